/*
 * paged_serve.h — C ABI of the B200 (sm_100a) KV-memory hot path of PagedServe.
 *
 * The library (paged_serve_b200/lib/libpaged_serve_b200.so) exports exactly the
 * functions declared here. Every entry point takes plain device pointers, sizes and
 * a CUDA stream handle (cudaStream_t passed as void*; NULL = legacy default stream),
 * launches asynchronously on that stream and returns a status code. Nothing here
 * allocates device memory, synchronises the stream, or keeps per-call global state,
 * so the ABI is re-entrant per device (one process per GPU).
 *
 * The reference (Vivek-Chaudhari30/Paged_Serve) has no native code: each entry
 * point below replaces a piece of its pure-PyTorch attention seam, cited as
 * pagedserve/<file>:<line> relative to that project's root.
 *
 * KV pool layout (one pool per layer for K and one for V):
 *     pool[num_blocks][num_kv_heads][block_size][head_dim]   (dtype elements)
 * so one (block, kv-head) tile — block_size x head_dim — is contiguous
 * (4 KiB for block_size 16, head_dim 128, bf16). A flat slot index is
 * block_id * block_size + offset_in_block, as in the reference's planned
 * StepInput.slot_mapping (pagedserve/attention/backend.py:104,113).
 *
 * Status codes: PS_OK on success; PS_ERR_INVALID for a bad argument (the Python
 * host maps it to ValueError, matching the reference's ValueError on bad
 * geometry, pagedserve/config.py:88-92 and pagedserve/attention/contiguous.py:117-121);
 * PS_ERR_UNSUPPORTED for a geometry the library has no kernel for (also ValueError);
 * PS_ERR_CUDA when a launch fails (RuntimeError). ps_last_error_string() gives the
 * calling thread's last message.
 *
 * Device-side errors: every kernel checks each block id, slot and position it
 * reads from an index array against the bounds it was given. An out-of-range
 * index is never dereferenced; the kernel skips the access and, when
 * `device_error` is non-NULL, ORs a PS_DEVERR_* bit into *device_error
 * (an int32 in device memory owned by the caller). Nothing traps.
 */
#ifndef PAGED_SERVE_B200_H
#define PAGED_SERVE_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define PS_API __attribute__((visibility("default")))
#else
#define PS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define PS_OK 0
#define PS_ERR_INVALID 1
#define PS_ERR_UNSUPPORTED 2
#define PS_ERR_CUDA 3

/* ---- element types (the pools, K/V/Q inputs and outputs share one type) ---- */
#define PS_DTYPE_F16 1
#define PS_DTYPE_BF16 2

/* ---- device error bits ORed into *device_error ---- */
#define PS_DEVERR_BLOCK_ID 1   /* block table entry outside [0, num_blocks)            */
#define PS_DEVERR_SLOT 2       /* slot_mapping entry outside [-1, num_blocks*block_size) */
#define PS_DEVERR_POSITION 4   /* RoPE position outside [0, table_positions)          */
#define PS_DEVERR_TIMEOUT 8    /* a bounded wait on an async copy gave up              */
#define PS_DEVERR_LENGTH 16    /* a context/query length exceeds the block table width */
#define PS_DEVERR_BLOCK_PAIRS 32 /* ps_copy_blocks: a destination repeated or used as a source */

/* Version of this ABI (bumped on any signature change). A caller compares
 * ps_abi_version() with the PS_ABI_VERSION it was compiled against. */
#define PS_ABI_VERSION 1
PS_API int ps_abi_version(void);

/* Message describing the calling thread's most recent non-PS_OK status. */
PS_API const char* ps_last_error_string(void);

/*
 * ps_cache_append — scatter this step's K and V rows into the paged pools.
 *
 * Replaces the KV write of ContiguousAttentionBackend.forward
 * (pagedserve/attention/contiguous.py:187-189: kv_cache[l,0,:n,s:e] = key, same for
 * value) under the write-then-attend contract of AttentionBackend.forward
 * (pagedserve/attention/backend.py:165-189).
 *
 * key/value: [num_tokens][num_kv_heads][head_dim]; row t starts at
 *   key + t*key_token_stride (elements), heads contiguous at stride head_dim.
 * slot_mapping: [num_tokens] int64; -1 skips the token (padding).
 * Bit-exact copy: pool row = input row.
 */
PS_API int ps_cache_append(void* k_pool, void* v_pool, const void* key, const void* value,
                    const int64_t* slot_mapping, int64_t num_tokens,
                    int64_t key_token_stride, int64_t value_token_stride, int num_kv_heads,
                    int head_dim, int block_size, int64_t num_blocks, int dtype,
                    int32_t* device_error, void* stream);

/*
 * ps_cache_append_rope — ps_cache_append with rotary position embedding applied
 * to K on the way into the pool (V is copied unchanged).
 *
 * Replaces the K half of apply_rotary (pagedserve/model/layers.py:62-77, split-half
 * rotate_half at :49-59) fused with the KV write (contiguous.py:187-189). The result
 * is bit-identical to the reference's bf16/fp16 arithmetic: each of k*cos,
 * rotate_half(k)*sin and their sum is rounded to the storage type separately.
 *
 * positions: [num_tokens] int64 absolute positions.
 * cos_sin_table: [table_positions][rope_dim] of dtype; row p holds
 *   cos(p*inv_freq[0..rope_dim/2)) followed by sin(p*inv_freq[0..rope_dim/2)),
 *   i.e. the first halves of the cos and sin that RotaryEmbedding.forward returns
 *   (pagedserve/model/layers.py:98-116), already cast to dtype.
 * rope_dim must equal head_dim (the reference rotates the whole head).
 */
PS_API int ps_cache_append_rope(void* k_pool, void* v_pool, const void* key, const void* value,
                         const int64_t* slot_mapping, const int64_t* positions,
                         int64_t num_tokens, int64_t key_token_stride,
                         int64_t value_token_stride, int num_kv_heads, int head_dim,
                         int block_size, int64_t num_blocks, const void* cos_sin_table,
                         int64_t table_positions, int rope_dim, int dtype,
                         int32_t* device_error, void* stream);

/*
 * ps_copy_blocks — copy whole KV blocks, pool[dst] = pool[src], for K and V of
 * num_layers layers (copy-on-write fork of a shared prefix block).
 *
 * No counterpart exists in the reference: block copies are planned there
 * (AGENTS.md "KV scatter/copy/swap kernels"; block manager fork/CoW) but unwritten.
 *
 * block_pairs: [num_pairs][2] int64 (src_block, dst_block).
 * Layer l's K pool is at k_pool + l*layer_stride_bytes (same for V).
 * block_bytes = num_kv_heads*block_size*head_dim*element size; must be a multiple
 * of 16, and both pools 16-byte aligned.
 *
 * All pairs of one call are copied concurrently, so the call is defined only for
 * a list in which every dst_block is distinct and no dst_block appears as the
 * src_block of another pair (a source may feed several pairs). A chain such as
 * [(a,b),(b,c)] must be split into two calls, in order, on one stream. For
 * lists of up to 4096 pairs the kernel checks this and ORs PS_DEVERR_BLOCK_PAIRS
 * into *device_error on a violation (the copies still run and their result is
 * unspecified); longer lists are not checked.
 */
PS_API int ps_copy_blocks(void* k_pool, void* v_pool, const int64_t* block_pairs, int64_t num_pairs,
                   int num_layers, int64_t layer_stride_bytes, int64_t block_bytes,
                   int64_t num_blocks, int32_t* device_error, void* stream);

/*
 * ps_swap_blocks — move whole KV blocks between two pools in different memories:
 * dst[pair.dst] = src[pair.src] for K and V of num_layers layers, in one launch.
 * Swap-out passes the HBM pool as src and a pinned host pool as dst; swap-in the
 * reverse (HBM to HBM also works).
 *
 * No counterpart exists in the reference: swap in/out is planned there for the
 * SWAP preemption policy (AGENTS.md:132-133 scheduler/policy, :149 cache_engine
 * "swap in/out", :158 "KV scatter/copy/swap kernels"; SchedulerConfig.preemption_policy,
 * pagedserve/config.py:228) but unwritten.
 *
 * Pools and block_pairs must each be device memory of the current device or
 * pinned host memory mapped into it (cudaHostAlloc / cudaMallocHost, or torch
 * pin_memory); pageable host memory and other devices' memory are rejected with
 * PS_ERR_INVALID. The kernel reads and writes host memory directly over the host
 * link (no staging copy, no per-block memcpy).
 *
 * block_pairs: [num_pairs][2] int64 (src_block, dst_block); ids outside
 *   [0, src_num_blocks) / [0, dst_num_blocks) set PS_DEVERR_BLOCK_ID and are skipped.
 * Layer l of a pool starts at pool + l*layer_stride_bytes.
 * max_ctas: grid cap; 0 = 32 CTAs when either side is host memory (enough to
 *   saturate the host link), two per SM for HBM to HBM.
 */
PS_API int ps_swap_blocks(void* dst_k_pool, void* dst_v_pool, int64_t dst_num_blocks,
                          int64_t dst_layer_stride_bytes, const void* src_k_pool,
                          const void* src_v_pool, int64_t src_num_blocks,
                          int64_t src_layer_stride_bytes, const int64_t* block_pairs,
                          int64_t num_pairs, int num_layers, int64_t block_bytes, int max_ctas,
                          int32_t* device_error, void* stream);

/*
 * ps_build_slot_mapping — the slot (and position) of every row of one step.
 *
 * The device half of the block manager the reference plans (memory/block_manager.py,
 * "block tables ... slot_mapping", AGENTS.md; the field it fills is
 * StepInput.slot_mapping, pagedserve/attention/backend.py:104,113). The step is laid
 * out as [num_seqs][query_len] rows with sequence b's q_lens[b] new tokens last
 * (left padding, as the reference engine pads, pagedserve/engine.py:245-274); row r
 * of b is logical position ctx_before[b] + r - (query_len - q_lens[b]) and slot
 * block_tables[b][pos / block_size] * block_size + pos % block_size. Padding rows
 * get -1 (slot and position). positions may be NULL.
 */
PS_API int ps_build_slot_mapping(int64_t* slot_mapping, int64_t* positions,
                                 const int32_t* block_tables, int64_t block_table_stride,
                                 const int32_t* ctx_before, const int32_t* q_lens,
                                 int num_seqs, int query_len, int block_size,
                                 int max_blocks_per_seq, int64_t num_blocks,
                                 int32_t* device_error, void* stream);

/*
 * ps_paged_decode_workspace_bytes — bytes of device workspace ps_paged_decode needs
 * for split-K (0 when split_tokens makes every sequence a single split).
 */
PS_API int64_t ps_paged_decode_workspace_bytes(int num_seqs, int num_q_heads, int head_dim,
                                        int block_size, int max_blocks_per_seq,
                                        int split_tokens);

/*
 * ps_paged_decode — one query token per sequence attending over its paged KV.
 *
 * Replaces the decode read of ContiguousAttentionBackend.forward: prefix read,
 * GQA repeat_interleave and masked SDPA (pagedserve/attention/contiguous.py:191-209)
 * with the padding/causal bias of _build_attn_bias (:136-169), which for one query
 * per sequence reduces to "keys [0, ctx_lens[b])".
 *
 * query/out: [num_seqs][num_q_heads][head_dim]; row b at +b*query_seq_stride /
 *   +b*out_seq_stride elements. Query head g uses KV head g / (num_q_heads/num_kv_heads).
 * block_tables: [num_seqs][block_table_stride] int32, first ceil(ctx/block_size)
 *   entries valid. ctx_lens: [num_seqs] int32 keys per sequence (0 -> output zeros).
 * scale: softmax scale (1/sqrt(head_dim) in the reference's SDPA default).
 * block_size: 8, 16 or 32 (PS_ERR_UNSUPPORTED otherwise); head_dim 64 or 128.
 * split_tokens: flash-decoding partition length in tokens (a multiple of 16 and of
 *   block_size), 0 = no split. Sequences longer than one partition are processed as independent
 *   partitions combined by a log-sum-exp merge; workspace must then hold
 *   ps_paged_decode_workspace_bytes(...) bytes (256-byte aligned): the fp32 partials and
 *   their LSEs, the list of (sequence, partition) units a small plan kernel writes from
 *   ctx_lens, and the counter the persistent decode CTAs claim units from. Every call
 *   rewrites all of it before reading it (no clearing needed); calls that share one
 *   workspace must not overlap on the GPU.
 * Softmax and accumulation are fp32; the output is rounded once to dtype.
 */
PS_API int ps_paged_decode(void* out, int64_t out_seq_stride, const void* query,
                    int64_t query_seq_stride, const void* k_pool, const void* v_pool,
                    int64_t num_blocks, const int32_t* block_tables,
                    int64_t block_table_stride, const int32_t* ctx_lens, int num_seqs,
                    int num_q_heads, int num_kv_heads, int head_dim, int block_size,
                    int max_blocks_per_seq, float scale, int split_tokens, void* workspace,
                    int64_t workspace_bytes, int dtype, int32_t* device_error, void* stream);

/*
 * ps_selftest_wait_timeout — exercises the failure path every kernel shares: one
 * thread waits, with the kernels' poll bound, on an mbarrier that nothing
 * arrives at, gives up, and ORs PS_DEVERR_TIMEOUT into *device_error. No GPU
 * fault and no hang: the context stays usable. For tests and health checks.
 */
PS_API int ps_selftest_wait_timeout(int32_t* device_error, void* stream);

/*
 * ps_paged_decode_order — longest-first launch order for a decode step. No
 * counterpart in the reference (its contiguous path has no launch order).
 *
 * Writes order[0 .. num_seqs) = a permutation of the sequence indices with the
 * longest ctx_lens first (a one-CTA counting sort into 1024 length buckets;
 * order inside a bucket is unspecified). Lengths are the same for every layer
 * of a step, so one call per step serves all its ps_paged_decode_ordered calls.
 * num_seqs <= 65535.
 */
PS_API int ps_paged_decode_order(const int32_t* ctx_lens, int num_seqs, int32_t* order,
                                 void* stream);

/*
 * ps_paged_decode_ordered — ps_paged_decode taking sequences in seq_order
 * (from ps_paged_decode_order; NULL = batch order). Starting the longest
 * sequences first shortens the last wave of the launch; results do not depend
 * on the order. An entry outside [0, num_seqs) sets PS_DEVERR_LENGTH and its
 * slot is skipped.
 */
PS_API int ps_paged_decode_ordered(void* out, int64_t out_seq_stride, const void* query,
                                   int64_t query_seq_stride, const void* k_pool,
                                   const void* v_pool, int64_t num_blocks,
                                   const int32_t* block_tables, int64_t block_table_stride,
                                   const int32_t* ctx_lens, int num_seqs, int num_q_heads,
                                   int num_kv_heads, int head_dim, int block_size,
                                   int max_blocks_per_seq, float scale, int split_tokens,
                                   void* workspace, int64_t workspace_bytes, int dtype,
                                   const int32_t* seq_order, int32_t* device_error, void* stream);

/*
 * ps_paged_decode_append — one decode step of a layer in one launch: writes
 * each sequence's new K/V row and attends, with the result and pool contents of
 * ps_cache_append followed by ps_paged_decode_ordered (the reference's
 * forward: write the step's K/V, then attend, pagedserve/attention/contiguous.py:188-209).
 *
 * key/value: [num_seqs][num_kv_heads][head_dim], row b at +b*key_seq_stride /
 *   +b*value_seq_stride elements (16-byte aligned, strides >= Hkv*D and % 8).
 * slot_mapping: [num_seqs] int64, the slot of each sequence's new token, which
 *   must be the position ctx_lens[b]-1 (the step's last key); -1 = no token.
 *   A slot >= num_blocks*block_size sets PS_DEVERR_SLOT and is not written.
 * Other arguments as ps_paged_decode_ordered. The CTA that attends over a
 * sequence's last partition writes its row before loading it, so the separate
 * append launch (and its tail) disappears from the step.
 */
PS_API int ps_paged_decode_append(void* out, int64_t out_seq_stride, const void* query,
                                  int64_t query_seq_stride, const void* key,
                                  int64_t key_seq_stride, const void* value,
                                  int64_t value_seq_stride, const int64_t* slot_mapping,
                                  void* k_pool, void* v_pool, int64_t num_blocks,
                                  const int32_t* block_tables, int64_t block_table_stride,
                                  const int32_t* ctx_lens, int num_seqs, int num_q_heads,
                                  int num_kv_heads, int head_dim, int block_size,
                                  int max_blocks_per_seq, float scale, int split_tokens,
                                  void* workspace, int64_t workspace_bytes, int dtype,
                                  const int32_t* seq_order, int32_t* device_error, void* stream);

/*
 * ps_paged_decode_plan / ps_paged_decode_append_planned — a split-K decode step
 * planned once for all its layers. No counterpart in the reference.
 *
 * The (sequence, partition) unit list a split decode works from depends only on
 * the step's ctx_lens, the launch order and the partition length, so it is the
 * same for every layer of a step. ps_paged_decode_plan writes it into the
 * workspace (and arms the claim counter); ps_paged_decode_append_planned then
 * behaves as ps_paged_decode_append for one layer without planning again (one
 * kernel fewer per layer), and its merge re-arms the counter for the next layer.
 * Plan with the same num_seqs, ctx_lens, seq_order, geometry, split_tokens and
 * workspace the layers use, and enqueue all of a step's layers before planning
 * the next step. A plan that does not fit the call is memory-safe (entries are
 * checked; PS_DEVERR_LENGTH is set) but gives wrong outputs. When split_tokens
 * leaves every sequence unsplit both calls plan nothing.
 */
PS_API int ps_paged_decode_plan(const int32_t* ctx_lens, int num_seqs, const int32_t* seq_order,
                                int num_q_heads, int head_dim, int block_size,
                                int max_blocks_per_seq, int split_tokens, void* workspace,
                                int64_t workspace_bytes, void* stream);
PS_API int ps_paged_decode_append_planned(void* out, int64_t out_seq_stride, const void* query,
                                          int64_t query_seq_stride, const void* key,
                                          int64_t key_seq_stride, const void* value,
                                          int64_t value_seq_stride, const int64_t* slot_mapping,
                                          void* k_pool, void* v_pool, int64_t num_blocks,
                                          const int32_t* block_tables,
                                          int64_t block_table_stride, const int32_t* ctx_lens,
                                          int num_seqs, int num_q_heads, int num_kv_heads,
                                          int head_dim, int block_size, int max_blocks_per_seq,
                                          float scale, int split_tokens, void* workspace,
                                          int64_t workspace_bytes, int dtype,
                                          const int32_t* seq_order, int32_t* device_error,
                                          void* stream);

/*
 * ps_paged_decode_listed — ps_paged_decode over a listed subset of a step's
 * sequences: for i < num_listed, sequence b = seq_list[i] (in [0, num_seqs))
 * attends over keys [0, ctx_lens[b]) and writes its output row; rows of
 * sequences not listed are left untouched. No counterpart in the reference (its
 * static engine runs whole-batch prefill or decode steps); it is the decode half
 * of a continuous-batching step whose other sequences prefill: query/out may
 * point at each sequence's last row of a [num_seqs][query_len] layout, with
 * query_seq_stride / out_seq_stride = query_len rows. Sequences are taken in
 * list order (list them longest first for the shortest last wave). The split-K
 * workspace is sized for num_seqs (ps_paged_decode_workspace_bytes). An entry
 * outside [0, num_seqs) sets PS_DEVERR_LENGTH and is skipped.
 */
PS_API int ps_paged_decode_listed(void* out, int64_t out_seq_stride, const void* query,
                                  int64_t query_seq_stride, const void* k_pool,
                                  const void* v_pool, int64_t num_blocks,
                                  const int32_t* block_tables, int64_t block_table_stride,
                                  const int32_t* ctx_lens, int num_seqs, const int32_t* seq_list,
                                  int num_listed, int num_q_heads, int num_kv_heads, int head_dim,
                                  int block_size, int max_blocks_per_seq, float scale,
                                  int split_tokens, void* workspace, int64_t workspace_bytes,
                                  int dtype, int32_t* device_error, void* stream);

/*
 * ps_paged_decode_noalloc — ps_paged_decode for callers that cannot allocate
 * device memory. It has no counterpart in the reference.
 *
 * Some hosts of this library cannot hand it a workspace: a plugin inside a
 * serving runtime or an FFI host (cgo, JNI, a C engine) whose allocator owns all
 * device memory and passes in only the input and output buffers, or a decode
 * loop that must not call cudaMalloc/cudaFree because they can synchronise the
 * device. This entry point takes the same arguments as ps_paged_decode minus the
 * workspace and keeps the split-K partials in a 64 MiB array compiled into the
 * library instead. It calls no allocator.
 *
 * - Limit: the partials, ps_paged_decode_workspace_bytes(...) bytes, must fit in
 *   64 MiB (67108864 bytes); larger requests return PS_ERR_INVALID. With
 *   split_tokens = 0 nothing is split and no scratch is used.
 * - Every GPU that loads the library holds the 64 MiB until the process exits.
 * - Arguments are checked as ps_paged_decode checks them before the scratch is
 *   sized, so an invalid argument reports its own error.
 * - The first call on a device that splits looks up the array's device address
 *   with that device current (cudaGetSymbolAddress) and caches it, keyed by the
 *   device's context; make that first call before any stream capture. After
 *   cudaDeviceReset the context is new and the next call looks the address up
 *   again (treat that call as a first call too).
 * - All calls on a device share the one array and it keeps the last call's
 *   contents. Nothing in it needs clearing: each call's plan kernel rewrites the
 *   list of split units and resets the claim counter before the decode reads
 *   them, and the combine reads only partials written by the same call. Calls
 *   that overlap on the GPU (different streams, or different host threads)
 *   race on it: serialise them.
 */
PS_API int ps_paged_decode_noalloc(void* out, int64_t out_seq_stride, const void* query,
                                   int64_t query_seq_stride, const void* k_pool,
                                   const void* v_pool, int64_t num_blocks,
                                   const int32_t* block_tables, int64_t block_table_stride,
                                   const int32_t* ctx_lens, int num_seqs, int num_q_heads,
                                   int num_kv_heads, int head_dim, int block_size,
                                   int max_blocks_per_seq, float scale, int split_tokens,
                                   int dtype, int32_t* device_error, void* stream);

/*
 * ps_paged_prefill — causal attention of a block of new query tokens per sequence
 * over that sequence's cached prefix plus the new tokens themselves.
 *
 * Replaces the prefill branch of ContiguousAttentionBackend.forward with the causal
 * mask of _build_attn_bias (pagedserve/attention/contiguous.py:136-169, query
 * position = context_len + i at :160-164) and SDPA (:208), generalised from one
 * shared context_len to per-sequence cached prefixes read through block tables.
 *
 * Sequence b owns query rows [q_starts[b], q_starts[b] + q_lens[b]) of
 *   query/out ([num_query_rows][num_q_heads][head_dim], row r at +r*token_stride
 *   elements); rows owned by no sequence are left untouched.
 * ctx_lens[b] = tokens cached before the first query row; query i of sequence b
 *   attends keys [0, ctx_lens[b] + i]. The K/V of the query tokens must already be
 *   in the pools (ps_cache_append / ps_cache_append_rope, or a block copy).
 * max_q_len bounds q_lens[] (sizes the launch grid).
 * head_dim must be 64 or 128, block_size 8, 16 or 32, and num_q_heads/num_kv_heads
 * at most 16. Runs on
 * tcgen05 tensor cores with TMEM accumulators, one persistent CTA per SM: a work
 * item is two tiles of 128 query rows = 128/G new tokens x the G query heads of
 * one KV head, so every K/V tile feeds all G heads.
 */
PS_API int ps_paged_prefill(void* out, int64_t out_token_stride, const void* query,
                     int64_t query_token_stride, int64_t num_query_rows, const void* k_pool,
                     const void* v_pool,
                     int64_t num_blocks, const int32_t* block_tables,
                     int64_t block_table_stride, const int32_t* q_starts,
                     const int32_t* q_lens, const int32_t* ctx_lens, int num_seqs,
                     int max_q_len, int num_q_heads, int num_kv_heads, int head_dim,
                     int block_size, int max_blocks_per_seq, float scale, int dtype,
                     int32_t* device_error, void* stream);

/*
 * ps_paged_prefill_split — ps_paged_prefill with split-K over the key range, for
 * steps with few query tiles over long cached prefixes (a long prompt's next
 * chunk): ps_paged_prefill runs one CTA per work item, so 64 items leave most
 * of the GPU idle while each walks its whole context.
 *
 * Same arguments, outputs and errors as ps_paged_prefill, plus:
 * split_keys: keys per piece, a positive multiple of 128 (0 = no split). Every
 *   item is cut into pieces of split_keys keys, run by different CTAs, and a
 *   second launch merges the pieces of the items that have more than one. With
 *   split_keys >= max_blocks_per_seq * block_size nothing is split and the call
 *   is ps_paged_prefill. Pieces per item, and so the workspace, follow
 *   max_blocks_per_seq: pass the longest sequence's blocks (context + new
 *   tokens), not a wider table's width (block_table_stride may be larger).
 * workspace: device memory of at least ps_paged_prefill_workspace_bytes(...)
 *   bytes (same sizes), 256-byte aligned, used by one call at a time; contents
 *   need no initialisation.
 * Results agree with ps_paged_prefill within rounding (a split row's sums are
 *   added in another order), not bit for bit.
 * No counterpart in the reference (its prefill is one dense SDPA per step).
 */
PS_API int ps_paged_prefill_split(void* out, int64_t out_token_stride, const void* query,
                                  int64_t query_token_stride, int64_t num_query_rows,
                                  const void* k_pool, const void* v_pool, int64_t num_blocks,
                                  const int32_t* block_tables, int64_t block_table_stride,
                                  const int32_t* q_starts, const int32_t* q_lens,
                                  const int32_t* ctx_lens, int num_seqs, int max_q_len,
                                  int num_q_heads, int num_kv_heads, int head_dim,
                                  int block_size, int max_blocks_per_seq, float scale,
                                  int split_keys, void* workspace, int64_t workspace_bytes,
                                  int dtype, int32_t* device_error, void* stream);

/*
 * ps_paged_prefill_workspace_bytes — bytes of workspace ps_paged_prefill_split
 * needs for these sizes: (query-tile pairs x pieces) x 256 rows x (head_dim + 2)
 * fp32 values; 0 when nothing is split or the sizes are invalid.
 */
PS_API int64_t ps_paged_prefill_workspace_bytes(int num_seqs, int max_q_len, int num_q_heads,
                                                int num_kv_heads, int head_dim, int block_size,
                                                int max_blocks_per_seq, int split_keys);

/*
 * ps_stream_read — diagnostic: read num_bytes of device memory once and XOR every
 * 32-bit word into *checksum (a device uint32 the caller zeroes first). No
 * counterpart in the reference. Timed alone over a buffer larger than L2 it
 * gives the HBM read bandwidth this GPU reaches, the ceiling for read-dominated
 * kernels such as ps_paged_decode (a copy moves bytes both ways and measures a
 * different bound).
 *
 * method: PS_STREAM_BULK — bulk asynchronous copies of 8 KB chunks into per-warp
 *   shared-memory rings (3 CTAs x 4 warps per SM; the way the decode loads K/V);
 *   PS_STREAM_LOADS — 16-byte loads, eight in flight per thread.
 * src 16-byte aligned, num_bytes a multiple of 16. A bulk copy that does not
 * complete within the kernels' wait bound sets PS_DEVERR_TIMEOUT in
 * *device_error (may be NULL).
 */
#define PS_STREAM_BULK 0
#define PS_STREAM_LOADS 1
PS_API int ps_stream_read(const void* src, int64_t num_bytes, uint32_t* checksum, int method,
                          int32_t* device_error, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PAGED_SERVE_B200_H */
