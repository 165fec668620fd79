// Paged decode attention (one query token per sequence, GQA) for sm_100a.
//
// Work decomposition: one CTA per (kv-head, partition, sequence). A partition
// is `split_tokens` keys of one sequence (the whole context when not split).
// The CTA's warps take the partition's KV blocks round-robin; each warp owns a
// private ring of NS shared-memory stages fed by TMA (two 64-column boxes per
// K or V tile, 128-byte swizzle) and runs its own fp32 online softmax, so the
// steady state needs no CTA-wide barrier. The group of G = Hq/Hkv query heads
// that share the KV head forms the 16-row A operand of a bf16/f16 warp MMA
// (rows >= G are zero; for G <= 8 rows 8-15 are not even carried through the
// softmax), so every K/V byte is read from HBM exactly once per step and
// consumed by all G heads:
//   S[16 x 16 keys]  = Q[16 x D] . K_blk^T      (D/16 MMAs per n-tile, 2 n-tiles)
//   O[16 x D]       += P[16 x 16 keys] . V_blk  (D/8 MMAs)
// The S accumulator fragment is re-used directly as the A fragment of P.V.
// At the end the warps merge (m, l, O) through shared memory; partitions of a
// split sequence are merged by ps_decode_combine_kernel with a log-sum-exp.
//
// Arithmetic intensity is ~4 flop per KV byte, so the tensor pipe is nearly
// idle and the kernel is bound by HBM bandwidth; what matters is keeping
// enough TMA bytes in flight per SM (NW * NS * 2 tiles per CTA).
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "capi_internal.h"
#include "common.cuh"

namespace ps {
namespace {

constexpr int kChunk = 16;  // keys per MMA step (one 16-row TMA tile per K and V half)

struct DecodeParams {
  void* out;
  const void* q;
  int64_t out_stride;
  int64_t q_stride;
  const int32_t* block_tables;
  int64_t bt_stride;
  const int32_t* ctx_lens;
  float* ws_o;    // [B][max_splits][Hq][D]
  float* ws_lse;  // [B][max_splits][Hq]   (log2 domain)
  int64_t num_blocks;
  int num_seqs;
  int num_launch;  // launch positions: num_seqs, or the length of a listed subset
  int num_q_heads;
  int num_kv_heads;
  int group;  // Hq / Hkv
  int max_blocks;
  int block_size;
  int part_tokens;  // partition length (multiple of 16 and of the block size)
  int max_splits;
  int table_cap;  // ints of block table staged per CTA
  float scale_log2;
  int32_t* err;
  // Split-K only: the (sequence, partition) pairs that have keys, as
  // b * max_splits + split, and their number; written by decode_plan_kernel.
  int32_t* items;
  int32_t* item_count;
  int32_t* item_next;  // claim counter of the persistent CTAs (reset by the plan and the combine)
  bool planned;        // the unit list was written by ps_paged_decode_plan for this step
  // Optional permutation of [0, num_seqs) (longest first, from
  // ps_paged_decode_order): the order CTAs / planned units take sequences in.
  const int32_t* seq_order;
  // Optional fused append of the step's new token (ps_paged_decode_append):
  // new_k/new_v [num_seqs][Hkv][D] rows go to slot new_slots[b] of the pools
  // (raw pointers; -1 = no token) before the unit that reads that slot loads it.
  void* k_pool_w;
  void* v_pool_w;
  const void* new_k;
  const void* new_v;
  int64_t new_k_stride;
  int64_t new_v_stride;
  const int64_t* new_slots;
  int64_t num_slots;
};

// Sequence at position i of the launch order; -1 (and an error bit) for an
// entry that is not a sequence index.
__device__ __forceinline__ int ordered_seq(const DecodeParams& p, int i) {
  if (!p.seq_order) return i;
  const int b = p.seq_order[i];
  if (b < 0 || b >= p.num_seqs) {
    set_device_error(p.err, PS_DEVERR_LENGTH);
    return -1;
  }
  return b;
}

template <int D>
struct TileGeom {
  static constexpr int kHalves = D / 64;              // 64-column TMA boxes per tile
  static constexpr int kHalfBytes = kChunk * 128;     // one chunk half: 16 rows x 128 B
  static constexpr int kTileBytes = kHalves * kHalfBytes;
  // Byte offset of 16-byte chunk c (0..D/8) of token row t inside a swizzled tile.
  __device__ __forceinline__ static uint32_t off(int t, int c) {
    return (c >> 3) * kHalfBytes + t * 128 + ((((c & 7) ^ (t & 7))) << 4);
  }
};

template <int D, int NW, int NS>
struct DecodeSmem {
  static constexpr int kStageBytes = 2 * TileGeom<D>::kTileBytes;  // K + V
  static constexpr int kRingBytes = NW * NS * kStageBytes;
  static constexpr int kMergeBytes = NW * 16 * (D + 2) * 4;  // m, l, O of up to 16 rows per warp
  static_assert(kMergeBytes <= kRingBytes, "merge area must fit in the ring");
  static constexpr int kBarOffset = kRingBytes;
  static constexpr int kTableOffset = kBarOffset + NW * NS * 8;
  static size_t bytes(int table_cap) {
    return 1024 /*alignment slack*/ + kTableOffset + static_cast<size_t>(table_cap) * 4;
  }
};

// BS = tokens per KV block (8, 16 or 32). A 16-key chunk is one 16-row box of
// its block (BS 16), the first or second half of a block (BS 32), or two 8-row
// boxes of consecutive blocks (BS 8); an 8-row box is one 1024-byte swizzle
// atom, so every case lands in the same shared-memory tile layout.
// R = MMA rows carried (8 when G <= 8, else 16).
// kList: persistent CTAs (one per resident slot) claim (kv head, unit) pairs of
// the split-K work list from an atomic counter, one ahead; otherwise one CTA
// per (kv head, 1, sequence).
template <typename T, int D, int NW, int NS, int BS, int R, bool kList>
__global__ void __launch_bounds__(NW * 32)
    paged_decode_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap) {
  static_assert(R == 8 || R == 16, "8 or 16 rows");
  using G = TileGeom<D>;
  using SM = DecodeSmem<D, NW, NS>;
  constexpr bool kWide = R == 16;
  constexpr int kKSteps = D / 16;
  constexpr int kNTiles = D / 8;

  int h = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int group = p.group;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::kBarOffset);
  int32_t* table = reinterpret_cast<int32_t*>(smem + SM::kTableOffset);
  // Launched with programmatic stream serialization: the set-up above touches
  // only shared memory and kernel parameters; global memory waits for the
  // previous kernel.
  pdl_trigger();
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&kmap);
    tma_prefetch_desc(&vmap);
    for (int i = 0; i < NW * NS; ++i) mbar_init(&bars[i], 1);
    fence_barrier_init();
  }
  pdl_wait();

  // Work units: one (sequence, partition) per CTA, or, for split-K, (kv head,
  // planned unit) pairs claimed one at a time (thread 0 claims the next while
  // the current one runs; the claimed index goes through a double-buffered
  // shared slot, so a barrier per unit suffices). Ring stages and barrier
  // phases carry over from one unit to the next (gbase = this warp's ring
  // iterations so far).
  __shared__ int claimed[2];
  int total = 0, next = 0;
  if constexpr (kList) {
    // A unit list planned for another step (a caller error) can hold more
    // entries than this launch's workspace holds, or sequences it does not
    // have: the count is clamped to the capacity and every entry is checked.
    const int cap = p.num_seqs * p.max_splits;
    total = min(max(*p.item_count, 0), cap) * p.num_kv_heads;
    if (threadIdx.x == 0) next = atomicAdd(p.item_next, 1);
  }
  uint32_t gbase = 0;
  for (int k = 0;; ++k) {
  int split, b;
  if constexpr (kList) {
    if (threadIdx.x == 0) {
      claimed[k & 1] = next;
      next = atomicAdd(p.item_next, 1);
    }
    __syncthreads();
    const int u = claimed[k & 1];
    if (u >= total) break;
    h = u % p.num_kv_heads;
    const int item = p.items[u / p.num_kv_heads];
    if (item < 0 || item >= p.num_seqs * p.max_splits) {
      if (threadIdx.x == 0) set_device_error(p.err, PS_DEVERR_LENGTH);
      continue;
    }
    split = item % p.max_splits;
    b = item / p.max_splits;
  } else {
    if (k > 0) break;
    split = blockIdx.y;
    b = ordered_seq(p, blockIdx.z);
    if (b < 0) break;
  }

  int ctx = p.ctx_lens[b];
  if (ctx > p.max_blocks * BS) {
    if (threadIdx.x == 0 && split == 0) set_device_error(p.err, PS_DEVERR_LENGTH);
    ctx = 0;
  }
  const int nsplit = (ctx + p.part_tokens - 1) / p.part_tokens;
  // Fused append: this (sequence, kv head)'s new K/V row goes to its slot, in
  // the last partition, which only this unit reads. Thread t < 2*D/8 moves 16 B.
  const bool writer = p.new_k != nullptr && split == (nsplit > 0 ? nsplit - 1 : 0);
  auto write_row = [&](int t) {
    constexpr int kPieces = D / 8;
    const int64_t slot = p.new_slots[b];
    if (slot >= p.num_slots) {
      if (t == 0) set_device_error(p.err, PS_DEVERR_SLOT);
      return false;
    }
    if (slot < 0 || t >= 2 * kPieces) return false;
    const bool is_v = t >= kPieces;
    const int piece = is_v ? t - kPieces : t;
    const int64_t blk = slot / BS;
    const int64_t row = ((blk * p.num_kv_heads + h) * BS + (slot - blk * BS)) * D + piece * 8;
    const T* src = static_cast<const T*>(is_v ? p.new_v : p.new_k) +
                   b * (is_v ? p.new_v_stride : p.new_k_stride) + static_cast<int64_t>(h) * D +
                   piece * 8;
    T* dst = static_cast<T*>(is_v ? p.v_pool_w : p.k_pool_w) + row;
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
    return true;
  };
  if (ctx <= 0) {
    if (writer) write_row(threadIdx.x);  // nothing of this launch reads it
    // No keys: the output is defined as zeros (nothing to attend to).
    if (split == 0) {
      T* o = static_cast<T*>(p.out) + b * p.out_stride + static_cast<int64_t>(h) * group * D;
      for (int i = threadIdx.x; i < group * D; i += blockDim.x) o[i] = from_f32<T>(0.f);
    }
    continue;
  }
  if (split >= nsplit) continue;

  const int t_begin = split * p.part_tokens;
  const int t_end = min(ctx, t_begin + p.part_tokens);
  const int chunk_begin = t_begin / kChunk;
  const int nchunk = (t_end - t_begin + kChunk - 1) / kChunk;
  const int blk_begin = t_begin / BS;  // partitions start on block and chunk boundaries
  const int nblk = (t_end - t_begin + BS - 1) / BS;

  // Stage this partition's block ids, validated, in shared memory.
  const int32_t* bt = p.block_tables + static_cast<int64_t>(b) * p.bt_stride + blk_begin;
  for (int i = threadIdx.x; i < nblk; i += blockDim.x) {
    int32_t id = bt[i];
    if (id < 0 || id >= p.num_blocks) {
      set_device_error(p.err, PS_DEVERR_BLOCK_ID);
      id = 0;  // read a valid block instead of faulting; the error bit reports it
    }
    table[i] = id;
  }
  __syncthreads();
  if (writer && warp == (nchunk - 1) % NW) {
    // The warp that loads the last chunk writes the row, then hands it to its
    // own TMA issue (lane 0) through the proxy fence and a warp barrier.
    if (write_row(lane)) fence_proxy_async_global();
    __syncwarp();
  }

  uint8_t* ring = smem + warp * NS * SM::kStageBytes;
  uint64_t* wbar = bars + warp * NS;
  constexpr int kBox = BS < kChunk ? BS : kChunk;  // rows per TMA box
  constexpr int kBoxes = kChunk / kBox;            // boxes per 16-key chunk

  // Issue the TMA loads of warp-local iteration `it` (chunk warp + it*NW).
  auto issue = [&](int it) {
    const int j = warp + it * NW;
    const int st = (gbase + it) % NS;
    uint8_t* kdst = ring + st * SM::kStageBytes;
    uint8_t* vdst = kdst + G::kTileBytes;
    mbar_arrive_expect_tx(&wbar[st], SM::kStageBytes);
#pragma unroll
    for (int x = 0; x < kBoxes; ++x) {
      const int tok = j * kChunk + x * kBox;  // first key of the box, from t_begin
      // A box past the partition's last block re-reads that block (its keys are masked).
      const int bi = min(tok / BS, nblk - 1);
      const int32_t row = (table[bi] * p.num_kv_heads + h) * BS + tok % BS;
#pragma unroll
      for (int half = 0; half < G::kHalves; ++half) {
        tma_load_2d(kdst + half * G::kHalfBytes + x * kBox * 128, &kmap, &wbar[st], half * 64, row);
        tma_load_2d(vdst + half * G::kHalfBytes + x * kBox * 128, &vmap, &wbar[st], half * 64, row);
      }
    }
  };

  if (lane == 0) {
#pragma unroll
    for (int it = 0; it < NS; ++it)
      if (warp + it * NW < nchunk) issue(it);
  }

  // Q fragments: lane (r = lane/4, q4 = lane%4) holds rows r and r + 8 of the
  // head group (A registers a0/a2 and a1/a3 of the m16n8k16 layout).
  const int r = lane >> 2;
  const int q4 = lane & 3;
  uint32_t qa0[kKSteps], qa1[kKSteps], qa2[kKSteps], qa3[kKSteps];
  {
    const bool real = r < group;
    const T* qrow = static_cast<const T*>(p.q) + b * p.q_stride +
                    static_cast<int64_t>(h * group + (real ? r : 0)) * D;
    const bool real_hi = kWide && r + 8 < group;
    const T* qrow_hi = static_cast<const T*>(p.q) + b * p.q_stride +
                       static_cast<int64_t>(h * group + (real_hi ? r + 8 : 0)) * D;
#pragma unroll
    for (int kk = 0; kk < kKSteps; ++kk) {
      qa0[kk] = real ? *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 2 * q4) : 0u;
      qa2[kk] = real ? *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 8 + 2 * q4) : 0u;
      qa1[kk] = real_hi ? *reinterpret_cast<const uint32_t*>(qrow_hi + kk * 16 + 2 * q4) : 0u;
      qa3[kk] = real_hi ? *reinterpret_cast<const uint32_t*>(qrow_hi + kk * 16 + 8 + 2 * q4) : 0u;
    }
  }

  float o[kNTiles][4];
#pragma unroll
  for (int n = 0; n < kNTiles; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_run = -INFINITY, m_hi = -INFINITY;  // rows r and r + 8
  float l_run = 0.f, l_hi = 0.f;
  int stuck_at = -1;  // warp-local iteration whose wait gave up

  // ldmatrix row/chunk selectors (see the fragment layouts above).
  const int qk_t = (lane & 7) + ((lane >> 4) << 3);
  const int qk_c = (lane >> 3) & 1;
  const int pv_t = (lane & 7) + (((lane >> 3) & 1) << 3);
  const int pv_c = lane >> 4;

  for (int it = 0; warp + it * NW < nchunk; ++it) {
    const int j = warp + it * NW;
    const int st = (gbase + it) % NS;
    if (!mbar_wait_bounded(&wbar[st], ((gbase + it) / NS) & 1)) {
      stuck_at = it;
      break;
    }
    const uint32_t kbase = smem_u32(ring + st * SM::kStageBytes);
    const uint32_t vbase = kbase + G::kTileBytes;

    // ---- S = Q K^T for the 16 keys of this block
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int kk = 0; kk < kKSteps; ++kk) {
      uint32_t b00, b01, b10, b11;
      ldsm_x4(kbase + G::off(qk_t, 2 * kk + qk_c), b00, b01, b10, b11);
      Mma<T>::run(s0, qa0[kk], qa1[kk], qa2[kk], qa3[kk], b00, b01);
      Mma<T>::run(s1, qa0[kk], qa1[kk], qa2[kk], qa3[kk], b10, b11);
    }

    // ---- online softmax (log2 domain): row r lives in s0[0..1], s1[0..1],
    // row r + 8 in s0[2..3], s1[2..3]
    const int tok0 = (chunk_begin + j) * kChunk;
    float x[4] = {s0[0] * p.scale_log2, s0[1] * p.scale_log2, s1[0] * p.scale_log2,
                  s1[1] * p.scale_log2};
    float y[4] = {s0[2] * p.scale_log2, s0[3] * p.scale_log2, s1[2] * p.scale_log2,
                  s1[3] * p.scale_log2};
    if (tok0 + kChunk > t_end) {
      const int tk[4] = {2 * q4, 2 * q4 + 1, 8 + 2 * q4, 9 + 2 * q4};
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (tok0 + tk[e] >= t_end) x[e] = y[e] = -INFINITY;
    }
    float mx = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx);
    const float alpha = exp2f(m_run - m_new);
    const uint32_t pa0 = pack2<T>(exp2f(x[0] - m_new), exp2f(x[1] - m_new));
    const uint32_t pa2 = pack2<T>(exp2f(x[2] - m_new), exp2f(x[3] - m_new));
    // Row sum of the rounded P the MMA consumes: normalisation matches the weights used.
    const float2 r0 = unpack2<T>(pa0);
    const float2 r1 = unpack2<T>(pa2);
    l_run = l_run * alpha + ((r0.x + r0.y) + (r1.x + r1.y));
    m_run = m_new;
    uint32_t pa1 = 0u, pa3 = 0u;
    float alpha_hi = 1.f;
    if constexpr (kWide) {
      float my = fmaxf(fmaxf(y[0], y[1]), fmaxf(y[2], y[3]));
      my = fmaxf(my, __shfl_xor_sync(0xffffffffu, my, 1));
      my = fmaxf(my, __shfl_xor_sync(0xffffffffu, my, 2));
      const float mh_new = fmaxf(m_hi, my);
      alpha_hi = exp2f(m_hi - mh_new);
      pa1 = pack2<T>(exp2f(y[0] - mh_new), exp2f(y[1] - mh_new));
      pa3 = pack2<T>(exp2f(y[2] - mh_new), exp2f(y[3] - mh_new));
      const float2 h0 = unpack2<T>(pa1);
      const float2 h1 = unpack2<T>(pa3);
      l_hi = l_hi * alpha_hi + ((h0.x + h0.y) + (h1.x + h1.y));
      m_hi = mh_new;
    }
#pragma unroll
    for (int n = 0; n < kNTiles; ++n) {
      o[n][0] *= alpha;
      o[n][1] *= alpha;
      if constexpr (kWide) {
        o[n][2] *= alpha_hi;
        o[n][3] *= alpha_hi;
      }
    }

    // ---- O += P V
#pragma unroll
    for (int jj = 0; jj < kNTiles / 2; ++jj) {
      uint32_t b00, b01, b10, b11;
      ldsm_x4_t(vbase + G::off(pv_t, 2 * jj + pv_c), b00, b01, b10, b11);
      Mma<T>::run(o[2 * jj], pa0, pa1, pa2, pa3, b00, b01);
      Mma<T>::run(o[2 * jj + 1], pa0, pa1, pa2, pa3, b10, b11);
    }

    __syncwarp();
    if (lane == 0 && warp + (it + NS) * NW < nchunk) {
      fence_proxy_async_smem();  // our ldmatrix reads of this stage precede the refill
      issue(it + NS);
    }
  }

  if (stuck_at >= 0) {
    set_device_error(p.err, PS_DEVERR_TIMEOUT);
    // Drain this warp's copies still in flight (iterations stuck_at ..
    // stuck_at+NS-1 were issued, each wait bounded) before the CTA moves on.
    if (lane == 0) {
      for (int k = 0; k < NS; ++k) {
        const int i2 = stuck_at + k;
        if (warp + i2 * NW < nchunk)
          (void)mbar_wait_bounded(&wbar[(gbase + i2) % NS], ((gbase + i2) / NS) & 1);
      }
    }
  }
  __syncwarp();

  // Row sums across the quad (each lane summed only its own 4 keys).
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  if constexpr (kWide) {
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
  }

  // ---- merge the NW warps' partial states through shared memory
  __syncthreads();  // every warp is done reading its ring; alias it as the merge area
  float* ms = reinterpret_cast<float*>(smem);   // [NW][R]
  float* ls = ms + NW * R;                      // [NW][R]
  float* os = ls + NW * R;                      // [NW][R][D]
  if (q4 == 0) {
    ms[warp * R + r] = m_run;
    ls[warp * R + r] = l_run;
    if constexpr (kWide) {
      ms[warp * R + r + 8] = m_hi;
      ls[warp * R + r + 8] = l_hi;
    }
  }
#pragma unroll
  for (int n = 0; n < kNTiles; ++n) {
    *reinterpret_cast<float2*>(&os[(warp * R + r) * D + n * 8 + 2 * q4]) =
        make_float2(o[n][0], o[n][1]);
    if constexpr (kWide)
      *reinterpret_cast<float2*>(&os[(warp * R + r + 8) * D + n * 8 + 2 * q4]) =
          make_float2(o[n][2], o[n][3]);
  }
  __syncthreads();

  const bool single = (nsplit == 1);
  for (int idx = threadIdx.x; idx < group * (D / 4); idx += blockDim.x) {
    const int g = idx / (D / 4);
    const int d = (idx % (D / 4)) * 4;
    float mmax = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) mmax = fmaxf(mmax, ms[w * R + g]);
    float lsum = 0.f;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float mw = ms[w * R + g];
      const float sc = (mw == -INFINITY) ? 0.f : exp2f(mw - mmax);
      lsum += ls[w * R + g] * sc;
      const float4 ov = *reinterpret_cast<const float4*>(&os[(w * R + g) * D + d]);
      acc[0] += ov.x * sc;
      acc[1] += ov.y * sc;
      acc[2] += ov.z * sc;
      acc[3] += ov.w * sc;
    }
    const float inv = (lsum > 0.f) ? 1.f / lsum : 0.f;
    const int qh = h * group + g;
    if (single) {
      T* orow = static_cast<T*>(p.out) + b * p.out_stride + static_cast<int64_t>(qh) * D + d;
      uint2 packed;
      packed.x = pack2<T>(acc[0] * inv, acc[1] * inv);
      packed.y = pack2<T>(acc[2] * inv, acc[3] * inv);
      *reinterpret_cast<uint2*>(orow) = packed;
    } else {
      const int64_t slot = (static_cast<int64_t>(b) * p.max_splits + split) * p.num_q_heads + qh;
      *reinterpret_cast<float4*>(p.ws_o + slot * D + d) =
          make_float4(acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv);
      if (d == 0) p.ws_lse[slot] = (lsum > 0.f) ? mmax + log2f(lsum) : -INFINITY;
    }
  }
  // This warp's ring iterations in the unit (its chunks warp, warp + NW, ...).
  gbase += nchunk > warp ? static_cast<uint32_t>((nchunk - warp + NW - 1) / NW) : 0u;
  if constexpr (kList) {
    // The merge area aliases the ring: every thread is done with it before the
    // next unit's TMA writes it.
    fence_proxy_async_smem();
    __syncthreads();
  }
  }  // work units
}

// Longest-first order of the sequences for a decode launch: a counting sort of
// ctx_lens into 1024 buckets spanning [0, max ctx], buckets taken from the
// longest down (order inside a bucket is unspecified). One CTA.
__global__ void __launch_bounds__(1024) decode_order_kernel(const int32_t* ctx_lens, int n,
                                                            int32_t* order) {
  constexpr int kBuckets = 1024;
  __shared__ int hist[kBuckets];
  __shared__ int cursor[kBuckets];
  __shared__ int wmax[32];
  const int t = threadIdx.x;
  const int lane = t & 31;
  const int warp = t >> 5;
  hist[t] = 0;
  int mx = 0;
  for (int b = t; b < n; b += 1024) mx = max(mx, ctx_lens[b]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) wmax[warp] = mx;
  __syncthreads();
  if (warp == 0) {
    int m = wmax[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) wmax[0] = m;
  }
  __syncthreads();
  const int64_t span = static_cast<int64_t>(wmax[0]) + 1;
  auto bucket = [&](int ctx) -> int {
    const int c = max(ctx, 0);
    return static_cast<int>((static_cast<int64_t>(c) * kBuckets) / span);  // < kBuckets
  };
  for (int b = t; b < n; b += 1024) atomicAdd(&hist[bucket(ctx_lens[b])], 1);
  __syncthreads();
  // Start of bucket k = sequences in buckets above k: an exclusive scan over the
  // buckets in descending order (thread t owns bucket kBuckets - 1 - t).
  const int mine = hist[kBuckets - 1 - t];
  int x = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();  // hist read; wmax reused for warp totals
  if (lane == 31) wmax[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const int w = wmax[lane];
    int y = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int z = __shfl_up_sync(0xffffffffu, y, o);
      if (lane >= o) y += z;
    }
    wmax[lane] = y - w;
  }
  __syncthreads();
  cursor[kBuckets - 1 - t] = wmax[warp] + x - mine;
  __syncthreads();
  for (int b = t; b < n; b += 1024) order[atomicAdd(&cursor[bucket(ctx_lens[b])], 1)] = b;
}

// Lists the (sequence, partition) units of a split-K launch in launch order
// (seq_order when given, else batch order):
// a sequence with ctx keys has ceil(ctx / part) partitions, and one unit even
// without keys (its output is written as zeros). One CTA of 1024 threads; a
// running block-wide prefix sum places each sequence's units.
__global__ void __launch_bounds__(1024) decode_plan_kernel(const DecodeParams p) {
  pdl_trigger();
  pdl_wait();
  __shared__ int wsum[32];
  __shared__ int carry;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < p.num_launch; base += 1024) {
    const int i = base + threadIdx.x;
    const int b = i < p.num_launch ? ordered_seq(p, i) : -1;
    int ns = 0;
    if (b >= 0) {
      int ctx = p.ctx_lens[b];
      if (ctx > p.max_blocks * p.block_size) ctx = 0;  // the decode kernel reports it
      ns = ctx <= 0 ? 1 : (ctx + p.part_tokens - 1) / p.part_tokens;
    }
    int x = ns;  // inclusive scan within the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) wsum[warp] = x;
    __syncthreads();
    if (warp == 0) {
      const int w = wsum[lane];
      int y = w;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int z = __shfl_up_sync(0xffffffffu, y, o);
        if (lane >= o) y += z;
      }
      wsum[lane] = y - w;  // exclusive, per warp
    }
    __syncthreads();
    const int off = carry + wsum[warp] + x - ns;
    for (int k = 0; k < ns; ++k) p.items[off + k] = b * p.max_splits + k;
    __syncthreads();  // every thread has read carry
    if (threadIdx.x == blockDim.x - 1) carry = off + ns;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    *p.item_count = carry;
    *p.item_next = 0;
  }
}

// Merge the partitions of each split sequence: out = sum_s w_s O_s, with
// w_s = 2^(lse_s - max lse) / sum. One warp per (sequence, query head).
template <typename T, int D>
__global__ void __launch_bounds__(128) decode_combine_kernel(const DecodeParams p) {
  pdl_trigger();
  pdl_wait();
  // The decode launch has finished claiming units: rearm the claim counter, so
  // the next layer of a planned step can reuse the unit list without a plan.
  if (blockIdx.x == 0 && threadIdx.x == 0) *p.item_next = 0;
  const int warp_global = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (warp_global >= p.num_launch * p.num_q_heads) return;
  const int b = ordered_seq(p, warp_global / p.num_q_heads);  // only launched sequences
  if (b < 0) return;
  const int qh = warp_global % p.num_q_heads;
  int ctx = p.ctx_lens[b];
  if (ctx > p.max_blocks * p.block_size) ctx = 0;
  const int nsplit = (ctx + p.part_tokens - 1) / p.part_tokens;
  if (nsplit <= 1) return;
  const int64_t base = static_cast<int64_t>(b) * p.max_splits * p.num_q_heads + qh;
  float mmax = -INFINITY;
  for (int s = lane; s < nsplit; s += 32)
    mmax = fmaxf(mmax, p.ws_lse[base + static_cast<int64_t>(s) * p.num_q_heads]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mmax = fmaxf(mmax, __shfl_xor_sync(0xffffffffu, mmax, o));
  constexpr int kPer = D / 32;  // dims per lane
  using Vec = typename std::conditional<kPer == 4, float4, float2>::type;
  float acc[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) acc[i] = 0.f;
  float wsum = 0.f;
  auto add = [&](float w, const Vec& v) {
    wsum += w;
    acc[0] += w * v.x;
    acc[1] += w * v.y;
    if constexpr (kPer == 4) {
      acc[2] += w * reinterpret_cast<const float4&>(v).z;
      acc[3] += w * reinterpret_cast<const float4&>(v).w;
    }
  };
  auto load = [&](int s) {
    return *reinterpret_cast<const Vec*>(p.ws_o + (base + static_cast<int64_t>(s) * p.num_q_heads) * D +
                                         lane * kPer);
  };
  // Partitions in order (the sum order is fixed); lane l computes the weight of
  // partition s0 + l. Eight partitions' loads are in flight at a time: when few
  // sequences are split, the longest one's chain of loads (64 partitions for
  // 32k tokens) sets the length of the launch (four in flight: 156.6 against
  // 153.3 us per 64-sequence 70B layer); sixteen gain a little more there but
  // cost occupancy when many sequences are split.
  for (int s0 = 0; s0 < nsplit; s0 += 32) {
    const int n = min(32, nsplit - s0);
    const float lse = lane < n ? p.ws_lse[base + static_cast<int64_t>(s0 + lane) * p.num_q_heads]
                               : -INFINITY;
    const float wl = (lse == -INFINITY) ? 0.f : exp2f(lse - mmax);
    int k = 0;
    for (; k + 8 <= n; k += 8) {
      Vec v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = load(s0 + k + u);
#pragma unroll
      for (int u = 0; u < 8; ++u) add(__shfl_sync(0xffffffffu, wl, k + u), v[u]);
    }
    for (; k + 4 <= n; k += 4) {
      Vec v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = load(s0 + k + u);
#pragma unroll
      for (int u = 0; u < 4; ++u) add(__shfl_sync(0xffffffffu, wl, k + u), v[u]);
    }
    for (; k < n; ++k) add(__shfl_sync(0xffffffffu, wl, k), load(s0 + k));
  }
  const float inv = (wsum > 0.f) ? 1.f / wsum : 0.f;
  T* orow = static_cast<T*>(p.out) + b * p.out_stride + static_cast<int64_t>(qh) * D + lane * kPer;
#pragma unroll
  for (int i = 0; i < kPer; i += 2)
    *reinterpret_cast<uint32_t*>(orow + i) = pack2<T>(acc[i] * inv, acc[i + 1] * inv);
}

// ------------------------------------------------------------ host side
constexpr int kNW = 4;  // warps per CTA
constexpr int kNS = 2;  // TMA stages per warp
// Warps per CTA of the unsplit launch. One CTA streams one (sequence, KV head)
// through its warps' chunk loops, so the longest sequences' CTAs set a layer's
// length when the grid is one short wave; at head dim 64 a 16-token chunk is
// half the bytes, and eight warps keep those CTAs at the pace of the rest
// (Qwen2.5-0.5B geometry, 256 sequences: 54.4 against 60.6 us per layer;
// sixteen warps, one CTA per SM, 66 us). At head dim 128 four are faster
// (eight: 381 against 347 us per 8B layer).
template <int D>
constexpr int unsplit_warps() { return D == 64 ? 8 : kNW; }

int effective_part_tokens(int split_tokens, int max_blocks, int block_size) {
  return split_tokens > 0 ? split_tokens : max_blocks * block_size;
}

// Guards the per-device launch caches below against concurrent host threads.
std::mutex g_launch_mu;

// The dynamic shared-memory attribute is per function and per device; raise it
// only when a larger block table than any seen so far needs more.
template <typename K>
int reserve_smem(K kern, size_t smem, size_t (&configured)[64]) {
  std::lock_guard<std::mutex> lock(g_launch_mu);
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || configured[dev] < smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess)
      return fail(PS_ERR_CUDA, "ps_paged_decode: cannot reserve %zu B shared memory: %s", smem,
                  cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) configured[dev] = smem;
  }
  return PS_OK;
}

template <typename T, int D, int BS, int R>
int launch_decode(const DecodeParams& p, const CUtensorMap& km, const CUtensorMap& vm,
                  cudaStream_t s) {
  using SM = DecodeSmem<D, kNW, kNS>;
  const size_t smem = SM::bytes(p.table_cap);
  if (p.max_splits <= 1) {
    constexpr int NWU = unsplit_warps<D>();
    auto kern = paged_decode_kernel<T, D, NWU, kNS, BS, R, false>;
    static size_t configured[64] = {};
    const size_t smem_u = DecodeSmem<D, NWU, kNS>::bytes(p.table_cap);
    int st = reserve_smem(kern, smem_u, configured);
    if (st != PS_OK) return st;
    dim3 grid(p.num_kv_heads, 1, p.num_launch);
    const cudaError_t e = launch_pdl(kern, grid, dim3(NWU * 32), smem_u, s, p, km, vm);
    if (e != cudaSuccess)
      return fail(PS_ERR_CUDA, "ps_paged_decode: launch failed: %s", cudaGetErrorString(e));
    return check_launch("ps_paged_decode");
  }
  // Split-K: plan the (sequence, partition) units on the device, then one
  // persistent CTA per resident slot claims them; the grid does not depend on
  // the lengths, so the launch sequence can be captured in a CUDA graph.
  auto kern = paged_decode_kernel<T, D, kNW, kNS, BS, R, true>;
  static size_t configured[64] = {};
  int st = reserve_smem(kern, smem, configured);
  if (st != PS_OK) return st;
  static int occ_dev[64], occ_blocks[64];
  static size_t occ_smem[64] = {};
  int dev = 0, sms = 148, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int slot = (dev >= 0 && dev < 64) ? dev : 0;
  std::unique_lock<std::mutex> lock(g_launch_mu);
  if (occ_smem[slot] == smem && occ_dev[slot] == dev) {
    per_sm = occ_blocks[slot];
  } else {
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kNW * 32, smem);
    if (e != cudaSuccess || per_sm <= 0)
      return fail(PS_ERR_CUDA, "ps_paged_decode: occupancy query failed: %s", cudaGetErrorString(e));
    occ_smem[slot] = smem;
    occ_dev[slot] = dev;
    occ_blocks[slot] = per_sm;
  }
  lock.unlock();
  cudaError_t e = cudaSuccess;
  if (!p.planned) {
    e = launch_pdl(decode_plan_kernel, dim3(1), dim3(1024), 0, s, p);
    if (e != cudaSuccess)
      return fail(PS_ERR_CUDA, "ps_paged_decode(plan): launch failed: %s", cudaGetErrorString(e));
  }
  e = launch_pdl(kern, dim3(per_sm * sms), dim3(kNW * 32), smem, s, p, km, vm);
  if (e != cudaSuccess)
    return fail(PS_ERR_CUDA, "ps_paged_decode: launch failed: %s", cudaGetErrorString(e));
  const int warps = p.num_launch * p.num_q_heads;
  e = launch_pdl(decode_combine_kernel<T, D>, dim3((warps + 3) / 4), dim3(128), 0, s, p);
  if (e != cudaSuccess)
    return fail(PS_ERR_CUDA, "ps_paged_decode(combine): launch failed: %s",
                cudaGetErrorString(e));
  return check_launch("ps_paged_decode(combine)");
}

template <typename T, int D, int R>
int dispatch_bs(const DecodeParams& p, const CUtensorMap& km, const CUtensorMap& vm,
                cudaStream_t s, int block_size) {
  if (block_size == 8) return launch_decode<T, D, 8, R>(p, km, vm, s);
  if (block_size == 32) return launch_decode<T, D, 32, R>(p, km, vm, s);
  return launch_decode<T, D, 16, R>(p, km, vm, s);
}

template <typename T, int D>
int dispatch_rows(const DecodeParams& p, const CUtensorMap& km, const CUtensorMap& vm,
                  cudaStream_t s, int block_size) {
  return p.group > 8 ? dispatch_bs<T, D, 16>(p, km, vm, s, block_size)
                     : dispatch_bs<T, D, 8>(p, km, vm, s, block_size);
}

int dispatch_decode(const DecodeParams& p, const CUtensorMap& km, const CUtensorMap& vm,
                    cudaStream_t s, int dtype, int head_dim, int block_size) {
  if (dtype == PS_DTYPE_BF16)
    return head_dim == 128 ? dispatch_rows<__nv_bfloat16, 128>(p, km, vm, s, block_size)
                           : dispatch_rows<__nv_bfloat16, 64>(p, km, vm, s, block_size);
  return head_dim == 128 ? dispatch_rows<__half, 128>(p, km, vm, s, block_size)
                         : dispatch_rows<__half, 64>(p, km, vm, s, block_size);
}

}  // namespace
}  // namespace ps

using namespace ps;

extern "C" int64_t ps_paged_decode_workspace_bytes(int num_seqs, int num_q_heads, int head_dim,
                                                   int block_size, int max_blocks_per_seq,
                                                   int split_tokens) {
  if (num_seqs <= 0 || num_q_heads <= 0 || head_dim <= 0 || max_blocks_per_seq <= 0 ||
      block_size <= 0)
    return 0;
  const int part = split_tokens > 0 ? split_tokens : max_blocks_per_seq * block_size;
  const int64_t max_splits = (static_cast<int64_t>(max_blocks_per_seq) * block_size + part - 1) / part;
  if (max_splits <= 1) return 0;
  const int64_t rows = static_cast<int64_t>(num_seqs) * max_splits * num_q_heads;
  const int64_t o_bytes = ((rows * head_dim * 4) + 255) / 256 * 256;
  const int64_t lse_bytes = ((rows * 4) + 255) / 256 * 256;
  const int64_t item_bytes = ((static_cast<int64_t>(num_seqs) * max_splits * 4) + 255) / 256 * 256;
  return o_bytes + lse_bytes + item_bytes + 256;  // + the unit count
}

extern "C" int ps_paged_decode_order(const int32_t* ctx_lens, int num_seqs, int32_t* order,
                                     void* stream) {
  ps::NvtxRange nvtx_range("ps_paged_decode_order");
  const char* fn = "ps_paged_decode_order";
  if (num_seqs < 0 || num_seqs > 65535)
    return fail(PS_ERR_INVALID, "%s: num_seqs %d outside [0, 65535]", fn, num_seqs);
  if (num_seqs == 0) return PS_OK;
  if (!ctx_lens || !order) return fail(PS_ERR_INVALID, "%s: null pointer argument", fn);
  decode_order_kernel<<<1, 1024, 0, as_stream(stream)>>>(ctx_lens, num_seqs, order);
  return check_launch(fn);
}

extern "C" int ps_paged_decode(void* out, int64_t out_seq_stride, const void* query,
                               int64_t query_seq_stride, const void* k_pool, const void* v_pool,
                               int64_t num_blocks, const int32_t* block_tables,
                               int64_t block_table_stride, const int32_t* ctx_lens, int num_seqs,
                               int num_q_heads, int num_kv_heads, int head_dim, int block_size,
                               int max_blocks_per_seq, float scale, int split_tokens,
                               void* workspace, int64_t workspace_bytes, int dtype,
                               int32_t* device_error, void* stream) {
  ps::NvtxRange nvtx_range("ps_paged_decode");
  return ps_paged_decode_ordered(out, out_seq_stride, query, query_seq_stride, k_pool, v_pool,
                                 num_blocks, block_tables, block_table_stride, ctx_lens, num_seqs,
                                 num_q_heads, num_kv_heads, head_dim, block_size,
                                 max_blocks_per_seq, scale, split_tokens, workspace,
                                 workspace_bytes, dtype, nullptr, device_error, stream);
}

namespace {
// The step's new token of each sequence, for the fused append.
struct NewToken {
  const void* key;
  int64_t key_stride;
  const void* value;
  int64_t value_stride;
  const int64_t* slots;
};

// Argument checks shared by every decode entry point; on success fills the
// partition length (tokens), the partitions per sequence and the block-table
// window a partition spans. Returns PS_OK, or the status of the first failure
// with its message naming `fn`.
int validate_decode(const char* fn, const void* out, int64_t out_seq_stride, const void* query,
                    int64_t query_seq_stride, const void* k_pool, const void* v_pool,
                    int64_t num_blocks, const int32_t* block_tables, int64_t block_table_stride,
                    const int32_t* ctx_lens, int num_seqs, int num_q_heads, int num_kv_heads,
                    int head_dim, int block_size, int max_blocks_per_seq, int split_tokens,
                    int dtype, int* part_out, int* max_splits_out, int* table_cap_out) {
  if (dtype != PS_DTYPE_BF16 && dtype != PS_DTYPE_F16)
    return fail(PS_ERR_UNSUPPORTED, "%s: dtype %d unsupported (bf16/f16 only)", fn, dtype);
  if (head_dim != 64 && head_dim != 128)
    return fail(PS_ERR_UNSUPPORTED, "%s: head_dim %d unsupported (64 or 128)", fn, head_dim);
  if (block_size != 8 && block_size != 16 && block_size != 32)
    return fail(PS_ERR_UNSUPPORTED, "%s: block_size %d unsupported (8, 16 or 32)", fn,
                block_size);
  if (num_seqs < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_blocks <= 0 ||
      max_blocks_per_seq <= 0)
    return fail(PS_ERR_INVALID, "%s: bad sizes", fn);
  if (num_q_heads % num_kv_heads != 0)
    return fail(PS_ERR_INVALID, "%s: num_q_heads %d not divisible by num_kv_heads %d", fn,
                num_q_heads, num_kv_heads);
  const int group = num_q_heads / num_kv_heads;
  if (group > 16)
    return fail(PS_ERR_UNSUPPORTED, "%s: %d query heads per kv head unsupported (max 16)", fn, group);
  if (num_seqs == 0) return PS_OK;  // nothing to launch; the caller checks num_seqs too
  if (num_seqs > 65535 || num_kv_heads > 65535)
    return fail(PS_ERR_INVALID, "%s: too many sequences/heads for one launch", fn);
  if (!out || !query || !k_pool || !v_pool || !block_tables || !ctx_lens)
    return fail(PS_ERR_INVALID, "%s: null pointer argument", fn);
  if (block_table_stride < max_blocks_per_seq)
    return fail(PS_ERR_INVALID, "%s: block_table_stride < max_blocks_per_seq", fn);
  if (query_seq_stride < static_cast<int64_t>(num_q_heads) * head_dim ||
      out_seq_stride < static_cast<int64_t>(num_q_heads) * head_dim || (query_seq_stride % 8) ||
      (out_seq_stride % 8) || !aligned(query, 16) || !aligned(out, 16))
    return fail(PS_ERR_INVALID, "%s: query/out must be 16-byte aligned, strides >= Hq*D and %% 8", fn);
  if (!aligned(k_pool, 16) || !aligned(v_pool, 16))
    return fail(PS_ERR_INVALID, "%s: pools must be 16-byte aligned", fn);
  const int64_t rows = num_blocks * num_kv_heads * block_size;
  if (rows >= (int64_t(1) << 31))
    return fail(PS_ERR_INVALID, "%s: pool too large for 32-bit TMA row coordinates", fn);
  const int unit = block_size > kChunk ? block_size : kChunk;
  if (split_tokens < 0 || (split_tokens % unit))
    return fail(PS_ERR_INVALID, "%s: split_tokens must be >= 0 and a multiple of %d", fn, unit);
  const int part = effective_part_tokens(split_tokens, max_blocks_per_seq, block_size);
  const int max_splits = (max_blocks_per_seq * block_size + part - 1) / part;
  const int table_cap = (part + block_size - 1) / block_size;
  if (table_cap > 8192)
    return fail(PS_ERR_UNSUPPORTED, "%s: partition of %d blocks too long; set split_tokens", fn,
                table_cap);
  if (max_splits > 65535) return fail(PS_ERR_INVALID, "%s: too many partitions", fn);
  *part_out = part;
  *max_splits_out = max_splits;
  *table_cap_out = table_cap;
  return PS_OK;
}

int decode_entry(const char* fn, void* out, int64_t out_seq_stride, const void* query,
                 int64_t query_seq_stride, const void* k_pool, const void* v_pool,
                 int64_t num_blocks, const int32_t* block_tables, int64_t block_table_stride,
                 const int32_t* ctx_lens, int num_seqs, int num_q_heads, int num_kv_heads,
                 int head_dim, int block_size, int max_blocks_per_seq, float scale,
                 int split_tokens, void* workspace, int64_t workspace_bytes, int dtype,
                 const int32_t* seq_order, const NewToken* nt, int32_t* device_error,
                 void* stream, int num_launch = -1, bool planned = false) {
  int part = 0, max_splits = 0, table_cap = 0;
  int vst = validate_decode(fn, out, out_seq_stride, query, query_seq_stride, k_pool, v_pool,
                            num_blocks, block_tables, block_table_stride, ctx_lens, num_seqs,
                            num_q_heads, num_kv_heads, head_dim, block_size, max_blocks_per_seq,
                            split_tokens, dtype, &part, &max_splits, &table_cap);
  if (vst != PS_OK || num_seqs == 0) return vst;
  if (num_launch < 0) num_launch = num_seqs;
  if (num_launch == 0) return PS_OK;
  const int group = num_q_heads / num_kv_heads;
  const int64_t rows = num_blocks * num_kv_heads * block_size;

  DecodeParams p{};
  if (max_splits > 1) {
    const int64_t need = ps_paged_decode_workspace_bytes(num_seqs, num_q_heads, head_dim, block_size,
                                                         max_blocks_per_seq, split_tokens);
    if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
      return fail(PS_ERR_INVALID, "%s: split-K needs a 256-byte aligned workspace of %lld bytes",
                  fn, (long long)need);
    if (static_cast<int64_t>(num_seqs) * max_splits >= (int64_t(1) << 31))
      return fail(PS_ERR_INVALID, "%s: too many (sequence, partition) units", fn);
    const int64_t rows_ws = static_cast<int64_t>(num_seqs) * max_splits * num_q_heads;
    const int64_t o_bytes = ((rows_ws * head_dim * 4) + 255) / 256 * 256;
    const int64_t lse_bytes = ((rows_ws * 4) + 255) / 256 * 256;
    const int64_t item_bytes = ((static_cast<int64_t>(num_seqs) * max_splits * 4) + 255) / 256 * 256;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    p.ws_o = reinterpret_cast<float*>(ws);
    p.ws_lse = reinterpret_cast<float*>(ws + o_bytes);
    p.items = reinterpret_cast<int32_t*>(ws + o_bytes + lse_bytes);
    p.item_count = reinterpret_cast<int32_t*>(ws + o_bytes + lse_bytes + item_bytes);
    p.item_next = p.item_count + 1;
  }
  p.out = out;
  p.q = query;
  p.out_stride = out_seq_stride;
  p.q_stride = query_seq_stride;
  p.block_tables = block_tables;
  p.bt_stride = block_table_stride;
  p.ctx_lens = ctx_lens;
  p.num_blocks = num_blocks;
  p.num_seqs = num_seqs;
  p.num_launch = num_launch;
  p.planned = planned;
  p.num_q_heads = num_q_heads;
  p.num_kv_heads = num_kv_heads;
  p.group = group;
  p.max_blocks = max_blocks_per_seq;
  p.block_size = block_size;
  p.part_tokens = part;
  p.max_splits = max_splits;
  p.table_cap = table_cap;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.err = device_error;
  p.seq_order = seq_order;
  if (nt) {
    if (!nt->key || !nt->value || !nt->slots)
      return fail(PS_ERR_INVALID, "%s: null key/value/slot_mapping", fn);
    if (nt->key_stride < static_cast<int64_t>(num_kv_heads) * head_dim ||
        nt->value_stride < static_cast<int64_t>(num_kv_heads) * head_dim ||
        (nt->key_stride % 8) || (nt->value_stride % 8) || !aligned(nt->key, 16) ||
        !aligned(nt->value, 16))
      return fail(PS_ERR_INVALID,
                  "%s: key/value must be 16-byte aligned with strides >= Hkv*D and %% 8", fn);
    if (num_blocks * block_size >= (int64_t(1) << 31))
      return fail(PS_ERR_INVALID, "%s: pool of %lld slots exceeds 2^31", fn,
                  (long long)(num_blocks * block_size));
    p.k_pool_w = const_cast<void*>(k_pool);
    p.v_pool_w = const_cast<void*>(v_pool);
    p.new_k = nt->key;
    p.new_v = nt->value;
    p.new_k_stride = nt->key_stride;
    p.new_v_stride = nt->value_stride;
    p.new_slots = nt->slots;
    p.num_slots = num_blocks * block_size;
  }

  CUtensorMap km, vm;
  const int box = block_size < kChunk ? block_size : kChunk;
  int st = get_pool_tmap(k_pool, static_cast<uint64_t>(rows), head_dim, box, &km);
  if (st != PS_OK) return st;
  st = get_pool_tmap(v_pool, static_cast<uint64_t>(rows), head_dim, box, &vm);
  if (st != PS_OK) return st;

  cudaStream_t s = as_stream(stream);
  return dispatch_decode(p, km, vm, s, dtype, head_dim, block_size);
}
}  // namespace

extern "C" int ps_paged_decode_ordered(void* out, int64_t out_seq_stride, const void* query,
                                       int64_t query_seq_stride, const void* k_pool,
                                       const void* v_pool, int64_t num_blocks,
                                       const int32_t* block_tables, int64_t block_table_stride,
                                       const int32_t* ctx_lens, int num_seqs, int num_q_heads,
                                       int num_kv_heads, int head_dim, int block_size,
                                       int max_blocks_per_seq, float scale, int split_tokens,
                                       void* workspace, int64_t workspace_bytes, int dtype,
                                       const int32_t* seq_order, int32_t* device_error,
                                       void* stream) {
  ps::NvtxRange nvtx_range("ps_paged_decode_ordered");
  return decode_entry("ps_paged_decode", out, out_seq_stride, query, query_seq_stride, k_pool,
                      v_pool, num_blocks, block_tables, block_table_stride, ctx_lens, num_seqs,
                      num_q_heads, num_kv_heads, head_dim, block_size, max_blocks_per_seq, scale,
                      split_tokens, workspace, workspace_bytes, dtype, seq_order, nullptr,
                      device_error, stream);
}

extern "C" int ps_paged_decode_append(void* out, int64_t out_seq_stride, const void* query,
                                      int64_t query_seq_stride, const void* key,
                                      int64_t key_seq_stride, const void* value,
                                      int64_t value_seq_stride, const int64_t* slot_mapping,
                                      void* k_pool, void* v_pool, int64_t num_blocks,
                                      const int32_t* block_tables, int64_t block_table_stride,
                                      const int32_t* ctx_lens, int num_seqs, int num_q_heads,
                                      int num_kv_heads, int head_dim, int block_size,
                                      int max_blocks_per_seq, float scale, int split_tokens,
                                      void* workspace, int64_t workspace_bytes, int dtype,
                                      const int32_t* seq_order, int32_t* device_error,
                                      void* stream) {
  ps::NvtxRange nvtx_range("ps_paged_decode_append");
  const NewToken nt{key, key_seq_stride, value, value_seq_stride, slot_mapping};
  return decode_entry("ps_paged_decode_append", out, out_seq_stride, query, query_seq_stride,
                      k_pool, v_pool, num_blocks, block_tables, block_table_stride, ctx_lens,
                      num_seqs, num_q_heads, num_kv_heads, head_dim, block_size,
                      max_blocks_per_seq, scale, split_tokens, workspace, workspace_bytes, dtype,
                      seq_order, &nt, device_error, stream);
}

extern "C" int ps_paged_decode_listed(void* out, int64_t out_seq_stride, const void* query,
                                      int64_t query_seq_stride, const void* k_pool,
                                      const void* v_pool, int64_t num_blocks,
                                      const int32_t* block_tables, int64_t block_table_stride,
                                      const int32_t* ctx_lens, int num_seqs,
                                      const int32_t* seq_list, int num_listed, int num_q_heads,
                                      int num_kv_heads, int head_dim, int block_size,
                                      int max_blocks_per_seq, float scale, int split_tokens,
                                      void* workspace, int64_t workspace_bytes, int dtype,
                                      int32_t* device_error, void* stream) {
  ps::NvtxRange nvtx_range("ps_paged_decode_listed");
  const char* fn = "ps_paged_decode_listed";
  if (num_listed < 0 || num_listed > num_seqs)
    return fail(PS_ERR_INVALID, "%s: num_listed %d outside [0, num_seqs %d]", fn, num_listed,
                num_seqs);
  if (num_listed > 0 && !seq_list) return fail(PS_ERR_INVALID, "%s: null seq_list", fn);
  return decode_entry(fn, out, out_seq_stride, query, query_seq_stride, k_pool, v_pool,
                      num_blocks, block_tables, block_table_stride, ctx_lens, num_seqs,
                      num_q_heads, num_kv_heads, head_dim, block_size, max_blocks_per_seq, scale,
                      split_tokens, workspace, workspace_bytes, dtype, seq_list, nullptr,
                      device_error, stream, num_listed);
}

extern "C" int ps_paged_decode_plan(const int32_t* ctx_lens, int num_seqs,
                                    const int32_t* seq_order, int num_q_heads, int head_dim,
                                    int block_size, int max_blocks_per_seq, int split_tokens,
                                    void* workspace, int64_t workspace_bytes, void* stream) {
  ps::NvtxRange nvtx_range("ps_paged_decode_plan");
  const char* fn = "ps_paged_decode_plan";
  if (num_seqs < 0 || num_seqs > 65535 || num_q_heads <= 0 || max_blocks_per_seq <= 0)
    return fail(PS_ERR_INVALID, "%s: bad sizes", fn);
  if (head_dim != 64 && head_dim != 128)
    return fail(PS_ERR_UNSUPPORTED, "%s: head_dim %d unsupported (64 or 128)", fn, head_dim);
  if (block_size != 8 && block_size != 16 && block_size != 32)
    return fail(PS_ERR_UNSUPPORTED, "%s: block_size %d unsupported (8, 16 or 32)", fn,
                block_size);
  const int unit = block_size > kChunk ? block_size : kChunk;
  if (split_tokens < 0 || (split_tokens % unit))
    return fail(PS_ERR_INVALID, "%s: split_tokens must be >= 0 and a multiple of %d", fn, unit);
  const int part = effective_part_tokens(split_tokens, max_blocks_per_seq, block_size);
  const int max_splits = (max_blocks_per_seq * block_size + part - 1) / part;
  if (num_seqs == 0 || max_splits <= 1) return PS_OK;  // nothing is split: no plan
  if (max_splits > 65535) return fail(PS_ERR_INVALID, "%s: too many partitions", fn);
  if (!ctx_lens) return fail(PS_ERR_INVALID, "%s: null ctx_lens", fn);
  const int64_t need = ps_paged_decode_workspace_bytes(num_seqs, num_q_heads, head_dim, block_size,
                                                       max_blocks_per_seq, split_tokens);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
    return fail(PS_ERR_INVALID, "%s: needs a 256-byte aligned workspace of %lld bytes", fn,
                (long long)need);
  const int64_t rows_ws = static_cast<int64_t>(num_seqs) * max_splits * num_q_heads;
  const int64_t o_bytes = ((rows_ws * head_dim * 4) + 255) / 256 * 256;
  const int64_t lse_bytes = ((rows_ws * 4) + 255) / 256 * 256;
  const int64_t item_bytes = ((static_cast<int64_t>(num_seqs) * max_splits * 4) + 255) / 256 * 256;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  DecodeParams p{};
  p.ctx_lens = ctx_lens;
  p.num_seqs = num_seqs;
  p.num_launch = num_seqs;
  p.max_blocks = max_blocks_per_seq;
  p.block_size = block_size;
  p.part_tokens = part;
  p.max_splits = max_splits;
  p.seq_order = seq_order;
  p.items = reinterpret_cast<int32_t*>(ws + o_bytes + lse_bytes);
  p.item_count = reinterpret_cast<int32_t*>(ws + o_bytes + lse_bytes + item_bytes);
  p.item_next = p.item_count + 1;
  const cudaError_t e =
      launch_pdl(decode_plan_kernel, dim3(1), dim3(1024), 0, as_stream(stream), p);
  if (e != cudaSuccess) return fail(PS_ERR_CUDA, "%s: launch failed: %s", fn, cudaGetErrorString(e));
  return check_launch(fn);
}

extern "C" int ps_paged_decode_append_planned(
    void* out, int64_t out_seq_stride, const void* query, int64_t query_seq_stride,
    const void* key, int64_t key_seq_stride, const void* value, int64_t value_seq_stride,
    const int64_t* slot_mapping, void* k_pool, void* v_pool, int64_t num_blocks,
    const int32_t* block_tables, int64_t block_table_stride, const int32_t* ctx_lens,
    int num_seqs, int num_q_heads, int num_kv_heads, int head_dim, int block_size,
    int max_blocks_per_seq, float scale, int split_tokens, void* workspace,
    int64_t workspace_bytes, int dtype, const int32_t* seq_order, int32_t* device_error,
    void* stream) {
  ps::NvtxRange nvtx_range("ps_paged_decode_append_planned");
  const NewToken nt{key, key_seq_stride, value, value_seq_stride, slot_mapping};
  return decode_entry("ps_paged_decode_append_planned", out, out_seq_stride, query,
                      query_seq_stride, k_pool, v_pool, num_blocks, block_tables,
                      block_table_stride, ctx_lens, num_seqs, num_q_heads, num_kv_heads, head_dim,
                      block_size, max_blocks_per_seq, scale, split_tokens, workspace,
                      workspace_bytes, dtype, seq_order, &nt, device_error, stream, -1, true);
}

// ------------------------------------------------------------ allocation-free variant
// Split-K partials of ps_paged_decode_noalloc live in this file-scope device
// array instead of a caller-provided workspace. It is part of the library's
// device image, so every GPU that loads the library holds these bytes until
// the process exits, and all calls on a device share them.
namespace ps {
namespace {
constexpr int64_t kNoAllocScratchBytes = int64_t(64) << 20;  // 64 MiB per device
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};
unsigned long long g_noalloc_ctx[kMaxDevices] = {};  // context id the address belongs to

// Driver calls that identify the calling thread's current context, fetched
// through the runtime (the library does not link libcuda directly).
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);
CtxGetCurrentFn g_ctx_get_current = nullptr;
CtxGetIdFn g_ctx_get_id = nullptr;
std::once_flag g_ctx_fns_once;

void load_ctx_fns() {
  cudaDriverEntryPointQueryResult q;
  void* fn = nullptr;
  if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
  fn = nullptr;
  if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_ctx_get_id = reinterpret_cast<CtxGetIdFn>(fn);
}

// Unique id of the calling thread's current context; 0 when none is current
// or the driver cannot say.
unsigned long long current_ctx_id() {
  std::call_once(g_ctx_fns_once, load_ctx_fns);
  if (!g_ctx_get_current || !g_ctx_get_id) return 0;
  CUcontext c = nullptr;
  unsigned long long id = 0;
  if (g_ctx_get_current(&c) != CUDA_SUCCESS || c == nullptr) return 0;
  if (g_ctx_get_id(c, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of g_noalloc_scratch on the current device. In host code the
// symbol name is only a host-side handle, so the address is looked up with
// cudaGetSymbolAddress (with the device current) the first time a device
// needs it and cached. The cache is keyed by the device's context id: after
// cudaDeviceReset the context, and with it the array's address, is new, and
// the next call looks the address up again instead of using a stale one.
int noalloc_scratch(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return fail(PS_ERR_CUDA, "ps_paged_decode_noalloc: cudaGetDevice failed: %s",
                cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return fail(PS_ERR_UNSUPPORTED, "ps_paged_decode_noalloc: device %d out of range", dev);
  const unsigned long long ctx = current_ctx_id();
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr || ctx == 0 || ctx != g_noalloc_ctx[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(PS_ERR_CUDA, "ps_paged_decode_noalloc: cudaGetSymbolAddress failed: %s",
                  cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
    g_noalloc_ctx[dev] = current_ctx_id();  // the lookup made the primary context current
  }
  *out = g_noalloc_ptr[dev];
  return PS_OK;
}
}  // namespace
}  // namespace ps

extern "C" int ps_paged_decode_noalloc(void* out, int64_t out_seq_stride, const void* query,
                                       int64_t query_seq_stride, const void* k_pool,
                                       const void* v_pool, int64_t num_blocks,
                                       const int32_t* block_tables, int64_t block_table_stride,
                                       const int32_t* ctx_lens, int num_seqs, int num_q_heads,
                                       int num_kv_heads, int head_dim, int block_size,
                                       int max_blocks_per_seq, float scale, int split_tokens,
                                       int dtype, int32_t* device_error, void* stream) {
  ps::NvtxRange nvtx_range("ps_paged_decode_noalloc");
  const char* fn = "ps_paged_decode_noalloc";
  // The arguments are checked before the scratch is sized, so a bad argument
  // is reported as itself rather than as a request the scratch cannot hold.
  int part = 0, max_splits = 0, table_cap = 0;
  const int vst = validate_decode(fn, out, out_seq_stride, query, query_seq_stride, k_pool,
                                  v_pool, num_blocks, block_tables, block_table_stride, ctx_lens,
                                  num_seqs, num_q_heads, num_kv_heads, head_dim, block_size,
                                  max_blocks_per_seq, split_tokens, dtype, &part, &max_splits,
                                  &table_cap);
  if (vst != PS_OK || num_seqs == 0) return vst;
  const int64_t need = max_splits > 1
                           ? ps_paged_decode_workspace_bytes(num_seqs, num_q_heads, head_dim,
                                                             block_size, max_blocks_per_seq,
                                                             split_tokens)
                           : 0;
  if (need > kNoAllocScratchBytes)
    return fail(PS_ERR_INVALID,
                "%s: split-K partials need %lld bytes, more than the %lld-byte built-in scratch; "
                "use fewer sequences, a larger split_tokens, or ps_paged_decode with a workspace",
                fn, (long long)need, (long long)kNoAllocScratchBytes);
  void* scratch = nullptr;
  if (need > 0) {
    const int st = noalloc_scratch(&scratch);
    if (st != PS_OK) return st;
  }
  // Nothing in the scratch needs clearing between calls: the plan kernel of
  // each call rewrites the unit list and count and resets the claim counter
  // before the decode reads them, and the combine reads only partials written
  // by the same call.
  return decode_entry(fn, out, out_seq_stride, query, query_seq_stride, k_pool, v_pool,
                      num_blocks, block_tables, block_table_stride, ctx_lens, num_seqs,
                      num_q_heads, num_kv_heads, head_dim, block_size, max_blocks_per_seq, scale,
                      split_tokens, scratch, need > 0 ? kNoAllocScratchBytes : 0, dtype, nullptr,
                      nullptr, device_error, stream);
}
