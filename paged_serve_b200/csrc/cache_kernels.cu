// KV-cache append (optionally with RoPE fused on K) and block copy.
//
// Both are HBM-bound byte movers: every thread moves 16-byte vectors, each
// (token, kv-head) row is handled by head_dim/16 consecutive threads so a warp
// covers whole 256-byte rows of the input and of the pool tile it scatters to.
#include "capi_internal.h"
#include "common.cuh"

namespace ps {
namespace {

struct AppendParams {
  void* k_pool;
  void* v_pool;
  const void* key;
  const void* value;
  const int64_t* slots;
  const int64_t* positions;  // RoPE only
  const void* table;         // RoPE only: [table_positions][head_dim] (cos half | sin half)
  int64_t num_tokens;
  int64_t key_stride;
  int64_t value_stride;
  int64_t num_slots;  // num_blocks * block_size
  int64_t table_positions;
  int num_kv_heads;
  int block_size;
  FastDiv div_heads;  // by num_kv_heads
  FastDiv div_block;  // by block_size
  int32_t* err;
};

// One thread owns elements [c*8, c*8+8) and [D/2 + c*8, D/2 + c*8 + 8) of one
// (token, kv-head) row, c in [0, D/16): exactly the pairs that rotate_half mixes.
// A "chunk" is that (row, c) pair; chunk ids run row-major, so consecutive
// threads read consecutive 16-byte vectors of the input.
template <typename T, int D, bool kRope>
struct AppendChunk {
  int64_t slot;
  int64_t pos;
  int h;
  uint4 klo, khi, vlo, vhi;
};

// Issues every load of one chunk that does not depend on another (slot,
// position, the four K/V vectors); K/V are read once, so they are evict-first.
template <typename T, int D, bool kRope>
__device__ __forceinline__ void append_load(const AppendParams& p, uint32_t chunk,
                                            AppendChunk<T, D, kRope>& a) {
  constexpr int kThreadsPerRow = D / 16;
  const uint32_t row = chunk / kThreadsPerRow;  // token * num_kv_heads + head
  const int c = static_cast<int>(chunk % kThreadsPerRow);
  const uint32_t t = p.div_heads.div(row);
  a.h = static_cast<int>(row - t * p.num_kv_heads);
  a.slot = p.slots[t];
  a.pos = 0;
  if constexpr (kRope) a.pos = p.positions[t];
  const T* k = static_cast<const T*>(p.key) + t * p.key_stride + a.h * D;
  const T* v = static_cast<const T*>(p.value) + t * p.value_stride + a.h * D;
  const int lo = c * 8;
  const int hi = D / 2 + c * 8;
  a.klo = __ldcs(reinterpret_cast<const uint4*>(k + lo));
  a.khi = __ldcs(reinterpret_cast<const uint4*>(k + hi));
  a.vlo = __ldcs(reinterpret_cast<const uint4*>(v + lo));
  a.vhi = __ldcs(reinterpret_cast<const uint4*>(v + hi));
}

// Rotates K (RoPE) and writes the chunk's K and V vectors into the pools.
template <typename T, int D, bool kRope>
__device__ __forceinline__ void append_store(const AppendParams& p, uint32_t chunk,
                                             AppendChunk<T, D, kRope>& a) {
  constexpr int kThreadsPerRow = D / 16;
  const int c = static_cast<int>(chunk % kThreadsPerRow);
  const int lo = c * 8;
  const int hi = D / 2 + c * 8;
  if (a.slot < 0) return;  // padding token: nothing to write
  if (a.slot >= p.num_slots) {
    set_device_error(p.err, PS_DEVERR_SLOT);
    return;
  }
  const uint32_t blk = p.div_block.div(static_cast<uint32_t>(a.slot));
  const int off = static_cast<int>(static_cast<uint32_t>(a.slot) - blk * p.block_size);
  const int64_t dst =
      ((static_cast<int64_t>(blk) * p.num_kv_heads + a.h) * p.block_size + off) * D;
  uint4 klo = a.klo, khi = a.khi;
  if constexpr (kRope) {
    if (a.pos < 0 || a.pos >= p.table_positions) {
      set_device_error(p.err, PS_DEVERR_POSITION);
      return;
    }
    const T* row_cs = static_cast<const T*>(p.table) + a.pos * D;
    const uint4 cv = *reinterpret_cast<const uint4*>(row_cs + lo);          // cos[lo..lo+8)
    const uint4 sv = *reinterpret_cast<const uint4*>(row_cs + D / 2 + lo);  // sin[lo..lo+8)
    // Reference arithmetic (layers.py:77 with rotate_half at :49-59), every
    // operation rounded to T: out = T(T(k*cos) + T(rotate_half(k)*sin)),
    // rotate_half(k)[d] = -k[d+D/2] for d < D/2 and k[d-D/2] above. Pairs of
    // elements go through packed fp32 multiplies/adds and one packed rounding.
    const uint32_t* kl = reinterpret_cast<const uint32_t*>(&a.klo);
    const uint32_t* kh = reinterpret_cast<const uint32_t*>(&a.khi);
    const uint32_t* cs = reinterpret_cast<const uint32_t*>(&cv);
    const uint32_t* sn = reinterpret_cast<const uint32_t*>(&sv);
    uint32_t* ol = reinterpret_cast<uint32_t*>(&klo);
    uint32_t* oh = reinterpret_cast<uint32_t*>(&khi);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x = unpack2<T>(kl[i]);
      const float2 y = unpack2<T>(kh[i]);
      const float2 cc = unpack2<T>(cs[i]);
      const float2 sg = unpack2<T>(sn[i]);
      const float2 ny = make_float2(-y.x, -y.y);
      const float2 lo_kc = unpack2<T>(pack2<T>(__fmul2_rn(x, cc)));
      const float2 lo_rs = unpack2<T>(pack2<T>(__fmul2_rn(ny, sg)));
      const float2 hi_kc = unpack2<T>(pack2<T>(__fmul2_rn(y, cc)));
      const float2 hi_rs = unpack2<T>(pack2<T>(__fmul2_rn(x, sg)));
      ol[i] = pack2<T>(__fadd2_rn(lo_kc, lo_rs));
      oh[i] = pack2<T>(__fadd2_rn(hi_kc, hi_rs));
    }
  }
  // Streaming (evict-first) stores: the pool rows are not read back by this
  // launch, and leaving L2 to the inputs measured 2.8% faster per launch.
  T* kd = static_cast<T*>(p.k_pool) + dst;
  T* vd = static_cast<T*>(p.v_pool) + dst;
  __stcs(reinterpret_cast<uint4*>(kd + lo), klo);
  __stcs(reinterpret_cast<uint4*>(kd + hi), khi);
  __stcs(reinterpret_cast<uint4*>(vd + lo), a.vlo);
  __stcs(reinterpret_cast<uint4*>(vd + hi), a.vhi);
}

// One chunk per thread (two rows per thread, or a persistent grid-stride
// loop with the next chunk's loads issued before the current stores, measured
// slower). Launched with programmatic stream serialization: the CTAs of the
// next launch are resident when this one ends, which hides the launch gap of
// back-to-back per-layer appends.
template <typename T, int D, bool kRope>
__global__ void __launch_bounds__(256) cache_append_kernel(AppendParams p, uint32_t num_chunks) {
  pdl_trigger();
  pdl_wait();
  // The host guarantees num_chunks and num_blocks*block_size < 2^31.
  const uint32_t chunk = blockIdx.x * blockDim.x + threadIdx.x;
  if (chunk >= num_chunks) return;
  AppendChunk<T, D, kRope> a;
  append_load(p, chunk, a);
  append_store(p, chunk, a);
}

template <typename T, int D, bool kRope>
void launch_append(const AppendParams& p, cudaStream_t s) {
  const uint32_t chunks = static_cast<uint32_t>(p.num_tokens * p.num_kv_heads * (D / 16));
  const uint32_t grid = (chunks + 255) / 256;
  launch_pdl(cache_append_kernel<T, D, kRope>, dim3(grid), dim3(256), 0, s, p, chunks);
}

template <bool kRope>
int append_dispatch(const AppendParams& p, int head_dim, int dtype, cudaStream_t s) {
  if (dtype == PS_DTYPE_BF16) {
    if (head_dim == 128) launch_append<__nv_bfloat16, 128, kRope>(p, s);
    else launch_append<__nv_bfloat16, 64, kRope>(p, s);
  } else {
    if (head_dim == 128) launch_append<__half, 128, kRope>(p, s);
    else launch_append<__half, 64, kRope>(p, s);
  }
  return check_launch(kRope ? "ps_cache_append_rope" : "ps_cache_append");
}

int check_append_args(const char* fn, void* k_pool, void* v_pool, const void* key,
                      const void* value, const int64_t* slots, int64_t num_tokens,
                      int64_t key_stride, int64_t value_stride, int num_kv_heads, int head_dim,
                      int block_size, int64_t num_blocks, int dtype) {
  if (dtype != PS_DTYPE_BF16 && dtype != PS_DTYPE_F16)
    return fail(PS_ERR_UNSUPPORTED, "%s: dtype %d unsupported (bf16/f16 only)", fn, dtype);
  if (head_dim != 64 && head_dim != 128)
    return fail(PS_ERR_UNSUPPORTED, "%s: head_dim %d unsupported (64 or 128)", fn, head_dim);
  if (num_tokens < 0 || num_kv_heads <= 0 || block_size <= 0 || num_blocks <= 0)
    return fail(PS_ERR_INVALID, "%s: bad sizes (tokens %lld, kv heads %d, block %d, blocks %lld)",
                fn, (long long)num_tokens, num_kv_heads, block_size, (long long)num_blocks);
  if (num_tokens == 0) return PS_OK;
  if (!k_pool || !v_pool || !key || !value || !slots)
    return fail(PS_ERR_INVALID, "%s: null pointer argument", fn);
  if (key_stride < (int64_t)num_kv_heads * head_dim || value_stride < (int64_t)num_kv_heads * head_dim)
    return fail(PS_ERR_INVALID, "%s: token stride smaller than num_kv_heads*head_dim", fn);
  if ((key_stride % 8) || (value_stride % 8) || !aligned(key, 16) || !aligned(value, 16) ||
      !aligned(k_pool, 16) || !aligned(v_pool, 16))
    return fail(PS_ERR_INVALID, "%s: key/value/pools must be 16-byte aligned with strides %% 8 == 0",
                fn);
  if (num_tokens * num_kv_heads * (head_dim / 16) >= (int64_t(1) << 31))
    return fail(PS_ERR_INVALID, "%s: too many tokens for one launch", fn);
  if (num_blocks * block_size >= (int64_t(1) << 31))
    return fail(PS_ERR_INVALID, "%s: pool of %lld slots exceeds 2^31", fn,
                (long long)(num_blocks * block_size));
  return PS_OK;
}

// ------------------------------------------------------------- block copy
// Lists up to this many pairs are checked on the device for the call's
// contract (no destination repeated, none used as another pair's source);
// the check reads num_pairs pairs per pair, so longer lists go unchecked.
constexpr int64_t kCopyPairCheckMax = 4096;

// One CTA per (pair, layer, K|V). The pairs of one call run concurrently, so
// the call is well defined only when every destination is distinct and no
// destination is another pair's source. The (layer 0, K) CTA of each pair
// verifies that for its destination and reports a violation as
// PS_DEVERR_BLOCK_PAIRS (the copies still run; their result is then unspecified).
__global__ void __launch_bounds__(256) copy_blocks_kernel(uint8_t* k_pool, uint8_t* v_pool,
                                                          const int64_t* pairs, int64_t num_pairs,
                                                          int64_t layer_stride,
                                                          int64_t block_bytes, int64_t num_blocks,
                                                          int32_t* err) {
  const int64_t pair = blockIdx.x;
  const int layer = blockIdx.y >> 1;
  uint8_t* base = ((blockIdx.y & 1) ? v_pool : k_pool) + layer * layer_stride;
  const int64_t src = pairs[2 * pair];
  const int64_t dst = pairs[2 * pair + 1];
  if (src < 0 || src >= num_blocks || dst < 0 || dst >= num_blocks) {
    if (threadIdx.x == 0) set_device_error(err, PS_DEVERR_BLOCK_ID);
    return;
  }
  if (blockIdx.y == 0 && num_pairs <= kCopyPairCheckMax) {
    bool clash = false;
    for (int64_t j = threadIdx.x; j < num_pairs; j += blockDim.x)
      if (j != pair && (pairs[2 * j] == dst || pairs[2 * j + 1] == dst)) clash = true;
    if (__syncthreads_or(clash) && threadIdx.x == 0) set_device_error(err, PS_DEVERR_BLOCK_PAIRS);
  }
  const uint4* s = reinterpret_cast<const uint4*>(base + src * block_bytes);
  uint4* d = reinterpret_cast<uint4*>(base + dst * block_bytes);
  const int64_t n = block_bytes / 16;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) d[i] = s[i];
}

}  // namespace
}  // namespace ps

using namespace ps;

extern "C" int ps_cache_append(void* k_pool, void* v_pool, const void* key, const void* value,
                               const int64_t* slot_mapping, int64_t num_tokens,
                               int64_t key_token_stride, int64_t value_token_stride,
                               int num_kv_heads, int head_dim, int block_size, int64_t num_blocks,
                               int dtype, int32_t* device_error, void* stream) {
  ps::NvtxRange nvtx_range("ps_cache_append");
  int st = check_append_args("ps_cache_append", k_pool, v_pool, key, value, slot_mapping,
                             num_tokens, key_token_stride, value_token_stride, num_kv_heads,
                             head_dim, block_size, num_blocks, dtype);
  if (st != PS_OK || num_tokens == 0) return st;
  AppendParams p{};
  p.k_pool = k_pool;
  p.v_pool = v_pool;
  p.key = key;
  p.value = value;
  p.slots = slot_mapping;
  p.num_tokens = num_tokens;
  p.key_stride = key_token_stride;
  p.value_stride = value_token_stride;
  p.num_slots = num_blocks * block_size;
  p.num_kv_heads = num_kv_heads;
  p.block_size = block_size;
  p.div_heads = FastDiv(static_cast<uint32_t>(num_kv_heads));
  p.div_block = FastDiv(static_cast<uint32_t>(block_size));
  p.err = device_error;
  return append_dispatch<false>(p, head_dim, dtype, as_stream(stream));
}

extern "C" int ps_cache_append_rope(void* k_pool, void* v_pool, const void* key,
                                    const void* value, const int64_t* slot_mapping,
                                    const int64_t* positions, int64_t num_tokens,
                                    int64_t key_token_stride, int64_t value_token_stride,
                                    int num_kv_heads, int head_dim, int block_size,
                                    int64_t num_blocks, const void* cos_sin_table,
                                    int64_t table_positions, int rope_dim, int dtype,
                                    int32_t* device_error, void* stream) {
  ps::NvtxRange nvtx_range("ps_cache_append_rope");
  int st = check_append_args("ps_cache_append_rope", k_pool, v_pool, key, value, slot_mapping,
                             num_tokens, key_token_stride, value_token_stride, num_kv_heads,
                             head_dim, block_size, num_blocks, dtype);
  if (st != PS_OK || num_tokens == 0) return st;
  if (rope_dim != head_dim)
    return fail(PS_ERR_UNSUPPORTED, "ps_cache_append_rope: rope_dim %d != head_dim %d", rope_dim,
                head_dim);
  if (!positions || !cos_sin_table || table_positions <= 0)
    return fail(PS_ERR_INVALID, "ps_cache_append_rope: positions/table missing");
  if (!aligned(cos_sin_table, 16))
    return fail(PS_ERR_INVALID, "ps_cache_append_rope: cos_sin_table must be 16-byte aligned");
  AppendParams p{};
  p.k_pool = k_pool;
  p.v_pool = v_pool;
  p.key = key;
  p.value = value;
  p.slots = slot_mapping;
  p.positions = positions;
  p.table = cos_sin_table;
  p.table_positions = table_positions;
  p.num_tokens = num_tokens;
  p.key_stride = key_token_stride;
  p.value_stride = value_token_stride;
  p.num_slots = num_blocks * block_size;
  p.num_kv_heads = num_kv_heads;
  p.block_size = block_size;
  p.div_heads = FastDiv(static_cast<uint32_t>(num_kv_heads));
  p.div_block = FastDiv(static_cast<uint32_t>(block_size));
  p.err = device_error;
  return append_dispatch<true>(p, head_dim, dtype, as_stream(stream));
}

extern "C" int ps_copy_blocks(void* k_pool, void* v_pool, const int64_t* block_pairs,
                              int64_t num_pairs, int num_layers, int64_t layer_stride_bytes,
                              int64_t block_bytes, int64_t num_blocks, int32_t* device_error,
                              void* stream) {
  ps::NvtxRange nvtx_range("ps_copy_blocks");
  if (num_pairs < 0 || num_layers <= 0 || block_bytes <= 0 || num_blocks <= 0)
    return fail(PS_ERR_INVALID, "ps_copy_blocks: bad sizes");
  if (num_pairs == 0) return PS_OK;
  if (!k_pool || !v_pool || !block_pairs)
    return fail(PS_ERR_INVALID, "ps_copy_blocks: null pointer argument");
  if ((block_bytes % 16) || (layer_stride_bytes % 16) || !aligned(k_pool, 16) || !aligned(v_pool, 16))
    return fail(PS_ERR_INVALID, "ps_copy_blocks: pools, block_bytes and layer stride must be 16-byte aligned");
  if (num_layers > 1 && layer_stride_bytes < num_blocks * block_bytes)
    return fail(PS_ERR_INVALID, "ps_copy_blocks: layer stride overlaps the previous layer's pool");
  if (num_pairs > 0x7fffffff || num_layers > 32767)
    return fail(PS_ERR_INVALID, "ps_copy_blocks: too many pairs/layers for one launch");
  dim3 grid(static_cast<unsigned>(num_pairs), static_cast<unsigned>(2 * num_layers));
  copy_blocks_kernel<<<grid, 256, 0, as_stream(stream)>>>(
      static_cast<uint8_t*>(k_pool), static_cast<uint8_t*>(v_pool), block_pairs, num_pairs,
      layer_stride_bytes, block_bytes, num_blocks, device_error);
  return check_launch("ps_copy_blocks");
}

// ------------------------------------------------------------- swap in / out
namespace ps {
namespace {
constexpr int kSwapThreads = 256;
constexpr int kSwapUnroll = 8;  // 16-byte vectors in flight per thread (32 KB per CTA)

// Moves whole blocks between two pools that may live in different memories
// (HBM, or pinned host memory mapped into the device's address space). Work
// units are (layer, K|V, pair), pair fastest, so consecutive CTAs touch
// consecutive blocks of one layer; a grid smaller than the unit count strides.
// Every thread issues all of its loads before its stores, which keeps enough
// reads in flight to cover the host link's latency.
__global__ void __launch_bounds__(kSwapThreads) swap_blocks_kernel(
    uint8_t* dst_k, uint8_t* dst_v, const uint8_t* src_k, const uint8_t* src_v,
    const int64_t* pairs, int64_t num_pairs, int64_t units, int64_t dst_layer_stride,
    int64_t src_layer_stride, int64_t block_bytes, int64_t dst_blocks, int64_t src_blocks,
    int32_t* err) {
  const int64_t vecs = block_bytes / 16;
  for (int64_t u = blockIdx.x; u < units; u += gridDim.x) {
    const int64_t pair = u % num_pairs;
    const int64_t lk = u / num_pairs;  // layer * 2 + (0 = K, 1 = V)
    const int64_t layer = lk >> 1;
    const int64_t src = pairs[2 * pair];
    const int64_t dst = pairs[2 * pair + 1];
    if (src < 0 || src >= src_blocks || dst < 0 || dst >= dst_blocks) {
      if (threadIdx.x == 0) set_device_error(err, PS_DEVERR_BLOCK_ID);
      continue;
    }
    const uint4* s = reinterpret_cast<const uint4*>(
        ((lk & 1) ? src_v : src_k) + layer * src_layer_stride + src * block_bytes);
    uint4* d = reinterpret_cast<uint4*>(((lk & 1) ? dst_v : dst_k) + layer * dst_layer_stride +
                                        dst * block_bytes);
    for (int64_t base = 0; base < vecs; base += kSwapThreads * kSwapUnroll) {
      uint4 r[kSwapUnroll];
#pragma unroll
      for (int j = 0; j < kSwapUnroll; ++j) {
        const int64_t i = base + j * kSwapThreads + threadIdx.x;
        if (i < vecs) r[j] = s[i];
      }
#pragma unroll
      for (int j = 0; j < kSwapUnroll; ++j) {
        const int64_t i = base + j * kSwapThreads + threadIdx.x;
        if (i < vecs) d[i] = r[j];
      }
    }
  }
}

// The address a kernel on the current device uses for `p`: device memory of
// this device, or pinned host memory mapped into its address space. Pageable
// host memory and other devices' memory are refused (the kernel would fault on
// the former and must not touch the latter).
int device_address(const void* p, const char* fn, const char* what, const void** out,
                   bool* on_host = nullptr) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return fail(PS_ERR_INVALID, "%s: %s is not memory CUDA knows", fn, what);
  }
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(PS_ERR_CUDA, "%s: no current device", fn);
  switch (a.type) {
    case cudaMemoryTypeDevice:
    case cudaMemoryTypeManaged:
      if (a.device != dev)
        return fail(PS_ERR_INVALID, "%s: %s lives on device %d, not the current device %d", fn,
                    what, a.device, dev);
      *out = a.devicePointer != nullptr ? a.devicePointer : p;
      return PS_OK;
    case cudaMemoryTypeHost:
      if (a.devicePointer == nullptr)
        return fail(PS_ERR_INVALID, "%s: %s is pinned host memory not mapped into the device", fn,
                    what);
      *out = a.devicePointer;
      if (on_host != nullptr) *on_host = true;
      return PS_OK;
    default:
      return fail(PS_ERR_INVALID,
                  "%s: %s is pageable host memory; pin it (cudaHostAlloc or torch pin_memory)", fn,
                  what);
  }
}
}  // namespace
}  // namespace ps

extern "C" int ps_swap_blocks(void* dst_k_pool, void* dst_v_pool, int64_t dst_num_blocks,
                              int64_t dst_layer_stride_bytes, const void* src_k_pool,
                              const void* src_v_pool, int64_t src_num_blocks,
                              int64_t src_layer_stride_bytes, const int64_t* block_pairs,
                              int64_t num_pairs, int num_layers, int64_t block_bytes, int max_ctas,
                              int32_t* device_error, void* stream) {
  ps::NvtxRange nvtx_range("ps_swap_blocks");
  const char* fn = "ps_swap_blocks";
  if (num_pairs < 0 || num_layers <= 0 || block_bytes <= 0 || dst_num_blocks <= 0 ||
      src_num_blocks <= 0 || max_ctas < 0)
    return fail(PS_ERR_INVALID, "%s: bad sizes", fn);
  if (num_pairs == 0) return PS_OK;
  if (!dst_k_pool || !dst_v_pool || !src_k_pool || !src_v_pool || !block_pairs)
    return fail(PS_ERR_INVALID, "%s: null pointer argument", fn);
  if ((block_bytes % 16) || (dst_layer_stride_bytes % 16) || (src_layer_stride_bytes % 16))
    return fail(PS_ERR_INVALID, "%s: block_bytes and layer strides must be multiples of 16", fn);
  if (num_layers > 1 && (dst_layer_stride_bytes < dst_num_blocks * block_bytes ||
                         src_layer_stride_bytes < src_num_blocks * block_bytes))
    return fail(PS_ERR_INVALID, "%s: a layer stride overlaps the previous layer's pool", fn);
  if (num_pairs > (int64_t(1) << 40) / (2 * num_layers))
    return fail(PS_ERR_INVALID, "%s: too many pairs for one launch", fn);
  const void* ptrs[5] = {dst_k_pool, dst_v_pool, src_k_pool, src_v_pool, block_pairs};
  const char* names[5] = {"dst_k_pool", "dst_v_pool", "src_k_pool", "src_v_pool", "block_pairs"};
  const void* dev[5];
  bool host_side = false;
  for (int i = 0; i < 5; ++i) {
    bool on_host = false;
    int st = device_address(ptrs[i], fn, names[i], &dev[i], &on_host);
    if (i < 4) host_side = host_side || on_host;
    if (st != PS_OK) return st;
    if (i < 4 && !aligned(dev[i], 16))
      return fail(PS_ERR_INVALID, "%s: %s must be 16-byte aligned", fn, names[i]);
  }
  if (!aligned(dev[4], 8)) return fail(PS_ERR_INVALID, "%s: block_pairs must be 8-byte aligned", fn);
  const int64_t units = num_pairs * num_layers * 2;
  int sms = 148;
  int device = 0;
  if (cudaGetDevice(&device) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  // 32 CTAs keep a PCIe Gen5 x16 link saturated (every cap from 16 to 4 per SM
  // moves the same ~52 GB/s), leaving the other SMs to concurrent work; an
  // HBM-to-HBM move gets two CTAs per SM.
  const int64_t cap = max_ctas > 0 ? max_ctas : (host_side ? 32 : 2 * static_cast<int64_t>(sms));
  const unsigned grid = static_cast<unsigned>(units < cap ? units : cap);
  swap_blocks_kernel<<<grid, kSwapThreads, 0, as_stream(stream)>>>(
      static_cast<uint8_t*>(const_cast<void*>(dev[0])),
      static_cast<uint8_t*>(const_cast<void*>(dev[1])), static_cast<const uint8_t*>(dev[2]),
      static_cast<const uint8_t*>(dev[3]), static_cast<const int64_t*>(dev[4]), num_pairs, units,
      dst_layer_stride_bytes, src_layer_stride_bytes, block_bytes, dst_num_blocks,
      src_num_blocks, device_error);
  return check_launch(fn);
}

// ------------------------------------------------------------- step metadata
namespace ps {
namespace {
// One thread per (sequence, row of the padded [B, query_len] step layout): the
// real tokens of sequence b are its last q_lens[b] rows (left padding); row r
// holds logical position ctx_before[b] + r - (query_len - q_lens[b]).
__global__ void __launch_bounds__(256) build_slot_mapping_kernel(
    int64_t* slots, int64_t* positions, const int32_t* tables, int64_t bt_stride,
    const int32_t* ctx_before, const int32_t* q_lens, int num_seqs, int query_len,
    int block_size, int max_blocks, int64_t num_blocks, int32_t* err) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(num_seqs) * query_len) return;
  const int b = static_cast<int>(i / query_len);
  const int r = static_cast<int>(i % query_len);
  const int ql = q_lens[b];
  int64_t slot = -1, pos = -1;
  if (ql < 0 || ql > query_len) {
    if (r == 0) set_device_error(err, PS_DEVERR_LENGTH);
  } else if (r >= query_len - ql) {
    const int pad = query_len - ql;
    pos = static_cast<int64_t>(ctx_before[b]) + (r - pad);
    const int64_t lb = pos / block_size;
    if (pos < 0 || lb >= max_blocks) {
      set_device_error(err, PS_DEVERR_LENGTH);
      pos = -1;
    } else {
      const int32_t blk = tables[b * bt_stride + lb];
      if (blk < 0 || blk >= num_blocks) {
        set_device_error(err, PS_DEVERR_BLOCK_ID);
      } else {
        slot = static_cast<int64_t>(blk) * block_size + pos % block_size;
      }
    }
  }
  slots[i] = slot;
  if (positions != nullptr) positions[i] = slot >= 0 ? pos : -1;
}
}  // namespace
}  // namespace ps

extern "C" int ps_build_slot_mapping(int64_t* slot_mapping, int64_t* positions,
                                     const int32_t* block_tables, int64_t block_table_stride,
                                     const int32_t* ctx_before, const int32_t* q_lens,
                                     int num_seqs, int query_len, int block_size,
                                     int max_blocks_per_seq, int64_t num_blocks,
                                     int32_t* device_error, void* stream) {
  ps::NvtxRange nvtx_range("ps_build_slot_mapping");
  const char* fn = "ps_build_slot_mapping";
  if (num_seqs < 0 || query_len < 0 || block_size <= 0 || max_blocks_per_seq <= 0 ||
      num_blocks <= 0)
    return fail(PS_ERR_INVALID, "%s: bad sizes", fn);
  const int64_t n = static_cast<int64_t>(num_seqs) * query_len;
  if (n == 0) return PS_OK;
  if (!slot_mapping || !block_tables || !ctx_before || !q_lens)
    return fail(PS_ERR_INVALID, "%s: null pointer argument", fn);
  if (block_table_stride < max_blocks_per_seq)
    return fail(PS_ERR_INVALID, "%s: block_table_stride < max_blocks_per_seq", fn);
  if (n >= (int64_t(1) << 31)) return fail(PS_ERR_INVALID, "%s: too many rows", fn);
  build_slot_mapping_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, as_stream(stream)>>>(
      slot_mapping, positions, block_tables, block_table_stride, ctx_before, q_lens, num_seqs,
      query_len, block_size, max_blocks_per_seq, num_blocks, device_error);
  return check_launch(fn);
}
