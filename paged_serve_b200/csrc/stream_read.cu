// Read-only streaming of a device buffer: the HBM read bandwidth a kernel that
// only reads (as the paged decode nearly does) can reach on this GPU. Used as
// the measured read ceiling beside the copy bandwidth (which reads and writes).
// Two ways to read, both folding every 32-bit word into an XOR (so no load can
// be dropped, and a test can verify the sum):
//
// - PS_STREAM_BULK: bulk asynchronous copies (cp.async.bulk, completion
//   counted on an mbarrier; no multicast) into per-warp shared-memory rings,
//   the way the decode's K/V arrive;
// - PS_STREAM_LOADS: every thread keeps eight 16-byte loads in flight
//   (evict-first), consecutive threads on consecutive vectors, grid-stride.
#include <algorithm>
#include <mutex>

#include "capi_internal.h"
#include "common.cuh"

namespace ps {
namespace {

constexpr int kStreamThreads = 256;
constexpr int kStreamUnroll = 8;

__global__ void __launch_bounds__(kStreamThreads)
    stream_read_kernel(const uint4* __restrict__ src, int64_t num_vec, uint32_t* checksum) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kStreamThreads;
  int64_t i = static_cast<int64_t>(blockIdx.x) * kStreamThreads + threadIdx.x;
  uint32_t acc = 0;
  for (; i + (kStreamUnroll - 1) * stride < num_vec; i += kStreamUnroll * stride) {
    uint4 r[kStreamUnroll];
#pragma unroll
    for (int u = 0; u < kStreamUnroll; ++u) r[u] = __ldcs(src + i + u * stride);
#pragma unroll
    for (int u = 0; u < kStreamUnroll; ++u) acc ^= r[u].x ^ r[u].y ^ r[u].z ^ r[u].w;
  }
  for (; i < num_vec; i += stride) {
    const uint4 r = __ldcs(src + i);
    acc ^= r.x ^ r.y ^ r.z ^ r.w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc ^= __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0 && acc != 0) atomicXor(checksum, acc);
}

// Bulk reader, shaped like the decode's K/V loads: 3 CTAs per SM, 4 warps per
// CTA, each warp an independent consumer with its own 2-stage ring of 8 KB
// chunks (one bulk copy each, completion counted on the stage's mbarrier).
// Warp g of G reads chunks g, g + G, ...
constexpr int kBulkWarps = 4;
constexpr int kBulkStages = 2;
constexpr int kBulkChunk = 8192;
constexpr int kBulkCtasPerSm = 3;
constexpr size_t kBulkSmem = kBulkWarps * kBulkStages * (kBulkChunk + 8) + 128;

__device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Every wait is bounded: a timeout sets PS_DEVERR_TIMEOUT, and the warp waits
// (bounded again) for its copies still in flight before the CTA's shared
// memory goes away.
__global__ void __launch_bounds__(kBulkWarps * 32)
    stream_read_bulk_kernel(const uint8_t* __restrict__ src, int64_t num_bytes,
                            uint32_t* checksum, int32_t* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                             ~static_cast<uintptr_t>(127));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint8_t* ring = smem + warp * kBulkStages * kBulkChunk;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBulkWarps * kBulkStages * kBulkChunk) +
                   warp * kBulkStages;
  const int64_t num_chunks = (num_bytes + kBulkChunk - 1) / kBulkChunk;
  const int64_t g = static_cast<int64_t>(blockIdx.x) * kBulkWarps + warp;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kBulkWarps;
  const int64_t mine = num_chunks > g ? (num_chunks - g + stride - 1) / stride : 0;
  if (lane == 0) {
    for (int i = 0; i < kBulkStages; ++i) mbar_init(&full[i], 1);
    fence_barrier_init();
  }
  __syncwarp();
  auto chunk_bytes = [&](int64_t k) -> uint32_t {
    return static_cast<uint32_t>(min64(kBulkChunk, num_bytes - (g + k * stride) * kBulkChunk));
  };
  auto issue = [&](int64_t k) {  // lane 0 only
    const int st = static_cast<int>(k % kBulkStages);
    const uint32_t bytes = chunk_bytes(k);
    mbar_arrive_expect_tx(&full[st], bytes);
    bulk_g2s(ring + st * kBulkChunk, src + (g + k * stride) * kBulkChunk, bytes, &full[st]);
  };
  if (lane == 0)
    for (int64_t k = 0; k < min64(kBulkStages, mine); ++k) issue(k);
  uint32_t acc = 0;
  bool ok = true;
  int64_t k = 0;
  for (; k < mine; ++k) {
    const int st = static_cast<int>(k % kBulkStages);
    ok = __all_sync(0xffffffffu,
                    mbar_wait_bounded(&full[st], static_cast<uint32_t>((k / kBulkStages) & 1)));
    if (!ok) break;
    const uint4* v = reinterpret_cast<const uint4*>(ring + st * kBulkChunk);
    const int n = static_cast<int>(chunk_bytes(k) / 16);
    for (int i = lane; i < n; i += 32) {
      const uint4 r = v[i];
      acc ^= r.x ^ r.y ^ r.z ^ r.w;
    }
    __syncwarp();  // every lane is done with this stage
    if (lane == 0 && k + kBulkStages < mine) {
      fence_proxy_async_smem();
      issue(k + kBulkStages);
    }
  }
  if (!ok && lane == 0) {
    set_device_error(err, PS_DEVERR_TIMEOUT);
    for (int64_t j = k; j < min64(mine, k + kBulkStages); ++j)
      (void)mbar_wait_bounded(&full[j % kBulkStages], static_cast<uint32_t>((j / kBulkStages) & 1));
  }
  __syncwarp();
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc ^= __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0 && acc != 0) atomicXor(checksum, acc);
}

}  // namespace
}  // namespace ps

using namespace ps;

extern "C" int ps_stream_read(const void* src, int64_t num_bytes, uint32_t* checksum, int method,
                              int32_t* device_error, void* stream) {
  ps::NvtxRange nvtx_range("ps_stream_read");
  const char* fn = "ps_stream_read";
  if (num_bytes < 0) return fail(PS_ERR_INVALID, "%s: bad sizes", fn);
  if (method != PS_STREAM_BULK && method != PS_STREAM_LOADS)
    return fail(PS_ERR_INVALID, "%s: unknown method %d", fn, method);
  if (num_bytes == 0) return PS_OK;
  if (!src || !checksum) return fail(PS_ERR_INVALID, "%s: null pointer argument", fn);
  if (!aligned(src, 16) || (num_bytes % 16) || !aligned(checksum, 4))
    return fail(PS_ERR_INVALID, "%s: buffer must be 16-byte aligned, num_bytes a multiple of 16",
                fn);
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaStream_t s = as_stream(stream);
  if (method == PS_STREAM_BULK) {
    static bool configured[64] = {};
    static std::mutex mu;
    {
      std::lock_guard<std::mutex> lock(mu);
      if (dev < 0 || dev >= 64 || !configured[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(
            stream_read_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
            static_cast<int>(kBulkSmem));
        if (e != cudaSuccess)
          return fail(PS_ERR_CUDA, "%s: cannot reserve shared memory: %s", fn,
                      cudaGetErrorString(e));
        if (dev >= 0 && dev < 64) configured[dev] = true;
      }
    }
    const int64_t chunks = (num_bytes + kBulkChunk - 1) / kBulkChunk;
    const int64_t warps_needed = chunks;
    const unsigned grid = static_cast<unsigned>(std::max<int64_t>(
        1, std::min<int64_t>(static_cast<int64_t>(sms) * kBulkCtasPerSm,
                             (warps_needed + kBulkWarps - 1) / kBulkWarps)));
    stream_read_bulk_kernel<<<grid, kBulkWarps * 32, kBulkSmem, s>>>(
        static_cast<const uint8_t*>(src), num_bytes, checksum, device_error);
    return check_launch(fn);
  }
  const int64_t num_vec = num_bytes / 16;
  // 8 CTAs of 256 threads fill an SM's 2048 thread slots.
  int64_t ctas = static_cast<int64_t>(sms) * 8;
  ctas = std::min<int64_t>(ctas, (num_vec + kStreamThreads - 1) / kStreamThreads);
  ctas = std::max<int64_t>(ctas, 1);
  stream_read_kernel<<<static_cast<unsigned>(ctas), kStreamThreads, 0, s>>>(
      static_cast<const uint4*>(src), num_vec, checksum);
  return check_launch(fn);
}
