// Read-only streaming of a device buffer: the HBM read bandwidth a kernel that
// only reads (as the paged decode nearly does) can reach on this GPU. Used as
// the measured read ceiling beside the copy bandwidth (which reads and writes).
//
// Every thread keeps eight 16-byte loads in flight (evict-first: the data is
// read once), consecutive threads read consecutive vectors, and the grid
// strides over the buffer. The loads are folded into an XOR of all 32-bit
// words so none can be dropped; that XOR is also a checksum a test can verify.
#include <algorithm>

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

}  // namespace
}  // namespace ps

using namespace ps;

extern "C" int ps_stream_read(const void* src, int64_t num_bytes, uint32_t* checksum,
                              int max_ctas, void* stream) {
  ps::NvtxRange nvtx_range("ps_stream_read");
  const char* fn = "ps_stream_read";
  if (num_bytes < 0 || max_ctas < 0) return fail(PS_ERR_INVALID, "%s: bad sizes", fn);
  if (num_bytes == 0) return PS_OK;
  if (!src || !checksum) return fail(PS_ERR_INVALID, "%s: null pointer argument", fn);
  if (!aligned(src, 16) || (num_bytes % 16) || !aligned(checksum, 4))
    return fail(PS_ERR_INVALID, "%s: buffer must be 16-byte aligned, num_bytes a multiple of 16",
                fn);
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t num_vec = num_bytes / 16;
  // 8 CTAs of 256 threads fill an SM's 2048 thread slots.
  int64_t ctas = max_ctas > 0 ? max_ctas : static_cast<int64_t>(sms) * 8;
  ctas = std::min<int64_t>(ctas, (num_vec + kStreamThreads - 1) / kStreamThreads);
  ctas = std::max<int64_t>(ctas, 1);
  stream_read_kernel<<<static_cast<unsigned>(ctas), kStreamThreads, 0, as_stream(stream)>>>(
      static_cast<const uint4*>(src), num_vec, checksum);
  return check_launch(fn);
}
