// C-ABI plumbing: version, per-thread last-error string, launch checks and the
// cuTensorMapEncodeTiled entry point (fetched from the driver through the
// runtime, so the library does not link libcuda directly).
#include <cudaTypedefs.h>

#include <mutex>

#include "capi_internal.h"
#include "common.cuh"

namespace ps {

namespace {
thread_local char g_last_error[512] = "no error";

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
cudaError_t g_encode_status = cudaSuccess;

void load_encode() {
  cudaDriverEntryPointQueryResult q;
  void* fn = nullptr;
  g_encode_status = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (g_encode_status == cudaSuccess && q == cudaDriverEntryPointSuccess) {
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
}
}  // namespace

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(PS_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  }
  return PS_OK;
}

int encode_tmap_16bit(CUtensorMap* map, void* base, int rank, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box,
                      CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, load_encode);
  if (g_encode == nullptr) {
    return fail(PS_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (%s)",
                cudaGetErrorString(g_encode_status));
  }
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
    if (i > 0) gstride[i - 1] = strides_bytes[i - 1];
  }
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, rank, base, gdim, gstride, bdim,
                        estride, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return fail(PS_ERR_CUDA, "cuTensorMapEncodeTiled failed with CUresult %d", static_cast<int>(r));
  }
  return PS_OK;
}

namespace {
struct TmapCacheEntry {
  const void* base = nullptr;
  uint64_t rows = 0;
  int d = 0;
  int box_rows = 0;
  CUtensorMap map;
};
thread_local TmapCacheEntry g_tmap_cache[128];
thread_local int g_tmap_next = 0;
}  // namespace

int get_pool_tmap(const void* pool, uint64_t rows, int head_dim, int box_rows, CUtensorMap* out) {
  for (auto& e : g_tmap_cache) {
    if (e.base == pool && e.rows == rows && e.d == head_dim && e.box_rows == box_rows) {
      *out = e.map;
      return PS_OK;
    }
  }
  const uint64_t dims[2] = {static_cast<uint64_t>(head_dim), rows};
  const uint64_t strides[1] = {static_cast<uint64_t>(head_dim) * 2};
  const uint32_t box[2] = {64, static_cast<uint32_t>(box_rows)};
  CUtensorMap map;
  int st = encode_tmap_16bit(&map, const_cast<void*>(pool), 2, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != PS_OK) return st;
  TmapCacheEntry& e = g_tmap_cache[g_tmap_next];
  g_tmap_next = (g_tmap_next + 1) % 128;
  e.base = pool;
  e.rows = rows;
  e.d = head_dim;
  e.box_rows = box_rows;
  e.map = map;
  *out = map;
  return PS_OK;
}

}  // namespace ps

namespace ps {
namespace {
// One thread waits, with the bound every kernel uses, on an mbarrier that
// nothing arrives at, then reports the timeout the way the kernels do.
__global__ void selftest_wait_timeout_kernel(int32_t* err) {
  __shared__ uint64_t bar;
  mbar_init(&bar, 1);
  fence_barrier_init();
  if (!mbar_wait_bounded(&bar, 0)) set_device_error(err, PS_DEVERR_TIMEOUT);
}
}  // namespace
}  // namespace ps

extern "C" int ps_selftest_wait_timeout(int32_t* device_error, void* stream) {
  ps::NvtxRange nvtx_range("ps_selftest_wait_timeout");
  if (!device_error) return ps::fail(PS_ERR_INVALID, "ps_selftest_wait_timeout: null device_error");
  ps::selftest_wait_timeout_kernel<<<1, 1, 0, ps::as_stream(stream)>>>(device_error);
  return ps::check_launch("ps_selftest_wait_timeout");
}

extern "C" int ps_abi_version(void) { return PS_ABI_VERSION; }

extern "C" const char* ps_last_error_string(void) { return ps::g_last_error; }
