// Host-side helpers shared by the C-ABI entry points: status/error-string
// handling, argument checks and the TMA tensor-map encoder.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <nvtx3/nvToolsExt.h>

#include <cstdarg>
#include <cstdio>
#include <utility>

#include "../../include/paged_serve.h"

namespace ps {

// Records a message for ps_last_error_string() (per calling thread) and
// returns `status`, so call sites read `return fail(PS_ERR_INVALID, "...")`.
int fail(int status, const char* fmt, ...);

// Maps the launch status of the kernels just enqueued to PS_OK / PS_ERR_CUDA.
int check_launch(const char* what);

inline bool aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Marks the host-side span of one C-ABI call (validation, descriptor set-up,
// launch) as an NVTX range named after the entry point, so a profiler
// timeline shows which call enqueued which kernels. NVTX is header-only: with
// no profiler attached a push/pop costs one pointer check.
class NvtxRange {
 public:
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

// Launches `kernel` with programmatic stream serialization: it may start while
// the previous kernel in the stream drains, and must begin with pdl_wait()
// (common.cuh) before touching global memory. Inside a CUDA graph capture the
// dependency becomes a programmatic edge.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Encodes a tiled TMA descriptor over a 16-bit tensor with up to 5 dims
// (dims/strides innermost first; strides in bytes for dims 1..rank-1).
// Returns PS_OK or PS_ERR_CUDA with a message.
int encode_tmap_16bit(CUtensorMap* map, void* base, int rank, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box,
                      CUtensorMapSwizzle swizzle);

// Tensor map over a KV pool viewed as 2-D [rows][head_dim] of 16-bit elements
// (rows = num_blocks * num_kv_heads * block_size): box = 64 columns x
// box_rows rows, 128-byte swizzle. Cached per thread by (pool, rows, head_dim,
// box_rows), since the same pools are used by every layer of every step.
int get_pool_tmap(const void* pool, uint64_t rows, int head_dim, int box_rows, CUtensorMap* out);

}  // namespace ps
