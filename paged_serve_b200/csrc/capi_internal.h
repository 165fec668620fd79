// Host-side helpers shared by the C-ABI entry points: status/error-string
// handling, argument checks and the TMA tensor-map encoder.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

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

// Encodes a tiled TMA descriptor over a 16-bit tensor with up to 5 dims
// (dims/strides innermost first; strides in bytes for dims 1..rank-1).
// Returns PS_OK or PS_ERR_CUDA with a message.
int encode_tmap_16bit(CUtensorMap* map, void* base, int rank, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box,
                      CUtensorMapSwizzle swizzle);

}  // namespace ps
