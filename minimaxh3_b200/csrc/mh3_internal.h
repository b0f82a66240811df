// Host-side helpers shared by the translation units of libmh3_b200.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>
#include <stdint.h>
#include <string.h>

#include <type_traits>

#include "mh3_b200.h"

namespace mh3 {

// Record ``msg`` as this thread's last error and return ``code``.
int fail(int code, const char* msg);
// Record a CUDA error with context and return it as a positive code.
int fail_cuda(cudaError_t e, const char* what);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// dependency on libcuda).  Returns MH3_OK or MH3_ERR_DRIVER.
int encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, void* base, const cuuint64_t* dims,
                 const cuuint64_t* strides_bytes, const cuuint32_t* box, const cuuint32_t* elem_strides,
                 CUtensorMapSwizzle swizzle);

// The library's device error word on the current device.
int* device_error_word();

// The calling thread's current CUDA context (CUcontext), or null; through
// the runtime's driver entry point, so the library does not link libcuda.
void* current_context();

// NVTX range named after a C entry point, over its host-side work (argument
// checks and launches), so a profiler can attribute kernels to entry points
// (e.g. ncu --nvtx --nvtx-include "mh3_fp8_attention_fwd/").  NVTX3 is
// header-only: without an attached tool a push/pop is a pointer check, and
// the library gains no link dependency.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

}  // namespace mh3
