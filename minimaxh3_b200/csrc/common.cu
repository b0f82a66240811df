// Host-side helpers of libmh3_b200: error reporting, tensor-map encoding,
// the library's device error word.
#include <mutex>
#include <string>

#include "mh3_internal.h"

namespace mh3 {

static thread_local std::string g_last_error;

int fail(int code, const char* msg) {
  g_last_error = msg ? msg : "";
  return code;
}

int fail_cuda(cudaError_t e, const char* what) {
  g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return (int)e;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

int encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, void* base, const cuuint64_t* dims,
                 const cuuint64_t* strides_bytes, const cuuint32_t* box, const cuuint32_t* elem_strides,
                 CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = get_encode();
  if (fn == nullptr) return fail(MH3_ERR_DRIVER, "cuTensorMapEncodeTiled entry point unavailable");
  CUresult r = fn(map, dtype, rank, base, dims, strides_bytes, box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    std::string msg = "cuTensorMapEncodeTiled failed (CUresult " + std::to_string((int)r) + ")";
    return fail(MH3_ERR_DRIVER, msg.c_str());
  }
  return MH3_OK;
}

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

void* current_context() {
  static std::once_flag once;
  static CtxGetCurrentFn fn = nullptr;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(ptr);
  });
  CUcontext ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != CUDA_SUCCESS) return nullptr;
  return ctx;
}

// One error word per device, in the module's global memory.
__device__ int g_device_error;

int* device_error_word() {
  constexpr int kMaxDevices = 64;
  static int* addr[kMaxDevices] = {};
  static void* ctx_of[kMaxDevices] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  // Looked up again when the device's context changed (e.g. after a device
  // reset): the module, and with it the word, is loaded anew there.
  void* ctx = current_context();
  if (addr[dev] == nullptr || ctx_of[dev] != ctx) {
    void* p = nullptr;
    addr[dev] = cudaGetSymbolAddress(&p, g_device_error) == cudaSuccess ? static_cast<int*>(p) : nullptr;
    ctx_of[dev] = ctx;
  }
  return addr[dev];
}

}  // namespace mh3

extern "C" int mh3_abi_version(void) { return MH3_ABI_VERSION; }

extern "C" const char* mh3_last_error(void) { return mh3::g_last_error.c_str(); }

extern "C" int* mh3_device_error_word(void) { return mh3::device_error_word(); }

extern "C" int mh3_copy_rows(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch, int64_t row_bytes,
                             int64_t rows, void* stream) {
  const mh3::NvtxRange nvtx_range("mh3_copy_rows");
  if (rows == 0 || row_bytes == 0) return MH3_OK;
  if (dst == nullptr || src == nullptr || rows < 0 || row_bytes < 0 || dst_pitch < row_bytes || src_pitch < row_bytes)
    return mh3::fail(MH3_ERR_INVALID, "mh3_copy_rows: bad pointers, pitches or sizes");
  cudaError_t e = cudaMemcpy2DAsync(dst, (size_t)dst_pitch, src, (size_t)src_pitch, (size_t)row_bytes, (size_t)rows,
                                    cudaMemcpyDefault, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MH3_OK : mh3::fail_cuda(e, "mh3_copy_rows");
}
