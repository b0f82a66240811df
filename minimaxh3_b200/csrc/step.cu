// Step-residual cache reductions (runtime/step_cache.py:39-52).
//
// The reference decides per denoising step whether to skip the transformer's
// middle blocks from
//   rel = mean|h1 - h1_prev| / max(mean|h1_prev|, 1e-6)
// computed as h1.float(), h1_prev.float(), a difference, two abs, two means
// (about ten passes over the hidden state), followed by a clone of h1 for the
// next step.  mh3_step_diff reads h1 and h1_prev once, accumulates both sums
// in double precision with a fixed reduction order (deterministic for a given
// size), and can overwrite h1_prev with h1 in the same pass - the clone.
#include <algorithm>

#include "mh3_b200.h"
#include "mh3_internal.h"
#include "ptx.cuh"

namespace mh3 {
namespace step {

constexpr int kThreads = 256;
constexpr int kBlocks = 148 * 4;  // fixed grid: the reduction order depends only on n
constexpr int kUnroll = 4;        // 16-byte vector pairs loaded ahead per thread

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// Block b handles elements [b*chunk, min(n, (b+1)*chunk)), 16-byte vectors
// first and then the ragged tail; partial[b] = (sum|h1-prev|, sum|prev|).
template <typename T>
__global__ void __launch_bounds__(kThreads) diff_kernel(const T* __restrict__ h1, T* __restrict__ prev, long long n,
                                                        long long chunk, int copy, double2* __restrict__ partial) {
  constexpr int V = 16 / sizeof(T);
  const long long lo = (long long)blockIdx.x * chunk;
  const long long hi = min(n, lo + chunk);
  double sd = 0.0, sp = 0.0;
  if (lo < hi) {
    const long long nvec = (hi - lo) / V;  // lo is a multiple of V (chunk is)
    const uint4* a4 = reinterpret_cast<const uint4*>(h1 + lo);
    uint4* p4 = reinterpret_cast<uint4*>(prev + lo);
    // One 16-byte vector pair: per-vector fp32 partials folded into the double sums.
    auto fold = [&](const uint4& ua, const uint4& up) {
      const T* ea = reinterpret_cast<const T*>(&ua);
      const T* ep = reinterpret_cast<const T*>(&up);
      float fd = 0.0f, fp = 0.0f;
#pragma unroll
      for (int k = 0; k < V; ++k) {
        const float x = to_f<T>(ea[k]), y = to_f<T>(ep[k]);
        fd += fabsf(x - y);
        fp += fabsf(y);
      }
      sd += (double)fd;
      sp += (double)fp;
    };
    // kUnroll vectors' loads are issued before any is folded (enough bytes in
    // flight per SM for HBM); each thread still folds its vectors i,
    // i + kThreads, i + 2*kThreads, ... in that order, so the sums do not
    // depend on the unrolling.
    long long i = threadIdx.x;
    for (; i + (kUnroll - 1) * kThreads < nvec; i += kUnroll * kThreads) {
      uint4 ua[kUnroll], up[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        ua[u] = __ldcs(a4 + i + u * kThreads);
        up[u] = __ldcs(p4 + i + u * kThreads);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        fold(ua[u], up[u]);
        if (copy) __stcs(p4 + i + u * kThreads, ua[u]);
      }
    }
    for (; i < nvec; i += kThreads) {
      const uint4 ua = __ldcs(a4 + i);
      const uint4 up = __ldcs(p4 + i);
      fold(ua, up);
      if (copy) __stcs(p4 + i, ua);
    }
    for (long long e = lo + nvec * V + threadIdx.x; e < hi; e += kThreads) {  // ragged tail
      const float x = to_f<T>(h1[e]), y = to_f<T>(prev[e]);
      sd += (double)fabsf(x - y);
      sp += (double)fabsf(y);
      if (copy) prev[e] = h1[e];
    }
  }
  __shared__ double rd[kThreads / 32], rp[kThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sd += __shfl_xor_sync(0xffffffffu, sd, o);
    sp += __shfl_xor_sync(0xffffffffu, sp, o);
  }
  if ((threadIdx.x & 31) == 0) {
    rd[threadIdx.x >> 5] = sd;
    rp[threadIdx.x >> 5] = sp;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double a = 0.0, b = 0.0;
    for (int w = 0; w < kThreads / 32; ++w) {
      a += rd[w];
      b += rp[w];
    }
    partial[blockIdx.x] = make_double2(a, b);
  }
}

// sums = (sum_b partial[b].x, sum_b partial[b].y), summed in block order.
__global__ void finish_kernel(const double2* __restrict__ partial, int nb, double* __restrict__ sums) {
  __shared__ double rd[32], rp[32];
  double a = 0.0, b = 0.0;
  for (int i = threadIdx.x; i < nb; i += 32) {
    a += partial[i].x;
    b += partial[i].y;
  }
  rd[threadIdx.x] = a;
  rp[threadIdx.x] = b;
  __syncwarp();
  if (threadIdx.x == 0) {
    double x = 0.0, y = 0.0;
    for (int w = 0; w < 32; ++w) {
      x += rd[w];
      y += rp[w];
    }
    sums[0] = x;
    sums[1] = y;
  }
}

}  // namespace step
}  // namespace mh3

using namespace mh3;

extern "C" uint64_t mh3_step_diff_workspace_bytes(void) { return (uint64_t)step::kBlocks * sizeof(double2); }

extern "C" int mh3_step_diff(const void* h1, void* prev, int32_t dtype, int64_t n, int32_t copy, double* sums,
                             void* workspace, void* stream) {
  const mh3::NvtxRange nvtx_range("mh3_step_diff");
  if (n < 0) return fail(MH3_ERR_INVALID, "mh3_step_diff: negative size");
  if (!sums || (n > 0 && (!h1 || !prev || !workspace))) return fail(MH3_ERR_INVALID, "mh3_step_diff: null pointer");
  if (((uintptr_t)h1 & 15u) || ((uintptr_t)prev & 15u) || ((uintptr_t)workspace & 15u))
    return fail(MH3_ERR_INVALID, "mh3_step_diff: h1, prev and workspace must be 16-byte aligned");
  if (dtype != MH3_DTYPE_BF16 && dtype != MH3_DTYPE_F16 && dtype != MH3_DTYPE_F32)
    return fail(MH3_ERR_INVALID, "mh3_step_diff: dtype must be bf16, f16 or f32");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (n == 0) {
    const cudaError_t z = cudaMemsetAsync(sums, 0, 2 * sizeof(double), st);
    return z == cudaSuccess ? MH3_OK : fail_cuda(z, "mh3_step_diff memset");
  }
  const long long vec = dtype == MH3_DTYPE_F32 ? 4 : 8;
  long long chunk = (n + step::kBlocks - 1) / step::kBlocks;
  chunk = std::max<long long>(vec, (chunk + vec - 1) / vec * vec);  // whole 16-byte vectors per block
  double2* part = static_cast<double2*>(workspace);
#define MH3_DIFF(T)                                                                                            \
  step::diff_kernel<T><<<step::kBlocks, step::kThreads, 0, st>>>(static_cast<const T*>(h1), static_cast<T*>(prev), \
                                                                 n, chunk, copy, part)
  if (dtype == MH3_DTYPE_BF16)
    MH3_DIFF(__nv_bfloat16);
  else if (dtype == MH3_DTYPE_F16)
    MH3_DIFF(__half);
  else
    MH3_DIFF(float);
#undef MH3_DIFF
  step::finish_kernel<<<1, 32, 0, st>>>(part, step::kBlocks, sums);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MH3_OK : fail_cuda(e, "mh3_step_diff launch");
}
