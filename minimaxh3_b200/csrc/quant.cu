#include <algorithm>
#include <string>
// e4m3 quantisation kernels (HBM-bound, CUDA cores).
//
//  * mh3_quantize_qkv: the drop-in path's Q/K/V quantisation, with the
//    reference's arithmetic (kernels/fp8_attention.py:39-170, :338).  The
//    reference walks each (b,h)'s V serially in one program (40 programs at
//    H=40, :122-170) and materialises an fp32 copy of K for its mean (:338);
//    here one grid-wide pass gathers per-chunk K sums and V absmax, a small
//    kernel finishes them in a fixed order (deterministic), and one 128-row
//    block per CTA is quantised for each of Q, K and V.
//  * mh3_quantize_rows: per-row scales for the FP8 linear
//    (kernels/fp8_linear.py:8-42).
//
// Quotients are correctly rounded (IEEE round-to-nearest, see div_rn_by) and
// the e4m3 cast is RNE with saturation at +-448 (the reference's clamp), so
// the bytes match the CPU restatement.
#include <mutex>

#include "mh3_internal.h"
#include "ptx.cuh"

namespace mh3 {
namespace quant {

constexpr int kThreads = 256;
constexpr int kBlockRows = 128;  // rows per scale block (fp8_attention.py:52, :93)
constexpr int kStatRows = 256;   // rows per K/V statistics chunk

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&x)[8]) {
  if constexpr (std::is_same<T, float>::value) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    return;
  }
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (std::is_same<T, __half>::value) {
      const __half2 h2 = *reinterpret_cast<const __half2*>(&w[i]);
      const float2 f = __half22float2(h2);
      x[2 * i] = f.x;
      x[2 * i + 1] = f.y;
    } else {
      const __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
      const float2 f = __bfloat1622float2(h2);
      x[2 * i] = f.x;
      x[2 * i + 1] = f.y;
    }
  }
}

// 8 packed 16-bit values -> floats (same conversion as load8).
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float (&x)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (std::is_same<T, __half>::value) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      x[2 * i] = f.x;
      x[2 * i + 1] = f.y;
    } else {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
      x[2 * i] = f.x;
      x[2 * i + 1] = f.y;
    }
  }
}

__device__ __forceinline__ float clamp448(float x) { return fminf(fmaxf(x, -448.0f), 448.0f); }

// x / s rounded to nearest even, given r = 1/s rounded to nearest (``__frcp_rn``,
// once per scale): Markstein's correction step - q = x*r, the remainder
// e = x - s*q is exact in one FMA, q + e*r rounds to the correctly rounded
// quotient (P. Markstein, "Computation of elementary functions on the IBM
// RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990; also the
// "Handbook of Floating-Point Arithmetic", ch. on division).  Holds while the
// quotient is a normal float; the quotients here are at most 448 in
// magnitude, and ones too small to be normal round to 0 in e4m3 and f16 alike.
// Three FMA-pipe operations where an IEEE division takes about ten: the
// quantisation kernels are otherwise issue-bound rather than HBM-bound.
__device__ __forceinline__ float div_rn_by(float x, float s, float r) {
  const float q = x * r;
  const float e = fmaf(-s, q, x);
  return fmaf(e, r, q);
}

// 8 floats -> 8 e4m3 bytes (element 0 in the lowest byte).
__device__ __forceinline__ uint2 pack8_e4m3(const float (&y)[8]) {
  uint32_t lo = cvt_e4m3x2_f32(y[1], y[0]) | (cvt_e4m3x2_f32(y[3], y[2]) << 16);
  uint32_t hi = cvt_e4m3x2_f32(y[5], y[4]) | (cvt_e4m3x2_f32(y[7], y[6]) << 16);
  return make_uint2(lo, hi);
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int i = 1; i < kThreads / 32; ++i) r = fmaxf(r, red[i]);
  return r;
}

// Per-chunk column sums of K and column absmax of V.
// part layout: [B*H, nchunk, D] (sums) and the same for absmax.
template <typename T, int D>
__global__ void __launch_bounds__(kThreads) kv_stats_kernel(const T* __restrict__ k, long long ksb, long long ksh,
                                                            long long kss, const T* __restrict__ v, long long vsb,
                                                            long long vsh, long long vss, int S, int H,
                                                            float* __restrict__ part_sum,
                                                            float* __restrict__ part_amax) {
  constexpr int CG = D / 8;           // column groups of 8 channels
  constexpr int RL = kThreads / CG;   // row lanes
  __shared__ float s_sum[RL][D];
  __shared__ float s_max[RL][D];
  const int chunk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int cg = threadIdx.x % CG, rl = threadIdx.x / CG;
  const int r_begin = chunk * kStatRows;
  const int r_end = min(S, r_begin + kStatRows);
  const T* kp = k + b * ksb + h * ksh + cg * 8;
  const T* vp = v + b * vsb + h * vsh + cg * 8;
  float sum[8], amax[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) sum[i] = 0.0f, amax[i] = 0.0f;
  for (int r = r_begin + rl; r < r_end; r += RL) {
    float xk[8], xv[8];
    load8(kp + (long long)r * kss, xk);
    load8(vp + (long long)r * vss, xv);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      sum[i] += xk[i];
      amax[i] = fmaxf(amax[i], fabsf(xv[i]));
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    s_sum[rl][cg * 8 + i] = sum[i];
    s_max[rl][cg * 8 + i] = amax[i];
  }
  __syncthreads();
  const int nchunk = gridDim.x;
  for (int d = threadIdx.x; d < D; d += kThreads) {
    float a = 0.0f, m = 0.0f;
    for (int i = 0; i < RL; ++i) {
      a += s_sum[i][d];
      m = fmaxf(m, s_max[i][d]);
    }
    const long long o = ((long long)(b * H + h) * nchunk + chunk) * D + d;
    part_sum[o] = a;
    part_amax[o] = m;
  }
}

// k_mean = sum / S and scale_v = max(absmax, 1e-12) / 448, chunks in order.
template <int D>
__global__ void kv_finalize_kernel(const float* __restrict__ part_sum, const float* __restrict__ part_amax,
                                   int nchunk, int S, float* __restrict__ k_mean, float* __restrict__ scale_v) {
  const int bh = blockIdx.x;
  const int d = threadIdx.x;
  if (d >= D) return;
  float a = 0.0f, m = 0.0f;
  for (int c = 0; c < nchunk; ++c) {
    const long long o = ((long long)bh * nchunk + c) * D + d;
    a += part_sum[o];
    m = fmaxf(m, part_amax[o]);
  }
  k_mean[(long long)bh * D + d] = a / (float)S;
  scale_v[(long long)bh * D + d] = fmaxf(m, 1.0e-12f) / 448.0f;
}

enum Mode { kQ = 0, kK = 1, kV = 2 };

// One 128-row block of one (b, h): transform, block absmax (Q, K), divide,
// clamp, e4m3.  Output contiguous [B,H,S,D]; scale [B,H,nblk].
// The block is held as raw 16-byte row pieces (8 channels x R rows per
// thread, 4 registers each) and converted twice - once for the absmax, once
// for the output - so that three CTAs fit on an SM and keep enough loads in
// flight for HBM.
template <typename T, int D, int MODE, bool OUT_F16 = false>
__global__ void __launch_bounds__(kThreads, 3) block_quant_kernel(const T* __restrict__ x, long long sb, long long sh,
                                                                  long long ss, int S, int H, float premul,
                                                                  const float* __restrict__ chan /* mean or sv */,
                                                                  uint8_t* __restrict__ out, float* __restrict__ scale) {
  constexpr int CG = D / 8;
  constexpr int RL = kThreads / CG;
  constexpr int R = kBlockRows / RL;  // rows per thread
  __shared__ float red[kThreads / 32];
  const int blk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int nblk = (S + kBlockRows - 1) / kBlockRows;
  if (blk >= nblk) return;
  const int cg = threadIdx.x % CG, rl = threadIdx.x / CG;
  const T* xp = x + b * sb + h * sh + cg * 8;
  const long long bh = (long long)b * H + h;
  uint4 raw[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int row = blk * kBlockRows + rl + r * RL;
    raw[r] = row < S ? __ldg(reinterpret_cast<const uint4*>(xp + (long long)row * ss)) : make_uint4(0u, 0u, 0u, 0u);
  }
  float c8[8], r8[8];
  if (MODE != kQ) {
#pragma unroll
    for (int i = 0; i < 8; ++i) c8[i] = __ldg(chan + bh * D + cg * 8 + i);
  }
  if (MODE == kV) {
#pragma unroll
    for (int i = 0; i < 8; ++i) r8[i] = __frcp_rn(c8[i]);
  }
  // transform (masked rows are 0, fp8_attention.py:69, :111)
  auto value = [&](int r, float (&v)[8]) {
    const int row = blk * kBlockRows + rl + r * RL;
    unpack8<T>(raw[r], v);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (MODE == kQ) v[i] = v[i] * premul;                 // :69
      if (MODE == kK) v[i] = row < S ? v[i] - c8[i] : 0.0f;  // :111
    }
  };
  float s = 1.0f;
  if (MODE != kV) {
    float amax = 0.0f;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float v[8];
      value(r, v);
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    }
    const float bm = block_max(amax, red);             // :70, :112
    s = fmaxf(bm, 1.0e-12f) / 448.0f;                  // :71, :113
    if (threadIdx.x == 0) scale[bh * nblk + blk] = s;
  }
  const float rs = __frcp_rn(s);
  // Convert again from the raw pieces instead of keeping R*8 floats alive
  // across the reduction (the empty asm hides the first conversion from CSE).
#pragma unroll
  for (int r = 0; r < R; ++r) asm volatile("" : "+r"(raw[r].x), "+r"(raw[r].y), "+r"(raw[r].z), "+r"(raw[r].w));
  constexpr int ES = OUT_F16 ? 2 : 1;  // output element size
  uint8_t* op = out + ((bh * S) * D + cg * 8) * ES;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int row = blk * kBlockRows + rl + r * RL;
    if (row < S) {
      float y[8];
      value(r, y);
#pragma unroll
      // divide (:72, :114, :167); the +-448 clamp is cvt.satfinite's for e4m3
      for (int i = 0; i < 8; ++i)
        y[i] = MODE == kV ? div_rn_by(y[i], c8[i], r8[i]) : div_rn_by(y[i], s, rs);
      if constexpr (OUT_F16) {
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = clamp448(y[i]);
      }
      if constexpr (OUT_F16) {
        uint4 u;
        u.x = cvt_f16x2(y[1], y[0]);
        u.y = cvt_f16x2(y[3], y[2]);
        u.z = cvt_f16x2(y[5], y[4]);
        u.w = cvt_f16x2(y[7], y[6]);
        *reinterpret_cast<uint4*>(op + (long long)row * D * ES) = u;
      } else {
        *reinterpret_cast<uint2*>(op + (long long)row * D) = pack8_e4m3(y);
      }
    }
  }
}

// Per-row absmax quantisation (fp8_linear.py:8-24): one CTA per row.
template <typename T>
__global__ void __launch_bounds__(kThreads) rows_quant_kernel(const T* __restrict__ x, long long xs, int K,
                                                              uint8_t* __restrict__ x8, float* __restrict__ scale) {
  __shared__ float red[kThreads / 32];
  const long long row = blockIdx.x;
  const T* xp = x + row * xs;
  float amax = 0.0f;
  for (int c = threadIdx.x * 8; c < K; c += kThreads * 8) {
    float v[8];
    load8(xp + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
  }
  const float s = fmaxf(block_max(amax, red), 1.0e-12f) / 448.0f;   // :20-21
  const float rs = __frcp_rn(s);
  if (threadIdx.x == 0) scale[row] = s;
  uint8_t* op = x8 + row * K;
  for (int c = threadIdx.x * 8; c < K; c += kThreads * 8) {
    float v[8], y[8];
    load8(xp + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = div_rn_by(v[i], s, rs);   // :22 (clamp: cvt.satfinite)
    *reinterpret_cast<uint2*>(op + c) = pack8_e4m3(y);
  }
}

// Same quantisation with the row held in registers: NT threads, R 16-byte
// chunks each (rows up to NT*8*R elements), so x is read from memory once;
// the absmax, the scale and every quotient are those of rows_quant_kernel.
// 128 threads up to 8192 elements, 256 threads up to 16384 (at most 8 chunks
// per thread: measured 13 % faster than 14 chunks per thread at K=13824).
template <typename T, int R, int NT>
__global__ void __launch_bounds__(NT) rows_quant_reg_kernel(const T* __restrict__ x, long long xs, int K,
                                                            uint8_t* __restrict__ x8, float* __restrict__ scale) {
  __shared__ float red[NT / 32];
  const long long row = blockIdx.x;
  const T* xp = x + row * xs;
  uint4 raw[R];
  float amax = 0.0f;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int c = (r * NT + (int)threadIdx.x) * 8;
    if (c < K) {
      raw[r] = __ldcs(reinterpret_cast<const uint4*>(xp + c));  // streamed: read once
      float v[8];
      unpack8<T>(raw[r], v);
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  float bm = red[0];
#pragma unroll
  for (int i = 1; i < NT / 32; ++i) bm = fmaxf(bm, red[i]);
  const float s = fmaxf(bm, 1.0e-12f) / 448.0f;   // fp8_linear.py:20-21
  const float rs = __frcp_rn(s);
  if (threadIdx.x == 0) scale[row] = s;
  uint8_t* op = x8 + row * K;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int c = (r * NT + (int)threadIdx.x) * 8;
    if (c < K) {
      float v[8], y[8];
      unpack8<T>(raw[r], v);
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = div_rn_by(v[i], s, rs);   // :22 (clamp: cvt.satfinite)
      *reinterpret_cast<uint2*>(op + c) = pack8_e4m3(y);
    }
  }
}

template <typename T>
static void launch_rows_quant(const T* x, long long xs, long long M, int K, uint8_t* x8, float* scale,
                              cudaStream_t st) {
  const int nt = K <= 128 * 8 * 8 ? 128 : 256;
  const int R = (K + nt * 8 - 1) / (nt * 8);
#define MH3_ROWS_REG(RR, NTT) rows_quant_reg_kernel<T, RR, NTT><<<(unsigned)M, NTT, 0, st>>>(x, xs, K, x8, scale)
  if (nt == 128) {
    switch (R) {
      case 1: MH3_ROWS_REG(1, 128); break;
      case 2: MH3_ROWS_REG(2, 128); break;
      case 3: MH3_ROWS_REG(3, 128); break;
      case 4: MH3_ROWS_REG(4, 128); break;
      case 5: MH3_ROWS_REG(5, 128); break;
      case 6: MH3_ROWS_REG(6, 128); break;
      case 7: MH3_ROWS_REG(7, 128); break;
      default: MH3_ROWS_REG(8, 128); break;
    }
  } else {
    switch (R) {
      case 5: MH3_ROWS_REG(5, 256); break;
      case 6: MH3_ROWS_REG(6, 256); break;
      case 7: MH3_ROWS_REG(7, 256); break;
      case 8: MH3_ROWS_REG(8, 256); break;
      default:  // rows longer than 16384 elements
        rows_quant_kernel<T><<<(unsigned)M, kThreads, 0, st>>>(x, xs, K, x8, scale);
    }
  }
#undef MH3_ROWS_REG
}

template <typename T, int D>
static cudaError_t run_qkv(const mh3_qkv_quant_args* a, cudaStream_t st) {
  const int B = a->batch, H = a->heads, Sq = a->seqlen_q, Sk = a->seqlen_k;
  const int nchunk = (Sk + kStatRows - 1) / kStatRows;
  float* part_sum = static_cast<float*>(a->workspace);
  float* part_amax = part_sum + (long long)B * H * nchunk * D;
  kv_stats_kernel<T, D><<<dim3(nchunk, H, B), kThreads, 0, st>>>(
      static_cast<const T*>(a->k), a->k_stride_b, a->k_stride_h, a->k_stride_s, static_cast<const T*>(a->v),
      a->v_stride_b, a->v_stride_h, a->v_stride_s, Sk, H, part_sum, part_amax);
  kv_finalize_kernel<D><<<B * H, D, 0, st>>>(part_sum, part_amax, nchunk, Sk, a->k_mean, a->scale_v);
  const int nq = (Sq + kBlockRows - 1) / kBlockRows;
  const int nk = (Sk + kBlockRows - 1) / kBlockRows;
  block_quant_kernel<T, D, kQ><<<dim3(nq, H, B), kThreads, 0, st>>>(
      static_cast<const T*>(a->q), a->q_stride_b, a->q_stride_h, a->q_stride_s, Sq, H, a->q_premul, nullptr,
      static_cast<uint8_t*>(a->q8), a->scale_q);
  block_quant_kernel<T, D, kK><<<dim3(nk, H, B), kThreads, 0, st>>>(
      static_cast<const T*>(a->k), a->k_stride_b, a->k_stride_h, a->k_stride_s, Sk, H, 1.0f, a->k_mean,
      static_cast<uint8_t*>(a->k8), a->scale_k);
  if (a->v_out_dtype == MH3_DTYPE_F16)
    block_quant_kernel<T, D, kV, true><<<dim3(nk, H, B), kThreads, 0, st>>>(
        static_cast<const T*>(a->v), a->v_stride_b, a->v_stride_h, a->v_stride_s, Sk, H, 1.0f, a->scale_v,
        static_cast<uint8_t*>(a->v8), nullptr);
  else
    block_quant_kernel<T, D, kV><<<dim3(nk, H, B), kThreads, 0, st>>>(
        static_cast<const T*>(a->v), a->v_stride_b, a->v_stride_h, a->v_stride_s, Sk, H, 1.0f, a->scale_v,
        static_cast<uint8_t*>(a->v8), nullptr);
  return cudaGetLastError();
}

// e4m3 -> f16, 16 elements per thread per step (exact: e4m3 is a subset of f16).
__global__ void widen_e4m3_f16_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, long long n16) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n16; i += (long long)gridDim.x * blockDim.x) {
    const uint4 u = src[i];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    uint32_t o[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t lo, hi;
      asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(lo) : "h"((uint16_t)(w[k] & 0xffffu)));
      asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(hi) : "h"((uint16_t)(w[k] >> 16)));
      o[2 * k] = lo;
      o[2 * k + 1] = hi;
    }
    dst[2 * i] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[2 * i + 1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

// Head selection shared by the two per-(batch, head) kernels: the H heads
// form H/hb blocks of hb; selected are heads p*hb + off + i for every block p
// and i < hs, numbered j = p*hs + i (hb = hs = H, off = 0: all heads).
struct HeadSel {
  int hb, off, hs;
  __device__ __forceinline__ int head(int j) const { return (j / hs) * hb + off + j % hs; }
};

// Segments of a packed shard: x is [S, H, D] (B = 1) and its rows
// [seg[z], seg[z+1]) form segment z (seg non-decreasing, each entry clamped
// to [0, S]); the per-segment kernels below index scales by z where the
// per-batch ones index them by b.
struct Segs {
  const int* seg;
  int nseg;
  __device__ __forceinline__ int bound(int z, int S) const { return min(max(__ldg(seg + z), 0), S); }
  // The segment holding row s, or -1 when s lies outside every segment.
  __device__ __forceinline__ int find(int s, int S) const {
    if (s < bound(0, S) || s >= bound(nseg, S)) return -1;
    int lo = 0, hi = nseg - 1;                 // largest z with bound(z) <= s
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (bound(mid, S) <= s) lo = mid; else hi = mid - 1;
    }
    return lo;
  }
};

// Per-(batch, head) absmax of x [B, S, H, D] (element strides sb/ss/sh, D
// contiguous) over the selected heads: one CTA per (256-row chunk, j, b),
// CTA max folded into amax[b*nsel+j] with an integer atomicMax (non-negative
// floats order like their bit patterns; amax starts at 0).  SEG: b is a
// segment z of a packed [S, H, D] shard and the chunks start at its first row.
template <typename T, int D, bool SEG>
__global__ void __launch_bounds__(kThreads) bh_absmax_kernel(const T* __restrict__ x, long long sb, long long ss,
                                                            long long sh, int S, HeadSel sel, Segs segs,
                                                            float* __restrict__ amax) {
  constexpr int CG = D / 8;
  constexpr int RL = kThreads / CG;
  __shared__ float red[kThreads / 32];
  const int j = blockIdx.y, b = blockIdx.z;
  const int h = sel.head(j);
  const int cg = threadIdx.x % CG, rl = threadIdx.x / CG;
  int first = 0, last = S;
  if constexpr (SEG) {
    first = segs.bound(b, S);
    last = max(first, segs.bound(b + 1, S));
  }
  const int r0 = first + blockIdx.x * kStatRows;
  if (r0 >= last) return;                       // uniform over the CTA
  const int r1 = min(last, r0 + kStatRows);
  const T* xp = x + (SEG ? 0 : b * sb) + h * sh + cg * 8;
  // 16-byte loads issued kBatch at a time (several in flight per thread),
  // rows past the chunk read as zeros.
  constexpr int kPass = kStatRows / RL;
  constexpr int kBatch = 4;
  float m = 0.0f;
#pragma unroll
  for (int k0 = 0; k0 < kPass; k0 += kBatch) {
    uint4 u[kBatch];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int r = r0 + rl + (k0 + i) * RL;
      u[i] = r < r1 ? *reinterpret_cast<const uint4*>(xp + (long long)r * ss) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      float v[8];
      unpack8<T>(u[i], v);
#pragma unroll
      for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(v[e]));
    }
  }
  m = block_max(m, red);
  if (threadIdx.x == 0) atomicMax(reinterpret_cast<int*>(amax) + (long long)b * gridDim.y + j, __float_as_int(m));
}

// y = x / scale[b, j] (IEEE division) for the selected heads, e4m3 (clamped
// to +-448, RNE) or f16 (RNE), written block-major: out [P, B, S, hs, D] with
// P = H/hb and selected head j = p*hs + i at [p, b, s, i] - the send buffer of
// a head-parallel all-to-all (all heads, hb = H: plain [B, S, H, D]).  SEG
// (B = 1): row s takes the scale of its segment z, scale[z, j]; rows outside
// every segment are written as zeros.  Grid (row chunk, j, b): one CTA per
// kQuantRows rows of one selected head, one thread per 8 channels of a row;
// each thread first issues all its row loads, then converts and stores.
constexpr int kQuantRows = 128;

template <typename T, int D, bool OUT_F16, bool SEG>
__global__ void __launch_bounds__(kThreads) bh_quant_kernel(const T* __restrict__ x, long long sb, long long ss,
                                                           long long sh, int S, HeadSel sel, Segs segs,
                                                           const float* __restrict__ scale,
                                                           uint8_t* __restrict__ out) {
  constexpr int CG = D / 8;
  constexpr int RPI = kThreads / CG;         // rows per pass
  constexpr int kPass = kQuantRows / RPI;
  constexpr int ES = OUT_F16 ? 2 : 1;
  const int j = blockIdx.y, b = blockIdx.z;
  const int nsel = gridDim.y, B = gridDim.z;
  const int h = sel.head(j);
  const int p = j / sel.hs, hl = j - p * sel.hs;
  const int g = threadIdx.x % CG;
  const int s0 = blockIdx.x * kQuantRows + threadIdx.x / CG;
  const T* xp = x + b * sb + h * sh + g * 8;
  const long long orow = (long long)sel.hs * D;  // output elements from one row to the next
  uint8_t* op = out + ((((long long)p * B + b) * S) * orow + (long long)hl * D + g * 8) * ES;
  uint4 u[kPass];
#pragma unroll
  for (int k = 0; k < kPass; ++k) {
    const int s = s0 + k * RPI;
    u[k] = s < S ? *reinterpret_cast<const uint4*>(xp + (long long)s * ss) : make_uint4(0u, 0u, 0u, 0u);
  }
  float sc = 1.0f, rc = 1.0f;
  if constexpr (!SEG) {
    sc = __ldg(scale + (long long)b * nsel + j);
    rc = __frcp_rn(sc);
  }
  // SEG: a thread's rows only move forward, so it keeps the row range
  // [zlo, zhi) of the sequence whose scale it holds and looks a sequence up
  // again only when a row leaves that range.
  int zlo = 0, zhi = 0;
#pragma unroll
  for (int k = 0; k < kPass; ++k) {
    const int s = s0 + k * RPI;
    if (s >= S) break;
    bool live = true;
    if constexpr (SEG) {
      if (s < zlo || s >= zhi) {
        const int z = segs.find(s, S);
        if (z >= 0) {
          zlo = segs.bound(z, S);
          zhi = segs.bound(z + 1, S);
          sc = __ldg(scale + (long long)z * nsel + j);
          rc = __frcp_rn(sc);
        } else {
          zlo = zhi = 0;
        }
      }
      live = s >= zlo && s < zhi;
    }
    float y[8];
    if (live) {
      float v[8];
      unpack8<T>(u[k], v);
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = div_rn_by(v[e], sc, rc);  // e4m3: clamp by cvt.satfinite
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = 0.0f;
    }
    uint8_t* dst = op + (long long)s * orow * ES;
    if constexpr (OUT_F16) {
      uint4 w;
      w.x = cvt_f16x2(y[1], y[0]);
      w.y = cvt_f16x2(y[3], y[2]);
      w.z = cvt_f16x2(y[5], y[4]);
      w.w = cvt_f16x2(y[7], y[6]);
      *reinterpret_cast<uint4*>(dst) = w;
    } else {
      *reinterpret_cast<uint2*>(dst) = pack8_e4m3(y);
    }
  }
}

}  // namespace quant
}  // namespace mh3

using namespace mh3;

namespace {
bool bh_shape_ok(const void* x, int32_t in_dtype, int64_t B, int64_t S, int64_t H, int64_t D, int64_t sb, int64_t ss,
                 int64_t sh, const char** why) {
  if (x == nullptr) return (*why = "null input"), false;
  if (in_dtype != MH3_DTYPE_BF16 && in_dtype != MH3_DTYPE_F16) return (*why = "in_dtype must be bf16 or f16"), false;
  if (B <= 0 || S <= 0 || H <= 0 || (D != 64 && D != 128)) return (*why = "bad sizes (D must be 64 or 128)"), false;
  if (B > 65535 || H > 65535 || S > (1ll << 30)) return (*why = "too many batches, heads or rows"), false;
  if (((uintptr_t)x & 15u) || (sb % 8) || (ss % 8) || (sh % 8))
    return (*why = "x must be 16-byte aligned with strides multiple of 8 elements"), false;
  return true;
}

template <typename T, int D, bool F16>
void launch_bh_quant_t(const void* x, int64_t sb, int64_t ss, int64_t sh, quant::HeadSel sel, quant::Segs segs,
                       const float* scale, void* out, dim3 grid, int S, bool seg, cudaStream_t st) {
  const T* xt = static_cast<const T*>(x);
  uint8_t* o = static_cast<uint8_t*>(out);
  if (seg)
    quant::bh_quant_kernel<T, D, F16, true><<<grid, quant::kThreads, 0, st>>>(xt, sb, ss, sh, S, sel, segs, scale, o);
  else
    quant::bh_quant_kernel<T, D, F16, false><<<grid, quant::kThreads, 0, st>>>(xt, sb, ss, sh, S, sel, segs, scale, o);
}

// Launches bh_quant_kernel for the dtypes and head dim; returns true when the launch failed.
bool launch_bh_quant(const void* x, int32_t in_dtype, int64_t D, int64_t sb, int64_t ss, int64_t sh,
                     quant::HeadSel sel, quant::Segs segs, const float* scale, int32_t out_dtype, void* out, dim3 grid,
                     int S, bool seg, cudaStream_t st) {
  const bool f16 = out_dtype == MH3_DTYPE_F16;
  const bool bf = in_dtype == MH3_DTYPE_BF16;
#define MH3_BHQ(T, DD, F)                                                                  \
  launch_bh_quant_t<T, DD, F>(x, sb, ss, sh, sel, segs, scale, out, grid, S, seg, st)
  if (D == 128) {
    if (bf) { if (f16) MH3_BHQ(__nv_bfloat16, 128, true); else MH3_BHQ(__nv_bfloat16, 128, false); }
    else { if (f16) MH3_BHQ(__half, 128, true); else MH3_BHQ(__half, 128, false); }
  } else {
    if (bf) { if (f16) MH3_BHQ(__nv_bfloat16, 64, true); else MH3_BHQ(__nv_bfloat16, 64, false); }
    else { if (f16) MH3_BHQ(__half, 64, true); else MH3_BHQ(__half, 64, false); }
  }
#undef MH3_BHQ
  return cudaPeekAtLastError() != cudaSuccess;
}
}  // namespace

extern "C" int mh3_absmax_bh(const void* x, int32_t in_dtype, int64_t B, int64_t S, int64_t H, int64_t D, int64_t sb,
                             int64_t ss, int64_t sh, int32_t head_block, int32_t head_off, int32_t heads_sel,
                             float* amax, void* stream) {
  const mh3::NvtxRange nvtx_range("mh3_absmax_bh");
  const char* why = nullptr;
  if (!bh_shape_ok(x, in_dtype, B, S, H, D, sb, ss, sh, &why)) return fail(MH3_ERR_INVALID, (std::string("mh3_absmax_bh: ") + why).c_str());
  if (amax == nullptr) return fail(MH3_ERR_INVALID, "mh3_absmax_bh: null amax");
  if (head_block <= 0 || H % head_block || head_off < 0 || heads_sel <= 0 || head_off + heads_sel > head_block)
    return fail(MH3_ERR_INVALID, "mh3_absmax_bh: bad head selection");
  const quant::HeadSel sel{head_block, head_off, heads_sel};
  const int64_t nsel = (H / head_block) * heads_sel;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(amax, 0, (size_t)(B * nsel) * sizeof(float), st);
  if (e != cudaSuccess) return fail_cuda(e, "mh3_absmax_bh memset");
  const dim3 grid((unsigned)((S + quant::kStatRows - 1) / quant::kStatRows), (unsigned)nsel, (unsigned)B);
  if (grid.x > 2147483647u) return fail(MH3_ERR_TOO_LARGE, "mh3_absmax_bh: too many rows");
#define MH3_ABSMAX(T, DD)                                                                                         \
  quant::bh_absmax_kernel<T, DD, false><<<grid, quant::kThreads, 0, st>>>(static_cast<const T*>(x), sb, ss, sh, (int)S, \
                                                                         sel, quant::Segs{nullptr, 0}, amax)
  if (in_dtype == MH3_DTYPE_BF16) {
    if (D == 128) MH3_ABSMAX(__nv_bfloat16, 128); else MH3_ABSMAX(__nv_bfloat16, 64);
  } else {
    if (D == 128) MH3_ABSMAX(__half, 128); else MH3_ABSMAX(__half, 64);
  }
#undef MH3_ABSMAX
  e = cudaGetLastError();
  return e == cudaSuccess ? MH3_OK : fail_cuda(e, "mh3_absmax_bh launch");
}

extern "C" int mh3_quantize_bh(const void* x, int32_t in_dtype, int64_t B, int64_t S, int64_t H, int64_t D, int64_t sb,
                               int64_t ss, int64_t sh, int32_t head_block, int32_t head_off, int32_t heads_sel,
                               const float* scale, int32_t out_dtype, void* out, void* stream) {
  const mh3::NvtxRange nvtx_range("mh3_quantize_bh");
  const char* why = nullptr;
  if (!bh_shape_ok(x, in_dtype, B, S, H, D, sb, ss, sh, &why)) return fail(MH3_ERR_INVALID, (std::string("mh3_quantize_bh: ") + why).c_str());
  if (scale == nullptr || out == nullptr) return fail(MH3_ERR_INVALID, "mh3_quantize_bh: null scale or out");
  if (out_dtype != MH3_DTYPE_E4M3 && out_dtype != MH3_DTYPE_F16)
    return fail(MH3_ERR_INVALID, "mh3_quantize_bh: out_dtype must be e4m3 or f16");
  if (head_block <= 0 || H % head_block || head_off < 0 || heads_sel <= 0 || head_off + heads_sel > head_block)
    return fail(MH3_ERR_INVALID, "mh3_quantize_bh: bad head selection");
  const quant::HeadSel sel{head_block, head_off, heads_sel};
  if ((uintptr_t)out & 15u) return fail(MH3_ERR_INVALID, "mh3_quantize_bh: out must be 16-byte aligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)((S + quant::kQuantRows - 1) / quant::kQuantRows),
                  (unsigned)((H / head_block) * heads_sel), (unsigned)B);
  return launch_bh_quant(x, in_dtype, D, sb, ss, sh, sel, quant::Segs{nullptr, 0}, scale, out_dtype, out, grid, (int)S,
                         false, st)
             ? fail_cuda(cudaGetLastError(), "mh3_quantize_bh launch")
             : MH3_OK;
}

extern "C" int mh3_absmax_seg(const void* x, int32_t in_dtype, int64_t S, int64_t H, int64_t D, int64_t ss,
                              int64_t sh, int32_t head_block, int32_t head_off, int32_t heads_sel, const int32_t* seg,
                              int32_t nseg, float* amax, void* stream) {
  const mh3::NvtxRange nvtx_range("mh3_absmax_seg");
  const char* why = nullptr;
  if (!bh_shape_ok(x, in_dtype, 1, S, H, D, 0, ss, sh, &why)) return fail(MH3_ERR_INVALID, (std::string("mh3_absmax_seg: ") + why).c_str());
  if (amax == nullptr || seg == nullptr) return fail(MH3_ERR_INVALID, "mh3_absmax_seg: null amax or seg");
  if (nseg <= 0 || nseg > 65535) return fail(MH3_ERR_INVALID, "mh3_absmax_seg: nseg must be in [1, 65535]");
  if (head_block <= 0 || H % head_block || head_off < 0 || heads_sel <= 0 || head_off + heads_sel > head_block)
    return fail(MH3_ERR_INVALID, "mh3_absmax_seg: bad head selection");
  const quant::HeadSel sel{head_block, head_off, heads_sel};
  const int64_t nsel = (H / head_block) * heads_sel;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(amax, 0, (size_t)(nseg * nsel) * sizeof(float), st);
  if (e != cudaSuccess) return fail_cuda(e, "mh3_absmax_seg memset");
  // Each segment gets as many chunks as the whole shard has (its own length is
  // only known on the device); chunks past a segment's end return at once.
  const dim3 grid((unsigned)((S + quant::kStatRows - 1) / quant::kStatRows), (unsigned)nsel, (unsigned)nseg);
  const quant::Segs segs{seg, nseg};
#define MH3_ABSMAX(T, DD)                                                                                        \
  quant::bh_absmax_kernel<T, DD, true><<<grid, quant::kThreads, 0, st>>>(static_cast<const T*>(x), 0, ss, sh, (int)S, \
                                                                         sel, segs, amax)
  if (in_dtype == MH3_DTYPE_BF16) {
    if (D == 128) MH3_ABSMAX(__nv_bfloat16, 128); else MH3_ABSMAX(__nv_bfloat16, 64);
  } else {
    if (D == 128) MH3_ABSMAX(__half, 128); else MH3_ABSMAX(__half, 64);
  }
#undef MH3_ABSMAX
  e = cudaGetLastError();
  return e == cudaSuccess ? MH3_OK : fail_cuda(e, "mh3_absmax_seg launch");
}

extern "C" int mh3_quantize_seg(const void* x, int32_t in_dtype, int64_t S, int64_t H, int64_t D, int64_t ss,
                                int64_t sh, int32_t head_block, int32_t head_off, int32_t heads_sel,
                                const int32_t* seg, int32_t nseg, const float* scale, int32_t out_dtype, void* out,
                                void* stream) {
  const mh3::NvtxRange nvtx_range("mh3_quantize_seg");
  const char* why = nullptr;
  if (!bh_shape_ok(x, in_dtype, 1, S, H, D, 0, ss, sh, &why)) return fail(MH3_ERR_INVALID, (std::string("mh3_quantize_seg: ") + why).c_str());
  if (scale == nullptr || out == nullptr || seg == nullptr)
    return fail(MH3_ERR_INVALID, "mh3_quantize_seg: null scale, out or seg");
  if (nseg <= 0 || nseg > 65535) return fail(MH3_ERR_INVALID, "mh3_quantize_seg: nseg must be in [1, 65535]");
  if (out_dtype != MH3_DTYPE_E4M3 && out_dtype != MH3_DTYPE_F16)
    return fail(MH3_ERR_INVALID, "mh3_quantize_seg: out_dtype must be e4m3 or f16");
  if (head_block <= 0 || H % head_block || head_off < 0 || heads_sel <= 0 || head_off + heads_sel > head_block)
    return fail(MH3_ERR_INVALID, "mh3_quantize_seg: bad head selection");
  const quant::HeadSel sel{head_block, head_off, heads_sel};
  if ((uintptr_t)out & 15u) return fail(MH3_ERR_INVALID, "mh3_quantize_seg: out must be 16-byte aligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)((S + quant::kQuantRows - 1) / quant::kQuantRows),
                  (unsigned)((H / head_block) * heads_sel), 1u);
  return launch_bh_quant(x, in_dtype, D, 0, ss, sh, sel, quant::Segs{seg, nseg}, scale, out_dtype, out, grid, (int)S,
                         true, st)
             ? fail_cuda(cudaGetLastError(), "mh3_quantize_seg launch")
             : MH3_OK;
}

extern "C" uint64_t mh3_qkv_workspace_bytes(int32_t batch, int32_t heads, int32_t seqlen_k, int32_t head_dim) {
  if (batch <= 0 || heads <= 0 || seqlen_k <= 0 || head_dim <= 0) return 0;
  const uint64_t nchunk = ((uint64_t)seqlen_k + quant::kStatRows - 1) / quant::kStatRows;
  return 2ull * (uint64_t)batch * (uint64_t)heads * nchunk * (uint64_t)head_dim * sizeof(float);
}

extern "C" int mh3_quantize_qkv(const mh3_qkv_quant_args* a, void* stream) {
  const mh3::NvtxRange nvtx_range("mh3_quantize_qkv");
  if (a == nullptr) return fail(MH3_ERR_INVALID, "mh3_quantize_qkv: null args");
  if (a->head_dim != 64 && a->head_dim != 128) return fail(MH3_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  if (a->batch <= 0 || a->heads <= 0 || a->seqlen_q <= 0 || a->seqlen_k <= 0)
    return fail(MH3_ERR_INVALID, "sizes must be positive");
  if (a->batch > 65535 || a->heads > 65535) return fail(MH3_ERR_INVALID, "too many batches or heads");
  if (!a->q || !a->k || !a->v || !a->q8 || !a->k8 || !a->v8 || !a->scale_q || !a->scale_k || !a->scale_v ||
      !a->k_mean || !a->workspace)
    return fail(MH3_ERR_INVALID, "null pointer");
  if (a->in_dtype != MH3_DTYPE_BF16 && a->in_dtype != MH3_DTYPE_F16)
    return fail(MH3_ERR_INVALID, "in_dtype must be bf16 or f16");
  if (a->v_out_dtype != MH3_DTYPE_E4M3 && a->v_out_dtype != MH3_DTYPE_F16)
    return fail(MH3_ERR_INVALID, "v_out_dtype must be e4m3 or f16");
  auto al16 = [](const void* p) { return ((uintptr_t)p & 15u) == 0; };
  if (!al16(a->q) || !al16(a->k) || !al16(a->v) || !al16(a->q8) || !al16(a->k8) || !al16(a->v8))
    return fail(MH3_ERR_INVALID, "tensors must be 16-byte aligned");
  const long long st[9] = {a->q_stride_b, a->q_stride_h, a->q_stride_s, a->k_stride_b, a->k_stride_h,
                           a->k_stride_s, a->v_stride_b, a->v_stride_h, a->v_stride_s};
  for (long long s : st)
    if (s % 8) return fail(MH3_ERR_INVALID, "q/k/v strides must be multiples of 8 elements");
  cudaStream_t stream_ = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e;
  const bool f16 = a->in_dtype == MH3_DTYPE_F16;
  if (a->head_dim == 128)
    e = f16 ? quant::run_qkv<__half, 128>(a, stream_) : quant::run_qkv<__nv_bfloat16, 128>(a, stream_);
  else
    e = f16 ? quant::run_qkv<__half, 64>(a, stream_) : quant::run_qkv<__nv_bfloat16, 64>(a, stream_);
  if (e != cudaSuccess) return fail_cuda(e, "mh3_quantize_qkv launch");
  return MH3_OK;
}

extern "C" int mh3_quantize_rows(const void* x, int64_t x_stride, int32_t in_dtype, int64_t M, int64_t K, void* x8,
                                 float* scale, void* stream) {
  const mh3::NvtxRange nvtx_range("mh3_quantize_rows");
  if (M < 0 || K < 0) return fail(MH3_ERR_INVALID, "negative size");
  if (M == 0 || K == 0) return MH3_OK;
  if (!x || !x8 || !scale) return fail(MH3_ERR_INVALID, "null pointer");
  if (K % 8 || x_stride % 8 || ((uintptr_t)x & 15u) || ((uintptr_t)x8 & 7u))
    return fail(MH3_ERR_UNSUPPORTED, "K and the row stride must be multiples of 8, x 16-byte aligned");
  if (M > 0x7fffffffLL) return fail(MH3_ERR_TOO_LARGE, "M too large");
  if (in_dtype != MH3_DTYPE_BF16 && in_dtype != MH3_DTYPE_F16 && in_dtype != MH3_DTYPE_F32)
    return fail(MH3_ERR_INVALID, "in_dtype must be bf16, f16 or f32");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (K > 0x7fffffffLL) return fail(MH3_ERR_TOO_LARGE, "K too large");
  if (in_dtype == MH3_DTYPE_F32)  // float rows (the reference loads any float dtype, fp8_linear.py:19)
    quant::rows_quant_kernel<float><<<(unsigned)M, quant::kThreads, 0, st>>>(static_cast<const float*>(x), x_stride,
                                                                            (int)K, static_cast<uint8_t*>(x8), scale);
  else if (in_dtype == MH3_DTYPE_F16)
    quant::launch_rows_quant<__half>(static_cast<const __half*>(x), x_stride, M, (int)K, static_cast<uint8_t*>(x8),
                                     scale, st);
  else
    quant::launch_rows_quant<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(x), x_stride, M, (int)K,
                                            static_cast<uint8_t*>(x8), scale, st);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail_cuda(e, "mh3_quantize_rows launch");
  return MH3_OK;
}

extern "C" int mh3_widen_e4m3_to_f16(const void* src, void* dst, int64_t n, void* stream) {
  const mh3::NvtxRange nvtx_range("mh3_widen_e4m3_to_f16");
  if (n < 0) return fail(MH3_ERR_INVALID, "negative size");
  if (n == 0) return MH3_OK;
  if (!src || !dst) return fail(MH3_ERR_INVALID, "null pointer");
  if ((n % 16) || ((uintptr_t)src & 15u) || ((uintptr_t)dst & 15u))
    return fail(MH3_ERR_UNSUPPORTED, "n must be a multiple of 16 and both buffers 16-byte aligned");
  const long long n16 = n / 16;
  const int threads = 256;
  const long long want = (n16 + threads - 1) / threads;
  const int blocks = (int)(want < 148 * 16 ? want : 148 * 16);
  quant::widen_e4m3_f16_kernel<<<blocks, threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), static_cast<uint4*>(dst), n16);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail_cuda(e, "mh3_widen_e4m3_to_f16 launch");
  return MH3_OK;
}

// ----------------------------------------------------------------------------
// mh3_quantize_qkv_noalloc: the same quantisation with library-owned scratch.
//
// Some callers cannot allocate device memory when they call this path: a
// plugin inside another inference runtime whose enqueue step may not allocate
// (the runtime plans every device buffer up front), a latency-critical
// serving loop where cudaMalloc's implicit device synchronisation would stall
// work already in flight, or a host program whose device memory all belongs
// to another framework's pool.  This entry point takes its K/V statistics
// scratch from a fixed array in the library's own device image instead of a
// caller workspace.  It never calls cudaMalloc, cudaFree or any allocating
// routine.
//
// The array is ``kNoAllocScratchBytes`` (8 MiB) and every GPU that loads the
// library holds it until the process exits.  Every call shares it and it
// keeps the last call's contents; the statistics kernel writes every partial
// the finishing kernel reads, so nothing has to start at zero.  Calls that
// overlap on the GPU (two streams, or two devices' work aimed at one device)
// race on the array: serialise them.
// ----------------------------------------------------------------------------
namespace mh3 {
namespace quant {

constexpr unsigned long long kNoAllocScratchBytes = 8ull << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device.  In host code
// the symbol names a host-side stand-in, not device memory, so the address
// is looked up once per device (with that device current) and cached; it is
// looked up again if the device's context changed since (a device reset
// loads the module, and the array, anew).
static int noalloc_scratch(void** out) {
  constexpr int kMaxDevices = 64;
  static void* addr[kMaxDevices] = {};
  static void* ctx_of[kMaxDevices] = {};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_cuda(e, "mh3_quantize_qkv_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(MH3_ERR_UNSUPPORTED, "device index out of range");
  std::lock_guard<std::mutex> lock(mu);
  void* ctx = current_context();
  if (addr[dev] == nullptr || ctx_of[dev] != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return fail_cuda(e, "mh3_quantize_qkv_noalloc: cudaGetSymbolAddress");
    addr[dev] = p;
    ctx_of[dev] = ctx;
  }
  *out = addr[dev];
  return MH3_OK;
}

}  // namespace quant
}  // namespace mh3

extern "C" int mh3_quantize_qkv_noalloc(const mh3_qkv_quant_args* a, void* stream) {
  if (a == nullptr) return fail(MH3_ERR_INVALID, "mh3_quantize_qkv_noalloc: null args");
  const uint64_t need = mh3_qkv_workspace_bytes(a->batch, a->heads, a->seqlen_k, a->head_dim);
  if (need > quant::kNoAllocScratchBytes)
    return fail(MH3_ERR_TOO_LARGE,
                "mh3_quantize_qkv_noalloc: scratch needed (2*batch*heads*ceil(seqlen_k/256)*head_dim*4 bytes) "
                "exceeds its fixed 8 MiB; use mh3_quantize_qkv with a caller workspace");
  void* scratch = nullptr;
  const int rc = quant::noalloc_scratch(&scratch);
  if (rc != MH3_OK) return rc;
  mh3_qkv_quant_args b = *a;
  b.workspace = scratch;
  return mh3_quantize_qkv(&b, stream);
}
