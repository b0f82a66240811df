// Per-key mask / bias of the drop-in attention path in the kernel's form.
//
// The reference applies ``key_bias`` and ``key_mask`` inside its attention
// loop (kernels/fp8_attention.py:256-264): a key is valid when its mask is
// true and its bias is above -1e8, a valid key's logit gains
// ``bias * 1.4426950408889634`` (log2 units), an invalid one is dropped.
// The attention kernel here takes both as one additive fp32 row per batch,
// bias2 = bias*log2(e) for a valid key and -inf otherwise (also for the
// padding up to a whole 128-key tile), plus kv_len = one past the last valid
// key, past which it skips whole tiles.  mh3_key_bias builds both: kv_len
// is zeroed (cudaMemsetAsync), then one launch over (4096-key chunk, batch)
// reads the mask and bias once, writes bias2 and folds each chunk's last
// valid key into kv_len with one integer atomicMax per CTA.
#include "mh3_b200.h"
#include "mh3_internal.h"

namespace mh3 {
namespace keymask {

constexpr int kThreads = 512;
constexpr int kPerThread = 8;                      // keys per thread, loads all in flight
constexpr int kChunk = kThreads * kPerThread;      // keys per CTA
constexpr int kTile = 128;                         // key tile of the attention kernel

// grid (chunks of the padded row, batch); key j = chunk*kChunk + i*kThreads + tid.
__global__ void __launch_bounds__(kThreads) key_bias_kernel(const uint8_t* __restrict__ mask, long long msb,
                                                            const float* __restrict__ bias, long long bsb, int Sk,
                                                            int padded, float* __restrict__ bias2, long long osb,
                                                            int* __restrict__ kv_len) {
  __shared__ int red[kThreads / 32];
  const long long b = blockIdx.y;
  const uint8_t* mrow = mask ? mask + b * msb : nullptr;
  const float* brow = bias ? bias + b * bsb : nullptr;
  float* orow = bias2 + b * osb;
  const int j0 = blockIdx.x * kChunk + threadIdx.x;
  uint8_t mv[kPerThread];
  float bv[kPerThread];
#pragma unroll
  for (int i = 0; i < kPerThread; ++i) {
    const int j = j0 + i * kThreads;
    const bool in = j < Sk;
    mv[i] = (mrow && in) ? mrow[j] : (uint8_t)1;
    bv[i] = (brow && in) ? brow[j] : 0.0f;
  }
  int last = 0;  // one past the last valid key of this thread
#pragma unroll
  for (int i = 0; i < kPerThread; ++i) {
    const int j = j0 + i * kThreads;
    if (j >= padded) break;
    // valid: mask true and bias > -1e8 (fp8_attention.py:258,261); bias2 = bias*log2(e) (:259)
    const bool valid = j < Sk && mv[i] != 0 && (brow == nullptr || bv[i] > -1.0e8f);
    orow[j] = valid ? __fmul_rn(bv[i], 1.4426950408889634f) : -INFINITY;
    if (valid) last = j + 1;
  }
  if (kv_len == nullptr) return;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = last;
  __syncthreads();
  if (threadIdx.x == 0) {
    int m = red[0];
#pragma unroll
    for (int i = 1; i < kThreads / 32; ++i) m = max(m, red[i]);
    if (m > 0) atomicMax(kv_len + b, m);
  }
}

}  // namespace keymask
}  // namespace mh3

using namespace mh3;

extern "C" int mh3_key_bias(const uint8_t* key_mask, int64_t mask_stride_b, const float* key_bias,
                            int64_t bias_stride_b, int64_t batch, int64_t seqlen_k, float* bias2,
                            int64_t bias2_stride_b, int32_t* kv_len, void* stream) {
  const mh3::NvtxRange nvtx_range("mh3_key_bias");
  if (batch <= 0 || seqlen_k <= 0) return fail(MH3_ERR_INVALID, "mh3_key_bias: batch and seqlen_k must be positive");
  if (batch > 65535 || seqlen_k > (1LL << 30))
    return fail(MH3_ERR_INVALID, "mh3_key_bias: batch must be <= 65535 and seqlen_k <= 2^30");
  if (bias2 == nullptr) return fail(MH3_ERR_INVALID, "mh3_key_bias: null bias2");
  if (mask_stride_b < 0 || bias_stride_b < 0) return fail(MH3_ERR_INVALID, "mh3_key_bias: negative batch stride");
  const long long padded = (seqlen_k + keymask::kTile - 1) / keymask::kTile * keymask::kTile;
  if (bias2_stride_b < padded)
    return fail(MH3_ERR_INVALID, "mh3_key_bias: bias2 rows must hold ceil(seqlen_k/128)*128 values");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (kv_len != nullptr) {
    const cudaError_t e = cudaMemsetAsync(kv_len, 0, (size_t)batch * sizeof(int32_t), st);
    if (e != cudaSuccess) return fail_cuda(e, "mh3_key_bias kv_len reset");
  }
  const dim3 grid((unsigned)((padded + keymask::kChunk - 1) / keymask::kChunk), (unsigned)batch);
  keymask::key_bias_kernel<<<grid, keymask::kThreads, 0, st>>>(key_mask, mask_stride_b, key_bias, bias_stride_b,
                                                               (int)seqlen_k, (int)padded, bias2, bias2_stride_b,
                                                               reinterpret_cast<int*>(kv_len));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MH3_OK : fail_cuda(e, "mh3_key_bias launch");
}
