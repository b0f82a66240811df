// Per-key mask / bias of the drop-in attention path in the kernel's form.
//
// The reference applies ``key_bias`` and ``key_mask`` inside its attention
// loop (kernels/fp8_attention.py:256-264): a key is valid when its mask is
// true and its bias is above -1e8, a valid key's logit gains
// ``bias * 1.4426950408889634`` (log2 units), an invalid one is dropped.
// The attention kernel here takes both as one additive fp32 row per batch,
// bias2 = bias*log2(e) for a valid key and -inf otherwise (also for the
// padding up to a whole 128-key tile), plus kv_len = one past the last valid
// key, past which it skips whole tiles.  mh3_key_bias builds both in one
// launch: one CTA per batch row reads the row's mask and bias once, writes
// bias2 and reduces kv_len (no atomics, so no zeroing pass).
#include "mh3_b200.h"
#include "mh3_internal.h"

namespace mh3 {
namespace keymask {

constexpr int kThreads = 512;
constexpr int kTile = 128;  // key tile of the attention kernel

__global__ void __launch_bounds__(kThreads) key_bias_kernel(const uint8_t* __restrict__ mask, long long msb,
                                                            const float* __restrict__ bias, long long bsb, long long Sk,
                                                            long long padded, float* __restrict__ bias2,
                                                            long long osb, int* __restrict__ kv_len) {
  __shared__ long long red[kThreads / 32];
  const long long b = blockIdx.x;
  const uint8_t* mrow = mask ? mask + b * msb : nullptr;
  const float* brow = bias ? bias + b * bsb : nullptr;
  float* orow = bias2 + b * osb;
  long long last = 0;  // one past the last valid key seen by this thread
  for (long long j = threadIdx.x; j < padded; j += kThreads) {
    float out = -INFINITY;
    if (j < Sk) {
      bool valid = true;
      float val = 0.0f;
      if (brow) {
        const float kb = brow[j];
        valid = kb > -1.0e8f;
        val = __fmul_rn(kb, 1.4426950408889634f);
      }
      if (mrow) valid = valid && mrow[j] != 0;
      if (valid) {
        out = val;
        last = j + 1;
      }
    }
    orow[j] = out;
  }
  if (kv_len == nullptr) return;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const long long other = __shfl_xor_sync(0xffffffffu, last, o);
    last = other > last ? other : last;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = last;
  __syncthreads();
  if (threadIdx.x == 0) {
    long long m = red[0];
    for (int i = 1; i < kThreads / 32; ++i) m = red[i] > m ? red[i] : m;
    kv_len[b] = (int)m;
  }
}

}  // namespace keymask
}  // namespace mh3

using namespace mh3;

extern "C" int mh3_key_bias(const uint8_t* key_mask, int64_t mask_stride_b, const float* key_bias,
                            int64_t bias_stride_b, int64_t batch, int64_t seqlen_k, float* bias2,
                            int64_t bias2_stride_b, int32_t* kv_len, void* stream) {
  if (batch <= 0 || seqlen_k <= 0) return fail(MH3_ERR_INVALID, "mh3_key_bias: batch and seqlen_k must be positive");
  if (batch > 0x7fffffffLL || seqlen_k > 0x7fffffffLL)
    return fail(MH3_ERR_INVALID, "mh3_key_bias: batch and seqlen_k must fit in 32 bits");
  if (bias2 == nullptr) return fail(MH3_ERR_INVALID, "mh3_key_bias: null bias2");
  if (mask_stride_b < 0 || bias_stride_b < 0) return fail(MH3_ERR_INVALID, "mh3_key_bias: negative batch stride");
  const long long padded = (seqlen_k + keymask::kTile - 1) / keymask::kTile * keymask::kTile;
  if (bias2_stride_b < padded)
    return fail(MH3_ERR_INVALID, "mh3_key_bias: bias2 rows must hold ceil(seqlen_k/128)*128 values");
  keymask::key_bias_kernel<<<(unsigned)batch, keymask::kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      key_mask, mask_stride_b, key_bias, bias_stride_b, seqlen_k, padded, bias2, bias2_stride_b,
      reinterpret_cast<int*>(kv_len));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MH3_OK : fail_cuda(e, "mh3_key_bias launch");
}
