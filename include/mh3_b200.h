/*
 * mh3_b200.h - C ABI of the B200 (sm_100a) FP8 attention / FP8 linear hot path
 * of MiniMax-H3.
 *
 * Every entry point takes plain pointers (device memory unless stated),
 * sizes and strides, and a CUDA stream passed as ``void*`` (a cudaStream_t;
 * NULL = legacy default stream).  Nothing allocates device memory: outputs
 * and scratch buffers are owned by the caller.  Calls are asynchronous on
 * the stream.  Return value: MH3_OK (0) on success; a negative MH3_ERR_*
 * code for an invalid argument (the message is available from
 * mh3_last_error() on the calling thread); a positive cudaError_t value if a
 * CUDA launch failed.
 *
 * Element strides are in elements of the tensor's own type; the last
 * dimension (channels / K) is always contiguous.
 *
 * Each entry point names the reference (viragadel6/minimaxh3) interface it
 * replaces, as path:line.
 */
#ifndef MH3_B200_H_
#define MH3_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define MH3_API
#else
#define MH3_API __attribute__((visibility("default")))
#endif

/* ABI history: 1: the first release, mh3_quantize_qkv_noalloc included;
 * 2: mh3_attn_args.kv_len; 3: head selection in mh3_absmax_bh /
 * mh3_quantize_bh, mh3_copy_rows, mh3_step_diff; 4: f32 input to
 * mh3_quantize_rows, test_flags in mh3_attn_args (was reserved0) and
 * mh3_gemm_args; 5: mh3_absmax_seg, mh3_quantize_seg; 6: mh3_peer_alloc,
 * mh3_peer_free, mh3_peer_handle, mh3_peer_open, mh3_peer_close;
 * 7: mh3_key_bias. */
#define MH3_ABI_VERSION 7

#define MH3_OK 0
#define MH3_ERR_INVALID (-1)     /* bad argument: shape, stride, alignment, null pointer */
#define MH3_ERR_UNSUPPORTED (-2) /* valid but not supported by this build (e.g. head_dim) */
#define MH3_ERR_DRIVER (-3)      /* CUDA driver call failed (tensor map encoding) */
#define MH3_ERR_TOO_LARGE (-4)   /* size exceeds a fixed limit of the entry point */

#define MH3_DTYPE_BF16 0
#define MH3_DTYPE_F16 1
#define MH3_DTYPE_E4M3 2
#define MH3_DTYPE_F32 3 /* mh3_step_diff and mh3_quantize_rows input */

/* Device-side error codes written by kernels into an ``err`` word. */
#define MH3_DEVERR_NONE 0
#define MH3_DEVERR_WAIT_TIMEOUT 1 /* an mbarrier wait exceeded timeout_ns */

/* test_flags bits (attention and GEMM arguments).  MH3_TEST_STALL_PRODUCER:
 * each CTA's load warp first waits on a barrier nothing arrives on, so its
 * bounded wait runs out after timeout_ns; the kernel then records
 * MH3_DEVERR_WAIT_TIMEOUT, issues no copy, runs its other waits to their
 * abort path, frees its tensor memory and returns (the output is
 * unspecified).  For testing the failure path without a GPU fault. */
#define MH3_TEST_STALL_PRODUCER 1

MH3_API int mh3_abi_version(void);

/* Message of the last failed call on this thread ("" if none). */
MH3_API const char* mh3_last_error(void);

/* Address of the library's own device error word on the current device
 * (used when a call passes err = NULL).  Kernels only ever set it from 0 to a
 * MH3_DEVERR_* code; read and clear it with ordinary copies. */
MH3_API int* mh3_device_error_word(void);

/* ------------------------------------------------------------------------ */
/* FP8 attention forward                                                     */
/* ------------------------------------------------------------------------ */
/*
 * Replaces ``_fp8_attn_kernel`` (kernels/fp8_attention.py:190-297) and the
 * launch at kernels/fp8_attention.py:379-402.
 *
 * Non-causal attention over e4m3 inputs:
 *   logit2[i,j] = (q8[i] . k8[j]) * scale_q[blk(i)] * scale_k[blk(j)]
 *                 * logit_scale_log2 + key_bias2[j]          (log2 units)
 *   out[i,d]    = scale_v[d] * sum_j 2^logit2[i,j] v8[j,d] / sum_j 2^logit2[i,j]
 * blk(i) = i / 128 within the sequence.  A per-(batch, head) scale is a
 * block stride of 0.  Rows whose keys are all masked produce 0.
 *
 * v_dtype selects the PV product: MH3_DTYPE_E4M3 (P rounded to e4m3, e4m3 V,
 * kind::f8f6f4) or MH3_DTYPE_F16 (P in f16, V an f16 tensor already divided
 * by scale_v, kind::f16 - the accurate default of the drop-in path).
 *
 * Dense mode (cu_seqlens_q == cu_seqlens_k == NULL): q8 is [B,H,Sq,D],
 * k8/v8 are [B,H,Sk,D] under the given strides.
 * Varlen mode: tensors are packed along the token dimension (the ``s``
 * stride steps one token; the ``b`` stride is ignored); sequence b owns
 * tokens [cu_seqlens[b], cu_seqlens[b+1]); ``batch`` = number of sequences;
 * scale/bias ``b`` strides index the sequence.
 *
 * key_bias2 (optional): f32 [B, ceil(Sk/128)*128] additive bias in log2
 * units, -inf for masked keys AND for the padding past Sk; 16-byte aligned.
 * It carries both the reference's key_mask and key_bias (:256-264).
 */
typedef struct mh3_attn_args {
  int32_t batch, heads, seqlen_q, seqlen_k, head_dim; /* head_dim: 64 or 128 */
  int32_t out_dtype;                                   /* MH3_DTYPE_BF16 / MH3_DTYPE_F16 */
  int32_t v_dtype;                                     /* MH3_DTYPE_E4M3 / MH3_DTYPE_F16 */
  int32_t test_flags;                                  /* 0; MH3_TEST_* bits for tests of the bounded waits */
  const void* q8;
  int64_t q_stride_b, q_stride_h, q_stride_s; /* multiples of 16 (v: of 16 bytes) */
  const void* k8;
  int64_t k_stride_b, k_stride_h, k_stride_s;
  const void* v8;
  int64_t v_stride_b, v_stride_h, v_stride_s;
  void* out;
  int64_t o_stride_b, o_stride_h, o_stride_s; /* multiples of 8 */
  const float* scale_q;
  int64_t sq_stride_b, sq_stride_h, sq_stride_blk;
  const float* scale_k;
  int64_t sk_stride_b, sk_stride_h, sk_stride_blk;
  const float* scale_v;
  int64_t sv_stride_b, sv_stride_h, sv_stride_d;
  float logit_scale_log2;
  int32_t max_seqlen_q; /* varlen only */
  const int32_t* cu_seqlens_q; /* [batch+1] device, or NULL */
  const int32_t* cu_seqlens_k;
  int64_t total_q, total_k; /* varlen only: packed token counts */
  const float* key_bias2;
  int64_t key_bias2_stride_b;
  int* err;            /* device error word, or NULL for the library's own */
  uint64_t timeout_ns; /* bound on every pipeline wait; 0 = 4 s */
  /* Optional int32 [batch] on the device: keys at or past kv_len[b] are
   * masked (a padded batch); the kernel skips their tiles.  NULL = none. */
  const int32_t* kv_len;
} mh3_attn_args;

MH3_API int mh3_fp8_attention_fwd(const mh3_attn_args* args, void* stream);

/*
 * The per-key inputs of the drop-in path in the form mh3_fp8_attention_fwd
 * takes (key_bias2 and kv_len), in one launch.  Replaces the reference's
 * in-kernel handling of ``key_bias`` / ``key_mask``
 * (kernels/fp8_attention.py:256-264): key j of batch b is valid when
 * key_mask[b,j] != 0 and key_bias[b,j] > -1e8;
 *   bias2[b,j] = key_bias[b,j] * 1.4426950408889634f (fp32 product; 0 with no
 *                bias) for a valid key, -inf for an invalid one and for
 *                j in [seqlen_k, ceil(seqlen_k/128)*128);
 *   kv_len[b]  = one past the last valid key (0 when none is).
 * key_mask: uint8 (bool) [batch, seqlen_k], keys contiguous, batch stride
 * mask_stride_b elements (0 = one row for every batch), or NULL.  key_bias:
 * f32, the same layout with bias_stride_b, or NULL.  bias2: f32 rows of
 * bias2_stride_b >= ceil(seqlen_k/128)*128.  kv_len: int32 [batch] or NULL
 * (zeroed on the stream, then reduced with atomics).  batch <= 65535,
 * seqlen_k <= 2^30.  (ABI version 7.)
 */
MH3_API int mh3_key_bias(const uint8_t* key_mask, int64_t mask_stride_b, const float* key_bias, int64_t bias_stride_b,
                         int64_t batch, int64_t seqlen_k, float* bias2, int64_t bias2_stride_b, int32_t* kv_len,
                         void* stream);

/* ------------------------------------------------------------------------ */
/* Q / K / V quantisation for the drop-in bf16/fp16 path                      */
/* ------------------------------------------------------------------------ */
/*
 * Replaces ``_quantize_q_kernel`` (kernels/fp8_attention.py:39-77), the K
 * channel mean ``k.float().mean(dim=2)`` (:338), ``_quantize_k_kernel``
 * (:80-119) and ``_quantize_v_kernel`` (:122-170), with the reference's
 * arithmetic:
 *   q8 = e4m3(clamp(q*q_premul / sq, +-448)), sq = max(absmax_128rows, 1e-12)/448
 *   k8 = e4m3(clamp((k-mean_k)/sk, +-448)),    sk per 128 keys likewise
 *   v8 = e4m3(clamp(v / sv[d], +-448)),        sv[d] = max(absmax over S, 1e-12)/448
 * (v_out_dtype = MH3_DTYPE_F16 stores f16(v / sv[d]) instead of e4m3, for the
 * attention kernel's f16 PV product.)
 * Outputs are contiguous: q8 [B,H,Sq,D], k8/v8 [B,H,Sk,D] (v8 in natural
 * [key, channel] order - the attention kernel needs no transposed copy),
 * scale_q [B,H,ceil(Sq/128)], scale_k [B,H,ceil(Sk/128)], scale_v and
 * k_mean [B,H,D].  ``workspace`` must hold mh3_qkv_workspace_bytes() bytes.
 */
typedef struct mh3_qkv_quant_args {
  int32_t batch, heads, seqlen_q, seqlen_k, head_dim;
  int32_t in_dtype; /* MH3_DTYPE_BF16 / MH3_DTYPE_F16 */
  const void* q;
  int64_t q_stride_b, q_stride_h, q_stride_s;
  const void* k;
  int64_t k_stride_b, k_stride_h, k_stride_s;
  const void* v;
  int64_t v_stride_b, v_stride_h, v_stride_s;
  float q_premul;      /* softmax scale * log2(e) */
  int32_t v_out_dtype; /* MH3_DTYPE_E4M3 (reference layout) or MH3_DTYPE_F16 */
  void* q8;
  void* k8;
  void* v8;
  float* scale_q;
  float* scale_k;
  float* scale_v;
  float* k_mean;
  void* workspace;
} mh3_qkv_quant_args;

MH3_API uint64_t mh3_qkv_workspace_bytes(int32_t batch, int32_t heads, int32_t seqlen_k, int32_t head_dim);
MH3_API int mh3_quantize_qkv(const mh3_qkv_quant_args* args, void* stream);

/*
 * mh3_quantize_qkv without a caller workspace.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory when
 * they call this path (a plugin whose enqueue step must not allocate, a
 * latency-critical loop that cannot afford cudaMalloc's implicit device
 * synchronisation, a host program whose device memory belongs to another
 * framework's pool).  It allocates nothing: its scratch is a fixed 8 MiB
 * array in the library's device image, held by every GPU that loads the
 * library until exit.  ``args->workspace`` is ignored.  Sizes needing more
 * than 8 MiB (mh3_qkv_workspace_bytes() > 8 MiB) are rejected with
 * MH3_ERR_TOO_LARGE.  The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress, with that device current); make that
 * first call before any stream capture.  All calls share the array: calls
 * that overlap on the GPU race and must be serialised.
 */
MH3_API int mh3_quantize_qkv_noalloc(const mh3_qkv_quant_args* args, void* stream);

/* ------------------------------------------------------------------------ */
/* Per-row e4m3 quantisation                                                 */
/* ------------------------------------------------------------------------ */
/*
 * Replaces ``_quantize_rows_kernel`` / ``quantize_rows``
 * (kernels/fp8_linear.py:8-42): x8[m,:] = e4m3(clamp(x[m,:]/s[m], +-448)),
 * s[m] = max(absmax(x[m,:]), 1e-12)/448.  x is [M,K] bf16, f16 or f32
 * (in_dtype; the reference's kernel loads any float dtype, :19) with row
 * stride x_stride (elements); x8 is contiguous [M,K]; scale is [M] f32.
 */
MH3_API int mh3_quantize_rows(const void* x, int64_t x_stride, int32_t in_dtype, int64_t M, int64_t K, void* x8,
                      float* scale, void* stream);

/* ------------------------------------------------------------------------ */
/* Scaled GEMM with fused bias and low-rank (LoRA) epilogue                  */
/* ------------------------------------------------------------------------ */
/*
 * Replaces ``torch._scaled_mm(x8, w8.t(), scale_a=x_scale, scale_b=w_scale,
 * bias=bias, out_dtype=bf16)`` plus the per-adapter LoRA loop of
 * ``FP8Linear.forward`` (kernels/fp8_linear.py:95-108, :45-55):
 *
 *   out[m,n] = bf16( (sum_k a[m,k]*b[n,k] + sum_r a2[m,r]*b2[n,r])
 *                    * rs[m] * cs[n] + bias[n] )
 *
 * a [M,K], b [N,K]: e4m3 or bf16 (ab_dtype), K contiguous, row strides lda /
 * ldb in elements (multiples of 16 bytes).  rs = row_scale[m] (or
 * 1/row_scale[m] with row_scale_inv), cs = col_scale[n]; NULL means 1.  bias:
 * bf16 [N] or NULL.  a2 [M,R], b2 [N,R]: optional bf16 low-rank operands
 * accumulated into the same fp32 accumulator (R = 0: none); FP8Linear passes
 * a2 = (x A^T)/x_scale and b2 = lora_scale*B/w_scale so the epilogue adds
 * the adapter delta.  out: bf16 [M,N], row stride ldo.  N, ldo, R multiples
 * of 8.
 */
typedef struct mh3_gemm_args {
  int64_t M, N, K, R;
  int32_t ab_dtype; /* MH3_DTYPE_E4M3 or MH3_DTYPE_BF16 */
  int32_t row_scale_inv;
  const void* a;
  int64_t lda;
  const void* b;
  int64_t ldb;
  const float* row_scale;
  const float* col_scale;
  const void* bias;
  const void* a2;
  int64_t lda2;
  const void* b2;
  int64_t ldb2;
  void* out;
  int64_t ldo;
  int* err;
  uint64_t timeout_ns;
  int32_t test_flags; /* 0; MH3_TEST_* bits (ABI version 4) */
  int32_t reserved1;
} mh3_gemm_args;

MH3_API int mh3_scaled_gemm(const mh3_gemm_args* args, void* stream);

/*
 * Exact widening of e4m3 to f16 (every e4m3 value is an f16 value): dst[i] =
 * src[i] for n contiguous elements.  Feeds pre-quantised e4m3 V to the
 * attention kernel's f16 PV product.  No reference counterpart (the
 * reference's PV product is e4m3 only).
 */
MH3_API int mh3_widen_e4m3_to_f16(const void* src, void* dst, int64_t n, void* stream);

/* ------------------------------------------------------------------------ */
/* Per-(batch, head) quantisation (the scale granularity of the benchmark workloads) */
/* ------------------------------------------------------------------------ */
/*
 * The per-(batch, head) form of the reference's Q/K/V quantisation
 * (kernels/fp8_attention.py:39-170 with one scale per (b,h) instead of per
 * 128-row block), as a sequence-sharded DiT block holds it: x is [B, S, H, D]
 * bf16/f16 under element strides sb/ss/sh (D contiguous, strides multiples
 * of 8, 16-byte aligned).
 *
 * Head selection: the H heads form P = H/head_block blocks (one per rank of
 * a head-parallel group); selected are heads p*head_block + head_off + i for
 * every block p and i < heads_sel, numbered j = p*heads_sel + i (nsel =
 * P*heads_sel).  All heads: head_block = heads_sel = H, head_off = 0.
 *
 * mh3_absmax_bh: amax[b*nsel+j] = max |x[b,:,head(j),:]| (f32; overwritten).
 * mh3_quantize_bh: y = x / scale[b*nsel+j] (IEEE division) rounded to e4m3
 * (after clamping to +-448) or f16 (out_dtype), written block-major: out
 * [P, B, S, heads_sel, D] contiguous - the send buffer of a head-parallel
 * (Ulysses) all-to-all, for all of a rank's heads or for a group of them.
 */
MH3_API int mh3_absmax_bh(const void* x, int32_t in_dtype, int64_t B, int64_t S, int64_t H, int64_t D, int64_t sb,
                          int64_t ss, int64_t sh, int32_t head_block, int32_t head_off, int32_t heads_sel,
                          float* amax, void* stream);
MH3_API int mh3_quantize_bh(const void* x, int32_t in_dtype, int64_t B, int64_t S, int64_t H, int64_t D, int64_t sb,
                            int64_t ss, int64_t sh, int32_t head_block, int32_t head_off, int32_t heads_sel,
                            const float* scale, int32_t out_dtype, void* out, void* stream);

/*
 * Per-(segment, head) variants for packed variable-length batches (the
 * cu_seqlens layout of the varlen attention): x is one packed [S, H, D]
 * shard (token stride ss, head stride sh, elements) whose rows
 * [seg[z], seg[z+1]) form segment z, z < nseg.  ``seg`` is int32 [nseg+1]
 * on the device, non-decreasing; each entry is clamped to [0, S], so a
 * sequence-parallel rank may pass the global cu_seqlens shifted by its first
 * token.  Head selection as above.
 *
 * mh3_absmax_seg: amax[z*nsel+j] = max |x[rows of z, head(j), :]| (f32,
 * overwritten; 0 for an empty segment).
 * mh3_quantize_seg: y = x / scale[z*nsel+j] for the rows of segment z, as
 * mh3_quantize_bh with B = 1: out [P, S, heads_sel, D] contiguous.  Rows
 * outside every segment are written as zeros.
 * No reference counterpart: the reference has no varlen path.  These give
 * the per-(sequence, head) absmax/448 scales of the packed video+audio
 * workload, on one GPU or across sequence-parallel ranks.
 */
MH3_API int mh3_absmax_seg(const void* x, int32_t in_dtype, int64_t S, int64_t H, int64_t D, int64_t ss, int64_t sh,
                           int32_t head_block, int32_t head_off, int32_t heads_sel, const int32_t* seg, int32_t nseg,
                           float* amax, void* stream);
MH3_API int mh3_quantize_seg(const void* x, int32_t in_dtype, int64_t S, int64_t H, int64_t D, int64_t ss, int64_t sh,
                             int32_t head_block, int32_t head_off, int32_t heads_sel, const int32_t* seg,
                             int32_t nseg, const float* scale, int32_t out_dtype, void* out, void* stream);

/* ------------------------------------------------------------------------ */
/* Exchange buffers shared between processes (CUDA IPC)                     */
/* ------------------------------------------------------------------------ */
/*
 * For a head-parallel exchange over copy engines: each rank allocates its
 * send buffers with mh3_peer_alloc (one device allocation each, on the
 * current device), exports them with mh3_peer_handle (MH3_PEER_HANDLE_BYTES
 * opaque bytes, to be passed to the other processes of the node), and maps a
 * peer's buffer with mh3_peer_open, which returns a pointer valid on the
 * current device (peer access enabled on first use).  Chunks are then
 * pulled with mh3_copy_rows.  mh3_peer_handle needs the pointer
 * mh3_peer_alloc returned.  Close every mapping (mh3_peer_close) before the
 * owner frees the buffer (mh3_peer_free).  Plain peer mappings only; no
 * multicast object is created.  No reference counterpart.
 */
#define MH3_PEER_HANDLE_BYTES 64
MH3_API int mh3_peer_alloc(int64_t bytes, void** ptr);
MH3_API int mh3_peer_free(void* ptr);
MH3_API int mh3_peer_handle(const void* ptr, void* handle);
MH3_API int mh3_peer_open(const void* handle, void** ptr);
MH3_API int mh3_peer_close(void* ptr);

/* ------------------------------------------------------------------------ */
/* Strided host<->device row copies                                         */
/* ------------------------------------------------------------------------ */
/*
 * rows x row_bytes from src (row pitch src_pitch bytes) to dst (row pitch
 * dst_pitch bytes), asynchronously on ``stream``, either direction between
 * pinned host memory and device memory, or device to device (also from a
 * peer's buffer mapped with mh3_peer_open: a copy-engine copy).  Moves one
 * head group of a host-resident [B, S, H, D] shard - a run of heads in every
 * token row - without staging it through a contiguous host copy.  No
 * reference counterpart (the reference's tensors are device-resident).
 */
MH3_API int mh3_copy_rows(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch, int64_t row_bytes,
                          int64_t rows, void* stream);

/* ------------------------------------------------------------------------ */
/* Step-residual cache reductions                                           */
/* ------------------------------------------------------------------------ */
/*
 * Replaces runtime/step_cache.py:39-52 (_rel_diff) and the clone of h1 that
 * follows it (:151): one pass over n elements of h1 and prev (bf16, f16 or
 * f32, 16-byte aligned) writes sums[0] = sum |h1 - prev| and
 * sums[1] = sum |prev| (double, summed in a fixed order: the same bits for
 * the same inputs), and with ``copy`` != 0 overwrites prev with h1 in the
 * same pass.  rel = (sums[0]/n) / max(sums[1]/n, 1e-6) on the caller's
 * side.  ``workspace``: mh3_step_diff_workspace_bytes() bytes of device
 * memory, 16-byte aligned.
 */
MH3_API uint64_t mh3_step_diff_workspace_bytes(void);
MH3_API int mh3_step_diff(const void* h1, void* prev, int32_t dtype, int64_t n, int32_t copy, double* sums,
                          void* workspace, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MH3_B200_H_ */
