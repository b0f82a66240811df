// FP8 (e4m3) non-causal flash-attention forward for sm_100a.
//
// Replaces the reference's ``_fp8_attn_kernel`` (kernels/fp8_attention.py:190-297
// of viragadel6/minimaxh3).  Same contract: e4m3 Q, K, V with fp32 dequant
// scales in, bf16/fp16 out, optional per-key mask or bias.  Different
// machinery:
//
//  * one CTA = two 128-row Q tiles sharing every K/V tile, 384 threads:
//      warps 0-3   softmax warpgroup for Q tile 0 (thread i owns row i)
//      warps 4-7   softmax warpgroup for Q tile 1
//      warp  8     TMA producer (K and V tiles through a 3-stage mbarrier ring)
//      warp  9     tcgen05 MMA issuer; owns the 512-column TMEM allocation
//      warps 10-11 idle (complete the third warpgroup for setmaxnreg)
//  * TMEM columns: S0 [0,128)  S1 [128,256)  O0 [256,256+D)  O1 [256+D,256+2D);
//    P (f16: 64 columns, e4m3: 32) is written over the first columns of S.
//  * S = Q K^T is tcgen05.mma kind::f8f6f4; O += P V is kind::f16 with f16 P
//    and V (default) or kind::f8f6f4 with e4m3 P and V.  V stays in its
//    natural [key, channel] layout: the PV MMA reads it as an MN-major B
//    operand, so no transposed copy of V is ever made.
//  * MMA order per Q tile t and KV step j: after P(t, j): PV(t, j), then
//    S(t, j+1).  With f16 PV, P(t, j) is released in two key halves and the
//    first half's PV runs while the softmax computes the second half.  With e4m3 PV the upper half of S(t, j+1) (keys 64..127,
//    columns P never touches) is issued earlier, as soon as the softmax has
//    read S(t, j) into registers, and only the lower half follows PV.  The
//    two Q tiles alternate, so the tensor core works on one tile while the
//    other tile's softmax runs.
//  * softmax (one thread per row): tile max, lazy running max (raised only
//    when a tile's max exceeds it by a threshold, the idea of the reference's
//    ``rowmax > m + 8`` at :267; the rare raise rescales the row of O in TMEM),
//    then P = 2^(s*c - m + offset) with the dequant scales folded into one
//    packed FMA per pair and two f32 MUFU ex2.
//  * every mbarrier wait is bounded; a timeout sets an error word and lets the
//    CTA run to teardown (TMEM is always freed, copies in flight drained).
#include <mutex>
#include <string>
#include <type_traits>

#include "mh3_b200.h"
#include "mh3_internal.h"
#include "ptx.cuh"

namespace mh3 {
namespace attn {

constexpr int BM = 128;  // rows per Q tile
constexpr int BN = 128;  // keys per K/V tile
constexpr int KST = 3;   // K ring depth
constexpr int VST = 3;   // V ring depth
constexpr int NUM_THREADS = 384;
// Lazy max threshold and P offset (log2 units), P = 2^(x - m + offset):
//  e4m3 P: P <= 2^(4 + 4.5) < 448, and the row max lands on 2^4 (exact);
//  f16 P:  P <= 2^12, far inside f16; the wide threshold makes the running
//          max (and the O rescale) rise in very few tiles.
constexpr float LAZY_T8 = 4.5f;
constexpr float P_OFFSET8 = 4.0f;
constexpr float LAZY_T16 = 12.0f;
constexpr float P_OFFSET16 = 0.0f;

// P(j) is handed to the PV MMAs in N key parts, each as soon as the softmax
// has stored it.  With f16 PV (the tensor core the busier side) splitting
// takes most of PV off the softmax -> PV -> S chain; with e4m3 PV the extra
// store waits cost more than they save.
#ifndef MH3_P_PARTS
#define MH3_P_PARTS 2
#endif
template <bool PV16>
struct PParts {
  static constexpr int N = PV16 ? MH3_P_PARTS : 1;
};

struct Params {
  CUtensorMap tmq;  // e4m3 (D, S, H, B), box (D, 128, 1, 1)
  CUtensorMap tmk;
  CUtensorMap tmv;
  void* out;
  long long osb, osh, oss;  // output strides in elements (d contiguous)
  const float* sq;
  long long sqb, sqh, sqblk;
  const float* sk;
  long long skb, skh, skblk;
  const float* sv;
  long long svb, svh, svd;
  float logit_scale_log2;
  int H, Sq, Sk;
  const int* cuq;  // varlen: cumulative sequence starts (B+1), or null
  const int* cuk;
  const float* kbias2;  // additive per-key bias in log2 units, [B, ceil(Sk/128)*128], or null
  long long kbias_sb;
  int* err;
  unsigned long long timeout_ns;
  const int* kv_len;  // per-batch key count (padding past it is skipped), or null
  int test_flags;     // MH3_TEST_* bits (tests of the bounded waits); 0 in normal use
};

template <int D, bool PV16>
struct __align__(1024) Smem {
  uint8_t q[2][BM * D];
  uint8_t k[KST][BN * D];
  uint8_t v[VST][BN * D * (PV16 ? 2 : 1)];
  uint64_t bar_q;
  uint64_t bar_kfull[KST];
  uint64_t bar_kempty[KST];
  uint64_t bar_vfull[VST];
  uint64_t bar_vempty[VST];
  uint64_t bar_s[2];
  uint64_t bar_sld[2];  // softmax has read S(j) into registers
  uint64_t bar_p[2][4];  // [tile][key part]: that part of P(j) is in TMEM
  uint64_t bar_o;
  uint64_t bar_never;  // nothing arrives on it (test hook)
  uint32_t tmem_base;
  int abort_flag;
};

template <int D, bool PV16>
constexpr uint32_t smem_bytes() {
  return (uint32_t)sizeof(Smem<D, PV16>) + 1024;
}

__device__ __forceinline__ float u2f(uint32_t x) { return __uint_as_float(x); }
__device__ __forceinline__ uint32_t f2u(float x) { return __float_as_uint(x); }

// PV16: the PV product runs on f16 operands (P = f16 straight from the packed
// ex2, V an f16 tensor pre-scaled per channel) instead of e4m3; same flow.
template <int D, bool OUT_F16, bool HAS_BIAS, bool PV16>
__global__ void __launch_bounds__(NUM_THREADS, 1) fwd_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  using SmemT = Smem<D, PV16>;
  SmemT& sm = *reinterpret_cast<SmemT*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int h = blockIdx.y;
  const int b = blockIdx.z;

  int q_start = 0, q_len = p.Sq, k_start = 0, k_len = p.Sk, bcoord = b;
  if (p.cuq != nullptr) {
    q_start = p.cuq[b];
    q_len = p.cuq[b + 1] - q_start;
    k_start = p.cuk[b];
    k_len = p.cuk[b + 1] - k_start;
    bcoord = 0;
  }
  if (p.kv_len != nullptr) k_len = min(k_len, max(0, __ldg(p.kv_len + b)));  // tiles past it are all masked
  const int qt0 = blockIdx.x * 2;
  if (qt0 * BM >= q_len) return;  // uniform over the CTA, before any barrier
  const int nk = (k_len + BN - 1) / BN;

  // Swizzle-128B (D=128) or swizzle-64B (D=64) tiles: row = D bytes.
  constexpr uint32_t kLayout = (D == 128) ? kLayoutSW128 : kLayoutSW64;
  constexpr uint32_t kRowBytes = D;
  constexpr uint32_t kTileBytes = BN * D;
  constexpr uint32_t kVTileBytes = BN * D * (PV16 ? 2 : 1);

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&sm.bar_q), 1);
    for (int i = 0; i < KST; ++i) {
      mbar_init(smem_u32(&sm.bar_kfull[i]), 1);
      mbar_init(smem_u32(&sm.bar_kempty[i]), 1);
    }
    for (int i = 0; i < VST; ++i) {
      mbar_init(smem_u32(&sm.bar_vfull[i]), 1);
      mbar_init(smem_u32(&sm.bar_vempty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&sm.bar_s[i]), 1);
      mbar_init(smem_u32(&sm.bar_sld[i]), 4);
      for (int k = 0; k < 4; ++k) mbar_init(smem_u32(&sm.bar_p[i][k]), 4);
    }
    mbar_init(smem_u32(&sm.bar_o), 1);
    mbar_init(smem_u32(&sm.bar_never), 1);
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(&sm.tmem_base), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const WaitGuard g{&sm.abort_flag, p.err, p.timeout_ns};

  if (warp >= 8) {
    setmaxnreg_dec<80>();
    if (warp == 8 && lane == 0) {
      // ---------------------------------------------------------------- producer
      tma_prefetch_desc(&p.tmq);
      tma_prefetch_desc(&p.tmk);
      tma_prefetch_desc(&p.tmv);
      // Test hook (MH3_TEST_STALL_PRODUCER): wait on a barrier nothing arrives
      // on, so the bounded wait runs out and the CTA takes its abort path
      // with no copy issued.
      const bool go = (p.test_flags & MH3_TEST_STALL_PRODUCER) == 0 || mbar_wait(smem_u32(&sm.bar_never), 0, g);
      const uint32_t bq = smem_u32(&sm.bar_q);
      if (go) {
        mbar_arrive_expect_tx(bq, 2 * BM * D);
        tma_load_4d(smem_u32(sm.q[0]), &p.tmq, bq, 0, q_start + qt0 * BM, h, bcoord);
        tma_load_4d(smem_u32(sm.q[1]), &p.tmq, bq, 0, q_start + (qt0 + 1) * BM, h, bcoord);
      }
      int issued = 0;
      for (int j = 0; go && j < nk; ++j) {
        const int ks = j % KST;
        const uint32_t kph = (uint32_t)(j / KST) & 1u;
        if (!mbar_wait(smem_u32(&sm.bar_kempty[ks]), kph ^ 1u, g)) break;
        mbar_arrive_expect_tx(smem_u32(&sm.bar_kfull[ks]), kTileBytes);
        tma_load_4d(smem_u32(sm.k[ks]), &p.tmk, smem_u32(&sm.bar_kfull[ks]), 0, k_start + j * BN, h, bcoord);
        const int vs = j % VST;
        const uint32_t vph = (uint32_t)(j / VST) & 1u;
        if (!mbar_wait(smem_u32(&sm.bar_vempty[vs]), vph ^ 1u, g)) {
          issued = -(j + 1);  // K(j) issued, V(j) not
          break;
        }
        mbar_arrive_expect_tx(smem_u32(&sm.bar_vfull[vs]), kVTileBytes);
        if constexpr (PV16) {
          // f16 V: 64-channel boxes (128 bytes wide), one swizzle-128B atom column each
#pragma unroll
          for (int c = 0; c < D / 64; ++c)
            tma_load_4d(smem_u32(sm.v[vs]) + c * (BN * 128), &p.tmv, smem_u32(&sm.bar_vfull[vs]), c * 64,
                        k_start + j * BN, h, bcoord);
        } else {
          tma_load_4d(smem_u32(sm.v[vs]), &p.tmv, smem_u32(&sm.bar_vfull[vs]), 0, k_start + j * BN, h, bcoord);
        }
        issued = j + 1;
      }
      // Teardown: let the last copy issued into each stage land before exit.
      const int nk_issued = issued >= 0 ? issued : -issued;
      const int nv_issued = issued >= 0 ? issued : -issued - 1;
      if (go) mbar_wait_teardown(bq, 0);
      for (int j = (nk_issued > KST ? nk_issued - KST : 0); j < nk_issued; ++j)
        mbar_wait_teardown(smem_u32(&sm.bar_kfull[j % KST]), (uint32_t)(j / KST) & 1u);
      for (int j = (nv_issued > VST ? nv_issued - VST : 0); j < nv_issued; ++j)
        mbar_wait_teardown(smem_u32(&sm.bar_vfull[j % VST]), (uint32_t)(j / VST) & 1u);
    } else if (warp == 9 && lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      constexpr uint32_t kIdescS = idesc_e4m3(BM, BN, false, false);
      constexpr uint32_t kIdescS64 = idesc_e4m3(BM, BN / 2, false, false);
      // Early upper half of the next S (see the header): pays with e4m3 PV;
      // with f16 PV the tensor core is the busier side and two N=64 halves
      // (Q read twice) cost more than one N=128 S after PV.
#ifndef MH3_EARLY_HALF
#define MH3_EARLY_HALF (PV16 ? 0 : 1)
#endif
      constexpr bool kEarlyHalf = MH3_EARLY_HALF;
      constexpr int kPHalves = PParts<PV16>::N;
      constexpr uint32_t kIdescO = PV16 ? idesc_f16(BM, D, false, true) : idesc_e4m3(BM, D, false, true);
      // Descriptors are built once: a Q tile, K/V stage or K step only moves
      // the start-address field (bytes >> 4).  K-major operands (Q, K): 8-row
      // swizzle atoms of D bytes per row, 32 bytes (32 e4m3) of K per MMA.
      // MN-major V: e4m3 - one swizzle atom across D channels, 32 keys per
      // MMA; f16 - 64-channel atom columns BN*128 bytes apart, 16 keys per MMA.
      const uint64_t dq0 = smem_desc(smem_u32(sm.q[0]), 16, 8 * kRowBytes, kLayout);
      const uint64_t dk0 = smem_desc(smem_u32(sm.k[0]), 16, 8 * kRowBytes, kLayout);
      const uint64_t dv0 = PV16 ? smem_desc(smem_u32(sm.v[0]), BN * 128, 8 * 128, kLayoutSW128)
                                : smem_desc(smem_u32(sm.v[0]), kTileBytes, 8 * kRowBytes, kLayout);
      constexpr uint64_t kQStep = (BM * D) >> 4;
      constexpr uint64_t kKStage = kTileBytes >> 4;
      constexpr uint64_t kVStage = kVTileBytes >> 4;
      constexpr uint64_t kVk = PV16 ? (16 * 128) >> 4 : (32 * kRowBytes) >> 4;
      auto tS = [&](int t) { return tmem + (uint32_t)(t * 128); };
      auto tO = [&](int t) { return tmem + 256u + (uint32_t)(t * D); };
      auto issue_s = [&](int t, int ks) {
        const uint64_t dq = dq0 + (uint64_t)t * kQStep;
        const uint64_t dk = dk0 + (uint64_t)ks * kKStage;
        mma_f8_ss(tS(t), dq, dk, kIdescS, 0u);
#pragma unroll
        for (int kk = 1; kk < D / 32; ++kk) mma_f8_ss(tS(t), dq + 2u * kk, dk + 2u * kk, kIdescS, 1u);
      };
      // Half of S(t, j+1): keys [half*64, half*64+64) into S columns
      // [half*64, half*64+64) (N = 64; K rows 64.. start on a swizzle atom).
      auto issue_s_half = [&](int t, int ks, int half) {
        const uint64_t dq = dq0 + (uint64_t)t * kQStep;
        const uint64_t dk = dk0 + (uint64_t)ks * kKStage + (uint64_t)((half * (BN / 2) * kRowBytes) >> 4);
        const uint32_t d = tS(t) + (uint32_t)(half * (BN / 2));
        mma_f8_ss(d, dq, dk, kIdescS64, 0u);
#pragma unroll
        for (int kk = 1; kk < D / 32; ++kk) mma_f8_ss(d, dq + 2u * kk, dk + 2u * kk, kIdescS64, 1u);
      };
      bool ok = mbar_wait(smem_u32(&sm.bar_q), 0, g);
      if (nk > 0) {
        ok = mbar_wait(smem_u32(&sm.bar_kfull[0]), 0, g) && ok;
        tc_fence_after();
        issue_s(0, 0);
        mma_commit(smem_u32(&sm.bar_s[0]));
        issue_s(1, 0);
        mma_commit(smem_u32(&sm.bar_s[1]));
        mma_commit(smem_u32(&sm.bar_kempty[0]));
      }
      // Per tile t and step j: S(t, j+1) keys 64..127 go into S columns
      // 64..127 as soon as the softmax has read S(t, j) (P only overwrites
      // columns 0..63); PV(t, j) then S(t, j+1) keys 0..63 follow P(t, j).
      for (int j = 0; j < nk; ++j) {
        const int vs = j % VST;
        mbar_wait(smem_u32(&sm.bar_vfull[vs]), (uint32_t)(j / VST) & 1u, g);
        const int ks = (j + 1) % KST;
        const bool has_next = j + 1 < nk;
        if (has_next) mbar_wait(smem_u32(&sm.bar_kfull[ks]), (uint32_t)((j + 1) / KST) & 1u, g);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (kEarlyHalf && has_next) {
            mbar_wait(smem_u32(&sm.bar_sld[t]), (uint32_t)j & 1u, g);
            tc_fence_after();
            issue_s_half(t, ks, 1);
          }
          // PV in key parts, each issued as soon as the softmax has stored
          // that part of P (only the last part follows the softmax).
#pragma unroll
          for (int hf = 0; hf < kPHalves; ++hf) {
            mbar_wait(smem_u32(&sm.bar_p[t][hf]), (uint32_t)j & 1u, g);
            tc_fence_after();
            constexpr int kPer = (PV16 ? BN / 16 : BN / 32) / kPHalves;
            const uint64_t dv = dv0 + (uint64_t)vs * kVStage;
#pragma unroll
            for (int kk = hf * kPer; kk < hf * kPer + kPer; ++kk) {
              const uint32_t acc = (j > 0 || kk > 0) ? 1u : 0u;
              if constexpr (PV16)
                mma_f16_ts(tO(t), tS(t) + (uint32_t)(kk * 8), dv + kVk * kk, kIdescO, acc);
              else
                mma_f8_ts(tO(t), tS(t) + (uint32_t)(kk * 8), dv + kVk * kk, kIdescO, acc);
            }
          }
          if (t == 1) mma_commit(smem_u32(&sm.bar_vempty[vs]));
          if (has_next) {
            if constexpr (kEarlyHalf)
              issue_s_half(t, ks, 0);
            else
              issue_s(t, ks);
            mma_commit(smem_u32(&sm.bar_s[t]));
            if (t == 1) mma_commit(smem_u32(&sm.bar_kempty[ks]));
          }
        }
      }
      mma_commit(smem_u32(&sm.bar_o));
      (void)ok;
      // Every MMA must be finished before the CTA frees TMEM.
      mbar_wait_teardown(smem_u32(&sm.bar_o), 0);
    }
  } else {
    // ------------------------------------------------------------------ softmax
    setmaxnreg_inc<200>();
    const int t = warp >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    const uint32_t tS = tmem + (uint32_t)(t * 128) + lane_off;
    const uint32_t tO = tmem + 256u + (uint32_t)(t * D) + lane_off;
    const int qt = qt0 + t;
    const bool tile_live = qt * BM < q_len;
    const float sq = tile_live ? __ldg(p.sq + b * p.sqb + h * p.sqh + (long long)qt * p.sqblk) : 1.0f;
    const float cq = p.logit_scale_log2 * sq;
    const float* skp = p.sk + b * p.skb + h * p.skh;
    const float* biasp = HAS_BIAS ? (p.kbias2 + b * p.kbias_sb) : nullptr;

    float m = -1.0e30f;  // running max (log2 units), raised lazily; -1e30 = no key yet
    float l = 0.0f;  // running sum of P
    // K scale of the current tile, loaded one tile ahead so that its latency
    // overlaps the wait for S (block scales change every tile).
    float sk_cur = nk > 0 ? __ldg(skp) : 1.0f;
    for (int j = 0; j < nk; ++j) {
      const float sk_next = (j + 1 < nk) ? __ldg(skp + (long long)(j + 1) * p.skblk) : 1.0f;
      mbar_wait(smem_u32(&sm.bar_s[t]), (uint32_t)j & 1u, g);
      tc_fence_after();
      uint32_t sr[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS + (uint32_t)(c * 32), sr[c]);
      tmem_wait_ld();
      // S(j) is in registers: S columns 64..127 may take the next S.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&sm.bar_sld[t]));

      const float c_tile = cq * sk_cur;
      sk_cur = sk_next;
      const int rem = k_len - j * BN;
      // Raw S chunk c (32 keys) -> the value P is taken from: s*c + bias2 with
      // bias2 = -inf for masked or padding keys (HAS_BIAS), else s with the
      // keys past the end of the sequence set to -inf.
      auto prep = [&](int c) {
        if constexpr (HAS_BIAS) {
          const float4* bp = reinterpret_cast<const float4*>(biasp + (long long)j * BN) + c * 8;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 bb = __ldg(bp + i);
            sr[c][4 * i + 0] = f2u(fmaf(u2f(sr[c][4 * i + 0]), c_tile, bb.x));
            sr[c][4 * i + 1] = f2u(fmaf(u2f(sr[c][4 * i + 1]), c_tile, bb.y));
            sr[c][4 * i + 2] = f2u(fmaf(u2f(sr[c][4 * i + 2]), c_tile, bb.z));
            sr[c][4 * i + 3] = f2u(fmaf(u2f(sr[c][4 * i + 3]), c_tile, bb.w));
          }
        } else {
          if (rem < BN) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (c * 32 + i >= rem) sr[c][i] = f2u(-INFINITY);
          }
        }
      };
#pragma unroll
      for (int c = 0; c < 4; ++c) prep(c);
      const float2 cc = HAS_BIAS ? make_float2(1.0f, 1.0f) : make_float2(c_tile, c_tile);
      constexpr float kLazy = PV16 ? LAZY_T16 : LAZY_T8;
      constexpr float kOffset = PV16 ? P_OFFSET16 : P_OFFSET8;

      // Tile max; raise the running max lazily and rescale this row of O in
      // TMEM on the rare raise (PV(j-1) has completed: the commit behind
      // bar_s(j) tracks every MMA issued before S(j)).
      float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        mx0 = fmax3(mx0, u2f(sr[0][i]), u2f(sr[0][i + 1]));
        mx1 = fmax3(mx1, u2f(sr[1][i]), u2f(sr[1][i + 1]));
        mx2 = fmax3(mx2, u2f(sr[2][i]), u2f(sr[2][i + 1]));
        mx3 = fmax3(mx3, u2f(sr[3][i]), u2f(sr[3][i + 1]));
      }
      const float rmax = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
      const float tmax = HAS_BIAS ? rmax : rmax * c_tile;
      const bool upd = tmax > m + kLazy;
      const float m_new = upd ? tmax : m;
      const float alpha = ex2_approx(m - m_new);  // 1 when kept, 0 from the sentinel
      if (j > 0 && __any_sync(0xffffffffu, upd)) {
#pragma unroll
        for (int c = 0; c < D / 16; ++c) {
          uint32_t o[16];
          tmem_ld16(tO + (uint32_t)(c * 16), o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = f2u(u2f(o[i]) * alpha);
          tmem_st16(tO + (uint32_t)(c * 16), o);
        }
      }
      l *= alpha;
      m = m_new;

      // P = 2^(s*c - m + offset), two f32 MUFU ex2 per pair, stored over the
      // first S columns as f16 pairs (PV16: 8 columns per 16 keys) or e4m3
      // quads (4 columns); the row sum takes the unrounded f32 values.
      const float nb = kOffset - m;
      const float2 nn = make_float2(nb, nb);
      float2 lsum2 = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int g16 = 0; g16 < 8; ++g16) {  // 16 keys per group
        const int c = g16 >> 1, i0 = (g16 & 1) * 8;
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float2 x = ffma2(make_float2(u2f(sr[c][2 * (i0 + i)]), u2f(sr[c][2 * (i0 + i) + 1])), cc, nn);
          const float2 pp = make_float2(ex2_approx(x.x), ex2_approx(x.y));
          lsum2 = __fadd2_rn(lsum2, pp);
          if constexpr (PV16) {
            pk[i] = cvt_f16x2(pp.y, pp.x);
          } else {
            const uint32_t p2 = cvt_e4m3x2_f32(pp.y, pp.x);
            if (i & 1)
              pk[i >> 1] |= p2 << 16;
            else
              pk[i >> 1] = p2;
          }
        }
        if constexpr (PV16)
          tmem_st8(tS + (uint32_t)(g16 * 8), pk);
        else
          tmem_st4(tS + (uint32_t)(g16 * 4), pk);
        constexpr int kGroupsPerPart = 8 / PParts<PV16>::N;
        if (g16 % kGroupsPerPart == kGroupsPerPart - 1) {  // a part of P is in TMEM: release it
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&sm.bar_p[t][g16 / kGroupsPerPart]));
        }
      }
      l += lsum2.x + lsum2.y;
    }

    // ---------------------------------------------------------------- epilogue
    const int grow = qt * BM + row;
    const bool row_ok = grow < q_len;
    using OutT = typename std::conditional<OUT_F16, __half, __nv_bfloat16>::type;
    OutT* orow = reinterpret_cast<OutT*>(p.out) + b * p.osb + h * p.osh + (long long)(q_start + grow) * p.oss;
    const float* svp = p.sv + b * p.svb + h * p.svh;
    if (nk > 0) {
      mbar_wait(smem_u32(&sm.bar_o), 0, g);
      tc_fence_after();
    }
    const float inv_l = 1.0f / fmaxf(l, 1.0e-30f);
#pragma unroll
    for (int c = 0; c < D / 32; ++c) {
      uint32_t o[32];
      if (nk > 0) {
        tmem_ld32(tO + (uint32_t)(c * 32), o);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0u;
      }
      uint32_t packed[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int d0 = c * 32 + 2 * i;
        const float a0 = u2f(o[2 * i]) * __ldg(svp + d0 * p.svd) * inv_l;
        const float a1 = u2f(o[2 * i + 1]) * __ldg(svp + (d0 + 1) * p.svd) * inv_l;
        if constexpr (OUT_F16) {
          __half2 hv = __floats2half2_rn(a0, a1);
          packed[i] = *reinterpret_cast<uint32_t*>(&hv);
        } else {
          __nv_bfloat162 hv = __floats2bfloat162_rn(a0, a1);
          packed[i] = *reinterpret_cast<uint32_t*>(&hv);
        }
      }
      if (row_ok) {
        uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          dst[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------

// dims (D, S, H, B) innermost first; element strides ss/sh/sb for dims 1..3.
// e4m3: box (D, 128) with a D-byte swizzle; f16: box (64, 128), swizzle 128B.
static int make_map(CUtensorMap* map, const void* base, int D, long long S, int H, int B, long long ss,
                    long long sh, long long sb, bool f16) {
  const long long es = f16 ? 2 : 1;
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)(ss * es), (cuuint64_t)(sh * es), (cuuint64_t)(sb * es)};
  const cuuint32_t box[4] = {(cuuint32_t)(f16 ? 64 : D), (cuuint32_t)BN, 1u, 1u};
  const cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  const CUtensorMapSwizzle sw =
      (f16 || D == 128) ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  return encode_tiled(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 4,
                      const_cast<void*>(base), dims, strides, box, estr, sw);
}

template <int D, bool F16, bool BIAS, bool PV16>
static cudaError_t launch(const Params& p, dim3 grid, cudaStream_t st) {
  auto kern = fwd_kernel<D, F16, BIAS, PV16>;
  constexpr uint32_t bytes = smem_bytes<D, PV16>();
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  });
  if (attr_err != cudaSuccess) return attr_err;
  kern<<<grid, NUM_THREADS, bytes, st>>>(p);
  return cudaGetLastError();
}

template <int D, bool PV16>
static cudaError_t dispatch(const Params& p, dim3 grid, cudaStream_t st, bool f16, bool bias) {
  if (f16) return bias ? launch<D, true, true, PV16>(p, grid, st) : launch<D, true, false, PV16>(p, grid, st);
  return bias ? launch<D, false, true, PV16>(p, grid, st) : launch<D, false, false, PV16>(p, grid, st);
}

}  // namespace attn
}  // namespace mh3

using namespace mh3;

extern "C" int mh3_fp8_attention_fwd(const mh3_attn_args* a, void* stream) {
  const mh3::NvtxRange nvtx_range("mh3_fp8_attention_fwd");
  if (a == nullptr) return fail(MH3_ERR_INVALID, "mh3_fp8_attention_fwd: null args");
  const int D = a->head_dim;
  if (D != 64 && D != 128) return fail(MH3_ERR_INVALID, "head_dim must be 64 or 128");
  if (a->batch <= 0 || a->heads <= 0) return fail(MH3_ERR_INVALID, "batch and heads must be positive");
  const bool varlen = a->cu_seqlens_q != nullptr || a->cu_seqlens_k != nullptr;
  if (varlen && (a->cu_seqlens_q == nullptr || a->cu_seqlens_k == nullptr))
    return fail(MH3_ERR_INVALID, "varlen needs both cu_seqlens_q and cu_seqlens_k");
  if (varlen && a->max_seqlen_q <= 0) return fail(MH3_ERR_INVALID, "varlen needs max_seqlen_q > 0");
  if (!varlen && (a->seqlen_q <= 0 || a->seqlen_k <= 0))
    return fail(MH3_ERR_INVALID, "seqlen_q and seqlen_k must be positive");
  if (!a->q8 || !a->k8 || !a->v8 || !a->out || !a->scale_q || !a->scale_k || !a->scale_v)
    return fail(MH3_ERR_INVALID, "null tensor pointer");
  if (a->out_dtype != MH3_DTYPE_BF16 && a->out_dtype != MH3_DTYPE_F16)
    return fail(MH3_ERR_INVALID, "out_dtype must be bf16 or f16");
  if (a->v_dtype != MH3_DTYPE_E4M3 && a->v_dtype != MH3_DTYPE_F16)
    return fail(MH3_ERR_INVALID, "v_dtype must be e4m3 or f16");
  // TMA: 16-byte aligned bases and strides; output rows written as 16-byte vectors.
  auto al16 = [](const void* p_) { return ((uintptr_t)p_ & 15u) == 0; };
  if (!al16(a->q8) || !al16(a->k8) || !al16(a->v8) || !al16(a->out))
    return fail(MH3_ERR_INVALID, "q8/k8/v8/out must be 16-byte aligned");
  const long long qs[3] = {a->q_stride_s, a->q_stride_h, a->q_stride_b};
  const long long ks[3] = {a->k_stride_s, a->k_stride_h, a->k_stride_b};
  const long long vs[3] = {a->v_stride_s, a->v_stride_h, a->v_stride_b};
  const long long vmul = a->v_dtype == MH3_DTYPE_F16 ? 8 : 16;
  for (int i = 0; i < 3; ++i) {
    if ((qs[i] % 16) || (ks[i] % 16) || (vs[i] % vmul))
      return fail(MH3_ERR_INVALID, "q8/k8 strides must be multiples of 16 elements, v of 16 bytes");
  }
  if ((a->o_stride_s % 8) || (a->o_stride_h % 8) || (a->o_stride_b % 8))
    return fail(MH3_ERR_INVALID, "output strides must be multiples of 8 elements");
  if (a->key_bias2 != nullptr && (((uintptr_t)a->key_bias2 & 15u) || (a->key_bias2_stride_b % 4)))
    return fail(MH3_ERR_INVALID, "key_bias2 must be 16-byte aligned with a row stride multiple of 4");

  attn::Params p;
  memset(&p, 0, sizeof(p));
  const int B = a->batch, H = a->heads;
  const long long Sq_dim = varlen ? a->total_q : a->seqlen_q;
  const long long Sk_dim = varlen ? a->total_k : a->seqlen_k;
  if (varlen && (Sq_dim <= 0 || Sk_dim <= 0)) return fail(MH3_ERR_INVALID, "varlen needs total_q/total_k > 0");
  const int Bdim = varlen ? 1 : B;
  const bool pv16 = a->v_dtype == MH3_DTYPE_F16;
  int rc = attn::make_map(&p.tmq, a->q8, D, Sq_dim, H, Bdim, a->q_stride_s, a->q_stride_h,
                          varlen ? Sq_dim * a->q_stride_s : a->q_stride_b, false);
  if (rc) return rc;
  rc = attn::make_map(&p.tmk, a->k8, D, Sk_dim, H, Bdim, a->k_stride_s, a->k_stride_h,
                      varlen ? Sk_dim * a->k_stride_s : a->k_stride_b, false);
  if (rc) return rc;
  rc = attn::make_map(&p.tmv, a->v8, D, Sk_dim, H, Bdim, a->v_stride_s, a->v_stride_h,
                      varlen ? Sk_dim * a->v_stride_s : a->v_stride_b, pv16);
  if (rc) return rc;
  p.out = a->out;
  p.osb = a->o_stride_b;
  p.osh = a->o_stride_h;
  p.oss = a->o_stride_s;
  p.sq = a->scale_q;
  p.sqb = a->sq_stride_b;
  p.sqh = a->sq_stride_h;
  p.sqblk = a->sq_stride_blk;
  p.sk = a->scale_k;
  p.skb = a->sk_stride_b;
  p.skh = a->sk_stride_h;
  p.skblk = a->sk_stride_blk;
  p.sv = a->scale_v;
  p.svb = a->sv_stride_b;
  p.svh = a->sv_stride_h;
  p.svd = a->sv_stride_d;
  p.logit_scale_log2 = a->logit_scale_log2;
  p.H = H;
  p.Sq = a->seqlen_q;
  p.Sk = a->seqlen_k;
  p.cuq = a->cu_seqlens_q;
  p.cuk = a->cu_seqlens_k;
  p.kbias2 = a->key_bias2;
  p.kbias_sb = a->key_bias2_stride_b;
  p.err = a->err ? a->err : device_error_word();
  p.timeout_ns = a->timeout_ns ? a->timeout_ns : 4000000000ull;
  p.kv_len = a->kv_len;
  p.test_flags = a->test_flags;

  const int max_q = varlen ? a->max_seqlen_q : a->seqlen_q;
  const int q_tiles = (max_q + attn::BM - 1) / attn::BM;
  const dim3 grid((unsigned)((q_tiles + 1) / 2), (unsigned)H, (unsigned)B);
  if (grid.y > 65535u || grid.z > 65535u) return fail(MH3_ERR_INVALID, "too many heads or batches");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool f16 = a->out_dtype == MH3_DTYPE_F16;
  const bool bias = a->key_bias2 != nullptr;
  cudaError_t e;
  if (D == 128)
    e = pv16 ? attn::dispatch<128, true>(p, grid, st, f16, bias) : attn::dispatch<128, false>(p, grid, st, f16, bias);
  else
    e = pv16 ? attn::dispatch<64, true>(p, grid, st, f16, bias) : attn::dispatch<64, false>(p, grid, st, f16, bias);
  if (e != cudaSuccess) return fail_cuda(e, "mh3_fp8_attention_fwd launch");
  return MH3_OK;
}
