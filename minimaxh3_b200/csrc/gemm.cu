// Scaled GEMM with a fused epilogue for sm_100a (tcgen05 + TMA).
//
// Replaces ``torch._scaled_mm(x8, w8.t(), scale_a, scale_b, bias, bf16)`` and
// the LoRA adapter loop that follows it in the reference's
// ``FP8Linear.forward`` (kernels/fp8_linear.py:95-108, :45-55):
//
//   out[m,n] = bf16( (sum_k a[m,k] b[n,k] + sum_r a2[m,r] b2[n,r])
//                    * rs[m] * cs[n] + bias[n] )
//
// a, b are e4m3 (kind::f8f6f4) or bf16 (kind::f16), K-major.  The optional
// low-rank term (a2 [M,R], b2 [N,R], bf16) is accumulated into the same TMEM
// accumulator after the main K loop; FP8Linear passes a2 = (x A^T)/sa and
// b2 = scale*B/sb so that the scaled epilogue yields main + LoRA delta.  rs
// may be replaced by 1/rs (``row_scale_inv``) - the form the LoRA-down
// product x A^T / sa uses.
//
// Persistent kernel, one CTA per SM, 192 threads:
//   warp 0      TMA producer (4-stage ring of 48 KB stages)
//   warp 1      MMA issuer; owns 512 TMEM columns = two 256-column accumulators
//   warps 2-5   epilogue (thread i of the warpgroup owns accumulator row i)
// The epilogue of one tile overlaps the main loop of the next.  Tiles are
// visited in groups of kGroupM M-blocks per N-column so the working set of
// A and B rows stays in L2.  Every mbarrier wait is bounded.
#include <cstdlib>
#include <mutex>

#include "mh3_b200.h"
#include "mh3_internal.h"
#include "ptx.cuh"

namespace mh3 {
namespace gemm {

constexpr int BM = 128;
constexpr int STAGES = 4;
constexpr int STAGE_K_BYTES = 128;  // bytes of K per stage: 128 e4m3 or 64 bf16
constexpr int kGroupM = 16;
constexpr int NUM_THREADS = 192;

struct Params {
  CUtensorMap tma_a;   // (K, M), box (128 B, 128)
  CUtensorMap tma_b;   // (K, N), box (128 B, BN)
  CUtensorMap tma_a2;  // bf16 (R, M), box (64, 128)
  CUtensorMap tma_b2;  // bf16 (R, N), box (64, BN)
  CUtensorMap tma_out; // bf16 (N, M), box (32, 32), 64B swizzle (CTA-pair kernel)
  int M, N, K, R;
  int bf16_ab;  // main operands are bf16 (else e4m3)
  const float* rs;
  int rs_inv;
  const float* cs;
  const __nv_bfloat16* bias;
  __nv_bfloat16* out;
  long long ldo;
  int* err;
  unsigned long long timeout_ns;
  int test_flags;  // MH3_TEST_* bits (tests of the bounded waits); 0 in normal use
};

template <int BN>
struct __align__(1024) Smem {
  uint8_t a[STAGES][BM * STAGE_K_BYTES];
  uint8_t b[STAGES][BN * STAGE_K_BYTES];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t mma_done;
  uint64_t bar_never;  // nothing arrives on it (test hook)
  uint32_t tmem_base;
  int abort_flag;
};

// TMEM per CTA: two accumulators of BN columns (rounded to the 32-column
// allocation granule; a power of two).  The narrow tile takes 128 columns, so
// two CTAs share an SM - the narrow GEMMs (the LoRA-down x A^T, N = rank) are
// memory-bound and the second CTA hides load latency and the tail wave.
template <int BN>
constexpr uint32_t kAccCols = BN <= 64 ? 64u : 256u;
template <int BN>
constexpr uint32_t kTmemCols = 2u * kAccCols<BN>;

template <int BN>
__global__ void __launch_bounds__(NUM_THREADS, BN == 64 ? 2 : 1) gemm_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem<BN>& sm = *reinterpret_cast<Smem<BN>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (p.M + BM - 1) / BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int kst_main = (p.K * (p.bf16_ab ? 2 : 1) + STAGE_K_BYTES - 1) / STAGE_K_BYTES;
  const int kst_lora = (p.R * 2 + STAGE_K_BYTES - 1) / STAGE_K_BYTES;
  const int kst = kst_main + kst_lora;

  // tile index -> (m-block, n-block): groups of kGroupM m-blocks sweep all n.
  auto coords = [&](int t, int& mb, int& nb) {
    const int per_group = kGroupM * num_n;
    const int g = t / per_group;
    const int r = t - g * per_group;
    const int gm = min(kGroupM, num_m - g * kGroupM);
    nb = r / gm;
    mb = g * kGroupM + (r - nb * gm);
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(smem_u32(&sm.full[i]), 1);
      mbar_init(smem_u32(&sm.empty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&sm.acc_full[i]), 1);
      mbar_init(smem_u32(&sm.acc_empty[i]), 4);
    }
    mbar_init(smem_u32(&sm.mma_done), 1);
    mbar_init(smem_u32(&sm.bar_never), 1);
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&sm.tmem_base), kTmemCols<BN>);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const WaitGuard g{&sm.abort_flag, p.err, p.timeout_ns};
  constexpr uint32_t kStageBytes = (BM + BN) * STAGE_K_BYTES;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- producer
      tma_prefetch_desc(&p.tma_a);
      tma_prefetch_desc(&p.tma_b);
      if (p.R > 0) {
        tma_prefetch_desc(&p.tma_a2);
        tma_prefetch_desc(&p.tma_b2);
      }
      int it = 0;
      int last_issued = -1;
      // Test hook (MH3_TEST_STALL_PRODUCER): a wait nothing ends runs out first.
      bool ok = (p.test_flags & MH3_TEST_STALL_PRODUCER) == 0 || mbar_wait(smem_u32(&sm.bar_never), 0, g);
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mb, nb;
        coords(t, mb, nb);
        for (int s = 0; s < kst; ++s, ++it) {
          const int st = it % STAGES;
          if (!mbar_wait(smem_u32(&sm.empty[st]), ((uint32_t)(it / STAGES) & 1u) ^ 1u, g)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&sm.full[st]);
          mbar_arrive_expect_tx(fb, kStageBytes);
          if (s < kst_main) {
            const int kc = s * (p.bf16_ab ? STAGE_K_BYTES / 2 : STAGE_K_BYTES);
            tma_load_2d(smem_u32(sm.a[st]), &p.tma_a, fb, kc, mb * BM);
            tma_load_2d(smem_u32(sm.b[st]), &p.tma_b, fb, kc, nb * BN);
          } else {
            const int rc = (s - kst_main) * (STAGE_K_BYTES / 2);
            tma_load_2d(smem_u32(sm.a[st]), &p.tma_a2, fb, rc, mb * BM);
            tma_load_2d(smem_u32(sm.b[st]), &p.tma_b2, fb, rc, nb * BN);
          }
          last_issued = it;
        }
      }
      // Teardown: the last copy issued into each stage must land.
      for (int i = max(0, last_issued - STAGES + 1); i <= last_issued; ++i)
        mbar_wait_teardown(smem_u32(&sm.full[i % STAGES]), (uint32_t)(i / STAGES) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      constexpr uint32_t kIdF8 = idesc_e4m3(BM, BN, false, false);
      constexpr uint32_t kIdBF = idesc_bf16(BM, BN, false, false);
      int it = 0, tcount = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tcount) {
        const int acc = tcount & 1;
        const uint32_t d_tmem = tmem + (uint32_t)(acc * kAccCols<BN>);
        mbar_wait(smem_u32(&sm.acc_empty[acc]), ((uint32_t)(tcount >> 1) & 1u) ^ 1u, g);
        tc_fence_after();
        for (int s = 0; s < kst; ++s, ++it) {
          const int st = it % STAGES;
          mbar_wait(smem_u32(&sm.full[st]), (uint32_t)(it / STAGES) & 1u, g);
          tc_fence_after();
          const uint32_t ab = smem_u32(sm.a[st]);
          const uint32_t bb = smem_u32(sm.b[st]);
          const bool f16kind = (s >= kst_main) || p.bf16_ab;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {  // 32 bytes of K per MMA
            const uint64_t ad = smem_desc(ab + kk * 32, 16, 1024, kLayoutSW128);
            const uint64_t bd = smem_desc(bb + kk * 32, 16, 1024, kLayoutSW128);
            const uint32_t accum = (s > 0 || kk > 0) ? 1u : 0u;
            if (f16kind)
              mma_f16_ss(d_tmem, ad, bd, kIdBF, accum);
            else
              mma_f8_ss(d_tmem, ad, bd, kIdF8, accum);
          }
          mma_commit(smem_u32(&sm.empty[st]));
        }
        mma_commit(smem_u32(&sm.acc_full[acc]));
      }
      // Every MMA must be finished before the CTA frees TMEM (also on the
      // abort path, where the epilogue's waits return early).
      mma_commit(smem_u32(&sm.mma_done));
      mbar_wait_teardown(smem_u32(&sm.mma_done), 0);
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    int tcount = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tcount) {
      int mb, nb;
      coords(t, mb, nb);
      const int acc = tcount & 1;
      mbar_wait(smem_u32(&sm.acc_full[acc]), (uint32_t)(tcount >> 1) & 1u, g);
      tc_fence_after();
      const int m = mb * BM + row;
      const bool row_ok = m < p.M;
      float rsv = 1.0f;
      if (p.rs != nullptr && row_ok) rsv = p.rs_inv ? 1.0f / __ldg(p.rs + m) : __ldg(p.rs + m);
      __nv_bfloat16* orow = p.out + (long long)(row_ok ? m : 0) * p.ldo;
      const int n0 = nb * BN;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + (uint32_t)(acc * kAccCols<BN> + c * 32) + lane_off, v);
        tmem_wait_ld();
        const int nc = n0 + c * 32;
        if (nc >= p.N) continue;
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int n = nc + 2 * i;
          float x0 = __uint_as_float(v[2 * i]) * rsv;
          float x1 = __uint_as_float(v[2 * i + 1]) * rsv;
          if (p.cs != nullptr) {
            x0 *= (n < p.N) ? __ldg(p.cs + n) : 0.0f;
            x1 *= (n + 1 < p.N) ? __ldg(p.cs + n + 1) : 0.0f;
          }
          if (p.bias != nullptr) {
            x0 += (n < p.N) ? __bfloat162float(p.bias[n]) : 0.0f;
            x1 += (n + 1 < p.N) ? __bfloat162float(p.bias[n + 1]) : 0.0f;
          }
          __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
          packed[i] = *reinterpret_cast<uint32_t*>(&h);
        }
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            if (nc + 8 * i < p.N)  // N is a multiple of 8
              *reinterpret_cast<uint4*>(orow + nc + 8 * i) =
                  make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&sm.acc_empty[acc]));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols<BN>);
  }
}

template <int BN>
constexpr uint32_t smem_bytes() {
  return (uint32_t)sizeof(Smem<BN>) + 1024;
}

// ---------------------------------------------------------------------------
// CTA-pair variant: a cluster of 2 CTAs computes a 256x256 tile with
// tcgen05.mma.cta_group::2 (M = 256 over both CTAs' TMEM lanes).  CTA c of
// the pair loads rows [c*128, c*128+128) of the tile's A rows and of its B
// rows into its own shared memory; the leader (c = 0) counts both CTAs'
// copies on its ``full`` barrier and issues every MMA; its commits arrive on
// both CTAs' ``empty`` / ``acc_full`` barriers; each CTA's epilogue drains
// its own 128 accumulator rows and arrives on the leader's ``acc_empty``.
// Per SM this halves the B bytes of a tile and doubles the work of each MMA
// instruction against the single-CTA 128x256 tile.  No TMA multicast.
//
// Epilogue: per 32-column chunk each warp scales its 32 rows (row scale in a
// register, column scale and bias staged in shared memory once per tile),
// packs bf16 into a 64B-swizzled 32x32 shared-memory box (conflict-free) and
// TMA-stores the box, double-buffered per warp; the TMA clips the M and N
// edges.  Row-per-thread global stores were the kernel's bottleneck.
// ---------------------------------------------------------------------------
// 3 stages of 256 bytes of K (8 MMAs per stage) measured faster than 6
// stages of 128 bytes: fp8 +3 %, bf16 +3-20 % (half the barrier round trips
// per MMA).
#ifndef MH3_PAIR_CHUNKS
#define MH3_PAIR_CHUNKS 2
#endif
#ifndef MH3_PAIR_STAGES
#define MH3_PAIR_STAGES 3
#endif
constexpr int PAIR_CHUNKS = MH3_PAIR_CHUNKS;  // 128-byte K chunks per stage
constexpr int PAIR_STAGES = MH3_PAIR_STAGES;
constexpr int PAIR_BM = 256;       // tile rows (both CTAs)
constexpr int PAIR_BN = 256;       // tile columns
constexpr int PAIR_HALF = 128;     // rows of A and of B per CTA
#ifndef MH3_PAIR_GROUP_M
#define MH3_PAIR_GROUP_M 8
#endif
constexpr int kPairGroupM = MH3_PAIR_GROUP_M;  // 256-row blocks per raster group
constexpr int PAIR_STAGE_BYTES = PAIR_HALF * STAGE_K_BYTES;  // one [128 rows x 128 B] SW128 block
constexpr int EPI_BOX = 32 * 32 * 2;                         // 32 rows x 32 bf16 columns

struct __align__(1024) SmemPair {
  uint8_t a[PAIR_STAGES][PAIR_CHUNKS][PAIR_STAGE_BYTES];
  uint8_t b[PAIR_STAGES][PAIR_CHUNKS][PAIR_STAGE_BYTES];
  uint8_t epi[4][2][EPI_BOX];  // per epilogue warp, double-buffered output boxes
  float col_scale[2][PAIR_BN]; // per accumulator buffer
  float col_bias[2][PAIR_BN];
  uint64_t full[PAIR_STAGES];  // used in the leader
  uint64_t empty[PAIR_STAGES];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];       // used in the leader: 4 warps x 2 CTAs
  uint64_t mma_done;
  uint64_t bar_never;  // nothing arrives on it (test hook)
  uint32_t tmem_base;
  int abort_flag;
};

__global__ void __launch_bounds__(NUM_THREADS, 1) gemm_pair_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  SmemPair& sm = *reinterpret_cast<SmemPair*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const int num_m = (p.M + PAIR_BM - 1) / PAIR_BM;
  const int num_n = (p.N + PAIR_BN - 1) / PAIR_BN;
  const int num_tiles = num_m * num_n;
  // K is walked in 128-byte stages (128 e4m3 / 64 bf16 elements): the main
  // stages first, then the low-rank (bf16) stages.
  const int ch_main = (p.K * (p.bf16_ab ? 2 : 1) + STAGE_K_BYTES - 1) / STAGE_K_BYTES;
  const int ch_lora = (p.R * 2 + STAGE_K_BYTES - 1) / STAGE_K_BYTES;
  const int kst_main = (ch_main + PAIR_CHUNKS - 1) / PAIR_CHUNKS;
  const int kst_lora = (ch_lora + PAIR_CHUNKS - 1) / PAIR_CHUNKS;
  const int kst = kst_main + kst_lora;
  // 128-byte chunks of stage s that hold data (the last main / low-rank stage may be short)
  auto stage_chunks = [&](int s) {
    return s < kst_main ? min(PAIR_CHUNKS, ch_main - s * PAIR_CHUNKS)
                        : min(PAIR_CHUNKS, ch_lora - (s - kst_main) * PAIR_CHUNKS);
  };

  auto coords = [&](int t, int& mb, int& nb) {
    const int per_group = kPairGroupM * num_n;
    const int g = t / per_group;
    const int r = t - g * per_group;
    const int gm = min(kPairGroupM, num_m - g * kPairGroupM);
    nb = r / gm;
    mb = g * kPairGroupM + (r - nb * gm);
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < PAIR_STAGES; ++i) {
      mbar_init(smem_u32(&sm.full[i]), 1);
      mbar_init(smem_u32(&sm.empty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&sm.acc_full[i]), 1);
      mbar_init(smem_u32(&sm.acc_empty[i]), 8);
    }
    mbar_init(smem_u32(&sm.mma_done), 1);
    mbar_init(smem_u32(&sm.bar_never), 1);
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(&sm.tmem_base), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers are initialised before any copy or arrive crosses
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const WaitGuard g{&sm.abort_flag, p.err, p.timeout_ns};

  // Warps 0 and 1 run their loops on the whole warp (warp-uniform state); one
  // elected lane issues each TMA, MMA and commit.
  if (warp == 0) {
    // ---------------------------------------------------------------- producer (both CTAs)
    if (elect_one_sync()) {
      tma_prefetch_desc(&p.tma_a);
      tma_prefetch_desc(&p.tma_b);
      if (p.R > 0) {
        tma_prefetch_desc(&p.tma_a2);
        tma_prefetch_desc(&p.tma_b2);
      }
    }
    __syncwarp();
    int it = 0;
    int last_issued = -1;
    // Test hook (MH3_TEST_STALL_PRODUCER): a wait nothing ends runs out first
    // (one lane waits, the warp takes its answer).
    bool ok = true;
    if (p.test_flags & MH3_TEST_STALL_PRODUCER) {
      bool w = true;
      if (lane == 0) w = mbar_wait(smem_u32(&sm.bar_never), 0, g);
      ok = __shfl_sync(0xffffffffu, w ? 1 : 0, 0) != 0;
    }
    for (int t = pair; t < num_tiles && ok; t += npairs) {
      int mb, nb;
      coords(t, mb, nb);
      const int row_a = mb * PAIR_BM + (int)crank * PAIR_HALF;
      const int row_b = nb * PAIR_BN + (int)crank * PAIR_HALF;
      for (int s = 0; s < kst; ++s, ++it) {
        const int st = it % PAIR_STAGES;
        // one lane waits and the warp takes its answer, so the warp stays converged
        bool w = true;
        if (lane == 0) w = mbar_wait(smem_u32(&sm.empty[st]), ((uint32_t)(it / PAIR_STAGES) & 1u) ^ 1u, g);
        if (!__shfl_sync(0xffffffffu, w ? 1 : 0, 0)) {
          ok = false;
          break;
        }
        last_issued = it;
        if (elect_one_sync()) {
          const int nch = stage_chunks(s);
          // the leader counts both CTAs' copies: 2 CTAs x (A + B) x nch chunks
          if (crank == 0) mbar_arrive_expect_tx(smem_u32(&sm.full[st]), (uint32_t)(4 * nch * PAIR_STAGE_BYTES));
          const uint32_t fb = mapa_shared(smem_u32(&sm.full[st]), 0);
          for (int c = 0; c < nch; ++c) {
            if (s < kst_main) {
              const int kc = (s * PAIR_CHUNKS + c) * (p.bf16_ab ? STAGE_K_BYTES / 2 : STAGE_K_BYTES);
              tma_load_2d_pair(smem_u32(sm.a[st][c]), &p.tma_a, fb, kc, row_a);
              tma_load_2d_pair(smem_u32(sm.b[st][c]), &p.tma_b, fb, kc, row_b);
            } else {
              const int rc = ((s - kst_main) * PAIR_CHUNKS + c) * (STAGE_K_BYTES / 2);
              tma_load_2d_pair(smem_u32(sm.a[st][c]), &p.tma_a2, fb, rc, row_a);
              tma_load_2d_pair(smem_u32(sm.b[st][c]), &p.tma_b2, fb, rc, row_b);
            }
          }
        }
        __syncwarp();
      }
    }
    // Teardown (leader): the last copies counted on each stage must land.
    if (crank == 0 && lane == 0)
      for (int i = max(0, last_issued - PAIR_STAGES + 1); i <= last_issued; ++i)
        mbar_wait_teardown(smem_u32(&sm.full[i % PAIR_STAGES]), (uint32_t)(i / PAIR_STAGES) & 1u);
  } else if (warp == 1) {
    if (crank == 0) {
      // -------------------------------------------------------------- MMA issuer (leader)
      constexpr uint32_t kIdF8 = idesc_e4m3(PAIR_BM, PAIR_BN, false, false);
      constexpr uint32_t kIdBF = idesc_bf16(PAIR_BM, PAIR_BN, false, false);
      int it = 0, tcount = 0;
      for (int t = pair; t < num_tiles; t += npairs, ++tcount) {
        const int acc = tcount & 1;
        const uint32_t d_tmem = tmem + (uint32_t)(acc * 256);
        mbar_wait_cluster(smem_u32(&sm.acc_empty[acc]), ((uint32_t)(tcount >> 1) & 1u) ^ 1u, g);
        tc_fence_after();
        for (int s = 0; s < kst; ++s, ++it) {
          const int st = it % PAIR_STAGES;
          mbar_wait(smem_u32(&sm.full[st]), (uint32_t)(it / PAIR_STAGES) & 1u, g);
          tc_fence_after();
          const bool f16kind = (s >= kst_main) || p.bf16_ab;
          const int nmma = 4 * stage_chunks(s);  // 32 bytes of K per MMA
          __syncwarp();
          if (elect_one_sync()) {
            for (int kk = 0; kk < nmma; ++kk) {
              const uint64_t ad = smem_desc(smem_u32(sm.a[st][kk >> 2]) + (kk & 3) * 32, 16, 1024, kLayoutSW128);
              const uint64_t bd = smem_desc(smem_u32(sm.b[st][kk >> 2]) + (kk & 3) * 32, 16, 1024, kLayoutSW128);
              const uint32_t accum = (s > 0 || kk > 0) ? 1u : 0u;
              if (f16kind)
                mma_f16_ss_pair(d_tmem, ad, bd, kIdBF, accum);
              else
                mma_f8_ss_pair(d_tmem, ad, bd, kIdF8, accum);
            }
            mma_commit_pair(smem_u32(&sm.empty[st]), 0x3);
          }
          __syncwarp();
        }
        if (elect_one_sync()) mma_commit_pair(smem_u32(&sm.acc_full[acc]), 0x3);
        __syncwarp();
      }
      if (elect_one_sync()) mma_commit_pair(smem_u32(&sm.mma_done), 0x3);
      __syncwarp();
    }
    // Both CTAs: every pair MMA (they write both CTAs' TMEM) must be
    // finished before TMEM is freed, also on the abort path.
    if (lane == 0) mbar_wait_teardown(smem_u32(&sm.mma_done), 0);
  } else {
    // ------------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;                    // TMEM lane quarter of this warp
    const int et = threadIdx.x - 64;           // 0..127 over the 4 epilogue warps
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    int tcount = 0, buf = 0;
    for (int t = pair; t < num_tiles; t += npairs, ++tcount) {
      int mb, nb;
      coords(t, mb, nb);
      const int acc = tcount & 1;
      const int n0 = nb * PAIR_BN;
      // this tile's column scale and bias (one buffer per accumulator: the
      // other may still be read by a slower warp for the previous tile)
      for (int j = et; j < PAIR_BN; j += 128) {
        const int n = n0 + j;
        const bool in = n < p.N;
        sm.col_scale[acc][j] = p.cs == nullptr ? 1.0f : (in ? __ldg(p.cs + n) : 0.0f);
        sm.col_bias[acc][j] = (p.bias != nullptr && in) ? __bfloat162float(p.bias[n]) : 0.0f;
      }
      named_barrier_sync(1, 128);
      mbar_wait(smem_u32(&sm.acc_full[acc]), (uint32_t)(tcount >> 1) & 1u, g);
      tc_fence_after();
      const int m0 = mb * PAIR_BM + (int)crank * PAIR_HALF + q * 32;  // first row of this warp's box
      const int m = m0 + lane;
      float rsv = 1.0f;
      if (p.rs != nullptr && m < p.M) rsv = p.rs_inv ? 1.0f / __ldg(p.rs + m) : __ldg(p.rs + m);
#pragma unroll 1
      for (int c = 0; c < PAIR_BN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + (uint32_t)(acc * 256 + c * 32) + lane_off, v);
        tmem_wait_ld();
        if (n0 + c * 32 >= p.N || m0 >= p.M) continue;  // warp-uniform: box wholly outside
        const float* cs = &sm.col_scale[acc][c * 32];
        const float* bs = &sm.col_bias[acc][c * 32];
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 8; ++i) {  // 4 columns per step (broadcast LDS.128)
          const float4 c4 = *reinterpret_cast<const float4*>(cs + 4 * i);
          const float4 b4 = *reinterpret_cast<const float4*>(bs + 4 * i);
          const float x0 = fmaf(__uint_as_float(v[4 * i + 0]) * rsv, c4.x, b4.x);
          const float x1 = fmaf(__uint_as_float(v[4 * i + 1]) * rsv, c4.y, b4.y);
          const float x2 = fmaf(__uint_as_float(v[4 * i + 2]) * rsv, c4.z, b4.z);
          const float x3 = fmaf(__uint_as_float(v[4 * i + 3]) * rsv, c4.w, b4.w);
          __nv_bfloat162 h0 = __floats2bfloat162_rn(x0, x1);
          __nv_bfloat162 h1 = __floats2bfloat162_rn(x2, x3);
          packed[2 * i] = *reinterpret_cast<uint32_t*>(&h0);
          packed[2 * i + 1] = *reinterpret_cast<uint32_t*>(&h1);
        }
        // the TMA store that last read this box (two chunks ago) must be done
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
        uint8_t* box = sm.epi[q][buf];
        // row ``lane`` at lane*64; 16-byte chunk j at (j ^ ((lane >> 1) & 3)) * 16 (64B swizzle)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          *reinterpret_cast<uint4*>(box + lane * 64 + ((j ^ ((lane >> 1) & 3)) * 16)) =
              make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&p.tma_out, smem_u32(box), n0 + c * 32, m0);
          bulk_commit_group();
        }
        buf ^= 1;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&sm.acc_empty[acc]), 0));
    }
    if (lane == 0) bulk_wait_group<0>();  // stores complete before the CTA's shared memory goes
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still arrive on or copy into it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

constexpr uint32_t smem_bytes_pair() { return (uint32_t)sizeof(SmemPair) + 1024; }

static cudaError_t launch_pair(const Params& p, cudaStream_t st) {
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [&] {
    attr = cudaFuncSetAttribute(gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)smem_bytes_pair());
  });
  if (attr != cudaSuccess) return attr;
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const long long tiles = (long long)((p.M + PAIR_BM - 1) / PAIR_BM) * ((p.N + PAIR_BN - 1) / PAIR_BN);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(nsm & ~1), 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes_pair();
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  // Persistent: no more pairs than can be resident at once (a pair needs two
  // SMs of one GPC, so this can be below nsm/2).
  static int max_pairs = 0;
  static std::once_flag once_occ;
  std::call_once(once_occ, [&] {
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel, &cfg) != cudaSuccess || n <= 0) n = nsm / 2;
    max_pairs = n;
  });
  const long long pairs = tiles < max_pairs ? tiles : max_pairs;
  cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
  return cudaLaunchKernelEx(&cfg, gemm_pair_kernel, p);
}


// 2-D K-major map: dims (K, rows), box (box_k elements, box_rows), swizzle 128B.
static int make_map_2d(CUtensorMap* map, const void* base, bool bf16, long long K, long long rows,
                       long long ld_elems, int box_rows) {
  const long long es = bf16 ? 2 : 1;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(ld_elems * es)};
  const cuuint32_t box[2] = {(cuuint32_t)(STAGE_K_BYTES / es), (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1u, 1u};
  return encode_tiled(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                      const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int BN>
static cudaError_t launch(const Params& p, cudaStream_t st) {
  auto kern = gemm_kernel<BN>;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [&] {
    attr = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes<BN>());
  });
  if (attr != cudaSuccess) return attr;
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const long long tiles = (long long)((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN);
  const long long slots = (long long)nsm * (BN == 64 ? 2 : 1);  // resident CTAs
  const int grid = (int)(tiles < slots ? tiles : slots);
  kern<<<grid, NUM_THREADS, smem_bytes<BN>(), st>>>(p);
  return cudaGetLastError();
}

}  // namespace gemm
}  // namespace mh3

using namespace mh3;

extern "C" int mh3_scaled_gemm(const mh3_gemm_args* a, void* stream) {
  const mh3::NvtxRange nvtx_range("mh3_scaled_gemm");
  if (a == nullptr) return fail(MH3_ERR_INVALID, "mh3_scaled_gemm: null args");
  if (a->M < 0 || a->N <= 0 || a->K <= 0) return fail(MH3_ERR_INVALID, "sizes must be positive");
  if (a->M == 0) return MH3_OK;
  if (a->M > 0x7fffffffLL || a->N > 0x7fffffffLL || a->K > 0x7fffffffLL || a->R > 0x7fffffffLL)
    return fail(MH3_ERR_TOO_LARGE, "dimension too large");
  if (a->ab_dtype != MH3_DTYPE_E4M3 && a->ab_dtype != MH3_DTYPE_BF16)
    return fail(MH3_ERR_INVALID, "ab_dtype must be e4m3 or bf16");
  const bool bf16 = a->ab_dtype == MH3_DTYPE_BF16;
  const long long es = bf16 ? 2 : 1;
  if (!a->a || !a->b || !a->out) return fail(MH3_ERR_INVALID, "null a/b/out");
  if ((a->K * es) % 16 || (a->lda * es) % 16 || (a->ldb * es) % 16)
    return fail(MH3_ERR_INVALID, "K and the row strides of a and b must be multiples of 16 bytes");
  if (a->N % 8 || a->ldo % 8) return fail(MH3_ERR_INVALID, "N and ldo must be multiples of 8");
  auto al16 = [](const void* p_) { return ((uintptr_t)p_ & 15u) == 0; };
  if (!al16(a->a) || !al16(a->b) || !al16(a->out)) return fail(MH3_ERR_INVALID, "a/b/out must be 16-byte aligned");
  if (a->R < 0) return fail(MH3_ERR_INVALID, "R must be >= 0");
  if (a->R > 0) {
    if (!a->a2 || !a->b2) return fail(MH3_ERR_INVALID, "R > 0 needs a2 and b2");
    if (a->R % 8 || a->lda2 % 8 || a->ldb2 % 8 || !al16(a->a2) || !al16(a->b2))
      return fail(MH3_ERR_INVALID, "R and the strides of a2/b2 must be multiples of 8 (16 bytes), 16-byte aligned");
  }
  gemm::Params p;
  memset(&p, 0, sizeof(p));
  const int BN = a->N <= 64 ? 64 : 256;
  // 256x256 tiles on CTA pairs unless the problem is a single 128-row block
  // (or MH3_GEMM_CTA_PAIR=0 asks for the single-CTA 128x256 kernel).
  const char* env = getenv("MH3_GEMM_CTA_PAIR");
  const bool use_pair = BN == 256 && a->M > gemm::BM && !(env != nullptr && env[0] == '0');
  const int b_rows = use_pair ? gemm::PAIR_HALF : BN;  // B rows per CTA copy
  int rc = gemm::make_map_2d(&p.tma_a, a->a, bf16, a->K, a->M, a->lda, gemm::BM);
  if (rc) return rc;
  rc = gemm::make_map_2d(&p.tma_b, a->b, bf16, a->K, a->N, a->ldb, b_rows);
  if (rc) return rc;
  if (a->R > 0) {
    rc = gemm::make_map_2d(&p.tma_a2, a->a2, true, a->R, a->M, a->lda2, gemm::BM);
    if (rc) return rc;
    rc = gemm::make_map_2d(&p.tma_b2, a->b2, true, a->R, a->N, a->ldb2, b_rows);
    if (rc) return rc;
  }
  if (use_pair) {
    const cuuint64_t dims[2] = {(cuuint64_t)a->N, (cuuint64_t)a->M};
    const cuuint64_t strides[1] = {(cuuint64_t)(a->ldo * 2)};
    const cuuint32_t box[2] = {32u, 32u};
    const cuuint32_t estr[2] = {1u, 1u};
    rc = encode_tiled(&p.tma_out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a->out, dims, strides, box, estr,
                      CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc) return rc;
  }
  p.M = (int)a->M;
  p.N = (int)a->N;
  p.K = (int)a->K;
  p.R = (int)a->R;
  p.bf16_ab = bf16 ? 1 : 0;
  p.rs = a->row_scale;
  p.rs_inv = a->row_scale_inv;
  p.cs = a->col_scale;
  p.bias = static_cast<const __nv_bfloat16*>(a->bias);
  p.out = static_cast<__nv_bfloat16*>(a->out);
  p.ldo = a->ldo;
  p.err = a->err ? a->err : device_error_word();
  p.timeout_ns = a->timeout_ns ? a->timeout_ns : 4000000000ull;
  p.test_flags = a->test_flags;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const cudaError_t e = use_pair ? gemm::launch_pair(p, st) : BN == 64 ? gemm::launch<64>(p, st) : gemm::launch<256>(p, st);
  if (e != cudaSuccess) return fail_cuda(e, "mh3_scaled_gemm launch");
  return MH3_OK;
}
