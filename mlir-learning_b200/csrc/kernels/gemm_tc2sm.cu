// gemm_tc2sm.cu -- the tcgen05 BF16 GEMM on CTA pairs: a cluster of two CTAs
// (two SMs) computes one 256 x 256 output tile with tcgen05.mma.cta_group::2
// (M = 256, N = 256, K = 16 per instruction).
//
// Replaces the reference's linalg.matmul launches (QKV, attention out-proj,
// MLP fc and proj, the tied lm_head; README.md:11) and the bias / GELU /
// residual generics fused around them (lib/ElementwiseFusion.cpp:43-109) in
// the BF16 and FP8 configurations; same epilogues as gemm_tc.cu.
//
// Why pairs: the single-CTA kernel (128 x 256 tiles) is bound by the
// operand bytes each SM pulls from L2 (a 128-wide tile is 30 % slower than a
// 256-wide one at the same M).  Here CTA r of the pair loads rows
// [r*128, r*128 + 128) of the A tile and of the B tile (B split along N);
// the MMA reads A from each CTA's own shared memory and B from both, so each
// SM loads 32 KB per 128 x 256 x 64 MACs instead of 48 KB.
//
// Roles (320 threads per CTA, one CTA per SM, persistent over the pair's
// tiles):
//   warp 0      TMA producer in both CTAs: its two 16 KB boxes per K step
//               land in its own shared memory and complete on the LEADER's
//               full[s] barrier (cp.async.bulk.tensor ... .cta_group::2);
//               the leader's producer arms that barrier for both CTAs' bytes.
//               No cluster multicast: every load reads this GPU's memory into
//               the issuing CTA.
//   warp 1      TMEM: both CTAs allocate 512 columns together
//               (tcgen05.alloc.cta_group::2); the leader's lane 0 issues the
//               MMAs into two 256-column accumulators (double buffered) and
//               releases each stage / signals each finished tile to both CTAs
//               with one tcgen05.commit aimed at the same barrier in both.
//   warps 2..9  epilogue in both CTAs: each CTA's TMEM holds its 128 rows x
//               256 columns; two warps per TMEM lane quarter, one per
//               128-column half (two epilogue warps per scheduler, so one
//               hides the other's latency); tcgen05.ld, bias / GELU /
//               residual / FP8 scale in registers, 128-byte-swizzled staging,
//               TMA store; every thread arrives on the leader's tempty
//               barrier once it has read its part of the accumulator.
// Every mbarrier wait is bounded (common.cuh); a timeout records
// GPT2_ERR_WAIT_TIMEOUT in the status word, which the other CTA of the pair
// (and every other CTA) sees through its own bounded waits, and both CTAs
// unwind to the closing cluster barrier, which every thread reaches.
#include <atomic>

#include "../common.cuh"
#include "../gemm_epi.cuh"
#include "../kernels.h"

namespace gpt2 {

namespace {
#ifndef GPT2_PAIR_STAGES
#define GPT2_PAIR_STAGES 6
#endif
#ifndef GPT2_PAIR_NBUF
#define GPT2_PAIR_NBUF 1
#endif
#ifndef GPT2_PAIR_STAGES_RESID
#define GPT2_PAIR_STAGES_RESID 5
#endif
#ifndef GPT2_PAIR_NBUF_RESID
#define GPT2_PAIR_NBUF_RESID 2
#endif
#ifndef GPT2_PAIR_GROUP_M_WIDE
#define GPT2_PAIR_GROUP_M_WIDE 16
#endif
constexpr int BM = 256, BN = 256, BK = 64, NTHREADS = 320;
constexpr int HALF_ROWS = 128;                   // rows of A (and of B) one CTA loads per tile
constexpr int A_BYTES = HALF_ROWS * BK * 2;      // 16 KB
constexpr int B_BYTES = HALF_ROWS * BK * 2;      // 16 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;   // per CTA
constexpr int EPI_WARPS = 8;
constexpr uint32_t TMEM_COLS = 512;              // two accumulators of BN columns

// Shared memory split between the operand ring and the epilogue's store
// staging (NBUF buffers of 32 rows x 128 bytes per epilogue warp).  Measured
// on B200 at M = 65536: a 6-deep ring with one staging buffer is fastest for
// the bias / GELU / no-epilogue shapes (QKV, fc, lm_head); the residual
// epilogue, which also loads a tile of the residual, does better with 5
// stages and 2 buffers.
template <int EPI, int OUT_F32>
struct PairCfg {
  static constexpr bool RESID = EpiKind<EPI>::resid;
  static constexpr int STAGES = RESID ? GPT2_PAIR_STAGES_RESID : GPT2_PAIR_STAGES;
  static constexpr int NBUF = RESID ? GPT2_PAIR_NBUF_RESID : GPT2_PAIR_NBUF;
  static constexpr int STAGING_BYTES = EPI_WARPS * NBUF * 4096;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + STAGING_BYTES + 256;
  static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
};

// ---- cluster / cta_group::2 helpers --------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// Address, in the cluster's shared window, of the variable at shared address
// `saddr` of this CTA, in the CTA of the given rank.
__device__ __forceinline__ uint32_t cluster_addr(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// Every thread of both CTAs: release this CTA's earlier writes, wait for the other CTA.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// Tiled load into this CTA's shared memory whose completion (bytes) is
// signalled on a barrier that may live in the other CTA of the pair.
__device__ __forceinline__ void tma_load_2d_pair(void *smem_dst, const CUtensorMap *map, uint32_t cluster_bar, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(cluster_bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_mma_f16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives once on the barrier at this shared offset in BOTH CTAs of the pair
// when every earlier MMA of this thread has completed.
__device__ __forceinline__ void tc_commit_pair_both(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}
__device__ __forceinline__ void tc_commit_pair_self(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Tiles are walked in groups of group_m M-blocks, M fastest, so that a
// group's A rows stay in L2 while every N-block of B passes once.
__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int group_m, int &mb, int &nb) {
  const int per_group = group_m * num_n;
  const int group = t / per_group;
  const int first_m = group * group_m;
  const int gsize = min(num_m - first_m, group_m);
  const int in = t - group * per_group;
  mb = first_m + in % gsize;
  nb = in / gsize;
}

template <int EPI, int OUT_F32>
__global__ void __launch_bounds__(NTHREADS, 1)
    gemm_tc2sm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                      const __grid_constant__ CUtensorMap map_c, int ldc, int M, int N, int K, int group_m,
                      const float *__restrict__ bias, const bf16 *resid, int *status,
                      const float *__restrict__ scale, const LnFold ln) {
  using Cfg = PairCfg<EPI, OUT_F32>;
  using Kind = EpiKind<EPI>;
  constexpr int STAGES = Cfg::STAGES, NBUF = Cfg::NBUF, STAGING_BYTES = Cfg::STAGING_BYTES;
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char *sa = smem;
  unsigned char *sb = smem + STAGES * A_BYTES;
  unsigned char *staging = smem + STAGES * STAGE_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(staging + STAGING_BYTES);
  uint64_t *full = bars, *empty = bars + STAGES, *tfull = bars + 2 * STAGES, *tempty = tfull + 2;
  uint64_t *drain = tempty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = static_cast<int>(cluster_id_x()), npairs = static_cast<int>(cluster_count_x());
  const int num_m = (M + BM - 1) / BM, num_n = (N + BN - 1) / BN, num_k = (K + BK - 1) / BK;
  const int total = num_m * num_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);   // the leader's arrive_expect_tx; both CTAs' bytes
      mbar_init(&empty[s], 1);  // one commit from the leader's MMA thread
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * EPI_WARPS * 32);  // every epilogue thread of both CTAs
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before either signals the other
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    prefetch_tmap(&map_a);
    prefetch_tmap(&map_b);
    const uint32_t full_leader = cluster_addr(smem_u32(full), 0);
    uint32_t issued[STAGES];
#pragma unroll
    for (int s = 0; s < STAGES; ++s) issued[s] = 0;
    int it = 0;
    bool ok = true;
    for (int t = pair; t < total && ok; t += npairs) {
      int mb, nb;
      tile_coords(t, num_m, num_n, group_m, mb, nb);
      for (int kb = 0; kb < num_k; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, status)) { ok = false; break; }
        if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * STAGE_BYTES);
        tma_load_2d_pair(sa + s * A_BYTES, &map_a, full_leader + 8 * s, kb * BK, mb * BM + rank * HALF_ROWS);
        tma_load_2d_pair(sb + s * B_BYTES, &map_b, full_leader + 8 * s, kb * BK, nb * BN + rank * HALF_ROWS);
        ++issued[s];
      }
    }
    if (ok) {
      // Wait for the leader's last releases of every stage, so that no commit
      // is still on its way to this CTA's barriers when the CTA exits.
      for (int i = 0; i < STAGES; ++i, ++it) {
        const int s = it % STAGES;
        if (!mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1, abort_flag, status)) break;
      }
    } else {
      set_status(status, GPT2_ERR_WAIT_TIMEOUT);
      *abort_flag = 1;
      // The leader's full[s] phases count both CTAs' bytes: waiting for the
      // phases the leader armed covers the loads both CTAs issued for them.
      if (rank == 0)
        for (int s = 0; s < STAGES; ++s)
          if (issued[s]) mbar_wait(&full[s], (issued[s] - 1) & 1, nullptr);
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ---------------- MMA issuer (leader CTA only) ----------------
    constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
    int it = 0, local = 0;
    bool ok = true;
    for (int t = pair; t < total && ok; t += npairs, ++local) {
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      if (!mbar_wait(&tempty[acc], aph ^ 1, abort_flag, status)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      for (int kb = 0; kb < num_k; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait(&full[s], ph, abort_flag, status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a0 = smem_u32(sa + s * A_BYTES), b0 = smem_u32(sb + s * B_BYTES);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          tc_mma_f16_pair(d_tmem, sdesc_kmajor_sw128(a0 + k * 32), sdesc_kmajor_sw128(b0 + k * 32), idesc,
                          (kb | k) != 0);
        tc_commit_pair_both(&empty[s]);
      }
      if (!ok) break;
      tc_commit_pair_both(&tfull[acc]);
    }
    if (!ok) {
      set_status(status, GPT2_ERR_WAIT_TIMEOUT);
      *abort_flag = 1;
    }
    // Drain: every MMA this thread issued has completed once this arrives.
    tc_commit_pair_self(drain);
    mbar_wait(drain, 0, nullptr);
  } else if (warp >= 2) {
    // ---------------- epilogue (both CTAs) ----------------
    constexpr int CH = OUT_F32 ? 32 : 64;  // columns per 128-byte chunk
    constexpr int NCH = BN / 2 / CH;          // chunks per warp (its 128-column half)
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int col_half = (warp - 2) >> 2;     // columns [col_half*128, +128) of the tile
    const int row_in_tile = static_cast<int>(rank) * HALF_ROWS + q * 32 + lane;
    const uint32_t tempty_leader = cluster_addr(smem_u32(tempty), 0);
    unsigned char *stage_buf = staging + (warp - 2) * NBUF * 4096;
    uint32_t chunk_count = 0;
    int local = 0;
    for (int t = pair; t < total; t += npairs, ++local) {
      int mb, nb;
      tile_coords(t, num_m, num_n, group_m, mb, nb);
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      const int row = mb * BM + row_in_tile;
      const bool row_ok = row < M;
      const int64_t row_off = (int64_t)row * ldc;
      const int tcol0 = nb * BN + col_half * (BN / 2);  // first column of this warp's half
      float ln_rstd = 0.f, ln_nmr = 0.f;  // folded LayerNorm of A's row, read while the main loop runs
      if (Kind::ln && row_ok) ln_row_stats(ln, row, ln_rstd, ln_nmr);
      float res_rstd = 0.f, res_nmr = 0.f;  // the residual's LayerNorm (EPI_LNRES_*)
      if (Kind::lnres && row_ok) ln_res_row_stats(ln, row, N, res_rstd, res_nmr);
      RowStats rs;
      if (Kind::resid && !OUT_F32 && row_ok) {
        // The residual row goes to L2 while the tile's main loop runs.
        const bf16 *rp = resid + row_off + tcol0;
#pragma unroll
        for (int i = 0; i < BN / 2 / 64; ++i)
          if (tcol0 + i * 64 < N) asm volatile("prefetch.global.L2 [%0];" ::"l"(rp + i * 64));
      }
      if (!mbar_wait(&tfull[acc], aph, abort_flag, status)) {
        set_status(status, GPT2_ERR_WAIT_TIMEOUT);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      uint4 res_cur[8], res_nxt[8];
      auto load_res = [&](uint4 (&dst)[8], int col0) {
        if (Kind::resid && !OUT_F32 && row_ok && col0 + CH <= N) {
          const uint4 *rp = reinterpret_cast<const uint4 *>(resid + row_off + col0);
#pragma unroll
          for (int g = 0; g < 8; ++g) dst[g] = rp[g];
        }
      };
      load_res(res_cur, tcol0);
#pragma unroll 1
      for (int c = 0; c < NCH; ++c) {
        const int col0 = tcol0 + c * CH;
        if (c + 1 < NCH) load_res(res_nxt, col0 + CH);
        uint32_t r[CH];
        const uint32_t taddr =
            tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN + col_half * (BN / 2) + c * CH;
        tmem_ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        if (CH == 64) tmem_ld_32x32b_x32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[CH == 64 ? 32 : 0]));
        tc_wait_ld();
        if (c == NCH - 1) {
          tc_fence_before();
          mbar_arrive_cluster(tempty_leader + 8 * acc);  // the leader may reuse this accumulator
        }
        float *v = reinterpret_cast<float *>(r);
        if (scale) {  // weight-only FP8: per-output-column dequantization scale
          const float s_lo = (col0 + lane < N) ? scale[col0 + lane] : 0.f;
          const float s_hi = (CH == 64 && col0 + 32 + lane < N) ? scale[col0 + 32 + lane] : 0.f;
#pragma unroll
          for (int j = 0; j < CH; ++j)
            r[j] = __float_as_uint(__uint_as_float(r[j]) * __shfl_sync(0xffffffffu, j < 32 ? s_lo : s_hi, j & 31));
        }
        if (Kind::ln) {
          ln_affine<CH, Kind::ln_act>(v, ln, col0, ln_rstd, ln_nmr);
        } else {
          float bias_lo = 0.f, bias_hi = 0.f;
          if (Kind::bias) {
            bias_lo = (col0 + lane < N) ? bias[col0 + lane] : 0.f;
            if (CH == 64) bias_hi = (col0 + 32 + lane < N) ? bias[col0 + 32 + lane] : 0.f;
          }
#pragma unroll
          for (int j = 0; j < CH; ++j) {
            float x = __uint_as_float(r[j]);
            if (Kind::bias) x += __shfl_sync(0xffffffffu, j < 32 ? bias_lo : bias_hi, j & 31);
            if (Kind::gelu_new) x = gelu_new_fast(x);
            if (Kind::gelu_erf) x = gelu_erf_fast(x);
            v[j] = x;
          }
        }
        if (Kind::resid && !OUT_F32 && row_ok) {
          if (col0 + CH <= N) {
#pragma unroll
            for (int g = 0; g < 8; ++g) {
              if (Kind::lnres) {
                float rr[8];
                ln_res_piece(res_cur[g], ln, col0 + 8 * g, res_rstd, res_nmr, rr);
#pragma unroll
                for (int j = 0; j < 8; ++j) v[g * 8 + j] += rr[j];
                continue;
              }
              const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&res_cur[g]);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float2 f = __bfloat1622float2(h[j]);
                v[g * 8 + 2 * j] += f.x;
                v[g * 8 + 2 * j + 1] += f.y;
              }
            }
          } else {
            for (int j = 0; j < CH; ++j)
              if (col0 + j < N) {
                float rj = __bfloat162float(resid[row_off + col0 + j]);
                if (Kind::lnres) rj = fmaf(fmaf(rj, res_rstd, res_nmr), ln.res_gain[col0 + j], ln.res_shift[col0 + j]);
                v[j] += rj;
              }
          }
          if (c + 1 < NCH) {
#pragma unroll
            for (int g = 0; g < 8; ++g) res_cur[g] = res_nxt[g];
          }
        }
        if (Kind::stats && !OUT_F32) {
          // Statistics of the stored bf16 row: this warp's 128 columns are one
          // LN_SEG segment (two chunks); columns past N are 0.
          rs.add_bf16<CH>(v);
          if (c == NCH - 1) rs.flush(ln, row, tcol0 / LN_SEG, row_ok);
        }
        // 16-byte piece g of this row: 4 f32 or 8 bf16 values, written with
        // the 128-byte swizzle (piece g of row r at g ^ (r & 7)); the TMA
        // store clips the ragged M / N edges.
        auto piece = [&](int g) -> uint4 {
          if (OUT_F32)
            return make_uint4(__float_as_uint(v[4 * g]), __float_as_uint(v[4 * g + 1]), __float_as_uint(v[4 * g + 2]),
                              __float_as_uint(v[4 * g + 3]));
          return make_uint4(pack_bf16x2(v[8 * g], v[8 * g + 1]), pack_bf16x2(v[8 * g + 2], v[8 * g + 3]),
                            pack_bf16x2(v[8 * g + 4], v[8 * g + 5]), pack_bf16x2(v[8 * g + 6], v[8 * g + 7]));
        };
        unsigned char *buf = stage_buf + (chunk_count % NBUF) * 4096;
        if (chunk_count >= NBUF) {
          if (lane == 0) bulk_wait_read<NBUF - 1>();
          __syncwarp();
        }
#pragma unroll
        for (int g = 0; g < 8; ++g)
          *reinterpret_cast<uint4 *>(buf + lane * 128 + ((g ^ (lane & 7)) << 4)) = piece(g);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&map_c, buf, col0, mb * BM + static_cast<int>(rank) * HALF_ROWS + q * 32);
          bulk_commit();
        }
        ++chunk_count;
      }
    }
    if (lane == 0) bulk_wait_all();
  }

  __syncthreads();
  if (*abort_flag || (status && *reinterpret_cast<volatile int *>(status) == GPT2_ERR_WAIT_TIMEOUT)) {
    // Unwinding after a timeout: give loads the other CTA may still have in
    // flight towards this CTA's barriers time to land (bounded pause).
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 200000ull) {
    }
  }
  cluster_sync_all();  // the leader's MMAs are drained and both CTAs' epilogues are done
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// Largest number of co-resident pairs of this kernel, per device (0 = not yet known).
template <int EPI, int OUT_F32>
int pair_slots(int num_sms) {
  static std::atomic<int> slots[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return num_sms / 2;
  std::atomic<int> &slot = slots[dev & 63];
  int n = slot.load();
  if (n > 0) return n;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(num_sms & ~1));
  cfg.blockDim = dim3(NTHREADS);
  cfg.dynamicSmemBytes = PairCfg<EPI, OUT_F32>::SMEM_BYTES;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_tc2sm_kernel<EPI, OUT_F32>, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = num_sms / 2;
  }
  if (n > num_sms / 2) n = num_sms / 2;
  slot.store(n);
  return n;
}

template <int EPI, int OUT_F32>
cudaError_t launch_pair(const TcGemmPlan &p, int ldc, const float *bias, const bf16 *resid, int *status, int num_sms,
                        cudaStream_t st, const float *scale, const LnFold &ln) {
  static std::atomic<uint64_t> attr_done{0};
  cudaError_t e = set_smem_once(gemm_tc2sm_kernel<EPI, OUT_F32>, PairCfg<EPI, OUT_F32>::SMEM_BYTES, attr_done);
  if (e != cudaSuccess) return e;
  const int tiles = ((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN);
  int pairs = pair_slots<EPI, OUT_F32>(num_sms);
  if (pairs < 1) pairs = 1;
  if (tiles < pairs) pairs = tiles;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
  cfg.blockDim = dim3(NTHREADS);
  cfg.dynamicSmemBytes = PairCfg<EPI, OUT_F32>::SMEM_BYTES;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // Wide outputs (the lm_head's vocabulary) take 16-block groups (4096 rows
  // of A, 6 MB at d = 768, reused by every N-block while in L2); measured 2.5 %
  // faster than 64-block groups and 4 % faster than 8-block groups.
  const int num_n = (p.N + BN - 1) / BN;
  const int group_m = num_n >= 64 ? GPT2_PAIR_GROUP_M_WIDE : 8;
  return cudaLaunchKernelEx(&cfg, gemm_tc2sm_kernel<EPI, OUT_F32>, p.map_a, p.map_b, p.map_c, ldc, p.M, p.N, p.K,
                            group_m, bias, resid, status, scale, ln);
}
}  // namespace

bool gemm_tc2sm_usable(const TcGemmPlan &plan, const void *C, int ldc, int out_f32) {
  return plan.two_sm && plan.bn == 128 && plan.has_c && plan.c_ptr == C && plan.c_ld == ldc &&
         plan.c_f32 == out_f32;
}

cudaError_t launch_gemm_tc2sm(const TcGemmPlan &plan, void *C, int ldc, int out_f32, const float *bias,
                              const bf16 *resid, int epi, int *status, int num_sms, cudaStream_t st,
                              const float *scale, const LnFold &ln) {
  if (!gemm_tc2sm_usable(plan, C, ldc, out_f32) || num_sms < 2) return cudaErrorInvalidValue;
  if (!ln_fold_valid(plan, epi, out_f32, &ln)) return cudaErrorInvalidValue;
#define GPT2_PAIR_CASE(E, F) \
  case E: return launch_pair<E, F>(plan, ldc, bias, resid, status, num_sms, st, scale, ln)
  if (out_f32) {
    switch (epi) {
      GPT2_PAIR_CASE(EPI_NONE, 1);
      GPT2_PAIR_CASE(EPI_BIAS, 1);
      GPT2_PAIR_CASE(EPI_LN_BIAS, 1);
    }
    return cudaErrorInvalidValue;
  }
  switch (epi) {
    GPT2_PAIR_CASE(EPI_NONE, 0);
    GPT2_PAIR_CASE(EPI_BIAS, 0);
    GPT2_PAIR_CASE(EPI_BIAS_GELU, 0);
    GPT2_PAIR_CASE(EPI_BIAS_RESID, 0);
    GPT2_PAIR_CASE(EPI_BIAS_GELU_ERF, 0);
    GPT2_PAIR_CASE(EPI_LN_BIAS, 0);
    GPT2_PAIR_CASE(EPI_LN_BIAS_GELU, 0);
    GPT2_PAIR_CASE(EPI_BIAS_RESID_STATS, 0);
    GPT2_PAIR_CASE(EPI_LN_BIAS_GELU_ERF, 0);
    GPT2_PAIR_CASE(EPI_LNRES_BIAS_RESID_STATS, 0);
  }
#undef GPT2_PAIR_CASE
  return cudaErrorInvalidValue;
}

}  // namespace gpt2
