// gemm_tc.cu -- BF16 GEMM on the 5th-generation tensor cores (tcgen05,
// accumulators in TMEM, operands staged by TMA) with fused epilogues.
//
// Replaces the reference's linalg.matmul launches (QKV, attention out-proj,
// MLP fc and proj, the tied lm_head; README.md:11) and the bias / GELU /
// residual generics fused around them (lib/ElementwiseFusion.cpp:43-109), in
// the BF16 configuration.
//
//   C[M, N] = epilogue(A[M, K] @ B[N, K]^T)
//   A: activations, bf16, row-major (K-major); B: weights packed [N, K]
//   (K-major) at load time; f32 accumulation in TMEM; bf16 or f32 output.
//
// Structure (one CTA per SM, persistent, 192 threads):
//   warp 0      TMA producer: 128 x 64 A and BN x 64 B tiles, 128-byte
//               swizzle, into a STAGES-deep shared-memory ring (mbarrier
//               full/empty pairs, transaction-count completion);
//   warp 1      TMEM allocator and MMA issuer: one thread issues
//               tcgen05.mma.cta_group::1.kind::f16 (M=128, N=BN, K=16) four
//               times per stage and tcgen05.commit's the stage back to the
//               producer; accumulators are double-buffered in TMEM (2 x BN
//               columns) so the epilogue of tile i overlaps the MMAs of i+1;
//   warps 2..5  epilogue: tcgen05.ld 32 rows x 32 columns per warp, bias /
//               gelu_new / residual in registers, 16-byte global stores.
// Tiles are walked in groups of 16 M-blocks so that the A rows and B columns
// live in L2 while they are reused.  No cluster multicast anywhere.
//
// Every mbarrier wait is bounded (common.cuh); on a timeout the kernel
// records GPT2_ERR_WAIT_TIMEOUT, stops issuing, drains what it issued and
// frees its TMEM before returning.
#include <atomic>

#include "../common.cuh"
#include "../gemm_epi.cuh"
#include "../kernels.h"

namespace gpt2 {

namespace {
constexpr int BM = 128, BK = 64, NTHREADS = 192, GROUP_M = 16;

template <int BN>
struct TcCfg {
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  // Epilogue staging: 4 warps x 2 buffers x (32 rows x 128 bytes).
  static constexpr int STAGING_BYTES = 4 * 2 * 4096;
  static constexpr int SMEM_BYTES = 1024 /*align slack*/ + STAGES * STAGE_BYTES + STAGING_BYTES + 256;
};

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int &mb, int &nb) {
  const int per_group = GROUP_M * num_n;
  const int group = t / per_group;
  const int first_m = group * GROUP_M;
  const int gsize = min(num_m - first_m, GROUP_M);
  const int in = t - group * per_group;
  mb = first_m + in % gsize;
  nb = in / gsize;
}

template <int BN, int EPI, int OUT_F32, int TMA_STORE>
__global__ void __launch_bounds__(NTHREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   const __grid_constant__ CUtensorMap map_c, void *C, int ldc, int M, int N, int K,
                   const float *__restrict__ bias, const bf16 *resid, int *status,
                   const float *__restrict__ scale, const LnFold ln, int withhold) {
  using Cfg = TcCfg<BN>;
  using Kind = EpiKind<EPI>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char *sa = smem;
  unsigned char *sb = smem + STAGES * Cfg::A_BYTES;
  unsigned char *staging = smem + STAGES * Cfg::STAGE_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(staging + Cfg::STAGING_BYTES);
  uint64_t *full = bars, *empty = bars + STAGES, *tfull = bars + 2 * STAGES, *tempty = bars + 2 * STAGES + 2;
  uint64_t *drain = bars + 2 * STAGES + 4;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 5);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM, num_n = (N + BN - 1) / BN, num_k = (K + BK - 1) / BK;
  const int total = num_m * num_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    prefetch_tmap(&map_a);
    prefetch_tmap(&map_b);
    uint32_t issued[STAGES];
#pragma unroll
    for (int s = 0; s < STAGES; ++s) issued[s] = 0;
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      int mb, nb;
      tile_coords(t, num_m, num_n, mb, nb);
      for (int kb = 0; kb < num_k; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, status)) { ok = false; break; }
        // Test hook of the timeout path (gpt2k_test_gemm_withheld_load): CTA 0
        // never fills its first stage, so its MMA thread's wait runs out.
        if (withhold >= 0 && blockIdx.x == 0 && it == withhold) continue;
        mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
        tma_load_2d(sa + s * Cfg::A_BYTES, &map_a, &full[s], kb * BK, mb * BM);
        tma_load_2d(sb + s * Cfg::B_BYTES, &map_b, &full[s], kb * BK, nb * BN);
        ++issued[s];
      }
    }
    if (!ok) {
      set_status(status, GPT2_ERR_WAIT_TIMEOUT);
      *abort_flag = 1;
      // Let the copies already in flight land before the CTA's shared memory goes away.
      for (int s = 0; s < STAGES; ++s)
        if (issued[s]) mbar_wait(&full[s], (issued[s] - 1) & 1, nullptr);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
    int it = 0, local = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++local) {
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
        const uint32_t a0 = smem_u32(sa + s * Cfg::A_BYTES), b0 = smem_u32(sb + s * Cfg::B_BYTES);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          tc_mma_f16(d_tmem, sdesc_kmajor_sw128(a0 + k * 32), sdesc_kmajor_sw128(b0 + k * 32), idesc,
                     (kb | k) != 0);
        tc_commit(&empty[s]);
      }
      if (!ok) break;
      tc_commit(&tfull[acc]);
    }
    if (!ok) {
      set_status(status, GPT2_ERR_WAIT_TIMEOUT);
      *abort_flag = 1;
    }
    // Drain: every MMA this thread issued has completed once this arrives.
    tc_commit(drain);
    mbar_wait(drain, 0, nullptr);
  } else if (warp >= 2) {
    // ---------------- epilogue ----------------
    // Chunks of 128 bytes per row: 32 f32 or 64 bf16 columns.  Thread i of
    // the warp owns row (q*32 + i) of the tile.  With TMA_STORE the chunk is
    // written to a 128-byte-swizzled staging buffer (16-byte piece j of row r
    // at piece j ^ (r & 7): conflict-free) and stored by one bulk tensor copy
    // that the hardware clips at the ragged M / N edges.
    constexpr int CH = OUT_F32 ? 32 : 64;
    constexpr int NCH = BN / CH;
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = q * 32 + lane;
    unsigned char *stage_buf = staging + (warp - 2) * 2 * 4096;
    uint32_t chunk_count = 0;
    int local = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++local) {
      int mb, nb;
      tile_coords(t, num_m, num_n, mb, nb);
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      if (Kind::resid && !OUT_F32) {
        // Pull this row's residual into L2 while the tile's main loop runs,
        // so the chunked loads below do not wait on HBM (short-K GEMMs
        // would otherwise be bound by the epilogue).
        const int prow = mb * BM + row_in_tile;
        if (prow < M) {
          const bf16 *rp = resid + (int64_t)prow * ldc + nb * BN;
#pragma unroll
          for (int i = 0; i < BN / 64; ++i)
            if (nb * BN + i * 64 < N) asm volatile("prefetch.global.L2 [%0];" ::"l"(rp + i * 64));
        }
      }
      const int row = mb * BM + row_in_tile;
      const bool row_ok = row < M;
      const int64_t row_off = (int64_t)row * ldc;
      float ln_rstd = 0.f, ln_nmr = 0.f;  // folded LayerNorm of A's row, read while the main loop runs
      if (Kind::ln && row_ok) ln_row_stats(ln, row, ln_rstd, ln_nmr);
      float res_rstd = 0.f, res_nmr = 0.f;  // the residual's LayerNorm (EPI_LNRES_*)
      if (Kind::lnres && row_ok) ln_res_row_stats(ln, row, N, res_rstd, res_nmr);
      RowStats rs;
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
      load_res(res_cur, nb * BN);
#pragma unroll 1
      for (int c = 0; c < NCH; ++c) {
        const int col0 = nb * BN + c * CH;
        if (c + 1 < NCH) load_res(res_nxt, col0 + CH);
        uint32_t r[CH];
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN + c * CH;
        tmem_ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        if (CH == 64) tmem_ld_32x32b_x32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[CH == 64 ? 32 : 0]));
        tc_wait_ld();
        if (c == NCH - 1) {
          tc_fence_before();
          mbar_arrive(&tempty[acc]);
        }
        float *v = reinterpret_cast<float *>(r);  // epilogue in place
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
        const bool full_chunk = col0 + CH <= N;
        if (Kind::resid && !OUT_F32 && row_ok) {
          if (full_chunk) {
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
          // Statistics of the stored bf16 row, one LN_SEG-column segment per
          // two chunks (BN is a multiple of LN_SEG); columns past N are 0.
          rs.add_bf16<CH>(v);
          if (c & 1) rs.flush(ln, row, (col0 + CH - LN_SEG) / LN_SEG, row_ok);
        }
        // 16-byte piece g of this row: 4 f32 or 8 bf16 values
        auto piece = [&](int g) -> uint4 {
          if (OUT_F32)
            return make_uint4(__float_as_uint(v[4 * g]), __float_as_uint(v[4 * g + 1]), __float_as_uint(v[4 * g + 2]),
                              __float_as_uint(v[4 * g + 3]));
          return make_uint4(pack_bf16x2(v[8 * g], v[8 * g + 1]), pack_bf16x2(v[8 * g + 2], v[8 * g + 3]),
                            pack_bf16x2(v[8 * g + 4], v[8 * g + 5]), pack_bf16x2(v[8 * g + 6], v[8 * g + 7]));
        };
        if (TMA_STORE) {
          unsigned char *buf = stage_buf + (chunk_count & 1) * 4096;
          if (chunk_count >= 2) {
            if (lane == 0) bulk_wait_read<1>();
            __syncwarp();
          }
#pragma unroll
          for (int g = 0; g < 8; ++g)
            *reinterpret_cast<uint4 *>(buf + lane * 128 + ((g ^ (lane & 7)) << 4)) = piece(g);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&map_c, buf, col0, mb * BM + q * 32);
            bulk_commit();
          }
          ++chunk_count;
        } else if (row_ok) {
          if (full_chunk && (!OUT_F32 || (ldc & 3) == 0)) {
            uint4 *cp = reinterpret_cast<uint4 *>(reinterpret_cast<unsigned char *>(C) +
                                                  (row_off + col0) * (OUT_F32 ? 4 : 2));
#pragma unroll
            for (int g = 0; g < 8; ++g) cp[g] = piece(g);
          } else if (OUT_F32) {
            float *cp = reinterpret_cast<float *>(C) + row_off + col0;
            for (int j = 0; j < CH; ++j)
              if (col0 + j < N) cp[j] = v[j];
          } else {
            bf16 *cp = reinterpret_cast<bf16 *>(C) + row_off + col0;
            for (int j = 0; j < CH; ++j)
              if (col0 + j < N) cp[j] = __float2bfloat16_rn(v[j]);
          }
        }
      }
    }
    if (TMA_STORE && lane == 0) bulk_wait_all();
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static std::atomic<EncodeTiledFn> fn{nullptr};
  EncodeTiledFn f = fn.load();
  if (f) return f;
  void *p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || !p)
    return nullptr;
  f = reinterpret_cast<EncodeTiledFn>(p);
  fn.store(f);
  return f;
}

// 2-D bf16 tensor [rows, cols] row-major, box [box_rows, 64 cols], 128-byte swizzle.
int make_map_2d(CUtensorMap *map, const void *base, int64_t rows, int64_t cols, int box_rows) {
  EncodeTiledFn f = encode_fn();
  if (!f) return -1;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (cols * 2) % 16) return -2;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols * 2)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = f(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -3;
}

// Output [rows, cols] (row stride ld elements) in boxes of 32 rows x 128
// bytes with the 128-byte swizzle of the staging buffers.
int make_map_out(CUtensorMap *map, const void *base, int64_t rows, int64_t cols, int64_t ld, int f32) {
  EncodeTiledFn f = encode_fn();
  if (!f) return -1;
  const int es = f32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld * es) % 16) return -2;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * es)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / es), 32};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = f(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                 const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                 CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -3;
}

template <int BN, int EPI, int OUT_F32, int TMA_STORE>
cudaError_t launch_variant(const TcGemmPlan &p, void *C, int ldc, const float *bias, const bf16 *resid, int *status,
                           int num_sms, cudaStream_t st, const float *scale, const LnFold &ln, int withhold = -1) {
  using Cfg = TcCfg<BN>;
  static std::atomic<uint64_t> attr_done{0};
  cudaError_t e = set_smem_once(gemm_tc_kernel<BN, EPI, OUT_F32, TMA_STORE>, Cfg::SMEM_BYTES, attr_done);
  if (e != cudaSuccess) return e;
  const int tiles = ((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN);
  const int grid = tiles < num_sms ? tiles : num_sms;
  gemm_tc_kernel<BN, EPI, OUT_F32, TMA_STORE><<<grid, NTHREADS, Cfg::SMEM_BYTES, st>>>(
      p.map_a, p.map_b, p.map_c, C, ldc, p.M, p.N, p.K, bias, resid, status, scale, ln, withhold);
  return cudaGetLastError();
}

template <int BN, int EPI, int OUT_F32>
cudaError_t launch_store(const TcGemmPlan &p, void *C, int ldc, const float *bias, const bf16 *resid, int *status,
                         int num_sms, cudaStream_t st, const float *scale, const LnFold &ln) {
  const bool tma = p.has_c && p.c_ptr == C && p.c_ld == ldc && p.c_f32 == OUT_F32;
  if (tma) return launch_variant<BN, EPI, OUT_F32, 1>(p, C, ldc, bias, resid, status, num_sms, st, scale, ln);
  return launch_variant<BN, EPI, OUT_F32, 0>(p, C, ldc, bias, resid, status, num_sms, st, scale, ln);
}

template <int BN>
cudaError_t dispatch_epi(const TcGemmPlan &p, void *C, int ldc, int out_f32, const float *bias, const bf16 *resid,
                         int epi, int *status, int num_sms, cudaStream_t st, const float *scale, const LnFold &ln) {
#define GPT2_TC_CASE(E, F) \
  case E: return launch_store<BN, E, F>(p, C, ldc, bias, resid, status, num_sms, st, scale, ln)
  if (out_f32) {
    switch (epi) {
      GPT2_TC_CASE(EPI_NONE, 1);
      GPT2_TC_CASE(EPI_BIAS, 1);
      GPT2_TC_CASE(EPI_LN_BIAS, 1);
    }
    return cudaErrorInvalidValue;
  }
  switch (epi) {
    GPT2_TC_CASE(EPI_NONE, 0);
    GPT2_TC_CASE(EPI_BIAS, 0);
    GPT2_TC_CASE(EPI_BIAS_GELU, 0);
    GPT2_TC_CASE(EPI_BIAS_RESID, 0);
    GPT2_TC_CASE(EPI_BIAS_GELU_ERF, 0);
    GPT2_TC_CASE(EPI_LN_BIAS, 0);
    GPT2_TC_CASE(EPI_LN_BIAS_GELU, 0);
    GPT2_TC_CASE(EPI_BIAS_RESID_STATS, 0);
    GPT2_TC_CASE(EPI_LN_BIAS_GELU_ERF, 0);
    GPT2_TC_CASE(EPI_LNRES_BIAS_RESID_STATS, 0);
  }
#undef GPT2_TC_CASE
  return cudaErrorInvalidValue;
}
}  // namespace

int tc_gemm_plan(TcGemmPlan *plan, const bf16 *A, const bf16 *B, int M, int N, int K, int bn) {
  if (!plan || M <= 0 || N <= 0 || K <= 0 || K % 8 || (bn != 128 && bn != 256 && bn != TC_TILE_PAIR)) return -10;
  plan->two_sm = bn == TC_TILE_PAIR;
  if (plan->two_sm) bn = 128;
  plan->has_c = 0;
  plan->c_ptr = nullptr;
  plan->M = M;
  plan->N = N;
  plan->K = K;
  plan->bn = bn;
  int r = make_map_2d(&plan->map_a, A, M, K, BM);
  if (r) return r;
  return make_map_2d(&plan->map_b, B, N, K, bn);
}

int tc_gemm_set_output(TcGemmPlan *plan, const void *C, int ldc, int out_f32) {
  plan->c_ptr = C;
  plan->c_ld = ldc;
  plan->c_f32 = out_f32;
  plan->has_c = make_map_out(&plan->map_c, C, plan->M, plan->N, ldc, out_f32) == 0;
  return plan->has_c;
}

cudaError_t launch_gemm_tc_withheld_load(const TcGemmPlan &plan, void *C, int *status, int num_sms,
                                         cudaStream_t st) {
  if (plan.two_sm || plan.bn != 128 || !status || num_sms <= 0) return cudaErrorInvalidValue;
  const LnFold none;
  return launch_variant<128, EPI_NONE, 0, 0>(plan, C, plan.N, nullptr, nullptr, status, num_sms, st, nullptr, none, 0);
}

bool ln_fold_valid(const TcGemmPlan &plan, int epi, int out_f32, const LnFold *ln) {
  auto aligned16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (epi == EPI_LN_BIAS || epi == EPI_LN_BIAS_GELU || epi == EPI_LN_BIAS_GELU_ERF)
    return ln && ln->c1 && ln->c2 && ln->stats_in && aligned16(ln->c1) && aligned16(ln->c2) && ln->k == plan.K &&
           ln->nseg_in == ln_segments(plan.K) && ln->eps > 0.f && !(epi != EPI_LN_BIAS && out_f32);
  if (epi == EPI_BIAS_RESID_STATS) return ln && ln->stats_out && ln->nseg_out == ln_segments(plan.N) && !out_f32;
  if (epi == EPI_LNRES_BIAS_RESID_STATS)
    return ln && ln->stats_out && ln->nseg_out == ln_segments(plan.N) && !out_f32 && ln->res_stats &&
           ln->res_gain && ln->res_shift && aligned16(ln->res_gain) && aligned16(ln->res_shift) && ln->eps > 0.f &&
           plan.N % 8 == 0;
  return true;
}

cudaError_t launch_gemm_tc(const TcGemmPlan &plan, void *C, int ldc, int out_f32, const float *bias,
                           const bf16 *resid, int epi, int *status, int num_sms, cudaStream_t st,
                           const float *scale, const LnFold *ln) {
  if (ldc < plan.N || num_sms <= 0) return cudaErrorInvalidValue;
  if (!out_f32 && ldc % 8) return cudaErrorInvalidValue;
  const bool ln_epi = epi == EPI_LN_BIAS || epi == EPI_LN_BIAS_GELU || epi == EPI_LN_BIAS_GELU_ERF;
  if (epi != EPI_NONE && !ln_epi && !bias) return cudaErrorInvalidValue;
  if ((epi == EPI_BIAS_RESID || epi == EPI_BIAS_RESID_STATS || epi == EPI_LNRES_BIAS_RESID_STATS) && !resid)
    return cudaErrorInvalidValue;
  if (!ln_fold_valid(plan, epi, out_f32, ln)) return cudaErrorInvalidValue;
  const LnFold none;
  const LnFold &lf = ln ? *ln : none;
  if (plan.two_sm && gemm_tc2sm_usable(plan, C, ldc, out_f32) && num_sms >= 2)
    return launch_gemm_tc2sm(plan, C, ldc, out_f32, bias, resid, epi, status, num_sms, st, scale, lf);
  if (plan.bn == 256)
    return dispatch_epi<256>(plan, C, ldc, out_f32, bias, resid, epi, status, num_sms, st, scale, lf);
  return dispatch_epi<128>(plan, C, ldc, out_f32, bias, resid, epi, status, num_sms, st, scale, lf);
}

}  // namespace gpt2
