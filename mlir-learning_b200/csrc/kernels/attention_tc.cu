// attention_tc.cu -- BF16 causal attention on the 5th-generation tensor cores
// (tcgen05, S and O accumulators in TMEM, Q / K / V staged by TMA), head
// dim 64.
//
// Replaces, per layer, the reference's q k^T and p v linalg.batch_matmul
// launches and the scale / causal where / additive mask / softmax generics
// between them (src/gpt/README.md:6, lib/DeadArgmaxElimination.cpp:4-6) in the
// BF16 configuration.  Semantics are those of attention_f32.cu: key k is
// attendable from query q iff k <= q and mask[b, k] != 0; masked keys weigh 0;
// rows without an attendable key are finished by attn_masked_rows_kernel.
//
// One CTA = one (batch, head) and two 128-query tiles (rows q0 .. q0+255),
// 320 threads:
//   warp 0       TMA: Q tiles once, then 128-key K and V tiles into a
//                3-stage ring (3-D tensor map over qkv [B][S][3D], so keys
//                past the sequence end read as zeros);
//   warp 1       TMEM allocation and the MMA thread: S_t = Q_t K^T
//                (M=128, N=128, K=16 x 4) and O_t += P_t V (M=128, N=64,
//                K=16 x 8, V as an MN-major operand), ping-ponging the two
//                tiles so that the tensor cores work on one tile while the
//                other tile's softmax runs;
//   warps 2-5    softmax of tile 0, warps 6-9 softmax of tile 1: one thread
//                per query row (its TMEM lane), scores read from TMEM in
//                32-column pieces, running max / sum in FP32 with exp2 and
//                the 1/8 * log2(e) scale folded in, P written as bf16 into a
//                128-byte-swizzled shared tile (the MMA's K-major A operand),
//                and the O rescale done lazily: only when the running max
//                grows by more than 8 (log2 units), so the un-normalised
//                partial sums stay below 2^8 and most tiles skip it.
// TMEM: S0 [0,128), S1 [128,256), O0 [256,320), O1 [320,384) of 512 columns.
// Every barrier wait is bounded; a timeout records status 2 and unwinds.
#include <atomic>

#include "../common.cuh"
#include "../kernels.h"

namespace gpt2 {

namespace {
constexpr int DH = 64, BQ = 128, BKV = 128, ST = 3, NTHREADS = 320;
constexpr int TILE_BYTES = 128 * 64 * 2;  // one Q, K or V tile: 128 rows x 128 bytes
constexpr int P_BYTES = 2 * TILE_BYTES;   // P: 128 rows x 128 keys bf16 = two 64-key blocks
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct AttnTcSmem {
  static constexpr int Q = 0;
  static constexpr int K = Q + 2 * TILE_BYTES;
  static constexpr int V = K + ST * TILE_BYTES;
  static constexpr int P = V + ST * TILE_BYTES;
  static constexpr int BARS = P + 2 * P_BYTES;
  // barriers: q, k_full[ST], v_full[ST], kv_empty[ST], s_full[2], s_free[2], p_full[2], o_done[2], drain
  static constexpr int NBARS = 1 + 3 * ST + 8 + 1;
  static constexpr int MISC = BARS + NBARS * 8;
  static constexpr int TOTAL = MISC + 16;
  static constexpr int ALLOC = TOTAL + 1024;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(NTHREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap map_qkv, const uint8_t *__restrict__ key_valid,
                        bf16 *__restrict__ out, int S, int H, int *status) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char *sm =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + AttnTcSmem::BARS);
  uint64_t *bar_q = bars;
  uint64_t *k_full = bars + 1, *v_full = k_full + ST, *kv_empty = v_full + ST;
  uint64_t *s_full = kv_empty + ST, *s_free = s_full + 2, *p_full = s_free + 2, *o_done = p_full + 2;
  uint64_t *drain = o_done + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + AttnTcSmem::MISC);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(sm + AttnTcSmem::MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_pairs = (S + 2 * BQ - 1) / (2 * BQ);
  const int pair = n_pairs - 1 - blockIdx.x;  // heaviest first
  const int h = blockIdx.y, b = blockIdx.z;
  const int D = H * DH;
  const int q0 = pair * 2 * BQ;
  // number of key tiles each query tile needs (causal), 0 if the tile is past the end
  const int n_kv_total = (S + BKV - 1) / BKV;
  int n_kv[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int qs = q0 + t * BQ;
    n_kv[t] = qs < S ? min(qs / BKV + 1, n_kv_total) : 0;
  }
  const int n_kv_max = max(n_kv[0], n_kv[1]);

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&s_free[t], 128);
      mbar_init(&p_full[t], 128);
      mbar_init(&o_done[t], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    prefetch_tmap(&map_qkv);
    mbar_arrive_expect_tx(bar_q, 2 * TILE_BYTES);
    tma_load_3d(sm + AttnTcSmem::Q, &map_qkv, bar_q, h * DH, q0, b);
    tma_load_3d(sm + AttnTcSmem::Q + TILE_BYTES, &map_qkv, bar_q, h * DH, q0 + BQ, b);
    uint32_t issued[ST] = {0, 0, 0};
    bool ok = true;
    for (int j = 0; j < n_kv_max; ++j) {
      const int s = j % ST;
      if (!mbar_wait(&kv_empty[s], ((j / ST) & 1) ^ 1, abort_flag, status)) {
        ok = false;
        break;
      }
      mbar_arrive_expect_tx(&k_full[s], TILE_BYTES);
      tma_load_3d(sm + AttnTcSmem::K + s * TILE_BYTES, &map_qkv, &k_full[s], D + h * DH, j * BKV, b);
      mbar_arrive_expect_tx(&v_full[s], TILE_BYTES);
      tma_load_3d(sm + AttnTcSmem::V + s * TILE_BYTES, &map_qkv, &v_full[s], 2 * D + h * DH, j * BKV, b);
      ++issued[s];
    }
    if (!ok) {
      set_status(status, GPT2_ERR_WAIT_TIMEOUT);
      *abort_flag = 1;
    }
    // Let every copy issued land before the CTA can exit.
    mbar_wait(bar_q, 0, nullptr);
    for (int s = 0; s < ST; ++s)
      if (issued[s]) {
        mbar_wait(&k_full[s], (issued[s] - 1) & 1, nullptr);
        mbar_wait(&v_full[s], (issued[s] - 1) & 1, nullptr);
      }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128, 0);  // Q K^T: both K-major
    constexpr uint32_t idesc_o = idesc_bf16_f32(128, 64, 1);   // P V: V is MN-major
    const uint32_t qa = smem_u32(sm + AttnTcSmem::Q), ka = smem_u32(sm + AttnTcSmem::K),
                   va = smem_u32(sm + AttnTcSmem::V), pa = smem_u32(sm + AttnTcSmem::P);
    bool ok = mbar_wait(bar_q, 0, abort_flag, status);
    auto issue_s = [&](int t, int j) -> bool {
      const int s = j % ST;
      if (j > 0 && !mbar_wait(&s_free[t], (j - 1) & 1, abort_flag, status)) return false;
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < DH / 16; ++k)
        tc_mma_f16(tmem + t * 128, sdesc_kmajor_sw128(qa + t * TILE_BYTES + k * 32),
                   sdesc_kmajor_sw128(ka + s * TILE_BYTES + k * 32), idesc_s, k != 0);
      tc_commit(&s_full[t]);
      return true;
    };
    auto issue_pv = [&](int t, int j) -> bool {
      const int s = j % ST;
      if (!mbar_wait(&p_full[t], j & 1, abort_flag, status)) return false;
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < BKV / 16; ++k)
        tc_mma_f16(tmem + 256 + t * 64, sdesc_kmajor_sw128(pa + t * P_BYTES + (k >> 2) * TILE_BYTES + (k & 3) * 32),
                   sdesc_mnmajor_sw128(va + s * TILE_BYTES + k * 2048, TILE_BYTES, 1024), idesc_o,
                   (j | k) != 0);
      tc_commit(&o_done[t]);
      return true;
    };
    if (ok && n_kv_max > 0) {
      ok = mbar_wait(&k_full[0], 0, abort_flag, status);
      for (int t = 0; t < 2 && ok; ++t)
        if (n_kv[t] > 0) ok = issue_s(t, 0);
    }
    for (int j = 0; j < n_kv_max && ok; ++j) {
      const int s = j % ST;
      const uint32_t ph = (j / ST) & 1;
      if (!mbar_wait(&v_full[s], ph, abort_flag, status)) { ok = false; break; }
      const bool next_k = j + 1 < n_kv_max;
      bool k_ready = false;
      for (int t = 0; t < 2 && ok; ++t) {
        if (j < n_kv[t]) ok = issue_pv(t, j);
        if (ok && j + 1 < n_kv[t]) {
          if (next_k && !k_ready) {
            ok = mbar_wait(&k_full[(j + 1) % ST], ((j + 1) / ST) & 1, abort_flag, status);
            k_ready = true;
          }
          if (ok) ok = issue_s(t, j + 1);
        }
      }
      tc_commit(&kv_empty[s]);
    }
    if (!ok) {
      set_status(status, GPT2_ERR_WAIT_TIMEOUT);
      *abort_flag = 1;
    }
    tc_commit(drain);
    mbar_wait(drain, 0, nullptr);
  } else if (warp >= 2) {
    // ---------------- softmax, one thread per query row ----------------
    const int t = (warp - 2) >> 2;          // query tile of this warpgroup
    const int qd = warp & 3;                // TMEM lane quarter
    const int r = qd * 32 + lane;           // row within the tile
    const int qrow = q0 + t * BQ + r;       // query index within the sequence
    const uint32_t lane_addr = static_cast<uint32_t>(qd * 32) << 16;
    const uint32_t s_tmem = tmem + lane_addr + t * 128;
    const uint32_t o_tmem = tmem + lane_addr + 256 + t * 64;
    unsigned char *p_row = sm + AttnTcSmem::P + t * P_BYTES + r * 128;
    const uint8_t *kv_ok = key_valid ? key_valid + (int64_t)b * S : nullptr;
    const float sl2 = 0.125f * 1.4426950408889634f;  // (1/sqrt(64)) * log2(e)
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv[t]; ++j) {
      if (!mbar_wait(&s_full[t], j & 1, abort_flag, status)) { ok = false; break; }
      tc_fence_after();
      const int kv0 = j * BKV;
      const bool diag = kv0 + BKV > q0 + t * BQ;        // tile touches the causal diagonal
      const bool tail = kv0 + BKV > S;                  // tile runs past the sequence end
      const bool need_mask = diag || tail || kv_ok != nullptr;
      // Pass 1: row max over the 128 scores (read from TMEM in 4 pieces).
      uint32_t sv[128];
#pragma unroll
      for (int c = 0; c < 4; ++c)
        tmem_ld_32x32b_x32(s_tmem + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[c * 32]));
      tc_wait_ld();
      tc_fence_before();
      mbar_arrive(&s_free[t]);  // S is in registers: the next Q K^T may overwrite it
      float mt = -INFINITY;
      if (need_mask) {
#pragma unroll
        for (int c = 0; c < 128; c += 16) {
          uint32_t fw[4] = {0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u};
          if (kv_ok) {
            const uint8_t *fp = kv_ok + kv0 + c;
            if (kv0 + c + 16 <= S && (reinterpret_cast<uintptr_t>(fp) & 15) == 0) {
              const uint4 f4 = *reinterpret_cast<const uint4 *>(fp);
              fw[0] = f4.x;
              fw[1] = f4.y;
              fw[2] = f4.z;
              fw[3] = f4.w;
            } else {
#pragma unroll
              for (int w4 = 0; w4 < 4; ++w4) {
                uint32_t wv = 0;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int key = kv0 + c + w4 * 4 + e;
                  wv |= static_cast<uint32_t>(key < S ? fp[w4 * 4 + e] : 0) << (8 * e);
                }
                fw[w4] = wv;
              }
            }
          }
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int key = kv0 + c + e;
            const bool okk = ((fw[e >> 2] >> (8 * (e & 3))) & 0xffu) != 0 && key <= qrow && key < S;
            const float x = okk ? __uint_as_float(sv[c + e]) * sl2 : -INFINITY;
            sv[c + e] = __float_as_uint(x);
            mt = fmaxf(mt, x);
          }
        }
      } else {
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          const float x = __uint_as_float(sv[c]) * sl2;
          sv[c] = __float_as_uint(x);
          mt = fmaxf(mt, x);
        }
      }
      // Lazy rescale: keep the old max unless the new one exceeds it by more
      // than the threshold (or no max exists yet).
      float m_use = m_run;
      bool rescale = false;
      float alpha = 1.f;
      if (mt > m_run + kRescaleThreshold || (m_run == -INFINITY && mt != -INFINITY)) {
        alpha = m_run == -INFINITY ? 0.f : ex2(m_run - mt);
        m_use = mt;
        rescale = j > 0 && m_run != -INFINITY;
        m_run = mt;
      }
      const float m_sub = m_use == -INFINITY ? 0.f : m_use;
      // P_t(j-1) must have been consumed (and O_t updated) before P and O are touched.
      if (j > 0 && !mbar_wait(&o_done[t], (j - 1) & 1, abort_flag, status)) { ok = false; break; }
      tc_fence_after();
      if (rescale) {
#pragma unroll 1
        for (int c = 0; c < 64; c += 16) {
          uint32_t ov[16];
          tmem_ld_32x32b_x16(o_tmem + c, ov);
          tc_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
          tmem_st_32x32b_x16(o_tmem + c, ov);
        }
        tc_wait_st();
      }
      l_run *= alpha;
      // Pass 2: probabilities, row sum, bf16 P into the swizzled shared tile.
      float rs = 0.f;
#pragma unroll
      for (int blk = 0; blk < 2; ++blk) {
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          float p[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            p[e] = ex2(__uint_as_float(sv[blk * 64 + g * 8 + e]) - m_sub);
            rs += p[e];
          }
          const uint4 w = make_uint4(pack_bf16x2(p[0], p[1]), pack_bf16x2(p[2], p[3]), pack_bf16x2(p[4], p[5]),
                                     pack_bf16x2(p[6], p[7]));
          *reinterpret_cast<uint4 *>(p_row + blk * TILE_BYTES + ((g ^ (r & 7)) << 4)) = w;
        }
      }
      l_run += rs;
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[t]);
    }
    // Epilogue: O / l for this row, bf16, 128 contiguous bytes.
    if (ok && n_kv[t] > 0) {
      if (mbar_wait(&o_done[t], (n_kv[t] - 1) & 1, abort_flag, status)) {
        tc_fence_after();
        uint32_t ov[64];
        tmem_ld_32x32b_x32(o_tmem, *reinterpret_cast<uint32_t(*)[32]>(&ov[0]));
        tmem_ld_32x32b_x32(o_tmem + 32, *reinterpret_cast<uint32_t(*)[32]>(&ov[32]));
        tc_wait_ld();
        if (qrow < S) {
          const float inv = l_run > 0.f ? 1.0f / l_run : 0.f;
          uint4 *dst = reinterpret_cast<uint4 *>(out + ((int64_t)b * S + qrow) * D + h * DH);
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            const float *f = reinterpret_cast<const float *>(&ov[g * 8]);
            dst[g] = make_uint4(pack_bf16x2(f[0] * inv, f[1] * inv), pack_bf16x2(f[2] * inv, f[3] * inv),
                                pack_bf16x2(f[4] * inv, f[5] * inv), pack_bf16x2(f[6] * inv, f[7] * inv));
          }
        }
      } else {
        ok = false;
      }
    }
    if (!ok) {
      set_status(status, GPT2_ERR_WAIT_TIMEOUT);
      *abort_flag = 1;
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn_attn() {
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
}  // namespace

int attention_tc_plan(AttnTcPlan *plan, const bf16 *qkv, int B, int S, int H) {
  EncodeTiledFn f = encode_fn_attn();
  if (!f) return -1;
  if (reinterpret_cast<uintptr_t>(qkv) & 15) return -2;
  const int64_t D3 = 3LL * H * DH;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(D3), static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(B)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(D3 * 2), static_cast<cuuint64_t>(D3 * 2 * S)};
  const cuuint32_t box[3] = {64, 128, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = f(&plan->map_qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<bf16 *>(qkv), dims, strides, box,
                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return -3;
  plan->qkv = qkv;
  plan->B = B;
  plan->S = S;
  plan->H = H;
  return 0;
}

cudaError_t launch_attention_tc(const AttnTcPlan &plan, const uint8_t *key_valid, bf16 *o, int *status,
                                cudaStream_t st) {
  if (plan.B <= 0 || plan.S <= 0 || plan.H <= 0 || plan.H > 65535 || plan.B > 65535) return cudaErrorInvalidValue;
  static std::atomic<uint64_t> attr_done{0};
  cudaError_t e = set_smem_once(attention_tc_kernel, AttnTcSmem::ALLOC, attr_done);
  if (e != cudaSuccess) return e;
  dim3 grid((plan.S + 2 * BQ - 1) / (2 * BQ), plan.H, plan.B);
  attention_tc_kernel<<<grid, NTHREADS, AttnTcSmem::ALLOC, st>>>(plan.map_qkv, key_valid, o, plan.S, plan.H, status);
  return cudaGetLastError();
}

}  // namespace gpt2
