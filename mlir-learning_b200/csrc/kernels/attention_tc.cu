// attention_tc.cu -- an earlier BF16 attention on the 5th-generation tensor
// cores (tcgen05, S and O accumulators in TMEM, Q / K / V staged by TMA,
// two softmax threads per query row, P through shared memory), head dim 64.
// The forward runs attention_tc2.cu; this kernel stays as an independent
// cross-check (gpt2k_attention_ex with GPT2K_ATTN_BF16_TC_SMEM_P) and owns
// the tensor-map plan both kernels use.
//
// Replaces, per layer, the reference's q k^T and p v linalg.batch_matmul
// launches and the scale / causal where / additive mask / softmax generics
// between them (src/gpt/README.md:6, lib/DeadArgmaxElimination.cpp:4-6) in the
// BF16 configuration, and the BERT encoder's self-attention
// (src/bert-base-uncased/lower_bert_model.py:12-18) with causal = 0.
// Semantics are those of attention_f32.cu: key k is attendable from query q
// iff mask[b, k] != 0 and, when causal, k <= q; masked keys weigh 0; rows
// without an attendable key are finished by attn_masked_rows_kernel.
//
// Persistent: one CTA per SM walks work items (batch, head, two 128-query
// tiles q0 .. q0+255), heaviest first; Q is double-buffered so the next
// item's Q lands while the current one finishes.  576 threads:
//   warp 0       TMA: Q tiles once, then 128-key K and V tiles into a
//                2-stage ring (3-D tensor map over qkv [B][S][3D], so keys
//                past the sequence end read as zeros);
//   warp 1       TMEM allocation and the MMA thread: S_t = Q_t K^T
//                (M=128, N=128, K=16 x 4) and O_t += P_t V (M=128, N=64,
//                K=16 x 8, V as an MN-major operand), ping-ponging the two
//                tiles so that the tensor cores work on one tile while the
//                other tile's softmax runs;
//   warps 2-9    softmax of tile 0, warps 10-17 softmax of tile 1: two
//                threads per query row (its TMEM lane), 64 key columns each,
//                the row max exchanged through shared memory, running max /
//                sum in FP32 with exp2 and
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
constexpr int DH = 64, BQ = 128, BKV = 128, ST = 2, NTHREADS = 576;
constexpr int SOFTMAX_THREADS = 256;  // per query tile: 8 warps, two threads per row
constexpr int TILE_BYTES = 128 * 64 * 2;  // one Q, K or V tile: 128 rows x 128 bytes
constexpr int P_BYTES = 2 * TILE_BYTES;   // P: 128 rows x 128 keys bf16 = two 64-key blocks
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct AttnTcSmem {
  static constexpr int Q = 0;                          // 2 buffers x 2 query tiles
  static constexpr int K = Q + 4 * TILE_BYTES;
  static constexpr int V = K + ST * TILE_BYTES;
  static constexpr int P = V + ST * TILE_BYTES;
  static constexpr int BARS = P + 2 * P_BYTES;
  // q_full[2], q_empty[2], k_full[ST], v_full[ST], k_empty[ST], v_empty[ST], s_full[2], s_free[2], p_full[2],
  // o_done[2], drain
  static constexpr int NBARS = 4 + 4 * ST + 8 + 1;
  static constexpr int XM = BARS + NBARS * 8;          // row max exchange [2 parity][2 tiles][2 halves][128]
  static constexpr int XL = XM + 2 * 2 * 2 * 128 * 4;  // row sum exchange [2 tiles][2 halves][128]
  static constexpr int MISC = XL + 2 * 2 * 128 * 4;
  static constexpr int TOTAL = MISC + 16;
  static constexpr int ALLOC = TOTAL + 1024;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed FP32 pairs (sm_100 f32x2 instructions): two elements per FMA / ADD.
__device__ __forceinline__ uint64_t pk2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void up2(uint64_t v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Work item w: (query-tile pair, batch, head), heaviest pairs first.
struct AttnItem {
  int b, h, q0, n_kv[2], n_kv_max;
};
__device__ __forceinline__ AttnItem attn_item(int w, int S, int B, int H, int causal, const int *kv_end) {
  AttnItem it;
  const int n_pairs = (S + 2 * BQ - 1) / (2 * BQ);
  const int pair = n_pairs - 1 - w / (B * H);
  const int bh = w % (B * H);
  it.b = bh / H;
  it.h = bh % H;
  it.q0 = pair * 2 * BQ;
  // Key tiles past the last unmasked key carry no weight; at least one tile
  // is kept so every role sees the same non-empty schedule (a sequence
  // without unmasked keys gets zeros here and is finished by the
  // masked-rows pass).
  int n_kv_total = (S + BKV - 1) / BKV;
  if (kv_end) n_kv_total = min(n_kv_total, max(1, (kv_end[it.b] + BKV - 1) / BKV));
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int qs = it.q0 + t * BQ;
    it.n_kv[t] = qs < S ? (causal ? min(qs / BKV + 1, n_kv_total) : n_kv_total) : 0;
  }
  it.n_kv_max = max(it.n_kv[0], it.n_kv[1]);
  return it;
}

__global__ void __launch_bounds__(NTHREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap map_qkv, const uint8_t *__restrict__ key_valid,
                        bf16 *__restrict__ out, int B, int S, int H, int *status, int causal,
                        const int *__restrict__ kv_end) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char *sm =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + AttnTcSmem::BARS);
  uint64_t *q_full = bars, *q_empty = bars + 2;
  uint64_t *k_full = bars + 4, *v_full = k_full + ST, *k_empty = v_full + ST, *v_empty = k_empty + ST;
  uint64_t *s_full = v_empty + ST, *s_free = s_full + 2, *p_full = s_free + 2, *o_done = p_full + 2;
  uint64_t *drain = o_done + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + AttnTcSmem::MISC);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(sm + AttnTcSmem::MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = H * DH;
  const int n_items = ((S + 2 * BQ - 1) / (2 * BQ)) * B * H;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int s = 0; s < ST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&s_free[t], SOFTMAX_THREADS / 32);  // one arrival per softmax warp
      mbar_init(&p_full[t], SOFTMAX_THREADS / 32);
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

  if (warp == 0) {
    // ---------------- TMA producer (whole warp, one elected lane issues) ----------------
    const bool leader = elect_one_sync();
    if (leader) prefetch_tmap(&map_qkv);
    uint32_t q_issued[2] = {0, 0}, kv_issued[ST] = {};
    int qi = 0, kvi = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, ++qi) {
      const AttnItem it = attn_item(w, S, B, H, causal, kv_end);
      const int qb = qi & 1;
      if (!mbar_wait_warp(&q_empty[qb], ((qi >> 1) & 1) ^ 1, abort_flag, status)) { ok = false; break; }
      if (leader) {
        mbar_arrive_expect_tx(&q_full[qb], 2 * TILE_BYTES);
        tma_load_3d(sm + AttnTcSmem::Q + qb * 2 * TILE_BYTES, &map_qkv, &q_full[qb], it.h * DH, it.q0, it.b);
        tma_load_3d(sm + AttnTcSmem::Q + qb * 2 * TILE_BYTES + TILE_BYTES, &map_qkv, &q_full[qb], it.h * DH,
                    it.q0 + BQ, it.b);
      }
      ++q_issued[qb];
      for (int j = 0; j < it.n_kv_max; ++j, ++kvi) {
        const int s = kvi % ST;
        // K slots free up once the S MMAs that read them complete, V slots
        // once the P V MMAs do, so K runs a full iteration ahead of V.
        if (!mbar_wait_warp(&k_empty[s], ((kvi / ST) & 1) ^ 1, abort_flag, status)) { ok = false; break; }
        if (leader) {
          mbar_arrive_expect_tx(&k_full[s], TILE_BYTES);
          tma_load_3d(sm + AttnTcSmem::K + s * TILE_BYTES, &map_qkv, &k_full[s], D + it.h * DH, j * BKV, it.b);
        }
        if (!mbar_wait_warp(&v_empty[s], ((kvi / ST) & 1) ^ 1, abort_flag, status)) { ok = false; break; }
        if (leader) {
          mbar_arrive_expect_tx(&v_full[s], TILE_BYTES);
          tma_load_3d(sm + AttnTcSmem::V + s * TILE_BYTES, &map_qkv, &v_full[s], 2 * D + it.h * DH, j * BKV,
                      it.b);
        }
        ++kv_issued[s];
      }
    }
    if (!ok) {
      set_status(status, GPT2_ERR_WAIT_TIMEOUT);
      *abort_flag = 1;
    }
    // Let every copy issued land before the CTA can exit.
    for (int i = 0; i < 2; ++i)
      if (q_issued[i]) mbar_wait_warp(&q_full[i], (q_issued[i] - 1) & 1, nullptr);
    for (int s = 0; s < ST; ++s)
      if (kv_issued[s]) {
        mbar_wait_warp(&k_full[s], (kv_issued[s] - 1) & 1, nullptr);
        mbar_wait_warp(&v_full[s], (kv_issued[s] - 1) & 1, nullptr);
      }
  } else if (warp == 1) {
    // ---------------- MMA issuer (whole warp, one elected lane issues) ----------------
    // The whole warp runs the schedule so that its state stays warp-uniform
    // (uniform registers); only the elected lane issues tcgen05 instructions.
    const bool leader = elect_one_sync();
    constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128, 0);  // Q K^T: both K-major
    constexpr uint32_t idesc_o = idesc_bf16_f32(128, 64, 1);   // P V: V is MN-major
    // Base descriptors, computed once: the MMA thread shares its SM sub-partition
    // with four busy softmax warps, so each MMA issue must cost only an add
    // per operand (start addresses are in 16-byte units in the low bits).
    const uint64_t dq0 = sdesc_kmajor_sw128(smem_u32(sm + AttnTcSmem::Q));
    const uint64_t dk0 = sdesc_kmajor_sw128(smem_u32(sm + AttnTcSmem::K));
    const uint64_t dp0 = sdesc_kmajor_sw128(smem_u32(sm + AttnTcSmem::P));
    const uint64_t dv0 = sdesc_mnmajor_sw128(smem_u32(sm + AttnTcSmem::V), TILE_BYTES, 1024);
    constexpr uint64_t kTile16 = TILE_BYTES >> 4;
    int g_base[2] = {0, 0};  // running per-tile iteration count (barrier phases)
    int qi = 0, kv_base = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, ++qi) {
      const AttnItem it = attn_item(w, S, B, H, causal, kv_end);
      const int qb = qi & 1;
      const uint64_t dq = dq0 + qb * 2 * kTile16;
      if (!mbar_wait_warp(&q_full[qb], (qi >> 1) & 1, abort_flag, status)) { ok = false; break; }
      // S_t(j) = Q_t K_j^T into TMEM columns [t*128, t*128+128)
      auto issue_s = [&](int t, int j) -> bool {
        const int g = g_base[t] + j;
        const int s = (kv_base + j) % ST;
        if (g > 0 && !mbar_wait_warp(&s_free[t], (g - 1) & 1, abort_flag, status)) return false;
        tc_fence_after();
        const uint64_t a = dq + t * kTile16, b = dk0 + s * kTile16;
        if (leader) {
#pragma unroll
          for (int k = 0; k < DH / 16; ++k) tc_mma_f16(tmem + t * 128, a + 2 * k, b + 2 * k, idesc_s, k != 0);
          tc_commit(&s_full[t]);
        }
        __syncwarp();
        return true;
      };
      // O_t (+)= P_t V_j into TMEM columns [256 + t*64, 256 + t*64 + 64)
      auto issue_pv = [&](int t, int j) -> bool {
        const int g = g_base[t] + j;
        const int s = (kv_base + j) % ST;
        if (!mbar_wait_warp(&p_full[t], g & 1, abort_flag, status)) return false;
        tc_fence_after();
        const uint64_t a = dp0 + t * 2 * kTile16, b = dv0 + s * kTile16;
        const uint32_t first = j == 0;
        if (leader) {
#pragma unroll
          for (int k = 0; k < BKV / 16; ++k)
            tc_mma_f16(tmem + 256 + t * 64, a + (k >> 2) * kTile16 + (k & 3) * 2, b + k * (2048 >> 4), idesc_o,
                       !(first && k == 0));
          tc_commit(&o_done[t]);
        }
        __syncwarp();
        return true;
      };
      ok = mbar_wait_warp(&k_full[kv_base % ST], (kv_base / ST) & 1, abort_flag, status);
      for (int t = 0; t < 2 && ok; ++t)
        if (it.n_kv[t] > 0) ok = issue_s(t, 0);
      if (ok && leader) tc_commit(&k_empty[kv_base % ST]);
      for (int j = 0; j < it.n_kv_max && ok; ++j) {
        const int kv = kv_base + j;
        // S_t(j+1) as soon as the softmax holds S_t(j) in registers, so the
        // next score tile is ready when the current softmax finishes.
        bool k_ready = false;
        for (int t = 0; t < 2 && ok; ++t) {
          if (j + 1 < it.n_kv[t]) {
            if (!k_ready) {
              ok = mbar_wait_warp(&k_full[(kv + 1) % ST], ((kv + 1) / ST) & 1, abort_flag, status);
              k_ready = true;
            }
            if (ok) ok = issue_s(t, j + 1);
          }
        }
        if (!ok) break;
        if (k_ready && leader) tc_commit(&k_empty[(kv + 1) % ST]);
        if (!mbar_wait_warp(&v_full[kv % ST], (kv / ST) & 1, abort_flag, status)) { ok = false; break; }
        for (int t = 0; t < 2 && ok; ++t)
          if (j < it.n_kv[t]) ok = issue_pv(t, j);
        if (leader) tc_commit(&v_empty[kv % ST]);
      }
      if (!ok) break;
      if (leader) tc_commit(&q_empty[qb]);  // this item's Q tiles are free once its MMAs complete
      g_base[0] += it.n_kv[0];
      g_base[1] += it.n_kv[1];
      kv_base += it.n_kv_max;
    }
    if (!ok) {
      set_status(status, GPT2_ERR_WAIT_TIMEOUT);
      *abort_flag = 1;
    }
    if (leader) tc_commit(drain);
    mbar_wait_warp(drain, 0, nullptr);
  } else if (warp >= 2) {
    // ---------------- softmax: two threads per query row ----------------
    // Warps 2-9 serve tile 0, warps 10-17 tile 1.  Within a tile, warps
    // (w, w + 4) share TMEM lane quarter w % 4: the first handles key columns
    // 0-63 of each row, the second 64-127.  The row max is exchanged through
    // shared memory with a 64-thread named barrier per warp pair; the row
    // sums stay per half until the epilogue.
    const int t = (warp - 2) >> 3;          // query tile
    const int half = ((warp - 2) >> 2) & 1; // key columns [half*64, half*64+64)
    const int qd = warp & 3;                // TMEM lane quarter
    const int r = qd * 32 + lane;           // row within the tile
    const int bar_id = 1 + t * 4 + qd;      // named barrier of the warp pair
    const uint32_t lane_addr = static_cast<uint32_t>(qd * 32) << 16;
    const uint32_t s_tmem = tmem + lane_addr + t * 128 + half * 64;
    const uint32_t o_tmem = tmem + lane_addr + 256 + t * 64 + half * 32;
    unsigned char *p_row = sm + AttnTcSmem::P + t * P_BYTES + half * TILE_BYTES + r * 128;
    float *xm = reinterpret_cast<float *>(sm + AttnTcSmem::XM);
    float *xl = reinterpret_cast<float *>(sm + AttnTcSmem::XL);
    const float sl2 = 0.125f * 1.4426950408889634f;  // (1/sqrt(64)) * log2(e)
    // A failed wait raises the abort flag but never changes the control flow:
    // the two threads of a row must execute the same named barriers, and
    // once the flag is up every later wait returns at once.
    // One lane per warp polls the barrier (keeping shared-memory barrier
    // traffic low for the MMA warp); the warp then proceeds together.
    auto wait = [&](uint64_t *bar, uint32_t parity) {
      if (lane == 0 && !mbar_wait(bar, parity, abort_flag, status)) {
        set_status(status, GPT2_ERR_WAIT_TIMEOUT);
        *abort_flag = 1;
      }
      __syncwarp();
    };
    // All lanes' tcgen05 / shared-memory work is done (each lane fenced) before one lane arrives.
    auto arrive = [&](uint64_t *bar) {
      __syncwarp();
      if (lane == 0) mbar_arrive(bar);
    };
    int g_base = 0;
    for (int w = blockIdx.x; w < n_items; w += gridDim.x) {
      const AttnItem it = attn_item(w, S, B, H, causal, kv_end);
      const int n = it.n_kv[t];
      if (n == 0) continue;
      const int qrow = it.q0 + t * BQ + r;  // query index within the sequence
      const uint8_t *kv_ok = key_valid ? key_valid + (int64_t)it.b * S : nullptr;
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; j < n; ++j) {
        const int g = g_base + j;
        wait(&s_full[t], g & 1);
        tc_fence_after();
        const int kv0 = j * BKV + half * 64;  // first key of this thread's 64 columns
        const bool diag = causal && j * BKV + BKV > it.q0 + t * BQ;  // tile touches the causal diagonal
        const bool tail = j * BKV + BKV > S;                // tile runs past the sequence end
        uint32_t sv[64];
        tmem_ld_32x32b_x32(s_tmem, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
        tmem_ld_32x32b_x32(s_tmem + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
        tc_wait_ld();
        tc_fence_before();
        arrive(&s_free[t]);  // S is in registers: the next Q K^T may overwrite it
        // Pass 1: masking (raw scores -> -inf) and the partial row max, 8 chains.
        float mx[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mx[e] = -INFINITY;
        // Key flags are checked element by element only when this half-tile
        // has a masked key (one 64-byte AND test, warp-uniform: every lane
        // of the warp reads the same 64 flags); right-padded batches take
        // the plain path on every tile but the last.
        bool need_mask = diag || tail;
        if (!need_mask && kv_ok) {
          const uint8_t *fp = kv_ok + kv0;
          if ((reinterpret_cast<uintptr_t>(fp) & 15) == 0) {
            const uint4 *f4 = reinterpret_cast<const uint4 *>(fp);
            uint32_t all = 0x01010101u;
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) {
              const uint4 v4 = f4[c4];
              all &= v4.x & v4.y & v4.z & v4.w;
            }
            need_mask = all != 0x01010101u;  // flags are 0 / 1 bytes
          } else {
            need_mask = true;
          }
        }
        if (need_mask) {
#pragma unroll
          for (int c = 0; c < 64; c += 16) {
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
              const bool okk = ((fw[e >> 2] >> (8 * (e & 3))) & 0xffu) != 0 && (!causal || key <= qrow) && key < S;
              const float x = okk ? __uint_as_float(sv[c + e]) : -INFINITY;
              sv[c + e] = __float_as_uint(x);
              mx[e & 7] = fmaxf(mx[e & 7], x);
            }
          }
        } else {
#pragma unroll
          for (int c = 0; c < 64; c += 2)
            mx[(c >> 1) & 7] = max3(mx[(c >> 1) & 7], __uint_as_float(sv[c]), __uint_as_float(sv[c + 1]));
        }
        float mraw = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                           fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
        // Exchange with the partner thread of the row (buffers alternate by iteration).
        float *xmb = xm + ((g & 1) * 2 + t) * 256;
        xmb[half * 128 + r] = mraw;
        named_bar_sync(bar_id, 64);
        mraw = fmaxf(mraw, xmb[(half ^ 1) * 128 + r]);
        const float mt = mraw * sl2;  // sl2 > 0: the max of the scaled scores
        // Lazy rescale (both halves take the same decision from the same max).
        float alpha = 1.f;
        bool rescale = false;
        if (mt > m_run + kRescaleThreshold || (m_run == -INFINITY && mt != -INFINITY)) {
          alpha = m_run == -INFINITY ? 0.f : ex2(m_run - mt);
          rescale = j > 0 && m_run != -INFINITY;
          m_run = mt;
        }
        const float neg_m = m_run == -INFINITY ? 0.f : -m_run;
        // P_t and O_t of the previous iteration must be consumed before they are touched.
        if (j > 0) wait(&o_done[t], (g - 1) & 1);
        tc_fence_after();
        // The TMEM loads and stores are warp-wide: when any row of the warp
        // rescales, every lane takes part, with a factor of 1 where its row does not.
        if (__any_sync(0xffffffffu, rescale)) {
          const float a = rescale ? alpha : 1.f;
#pragma unroll 1
          for (int c = 0; c < 32; c += 16) {
            uint32_t ov[16];
            tmem_ld_32x32b_x16(o_tmem + c, ov);
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * a);
            tmem_st_32x32b_x16(o_tmem + c, ov);
          }
          tc_wait_st();
        }
        l_run *= alpha;
        // Pass 2: p = 2^(s * scale * log2e - m), bf16 P (this half's 64-key block); the scale
        // and the sums run on packed pairs.
        const uint64_t sl2x2 = pk2(sl2, sl2), negm2 = pk2(neg_m, neg_m);
        uint64_t rs2[4] = {0, 0, 0, 0};
#pragma unroll
        for (int gi = 0; gi < 8; ++gi) {
          uint32_t wv[4];
#pragma unroll
          for (int e2 = 0; e2 < 4; ++e2) {
            const uint64_t x2 = fma2(pk2(__uint_as_float(sv[gi * 8 + 2 * e2]), __uint_as_float(sv[gi * 8 + 2 * e2 + 1])),
                                     sl2x2, negm2);
            float x0, x1;
            up2(x2, x0, x1);
            const float p0 = ex2(x0), p1 = ex2(x1);
            rs2[e2] = add2(rs2[e2], pk2(p0, p1));
            wv[e2] = pack_bf16x2(p0, p1);
          }
          *reinterpret_cast<uint4 *>(p_row + ((gi ^ (r & 7)) << 4)) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
        }
        {
          const uint64_t s01 = add2(rs2[0], rs2[1]), s23 = add2(rs2[2], rs2[3]);
          float a0, a1;
          up2(add2(s01, s23), a0, a1);
          l_run += a0 + a1;
        }
        fence_proxy_async_smem();
        tc_fence_before();
        arrive(&p_full[t]);
      }
      // Epilogue: O / l (l = sum of both halves), bf16; each half stores 32 columns.
      xl[(t * 2 + half) * 128 + r] = l_run;
      wait(&o_done[t], (g_base + n - 1) & 1);
      tc_fence_after();
      named_bar_sync(bar_id, 64);
      const float l_tot = l_run + xl[(t * 2 + (half ^ 1)) * 128 + r];
      uint32_t ov[32];
      tmem_ld_32x32b_x32(o_tmem, ov);
      tc_wait_ld();
      if (qrow < S) {
        const float inv = l_tot > 0.f ? 1.0f / l_tot : 0.f;
        uint4 *dst = reinterpret_cast<uint4 *>(out + ((int64_t)it.b * S + qrow) * D + it.h * DH + half * 32);
#pragma unroll
        for (int gi = 0; gi < 4; ++gi) {
          const float *f = reinterpret_cast<const float *>(&ov[gi * 8]);
          dst[gi] = make_uint4(pack_bf16x2(f[0] * inv, f[1] * inv), pack_bf16x2(f[2] * inv, f[3] * inv),
                               pack_bf16x2(f[4] * inv, f[5] * inv), pack_bf16x2(f[6] * inv, f[7] * inv));
        }
      }
      // The partner reads xl before either thread reuses it for the next item.
      named_bar_sync(bar_id, 64);
      g_base += n;
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

int attention_tc_plan(AttnTcPlan *plan, const bf16 *qkv, int B, int S, int H, const bf16 *o) {
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
  plan->out = nullptr;
  if (o) {
    if (reinterpret_cast<uintptr_t>(o) & 15) return -2;
    const int64_t D = (int64_t)H * DH;
    const cuuint64_t odims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(B)};
    const cuuint64_t ostrides[2] = {static_cast<cuuint64_t>(D * 2), static_cast<cuuint64_t>(D * 2 * S)};
    const cuuint32_t obox[3] = {64, 32, 1};
    r = f(&plan->map_out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<bf16 *>(o), odims, ostrides, obox, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return -3;
    plan->out = o;
  }
  plan->qkv = qkv;
  plan->B = B;
  plan->S = S;
  plan->H = H;
  return 0;
}

cudaError_t launch_attention_tc(const AttnTcPlan &plan, const uint8_t *key_valid, bf16 *o, int *status,
                                cudaStream_t st, int causal, const int *kv_end) {
  if (plan.B <= 0 || plan.S <= 0 || plan.H <= 0 || plan.H > 65535 || plan.B > 65535) return cudaErrorInvalidValue;
  static std::atomic<uint64_t> attr_done{0};
  cudaError_t e = set_smem_once(attention_tc_kernel, AttnTcSmem::ALLOC, attr_done);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int items = ((plan.S + 2 * BQ - 1) / (2 * BQ)) * plan.B * plan.H;
  const int grid = items < sms ? items : sms;
  attention_tc_kernel<<<grid, NTHREADS, AttnTcSmem::ALLOC, st>>>(plan.map_qkv, key_valid, o, plan.B, plan.S, plan.H,
                                                                  status, causal, kv_end);
  return cudaGetLastError();
}

}  // namespace gpt2
