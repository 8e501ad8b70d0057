// attention_tc2.cu -- BF16 attention on the 5th-generation tensor cores with
// one softmax thread per query row and the probabilities P kept in tensor
// memory: the P.V product reads P as its A operand straight from TMEM
// (tcgen05.mma with A in TMEM), so P never touches shared memory.  Head
// dim 64.
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
// tiles), heaviest first; Q is double-buffered across items.  320 threads,
// so that a thread may hold a whole 128-key score row in registers (10
// warps: at most 3 per SM sub-partition, 168 registers each):
//   warp 0       TMA: Q tiles once per item, then 128-key K and V tiles into
//                a 3-stage ring (3-D tensor map over qkv [B][S][3D]; keys
//                past the sequence end read as zeros);
//   warp 1       TMEM allocation and the MMA thread: S_t = Q_t K^T (M=128,
//                N=128, K=16 x 4, both operands in shared memory) and
//                O_t += P_t V (M=128, N=64, K=16 x 8, P from TMEM, V an
//                MN-major shared-memory operand), S_t(j+1) issued as soon as
//                the softmax holds S_t(j) in registers;
//   warps 2-5    softmax of tile 0, warps 6-9 softmax of tile 1: thread =
//                query row (its TMEM lane), all 128 key columns: masking,
//                row max, lazy rescale of O (only when the running max grows
//                by more than 8 in log2 units), exp2 with the 1/8 * log2(e)
//                scale folded in, running sum in FP32, P packed to bf16 pairs
//                and stored into its TMEM columns; the epilogue divides O by
//                the row sum and writes bf16 through shared memory and a TMA
//                store.  The two tiles' softmax warps of a sub-partition
//                issue independently: the kernel is bound by instruction
//                issue and latency, not by the MUFU unit (measured: making
//                them take turns on it, or moving a quarter of the
//                exponentials to an FMA-pipe polynomial, was slower).
// TMEM (512 columns): S0 [0,128), S1 [128,256), O0 [256,320), O1 [320,384),
// P0 [384,448), P1 [448,512) (P: 128 bf16 per row = 64 columns).
// Every barrier wait is bounded; a timeout records status 2 and unwinds.
#include <atomic>

#include "../common.cuh"
#include "../kernels.h"

namespace gpt2 {

namespace {
constexpr int DH = 64, BQ = 128, BKV = 128, ST = 3, NTHREADS = 320;
constexpr int SOFTMAX_WARPS = 4;          // per query tile: one thread per row
constexpr int TILE_BYTES = 128 * 64 * 2;  // one Q, K or V tile: 128 rows x 128 bytes
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr uint32_t kColS = 0, kColO = 256, kColP = 384;

constexpr int OST_BYTES = 32 * 128;       // output staging of one softmax warp: 32 rows x 128 bytes

struct Smem2 {
  static constexpr int Q = 0;  // 2 buffers x 2 query tiles
  static constexpr int K = Q + 4 * TILE_BYTES;
  static constexpr int V = K + ST * TILE_BYTES;
  static constexpr int OST = V + ST * TILE_BYTES;  // [tile][quarter] output staging (128-byte swizzle)
  static constexpr int BARS = OST + 8 * OST_BYTES;
  // q_full[2], q_empty[2], k_full[ST], v_full[ST], k_empty[ST], v_empty[ST], s_full[2], s_free[2], p_full[2],
  // o_done[2], drain
  static constexpr int NBARS = 4 + 4 * ST + 8 + 1;
  static constexpr int MISC = BARS + NBARS * 8;
  static constexpr int TOTAL = MISC + 16;
  static constexpr int ALLOC = TOTAL + 1024;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

struct AttnItem {
  int b, h, q0, n_kv[2], n_kv_max;
};
// Work item w: (query-tile pair, batch, head), heaviest pairs first; key
// tiles past the last unmasked key are dropped (at least one is kept so
// every role sees the same non-empty schedule).
__device__ __forceinline__ AttnItem attn_item(int w, int S, int B, int H, int causal, const int *kv_end) {
  AttnItem it;
  const int n_pairs = (S + 2 * BQ - 1) / (2 * BQ);
  const int pair = n_pairs - 1 - w / (B * H);
  const int bh = w % (B * H);
  it.b = bh / H;
  it.h = bh % H;
  it.q0 = pair * 2 * BQ;
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
    attention_tc2_kernel(const __grid_constant__ CUtensorMap map_qkv, const __grid_constant__ CUtensorMap map_out,
                         const uint8_t *__restrict__ key_valid, int B, int S, int H, int *status, int causal,
                         const int *__restrict__ kv_end) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char *sm =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + Smem2::BARS);
  uint64_t *q_full = bars, *q_empty = bars + 2;
  uint64_t *k_full = bars + 4, *v_full = k_full + ST, *k_empty = v_full + ST, *v_empty = k_empty + ST;
  uint64_t *s_full = v_empty + ST, *s_free = s_full + 2, *p_full = s_free + 2, *o_done = p_full + 2;
  uint64_t *drain = o_done + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + Smem2::MISC);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(sm + Smem2::MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
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
      mbar_init(&s_free[t], SOFTMAX_WARPS);  // one arrival per softmax warp
      mbar_init(&p_full[t], SOFTMAX_WARPS);
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
    const int D = H * DH;
    uint32_t q_issued[2] = {0, 0}, kv_issued[ST] = {};
    int qi = 0, kvi = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, ++qi) {
      const AttnItem it = attn_item(w, S, B, H, causal, kv_end);
      const int qb = qi & 1;
      if (!mbar_wait_warp(&q_empty[qb], ((qi >> 1) & 1) ^ 1, abort_flag, status)) { ok = false; break; }
      if (leader) {
        mbar_arrive_expect_tx(&q_full[qb], 2 * TILE_BYTES);
        tma_load_3d(sm + Smem2::Q + qb * 2 * TILE_BYTES, &map_qkv, &q_full[qb], it.h * DH, it.q0, it.b);
        tma_load_3d(sm + Smem2::Q + qb * 2 * TILE_BYTES + TILE_BYTES, &map_qkv, &q_full[qb], it.h * DH, it.q0 + BQ,
                    it.b);
      }
      ++q_issued[qb];
      for (int j = 0; j < it.n_kv_max; ++j, ++kvi) {
        const int s = kvi % ST;
        // K slots free up once the S MMAs that read them complete, V slots
        // once the P V MMAs do.
        if (!mbar_wait_warp(&k_empty[s], ((kvi / ST) & 1) ^ 1, abort_flag, status)) { ok = false; break; }
        if (leader) {
          mbar_arrive_expect_tx(&k_full[s], TILE_BYTES);
          tma_load_3d(sm + Smem2::K + s * TILE_BYTES, &map_qkv, &k_full[s], D + it.h * DH, j * BKV, it.b);
        }
        if (!mbar_wait_warp(&v_empty[s], ((kvi / ST) & 1) ^ 1, abort_flag, status)) { ok = false; break; }
        if (leader) {
          mbar_arrive_expect_tx(&v_full[s], TILE_BYTES);
          tma_load_3d(sm + Smem2::V + s * TILE_BYTES, &map_qkv, &v_full[s], 2 * D + it.h * DH, j * BKV, it.b);
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
    const bool leader = elect_one_sync();
    constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128, 0);  // Q K^T: both K-major
    constexpr uint32_t idesc_o = idesc_bf16_f32(128, 64, 1);   // P V: V is MN-major
    const uint64_t dq0 = sdesc_kmajor_sw128(smem_u32(sm + Smem2::Q));
    const uint64_t dk0 = sdesc_kmajor_sw128(smem_u32(sm + Smem2::K));
    const uint64_t dv0 = sdesc_mnmajor_sw128(smem_u32(sm + Smem2::V), TILE_BYTES, 1024);
    constexpr uint64_t kTile16 = TILE_BYTES >> 4;
    int g_base[2] = {0, 0};  // running per-tile iteration count (barrier phases)
    int qi = 0, kv_base = 0;
    bool ok = true;
    bool pre_s0 = false;  // S_0(0) of this item was issued while the previous item finished
    for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, ++qi) {
      const AttnItem it = attn_item(w, S, B, H, causal, kv_end);
      const int qb = qi & 1;
      const uint64_t dq = dq0 + qb * 2 * kTile16;
      bool pre_next = false;
      if (!mbar_wait_warp(&q_full[qb], (qi >> 1) & 1, abort_flag, status)) { ok = false; break; }
      // S_t = Q_t K^T into TMEM columns [t*128, t*128+128): global step g of
      // tile t, K from ring slot `slot`, Q tiles at descriptor dqx.
      auto issue_s_at = [&](int t, int g, int slot, uint64_t dqx) -> bool {
        if (g > 0 && !mbar_wait_warp(&s_free[t], (g - 1) & 1, abort_flag, status)) return false;
        tc_fence_after();
        const uint64_t a = dqx + t * kTile16, b = dk0 + slot * kTile16;
        if (leader) {
#pragma unroll
          for (int k = 0; k < DH / 16; ++k)
            tc_mma_f16(tmem + kColS + t * 128, a + 2 * k, b + 2 * k, idesc_s, k != 0);
          tc_commit(&s_full[t]);
        }
        __syncwarp();
        return true;
      };
      auto issue_s = [&](int t, int j) -> bool { return issue_s_at(t, g_base[t] + j, (kv_base + j) % ST, dq); };
      // Once tile 0 has its last P.V of this item, the next item's first
      // S_0 goes out (its Q and first K tile are loaded independently of the
      // rest of this item), so tile 0's softmax starts the next item while
      // tile 1 finishes this one.
      auto prefetch_next_s0 = [&]() -> bool {
        if (w + (int)gridDim.x >= n_items) return true;
        const int qn = qi + 1, qbn = qn & 1, kvn = kv_base + it.n_kv_max;
        if (!mbar_wait_warp(&q_full[qbn], (qn >> 1) & 1, abort_flag, status)) return false;
        if (!mbar_wait_warp(&k_full[kvn % ST], (kvn / ST) & 1, abort_flag, status)) return false;
        if (!issue_s_at(0, g_base[0] + it.n_kv[0], kvn % ST, dq0 + qbn * 2 * kTile16)) return false;
        pre_next = true;
        return true;
      };
      // O_t (+)= P_t V_j: P_t from TMEM columns [384 + t*64, +64), 8 columns per K=16 step
      auto issue_pv = [&](int t, int j) -> bool {
        const int g = g_base[t] + j;
        const int s = (kv_base + j) % ST;
        if (!mbar_wait_warp(&p_full[t], g & 1, abort_flag, status)) return false;
        tc_fence_after();
        const uint64_t b = dv0 + s * kTile16;
        const uint32_t first = j == 0;
        if (leader) {
#pragma unroll
          for (int k = 0; k < BKV / 16; ++k)
            tc_mma_f16_ts(tmem + kColO + t * 64, tmem + kColP + t * 64 + k * 8, b + k * (2048 >> 4), idesc_o,
                          !(first && k == 0));
          tc_commit(&o_done[t]);
        }
        __syncwarp();
        return true;
      };
      ok = mbar_wait_warp(&k_full[kv_base % ST], (kv_base / ST) & 1, abort_flag, status);
      for (int t = 0; t < 2 && ok; ++t)
        if (it.n_kv[t] > 0 && !(t == 0 && pre_s0)) ok = issue_s(t, 0);
      if (ok && leader) tc_commit(&k_empty[kv_base % ST]);
      for (int j = 0; j < it.n_kv_max && ok; ++j) {
        const int kv = kv_base + j;
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
        for (int t = 0; t < 2 && ok; ++t) {
          if (j < it.n_kv[t]) ok = issue_pv(t, j);
          if (ok && t == 0 && j == it.n_kv[0] - 1) ok = prefetch_next_s0();
        }
        if (leader) tc_commit(&v_empty[kv % ST]);
      }
      if (!ok) break;
      if (leader) tc_commit(&q_empty[qb]);
      g_base[0] += it.n_kv[0];
      g_base[1] += it.n_kv[1];
      kv_base += it.n_kv_max;
      pre_s0 = pre_next;
    }
    if (!ok) {
      set_status(status, GPT2_ERR_WAIT_TIMEOUT);
      *abort_flag = 1;
    }
    if (leader) tc_commit(drain);
    mbar_wait_warp(drain, 0, nullptr);
  } else {
    // ---------------- softmax: one thread per query row ----------------
    const int t = (warp - 2) >> 2;  // query tile
    const int qd = warp & 3;        // TMEM lane quarter this warp may access
    const int r = qd * 32 + lane;   // row within the tile
    const uint32_t lane_addr = static_cast<uint32_t>(qd * 32) << 16;
    const uint32_t s_tmem = tmem + lane_addr + kColS + t * 128;
    const uint32_t o_tmem = tmem + lane_addr + kColO + t * 64;
    const uint32_t p_tmem = tmem + lane_addr + kColP + t * 64;
    const float sl2 = 0.125f * 1.4426950408889634f;  // (1/sqrt(64)) * log2(e)
    unsigned char *ostage = sm + Smem2::OST + (t * 4 + qd) * OST_BYTES;
    if (lane == 0) prefetch_tmap(&map_out);
    // A failed wait raises the abort flag; once it is up every later wait
    // returns at once, so the loop runs out without blocking.
    auto wait = [&](uint64_t *bar, uint32_t parity) {
      if (lane == 0 && !mbar_wait(bar, parity, abort_flag, status)) {
        set_status(status, GPT2_ERR_WAIT_TIMEOUT);
        *abort_flag = 1;
      }
      __syncwarp();
    };
    auto arrive = [&](uint64_t *bar) {
      __syncwarp();
      if (lane == 0) mbar_arrive(bar);
    };
    int g_base = 0;  // steps of this tile so far
    for (int w = blockIdx.x; w < n_items; w += gridDim.x) {
      const AttnItem it = attn_item(w, S, B, H, causal, kv_end);
      const int n = it.n_kv[t];
      if (n == 0) continue;
      const int qrow = it.q0 + t * BQ + r;
      const uint8_t *kv_ok = key_valid ? key_valid + (int64_t)it.b * S : nullptr;
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; j < n; ++j) {
        const int g = g_base + j;
        wait(&s_full[t], g & 1);
        tc_fence_after();
        const int kv0 = j * BKV;
        uint32_t sv[128];
        tmem_ld_32x32b_x32(s_tmem, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
        tmem_ld_32x32b_x32(s_tmem + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
        tmem_ld_32x32b_x32(s_tmem + 64, *reinterpret_cast<uint32_t(*)[32]>(&sv[64]));
        tmem_ld_32x32b_x32(s_tmem + 96, *reinterpret_cast<uint32_t(*)[32]>(&sv[96]));
        tc_wait_ld();
        tc_fence_before();
        arrive(&s_free[t]);  // S is in registers: the next Q K^T may overwrite it
        // Masking (raw scores -> -inf) and the row max, 8 independent chains.
        // A tile that touches the causal diagonal or the sequence end, or has
        // a masked key, is masked through a 128-bit keep mask: bit c keeps key
        // kv0 + c.  The mask is the key range [0, lim) of this row ANDed with
        // the key flags, so the per-key work is one bit test and one select.
        const bool diag = causal && j * BKV + BKV > it.q0 + t * BQ;
        const bool tail = j * BKV + BKV > S;
        uint32_t keep[4] = {~0u, ~0u, ~0u, ~0u};
        bool need_mask = diag || tail;
        if (kv_ok) {
          const uint8_t *fp = kv_ok + kv0;
          if (!tail && (reinterpret_cast<uintptr_t>(fp) & 15) == 0) {
            // Warp-uniform: every lane reads the same 128 flags (0 / 1 bytes);
            // x * 0x00204081 >> 21 gathers the low bits of a word's 4 bytes.
            const uint4 *f4 = reinterpret_cast<const uint4 *>(fp);
            uint32_t all = 0x01010101u;
#pragma unroll
            for (int c4 = 0; c4 < 8; ++c4) {
              const uint4 v4 = f4[c4];
              all &= v4.x & v4.y & v4.z & v4.w;
              const uint32_t nib = (((v4.x * 0x00204081u) >> 21) & 0xFu) | ((((v4.y * 0x00204081u) >> 21) & 0xFu) << 4) |
                                   ((((v4.z * 0x00204081u) >> 21) & 0xFu) << 8) |
                                   ((((v4.w * 0x00204081u) >> 21) & 0xFu) << 12);
              if (c4 & 1) keep[c4 >> 1] = (keep[c4 >> 1] & 0xFFFFu) | (nib << 16);
              else keep[c4 >> 1] = nib;
            }
            if (all != 0x01010101u) need_mask = true;
          } else {
            need_mask = true;
#pragma unroll 1
            for (int w4 = 0; w4 < 4; ++w4) {
              uint32_t m = 0;
#pragma unroll 1
              for (int e = 0; e < 32; ++e) {
                const int key = kv0 + w4 * 32 + e;
                m |= static_cast<uint32_t>(key < S && fp[w4 * 32 + e] != 0) << e;
              }
              keep[w4] = m;
            }
          }
        }
        float mx[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mx[e] = -INFINITY;
        if (need_mask) {
          int lim = min(BKV, S - kv0);
          if (causal) lim = min(lim, qrow - kv0 + 1);
#pragma unroll
          for (int w4 = 0; w4 < 4; ++w4) {
            const int lo = w4 * 32;
            keep[w4] &= lim >= lo + 32 ? ~0u : (lim <= lo ? 0u : (1u << (lim - lo)) - 1u);
          }
#pragma unroll
          for (int c = 0; c < 128; ++c) {
            const float x = (keep[c >> 5] >> (c & 31)) & 1u ? __uint_as_float(sv[c]) : -INFINITY;
            sv[c] = __float_as_uint(x);
            mx[c & 7] = fmaxf(mx[c & 7], x);
          }
        } else {
#pragma unroll
          for (int c = 0; c < 128; c += 2)
            mx[(c >> 1) & 7] = max3(mx[(c >> 1) & 7], __uint_as_float(sv[c]), __uint_as_float(sv[c + 1]));
        }
        const float mraw = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                                 fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
        const float mt = mraw * sl2;  // sl2 > 0: the max of the scaled scores
        // Lazy rescale: the running max moves only when it grows by more than
        // the threshold, so the unnormalised terms stay below 2^8.
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
          for (int c = 0; c < 64; c += 16) {
            uint32_t ov[16];
            tmem_ld_32x32b_x16(o_tmem + c, ov);
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * a);
            tmem_st_32x32b_x16(o_tmem + c, ov);
          }
        }
        l_run *= alpha;
        // p = 2^(s * scale * log2e - m): packed pairs for the scale and the sums,
        // bf16 pairs stored into P's TMEM columns 32 at a time.
        const uint64_t sl2x2 = pk2(sl2, sl2), negm2 = pk2(neg_m, neg_m);
        uint64_t rs2[4] = {0, 0, 0, 0};
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          uint32_t pw[16];
#pragma unroll
          for (int e2 = 0; e2 < 16; ++e2) {
            const int c = q4 * 32 + 2 * e2;
            const uint64_t x2 = fma2(pk2(__uint_as_float(sv[c]), __uint_as_float(sv[c + 1])), sl2x2, negm2);
            float x0, x1;
            up2(x2, x0, x1);
            const float p0 = ex2(x0), p1 = ex2(x1);
            rs2[e2 & 3] = add2(rs2[e2 & 3], pk2(p0, p1));
            pw[e2] = pack_bf16x2(p0, p1);
          }
          tmem_st_32x32b_x16(p_tmem + q4 * 16, pw);
        }
        {
          const uint64_t s01 = add2(rs2[0], rs2[1]), s23 = add2(rs2[2], rs2[3]);
          float a0, a1;
          up2(add2(s01, s23), a0, a1);
          l_run += a0 + a1;
        }
        tc_wait_st();  // P (and a rescaled O) are in TMEM before the MMA may read them
        tc_fence_before();
        arrive(&p_full[t]);
      }
      // Epilogue: O / l in bf16, staged in shared memory (128-byte swizzle)
      // and written by one TMA store per warp (32 rows x 64 columns); rows
      // past the sequence end are clipped by the tensor map.
      wait(&o_done[t], (g_base + n - 1) & 1);
      tc_fence_after();
      uint32_t ov[64];
      tmem_ld_32x32b_x32(o_tmem, *reinterpret_cast<uint32_t(*)[32]>(&ov[0]));
      tmem_ld_32x32b_x32(o_tmem + 32, *reinterpret_cast<uint32_t(*)[32]>(&ov[32]));
      tc_wait_ld();
      tc_fence_before();
      if (lane == 0) bulk_wait_read<0>();  // the previous item's store has read the staging rows
      __syncwarp();
      {
        const float inv = l_run > 0.f ? 1.0f / l_run : 0.f;
        unsigned char *row = ostage + lane * 128;
#pragma unroll
        for (int gi = 0; gi < 8; ++gi) {
          const float *f = reinterpret_cast<const float *>(&ov[gi * 8]);
          *reinterpret_cast<uint4 *>(row + ((gi ^ (lane & 7)) << 4)) =
              make_uint4(pack_bf16x2(f[0] * inv, f[1] * inv), pack_bf16x2(f[2] * inv, f[3] * inv),
                         pack_bf16x2(f[4] * inv, f[5] * inv), pack_bf16x2(f[6] * inv, f[7] * inv));
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_3d(&map_out, ostage, it.h * DH, it.q0 + t * BQ + qd * 32, it.b);
        bulk_commit();
      }
      g_base += n;
    }
    if (lane == 0) bulk_wait_all();  // stores complete before the CTA (and its shared memory) goes away
    __syncwarp();
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

cudaError_t launch_attention_tc2(const AttnTcPlan &plan, const uint8_t *key_valid, bf16 *o, int *status,
                                 cudaStream_t st, int causal, const int *kv_end) {
  if (plan.B <= 0 || plan.S <= 0 || plan.H <= 0 || plan.H > 65535 || plan.B > 65535) return cudaErrorInvalidValue;
  if (!o || plan.out != o) return cudaErrorInvalidValue;  // the output descriptor must describe o
  static std::atomic<uint64_t> attr_done{0};
  cudaError_t e = set_smem_once(attention_tc2_kernel, Smem2::ALLOC, attr_done);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int items = ((plan.S + 2 * BQ - 1) / (2 * BQ)) * plan.B * plan.H;
  const int grid = items < sms ? items : sms;
  attention_tc2_kernel<<<grid, NTHREADS, Smem2::ALLOC, st>>>(plan.map_qkv, plan.map_out, key_valid, plan.B, plan.S,
                                                             plan.H, status, causal, kv_end);
  return cudaGetLastError();
}

}  // namespace gpt2
