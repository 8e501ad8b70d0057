// attention_tc3.cu -- BF16 attention on the 5th-generation tensor cores with
// three independent query-tile slots per SM, 64-key blocks, one softmax
// thread per query row and the probabilities P kept in tensor memory (the
// P.V product reads P as its A operand straight from TMEM).  Head dim 64.
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
// Why three slots.  With head dim 64 one exponential stands for 256 FLOPs of
// tensor-core work; the MUFU unit (16 exponentials per clock per SM) needs
// about twice as long for a block as the tensor cores do, so the kernel is
// bound by how busy the softmax warps keep that unit.  A softmax warp spends
// part of every block on its TMEM loads, its row max and its barrier waits,
// when it issues no exponential.  Here every SM sub-partition runs three
// softmax warps, one per slot, and slots never wait for one another: each
// has its own Q buffers, K / V rings, TMEM columns and barriers and walks its
// own list of query tiles, so while one warp is in those phases the other
// two keep the unit busy.
//
// Work.  A pair-unit (batch, head, i) is query tile n_tiles-1-i followed by
// tile i: under the causal mask every pair costs the same number of key
// blocks.  Slot p (CTA c, slot s, p = 3c + s) takes pair-units p, p + P,
// p + 2P, ... with P = 3 * grid; units are numbered batch-head-major, so the
// slots at work at any time cover a window of consecutive (batch, head)s
// whose keys and values stay in L2.
//
// Roles, 480 threads:
//   warps 0-2    one control warp per slot (warp 0 also allocates TMEM): the
//                slot's TMA loads -- Q tiles (two 64-row boxes, double-
//                buffered), K blocks into a 3-stage and V blocks into a
//                2-stage ring (3-D tensor map over qkv [B][S][3D]: keys past
//                the sequence end read as zeros) -- and its MMAs: S = Q K^T
//                (M=128, N=64, K=16 x 4) once the softmax holds the previous S
//                in registers, O (+)= P V (M=128, N=64, K=16 x 4, P from TMEM,
//                V an MN-major shared-memory operand) once the softmax has
//                stored P.  The warp sleeps in one barrier at a time, in a
//                fixed order.  (A single producer and a single MMA warp that
//                polled all three slots were measured to be the bottleneck:
//                each pass over the slots' barriers took longer than a block.)
//   warps 3-14   softmax, four warps per slot (one per TMEM lane quarter),
//                thread = query row: masking, row max, exp2 with the
//                1/8 * log2(e) scale folded in, running sum in FP32, lazy O
//                rescale (only when the running max grows by more than 8 in
//                log2 units), P packed to bf16 pairs and stored into its TMEM
//                columns; the epilogue divides O by the row sum and writes
//                bf16 through the slot's no longer needed Q buffer and a TMA
//                store per warp.
// TMEM (512 columns allocated): S_s [64 s, +64), O_s [192 + 64 s, +64),
// P_s [384 + 32 s, +32) (P: 64 bf16 per row = 32 columns).
// Every barrier wait is bounded; a timeout records status 2 and unwinds.
#include <atomic>

#include "../common.cuh"
#include "../kernels.h"

namespace gpt2 {

namespace {
constexpr int DH = 64, BQ = 128, BK = 64, NSLOT = 3, KST = 3, VST = 2;
constexpr int SOFTMAX_WARPS = 4;  // per slot: one thread per query row
constexpr int NTHREADS = 32 * NSLOT * (1 + SOFTMAX_WARPS);
constexpr int QBYTES = BQ * DH * 2;   // one Q tile: 128 rows x 128 bytes
constexpr int KVBYTES = BK * DH * 2;  // one K or V block: 64 rows x 128 bytes
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr uint32_t kColS = 0, kColO = 192, kColP = 384;

struct SlotBars {
  uint64_t q_full[2], q_empty[2], k_full[KST], v_full[VST];
  uint64_t s_full, s_free, p_full, o_done;
};

struct Smem3 {
  static constexpr int Q = 0;                          // [slot][2] Q tiles (later the output staging)
  static constexpr int K = Q + NSLOT * 2 * QBYTES;     // [slot][KST]
  static constexpr int V = K + NSLOT * KST * KVBYTES;  // [slot][VST]
  static constexpr int BARS = V + NSLOT * VST * KVBYTES;
  static constexpr int DRAIN = BARS + NSLOT * static_cast<int>(sizeof(SlotBars));
  static constexpr int MISC = DRAIN + 8 * NSLOT;
  static constexpr int TOTAL = MISC + 16;
  static constexpr int ALLOC = TOTAL + 1024;
};
static_assert(Smem3::ALLOC <= 227 * 1024, "shared memory");

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 2^x on the FMA pipe, for a pair of inputs: an eighth of the softmax's
// exponentials go here instead of the MUFU unit, which the three slots'
// softmax warps of a sub-partition share (measured: 0.202 -> 0.197 ms at
// B64xS1024; a quarter made the kernel spill and gained less).
// x = n + f with n = round(x) from the 1.5 * 2^23 rounding trick and
// f in [-0.5, 0.5]; 2^f from a cubic fitted here to minimise the relative
// error on that interval (iteratively reweighted least squares,
// max relative error 7.5e-5, far below the bf16 rounding of P); 2^n added to
// the exponent field.  Inputs below -126 (masked keys: -inf) are clamped and
// give at most 2.4e-38 instead of 0, nothing next to a row sum of at least 1.
__device__ __forceinline__ void ex2_fma2(float x0, float x1, float &p0, float &p1) {
  const uint64_t x2 = pk2(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
  const uint64_t t2 = add2(x2, pk2(12582912.f, 12582912.f));
  const uint64_t n2 = add2(t2, pk2(-12582912.f, -12582912.f));
  const uint64_t f2 = fma2(n2, pk2(-1.f, -1.f), x2);
  uint64_t q2 = fma2(pk2(0.05517132f, 0.05517132f), f2, pk2(0.24261054f, 0.24261054f));
  q2 = fma2(q2, f2, pk2(0.69326097f, 0.69326097f));
  q2 = fma2(q2, f2, pk2(0.99992812f, 0.99992812f));
  float q0, q1, t0, t1;
  up2(q2, q0, q1);
  up2(t2, t0, t1);
  // The rounded t = 1.5 * 2^23 + n: its bits shifted left by 23 are n << 23.
  p0 = __int_as_float(__float_as_int(q0) + (__float_as_int(t0) << 23));
  p1 = __int_as_float(__float_as_int(q1) + (__float_as_int(t1) << 23));
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Unsigned division by a divisor fixed for the launch, as a multiply-high
// and shifts (Granlund and Montgomery, "Division by invariant integers using
// multiplication", PLDI 1994, figure 4.1): l = ceil(log2 d),
// m = floor(2^32 (2^l - d) / d) + 1, n / d = (t + ((n - t) >> 1)) >> (l - 1)
// with t = umulhi(m, n), exact for every 32-bit n when d >= 2.  The tile
// walk divides by the pair count and the head count on every tile; as
// integer divisions those cost several hundred clocks per tile.  The
// constants are made on the host and reach the kernel as parameters (made in
// the kernel, the compiler recomputed their 64-bit division wherever it ran
// short of registers).
struct FastDiv {
  uint32_t d, m, l;
};
FastDiv make_fastdiv(uint32_t d) {
  FastDiv f;
  f.d = d;
  uint32_t l = 0;
  while (l < 32 && (1ull << l) < d) ++l;
  f.l = l;
  f.m = static_cast<uint32_t>(((1ull << 32) * ((1ull << l) - d)) / d + 1);
  return f;
}
__device__ __forceinline__ uint32_t fast_div(uint32_t n, const FastDiv &f) {
  if (f.d == 1) return n;
  const uint32_t t = __umulhi(n, f.m);
  return (t + ((n - t) >> 1)) >> (f.l - 1);
}

struct Geo {
  int S, H, n_tiles, n_pairs, n_units, nk_total, causal, P;
  FastDiv div_pairs, div_h;
  const int *kv_end;
};
struct Tile {
  int b, h, qs, n;  // batch, head, first query row, key blocks
};

// The tile walk of one launch (host side; grid CTAs).
Geo make_geo(int B, int S, int H, int causal, const int *kv_end, int grid) {
  Geo g;
  g.S = S;
  g.H = H;
  g.n_tiles = (S + BQ - 1) / BQ;
  g.n_pairs = (g.n_tiles + 1) / 2;
  g.n_units = B * H * g.n_pairs;
  g.nk_total = (S + BK - 1) / BK;
  g.causal = causal;
  g.P = grid * NSLOT;
  g.div_pairs = make_fastdiv(g.n_pairs);
  g.div_h = make_fastdiv(H);
  g.kv_end = kv_end;
  return g;
}
// The slot's next tile after (u, sec): the second tile of the pair, or the
// first of the slot's next pair-unit.
__device__ __forceinline__ void next_tile(const Geo &g, int &u, int &sec) {
  const int i = u - static_cast<int>(fast_div(u, g.div_pairs)) * g.n_pairs;
  if (sec == 0 && g.n_tiles - 1 - i != i) {
    sec = 1;
  } else {
    u += g.P;
    sec = 0;
  }
}
__device__ __forceinline__ Tile tile_of(const Geo &g, int u, int sec) {
  Tile t;
  const int bh = static_cast<int>(fast_div(u, g.div_pairs)), i = u - bh * g.n_pairs;
  t.b = static_cast<int>(fast_div(bh, g.div_h));
  t.h = bh - t.b * g.H;
  t.qs = (sec ? i : g.n_tiles - 1 - i) * BQ;
  int nk = g.nk_total;
  if (g.kv_end) nk = min(nk, max(1, (g.kv_end[t.b] + BK - 1) / BK));
  // Key tiles past the last unmasked key are dropped (at least one is kept so
  // every role sees the same non-empty schedule).
  t.n = g.causal ? min((min(t.qs + BQ, g.S) + BK - 1) / BK, nk) : nk;
  return t;
}

// A position in a slot's list of key blocks: the tile (pair-unit u, sec),
// its block j of n, and the tile's batch, head and first query row.
struct Cursor {
  int u, sec, j, n, b, h, qs;
};
__device__ __forceinline__ void cursor_load(Cursor &c, const Geo &g) {
  if (c.u >= g.n_units) return;
  const Tile t = tile_of(g, c.u, c.sec);
  c.n = t.n;
  c.b = t.b;
  c.h = t.h;
  c.qs = t.qs;
}
__device__ __forceinline__ void cursor_init(Cursor &c, const Geo &g, int p) {
  c.u = p;
  c.sec = c.j = 0;
  c.n = 1;
  c.b = c.h = c.qs = 0;
  cursor_load(c, g);
}
__device__ __forceinline__ bool cursor_valid(const Cursor &c, const Geo &g) { return c.u < g.n_units; }
__device__ __forceinline__ void cursor_next_tile(Cursor &c, const Geo &g) {
  next_tile(g, c.u, c.sec);
  c.j = 0;
  cursor_load(c, g);
}
__device__ __forceinline__ void cursor_next_block(Cursor &c, const Geo &g) {
  if (++c.j == c.n) cursor_next_tile(c, g);
}

__global__ void __launch_bounds__(NTHREADS, 1)
    attention_tc3_kernel(const __grid_constant__ CUtensorMap map_qkv, const __grid_constant__ CUtensorMap map_out,
                         const uint8_t *__restrict__ key_valid, const Geo g, int *status) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char *sm =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  SlotBars *sb = reinterpret_cast<SlotBars *>(sm + Smem3::BARS);
  uint64_t *drain = reinterpret_cast<uint64_t *>(sm + Smem3::DRAIN);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + Smem3::MISC);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(sm + Smem3::MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = g.S, H = g.H, causal = g.causal;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NSLOT; ++s) {
      SlotBars &b = sb[s];
      for (int i = 0; i < 2; ++i) {
        mbar_init(&b.q_full[i], 1);
        mbar_init(&b.q_empty[i], SOFTMAX_WARPS * 32);  // every softmax thread, once its warp's output store has read the buffer
      }
      for (int i = 0; i < KST; ++i) mbar_init(&b.k_full[i], 1);
      for (int i = 0; i < VST; ++i) mbar_init(&b.v_full[i], 1);
      mbar_init(&b.s_full, 1);
      mbar_init(&b.s_free, SOFTMAX_WARPS * 32);
      mbar_init(&b.p_full, SOFTMAX_WARPS * 32);
      mbar_init(&b.o_done, 1);
    }
    for (int s = 0; s < NSLOT; ++s) mbar_init(&drain[s], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < NSLOT) {
    // ---------------- control warp of slot `warp`: its TMA loads and its MMAs ----------------
    // The whole warp waits in each barrier; one elected lane issues.  Fixed
    // order: Q(0), K(0..KST-1), V(0..VST-2), S(0); then for every block g of
    // the slot (blocks run on across its tiles) S(g + 1), P.V(g), K(g + KST)
    // and V(g + VST - 1).  The ring stages those two loads refill need no
    // barrier of their own: K(g + KST) replaces K(g), whose only reader S(g)
    // has completed once the softmax freed S(g) (S(g + 1) waited for that);
    // V(g + VST - 1) replaces V(g - 1), whose only reader P.V(g - 1) has
    // completed once the softmax stored P(g) (it waits for P.V(g - 1) first,
    // and P.V(g) waited for P(g)).  The Q tile of the next tile goes out
    // right after the P.V of a tile's second block (its only block, if it
    // has one): the softmax hands that buffer back (the previous tile's
    // output store has read it) just after that P.
    const int s = warp;
    SlotBars &b = sb[s];
    const bool leader = elect_one_sync();
    if (leader) prefetch_tmap(&map_qkv);
    const int D = H * DH;
    constexpr uint32_t idesc_s = idesc_bf16_f32(128, 64, 0);  // Q K^T: both K-major
    constexpr uint32_t idesc_o = idesc_bf16_f32(128, 64, 1);  // P V: V is MN-major
    unsigned char *q_sm = sm + Smem3::Q + s * 2 * QBYTES;
    unsigned char *k_sm = sm + Smem3::K + s * KST * KVBYTES;
    unsigned char *v_sm = sm + Smem3::V + s * VST * KVBYTES;
    const uint32_t d_s = tmem + kColS + 64 * s, d_o = tmem + kColO + 64 * s, a_p = tmem + kColP + 32 * s;
    const int p0 = blockIdx.x * NSLOT + s;
    // Cursors over the slot's blocks: next Q tile, K, V, S and P.V.
    Cursor qc, kcur, vcur, sc, pc;
    cursor_init(qc, g, p0);
    kcur = vcur = sc = pc = qc;
    int nq = 0, nk = 0, nv = 0, ns = 0, npv = 0, s_tile = 0, pv_tile = 0;
    auto load_q = [&]() -> bool {
      const int qb = nq & 1;
      if (!mbar_wait_warp(&b.q_empty[qb], ((nq >> 1) & 1) ^ 1, abort_flag, status)) return false;
      if (leader) {
        mbar_arrive_expect_tx(&b.q_full[qb], QBYTES);
        tma_load_3d(q_sm + qb * QBYTES, &map_qkv, &b.q_full[qb], qc.h * DH, qc.qs, qc.b);
        tma_load_3d(q_sm + qb * QBYTES + KVBYTES, &map_qkv, &b.q_full[qb], qc.h * DH, qc.qs + BK, qc.b);
      }
      __syncwarp();
      ++nq;
      cursor_next_tile(qc, g);
      return true;
    };
    auto load_k = [&]() -> bool {
      const int st = nk % KST;
      if (leader) {
        mbar_arrive_expect_tx(&b.k_full[st], KVBYTES);
        tma_load_3d(k_sm + st * KVBYTES, &map_qkv, &b.k_full[st], D + kcur.h * DH, kcur.j * BK, kcur.b);
      }
      __syncwarp();
      ++nk;
      cursor_next_block(kcur, g);
      return true;
    };
    auto load_v = [&]() -> bool {
      const int st = nv % VST;
      if (leader) {
        mbar_arrive_expect_tx(&b.v_full[st], KVBYTES);
        tma_load_3d(v_sm + st * KVBYTES, &map_qkv, &b.v_full[st], 2 * D + vcur.h * DH, vcur.j * BK, vcur.b);
      }
      __syncwarp();
      ++nv;
      cursor_next_block(vcur, g);
      return true;
    };
    auto issue_s = [&]() -> bool {
      const int st = ns % KST, qb = s_tile & 1;
      if (sc.j == 0 && !mbar_wait_warp(&b.q_full[qb], (s_tile >> 1) & 1, abort_flag, status)) return false;
      if (!mbar_wait_warp(&b.k_full[st], (ns / KST) & 1, abort_flag, status)) return false;
      if (ns > 0 && !mbar_wait_warp(&b.s_free, (ns - 1) & 1, abort_flag, status)) return false;
      tc_fence_after();
      if (leader) {
        const uint64_t a = sdesc_kmajor_sw128(smem_u32(q_sm + qb * QBYTES));
        const uint64_t bd = sdesc_kmajor_sw128(smem_u32(k_sm + st * KVBYTES));
#pragma unroll
        for (int k = 0; k < DH / 16; ++k) tc_mma_f16(d_s, a + 2 * k, bd + 2 * k, idesc_s, k != 0);
        tc_commit(&b.s_full);
      }
      __syncwarp();
      ++ns;
      if (sc.j + 1 == sc.n) ++s_tile;
      cursor_next_block(sc, g);
      return true;
    };
    auto issue_pv = [&]() -> bool {
      const int st = npv % VST;
      if (!mbar_wait_warp(&b.p_full, npv & 1, abort_flag, status)) return false;
      if (!mbar_wait_warp(&b.v_full[st], (npv / VST) & 1, abort_flag, status)) return false;
      tc_fence_after();
      if (leader) {
        const uint64_t bd = sdesc_mnmajor_sw128(smem_u32(v_sm + st * KVBYTES), KVBYTES, 1024);
        const uint32_t first = pc.j == 0;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          tc_mma_f16_ts(d_o, a_p + k * 8, bd + k * (2048 >> 4), idesc_o, !(first && k == 0));
        tc_commit(&b.o_done);
      }
      __syncwarp();
      ++npv;
      if (pc.j + 1 == pc.n) ++pv_tile;
      cursor_next_block(pc, g);
      return true;
    };
    bool ok = true;
    if (cursor_valid(sc, g)) {
      ok = load_q();
      for (int i = 0; i < KST && ok && cursor_valid(kcur, g); ++i) ok = load_k();
      for (int i = 0; i < VST - 1 && ok && cursor_valid(vcur, g); ++i) ok = load_v();
      if (ok) ok = issue_s();
    }
    while (ok && cursor_valid(pc, g)) {
      // S(g + 1) first, unless it opens a tile whose Q is not loaded yet: that
      // Q waits for the P.V of this (one-block) tile.
      const bool q_first = cursor_valid(sc, g) && sc.j == 0 && s_tile >= nq;
      if (cursor_valid(sc, g) && !q_first) ok = issue_s();
      const int tile_of_pv = pv_tile;
      const bool q_block = pc.j == min(1, pc.n - 1);
      if (ok) ok = issue_pv();
      if (ok && q_block && nq == tile_of_pv + 1 && cursor_valid(qc, g)) ok = load_q();
      if (ok && q_first) ok = issue_s();
      if (ok && cursor_valid(kcur, g)) ok = load_k();
      if (ok && cursor_valid(vcur, g)) ok = load_v();
    }
    if (!ok) {
      set_status(status, GPT2_ERR_WAIT_TIMEOUT);
      *abort_flag = 1;
    }
    // Every product done and every copy landed before the CTA can exit.
    if (leader) tc_commit(&drain[s]);
    mbar_wait_warp(&drain[s], 0, nullptr);
    for (int i = 0; i < 2; ++i) {
      const int cnt = (nq + 1 - i) / 2;  // Q tiles that went into buffer i
      if (cnt) mbar_wait_warp(&b.q_full[i], (cnt - 1) & 1, nullptr);
    }
    for (int i = 0; i < KST; ++i) {
      const int cnt = (nk + KST - 1 - i) / KST;
      if (cnt) mbar_wait_warp(&b.k_full[i], (cnt - 1) & 1, nullptr);
    }
    for (int i = 0; i < VST; ++i) {
      const int cnt = (nv + VST - 1 - i) / VST;
      if (cnt) mbar_wait_warp(&b.v_full[i], (cnt - 1) & 1, nullptr);
    }
  } else {
    // ---------------- softmax: one thread per query row ----------------
    const int s = (warp - NSLOT) >> 2;  // slot
    const int qd = warp & 3;        // TMEM lane quarter this warp may access
    const int r = qd * 32 + lane;   // row within the tile
    const uint32_t lane_addr = static_cast<uint32_t>(qd * 32) << 16;
    const uint32_t s_tmem = tmem + lane_addr + kColS + 64 * s;
    const uint32_t o_tmem = tmem + lane_addr + kColO + 64 * s;
    const uint32_t p_tmem = tmem + lane_addr + kColP + 32 * s;
    const float sl2 = 0.125f * 1.4426950408889634f;  // (1/sqrt(64)) * log2(e)
    SlotBars &bb = sb[s];
    if (lane == 0) prefetch_tmap(&map_out);
    // Every thread waits and arrives itself (the softmax barriers count all
    // 128 threads of the slot): measured 5 % faster than one lane per warp
    // with the warp reconverging around it.  A failed wait raises the abort
    // flag; once it is up every later wait returns at once, so the loop runs
    // out without blocking.
    auto wait = [&](uint64_t *bar, uint32_t parity) {
      if (!mbar_wait(bar, parity, abort_flag, status)) {
        set_status(status, GPT2_ERR_WAIT_TIMEOUT);
        *abort_flag = 1;
      }
    };
    auto arrive = [&](uint64_t *bar) { mbar_arrive(bar); };
    // Output of a finished tile: O / l in bf16, staged (128-byte swizzle) in
    // the tile's Q buffer, whose Q K^T products are all done, and written by
    // one TMA store per warp (32 rows x 64 columns); rows past the sequence
    // end are clipped by the tensor map.  O is read in two 32-column halves.
    auto write_out = [&](float l, int ob, int oh, int oqs, int buf) {
      const float inv = l > 0.f ? 1.0f / l : 0.f;
      unsigned char *ostage = sm + Smem3::Q + (s * 2 + buf) * QBYTES + qd * 32 * 128;
      unsigned char *row = ostage + lane * 128;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t ov[32];
        tmem_ld_32x32b_x32(o_tmem + 32 * half, ov);
        tc_wait_ld();
#pragma unroll
        for (int gi = 0; gi < 4; ++gi) {
          const float *f = reinterpret_cast<const float *>(&ov[gi * 8]);
          const int chunk = half * 4 + gi;
          *reinterpret_cast<uint4 *>(row + ((chunk ^ (lane & 7)) << 4)) =
              make_uint4(pack_bf16x2(f[0] * inv, f[1] * inv), pack_bf16x2(f[2] * inv, f[3] * inv),
                         pack_bf16x2(f[4] * inv, f[5] * inv), pack_bf16x2(f[6] * inv, f[7] * inv));
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_3d(&map_out, ostage, oh * DH, oqs + qd * 32, ob);
        bulk_commit();
      }
      __syncwarp();
    };
    // A tile's output is written during the next tile's first block (after
    // its exponentials, when the tile's last P.V is long done and before that
    // block's P lets the next P.V overwrite O), so the wait for the last P.V
    // hides behind the next tile's work; the slot's last tile is written
    // after the loop.
    bool has_prev = false;
    float prev_l = 0.f;
    int prev_b = 0, prev_h = 0, prev_qs = 0;
    int gb = 0, nt = 0;  // blocks and tiles of this slot so far
    int u = blockIdx.x * NSLOT + s, sec = 0;
    for (; u < g.n_units; next_tile(g, u, sec), ++nt) {
      const Tile t = tile_of(g, u, sec);
      const int qrow = t.qs + r;
      const uint8_t *kv_ok = key_valid ? key_valid + (int64_t)t.b * S : nullptr;
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; j < t.n; ++j, ++gb) {
        const int kv0 = j * BK;
        const bool diag = causal && kv0 + BK > t.qs;
        const bool tail = kv0 + BK > S;
        // keep bit c: key kv0 + c may be attended (key flags only; the key
        // range of the row is ANDed in below).  Read before the wait for S.
        uint32_t keep[2] = {~0u, ~0u};
        bool need_mask = diag || tail;
        if (kv_ok) {
          const uint8_t *fp = kv_ok + kv0;
          if (!tail && (reinterpret_cast<uintptr_t>(fp) & 15) == 0) {
            // Warp-uniform: every lane reads the same 64 flags (0 / 1 bytes);
            // x * 0x00204081 >> 21 gathers the low bits of a word's 4 bytes.
            const uint4 *f4 = reinterpret_cast<const uint4 *>(fp);
            uint32_t all = 0x01010101u;
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) {
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
            for (int w2 = 0; w2 < 2; ++w2) {
              uint32_t m = 0;
#pragma unroll 1
              for (int e = 0; e < 32; ++e) {
                const int key = kv0 + w2 * 32 + e;
                m |= static_cast<uint32_t>(key < S && fp[w2 * 32 + e] != 0) << e;
              }
              keep[w2] = m;
            }
          }
        }
        wait(&bb.s_full, gb & 1);
        tc_fence_after();
        uint32_t sv[64];
        tmem_ld_32x32b_x32(s_tmem, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
        tmem_ld_32x32b_x32(s_tmem + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
        tc_wait_ld();
        tc_fence_before();
        arrive(&bb.s_free);  // S is in registers: the next Q K^T may overwrite it
        // Masking (raw scores -> -inf) and the row max, 8 independent chains.
        float mx[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mx[e] = -INFINITY;
        if (need_mask) {
          int lim = min(BK, S - kv0);
          if (causal) lim = min(lim, qrow - kv0 + 1);
          if (kv_ok) {
            keep[0] &= lim >= 32 ? ~0u : (lim <= 0 ? 0u : (1u << lim) - 1u);
            keep[1] &= lim >= 64 ? ~0u : (lim <= 32 ? 0u : (1u << (lim - 32)) - 1u);
#pragma unroll
            for (int c = 0; c < 64; ++c) {
              const float x = (keep[c >> 5] >> (c & 31)) & 1u ? __uint_as_float(sv[c]) : -INFINITY;
              sv[c] = __float_as_uint(x);
              mx[c & 7] = fmaxf(mx[c & 7], x);
            }
          } else {
            // No key flags: the keys kept are exactly [0, lim).
#pragma unroll
            for (int c = 0; c < 64; ++c) {
              const float x = c < lim ? __uint_as_float(sv[c]) : -INFINITY;
              sv[c] = __float_as_uint(x);
              mx[c & 7] = fmaxf(mx[c & 7], x);
            }
          }
        } else {
#pragma unroll
          for (int c = 0; c < 64; c += 2)
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
        // p = 2^(s * scale * log2e - m): packed pairs for the scale and the
        // sums; P is kept in registers until its TMEM columns are free.
        const uint64_t sl2x2 = pk2(sl2, sl2), negm2 = pk2(neg_m, neg_m);
        uint64_t rs2[4] = {0, 0, 0, 0};
        uint32_t pw[32];
#pragma unroll
        for (int e2 = 0; e2 < 32; ++e2) {
          const uint64_t x2 =
              fma2(pk2(__uint_as_float(sv[2 * e2]), __uint_as_float(sv[2 * e2 + 1])), sl2x2, negm2);
          float x0, x1;
          up2(x2, x0, x1);
          float p0, p1;
          if ((e2 & 7) == 7) {
            ex2_fma2(x0, x1, p0, p1);
          } else {
            p0 = ex2(x0);
            p1 = ex2(x1);
          }
          rs2[e2 & 3] = add2(rs2[e2 & 3], pk2(p0, p1));
          pw[e2] = pack_bf16x2(p0, p1);
        }
        {
          const uint64_t s01 = add2(rs2[0], rs2[1]), s23 = add2(rs2[2], rs2[3]);
          float a0, a1;
          up2(add2(s01, s23), a0, a1);
          l_run = l_run * alpha + (a0 + a1);
        }
        // The previous P.V must be done before P is overwritten and O rescaled
        // (or, at a tile's first block, before O of the previous tile is read).
        if (j > 0 || has_prev) wait(&bb.o_done, (gb - 1) & 1);
        tc_fence_after();
        if (j == 0 && has_prev) write_out(prev_l, prev_b, prev_h, prev_qs, (nt - 1) & 1);
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
        tmem_st_32x32b_x32(p_tmem, pw);
        tc_wait_st();  // P (and a rescaled O) are in TMEM before the MMA may read them
        tc_fence_before();
        arrive(&bb.p_full);
        // The previous tile's output store has read its staging rows by the
        // end of this tile's second block (or of its only one): hand that Q
        // buffer back.  The control warp asks for it only after this P, to
        // load the tile after this one.
        if (j == min(1, t.n - 1) && nt > 0) {
          if (lane == 0) bulk_wait_read<0>();
          arrive(&bb.q_empty[(nt - 1) & 1]);
        }
      }
      has_prev = true;
      prev_l = l_run;
      prev_b = t.b;
      prev_h = t.h;
      prev_qs = t.qs;
    }
    if (has_prev) {
      wait(&bb.o_done, (gb - 1) & 1);
      tc_fence_after();
      write_out(prev_l, prev_b, prev_h, prev_qs, (nt - 1) & 1);
    }
    if (lane == 0) bulk_wait_all();  // stores complete before the CTA (and its shared memory) goes away
    __syncwarp();
  }

  __syncthreads();
  if (warp == 0) {
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
  const cuuint32_t box[3] = {64, 64, 1};  // one K or V block, half a Q tile
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

cudaError_t launch_attention_tc3(const AttnTcPlan &plan, const uint8_t *key_valid, bf16 *o, int *status,
                                 cudaStream_t st, int causal, const int *kv_end) {
  if (plan.B <= 0 || plan.S <= 0 || plan.H <= 0 || plan.H > 65535 || plan.B > 65535) return cudaErrorInvalidValue;
  if (!o || plan.out != o) return cudaErrorInvalidValue;  // the output descriptor must describe o
  const int64_t units = (int64_t)plan.B * plan.H * (((plan.S + BQ - 1) / BQ + 1) / 2);
  if (units > (int64_t)1 << 30) return cudaErrorInvalidValue;  // unit numbers stay far from int overflow
  static std::atomic<uint64_t> attr_done{0};
  cudaError_t e = set_smem_once(attention_tc3_kernel, Smem3::ALLOC, attr_done);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t ctas = (units + NSLOT - 1) / NSLOT;
  const int grid = static_cast<int>(ctas < sms ? ctas : sms);
  const Geo g = make_geo(plan.B, plan.S, plan.H, causal ? 1 : 0, kv_end, grid);
  attention_tc3_kernel<<<grid, NTHREADS, Smem3::ALLOC, st>>>(plan.map_qkv, plan.map_out, key_valid, g, status);
  return cudaGetLastError();
}

}  // namespace gpt2
