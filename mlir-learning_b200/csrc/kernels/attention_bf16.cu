// attention_bf16.cu -- BF16 fused causal attention (online softmax, FP32
// statistics) for head dim 64.
//
// Replaces, per layer, the reference's q k^T and p v linalg.batch_matmul
// launches plus the scale / causal where / additive mask / softmax generics
// (src/gpt/README.md:6, lib/DeadArgmaxElimination.cpp:4-6) in the BF16
// configuration; the S x S scores never reach memory.
//
// Semantics match attention_f32.cu (key k attendable from q iff k <= q and
// mask[b, k] != 0; rows without an attendable key are finished by
// attn_masked_rows_kernel).  P is rounded to bf16 before the P.V product;
// the running max / sum are FP32; exponentials use exp2 with log2(e) folded
// into the 1/8 scale.
//
// Block: 64 queries of one (batch, head), 4 warps x 16 query rows, K/V
// tiles of 64 keys double-buffered in shared memory with cp.async (rows of
// 128 bytes, 16-byte chunks XOR-swizzled by row so ldmatrix is conflict
// free), warp-level m16n8k16 BF16 MMAs.
#include "../common.cuh"
#include "../kernels.h"

namespace gpt2 {

namespace {
constexpr int DH = 64, BQ = 64, BKV = 64, NT = 128;

__device__ __forceinline__ uint32_t swz(int row, int chunk) {  // byte offset inside a [64][64] bf16 tile
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(NT) attention_bf16_kernel(const bf16 *__restrict__ qkv,
                                                            const uint8_t *__restrict__ key_valid,
                                                            bf16 *__restrict__ o, int S, int H, int causal) {
  __shared__ __align__(128) unsigned char sq[BQ * DH * 2];
  __shared__ __align__(128) unsigned char sk[2][BKV * DH * 2];
  __shared__ __align__(128) unsigned char sv[2][BKV * DH * 2];

  const int nqb = (S + BQ - 1) / BQ;
  const int qb = nqb - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int D = H * DH;
  const int64_t ld = 3 * (int64_t)D;
  const bf16 *base = qkv + (int64_t)b * S * ld;
  const uint8_t *kv_ok = key_valid ? key_valid + (int64_t)b * S : nullptr;
  const int q0 = qb * BQ;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;

  auto load_tile = [&](unsigned char *dst, int row0, int col_off) {
#pragma unroll
    for (int i = 0; i < (BKV * 8) / NT; ++i) {
      const int idx = tid + i * NT;
      const int r = idx >> 3, c = idx & 7;
      const bool valid = row0 + r < S;
      const bf16 *src = base + (int64_t)(valid ? row0 + r : 0) * ld + col_off + c * 8;
      cp_async16(smem_u32(dst) + swz(r, c), src, valid);
    }
  };

  load_tile(sq, q0, h * DH);
  load_tile(sk[0], 0, D + h * DH);
  load_tile(sv[0], 0, 2 * D + h * DH);
  cp_async_commit();

  const int n_tiles = causal ? qb + 1 : (S + BKV - 1) / BKV;  // causal: key tiles 0..qb
  uint32_t qf[4][4];
  float oacc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) oacc[i][j] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const float sl2 = 0.125f * 1.4426950408889634f;  // (1/sqrt(64)) * log2(e)

  for (int it = 0; it < n_tiles; ++it) {
    const int cur = it & 1;
    if (it + 1 < n_tiles) {
      load_tile(sk[cur ^ 1], (it + 1) * BKV, D + h * DH);
      load_tile(sv[cur ^ 1], (it + 1) * BKV, 2 * D + h * DH);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (it == 0) {
      // Q fragments for this warp's 16 rows, all 64 columns.
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = kk * 2 + (lane >> 4);
        ldsm_x4(smem_u32(sq) + swz(r, c), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    const int kv0 = it * BKV;

    // S = Q K^T for 16 rows x 64 keys (8 n-tiles of 8 keys).
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
      uint32_t k0, k1, k2, k3, k4, k5, k6, k7;
      const int r = j * 8 + (lane & 7);
      ldsm_x4(smem_u32(sk[cur]) + swz(r, (lane >> 3)), k0, k1, k2, k3);
      ldsm_x4(smem_u32(sk[cur]) + swz(r, 4 + (lane >> 3)), k4, k5, k6, k7);
      mma_bf16(s[j], qf[0], k0, k1);
      mma_bf16(s[j], qf[1], k2, k3);
      mma_bf16(s[j], qf[2], k4, k5);
      mma_bf16(s[j], qf[3], k6, k7);
    }

    // Masking: causal only on the diagonal tile; key validity everywhere.
    const bool diag = causal && it == qb;
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kv0 + j * 8 + 2 * t + (e & 1);
        const int row = q0 + warp * 16 + g + (e >> 1) * 8;
        bool ok = key < S && (!kv_ok || kv_ok[key]);
        if (diag) ok = ok && key <= row;
        s[j][e] = ok ? s[j][e] * sl2 : -INFINITY;
      }

    // Online softmax (rows g and g+8 of the warp's 16).
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      float mt = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; ++j) mt = fmaxf(mt, fmaxf(s[j][2 * hr], s[j][2 * hr + 1]));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
      const float m_new = fmaxf(m_run[hr], mt);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = fast_exp2(m_run[hr] - m_use);
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        s[j][2 * hr] = fast_exp2(s[j][2 * hr] - m_use);
        s[j][2 * hr + 1] = fast_exp2(s[j][2 * hr + 1] - m_use);
        rs += s[j][2 * hr] + s[j][2 * hr + 1];
      }
      rs += __shfl_xor_sync(0xffffffffu, rs, 1);
      rs += __shfl_xor_sync(0xffffffffu, rs, 2);
      l_run[hr] = l_run[hr] * alpha + rs;
      m_run[hr] = m_new;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        oacc[j][2 * hr] *= alpha;
        oacc[j][2 * hr + 1] *= alpha;
      }
    }

    // O += P V: P as bf16 A fragments (16 rows x 64 keys = 4 k-steps).
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {  // pairs of 8-column output tiles
        uint32_t v0, v1, v2, v3;
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = jj * 2 + (lane >> 4);
        ldsm_x4_t(smem_u32(sv[cur]) + swz(r, c), v0, v1, v2, v3);
        mma_bf16(oacc[2 * jj], pa, v0, v1);
        mma_bf16(oacc[2 * jj + 1], pa, v2, v3);
      }
    }
    __syncthreads();
  }

#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int row = q0 + warp * 16 + g + hr * 8;
    if (row >= S) continue;
    const float inv = l_run[hr] > 0.f ? 1.0f / l_run[hr] : 0.f;
    bf16 *op = o + ((int64_t)b * S + row) * D + h * DH;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<uint32_t *>(op + j * 8 + 2 * t) = pack_bf16x2(oacc[j][2 * hr] * inv, oacc[j][2 * hr + 1] * inv);
  }
}
}  // namespace

cudaError_t launch_attention_bf16(const bf16 *qkv, const uint8_t *key_valid, bf16 *o, int B, int S, int H,
                                  cudaStream_t st, int causal) {
  if (B <= 0 || S <= 0 || H <= 0 || H > 65535 || B > 65535) return cudaErrorInvalidValue;
  dim3 grid((S + BQ - 1) / BQ, H, B);
  attention_bf16_kernel<<<grid, NT, 0, st>>>(qkv, key_valid, o, S, H, causal);
  return cudaGetLastError();
}

}  // namespace gpt2
