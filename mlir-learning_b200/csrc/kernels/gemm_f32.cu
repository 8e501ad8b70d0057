// gemm_f32.cu -- exact-FP32 SIMT GEMM with fused epilogues (bias, gelu_new,
// residual add), the verification path of the GPT-2 forward.
//
// Replaces the reference's linalg.matmul kernels (QKV, attention out-proj,
// MLP fc/proj, lm_head: README.md:11, one thread per output element with a
// sequential K loop) plus the linalg.fill zero-init and the bias / GELU /
// residual generics that follow them.  FP32 FFMA only (no TF32), so the
// result stays within 1e-4 of the CPU lowering's cblas_sgemm
// (lib/ConvertMatMulToBlas.cpp:156-160).
//
// Tiling: 128 x 128 output tile per 256-thread block, K step 8, each thread
// an 8 x 8 sub-tile (two 4-row x two 4-column groups 64 apart, so the
// shared-memory float4 reads are conflict free), register-prefetched double
// buffering of the shared tiles.
#include "../common.cuh"
#include "../kernels.h"

namespace gpt2 {

namespace {
constexpr int BM = 128, BN = 128, BK = 8, NT = 256;

template <int EPI>
__device__ __forceinline__ float apply_epi(float acc, const float *bias, const float *resid, int64_t ridx, int col) {
  if (EPI == EPI_NONE) return acc;
  float v = acc + bias[col];
  if (EPI == EPI_BIAS_GELU) v = gelu_new_exact(v);
  if (EPI == EPI_BIAS_GELU_ERF) v = gelu_erf(v);
  if (EPI == EPI_BIAS_RESID) v = resid[ridx] + v;
  return v;
}

template <int EPI, int BNK>
__global__ void __launch_bounds__(NT) gemm_f32_kernel(const float *__restrict__ A, const float *__restrict__ B,
                                                      float *C, int M, int N, int K, int ldc,
                                                      const float *__restrict__ bias, const float *resid) {
  __shared__ __align__(16) float As[2][BK][BM];
  __shared__ __align__(16) float Bs[2][BK][BN];
  const int tid = threadIdx.x;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;

  // A tile: thread loads A[m0 + tid/2][k0 + (tid&1)*4 .. +3]
  const int a_row = tid >> 1, a_col = (tid & 1) * 4;
  // B tile, [K,N] layout: B[k0 + tid/32][n0 + (tid&31)*4 .. +3]
  // B tile, [N,K] layout: B[n0 + tid/2][k0 + (tid&1)*4 .. +3]
  const int bkn_row = tid >> 5, bkn_col = (tid & 31) * 4;
  const int bnk_row = tid >> 1, bnk_col = (tid & 1) * 4;

  const bool a_ok = m0 + a_row < M;
  const float *a_ptr = A + (int64_t)(a_ok ? m0 + a_row : 0) * K + a_col;
  bool b_ok;
  const float *b_ptr;
  if (BNK) {
    b_ok = n0 + bnk_row < N;
    b_ptr = B + (int64_t)(b_ok ? n0 + bnk_row : 0) * K + bnk_col;
  } else {
    b_ok = n0 + bkn_col < N;  // N % 4 == 0 for this layout
    b_ptr = B + (int64_t)bkn_row * N + (b_ok ? n0 + bkn_col : 0);
  }

  float4 a_reg, b_reg;
  auto load_regs = [&](int k0) {
    a_reg = a_ok ? *reinterpret_cast<const float4 *>(a_ptr + k0) : make_float4(0.f, 0.f, 0.f, 0.f);
    if (BNK) b_reg = b_ok ? *reinterpret_cast<const float4 *>(b_ptr + k0) : make_float4(0.f, 0.f, 0.f, 0.f);
    else b_reg = b_ok ? *reinterpret_cast<const float4 *>(b_ptr + (int64_t)k0 * N) : make_float4(0.f, 0.f, 0.f, 0.f);
  };
  auto store_regs = [&](int buf) {
    As[buf][a_col + 0][a_row] = a_reg.x;
    As[buf][a_col + 1][a_row] = a_reg.y;
    As[buf][a_col + 2][a_row] = a_reg.z;
    As[buf][a_col + 3][a_row] = a_reg.w;
    if (BNK) {
      Bs[buf][bnk_col + 0][bnk_row] = b_reg.x;
      Bs[buf][bnk_col + 1][bnk_row] = b_reg.y;
      Bs[buf][bnk_col + 2][bnk_row] = b_reg.z;
      Bs[buf][bnk_col + 3][bnk_row] = b_reg.w;
    } else {
      *reinterpret_cast<float4 *>(&Bs[buf][bkn_row][bkn_col]) = b_reg;
    }
  };

  const int ty = tid >> 4, tx = tid & 15;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  load_regs(0);
  store_regs(0);
  __syncthreads();
  int buf = 0;
  for (int k0 = 0; k0 < K; k0 += BK) {
    const bool more = k0 + BK < K;
    if (more) load_regs(k0 + BK);
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      float a[8], b[8];
      *reinterpret_cast<float4 *>(&a[0]) = *reinterpret_cast<const float4 *>(&As[buf][k][ty * 4]);
      *reinterpret_cast<float4 *>(&a[4]) = *reinterpret_cast<const float4 *>(&As[buf][k][64 + ty * 4]);
      *reinterpret_cast<float4 *>(&b[0]) = *reinterpret_cast<const float4 *>(&Bs[buf][k][tx * 4]);
      *reinterpret_cast<float4 *>(&b[4]) = *reinterpret_cast<const float4 *>(&Bs[buf][k][64 + tx * 4]);
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (more) {
      store_regs(buf ^ 1);
      __syncthreads();
      buf ^= 1;
    }
  }

  const bool vec_ok = (ldc & 3) == 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int row = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
    if (row >= M) continue;
#pragma unroll
    for (int jg = 0; jg < 2; ++jg) {
      const int col = n0 + jg * 64 + tx * 4;
      const int64_t base = (int64_t)row * ldc + col;
      float v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        v[j] = col + j < N ? apply_epi<EPI>(acc[i][jg * 4 + j], bias, resid, base + j, col + j) : 0.f;
      if (vec_ok && col + 3 < N) {
        *reinterpret_cast<float4 *>(C + base) = make_float4(v[0], v[1], v[2], v[3]);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (col + j < N) C[base + j] = v[j];
      }
    }
  }
}

template <int EPI>
cudaError_t launch_epi(const float *A, const float *B, int b_nk, float *C, int M, int N, int K, int ldc,
                       const float *bias, const float *resid, cudaStream_t st) {
  dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
  if (b_nk) gemm_f32_kernel<EPI, 1><<<grid, NT, 0, st>>>(A, B, C, M, N, K, ldc, bias, resid);
  else gemm_f32_kernel<EPI, 0><<<grid, NT, 0, st>>>(A, B, C, M, N, K, ldc, bias, resid);
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_gemm_f32(const float *A, const float *B, int b_nk, float *C, int M, int N, int K, int ldc,
                            const float *bias, const float *resid, int epi, cudaStream_t st) {
  if (M <= 0 || N <= 0 || K <= 0 || K % BK || ldc < N) return cudaErrorInvalidValue;
  if (!b_nk && N % 4) return cudaErrorInvalidValue;
  if (epi != EPI_NONE && !bias) return cudaErrorInvalidValue;
  if (epi == EPI_BIAS_RESID && !resid) return cudaErrorInvalidValue;
  if (M > 65535 * BM) return cudaErrorInvalidValue;
  switch (epi) {
    case EPI_NONE: return launch_epi<EPI_NONE>(A, B, b_nk, C, M, N, K, ldc, bias, resid, st);
    case EPI_BIAS: return launch_epi<EPI_BIAS>(A, B, b_nk, C, M, N, K, ldc, bias, resid, st);
    case EPI_BIAS_GELU: return launch_epi<EPI_BIAS_GELU>(A, B, b_nk, C, M, N, K, ldc, bias, resid, st);
    case EPI_BIAS_RESID: return launch_epi<EPI_BIAS_RESID>(A, B, b_nk, C, M, N, K, ldc, bias, resid, st);
    case EPI_BIAS_GELU_ERF: return launch_epi<EPI_BIAS_GELU_ERF>(A, B, b_nk, C, M, N, K, ldc, bias, resid, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace gpt2
