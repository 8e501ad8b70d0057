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
// Tiling: a 128 x BN output tile (BN = 128 or 64) per 256-thread block, K
// step 16, two blocks per SM.  The 8 warps sit 2 (M) x 4 (N), a warp covers
// 64 x BN/4 and a thread 8 x TN (TN = BN / 16) in groups of 4 rows 32 apart
// and 4 columns 16 apart, so the shared-memory float4 reads of one k are 2
// (A) + TN/4 (B) conflict-free wavefronts per warp.  Operands are staged
// through registers into K-outer shared tiles (A and [N, K] B transposed on
// the way), double-buffered with one barrier per K step.  Every output is a
// single fmaf chain over k = 0 .. K-1 in order, whatever the tile shape, so a
// row's result does not depend on how many rows the call has.
//
// BN = 64 is used when 128-wide tiles would leave the last wave of blocks
// mostly empty (narrow N: the d x d and ff x d products of a few thousand
// tokens), since both shapes give identical results.
#include "../common.cuh"
#include "../kernels.h"

namespace gpt2 {

namespace {
constexpr int BM = 128, BK = 16, NT = 256;
constexpr int APAD = 4;  // As row stride BM + 4 floats: the transposing stores hit 2 banks-ways, not 4

template <int EPI>
__device__ __forceinline__ float apply_epi(float acc, const float *bias, const float *resid, int64_t ridx, int col) {
  if (EPI == EPI_NONE) return acc;
  float v = acc + bias[col];
  if (EPI == EPI_BIAS_GELU) v = gelu_new_exact(v);
  if (EPI == EPI_BIAS_GELU_ERF) v = gelu_erf(v);
  if (EPI == EPI_BIAS_RESID) v = resid[ridx] + v;
  return v;
}

template <int EPI, int BNK, int BN>
__global__ void __launch_bounds__(NT, 2) gemm_f32_kernel(const float *__restrict__ A, const float *__restrict__ B,
                                                         float *C, int M, int N, int K, int ldc,
                                                         const float *__restrict__ bias, const float *resid) {
  constexpr int TN = BN / 16;       // columns per thread: 8 or 4
  constexpr int BSTRIDE = BN + 4;   // Bs row stride (floats)
  constexpr int A_LD = BM * BK / 4 / NT;            // float4 loads of A per thread per K step: 2
  constexpr int B_LD = BN * BK / 4 / NT;            // of B: 2 (BN 128) or 1 (BN 64)
  __shared__ __align__(16) float As[2][BK][BM + APAD];
  __shared__ __align__(16) float Bs[2][BK][BSTRIDE];
  const int tid = threadIdx.x;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;

  // Staging: float4 f = tid + NT * r of a tile.  A (and [N, K] B): row f / 4,
  // k (f % 4) * 4 -- four threads read one row's 16 k values (64 bytes).
  // [K, N] B: k f / (BN / 4), column (f % (BN / 4)) * 4.
  float4 a_reg[A_LD], b_reg[B_LD];
  auto load_regs = [&](int k0) {
#pragma unroll
    for (int r = 0; r < A_LD; ++r) {
      const int f = tid + NT * r, row = m0 + f / 4, k = k0 + (f % 4) * 4;
      a_reg[r] = row < M && k < K ? *reinterpret_cast<const float4 *>(A + (int64_t)row * K + k)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int r = 0; r < B_LD; ++r) {
      const int f = tid + NT * r;
      if (BNK) {
        const int col = n0 + f / 4, k = k0 + (f % 4) * 4;
        b_reg[r] = col < N && k < K ? *reinterpret_cast<const float4 *>(B + (int64_t)col * K + k)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
      } else {
        const int k = k0 + f / (BN / 4), col = n0 + (f % (BN / 4)) * 4;  // N % 4 == 0 for this layout
        b_reg[r] = col < N && k < K ? *reinterpret_cast<const float4 *>(B + (int64_t)k * N + col)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  };
  auto store_regs = [&](int buf) {
#pragma unroll
    for (int r = 0; r < A_LD; ++r) {
      const int f = tid + NT * r, row = f / 4, k = (f % 4) * 4;
      As[buf][k + 0][row] = a_reg[r].x;
      As[buf][k + 1][row] = a_reg[r].y;
      As[buf][k + 2][row] = a_reg[r].z;
      As[buf][k + 3][row] = a_reg[r].w;
    }
#pragma unroll
    for (int r = 0; r < B_LD; ++r) {
      const int f = tid + NT * r;
      if (BNK) {
        const int col = f / 4, k = (f % 4) * 4;
        Bs[buf][k + 0][col] = b_reg[r].x;
        Bs[buf][k + 1][col] = b_reg[r].y;
        Bs[buf][k + 2][col] = b_reg[r].z;
        Bs[buf][k + 3][col] = b_reg[r].w;
      } else {
        *reinterpret_cast<float4 *>(&Bs[buf][f / (BN / 4)][(f % (BN / 4)) * 4]) = b_reg[r];
      }
    }
  };

  // This thread's rows: wm * 64 + g * 32 + lm * 4 + i (g < 2, i < 4); its
  // columns: wn * (BN / 4) + h * 16 + ln * 4 + j (h < TN / 4, j < 4).
  const int warp = tid >> 5, lane = tid & 31;
  const int wm = warp >> 2, wn = warp & 3, lm = lane >> 2, ln = lane & 3;
  const int row_base = wm * 64 + lm * 4, col_base = wn * (BN / 4) + ln * 4;
  float acc[8][TN];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

  load_regs(0);
  store_regs(0);
  __syncthreads();
  int buf = 0;
  for (int k0 = 0; k0 < K; k0 += BK) {
    const bool more = k0 + BK < K;
    if (more) load_regs(k0 + BK);
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      float a[8], b[TN];
      *reinterpret_cast<float4 *>(&a[0]) = *reinterpret_cast<const float4 *>(&As[buf][k][row_base]);
      *reinterpret_cast<float4 *>(&a[4]) = *reinterpret_cast<const float4 *>(&As[buf][k][row_base + 32]);
#pragma unroll
      for (int h = 0; h < TN / 4; ++h)
        *reinterpret_cast<float4 *>(&b[4 * h]) = *reinterpret_cast<const float4 *>(&Bs[buf][k][col_base + 16 * h]);
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
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
    const int row = m0 + row_base + (i >> 2) * 32 + (i & 3);
    if (row >= M) continue;
#pragma unroll
    for (int h = 0; h < TN / 4; ++h) {
      const int col = n0 + col_base + 16 * h;
      const int64_t base = (int64_t)row * ldc + col;
      float v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        v[j] = col + j < N ? apply_epi<EPI>(acc[i][4 * h + j], bias, resid, base + j, col + j) : 0.f;
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

// Fraction of the block slots of the last wave that hold a tile.
double wave_fill(int64_t tiles, int64_t slots) {
  const int64_t waves = (tiles + slots - 1) / slots;
  return static_cast<double>(tiles) / static_cast<double>(waves * slots);
}

template <int EPI>
cudaError_t launch_epi(const float *A, const float *B, int b_nk, float *C, int M, int N, int K, int ldc,
                       const float *bias, const float *resid, cudaStream_t st) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t mb = (M + BM - 1) / BM, slots = 2LL * sms;
  const bool narrow = wave_fill(mb * ((N + 127) / 128), slots) < 0.8 &&
                      wave_fill(mb * ((N + 63) / 64), slots) > wave_fill(mb * ((N + 127) / 128), slots);
  if (narrow) {
    dim3 grid((N + 63) / 64, mb);
    if (b_nk) gemm_f32_kernel<EPI, 1, 64><<<grid, NT, 0, st>>>(A, B, C, M, N, K, ldc, bias, resid);
    else gemm_f32_kernel<EPI, 0, 64><<<grid, NT, 0, st>>>(A, B, C, M, N, K, ldc, bias, resid);
  } else {
    dim3 grid((N + 127) / 128, mb);
    if (b_nk) gemm_f32_kernel<EPI, 1, 128><<<grid, NT, 0, st>>>(A, B, C, M, N, K, ldc, bias, resid);
    else gemm_f32_kernel<EPI, 0, 128><<<grid, NT, 0, st>>>(A, B, C, M, N, K, ldc, bias, resid);
  }
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_gemm_f32(const float *A, const float *B, int b_nk, float *C, int M, int N, int K, int ldc,
                            const float *bias, const float *resid, int epi, cudaStream_t st) {
  if (M <= 0 || N <= 0 || K <= 0 || K % 8 || ldc < N) return cudaErrorInvalidValue;
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
