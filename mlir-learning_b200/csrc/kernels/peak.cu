// peak.cu -- the FP32 SIMT (FFMA) throughput of this GPU, measured: the
// denominator of the roofline of the exact-FP32 configuration, whose GEMMs
// and attention run on FFMA rather than the tensor cores.
//
// Every thread runs 16 independent FMA chains (enough to cover the FMA
// pipeline's latency with 8 resident blocks of 256 threads per SM) through
// inline PTX, so nothing is folded or reordered away; the chains' sum is
// stored so the work is live.
#include "../common.cuh"
#include "../kernels.h"

namespace gpt2 {

namespace {
constexpr int FFMA_CHAINS = 16, FFMA_THREADS = 256, FFMA_BLOCKS_PER_SM = 8;

__global__ void __launch_bounds__(FFMA_THREADS) ffma_peak_kernel(float *out, int iters, float a, float b) {
  float acc[FFMA_CHAINS];
#pragma unroll
  for (int i = 0; i < FFMA_CHAINS; ++i) acc[i] = threadIdx.x * 1e-3f + i;
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int i = 0; i < FFMA_CHAINS; ++i) asm volatile("fma.rn.f32 %0, %0, %1, %2;" : "+f"(acc[i]) : "f"(a), "f"(b));
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < FFMA_CHAINS; ++i) s += acc[i];
  out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}
}  // namespace

cudaError_t measure_ffma_peak(float *tflops, cudaStream_t st) {
  if (!tflops) return cudaErrorInvalidValue;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  const int blocks = sms * FFMA_BLOCKS_PER_SM, iters = 1 << 16;
  float *out = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  e = cudaMalloc(&out, sizeof(float) * blocks * FFMA_THREADS);
  if (e == cudaSuccess) e = cudaEventCreate(&e0);
  if (e == cudaSuccess) e = cudaEventCreate(&e1);
  float best_ms = 0.f;
  // one warm-up launch, then the best of three
  for (int rep = 0; rep < 4 && e == cudaSuccess; ++rep) {
    cudaEventRecord(e0, st);
    ffma_peak_kernel<<<blocks, FFMA_THREADS, 0, st>>>(out, iters, 0.9999f, 1e-4f);
    cudaEventRecord(e1, st);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaEventSynchronize(e1);
    float ms = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
    if (e == cudaSuccess && rep > 0 && (best_ms == 0.f || ms < best_ms)) best_ms = ms;
  }
  if (e == cudaSuccess)
    *tflops = static_cast<float>(2.0 * FFMA_CHAINS * (double)iters * blocks * FFMA_THREADS / (best_ms * 1e-3) / 1e12);
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  if (out) cudaFree(out);
  return e;
}

}  // namespace gpt2
