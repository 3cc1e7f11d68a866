// AWQ int4 weights kept packed on the device (W4A16), for sm_100a:
//   awq_gemv     decode-sized batches on the CUDA cores, up to 8 rows per
//                launch (the Python dispatcher runs batches of up to 64 rows
//                as 8-row chunks). At that size a layer is weight-bandwidth-
//                bound, and int4 moves a quarter of bf16's bytes.
//   awq_dequant  expands a layer to bf16 [N, K] for the tcgen05 GEMM of
//                prefill-sized batches.
// Layout (AutoAWQ "gemm" packing, the one Hugging Face AWQ checkpoints hold):
//   qweight int32 [K, N/8], qzeros int32 [K/G, N/8], scales fp16 [K/G, N];
//   bits 4i..4i+3 of a word hold output column 8c + {0,2,4,6,1,3,5,7}[i];
//   W[k, n] = (q[k, n] - z[k/G, n]) * s[k/G, n].
// Neither kernel waits on anything: no flags, no cross-CTA dependencies.
#include <cuda_fp16.h>

#include <stdexcept>
#include <string>

#include "../common.cuh"
#include "../kernels.h"

namespace mbx {

namespace {

// the 8 values of one packed word, in natural column order
__device__ __forceinline__ void unpack8(uint32_t w, float (&v)[8]) {
  v[0] = (float)(w & 0xFu);
  v[2] = (float)((w >> 4) & 0xFu);
  v[4] = (float)((w >> 8) & 0xFu);
  v[6] = (float)((w >> 12) & 0xFu);
  v[1] = (float)((w >> 16) & 0xFu);
  v[3] = (float)((w >> 20) & 0xFu);
  v[5] = (float)((w >> 24) & 0xFu);
  v[7] = (float)((w >> 28) & 0xFu);
}

constexpr int kGemvThreads = 64;  // packed columns (512 outputs) per CTA

// One CTA: one quantization group (G rows of k) x 64 packed columns. Per group
// sum_k x[m,k] * (q - z) * s = s * (sum_k x[m,k] q[k] - z * sum_k x[m,k]),
// so the inner loop is 8 FMAs per row per packed word. Partial sums of each
// group go to ws[g, m, n] (fp32), folded in order by awq_reduce_kernel.
template <int M>
__global__ void __launch_bounds__(kGemvThreads) awq_gemv_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ldx, const uint32_t* __restrict__ qw,
    const uint32_t* __restrict__ qz, const __half* __restrict__ sc, float* __restrict__ ws, int N, int G) {
  extern __shared__ float xs[];  // [M][G] activations of this group
  __shared__ float sumx[M];
  const int Nq = N / 8;
  const int g = blockIdx.y;
  const int c = blockIdx.x * kGemvThreads + threadIdx.x;
  const int64_t k0 = (int64_t)g * G;
  for (int i = threadIdx.x; i < M * G; i += blockDim.x) {
    const int m = i / G, k = i % G;
    xs[i] = __bfloat162float(x[m * ldx + k0 + k]);
  }
  __syncthreads();
  if (threadIdx.x < M) {
    float s = 0.f;
    for (int k = 0; k < G; ++k) s += xs[threadIdx.x * G + k];
    sumx[threadIdx.x] = s;
  }
  __syncthreads();
  if (c >= Nq) return;
  float acc[M][8];
#pragma unroll
  for (int m = 0; m < M; ++m)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[m][j] = 0.f;
  const uint32_t* wp = qw + k0 * Nq + c;
  // 8 rows of k per step, their loads issued before any is used: 8 loads in
  // flight per thread (G is a multiple of 8)
#pragma unroll 1
  for (int k = 0; k < G; k += 8) {
    uint32_t wv[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) wv[u] = __ldg(wp + (int64_t)(k + u) * Nq);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      float q[8];
      unpack8(wv[u], q);
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const float xv = xs[m * G + k + u];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[m][j] = fmaf(xv, q[j], acc[m][j]);
      }
    }
  }
  float z[8];
  unpack8(__ldg(qz + (int64_t)g * Nq + c), z);
  const uint4 sv = __ldg(reinterpret_cast<const uint4*>(sc + (int64_t)g * N + 8 * c));
  const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
  float sf[8];
#pragma unroll
  for (int j = 0; j < 8; ++j)  // halves j = 2i (low) and 2i + 1 (high) of word i
    sf[j] = __half2float(__ushort_as_half((unsigned short)(sw[j / 2] >> (16 * (j % 2)))));
#pragma unroll
  for (int m = 0; m < M; ++m) {
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = sf[j] * (acc[m][j] - z[j] * sumx[m]);
    float4* dst = reinterpret_cast<float4*>(ws + ((int64_t)g * M + m) * N + 8 * c);
    dst[0] = make_float4(o[0], o[1], o[2], o[3]);
    dst[1] = make_float4(o[4], o[5], o[6], o[7]);
  }
}

// out[m, n] = bf16(sum_g ws[g, m, n]) (+ residual[m, n], a second rounding,
// like the GEMM's residual epilogue). out may alias residual.
__global__ void awq_reduce_kernel(const float* __restrict__ ws, int groups, int M, int N,
                                  const __nv_bfloat16* residual, __nv_bfloat16* out, int64_t ldo) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t MN = (int64_t)M * N;
  if (i >= MN) return;
  float s = 0.f;
  for (int g = 0; g < groups; ++g) s += ws[(int64_t)g * MN + i];
  const int64_t m = i / N, n = i % N;
  if (residual != nullptr)
    s = __bfloat162float(__float2bfloat16(s)) + __bfloat162float(residual[m * ldo + n]);
  out[m * ldo + n] = __float2bfloat16(s);
}

// bf16 [N, K] from the packed layout. A CTA transposes a tile of 64 rows of k
// x 32 packed columns through shared memory, so the int32 reads (along the
// packed columns) and the bf16 writes (along k) are both coalesced.
constexpr int kDqK = 64, kDqC = 32, kDqThreads = 256;

__global__ void __launch_bounds__(kDqThreads) awq_dequant_kernel(
    const uint32_t* __restrict__ qw, const uint32_t* __restrict__ qz, const __half* __restrict__ sc,
    __nv_bfloat16* __restrict__ out, int K, int N, int G) {
  __shared__ uint32_t tile[kDqK][kDqC + 1];
  const int Nq = N / 8;
  const int c0 = blockIdx.x * kDqC, k0 = blockIdx.y * kDqK;
  for (int r = 0; r < kDqK * kDqC / kDqThreads; ++r) {
    const int kk = threadIdx.x / kDqC + (kDqThreads / kDqC) * r, cc = threadIdx.x % kDqC;
    const int k = k0 + kk, c = c0 + cc;
    tile[kk][cc] = (k < K && c < Nq) ? __ldg(qw + (int64_t)k * Nq + c) : 0u;
  }
  __syncthreads();
  const int kk = threadIdx.x % kDqK, k = k0 + kk;
  if (k >= K) return;
  const int g = k / G;
  for (int r = 0; r < kDqC / (kDqThreads / kDqK); ++r) {
    const int cc = threadIdx.x / kDqK + (kDqThreads / kDqK) * r, c = c0 + cc;
    if (c >= Nq) break;
    float q[8], z[8];
    unpack8(tile[kk][cc], q);
    unpack8(__ldg(qz + (int64_t)g * Nq + c), z);
    const __half* s = sc + (int64_t)g * N + 8 * c;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      out[(int64_t)(8 * c + j) * K + k] = __float2bfloat16((q[j] - z[j]) * __half2float(s[j]));
  }
}

template <int M>
void gemv_launch(const AwqGemvArgs& a, cudaStream_t s) {
  const int Nq = a.N / 8;
  dim3 grid((Nq + kGemvThreads - 1) / kGemvThreads, a.K / a.G);
  awq_gemv_kernel<M><<<grid, kGemvThreads, M * a.G * sizeof(float), s>>>(
      (const __nv_bfloat16*)a.x, a.ldx, (const uint32_t*)a.qweight, (const uint32_t*)a.qzeros,
      (const __half*)a.scales, a.ws, a.N, a.G);
}

}  // namespace

void awq_gemv_launch(const AwqGemvArgs& a, cudaStream_t s) {
  if (a.M < 1 || a.M > kAwqGemvMaxRows) throw std::runtime_error("awq_gemv: 1..8 rows");
  if (a.N % 8 || a.G <= 0 || a.G > 256 || a.G % 8 || a.K % a.G)
    throw std::runtime_error("awq_gemv: unsupported shape");
  switch (a.M) {
    case 1: gemv_launch<1>(a, s); break;
    case 2: gemv_launch<2>(a, s); break;
    case 3: gemv_launch<3>(a, s); break;
    case 4: gemv_launch<4>(a, s); break;
    case 5: gemv_launch<5>(a, s); break;
    case 6: gemv_launch<6>(a, s); break;
    case 7: gemv_launch<7>(a, s); break;
    default: gemv_launch<8>(a, s); break;
  }
  MBX_CUDA_CHECK(cudaGetLastError());
  const int64_t MN = (int64_t)a.M * a.N;
  awq_reduce_kernel<<<(unsigned)((MN + 255) / 256), 256, 0, s>>>(a.ws, a.K / a.G, a.M, a.N,
                                                                  (const __nv_bfloat16*)a.residual,
                                                                  (__nv_bfloat16*)a.out, a.ldo);
  MBX_CUDA_CHECK(cudaGetLastError());
}

void awq_dequant_launch(const void* qweight, const void* qzeros, const void* scales, void* out, int K, int N, int G,
                        cudaStream_t s) {
  if (N % 8 || G <= 0 || K % G) throw std::runtime_error("awq_dequant: unsupported shape");
  const int Nq = N / 8;
  dim3 grid((Nq + kDqC - 1) / kDqC, (K + kDqK - 1) / kDqK);
  awq_dequant_kernel<<<grid, kDqThreads, 0, s>>>((const uint32_t*)qweight, (const uint32_t*)qzeros,
                                                 (const __half*)scales, (__nv_bfloat16*)out, K, N, G);
  MBX_CUDA_CHECK(cudaGetLastError());
}

}  // namespace mbx
