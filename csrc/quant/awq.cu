// AWQ int4 weights kept packed on the device (W4A16), for sm_100a:
//   awq_gemv     decode-sized batches on the CUDA cores, up to 8 rows per
//                launch (the Python dispatcher runs small batches as 8-row
//                chunks). At that size a layer is weight-bandwidth-bound, and
//                int4 moves a quarter of bf16's bytes.
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

// GEMV CTA: kGemvCols packed columns (8 outputs each) x kGemvSplit slices of
// one quantization group's rows. A thread owns one packed column of one slice
// (G / kGemvSplit rows), so a group's weight column is read by kGemvSplit
// threads at once; the slices meet in shared memory at the end.
constexpr int kGemvCols = 64;
constexpr int kGemvSplit = 4;
constexpr int kGemvThreads = kGemvCols * kGemvSplit;
constexpr int kGemvBatch = 16;  // weight loads in flight per thread

// Dynamic shared memory of the GEMV: activations [M][G] + the partial sums of
// slices 1.. [kGemvSplit - 1][M][8][kGemvCols].
constexpr int gemv_smem_bytes(int M, int G) { return (M * G + (kGemvSplit - 1) * M * 8 * kGemvCols) * 4; }

// One CTA: one quantization group (G rows of k) x kGemvCols packed columns.
// Per group sum_k x[m,k] * (q - z) * s = s * (sum_k x[m,k] q[k] - z * sum_k
// x[m,k]), so the inner loop is 8 FMAs per row per packed word. The first
// batch of weight loads is issued before the activations are staged, and the
// next batch before the current one is used. Partial sums of each group go to
// ws[g, m, n] (fp32), folded by awq_reduce_kernel.
template <int M>
__global__ void __launch_bounds__(kGemvThreads) awq_gemv_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ldx, const uint32_t* __restrict__ qw,
    const uint32_t* __restrict__ qz, const __half* __restrict__ sc, float* __restrict__ ws, int N, int G) {
  extern __shared__ float smem[];
  float* xs = smem;          // [M][G]
  float* red = smem + M * G;  // [kGemvSplit - 1][M][8][kGemvCols]
  __shared__ float sumx[M];
  const int Nq = N / 8;
  const int g = blockIdx.y;
  const int col = threadIdx.x % kGemvCols, part = threadIdx.x / kGemvCols;
  const int c = blockIdx.x * kGemvCols + col;
  const bool live = c < Nq;
  const int64_t k0 = (int64_t)g * G;
  const int R = G / kGemvSplit;  // rows of this slice (a multiple of 8)
  const int kr = part * R;
  const uint32_t* wp = qw + (k0 + kr) * Nq + (live ? c : 0);
  uint32_t wv[kGemvBatch];
#pragma unroll
  for (int u = 0; u < kGemvBatch; ++u) wv[u] = (live && u < R) ? __ldg(wp + (int64_t)u * Nq) : 0u;
  pdl_wait();  // the weights do not depend on earlier kernels; the activations do
  for (int i = threadIdx.x; i < M * G; i += blockDim.x) {
    const int m = i / G, k = i % G;
    xs[i] = __bfloat162float(x[m * ldx + k0 + k]);
  }
  __syncthreads();
  {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp < M) {
      float sx = 0.f;
      for (int k = lane; k < G; k += 32) sx += xs[warp * G + k];
      sx = warp_sum(sx);
      if (lane == 0) sumx[warp] = sx;
    }
  }
  float acc[M][8];
#pragma unroll
  for (int m = 0; m < M; ++m)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[m][j] = 0.f;
#pragma unroll 1
  for (int r0 = 0; r0 < R; r0 += kGemvBatch) {
    uint32_t nv[kGemvBatch];
    const bool more = r0 + kGemvBatch < R;
    if (more) {
#pragma unroll
      for (int u = 0; u < kGemvBatch; ++u) {
        const int r = r0 + kGemvBatch + u;
        nv[u] = (live && r < R) ? __ldg(wp + (int64_t)r * Nq) : 0u;
      }
    }
#pragma unroll
    for (int u = 0; u < kGemvBatch; ++u) {
      if (r0 + u < R) {
        float q[8];
        unpack8(wv[u], q);
#pragma unroll
        for (int m = 0; m < M; ++m) {
          const float xv = xs[m * G + kr + r0 + u];
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[m][j] = fmaf(xv, q[j], acc[m][j]);
        }
      }
    }
    if (more) {
#pragma unroll
      for (int u = 0; u < kGemvBatch; ++u) wv[u] = nv[u];
    }
  }
  if (part > 0) {
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int j = 0; j < 8; ++j) red[(((part - 1) * M + m) * 8 + j) * kGemvCols + col] = acc[m][j];
  }
  __syncthreads();
  if (part != 0 || !live) return;
  for (int p = 1; p < kGemvSplit; ++p)
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[m][j] += red[(((p - 1) * M + m) * 8 + j) * kGemvCols + col];
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
// like the GEMM's residual epilogue). out may alias residual. A CTA folds 32
// outputs: kRedSlices threads per output take the groups g = slice, slice +
// kRedSlices, ... (independent loads in flight), then the slices meet in
// shared memory in slice order.
constexpr int kRedOut = 32, kRedSlices = 8;
__global__ void __launch_bounds__(kRedOut * kRedSlices) awq_reduce_kernel(
    const float* __restrict__ ws, int groups, int M, int N, const __nv_bfloat16* residual, __nv_bfloat16* out,
    int64_t ldo) {
  pdl_wait();
  __shared__ float part[kRedSlices][kRedOut];
  const int o = threadIdx.x % kRedOut, sl = threadIdx.x / kRedOut;
  const int64_t i = (int64_t)blockIdx.x * kRedOut + o;
  const int64_t MN = (int64_t)M * N;
  float s = 0.f;
  if (i < MN) {
#pragma unroll 4
    for (int g = sl; g < groups; g += kRedSlices) s += ws[(int64_t)g * MN + i];
  }
  part[sl][o] = s;
  __syncthreads();
  if (sl != 0 || i >= MN) return;
  for (int k = 1; k < kRedSlices; ++k) s += part[k][o];
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
  static SmemLimit limit;
  const int Nq = a.N / 8;
  const int bytes = gemv_smem_bytes(M, a.G);
  if (bytes > 48 * 1024) limit.ensure((const void*)awq_gemv_kernel<M>, gemv_smem_bytes(M, 256));
  dim3 grid((Nq + kGemvCols - 1) / kGemvCols, a.K / a.G);
  launch_k(awq_gemv_kernel<M>, grid, dim3(kGemvThreads), bytes, s, (const __nv_bfloat16*)a.x, a.ldx,
           (const uint32_t*)a.qweight, (const uint32_t*)a.qzeros, (const __half*)a.scales, a.ws, a.N, a.G);
}

}  // namespace

void awq_gemv_launch(const AwqGemvArgs& a, cudaStream_t s) {
  if (a.M < 1 || a.M > kAwqGemvMaxRows) throw std::runtime_error("awq_gemv: 1..8 rows");
  if (a.N % 8 || a.G <= 0 || a.G > 256 || a.G % (8 * kGemvSplit) || a.K % a.G)
    throw std::runtime_error("awq_gemv: unsupported shape (N % 8, group a multiple of 32 up to 256)");
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
  launch_k(awq_reduce_kernel, dim3((unsigned)((MN + kRedOut - 1) / kRedOut)), dim3(kRedOut * kRedSlices), 0, s,
           (const float*)a.ws, a.K / a.G, a.M, a.N, (const __nv_bfloat16*)a.residual, (__nv_bfloat16*)a.out, a.ldo);
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
