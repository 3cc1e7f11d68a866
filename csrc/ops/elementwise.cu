// Memory-bound hot ops of the served decoder, written for sm_100a:
//   rmsnorm / fused_add_rmsnorm, rope_and_cache (neox RoPE on q/k + paged-KV
//   write of k/v in one pass), silu_mul, vocab-parallel embedding gather,
//   greedy argmax over a vocab shard, and a plain paged-KV write.
// All of them move 16-byte packs and accumulate in fp32. The reference has no
// model code (these are sglang kernels there, docs/performance.md:3-5).
#include <algorithm>
#include <stdexcept>
#include <string>

#include "../common.cuh"
#include "../kernels.h"

namespace mbx {

namespace {

__device__ __forceinline__ float block_reduce_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += red[i];
  __syncthreads();
  return s;
}

// out = bf16(x * rsqrt(mean(x^2) + eps) * w); optional residual: x = bf16(x + res), res <- x.
template <bool kResidual>
__global__ void rmsnorm_kernel(const uint4* __restrict__ x, uint4* residual, const uint4* __restrict__ w,
                               uint4* __restrict__ out, int hvec, float inv_h, float eps) {
  pdl_wait();
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const uint4* xr = x + row * hvec;
  uint4* rr = kResidual ? residual + row * hvec : nullptr;
  uint4* orow = out + row * hvec;
  constexpr int kMaxPer = 4;  // up to 4 packs per thread held in registers
  uint4 vals[kMaxPer];
  float ss = 0.f;
  int k = 0;
  for (int p = threadIdx.x; p < hvec; p += blockDim.x, ++k) {
    float a[8] = {};
    unpack_add<__nv_bfloat16>(xr[p], a);
    if (kResidual) unpack_add<__nv_bfloat16>(rr[p], a);
    const uint4 v = pack_from<__nv_bfloat16>(a);
    if (kResidual) rr[p] = v;
    float q[8] = {};
    unpack_add<__nv_bfloat16>(v, q);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += q[i] * q[i];
    if (k < kMaxPer) vals[k] = v;
  }
  const float rstd = rsqrtf(block_reduce_sum(ss, red) * inv_h + eps);
  k = 0;
  for (int p = threadIdx.x; p < hvec; p += blockDim.x, ++k) {
    float q[8] = {}, wv[8] = {};
    const uint4 v = k < kMaxPer ? vals[k] : (kResidual ? rr[p] : xr[p]);
    unpack_add<__nv_bfloat16>(v, q);
    unpack_add<__nv_bfloat16>(w[p], wv);
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = q[i] * rstd * wv[i];
    orow[p] = pack_from<__nv_bfloat16>(q);
  }
}

// NeoX-style rotary embedding on q and k (rotate the two halves of each head)
// using a precomputed [max_pos, head_dim/2] cos/sin table, plus the paged-KV
// write of the rotated k and of v. qkv rows are [q heads | k heads | v heads].
// Cache layout: [num_blocks, kv_heads, page, head_dim]; slot = block*page + off.
// q is written (rotated) to q_out [T, nq, D].
template <int D>
__global__ void rope_and_cache_kernel(const __nv_bfloat16* __restrict__ qkv, const int* __restrict__ pos,
                                      const float* __restrict__ cos_sin, const int64_t* __restrict__ slots,
                                      __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_cache,
                                      __nv_bfloat16* __restrict__ v_cache, int nq, int nkv, int page) {
  constexpr int H2 = D / 2;
  pdl_wait();
  const int t = blockIdx.x;
  const int p = pos[t];
  const float* cs = cos_sin + (int64_t)p * D;  // [cos(H2) | sin(H2)]
  const __nv_bfloat16* row = qkv + (int64_t)t * (nq + 2 * nkv) * D;
  const int64_t slot = slots ? slots[t] : -1;
  const int64_t blk = slot >= 0 ? slot / page : 0, off = slot >= 0 ? slot % page : 0;
  // one thread per (head, pair index)
  const int total = (nq + nkv) * H2;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int h = i / H2, j = i % H2;
    const __nv_bfloat16* src = row + h * D;
    const float x1 = __bfloat162float(src[j]), x2 = __bfloat162float(src[j + H2]);
    const float c = cs[j], s = cs[H2 + j];
    const __nv_bfloat16 y1 = __float2bfloat16(x1 * c - x2 * s);
    const __nv_bfloat16 y2 = __float2bfloat16(x2 * c + x1 * s);
    if (h < nq) {
      __nv_bfloat16* dst = q_out + ((int64_t)t * nq + h) * D;
      dst[j] = y1;
      dst[j + H2] = y2;
    } else if (slot >= 0) {
      const int kh = h - nq;
      __nv_bfloat16* dst = k_cache + ((blk * nkv + kh) * page + off) * D;
      dst[j] = y1;
      dst[j + H2] = y2;
    }
  }
  if (slot >= 0) {
    // v: plain copy, 16-byte packs
    const uint4* vsrc = reinterpret_cast<const uint4*>(row + (nq + nkv) * D);
    constexpr int PV = D / 8;
    for (int i = threadIdx.x; i < nkv * PV; i += blockDim.x) {
      const int kh = i / PV, j = i % PV;
      uint4* dst = reinterpret_cast<uint4*>(v_cache + ((blk * nkv + kh) * page + off) * D);
      dst[j] = vsrc[kh * PV + j];
    }
  }
}

// Qwen3: per-head RMSNorm of q and k (weights q_norm / k_norm [D], fp32
// statistics, one rounding after the rotation) fused in front of the NeoX
// rotation, then the stores of rope_and_cache_kernel. One warp per head:
// lane l holds elements 2l, 2l+1 and their rotation partners 2l+64, 2l+65, so
// a head's sum of squares is one warp reduction and the rotation stays in the
// lane. v is copied unnormalised (the model norms q and k only).
__global__ void rope_qknorm_cache_kernel(const __nv_bfloat16* __restrict__ qkv, const int* __restrict__ pos,
                                         const float* __restrict__ cos_sin, const int64_t* __restrict__ slots,
                                         const __nv_bfloat16* __restrict__ q_norm,
                                         const __nv_bfloat16* __restrict__ k_norm, float eps,
                                         __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_cache,
                                         __nv_bfloat16* __restrict__ v_cache, int nq, int nkv, int page) {
  constexpr int D = 128, H2 = 64;
  pdl_wait();
  const int t = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const float* cs = cos_sin + (int64_t)pos[t] * D;  // [cos(H2) | sin(H2)]
  const __nv_bfloat16* row = qkv + (int64_t)t * (nq + 2 * nkv) * D;
  const int64_t slot = slots ? slots[t] : -1;
  const int64_t blk = slot >= 0 ? slot / page : 0, off = slot >= 0 ? slot % page : 0;
  const int j = 2 * lane;
  const float c0 = cs[j], c1 = cs[j + 1], s0 = cs[H2 + j], s1 = cs[H2 + j + 1];
  // k heads only feed the cache: without slots the warps stop after the q heads
  const int heads = slot >= 0 ? nq + nkv : nq;
  for (int h = warp; h < heads; h += nwarps) {
    const __nv_bfloat16* src = row + h * D;
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + j));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + H2 + j));
    float ss = a.x * a.x + a.y * a.y + b.x * b.x + b.y * b.y;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss * (1.f / D) + eps);
    const __nv_bfloat16* w = h < nq ? q_norm : k_norm;
    const float a0 = a.x * r * __bfloat162float(w[j]), a1 = a.y * r * __bfloat162float(w[j + 1]);
    const float b0 = b.x * r * __bfloat162float(w[H2 + j]), b1 = b.y * r * __bfloat162float(w[H2 + j + 1]);
    __nv_bfloat16* dst = h < nq ? q_out + ((int64_t)t * nq + h) * D
                                : k_cache + ((blk * nkv + (h - nq)) * page + off) * D;
    *reinterpret_cast<__nv_bfloat162*>(dst + j) = __floats2bfloat162_rn(a0 * c0 - b0 * s0, a1 * c1 - b1 * s1);
    *reinterpret_cast<__nv_bfloat162*>(dst + H2 + j) = __floats2bfloat162_rn(b0 * c0 + a0 * s0, b1 * c1 + a1 * s1);
  }
  if (slot >= 0) {
    const uint4* vsrc = reinterpret_cast<const uint4*>(row + (nq + nkv) * D);
    constexpr int PV = D / 8;
    for (int i = threadIdx.x; i < nkv * PV; i += blockDim.x) {
      const int kh = i / PV, jj = i % PV;
      uint4* dst = reinterpret_cast<uint4*>(v_cache + ((blk * nkv + kh) * page + off) * D);
      dst[jj] = vsrc[kh * PV + jj];
    }
  }
}

// out[m, j] = silu(x[m, j]) * x[m, I + j]
__global__ void silu_mul_kernel(const uint4* __restrict__ x, uint4* __restrict__ out, int ivec) {
  pdl_wait();
  const int64_t row = blockIdx.y;
  const uint4* g = x + row * 2 * ivec;
  const uint4* u = g + ivec;
  uint4* o = out + row * ivec;
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < ivec; p += gridDim.x * blockDim.x) {
    float a[8] = {}, b[8] = {};
    unpack_add<__nv_bfloat16>(g[p], a);
    unpack_add<__nv_bfloat16>(u[p], b);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      // round silu(gate) to bf16 before the product (matches torch's
      // F.silu(gate) * up evaluated in bf16)
      const float sg = __bfloat162float(__float2bfloat16(a[i] / (1.f + __expf(-a[i]))));
      a[i] = sg * b[i];
    }
    o[p] = pack_from<__nv_bfloat16>(a);
  }
}

// Vocab-parallel embedding: rows whose id is outside [start, start + rows) are
// zero (the tensor-parallel allreduce then sums the shards).
__global__ void embedding_kernel(const int* __restrict__ ids, const uint4* __restrict__ table, uint4* __restrict__ out,
                                 int hvec, int64_t start, int64_t rows) {
  pdl_wait();
  const int t = blockIdx.x;
  const int64_t id = (int64_t)ids[t] - start;
  const bool in = id >= 0 && id < rows;
  for (int p = threadIdx.x; p < hvec; p += blockDim.x)
    out[(int64_t)t * hvec + p] = in ? table[id * hvec + p] : make_uint4(0, 0, 0, 0);
}

MBX_DEVICE float to_f32(float x) { return x; }
MBX_DEVICE float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

// Greedy argmax over a vocab shard; ties resolve to the smallest index.
template <typename T>
__global__ void argmax_kernel(const T* __restrict__ logits, int64_t ld, int V, int64_t offset,
                              float* __restrict__ best_val, int64_t* __restrict__ best_idx) {
  pdl_wait();
  __shared__ float sv[32];
  __shared__ int si[32];
  const int64_t row = blockIdx.x;
  const T* lr = logits + row * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int j = threadIdx.x; j < V; j += blockDim.x) {
    const float v = to_f32(lr[j]);
    if (v > bv || (v == bv && j < bi)) {
      bv = v;
      bi = j;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sv[w] = bv;
    si[w] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i)
      if (sv[i] > bv || (sv[i] == bv && si[i] < bi)) {
        bv = sv[i];
        bi = si[i];
      }
    best_val[row] = bv;
    best_idx[row] = (int64_t)bi + offset;
  }
}

// Pick the winner among per-rank (value, index) candidates: [W, B] -> [B].
__global__ void argmax_combine_kernel(const float* __restrict__ vals, const int64_t* __restrict__ idxs, int W, int B,
                                      int64_t* __restrict__ out) {
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  float bv = vals[b];
  int64_t bi = idxs[b];
  for (int r = 1; r < W; ++r) {
    const float v = vals[r * B + b];
    const int64_t i = idxs[r * B + b];
    if (v > bv || (v == bv && i < bi)) {
      bv = v;
      bi = i;
    }
  }
  out[b] = bi;
}

int norm_threads(int hvec) {
  int t = std::min(1024, std::max(32, hvec));
  return (t + 31) / 32 * 32;
}

}  // namespace

void rmsnorm_launch(const void* x, void* residual, const void* w, void* out, int64_t M, int H, float eps,
                    cudaStream_t s) {
  if (M == 0) return;
  if (H % 8 != 0 || H / 8 > 4 * 1024) throw std::runtime_error("rmsnorm: bad hidden size");
  const int hvec = H / 8;
  if (residual)
    launch_k(rmsnorm_kernel<true>, dim3((unsigned)M), dim3(norm_threads(hvec)), 0, s, (const uint4*)x,
             (uint4*)residual, (const uint4*)w, (uint4*)out, hvec, 1.f / H, eps);
  else
    launch_k(rmsnorm_kernel<false>, dim3((unsigned)M), dim3(norm_threads(hvec)), 0, s, (const uint4*)x,
             (uint4*)nullptr, (const uint4*)w, (uint4*)out, hvec, 1.f / H, eps);
  MBX_CUDA_CHECK(cudaGetLastError());
}

void rope_and_cache_launch(const void* qkv, const int* pos, const float* cos_sin, const int64_t* slots, void* q_out,
                           void* k_cache, void* v_cache, int64_t T, int nq, int nkv, int page, cudaStream_t s,
                           const void* q_norm, const void* k_norm, float eps) {
  if (T == 0) return;
  if (q_norm != nullptr) {
    launch_k(rope_qknorm_cache_kernel, dim3((unsigned)T), dim3(256), 0, s, (const __nv_bfloat16*)qkv, pos, cos_sin,
             slots, (const __nv_bfloat16*)q_norm, (const __nv_bfloat16*)k_norm, eps, (__nv_bfloat16*)q_out,
             (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache, nq, nkv, page);
  } else {
    launch_k(rope_and_cache_kernel<128>, dim3((unsigned)T), dim3(256), 0, s, (const __nv_bfloat16*)qkv, pos, cos_sin,
             slots, (__nv_bfloat16*)q_out, (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache, nq, nkv, page);
  }
  MBX_CUDA_CHECK(cudaGetLastError());
}

void silu_mul_launch(const void* x, void* out, int64_t M, int I2, cudaStream_t s) {
  if (M == 0) return;
  if (I2 % 16 != 0) throw std::runtime_error("silu_mul: width must be a multiple of 16");
  const int ivec = I2 / 16;
  const int threads = 256;
  const int64_t rows_per = 65535;
  for (int64_t r0 = 0; r0 < M; r0 += rows_per) {
    const int64_t rows = std::min(rows_per, M - r0);
    dim3 grid((ivec + threads - 1) / threads, (unsigned)rows);
    launch_k(silu_mul_kernel, grid, dim3(threads), 0, s, (const uint4*)x + r0 * 2 * ivec, (uint4*)out + r0 * ivec,
             ivec);
  }
  MBX_CUDA_CHECK(cudaGetLastError());
}

void embedding_launch(const int* ids, const void* table, void* out, int64_t T, int H, int64_t start, int64_t rows,
                      cudaStream_t s) {
  if (T == 0) return;
  if (H % 8 != 0) throw std::runtime_error("embedding: hidden must be a multiple of 8");
  launch_k(embedding_kernel, dim3((unsigned)T), dim3(256), 0, s, ids, (const uint4*)table, (uint4*)out, H / 8, start,
           rows);
  MBX_CUDA_CHECK(cudaGetLastError());
}

void argmax_launch(const void* logits, bool bf16, int64_t ld, int64_t B, int V, int64_t offset, float* best_val,
                   int64_t* best_idx, cudaStream_t s) {
  if (B == 0) return;
  if (bf16)
    launch_k(argmax_kernel<__nv_bfloat16>, dim3((unsigned)B), dim3(1024), 0, s, (const __nv_bfloat16*)logits, ld, V,
             offset, best_val, best_idx);
  else
    launch_k(argmax_kernel<float>, dim3((unsigned)B), dim3(1024), 0, s, (const float*)logits, ld, V, offset, best_val,
             best_idx);
  MBX_CUDA_CHECK(cudaGetLastError());
}

void argmax_combine_launch(const float* vals, const int64_t* idxs, int W, int B, int64_t* out, cudaStream_t s) {
  if (B == 0) return;
  launch_k(argmax_combine_kernel, dim3((B + 127) / 128), dim3(128), 0, s, vals, idxs, W, B, out);
  MBX_CUDA_CHECK(cudaGetLastError());
}

}  // namespace mbx
