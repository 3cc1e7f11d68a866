// bf16 GEMV for decode batches of 1-2 rows, for sm_100a:
//   out[m, n] = bf16(sum_k x[m, k] * W[n, k])            (fp32 accumulation)
//   out[m, n] = bf16(bf16(sum_k ...) + residual[m, n])    (residual form, the
//                                                          GEMM epilogue's rounding)
// plus two fused epilogues of the decoder (SiLU-mul of a gate_up projection;
// RoPE and paged-KV writes of a qkv projection).
// At one or two rows a linear layer is a weight stream: 2 bytes per weight
// against 2-4 FLOPs, far below what the tensor cores need to pay off, and the
// tile machinery (128-row MMA side, TMEM epilogue, split-K partials and their
// reduce launch) costs more than the stream itself. Here every weight byte is
// read once with 16-byte loads, 8 in flight per lane, by a warp per pair of
// output rows (several warps per pair when K is long or the rows are few);
// the x rows (a few KB, shared by every warp) come through L1. Measured on 8B
// decode at TP=1: 15 % faster per step at one row, 7 % at two, 8 % slower at
// four (the FMAs then bind), hence the two-row limit. The first weight loads
// are issued before the programmatic-launch wait, since the weights do not
// depend on earlier kernels.
#include <stdexcept>

#include "../common.cuh"
#include "../kernels.h"

namespace mbx {

namespace {

constexpr int kWarps = 8;        // warps per CTA
constexpr int kRowsPerWarp = 2;  // output rows of a warp (a row pair)
constexpr int kU = 4;            // 16-byte chunks per row per lane per batch (8 loads in flight)

MBX_DEVICE void bf16x8_to_f32(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// Epilogue modes.
//   kPlain: out[m, n] (+ residual).
//   kSilu:  W is a gate_up weight [2F, K] (gate rows, then up rows); a warp's
//           row pair is (j, F + j) and it writes out[m, j] = silu(gate) * up
//           with the roundings of the separate GEMM + silu_mul pair (gate and
//           up rounded to bf16, silu(gate) rounded to bf16, the product
//           rounded to bf16).
//   kRope:  W is a qkv weight [(nq + 2 nkv) * 128, K]; a warp's row pair is
//           dims (j, j + 64) of one head, so it applies the neox rotation at
//           the token's position to q and k heads (q to q_out [M, nq, 128], k
//           to the paged cache at the token's slot) and copies v heads to the
//           cache, with the roundings of the separate GEMM + rope_and_cache
//           pair (the projection rounded to bf16 first).
enum GemvEpi : int { kPlain = 0, kSilu = 1, kRope = 2 };

struct RopeArgs {
  const int* pos;         // [M] positions
  const float* cos_sin;   // [max_pos, 128]: cos(64) | sin(64)
  const int64_t* slots;   // [M] block * page + offset, or nullptr (no cache write)
  __nv_bfloat16* q_out;   // [M, nq, 128]
  __nv_bfloat16* k_cache; // [blocks, nkv, page, 128]
  __nv_bfloat16* v_cache;
  int nq, nkv, page;
};

// A warp owns a pair of output rows and a slice of K: `wpr` warps (a power of
// two up to kWarps) share a pair when K is long or the rows are few; lanes are
// 8 elements apart inside the slice. With wpr > 1 the slices' sums meet in
// shared memory in slice order.
template <int M, int EPI>
__global__ void __launch_bounds__(kWarps * 32) gemv_bf16_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                                const __nv_bfloat16* __restrict__ w, int64_t ldw,
                                                                __nv_bfloat16* __restrict__ out, int64_t ldo,
                                                                const __nv_bfloat16* residual, int N, int K,
                                                                int wpr, RopeArgs ra) {
  __shared__ float red[kWarps][kRowsPerWarp][M];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pair = warp / wpr, slice = warp % wpr;
  const int p = blockIdx.x * (kWarps / wpr) + pair;  // row pair index
  const int F = N / 2;                                // kSilu: output width
  const int n0 = EPI == kSilu ? p : (EPI == kRope ? (p / 64) * 128 + p % 64 : p * kRowsPerWarp);
  const int chunks = K / 8;  // 16-byte chunks per row
  const int per = (chunks + wpr - 1) / wpr;
  const int c_beg = slice * per, c_end = min(chunks, c_beg + per);
  const uint4* wr[kRowsPerWarp];
  bool live[kRowsPerWarp];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const int n = EPI == kSilu ? p + r * F : (EPI == kRope ? n0 + r * 64 : n0 + r);
    live[r] = EPI == kSilu ? p < F : (EPI == kRope ? p < N / 2 : n < N);
    wr[r] = reinterpret_cast<const uint4*>(w + (int64_t)(live[r] ? n : 0) * ldw);
  }
  float acc[kRowsPerWarp][M];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) acc[r][m] = 0.f;

  uint4 wv[kRowsPerWarp][kU];
  auto load_w = [&](int c0) {
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int c = c0 + u * 32 + lane;
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r)
        wv[r][u] = (live[r] && c < c_end) ? __ldg(wr[r] + c) : make_uint4(0, 0, 0, 0);
    }
  };
  load_w(c_beg);
  pdl_wait();  // x and residual may come from the previous kernel
#pragma unroll 1
  for (int c0 = c_beg; c0 < c_end; c0 += 32 * kU) {
    if (c0 > c_beg) load_w(c0);
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int c = c0 + u * 32 + lane;
      float xf[M][8];
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const uint4 xv = c < c_end ? __ldg(reinterpret_cast<const uint4*>(x + (int64_t)m * ldx) + c)
                                   : make_uint4(0, 0, 0, 0);
        bf16x8_to_f32(xv, xf[m]);
      }
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) {
        float wf[8];
        bf16x8_to_f32(wv[r][u], wf);
#pragma unroll
        for (int m = 0; m < M; ++m)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[r][m] = fmaf(xf[m][j], wf[j], acc[r][m]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) acc[r][m] = warp_sum(acc[r][m]);
  if (wpr > 1) {
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
        for (int m = 0; m < M; ++m) red[warp][r][m] = acc[r][m];
    }
    __syncthreads();
    if (slice != 0 || lane != 0) return;
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float v = red[warp][r][m];
        for (int i = 1; i < wpr; ++i) v += red[warp + i][r][m];
        acc[r][m] = v;
      }
  } else if (lane != 0) {
    return;
  }
  if constexpr (EPI == kRope) {
    if (p >= N / 2) return;
    const int h = p / 64, j = p % 64;
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const float x1 = __bfloat162float(__float2bfloat16(acc[0][m]));
      const float x2 = __bfloat162float(__float2bfloat16(acc[1][m]));
      const int64_t slot = ra.slots ? ra.slots[m] : -1;
      const int64_t blk = slot >= 0 ? slot / ra.page : 0, off = slot >= 0 ? slot % ra.page : 0;
      if (h < ra.nq + ra.nkv) {
        const float* cs = ra.cos_sin + (int64_t)ra.pos[m] * 128;
        const float c = cs[j], sn = cs[64 + j];
        const __nv_bfloat16 y1 = __float2bfloat16(x1 * c - x2 * sn);
        const __nv_bfloat16 y2 = __float2bfloat16(x2 * c + x1 * sn);
        __nv_bfloat16* dst = nullptr;
        if (h < ra.nq) dst = ra.q_out + ((int64_t)m * ra.nq + h) * 128;
        else if (slot >= 0) dst = ra.k_cache + ((blk * ra.nkv + (h - ra.nq)) * ra.page + off) * 128;
        if (dst != nullptr) {
          dst[j] = y1;
          dst[j + 64] = y2;
        }
      } else if (slot >= 0) {
        __nv_bfloat16* dst = ra.v_cache + ((blk * ra.nkv + (h - ra.nq - ra.nkv)) * ra.page + off) * 128;
        dst[j] = __float2bfloat16(x1);
        dst[j + 64] = __float2bfloat16(x2);
      }
    }
    return;
  }
  if constexpr (EPI == kSilu) {
    if (p >= F) return;
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const float g = __bfloat162float(__float2bfloat16(acc[0][m]));
      const float u = __bfloat162float(__float2bfloat16(acc[1][m]));
      const float sg = __bfloat162float(__float2bfloat16(g / (1.f + __expf(-g))));
      out[(int64_t)m * ldo + p] = __float2bfloat16(sg * u);
    }
    return;
  }
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const int n = n0 + r;
    if (n >= N) continue;
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float v = acc[r][m];
      if (residual != nullptr)
        v = __bfloat162float(__float2bfloat16(v)) + __bfloat162float(residual[(int64_t)m * ldo + n]);
      out[(int64_t)m * ldo + n] = __float2bfloat16(v);
    }
  }
}

template <int M, int EPI>
void launch_rows(const void* x, int64_t ldx, const void* w, int64_t ldw, void* out, int64_t ldo,
                 const void* residual, int N, int K, cudaStream_t s, const RopeArgs& ra = RopeArgs{}) {
  // warps per row pair: enough that no warp walks more than 4096 elements of a
  // row, and that the grid holds about 4096 warps (narrow tensor-parallel
  // shards: 384 row pairs of an 8B qkv shard at TP=8)
  const int pairs = EPI == kPlain ? (N + kRowsPerWarp - 1) / kRowsPerWarp : N / 2;
  int wpr = 1;
  while (wpr < kWarps && ((int64_t)K > 4096 * wpr || (int64_t)pairs * wpr < 4096)) wpr *= 2;
  const int pairs_per_cta = kWarps / wpr;
  launch_k(gemv_bf16_kernel<M, EPI>, dim3((unsigned)((pairs + pairs_per_cta - 1) / pairs_per_cta)),
           dim3(kWarps * 32), 0, s,
           static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(w), ldw,
           static_cast<__nv_bfloat16*>(out), ldo, static_cast<const __nv_bfloat16*>(residual), N, K, wpr, ra);
}

}  // namespace

bool gemv_bf16_supported(const void* x, int64_t ldx, const void* w, int64_t ldw, int64_t M, int64_t K) {
  return M >= 1 && M <= kGemvMaxRows && K % 8 == 0 && ldx % 8 == 0 && ldw % 8 == 0 &&
         ((uintptr_t)x & 15) == 0 && ((uintptr_t)w & 15) == 0;
}

void gemv_bf16_launch(const void* x, int64_t ldx, const void* w, int64_t ldw, void* out, int64_t ldo,
                      const void* residual, int64_t M, int64_t N, int64_t K, cudaStream_t s) {
  if (!gemv_bf16_supported(x, ldx, w, ldw, M, K)) throw std::runtime_error("gemv: unsupported shape or alignment");
  if (M == 1) launch_rows<1, kPlain>(x, ldx, w, ldw, out, ldo, residual, (int)N, (int)K, s);
  else launch_rows<2, kPlain>(x, ldx, w, ldw, out, ldo, residual, (int)N, (int)K, s);
  MBX_CUDA_CHECK(cudaGetLastError());
}

void gemv_silu_launch(const void* x, int64_t ldx, const void* w, int64_t ldw, void* out, int64_t ldo, int64_t M,
                      int64_t N2, int64_t K, cudaStream_t s) {
  if (!gemv_bf16_supported(x, ldx, w, ldw, M, K) || N2 % 2 != 0)
    throw std::runtime_error("gemv_silu: unsupported shape or alignment");
  if (M == 1) launch_rows<1, kSilu>(x, ldx, w, ldw, out, ldo, nullptr, (int)N2, (int)K, s);
  else launch_rows<2, kSilu>(x, ldx, w, ldw, out, ldo, nullptr, (int)N2, (int)K, s);
  MBX_CUDA_CHECK(cudaGetLastError());
}

void gemv_rope_launch(const void* x, int64_t ldx, const void* w, int64_t ldw, int64_t M, int64_t K, const int* pos,
                      const float* cos_sin, const int64_t* slots, void* q_out, void* k_cache, void* v_cache, int nq,
                      int nkv, int page, cudaStream_t s) {
  if (!gemv_bf16_supported(x, ldx, w, ldw, M, K)) throw std::runtime_error("gemv_rope: unsupported shape or alignment");
  RopeArgs ra;
  ra.pos = pos;
  ra.cos_sin = cos_sin;
  ra.slots = slots;
  ra.q_out = static_cast<__nv_bfloat16*>(q_out);
  ra.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  ra.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  ra.nq = nq;
  ra.nkv = nkv;
  ra.page = page;
  const int N = (nq + 2 * nkv) * 128;
  if (M == 1) launch_rows<1, kRope>(x, ldx, w, ldw, nullptr, 0, nullptr, N, (int)K, s, ra);
  else launch_rows<2, kRope>(x, ldx, w, ldw, nullptr, 0, nullptr, N, (int)K, s, ra);
  MBX_CUDA_CHECK(cudaGetLastError());
}

}  // namespace mbx
