// Paged attention for the served decoder (head_dim 128, bf16, GQA).
//
//  * prefill_attention: causal, chunked prefill over a ragged batch. Each
//    (q-tile of 64 tokens, q-head) block streams the request's keys/values
//    from the paged cache (page 16, layout [blocks, kv_heads, 16, 128]) in
//    64-key tiles with cp.async double buffering, computes S = QK^T and
//    O += PV with m16n8k16 bf16 tensor-core MMAs and an online softmax in
//    fp32 (exp2 domain). Query i of a request with kv_len L and q_len Lq sits
//    at position L - Lq + i and attends keys 0..that position.
//  * decode_attention: one query per request, GQA heads packed as the rows of
//    one tensor-core tile so each KV page is read once; the request's keys are
//    split across blocks (split-KV) for parallelism at small batch, each split
//    writes a normalised partial output and its log-sum-exp, and a combine
//    kernel merges the splits (LSE-weighted). A single split writes the
//    output directly.
// The reference has no attention code (sglang provides it,
// docs/performance.md:3-5; prefix cache noted in tests/pp_bench.py:1-2).
#include <algorithm>
#include <stdexcept>
#include <string>

#include "../common.cuh"
#include "../kernels.h"

namespace mbx {
namespace {

constexpr int D = 128;
constexpr int BQ = 64;
constexpr int BKV = 64;
constexpr int PAGE = 16;
constexpr int kAttnThreads = 128;

MBX_DEVICE uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Swizzled [rows][128] bf16 tile: 16-byte chunk c of row r lives at chunk c ^ (r & 7).
MBX_DEVICE uint32_t swz(int row, int chunk) { return row * 256 + ((chunk ^ (row & 7)) << 4); }

MBX_DEVICE void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
MBX_DEVICE void cp_async16_zfill(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
MBX_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
MBX_DEVICE void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

MBX_DEVICE void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
MBX_DEVICE void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

MBX_DEVICE void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

MBX_DEVICE uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

struct PrefillArgs {
  const __nv_bfloat16* q;   // [T, nq, D]
  const __nv_bfloat16* kc;  // [blocks, nkv, PAGE, D]
  const __nv_bfloat16* vc;
  __nv_bfloat16* o;         // [T, nq, D]
  const int* cu_q;          // [R+1]
  const int* kv_len;        // [R]
  const int* block_table;   // [R, max_blocks]
  const int2* tiles;        // [num_tiles] (request, q offset within request)
  int max_blocks;
  int nq, nkv;
  float scale_log2;         // softmax scale * log2(e)
};

// Load a 64-key K or V tile (keys kv0..kv0+63 of request r, kv head h) into a
// swizzled smem tile; keys >= kv_end are zero-filled.
MBX_DEVICE void load_kv_tile(uint32_t dst, const __nv_bfloat16* cache, const int* bt, int nkv, int h, int kv0,
                             int kv_end) {
  // 64 keys x 16 chunks = 1024 16-byte copies, 8 per thread
#pragma unroll
  for (int i = 0; i < (BKV * 16) / kAttnThreads; ++i) {
    const int idx = threadIdx.x + i * kAttnThreads;
    const int row = idx >> 4, chunk = idx & 15;
    const int key = kv0 + row;
    const bool valid = key < kv_end;
    const int kk = valid ? key : 0;
    const int blk = bt[kk / PAGE];
    const __nv_bfloat16* src = cache + (((int64_t)blk * nkv + h) * PAGE + (kk % PAGE)) * D + chunk * 8;
    cp_async16_zfill(dst + swz(row, chunk), src, valid);
  }
}

__global__ void __launch_bounds__(kAttnThreads) prefill_attention_kernel(PrefillArgs a) {
  pdl_wait();
  extern __shared__ __align__(128) uint8_t smem[];
  // [Q 64x128][K0][V0][K1][V1], each 16 KB
  const uint32_t sQ = smem_addr(smem);
  const uint32_t sK[2] = {sQ + 16384, sQ + 16384 * 3};
  const uint32_t sV[2] = {sQ + 16384 * 2, sQ + 16384 * 4};

  const int2 tile = a.tiles[blockIdx.x];
  const int r = tile.x, qoff = tile.y;
  const int head = blockIdx.y;
  const int kvh = head / (a.nq / a.nkv);
  const int q_begin = a.cu_q[r], q_len = a.cu_q[r + 1] - q_begin;
  const int L = a.kv_len[r];
  const int pos0 = L - q_len;  // position of the request's first query
  const int* bt = a.block_table + (int64_t)r * a.max_blocks;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;

  // Q tile -> smem (rows beyond q_len zero-filled)
  const int rows_here = min(BQ, q_len - qoff);
#pragma unroll
  for (int i = 0; i < (BQ * 16) / kAttnThreads; ++i) {
    const int idx = threadIdx.x + i * kAttnThreads;
    const int row = idx >> 4, chunk = idx & 15;
    const bool valid = row < rows_here;
    const __nv_bfloat16* src = a.q + ((int64_t)(q_begin + qoff + (valid ? row : 0)) * a.nq + head) * D + chunk * 8;
    cp_async16_zfill(sQ + swz(row, chunk), src, valid);
  }
  // causal bound: last query position in this tile
  const int last_pos = pos0 + qoff + rows_here - 1;
  const int kv_end = min(L, last_pos + 1);
  const int n_tiles = (kv_end + BKV - 1) / BKV;
  if (n_tiles > 0) {
    load_kv_tile(sK[0], a.kc, bt, a.nkv, kvh, 0, kv_end);
    load_kv_tile(sV[0], a.vc, bt, a.nkv, kvh, 0, kv_end);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();

  // Q fragments for this warp's 16 rows, 8 k-steps.
  uint32_t qf[8][4];
  {
    const int row = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int chunk = ks * 2 + (lane >> 4);
      ldsm_x4(sQ + swz(row, chunk), qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3]);
    }
  }

  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  const int qpos_r0 = pos0 + qoff + warp * 16 + g;  // rows g and g+8
  const int qpos_r1 = qpos_r0 + 8;

  for (int it = 0; it < n_tiles; ++it) {
    const int buf = it & 1;
    if (it + 1 < n_tiles) {
      load_kv_tile(sK[buf ^ 1], a.kc, bt, a.nkv, kvh, (it + 1) * BKV, kv_end);
      load_kv_tile(sV[buf ^ 1], a.vc, bt, a.nkv, kvh, (it + 1) * BKV, kv_end);
    }
    cp_async_commit();

    // S = Q K^T : 16 x 64 per warp (8 n-tiles)
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int jn = 0; jn < 4; ++jn) {  // pairs of key n-tiles
        const int key = jn * 16 + (lane & 7) + 8 * (lane >> 4);
        const int chunk = ks * 2 + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(sK[buf] + swz(key, chunk), b0, b1, b2, b3);
        mma16816(s[2 * jn], qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], b0, b1);
        mma16816(s[2 * jn + 1], qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], b2, b3);
      }
    }
    // mask + online softmax
    const int kv0 = it * BKV;
    const bool need_mask = (kv0 + BKV > kv_end) || (kv0 + BKV - 1 > pos0 + qoff + warp * 16);
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = s[j][e] * a.scale_log2;
        if (need_mask) {
          const int key = kv0 + j * 8 + 2 * t4 + (e & 1);
          const int qp = (e < 2) ? qpos_r0 : qpos_r1;
          if (key > qp || key >= kv_end) v = -INFINITY;
        }
        s[j][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
    }
    float corr[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float mnew = mx[h];
      corr[h] = (mnew == -INFINITY) ? 1.f : exp2f(m_r[h] - mnew);
      m_r[h] = mnew;
    }
    uint32_t pf[4][4];  // P as A fragments, 4 k-steps of 16 keys
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float p[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mm = m_r[e >> 1];
        p[e] = (mm == -INFINITY) ? 0.f : exp2f(s[j][e] - mm);
        rs[e >> 1] += p[e];
      }
      const int kstep = j >> 1, hi = j & 1;
      pf[kstep][hi * 2 + 0] = pack_bf16(p[0], p[1]);
      pf[kstep][hi * 2 + 1] = pack_bf16(p[2], p[3]);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 1);
      rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 2);
      l_r[h] = l_r[h] * corr[h] + rs[h];
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= corr[0];
      o[j][1] *= corr[0];
      o[j][2] *= corr[1];
      o[j][3] *= corr[1];
    }
    // O += P V : for each 16-key k-step, 16 dim n-tiles (8 ldmatrix.x4.trans)
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      // A-fragment register order: a0 (row g, k lo), a1 (row g+8, k lo), a2 (row g, k hi), a3 (row g+8, k hi)
      const uint32_t a0 = pf[ks][0], a1 = pf[ks][1], a2 = pf[ks][2], a3 = pf[ks][3];
#pragma unroll
      for (int jn = 0; jn < 8; ++jn) {
        const int key = ks * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
        const int chunk = jn * 2 + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(sV[buf] + swz(key, chunk), b0, b1, b2, b3);
        mma16816(o[2 * jn], a0, a1, a2, a3, b0, b1);
        mma16816(o[2 * jn + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    cp_async_wait<0>();
    __syncthreads();
  }

  // normalise and store
  const float inv0 = l_r[0] > 0.f ? 1.f / l_r[0] : 0.f;
  const float inv1 = l_r[1] > 0.f ? 1.f / l_r[1] : 0.f;
  const int row0 = warp * 16 + g, row1 = row0 + 8;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int col = j * 8 + 2 * t4;
    if (row0 < rows_here) {
      __nv_bfloat16* dst = a.o + ((int64_t)(q_begin + qoff + row0) * a.nq + head) * D + col;
      *reinterpret_cast<uint32_t*>(dst) = pack_bf16(o[j][0] * inv0, o[j][1] * inv0);
    }
    if (row1 < rows_here) {
      __nv_bfloat16* dst = a.o + ((int64_t)(q_begin + qoff + row1) * a.nq + head) * D + col;
      *reinterpret_cast<uint32_t*>(dst) = pack_bf16(o[j][2] * inv1, o[j][3] * inv1);
    }
  }
}

// ------------------------------------------------------------------- decode
// One query token per request. The G = nq/nkv query heads that share a KV head
// form the rows of one 16-row m16n8k16 tile (rows >= G are zero), so each KV
// page is read once per (request, kv head). A block of 4 warps handles one
// split of the request's keys; each warp streams its own pages (16 keys x 128
// dims, 4 KB of K + 4 KB of V) through a 3-stage cp.async ring, computes
// S = Q K^T and O += P V with tensor-core MMAs and keeps an online softmax;
// the warps then merge (m, l, O) through shared memory.
struct DecodeArgs {
  const __nv_bfloat16* q;   // [B, nq, D]
  const __nv_bfloat16* kc;
  const __nv_bfloat16* vc;
  __nv_bfloat16* o;         // [B, nq, D]
  float* part_o;            // [B, nq, splits, D] (splits > 1)
  float* part_lse;          // [B, nq, splits]
  const int* kv_len;        // [B]
  const int* block_table;   // [B, max_blocks]
  int* counters;            // [B, nkv] arrival counts (zero; the last CTA resets) or nullptr
  int max_blocks, nq, nkv, splits;
  float scale_log2;
};

constexpr int kDecWarps = 4;
constexpr int kDecThreads = kDecWarps * 32;
constexpr int kDecStages = 3;
constexpr int kPageBytes = PAGE * D * 2;               // 4 KB
constexpr int kDecStageBytes = 2 * kPageBytes;         // K + V page
constexpr int kDecSmem = kDecWarps * kDecStages * kDecStageBytes;  // 96 KB
constexpr int kMaxG = 16;

MBX_DEVICE void load_page(uint32_t dst, const __nv_bfloat16* base, int lane) {
  // 16 rows x 16 chunks of 16 B, 8 per lane, swizzled like the prefill tiles
#pragma unroll
  for (int i = 0; i < (PAGE * 16) / 32; ++i) {
    const int idx = lane + i * 32;
    const int row = idx >> 4, chunk = idx & 15;
    cp_async16(dst + swz(row, chunk), base + row * D + chunk * 8);
  }
}

// One (row, head) of the split-KV merge, by one warp: lane l owns dims
// 4l..4l+3. Reads go through L2 (__ldcg): the partials may have been written
// by other CTAs of the same kernel.
MBX_DEVICE void combine_row(const float* part_o, const float* part_lse, int splits, int64_t bh, int lane,
                            __nv_bfloat16* o) {
  const float* lse = part_lse + bh * splits;
  float mx = -INFINITY;
  for (int s = lane; s < splits; s += 32) mx = fmaxf(mx, __ldcg(lse + s));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  const float4* po = reinterpret_cast<const float4*>(part_o + bh * splits * D) + lane;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float den = 0.f;
#pragma unroll 4
  for (int s = 0; s < splits; ++s) {
    const float ls = __ldcg(lse + s);
    const float w = (ls == -INFINITY) ? 0.f : exp2f(ls - mx);
    const float4 v = __ldcg(po + s * (D / 4));
    den += w;
    acc.x += w * v.x;
    acc.y += w * v.y;
    acc.z += w * v.z;
    acc.w += w * v.w;
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x * inv, acc.y * inv);
  __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z * inv, acc.w * inv);
  uint2 packed;
  packed.x = *reinterpret_cast<uint32_t*>(&lo);
  packed.y = *reinterpret_cast<uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(o + bh * D + lane * 4) = packed;
}

__global__ void __launch_bounds__(kDecThreads) decode_attention_kernel(DecodeArgs a) {
  pdl_wait();
  extern __shared__ __align__(128) uint8_t dsm[];
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int G = a.nq / a.nkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int L = a.kv_len[b];
  const int pages = (L + PAGE - 1) / PAGE;
  const int per = (pages + a.splits - 1) / a.splits;
  const int p_begin = split * per, p_end = min(pages, p_begin + per);
  const int* bt = a.block_table + (int64_t)b * a.max_blocks;
  const uint32_t ring = smem_addr(dsm) + warp * kDecStages * kDecStageBytes;

  // Q fragments (16 rows = heads kvh*G .. +G-1; rows >= G zero), 8 k-steps
  uint32_t qf[8][4];
  {
    const __nv_bfloat16* qb = a.q + ((int64_t)b * a.nq + kvh * G) * D;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int c0 = ks * 16 + 2 * t4;
      qf[ks][0] = g < G ? *reinterpret_cast<const uint32_t*>(qb + g * D + c0) : 0u;
      qf[ks][1] = g + 8 < G ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * D + c0) : 0u;
      qf[ks][2] = g < G ? *reinterpret_cast<const uint32_t*>(qb + g * D + c0 + 8) : 0u;
      qf[ks][3] = g + 8 < G ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * D + c0 + 8) : 0u;
    }
  }
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};

  // pages of this warp: p_begin + warp, + kDecWarps, ...
  auto page_src = [&](int p, const __nv_bfloat16* cache) {
    return cache + (((int64_t)bt[p] * a.nkv + kvh) * PAGE) * D;
  };
  int issue = p_begin + warp;
#pragma unroll
  for (int st = 0; st < kDecStages - 1; ++st) {
    if (issue < p_end) {
      const uint32_t dst = ring + st * kDecStageBytes;
      load_page(dst, page_src(issue, a.kc), lane);
      load_page(dst + kPageBytes, page_src(issue, a.vc), lane);
    }
    cp_async_commit();
    issue += kDecWarps;
  }
  int stage = 0;
  for (int p = p_begin + warp; p < p_end; p += kDecWarps) {
    {  // keep the ring full
      const int st = (stage + kDecStages - 1) % kDecStages;
      if (issue < p_end) {
        const uint32_t dst = ring + st * kDecStageBytes;
        load_page(dst, page_src(issue, a.kc), lane);
        load_page(dst + kPageBytes, page_src(issue, a.vc), lane);
      }
      cp_async_commit();
      issue += kDecWarps;
    }
    cp_async_wait<kDecStages - 1>();
    __syncwarp();
    const uint32_t sK = ring + stage * kDecStageBytes;
    const uint32_t sV = sK + kPageBytes;
    // S = Q K^T: 16 rows x 16 keys (2 n-tiles)
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int key = (lane & 7) + 8 * (lane >> 4);
      const int chunk = ks * 2 + ((lane >> 3) & 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4(sK + swz(key, chunk), b0, b1, b2, b3);
      mma16816(s[0], qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], b0, b1);
      mma16816(s[1], qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], b2, b3);
    }
    const int key0 = p * PAGE;
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = key0 + j * 8 + 2 * t4 + (e & 1);
        const float v = key < L ? s[j][e] * a.scale_log2 : -INFINITY;
        s[j][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
    }
    float corr[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      corr[h] = (mx[h] == -INFINITY) ? 1.f : exp2f(m_r[h] - mx[h]);
      m_r[h] = mx[h];
    }
    uint32_t pf[4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float pv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mm = m_r[e >> 1];
        pv[e] = (mm == -INFINITY) ? 0.f : exp2f(s[j][e] - mm);
        rs[e >> 1] += pv[e];
      }
      pf[j * 2 + 0] = pack_bf16(pv[0], pv[1]);
      pf[j * 2 + 1] = pack_bf16(pv[2], pv[3]);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 1);
      rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 2);
      l_r[h] = l_r[h] * corr[h] + rs[h];
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= corr[0];
      o[j][1] *= corr[0];
      o[j][2] *= corr[1];
      o[j][3] *= corr[1];
    }
    // O += P V (16 keys = one k-step), 8 pairs of dim n-tiles
#pragma unroll
    for (int jn = 0; jn < 8; ++jn) {
      const int key = (lane & 7) + 8 * ((lane >> 3) & 1);
      const int chunk = jn * 2 + (lane >> 4);
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(sV + swz(key, chunk), b0, b1, b2, b3);
      mma16816(o[2 * jn], pf[0], pf[1], pf[2], pf[3], b0, b1);
      mma16816(o[2 * jn + 1], pf[0], pf[1], pf[2], pf[3], b2, b3);
    }
    __syncwarp();
    stage = (stage + 1) % kDecStages;
  }
  cp_async_wait<0>();
  __syncthreads();

  // merge the warps' states: smem [warp][16 rows][D] fp32 + m, l per row
  float* so = reinterpret_cast<float*>(dsm);                 // 4 * 16 * 128 * 4 = 32 KB
  float* sm = so + kDecWarps * 16 * D;                       // [warp][16]
  float* sl = sm + kDecWarps * 16;                           // [warp][16]
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int col = j * 8 + 2 * t4;
    so[(warp * 16 + g) * D + col] = o[j][0];
    so[(warp * 16 + g) * D + col + 1] = o[j][1];
    so[(warp * 16 + g + 8) * D + col] = o[j][2];
    so[(warp * 16 + g + 8) * D + col + 1] = o[j][3];
  }
  if (t4 == 0) {
    sm[warp * 16 + g] = m_r[0];
    sm[warp * 16 + g + 8] = m_r[1];
    sl[warp * 16 + g] = l_r[0];
    sl[warp * 16 + g + 8] = l_r[1];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += kDecThreads) {
    const int row = i / D, d = i % D;
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) mm = fmaxf(mm, sm[w * 16 + row]);
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) {
      const float mw = sm[w * 16 + row];
      const float e = (mw == -INFINITY) ? 0.f : exp2f(mw - mm);
      num += e * so[(w * 16 + row) * D + d];
      den += e * sl[w * 16 + row];
    }
    const int qh = kvh * G + row;
    if (a.splits == 1) {
      a.o[((int64_t)b * a.nq + qh) * D + d] = __float2bfloat16(den > 0.f ? num / den : 0.f);
    } else {
      a.part_o[(((int64_t)b * a.nq + qh) * a.splits + split) * D + d] = den > 0.f ? num / den : 0.f;
      if (d == 0)
        a.part_lse[((int64_t)b * a.nq + qh) * a.splits + split] = (den > 0.f) ? mm + log2f(den) : -INFINITY;
    }
  }
  if (a.splits == 1 || a.counters == nullptr) return;
  // Split-KV merge in the kernel: the last CTA of (b, kvh) to finish combines
  // the G heads' partials (the combine kernel's arithmetic, one launch fewer).
  // Classic arrival counting: every CTA's partial stores are fenced before its
  // count; the last one fences again before reading the others'.
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    int* cnt = a.counters + (int64_t)b * a.nkv + kvh;
    s_last = atomicAdd(cnt, 1) == a.splits - 1;
    if (s_last) *cnt = 0;  // ready for the next launch
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int row = warp; row < G; row += kDecWarps) {
    const int64_t bh = (int64_t)b * a.nq + kvh * G + row;
    combine_row(a.part_o, a.part_lse, a.splits, bh, lane, a.o);
  }
}

// Split-KV combine: one warp per (row, head), lane l owns dims 4l..4l+3.
// o = sum_s 2^(lse_s - max) o_s / sum_s 2^(lse_s - max); splits that saw no
// key have lse = -inf and weight 0; a row with no key at all gets zeros.
constexpr int kCombineRows = 8;  // warps (rows) per block
__global__ void __launch_bounds__(32 * kCombineRows) decode_combine_kernel(const float* __restrict__ part_o,
                                                                          const float* __restrict__ part_lse,
                                                                          int splits, int64_t rows,
                                                                          __nv_bfloat16* __restrict__ o) {
  pdl_wait();
  const int64_t bh = (int64_t)blockIdx.x * kCombineRows + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (bh >= rows) return;
  combine_row(part_o, part_lse, splits, bh, lane, o);
}

}  // namespace

void prefill_attention_launch(const void* q, const void* kc, const void* vc, void* o, const int* cu_q,
                              const int* kv_len, const int* block_table, int max_blocks, const int* tiles,
                              int n_tiles, int nq, int nkv, float scale, cudaStream_t s) {
  if (n_tiles == 0) return;
  if (nq % nkv != 0) throw std::runtime_error("attention: nq must be a multiple of nkv");
  PrefillArgs a;
  a.q = (const __nv_bfloat16*)q;
  a.kc = (const __nv_bfloat16*)kc;
  a.vc = (const __nv_bfloat16*)vc;
  a.o = (__nv_bfloat16*)o;
  a.cu_q = cu_q;
  a.kv_len = kv_len;
  a.block_table = block_table;
  a.tiles = reinterpret_cast<const int2*>(tiles);
  a.max_blocks = max_blocks;
  a.nq = nq;
  a.nkv = nkv;
  a.scale_log2 = scale * 1.4426950408889634f;
  const int smem = 5 * 16384;
  static SmemLimit limit;
  limit.ensure((const void*)prefill_attention_kernel, smem);
  dim3 grid(n_tiles, nq);
  launch_k(prefill_attention_kernel, grid, dim3(kAttnThreads), smem, s, a);
  MBX_CUDA_CHECK(cudaGetLastError());
}

void attn_combine_launch(const float* part_o, const float* part_lse, int64_t rows, int splits, void* out,
                         cudaStream_t s) {
  if (rows == 0) return;
  const unsigned blocks = (unsigned)((rows + kCombineRows - 1) / kCombineRows);
  launch_k(decode_combine_kernel, dim3(blocks), dim3(32 * kCombineRows), 0, s, part_o, part_lse, splits, rows,
           static_cast<__nv_bfloat16*>(out));
  MBX_CUDA_CHECK(cudaGetLastError());
}

void decode_attention_launch(const void* q, const void* kc, const void* vc, void* o, const int* kv_len,
                             const int* block_table, int max_blocks, int B, int nq, int nkv, int splits,
                             float* part_o, float* part_lse, float scale, cudaStream_t s, int* counters) {
  if (B == 0) return;
  if (nq % nkv != 0 || nq / nkv > kMaxG) throw std::runtime_error("decode: group size must be <= 16");
  DecodeArgs a;
  a.q = (const __nv_bfloat16*)q;
  a.kc = (const __nv_bfloat16*)kc;
  a.vc = (const __nv_bfloat16*)vc;
  a.o = (__nv_bfloat16*)o;
  a.kv_len = kv_len;
  a.block_table = block_table;
  a.max_blocks = max_blocks;
  a.nq = nq;
  a.nkv = nkv;
  a.splits = std::max(1, splits);
  a.scale_log2 = scale * 1.4426950408889634f;
  a.part_o = part_o;
  a.part_lse = part_lse;
  a.counters = counters;
  if (a.splits > 1 && (!part_o || !part_lse)) throw std::runtime_error("decode: split-KV needs scratch buffers");
  static SmemLimit limit;
  limit.ensure((const void*)decode_attention_kernel, kDecSmem);
  dim3 grid(a.splits, nkv, B);
  launch_k(decode_attention_kernel, grid, dim3(kDecThreads), kDecSmem, s, a);
  MBX_CUDA_CHECK(cudaGetLastError());
  if (a.splits > 1 && counters == nullptr) {
    attn_combine_launch(a.part_o, a.part_lse, (int64_t)B * nq, a.splits, a.o, s);
    MBX_CUDA_CHECK(cudaGetLastError());
  }
}

}  // namespace mbx
