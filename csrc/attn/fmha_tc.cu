// Prefill attention on the Blackwell tensor cores (tcgen05 + TMEM + TMA).
//
// One CTA = two 128-row query tiles (256 queries) of one q-head, each with
// its own softmax warpgroup, sharing the K/V stages; the single MMA thread
// interleaves both tiles' S and PV MMAs so the tensor core has independent
// work while either softmax runs. For every 64-key tile of the request's
// paged KV cache (per query tile):
//   S_j  = Q K_j^T      tcgen05.mma (M=128, N=128, K=128 head dims), fp32 in
//                       TMEM, double-buffered (S_{j+1} overlaps softmax_j)
//   P_j  = exp2(S_j*scale - m)   online softmax by 4 warps (one row per
//                       thread, tcgen05.ld of the S row), written as bf16 to
//                       shared memory in the canonical K-major 128B-swizzled
//                       layout; the running output is rescaled in TMEM
//                       (tcgen05.ld/st) when a row's max grows
//   O   += P_j V_j      tcgen05.mma with V read MN-major (dims contiguous, as
//                       stored in the cache), fp32 accumulator in TMEM
// Warp roles (320 threads): warp 0 TMA producer (Q once; K/V pages of 16
// keys x 64 dims per box, double-buffered stages), warp 1 TMEM allocator +
// single-thread MMA issuer, warps 2-9 softmax + epilogue, two threads per
// row (each owns 64 of the 128 keys; row maxima exchanged through shared
// memory), so two softmax warps share every SM sub-partition. The running
// output is rescaled only when a row max grows by more than 2^8. No cluster
// multicast. Causal masking / kv-length masking per element in softmax.
// Every mbarrier wait is bounded; on timeout the CTA records an error, drains
// its in-flight copies and MMAs, frees TMEM and exits.
#include <cudaTypedefs.h>

#include <algorithm>
#include <functional>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>

#include "../gemm/tcgen05.cuh"
#include "../kernels.h"

namespace mbx {
namespace {

constexpr int D = 128;
constexpr int BQ = 128;             // rows per query tile
constexpr int QT = 2;               // query tiles per CTA (ping-pong)
constexpr int BKV = 64;             // keys per KV tile
constexpr int NS = 3;               // K/V pipeline stages
constexpr int PAGE = 16;
constexpr int kThreads = 320;       // warp 0 TMA, warp 1 MMA, warps 2-5 / 6-9 softmax of tile 0 / 1
constexpr int kQBytes = BQ * D * 2;           // 32 KB, two 16 KB column chunks
constexpr int kQChunk = BQ * 64 * 2;          // 16 KB
constexpr int kKVBytes = BKV * D * 2;         // 16 KB, two 8 KB column chunks
constexpr int kKVChunk = BKV * 64 * 2;        // 8 KB
constexpr int kPBytes = BQ * BKV * 2;         // 16 KB: [128 rows x 64 keys], one 128B-wide chunk
// Rescale the running output only when a row max grows by more than this
// (log2 units): exponents stay <= 2^8, harmless in fp32/bf16.
constexpr float kRescaleThreshold = 8.f;

struct FmhaArgs {
  __nv_bfloat16* o;         // [T, nq, D]
  const int* cu_q;          // [R+1]
  const int* kv_len;        // [R]
  const int* block_table;   // [R, max_blocks]
  const int2* tiles;        // (request, q offset): 256-row query-tile pairs
  float* part_o;            // splits > 1: [T, nq, splits, D] normalised partial outputs
  float* part_lse;          //             [T, nq, splits] log2-sum-exp
  int splits;
  int max_blocks, nq, nkv;
  float scale_log2;
  uint32_t* err;
  uint64_t timeout_ns;
};

struct Smem {
  static constexpr int kQ = 0;                          // [QT] query tiles
  static constexpr int kK = kQ + QT * kQBytes;          // [NS] key tiles
  static constexpr int kV = kK + NS * kKVBytes;         // [NS] value tiles
  static constexpr int kP = kV + NS * kKVBytes;         // [QT] probability tiles
  static constexpr int kBar = kP + QT * kPBytes;
  static constexpr int kTotal = kBar + 256 + 1024;
};

MBX_DEVICE void set_err(uint32_t* err, uint32_t code, volatile int* abort) {
  *abort = 1;
  if (err) atomicCAS(err, 0u, code);
}

__global__ void __launch_bounds__(kThreads, 1)
    fmha_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, FmhaArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Smem::kBar);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;          // [NS]
  uint64_t* kv_empty = kv_full + NS;     // [NS]
  uint64_t* s_full = kv_empty + NS;      // [QT][2]
  uint64_t* p_full = s_full + 2 * QT;    // [QT]
  uint64_t* o_done = p_full + QT;        // [QT]
  uint64_t* mma_done = o_done + QT;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();  // the tile list, lengths and block table may come from the previous kernel
  const int2 tile = a.tiles[blockIdx.x];
  const int r = tile.x, qoff = tile.y;
  const int head = blockIdx.y;
  const int kvh = head / (a.nq / a.nkv);
  const int q_begin = a.cu_q[r], q_len = a.cu_q[r + 1] - q_begin;
  const int L = a.kv_len[r];
  const int pos0 = L - q_len;
  const int* bt = a.block_table + (int64_t)r * a.max_blocks;
  // per query tile: valid rows, causal key bound, KV tiles needed
  int rows_t[QT], kvend_t[QT], n_t[QT];
#pragma unroll
  for (int t = 0; t < QT; ++t) {
    rows_t[t] = max(0, min(BQ, q_len - qoff - t * BQ));
    kvend_t[t] = rows_t[t] > 0 ? min(L, pos0 + qoff + t * BQ + rows_t[t]) : 0;
    n_t[t] = (kvend_t[t] + BKV - 1) / BKV;
  }
  const int n_all = max(n_t[0], n_t[1]);
  const int kv_end_all = max(kvend_t[0], kvend_t[1]);
  // split-KV: this CTA takes KV tiles [tb, te)
  const int split = blockIdx.z;
  const int per = (n_all + a.splits - 1) / a.splits;
  const int tb = min(n_all, split * per);
  const int te = min(n_all, tb + per);
  const int n_cta = te - tb;
  int nt[QT];
#pragma unroll
  for (int t = 0; t < QT; ++t) nt[t] = max(0, min(te, n_t[t]) - tb);

  if (threadIdx.x == 0) {
    tc::mbar_init(q_full, 1);
    for (int i = 0; i < NS; ++i) {
      tc::mbar_init(&kv_full[i], 1);
      tc::mbar_init(&kv_empty[i], 1);
    }
    for (int t = 0; t < QT; ++t) {
      tc::mbar_init(&s_full[2 * t], 1);
      tc::mbar_init(&s_full[2 * t + 1], 1);
      tc::mbar_init(&p_full[t], 4);
      tc::mbar_init(&o_done[t], 1);
    }
    tc::mbar_init(mma_done, 1);
    *abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: S[t][b] at (2t + b) * 64, O[t] at 256 + 128 t
  auto tS = [&](int t, int b) { return tmem + (uint32_t)((2 * t + b) * BKV); };
  auto tO = [&](int t) { return tmem + 256u + (uint32_t)(t * D); };

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (tc::elect_one()) {
      tc::tma_prefetch_desc(&tmQ);
      tc::tma_prefetch_desc(&tmK);
      tc::tma_prefetch_desc(&tmV);
      tc::mbar_arrive_expect_tx(q_full, QT * kQBytes);
      for (int t = 0; t < QT; ++t)
        for (int c = 0; c < 2; ++c)
          tc::tma_load_3d(smem + Smem::kQ + t * kQBytes + c * kQChunk, &tmQ, q_full, c * 64, head,
                          q_begin + qoff + t * BQ);
      const int last_page = max(0, (kv_end_all - 1) / PAGE);
      int issued = 0;
      for (int j = 0; j < n_cta && !*abort; ++j, ++issued) {
        const int s = j % NS;
        if (!tc::mbar_wait(&kv_empty[s], ((j / NS) & 1) ^ 1, abort, a.timeout_ns)) {
          set_err(a.err, 11, abort);
          break;
        }
        tc::mbar_arrive_expect_tx(&kv_full[s], 2 * kKVBytes);
        uint8_t* sk = smem + Smem::kK + s * kKVBytes;
        uint8_t* sv = smem + Smem::kV + s * kKVBytes;
#pragma unroll 1
        for (int p = 0; p < BKV / PAGE; ++p) {
          const int page = min((tb + j) * (BKV / PAGE) + p, last_page);  // clamp: masked keys read finite data
          const int blk = bt[page];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            tc::tma_load_4d(sk + c * kKVChunk + p * (PAGE * 128), &tmK, &kv_full[s], c * 64, 0, kvh, blk);
            tc::tma_load_4d(sv + c * kKVChunk + p * (PAGE * 128), &tmV, &kv_full[s], c * 64, 0, kvh, blk);
          }
        }
      }
      volatile int never = 0;
      tc::mbar_wait(q_full, 0, &never, 200000000ull);
      for (int j = max(0, issued - NS); j < issued; ++j)
        tc::mbar_wait(&kv_full[j % NS], (j / NS) & 1, &never, 200000000ull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (tc::elect_one()) {
      constexpr uint32_t idS = tc::idesc_bf16_f32_major(BQ, BKV, 0, 0);  // Q K-major, K K-major
      constexpr uint32_t idO = tc::idesc_bf16_f32_major(BQ, D, 0, 1);    // P K-major, V MN-major
      bool ok = tc::mbar_wait(q_full, 0, abort, a.timeout_ns);
      if (!ok) set_err(a.err, 12, abort);
      auto issue_s = [&](int j) -> bool {
        const int s = j % NS;
        if (!tc::mbar_wait(&kv_full[s], (j / NS) & 1, abort, a.timeout_ns)) {
          set_err(a.err, 12, abort);
          return false;
        }
        tc::tc_fence_after();
        const uint32_t sK = tc::smem_u32(smem + Smem::kK + s * kKVBytes);
#pragma unroll
        for (int t = 0; t < QT; ++t) {
          if (j >= nt[t]) continue;
          const uint32_t sQ = tc::smem_u32(smem + Smem::kQ + t * kQBytes);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t qoff_b = (kk >> 2) * kQChunk + (kk & 3) * 32;
            const uint32_t koff_b = (kk >> 2) * kKVChunk + (kk & 3) * 32;
            tc::mma_bf16(tS(t, j & 1), tc::sw128_desc(sQ + qoff_b, 16, 1024), tc::sw128_desc(sK + koff_b, 16, 1024),
                         idS, kk > 0 ? 1u : 0u);
          }
          tc::mma_commit(&s_full[2 * t + (j & 1)]);
        }
        return true;
      };
      if (ok && n_cta > 0) ok = issue_s(0);
      for (int j = 0; ok && j < n_cta; ++j) {
        if (j + 1 < n_cta && !issue_s(j + 1)) break;
        const uint32_t sV = tc::smem_u32(smem + Smem::kV + (j % NS) * kKVBytes);
#pragma unroll
        for (int t = 0; t < QT; ++t) {
          if (j >= nt[t]) continue;
          if (!tc::mbar_wait(&p_full[t], j & 1, abort, a.timeout_ns)) {
            set_err(a.err, 12, abort);
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t sP = tc::smem_u32(smem + Smem::kP + t * kPBytes);
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk) {
            // P: keys along K within one 128B chunk; V: 16 key rows of 128 B per step, MN atoms 8 KB apart
            tc::mma_bf16(tO(t), tc::sw128_desc(sP + kk * 32, 16, 1024), tc::sw128_desc(sV + kk * 16 * 128, kKVChunk, 1024),
                         idO, (j > 0 || kk > 0) ? 1u : 0u);
          }
          tc::mma_commit(&o_done[t]);
        }
        if (!ok) break;
        tc::mma_commit(&kv_empty[j % NS]);
      }
      tc::mma_commit(mma_done);
      volatile int never = 0;
      tc::mbar_wait(mma_done, 0, &never, 200000000ull);
    }
  } else {
    // ------------------------------------------------------------------ softmax / epilogue
    // Warps 2-5 own query tile 0, warps 6-9 tile 1; one thread per row.
    const int t = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
    const int q_pos = pos0 + qoff + t * BQ + row;
    const float sc = a.scale_log2;
    const int my_n = nt[t];
    float m = -INFINITY, l = 0.f;
    uint8_t* sP = smem + Smem::kP + t * kPBytes;
    bool ok = true;
    for (int j = 0; j < my_n; ++j) {
      const int b = j & 1;
      if (!tc::mbar_wait(&s_full[2 * t + b], (j >> 1) & 1, abort, a.timeout_ns)) {
        if (lane == 0) set_err(a.err, 13, abort);
        ok = false;
        break;
      }
      tc::tc_fence_after();
      uint32_t v[BKV];
#pragma unroll
      for (int c = 0; c < BKV / 32; ++c) {
        uint32_t tt[32];
        tc::tmem_ld_32x32b_x32(tS(t, b) + lane_addr + c * 32, tt);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[c * 32 + i] = tt[i];
      }
      tc::tmem_ld_wait();
      const int kv0 = (tb + j) * BKV;
      const int lim = min(q_pos + 1, kvend_t[t]) - kv0;  // keys [kv0, kv0 + lim) are visible
      if (lim < BKV) {
#pragma unroll
        for (int i = 0; i < BKV; ++i)
          if (i >= lim) v[i] = __float_as_uint(-INFINITY);
      }
      // Row max of the raw scores over 8 independent partial maxima (a
      // 64-deep dependent fmax chain would sit on the softmax's critical
      // path), then scaled once: sc > 0, so max(x * sc) = max(x) * sc.
      float m8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) m8[k] = __uint_as_float(v[k]);
#pragma unroll
      for (int i = 8; i < BKV; ++i) m8[i & 7] = fmaxf(m8[i & 7], __uint_as_float(v[i]));
#pragma unroll
      for (int k = 4; k > 0; k >>= 1)
#pragma unroll
        for (int q = 0; q < k; ++q) m8[q] = fmaxf(m8[q], m8[q + k]);
      const float mx = m8[0] * sc;
      const bool grow = mx > m + kRescaleThreshold || (m == -INFINITY && mx != -INFINITY);
      const float m_new = grow ? mx : m;
      const float corr = (m == -INFINITY || !grow) ? 1.f : tc::ex2(m - m_new);
      // p = 2^(x * sc - m_new) in one FMA per score; row sum over 8 partial sums
      const float neg = -m_new;
      float s8[8] = {};
      uint32_t pk[BKV / 2];
#pragma unroll
      for (int i = 0; i < BKV; i += 2) {
        const float p0 = (m_new == -INFINITY) ? 0.f : tc::ex2(fmaf(__uint_as_float(v[i]), sc, neg));
        const float p1 = (m_new == -INFINITY) ? 0.f : tc::ex2(fmaf(__uint_as_float(v[i + 1]), sc, neg));
        s8[(i >> 1) & 7] += p0 + p1;
        __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
        pk[i / 2] = *reinterpret_cast<uint32_t*>(&h2);
      }
#pragma unroll
      for (int k = 4; k > 0; k >>= 1)
#pragma unroll
        for (int q = 0; q < k; ++q) s8[q] += s8[q + k];
      const float sum = s8[0];
      l = l * corr + sum;
      m = m_new;
      if (j > 0) {
        // PV_{j-1} must be complete before P is overwritten and O is rescaled
        if (!tc::mbar_wait(&o_done[t], (j - 1) & 1, abort, a.timeout_ns)) {
          if (lane == 0) set_err(a.err, 13, abort);
          ok = false;
          break;
        }
        tc::tc_fence_after();
      }
#pragma unroll
      for (int cc = 0; cc < BKV / 8; ++cc) {
        uint8_t* dst = sP + (row >> 3) * 1024 + (row & 7) * 128 + ((cc ^ (row & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) = make_uint4(pk[cc * 4], pk[cc * 4 + 1], pk[cc * 4 + 2], pk[cc * 4 + 3]);
      }
      if (j > 0 && __any_sync(0xffffffffu, corr < 1.f)) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t tt[32];
          tc::tmem_ld_32x32b_x32(tO(t) + lane_addr + c * 32, tt);
          tc::tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) tt[i] = __float_as_uint(__uint_as_float(tt[i]) * corr);
          tc::tmem_st_32x32b_x32(tO(t) + lane_addr + c * 32, tt);
        }
        tc::tmem_st_wait();
      }
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&p_full[t]);
    }
    const int rows_here = rows_t[t];
    const int64_t tok = q_begin + qoff + t * BQ + row;
    if (ok && my_n > 0) {
      if (!tc::mbar_wait(&o_done[t], (my_n - 1) & 1, abort, a.timeout_ns)) {
        if (lane == 0) set_err(a.err, 13, abort);
      } else {
        tc::tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t tt[32];
          tc::tmem_ld_32x32b_x32(tO(t) + lane_addr + c * 32, tt);
          tc::tmem_ld_wait();
          if (row < rows_here) {
            if (a.splits == 1) {
              __nv_bfloat16* dst = a.o + (tok * a.nq + head) * D + c * 32;
              float f[8];
#pragma unroll
              for (int g = 0; g < 4; ++g) {
#pragma unroll
                for (int i = 0; i < 8; ++i) f[i] = __uint_as_float(tt[g * 8 + i]) * inv;
                *reinterpret_cast<uint4*>(dst + g * 8) = pack_from<__nv_bfloat16>(f);
              }
            } else {
              float* dst = a.part_o + ((tok * a.nq + head) * a.splits + split) * D + c * 32;
#pragma unroll
              for (int g = 0; g < 8; ++g)
                *reinterpret_cast<float4*>(dst + g * 4) =
                    make_float4(__uint_as_float(tt[g * 4]) * inv, __uint_as_float(tt[g * 4 + 1]) * inv,
                                __uint_as_float(tt[g * 4 + 2]) * inv, __uint_as_float(tt[g * 4 + 3]) * inv);
            }
          }
        }
        if (a.splits > 1 && row < rows_here)
          a.part_lse[(tok * a.nq + head) * a.splits + split] = (l > 0.f) ? m + log2f(l) : -INFINITY;
      }
    } else if (ok && my_n == 0 && a.splits > 1 && row < rows_here) {
      // this split holds no keys of the tile: contributes nothing to the combine
      float* dst = a.part_o + ((tok * a.nq + head) * a.splits + split) * D;
      for (int d = 0; d < D; d += 4) *reinterpret_cast<float4*>(dst + d) = make_float4(0.f, 0.f, 0.f, 0.f);
      a.part_lse[(tok * a.nq + head) * a.splits + split] = -INFINITY;
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 1) tc::tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  if (!fn) throw std::runtime_error("cuTensorMapEncodeTiled unavailable (no CUDA driver)");
  return fn;
}

CUtensorMap encode(const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides_bytes,
                   const cuuint32_t* box) {
  if (((uint64_t)base & 15) != 0) throw std::runtime_error("fmha: tensor base must be 16-byte aligned");
  CUtensorMap m;
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult res = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims, strides_bytes,
                             box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS) throw std::runtime_error("fmha: cuTensorMapEncodeTiled failed " + std::to_string((int)res));
  return m;
}

struct Key {
  uint64_t p, a, b, c;
  bool operator==(const Key& o) const { return p == o.p && a == o.a && b == o.b && c == o.c; }
};
struct KeyHash {
  size_t operator()(const Key& k) const {
    return (size_t)(k.p * 0x9E3779B97F4A7C15ull ^ (k.a << 1) ^ (k.b << 21) ^ (k.c << 41));
  }
};
std::mutex g_mu;
std::unordered_map<Key, CUtensorMap, KeyHash> g_maps;

CUtensorMap cached(const Key& k, const std::function<CUtensorMap()>& make) {
  {
    std::lock_guard<std::mutex> g(g_mu);
    auto it = g_maps.find(k);
    if (it != g_maps.end()) return it->second;
  }
  CUtensorMap m = make();
  std::lock_guard<std::mutex> g(g_mu);
  if (g_maps.size() > 4096) g_maps.clear();
  g_maps.emplace(k, m);
  return m;
}

}  // namespace

void prefill_attention_tc_launch(const void* q, const void* kc, const void* vc, void* o, const int* cu_q,
                                 const int* kv_len, const int* block_table, int max_blocks, const int* tiles,
                                 int n_tiles, int T, int nq, int nkv, int num_blocks, float scale, int splits,
                                 float* part_o, float* part_lse, uint32_t* err, cudaStream_t s) {
  if (n_tiles == 0 || T == 0) return;
  if (nq % nkv != 0) throw std::runtime_error("fmha: nq must be a multiple of nkv");
  // Q: [T, nq, D] -> dims {D, nq, T}, box {64, 1, 128}
  const CUtensorMap tq = cached(Key{(uint64_t)q, (uint64_t)T, (uint64_t)nq, 1}, [&] {
    cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)nq, (cuuint64_t)T};
    cuuint64_t str[2] = {(cuuint64_t)D * 2, (cuuint64_t)nq * D * 2};
    cuuint32_t box[3] = {64, 1, BQ};
    return encode(q, 3, dims, str, box);
  });
  // K/V cache: [blocks, nkv, PAGE, D] -> dims {D, PAGE, nkv, blocks}, box {64, PAGE, 1, 1}
  auto cache_map = [&](const void* base) {
    return cached(Key{(uint64_t)base, (uint64_t)num_blocks, (uint64_t)nkv, 2}, [&] {
      cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)PAGE, (cuuint64_t)nkv, (cuuint64_t)num_blocks};
      cuuint64_t str[3] = {(cuuint64_t)D * 2, (cuuint64_t)PAGE * D * 2, (cuuint64_t)nkv * PAGE * D * 2};
      cuuint32_t box[4] = {64, PAGE, 1, 1};
      return encode(base, 4, dims, str, box);
    });
  };
  const CUtensorMap tk = cache_map(kc);
  const CUtensorMap tv = cache_map(vc);
  FmhaArgs a;
  a.o = static_cast<__nv_bfloat16*>(o);
  a.cu_q = cu_q;
  a.kv_len = kv_len;
  a.block_table = block_table;
  a.tiles = reinterpret_cast<const int2*>(tiles);
  a.max_blocks = max_blocks;
  a.nq = nq;
  a.nkv = nkv;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.err = err;
  a.timeout_ns = 2000000000ull;
  a.splits = std::max(1, splits);
  a.part_o = part_o;
  a.part_lse = part_lse;
  if (a.splits > 1 && (!part_o || !part_lse)) throw std::runtime_error("fmha: split-KV needs scratch buffers");
  static SmemLimit limit;
  limit.ensure((const void*)fmha_tc_kernel, Smem::kTotal);
  dim3 grid(n_tiles, nq, a.splits);
  launch_k(fmha_tc_kernel, grid, dim3(kThreads), Smem::kTotal, s, tq, tk, tv, a);
  MBX_CUDA_CHECK(cudaGetLastError());
  if (a.splits > 1) attn_combine_launch(part_o, part_lse, (int64_t)T * nq, a.splits, o, s);
}

}  // namespace mbx
