// Persistent tcgen05 / TMEM GEMM for sm_100a:  C[M,N] = A[M,K] * B[N,K]^T
// (bf16 operands, both K-major as in torch's Linear: activations [T, in],
// weights [out, in]; fp32 accumulation in tensor memory).
//
// Structure (one CTA per SM, 192 threads):
//   warp 0     TMA producer: 128x64 A tile + BNx64 B tile per stage, 128-byte
//              swizzle, S-stage mbarrier ring (full/empty). No multicast.
//   warp 1     TMEM allocator + single-thread tcgen05.mma issuer (M=128,
//              N=BN, K=16 per instruction, 4 per 64-wide k-block); commits
//              free smem stages and signal finished accumulators.
//   warps 2-5  epilogue: tcgen05.ld (32 lanes x 32 columns per warp), convert,
//              store; double-buffered accumulators (2 x BN TMEM columns) so the
//              epilogue of tile i overlaps the mainloop of tile i+1.
// Work units = (m-block, n-block, k-split), strided over the persistent grid.
// split_k > 1 writes fp32 partials that a reduce kernel folds (decode shapes
// with few output tiles).
//
// Every mbarrier wait is bounded (%globaltimer); on timeout the CTA records an
// error word, drains its own in-flight TMA/MMA, frees TMEM and exits.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>

#include <algorithm>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>

#include "../kernels.h"
#include "tcgen05.cuh"

namespace mbx {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int kThreads = 192;
constexpr int kEpiWarps = 4;

// kEpiSwapF32Partial: the kernel runs on swapped operands (A = weights
// [N_w, K], B = activations [M_tok, K], tile rows = output features, tile
// columns = tokens) and writes fp32 partials transposed to [split][token][feature].
enum EpiMode : int { kEpiBf16 = 0, kEpiF32Partial = 1, kEpiBf16AddResidual = 2, kEpiPushRS = 3, kEpiSwapF32Partial = 4 };

struct GemmArgs {
  void* out;             // bf16 C (ldc) or fp32 partials [splits][M][N]
  const __nv_bfloat16* residual;  // kEpiBf16AddResidual: C = acc + residual (ld = ldc)
  int64_t ldc;
  int M, N, K;
  int num_m, num_n, splits, kb_per_split, kb_total;
  uint32_t* err;
  uint64_t timeout_ns;
  // kEpiPushRS: row r of C goes to owner r / Mo's fused region A, slot `rank`;
  // with push_all every rank receives every row (slot `rank` of [M, N] slots)
  ArCtx ar;
  int Mo;
  int push_all;
  // Sequence-parallel all-gather consumer: before the first load of m-tile m
  // the producer waits until every owner of its rows (row / ag_Mo) has
  // released ag_flags[owner] >= *ag_epoch_word (nullptr = no wait).
  const uint32_t* ag_flags;
  const uint32_t* ag_epoch_word;
  int ag_Mo;
  // split-K: per-tile arrival counters (zeroed once; the last CTA of a tile
  // resets its counter) and the final bf16 output of the in-kernel reduction
  uint32_t* tile_counters;
  __nv_bfloat16* final_out;
  int64_t final_ld;
};

MBX_DEVICE char* fused_half(const ArCtx& c, char* base, uint32_t epoch) {
  return base + c.fuse_off + (uint64_t)(epoch & 1u) * c.fuse_half_bytes;
}

// ---------------------------------------------------------------------------
// Peer-push epilogue (GEMM -> allreduce / reduce-scatter), shared by the
// single-CTA and the CTA-pair kernels. Each epilogue warp owns 32 rows of a
// tile. Rows go to every rank's fused half (push-all: slot `rank` of
// [W][M][N]) or to the row owner's (owner push: slot `rank` of [W][Mo][N]).
// ---------------------------------------------------------------------------
struct PushDst {
  char* all[kMaxRanks];  // push-all: this rank's slot in every rank's buffer, rank-staggered; else nullptr
};

MBX_DEVICE void push_dst_init(const GemmArgs& args, uint32_t fepoch, PushDst& d) {
#pragma unroll
  for (int j = 0; j < kMaxRanks; ++j) {
    const int r = (args.ar.rank + j) % max(1, args.ar.world);
    d.all[j] = (j < args.ar.world && args.push_all)
                   ? fused_half(args.ar, args.ar.bufs[r], fepoch) + (uint64_t)args.ar.rank * args.M * args.N * 2
                   : nullptr;
  }
}

// The 8 rows a lane flushes (row k*4 + lane/8 of the warp's 32, whose first
// global row is row0): byte offsets from PushDst (push-all) or the owner's
// destination row (owner push); ~0 / nullptr past M.
struct PushRows {
  char* row[8];
  uint64_t off[8];
};

MBX_DEVICE void push_rows_init(const GemmArgs& args, uint32_t fepoch, int row0, int lane, PushRows& pr) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int grow2 = row0 + k * 4 + (lane >> 3);
    pr.row[k] = nullptr;
    pr.off[k] = ~0ull;
    if (grow2 < args.M) {
      if (args.push_all) {
        pr.off[k] = (uint64_t)grow2 * args.N * 2;
      } else {
        const int owner = grow2 / args.Mo;
        const int lrow = grow2 - owner * args.Mo;
        pr.row[k] = fused_half(args.ar, args.ar.bufs[owner], fepoch) +
                    (uint64_t)(args.ar.rank * args.Mo + lrow) * args.N * 2;
      }
    }
  }
}

// Stage this warp's 32 rows x 32 columns (chunk c0 of a tile starting at
// column col0; bf16, 64 B per row) into a [32 x 128 B] tile (16-byte units
// XOR-swizzled by row); every second chunk, write 4 full 128-byte row
// segments per store instruction to the destinations (NVLink moves whole
// lines instead of 16-byte pieces of 32 different rows).
template <int BN>
MBX_DEVICE void push_chunk(const GemmArgs& args, uint8_t* stg, const uint32_t (&r)[32], int c0, int col0,
                           const PushRows& pr, const PushDst& d, int lane) {
  const int half64 = (c0 >> 5) & 1;
  {
    float f[8];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = __uint_as_float(r[g * 8 + j]);
      const int unit = half64 * 4 + g;
      *reinterpret_cast<uint4*>(stg + lane * 128 + ((unit ^ (lane & 7)) << 4)) = pack_from<__nv_bfloat16>(f);
    }
  }
  if (half64 == 1 || c0 + 32 >= BN) {
    __syncwarp();
    const int unit = lane & 7;
    const int col = col0 + (c0 & ~63) + unit * 8;  // this lane's 8 columns of the staged 64
    const bool col_ok = col < args.N && (half64 == 1 || unit < 4);
    const uint64_t col_b = (uint64_t)col * 2;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int srow = k * 4 + (lane >> 3);
      if (!col_ok) continue;
      if (args.push_all) {
        if (pr.off[k] == ~0ull) continue;
        const uint4 v = *reinterpret_cast<const uint4*>(stg + srow * 128 + ((unit ^ (srow & 7)) << 4));
        const uint64_t off = pr.off[k] + col_b;
#pragma unroll
        for (int j = 0; j < kMaxRanks; ++j)
          if (d.all[j] != nullptr) *reinterpret_cast<uint4*>(d.all[j] + off) = v;
      } else {
        if (pr.row[k] == nullptr) continue;
        const uint4 v = *reinterpret_cast<const uint4*>(stg + srow * 128 + ((unit ^ (srow & 7)) << 4));
        *reinterpret_cast<uint4*>(pr.row[k] + col_b) = v;
      }
    }
    __syncwarp();
  }
}

// This CTA's rows are stored; the last CTA of the grid releases one flag per
// rank (epoch fepoch) after every CTA's pushes (called by all epilogue warps).
MBX_DEVICE void push_release(const GemmArgs& args, uint32_t fepoch, int warp, int lane, volatile int* abort) {
  tc::named_bar_sync(1, kEpiWarps * 32);
  if (warp == 2 && lane == 0 && !*abort) {
    fence_acq_rel_sys();
    const uint32_t prev = atomicAdd(args.ar.state + kStFuseGemmDone, 1u);
    if (prev == gridDim.x - 1) {
      fence_acq_rel_sys();
      args.ar.state[kStFuseGemmDone] = 0;
      for (int o = 0; o < args.ar.world; ++o)
        st_release_sys(reinterpret_cast<uint32_t*>(args.ar.bufs[o] + kTileFlagOff) + args.ar.rank, fepoch);
    }
  }
}

// TMEM columns per accumulator buffer (power of two >= BN, so both buffers
// start on aligned columns and the allocation is a power of two).
template <int BN>
struct Tmem {
  static constexpr int kAccStride = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
  static constexpr int kCols = 2 * kAccStride;
};

template <int BN, int STAGES, bool kStaging = false>
struct Smem {
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOff = STAGES * kStageBytes;
  // push epilogue: per epilogue warp a [32 rows x 128 B] staging tile
  static constexpr int kStageOut = kBarOff + 256;
  static constexpr int kTotal = kStageOut + (kStaging ? 4 * 32 * 128 : 0) + 1024;  // + alignment slack
};

MBX_DEVICE void set_err(uint32_t* err, uint32_t code, volatile int* abort) {
  *abort = 1;
  if (err) atomicCAS(err, 0u, code);
}

MBX_DEVICE void store_row_bf16(__nv_bfloat16* dst, const uint32_t (&r)[32], int ncols_valid,
                               const __nv_bfloat16* res) {
  // r holds 32 fp32 bit patterns of consecutive columns; write ncols_valid
  // (multiple of 8) of them as bf16 in 16-byte packs.
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    if (g * 8 < ncols_valid) {
      float f[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = __uint_as_float(r[g * 8 + j]);
      if (res) {
        float rr[8] = {};
        unpack_add<__nv_bfloat16>(*reinterpret_cast<const uint4*>(res + g * 8), rr);
        // round the GEMM result first: same as a separate bf16 add
        const uint4 pb = pack_from<__nv_bfloat16>(f);
        float q[8] = {};
        unpack_add<__nv_bfloat16>(pb, q);
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = q[j] + rr[j];
      }
      *reinterpret_cast<uint4*>(dst + g * 8) = pack_from<__nv_bfloat16>(f);
    }
  }
}

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        GemmArgs args) {
  using L = Smem<BN, STAGES, EPI == kEpiPushRS>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled tiles.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;   // [2]
  uint64_t* tempty = tfull + 2;       // [2]
  uint64_t* mma_done = tempty + 2;    // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int units = args.num_m * args.num_n * args.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(&tfull[a], 1);
      tc::mbar_init(&tempty[a], kEpiWarps);
    }
    tc::mbar_init(mma_done, 1);
    *abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, Tmem<BN>::kCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // set-up above overlaps the previous kernel; its outputs are read below

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (tc::elect_one()) {
      tc::tma_prefetch_desc(&tmA);
      tc::tma_prefetch_desc(&tmB);
      const uint32_t ag_epoch = args.ag_flags ? *reinterpret_cast<const volatile uint32_t*>(args.ag_epoch_word) : 0u;
      int ready_m = -1;
      uint32_t it = 0;
      for (int u = blockIdx.x; u < units && !*abort; u += gridDim.x) {
        const int m = u % args.num_m;
        const int rest = u / args.num_m;
        const int n = rest % args.num_n;
        const int ks = rest / args.num_n;
        const int kb0 = ks * args.kb_per_split;
        const int kb1 = min(args.kb_total, kb0 + args.kb_per_split);
        if (args.ag_flags != nullptr && m != ready_m) {
          // rows [m*BM, m*BM+BM) come from their owners' all-gather pushes
          const int o0 = (m * BM) / args.ag_Mo;
          const int o1 = (min(args.M, m * BM + BM) - 1) / args.ag_Mo;
          bool ok = true;
          for (int o = o0; o <= o1 && ok; ++o) ok = wait_flag_geq(args.ag_flags + o, ag_epoch, args.timeout_ns);
          if (!ok) {
            set_err(args.err, 4, abort);
            break;
          }
          // the rows were written by peers' generic-proxy stores; TMA reads
          // through the async proxy
          asm volatile("fence.proxy.async.global;" ::: "memory");
          ready_m = m;
        }
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!tc::mbar_wait(&empty[s], ph ^ 1, abort, args.timeout_ns)) {
            set_err(args.err, 1, abort);
            break;
          }
          uint8_t* sa = smem + s * L::kStageBytes;
          uint8_t* sb = sa + L::kABytes;
          tc::mbar_arrive_expect_tx(&full[s], L::kStageBytes);
          tc::tma_load_2d(sa, &tmA, &full[s], kb * BK, m * BM);
          tc::tma_load_2d(sb, &tmB, &full[s], kb * BK, n * BN);
        }
      }
      // Drain: wait for the last (up to STAGES) loads this thread issued.
      const uint32_t first = it > (uint32_t)STAGES ? it - STAGES : 0;
      for (uint32_t j = first; j < it; ++j) {
        volatile int never = 0;
        tc::mbar_wait(&full[j % STAGES], (j / STAGES) & 1, &never, 200000000ull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (tc::elect_one()) {
      constexpr uint32_t idesc = tc::idesc_bf16_f32(BM, BN);
      uint32_t it = 0, t = 0;
      for (int u = blockIdx.x; u < units && !*abort; u += gridDim.x, ++t) {
        const int rest = u / args.num_m;
        const int ks = rest / args.num_n;
        const int kb0 = ks * args.kb_per_split;
        const int kb1 = min(args.kb_total, kb0 + args.kb_per_split);
        const int acc = t & 1;
        const uint32_t aph = (t >> 1) & 1;
        if (!tc::mbar_wait(&tempty[acc], aph ^ 1, abort, args.timeout_ns)) {
          set_err(args.err, 2, abort);
          break;
        }
        tc::tc_fence_after();
        const uint32_t d = tmem_base + acc * Tmem<BN>::kAccStride;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!tc::mbar_wait(&full[s], ph, abort, args.timeout_ns)) {
            set_err(args.err, 2, abort);
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t sa = tc::smem_u32(smem + s * L::kStageBytes);
          const uint32_t sb = sa + L::kABytes;
          const uint64_t da = tc::sw128_kmajor_desc(sa);
          const uint64_t db = tc::sw128_kmajor_desc(sb);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // advance 16 bf16 = 32 bytes (2 in descriptor units) along K
            tc::mma_bf16(d, da + 2 * k, db + 2 * k, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          tc::mma_commit(&empty[s]);
        }
        if (!ok) break;
        tc::mma_commit(&tfull[acc]);
      }
      // All issued MMAs complete before TMEM is released.
      tc::mma_commit(mma_done);
      volatile int never = 0;
      tc::mbar_wait(mma_done, 0, &never, 200000000ull);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_in_tile = quad * 32 + lane;
    const uint32_t fepoch =
        EPI == kEpiPushRS ? *reinterpret_cast<volatile uint32_t*>(args.ar.state + kStFuseEpoch) + 1u : 0u;
    // push epilogue: destination bases fixed for the whole launch
    PushDst pdst;
    if (EPI == kEpiPushRS) push_dst_init(args, fepoch, pdst);
    uint32_t t = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++t) {
      const int m = u % args.num_m;
      const int rest = u / args.num_m;
      const int n = rest % args.num_n;
      const int ks = rest / args.num_n;
      const int acc = t & 1;
      const uint32_t aph = (t >> 1) & 1;
      if (!tc::mbar_wait(&tfull[acc], aph, abort, args.timeout_ns)) {
        if (lane == 0) set_err(args.err, 3, abort);
        break;
      }
      tc::tc_fence_after();
      const int grow = m * BM + row_in_tile;
      const bool row_ok = grow < args.M;
      PushRows prows;
      if (EPI == kEpiPushRS) push_rows_init(args, fepoch, m * BM + quad * 32, lane, prows);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        tc::tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * Tmem<BN>::kAccStride + c0, r);
        tc::tmem_ld_wait();
        const int gcol = n * BN + c0;
        const int valid = min(32, args.N - gcol);
        if (EPI == kEpiPushRS)
          push_chunk<BN>(args, smem + L::kStageOut + (warp - 2) * (32 * 128), r, c0, n * BN, prows, pdst, lane);
        if (EPI != kEpiPushRS && row_ok && valid > 0) {
          if (EPI == kEpiPushRS) {
            // staged below (coalesced 128-byte row segments)
          } else if (EPI == kEpiSwapF32Partial) {
            // row = output feature, columns = tokens: store column j of the tile as
            // partial[ks][token][feature] (consecutive threads = consecutive features)
            float* base = static_cast<float*>(args.out) + (int64_t)ks * args.N * args.M + grow;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < valid) base[(int64_t)(gcol + j) * args.M] = __uint_as_float(r[j]);
          } else if (EPI == kEpiF32Partial) {
            float* dst = static_cast<float*>(args.out) + ((int64_t)ks * args.M + grow) * args.N + gcol;
#pragma unroll
            for (int g = 0; g < 8; ++g)
              if (g * 4 < valid)
                *reinterpret_cast<uint4*>(dst + g * 4) = make_uint4(r[g * 4], r[g * 4 + 1], r[g * 4 + 2], r[g * 4 + 3]);
          } else {
            __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(args.out) + (int64_t)grow * args.ldc + gcol;
            const __nv_bfloat16* res =
                EPI == kEpiBf16AddResidual ? args.residual + (int64_t)grow * args.ldc + gcol : nullptr;
            store_row_bf16(dst, r, valid, res);
          }
        }
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&tempty[acc]);
      if ((EPI == kEpiF32Partial || EPI == kEpiSwapF32Partial) && args.splits > 1 && args.tile_counters) {
        // In-kernel split-K: the last CTA to finish a tile sums every split's
        // partial (split order 0..S-1, deterministic) and writes bf16 output.
        volatile uint32_t* s_last = reinterpret_cast<volatile uint32_t*>(tmem_slot + 2);
        tc::named_bar_sync(1, kEpiWarps * 32);
        if (warp == 2 && lane == 0) {
          __threadfence();
          const int tile = m + n * args.num_m;
          const uint32_t prev = atomicAdd(args.tile_counters + tile, 1u);
          const bool last = prev == (uint32_t)(args.splits - 1);
          if (last) {
            args.tile_counters[tile] = 0;
            __threadfence();
          }
          *s_last = last ? 1u : 0u;
        }
        tc::named_bar_sync(1, kEpiWarps * 32);
        if (*s_last) {
          const float* ws = static_cast<const float*>(args.out);
          const int64_t plane = (int64_t)args.M * args.N;
          if (EPI == kEpiSwapF32Partial) {
            // row = feature `grow`, columns = tokens: C[token][feature]
            if (row_ok) {
              const int t_end = min(args.N, n * BN + BN);
              for (int tk = n * BN; tk < t_end; ++tk) {
                float acc2 = 0.f;
                for (int sp = 0; sp < args.splits; ++sp)
                  acc2 += __ldcg(ws + sp * plane + (int64_t)tk * args.M + grow);
                __nv_bfloat16* dst = args.final_out + (int64_t)tk * args.final_ld + grow;
                if (args.residual)
                  acc2 = __bfloat162float(__float2bfloat16(acc2)) +
                         __bfloat162float(args.residual[(int64_t)tk * args.final_ld + grow]);
                *dst = __float2bfloat16(acc2);
              }
            }
          } else if (row_ok) {
            const int c_end = min(args.N, n * BN + BN);
            for (int col = n * BN; col < c_end; col += 8) {
              float f[8] = {};
              for (int sp = 0; sp < args.splits; ++sp) {
                const float4* src = reinterpret_cast<const float4*>(ws + sp * plane + (int64_t)grow * args.N + col);
                const float4 lo = __ldcg(src), hi = __ldcg(src + 1);
                f[0] += lo.x; f[1] += lo.y; f[2] += lo.z; f[3] += lo.w;
                f[4] += hi.x; f[5] += hi.y; f[6] += hi.z; f[7] += hi.w;
              }
              uint32_t rr[32];
#pragma unroll
              for (int j = 0; j < 8; ++j) rr[j] = __float_as_uint(f[j]);
              __nv_bfloat16* dst = args.final_out + (int64_t)grow * args.final_ld + col;
              const __nv_bfloat16* res = args.residual ? args.residual + (int64_t)grow * args.final_ld + col : nullptr;
              store_row_bf16(dst, rr, 8, res);
            }
          }
        }
      }
    }
    if (EPI == kEpiPushRS) push_release(args, fepoch, warp, lane, abort);
  }

  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 1) tc::tmem_dealloc(tmem_base, Tmem<BN>::kCols);
}

// Sum split-K partials (fp32, in split order) into bf16 C, optional residual.
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int splits, int64_t MN, int N,
                                     __nv_bfloat16* __restrict__ out, int64_t ldc,
                                     const __nv_bfloat16* __restrict__ residual) {
  pdl_wait();
  const int64_t nvec = MN / 4;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += (int64_t)gridDim.x * blockDim.x) {
    float4 acc = reinterpret_cast<const float4*>(part)[v];
    for (int s = 1; s < splits; ++s) {
      const float4 p = reinterpret_cast<const float4*>(part + s * MN)[v];
      acc.x += p.x;
      acc.y += p.y;
      acc.z += p.z;
      acc.w += p.w;
    }
    const int64_t e = v * 4;
    const int64_t row = e / N, col = e % N;
    __nv_bfloat16* o = out + row * ldc + col;
    __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y);
    __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z, acc.w);
    if (residual) {
      const __nv_bfloat16* rr = residual + row * ldc + col;
      float2 a = __bfloat1622float2(lo), b = __bfloat1622float2(hi);
      float2 ra = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(rr));
      float2 rb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(rr + 2));
      lo = __floats2bfloat162_rn(a.x + ra.x, a.y + ra.y);
      hi = __floats2bfloat162_rn(b.x + rb.x, b.y + rb.y);
    }
    reinterpret_cast<__nv_bfloat162*>(o)[0] = lo;
    reinterpret_cast<__nv_bfloat162*>(o)[1] = hi;
  }
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

struct MapKey {
  uint64_t ptr, rows, cols, ld, box_rows;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rows == o.rows && cols == o.cols && ld == o.ld && box_rows == o.box_rows;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    uint64_t h = k.ptr * 0x9E3779B97F4A7C15ull;
    h ^= k.rows + 0x9E3779B97F4A7C15ull + (h << 6) + (h >> 2);
    h ^= k.cols + 0x9E3779B97F4A7C15ull + (h << 6) + (h >> 2);
    h ^= k.ld + 0x9E3779B97F4A7C15ull + (h << 6) + (h >> 2);
    h ^= k.box_rows + 0x9E3779B97F4A7C15ull + (h << 6) + (h >> 2);
    return (size_t)h;
  }
};

std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

// 2-D bf16 row-major [rows, cols] (row stride ld elements), box = box_rows x 64,
// 128-byte swizzle. Out-of-range rows/columns of a box read as zero.
CUtensorMap make_map(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  MapKey key{(uint64_t)ptr, (uint64_t)rows, (uint64_t)cols, (uint64_t)ld, (uint64_t)box_rows};
  {
    std::lock_guard<std::mutex> g(g_map_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) return it->second;
  }
  if (((uint64_t)ptr & 15) != 0) throw std::runtime_error("gemm: operand base must be 16-byte aligned");
  if ((ld * 2) % 16 != 0) throw std::runtime_error("gemm: row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  std::lock_guard<std::mutex> g(g_map_mu);
  if (g_maps.size() > 8192) g_maps.clear();
  g_maps.emplace(key, m);
  return m;
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
  }
  return n;
}

// ==========================================================================
// CTA-pair GEMM (cta_group::2): a cluster of two CTAs computes one 256 x BN
// tile. CTA r stages rows [256m + 128r, +128) of A and rows [BN n + BN/2 r,
// +BN/2) of B in its own shared memory; the leader (r = 0) issues M=256
// tcgen05.mma over both CTAs' tiles, so each SM streams half of B per k-step
// instead of all of it (the per-SM operand traffic drops from 48 KB to 32 KB
// per 64-deep k-block at BN = 256). Accumulator rows land in each CTA's own
// TMEM; each CTA's epilogue stores its 128 rows. Plain / residual epilogues.
// Barriers: full[s] lives in the leader (both CTAs' loads count on it; the
// leader expects both CTAs' bytes), empty[s] and tfull[acc] in both CTAs (the
// MMA commit arrives on both), tempty[acc] in the leader (both CTAs'
// epilogue warps arrive). Every wait is bounded; the only unbounded waits are
// the two cluster barriers, at the start and at the end, which every thread
// of both CTAs reaches on every path.
// ==========================================================================
template <int BN, int STAGES, bool kStaging = false>
struct Smem2 {
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = (BN / 2) * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOff = STAGES * kStageBytes;
  // push epilogue: per epilogue warp a [32 rows x 128 B] staging tile
  static constexpr int kStageOut = kBarOff + 256;
  static constexpr int kTotal = kStageOut + (kStaging ? 4 * 32 * 128 : 0) + 1024;
};

template <int BN, int STAGES, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm2_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         GemmArgs args) {
  using L = Smem2<BN, STAGES, EPI == kEpiPushRS>;
  static_assert(BN % 32 == 0 && BN <= 256, "pair tile width");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;   // [2]
  uint64_t* tempty = tfull + 2;       // [2]
  uint64_t* mma_done = tempty + 2;    // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = tc::cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int num_m2 = (args.M + 2 * BM - 1) / (2 * BM);
  const int units = num_m2 * args.num_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(&tfull[a], 1);
      tc::mbar_init(&tempty[a], 2 * kEpiWarps);
    }
    tc::mbar_init(mma_done, 1);
    *abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc_pair(tmem_slot, Tmem<BN>::kCols);
    tc::tmem_relinquish_pair();
  }
  tc::tc_fence_before();
  __syncwarp();
  tc::cluster_sync();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // set-up above overlaps the previous kernel; its outputs are read below

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (tc::elect_one()) {
      tc::tma_prefetch_desc(&tmA);
      tc::tma_prefetch_desc(&tmB);
      uint32_t it = 0;
      for (int u = pair; u < units && !*abort; u += npairs) {
        const int m = u % num_m2;
        const int n = u / num_m2;
        for (int kb = 0; kb < args.kb_total; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!tc::mbar_wait(&empty[s], ph ^ 1, abort, args.timeout_ns)) {
            set_err(args.err, 5, abort);
            break;
          }
          uint8_t* sa = smem + s * L::kStageBytes;
          uint8_t* sb = sa + L::kABytes;
          if (rank == 0) tc::mbar_arrive_expect_tx(&full[s], 2 * L::kStageBytes);
          tc::tma_load_2d_pair(sa, &tmA, &full[s], kb * BK, m * 2 * BM + (int)rank * BM);
          tc::tma_load_2d_pair(sb, &tmB, &full[s], kb * BK, n * BN + (int)rank * (BN / 2));
        }
      }
      if (rank == 0) {
        // Drain: the last (up to STAGES) stages' loads of both CTAs have landed
        // (the leader's full barriers count both) before the final cluster
        // barrier lets either CTA exit.
        const uint32_t first = it > (uint32_t)STAGES ? it - STAGES : 0;
        for (uint32_t j = first; j < it; ++j) {
          volatile int never = 0;
          tc::mbar_wait(&full[j % STAGES], (j / STAGES) & 1, &never, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (rank == 0 && tc::elect_one()) {
      constexpr uint32_t idesc = tc::idesc_bf16_f32(2 * BM, BN);
      uint32_t it = 0, t = 0;
      for (int u = pair; u < units && !*abort; u += npairs, ++t) {
        const int acc = t & 1;
        const uint32_t aph = (t >> 1) & 1;
        if (!tc::mbar_wait(&tempty[acc], aph ^ 1, abort, args.timeout_ns)) {
          set_err(args.err, 6, abort);
          break;
        }
        tc::tc_fence_after();
        const uint32_t d = tmem_base + acc * Tmem<BN>::kAccStride;
        bool ok = true;
        for (int kb = 0; kb < args.kb_total; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!tc::mbar_wait(&full[s], ph, abort, args.timeout_ns)) {
            set_err(args.err, 6, abort);
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t sa = tc::smem_u32(smem + s * L::kStageBytes);
          const uint64_t da = tc::sw128_kmajor_desc(sa);
          const uint64_t db = tc::sw128_kmajor_desc(sa + L::kABytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) tc::mma_bf16_pair(d, da + 2 * k, db + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          tc::mma_commit_pair(&empty[s], 0x3);
        }
        if (!ok) break;
        tc::mma_commit_pair(&tfull[acc], 0x3);
      }
      // every issued MMA completes before the pair's TMEM is released
      tc::mma_commit_pair(mma_done, 0x1);
      volatile int never = 0;
      tc::mbar_wait(mma_done, 0, &never, 200000000ull);
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quad = warp & 3;
    const uint32_t fepoch =
        EPI == kEpiPushRS ? *reinterpret_cast<volatile uint32_t*>(args.ar.state + kStFuseEpoch) + 1u : 0u;
    PushDst pdst;
    if (EPI == kEpiPushRS) push_dst_init(args, fepoch, pdst);
    uint32_t t = 0;
    for (int u = pair; u < units; u += npairs, ++t) {
      const int m = u % num_m2;
      const int n = u / num_m2;
      const int acc = t & 1;
      const uint32_t aph = (t >> 1) & 1;
      if (!tc::mbar_wait(&tfull[acc], aph, abort, args.timeout_ns)) {
        if (lane == 0) set_err(args.err, 7, abort);
        break;
      }
      tc::tc_fence_after();
      const int grow = m * 2 * BM + (int)rank * BM + quad * 32 + lane;
      const bool row_ok = grow < args.M;
      PushRows prows;
      if (EPI == kEpiPushRS) push_rows_init(args, fepoch, m * 2 * BM + (int)rank * BM + quad * 32, lane, prows);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        tc::tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * Tmem<BN>::kAccStride + c0, r);
        tc::tmem_ld_wait();
        const int gcol = n * BN + c0;
        const int valid = min(32, args.N - gcol);
        if (EPI == kEpiPushRS) {
          push_chunk<BN>(args, smem + L::kStageOut + (warp - 2) * (32 * 128), r, c0, n * BN, prows, pdst, lane);
        } else if (row_ok && valid > 0) {
          __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(args.out) + (int64_t)grow * args.ldc + gcol;
          const __nv_bfloat16* res =
              EPI == kEpiBf16AddResidual ? args.residual + (int64_t)grow * args.ldc + gcol : nullptr;
          store_row_bf16(dst, r, valid, res);
        }
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0) tc::mbar_arrive(&tempty[acc]);
        else tc::mbar_arrive_remote(&tempty[acc], 0);
      }
    }
    if (EPI == kEpiPushRS) push_release(args, fepoch, warp, lane, abort);
  }

  tc::tc_fence_before();
  __syncwarp();
  tc::cluster_sync();
  tc::tc_fence_after();
  if (warp == 1) tc::tmem_dealloc_pair(tmem_base, Tmem<BN>::kCols);
}

template <int BN, int STAGES, int EPI>
void launch_pair_cfg(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int grid, cudaStream_t s) {
  using L = Smem2<BN, STAGES, EPI == kEpiPushRS>;
  auto kern = gemm2_tcgen05_kernel<BN, STAGES, EPI>;
  static SmemLimit limit;
  limit.ensure((const void*)kern, L::kTotal);
  launch_k(kern, dim3(grid), dim3(kThreads), L::kTotal, s, ta, tb, a);
}

template <int BN, int STAGES, int EPI>
void launch_cfg(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int grid, cudaStream_t s) {
  using L = Smem<BN, STAGES, EPI == kEpiPushRS>;
  auto kern = gemm_tcgen05_kernel<BN, STAGES, EPI>;
  static SmemLimit limit;
  limit.ensure((const void*)kern, L::kTotal);
  launch_k(kern, dim3(grid), dim3(kThreads), L::kTotal, s, ta, tb, a);
}

template <int EPI>
void launch_bn(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int grid, cudaStream_t s) {
  if (EPI == kEpiSwapF32Partial) {
    if (bn == 32) launch_cfg<32, 8, EPI>(ta, tb, a, grid, s);
    else launch_cfg<64, 8, EPI>(ta, tb, a, grid, s);
    return;
  }
  switch (bn) {
    case 256: launch_cfg<256, 4, EPI>(ta, tb, a, grid, s); break;
    case 224: launch_cfg<224, EPI == kEpiPushRS ? 4 : 5, EPI>(ta, tb, a, grid, s); break;
    case 192: launch_cfg<192, 5, EPI>(ta, tb, a, grid, s); break;
    case 160: launch_cfg<160, 5, EPI>(ta, tb, a, grid, s); break;
    case 128: launch_cfg<128, 6, EPI>(ta, tb, a, grid, s); break;
    default: launch_cfg<64, 8, EPI>(ta, tb, a, grid, s); break;
  }
}

GemmPlan plan_for(int64_t M, int64_t N, int64_t K, int sms) {
  GemmPlan p;
  const int64_t num_m = (M + BM - 1) / BM;
  const int64_t kb_total = (K + BK - 1) / BK;
  // Tile width by estimated time: waves of the persistent grid x per-tile
  // cost. Narrow tiles pay more shared-memory traffic per FLOP (A is
  // re-read for every BN columns), which the factor models.
  static const int kBN[] = {256, 224, 192, 160, 128};
  static const double kCost[] = {1.00, 1.00, 1.02, 1.10, 1.25};
  double best = 1e30;
  for (int i = 0; i < 5; ++i) {
    const int bn = kBN[i];
    const int64_t tiles = num_m * ((N + bn - 1) / bn);
    const int64_t waves = (tiles + sms - 1) / sms;
    const double t = (double)waves * bn * kCost[i];
    if (t < best * 0.999) {
      best = t;
      p.bn = bn;
    }
  }
  const int64_t tiles = num_m * ((N + p.bn - 1) / p.bn);
  p.splits = 1;
  if (tiles * 2 <= sms && kb_total >= 8) {
    // few output tiles (decode, narrow TP shards): split K so every SM streams weights
    if (p.bn > 128) {
      p.bn = 128;
    }
    const int64_t t128 = num_m * ((N + 127) / 128);
    const int64_t s = std::min<int64_t>(sms / std::max<int64_t>(1, t128), kb_total / 4);
    p.splits = (int)std::max<int64_t>(1, std::min<int64_t>(s, 16));
  }
  // every split gets at least one k-block
  const int64_t per = (kb_total + p.splits - 1) / p.splits;
  p.splits = (int)((kb_total + per - 1) / per);
  return p;
}

// Decode shapes (M <= 64 tokens): operands swapped, tokens on the N side.
GemmPlan swap_plan(int64_t M, int64_t N, int64_t K, int sms) {
  GemmPlan p;
  p.bn = M <= 32 ? 32 : 64;
  const int64_t kb_total = (K + BK - 1) / BK;
  const int64_t num_f = (N + BM - 1) / BM;
  const int64_t want = std::max<int64_t>(1, (sms + num_f - 1) / num_f);
  int64_t sp = std::min<int64_t>(want, std::max<int64_t>(1, kb_total / 2));
  sp = std::min<int64_t>(sp, 32);
  const int64_t per = (kb_total + sp - 1) / sp;
  p.splits = (int)((kb_total + per - 1) / per);
  return p;
}

}  // namespace

GemmPlan gemm_plan(int64_t M, int64_t N, int64_t K) {
  if (M <= 64 && N % 4 == 0) {
    GemmPlan sp = swap_plan(M, N, K, num_sms());
    if (sp.splits > 1) return sp;
  }
  return plan_for(M, N, K, num_sms());
}

static int pair_gemm_bn(int64_t M, int64_t N, const GemmPlan& p, int sms);

namespace {
GemmArgs push_args(const ArCtx& c, int64_t M, int64_t N, int64_t K, int bn, int64_t Mo, bool push_all, uint32_t* err) {
  GemmArgs a;
  std::memset(&a, 0, sizeof(a));
  a.ldc = N;
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.num_m = (int)((M + BM - 1) / BM);
  a.num_n = (int)((N + bn - 1) / bn);
  a.kb_total = (int)((K + BK - 1) / BK);
  a.splits = 1;
  a.kb_per_split = a.kb_total;
  a.err = err;
  a.timeout_ns = 2000000000ull;
  a.ar = c;
  a.Mo = (int)Mo;
  a.push_all = push_all ? 1 : 0;
  return a;
}

void launch_push_gemm(const ArCtx& c, const void* A, int64_t lda, const void* B, int64_t ldb, int64_t M, int64_t N,
                      int64_t K, int64_t Mo, bool push_all, uint32_t* err, cudaStream_t s) {
  const int sms = num_sms();
  GemmPlan p = plan_for(M, N, K, sms);
  int bn2 = pair_gemm_bn(M, N, p, sms);
  // MBX_PUSH_GEMM_BN=256|192|128 forces the pair tile width of the push GEMM
  // alone (narrower tiles give more waves, whose pushes then overlap later
  // tiles' MMAs; tuning)
  static const int push_bn = [] {
    const char* v = std::getenv("MBX_PUSH_GEMM_BN");
    const int b = v ? std::atoi(v) : 0;
    return (b == 256 || b == 192 || b == 128) ? b : 0;
  }();
  if (push_bn && M >= 2 * BM) bn2 = push_bn;
  if (bn2 > 0) {
    // CTA-pair tiles, same tile choice as the plain GEMM of this shape
    GemmArgs pa = push_args(c, M, N, K, bn2, Mo, push_all, err);
    const CUtensorMap ta2 = make_map(A, M, K, lda, BM);
    const CUtensorMap tb2 = make_map(B, N, K, ldb, bn2 / 2);
    const int units2 = (int)((M + 2 * BM - 1) / (2 * BM)) * pa.num_n;
    const int grid2 = 2 * std::min(units2, sms / 2);
    if (bn2 == 256) launch_pair_cfg<256, 6, kEpiPushRS>(ta2, tb2, pa, grid2, s);
    else if (bn2 == 192) launch_pair_cfg<192, 7, kEpiPushRS>(ta2, tb2, pa, grid2, s);
    else launch_pair_cfg<128, 8, kEpiPushRS>(ta2, tb2, pa, grid2, s);
    MBX_CUDA_CHECK(cudaGetLastError());
    return;
  }
  GemmArgs a = push_args(c, M, N, K, p.bn, Mo, push_all, err);
  const CUtensorMap ta = make_map(A, M, K, lda, BM);
  const CUtensorMap tb = make_map(B, N, K, ldb, p.bn);
  const int units = a.num_m * a.num_n;
  launch_bn<kEpiPushRS>(p.bn, ta, tb, a, std::min(units, sms), s);
  MBX_CUDA_CHECK(cudaGetLastError());
}
}  // namespace

void gemm_ar_rmsnorm_launch(const ArCtx& c, const void* A, int64_t lda, const void* B, int64_t ldb, int64_t M,
                            int64_t N, int64_t K, void* residual, const void* norm_w, void* out, float eps,
                            uint32_t* err, int max_blocks, bool push_all, cudaStream_t s) {
  if (M == 0) return;
  if (K % 8 != 0 || N % 8 != 0) throw std::runtime_error("gemm_ar: K and N must be multiples of 8");
  const int W = c.world;
  const int64_t Mo = (M + W - 1) / W;
  const uint64_t need = push_all ? (uint64_t)W * M * N * 2 : (uint64_t)W * Mo * N * 2 + (uint64_t)M * N * 2;
  if (c.fuse_half_bytes == 0 || need > c.fuse_half_bytes)
    throw std::runtime_error("gemm_ar: message needs " + std::to_string(need) + " bytes of fused buffer, have " +
                             std::to_string(c.fuse_half_bytes));
  launch_push_gemm(c, A, lda, B, ldb, M, N, K, Mo, push_all, err, s);
  if (push_all) fused_allsum_norm_launch(c, (int)M, (int)N, residual, norm_w, out, eps, max_blocks, s);
  else fused_rs_norm_launch(c, (int)M, (int)N, (int)Mo, residual, norm_w, out, eps, max_blocks, s);
}

void gemm_push_launch(const ArCtx& c, const void* A, int64_t lda, const void* B, int64_t ldb, int64_t M, int64_t N,
                      int64_t K, bool push_all, uint32_t* err, cudaStream_t s) {
  if (M == 0) return;
  if (K % 8 != 0 || N % 8 != 0) throw std::runtime_error("gemm_push: K and N must be multiples of 8");
  const int W = c.world;
  const int64_t Mo = (M + W - 1) / W;
  const uint64_t need = push_all ? (uint64_t)W * M * N * 2 : (uint64_t)W * Mo * N * 2 + (uint64_t)M * N * 2;
  if (c.fuse_half_bytes == 0 || need > c.fuse_half_bytes)
    throw std::runtime_error("gemm_push: message exceeds the fused buffer");
  launch_push_gemm(c, A, lda, B, ldb, M, N, K, Mo, push_all, err, s);
}

void gemm_rs_launch(const ArCtx& c, const void* A, int64_t lda, const void* B, int64_t ldb, int64_t M, int64_t N,
                    int64_t K, uint32_t* err, cudaStream_t s) {
  if (M == 0) return;
  if (K % 8 != 0 || N % 8 != 0) throw std::runtime_error("gemm_rs: K and N must be multiples of 8");
  const int64_t Mo = (M + c.world - 1) / c.world;
  if ((uint64_t)c.world * Mo * N * 2 > c.fuse_half_bytes)
    throw std::runtime_error("gemm_rs: [" + std::to_string(M) + ", " + std::to_string(N) +
                             "] exceeds the reduce-scatter buffer");
  launch_push_gemm(c, A, lda, B, ldb, M, N, K, Mo, false, err, s);
}

// CTA-pair GEMM selection: MBX_GEMM_2CTA=0 never, =1 whenever M >= 256,
// unset: when its wave cost is lower. A 256x256 pair tile occupies two SMs
// and, per SM, costs 0.85 of a 128x256 single-CTA tile (measured on the 8B
// shapes: down_proj K=14336 98.3 -> 80.7 us, o_proj K=4096 36.9 -> 32.8 us);
// its coarser tiles lose where they fill the pairs worse than the single-CTA
// plan fills the SMs (qkv N=6144: 53.2 vs 51.2 us). This rule picks the
// faster kernel on all eight measured 8B TP=1/2 shapes.
static int pair_gemm_mode() {
  static const int mode = [] {
    const char* v = std::getenv("MBX_GEMM_2CTA");
    if (v == nullptr || v[0] == '\0') return -1;
    return v[0] == '1' ? 1 : 0;
  }();
  return mode;
}

// Pair tile width (256, 192 or 128; 0 = single-CTA tiles). The pair widths
// share the wave-cost model of plan_for: per SM a pair tile reads half of B,
// which the per-width factors credit (0.85 at 256 measured; the narrower pair
// tiles re-read A more often per FLOP, like their single-CTA counterparts).
// MBX_GEMM_2CTA_BN=256|192|128 forces one width (tuning, tests).
static int pair_gemm_bn(int64_t M, int64_t N, const GemmPlan& p, int sms) {
  const int mode = pair_gemm_mode();
  if (mode == 0 || M < 2 * BM || p.splits > 1) return 0;
  static const int forced = [] {
    const char* v = std::getenv("MBX_GEMM_2CTA_BN");
    const int b = v ? std::atoi(v) : 0;
    return (b == 256 || b == 192 || b == 128) ? b : 0;
  }();
  if (forced) return forced;
  static const int kBN[] = {256, 224, 192, 160, 128};
  static const double kCost[] = {1.00, 1.00, 1.02, 1.10, 1.25};
  double c1 = 0.0;
  for (int i = 0; i < 5; ++i)
    if (kBN[i] == p.bn) c1 = kCost[i];
  if (c1 == 0.0) return 0;
  const int64_t tiles1 = ((M + BM - 1) / BM) * ((N + p.bn - 1) / p.bn);
  const double t1 = (double)((tiles1 + sms - 1) / sms) * p.bn * c1;
  static const int kBN2[] = {256, 192, 128};
  static const double kCost2[] = {0.85, 0.88, 1.0};
  const int64_t slots = std::max(1, sms / 2);
  double best = t1;
  int bn2 = 0;
  for (int i = 0; i < 3; ++i) {
    const int64_t pairs = ((M + 2 * BM - 1) / (2 * BM)) * ((N + kBN2[i] - 1) / kBN2[i]);
    const double t2 = (double)((pairs + slots - 1) / slots) * kBN2[i] * kCost2[i];
    if (t2 < best * 0.999) {
      best = t2;
      bn2 = kBN2[i];
    }
  }
  if (mode == 1 && bn2 == 0) bn2 = 256;
  return bn2;
}

void gemm_launch(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, const void* residual,
                 int64_t M, int64_t N, int64_t K, int bn, int splits, float* workspace, uint32_t* counters,
                 uint32_t* err, cudaStream_t s, const GemmAgWait* ag) {
  if (M == 0 || N == 0) return;
  // explicit bn/splits requests keep the regular orientation (tests, tuning);
  // an all-gather consumer keeps it too (its rows arrive per m-tile)
  const bool swap_ok = bn <= 0 && splits <= 0 && N % 4 == 0 && ag == nullptr;
  if (K % 8 != 0 || N % 8 != 0) throw std::runtime_error("gemm: K and N must be multiples of 8");
  if (ldc % 8 != 0 || ((uint64_t)C & 15) != 0) throw std::runtime_error("gemm: C must be 16-byte aligned rows");
  // 1-2 rows (decode): a weight stream, served by the CUDA-core GEMV
  // (MBX_GEMV=0 keeps the tensor-core kernels)
  static const bool gemv_on = [] {
    const char* v = std::getenv("MBX_GEMV");
    return !(v != nullptr && v[0] == '0');
  }();
  if (gemv_on && bn <= 0 && splits <= 0 && ag == nullptr && gemv_bf16_supported(A, lda, B, ldb, M, K)) {
    gemv_bf16_launch(A, lda, B, ldb, C, ldc, residual, M, N, K, s);
    return;
  }
  const int sms = num_sms();
  GemmPlan p = plan_for(M, N, K, sms);
  if (bn > 0) p.bn = bn;
  if (splits > 0) p.splits = splits;
  if (p.bn != 64 && p.bn != 128 && p.bn != 160 && p.bn != 192 && p.bn != 224 && p.bn != 256)
    throw std::runtime_error("gemm: BN must be one of 64, 128, 160, 192, 224, 256");
  GemmArgs a;
  std::memset(&a, 0, sizeof(a));
  if (ag != nullptr) {
    a.ag_flags = ag->flags;
    a.ag_epoch_word = ag->epoch_word;
    a.ag_Mo = ag->Mo;
  }
  a.residual = static_cast<const __nv_bfloat16*>(residual);
  a.ldc = ldc;
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.num_m = (int)((M + BM - 1) / BM);
  a.num_n = (int)((N + p.bn - 1) / p.bn);
  a.kb_total = (int)((K + BK - 1) / BK);
  a.splits = std::max(1, std::min(p.splits, a.kb_total));
  a.kb_per_split = (a.kb_total + a.splits - 1) / a.splits;
  a.splits = (a.kb_total + a.kb_per_split - 1) / a.kb_per_split;
  a.err = err;
  a.timeout_ns = 2000000000ull;
  const GemmPlan swp = swap_plan(M, N, K, sms);
  if (M <= 64 && workspace != nullptr && swap_ok && swp.splits > 1) {
    // Decode shapes: weights take the 128-row MMA side, the <= 64 tokens the
    // N side (32 or 64), K split so every SM streams its share of the weights.
    const int bnt = swp.bn;
    const int64_t num_f = (N + BM - 1) / BM;
    const int64_t sp = swp.splits;
    const int64_t per = (a.kb_total + sp - 1) / sp;
    GemmArgs sw = a;
    sw.M = (int)N;  // kernel rows = features
    sw.N = (int)M;  // kernel columns = tokens
    sw.num_m = (int)num_f;
    sw.num_n = 1;
    sw.splits = (int)sp;
    sw.kb_per_split = (int)per;
    sw.out = workspace;
    sw.tile_counters = counters;
    sw.final_out = static_cast<__nv_bfloat16*>(C);
    sw.final_ld = ldc;
    const CUtensorMap tw = make_map(B, N, K, ldb, BM);
    const CUtensorMap tx = make_map(A, M, K, lda, bnt);
    // with counters the last CTA of each tile folds the partials in-kernel,
    // otherwise the reduce kernel below does
    launch_bn<kEpiSwapF32Partial>(bnt, tw, tx, sw, (int)std::min<int64_t>(num_f * sp, sms), s);
    if (!counters) {
      const int64_t MN = M * N;
      const int threads = 256;
      const int64_t blocks = std::min<int64_t>((MN / 4 + threads - 1) / threads, (int64_t)sms * 8);
      launch_k(splitk_reduce_kernel, dim3((unsigned)std::max<int64_t>(1, blocks)), dim3(threads), 0, s,
               (const float*)workspace, (int)sp, MN, (int)N, (__nv_bfloat16*)C, (int64_t)ldc, a.residual);
    }
    MBX_CUDA_CHECK(cudaGetLastError());
    return;
  }
  const int bn2 = (ag == nullptr && bn <= 0 && splits <= 0 && N % 8 == 0) ? pair_gemm_bn(M, N, p, sms) : 0;
  if (bn2 > 0) {
    // CTA-pair tiles (256 x bn2): same grid of SMs, half of B per SM per k-step
    GemmArgs pa = a;
    pa.splits = 1;
    pa.kb_per_split = pa.kb_total;
    pa.num_n = (int)((N + bn2 - 1) / bn2);
    pa.out = C;
    const CUtensorMap ta2 = make_map(A, M, K, lda, BM);
    const CUtensorMap tb2 = make_map(B, N, K, ldb, bn2 / 2);
    const int units2 = (int)((M + 2 * BM - 1) / (2 * BM)) * pa.num_n;
    const int grid2 = 2 * std::min(units2, sms / 2);
    if (bn2 == 256) {
      if (residual) launch_pair_cfg<256, 6, kEpiBf16AddResidual>(ta2, tb2, pa, grid2, s);
      else launch_pair_cfg<256, 6, kEpiBf16>(ta2, tb2, pa, grid2, s);
    } else if (bn2 == 192) {
      if (residual) launch_pair_cfg<192, 7, kEpiBf16AddResidual>(ta2, tb2, pa, grid2, s);
      else launch_pair_cfg<192, 7, kEpiBf16>(ta2, tb2, pa, grid2, s);
    } else {
      if (residual) launch_pair_cfg<128, 8, kEpiBf16AddResidual>(ta2, tb2, pa, grid2, s);
      else launch_pair_cfg<128, 8, kEpiBf16>(ta2, tb2, pa, grid2, s);
    }
    MBX_CUDA_CHECK(cudaGetLastError());
    return;
  }
  const CUtensorMap ta = make_map(A, M, K, lda, BM);
  const CUtensorMap tb = make_map(B, N, K, ldb, p.bn);
  const int units = a.num_m * a.num_n * a.splits;
  const int grid = std::min(units, sms);
  if (a.splits == 1) {
    a.out = C;
    if (residual) launch_bn<kEpiBf16AddResidual>(p.bn, ta, tb, a, grid, s);
    else launch_bn<kEpiBf16>(p.bn, ta, tb, a, grid, s);
  } else {
    if (!workspace) throw std::runtime_error("gemm: split-K needs an fp32 workspace of splits*M*N elements");
    if (N % 4 != 0) throw std::runtime_error("gemm: split-K needs N % 4 == 0");
    a.out = workspace;
    a.tile_counters = counters;
    a.final_out = static_cast<__nv_bfloat16*>(C);
    a.final_ld = ldc;
    launch_bn<kEpiF32Partial>(p.bn, ta, tb, a, grid, s);
    if (!counters) {
      const int64_t MN = M * N;
      const int threads = 256;
      const int64_t blocks = std::min<int64_t>((MN / 4 + threads - 1) / threads, (int64_t)sms * 8);
      launch_k(splitk_reduce_kernel, dim3((unsigned)blocks), dim3(threads), 0, s, (const float*)workspace, a.splits,
               MN, (int)N, (__nv_bfloat16*)C, (int64_t)ldc, a.residual);
    }
  }
  MBX_CUDA_CHECK(cudaGetLastError());
}

}  // namespace mbx
