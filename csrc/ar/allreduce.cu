// Cross-GPU allreduce kernels over NVLink 5 / NVSwitch symmetric memory.
//
// Replaces the reference's 5/6-kernel lockstep push (waitack -> produce ->
// flag -> wait_local -> reduce -> ack, sglang/mailbox_ar_ext.cu:124-167) with
// ONE launch per call for every algorithm:
//
//   kOneShotPush  each rank stores its input into slot[rank] of every peer's
//                 buffer ("mailbox push", the reference's data path), block
//                 barrier, then reduces its own buffer locally.
//   kOneShotPull  each rank copies its input into its own buffer, barrier,
//                 then every rank loads all peers' copies over NVLink.
//   kTwoShot      reduce-scatter by pull + all-gather by pull (2(n-1)/n bytes).
//   kNvls         reduce-scatter with multimem.ld_reduce through the switch and
//                 all-gather with multimem.st (NVLS), when multicast exists.
//
// All sums are fp32 in rank order 0..n-1 with a single final rounding (the
// reference's mb_add semantics, sglang/mailbox_ar_ext.cu:91-99), so every rank
// gets the bit-identical result and x + x is exact.
//
// Every wait is bounded by %globaltimer; a timeout records (code, block, peer,
// phase, epoch) in host-mapped memory and the block returns. There is no trap.
#include <algorithm>
#include <stdexcept>
#include <string>
#include <type_traits>

#include "../kernels.h"
#include "ar_common.cuh"

namespace mbx {

enum Algo : int { kAuto = 0, kOneShotPush = 1, kOneShotPull = 2, kTwoShot = 3, kNvls = 4, kTwoShotPush = 5 };

constexpr int kArThreads = 512;

MBX_DEVICE uint32_t call_epoch(const ArCtx& c) {
  return *reinterpret_cast<volatile uint32_t*>(c.state + kStEpoch) + 1u;
}
MBX_DEVICE bool poisoned(const ArCtx& c) {
  return *reinterpret_cast<volatile uint32_t*>(c.state + kStErr) != 0u;
}

// --------------------------------------------------------------------------
// One-shot push ("mailbox"): slot size = half / world (256-byte aligned).
// --------------------------------------------------------------------------
template <typename T, int W>
MBX_DEVICE void ar_oneshot_push(const ArCtx& c, const uint4* __restrict__ in, uint4* __restrict__ out, uint64_t nvec) {
  __shared__ bool s_ok;
  const uint32_t epoch = call_epoch(c);
  trace_mark(c, 0);
  if (!poisoned(c)) {
    const uint64_t slot = oneshot_slot_bytes(c.half_bytes, W);
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t i0 = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (uint64_t i = i0; i < nvec; i += stride) {
      const uint4 v = ld_nc_v4(in + i);
#pragma unroll
      for (int j = 0; j < W; ++j) {
        const int r = (c.rank + j) % W;  // stagger destinations across ranks
        st_v4(data_half(c.bufs[r], epoch, c.half_bytes) + c.rank * slot + i * 16, v);
      }
    }
    trace_mark(c, 1);
    if (block_barrier(c, 0, epoch, &s_ok)) {
      trace_mark(c, 2);
      const char* mine = data_half(c.bufs[c.rank], epoch, c.half_bytes);
      for (uint64_t i = i0; i < nvec; i += stride) {
        uint4 v[W];
#pragma unroll
        for (int r = 0; r < W; ++r) v[r] = ld_cg_v4(mine + r * slot + i * 16);
        float acc[Pack<T>::N] = {};
#pragma unroll
        for (int r = 0; r < W; ++r) unpack_add<T>(v[r], acc);
        out[i] = pack_from<T>(acc);
      }
    }
  }
  trace_mark(c, 5);
  finish_call(c, epoch);
}

template <typename T, int W>
__global__ void __launch_bounds__(kArThreads) ar_oneshot_push_kernel(ArCtx c, const uint4* __restrict__ in,
                                                                     uint4* __restrict__ out, uint64_t nvec) {
  pdl_wait();
  ar_oneshot_push<T, W>(c, in, out, nvec);
}

// --------------------------------------------------------------------------
// One-shot pull.
// --------------------------------------------------------------------------
template <typename T, int W>
MBX_DEVICE void ar_oneshot_pull(const ArCtx& c, const uint4* __restrict__ in, uint4* __restrict__ out, uint64_t nvec) {
  __shared__ bool s_ok;
  const uint32_t epoch = call_epoch(c);
  if (!poisoned(c)) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t i0 = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    char* mine = data_half(c.bufs[c.rank], epoch, c.half_bytes);
    for (uint64_t i = i0; i < nvec; i += stride) st_v4(mine + i * 16, ld_nc_v4(in + i));
    if (block_barrier(c, 0, epoch, &s_ok)) {
#pragma unroll 2
      for (uint64_t i = i0; i < nvec; i += stride) {
        uint4 v[W];
#pragma unroll
        for (int j = 0; j < W; ++j) {
          const int r = (c.rank + j) % W;
          v[r] = ld_cg_v4(data_half(c.bufs[r], epoch, c.half_bytes) + i * 16);
        }
        float acc[Pack<T>::N] = {};
#pragma unroll
        for (int r = 0; r < W; ++r) unpack_add<T>(v[r], acc);
        out[i] = pack_from<T>(acc);
      }
    }
  }
  finish_call(c, epoch);
}

template <typename T, int W>
__global__ void __launch_bounds__(kArThreads) ar_oneshot_pull_kernel(ArCtx c, const uint4* __restrict__ in,
                                                                     uint4* __restrict__ out, uint64_t nvec) {
  pdl_wait();
  ar_oneshot_pull<T, W>(c, in, out, nvec);
}

// --------------------------------------------------------------------------
// Two-shot: chunk c of the message is owned by rank c.
//   A: copy input -> own slot0             B: owner reduces its chunk from all
//   slot0s into own slot1 (+ out)          C: gather the other chunks' slot1s.
// Block b always handles the same element partition of every chunk, so the
// pairwise block barrier orders exactly the data each block consumes.
// --------------------------------------------------------------------------
template <typename T, int W>
MBX_DEVICE void ar_twoshot(const ArCtx& c, const uint4* __restrict__ in, uint4* __restrict__ out, uint64_t nvec) {
  __shared__ bool s_ok;
  const uint32_t epoch = call_epoch(c);
  if (!poisoned(c)) {
    const uint64_t slot1 = c.half_bytes / 2;
    const uint64_t cs = (nvec + W - 1) / W;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t o0 = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    char* mine = data_half(c.bufs[c.rank], epoch, c.half_bytes);
    for (int ch = 0; ch < W; ++ch) {
      const uint64_t beg = ch * cs, end = min(nvec, beg + cs);
      for (uint64_t i = beg + o0; i < end; i += stride) st_v4(mine + i * 16, ld_nc_v4(in + i));
    }
    if (!block_barrier(c, 0, epoch, &s_ok)) goto done;
    {
      const uint64_t beg = c.rank * cs, end = min(nvec, beg + cs);
      for (uint64_t i = beg + o0; i < end; i += stride) {
        uint4 v[W];
#pragma unroll
        for (int j = 0; j < W; ++j) {
          const int r = (c.rank + j) % W;
          v[r] = ld_cg_v4(data_half(c.bufs[r], epoch, c.half_bytes) + i * 16);
        }
        float acc[Pack<T>::N] = {};
#pragma unroll
        for (int r = 0; r < W; ++r) unpack_add<T>(v[r], acc);
        const uint4 s = pack_from<T>(acc);
        st_v4(mine + slot1 + i * 16, s);
        out[i] = s;
      }
    }
    if (!block_barrier(c, 1, epoch, &s_ok)) goto done;
    for (int j = 1; j < W; ++j) {
      const int p = (c.rank + j) % W;
      const uint64_t beg = p * cs, end = min(nvec, beg + cs);
      const char* src = data_half(c.bufs[p], epoch, c.half_bytes) + slot1;
      for (uint64_t i = beg + o0; i < end; i += stride) out[i] = ld_cg_v4(src + i * 16);
    }
  }
done:
  finish_call(c, epoch);
}

template <typename T, int W>
__global__ void __launch_bounds__(kArThreads) ar_twoshot_kernel(ArCtx c, const uint4* __restrict__ in,
                                                                uint4* __restrict__ out, uint64_t nvec) {
  pdl_wait();
  ar_twoshot<T, W>(c, in, out, nvec);
}

// --------------------------------------------------------------------------
// Two-shot, push-push: every NVLink byte is a posted store.
//   A: element i of chunk ch is stored into owner ch's slot[rank]
//   B: the owner sums its W slots locally (rank order) and stores the result
//      into every rank's result region (slot of chunk ch)
//   C: each rank copies the result region to `out` (local reads)
// Region A = W slots of cs vectors, region B = W chunks of cs vectors.
// --------------------------------------------------------------------------
constexpr int kU = 4;  // vectors in flight per thread per loop trip

template <typename T, int W>
MBX_DEVICE void ar_twoshot_push(const ArCtx& c, const uint4* __restrict__ in, uint4* __restrict__ out, uint64_t nvec) {
  __shared__ bool s_ok;
  const uint32_t epoch = call_epoch(c);
  trace_mark(c, 0);
  if (!poisoned(c)) {
    const uint64_t cs = (nvec + W - 1) / W;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t o0 = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    char* mine = data_half(c.bufs[c.rank], epoch, c.half_bytes);
    // A: push every chunk's share to its owner
#pragma unroll 1
    for (int j = 0; j < W; ++j) {
      const int ch = (c.rank + j) % W;
      const uint64_t beg = ch * cs, end = min(nvec, beg + cs);
      char* dst = data_half(c.bufs[ch], epoch, c.half_bytes) + (uint64_t)c.rank * cs * 16;
      for (uint64_t i = beg + o0; i < end; i += stride * kU) {
        uint4 v[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const uint64_t k = i + u * stride;
          if (k < end) v[u] = ld_nc_v4(in + k);
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const uint64_t k = i + u * stride;
          if (k < end) st_v4(dst + (k - beg) * 16, v[u]);
        }
      }
    }
    trace_mark(c, 1);
    if (!block_barrier(c, 0, epoch, &s_ok)) goto done;
    trace_mark(c, 2);
    {
      // B: reduce the own chunk, broadcast the result
      const uint64_t beg = c.rank * cs, end = min(nvec, beg + cs);
      const uint64_t resoff = (uint64_t)W * cs * 16 + (uint64_t)c.rank * cs * 16;
      for (uint64_t i = beg + o0; i < end; i += stride * kU) {
        uint4 s4[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const uint64_t k = i + u * stride;
          if (k < end) {
            uint4 v[W];
#pragma unroll
            for (int r = 0; r < W; ++r) v[r] = ld_cg_v4(mine + ((uint64_t)r * cs + (k - beg)) * 16);
            float acc[Pack<T>::N] = {};
#pragma unroll
            for (int r = 0; r < W; ++r) unpack_add<T>(v[r], acc);
            s4[u] = pack_from<T>(acc);
          }
        }
#pragma unroll
        for (int j = 0; j < W; ++j) {
          const int r = (c.rank + j) % W;
          char* dst = data_half(c.bufs[r], epoch, c.half_bytes) + resoff;
#pragma unroll
          for (int u = 0; u < kU; ++u) {
            const uint64_t k = i + u * stride;
            if (k < end) st_v4(dst + (k - beg) * 16, s4[u]);
          }
        }
      }
    }
    trace_mark(c, 3);
    if (!block_barrier(c, 1, epoch, &s_ok)) goto done;
    trace_mark(c, 4);
    {
      // C: gather locally
      const char* res = mine + (uint64_t)W * cs * 16;
#pragma unroll 1
      for (int ch = 0; ch < W; ++ch) {
        const uint64_t beg = ch * cs, end = min(nvec, beg + cs);
        for (uint64_t i = beg + o0; i < end; i += stride * kU) {
          uint4 v[kU];
#pragma unroll
          for (int u = 0; u < kU; ++u) {
            const uint64_t k = i + u * stride;
            if (k < end) v[u] = ld_cg_v4(res + k * 16);
          }
#pragma unroll
          for (int u = 0; u < kU; ++u) {
            const uint64_t k = i + u * stride;
            if (k < end) out[k] = v[u];
          }
        }
      }
    }
  }
done:
  trace_mark(c, 5);
  finish_call(c, epoch);
}

template <typename T, int W>
__global__ void __launch_bounds__(kArThreads) ar_twoshot_push_kernel(ArCtx c, const uint4* __restrict__ in,
                                                                     uint4* __restrict__ out, uint64_t nvec) {
  pdl_wait();
  ar_twoshot_push<T, W>(c, in, out, nvec);
}

// --------------------------------------------------------------------------
// NVLS: multimem.ld_reduce (switch-side sum, fp32 accumulation for 16-bit
// types) + multimem.st broadcast of the owner's chunk.
// The switch serves multicast loads and stores from/to every GPU's L2, the
// same point of coherence as the local .cg loads and the unicast stores, so
// the system-scope release/acquire barriers alone order the phases (no
// fence.proxy.alias, which measured 3-30 us per barrier, growing with size).
// Loads and stores of different warps overlap: the loads use a GPU's egress
// (its memory is read by every owner), the stores its ingress.
// --------------------------------------------------------------------------
template <typename T>
MBX_DEVICE uint4 multimem_ld_reduce(const void* mc);
template <>
MBX_DEVICE uint4 multimem_ld_reduce<__nv_bfloat16>(const void* mc) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}
template <>
MBX_DEVICE uint4 multimem_ld_reduce<__half>(const void* mc) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}
template <>
MBX_DEVICE uint4 multimem_ld_reduce<float>(const void* mc) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}
MBX_DEVICE void multimem_st(void* mc, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

template <typename T, int W>
__global__ void __launch_bounds__(kArThreads) ar_nvls_kernel(ArCtx c, const uint4* __restrict__ in,
                                                             uint4* __restrict__ out, uint64_t nvec) {
  pdl_wait();
  __shared__ bool s_ok;
  const uint32_t epoch = call_epoch(c);
  trace_mark(c, 0);
  if (!poisoned(c)) {
    const uint64_t slot1 = c.half_bytes / 2;
    const uint64_t cs = (nvec + W - 1) / W;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t o0 = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    char* mine = data_half(c.bufs[c.rank], epoch, c.half_bytes);
    char* mc = data_half(c.mc, epoch, c.half_bytes);
    for (int ch = 0; ch < W; ++ch) {
      const uint64_t beg = ch * cs, end = min(nvec, beg + cs);
      for (uint64_t i = beg + o0; i < end; i += stride) st_v4(mine + i * 16, ld_nc_v4(in + i));
    }
    trace_mark(c, 1);
    if (!block_barrier(c, 0, epoch, &s_ok)) goto done;
    trace_mark(c, 2);
    {
      const uint64_t beg = c.rank * cs, end = min(nvec, beg + cs);
      for (uint64_t i = beg + o0; i < end; i += stride * kU) {
        uint4 v[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const uint64_t k = i + u * stride;
          if (k < end) v[u] = multimem_ld_reduce<T>(mc + k * 16);
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const uint64_t k = i + u * stride;
          if (k < end) multimem_st(mc + slot1 + k * 16, v[u]);
        }
      }
    }
    trace_mark(c, 3);
    if (!block_barrier(c, 1, epoch, &s_ok)) goto done;
    trace_mark(c, 4);
    for (int ch = 0; ch < W; ++ch) {
      const uint64_t beg = ch * cs, end = min(nvec, beg + cs);
      for (uint64_t i = beg + o0; i < end; i += stride) out[i] = ld_cg_v4(mine + slot1 + i * 16);
    }
  }
done:
  trace_mark(c, 5);
  finish_call(c, epoch);
}

// --------------------------------------------------------------------------
// Fused allreduce + residual add + RMSNorm (bf16, rows of H elements).
//   ar   = bf16(sum_r in_r)                 (same rounding as a plain AR)
//   res  = bf16(ar + residual)   -> residual (in place)
//   out  = bf16(res * rsqrt(mean(res^2) + eps) * w)
// One-shot push by rows, or two-shot (rows split by owner rank, all-gather of
// the reduced rows, each rank normalises every row locally).
// --------------------------------------------------------------------------
MBX_DEVICE float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
  const int nw = blockDim.x >> 5;
  for (int i = 0; i < nw; ++i) s += red[i];
  return s;
}

// res/out for one row given the reduced bf16 row `ar` (read through `ld`).
// Row kernels. Row l of a phase's range belongs to block l % gridDim.x (rows
// b, b+g, b+2g, ...); every phase that reads rows another rank's block wrote
// keeps this assignment, so the block-pairwise barriers between phases cover
// every row. Inside a block, a normalisation phase works on one row with the
// whole block (decode: few rows, lowest latency) or, when the block owns
// several rows, on one row per warp (prefill: one row in flight per warp, no
// block-wide reductions).

struct RowCtx {
  int t0, tstep;  // this thread's first 16-byte vector of the row and its stride
  int group;      // warps per row: 1 (warp reduction), G > 1 (G warps, named barrier), 0 (whole block)
};

// Rows b, b+g, ... below n owned by this block.
MBX_DEVICE int block_rows(int n) {
  return n > (int)blockIdx.x ? (n - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
}

// fn(rc, k) for k in [0, count) (count uniform over the block). One row: the
// whole block. Several rows: groups of G warps per row, G the largest power of
// two up to 8 with 2 * count * G <= warps (more warps in flight per row when the
// block has few rows); groups take rows k, k + groups, ... A row's partial sums
// meet through the group's own named barrier, so a group whose rows run out
// stops without the others.
template <typename Fn>
MBX_DEVICE void for_norm_rows(int count, Fn fn) {
  if (count == 1) {
    fn(RowCtx{(int)threadIdx.x, (int)blockDim.x, 0}, 0);
    return;
  }
  const int warps = (int)(blockDim.x >> 5);
  int G = 1;
  while (G < 8 && count * G * 2 <= warps) G *= 2;
  const int w = (int)(threadIdx.x >> 5);
  const int groups = warps / G;
  for (int k = w / G; k < count; k += groups) fn(RowCtx{(w % G) * 32 + (int)(threadIdx.x & 31), 32 * G, G}, k);
}

// Sum over the G warps of this thread's group (groups of G consecutive warps),
// through red[] (one word per warp) and the group's named barrier 1 + group
// (G >= 2 and at most 16 warps per block give ids 1..8 of the 16).
MBX_DEVICE float group_sum(float v, float* red, int G) {
  v = warp_sum(v);
  const int w = (int)(threadIdx.x >> 5), g = w / G;
  asm volatile("bar.sync %0, %1;" ::"r"(1 + g), "r"(G * 32) : "memory");  // earlier readers of red[] are done
  if ((threadIdx.x & 31) == 0) red[w] = v;
  asm volatile("bar.sync %0, %1;" ::"r"(1 + g), "r"(G * 32) : "memory");
  float s = 0.f;
  for (int i = 0; i < G; ++i) s += red[g * G + i];
  return s;
}

// Copy/reduce phases over the block's rows (row j = b + j*g of a range):
// out(j, p, sum of the NV source vectors src(j, p, r)) for every vector p <
// hvec, flattened over the block's threads. Each thread issues the loads of
// KU vectors before it combines any (the load wrappers are ordered asm), so
// about 8 loads are in flight per thread.
template <int NV, typename Src, typename Out>
MBX_DEVICE void reduce_block_vectors(int rows, int hvec, Src src, Out out) {
  constexpr int KU = NV >= 8 ? 1 : (NV == 1 ? 4 : 8 / NV);
  const int total = rows * hvec;
  for (int i0 = threadIdx.x; i0 < total; i0 += blockDim.x * KU) {
    uint4 v[KU][NV];
#pragma unroll
    for (int u = 0; u < KU; ++u) {
      const int i = i0 + u * (int)blockDim.x;
      if (i < total) {
        const int j = i / hvec, pv = i - j * hvec;
#pragma unroll
        for (int r = 0; r < NV; ++r) v[u][r] = src(j, pv, r);
      }
    }
#pragma unroll
    for (int u = 0; u < KU; ++u) {
      const int i = i0 + u * (int)blockDim.x;
      if (i < total) {
        const int j = i / hvec, pv = i - j * hvec;
        if (NV == 1) {
          out(j, pv, v[u][0]);
        } else {
          float acc[8] = {};
#pragma unroll
          for (int r = 0; r < NV; ++r) unpack_add<__nv_bfloat16>(v[u][r], acc);
          out(j, pv, pack_from<__nv_bfloat16>(acc));
        }
      }
    }
  }
}

// res = bf16(bf16(sum_r src(p, r)) + residual) -> residual (in place);
// st(p, bf16(res * rsqrt(mean(res^2) + eps) * w)). NV sources per vector,
// summed in order r = 0..NV-1 in fp32 with one rounding; loads batched as in
// reduce_block_vectors.
template <int NV, typename Src, typename StoreOut>
MBX_DEVICE void residual_rmsnorm_row(const RowCtx& rc, Src src, uint4* residual_row, const uint4* w_row,
                                     StoreOut st, int hvec, int H, float eps, float* red) {
  constexpr int KU = NV >= 8 ? 1 : (NV == 1 ? 4 : 8 / NV);
  float ss = 0.f;
  if (hvec <= rc.tstep * KU) {
    // The thread's share of the row is one batch (decode rows on a whole block,
    // prefill rows on 8-warp groups): the new residual and the weights stay in
    // registers, so the scaling needs no second round of loads. Same arithmetic
    // in the same order as the two-pass form below.
    uint4 v[KU][NV];
    uint4 rv[KU], wv[KU], rb[KU];
#pragma unroll
    for (int u = 0; u < KU; ++u) {
      const int pv = rc.t0 + u * rc.tstep;
      if (pv < hvec) {
#pragma unroll
        for (int r = 0; r < NV; ++r) v[u][r] = ld_cg_v4(src(pv, r));
        rv[u] = residual_row[pv];
        wv[u] = w_row[pv];
      }
    }
#pragma unroll
    for (int u = 0; u < KU; ++u) {
      const int pv = rc.t0 + u * rc.tstep;
      if (pv < hvec) {
        float a[8] = {};
#pragma unroll
        for (int r = 0; r < NV; ++r) unpack_add<__nv_bfloat16>(v[u][r], a);
        const uint4 arb = pack_from<__nv_bfloat16>(a);
        float q[8] = {};
        unpack_add<__nv_bfloat16>(arb, q);
        unpack_add<__nv_bfloat16>(rv[u], q);
        rb[u] = pack_from<__nv_bfloat16>(q);
        residual_row[pv] = rb[u];
        float f[8] = {};
        unpack_add<__nv_bfloat16>(rb[u], f);
#pragma unroll
        for (int k = 0; k < 8; ++k) ss += f[k] * f[k];
      }
    }
    const float tot1 =
        rc.group == 1 ? warp_sum(ss) : (rc.group == 0 ? block_sum(ss, red) : group_sum(ss, red, rc.group));
    const float rstd1 = rsqrtf(tot1 / (float)H + eps);
#pragma unroll
    for (int u = 0; u < KU; ++u) {
      const int pv = rc.t0 + u * rc.tstep;
      if (pv < hvec) {
        float q[8] = {}, ww[8] = {};
        unpack_add<__nv_bfloat16>(rb[u], q);
        unpack_add<__nv_bfloat16>(wv[u], ww);
#pragma unroll
        for (int k = 0; k < 8; ++k) q[k] = q[k] * rstd1 * ww[k];
        st(pv, pack_from<__nv_bfloat16>(q));
      }
    }
    return;
  }
  for (int p0 = rc.t0; p0 < hvec; p0 += rc.tstep * KU) {
    uint4 v[KU][NV];
    uint4 rv[KU];
#pragma unroll
    for (int u = 0; u < KU; ++u) {
      const int pv = p0 + u * rc.tstep;
      if (pv < hvec) {
#pragma unroll
        for (int r = 0; r < NV; ++r) v[u][r] = ld_cg_v4(src(pv, r));
        rv[u] = residual_row[pv];
      }
    }
#pragma unroll
    for (int u = 0; u < KU; ++u) {
      const int pv = p0 + u * rc.tstep;
      if (pv < hvec) {
        float a[8] = {};
#pragma unroll
        for (int r = 0; r < NV; ++r) unpack_add<__nv_bfloat16>(v[u][r], a);
        // round the AR result to bf16 first (matches AR-then-add unfused order)
        const uint4 arb = pack_from<__nv_bfloat16>(a);
        float q[8] = {};
        unpack_add<__nv_bfloat16>(arb, q);
        unpack_add<__nv_bfloat16>(rv[u], q);
        const uint4 rb = pack_from<__nv_bfloat16>(q);
        residual_row[pv] = rb;
        float f[8] = {};
        unpack_add<__nv_bfloat16>(rb, f);
#pragma unroll
        for (int k = 0; k < 8; ++k) ss += f[k] * f[k];
      }
    }
  }
  const float tot = rc.group == 1 ? warp_sum(ss) : (rc.group == 0 ? block_sum(ss, red) : group_sum(ss, red, rc.group));
  const float rstd = rsqrtf(tot / (float)H + eps);
  constexpr int KU2 = 4;
  for (int p0 = rc.t0; p0 < hvec; p0 += rc.tstep * KU2) {
    uint4 rv[KU2], wv[KU2];
#pragma unroll
    for (int u = 0; u < KU2; ++u) {
      const int pv = p0 + u * rc.tstep;
      if (pv < hvec) {
        rv[u] = residual_row[pv];
        wv[u] = w_row[pv];
      }
    }
#pragma unroll
    for (int u = 0; u < KU2; ++u) {
      const int pv = p0 + u * rc.tstep;
      if (pv < hvec) {
        float q[8] = {}, ww[8] = {};
        unpack_add<__nv_bfloat16>(rv[u], q);
        unpack_add<__nv_bfloat16>(wv[u], ww);
#pragma unroll
        for (int k = 0; k < 8; ++k) q[k] = q[k] * rstd * ww[k];
        st(pv, pack_from<__nv_bfloat16>(q));
      }
    }
  }
}

// Norm rows of a per-owner layout: for every owner o (rows [o*Mo, o*Mo+Mo) of
// M), this block's rows o*Mo + b + j*g; fn(rc, row).
template <int NO, typename Fn>
MBX_DEVICE void for_owner_norm_rows(int M, int Mo, Fn fn) {
  const int per = block_rows(Mo);
  for_norm_rows(NO * per, [&](const RowCtx& rc, int k) {
    const int o = k / per, j = k - (k / per) * per;
    const int row = o * Mo + (int)blockIdx.x + j * (int)gridDim.x;
    if (row < min(M, o * Mo + Mo)) fn(rc, row);
  });
}

template <int W>
MBX_DEVICE void ar_rmsnorm_oneshot(const ArCtx& c, const uint4* __restrict__ in, uint4* residual,
                                   const uint4* __restrict__ w, uint4* __restrict__ out, int M, int H, float eps) {
  __shared__ bool s_ok;
  __shared__ float red[32];
  const uint32_t epoch = call_epoch(c);
  const int hvec = H / 8;
  trace_mark(c, 0);
  if (!poisoned(c)) {
    const uint64_t slot = oneshot_slot_bytes(c.half_bytes, W);
    const int nrows = block_rows(M);
    const int b = blockIdx.x, g = gridDim.x;
    reduce_block_vectors<1>(
        nrows, hvec, [&](int j, int pv, int) { return ld_nc_v4(in + (uint64_t)(b + j * g) * hvec + pv); },
        [&](int j, int pv, const uint4& v) {
          const uint64_t i = (uint64_t)(b + j * g) * hvec + pv;
#pragma unroll
          for (int t = 0; t < W; ++t)
            st_v4(data_half(c.bufs[(c.rank + t) % W], epoch, c.half_bytes) + c.rank * slot + i * 16, v);
        });
    trace_mark(c, 1);
    if (block_barrier(c, 0, epoch, &s_ok)) {
      trace_mark(c, 2);
      const char* mine = data_half(c.bufs[c.rank], epoch, c.half_bytes);
      for_norm_rows(nrows, [&](const RowCtx& rc, int k) {
        const uint64_t base = (uint64_t)(b + k * g) * hvec;
        residual_rmsnorm_row<W>(
            rc, [&](int pv, int r) { return mine + r * slot + (base + pv) * 16; }, residual + base, w,
            [&](int pv, const uint4& v) { out[base + pv] = v; }, hvec, H, eps, red);
      });
    }
  }
  trace_mark(c, 5);
  finish_call(c, epoch);
}

template <int W>
__global__ void __launch_bounds__(kArThreads) ar_rmsnorm_oneshot_kernel(ArCtx c, const uint4* __restrict__ in,
                                                                        uint4* residual, const uint4* __restrict__ w,
                                                                        uint4* __restrict__ out, int M, int H,
                                                                        float eps) {
  pdl_wait();
  ar_rmsnorm_oneshot<W>(c, in, residual, w, out, M, H, eps);
}

template <int W>
MBX_DEVICE void ar_rmsnorm_twoshot(const ArCtx& c, const uint4* __restrict__ in, uint4* residual,
                                   const uint4* __restrict__ w, uint4* __restrict__ out, int M, int H, float eps) {
  __shared__ bool s_ok;
  __shared__ float red[32];
  const uint32_t epoch = call_epoch(c);
  const int hvec = H / 8;
  if (!poisoned(c)) {
    const uint64_t slot1 = c.half_bytes / 2;
    const int rc = (M + W - 1) / W;
    const int b = blockIdx.x, g = gridDim.x;
    char* mine = data_half(c.bufs[c.rank], epoch, c.half_bytes);
    for (int ch = 0; ch < W; ++ch) {
      const int beg = ch * rc, end = min(M, beg + rc);
      reduce_block_vectors<1>(
          block_rows(end - beg), hvec,
          [&](int j, int pv, int) { return ld_nc_v4(in + (uint64_t)(beg + b + j * g) * hvec + pv); },
          [&](int j, int pv, const uint4& v) { st_v4(mine + ((uint64_t)(beg + b + j * g) * hvec + pv) * 16, v); });
    }
    if (!block_barrier(c, 0, epoch, &s_ok)) goto done;
    {
      const int beg = c.rank * rc, end = min(M, beg + rc);
      reduce_block_vectors<W>(
          block_rows(end - beg), hvec,
          [&](int j, int pv, int r) {
            return ld_cg_v4(data_half(c.bufs[r], epoch, c.half_bytes) + ((uint64_t)(beg + b + j * g) * hvec + pv) * 16);
          },
          [&](int j, int pv, const uint4& sum) {
            st_v4(mine + slot1 + ((uint64_t)(beg + b + j * g) * hvec + pv) * 16, sum);
          });
    }
    if (!block_barrier(c, 1, epoch, &s_ok)) goto done;
    for_owner_norm_rows<W>(M, rc, [&](const RowCtx& rx, int row) {
      const char* src = data_half(c.bufs[row / rc], epoch, c.half_bytes) + slot1;
      const uint64_t base = (uint64_t)row * hvec;
      residual_rmsnorm_row<1>(
          rx, [&](int pv, int) { return src + (base + pv) * 16; }, residual + base, w,
          [&](int pv, const uint4& v) { out[base + pv] = v; }, hvec, H, eps, red);
    });
  }
done:
  finish_call(c, epoch);
}

template <int W>
__global__ void __launch_bounds__(kArThreads) ar_rmsnorm_twoshot_kernel(ArCtx c, const uint4* __restrict__ in,
                                                                        uint4* residual, const uint4* __restrict__ w,
                                                                        uint4* __restrict__ out, int M, int H,
                                                                        float eps) {
  pdl_wait();
  ar_rmsnorm_twoshot<W>(c, in, residual, w, out, M, H, eps);
}

// --------------------------------------------------------------------------
// Fused row-parallel GEMM -> allreduce -> residual + RMSNorm, second half.
// The GEMM epilogue (gemm.cu, push-RS mode) has stored every rank's partial
// rows into the owner's region A (W source slots of [Mo, N] bf16) and the last
// CTA of each rank's GEMM released one flag per owner. Here each owner waits
// for all W flags, sums its rows in rank order (fp32, one rounding), stores the
// reduced rows into every rank's region B (all-gather by posted stores), and
// after a block barrier every rank applies residual add + RMSNorm to all rows
// from its local region B.
// --------------------------------------------------------------------------
MBX_DEVICE char* fuse_half(const ArCtx& c, char* base, uint32_t epoch) {
  return base + c.fuse_off + (uint64_t)(epoch & 1u) * c.fuse_half_bytes;
}
MBX_DEVICE uint32_t* fuse_flag(char* base, int src) { return reinterpret_cast<uint32_t*>(base + kTileFlagOff) + src; }

template <int W>
MBX_DEVICE void fused_rs_norm(const ArCtx& c, int M, int N, int Mo, uint4* residual, const uint4* __restrict__ w,
                              uint4* __restrict__ out, float eps) {
  __shared__ bool s_ok;
  __shared__ float red[32];
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(c.state + kStFuseEpoch) + 1u;
  const int nvec = N / 8;
  if (!poisoned(c)) {
    if (threadIdx.x == 0) s_ok = true;
    __syncthreads();
    if (threadIdx.x < W) {
      if (!wait_flag_geq(fuse_flag(c.bufs[c.rank], threadIdx.x), epoch, c.timeout_ns)) {
        record_error(c, kErrFuseWait, blockIdx.x, threadIdx.x, 4, epoch);
        s_ok = false;
      }
    }
    __syncthreads();
    if (!s_ok) goto done;
    {
      char* mine = fuse_half(c, c.bufs[c.rank], epoch);
      const uint64_t slot = (uint64_t)Mo * N * 2;
      const uint64_t regB = (uint64_t)W * slot;
      const int r0 = c.rank * Mo, r1 = min(M, r0 + Mo);
      const int b = blockIdx.x, g = gridDim.x;
      reduce_block_vectors<W>(
          block_rows(r1 - r0), nvec,
          [&](int j, int pv, int r) { return ld_cg_v4(mine + r * slot + ((uint64_t)(b + j * g) * nvec + pv) * 16); },
          [&](int j, int pv, const uint4& sum) {
            const uint64_t row = r0 + b + j * g;
#pragma unroll
            for (int t = 0; t < W; ++t)
              st_v4(fuse_half(c, c.bufs[(c.rank + t) % W], epoch) + regB + (row * nvec + pv) * 16, sum);
          });
      if (!block_barrier(c, 2, epoch, &s_ok)) goto done;
      for_owner_norm_rows<W>(M, Mo, [&](const RowCtx& rc, int row) {
        const uint64_t base = (uint64_t)row * nvec;
        residual_rmsnorm_row<1>(
            rc, [&](int pv, int) { return mine + regB + (base + pv) * 16; }, residual + base, w,
            [&](int pv, const uint4& v) { out[base + pv] = v; }, nvec, N, eps, red);
      });
    }
  }
done:
  finish_call(c, epoch, kStFuseEpoch, kStFuseDone);
}

template <int W>
__global__ void __launch_bounds__(kArThreads) fused_rs_norm_kernel(ArCtx c, int M, int N, int Mo, uint4* residual,
                                                                   const uint4* __restrict__ w,
                                                                   uint4* __restrict__ out, float eps) {
  pdl_wait();
  fused_rs_norm<W>(c, M, N, Mo, residual, w, out, eps);
}

// --------------------------------------------------------------------------
// Fused GEMM -> allreduce, push-all variant (small worlds): the GEMM epilogue
// stored every row of its partial output into every rank's slot[rank]
// ([W][M][N] bf16) and released one flag per rank. Each rank waits for all W
// flags, then sums the W partials of every row locally (rank order, fp32,
// one rounding) and applies residual add + RMSNorm. No second exchange.
// --------------------------------------------------------------------------
template <int W>
__global__ void __launch_bounds__(kArThreads) fused_allsum_norm_kernel(ArCtx c, int M, int N, uint4* residual,
                                                                       const uint4* __restrict__ w,
                                                                       uint4* __restrict__ out, float eps) {
  pdl_wait();
  __shared__ bool s_ok;
  __shared__ float red[32];
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(c.state + kStFuseEpoch) + 1u;
  const int nvec = N / 8;
  if (!poisoned(c)) {
    if (threadIdx.x == 0) s_ok = true;
    __syncthreads();
    if (threadIdx.x < W) {
      if (!wait_flag_geq(fuse_flag(c.bufs[c.rank], threadIdx.x), epoch, c.timeout_ns)) {
        record_error(c, kErrFuseWait, blockIdx.x, threadIdx.x, 5, epoch);
        s_ok = false;
      }
    }
    __syncthreads();
    if (s_ok) {
      const char* mine = fuse_half(c, c.bufs[c.rank], epoch);
      const uint64_t slot = (uint64_t)M * N * 2;
      const int b = blockIdx.x, g = gridDim.x;
      for_norm_rows(block_rows(M), [&](const RowCtx& rc, int k) {
        const uint64_t base = (uint64_t)(b + k * g) * nvec;
        residual_rmsnorm_row<W>(
            rc, [&](int pv, int r) { return mine + r * slot + (base + pv) * 16; }, residual + base, w,
            [&](int pv, const uint4& v) { out[base + pv] = v; }, nvec, N, eps, red);
      });
    }
  }
  finish_call(c, epoch, kStFuseEpoch, kStFuseDone);
}

// ==========================================================================
// Sequence parallel. Rank r owns rows [r*Mo, r*Mo+Mo) of the residual stream.
// Row-parallel GEMMs push each output row to its owner's reduce-scatter slot
// (gemm_rs_launch, or sp_rs_push for a local tensor); sp_rs_norm_ag reduces
// the owned rows, adds them to the residual shard, normalises them and pushes
// the normed rows into every rank's gather buffer G, where the next
// column-parallel GEMM's TMA producer loads an m-tile as soon as its owners'
// flags are up (all-gather -> GEMM without a separate all-gather launch).
// Buffers: the reduce-scatter slots live in the fused halves (epoch parity),
// G is one fixed buffer: a rank only pushes into a peer's G after every rank's
// previous row-parallel GEMM ran, which comes after that rank's last read of G.
// ==========================================================================
MBX_DEVICE uint32_t* ag_flag(char* base, int owner) {
  return reinterpret_cast<uint32_t*>(base + kAgFlagOff) + owner;
}

// Once every block of the grid got here, release *flag_of(o) = epoch on every
// rank o (the blocks' earlier stores, local or remote, are visible first).
template <typename FlagOf>
MBX_DEVICE void grid_done_release(const ArCtx& c, int counter_word, uint32_t epoch, FlagOf flag_of) {
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_acq_rel_sys();
    const uint32_t prev = atomicAdd(c.state + counter_word, 1u);
    if (prev == gridDim.x - 1) {
      c.state[counter_word] = 0;
      fence_acq_rel_sys();
      for (int o = 0; o < c.world; ++o) st_release_sys(flag_of(o), epoch);
    }
  }
}

template <int W>
__global__ void __launch_bounds__(kArThreads) sp_rs_push_kernel(ArCtx c, const uint4* __restrict__ x, int M, int N,
                                                                 int Mo) {
  pdl_wait();
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(c.state + kStFuseEpoch) + 1u;
  if (poisoned(c)) return;
  const int nvec = N / 8;
  const uint64_t total = (uint64_t)M * nvec;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int row = (int)(i / nvec);
    const int p = (int)(i - (uint64_t)row * nvec);
    const int owner = row / Mo;
    const int lrow = row - owner * Mo;
    char* dst = fuse_half(c, c.bufs[owner], epoch) + ((uint64_t)(c.rank * Mo + lrow) * nvec + p) * 16;
    st_v4(dst, ld_nc_v4(x + i));
  }
  grid_done_release(c, kStFuseGemmDone, epoch, [&](int o) { return fuse_flag(c.bufs[o], c.rank); });
}

template <int W>
__global__ void __launch_bounds__(kArThreads) sp_rs_norm_ag_kernel(ArCtx c, int M, int N, int Mo, uint4* res_own,
                                                                   const uint4* __restrict__ w, float eps) {
  pdl_wait();
  __shared__ bool s_ok;
  __shared__ float red[32];
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(c.state + kStFuseEpoch) + 1u;
  const int nvec = N / 8;
  bool ok = false;
  if (!poisoned(c)) {
    if (threadIdx.x == 0) s_ok = true;
    __syncthreads();
    if (threadIdx.x < W) {
      if (!wait_flag_geq(fuse_flag(c.bufs[c.rank], threadIdx.x), epoch, c.timeout_ns)) {
        record_error(c, kErrFuseWait, blockIdx.x, threadIdx.x, 6, epoch);
        s_ok = false;
      }
    }
    __syncthreads();
    ok = s_ok;
    if (ok) {
      const char* mine = fuse_half(c, c.bufs[c.rank], epoch);
      const uint64_t slot = (uint64_t)Mo * N * 2;
      const int r0 = c.rank * Mo, r1 = min(M, r0 + Mo);
      const int b = blockIdx.x, g = gridDim.x;
      for_norm_rows(block_rows(r1 - r0), [&](const RowCtx& rc, int k) {
        const int lrow = b + k * g;
        const uint64_t row = r0 + lrow;
        residual_rmsnorm_row<W>(
            rc, [&](int pv, int r) { return mine + r * slot + ((uint64_t)lrow * nvec + pv) * 16; },
            res_own + (uint64_t)lrow * nvec, w,
            [&](int pv, const uint4& v) {
#pragma unroll
              for (int t = 0; t < W; ++t)
                st_v4(c.bufs[(c.rank + t) % W] + c.sp_off + (row * nvec + pv) * 16, v);
            },
            nvec, N, eps, red);
      });
    }
  }
  if (ok) grid_done_release(c, kStSpAgDone, epoch, [&](int o) { return ag_flag(c.bufs[o], c.rank); });
  finish_call(c, epoch, kStFuseEpoch, kStFuseDone);
}

__global__ void sp_ag_wait_kernel(ArCtx c, int owners) {
  pdl_wait();
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(c.state + kStFuseEpoch);
  if (poisoned(c)) return;
  const int o = threadIdx.x;
  if (o < owners && !wait_flag_geq(ag_flag(c.bufs[c.rank], o), epoch, c.timeout_ns))
    record_error(c, kErrFuseWait, 0, o, 7, epoch);
}

// --------------------------------------------------------------------------
// Allreduce + residual + RMSNorm, two-shot with posted stores only:
//   A: every row is stored into its owner's region A slot[rank]
//   B: the owner sums its rows (rank order, fp32, one rounding) and stores
//      the reduced rows into every rank's region B
//   C: every rank applies residual add + RMSNorm to all rows from region B
// Rows are owned in contiguous blocks of Mo = ceil(M / W).
// --------------------------------------------------------------------------
template <int W>
MBX_DEVICE void ar_rmsnorm_twoshot_push(const ArCtx& c, const uint4* __restrict__ in, uint4* residual,
                                        const uint4* __restrict__ w, uint4* __restrict__ out, int M, int H, float eps) {
  __shared__ bool s_ok;
  __shared__ float red[32];
  const uint32_t epoch = call_epoch(c);
  const int hvec = H / 8;
  const int Mo = (M + W - 1) / W;
  trace_mark(c, 0);
  if (!poisoned(c)) {
    const uint64_t slot = (uint64_t)Mo * hvec * 16;
    const uint64_t regB = (uint64_t)W * slot;
    char* mine = data_half(c.bufs[c.rank], epoch, c.half_bytes);
    const int b = blockIdx.x, g = gridDim.x;
    // A: rows of owner o -> o's region A, slot `rank`; block b takes rows o*Mo + b + j*g
#pragma unroll 1
    for (int t = 0; t < W; ++t) {
      const int o = (c.rank + t) % W;
      const int a0 = o * Mo, a1 = min(M, a0 + Mo);
      char* dst = data_half(c.bufs[o], epoch, c.half_bytes) + (uint64_t)c.rank * slot;
      reduce_block_vectors<1>(
          block_rows(a1 - a0), hvec,
          [&](int j, int pv, int) { return ld_nc_v4(in + (uint64_t)(a0 + b + j * g) * hvec + pv); },
          [&](int j, int pv, const uint4& v) { st_v4(dst + ((uint64_t)(b + j * g) * hvec + pv) * 16, v); });
    }
    trace_mark(c, 1);
    if (!block_barrier(c, 0, epoch, &s_ok)) goto done;
    trace_mark(c, 2);
    {
      // B: sum the own rows (rank order) and push the sums into every rank's region B
      const int r0 = c.rank * Mo, r1 = min(M, r0 + Mo);
      reduce_block_vectors<W>(
          block_rows(r1 - r0), hvec,
          [&](int j, int pv, int r) { return ld_cg_v4(mine + r * slot + ((uint64_t)(b + j * g) * hvec + pv) * 16); },
          [&](int j, int pv, const uint4& sum) {
            const uint64_t row = r0 + b + j * g;
#pragma unroll
            for (int t = 0; t < W; ++t)
              st_v4(data_half(c.bufs[(c.rank + t) % W], epoch, c.half_bytes) + regB + (row * hvec + pv) * 16, sum);
          });
    }
    trace_mark(c, 3);
    if (!block_barrier(c, 1, epoch, &s_ok)) goto done;
    trace_mark(c, 4);
    // C: residual + norm of every row from the local region B
    for_owner_norm_rows<W>(M, Mo, [&](const RowCtx& rc, int row) {
      const uint64_t base = (uint64_t)row * hvec;
      residual_rmsnorm_row<1>(
          rc, [&](int pv, int) { return mine + regB + (base + pv) * 16; }, residual + base, w,
          [&](int pv, const uint4& v) { out[base + pv] = v; }, hvec, H, eps, red);
    });
  }
done:
  trace_mark(c, 5);
  finish_call(c, epoch);
}

template <int W>
__global__ void __launch_bounds__(kArThreads) ar_rmsnorm_twoshot_push_kernel(ArCtx c, const uint4* __restrict__ in,
                                                                             uint4* residual,
                                                                             const uint4* __restrict__ w,
                                                                             uint4* __restrict__ out, int M, int H,
                                                                             float eps) {
  pdl_wait();
  ar_rmsnorm_twoshot_push<W>(c, in, residual, w, out, M, H, eps);
}

// --------------------------------------------------------------------------
// Segmented allreduce (overlap path). The reference pushes row segments with
// the copy engine and flags a peer slot from the host-maintained seq
// (sglang/mailbox_ar_ext.cu:233-342), which is not graph-replay safe. Here the
// seq is device-resident: submit (side stream) pushes segment s into
// slot s%3 of every peer after that peer freed the slot, then releases a
// ready flag; wait (main stream) waits for every peer's flag, reduces, and
// acks the slot free to each pusher.
// --------------------------------------------------------------------------
MBX_DEVICE uint32_t* seg_ready(char* base, int slot, int src) {
  return reinterpret_cast<uint32_t*>(base + kSegReadyOff) + slot * kMaxRanks + src;
}
MBX_DEVICE uint32_t* seg_free(char* base, int slot, int src) {
  return reinterpret_cast<uint32_t*>(base + kSegFreeOff) + slot * kMaxRanks + src;
}
MBX_DEVICE char* seg_data(const ArCtx& c, char* base, int slot, int src) {
  return base + c.fuse_off + 2 * c.fuse_half_bytes + ((uint64_t)slot * kMaxRanks + src) * c.seg_slot_bytes;
}

template <int W>
__global__ void __launch_bounds__(kArThreads) seg_submit_kernel(ArCtx c, const uint4* __restrict__ in, uint64_t nvec) {
  __shared__ bool s_ok;
  const uint32_t seq = *reinterpret_cast<volatile uint32_t*>(c.state + kStSegSubmit) + 1u;
  const int slot = seq % kSegSlots;
  if (threadIdx.x == 0) s_ok = true;
  __syncthreads();
  if (!poisoned(c)) {
    // Slot reuse: every peer must have acked seq - kSegSlots. Only peers take
    // part (the own contribution never goes through a slot), so no kernel
    // waits on another kernel of the same GPU.
    if (threadIdx.x < W && threadIdx.x != c.rank && seq > (uint32_t)kSegSlots) {
      const int r = threadIdx.x;
      if (!wait_flag_geq(seg_free(c.bufs[c.rank], slot, r), seq - kSegSlots, c.timeout_ns)) {
        record_error(c, kErrSegFree, blockIdx.x, r, 10, seq);
        s_ok = false;
      }
    }
    __syncthreads();
    if (s_ok) {
      const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
      for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
        const uint4 v = ld_nc_v4(in + i);
#pragma unroll
        for (int j = 1; j < W; ++j) {
          const int r = (c.rank + j) % W;
          st_v4(seg_data(c, c.bufs[r], slot, c.rank) + i * 16, v);
        }
      }
    }
  }
  // Every block's stores must land before the single ready flag per peer: the
  // last block to finish releases the flags and advances the device seq (all
  // blocks have read it by then).
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_acq_rel_sys();
    const uint32_t prev = atomicAdd(c.state + kStSegSubmitDone, 1u);
    if (prev == gridDim.x - 1) {
      c.state[kStSegSubmitDone] = 0;
      if (!poisoned(c))
        for (int j = 1; j < W; ++j) st_release_sys(seg_ready(c.bufs[(c.rank + j) % W], slot, c.rank), seq);
      c.state[kStSegSubmit] = seq;
      __threadfence();
    }
  }
}

template <typename T, int W>
__global__ void __launch_bounds__(kArThreads) seg_wait_kernel(ArCtx c, const uint4* __restrict__ local,
                                                              uint4* __restrict__ out, uint64_t nvec) {
  __shared__ bool s_ok;
  const uint32_t seq = *reinterpret_cast<volatile uint32_t*>(c.state + kStSegWait) + 1u;
  const int slot = seq % kSegSlots;
  if (threadIdx.x == 0) s_ok = true;
  __syncthreads();
  if (!poisoned(c)) {
    if (threadIdx.x < W && threadIdx.x != c.rank) {
      const int r = threadIdx.x;
      if (!wait_flag_geq(seg_ready(c.bufs[c.rank], slot, r), seq, c.timeout_ns)) {
        record_error(c, kErrSegWait, blockIdx.x, r, 11, seq);
        s_ok = false;
      }
    }
    __syncthreads();
    if (s_ok) {
      const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
      for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
        float acc[Pack<T>::N] = {};
#pragma unroll
        for (int r = 0; r < W; ++r) {
          // rank order; the own contribution comes from the caller's tensor
          const uint4 v = (r == c.rank) ? ld_nc_v4(local + i) : ld_cg_v4(seg_data(c, c.bufs[c.rank], slot, r) + i * 16);
          unpack_add<T>(v, acc);
        }
        out[i] = pack_from<T>(acc);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_acq_rel_sys();
    const uint32_t prev = atomicAdd(c.state + kStSegWaitDone, 1u);
    if (prev == gridDim.x - 1) {
      c.state[kStSegWaitDone] = 0;
      c.state[kStSegWait] = seq;
      // free the slot for every pushing peer
      if (!poisoned(c))
        for (int j = 1; j < W; ++j) st_release_sys(seg_free(c.bufs[(c.rank + j) % W], slot, c.rank), seq);
      __threadfence();
    }
  }
}

// --------------------------------------------------------------------------
// All-gather (one-shot push): out[r] = in of rank r, for every rank r. Used
// by the vocab-parallel argmax combine and the sequence-parallel paths.
// --------------------------------------------------------------------------
template <int W>
MBX_DEVICE void ar_allgather(const ArCtx& c, const uint4* __restrict__ in, uint4* __restrict__ out, uint64_t nvec) {
  __shared__ bool s_ok;
  const uint32_t epoch = call_epoch(c);
  trace_mark(c, 0);
  if (!poisoned(c)) {
    const uint64_t slot = oneshot_slot_bytes(c.half_bytes, W);
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t i0 = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (uint64_t i = i0; i < nvec; i += stride) {
      const uint4 v = ld_nc_v4(in + i);
#pragma unroll
      for (int j = 0; j < W; ++j) {
        const int r = (c.rank + j) % W;
        st_v4(data_half(c.bufs[r], epoch, c.half_bytes) + c.rank * slot + i * 16, v);
      }
    }
    trace_mark(c, 1);
    if (block_barrier(c, 0, epoch, &s_ok)) {
      trace_mark(c, 2);
      const char* mine = data_half(c.bufs[c.rank], epoch, c.half_bytes);
      for (uint64_t i = i0; i < nvec; i += stride) {
#pragma unroll
        for (int r = 0; r < W; ++r) out[r * nvec + i] = ld_cg_v4(mine + r * slot + i * 16);
      }
    }
  }
  finish_call(c, epoch);
}

template <int W>
__global__ void __launch_bounds__(kArThreads) ar_allgather_kernel(ArCtx c, const uint4* __restrict__ in,
                                                                  uint4* __restrict__ out, uint64_t nvec) {
  pdl_wait();
  ar_allgather<W>(c, in, out, nvec);
}

// --------------------------------------------------------------------------
// Raw peer-store bench kernel (16-byte stores, capped grid): same role as the
// reference's push microbench (sglang/mailbox_ar_ext.cu:201-221).
// --------------------------------------------------------------------------
// --------------------------------------------------------------------------
// Raw transport kernels for the NVLink bandwidth benchmarks (the counterpart
// of the reference's raw mailbox push bench, sglang/mailbox_ar_ext.cu:201-221):
// SM stores into a peer (U vectors in flight per thread), SM loads from a
// peer, NVLS multimem.ld_reduce from a multicast address (with or without
// fp32 accumulation) and multimem.st to one.
// --------------------------------------------------------------------------
template <int U>
__global__ void push_raw_kernel(uint4* __restrict__ dst, const uint4* __restrict__ src, uint64_t nvec) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride * U) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (i + u * stride < nvec) v[u] = ld_nc_v4(src + i + u * stride);
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (i + u * stride < nvec) st_v4(dst + i + u * stride, v[u]);
  }
}

__global__ void pull_raw_kernel(uint4* __restrict__ dst, const uint4* __restrict__ src, uint64_t nvec) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride * kU) {
    uint4 v[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (i + u * stride < nvec) v[u] = ld_cg_v4(src + i + u * stride);
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (i + u * stride < nvec) dst[i + u * stride] = v[u];
  }
}

MBX_DEVICE uint4 multimem_ld_reduce_bf16_noacc(const void* mc) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}

template <bool kAcc>
__global__ void mc_reduce_raw_kernel(uint4* __restrict__ dst, const char* mc, uint64_t nvec) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride * kU) {
    uint4 v[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (i + u * stride < nvec)
        v[u] = kAcc ? multimem_ld_reduce<__nv_bfloat16>(mc + (i + u * stride) * 16)
                    : multimem_ld_reduce_bf16_noacc(mc + (i + u * stride) * 16);
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (i + u * stride < nvec) dst[i + u * stride] = v[u];
  }
}

__global__ void mc_store_raw_kernel(char* mc, const uint4* __restrict__ src, uint64_t nvec) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride * kU) {
    uint4 v[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (i + u * stride < nvec) v[u] = ld_nc_v4(src + i + u * stride);
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (i + u * stride < nvec) multimem_st(mc + (i + u * stride) * 16, v[u]);
  }
}

// ==========================================================================
// Host side
// ==========================================================================
#define MBX_DISPATCH_W(W_, ...)                   \
  switch (W_) {                                   \
    case 2: { constexpr int W = 2; __VA_ARGS__; } break; \
    case 4: { constexpr int W = 4; __VA_ARGS__; } break; \
    case 8: { constexpr int W = 8; __VA_ARGS__; } break; \
    case 3: { constexpr int W = 3; __VA_ARGS__; } break; \
    case 5: { constexpr int W = 5; __VA_ARGS__; } break; \
    case 6: { constexpr int W = 6; __VA_ARGS__; } break; \
    case 7: { constexpr int W = 7; __VA_ARGS__; } break; \
    default: throw std::runtime_error("allreduce: unsupported world size " + std::to_string(W_)); \
  }

// The fused GEMM/norm launches also take world 1: a single-GPU emulation in
// which every push lands in the rank's own buffer (kernel profiling on one GPU).
#define MBX_DISPATCH_W1(W_, ...)                                   \
  if ((W_) == 1) {                                                 \
    constexpr int W = 1;                                           \
    __VA_ARGS__;                                                   \
  } else {                                                         \
    MBX_DISPATCH_W(W_, __VA_ARGS__)                                \
  }

#define MBX_DISPATCH_T(D_, ...)                                  \
  switch (D_) {                                                  \
    case kF32: { using T = float; __VA_ARGS__; } break;          \
    case kF16: { using T = __half; __VA_ARGS__; } break;         \
    case kBF16: { using T = __nv_bfloat16; __VA_ARGS__; } break; \
    default: throw std::runtime_error("allreduce: unsupported dtype id"); \
  }

static inline int ar_grid(uint64_t work_vec, int max_blocks) {
  uint64_t g = (work_vec + kArThreads - 1) / kArThreads;
  if (g < 1) g = 1;
  if (g > (uint64_t)max_blocks) g = max_blocks;
  if (g > (uint64_t)kMaxBlocks) g = kMaxBlocks;
  return (int)g;
}

// Largest message (bytes) one launch of `algo` can carry through the buffer.
uint64_t ar_chunk_limit(const ArCtx& c, int algo) {
  switch (algo) {
    case kOneShotPush: return oneshot_slot_bytes(c.half_bytes, c.world);
    case kOneShotPull: return c.half_bytes & ~uint64_t(15);
    case kTwoShot:
    case kNvls: return (c.half_bytes / 2) & ~uint64_t(15);
    case kTwoShotPush: return ((c.half_bytes / 2 - 16 * (uint64_t)c.world) / 16) * 16;
  }
  return 0;
}

void ar_launch(const ArCtx& c, int algo, int dtype, const void* in, void* out, uint64_t nbytes,
               int max_blocks, cudaStream_t stream) {
  if (nbytes % 16 != 0) throw std::runtime_error("allreduce: byte size must be a multiple of 16");
  if (algo == kNvls && c.mc == nullptr) throw std::runtime_error("allreduce: NVLS requested without multicast");
  const uint64_t limit = ar_chunk_limit(c, algo);
  if (limit == 0) throw std::runtime_error("allreduce: bad algorithm id");
  const char* ip = static_cast<const char*>(in);
  char* op = static_cast<char*>(out);
  for (uint64_t off = 0; off < nbytes || (nbytes == 0 && off == 0); off += limit) {
    const uint64_t cur = std::min(limit, nbytes - off);
    const uint64_t nvec = cur / 16;
    const uint4* i4 = reinterpret_cast<const uint4*>(ip + off);
    uint4* o4 = reinterpret_cast<uint4*>(op + off);
    const int W_ = c.world;
    if (algo == kOneShotPush || algo == kOneShotPull) {
      const int g = ar_grid(nvec, max_blocks);
      MBX_DISPATCH_T(dtype, MBX_DISPATCH_W(W_, {
        if (algo == kOneShotPush) launch_k(ar_oneshot_push_kernel<T, W>, dim3(g), dim3(kArThreads), 0, stream,
                                           c, i4, o4, nvec);
        else launch_k(ar_oneshot_pull_kernel<T, W>, dim3(g), dim3(kArThreads), 0, stream, c, i4, o4, nvec);
      }));
    } else {
      const int g = ar_grid((nvec + W_ - 1) / W_, max_blocks);
      MBX_DISPATCH_T(dtype, MBX_DISPATCH_W(W_, {
        if (algo == kTwoShot) launch_k(ar_twoshot_kernel<T, W>, dim3(g), dim3(kArThreads), 0, stream, c, i4, o4, nvec);
        else if (algo == kTwoShotPush) launch_k(ar_twoshot_push_kernel<T, W>, dim3(g), dim3(kArThreads), 0, stream,
                                                c, i4, o4, nvec);
        else launch_k(ar_nvls_kernel<T, W>, dim3(g), dim3(kArThreads), 0, stream, c, i4, o4, nvec);
      }));
    }
    MBX_CUDA_CHECK(cudaGetLastError());
    if (nbytes == 0) break;
  }
}

void ar_rmsnorm_launch(const ArCtx& c, int algo, const void* in, void* residual, const void* weight, void* out,
                       int M, int H, float eps, int max_blocks, cudaStream_t stream, int threads) {
  if (H % 8 != 0) throw std::runtime_error("ar_rmsnorm: hidden size must be a multiple of 8");
  if (threads != 256 && threads != kArThreads) throw std::runtime_error("ar_rmsnorm: threads must be 256 or 512");
  const uint64_t bytes = (uint64_t)M * H * 2;
  const int g = std::max(1, std::min(M, std::min(max_blocks, (int)kMaxBlocks)));
  const int W_ = c.world;
  auto i4 = static_cast<const uint4*>(in);
  auto r4 = static_cast<uint4*>(residual);
  auto w4 = static_cast<const uint4*>(weight);
  auto o4 = static_cast<uint4*>(out);
  if (algo == kOneShotPush) {
    if (bytes > ar_chunk_limit(c, kOneShotPush)) throw std::runtime_error("ar_rmsnorm: message exceeds one-shot slot");
    MBX_DISPATCH_W1(W_, launch_k(ar_rmsnorm_oneshot_kernel<W>, dim3(g), dim3(threads), 0, stream,
                                 c, i4, r4, w4, o4, M, H, eps));
  } else if (algo == kTwoShotPush) {
    const int Mo = (M + W_ - 1) / W_;
    if ((uint64_t)W_ * Mo * H * 2 + bytes > c.half_bytes)
      throw std::runtime_error("ar_rmsnorm: message exceeds the two-shot buffer");
    const int gp = std::max(1, std::min(Mo, std::min(max_blocks, (int)kMaxBlocks)));
    MBX_DISPATCH_W1(W_, launch_k(ar_rmsnorm_twoshot_push_kernel<W>, dim3(gp), dim3(threads), 0, stream,
                                 c, i4, r4, w4, o4, M, H, eps));
  } else {
    if (bytes > ar_chunk_limit(c, kTwoShot)) throw std::runtime_error("ar_rmsnorm: message exceeds two-shot slot");
    MBX_DISPATCH_W(W_, launch_k(ar_rmsnorm_twoshot_kernel<W>, dim3(g), dim3(threads), 0, stream,
                                c, i4, r4, w4, o4, M, H, eps));
  }
  MBX_CUDA_CHECK(cudaGetLastError());
}

void ar_allgather_launch(const ArCtx& c, const void* in, void* out, uint64_t nbytes, int max_blocks,
                         cudaStream_t stream) {
  if (nbytes % 16 != 0) throw std::runtime_error("allgather: byte size must be a multiple of 16");
  if (nbytes > ar_chunk_limit(c, kOneShotPush)) throw std::runtime_error("allgather: message exceeds slot");
  const uint64_t nvec = nbytes / 16;
  const int g = ar_grid(nvec, max_blocks);
  const int W_ = c.world;
  MBX_DISPATCH_W(W_, launch_k(ar_allgather_kernel<W>, dim3(g), dim3(kArThreads), 0, stream,
                              c, static_cast<const uint4*>(in),
                                                                           static_cast<uint4*>(out), nvec));
  MBX_CUDA_CHECK(cudaGetLastError());
}

void fused_rs_norm_launch(const ArCtx& c, int M, int N, int Mo, void* residual, const void* weight, void* out,
                          float eps, int max_blocks, cudaStream_t stream) {
  const int g = std::max(1, std::min(Mo, std::min(max_blocks, (int)kMaxBlocks)));
  const int W_ = c.world;
  MBX_DISPATCH_W1(W_, launch_k(fused_rs_norm_kernel<W>, dim3(g), dim3(kArThreads), 0, stream,
                         c, M, N, Mo, static_cast<uint4*>(residual), static_cast<const uint4*>(weight),
                         static_cast<uint4*>(out), eps));
  MBX_CUDA_CHECK(cudaGetLastError());
}

void fused_allsum_norm_launch(const ArCtx& c, int M, int N, void* residual, const void* weight, void* out, float eps,
                              int max_blocks, cudaStream_t stream) {
  const int g = std::max(1, std::min(M, std::min(max_blocks, (int)kMaxBlocks)));
  const int W_ = c.world;
  MBX_DISPATCH_W1(W_, launch_k(fused_allsum_norm_kernel<W>, dim3(g), dim3(kArThreads), 0, stream,
                         c, M, N, static_cast<uint4*>(residual), static_cast<const uint4*>(weight),
                         static_cast<uint4*>(out), eps));
  MBX_CUDA_CHECK(cudaGetLastError());
}

void sp_rs_push_launch(const ArCtx& c, const void* x, int M, int N, int max_blocks, cudaStream_t stream) {
  if (M == 0) return;
  if (N % 8 != 0) throw std::runtime_error("sp_rs_push: N must be a multiple of 8");
  const int W_ = c.world;
  const int Mo = (M + W_ - 1) / W_;
  if ((uint64_t)W_ * Mo * N * 2 > c.fuse_half_bytes)
    throw std::runtime_error("sp_rs_push: message exceeds the reduce-scatter buffer");
  const int g = ar_grid((uint64_t)M * N / 8, max_blocks);
  MBX_DISPATCH_W1(W_, launch_k(sp_rs_push_kernel<W>, dim3(g), dim3(kArThreads), 0, stream,
                               c, static_cast<const uint4*>(x), M, N, Mo));
  MBX_CUDA_CHECK(cudaGetLastError());
}

void sp_rs_norm_ag_launch(const ArCtx& c, int M, int N, void* res_own, const void* w, float eps, int max_blocks,
                          cudaStream_t stream) {
  if (M == 0) return;
  if (N % 8 != 0) throw std::runtime_error("sp_rs_norm_ag: N must be a multiple of 8");
  const int W_ = c.world;
  const int Mo = (M + W_ - 1) / W_;
  if ((uint64_t)M * N * 2 > c.sp_bytes) throw std::runtime_error("sp_rs_norm_ag: rows exceed the gather buffer");
  const int g = std::max(1, std::min(Mo, std::min(max_blocks, (int)kMaxBlocks)));
  MBX_DISPATCH_W1(W_, launch_k(sp_rs_norm_ag_kernel<W>, dim3(g), dim3(kArThreads), 0, stream,
                         c, M, N, Mo, static_cast<uint4*>(res_own), static_cast<const uint4*>(w), eps));
  MBX_CUDA_CHECK(cudaGetLastError());
}

void sp_ag_wait_launch(const ArCtx& c, int M, cudaStream_t stream) {
  if (M == 0) return;
  const int Mo = (M + c.world - 1) / c.world;
  const int owners = std::min(c.world, (M + Mo - 1) / Mo);
  launch_k(sp_ag_wait_kernel, dim3(1), dim3(32), 0, stream, c, owners);
  MBX_CUDA_CHECK(cudaGetLastError());
}

void seg_submit_launch(const ArCtx& c, const void* in, uint64_t nbytes, int max_blocks, cudaStream_t stream) {
  if (nbytes % 16 != 0 || nbytes > c.seg_slot_bytes)
    throw std::runtime_error("submit_seg: segment must be a multiple of 16 bytes and <= slot size " +
                             std::to_string(c.seg_slot_bytes));
  const uint64_t nvec = nbytes / 16;
  const int g = ar_grid(nvec, max_blocks);
  const int W_ = c.world;
  MBX_DISPATCH_W(W_, seg_submit_kernel<W><<<g, kArThreads, 0, stream>>>(c, static_cast<const uint4*>(in), nvec));
  MBX_CUDA_CHECK(cudaGetLastError());
}

void seg_wait_launch(const ArCtx& c, int dtype, const void* local, void* out, uint64_t nbytes, int max_blocks,
                     cudaStream_t stream) {
  if (nbytes % 16 != 0 || nbytes > c.seg_slot_bytes)
    throw std::runtime_error("wait_seg: bad segment size");
  const uint64_t nvec = nbytes / 16;
  const int g = ar_grid(nvec, max_blocks);
  const int W_ = c.world;
  MBX_DISPATCH_T(dtype, MBX_DISPATCH_W(W_, seg_wait_kernel<T, W><<<g, kArThreads, 0, stream>>>(
                                              c, static_cast<const uint4*>(local), static_cast<uint4*>(out), nvec)));
  MBX_CUDA_CHECK(cudaGetLastError());
}

void raw_transport_launch(int kind, void* dst, const void* src, uint64_t nbytes, int grid, int threads,
                          cudaStream_t stream) {
  if (nbytes % 16 != 0) throw std::runtime_error("raw transport: bytes must be a multiple of 16");
  if (grid < 1 || grid > 65535 || threads < 32 || threads > 1024 || threads % 32)
    throw std::runtime_error("raw transport: bad launch shape");
  const uint64_t nvec = nbytes / 16;
  auto d4 = static_cast<uint4*>(dst);
  auto s4 = static_cast<const uint4*>(src);
  switch (kind) {
    case kRawPush1: push_raw_kernel<1><<<grid, threads, 0, stream>>>(d4, s4, nvec); break;
    case kRawPush4: push_raw_kernel<4><<<grid, threads, 0, stream>>>(d4, s4, nvec); break;
    case kRawPull4: pull_raw_kernel<<<grid, threads, 0, stream>>>(d4, s4, nvec); break;
    case kRawMcReduce: mc_reduce_raw_kernel<true><<<grid, threads, 0, stream>>>(d4, static_cast<const char*>(src), nvec); break;
    case kRawMcReduceNoAcc:
      mc_reduce_raw_kernel<false><<<grid, threads, 0, stream>>>(d4, static_cast<const char*>(src), nvec);
      break;
    case kRawMcStore: mc_store_raw_kernel<<<grid, threads, 0, stream>>>(static_cast<char*>(dst), s4, nvec); break;
    default: throw std::runtime_error("raw transport: unknown kind");
  }
  MBX_CUDA_CHECK(cudaGetLastError());
}


// --------------------------------------------------------------------------
// One-GPU emulation of a W-rank call, for tests and single-GPU profiling.
// Kernels that wait on one another cannot run as separate launches on one
// GPU: nothing makes them co-resident. So every emulated rank's blocks run in
// ONE cooperative launch (co-residency guaranteed, or the launch is refused):
// blockIdx.y is the rank, blockIdx.x / gridDim.x keep their per-rank meaning,
// and each rank brings its own context (symmetric buffers of all emulated
// ranks, its own state and status words). The device code is the same body
// the multi-GPU launch runs; only the memory behind the "peer" pointers is
// local.
// --------------------------------------------------------------------------
template <typename T, int W>
__global__ void __launch_bounds__(kArThreads) ar_emulated_kernel(const EmuRank* __restrict__ ranks, int op, int algo,
                                                                 uint64_t nvec, int M, int N, float eps) {
  const EmuRank& er = ranks[blockIdx.y];
  const ArCtx c = er.c;
  const uint4* in = static_cast<const uint4*>(er.in);
  uint4* out = static_cast<uint4*>(er.out);
  uint4* res = static_cast<uint4*>(er.residual);
  const uint4* w = static_cast<const uint4*>(er.weight);
  if (op == kEmuAllreduce) {
    switch (algo) {
      case kOneShotPush: ar_oneshot_push<T, W>(c, in, out, nvec); break;
      case kOneShotPull: ar_oneshot_pull<T, W>(c, in, out, nvec); break;
      case kTwoShot: ar_twoshot<T, W>(c, in, out, nvec); break;
      case kTwoShotPush: ar_twoshot_push<T, W>(c, in, out, nvec); break;
    }
  } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    if (op == kEmuArRmsnorm) {
      if (algo == kOneShotPush) ar_rmsnorm_oneshot<W>(c, in, res, w, out, M, N, eps);
      else if (algo == kTwoShotPush) ar_rmsnorm_twoshot_push<W>(c, in, res, w, out, M, N, eps);
      else ar_rmsnorm_twoshot<W>(c, in, res, w, out, M, N, eps);
    } else if (op == kEmuFusedRsNorm) {
      fused_rs_norm<W>(c, M, N, (M + W - 1) / W, res, w, out, eps);
    } else if (op == kEmuAllgather) {
      ar_allgather<W>(c, in, out, nvec);
    }
  }
}

void ar_emulated_launch(const EmuRank* ranks_host, int world, int op, int algo, int dtype, uint64_t nbytes, int M,
                        int N, float eps, int blocks, void* dev_scratch, cudaStream_t stream, int threads) {
  if (threads != 256 && threads != kArThreads) throw std::runtime_error("emulated allreduce: threads must be 256 or 512");
  if (world < 2 || world > kMaxRanks) throw std::runtime_error("emulated allreduce: world must be 2..8");
  if (nbytes % 16 != 0) throw std::runtime_error("emulated allreduce: byte size must be a multiple of 16");
  if (op == kEmuAllreduce) {
    if (algo != kOneShotPush && algo != kOneShotPull && algo != kTwoShot && algo != kTwoShotPush)
      throw std::runtime_error("emulated allreduce: algorithm must be one-shot push/pull or two-shot (push)");
    if (nbytes > ar_chunk_limit(ranks_host[0].c, algo))
      throw std::runtime_error("emulated allreduce: message exceeds one launch of the algorithm");
  } else if (dtype != kBF16) {
    throw std::runtime_error("emulated fused kernels are bf16 only");
  } else if (op == kEmuArRmsnorm || op == kEmuFusedRsNorm) {
    if (N % 8 != 0 || M < 1) throw std::runtime_error("emulated norm: bad shape");
    const uint64_t bytes = (uint64_t)M * N * 2;
    const int Mo = (M + world - 1) / world;
    const ArCtx& c0 = ranks_host[0].c;
    if (op == kEmuFusedRsNorm) {
      if ((uint64_t)world * Mo * N * 2 + bytes > c0.fuse_half_bytes)
        throw std::runtime_error("emulated fused reduce: rows exceed the fused buffer");
    } else if (algo == kOneShotPush) {
      if (bytes > ar_chunk_limit(c0, kOneShotPush)) throw std::runtime_error("emulated norm: exceeds one-shot slot");
    } else if (algo == kTwoShotPush) {
      if ((uint64_t)world * Mo * N * 2 + bytes > c0.half_bytes)
        throw std::runtime_error("emulated norm: exceeds the two-shot buffer");
    } else if (bytes > ar_chunk_limit(c0, kTwoShot)) {
      throw std::runtime_error("emulated norm: exceeds two-shot slot");
    }
  } else if (op == kEmuAllgather) {
    if (nbytes > ar_chunk_limit(ranks_host[0].c, kOneShotPush))
      throw std::runtime_error("emulated all-gather: message exceeds slot");
  } else {
    throw std::runtime_error("emulated allreduce: unknown op");
  }
  if (dtype != kBF16 && dtype != kF32) throw std::runtime_error("emulated allreduce: dtype must be bf16 or fp32");
  if (blocks < 1 || blocks > kMaxBlocks) throw std::runtime_error("emulated allreduce: bad block count");
  MBX_CUDA_CHECK(cudaMemcpyAsync(dev_scratch, ranks_host, sizeof(EmuRank) * world, cudaMemcpyHostToDevice, stream));
  const EmuRank* ranks = static_cast<const EmuRank*>(dev_scratch);
  uint64_t nvec = nbytes / 16;
  dim3 grid(blocks, world);
  void* args[] = {&ranks, &op, &algo, &nvec, &M, &N, &eps};
  auto go = [&](const void* fn) {
    MBX_CUDA_CHECK(cudaLaunchCooperativeKernel(fn, grid, dim3(threads), args, 0, stream));
  };
  const bool f32 = dtype == kF32;
  auto pick = [&](auto wc) -> const void* {
    constexpr int W = decltype(wc)::value;
    return f32 ? (const void*)ar_emulated_kernel<float, W> : (const void*)ar_emulated_kernel<__nv_bfloat16, W>;
  };
  switch (world) {
    case 2: go(pick(std::integral_constant<int, 2>{})); break;
    case 3: go(pick(std::integral_constant<int, 3>{})); break;
    case 4: go(pick(std::integral_constant<int, 4>{})); break;
    case 8: go(pick(std::integral_constant<int, 8>{})); break;
    default: throw std::runtime_error("emulated allreduce: world sizes 2, 3, 4 and 8");
  }
}

}  // namespace mbx
