// Device-side helpers of the cross-GPU protocols (barriers, epochs, error
// recording, cache-bypassing vector loads). Layout constants and the launch
// context are in ar_ctx.h.
#pragma once
#include "../common.cuh"
#include "ar_ctx.h"

namespace mbx {

MBX_DEVICE uint32_t* bar_flag(char* base, int phase, int block, int src) {
  return reinterpret_cast<uint32_t*>(base + kBarOff) +
         ((phase * kMaxBlocks + block) * kMaxRanks + src);
}

MBX_DEVICE char* data_half(char* base, uint32_t epoch, uint64_t half_bytes) {
  return base + kSigBytes + (uint64_t)(epoch & 1u) * half_bytes;
}

MBX_DEVICE void record_error(const ArCtx& c, uint32_t code, int block, int peer, int phase,
                             uint32_t epoch) {
  // First error wins; later ones keep the original diagnosis. The atomic is on
  // device memory; the host-mapped copy is written with plain stores (PCIe
  // atomics to host memory are not assumed).
  if (atomicCAS(c.state + kStErr, 0u, code) == 0u) {
    volatile uint32_t* s = c.status;
    s[kStatusBlock] = block;
    s[kStatusPeer] = peer;
    s[kStatusPhase] = phase;
    s[kStatusEpoch] = epoch;
    __threadfence_system();
    s[kStatusErr] = code;
    __threadfence_system();
  }
}

// Pairwise block barrier across ranks: block `b` of this rank tells block `b`
// of every rank that it reached `phase` of call `epoch`, then waits for all of
// them. Data written before the barrier (by any thread of the block) is
// visible to the peers after it: __syncthreads orders the block's stores
// before the signalling thread's system-scope release, and the waiting
// thread's acquire is ordered before the block's later loads by the trailing
// __syncthreads. Returns false (after recording the error) on timeout.
// Phase timestamp of block 0 (benchmarks only; c.trace is null otherwise).
// Slot k holds %globaltimer at mark k of the last call.
MBX_DEVICE void trace_mark(const ArCtx& c, int k) {
  if (c.trace != nullptr && blockIdx.x == 0 && threadIdx.x == 0) c.trace[k] = globaltimer_ns();
}

MBX_DEVICE bool block_barrier(const ArCtx& c, int phase, uint32_t epoch, bool* s_ok) {
  const int b = blockIdx.x;
  const int t = threadIdx.x;
  if (t == 0) *s_ok = true;
  __syncthreads();
  if (t < c.world) {
    st_release_sys(bar_flag(c.bufs[t], phase, b, c.rank), epoch);
  }
  if (t < c.world) {
    if (!wait_flag_geq(bar_flag(c.bufs[c.rank], phase, b, t), epoch, c.timeout_ns)) {
      record_error(c, kErrBarrier, b, t, phase, epoch);
      *s_ok = false;
    }
  }
  __syncthreads();
  return *s_ok;
}

// Every block of a call ends here. The last block to finish publishes the new
// epoch (device-resident, so CUDA-graph replays advance it without the host;
// same role as the reference's round counter, sglang/mailbox_ar_ext.cu:112-115).
MBX_DEVICE void finish_call(const ArCtx& c, uint32_t epoch, int word_epoch = kStEpoch,
                            int word_done = kStDone) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(c.state + word_done, 1u);
    if (prev == gridDim.x - 1) {
      c.state[word_done] = 0;
      c.state[word_epoch] = epoch;
      __threadfence();
    }
  }
}

MBX_DEVICE uint4 ld_cg_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

MBX_DEVICE uint4 ld_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

}  // namespace mbx
