// Symmetric-buffer layout constants and the allreduce launch context
// (host-safe: no device code). Device helpers are in ar_common.cuh.
//
// Layout of every rank's symmetric buffer (identical offsets on all ranks, so a
// peer address is peer_base + offset):
//
//   [0, kSigBytes)        signal words
//       bar[phase][block][src]     u32 epoch written by rank `src`
//       seg_ready[slot][src]       u32 segment seq written by the pusher
//       seg_free[slot][src]        u32 segment seq acked by the receiver
//       tile_ready[slot][src]      u32 per-row-block flags of fused epilogues
//   [kSigBytes, +2*half)  two ping-pong data halves (call epoch parity)
//   [fuse_off, +2*fuse)   two ping-pong halves of the fused GEMM->allreduce
//                         path (own epoch, so it never shares memory with
//                         a plain allreduce that may overlap it across ranks)
//   [.., + seg region)    segmented-allreduce slots
//
// The reference keeps a [flag][ack][pad] header plus two 24 MB halves in a
// 64 MB pairwise mailbox (sglang/mailbox_ar_ext.cu:6-7,16-23); here the header
// is generalised to per-(phase, block, source-rank) epoch words so one buffer
// serves TP=2/4/8 and every algorithm.
#pragma once
#include <stddef.h>
#include <stdint.h>

namespace mbx {


constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 256;
constexpr int kPhases = 4;
constexpr int kSegSlots = 3;
constexpr int kTileFlagSlots = 4096;  // row-block flags for the fused GEMM epilogues
constexpr size_t kBarOff = 0;
constexpr size_t kSegReadyOff = kBarOff + sizeof(uint32_t) * kPhases * kMaxBlocks * kMaxRanks;
constexpr size_t kSegFreeOff = kSegReadyOff + sizeof(uint32_t) * kSegSlots * kMaxRanks;
constexpr size_t kTileFlagOff = kSegFreeOff + sizeof(uint32_t) * kSegSlots * kMaxRanks;
constexpr size_t kSigBytes = 1 << 20;  // 1 MiB signal area (keeps data 1 MiB aligned)
// Sequence-parallel all-gather flags: word `owner` = epoch of the last
// all-gather whose rows from `owner` have landed in this rank's gather buffer.
constexpr size_t kAgFlagOff = kTileFlagOff + sizeof(uint32_t) * 64;
static_assert(kTileFlagOff + sizeof(uint32_t) * kTileFlagSlots * kMaxRanks <= kSigBytes,
              "signal area overflow");

// One rank's slot of a one-shot half: half / world rounded down to 256 bytes.
// Every slot must start 16-byte aligned for the vector stores whatever the
// world size (half / 3 of a power of two is not even a multiple of 16).
// constexpr, so host code and device code (--expt-relaxed-constexpr) share it.
constexpr uint64_t oneshot_slot_bytes(uint64_t half_bytes, int world) {
  return (half_bytes / (uint64_t)world) & ~uint64_t(255);
}

// Device-local (not symmetric) state words.
enum StateWord : int {
  kStEpoch = 0,     // epoch of the last completed allreduce call
  kStDone = 1,      // blocks finished in the current call
  kStErr = 2,       // sticky device-side error copy (fast early-exit check)
  kStSegSubmit = 3,      // segmented path: last submitted seq
  kStSegWait = 4,        // segmented path: last reduced seq
  kStSegSubmitDone = 5,  // blocks finished in the current submit
  kStSegWaitDone = 6,    // blocks finished in the current wait
  kStFuseEpoch = 7,      // fused GEMM-epilogue path epoch
  kStFuseDone = 8,       // blocks finished in the current fused reduce kernel
  kStFuseGemmDone = 9,   // GEMM CTAs finished pushing in the current fused call
  kStSpAgDone = 10,      // blocks finished pushing in the current sequence-parallel all-gather
  kStWords = 16
};

// Host-mapped status words (readable without a device sync).
enum StatusWord : int {
  kStatusErr = 0,    // 0 ok; else error code (below)
  kStatusBlock = 1,  // block that gave up
  kStatusPeer = 2,   // peer it was waiting for
  kStatusPhase = 3,  // protocol phase
  kStatusEpoch = 4,  // epoch it waited for
  kStatusWords = 8
};

// Error codes. 2/3/4/5 keep the meaning of the reference's codes
// (sglang/mailbox_ar_ext.cu:30,41,259,290: ack wait, flag wait, segment wait,
// slot-free wait).
enum ErrCode : uint32_t {
  kErrNone = 0,
  kErrBarrier = 3,
  kErrSegWait = 4,
  kErrSegFree = 5,
  kErrFuseWait = 6,
};

struct ArCtx {
  char* bufs[kMaxRanks];   // symmetric buffer base of every rank (bufs[rank] is local)
  char* mc;                // multicast (NVLS) mapping of the same buffers, or nullptr
  uint32_t* state;         // device-local state words (StateWord)
  uint32_t* status;        // host-mapped status words (StatusWord)
  uint64_t timeout_ns;     // bound of every device-side wait
  uint64_t half_bytes;     // size of one ping-pong data half
  uint64_t seg_slot_bytes; // size of one segmented slot (per source rank)
  uint64_t fuse_off;       // byte offset of the fused path's halves
  uint64_t fuse_half_bytes;// size of one fused half (0 = fused path disabled)
  uint64_t sp_off;         // byte offset of the sequence-parallel gather buffer G (0 = none)
  uint64_t sp_bytes;       // its size
  uint64_t* trace;         // optional device array of phase timestamps (block 0), or nullptr
  int rank;
  int world;
};

}  // namespace mbx
