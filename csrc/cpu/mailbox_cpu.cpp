// CPU mailbox allreduce: the lockstep push protocol run by host processes over
// a shared mmap, with std::atomic flags.
//
// It is the host-side model of the device protocol in csrc/ar/allreduce.cu
// (one-shot push, one epoch per call, two ping-pong halves, wrap-safe epoch
// compare, fp32 accumulation in rank order with a single rounding) and is what
// the communicator uses when its tensors live on the CPU (gloo groups). The
// reference's protocol is pairwise and GPU-only (sglang/mailbox_ar_ext.cu:
// 124-167: waitack -> push -> flag -> wait -> reduce -> ack); this engine
// generalises it to world sizes 2..8.
//
// Shared file layout (all ranks map the same file):
//   [0, 4096)                    flags[dst][src] (u32, written by src)
//   [4096, ..)                   mailbox[dst][half][src][slot_bytes]
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "mailbox_cpu.h"

namespace mbx {

namespace {
constexpr size_t kHdr = 4096;
constexpr int kMaxW = 8;

inline float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// Round-to-nearest-even float -> bf16 (NaN stays NaN).
inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  const uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

inline float f16_to_f32(uint16_t h) {
  _Float16 x;
  std::memcpy(&x, &h, 2);
  return (float)x;
}

inline uint16_t f32_to_f16(float f) {
  _Float16 x = (_Float16)f;  // IEEE round-to-nearest-even
  uint16_t h;
  std::memcpy(&h, &x, 2);
  return h;
}

inline int elem_size(int dtype) { return dtype == 0 ? 4 : 2; }
}  // namespace

CpuMailbox::CpuMailbox(const std::string& path, int rank, int world, size_t slot_bytes, bool create,
                       int64_t timeout_ms)
    : path_(path), rank_(rank), world_(world), slot_bytes_(slot_bytes), timeout_ms_(timeout_ms), owner_(create) {
  if (world < 1 || world > kMaxW) throw std::runtime_error("CpuMailbox: world size must be 1..8");
  if (rank < 0 || rank >= world) throw std::runtime_error("CpuMailbox: bad rank");
  if (slot_bytes % 64 != 0) throw std::runtime_error("CpuMailbox: slot_bytes must be a multiple of 64");
  size_ = kHdr + (size_t)world * 2 * world * slot_bytes;
  int flags = O_RDWR | O_CLOEXEC | (create ? (O_CREAT | O_TRUNC) : 0);
  fd_ = ::open(path.c_str(), flags, 0600);
  if (fd_ < 0) throw std::runtime_error("CpuMailbox: open(" + path + ") failed: " + std::strerror(errno));
  if (create && ::ftruncate(fd_, (off_t)size_) != 0) {
    ::close(fd_);
    throw std::runtime_error("CpuMailbox: ftruncate failed");
  }
  struct stat st;
  if (::fstat(fd_, &st) != 0 || (size_t)st.st_size < size_) {
    ::close(fd_);
    throw std::runtime_error("CpuMailbox: shared file too small (creator not ready?)");
  }
  void* p = ::mmap(nullptr, size_, PROT_READ | PROT_WRITE, MAP_SHARED, fd_, 0);
  if (p == MAP_FAILED) {
    ::close(fd_);
    throw std::runtime_error("CpuMailbox: mmap failed");
  }
  base_ = static_cast<char*>(p);
  if (create) std::memset(base_, 0, kHdr);
}

CpuMailbox::~CpuMailbox() { close(); }

void CpuMailbox::close() {
  if (base_) {
    ::munmap(base_, size_);
    base_ = nullptr;
  }
  if (fd_ >= 0) {
    ::close(fd_);
    fd_ = -1;
    if (owner_) ::unlink(path_.c_str());
  }
}

std::atomic<uint32_t>* CpuMailbox::flag(int dst, int src) const {
  return reinterpret_cast<std::atomic<uint32_t>*>(base_) + dst * kMaxW + src;
}

char* CpuMailbox::slot(int dst, int half, int src) const {
  return base_ + kHdr + (((size_t)dst * 2 + half) * world_ + src) * slot_bytes_;
}

int CpuMailbox::allreduce(const void* in, void* out, size_t nbytes, int dtype) {
  if (!base_) throw std::runtime_error("CpuMailbox: closed");
  if (err_) return err_;
  if (nbytes > slot_bytes_) throw std::runtime_error("CpuMailbox: message larger than slot");
  const int es = elem_size(dtype);
  if (nbytes % es) throw std::runtime_error("CpuMailbox: size not a multiple of the element size");
  const uint32_t epoch = epoch_ + 1;
  const int half = epoch & 1;
  // 1. push: store my input into slot[rank] of every rank's mailbox.
  for (int j = 0; j < world_; ++j) {
    const int dst = (rank_ + j) % world_;
    std::memcpy(slot(dst, half, rank_), in, nbytes);
  }
  // 2. flag: publish epoch to every rank (release orders the copies before it).
  for (int dst = 0; dst < world_; ++dst) flag(dst, rank_)->store(epoch, std::memory_order_release);
  // 3. wait for every source (bounded).
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms_);
  for (int src = 0; src < world_; ++src) {
    int spins = 0;
    while ((int32_t)(flag(rank_, src)->load(std::memory_order_acquire) - epoch) < 0) {
      if (++spins > 64) {
        std::this_thread::yield();
        if (std::chrono::steady_clock::now() > deadline) {
          err_ = 3;
          err_peer_ = src;
          return err_;
        }
      }
    }
  }
  // 4. reduce in rank order, fp32 accumulate, one rounding.
  const size_t n = nbytes / es;
  if (dtype == 0) {
    float* o = static_cast<float*>(out);
    for (size_t i = 0; i < n; ++i) {
      float acc = 0.f;
      for (int src = 0; src < world_; ++src) acc += reinterpret_cast<const float*>(slot(rank_, half, src))[i];
      o[i] = acc;
    }
  } else {
    uint16_t* o = static_cast<uint16_t*>(out);
    for (size_t i = 0; i < n; ++i) {
      float acc = 0.f;
      for (int src = 0; src < world_; ++src) {
        const uint16_t h = reinterpret_cast<const uint16_t*>(slot(rank_, half, src))[i];
        acc += dtype == 2 ? bf16_to_f32(h) : f16_to_f32(h);
      }
      o[i] = dtype == 2 ? f32_to_bf16(acc) : f32_to_f16(acc);
    }
  }
  epoch_ = epoch;
  return 0;
}

void CpuMailbox::set_epoch(uint32_t e) {
  epoch_ = e;
  for (int src = 0; src < world_; ++src) flag(rank_, src)->store(e, std::memory_order_release);
}

void CpuMailbox::reset() {
  epoch_ = 0;
  err_ = 0;
  err_peer_ = -1;
  for (int src = 0; src < world_; ++src) flag(rank_, src)->store(0, std::memory_order_release);
}

}  // namespace mbx
