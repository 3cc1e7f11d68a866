// CPU mailbox allreduce engine (see mailbox_cpu.cpp).
#pragma once
#include <atomic>
#include <cstddef>
#include <cstdint>
#include <string>

namespace mbx {

class CpuMailbox {
 public:
  CpuMailbox(const std::string& path, int rank, int world, size_t slot_bytes, bool create, int64_t timeout_ms);
  ~CpuMailbox();
  // Returns 0, or a sticky error code (3 = timed out waiting for a peer's flag).
  int allreduce(const void* in, void* out, size_t nbytes, int dtype);
  void reset();
  // Test support: put this rank at epoch `e` with every inbound flag at `e`
  // (a consistent state, as if e calls had completed; used to run across the
  // 2^32 wrap). Every rank must call it before the next allreduce.
  void set_epoch(uint32_t e);
  void close();
  uint32_t epoch() const { return epoch_; }
  int error() const { return err_; }
  int error_peer() const { return err_peer_; }
  size_t slot_bytes() const { return slot_bytes_; }

 private:
  std::atomic<uint32_t>* flag(int dst, int src) const;
  char* slot(int dst, int half, int src) const;

  std::string path_;
  int rank_, world_;
  size_t slot_bytes_, size_ = 0;
  int64_t timeout_ms_;
  bool owner_;
  int fd_ = -1;
  char* base_ = nullptr;
  uint32_t epoch_ = 0;
  int err_ = 0;
  int err_peer_ = -1;
};

}  // namespace mbx
