// Host API of the symmetric-memory layer (see symm.cpp).
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>

namespace mbx {

struct SymmAlloc {
  int64_t id = 0;   // registry id (for free / bind)
  int64_t ptr = 0;  // mapped device address (0 for an unmapped multicast object)
  int fd = -1;      // exported POSIX FD (owner side), -1 on import
};

struct HostMapped {
  int64_t host = 0;
  int64_t dev = 0;
};

size_t symm_granularity(int device, bool multicast, int ndev);
SymmAlloc symm_create(int device, size_t size);
SymmAlloc symm_import(int device, int fd, size_t size);
void symm_free(int64_t id);

bool mc_supported(int device);
SymmAlloc mc_create(int ndev, size_t size);
int64_t mc_import(int fd, size_t size);
void mc_add_device(int64_t mc_id, int device);
void mc_bind(int64_t mc_id, int64_t mem_id, size_t size);
int64_t mc_map(int64_t mc_id, int device, size_t size);
void mc_unbind(int64_t mc_id, int device, size_t size);
void close_fd(int fd);

std::string ipc_get_handle(int64_t ptr);
int64_t ipc_open(const std::string& handle);
void ipc_close(int64_t ptr);

HostMapped host_mapped_alloc(size_t bytes);
void host_mapped_free(int64_t host_ptr);

}  // namespace mbx
