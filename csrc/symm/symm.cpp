// Symmetric memory over NVLink 5 / NVSwitch.
//
// The reference gets a peer-visible 64 MB mailbox by patching the GeForce
// kernel driver (BAR1 P2P + a second static BAR1 window,
// driver/p2p-mailbox-595.91.07.patch:673-970) and then opening the peer's
// allocation with cudaIpcOpenMemHandle (sglang/mailbox_ar_ext.cu:169-186),
// retrying up to 16 allocations until one "lands in the window"
// (sglang/mailbox_all_reduce.py:91-146). B200 peers are natively reachable
// over NVLink, so this layer instead:
//
//   * allocates each rank's buffer with cuMemCreate (VMM, POSIX-FD shareable),
//   * exports the handle as a file descriptor, which the Python side passes
//     to the peers over a Unix socket (SCM_RIGHTS, csrc/cpu/fdx.cpp),
//   * imports every peer's handle and maps it at a fixed virtual address once
//     (so CUDA-graph replays can record raw pointers),
//   * optionally creates an NVLS multicast object (cuMulticastCreate / AddDevice
//     / BindMem) and maps it, giving multimem.* access to all ranks' buffers,
//   * keeps the reference's legacy CUDA IPC path (cudaIpcGetMemHandle /
//     cudaIpcOpenMemHandle) as a unicast fallback.
//
// Driver entry points are resolved at run time with cudaGetDriverEntryPoint,
// so the module imports (and its host code is testable) without libcuda.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <unistd.h>

#include <cstring>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "symm.h"

namespace mbx {
namespace {

struct DriverApi {
  PFN_cuMemCreate_v10020 memCreate = nullptr;
  PFN_cuMemRelease_v10020 memRelease = nullptr;
  PFN_cuMemAddressReserve_v10020 addrReserve = nullptr;
  PFN_cuMemAddressFree_v10020 addrFree = nullptr;
  PFN_cuMemMap_v10020 memMap = nullptr;
  PFN_cuMemUnmap_v10020 memUnmap = nullptr;
  PFN_cuMemSetAccess_v10020 setAccess = nullptr;
  PFN_cuMemGetAllocationGranularity_v10020 granularity = nullptr;
  PFN_cuMemExportToShareableHandle_v10020 exportHandle = nullptr;
  PFN_cuMemImportFromShareableHandle_v10020 importHandle = nullptr;
  PFN_cuDeviceGetAttribute_v2000 devAttr = nullptr;
  PFN_cuDeviceGet_v2000 devGet = nullptr;
  PFN_cuGetErrorString_v6000 errString = nullptr;
  PFN_cuMulticastCreate_v12010 mcCreate = nullptr;
  PFN_cuMulticastAddDevice_v12010 mcAddDevice = nullptr;
  PFN_cuMulticastBindMem_v12010 mcBindMem = nullptr;
  PFN_cuMulticastUnbind_v12010 mcUnbind = nullptr;
  PFN_cuMulticastGetGranularity_v12010 mcGranularity = nullptr;
  bool loaded = false;
};

DriverApi& api() {
  static DriverApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    auto get = [](const char* name, void** fn) {
      cudaDriverEntryPointQueryResult q;
      cudaError_t e = cudaGetDriverEntryPoint(name, fn, cudaEnableDefault, &q);
      if (e != cudaSuccess || q != cudaDriverEntryPointSuccess) *fn = nullptr;
    };
    get("cuMemCreate", (void**)&a.memCreate);
    get("cuMemRelease", (void**)&a.memRelease);
    get("cuMemAddressReserve", (void**)&a.addrReserve);
    get("cuMemAddressFree", (void**)&a.addrFree);
    get("cuMemMap", (void**)&a.memMap);
    get("cuMemUnmap", (void**)&a.memUnmap);
    get("cuMemSetAccess", (void**)&a.setAccess);
    get("cuMemGetAllocationGranularity", (void**)&a.granularity);
    get("cuMemExportToShareableHandle", (void**)&a.exportHandle);
    get("cuMemImportFromShareableHandle", (void**)&a.importHandle);
    get("cuDeviceGetAttribute", (void**)&a.devAttr);
    get("cuDeviceGet", (void**)&a.devGet);
    get("cuGetErrorString", (void**)&a.errString);
    get("cuMulticastCreate", (void**)&a.mcCreate);
    get("cuMulticastAddDevice", (void**)&a.mcAddDevice);
    get("cuMulticastBindMem", (void**)&a.mcBindMem);
    get("cuMulticastUnbind", (void**)&a.mcUnbind);
    get("cuMulticastGetGranularity", (void**)&a.mcGranularity);
    a.loaded = a.memCreate && a.memMap && a.exportHandle && a.importHandle;
  });
  if (!a.loaded) throw std::runtime_error("symm: CUDA driver VMM entry points unavailable (no GPU driver?)");
  return a;
}

void check(CUresult r, const char* what) {
  if (r != CUDA_SUCCESS) {
    const char* s = nullptr;
    if (api().errString) api().errString(r, &s);
    throw std::runtime_error(std::string("symm: ") + what + " failed: " + (s ? s : "?") + " (" +
                             std::to_string((int)r) + ")");
  }
}

struct Mem {
  CUmemGenericAllocationHandle h = 0;
  CUdeviceptr va = 0;
  size_t size = 0;
  bool multicast = false;
  int device = 0;
};

std::mutex g_mu;
std::map<int64_t, Mem> g_mem;
int64_t g_next = 1;

CUmemAllocationProp alloc_prop(int device) {
  CUmemAllocationProp p;
  std::memset(&p, 0, sizeof(p));
  p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  p.location.id = device;
  p.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  return p;
}

CUdeviceptr map_handle(CUmemGenericAllocationHandle h, size_t size, size_t align, int device) {
  auto& a = api();
  CUdeviceptr va = 0;
  check(a.addrReserve(&va, size, align, 0, 0), "cuMemAddressReserve");
  CUresult r = a.memMap(va, size, 0, h, 0);
  if (r != CUDA_SUCCESS) {
    a.addrFree(va, size);
    check(r, "cuMemMap");
  }
  CUmemAccessDesc acc;
  std::memset(&acc, 0, sizeof(acc));
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = device;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  r = a.setAccess(va, size, &acc, 1);
  if (r != CUDA_SUCCESS) {
    a.memUnmap(va, size);
    a.addrFree(va, size);
    check(r, "cuMemSetAccess");
  }
  return va;
}

int64_t register_mem(const Mem& m) {
  std::lock_guard<std::mutex> g(g_mu);
  int64_t id = g_next++;
  g_mem[id] = m;
  return id;
}

Mem& lookup(int64_t id) {
  std::lock_guard<std::mutex> g(g_mu);
  auto it = g_mem.find(id);
  if (it == g_mem.end()) throw std::runtime_error("symm: unknown handle id " + std::to_string(id));
  return it->second;
}

}  // namespace

size_t symm_granularity(int device, bool multicast, int ndev) {
  auto& a = api();
  size_t g = 0;
  CUmemAllocationProp p = alloc_prop(device);
  check(a.granularity(&g, &p, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED), "cuMemGetAllocationGranularity");
  if (multicast && a.mcGranularity) {
    CUmulticastObjectProp mp;
    std::memset(&mp, 0, sizeof(mp));
    mp.numDevices = ndev;
    mp.size = g;
    mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    size_t mg = 0;
    check(a.mcGranularity(&mg, &mp, CU_MULTICAST_GRANULARITY_RECOMMENDED), "cuMulticastGetGranularity");
    if (mg > g) g = mg;
  }
  return g;
}

SymmAlloc symm_create(int device, size_t size) {
  auto& a = api();
  cudaSetDevice(device);
  Mem m;
  m.size = size;
  m.device = device;
  CUmemAllocationProp p = alloc_prop(device);
  check(a.memCreate(&m.h, size, &p, 0), "cuMemCreate");
  try {
    m.va = map_handle(m.h, size, 0, device);
  } catch (...) {
    a.memRelease(m.h);
    throw;
  }
  int fd = -1;
  CUresult r = a.exportHandle(&fd, m.h, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0);
  if (r != CUDA_SUCCESS) {
    a.memUnmap(m.va, size);
    a.addrFree(m.va, size);
    a.memRelease(m.h);
    check(r, "cuMemExportToShareableHandle");
  }
  // Fresh memory: zero it so every signal word starts at epoch 0 (the
  // reference relies on fresh VRAM being zero for its header words).
  if (cudaMemset((void*)m.va, 0, size) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess)
    throw std::runtime_error("symm: zeroing the new buffer failed");
  SymmAlloc out;
  out.id = register_mem(m);
  out.ptr = (int64_t)m.va;
  out.fd = fd;
  return out;
}

SymmAlloc symm_import(int device, int fd, size_t size) {
  auto& a = api();
  cudaSetDevice(device);
  Mem m;
  m.size = size;
  m.device = device;
  check(a.importHandle(&m.h, (void*)(intptr_t)fd, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
        "cuMemImportFromShareableHandle");
  try {
    m.va = map_handle(m.h, size, 0, device);
  } catch (...) {
    a.memRelease(m.h);
    throw;
  }
  SymmAlloc out;
  out.id = register_mem(m);
  out.ptr = (int64_t)m.va;
  out.fd = -1;
  return out;
}

void symm_free(int64_t id) {
  Mem m;
  {
    std::lock_guard<std::mutex> g(g_mu);
    auto it = g_mem.find(id);
    if (it == g_mem.end()) return;
    m = it->second;
    g_mem.erase(it);
  }
  auto& a = api();
  if (m.va) {
    a.memUnmap(m.va, m.size);
    a.addrFree(m.va, m.size);
  }
  if (m.h) a.memRelease(m.h);
}

bool mc_supported(int device) {
  auto& a = api();
  if (!a.mcCreate || !a.devAttr || !a.devGet) return false;
  CUdevice d;
  if (a.devGet(&d, device) != CUDA_SUCCESS) return false;
  int v = 0;
  if (a.devAttr(&v, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, d) != CUDA_SUCCESS) return false;
  return v != 0;
}

SymmAlloc mc_create(int ndev, size_t size) {
  auto& a = api();
  CUmulticastObjectProp mp;
  std::memset(&mp, 0, sizeof(mp));
  mp.numDevices = ndev;
  mp.size = size;
  mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  Mem m;
  m.size = size;
  m.multicast = true;
  check(a.mcCreate(&m.h, &mp), "cuMulticastCreate");
  int fd = -1;
  CUresult r = a.exportHandle(&fd, m.h, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0);
  if (r != CUDA_SUCCESS) {
    a.memRelease(m.h);
    check(r, "cuMemExportToShareableHandle(multicast)");
  }
  SymmAlloc out;
  out.id = register_mem(m);
  out.ptr = 0;
  out.fd = fd;
  return out;
}

int64_t mc_import(int fd, size_t size) {
  auto& a = api();
  Mem m;
  m.size = size;
  m.multicast = true;
  check(a.importHandle(&m.h, (void*)(intptr_t)fd, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
        "cuMemImportFromShareableHandle(multicast)");
  return register_mem(m);
}

void mc_add_device(int64_t mc_id, int device) {
  auto& a = api();
  CUdevice d;
  check(a.devGet(&d, device), "cuDeviceGet");
  check(a.mcAddDevice(lookup(mc_id).h, d), "cuMulticastAddDevice");
}

void mc_bind(int64_t mc_id, int64_t mem_id, size_t size) {
  auto& a = api();
  check(a.mcBindMem(lookup(mc_id).h, 0, lookup(mem_id).h, 0, size, 0), "cuMulticastBindMem");
}

int64_t mc_map(int64_t mc_id, int device, size_t size) {
  Mem& m = lookup(mc_id);
  m.device = device;
  m.va = map_handle(m.h, size, 0, device);
  return (int64_t)m.va;
}

void mc_unbind(int64_t mc_id, int device, size_t size) {
  auto& a = api();
  if (!a.mcUnbind) return;
  CUdevice d;
  if (a.devGet(&d, device) != CUDA_SUCCESS) return;
  a.mcUnbind(lookup(mc_id).h, d, 0, size);
}

void close_fd(int fd) {
  if (fd >= 0) ::close(fd);
}

// ---- legacy CUDA IPC (same entry points as the reference's ext) ----------
std::string ipc_get_handle(int64_t ptr) {
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, (void*)ptr);
  if (e != cudaSuccess) throw std::runtime_error(std::string("cudaIpcGetMemHandle failed: ") + cudaGetErrorString(e));
  return std::string(reinterpret_cast<const char*>(&h), sizeof(h));
}

int64_t ipc_open(const std::string& handle) {
  if (handle.size() != sizeof(cudaIpcMemHandle_t)) throw std::runtime_error("ipc_open: bad handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) throw std::runtime_error(std::string("cudaIpcOpenMemHandle failed: ") + cudaGetErrorString(e));
  return (int64_t)p;
}

void ipc_close(int64_t ptr) {
  if (ptr) cudaIpcCloseMemHandle((void*)ptr);
}

// ---- host-mapped status words ------------------------------------------
HostMapped host_mapped_alloc(size_t bytes) {
  void* h = nullptr;
  cudaError_t e = cudaHostAlloc(&h, bytes, cudaHostAllocMapped | cudaHostAllocPortable);
  if (e != cudaSuccess) throw std::runtime_error(std::string("cudaHostAlloc failed: ") + cudaGetErrorString(e));
  std::memset(h, 0, bytes);
  void* d = nullptr;
  e = cudaHostGetDevicePointer(&d, h, 0);
  if (e != cudaSuccess) {
    cudaFreeHost(h);
    throw std::runtime_error(std::string("cudaHostGetDevicePointer failed: ") + cudaGetErrorString(e));
  }
  return HostMapped{(int64_t)h, (int64_t)d};
}

void host_mapped_free(int64_t host_ptr) {
  if (host_ptr) cudaFreeHost((void*)host_ptr);
}

}  // namespace mbx
