// Allocation-free split-KV decode attention (declaration and caller rules in
// decode_noalloc.h). It runs the existing decode kernels with their scratch in
// a file-scope device array; no existing code path changes.
#include <cuda_runtime.h>

#include <cstdio>
#include <exception>
#include <mutex>

#include "../kernels.h"
#include "decode_noalloc.h"

namespace {

constexpr int kHeadDim = 128;
constexpr size_t kMaxRows = MBX_NOALLOC_MAX_PARTIAL_ROWS;

// The scratch: one copy per GPU that loads this library, alive until exit.
static __device__ __align__(256) float g_part_o[kMaxRows * kHeadDim];  // 8 MiB
static __device__ __align__(256) float g_part_lse[kMaxRows];           // 64 KiB

constexpr int kMaxDevices = 128;
struct DeviceScratch {
  float* o = nullptr;
  float* lse = nullptr;
  bool ready = false;
};
DeviceScratch g_scratch[kMaxDevices];
std::mutex g_mu;
thread_local char g_last_error[512] = "";

int fail(int code, const char* msg) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s", msg);
  return code;
}

// Host code only holds a stand-in for the array's name: its device address is
// looked up here, once per device, with that device current.
int scratch_for_current_device(DeviceScratch** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(3, cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(3, "mbx_decode_attention_noalloc: device index out of range");
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceScratch& s = g_scratch[dev];
  if (!s.ready) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_part_o);
    if (e != cudaSuccess) return fail(3, cudaGetErrorString(e));
    s.o = static_cast<float*>(p);
    e = cudaGetSymbolAddress(&p, g_part_lse);
    if (e != cudaSuccess) return fail(3, cudaGetErrorString(e));
    s.lse = static_cast<float*>(p);
    s.ready = true;
  }
  *out = &s;
  return 0;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int mbx_decode_attention_noalloc(
    const void* q, const void* k_cache, const void* v_cache, void* out, const int32_t* kv_len,
    const int32_t* block_table, int max_blocks, int batch, int q_heads, int kv_heads, int splits, float scale,
    void* stream) {
  g_last_error[0] = '\0';
  if (!q || !k_cache || !v_cache || !out || !kv_len || !block_table)
    return fail(1, "mbx_decode_attention_noalloc: null pointer argument");
  if (batch < 0 || q_heads <= 0 || kv_heads <= 0 || max_blocks <= 0 || splits < 1)
    return fail(1, "mbx_decode_attention_noalloc: bad sizes (need batch >= 0, heads > 0, splits >= 1)");
  const size_t rows = (size_t)batch * (size_t)q_heads * (size_t)splits;
  if (splits > 1 && rows > kMaxRows) {
    char msg[256];
    std::snprintf(msg, sizeof(msg),
                  "mbx_decode_attention_noalloc: batch*q_heads*splits = %zu exceeds the fixed scratch of %zu rows; "
                  "lower splits or call the allocating entry point",
                  rows, kMaxRows);
    return fail(2, msg);
  }
  if (batch == 0) return 0;
  // one split writes the output directly and needs no scratch
  DeviceScratch* s = nullptr;
  if (splits > 1) {
    if (int rc = scratch_for_current_device(&s)) return rc;
  }
  try {
    mbx::decode_attention_launch(q, k_cache, v_cache, out, kv_len, block_table, max_blocks, batch, q_heads,
                                 kv_heads, splits, s ? s->o : nullptr, s ? s->lse : nullptr, scale,
                                 static_cast<cudaStream_t>(stream));
  } catch (const std::exception& ex) {
    return fail(4, ex.what());
  }
  return 0;
}

extern "C" __attribute__((visibility("default"))) size_t mbx_decode_attention_noalloc_max_rows(void) {
  return kMaxRows;
}

extern "C" __attribute__((visibility("default"))) const char* mbx_noalloc_last_error(void) {
  return g_last_error;
}
