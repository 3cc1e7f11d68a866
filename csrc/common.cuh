// Shared device helpers for every sm_100a kernel in this package.
//
// Memory-ordering primitives used by the cross-GPU protocols: system-scope
// acquire loads / release stores on flags that live in symmetric (peer-mapped)
// memory, a %globaltimer based clock for bounded waits, and 16-byte vector
// helpers for bf16/fp16/fp32 element packs.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <atomic>
#include <cstdlib>
#include <utility>
#include <mutex>
#include <stdexcept>
#include <string>

#define MBX_DEVICE __device__ __forceinline__

#define MBX_CUDA_CHECK(expr)                                                    \
  do {                                                                          \
    cudaError_t _e = (expr);                                                    \
    if (_e != cudaSuccess) {                                                    \
      throw std::runtime_error(std::string(#expr " failed: ") +                 \
                               cudaGetErrorString(_e) + " at " + __FILE__ +     \
                               ":" + std::to_string(__LINE__));                 \
    }                                                                           \
  } while (0)

namespace mbx {

// ---------------------------------------------------------------------------
// Programmatic dependent launch. A kernel launched with `launch_k` may start
// while the kernel before it on the stream is still finishing (its launch and
// its own set-up overlap the other's tail). Every kernel launched that way
// calls pdl_wait() before its first global-memory access that can depend on
// earlier work: the wait returns once the preceding grids have completed and
// their memory is visible (at once when the kernel was launched normally).
// MBX_PDL=0 turns the attribute off (plain serialised launches).
// ---------------------------------------------------------------------------
MBX_DEVICE void pdl_wait() {
#if defined(__CUDA_ARCH__)
  asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
}

inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("MBX_PDL");
    return !(v != nullptr && v[0] == '0');
  }();
  return on;
}

template <typename... Params, typename... Args>
inline void launch_k(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                     Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  MBX_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

// Raises one kernel's dynamic shared-memory limit on every device it runs on.
// The attribute belongs to a device, so a process that launches on several
// GPUs must set it on each of them: one record per launch site (a function-
// local static), bit d set once device d has it. The lock orders host threads
// that reach the same site at once; after the first launch on a device the
// check is one atomic load.
struct SmemLimit {
  std::atomic<uint64_t> done{0};
  std::mutex mu;
  void ensure(const void* kernel, int bytes) {
    int dev = 0;
    MBX_CUDA_CHECK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) throw std::runtime_error("device index out of range for the kernel attribute record");
    const uint64_t bit = 1ull << dev;
    if (done.load(std::memory_order_acquire) & bit) return;
    std::lock_guard<std::mutex> g(mu);
    if (done.load(std::memory_order_relaxed) & bit) return;
    MBX_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done.fetch_or(bit, std::memory_order_release);
  }
};

// dtype ids shared with Python (same numbering as the reference's dtype_id:
// 0 = fp32, 1 = fp16, 2 = bf16).
enum DType : int { kF32 = 0, kF16 = 1, kBF16 = 2 };

// ---------------------------------------------------------------------------
// Timers and flag access with explicit scopes.
// ---------------------------------------------------------------------------
MBX_DEVICE uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

MBX_DEVICE uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

MBX_DEVICE uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

MBX_DEVICE void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

MBX_DEVICE void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

MBX_DEVICE void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

MBX_DEVICE void nanosleep_ns(uint32_t ns) { asm volatile("nanosleep.u32 %0;" ::"r"(ns)); }

// Wrap-safe "a has reached b" for monotone 32-bit epochs.
MBX_DEVICE bool epoch_reached(uint32_t a, uint32_t b) { return (int32_t)(a - b) >= 0; }

// Bounded wait for *flag to reach `want` (monotone epoch compare). Returns
// false if `timeout_ns` elapsed first. Never traps; the caller records the
// error and returns so the context stays usable.
MBX_DEVICE bool wait_flag_geq(const uint32_t* flag, uint32_t want, uint64_t timeout_ns) {
  if (epoch_reached(ld_acquire_sys(flag), want)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    nanosleep_ns(32);
    if (epoch_reached(ld_acquire_sys(flag), want)) return true;
    if (globaltimer_ns() - t0 > timeout_ns) return false;
  }
}

// ---------------------------------------------------------------------------
// 16-byte packs: 8 x bf16 / 8 x fp16 / 4 x fp32, accumulated in fp32.
// ---------------------------------------------------------------------------
template <typename T> struct Pack;
template <> struct Pack<float> {
  static constexpr int N = 4;
};
template <> struct Pack<__half> {
  static constexpr int N = 8;
};
template <> struct Pack<__nv_bfloat16> {
  static constexpr int N = 8;
};

template <typename T>
MBX_DEVICE void unpack_add(const uint4& v, float* acc);

template <>
MBX_DEVICE void unpack_add<float>(const uint4& v, float* acc) {
  acc[0] += __uint_as_float(v.x);
  acc[1] += __uint_as_float(v.y);
  acc[2] += __uint_as_float(v.z);
  acc[3] += __uint_as_float(v.w);
}

template <>
MBX_DEVICE void unpack_add<__nv_bfloat16>(const uint4& v, float* acc) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
    float2 f = __bfloat1622float2(h);
    acc[2 * i] += f.x;
    acc[2 * i + 1] += f.y;
  }
}

template <>
MBX_DEVICE void unpack_add<__half>(const uint4& v, float* acc) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
    float2 f = __half22float2(h);
    acc[2 * i] += f.x;
    acc[2 * i + 1] += f.y;
  }
}

template <typename T>
MBX_DEVICE uint4 pack_from(const float* acc);

template <>
MBX_DEVICE uint4 pack_from<float>(const float* acc) {
  return make_uint4(__float_as_uint(acc[0]), __float_as_uint(acc[1]), __float_as_uint(acc[2]),
                    __float_as_uint(acc[3]));
}

template <>
MBX_DEVICE uint4 pack_from<__nv_bfloat16>(const float* acc) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <>
MBX_DEVICE uint4 pack_from<__half>(const float* acc) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = __floats2half2_rn(acc[2 * i], acc[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

MBX_DEVICE uint4 ld_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// Peer-memory load that bypasses L1 (data written by another GPU must not be
// served from a stale L1 line).
MBX_DEVICE uint4 ld_v4_volatile(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

MBX_DEVICE void st_v4(void* p, const uint4& v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

MBX_DEVICE float bf16_to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

MBX_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace mbx
