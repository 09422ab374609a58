// Shared helpers for the lightserve_b200 CUDA kernels (sm_100a only).
//
// Every kernel in this library is launched through an `extern "C"` entry point
// declared in include/lightserve_b200.h. Entry points never allocate device
// memory and never synchronise the stream, so every one of them can be
// recorded into a CUDA graph. Errors are reported as an int status plus a
// thread-local message readable through lsb_last_error().
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include <atomic>
#include <mutex>
#include <utility>

#include "../../include/lightserve_b200.h"

namespace lsb {

// ---------------------------------------------------------------- errors ---

void set_error(const char* fmt, ...);

#define LSB_CHECK_ARG(cond, ...)                                   \
  do {                                                             \
    if (!(cond)) {                                                 \
      ::lsb::set_error(__VA_ARGS__);                               \
      return LSB_ERR_INVALID;                                      \
    }                                                              \
  } while (0)

#define LSB_CHECK_LAUNCH(what)                                                    \
  do {                                                                            \
    cudaError_t _e = cudaGetLastError();                                          \
    if (_e != cudaSuccess) {                                                      \
      ::lsb::set_error("%s: CUDA launch failed: %s", what, cudaGetErrorString(_e)); \
      return LSB_ERR_CUDA;                                                        \
    }                                                                             \
  } while (0)

#define LSB_CUDA_OK(call, what)                                                   \
  do {                                                                            \
    cudaError_t _e = (call);                                                      \
    if (_e != cudaSuccess) {                                                      \
      ::lsb::set_error("%s: %s", what, cudaGetErrorString(_e));                   \
      return LSB_ERR_CUDA;                                                        \
    }                                                                             \
  } while (0)

// Per-device state is kept for device ordinals [0, kMaxDevices).
constexpr int kMaxDevices = 64;

// The current device, or -1 (with the error message set) when it cannot be
// read or lies outside [0, kMaxDevices).
inline int current_device(const char* who) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_error("%s: no usable current device (%s, ordinal %d)", who,
              e == cudaSuccess ? "ordinal out of range" : cudaGetErrorString(e), dev);
    return -1;
  }
  return dev;
}

// Runs a set-up step once per device, thread-safely; a failed step is retried
// on the next call.
class PerDeviceOnce {
 public:
  template <class F>
  cudaError_t run(int dev, F&& fn) {
    const uint64_t bit = 1ull << dev;
    if (done_.load(std::memory_order_acquire) & bit) return cudaSuccess;
    std::lock_guard<std::mutex> lock(mu_);
    if (done_.load(std::memory_order_relaxed) & bit) return cudaSuccess;
    const cudaError_t e = fn();
    if (e == cudaSuccess) done_.fetch_or(bit, std::memory_order_release);
    return e;
  }

 private:
  std::atomic<uint64_t> done_{0};
  std::mutex mu_;
};

// A kernel's dynamic shared-memory limit per device: cudaFuncSetAttribute is
// called only when a launch needs more than the limit already set on the
// current device. One static instance per kernel, owned by its launcher.
class SmemLimit {
 public:
  template <class K>
  int ensure(K kern, size_t bytes, const char* what) {
    const int dev = current_device(what);
    if (dev < 0) return LSB_ERR_CUDA;
    if ((size_t)set_[dev].load(std::memory_order_acquire) >= bytes) return LSB_OK;
    std::lock_guard<std::mutex> lock(mu_);
    if ((size_t)set_[dev].load(std::memory_order_relaxed) >= bytes) return LSB_OK;
    LSB_CUDA_OK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes),
                what);
    set_[dev].store((int)bytes, std::memory_order_release);
    return LSB_OK;
  }

 private:
  std::atomic<int> set_[kMaxDevices] = {};
  std::mutex mu_;
};

inline int num_sms() {
  static int cached[kMaxDevices] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

// ----------------------------------------------------------- dtype traits ---

template <typename T> struct Dt;
template <> struct Dt<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <> struct Dt<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};
template <> struct Dt<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};

template <typename T> __device__ __forceinline__ float to_f(T x) { return Dt<T>::to_f(x); }
template <typename T> __device__ __forceinline__ T from_f(float x) { return Dt<T>::from_f(x); }

inline int dtype_size(int dtype) {
  switch (dtype) {
    case LSB_DTYPE_F32: return 4;
    case LSB_DTYPE_BF16: return 2;
    case LSB_DTYPE_F16: return 2;
    default: return 0;
  }
}

// Dispatch a templated body over the three element types.
#define LSB_DISPATCH_DTYPE(dtype, T, ...)                 \
  [&]() -> int {                                          \
    switch (dtype) {                                      \
      case LSB_DTYPE_F32: { using T = float; return __VA_ARGS__(); }          \
      case LSB_DTYPE_BF16: { using T = __nv_bfloat16; return __VA_ARGS__(); } \
      case LSB_DTYPE_F16: { using T = __half; return __VA_ARGS__(); }         \
      default: ::lsb::set_error("unsupported dtype code %d", (int)dtype); return LSB_ERR_UNSUPPORTED; \
    }                                                     \
  }()

// 16-byte vector of T.
template <typename T>
struct alignas(16) Vec16 {
  static constexpr int N = 16 / sizeof(T);
  T v[N];
};

template <typename T>
__device__ __forceinline__ Vec16<T> ld_vec16(const T* p) {
  Vec16<T> r;
  *reinterpret_cast<uint4*>(&r) = *reinterpret_cast<const uint4*>(p);
  return r;
}

template <typename T>
__device__ __forceinline__ Vec16<T> ld_vec16_stream(const T* p) {
  // Streaming load: data read once, do not keep in L1.
  Vec16<T> r;
  *reinterpret_cast<uint4*>(&r) = __ldcs(reinterpret_cast<const uint4*>(p));
  return r;
}

template <typename T>
__device__ __forceinline__ void st_vec16(T* p, const Vec16<T>& v) {
  *reinterpret_cast<uint4*>(p) = *reinterpret_cast<const uint4*>(&v);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Lets the next kernel of the stream, when it was launched with programmatic
// stream serialisation, start before this one finishes (it still waits for
// this kernel's completion before reading its results). No effect otherwise.
__device__ __forceinline__ void allow_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Waits until the kernels this one depends on (the previous kernel of the
// stream, when this one was launched with programmatic stream serialisation)
// have completed and their writes are visible. Returns at once otherwise.
// Every kernel launched through launch_kernel() executes it before it reads
// its inputs or writes its outputs.
__device__ __forceinline__ void wait_prerequisites() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Process-wide switch (lsb_set_programmatic_launch, default on): kernels
// launched through launch_kernel() may start while the previous kernel of
// the stream finishes, hiding the launch gap between consecutive kernels.
bool programmatic_launch();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                 cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = programmatic_launch() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Workspace regions are padded to 256 bytes.
inline int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

}  // namespace lsb
