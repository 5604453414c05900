// Shared device/host helpers for the sm_100a kernels of libdli_sm100.so.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "dli_sm100.h"

namespace dli_sm100 {

// ---------------------------------------------------------------------------
// Host-side status plumbing.
// ---------------------------------------------------------------------------

// Stores `msg` as this thread's last error and returns `status`.
dli_status fail(dli_status status, const std::string& msg);
// Clears the last error and returns DLI_OK.
dli_status ok();
// Maps the last launch error (cudaGetLastError) to a status naming `what`; on
// success adds `launches` kernels to the library's launch counter.
dli_status check_launch(const char* what, int launches = 1);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool is_float_dtype(dli_dtype d) {
  return d == DLI_DTYPE_F32 || d == DLI_DTYPE_BF16 || d == DLI_DTYPE_F16;
}
inline size_t dtype_bytes(dli_dtype d) {
  switch (d) {
    case DLI_DTYPE_F32: return 4;
    case DLI_DTYPE_I64: return 8;
    case DLI_DTYPE_BF16: return 2;
    case DLI_DTYPE_F16: return 2;
    case DLI_DTYPE_I32: return 4;
  }
  return 0;
}
inline bool aligned(const void* p, size_t bytes) {
  return (reinterpret_cast<uintptr_t>(p) % bytes) == 0;
}
inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Number of SMs of the current device (cached per device).
int sm_count();

// Raises a kernel's dynamic shared-memory limit to `bytes` once per device.
dli_status ensure_smem(const void* kernel, int bytes, const char* what);

// Integer tuning knob read once from the environment (DLI_SM100_<name>),
// `fallback` when unset. Knobs change launch shapes only, never the result.
int tuning_knob(const char* name, int fallback);
inline bool pdl_enabled() {
  static const bool on = tuning_knob("PDL", 1) != 0;
  return on;
}

// Dispatches a functor templated on the element type of a float dtype.
template <typename F>
dli_status dispatch_float(dli_dtype dtype, const char* what, F&& f) {
  switch (dtype) {
    case DLI_DTYPE_F32: f(float{}); return DLI_OK;
    case DLI_DTYPE_BF16: f(__nv_bfloat16{}); return DLI_OK;
    case DLI_DTYPE_F16: f(__half{}); return DLI_OK;
    default: break;
  }
  return fail(DLI_ERR_INVALID_ARGUMENT, std::string(what) + " expects a float32/bfloat16/float16 dtype");
}

// ---------------------------------------------------------------------------
// Device error word: kernels with bounded waits or data-dependent bounds set a
// code here instead of trapping; dli_sm100_check_device_error() reads it.
// ---------------------------------------------------------------------------
enum DeviceError : unsigned {
  kDevErrNone = 0,
  kDevErrGemmTimeout = 1,
  kDevErrEmbeddingIndex = 2,
  kDevErrRotaryPosition = 3,
  kDevErrAttentionTimeout = 4,
  kDevErrKvCapacity = 5,
  kDevErrExchangeTimeout = 6,
};
// Device address of the error word of the current device (resolved once per
// device with cudaGetSymbolAddress); kernels receive it as an argument.
unsigned* device_error_word();

__device__ __forceinline__ void set_device_error(unsigned* word, unsigned code) {
  if (word != nullptr) atomicCAS(word, 0u, code);
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch. Every kernel of this library is launched with
// the programmatic-stream-serialization attribute, so it may be scheduled while
// the previous kernel of the stream is still running. Before its first global
// read of data a previous kernel produces and before its first global write, a
// kernel calls pdl_wait() (griddepcontrol.wait: returns once the preceding grid
// has completed and its memory is visible; a no-op without a programmatic
// dependency). Only reads of operands no kernel writes (weights) may precede
// it. pdl_trigger() lets the next kernel's CTAs be scheduled early; correctness
// never depends on it because the next kernel's pdl_wait() still waits for this
// grid to finish.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Entry of a kernel whose every global access may depend on the previous kernel.
#define DLI_PDL_ENTRY()          \
  do {                           \
    ::dli_sm100::pdl_wait();     \
    ::dli_sm100::pdl_trigger();  \
  } while (0)

// Launches `kernel` on `stream` with programmatic dependent launch enabled and,
// when cluster_y > 1, thread-block clusters of (1, cluster_y, 1) CTAs.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                               cudaStream_t stream, unsigned cluster_y, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_y > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 1;
    attr[n].val.clusterDim.y = cluster_y;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
  return launch_pdl_cluster(kernel, grid, block, smem, stream, 1u, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------
// Element conversions.
// ---------------------------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// Rounds an fp32 value through T (identity for float).
template <typename T> __device__ __forceinline__ float round_through(float v) {
  return to_f32<T>(from_f32<T>(v));
}

// 16-byte vector of T.
template <typename T> struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
  union {
    uint4 raw;
    T e[N];
  };
};

template <typename T>
__device__ __forceinline__ Vec16<T> load16(const T* p) {
  Vec16<T> v;
  v.raw = *reinterpret_cast<const uint4*>(p);
  return v;
}
template <typename T>
__device__ __forceinline__ void store16(T* p, const Vec16<T>& v) {
  *reinterpret_cast<uint4*>(p) = v.raw;
}

// ---------------------------------------------------------------------------
// Reductions.
// ---------------------------------------------------------------------------
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

// Block-wide sum; `scratch` holds >= 32 floats. All threads get the result.
__device__ __forceinline__ float block_sum(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float r = (lane < nwarps) ? scratch[lane] : 0.f;
  r = warp_sum(r);
  return r;
}
__device__ __forceinline__ float block_max(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float r = (lane < nwarps) ? scratch[lane] : -INFINITY;
  r = warp_max(r);
  return r;
}

}  // namespace dli_sm100
