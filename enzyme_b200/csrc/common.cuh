// Shared helpers for the Axon B200 kernel library: status handling, element
// conversion, 16-byte vector access and CTA reductions. sm_100a only.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>
#include <utility>

#include "../../include/axon_b200.h"

namespace axon {

// ---- error reporting --------------------------------------------------------

// Records the message for axon_last_error() (thread-local) and returns `code`.
int fail(int code, const char* fmt, ...);
void clear_error();

#define AXON_CHECK_ARG(cond, ...)                  \
  do {                                             \
    if (!(cond)) return ::axon::fail(AXON_E_ARG, __VA_ARGS__); \
  } while (0)

#define AXON_CHECK_SHAPE(cond, ...)                \
  do {                                             \
    if (!(cond)) return ::axon::fail(AXON_E_SHAPE, __VA_ARGS__); \
  } while (0)

// Turns the launch status into an AXON code (does not synchronise).
int launch_status(const char* what);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int dtype_size(int32_t dt) { return dt == AXON_F32 ? 4 : 2; }

inline bool valid_dtype(int32_t dt) { return dt == AXON_F32 || dt == AXON_BF16 || dt == AXON_F16; }

// Number of SMs of the current device (cached per device).
int sm_count();

// Elementwise dtype conversion of n elements (the body of axon_cast).
int cast_impl(const void* src, void* dst, int64_t n, int32_t src_dtype, int32_t dst_dtype, cudaStream_t s);

// Resolves a tune pointer (NULL = all defaults).
inline axon_tune_t tune_or_default(const axon_tune_t* t) {
  axon_tune_t d{};
  return t ? *t : d;
}

// ---- programmatic dependent launch --------------------------------------------
//
// Memory-bound kernels are launched with programmatic stream serialization:
// the next kernel in the stream may be scheduled while this one drains, and
// every such kernel starts with pdl_wait() (griddepcontrol.wait), which
// blocks until the previous grid has completed and its writes are visible.
// Data dependencies are therefore exactly those of a plain launch; only the
// launch latency between back-to-back kernels is hidden. AXON_B200_PDL=0 in
// the environment turns the attribute off.

bool pdl_enabled();

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// ---- element conversion -------------------------------------------------------

template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// Loads element i of a runtime-typed array as float (used for small side
// vectors such as per-row scalars and norm weights).
__device__ __forceinline__ float load_any(const void* p, int64_t i, int32_t dt) {
  if (dt == AXON_F32) return static_cast<const float*>(p)[i];
  if (dt == AXON_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}

// ---- 16-byte vectors ----------------------------------------------------------

// A 16-byte packet of E = 16 / sizeof(T) elements.
template <typename T>
struct Vec {
  static constexpr int E = 16 / sizeof(T);
  union {
    uint4 u;
    T e[E];
  };
};

template <typename T>
__device__ __forceinline__ Vec<T> ld_vec(const T* p) {
  Vec<T> v;
  v.u = *reinterpret_cast<const uint4*>(p);
  return v;
}

// Streaming load: the data is used once, keep it out of L1.
template <typename T>
__device__ __forceinline__ Vec<T> ld_vec_stream(const T* p) {
  Vec<T> v;
  v.u = __ldcs(reinterpret_cast<const uint4*>(p));
  return v;
}

template <typename T>
__device__ __forceinline__ void st_vec(T* p, const Vec<T>& v) {
  *reinterpret_cast<uint4*>(p) = v.u;
}

template <typename T>
__device__ __forceinline__ void st_vec_stream(T* p, const Vec<T>& v) {
  __stcs(reinterpret_cast<uint4*>(p), v.u);
}

// ---- reductions -----------------------------------------------------------------

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

}  // namespace axon
