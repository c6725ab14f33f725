// Elementwise dtype conversion (f32 / bf16 / f16 in any direction), HBM-bound:
// 8 elements per thread-iteration, 16-byte loads and stores when both sides are
// aligned. Used for the f16 copy of W_down in the SwiGLU f16-activation mode.
#include "common.cuh"

namespace axon {
namespace {

template <typename S, typename D>
__global__ void __launch_bounds__(256) cast_vec(const S* __restrict__ src, D* __restrict__ dst, int64_t groups) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < groups;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float v[8];
    if constexpr (sizeof(S) == 4) {
      const float4 a = __ldcs(reinterpret_cast<const float4*>(src + i * 8));
      const float4 b = __ldcs(reinterpret_cast<const float4*>(src + i * 8) + 1);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
      const Vec<S> p = ld_vec_stream(src + i * 8);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = to_f(p.e[e]);
    }
    if constexpr (sizeof(D) == 4) {
      __stcs(reinterpret_cast<float4*>(dst + i * 8), make_float4(v[0], v[1], v[2], v[3]));
      __stcs(reinterpret_cast<float4*>(dst + i * 8) + 1, make_float4(v[4], v[5], v[6], v[7]));
    } else {
      Vec<D> q;
#pragma unroll
      for (int e = 0; e < 8; ++e) q.e[e] = from_f<D>(v[e]);
      st_vec(dst + i * 8, q);
    }
  }
}

template <typename S, typename D>
__global__ void cast_scalar(const S* __restrict__ src, D* __restrict__ dst, int64_t n) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = from_f<D>(to_f(src[i]));
}

template <typename S, typename D>
int launch_cast(const void* src, void* dst, int64_t n, cudaStream_t s) {
  const bool vec = n % 8 == 0 && aligned16(src) && aligned16(dst);
  const int64_t work = vec ? n / 8 : n;
  int64_t grid = (work + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  if (vec)
    launch_k(cast_vec<S, D>, dim3(static_cast<unsigned>(grid)), dim3(256), 0, s, static_cast<const S*>(src),
             static_cast<D*>(dst), work);
  else
    launch_k(cast_scalar<S, D>, dim3(static_cast<unsigned>(grid)), dim3(256), 0, s, static_cast<const S*>(src),
             static_cast<D*>(dst), n);
  return launch_status("axon_cast");
}

template <typename S>
int cast_to(int32_t dst_dtype, const void* src, void* dst, int64_t n, cudaStream_t s) {
  switch (dst_dtype) {
    case AXON_F32: return launch_cast<S, float>(src, dst, n, s);
    case AXON_BF16: return launch_cast<S, __nv_bfloat16>(src, dst, n, s);
    case AXON_F16: return launch_cast<S, __half>(src, dst, n, s);
    default: return fail(AXON_E_UNSUPPORTED, "axon_cast: unsupported destination dtype %d", dst_dtype);
  }
}

}  // namespace

int cast_impl(const void* src, void* dst, int64_t n, int32_t src_dtype, int32_t dst_dtype, cudaStream_t s) {
  if (n < 0) return fail(AXON_E_SHAPE, "axon_cast: negative size");
  if (n == 0) return AXON_OK;
  if (!src || !dst) return fail(AXON_E_ARG, "axon_cast: NULL pointer");
  switch (src_dtype) {
    case AXON_F32: return cast_to<float>(dst_dtype, src, dst, n, s);
    case AXON_BF16: return cast_to<__nv_bfloat16>(dst_dtype, src, dst, n, s);
    case AXON_F16: return cast_to<__half>(dst_dtype, src, dst, n, s);
    default: return fail(AXON_E_UNSUPPORTED, "axon_cast: unsupported source dtype %d", src_dtype);
  }
}

}  // namespace axon

extern "C" int axon_cast(const void* src, void* dst, int64_t n, int32_t src_dtype, int32_t dst_dtype, void* stream) {
  return axon::cast_impl(src, dst, n, src_dtype, dst_dtype, axon::as_stream(stream));
}
