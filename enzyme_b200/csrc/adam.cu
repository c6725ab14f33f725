// Fused L2-regularised Adam (Axon kernels/fused_adam/refs.py:38-46):
//   g' = g + wd*p;  m' = b1*m + (1-b1)*g';  v' = b2*v + (1-b2)*g'^2;
//   p' = p - m' / (sqrt(v')*inv_bc2_sqrt + eps) * step_size
// in fp32 with IEEE division and square root, in the reference's operation
// order. A grid-stride loop over 8-element groups: each group is one or two
// 16-byte packets per tensor (fp32 state: 2, bf16 state: 1), read once with
// evict-first hints and written once -- 26 bytes per parameter for fp32 state
// with bf16 gradients, HBM-bound.
#include "common.cuh"

namespace axon {
namespace {

constexpr int G = 8;  // elements per thread-iteration

struct AdamArgs {
  const void* p;
  const void* g;
  const void* m;
  const void* v;
  void* po;
  void* mo;
  void* vo;
  const void* ss_rows;
  const void* ib_rows;
  const void* wd_rows;
  int32_t row_dtype;
  int64_t cols;
  int64_t n;
  float b1, b2, eps, ss, ib, wd;
};

template <typename T>
__device__ __forceinline__ void ld8(const T* p, float* out) {
  if constexpr (sizeof(T) == 4) {
    float4 a = __ldcs(reinterpret_cast<const float4*>(p));
    float4 b = __ldcs(reinterpret_cast<const float4*>(p) + 1);
    out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
    out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
  } else {
    Vec<T> v = ld_vec_stream(p);
#pragma unroll
    for (int e = 0; e < 8; ++e) out[e] = to_f(v.e[e]);
  }
}

template <typename T>
__device__ __forceinline__ void st8(T* p, const float* in) {
  if constexpr (sizeof(T) == 4) {
    __stcs(reinterpret_cast<float4*>(p), make_float4(in[0], in[1], in[2], in[3]));
    __stcs(reinterpret_cast<float4*>(p) + 1, make_float4(in[4], in[5], in[6], in[7]));
  } else {
    Vec<T> v;
#pragma unroll
    for (int e = 0; e < 8; ++e) v.e[e] = from_f<T>(in[e]);
    st_vec_stream(p, v);
  }
}

__device__ __forceinline__ void adam_one(const AdamArgs& a, float ss, float ib, float wd, float& p, float g,
                                         float& m, float& v) {
  g = g + wd * p;
  m = a.b1 * m + (1.0f - a.b1) * g;
  v = a.b2 * v + (1.0f - a.b2) * (g * g);
  const float denom = sqrtf(v) * ib + a.eps;
  p = p - m / denom * ss;
}

__device__ __forceinline__ void row_scalars(const AdamArgs& a, int64_t idx, float& ss, float& ib, float& wd) {
  const int64_t row = idx / a.cols;
  ss = a.ss_rows ? load_any(a.ss_rows, row, a.row_dtype) : a.ss;
  ib = a.ib_rows ? load_any(a.ib_rows, row, a.row_dtype) : a.ib;
  wd = a.wd_rows ? load_any(a.wd_rows, row, a.row_dtype) : a.wd;
}

// Vector path: n % 8 == 0, cols % 8 == 0 (a group never straddles a row), all
// tensors 16-byte aligned.
template <typename TS, typename TG>
__global__ void __launch_bounds__(256) adam_vec(AdamArgs a) {
  const int64_t groups = a.n / G;
  const bool per_row = a.ss_rows || a.ib_rows || a.wd_rows;
  pdl_wait();
  pdl_trigger();
  for (int64_t gi = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; gi < groups;
       gi += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t off = gi * G;
    float p[G], g[G], m[G], v[G];
    ld8(static_cast<const TS*>(a.p) + off, p);
    ld8(static_cast<const TG*>(a.g) + off, g);
    ld8(static_cast<const TS*>(a.m) + off, m);
    ld8(static_cast<const TS*>(a.v) + off, v);
    float ss = a.ss, ib = a.ib, wd = a.wd;
    if (per_row) row_scalars(a, off, ss, ib, wd);
#pragma unroll
    for (int e = 0; e < G; ++e) adam_one(a, ss, ib, wd, p[e], g[e], m[e], v[e]);
    st8(static_cast<TS*>(a.po) + off, p);
    st8(static_cast<TS*>(a.mo) + off, m);
    st8(static_cast<TS*>(a.vo) + off, v);
  }
}

template <typename TS, typename TG>
__global__ void adam_scalar(AdamArgs a) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < a.n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float p = to_f(static_cast<const TS*>(a.p)[i]);
    float g = to_f(static_cast<const TG*>(a.g)[i]);
    float m = to_f(static_cast<const TS*>(a.m)[i]);
    float v = to_f(static_cast<const TS*>(a.v)[i]);
    float ss, ib, wd;
    row_scalars(a, i, ss, ib, wd);
    adam_one(a, ss, ib, wd, p, g, m, v);
    static_cast<TS*>(a.po)[i] = from_f<TS>(p);
    static_cast<TS*>(a.mo)[i] = from_f<TS>(m);
    static_cast<TS*>(a.vo)[i] = from_f<TS>(v);
  }
}

template <typename TS, typename TG>
int launch_adam(const AdamArgs& a, int threads, cudaStream_t s) {
  const bool vec = a.n % G == 0 && a.cols % G == 0 && aligned16(a.p) && aligned16(a.g) && aligned16(a.m) &&
                   aligned16(a.v) && aligned16(a.po) && aligned16(a.mo) && aligned16(a.vo);
  const int64_t work = vec ? a.n / G : a.n;
  int64_t grid = (work + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * (2048 / threads);
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  if (vec)
    launch_k(adam_vec<TS, TG>, dim3(static_cast<unsigned>(grid)), dim3(threads), 0, s, a);
  else
    adam_scalar<TS, TG><<<static_cast<int>(grid), threads, 0, s>>>(a);
  return launch_status("axon_adam");
}

template <typename TS>
int dispatch_grad(const AdamArgs& a, int32_t gdt, int threads, cudaStream_t s) {
  switch (gdt) {
    case AXON_F32: return launch_adam<TS, float>(a, threads, s);
    case AXON_BF16: return launch_adam<TS, __nv_bfloat16>(a, threads, s);
    case AXON_F16: return launch_adam<TS, __half>(a, threads, s);
    default: return fail(AXON_E_UNSUPPORTED, "axon_adam: unsupported grad dtype %d", gdt);
  }
}

}  // namespace
}  // namespace axon

using namespace axon;

extern "C" int axon_adam(const void* param, const void* grad, const void* exp_avg, const void* exp_avg_sq,
                         void* param_out, void* exp_avg_out, void* exp_avg_sq_out, int64_t rows, int64_t cols,
                         int32_t state_dtype, int32_t grad_dtype, const void* step_size_rows,
                         const void* inv_bc2_sqrt_rows, const void* wd_rows, int32_t row_dtype,
                         const axon_adam_hparams_t* hp, const axon_tune_t* tune, void* stream) {
  axon_tune_t t = tune_or_default(tune);
  if (rows < 0 || cols < 0) return fail(AXON_E_SHAPE, "axon_adam: negative size");
  if (!hp) return fail(AXON_E_ARG, "axon_adam: NULL hyper-parameters");
  if (rows * cols > 0 && (!param || !grad || !exp_avg || !exp_avg_sq || !param_out || !exp_avg_out || !exp_avg_sq_out))
    return fail(AXON_E_ARG, "axon_adam: NULL pointer");
  if ((step_size_rows || inv_bc2_sqrt_rows || wd_rows) && !valid_dtype(row_dtype))
    return fail(AXON_E_UNSUPPORTED, "axon_adam: unsupported per-row scalar dtype %d", row_dtype);
  if (t.variant != 0) return fail(AXON_E_ARG, "axon_adam: unknown variant %d", t.variant);
  // 128-thread CTAs (16 per SM) measured 6.26 TB/s at 1e9 parameters on B200,
  // 256-thread CTAs 5.76 TB/s
  const int threads = t.threads > 0 ? t.threads : 128;
  if (threads > 256 || threads % 32) return fail(AXON_E_ARG, "axon_adam: threads must be 32..256, multiple of 32");
  const int64_t n = rows * cols;
  if (n == 0) return AXON_OK;
  AdamArgs a{param, grad, exp_avg, exp_avg_sq, param_out, exp_avg_out, exp_avg_sq_out,
             step_size_rows, inv_bc2_sqrt_rows, wd_rows, row_dtype, cols, n,
             hp->beta1, hp->beta2, hp->eps, hp->step_size, hp->inv_bc2_sqrt, hp->wd};
  cudaStream_t s = as_stream(stream);
  switch (state_dtype) {
    case AXON_F32: return dispatch_grad<float>(a, grad_dtype, threads, s);
    case AXON_BF16: return dispatch_grad<__nv_bfloat16>(a, grad_dtype, threads, s);
    case AXON_F16: return dispatch_grad<__half>(a, grad_dtype, threads, s);
    default: return fail(AXON_E_UNSUPPORTED, "axon_adam: unsupported state dtype %d", state_dtype);
  }
}
