// Rotary position embedding.
//
// axon_rope_split: Axon's `rope` spec layout (kernels/rope/refs.py:26-30), four
// [half_d, free] tensors -> two, a pure elementwise stream of 16-byte packets.
//
// axon_rope_rotate_half: the Llama layout. One work item is one 16-byte packet
// of x1 = x[..., :D/2] plus the matching packet of x2 = x[..., D/2:]; items are
// ordered token-major so all heads of a token (q and k) hit the same cos/sin
// row, which is read from HBM once and then from L1/L2. q and k are streamed
// once in and once out; the work is HBM-bound.
#include "common.cuh"

namespace axon {
namespace {

template <typename T>
__global__ void __launch_bounds__(256) rope_split_vec(const T* __restrict__ xe, const T* __restrict__ xo,
                                                      const T* __restrict__ c, const T* __restrict__ s, T* oe,
                                                      T* oo, int64_t npk) {
  constexpr int E = Vec<T>::E;
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < npk;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t off = i * E;
    Vec<T> a = ld_vec_stream(xe + off), b = ld_vec_stream(xo + off), cc = ld_vec_stream(c + off),
           ss = ld_vec_stream(s + off);
    Vec<T> re, ro;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      float x1 = to_f(a.e[e]), x2 = to_f(b.e[e]), cv = to_f(cc.e[e]), sv = to_f(ss.e[e]);
      re.e[e] = from_f<T>(x1 * cv - x2 * sv);
      ro.e[e] = from_f<T>(x2 * cv + x1 * sv);
    }
    st_vec_stream(oe + off, re);
    st_vec_stream(oo + off, ro);
  }
}

template <typename T>
__global__ void rope_split_scalar(const T* xe, const T* xo, const T* c, const T* s, T* oe, T* oo, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float x1 = to_f(xe[i]), x2 = to_f(xo[i]), cv = to_f(c[i]), sv = to_f(s[i]);
    oe[i] = from_f<T>(x1 * cv - x2 * sv);
    oo[i] = from_f<T>(x2 * cv + x1 * sv);
  }
}

struct RotArgs {
  const void* q;
  const void* k;
  const float* cos_t;
  const float* sin_t;
  void* q_out;
  void* k_out;
  int64_t seq, nq, nkv, half;
};

// Vector path: half % E == 0 and every tensor 16-byte aligned.
template <typename T>
__global__ void __launch_bounds__(256) rope_rotate_half_vec(RotArgs a, int64_t items) {
  constexpr int E = Vec<T>::E;
  const int64_t ppr = a.half / E;               // packets per half-row
  const int64_t heads = a.nq + a.nkv;
  const int64_t per_tok = heads * ppr;
  pdl_wait();
  pdl_trigger();
  for (int64_t it = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; it < items;
       it += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t tok = it / per_tok;
    const int64_t r = it - tok * per_tok;
    const int64_t h = r / ppr;
    const int64_t p = r - h * ppr;
    const T* src;
    T* dst;
    if (h < a.nq) {
      const int64_t base = (tok * a.nq + h) * 2 * a.half;
      src = static_cast<const T*>(a.q) + base;
      dst = static_cast<T*>(a.q_out) + base;
    } else {
      const int64_t base = (tok * a.nkv + (h - a.nq)) * 2 * a.half;
      src = static_cast<const T*>(a.k) + base;
      dst = static_cast<T*>(a.k_out) + base;
    }
    const int64_t col = p * E;
    Vec<T> x1 = ld_vec_stream(src + col), x2 = ld_vec_stream(src + a.half + col);
    const float* cr = a.cos_t + tok * a.half + col;
    const float* sr = a.sin_t + tok * a.half + col;
    float cv[E], sv[E];
#pragma unroll
    for (int j = 0; j < E; j += 4) {
      float4 c4 = __ldg(reinterpret_cast<const float4*>(cr + j));
      float4 s4 = __ldg(reinterpret_cast<const float4*>(sr + j));
      cv[j] = c4.x; cv[j + 1] = c4.y; cv[j + 2] = c4.z; cv[j + 3] = c4.w;
      sv[j] = s4.x; sv[j + 1] = s4.y; sv[j + 2] = s4.z; sv[j + 3] = s4.w;
    }
    Vec<T> o1, o2;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      float a1 = to_f(x1.e[e]), a2 = to_f(x2.e[e]);
      o1.e[e] = from_f<T>(a1 * cv[e] - a2 * sv[e]);
      o2.e[e] = from_f<T>(a2 * cv[e] + a1 * sv[e]);
    }
    st_vec_stream(dst + col, o1);
    st_vec_stream(dst + a.half + col, o2);
  }
}

// Token-blocked vector path (variant 0), used when one token's packets (heads
// x packets per half-row, at most 512) fit in one CTA: thread t owns head
// t / ppr and packet t % ppr for TOK consecutive tokens, so all index math is
// done once per thread and the TOK tokens' q/k loads are issued together
// (only the raw packets are held in registers). The cos/sin rows are read in
// the compute loop: every head of a token reads the same row, so after the
// first head they are L1 hits.
template <typename T, int TOK>
__global__ void __launch_bounds__(512) rope_rotate_half_tok(RotArgs a, int ppr) {
  constexpr int E = Vec<T>::E;
  pdl_wait();
  pdl_trigger();
  const int t = threadIdx.x;
  const int h = t / ppr;
  const int p = t - h * ppr;
  if (h >= a.nq + a.nkv) return;
  const int64_t half = a.half;
  const bool is_q = h < a.nq;
  const int64_t hh = is_q ? h : h - a.nq;
  const int64_t nh = is_q ? a.nq : a.nkv;
  const T* src = static_cast<const T*>(is_q ? a.q : a.k);
  T* dst = static_cast<T*>(is_q ? a.q_out : a.k_out);
  const int64_t tok0 = static_cast<int64_t>(blockIdx.x) * TOK;
  const int col = p * E;
  Vec<T> x1[TOK], x2[TOK];
#pragma unroll
  for (int i = 0; i < TOK; ++i) {
    const int64_t tok = tok0 + i;
    if (tok < a.seq) {
      const T* s = src + (tok * nh + hh) * 2 * half + col;
      x1[i] = ld_vec_stream(s);
      x2[i] = ld_vec_stream(s + half);
    }
  }
#pragma unroll
  for (int i = 0; i < TOK; ++i) {
    const int64_t tok = tok0 + i;
    if (tok >= a.seq) continue;
    float c[E], s[E];
#pragma unroll
    for (int j = 0; j < E; j += 4) {
      const float4 c4 = __ldg(reinterpret_cast<const float4*>(a.cos_t + tok * half + col + j));
      const float4 s4 = __ldg(reinterpret_cast<const float4*>(a.sin_t + tok * half + col + j));
      c[j] = c4.x; c[j + 1] = c4.y; c[j + 2] = c4.z; c[j + 3] = c4.w;
      s[j] = s4.x; s[j + 1] = s4.y; s[j + 2] = s4.z; s[j + 3] = s4.w;
    }
    Vec<T> o1, o2;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float a1 = to_f(x1[i].e[e]), a2 = to_f(x2[i].e[e]);
      o1.e[e] = from_f<T>(a1 * c[e] - a2 * s[e]);
      o2.e[e] = from_f<T>(a2 * c[e] + a1 * s[e]);
    }
    T* d = dst + (tok * nh + hh) * 2 * half + col;
    st_vec_stream(d, o1);
    st_vec_stream(d + half, o2);
  }
}

template <typename T>
__global__ void rope_rotate_half_scalar(RotArgs a, int64_t items) {
  const int64_t heads = a.nq + a.nkv;
  for (int64_t it = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; it < items;
       it += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t tok = it / (heads * a.half);
    const int64_t r = it - tok * heads * a.half;
    const int64_t h = r / a.half;
    const int64_t j = r - h * a.half;
    const T* src;
    T* dst;
    if (h < a.nq) {
      const int64_t base = (tok * a.nq + h) * 2 * a.half;
      src = static_cast<const T*>(a.q) + base;
      dst = static_cast<T*>(a.q_out) + base;
    } else {
      const int64_t base = (tok * a.nkv + (h - a.nq)) * 2 * a.half;
      src = static_cast<const T*>(a.k) + base;
      dst = static_cast<T*>(a.k_out) + base;
    }
    float x1 = to_f(src[j]), x2 = to_f(src[a.half + j]);
    float cv = a.cos_t[tok * a.half + j], sv = a.sin_t[tok * a.half + j];
    dst[j] = from_f<T>(x1 * cv - x2 * sv);
    dst[a.half + j] = from_f<T>(x2 * cv + x1 * sv);
  }
}

int grid_for(int64_t items, int threads) {
  int64_t want = (items + threads - 1) / threads;
  int64_t cap = static_cast<int64_t>(sm_count()) * (2048 / threads) * 4;
  if (want > cap) want = cap;
  return static_cast<int>(want < 1 ? 1 : want);
}

template <typename T>
int launch_split(const void* xe, const void* xo, const void* c, const void* s, void* oe, void* oo, int64_t n,
                 int threads, cudaStream_t st) {
  constexpr int E = Vec<T>::E;
  const bool vec = aligned16(xe) && aligned16(xo) && aligned16(c) && aligned16(s) && aligned16(oe) &&
                   aligned16(oo) && n % E == 0;
  if (vec) {
    const int64_t npk = n / E;
    launch_k(rope_split_vec<T>, dim3(grid_for(npk, threads)), dim3(threads), 0, st, static_cast<const T*>(xe),
             static_cast<const T*>(xo), static_cast<const T*>(c), static_cast<const T*>(s), static_cast<T*>(oe),
             static_cast<T*>(oo), npk);
  } else {
    rope_split_scalar<T><<<grid_for(n, threads), threads, 0, st>>>(
        static_cast<const T*>(xe), static_cast<const T*>(xo), static_cast<const T*>(c),
        static_cast<const T*>(s), static_cast<T*>(oe), static_cast<T*>(oo), n);
  }
  return launch_status("axon_rope_split");
}

template <typename T>
int launch_rot(const RotArgs& a, int variant, int threads, int rows_per_cta, cudaStream_t st) {
  constexpr int E = Vec<T>::E;
  bool vec = a.half % E == 0 && aligned16(a.q) && aligned16(a.q_out) && aligned16(a.cos_t) &&
             aligned16(a.sin_t);
  if (a.nkv > 0) vec = vec && aligned16(a.k) && aligned16(a.k_out);
  const int64_t heads = a.nq + a.nkv;
  const int64_t per_tok = vec ? heads * (a.half / E) : 0;
  if (vec && variant == 0 && per_tok <= 512) {
    // tokens per CTA: tune.rows_per_cta in {1, 2, 4, 8}; default 1 (measured
    // on B200 at the Llama-3-8B GQA config: 1 token 14.0 us, 2 14.5, 4 16.9)
    const int tok = rows_per_cta > 0 ? rows_per_cta : 1;
    const int block = static_cast<int>((per_tok + 31) / 32 * 32);
    const int64_t grid = (a.seq + tok - 1) / tok;
    if (grid > 0x7fffffff) return fail(AXON_E_SHAPE, "axon_rope_rotate_half: sequence too long");
    const dim3 g(static_cast<unsigned>(grid)), b(block);
    const int ppr = static_cast<int>(a.half / E);
    switch (tok) {
      case 1: launch_k(rope_rotate_half_tok<T, 1>, g, b, 0, st, a, ppr); break;
      case 2: launch_k(rope_rotate_half_tok<T, 2>, g, b, 0, st, a, ppr); break;
      case 4: launch_k(rope_rotate_half_tok<T, 4>, g, b, 0, st, a, ppr); break;
      case 8: launch_k(rope_rotate_half_tok<T, 8>, g, b, 0, st, a, ppr); break;
      default: return fail(AXON_E_ARG, "axon_rope_rotate_half: rows_per_cta (tokens per CTA) must be 1, 2, 4 or 8");
    }
  } else if (vec) {
    const int64_t items = a.seq * heads * (a.half / E);
    launch_k(rope_rotate_half_vec<T>, dim3(grid_for(items, threads)), dim3(threads), 0, st, a, items);
  } else {
    const int64_t items = a.seq * heads * a.half;
    rope_rotate_half_scalar<T><<<grid_for(items, threads), threads, 0, st>>>(a, items);
  }
  return launch_status("axon_rope_rotate_half");
}

}  // namespace
}  // namespace axon

using namespace axon;

extern "C" int axon_rope_split(const void* x_even, const void* x_odd, const void* cos_t, const void* sin_t,
                               void* out_even, void* out_odd, int64_t half_d, int64_t free_n, int32_t dtype,
                               const axon_tune_t* tune, void* stream) {
  axon_tune_t t = tune_or_default(tune);
  if (half_d < 0 || free_n < 0) return fail(AXON_E_SHAPE, "axon_rope_split: negative size");
  if (half_d == 0 || free_n == 0) return AXON_OK;
  if (!x_even || !x_odd || !cos_t || !sin_t || !out_even || !out_odd)
    return fail(AXON_E_ARG, "axon_rope_split: NULL tensor pointer");
  if (t.variant != 0) return fail(AXON_E_ARG, "axon_rope_split: unknown variant %d", t.variant);
  const int threads = t.threads > 0 ? t.threads : 256;
  if (threads > 256 || threads % 32) return fail(AXON_E_ARG, "axon_rope_split: threads must be 32..256, multiple of 32");
  const int64_t n = half_d * free_n;
  if (n == 0) return AXON_OK;
  cudaStream_t s = as_stream(stream);
  switch (dtype) {
    case AXON_F32: return launch_split<float>(x_even, x_odd, cos_t, sin_t, out_even, out_odd, n, threads, s);
    case AXON_BF16: return launch_split<__nv_bfloat16>(x_even, x_odd, cos_t, sin_t, out_even, out_odd, n, threads, s);
    case AXON_F16: return launch_split<__half>(x_even, x_odd, cos_t, sin_t, out_even, out_odd, n, threads, s);
    default: return fail(AXON_E_UNSUPPORTED, "axon_rope_split: unsupported dtype %d", dtype);
  }
}

extern "C" int axon_rope_rotate_half(const void* q, const void* k, const float* cos_t, const float* sin_t,
                                     void* q_out, void* k_out, int64_t seq, int64_t n_q, int64_t n_kv,
                                     int64_t head_dim, int32_t dtype, const axon_tune_t* tune, void* stream) {
  axon_tune_t t = tune_or_default(tune);
  if (seq < 0 || n_q < 0 || n_kv < 0 || head_dim < 0 || head_dim % 2)
    return fail(AXON_E_SHAPE, "axon_rope_rotate_half: bad shape (head_dim must be even)");
  if (seq == 0 || head_dim == 0 || n_q + n_kv == 0) return AXON_OK;
  if (!q || !q_out || !cos_t || !sin_t) return fail(AXON_E_ARG, "axon_rope_rotate_half: NULL tensor pointer");
  if (n_kv > 0 && (!k || !k_out)) return fail(AXON_E_ARG, "axon_rope_rotate_half: NULL k pointer with n_kv > 0");
  if (t.variant < 0 || t.variant > 1) return fail(AXON_E_ARG, "axon_rope_rotate_half: unknown variant %d", t.variant);
  const int threads = t.threads > 0 ? t.threads : 256;
  if (threads > 256 || threads % 32) return fail(AXON_E_ARG, "axon_rope_rotate_half: threads must be 32..256, multiple of 32");
  if (seq == 0 || head_dim == 0 || n_q + n_kv == 0) return AXON_OK;
  RotArgs a{q, k, cos_t, sin_t, q_out, k_out, seq, n_q, n_kv, head_dim / 2};
  cudaStream_t s = as_stream(stream);
  switch (dtype) {
    case AXON_F32: return launch_rot<float>(a, t.variant, threads, t.rows_per_cta, s);
    case AXON_BF16: return launch_rot<__nv_bfloat16>(a, t.variant, threads, t.rows_per_cta, s);
    case AXON_F16: return launch_rot<__half>(a, t.variant, threads, t.rows_per_cta, s);
    default: return fail(AXON_E_UNSUPPORTED, "axon_rope_rotate_half: unsupported dtype %d", dtype);
  }
}
