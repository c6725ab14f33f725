// The GEMM-backed specs next to the hot path: qkv_cte, softmax_mm and
// attention_nkilib (the reference's kernels/<name>/kernel.py). Each is a
// row-wise map feeding a tcgen05 GEMM whose epilogue applies a per-row
// scale, so the normalisation costs no pass of its own:
//
//   qkv_cte     h = x + mlp_prev + attention_prev, r = rsqrt(mean(h^2) + eps),
//               y = r * (h @ w): by default one kernel (axon_gemm_resid3,
//               gemm.cu) that forms h while staging the GEMM's A operand;
//               variants 1 / 2 run a row pass writing h, then the GEMM
//   softmax_mm  e = exp(x), r = 1 / sum(e) (one row pass writing e), then
//               y = r * (e @ w)
//   attention   by default (head dim 64 or 128) one kernel that keeps the
//               scores on chip (axon_attention_fused, gemm.cu); variant 1:
//               e = exp(q @ k_t) written by the first GEMM's epilogue, which
//               also leaves each row's sum per 256-column tile; r = 1 / sum
//               of those (a tiny pass over s x tiles floats), then
//               y = r * (e @ v)
//
// The exponentials are bare, as in the specs (no max shift). The GEMM's A
// operand e (or h) is stored in the input dtype (bf16 / f16) and the row
// sums are taken over the values as stored, so the normaliser matches the
// operand the tensor cores read.
#include "common.cuh"

namespace axon {
namespace {

constexpr int kOpResidRms = 0;  // h = x + a + b; r = rsqrt(sum(h^2) / n + eps)
constexpr int kOpExpSum = 1;    // e = exp(x);    r = 1 / sum(e)
constexpr int kPrologueWarps = 8;

// One warp per row, 16-byte packets; n a multiple of the packet size.
template <typename T, int OP>
__global__ void __launch_bounds__(kPrologueWarps * 32) row_prologue_kernel(const T* __restrict__ x,
                                                                             const T* __restrict__ a,
                                                                             const T* __restrict__ b,
                                                                             T* __restrict__ h, float* __restrict__ r,
                                                                             int64_t m, int64_t n, float eps) {
  constexpr int E = Vec<T>::E;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kPrologueWarps + (threadIdx.x >> 5);
  pdl_wait();
  pdl_trigger();
  if (row >= m) return;
  const int64_t npk = n / E;
  const T* xr = x + row * n;
  T* hr = h + row * n;
  float acc = 0.f;
#pragma unroll 4
  for (int64_t pk = lane; pk < npk; pk += 32) {
    const Vec<T> vx = ld_vec_stream(xr + pk * E);
    Vec<T> o;
    if constexpr (OP == kOpResidRms) {
      const Vec<T> va = ld_vec_stream(a + row * n + pk * E);
      const Vec<T> vb = ld_vec_stream(b + row * n + pk * E);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float f = (to_f(vx.e[e]) + to_f(va.e[e])) + to_f(vb.e[e]);  // the spec's order
        acc = fmaf(f, f, acc);
        o.e[e] = from_f<T>(f);
      }
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        o.e[e] = from_f<T>(__expf(to_f(vx.e[e])));
        acc += to_f(o.e[e]);
      }
    }
    st_vec(hr + pk * E, o);
  }
  acc = warp_sum(acc);
  if (lane == 0) r[row] = OP == kOpResidRms ? rsqrtf(acc / static_cast<float>(n) + eps) : 1.0f / acc;
}

// r[i] = 1 / sum_t part[t * ld + i], t < tiles, in tile order.
__global__ void __launch_bounds__(256) recip_sum_kernel(const float* __restrict__ part, float* __restrict__ r,
                                                        int64_t m, int64_t tiles, int64_t ld) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  pdl_wait();
  pdl_trigger();
  if (row >= m) return;
  float s = 0.f;
  for (int64_t t = 0; t < tiles; ++t) s += part[t * ld + row];
  r[row] = 1.0f / s;
}

int64_t round256(int64_t v) { return (v + 255) / 256 * 256; }

int check_gemm_dtype(int32_t ab_dtype, const char* name) {
  if (ab_dtype != AXON_BF16 && ab_dtype != AXON_F16)
    return fail(AXON_E_UNSUPPORTED, "%s: inputs must be bf16 or f16 (the tensor-core operand types), got %d", name,
                ab_dtype);
  return AXON_OK;
}

template <int OP>
int launch_prologue(const void* x, const void* a, const void* b, void* h, float* r, int64_t m, int64_t n,
                    int32_t dtype, cudaStream_t s, const char* name) {
  const int64_t grid = (m + kPrologueWarps - 1) / kPrologueWarps;
  if (grid > 0x7fffffffLL) return fail(AXON_E_SHAPE, "%s: too many rows (%lld)", name, (long long)m);
  if (dtype == AXON_BF16) {
    launch_k(row_prologue_kernel<__nv_bfloat16, OP>, dim3(static_cast<unsigned>(grid)), dim3(kPrologueWarps * 32), 0,
             s, static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(a),
             static_cast<const __nv_bfloat16*>(b), static_cast<__nv_bfloat16*>(h), r, m, n, 1e-6f);
  } else {
    launch_k(row_prologue_kernel<__half, OP>, dim3(static_cast<unsigned>(grid)), dim3(kPrologueWarps * 32), 0, s,
             static_cast<const __half*>(x), static_cast<const __half*>(a), static_cast<const __half*>(b),
             static_cast<__half*>(h), r, m, n, 1e-6f);
  }
  return launch_status(name);
}

// Default GEMM column tile for n output columns (the rule axon_gemm applies).
int default_block_n(int64_t n) { return n <= 64 ? 64 : n <= 128 ? 128 : 256; }

}  // namespace
}  // namespace axon

using namespace axon;

namespace axon {
namespace {
int64_t qkv_rowpass_bytes(int64_t m, int64_t k) { return round256(m * k * 2) + 4 * m; }
}  // namespace
}  // namespace axon

extern "C" int64_t axon_qkv_cte_workspace_bytes(int64_t m, int64_t n, int64_t k, const axon_tune_t* tune) {
  if (m < 0 || n < 0 || k < 0) return fail(AXON_E_SHAPE, "axon_qkv_cte_workspace_bytes: negative size");
  if (tune_or_default(tune).variant == 0) return axon_gemm_resid3_workspace_bytes(m, n, k, tune);
  return qkv_rowpass_bytes(m, k);
}

extern "C" int axon_qkv_cte(const void* x, const void* mlp_prev, const void* attention_prev, const void* w, void* y,
                            void* workspace, int64_t workspace_bytes, int64_t m, int64_t n, int64_t k,
                            int32_t ab_dtype, int32_t c_dtype, const axon_tune_t* tune, void* stream) {
  int rc = check_gemm_dtype(ab_dtype, "axon_qkv_cte");
  if (rc) return rc;
  if (m < 0 || n < 0 || k < 0) return fail(AXON_E_SHAPE, "axon_qkv_cte: negative size");
  if (m == 0 || n == 0) return AXON_OK;
  if (k == 0 || k % 8) return fail(AXON_E_SHAPE, "axon_qkv_cte: k must be a positive multiple of 8");
  if (!x || !mlp_prev || !attention_prev || !w || !y) return fail(AXON_E_ARG, "axon_qkv_cte: NULL tensor");
  if (!aligned16(x) || !aligned16(mlp_prev) || !aligned16(attention_prev))
    return fail(AXON_E_ALIGN, "axon_qkv_cte: inputs must be 16-byte aligned");
  const axon_tune_t t = tune_or_default(tune);
  if (t.variant == 0)
    return axon_gemm_resid3(x, mlp_prev, attention_prev, w, y, workspace, workspace_bytes, m, n, k, ab_dtype, c_dtype,
                            1e-6f, tune, stream);
  if (t.variant != 1 && t.variant != 2) return fail(AXON_E_ARG, "axon_qkv_cte: variant must be 0, 1 or 2");
  const int64_t need = qkv_rowpass_bytes(m, k);
  if (!workspace || workspace_bytes < need || !aligned16(workspace))
    return fail(AXON_E_ARG, "axon_qkv_cte: workspace of %lld bytes needed", (long long)need);
  void* h = workspace;
  float* r = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + round256(m * k * 2));
  cudaStream_t s = as_stream(stream);
  rc = launch_prologue<kOpResidRms>(x, mlp_prev, attention_prev, h, r, m, k, ab_dtype, s, "axon_qkv_cte");
  if (rc) return rc;
  return axon_gemm(h, w, nullptr, y, r, m, n, k, k, n, n, ab_dtype, c_dtype, AXON_EPI_ROWSCALE, tune, stream);
}

extern "C" int64_t axon_softmax_mm_workspace_bytes(int64_t m, int64_t k) {
  if (m < 0 || k < 0) return fail(AXON_E_SHAPE, "axon_softmax_mm_workspace_bytes: negative size");
  return round256(m * k * 2) + 4 * m;
}

extern "C" int axon_softmax_mm(const void* x, const void* w, void* y, void* workspace, int64_t workspace_bytes,
                               int64_t m, int64_t n, int64_t k, int32_t ab_dtype, int32_t c_dtype,
                               const axon_tune_t* tune, void* stream) {
  int rc = check_gemm_dtype(ab_dtype, "axon_softmax_mm");
  if (rc) return rc;
  if (m < 0 || n < 0 || k < 0) return fail(AXON_E_SHAPE, "axon_softmax_mm: negative size");
  if (m == 0 || n == 0) return AXON_OK;
  if (k == 0 || k % 8) return fail(AXON_E_SHAPE, "axon_softmax_mm: k must be a positive multiple of 8");
  if (!x || !w || !y) return fail(AXON_E_ARG, "axon_softmax_mm: NULL tensor");
  if (!aligned16(x)) return fail(AXON_E_ALIGN, "axon_softmax_mm: x must be 16-byte aligned");
  const int64_t need = axon_softmax_mm_workspace_bytes(m, k);
  if (!workspace || workspace_bytes < need || !aligned16(workspace))
    return fail(AXON_E_ARG, "axon_softmax_mm: workspace of %lld bytes needed", (long long)need);
  void* e = workspace;
  float* r = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + round256(m * k * 2));
  cudaStream_t s = as_stream(stream);
  rc = launch_prologue<kOpExpSum>(x, nullptr, nullptr, e, r, m, k, ab_dtype, s, "axon_softmax_mm");
  if (rc) return rc;
  return axon_gemm(e, w, nullptr, y, r, m, n, k, k, n, n, ab_dtype, c_dtype, AXON_EPI_ROWSCALE, tune, stream);
}

namespace axon {
namespace {
// scores [s, s], per-tile row sums, 1 / row sums: the two-GEMM form
int64_t attention_composed_bytes(int64_t s) {
  const int64_t tiles = (s + 63) / 64;  // the most column tiles the first GEMM can use
  return round256(s * s * 2) + round256(tiles * s * 4) + 4 * s;
}
bool attention_fused_ok(int64_t d, const axon_tune_t& t) { return t.variant == 0 && (d == 64 || d == 128); }
}  // namespace
}  // namespace axon

extern "C" int64_t axon_attention_workspace_bytes(int64_t s, int64_t d, const axon_tune_t* tune) {
  if (s < 0 || d < 0) return fail(AXON_E_SHAPE, "axon_attention_workspace_bytes: negative size");
  if (attention_fused_ok(d, tune_or_default(tune))) return axon_attention_fused_workspace_bytes(s, d, tune);
  return attention_composed_bytes(s);
}

extern "C" int axon_attention(const void* q, const void* k_t, const void* v, void* y, void* workspace,
                              int64_t workspace_bytes, int64_t s, int64_t d, int32_t ab_dtype, int32_t c_dtype,
                              const axon_tune_t* tune, void* stream) {
  int rc = check_gemm_dtype(ab_dtype, "axon_attention");
  if (rc) return rc;
  if (s < 0 || d < 0) return fail(AXON_E_SHAPE, "axon_attention: negative size");
  if (s == 0 || d == 0) return AXON_OK;
  if (s % 8 || d % 8) return fail(AXON_E_SHAPE, "axon_attention: s and d must be multiples of 8");
  if (!q || !k_t || !v || !y) return fail(AXON_E_ARG, "axon_attention: NULL tensor");
  const axon_tune_t t = tune_or_default(tune);
  if (t.variant != 0 && t.variant != 1) return fail(AXON_E_ARG, "axon_attention: variant must be 0 or 1");
  if (attention_fused_ok(d, t))
    return axon_attention_fused(q, k_t, v, y, workspace, workspace_bytes, s, d, ab_dtype, c_dtype, tune, stream);
  const int64_t need = attention_composed_bytes(s);
  if (!workspace || workspace_bytes < need || !aligned16(workspace))
    return fail(AXON_E_ARG, "axon_attention: workspace of %lld bytes needed", (long long)need);
  // scores: e = exp(q @ k_t) [s, s], row sums per column tile of the first GEMM
  axon_tune_t t1 = t;
  t1.variant = 0;  // the GEMMs' own automatic choice
  if (t1.block_n == 0) t1.block_n = default_block_n(s);
  if (t1.block_n != 64 && t1.block_n != 128 && t1.block_n != 256)
    return fail(AXON_E_ARG, "axon_attention: block_n must be 64, 128 or 256");
  const int64_t tiles = (s + t1.block_n - 1) / t1.block_n;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  void* e = ws;
  float* part = reinterpret_cast<float*>(ws + round256(s * s * 2));
  float* r = reinterpret_cast<float*>(ws + round256(s * s * 2) + round256(((s + 63) / 64) * s * 4));
  rc = axon_gemm_exp(q, k_t, e, part, s, s, s, d, d, s, s, ab_dtype, ab_dtype, &t1, stream);
  if (rc) return rc;
  cudaStream_t st = as_stream(stream);
  launch_k(recip_sum_kernel, dim3(static_cast<unsigned>((s + 255) / 256)), dim3(256), 0, st,
           static_cast<const float*>(part), r, s, tiles, s);
  rc = launch_status("axon_attention");
  if (rc) return rc;
  // output: y = r * (e @ v), the second GEMM with its own default tile
  axon_tune_t t2 = t;
  t2.variant = 0;
  t2.block_n = 0;
  return axon_gemm(e, v, nullptr, y, r, s, d, s, s, d, d, ab_dtype, c_dtype, AXON_EPI_ROWSCALE, &t2, stream);
}
