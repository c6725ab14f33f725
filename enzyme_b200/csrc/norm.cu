// Row-wise kernels: rmsnorm (sum and mean forms, optional weight), layernorm,
// softmax, and the per-row rsqrt(sum x^2) prologue of rmsnorm_matmul.
//
// Variant 0 ("row_resident") keeps each row in registers as raw 16-byte
// packets: one group of threads per row (a warp up to a full 1024-thread CTA)
// issues every load of the row before it reduces, so each row costs exactly
// one HBM read and one HBM write. Statistics are fp32, reduced with warp
// shuffles and (for multi-warp rows) a small shared-memory exchange.
// Variant 1 ("row_streaming") handles rows too long for registers, and rows
// whose starts are not 16-byte aligned: a CTA walks its row once per pass;
// the second pass re-reads the row from L2 (rows in flight are far smaller
// than the 126 MB L2). Variant 2 ("row_bulk_warp", below) stages rows in
// shared memory with bulk copies and reduces one row per warp. Variant 3
// ("row_bulk_cta") stages rows of up to ~200 KB in shared memory chunk by
// chunk, one persistent CTA per row at a time, refilling each chunk with the
// CTA's next row as soon as the output pass has read it. Variant 0 picks
// variant 3 for rows of 16 KB and more, variant 2 for shorter rows, when
// there is at least a row per SM, else the register-resident kernel.
#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace axon {

__device__ int g_row_error;

namespace {

enum RowOp { OP_RMS = 0, OP_LN = 1, OP_SM = 2, OP_RSQRT = 3 };

struct RowArgs {
  const void* x;
  void* y;
  const void* w;   // rmsnorm weight [n] or NULL
  float* r_out;    // OP_RSQRT output [m]
  int64_t m, n, ld_x, ld_y;
  int32_t w_dtype;
  float scale, eps;
};

// Sum (or max) across the threads that own one row. `red` holds one slot per
// warp of the CTA; rows never share a warp.
template <bool MAX>
__device__ __forceinline__ float row_allreduce(float v, float* red, int gw, int row_in_cta) {
  v = MAX ? warp_max(v) : warp_sum(v);
  if (gw == 1) return v;
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  __syncthreads();
  float r = red[row_in_cta * gw];
  for (int i = 1; i < gw; ++i) {
    float o = red[row_in_cta * gw + i];
    r = MAX ? fmaxf(r, o) : r + o;
  }
  __syncthreads();
  return r;
}

__device__ __forceinline__ float weight_at(const RowArgs& a, int64_t col) {
  return a.w ? load_any(a.w, col, a.w_dtype) : 1.0f;
}

// 16-bit rows are capped at 512 threads per CTA so a thread may hold up to
// eight 16-byte packets (64 elements) without spilling.
template <typename T>
constexpr int max_row_threads() { return sizeof(T) == 2 ? 512 : 1024; }

template <typename T, int VPT, int OP>
__global__ void __launch_bounds__(max_row_threads<T>()) row_resident_kernel(RowArgs a, int gw, int rows_per_cta) {
  constexpr int E = Vec<T>::E;
  __shared__ float red[32];
  const int tpr = gw * 32;
  const int lane = threadIdx.x % tpr;
  const int row_in_cta = threadIdx.x / tpr;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * rows_per_cta + row_in_cta;
  const bool active = row < a.m;
  const int64_t n = a.n;
  pdl_wait();
  pdl_trigger();
  const T* xr = static_cast<const T*>(a.x) + (active ? row : 0) * a.ld_x;

  Vec<T> raw[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t col = (static_cast<int64_t>(i) * tpr + lane) * E;
    if (active && col + E <= n) {
      raw[i] = ld_vec(xr + col);
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) raw[i].e[e] = (active && col + e < n) ? xr[col + e] : from_f<T>(0.f);
    }
  }
  auto valid = [&](int i, int e) -> bool {
    return active && (static_cast<int64_t>(i) * tpr + lane) * E + e < n;
  };
  // Keep only the raw packets live between passes: without this the compiler
  // holds every converted fp32 value of the previous pass, doubling the
  // registers (and halving the resident rows).
  auto pin_raw = [&]() {
#pragma unroll
    for (int i = 0; i < VPT; ++i)
      asm volatile("" : "+r"(raw[i].u.x), "+r"(raw[i].u.y), "+r"(raw[i].u.z), "+r"(raw[i].u.w));
  };

  float s0 = 0.f, s1 = 0.f;  // op-specific statistics
  if constexpr (OP == OP_RMS || OP == OP_RSQRT) {
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int e = 0; e < E; ++e) {
        float v = to_f(raw[i].e[e]);
        s0 = fmaf(v, v, s0);
      }
    s0 = row_allreduce<false>(s0, red, gw, row_in_cta);
    s1 = rsqrtf(a.scale * s0 + a.eps);
    if constexpr (OP == OP_RSQRT) {
      if (active && lane == 0) a.r_out[row] = s1;
      return;
    }
  } else if constexpr (OP == OP_LN) {
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int e = 0; e < E; ++e) s0 += to_f(raw[i].e[e]);
    const float mean = row_allreduce<false>(s0, red, gw, row_in_cta) / static_cast<float>(n);
    pin_raw();
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int e = 0; e < E; ++e) {
        float c = valid(i, e) ? to_f(raw[i].e[e]) - mean : 0.f;
        ss = fmaf(c, c, ss);
      }
    ss = row_allreduce<false>(ss, red, gw, row_in_cta);
    s0 = mean;
    s1 = rsqrtf(ss / static_cast<float>(n) + a.eps);
  } else {  // OP_SM
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int e = 0; e < E; ++e)
        if (valid(i, e)) mx = fmaxf(mx, to_f(raw[i].e[e]));
    mx = row_allreduce<true>(mx, red, gw, row_in_cta);
    pin_raw();
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int e = 0; e < E; ++e)
        if (valid(i, e)) sum += __expf(to_f(raw[i].e[e]) - mx);
    sum = row_allreduce<false>(sum, red, gw, row_in_cta);
    s0 = mx;
    s1 = 1.0f / sum;
  }

  if (!active) return;
  pin_raw();
  T* yr = static_cast<T*>(a.y) + row * a.ld_y;
  // The resident path only takes a weight of the row's own dtype, read as
  // 16-byte packets (all rows share it, so it stays in L1/L2).
  const T* w = static_cast<const T*>(a.w);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t col = (static_cast<int64_t>(i) * tpr + lane) * E;
    if (col >= n) continue;
    Vec<T> wv;
    if constexpr (OP == OP_RMS) {
      if (w != nullptr && col + E <= n) {
        wv = ld_vec(w + col);
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) wv.e[e] = (w != nullptr && col + e < n) ? w[col + e] : from_f<T>(1.f);
      }
    }
    Vec<T> o;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      float v = to_f(raw[i].e[e]);
      float r;
      if constexpr (OP == OP_RMS) r = v * s1 * to_f(wv.e[e]);
      else if constexpr (OP == OP_LN) r = (v - s0) * s1;
      else r = __expf(v - s0) * s1;
      o.e[e] = from_f<T>(r);
    }
    if (col + E <= n) {
      st_vec(yr + col, o);
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e)
        if (col + e < n) yr[col + e] = o.e[e];
    }
  }
}

// One CTA per row, any length / alignment. VEC selects 16-byte packets (the
// row start and length must then be packet-aligned) or single elements.
template <typename T, bool VEC, int OP>
__global__ void __launch_bounds__(1024) row_streaming_kernel(RowArgs a) {
  constexpr int E = VEC ? Vec<T>::E : 1;
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int64_t n = a.n;
  const int gw = blockDim.x / 32;
  const T* xr = static_cast<const T*>(a.x) + row * a.ld_x;
  T* yr = static_cast<T*>(a.y) + row * a.ld_y;
  const int64_t nchunks = (n + E - 1) / E;
  pdl_wait();
  pdl_trigger();

  auto load = [&](int64_t c, float* v) {
    const int64_t col = c * E;
    if constexpr (VEC) {
      if (col + E <= n) {
        Vec<T> p = ld_vec(xr + col);
#pragma unroll
        for (int e = 0; e < E; ++e) v[e] = to_f(p.e[e]);
        return;
      }
    }
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = col + e < n ? to_f(xr[col + e]) : 0.f;
  };

  float s0 = 0.f, s1 = 0.f;
  float v[E];
  if constexpr (OP == OP_RMS || OP == OP_RSQRT) {
    for (int64_t c = threadIdx.x; c < nchunks; c += blockDim.x) {
      load(c, v);
#pragma unroll
      for (int e = 0; e < E; ++e) s0 = fmaf(v[e], v[e], s0);
    }
    s0 = row_allreduce<false>(s0, red, gw, 0);
    s1 = rsqrtf(a.scale * s0 + a.eps);
    if constexpr (OP == OP_RSQRT) {
      if (threadIdx.x == 0) a.r_out[row] = s1;
      return;
    }
  } else if constexpr (OP == OP_LN) {
    for (int64_t c = threadIdx.x; c < nchunks; c += blockDim.x) {
      load(c, v);
#pragma unroll
      for (int e = 0; e < E; ++e) s0 += v[e];
    }
    const float mean = row_allreduce<false>(s0, red, gw, 0) / static_cast<float>(n);
    float ss = 0.f;
    for (int64_t c = threadIdx.x; c < nchunks; c += blockDim.x) {
      load(c, v);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        float d = c * E + e < n ? v[e] - mean : 0.f;
        ss = fmaf(d, d, ss);
      }
    }
    ss = row_allreduce<false>(ss, red, gw, 0);
    s0 = mean;
    s1 = rsqrtf(ss / static_cast<float>(n) + a.eps);
  } else {  // OP_SM: online max / rescaled sum in one pass
    float mx = -INFINITY, sum = 0.f;
    for (int64_t c = threadIdx.x; c < nchunks; c += blockDim.x) {
      load(c, v);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        if (c * E + e >= n) continue;
        if (v[e] > mx) {
          sum = sum * __expf(mx - v[e]) + 1.f;
          mx = v[e];
        } else {
          sum += __expf(v[e] - mx);
        }
      }
    }
    const float gmx = row_allreduce<true>(mx, red, gw, 0);
    sum = mx == -INFINITY ? 0.f : sum * __expf(mx - gmx);
    sum = row_allreduce<false>(sum, red, gw, 0);
    s0 = gmx;
    s1 = 1.0f / sum;
  }

  if constexpr (OP != OP_RSQRT) {
  for (int64_t c = threadIdx.x; c < nchunks; c += blockDim.x) {
    load(c, v);
    const int64_t col = c * E;
    float r[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      if constexpr (OP == OP_RMS) r[e] = v[e] * s1 * weight_at(a, col + e < n ? col + e : 0);
      else if constexpr (OP == OP_LN) r[e] = (v[e] - s0) * s1;
      else r[e] = __expf(v[e] - s0) * s1;
    }
    if constexpr (VEC) {
      if (col + E <= n) {
        Vec<T> o;
#pragma unroll
        for (int e = 0; e < E; ++e) o.e[e] = from_f<T>(r[e]);
        st_vec(yr + col, o);
        continue;
      }
    }
#pragma unroll
    for (int e = 0; e < E; ++e)
      if (col + e < n) yr[col + e] = from_f<T>(r[e]);
  }
  }
}

// Variant 2 ("row_bulk_warp"): one warp per row, rows staged in shared
// memory by the bulk-copy engine. Each warp owns `slots` row buffers and an
// mbarrier per buffer; its lane 0 issues cp.async.bulk for its first rows as
// soon as the grid starts, so every SM has all of its rows (up to ~200 KB)
// in flight at once -- the whole [2048, 4096] bf16 input of the Llama
// rmsnorm config fits in the GPU's shared memory. The warp then reduces the
// row from shared memory with shuffles only (no CTA barrier), writes the
// output with 16-byte stores, and refills the buffer with its row + slots*G.
// The rmsnorm weight is staged once per CTA. Rows must be 16-byte aligned
// with n * sizeof(T) a multiple of 16 and at most 32 KB.
constexpr uint64_t kRowWaitNs = 2000000000ull;
constexpr int kBulkSmemBudget = 200 * 1024;
constexpr int kBulkMaxRowBytes = 32 * 1024;
constexpr int kBulkTargetBytes = 136 * 1024;  // rows (+ weight) per CTA by default

template <typename T>
__device__ __forceinline__ Vec<T> ld_smem_vec(const T* p) {
  Vec<T> v;
  v.u = *reinterpret_cast<const uint4*>(p);
  return v;
}

template <typename T, int OP>
__global__ void __launch_bounds__(1024) row_bulk_kernel(RowArgs a, int slots, uint32_t row_bytes) {
  constexpr int E = Vec<T>::E;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool has_w = OP == OP_RMS && a.w != nullptr;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  T* sw = reinterpret_cast<T*>(smem + 512);  // after the mbarriers (32 warps x 2 slots at most)
  uint8_t* rows = reinterpret_cast<uint8_t*>(sw) + (has_w ? row_bytes : 0);
  uint64_t* my_bar = bars + warp * slots;
  uint8_t* my_buf = rows + static_cast<size_t>(warp) * slots * row_bytes;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * warps + warp;
  const int64_t G = static_cast<int64_t>(gridDim.x) * warps;
  const int64_t npk = a.n / E;
  const T* x = static_cast<const T*>(a.x);

  if (lane == 0) {
    for (int s = 0; s < slots; ++s) sm100::mbar_init(&my_bar[s], 1);
    sm100::mbar_init_fence();
  }
  __syncwarp();
  pdl_wait();
  pdl_trigger();
  if (lane == 0) {
    for (int s = 0; s < slots; ++s) {
      const int64_t row = gw + s * G;
      if (row < a.m) {
        sm100::mbar_expect_tx(&my_bar[s], row_bytes);
        sm100::bulk_g2s(my_buf + s * row_bytes, x + row * a.ld_x, row_bytes, &my_bar[s]);
      }
    }
  }
  if (has_w) {
    const T* w = static_cast<const T*>(a.w);
    for (int64_t p = threadIdx.x; p < npk; p += blockDim.x) st_vec(sw + p * E, ld_vec(w + p * E));
  }
  __syncthreads();

  int i = 0;
  bool clean = true;
  for (int64_t row = gw; row < a.m; row += G, ++i) {
    const int s = slots == 1 ? 0 : (i & 1);
    const uint32_t parity = static_cast<uint32_t>((slots == 1 ? i : i >> 1) & 1);
    const bool ok = __all_sync(0xffffffffu, sm100::mbar_wait_bounded(&my_bar[s], parity, kRowWaitNs));
    if (!ok) {
      if (lane == 0) atomicExch(&g_row_error, AXON_E_TIMEOUT);
      clean = false;
      break;
    }
    const T* sx = reinterpret_cast<const T*>(my_buf + s * row_bytes);
    float s0 = 0.f, s1 = 0.f;
    if constexpr (OP == OP_RMS || OP == OP_RSQRT) {
#pragma unroll 4
      for (int64_t p = lane; p < npk; p += 32) {
        const Vec<T> v = ld_smem_vec(sx + p * E);
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const float f = to_f(v.e[e]);
          s0 = fmaf(f, f, s0);
        }
      }
      s1 = rsqrtf(a.scale * warp_sum(s0) + a.eps);
    } else if constexpr (OP == OP_LN) {
#pragma unroll 4
      for (int64_t p = lane; p < npk; p += 32) {
        const Vec<T> v = ld_smem_vec(sx + p * E);
#pragma unroll
        for (int e = 0; e < E; ++e) s0 += to_f(v.e[e]);
      }
      s0 = warp_sum(s0) / static_cast<float>(a.n);
      float ss = 0.f;
#pragma unroll 4
      for (int64_t p = lane; p < npk; p += 32) {
        const Vec<T> v = ld_smem_vec(sx + p * E);
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const float c = to_f(v.e[e]) - s0;
          ss = fmaf(c, c, ss);
        }
      }
      s1 = rsqrtf(warp_sum(ss) / static_cast<float>(a.n) + a.eps);
    } else {  // OP_SM
      float mx = -INFINITY;
#pragma unroll 4
      for (int64_t p = lane; p < npk; p += 32) {
        const Vec<T> v = ld_smem_vec(sx + p * E);
#pragma unroll
        for (int e = 0; e < E; ++e) mx = fmaxf(mx, to_f(v.e[e]));
      }
      s0 = warp_max(mx);
      float sum = 0.f;
#pragma unroll 4
      for (int64_t p = lane; p < npk; p += 32) {
        const Vec<T> v = ld_smem_vec(sx + p * E);
#pragma unroll
        for (int e = 0; e < E; ++e) sum += __expf(to_f(v.e[e]) - s0);
      }
      s1 = 1.0f / warp_sum(sum);
    }
    if constexpr (OP == OP_RSQRT) {
      if (lane == 0) a.r_out[row] = s1;
    } else {
      T* yr = static_cast<T*>(a.y) + row * a.ld_y;
#pragma unroll 4
      for (int64_t p = lane; p < npk; p += 32) {
        const Vec<T> v = ld_smem_vec(sx + p * E);
        Vec<T> wv;
        if constexpr (OP == OP_RMS) {
          if (has_w) wv = ld_smem_vec(sw + p * E);
        }
        Vec<T> o;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const float f = to_f(v.e[e]);
          float r;
          if constexpr (OP == OP_RMS) r = has_w ? f * s1 * to_f(wv.e[e]) : f * s1;
          else if constexpr (OP == OP_LN) r = (f - s0) * s1;
          else r = __expf(f - s0) * s1;
          o.e[e] = from_f<T>(r);
        }
        st_vec(yr + p * E, o);
      }
    }
    __syncwarp();  // every lane has read the buffer before it is refilled
    if (lane == 0) {
      const int64_t next = row + slots * G;
      if (next < a.m) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        sm100::mbar_expect_tx(&my_bar[s], row_bytes);
        sm100::bulk_g2s(my_buf + s * row_bytes, x + next * a.ld_x, row_bytes, &my_bar[s]);
      }
    }
  }
  // A warp that gave up may leave copies in flight: give them time to land
  // before the CTA's shared memory is released (failure path only).
  if (!clean && lane == 0)
    for (int k = 0; k < 2000; ++k) __nanosleep(1000);
}

// Variant 3 ("row_bulk_cta"): one CTA per row, for rows past a warp's share
// of shared memory (up to ~200 KB). The row is staged in shared memory by
// 1-D bulk copies in chunks, each completing on its own mbarrier, so the
// statistics pass starts on the first chunk while the others are landing.
// CTAs are persistent over rows (row, row + grid, ...): as soon as the
// output pass has read a chunk, that chunk's buffer is refilled with the same
// chunk of the CTA's next row, so the next row's reads overlap this row's
// writes -- the register-resident kernel (one CTA of a whole-row register
// file per SM) loads, reduces and stores strictly in turn. One HBM read and
// one HBM write per row; the rmsnorm weight is read from global memory (it
// stays in L1/L2). Statistics are those of the other variants: fp32, two
// passes over the staged row for layernorm and softmax.
constexpr int kCtaThreads = 512;
constexpr int kCtaBarBytes = 256;  // one mbarrier per chunk
constexpr int kCtaMaxChunks = kCtaBarBytes / 8;
constexpr int64_t kCtaMaxRowBytes = kBulkSmemBudget - kCtaBarBytes;
constexpr int64_t kCtaChunkBytes = 16384;
constexpr int64_t kCtaDefaultMinRowBytes = 16384;  // variant 0 runs variant 3 from this row size

// Sum (or max) over all threads of the CTA. Ends with a CTA barrier, so every
// shared-memory read issued before the call is complete on return.
template <bool MAX>
__device__ __forceinline__ float cta_allreduce(float v, float* red) {
  v = MAX ? warp_max(v) : warp_sum(v);
  const int nw = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
  for (int i = 1; i < nw; ++i) r = MAX ? fmaxf(r, red[i]) : r + red[i];
  __syncthreads();
  return r;
}

// rmsnorm, layernorm and softmax (the rsqrt prologue of rmsnorm_matmul keeps
// the warp-per-row kernel).
template <typename T, int OP>
__global__ void __launch_bounds__(1024) row_cta_bulk_kernel(RowArgs a, uint32_t row_bytes, uint32_t chunk_bytes,
                                                          int nch) {
  static_assert(OP == OP_RMS || OP == OP_LN || OP == OP_SM, "row_cta_bulk_kernel: rmsnorm, layernorm, softmax");
  constexpr int E = Vec<T>::E;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float red[32];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint8_t* buf = smem + kCtaBarBytes;
  const T* sx = reinterpret_cast<const T*>(buf);
  const uint8_t* xb = static_cast<const uint8_t*>(a.x);
  const int tid = threadIdx.x;
  const uint32_t nt = blockDim.x;
  const int64_t ld_bytes = a.ld_x * static_cast<int64_t>(sizeof(T));
  const uint32_t pkc = chunk_bytes / 16;  // packets in a full chunk
  const uint32_t npk = row_bytes / 16;    // packets in a row

  // chunk c of `row` into its buffer; the last chunk may be shorter
  auto issue = [&](int64_t row, int c) {
    const uint32_t off = static_cast<uint32_t>(c) * chunk_bytes;
    const uint32_t bytes = row_bytes - off < chunk_bytes ? row_bytes - off : chunk_bytes;
    sm100::mbar_expect_tx(&bars[c], bytes);
    sm100::bulk_g2s(buf + off, xb + row * ld_bytes + off, bytes, &bars[c]);
  };
  auto chunk_end = [&](int c) -> uint32_t {
    const uint32_t e = static_cast<uint32_t>(c + 1) * pkc;
    return e < npk ? e : npk;
  };

  if (tid == 0) {
    for (int c = 0; c < nch; ++c) sm100::mbar_init(&bars[c], 1);
    sm100::mbar_init_fence();
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  if (tid == 0 && blockIdx.x < a.m)
    for (int c = 0; c < nch; ++c) issue(blockIdx.x, c);

  bool clean = true;
  uint32_t parity = 0;
  for (int64_t row = blockIdx.x; row < a.m; row += gridDim.x, parity ^= 1u) {
    const int64_t next = row + gridDim.x;
    // statistics pass, each chunk as soon as it has landed (every thread
    // waits on every chunk, so the whole row is visible to it afterwards)
    bool ok = true;
    float s0 = OP == OP_SM ? -INFINITY : 0.f, s1 = 0.f;
    for (int c = 0; c < nch; ++c) {
      if (ok) ok = sm100::mbar_wait_bounded(&bars[c], parity, kRowWaitNs);
      const uint32_t end = chunk_end(c);
      for (uint32_t p = static_cast<uint32_t>(c) * pkc + tid; p < end; p += nt) {
        const Vec<T> v = ld_smem_vec(sx + static_cast<size_t>(p) * E);
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const float f = to_f(v.e[e]);
          if constexpr (OP == OP_RMS) s0 = fmaf(f, f, s0);
          else if constexpr (OP == OP_LN) s0 += f;
          else s0 = fmaxf(s0, f);
        }
      }
    }
    if (!__syncthreads_and(ok)) {  // the same decision in every thread
      if (tid == 0) atomicExch(&g_row_error, AXON_E_TIMEOUT);
      clean = false;
      break;
    }
    if constexpr (OP == OP_RMS) {
      s1 = rsqrtf(a.scale * cta_allreduce<false>(s0, red) + a.eps);
    } else if constexpr (OP == OP_LN) {
      s0 = cta_allreduce<false>(s0, red) / static_cast<float>(a.n);
      float ss = 0.f;
      for (uint32_t p = tid; p < npk; p += nt) {
        const Vec<T> v = ld_smem_vec(sx + static_cast<size_t>(p) * E);
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const float d = to_f(v.e[e]) - s0;
          ss = fmaf(d, d, ss);
        }
      }
      s1 = rsqrtf(cta_allreduce<false>(ss, red) / static_cast<float>(a.n) + a.eps);
    } else {  // OP_SM
      s0 = cta_allreduce<true>(s0, red);
      float sum = 0.f;
      for (uint32_t p = tid; p < npk; p += nt) {
        const Vec<T> v = ld_smem_vec(sx + static_cast<size_t>(p) * E);
#pragma unroll
        for (int e = 0; e < E; ++e) sum += __expf(to_f(v.e[e]) - s0);
      }
      s1 = 1.0f / cta_allreduce<false>(sum, red);
    }
    T* yr = static_cast<T*>(a.y) + row * a.ld_y;
    const T* w = static_cast<const T*>(a.w);
    for (int c = 0; c < nch; ++c) {
      const uint32_t end = chunk_end(c);
      for (uint32_t p = static_cast<uint32_t>(c) * pkc + tid; p < end; p += nt) {
        const Vec<T> v = ld_smem_vec(sx + static_cast<size_t>(p) * E);
        Vec<T> wv;
        if constexpr (OP == OP_RMS) {
          if (w != nullptr) wv = ld_vec(w + static_cast<size_t>(p) * E);
        }
        Vec<T> o;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const float f = to_f(v.e[e]);
          float r;
          if constexpr (OP == OP_RMS) r = w != nullptr ? f * s1 * to_f(wv.e[e]) : f * s1;
          else if constexpr (OP == OP_LN) r = (f - s0) * s1;
          else r = __expf(f - s0) * s1;
          o.e[e] = from_f<T>(r);
        }
        st_vec(yr + static_cast<size_t>(p) * E, o);
      }
      __syncthreads();  // every thread has read chunk c: refill it
      if (tid == 0 && next < a.m) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        issue(next, c);
      }
    }
  }
  // A CTA that gave up may leave copies in flight: give them time to land
  // before its shared memory is released (failure path only).
  if (!clean && tid == 0)
    for (int k = 0; k < 2000; ++k) __nanosleep(1000);
}

// tune: threads (a multiple of 32 in [64, 1024], default 512), block_k = chunk
// size in KB (1..64, default 16 KB, doubled until the row has at most 32
// chunks), max_ctas caps the persistent grid (default: every CTA that fits).
template <typename T, int OP>
int launch_rows_cta(const RowArgs& a, const axon_tune_t& t, cudaStream_t s, const char* name) {
  const int64_t row_bytes = a.n * static_cast<int64_t>(sizeof(T));
  if (row_bytes > kCtaMaxRowBytes)
    return fail(AXON_E_UNSUPPORTED, "%s: rows of %lld bytes exceed the CTA bulk variant's %lld", name,
                (long long)row_bytes, (long long)kCtaMaxRowBytes);
  int threads = t.threads > 0 ? t.threads : kCtaThreads;
  if (threads < 64) return fail(AXON_E_ARG, "%s: the CTA bulk variant runs at least 64 threads", name);
  if (t.block_k < 0 || t.block_k > 64) return fail(AXON_E_ARG, "%s: block_k (chunk KB) must be in 1..64", name);
  int64_t chunk = t.block_k > 0 ? static_cast<int64_t>(t.block_k) * 1024 : kCtaChunkBytes;
  if (t.block_k == 0)
    while ((row_bytes + chunk - 1) / chunk > kCtaMaxChunks) chunk *= 2;
  const int64_t nch = (row_bytes + chunk - 1) / chunk;
  if (nch > kCtaMaxChunks)
    return fail(AXON_E_ARG, "%s: %lld chunks of %lld bytes, at most %d", name, (long long)nch, (long long)chunk,
                kCtaMaxChunks);
  if (t.max_ctas < 0) return fail(AXON_E_ARG, "%s: max_ctas must be >= 0", name);
  const size_t smem = static_cast<size_t>(kCtaBarBytes + row_bytes);
  auto kern = row_cta_bulk_kernel<T, OP>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return fail(AXON_E_LAUNCH, "%s: smem attribute: %s", name, cudaGetErrorString(e));
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem);
  if (t.threads == 0 && e == cudaSuccess) {
    // Rows in flight per SM set the pace: take 256 threads where 512 would
    // let fewer rows (CTAs) be resident than shared memory allows. Measured
    // on B200 (graph replay, inputs rotating past L2): layernorm 4096 x 16384
    // bf16 48.7 us at 256 threads (6 CTAs per SM) vs 55.6 at 512 (4); 2048 x
    // 8192 bf16 16.1 vs 20.7; softmax 2048 x 16384 fp32 (3 CTAs per SM
    // either way) 49.3 at 512 vs 54.1; 4096 x 32768 fp32 (one) 211 vs 231.
    int per_sm_256 = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm_256, kern, 256, smem) == cudaSuccess &&
        per_sm_256 > per_sm) {
      threads = 256;
      per_sm = per_sm_256;
    }
  }
  if (e != cudaSuccess || per_sm < 1)
    return fail(AXON_E_LAUNCH, "%s: %d threads with %zu bytes of shared memory do not fit an SM", name, threads, smem);
  int64_t grid = static_cast<int64_t>(sm_count()) * per_sm;
  if (t.max_ctas > 0 && grid > t.max_ctas) grid = t.max_ctas;
  if (grid > a.m) grid = a.m;
  launch_k(kern, dim3(static_cast<unsigned>(grid)), dim3(threads), smem, s, a, static_cast<uint32_t>(row_bytes),
           static_cast<uint32_t>(chunk), static_cast<int>(nch));
  return launch_status(name);
}

template <typename T, int OP>
int launch_rows_bulk(const RowArgs& a, const axon_tune_t& t, cudaStream_t s, const char* name) {
  const int64_t row_bytes = a.n * static_cast<int64_t>(sizeof(T));
  const bool has_w = OP == OP_RMS && a.w != nullptr;
  const int sms = sm_count();
  const int64_t fixed = has_w ? row_bytes : 0;
  constexpr int64_t kBarBytes = 512;  // the kernel's mbarrier block: 32 warps x 2 slots
  int warps, slots;
  if (t.threads > 0) {
    // explicit CTA size: double-buffer each warp's rows when two slots fit
    warps = t.threads / 32;
    slots = 2;
    while (slots > 1 && kBarBytes + fixed + static_cast<int64_t>(warps) * slots * row_bytes > kBulkSmemBudget)
      --slots;
  } else {
    // One row per warp, about 128 KB of rows per CTA (16 warps of 8 KB rows,
    // 8 of 16 KB), fewer warps when there are few rows per SM. Measured on
    // B200 (CUDA graph, inputs rotating past L2): rmsnorm 2048 x 4096 bf16
    // 8.2 us at 16 warps vs 8.5 at 14 and 9.9 at 12; layernorm 2048 x 8192
    // 18.2 us at 8 warps vs 19.7 with persistent double-buffered warps.
    slots = 1;
    int64_t cap = (kBulkTargetBytes - fixed) / row_bytes;
    cap = cap < 1 ? 1 : cap > 16 ? 16 : cap;
    const int64_t per_sm = (a.m + sms - 1) / sms;
    warps = static_cast<int>(per_sm * 2 >= cap ? cap : per_sm);
  }
  if (warps < 1) return fail(AXON_E_UNSUPPORTED, "%s: rows of %lld bytes do not fit the bulk variant", name,
                             (long long)row_bytes);
  const size_t smem = kBarBytes + fixed + static_cast<size_t>(warps) * slots * row_bytes;
  if (smem > 232448) return fail(AXON_E_ARG, "%s: %d threads need %zu bytes of shared memory", name, warps * 32, smem);
  const int64_t per_cta = warps;
  int64_t grid = (a.m + per_cta - 1) / per_cta;
  if (slots == 2 && grid > sms) grid = sms;
  if (grid > 0x7fffffff) return fail(AXON_E_SHAPE, "%s: too many rows (%lld)", name, (long long)a.m);
  auto kern = row_bulk_kernel<T, OP>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return fail(AXON_E_LAUNCH, "%s: smem attribute: %s", name, cudaGetErrorString(e));
  launch_k(kern, dim3(static_cast<unsigned>(grid)), dim3(warps * 32), smem, s, a, slots,
           static_cast<uint32_t>(row_bytes));
  return launch_status(name);
}

template <typename T, int OP>
int launch_rows(const RowArgs& a, const axon_tune_t& t, cudaStream_t s, const char* name) {
  constexpr int E = Vec<T>::E;
  if (a.m == 0 || a.n == 0) return AXON_OK;
  constexpr int32_t kCode = sizeof(T) == 4 ? AXON_F32 : std::is_same<T, __half>::value ? AXON_F16 : AXON_BF16;
  const bool w_ok = a.w == nullptr || (a.w_dtype == kCode && aligned16(a.w));
  const bool vec_ok = aligned16(a.x) && (a.ld_x * sizeof(T)) % 16 == 0 && w_ok &&
                      (OP == OP_RSQRT || (aligned16(a.y) && (a.ld_y * sizeof(T)) % 16 == 0));
  const int64_t nv = (a.n + E - 1) / E;
  const int64_t row_bytes = a.n * static_cast<int64_t>(sizeof(T));
  const bool bulk_ok = vec_ok && row_bytes % 16 == 0 && row_bytes <= kBulkMaxRowBytes;
  // Default (variant 0, no thread count), once there is at least a row per
  // SM: rows of 16 KB up to the shared-memory limit run the CTA-per-row bulk
  // kernel (variant 3), shorter rows the bulk warp-per-row kernel (variant 2).
  // Measured on B200 against the previous defaults: softmax 4096 x 32768 fp32
  // 211 vs 261 us (register-resident), layernorm 4096 x 16384 bf16 48.7 vs
  // 73.8 us and 2048 x 8192 bf16 16.1 vs 18.3 us (warp per row); at 8 KB rows
  // the warp-per-row kernel stays ahead (rmsnorm 2048 x 4096 bf16 8.5 vs 9.5
  // us). The warp-per-row kernel beat the register-resident one on every
  // measured shape it takes (softmax 16384 x 4096 bf16: 62 vs 111 us).
  if constexpr (OP != OP_RSQRT) {
    if (t.variant == 0 && t.threads == 0 && vec_ok && row_bytes % 16 == 0 && row_bytes >= kCtaDefaultMinRowBytes &&
        row_bytes <= kCtaMaxRowBytes && a.m >= sm_count())
      return launch_rows_cta<T, OP>(a, t, s, name);
  }
  if (t.variant == 0 && t.threads == 0 && bulk_ok && a.m >= sm_count()) return launch_rows_bulk<T, OP>(a, t, s, name);
  if (t.variant == 2) {
    if (!bulk_ok)
      return fail(AXON_E_UNSUPPORTED,
                  "%s: the bulk variant needs 16-byte aligned rows of a multiple of 16 bytes, at most %d bytes",
                  name, kBulkMaxRowBytes);
    return launch_rows_bulk<T, OP>(a, t, s, name);
  }
  if (t.variant == 3) {
    if constexpr (OP == OP_RSQRT) {
      return fail(AXON_E_UNSUPPORTED, "%s: no CTA bulk variant", name);
    } else {
      if (!vec_ok || row_bytes % 16 || row_bytes > kCtaMaxRowBytes)
        return fail(AXON_E_UNSUPPORTED,
                    "%s: the CTA bulk variant needs 16-byte aligned rows of a multiple of 16 bytes, at most %lld "
                    "bytes",
                    name, (long long)kCtaMaxRowBytes);
      return launch_rows_cta<T, OP>(a, t, s, name);
    }
  }
  int tpr = 0, vpt = 0;
  if (t.variant == 0 && vec_ok) {
    if (t.threads > 0) {
      tpr = t.threads;
      if (tpr > max_row_threads<T>())
        return fail(AXON_E_ARG, "%s: at most %d threads per row for this dtype", name, max_row_threads<T>());
    } else {
      // About two 16-byte packets per thread with up to 256 threads per row,
      // wider rows only when a thread would otherwise hold more than eight
      // packets. Measured on B200: rmsnorm 2048x4096 bf16 8.8 us at 256
      // threads (2 packets) vs 9.8 at 128 and 12.0 at 512; layernorm
      // 2048x8192 bf16 best at 256 threads (4 packets).
      tpr = 32;
      while (tpr < 256 && tpr < max_row_threads<T>() && (nv + tpr - 1) / tpr > 2) tpr *= 2;
      while (tpr < max_row_threads<T>() && (nv + tpr - 1) / tpr > 8) tpr *= 2;
    }
    int64_t need = (nv + tpr - 1) / tpr;
    vpt = need <= 1 ? 1 : need <= 2 ? 2 : need <= 4 ? 4 : need <= 8 ? 8 : 0;
  }
  if (vpt > 0) {
    const int gw = tpr / 32;
    const int rows_per_cta = tpr >= 128 ? 1 : 128 / tpr;
    const int64_t grid = (a.m + rows_per_cta - 1) / rows_per_cta;
    if (grid > 0x7fffffff) return fail(AXON_E_SHAPE, "%s: too many rows (%lld)", name, (long long)a.m);
    dim3 block(tpr * rows_per_cta);
    switch (vpt) {
      case 1: launch_k(row_resident_kernel<T, 1, OP>, dim3(grid), block, 0, s, a, gw, rows_per_cta); break;
      case 2: launch_k(row_resident_kernel<T, 2, OP>, dim3(grid), block, 0, s, a, gw, rows_per_cta); break;
      case 4: launch_k(row_resident_kernel<T, 4, OP>, dim3(grid), block, 0, s, a, gw, rows_per_cta); break;
      default: launch_k(row_resident_kernel<T, 8, OP>, dim3(grid), block, 0, s, a, gw, rows_per_cta); break;
    }
    return launch_status(name);
  }
  if (a.m > 0x7fffffff) return fail(AXON_E_SHAPE, "%s: too many rows (%lld)", name, (long long)a.m);
  int threads = t.threads > 0 ? t.threads : 1024;
  if (vec_ok)
    launch_k(row_streaming_kernel<T, true, OP>, dim3(a.m), dim3(threads), 0, s, a);
  else
    launch_k(row_streaming_kernel<T, false, OP>, dim3(a.m), dim3(threads), 0, s, a);
  return launch_status(name);
}

template <int OP>
int dispatch_rows(const RowArgs& a, int32_t dtype, const axon_tune_t* tune, void* stream, const char* name) {
  axon_tune_t t = tune_or_default(tune);
  if (t.variant < 0 || t.variant > 3) return fail(AXON_E_ARG, "%s: unknown variant %d", name, t.variant);
  if (t.variant >= 2 && t.threads != 0 && (t.threads < 32 || t.threads > 1024 || t.threads % 32))
    return fail(AXON_E_ARG, "%s: threads must be a multiple of 32 in [32, 1024], got %d", name, t.threads);
  if (t.variant < 2 && t.threads != 0 && (t.threads < 32 || t.threads > 1024 || (t.threads & (t.threads - 1))))
    return fail(AXON_E_ARG, "%s: threads must be a power of two in [32, 1024], got %d", name, t.threads);
  if (a.m < 0 || a.n < 0) return fail(AXON_E_SHAPE, "%s: negative size", name);
  if (a.ld_x < a.n || (OP != OP_RSQRT && a.ld_y < a.n))
    return fail(AXON_E_SHAPE, "%s: leading dimension smaller than n", name);
  if (a.m == 0 || a.n == 0) return AXON_OK;  // empty tensors may carry NULL pointers
  if (a.x == nullptr || (OP != OP_RSQRT && a.y == nullptr) || (OP == OP_RSQRT && a.r_out == nullptr))
    return fail(AXON_E_ARG, "%s: NULL tensor pointer", name);
  cudaStream_t s = as_stream(stream);
  switch (dtype) {
    case AXON_F32: return launch_rows<float, OP>(a, t, s, name);
    case AXON_BF16: return launch_rows<__nv_bfloat16, OP>(a, t, s, name);
    case AXON_F16: return launch_rows<__half, OP>(a, t, s, name);
    default: return fail(AXON_E_UNSUPPORTED, "%s: unsupported dtype %d", name, dtype);
  }
}

}  // namespace
}  // namespace axon

using namespace axon;

extern "C" int axon_rmsnorm(const void* x, const void* w, void* y, int64_t m, int64_t n, int64_t ld_x,
                            int64_t ld_y, int32_t dtype, int32_t w_dtype, float scale, float eps,
                            const axon_tune_t* tune, void* stream) {
  if (w != nullptr && !valid_dtype(w_dtype)) return fail(AXON_E_UNSUPPORTED, "axon_rmsnorm: bad weight dtype %d", w_dtype);
  RowArgs a{x, y, w, nullptr, m, n, ld_x, ld_y, w_dtype, scale, eps};
  return dispatch_rows<OP_RMS>(a, dtype, tune, stream, "axon_rmsnorm");
}

extern "C" int axon_layernorm(const void* x, void* y, int64_t m, int64_t n, int64_t ld_x, int64_t ld_y,
                              int32_t dtype, float eps, const axon_tune_t* tune, void* stream) {
  RowArgs a{x, y, nullptr, nullptr, m, n, ld_x, ld_y, 0, 1.f, eps};
  return dispatch_rows<OP_LN>(a, dtype, tune, stream, "axon_layernorm");
}

extern "C" int axon_softmax(const void* x, void* y, int64_t m, int64_t n, int64_t ld_x, int64_t ld_y,
                            int32_t dtype, const axon_tune_t* tune, void* stream) {
  RowArgs a{x, y, nullptr, nullptr, m, n, ld_x, ld_y, 0, 1.f, 0.f};
  return dispatch_rows<OP_SM>(a, dtype, tune, stream, "axon_softmax");
}

extern "C" int axon_row_status(void* stream) {
  int v = 0;
  cudaStream_t s = as_stream(stream);
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_row_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return fail(AXON_E_CUDA, "axon_row_status: %s", cudaGetErrorString(e));
  if (v != 0) {
    int zero = 0;
    cudaMemcpyToSymbolAsync(g_row_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
    cudaStreamSynchronize(s);
    return fail(v, "row kernel: a bulk-copy wait gave up (status %d)", v);
  }
  return AXON_OK;
}

extern "C" int axon_row_rsqrt(const void* x, float* r, int64_t m, int64_t n, int64_t ld_x, int32_t dtype,
                              float scale, float eps, void* stream) {
  RowArgs a{x, nullptr, nullptr, r, m, n, ld_x, 0, 0, scale, eps};
  return dispatch_rows<OP_RSQRT>(a, dtype, nullptr, stream, "axon_row_rsqrt");
}
