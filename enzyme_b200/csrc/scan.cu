// Inclusive prefix sum along the last axis (Axon kernels/cumsum/refs.py:20-22).
//
// Variant 0 -- single-pass decoupled look-back (Merrill & Garland, "Single-pass
// Parallel Prefix Scan with Decoupled Look-back", NVIDIA TR 2016). Each CTA
// takes the next tile id from an atomic counter, so a tile's predecessors in
// its row were always claimed by CTAs that are already running; it scans its
// tile in registers (warp-striped 16-byte packets: packet-serial, then warp
// shuffles per segment, then across warps),
// publishes the tile aggregate, looks back over predecessor descriptors with
// one warp until it meets an inclusive prefix, publishes its own inclusive
// prefix and writes the tile. Every input byte is read once and every output
// byte written once. Tile sums and carries are float64, so the error of an
// element is a few fp32 roundings regardless of the row length. Every wait on
// a predecessor is bounded: a wait that gives up records AXON_E_TIMEOUT in the
// workspace status word and the CTA finishes (with a wrong prefix) rather than
// spinning forever.
//
// Variant 1 -- one thread-block cluster per row (2..8 CTAs, or one CTA for
// short rows). Each CTA pulls its contiguous chunk of the row (at most 64 KB
// at the automatic cluster size) into shared memory with 1-D bulk copies
// (cp.async.bulk, no multicast), sums it warp by warp, and the chunk sums are
// exchanged through distributed shared memory between two hardware cluster
// barriers; each CTA then scans its chunk from shared memory and writes it
// out. No global flags, no atomics and no scratch memory; the barrier cannot
// hang because every CTA of a cluster is co-scheduled and runs the same path.
// The only wait on memory, the bulk copy's mbarrier, is bounded and records
// AXON_E_TIMEOUT in a device status word (axon_cumsum_status with a NULL
// workspace reads it).
#include <cooperative_groups.h>

#include "common.cuh"
#include "sm100.cuh"

namespace axon {

__device__ int g_scan_error;

namespace {

struct alignas(32) TileDesc {
  unsigned flag;  // 0 = empty, 1 = aggregate ready, 2 = inclusive prefix ready
  unsigned pad;
  double agg;
  double incl;
  double pad2;
};

constexpr int64_t kHeaderBytes = 32;  // int status, unsigned counter, padding
constexpr long long kSpinLimit = 1ll << 22;

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Warp-striped tile layout: warp w of the CTA owns the ITEMS*32 contiguous
// elements starting at w*ITEMS*32 of the tile, split into S = ITEMS/E
// segments of 32 packets; lane l holds packet l of every segment. Every warp
// load or store instruction therefore touches 32 consecutive 16-byte packets.
template <typename Tin, int ITEMS>
__device__ __forceinline__ void load_striped(const Tin* row, int64_t wbase, int lane, int64_t n, bool vec,
                                             float* v) {
  constexpr int E = Vec<Tin>::E;
#pragma unroll
  for (int sgi = 0; sgi < ITEMS / E; ++sgi) {
    const int64_t col = wbase + (static_cast<int64_t>(sgi) * 32 + lane) * E;
    if (vec && col + E <= n) {
      Vec<Tin> p = ld_vec_stream(row + col);
#pragma unroll
      for (int e = 0; e < E; ++e) v[sgi * E + e] = to_f(p.e[e]);
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) v[sgi * E + e] = col + e < n ? to_f(row[col + e]) : 0.f;
    }
  }
}

template <typename Tin, typename Tout, int ITEMS>
__device__ __forceinline__ void store_striped(Tout* row, int64_t wbase, int lane, int64_t n, bool vec,
                                              const float* v) {
  constexpr int E = Vec<Tin>::E;  // same packet geometry as the loads
#pragma unroll
  for (int sgi = 0; sgi < ITEMS / E; ++sgi) {
    const int64_t col = wbase + (static_cast<int64_t>(sgi) * 32 + lane) * E;
    if (vec && col + E <= n && (sizeof(Tout) * E) % 16 == 0) {
#pragma unroll
      for (int h = 0; h < E; h += Vec<Tout>::E) {
        Vec<Tout> p;
#pragma unroll
        for (int e = 0; e < Vec<Tout>::E; ++e) p.e[e] = from_f<Tout>(v[sgi * E + h + e]);
        st_vec_stream(row + col + h, p);
      }
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e)
        if (col + e < n) row[col + e] = from_f<Tout>(v[sgi * E + e]);
    }
  }
}

template <typename Tin, typename Tout, int ITEMS>
__global__ void __launch_bounds__(1024) cumsum_lookback(const Tin* __restrict__ x, Tout* __restrict__ y,
                                                        int64_t n, int64_t ld_x, int64_t ld_y,
                                                        int64_t tiles_per_row, bool vec, unsigned char* ws) {
  constexpr int E = Vec<Tin>::E;
  constexpr int SEG = ITEMS / E;
  __shared__ unsigned s_tile;
  __shared__ float s_warp[32];
  __shared__ double s_prefix;
  int* status = reinterpret_cast<int*>(ws);
  unsigned* counter = reinterpret_cast<unsigned*>(ws + 4);
  TileDesc* desc = reinterpret_cast<TileDesc*>(ws + kHeaderBytes);

  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  if (tid == 0) s_tile = atomicAdd(counter, 1u);
  __syncthreads();
  const int64_t t = s_tile;
  const int64_t row = t / tiles_per_row;
  const int64_t tr = t - row * tiles_per_row;
  const int64_t tile_elems = static_cast<int64_t>(blockDim.x) * ITEMS;
  const int64_t wbase = tr * tile_elems + static_cast<int64_t>(warp) * ITEMS * 32;
  const Tin* xr = x + row * ld_x;
  Tout* yr = y + row * ld_y;

  float v[ITEMS];
  load_striped<Tin, ITEMS>(xr, wbase, lane, n, vec, v);
  // Per segment: scan the lane's packet, then across lanes; `carry` runs over
  // the warp's segments in order.
  float carry = 0.f;
#pragma unroll
  for (int sg = 0; sg < SEG; ++sg) {
#pragma unroll
    for (int e = 1; e < E; ++e) v[sg * E + e] += v[sg * E + e - 1];
    const float own = v[sg * E + E - 1];
    float incl = own;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float up = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += up;
    }
    const float base = carry + (incl - own);
#pragma unroll
    for (int e = 0; e < E; ++e) v[sg * E + e] += base;
    carry += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) s_warp[warp] = carry;
  __syncthreads();
  if (warp == 0) {
    float w = lane < nwarps ? s_warp[lane] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float up = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += up;
    }
    if (lane < nwarps) s_warp[lane] = w;
  }
  __syncthreads();
  const float warp_excl = warp > 0 ? s_warp[warp - 1] : 0.f;
  const double tile_agg = static_cast<double>(s_warp[nwarps - 1]);

  if (warp == 0) {
    double prefix = 0.0;
    if (tr == 0) {
      if (lane == 0) {
        desc[t].incl = tile_agg;
        st_release(&desc[t].flag, 2u);
      }
    } else {
      if (lane == 0) {
        desc[t].agg = tile_agg;
        st_release(&desc[t].flag, 1u);
      }
      const int64_t first = t - tr;
      int64_t base = t - 1;
      long long spins = 0;
      bool timed_out = false;
      while (true) {
        const int64_t idx = base - lane;
        const unsigned f = idx >= first ? ld_acquire(&desc[idx].flag) : 2u;
        const unsigned pmask = __ballot_sync(0xffffffffu, f == 2u);
        const unsigned zmask = __ballot_sync(0xffffffffu, f == 0u);
        const int plane = pmask ? __ffs(pmask) - 1 : 32;
        const unsigned need = plane >= 31 ? 0xffffffffu : ((2u << plane) - 1u);
        if ((zmask & need) && !timed_out) {
          if (++spins > kSpinLimit) {
            timed_out = true;
            // recorded in the workspace header and in the library's device
            // status word: the allocation-free entry point's scratch is
            // cleared by the next call, so only the latter survives for it
            if (lane == 0) {
              atomicExch(status, AXON_E_TIMEOUT);
              atomicExch(&g_scan_error, AXON_E_TIMEOUT);
            }
          } else {
            __nanosleep(spins < 64 ? 32 : 256);
          }
          continue;
        }
        double c = 0.0;
        if (idx >= first && f != 0u) {
          if (lane < plane) c = desc[idx].agg;
          else if (lane == plane) c = desc[idx].incl;
        }
        prefix += warp_sum_d(c);
        if (plane < 32) break;
        base -= 32;
        if (base < first) break;
      }
      if (lane == 0) {
        desc[t].incl = prefix + tile_agg;
        st_release(&desc[t].flag, 2u);
      }
    }
    if (lane == 0) s_prefix = prefix;
  }
  __syncthreads();
  const double p = s_prefix;
#pragma unroll
  for (int j = 0; j < ITEMS; ++j) v[j] = static_cast<float>(p + static_cast<double>(warp_excl + v[j]));
  store_striped<Tin, Tout, ITEMS>(yr, wbase, lane, n, vec, v);
}

// ---- variant 1: cluster scan ------------------------------------------------------

constexpr int kClusterThreads = 512;
constexpr int64_t kChunkTargetBytes = 64 * 1024;
constexpr int64_t kChunkMaxBytes = 200 * 1024;
constexpr uint64_t kBulkWaitNs = 2000000000ull;

// Store E consecutive outputs (the first `valid` of them) at dst.
template <typename Tout, int E>
__device__ __forceinline__ void store_packet(Tout* dst, const float* v, int64_t valid, bool vec) {
  if (vec && valid >= E) {
    if constexpr (sizeof(Tout) * E >= 16) {
#pragma unroll
      for (int h = 0; h < E; h += Vec<Tout>::E) {
        Vec<Tout> p;
#pragma unroll
        for (int e = 0; e < Vec<Tout>::E; ++e) p.e[e] = from_f<Tout>(v[h + e]);
        st_vec_stream(dst + h, p);
      }
      return;
    } else if constexpr (sizeof(Tout) * E == 8) {
      union {
        uint2 u;
        Tout e[E];
      } p;
#pragma unroll
      for (int e = 0; e < E; ++e) p.e[e] = from_f<Tout>(v[e]);
      *reinterpret_cast<uint2*>(dst) = p.u;
      return;
    }
  }
#pragma unroll
  for (int e = 0; e < E; ++e)
    if (e < valid) dst[e] = from_f<Tout>(v[e]);
}

template <typename Tin, typename Tout>
__global__ void __launch_bounds__(kClusterThreads) cumsum_cluster(const Tin* __restrict__ x, Tout* __restrict__ y,
                                                                  int64_t n, int64_t ld_x, int64_t ld_y,
                                                                  int64_t chunk, int csize, bool vec) {
  namespace cg = cooperative_groups;
  constexpr int E = Vec<Tin>::E;
  extern __shared__ __align__(128) unsigned char dyn_smem[];
  Tin* buf = reinterpret_cast<Tin*>(dyn_smem);
  __shared__ __align__(8) uint64_t bar;
  __shared__ float s_warp[32];
  __shared__ double s_total;
  __shared__ double s_prefix;

  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int64_t row = blockIdx.x / csize;
  const int64_t c0 = static_cast<int64_t>(rank) * chunk;
  const int64_t len = c0 < n ? (chunk < n - c0 ? chunk : n - c0) : 0;
  const Tin* src = x + row * ld_x + c0;
  Tout* dst = y + row * ld_y + c0;

  pdl_wait();
  pdl_trigger();
  // 1. chunk -> shared memory: bulk copies for the 16-byte-aligned body,
  // plain loads for a ragged tail
  const int64_t bulk = vec ? (len * static_cast<int64_t>(sizeof(Tin))) / 16 * 16 : 0;
  if (tid == 0) {
    sm100::mbar_init(&bar, 1);
    sm100::mbar_init_fence();
  }
  __syncthreads();
  if (tid == 0 && bulk > 0) {
    sm100::mbar_expect_tx(&bar, static_cast<uint32_t>(bulk));
    constexpr int64_t kPiece = 32768;
    for (int64_t off = 0; off < bulk; off += kPiece) {
      const int64_t b = bulk - off < kPiece ? bulk - off : kPiece;
      sm100::bulk_g2s(dyn_smem + off, reinterpret_cast<const unsigned char*>(src) + off, static_cast<uint32_t>(b),
                      &bar);
    }
  }
  for (int64_t i = bulk / static_cast<int64_t>(sizeof(Tin)) + tid; i < len; i += blockDim.x) buf[i] = src[i];
  if (bulk > 0 && !sm100::mbar_wait_bounded(&bar, 0, kBulkWaitNs)) {
    if (tid == 0) atomicExch(&g_scan_error, AXON_E_TIMEOUT);
    sm100::mbar_wait_bounded(&bar, 0, kBulkWaitNs);  // second bound for copies still in flight
  }
  __syncthreads();

  // 2. warp sums over warp-striped packets of E elements
  const int64_t packets = (len + E - 1) / E;
  const int64_t ppw = ((packets + nwarps - 1) / nwarps + 31) / 32 * 32;  // packets per warp, whole segments
  const int64_t wp0 = static_cast<int64_t>(warp) * ppw;
  auto load = [&](int64_t pk, float* v) {
    const int64_t e0 = pk * E;
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = (pk < packets && e0 + e < len) ? to_f(buf[e0 + e]) : 0.f;
  };
  float wsum = 0.f;
  for (int64_t j = 0; j < ppw; j += 32) {
    float v[E];
    load(wp0 + j + lane, v);
#pragma unroll
    for (int e = 0; e < E; ++e) wsum += v[e];
  }
  wsum = warp_sum(wsum);
  if (lane == 0) s_warp[warp] = wsum;
  __syncthreads();
  if (warp == 0) {
    float w = lane < nwarps ? s_warp[lane] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float up = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += up;
    }
    if (lane < nwarps) s_warp[lane] = w;
  }
  __syncthreads();
  const float warp_excl = warp > 0 ? s_warp[warp - 1] : 0.f;

  // 3. chunk sums across the cluster through distributed shared memory
  if (tid == 0) s_total = static_cast<double>(s_warp[nwarps - 1]);
  cluster.sync();
  if (tid == 0) {
    double p = 0.0;
    for (int r = 0; r < rank; ++r) p += *cluster.map_shared_rank(&s_total, r);
    s_prefix = p;
  }
  cluster.sync();  // also keeps every CTA's s_total alive until all reads are done
  const double prefix = s_prefix;

  // 4. scan the chunk from shared memory and write it out
  float carry = warp_excl;
  for (int64_t j = 0; j < ppw; j += 32) {
    const int64_t pk = wp0 + j + lane;
    float v[E];
    load(pk, v);
#pragma unroll
    for (int e = 1; e < E; ++e) v[e] += v[e - 1];
    const float own = v[E - 1];
    float incl = own;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float up = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += up;
    }
    const float base = carry + (incl - own);
    float out[E];
#pragma unroll
    for (int e = 0; e < E; ++e) out[e] = static_cast<float>(prefix + static_cast<double>(base + v[e]));
    if (pk < packets) store_packet<Tout, E>(dst + pk * E, out, len - pk * E, vec);
    carry += __shfl_sync(0xffffffffu, incl, 31);
  }
}

// Cluster size and chunk for a row of n elements of `size` bytes: the
// smallest power of two (at most 8) whose chunks fit the 64 KB target, chunks
// a multiple of 8 elements so every CTA's slice starts 16-byte aligned.
bool cluster_shape(int64_t n, int size, int want, int& csize, int64_t& chunk) {
  csize = want;
  if (csize == 0) {
    csize = 1;
    while (csize < 8 && (n + csize - 1) / csize * size > kChunkTargetBytes) csize *= 2;
  }
  chunk = ((n + csize - 1) / csize + 7) / 8 * 8;
  return chunk * size <= kChunkMaxBytes;
}

template <typename Tin, typename Tout>
int launch_cluster(const void* x, void* y, int64_t m, int64_t n, int64_t ld_x, int64_t ld_y, const axon_tune_t& t,
                   cudaStream_t s) {
  int csize;
  int64_t chunk;
  if (!cluster_shape(n, sizeof(Tin), t.split, csize, chunk))
    return fail(AXON_E_SHAPE, "axon_cumsum: rows of %lld elements are too long for the cluster variant (use 0)",
                (long long)n);
  if (m * csize > 0x7fffffffLL) return fail(AXON_E_SHAPE, "axon_cumsum: too many rows (%lld)", (long long)m);
  const bool vec = aligned16(x) && aligned16(y) && (ld_x * sizeof(Tin)) % 16 == 0 && (ld_y * sizeof(Tout)) % 16 == 0;
  const size_t smem = static_cast<size_t>(chunk) * sizeof(Tin);
  auto kern = cumsum_cluster<Tin, Tout>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return fail(AXON_E_LAUNCH, "axon_cumsum: smem attribute: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(m * csize));
  cfg.blockDim = dim3(kClusterThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = csize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  e = cudaLaunchKernelEx(&cfg, kern, static_cast<const Tin*>(x), static_cast<Tout*>(y), n, ld_x, ld_y, chunk, csize,
                         vec);
  if (e != cudaSuccess) return fail(AXON_E_LAUNCH, "axon_cumsum: cluster launch failed: %s", cudaGetErrorString(e));
  return launch_status("axon_cumsum");
}

// ---- variant 2: one CTA streams a whole row --------------------------------------
//
// Rows are independent, so a CTA can own a row and walk it chunk by chunk
// with the running sum in a register: no flags, no cluster barriers, no
// scratch. Chunks (24 KB by default) arrive in a ring of shared-memory
// stages by 1-D bulk copies; a stage is refilled as soon as
// its chunk has moved into registers, so up to `stages` chunks are in flight
// per CTA, and two CTAs share an SM (the nucleus config's 256 rows all run at
// once on 148 SMs). Per chunk: packets into registers and warp sums
// (warp-striped packets), one CTA exchange of the warp sums, then a shuffle
// scan per 32-packet segment written out with streaming stores. The running
// row sum is float64.
constexpr int kRowThreads = 512;
constexpr int kRowMaxStages = 8;
constexpr int kRowStageBytes = 32768;  // default chunk: 8192 fp32 or 16384 bf16 elements
constexpr int kRowStages = 2;          // default ring depth
constexpr int64_t kRowStreamMinRows = 128;

// NW warps; `stages` chunks of SKB KB (a multiple of NW / 2 KB, so every
// warp owns whole 32-packet segments of a chunk).
// A segment is 32 * K consecutive packets of a warp's range, lane l holding
// packets l*K .. l*K + K - 1 of it: one shuffle scan covers K packets.
template <typename Tin, typename Tout, int NW, int SKB, int KREQ>
__global__ void __launch_bounds__(NW * 32, 2) cumsum_rowstream(const Tin* __restrict__ x, Tout* __restrict__ y,
                                                               int64_t n, int64_t ld_x, int64_t ld_y, bool vec_out,
                                                               int stages, int* ws_status) {
  constexpr int E = Vec<Tin>::E;
  constexpr int64_t kRowChunk = SKB * 1024 / static_cast<int64_t>(sizeof(Tin));
  constexpr int64_t PPW = kRowChunk / E / NW;  // packets per warp per chunk
  constexpr int K = PPW % (32 * KREQ) == 0 ? KREQ : 1;  // whole segments per warp
  static_assert(PPW % 32 == 0, "whole segments per warp");
  const int kRowStages = stages;
  extern __shared__ __align__(128) unsigned char dyn_smem[];
  __shared__ __align__(8) uint64_t full[kRowMaxStages];
  __shared__ float s_warp[2][NW];
  __shared__ int s_abort;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row = blockIdx.x;
  const Tin* src = x + row * ld_x;
  Tout* dst = y + row * ld_y;
  const int64_t nchunks = (n + kRowChunk - 1) / kRowChunk;
  constexpr int64_t kStageBytes = SKB * 1024;

  // chunk c: elements [c * kRowChunk, +len); the 16-byte multiple of its bytes
  // comes by bulk copy, a ragged tail (< 16 bytes) is read from global memory
  auto chunk_len = [&](int64_t c) { return n - c * kRowChunk < kRowChunk ? n - c * kRowChunk : kRowChunk; };
  auto issue = [&](int64_t c) {
    const int st = static_cast<int>(c % kRowStages);
    const uint32_t bytes = static_cast<uint32_t>(chunk_len(c) * static_cast<int64_t>(sizeof(Tin)) / 16 * 16);
    if (bytes == 0) {
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sm100::smem_addr(&full[st])) : "memory");
      return;
    }
    sm100::mbar_expect_tx(&full[st], bytes);
    sm100::bulk_g2s(dyn_smem + st * kStageBytes, src + c * kRowChunk, bytes, &full[st]);
  };

  if (tid == 0) {
    for (int st = 0; st < kRowStages; ++st) sm100::mbar_init(&full[st], 1);
    s_abort = 0;
    sm100::mbar_init_fence();
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  // a caller workspace, if any, reports OK (waits that give up go to g_scan_error)
  if (ws_status != nullptr && row == 0 && tid == 0) *ws_status = AXON_OK;
  if (tid == 0)
    for (int64_t c = 0; c < nchunks && c < kRowStages; ++c) issue(c);

  double carry = 0.0;
  for (int64_t c = 0; c < nchunks; ++c) {
    const int st = static_cast<int>(c % kRowStages);
    const int b = static_cast<int>(c & 1);
    const int64_t len = chunk_len(c);
    const int64_t bulk_elems = len * static_cast<int64_t>(sizeof(Tin)) / 16 * 16 / static_cast<int64_t>(sizeof(Tin));
    const Tin* buf = reinterpret_cast<const Tin*>(dyn_smem + st * kStageBytes);
    const Tin* gsrc = src + c * kRowChunk;
    if (!s_abort && !sm100::mbar_wait_bounded(&full[st], static_cast<uint32_t>((c / kRowStages) & 1), kBulkWaitNs)) {
      s_abort = 1;
      atomicExch(&g_scan_error, AXON_E_TIMEOUT);
    }
    // pass 1: this thread's packets -> registers, and the warp sums. Full
    // chunks (all but a row's last) take a path with no bounds checks.
    constexpr int NSEG = static_cast<int>(PPW / (32 * K));
    const bool full_chunk = len == kRowChunk;
    const int wbase = warp * static_cast<int>(PPW) + lane * K;  // this lane's first packet
    Vec<Tin> raw[NSEG * K];
    float wsum = 0.f;
#pragma unroll
    for (int q = 0; q < NSEG * K; ++q) {
      const int e0 = (wbase + (q / K) * 32 * K + q % K) * E;
      if (full_chunk || e0 + E <= bulk_elems) {
        raw[q] = *reinterpret_cast<const Vec<Tin>*>(buf + e0);
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const int64_t i = e0 + e;
          raw[q].e[e] = i < bulk_elems ? buf[i] : i < len ? gsrc[i] : from_f<Tin>(0.f);
        }
      }
#pragma unroll
      for (int e = 0; e < E; ++e) wsum += to_f(raw[q].e[e]);
    }
    wsum = warp_sum(wsum);
    if (lane == 0) s_warp[b][warp] = wsum;
    __syncthreads();
    // the chunk is in registers: its stage takes chunk c + stages right away
    if (tid == 0 && c + kRowStages < nchunks) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(c + kRowStages);
    }
    // every warp scans the NW warp sums itself (no second CTA barrier)
    float wi = lane < NW ? s_warp[b][lane] : 0.f;
#pragma unroll
    for (int o = 1; o < NW; o <<= 1) {
      const float up = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += up;
    }
    const float chunk_total = __shfl_sync(0xffffffffu, wi, NW - 1);
    const float warp_excl = __shfl_sync(0xffffffffu, wi, warp > 0 ? warp - 1 : 0);
    // The row's running sum is float64 across chunks; an output is
    // (float)carry + its chunk-local fp32 prefix: two roundings at the
    // output's magnitude, the rest at the (smaller) chunk-local one.
    const float carry_f = static_cast<float>(carry);
    float seg_carry = warp > 0 ? warp_excl : 0.f;
    // pass 2: scan 32-packet segments and write them out
    Tout* cdst = dst + c * kRowChunk;
#pragma unroll
    for (int j = 0; j < NSEG; ++j) {
      const int e0 = (wbase + j * 32 * K) * E;
      float v[K * E];
#pragma unroll
      for (int q = 0; q < K * E; ++q) v[q] = to_f(raw[j * K + q / E].e[q % E]);
#pragma unroll
      for (int q = 1; q < K * E; ++q) v[q] += v[q - 1];
      const float own = v[K * E - 1];
      float incl = own;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float up = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += up;
      }
      const float base = seg_carry + (incl - own);
#pragma unroll
      for (int q = 0; q < K * E; ++q) v[q] = carry_f + (base + v[q]);
#pragma unroll
      for (int k = 0; k < K; ++k) {
        if (full_chunk) store_packet<Tout, E>(cdst + e0 + k * E, v + k * E, E, vec_out);
        else if (e0 + k * E < len) store_packet<Tout, E>(cdst + e0 + k * E, v + k * E, len - e0 - k * E, vec_out);
      }
      seg_carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    carry += static_cast<double>(chunk_total);
  }
  // copies may still be landing only if a wait gave up: let them finish
  // before the CTA's shared memory is released (failure path only)
  if (tid == 0 && s_abort)
    for (int k = 0; k < 2000; ++k) __nanosleep(1000);
}

// tune: stages 2..8 (default 2), block_k = stage size in KB: 16, 24, 32
// (default) or 48; stages x block_k at most 200 KB. Measured on B200 at
// 256 x 128256 fp32: 51.2 us at 2 x 32 KB, 52.1 at 3 x 24, 53.7 at 4 x 16.
template <typename Tin, typename Tout>
int launch_rowstream(const void* x, void* y, int64_t m, int64_t n, int64_t ld_x, int64_t ld_y,
                     const axon_tune_t& t, void* ws, cudaStream_t s) {
  if (!aligned16(x) || (m > 1 && (ld_x * sizeof(Tin)) % 16))
    return fail(AXON_E_UNSUPPORTED, "axon_cumsum: variant 2 needs 16-byte aligned input rows");
  if (m > 0x7fffffffLL) return fail(AXON_E_SHAPE, "axon_cumsum: too many rows (%lld)", (long long)m);
  const int stages = t.stages ? t.stages : kRowStages;
  const int kb = t.block_k ? t.block_k : kRowStageBytes / 1024;
  if (t.threads != 0 && t.threads != kRowThreads)
    return fail(AXON_E_ARG, "axon_cumsum: variant 2 runs %d threads", kRowThreads);
  if (stages < 2 || stages > kRowMaxStages) return fail(AXON_E_ARG, "axon_cumsum: variant 2 stages must be 2..8");
  if ((kb != 16 && kb != 24 && kb != 32 && kb != 48) || stages * kb > 200)
    return fail(AXON_E_ARG, "axon_cumsum: variant 2 stage size must be 16, 24, 32 or 48 KB, ring <= 200 KB");
  const bool vec_out = aligned16(y) && (ld_y * sizeof(Tout)) % 16 == 0;
  const size_t smem = static_cast<size_t>(stages) * kb * 1024;
  constexpr int NW = kRowThreads / 32;
  const bool k2 = t.split == 2;  // tune.split: packets per lane per segment (1 or 2)
  auto kern = kb == 16   ? (k2 ? cumsum_rowstream<Tin, Tout, NW, 16, 2> : cumsum_rowstream<Tin, Tout, NW, 16, 1>)
              : kb == 24 ? (k2 ? cumsum_rowstream<Tin, Tout, NW, 24, 2> : cumsum_rowstream<Tin, Tout, NW, 24, 1>)
              : kb == 32 ? (k2 ? cumsum_rowstream<Tin, Tout, NW, 32, 2> : cumsum_rowstream<Tin, Tout, NW, 32, 1>)
                         : (k2 ? cumsum_rowstream<Tin, Tout, NW, 48, 2> : cumsum_rowstream<Tin, Tout, NW, 48, 1>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return fail(AXON_E_LAUNCH, "axon_cumsum: smem attribute: %s", cudaGetErrorString(e));
  launch_k(kern, dim3(static_cast<unsigned>(m)), dim3(kRowThreads), smem, s, static_cast<const Tin*>(x),
           static_cast<Tout*>(y), n, ld_x, ld_y, vec_out, stages, static_cast<int*>(ws));
  return launch_status("axon_cumsum");
}

// ---- variant 3: balanced chunk ranges --------------------------------------------
//
// One CTA per row loads the SMs unevenly whenever the row count is not a
// multiple of the resident CTAs (256 rows over 148 SMs with two CTAs each:
// 108 SMs stream two rows, 40 stream one, and the slowest SM sets the time).
// Here rows are cut into the same fixed chunks as variant 2 and every CTA --
// two 512-thread CTAs per SM, as variant 2 runs, G = 2 x SMs of them --
// takes an equal contiguous range of the row-major chunk sequence. A range
// is: a lead (the tail of a row whose head belongs to the previous CTA),
// whole rows, and a trail (the head of a row whose tail belongs to the next
// CTA), or, when it lies inside one row, a single middle piece. A CTA streams
// its trail first and publishes the trail's float64 running sum in its
// workspace slot (a release store of a ready word), then its whole rows, and
// its lead last, taking the lead's carry from the previous CTA's slot
// (acquire load, bounded wait): published early in that CTA's run, so a lead
// rarely waits. A middle piece waits for its carry first and publishes after
// its last chunk. The reader clears the ready word, so a call leaves the
// slots as it found them. Numerics are those of variant 2: a float64 running
// sum across chunks and a chunk-local fp32 prefix, same warp split.
struct ScanSlot {
  double prefix;
  int ready;
  int pad;
};
constexpr int kSlotReady = 0x5ca11ed;    // a slot holds a published sum
constexpr int kBalThreads = 512;
constexpr int kBalStages = 2;            // default ring: 2 x 32 KB per CTA
constexpr int64_t kBalSlotOffset = 256;  // slots follow the status word's block
constexpr int kBalMaxSlots = 1024;
constexpr int64_t kBalShortRowBytes = 32768;  // variant 0 runs variant 3 for rows up to this

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

template <typename Tin, typename Tout, int NW, int SKB>
__global__ void __launch_bounds__(NW * 32, 2) cumsum_balanced(const Tin* __restrict__ x, Tout* __restrict__ y,
                                                              int64_t m, int64_t n, int64_t ld_x, int64_t ld_y,
                                                              bool vec_out, int stages, unsigned char* ws) {
  constexpr int E = Vec<Tin>::E;
  constexpr int64_t kChunk = SKB * 1024 / static_cast<int64_t>(sizeof(Tin));
  constexpr int64_t PPW = kChunk / E / NW;  // packets per warp per chunk
  static_assert(PPW % 32 == 0, "whole segments per warp");
  constexpr int NSEG = static_cast<int>(PPW / 32);
  constexpr int64_t kStageBytes = SKB * 1024;
  extern __shared__ __align__(128) unsigned char dyn_smem[];
  __shared__ __align__(8) uint64_t full[kRowMaxStages];
  __shared__ float s_warp[2][NW];
  __shared__ double s_lead;
  __shared__ int s_abort;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  ScanSlot* slots = reinterpret_cast<ScanSlot*>(ws + kBalSlotOffset);

  // this CTA's chunks [g0, g1) of the row-major sequence, split into
  // trail (row rb, chunks [0, k1)), whole rows [full0, rb), lead (row ra,
  // chunks [k0, cpr)), processed in that order; or one middle piece (row ra,
  // chunks [k0, k1)), handled as a lead that also publishes
  // (chunk counts fit in 32 bits: the launcher checks m * cpr < 2^31)
  const int cpr = static_cast<int>((n + kChunk - 1) / kChunk);
  const int64_t total = m * cpr;
  const int b = blockIdx.x;
  const int g0 = static_cast<int>(b * total / gridDim.x), g1 = static_cast<int>((b + 1) * total / gridDim.x);
  const int ra = g0 / cpr, k0 = g0 - ra * cpr;
  const int rb = g1 / cpr, k1 = g1 - rb * cpr;
  const bool mid = ra == rb && k0 > 0;  // then k1 > k0
  const int n_trail = mid ? 0 : k1;
  const int full0 = k0 > 0 ? ra + 1 : ra;
  const int n_full = mid ? 0 : (rb - full0) * cpr;
  const int n_lead = mid ? k1 - k0 : k0 > 0 ? cpr - k0 : 0;
  const int npos = n_trail + n_full + n_lead;
  auto locate = [&](int p, int& row, int& c) {
    if (p < n_trail) {
      row = rb;
      c = p;
    } else if (p < n_trail + n_full) {
      const int q = p - n_trail;
      row = full0 + q / cpr;
      c = q - (q / cpr) * cpr;
    } else {
      row = ra;
      c = k0 + (p - n_trail - n_full);
    }
  };
  auto chunk_len = [&](int c) {
    const int64_t left = n - static_cast<int64_t>(c) * kChunk;
    return left < kChunk ? left : kChunk;
  };
  auto issue = [&](int p) {
    int row, c;
    locate(p, row, c);
    const int st = p % stages;
    const uint32_t bytes = static_cast<uint32_t>(chunk_len(c) * static_cast<int64_t>(sizeof(Tin)) / 16 * 16);
    if (bytes == 0) {
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sm100::smem_addr(&full[st])) : "memory");
      return;
    }
    sm100::mbar_expect_tx(&full[st], bytes);
    sm100::bulk_g2s(dyn_smem + st * kStageBytes, x + row * ld_x + static_cast<int64_t>(c) * kChunk, bytes,
                    &full[st]);
  };

  if (tid == 0) {
    for (int st = 0; st < stages; ++st) sm100::mbar_init(&full[st], 1);
    s_abort = 0;
    sm100::mbar_init_fence();
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  if (b == 0 && tid == 0) *reinterpret_cast<int*>(ws) = AXON_OK;
  if (tid == 0)
    for (int p = 0; p < npos && p < stages; ++p) issue(p);

  double carry = 0.0;
  for (int p = 0; p < npos; ++p) {
    int row, c;
    locate(p, row, c);
    const int st = p % stages;
    const int bsel = p & 1;
    const int len = static_cast<int>(chunk_len(c));
    const int bulk_elems = static_cast<int>(len * sizeof(Tin) / 16 * 16 / sizeof(Tin));
    const Tin* buf = reinterpret_cast<const Tin*>(dyn_smem + st * kStageBytes);
    const Tin* gsrc = x + row * ld_x + static_cast<int64_t>(c) * kChunk;
    const bool lead_start = n_lead > 0 && p == n_trail + n_full;
    if (tid == 0 && lead_start) {
      // the previous CTA's trail sum, read once and cleared
      ScanSlot* prev = slots + (b - 1);
      const uint64_t t0 = sm100::globaltimer_ns();
      bool ok = true;
      while (ld_acquire_gpu(&prev->ready) != kSlotReady) {
        if (sm100::globaltimer_ns() - t0 > kBulkWaitNs) {
          ok = false;
          break;
        }
        __nanosleep(100);
      }
      if (ok) {
        s_lead = __ldcg(&prev->prefix);
        prev->ready = 0;
      } else {
        s_lead = 0.0;
        atomicExch(&g_scan_error, AXON_E_TIMEOUT);
      }
    }
    if (!s_abort &&
        !sm100::mbar_wait_bounded(&full[st], static_cast<uint32_t>((p / stages) & 1), kBulkWaitNs)) {
      s_abort = 1;
      atomicExch(&g_scan_error, AXON_E_TIMEOUT);
    }
    // pass 1: this thread's packets -> registers, and the warp sums
    const bool full_chunk = len == kChunk;
    const int wbase = warp * static_cast<int>(PPW) + lane;  // this lane's first packet
    Vec<Tin> raw[NSEG];
    float wsum = 0.f;
#pragma unroll
    for (int q = 0; q < NSEG; ++q) {
      const int e0 = (wbase + q * 32) * E;
      if (full_chunk || e0 + E <= bulk_elems) {
        raw[q] = *reinterpret_cast<const Vec<Tin>*>(buf + e0);
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const int i = e0 + e;
          raw[q].e[e] = i < bulk_elems ? buf[i] : i < len ? gsrc[i] : from_f<Tin>(0.f);
        }
      }
#pragma unroll
      for (int e = 0; e < E; ++e) wsum += to_f(raw[q].e[e]);
    }
    wsum = warp_sum(wsum);
    if (lane == 0) s_warp[bsel][warp] = wsum;
    __syncthreads();
    if (tid == 0 && p + stages < npos) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(p + stages);
    }
    if (c == 0) carry = 0.0;  // a row starts: the trail, or a whole row
    if (lead_start) carry = s_lead;
    float wi = lane < NW ? s_warp[bsel][lane] : 0.f;
#pragma unroll
    for (int o = 1; o < NW; o <<= 1) {
      const float up = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += up;
    }
    const float chunk_total = __shfl_sync(0xffffffffu, wi, NW - 1);
    const float warp_excl = __shfl_sync(0xffffffffu, wi, warp > 0 ? warp - 1 : 0);
    const float carry_f = static_cast<float>(carry);
    float seg_carry = warp > 0 ? warp_excl : 0.f;
    // pass 2: scan 32-packet segments and write them out
    Tout* cdst = y + row * ld_y + static_cast<int64_t>(c) * kChunk;
#pragma unroll
    for (int j = 0; j < NSEG; ++j) {
      const int e0 = (wbase + j * 32) * E;
      float v[E];
#pragma unroll
      for (int q = 0; q < E; ++q) v[q] = to_f(raw[j].e[q]);
#pragma unroll
      for (int q = 1; q < E; ++q) v[q] += v[q - 1];
      const float own = v[E - 1];
      float incl = own;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float up = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += up;
      }
      const float base = seg_carry + (incl - own);
#pragma unroll
      for (int q = 0; q < E; ++q) v[q] = carry_f + (base + v[q]);
      if (full_chunk) store_packet<Tout, E>(cdst + e0, v, E, vec_out);
      else if (e0 < len) store_packet<Tout, E>(cdst + e0, v, len - e0, vec_out);
      seg_carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    carry += static_cast<double>(chunk_total);
    if (tid == 0 && ((n_trail > 0 && p == n_trail - 1) || (mid && p == npos - 1))) {
      // the trail (or middle piece) is done: its running sum carries into
      // the next CTA's lead
      slots[b].prefix = carry;
      st_release_gpu(&slots[b].ready, kSlotReady);
    }
  }
  // copies may still be landing only if a wait gave up: let them finish
  // before the CTA's shared memory is released (failure path only)
  if (tid == 0 && s_abort)
    for (int k = 0; k < 2000; ++k) __nanosleep(1000);
}

// Launch of variant 3: `ws` holds the status word and one slot per CTA
// (kBalSlotOffset + 16 * G bytes); its slots must read as not ready (zero-filled
// before the first call; every completed call leaves them so).
template <typename Tin, typename Tout>
int launch_balanced(const void* x, void* y, int64_t m, int64_t n, int64_t ld_x, int64_t ld_y, const axon_tune_t& t,
                    void* ws, int64_t ws_bytes, cudaStream_t s) {
  if (!aligned16(x) || (m > 1 && (ld_x * sizeof(Tin)) % 16))
    return fail(AXON_E_UNSUPPORTED, "axon_cumsum: variant 3 needs 16-byte aligned input rows");
  const int64_t chunk_elems = (t.block_k ? t.block_k : 32) * 1024 / static_cast<int64_t>(sizeof(Tin));
  const int64_t chunks = m * ((n + chunk_elems - 1) / chunk_elems);
  if (chunks > 0x7fffffffLL) return fail(AXON_E_SHAPE, "axon_cumsum: variant 3 takes fewer than 2^31 chunks");
  // two CTAs per SM, every CTA at least one chunk
  int64_t G = t.max_ctas > 0 ? t.max_ctas : 2 * sm_count();
  if (G > 2 * sm_count()) G = 2 * sm_count();
  if (G > chunks) G = chunks;
  if (G > kBalMaxSlots) G = kBalMaxSlots;
  const int64_t need = kBalSlotOffset + static_cast<int64_t>(sizeof(ScanSlot)) * G;
  if (ws == nullptr || ws_bytes < need || !aligned16(ws))
    return fail(AXON_E_ARG, "axon_cumsum: variant 3 needs a zero-filled, 16-byte aligned workspace of %lld bytes",
                (long long)need);
  const int stages = t.stages ? t.stages : kBalStages;
  const int kb = t.block_k ? t.block_k : 32;
  if (t.threads != 0 && t.threads != kBalThreads)
    return fail(AXON_E_ARG, "axon_cumsum: variant 3 runs %d threads", kBalThreads);
  if (stages < 2 || stages > kRowMaxStages) return fail(AXON_E_ARG, "axon_cumsum: variant 3 stages must be 2..8");
  if ((kb != 16 && kb != 32) || stages * kb > 200)
    return fail(AXON_E_ARG, "axon_cumsum: variant 3 stage size must be 16 or 32 KB, ring <= 200 KB");
  const bool vec_out = aligned16(y) && (ld_y * sizeof(Tout)) % 16 == 0;
  const size_t smem = static_cast<size_t>(stages) * kb * 1024;
  constexpr int NW = kBalThreads / 32;
  auto kern = kb == 16 ? cumsum_balanced<Tin, Tout, NW, 16> : cumsum_balanced<Tin, Tout, NW, 32>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return fail(AXON_E_LAUNCH, "axon_cumsum: smem attribute: %s", cudaGetErrorString(e));
  launch_k(kern, dim3(static_cast<unsigned>(G)), dim3(kBalThreads), smem, s, static_cast<const Tin*>(x),
           static_cast<Tout*>(y), m, n, ld_x, ld_y, vec_out, stages, static_cast<unsigned char*>(ws));
  return launch_status("axon_cumsum");
}

template <typename Tin>
int dispatch_balanced(int32_t out_dtype, const void* x, void* y, int64_t m, int64_t n, int64_t ld_x, int64_t ld_y,
                      const axon_tune_t& t, void* ws, int64_t ws_bytes, cudaStream_t s) {
  switch (out_dtype) {
    case AXON_F32: return launch_balanced<Tin, float>(x, y, m, n, ld_x, ld_y, t, ws, ws_bytes, s);
    case AXON_BF16: return launch_balanced<Tin, __nv_bfloat16>(x, y, m, n, ld_x, ld_y, t, ws, ws_bytes, s);
    default: return fail(AXON_E_UNSUPPORTED, "axon_cumsum: unsupported output dtype %d", out_dtype);
  }
}

template <typename Tin>
int dispatch_rowstream(int32_t out_dtype, const void* x, void* y, int64_t m, int64_t n, int64_t ld_x, int64_t ld_y,
                       const axon_tune_t& t, void* ws, cudaStream_t s) {
  switch (out_dtype) {
    case AXON_F32: return launch_rowstream<Tin, float>(x, y, m, n, ld_x, ld_y, t, ws, s);
    case AXON_BF16: return launch_rowstream<Tin, __nv_bfloat16>(x, y, m, n, ld_x, ld_y, t, ws, s);
    default: return fail(AXON_E_UNSUPPORTED, "axon_cumsum: unsupported output dtype %d", out_dtype);
  }
}

template <typename Tin>
int dispatch_cluster(int32_t out_dtype, const void* x, void* y, int64_t m, int64_t n, int64_t ld_x, int64_t ld_y,
                     const axon_tune_t& t, cudaStream_t s) {
  switch (out_dtype) {
    case AXON_F32: return launch_cluster<Tin, float>(x, y, m, n, ld_x, ld_y, t, s);
    case AXON_BF16: return launch_cluster<Tin, __nv_bfloat16>(x, y, m, n, ld_x, ld_y, t, s);
    default: return fail(AXON_E_UNSUPPORTED, "axon_cumsum: unsupported output dtype %d", out_dtype);
  }
}

void tile_shape(const axon_tune_t& t, int& threads, int& items) {
  switch (t.split) {
    case 2048: threads = 128; items = 16; break;
    case 4096: threads = 256; items = 16; break;
    case 16384: threads = 1024; items = 16; break;
    default: threads = 512; items = 16; break;  // 8192
  }
}

int64_t lookback_ws_bytes(int64_t m, int64_t n, const axon_tune_t& t) {
  int threads, items;
  tile_shape(t, threads, items);
  const int64_t tile = static_cast<int64_t>(threads) * items;
  const int64_t tpr = n > 0 ? (n + tile - 1) / tile : 0;
  return kHeaderBytes + static_cast<int64_t>(sizeof(TileDesc)) * m * tpr;
}

template <typename Tin, typename Tout>
int launch_lookback(const void* x, void* y, int64_t m, int64_t n, int64_t ld_x, int64_t ld_y, void* ws,
                    const axon_tune_t& t, cudaStream_t s) {
  int threads, items;
  tile_shape(t, threads, items);
  const int64_t tile = static_cast<int64_t>(threads) * items;
  const int64_t tpr = (n + tile - 1) / tile;
  const int64_t tiles = m * tpr;
  if (tiles > 0x7fffffffLL) return fail(AXON_E_SHAPE, "axon_cumsum: too many tiles (%lld)", (long long)tiles);
  const bool vec = aligned16(x) && aligned16(y) && (ld_x * sizeof(Tin)) % 16 == 0 &&
                   (ld_y * sizeof(Tout)) % 16 == 0;
  cudaError_t e = cudaMemsetAsync(ws, 0, lookback_ws_bytes(m, n, t), s);
  if (e != cudaSuccess) return fail(AXON_E_CUDA, "axon_cumsum: workspace clear failed: %s", cudaGetErrorString(e));
  auto* ws8 = static_cast<unsigned char*>(ws);
  if (items == 8)
    launch_k(cumsum_lookback<Tin, Tout, 8>, dim3(static_cast<unsigned>(tiles)), dim3(threads), 0, s,
             static_cast<const Tin*>(x), static_cast<Tout*>(y), n, ld_x, ld_y, tpr, vec, ws8);
  else
    launch_k(cumsum_lookback<Tin, Tout, 16>, dim3(static_cast<unsigned>(tiles)), dim3(threads), 0, s,
             static_cast<const Tin*>(x), static_cast<Tout*>(y), n, ld_x, ld_y, tpr, vec, ws8);
  return launch_status("axon_cumsum");
}

template <typename Tin>
int dispatch_out(int32_t out_dtype, const void* x, void* y, int64_t m, int64_t n, int64_t ld_x, int64_t ld_y,
                 void* ws, const axon_tune_t& t, cudaStream_t s) {
  switch (out_dtype) {
    case AXON_F32: return launch_lookback<Tin, float>(x, y, m, n, ld_x, ld_y, ws, t, s);
    case AXON_BF16: return launch_lookback<Tin, __nv_bfloat16>(x, y, m, n, ld_x, ld_y, ws, t, s);
    default: return fail(AXON_E_UNSUPPORTED, "axon_cumsum: unsupported output dtype %d", out_dtype);
  }
}

}  // namespace
}  // namespace axon

using namespace axon;

extern "C" int64_t axon_cumsum_workspace_bytes(int64_t m, int64_t n, const axon_tune_t* tune) {
  axon_tune_t t = tune_or_default(tune);
  if (m < 0 || n < 0) return fail(AXON_E_SHAPE, "axon_cumsum_workspace_bytes: negative size");
  if (t.variant == 1 || t.variant == 2) return 0;
  const int64_t balanced = kBalSlotOffset + static_cast<int64_t>(sizeof(ScanSlot)) * kBalMaxSlots;
  if (t.variant == 3) return balanced;
  // variant 0 may run variant 3 (short aligned rows): room for either
  const int64_t lookback = lookback_ws_bytes(m, n, t);
  return lookback > balanced ? lookback : balanced;
}

extern "C" int axon_cumsum(const void* x, void* y, int64_t m, int64_t n, int64_t ld_x, int64_t ld_y,
                           int32_t in_dtype, int32_t out_dtype, void* workspace, int64_t workspace_bytes,
                           const axon_tune_t* tune, void* stream) {
  axon_tune_t t = tune_or_default(tune);
  if (m < 0 || n < 0) return fail(AXON_E_SHAPE, "axon_cumsum: negative size");
  if (m > 0 && n > 0 && (!x || !y)) return fail(AXON_E_ARG, "axon_cumsum: NULL tensor pointer");
  if (ld_x < n || ld_y < n) return fail(AXON_E_SHAPE, "axon_cumsum: leading dimension smaller than n");
  if (t.variant == 1) {
    if (t.split != 0 && t.split != 1 && t.split != 2 && t.split != 4 && t.split != 8)
      return fail(AXON_E_ARG, "axon_cumsum: variant 1 split (CTAs per row cluster) must be 1, 2, 4 or 8");
    if (m == 0 || n == 0) return AXON_OK;
    cudaStream_t s = as_stream(stream);
    switch (in_dtype) {
      case AXON_F32: return dispatch_cluster<float>(out_dtype, x, y, m, n, ld_x, ld_y, t, s);
      case AXON_BF16: return dispatch_cluster<__nv_bfloat16>(out_dtype, x, y, m, n, ld_x, ld_y, t, s);
      default: return fail(AXON_E_UNSUPPORTED, "axon_cumsum: unsupported input dtype %d", in_dtype);
    }
  }
  if (t.variant == 2) {
    if (t.split != 0 && t.split != 1 && t.split != 2)
      return fail(AXON_E_ARG, "axon_cumsum: variant 2 split (packets per lane) must be 1 or 2");
    if (m == 0 || n == 0) return AXON_OK;
    cudaStream_t s = as_stream(stream);
    switch (in_dtype) {
      case AXON_F32: return dispatch_rowstream<float>(out_dtype, x, y, m, n, ld_x, ld_y, t, workspace, s);
      case AXON_BF16:
        return dispatch_rowstream<__nv_bfloat16>(out_dtype, x, y, m, n, ld_x, ld_y, t, workspace, s);
      default: return fail(AXON_E_UNSUPPORTED, "axon_cumsum: unsupported input dtype %d", in_dtype);
    }
  }
  if (t.variant == 3) {
    if (m == 0 || n == 0) return AXON_OK;
    cudaStream_t s = as_stream(stream);
    switch (in_dtype) {
      case AXON_F32:
        return dispatch_balanced<float>(out_dtype, x, y, m, n, ld_x, ld_y, t, workspace, workspace_bytes, s);
      case AXON_BF16:
        return dispatch_balanced<__nv_bfloat16>(out_dtype, x, y, m, n, ld_x, ld_y, t, workspace, workspace_bytes,
                                                s);
      default: return fail(AXON_E_UNSUPPORTED, "axon_cumsum: unsupported input dtype %d", in_dtype);
    }
  }
  if (t.split != 0 && t.split != 2048 && t.split != 4096 && t.split != 8192 && t.split != 16384)
    return fail(AXON_E_ARG, "axon_cumsum: split must be one of 2048, 4096, 8192, 16384 (got %d)", t.split);
  if (t.variant != 0) return fail(AXON_E_UNSUPPORTED, "axon_cumsum: unknown variant %d", t.variant);
  if (m == 0 || n == 0) return AXON_OK;
  // Default (variant 0 without a split): the chunk-streaming scans when there
  // are enough rows to fill the GPU and the rows are 16-byte aligned; the
  // row-streaming scan beat the look-back scan on B200 at 256 x 128256 (51
  // vs 85 us), 1024 x 32768 and 4096 x 4096, and lost at 64 x 1e6 (228 vs
  // 211 us).
  const int64_t in_size = in_dtype == AXON_F32 ? 4 : 2;
  if (t.split == 0 && t.threads == 0 && m >= kRowStreamMinRows && aligned16(x) && (ld_x * in_size) % 16 == 0 &&
      (in_dtype == AXON_F32 || in_dtype == AXON_BF16)) {
    cudaStream_t s = as_stream(stream);
    // Rows of at most 32 KB: balanced chunk ranges of 16 KB chunks, which
    // stream across row ends instead of paying a CTA's start per row
    // (4096 x 4096 fp32 on B200: 30.9 us vs 53.9 for one CTA per row); longer
    // rows: the row-streaming scan (1024 x 32768: 45.1 vs 49.3 us).
    if (n * in_size <= kBalShortRowBytes && workspace != nullptr &&
        workspace_bytes >= kBalSlotOffset + static_cast<int64_t>(sizeof(ScanSlot)) * 2 * sm_count()) {
      axon_tune_t tb = t;
      tb.variant = 3;
      tb.block_k = 16;
      tb.stages = 4;
      return in_dtype == AXON_F32
                 ? dispatch_balanced<float>(out_dtype, x, y, m, n, ld_x, ld_y, tb, workspace, workspace_bytes, s)
                 : dispatch_balanced<__nv_bfloat16>(out_dtype, x, y, m, n, ld_x, ld_y, tb, workspace,
                                                    workspace_bytes, s);
    }
    return in_dtype == AXON_F32
               ? dispatch_rowstream<float>(out_dtype, x, y, m, n, ld_x, ld_y, t, workspace, s)
               : dispatch_rowstream<__nv_bfloat16>(out_dtype, x, y, m, n, ld_x, ld_y, t, workspace, s);
  }
  const int64_t need = lookback_ws_bytes(m, n, t);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(AXON_E_ARG, "axon_cumsum: workspace of %lld bytes needed, got %lld", (long long)need,
                (long long)workspace_bytes);
  cudaStream_t s = as_stream(stream);
  switch (in_dtype) {
    case AXON_F32: return dispatch_out<float>(out_dtype, x, y, m, n, ld_x, ld_y, workspace, t, s);
    case AXON_BF16: return dispatch_out<__nv_bfloat16>(out_dtype, x, y, m, n, ld_x, ld_y, workspace, t, s);
    default: return fail(AXON_E_UNSUPPORTED, "axon_cumsum: unsupported input dtype %d", in_dtype);
  }
}

extern "C" int axon_cumsum_status(const void* workspace, void* stream) {
  int status = 0, device_word = 0;
  cudaError_t e = cudaSuccess;
  if (workspace) e = cudaMemcpyAsync(&status, workspace, sizeof(int), cudaMemcpyDeviceToHost, as_stream(stream));
  // the device status word of the bulk-copy variants; reading clears it
  if (e == cudaSuccess)
    e = cudaMemcpyFromSymbolAsync(&device_word, g_scan_error, sizeof(int), 0, cudaMemcpyDeviceToHost,
                                  as_stream(stream));
  if (e == cudaSuccess) e = cudaStreamSynchronize(as_stream(stream));
  if (e == cudaSuccess && device_word != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_scan_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, as_stream(stream));
  }
  if (status == 0) status = device_word;
  if (e == cudaSuccess) e = cudaStreamSynchronize(as_stream(stream));
  if (e != cudaSuccess) return fail(AXON_E_CUDA, "axon_cumsum_status: %s", cudaGetErrorString(e));
  if (status != 0) return fail(status, "axon_cumsum: a bounded wait gave up (status %d)", status);
  return AXON_OK;
}

// ---- allocation-free variant ----------------------------------------------------
//
// axon_cumsum_noalloc serves callers that must not allocate device memory
// themselves: a plugin whose host framework owns every device allocation
// through its own memory planner, or a latency-critical caller for whom
// cudaMalloc (which can synchronise the whole device) is off limits. It runs
// the same look-back kernel as axon_cumsum, with its scratch in a fixed
// file-scope device array instead of a caller workspace. The array exists
// once per device that loads this library and lives until the process exits.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

namespace axon {
namespace {

constexpr int64_t kNoAllocScratchBytes = 1 << 20;  // 1 MiB: up to 32767 look-back tiles
static __device__ __align__(256) unsigned char g_cumsum_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};
CUcontext g_scratch_ctx[kMaxDevices] = {};

PFN_cuCtxGetCurrent_v4000 ctx_current_fn() {
  static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
  });
  return fn;
}

// The device address of g_cumsum_scratch on the current device. In host code
// the symbol is only a stand-in, so the address is looked up with
// cudaGetSymbolAddress, once per device, with that device current. The
// device's context is recorded with it: a reset device gets a new context,
// and the address is then looked up again instead of reusing a stale one.
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(AXON_E_CUDA, "axon_cumsum_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(AXON_E_UNSUPPORTED, "axon_cumsum_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  void* p = nullptr;
  if (g_scratch_addr[dev] == nullptr) {
    // the first runtime call on this device makes its primary context current
    e = cudaGetSymbolAddress(&p, g_cumsum_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(AXON_E_CUDA, "axon_cumsum_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
  }
  CUcontext ctx = nullptr;
  auto current = ctx_current_fn();
  if (current == nullptr || current(&ctx) != CUDA_SUCCESS)
    return fail(AXON_E_CUDA, "axon_cumsum_noalloc: cuCtxGetCurrent unavailable");
  if (g_scratch_addr[dev] == nullptr || g_scratch_ctx[dev] != ctx) {
    if (p == nullptr) {
      e = cudaGetSymbolAddress(&p, g_cumsum_scratch);
      if (e != cudaSuccess || p == nullptr)
        return fail(AXON_E_CUDA, "axon_cumsum_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    }
    g_scratch_addr[dev] = p;
    g_scratch_ctx[dev] = ctx;
  }
  *out = g_scratch_addr[dev];
  return AXON_OK;
}

}  // namespace
}  // namespace axon

extern "C" int axon_cumsum_noalloc(const void* x, void* y, int64_t m, int64_t n, int64_t ld_x, int64_t ld_y,
                                   int32_t in_dtype, int32_t out_dtype, const axon_tune_t* tune, void* stream) {
  axon_tune_t t = tune_or_default(tune);
  if (m < 0 || n < 0) return fail(AXON_E_SHAPE, "axon_cumsum_noalloc: negative size");
  if (m > 0 && n > 0 && (!x || !y)) return fail(AXON_E_ARG, "axon_cumsum_noalloc: NULL tensor pointer");
  if (ld_x < n || ld_y < n) return fail(AXON_E_SHAPE, "axon_cumsum_noalloc: leading dimension smaller than n");
  if (t.split != 0 && t.split != 2048 && t.split != 4096 && t.split != 8192 && t.split != 16384)
    return fail(AXON_E_ARG, "axon_cumsum_noalloc: split must be one of 2048, 4096, 8192, 16384 (got %d)", t.split);
  if (t.variant != 0) return fail(AXON_E_UNSUPPORTED, "axon_cumsum_noalloc: only variant 0 uses scratch");
  if (m == 0 || n == 0) return AXON_OK;
  const int64_t need = lookback_ws_bytes(m, n, t);
  if (need > kNoAllocScratchBytes)
    return fail(AXON_E_SHAPE,
                "axon_cumsum_noalloc: a %lld x %lld scan needs %lld bytes of look-back scratch but the static "
                "scratch holds %lld; use a larger split or axon_cumsum with a workspace",
                (long long)m, (long long)n, (long long)need, (long long)kNoAllocScratchBytes);
  void* ws = nullptr;
  const int rc = scratch_address(&ws);
  if (rc != AXON_OK) return rc;
  cudaStream_t s = as_stream(stream);
  switch (in_dtype) {
    case AXON_F32: return dispatch_out<float>(out_dtype, x, y, m, n, ld_x, ld_y, ws, t, s);
    case AXON_BF16: return dispatch_out<__nv_bfloat16>(out_dtype, x, y, m, n, ld_x, ld_y, ws, t, s);
    default: return fail(AXON_E_UNSUPPORTED, "axon_cumsum_noalloc: unsupported input dtype %d", in_dtype);
  }
}
