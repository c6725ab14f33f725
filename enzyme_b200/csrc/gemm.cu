// Dense path: a persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   C[m, n] = epilogue(A[m, k] @ B[k, n])      A, B bf16 (or both f16)
//
// A is row-major (K-major for the MMA); B is the [k, n] row-major weight the
// Axon specs pass (kernels/matmul/refs.py:24-25), consumed in place as an
// MN-major operand, so no transpose pass runs.
//
// One CTA per SM, 192 threads:
//   warp 0      TMA producer: streams 128x64 A slabs and BNx64 B slabs into a
//               ring of `stages` shared-memory buffers (128-byte swizzle),
//               one mbarrier per stage carrying the transaction bytes;
//   warp 1      TMEM owner and MMA issuer: one thread issues
//               tcgen05.mma.cta_group::1.kind::f16 (M=128, N=BN, K=16) into a
//               double-buffered fp32 accumulator in tensor memory, and frees
//               each smem stage with tcgen05.commit when its MMAs retire;
//   warps 2..5  epilogue: tcgen05.ld the accumulator (each warp owns its
//               32-lane quarter of TMEM), apply the epilogue in registers and
//               store to global memory, overlapping the next tile's mainloop.
// Epilogues: NONE; ROWSCALE (C = r[i] * acc, the rmsnorm_matmul norm);
// SILU_GATE (the B tile holds BN/2 gate columns from w1 and the matching BN/2
// up columns from w2, so one N=BN MMA yields both and C = silu(g) * u).
//
// Variant 2 (below) runs the same roles on a cluster of two CTAs that share one
// tcgen05.mma.cta_group::2 (M = 256) per k-step, halving the B bytes each SM
// stages per FLOP.
//
// No TMA multicast is used anywhere, so the kernel is legal when its operands
// live in any GPU's memory. Every mbarrier wait is bounded (about two seconds
// of %globaltimer); a wait that gives up raises a CTA-wide abort flag and the
// device error word read by axon_gemm_status(), and every role drains out.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace axon {

__device__ int g_gemm_error;

namespace {

constexpr int BM = 128;
constexpr int BK = 64;              // bf16 elements per 128-byte swizzle row
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_CHUNK = 64 * BK * 2;  // one 64-column MN-major swizzle block
constexpr int EPI_THREADS = 128;
constexpr unsigned long long kTimeoutNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase. Returns false if this CTA has aborted or
// the wait ran past the time limit (which then aborts the CTA).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 127) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > kTimeoutNs) {
        *abort_flag = 1;
        atomicExch(&g_gemm_error, AXON_E_TIMEOUT);
        return false;
      }
    }
  }
}

// mbar_wait for threads with slack: after a few failed tries it sleeps
// between polls, leaving the issue slots to the warps doing the work.
__device__ __forceinline__ bool mbar_wait_backoff(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (i > 4) __nanosleep(64);
    if ((i & 31) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > kTimeoutNs) {
        *abort_flag = 1;
        atomicExch(&g_gemm_error, AXON_E_TIMEOUT);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* dst, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit TMEM columns -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor (sm_100 format): start address, leading and
// stride byte offsets (all >> 4), descriptor version 1 at bit 46, 128-byte
// swizzle (layout type 2) at bits 61..63, base offset 0 (buffers are
// 1024-byte aligned).
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

template <typename TC>
__device__ __forceinline__ void store32(TC* dst, const float* v, int64_t col, int64_t n) {
  if (col + 32 <= n) {
    if constexpr (sizeof(TC) == 4) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        Vec<TC> p;
#pragma unroll
        for (int e = 0; e < 8; ++e) p.e[e] = from_f<TC>(v[j + e]);
        st_vec(dst + j, p);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col + j < n) dst[j] = from_f<TC>(v[j]);
  }
}

// Epilogue of the tensor-parallel down projection (internal to
// axon_tp_down_partial, not an axon_gemm epilogue): output row r goes to the
// inbox of its owner rank o = r / rows_per_owner, a peer buffer laid out
// [world][rows_per_owner][ldc], at slot `peer_rank`.
constexpr int kEpiPeer = 7;
constexpr int kMaxPeers = 8;

struct GemmParams {
  void* c;
  void* peers[kMaxPeers];  // kEpiPeer: each owner's inbox for this output
  int peer_rank;
  int rows_per_owner;
  int world;               // kEpiPeer with interleave: ranks owning 8-row granules in turn
  int interleave;
  const float* row_scale;
  int m, n, k;         // n = output columns
  int64_t ldc;
  int stages;
  uint32_t idesc;
  int terms;           // SILU_GATE: write the activation as this many bf16/f16 terms
  int64_t term_stride; // columns between the terms in C
  int b_kwrap;         // > 0: B's k coordinate wraps modulo this (B re-read per term)
  int max_ctas;        // > 0: cap on the persistent grid
  int raster;          // > 0: tiles ordered in bands of this many row tiles (see tile_coords)
  float* row_part;     // EXP: sums of the stored values per (column tile, row), or NULL
  int64_t part_ld;     // row_part stride between column tiles (>= m)
};

// Ownership of output row r: contiguous blocks of rows_per_owner rows, or
// (interleave) 8-row granules dealt to the ranks in turn, so every owner's
// rows are spread over the whole output. `local` is the row's index among
// its owner's rows.
__device__ __forceinline__ int row_owner(const GemmParams& p, int64_t row, int64_t& local) {
  if (p.interleave) {
    const int o = static_cast<int>((row >> 3) % p.world);
    local = (row / (8 * p.world)) * 8 + (row & 7);
    return o;
  }
  const int o = static_cast<int>(row / p.rows_per_owner);
  local = row - static_cast<int64_t>(o) * p.rows_per_owner;
  return o;
}

// Tile t of the persistent loop: column-major over the whole grid of tiles
// (raster 0), or in bands of `raster` row tiles, each band column-major, so
// the tiles in flight share fewer A rows and B columns and more of both stay
// in L2.
__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int raster, int& tm, int& tn) {
  if (raster <= 0 || raster >= num_m) {
    tm = t % num_m;
    tn = t / num_m;
    return;
  }
  const int band = t / (raster * num_n);
  const int within = t - band * raster * num_n;
  const int rows = num_m - band * raster < raster ? num_m - band * raster : raster;
  tm = band * raster + within % rows;
  tn = within / rows;
}

template <int EPI, typename TC>
__device__ __forceinline__ TC* out_row(const GemmParams& p, TC* C, int64_t row) {
  if constexpr (EPI == kEpiPeer) {
    int64_t local;
    const int o = row_owner(p, row, local);
    return static_cast<TC*>(p.peers[o]) + (static_cast<int64_t>(p.peer_rank) * p.rows_per_owner + local) * p.ldc;
  } else {
    return C + row * p.ldc;
  }
}

constexpr int kPeerStageHalves = 72;                              // 64 columns + 8 of padding per row
constexpr int kPeerStageBytes = 4 * 32 * kPeerStageHalves * 2;    // one 32-row piece per epilogue warp

// kEpiPeer: the warp's 32 accumulator rows leave in 64-column pieces through a
// shared-memory transpose, so each store instruction writes 4 rows x 128
// contiguous bytes of an owner's inbox: whole lines cross NVLink instead of
// 32 scattered 16-byte pieces.
template <int BN>
__device__ __forceinline__ void peer_store_tile(const GemmParams& p, __half* stg, uint32_t tbase, int64_t row0,
                                                int64_t col0, int lane) {
#pragma unroll 1
  for (int c = 0; c < BN / 64; ++c) {
    float v[64];
    __syncwarp();
    tmem_ld32(tbase + c * 64, v);
    tmem_ld32(tbase + c * 64 + 32, v + 32);
    tmem_wait_ld();
    __half* mine = stg + lane * kPeerStageHalves;
#pragma unroll
    for (int j = 0; j < 64; j += 8) {
      Vec<__half> pk;
#pragma unroll
      for (int e = 0; e < 8; ++e) pk.e[e] = __float2half_rn(v[j + e]);
      *reinterpret_cast<uint4*>(mine + j) = pk.u;
    }
    __syncwarp();
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int r = it * 4 + (lane >> 3), seg = lane & 7;
      const int64_t row = row0 + r;
      const int64_t col = col0 + c * 64 + seg * 8;
      const uint4 val = *reinterpret_cast<const uint4*>(stg + r * kPeerStageHalves + seg * 8);
      if (row < p.m && col < p.n) *reinterpret_cast<uint4*>(out_row<kEpiPeer, __half>(p, nullptr, row) + col) = val;
    }
  }
}

template <int BN, int EPI, typename TC>
__global__ void __launch_bounds__(192, 1)
    gemm_tcgen05(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmB2, GemmParams p) {
  constexpr int B_BYTES = BN * BK * 2;
  constexpr int STAGE = A_BYTES + B_BYTES;
  constexpr int BN_OUT = EPI == AXON_EPI_SILU_GATE ? BN / 2 : BN;
  constexpr uint32_t TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * STAGE);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* issued = reinterpret_cast<int*>(tmem_slot + 2);  // TMA slabs issued, per stage
  int* consumed = issued + S;                            // slabs the MMA warp consumed, per stage

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (p.m + BM - 1) / BM;
  const int num_n = (p.n + BN_OUT - 1) / BN_OUT;
  const int tiles = num_m * num_n;
  const int kblocks = (p.k + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      issued[s] = 0;
      consumed[s] = 0;
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], EPI_THREADS);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
    int stage = 0;
    uint32_t phase = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      int tm, tn;
      tile_coords(t, num_m, num_n, p.raster, tm, tn);
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) goto producer_done;
        mbar_expect_tx(&full[stage], STAGE);
        uint8_t* sa = smem + stage * STAGE;
        uint8_t* sb = sa + A_BYTES;
        tma_load_2d(&tmA, &full[stage], sa, kb * BK, tm * BM);
        if constexpr (EPI == AXON_EPI_SILU_GATE) {
#pragma unroll
          for (int j = 0; j < BN / 128; ++j)
            tma_load_2d(&tmB, &full[stage], sb + j * B_CHUNK, tn * BN_OUT + j * 64, kb * BK);
#pragma unroll
          for (int j = 0; j < BN / 128; ++j)
            tma_load_2d(&tmB2, &full[stage], sb + (BN / 128 + j) * B_CHUNK, tn * BN_OUT + j * 64, kb * BK);
        } else {
          const int kb_b = p.b_kwrap > 0 ? (kb * BK) % p.b_kwrap : kb * BK;
#pragma unroll
          for (int j = 0; j < BN / 64; ++j)
            tma_load_2d(&tmB, &full[stage], sb + j * B_CHUNK, tn * BN + j * 64, kb_b);
        }
        issued[stage] += 1;
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  producer_done:;
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    int stage = 0;
    uint32_t phase = 0;
    int local = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++local) {
      const int buf = local & 1;
      if (!mbar_wait(&tempty[buf], ((local >> 1) & 1) ^ 1u, abort_flag)) break;
      tc_fence_after();
      const uint32_t d = tmem_base + static_cast<uint32_t>(buf * BN);
      bool ok = true;
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + stage * STAGE);
        const uint32_t sb = sa + A_BYTES;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          const uint64_t ad = sdesc(sa + k * 32, 16, 1024);
          const uint64_t bd = sdesc(sb + k * 2048, B_CHUNK, 1024);
          tc_mma(d, ad, bd, p.idesc, (kb | k) != 0);
        }
        tc_commit(&empty[stage]);
        consumed[stage] += 1;
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      tc_commit(&tfull[buf]);
    }
  } else if (warp >= 2) {
    // ---------------- epilogue ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int local = 0;
    TC* C = static_cast<TC*>(p.c);
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++local) {
      int tm, tn;
      tile_coords(t, num_m, num_n, p.raster, tm, tn);
      const int buf = local & 1;
      if (!mbar_wait(&tfull[buf], (local >> 1) & 1, abort_flag)) break;
      tc_fence_after();
      const int64_t row = static_cast<int64_t>(tm) * BM + q * 32 + lane;
      const bool row_ok = row < p.m;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * BN);
      TC* crow = out_row<EPI, TC>(p, C, row_ok ? row : 0);
      float scale = 1.f;
      if constexpr (EPI == AXON_EPI_ROWSCALE) scale = row_ok ? p.row_scale[row] : 0.f;
      if constexpr (EPI == AXON_EPI_SILU_GATE) {
#pragma unroll 1
        for (int c = 0; c < BN_OUT / 32; ++c) {
          float g[32], u[32];
          __syncwarp();
          tmem_ld32(tbase + c * 32, g);
          tmem_ld32(tbase + BN_OUT + c * 32, u);
          tmem_wait_ld();
          const int64_t col = static_cast<int64_t>(tn) * BN_OUT + c * 32;
#pragma unroll
          for (int j = 0; j < 32; ++j) g[j] = g[j] / (1.0f + __expf(-g[j])) * u[j];
          if (row_ok && col < p.n) {
            if (p.terms <= 1) {
              store32<TC>(crow + col, g, col, p.n);
            } else {
              // Split the fp32 activation into `terms` values of TC whose sum
              // carries 8 more mantissa bits per term: t_0 = round(a),
              // t_i = round(a - t_0 - ... - t_{i-1}).
#pragma unroll 1
              for (int tt = 0; tt < p.terms; ++tt) {
                float part[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                  part[j] = to_f(from_f<TC>(g[j]));
                  g[j] -= part[j];
                }
                store32<TC>(crow + tt * p.term_stride + col, part, col, p.n);
              }
            }
          }
        }
      } else if constexpr (EPI == kEpiPeer) {
        __half* stg = reinterpret_cast<__half*>(smem + S * STAGE + 256) + q * 32 * kPeerStageHalves;
        peer_store_tile<BN>(p, stg, tbase, static_cast<int64_t>(tm) * BM + q * 32, static_cast<int64_t>(tn) * BN,
                            lane);
      } else {
        float psum = 0.f;  // EXP: this row's sum over the tile, of the values as stored
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          __syncwarp();
          tmem_ld32(tbase + c * 32, v);
          tmem_wait_ld();
          const int64_t col = static_cast<int64_t>(tn) * BN + c * 32;
          if constexpr (EPI == AXON_EPI_ROWSCALE) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] *= scale;
          }
          if constexpr (EPI == AXON_EPI_EXP) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              v[j] = to_f(from_f<TC>(__expf(v[j])));
              if (col + j < p.n) psum += v[j];
            }
          }
          if (row_ok && col < p.n) store32<TC>(crow + col, v, col, p.n);
        }
        if constexpr (EPI == AXON_EPI_EXP) {
          if (row_ok && p.row_part != nullptr) p.row_part[tn * p.part_ld + row] = psum;
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
    }
  }

  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) {
    // Drain TMA copies that were issued but never consumed, so no copy is in
    // flight into shared memory when the CTA exits.
    for (int s = 0; s < S; ++s) {
      if (issued[s] > consumed[s]) {
        volatile int never = 0;
        mbar_wait(&full[s], static_cast<uint32_t>((issued[s] - 1) & 1), &never);
      }
    }
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
  }
}

// ---- qkv_cte in one pass: the residual sum staged as the A operand ----------------
//
// C = rsqrt(sum_k h^2 / k + eps)[i] * (h @ B), h = x + r1 + r2 (the qkv_cte
// spec's residual add, norm and projection), without h reaching global
// memory. A transform group of 8 warps is the A producer: per k-block each
// thread loads its four 16-byte chunks of each input straight from global
// memory (a warp's load covers four whole 128-byte row segments; two
// k-blocks stay in flight in registers), adds them in fp32 in the spec's
// order, accumulates the rows' sums of h^2 and writes h, rounded to the
// operand type, into a ring of 128-byte-swizzled A slabs -- the layout TMA's
// swizzle would produce -- for the MMA warp. TMA streams only B. A tile is up
// to 512 columns wide -- the whole fused QKV width of the reference's
// cases -- as two MMAs per k-step (N = 256 and BN - 256) into the 512 TMEM
// columns, so each row block's inputs are read and summed once. When the
// row blocks cannot fill the GPU, k is split: each unit writes its fp32
// partial tile and partial sums of h^2, and resid3_reduce_kernel adds the
// splits in a fixed order and applies the scale. Roles: warp 0 TMA, warp 1
// TMEM + MMA, warps 2..5 epilogue, warps 6..13 transform; every wait is
// bounded.
constexpr int kResidXformWarps = 8;
constexpr int kResidThreads = (6 + kResidXformWarps) * 32;

struct Resid3Params {
  void* c;          // [m, ldc] output (splits == 1)
  float* part;      // [splits][m][n] fp32 partial tiles (splits > 1)
  float* ss_part;   // [splits][m] partial sums of h^2 (splits > 1)
  int m, n, k;
  int64_t ldc;
  int stages;
  uint32_t idesc_lo;  // N = min(BN, 256)
  uint32_t idesc_hi;  // N = BN - 256 (BN > 256)
  int splits;
  int kb_per_split;
  int raster;
  float inv_k, eps;
};

constexpr int kResidHSlots = 4;  // h ring depth (16 KB each)

// One k-block of this transform thread's share of the three inputs: chunk
// (t & 7) of rows (t >> 3) + 32 i, i < 4, so each load instruction of a warp
// reads four whole 128-byte row segments. Rows past m and k-blocks past k
// read as zero.
template <typename TA>
struct Resid3Regs {
  uint4 x[4], r1[4], r2[4];
};

template <typename TA>
__device__ __forceinline__ void resid3_load(Resid3Regs<TA>& g, const TA* x, const TA* r1, const TA* r2,
                                            int64_t row0, int m, int k, int kb, int t) {
  const int c = t & 7;
  const int64_t col = static_cast<int64_t>(kb) * BK + c * 8;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t row = row0 + (t >> 3) + 32 * i;
    if (row < m && col < k) {
      const int64_t off = row * k + col;
      g.x[i] = __ldcs(reinterpret_cast<const uint4*>(x + off));
      g.r1[i] = __ldcs(reinterpret_cast<const uint4*>(r1 + off));
      g.r2[i] = __ldcs(reinterpret_cast<const uint4*>(r2 + off));
    } else {
      g.x[i] = g.r1[i] = g.r2[i] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

// h = (x + r1) + r2 in fp32 into the 128-byte-swizzled A slab (chunk c of row
// r at r * 128 + ((c ^ (r & 7)) * 16), the layout TMA's 128-byte swizzle
// writes), and the rows' sums of h^2.
template <typename TA>
__device__ __forceinline__ void resid3_store(const Resid3Regs<TA>& g, uint8_t* slab, float* ss, int t) {
  const int c = t & 7;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = (t >> 3) + 32 * i;
    Vec<TA> a, b, d;
    a.u = g.x[i];
    b.u = g.r1[i];
    d.u = g.r2[i];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float h = (to_f(a.e[e]) + to_f(b.e[e])) + to_f(d.e[e]);
      ss[i] = fmaf(h, h, ss[i]);
      a.e[e] = from_f<TA>(h);
    }
    *reinterpret_cast<uint4*>(slab + r * 128 + ((c ^ (r & 7)) * 16)) = a.u;
  }
}

template <int BN, typename TA, typename TC>
__global__ void __launch_bounds__(kResidThreads, 1)
    gemm_resid3(const TA* __restrict__ x, const TA* __restrict__ r1, const TA* __restrict__ r2,
                const __grid_constant__ CUtensorMap tmB, Resid3Params p) {
  constexpr int B_BYTES = BN * BK * 2;
  constexpr int NBUF = 2 * BN <= 512 ? 2 : 1;  // accumulator buffers in TMEM
  constexpr uint32_t TMEM_COLS = 512;
  constexpr int XT = kResidXformWarps * 32;
  constexpr int H = kResidHSlots;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.stages;                                   // B ring depth
  uint8_t* hbase = smem + S * B_BYTES;                      // h ring: H slabs of A_BYTES
  uint64_t* bfull = reinterpret_cast<uint64_t*>(hbase + H * A_BYTES);
  uint64_t* bempty = bfull + S;
  uint64_t* hfull = bempty + S;
  uint64_t* hempty = hfull + H;
  uint64_t* tfull = hempty + H;
  uint64_t* tempty = tfull + 2;
  uint64_t* rsfull = tempty + 2;
  uint64_t* rsempty = rsfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rsempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* issued = reinterpret_cast<int*>(tmem_slot + 2);
  int* consumed = issued + S;
  float* rs = reinterpret_cast<float*>(hbase + H * A_BYTES + 512);  // [2][BM] row scales

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (p.m + BM - 1) / BM;
  const int num_n = (p.n + BN - 1) / BN;
  const int units = num_m * num_n * p.splits;
  const int kblocks = (p.k + BK - 1) / BK;
  auto unit_k = [&](int u, int& kb0, int& kb1) {
    kb0 = (u % p.splits) * p.kb_per_split;
    kb1 = kb0 + p.kb_per_split < kblocks ? kb0 + p.kb_per_split : kblocks;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&bfull[s], 1);
      mbar_init(&bempty[s], 1);
      issued[s] = 0;
      consumed[s] = 0;
    }
    for (int h = 0; h < H; ++h) {
      mbar_init(&hfull[h], XT);
      mbar_init(&hempty[h], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], EPI_THREADS);
      mbar_init(&rsfull[b], XT);
      mbar_init(&rsempty[b], EPI_THREADS);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer: the B slabs ----------------
    int stage = 0;
    uint32_t phase = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      int tm, tn, kb0, kb1;
      tile_coords(u / p.splits, num_m, num_n, p.raster, tm, tn);
      unit_k(u, kb0, kb1);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&bempty[stage], phase ^ 1u, abort_flag)) goto producer_done;
        mbar_expect_tx(&bfull[stage], B_BYTES);
        uint8_t* sb = smem + stage * B_BYTES;
#pragma unroll
        for (int j = 0; j < BN / 64; ++j)
          tma_load_2d(&tmB, &bfull[stage], sb + j * B_CHUNK, tn * BN + j * 64, kb * BK);
        issued[stage] += 1;
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  producer_done:;
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer: A = an h slab, B = a B slab ----------------
    int stage = 0, hs = 0;
    uint32_t phase = 0, hphase = 0;
    int local = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++local) {
      const int buf = local % NBUF;
      const uint32_t use = static_cast<uint32_t>(local / NBUF);
      if (!mbar_wait(&tempty[buf], (use & 1) ^ 1u, abort_flag)) break;
      tc_fence_after();
      const uint32_t d = tmem_base + static_cast<uint32_t>(buf * BN);
      int kb0, kb1;
      unit_k(u, kb0, kb1);
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&bfull[stage], phase, abort_flag) || !mbar_wait(&hfull[hs], hphase, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(hbase + hs * A_BYTES);
        const uint32_t sb = smem_u32(smem + stage * B_BYTES);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          const uint64_t ad = sdesc(sa + k * 32, 16, 1024);
          const uint32_t acc = (kb != kb0 || k != 0) ? 1u : 0u;
          tc_mma(d, ad, sdesc(sb + k * 2048, B_CHUNK, 1024), p.idesc_lo, acc);
          if constexpr (BN > 256)
            tc_mma(d + 256, ad, sdesc(sb + 4 * B_CHUNK + k * 2048, B_CHUNK, 1024), p.idesc_hi, acc);
        }
        tc_commit(&bempty[stage]);
        tc_commit(&hempty[hs]);
        consumed[stage] += 1;
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
        if (++hs == H) {
          hs = 0;
          hphase ^= 1u;
        }
      }
      if (!ok) break;
      tc_commit(&tfull[buf]);
    }
  } else if (warp >= 2 && warp < 6) {
    // ---------------- epilogue: C = rs[row] * acc, or the fp32 partial ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int local = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++local) {
      int tm, tn;
      tile_coords(u / p.splits, num_m, num_n, p.raster, tm, tn);
      const int buf = local % NBUF;
      const uint32_t use = static_cast<uint32_t>(local / NBUF);
      // the epilogue idles through a tile's mainloop: poll with sleeps
      if (!mbar_wait_backoff(&tfull[buf], use & 1, abort_flag)) break;
      if (!mbar_wait_backoff(&rsfull[buf], use & 1, abort_flag)) break;
      tc_fence_after();
      const float scale = rs[buf * BM + q * 32 + lane];
      mbar_arrive(&rsempty[buf]);
      const int64_t row = static_cast<int64_t>(tm) * BM + q * 32 + lane;
      const bool row_ok = row < p.m;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * BN);
      const int64_t r = row_ok ? row : 0;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
        __syncwarp();
        tmem_ld32(tbase + c * 32, v);
        tmem_wait_ld();
        const int64_t col = static_cast<int64_t>(tn) * BN + c * 32;
        if (p.splits == 1) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] *= scale;
          if (row_ok && col < p.n) store32<TC>(static_cast<TC*>(p.c) + r * p.ldc + col, v, col, p.n);
        } else if (row_ok && col < p.n) {
          float* dst = p.part + (static_cast<int64_t>(u % p.splits) * p.m + r) * p.n + col;
          store32<float>(dst, v, col, p.n);
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
    }
  } else if (warp >= 6) {
    // ---------------- transform: loads x, r1, r2, forms h into the h ring ----------------
    const int t = threadIdx.x - 192;
    int hs = 0;
    uint32_t hphase = 0;
    int local = 0;
    bool ok = true;
    // one k-block: wait for the slot, write h, hand it to the MMA warp
    auto put = [&](const Resid3Regs<TA>& g, float* ss) {
      if (!mbar_wait_backoff(&hempty[hs], hphase ^ 1u, abort_flag)) {
        ok = false;
        return;
      }
      resid3_store<TA>(g, hbase + hs * A_BYTES, ss, t);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // h -> the tensor cores' reads
      mbar_arrive(&hfull[hs]);
      if (++hs == H) {
        hs = 0;
        hphase ^= 1u;
      }
    };
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++local) {
      int tm, tn, kb0, kb1;
      tile_coords(u / p.splits, num_m, num_n, p.raster, tm, tn);
      unit_k(u, kb0, kb1);
      const int64_t row0 = static_cast<int64_t>(tm) * BM;
      const int buf = local % NBUF;
      const uint32_t use = static_cast<uint32_t>(local / NBUF);
      float ss[4] = {0.f, 0.f, 0.f, 0.f};
      Resid3Regs<TA> g0, g1;  // two k-blocks in flight
      resid3_load<TA>(g0, x, r1, r2, row0, p.m, p.k, kb0, t);
      if (kb0 + 1 < kb1) resid3_load<TA>(g1, x, r1, r2, row0, p.m, p.k, kb0 + 1, t);
      for (int kb = kb0; kb < kb1 && ok; kb += 2) {
        put(g0, ss);
        if (kb + 2 < kb1) resid3_load<TA>(g0, x, r1, r2, row0, p.m, p.k, kb + 2, t);
        if (kb + 1 < kb1 && ok) {
          put(g1, ss);
          if (kb + 3 < kb1) resid3_load<TA>(g1, x, r1, r2, row0, p.m, p.k, kb + 3, t);
        }
      }
      if (__any_sync(0xffffffffu, !ok)) {  // warp-uniform exit before the shuffles
        ok = false;
        break;
      }
      // a row's eight chunks sit in eight consecutive lanes
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        ss[i] += __shfl_xor_sync(0xffffffffu, ss[i], 1);
        ss[i] += __shfl_xor_sync(0xffffffffu, ss[i], 2);
        ss[i] += __shfl_xor_sync(0xffffffffu, ss[i], 4);
      }
      if (!mbar_wait(&rsempty[buf], (use & 1) ^ 1u, abort_flag)) break;
      if ((t & 7) == 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = (t >> 3) + 32 * i;
          rs[buf * BM + row] = rsqrtf(ss[i] * p.inv_k + p.eps);
          const int64_t grow = row0 + row;
          // a split's partial sum, added up by the reduce pass
          if (p.splits > 1 && tn == 0 && grow < p.m) p.ss_part[static_cast<int64_t>(u % p.splits) * p.m + grow] = ss[i];
        }
      }
      mbar_arrive(&rsfull[buf]);
    }
  }

  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) {
    for (int s = 0; s < S; ++s) {
      if (issued[s] > consumed[s]) {
        volatile int never = 0;
        mbar_wait(&bfull[s], static_cast<uint32_t>((issued[s] - 1) & 1), &never);
      }
    }
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
  }
}

// Split-k finish of gemm_resid3: c[i, j] = rsqrt(sum_s ss[s][i] / k + eps) *
// sum_s part[s][i][j], splits added in order (deterministic). Four outputs
// per thread; n a multiple of 8.
template <typename TC>
__global__ void __launch_bounds__(256) resid3_reduce_kernel(const float* __restrict__ part,
                                                            const float* __restrict__ ss_part, TC* __restrict__ c,
                                                            int64_t m, int64_t n, int64_t ldc, int splits, float inv_k,
                                                            float eps) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  pdl_wait();
  pdl_trigger();
  const int64_t per_row = n / 4;
  if (idx >= m * per_row) return;
  const int64_t i = idx / per_row, j = (idx - i * per_row) * 4;
  float ss = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s = 0; s < splits; ++s) {
    ss += ss_part[static_cast<int64_t>(s) * m + i];
    const float4 v = *reinterpret_cast<const float4*>(part + (static_cast<int64_t>(s) * m + i) * n + j);
    acc.x += v.x;
    acc.y += v.y;
    acc.z += v.z;
    acc.w += v.w;
  }
  const float r = rsqrtf(ss * inv_k + eps);
  TC* dst = c + i * ldc + j;
  dst[0] = from_f<TC>(acc.x * r);
  dst[1] = from_f<TC>(acc.y * r);
  dst[2] = from_f<TC>(acc.z * r);
  dst[3] = from_f<TC>(acc.w * r);
}

// ---- attention_nkilib in one kernel: softmax(q @ k_t) @ v, bare exponential ----------
//
// The spec's softmax has no max shift, so no running maximum and no
// rescaling are needed: P = exp(S) feeds the second product directly and the
// row sums add up. One CTA (608 threads) owns 128 query rows and a range of
// 128-key blocks:
//   warp 0     TMA: the Q tile once per unit, then per key block the k_t slab
//              [D, 128 keys] (consumed as an MN-major B operand, as the GEMM
//              consumes weights), two stages, a stage refilled as soon as
//              its scores are computed;
//   warp 18    TMA: per key block the v slab [128 keys, D], two stages, each
//              refilled once its second product has read it;
//   warp 1     TMEM + MMA: S_j = Q @ k_t_j (M 128, N 128, K D) into one of two
//              TMEM score buffers, then O += P_{j-1} @ v_{j-1} (N = D) into the
//              TMEM output, so the next block's scores overlap this block's
//              softmax;
//   warps 2-17 softmax: four warps per TMEM lane quarter, each on 32 of the
//              block's 128 keys (thread = query row = TMEM lane): tcgen05.ld
//              the 32 scores, e = exp(s) (keys past s are 0), l += e in
//              fp32, and e rounded to bf16 into a 128-byte-swizzled P
//              slab (the A operand of the second product; two slabs); after
//              the last block the four partial row sums meet in shared
//              memory and the key-quarter-0 warps add them in a fixed order
//              and store O / l, or, when the keys are split over CTAs, the
//              fp32 partial O and l.
// Scores never reach global memory. Split keys are combined by
// attn_reduce_kernel in a fixed order. Every wait is bounded.
// exp of a pair of scores as 2^(x log2 e): one packed f32x2 multiply by
// log2 e and the ISA's ex2.approx (flush-to-zero: the scores' exponentials
// are never subnormal; keys past s come in as -inf and give +0).
__device__ __forceinline__ float2 exp_pair(float a, float b) {
  constexpr float kLog2e = 1.4426950408889634f;
  uint64_t x, y;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a), "f"(b));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(y) : "l"(x), "l"(static_cast<uint64_t>(__float_as_uint(kLog2e)) << 32 |
                                                          __float_as_uint(kLog2e)));
  float ya, yb, ea, eb;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(ya), "=f"(yb) : "l"(y));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(ea) : "f"(ya));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(eb) : "f"(yb));
  return make_float2(ea, eb);
}

// Two floats rounded to the operand type by one packed conversion, the
// first in the low half.
template <typename T>
__device__ __forceinline__ uint32_t cvt_pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t cvt_pack2<__nv_bfloat16>(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
template <>
__device__ __forceinline__ uint32_t cvt_pack2<__half>(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// sum += (a, b), two lanes of fp32 in one packed add
__device__ __forceinline__ void add_pair(float2& sum, float2 v) {
  uint64_t x, y, z;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(sum.x), "f"(sum.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(y) : "f"(v.x), "f"(v.y));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(z) : "l"(x), "l"(y));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(sum.x), "=f"(sum.y) : "l"(z));
}

constexpr int kAttnSoftmaxWarps = 16;
constexpr int kAttnThreads = (3 + kAttnSoftmaxWarps) * 32;  // + the v producer warp, last
constexpr int kAttnSoftmaxThreads = kAttnSoftmaxWarps * 32;

struct AttnParams {
  void* y;        // [s, D] output (splits == 1)
  float* part;    // [splits][s][D] partial O (splits > 1)
  float* lpart;   // [splits][s] partial row sums
  int s;
  int splits, kblk_per_split;  // key blocks (128 keys) per split
  uint32_t idesc_s, idesc_o;
};

template <int D, typename TA, typename TC>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_fused(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmV, AttnParams p) {
  constexpr int KA = D / 64;                 // 64-wide k-atoms of the head dim
  constexpr int Q_BYTES = KA * A_BYTES;      // [128, D]
  constexpr int KT_BYTES = KA * 2 * B_CHUNK;  // [D, 128 keys]: per k-atom two 64-key chunks
  constexpr int V_BYTES = 2 * KA * B_CHUNK;   // [128 keys, D]: per 64-key block KA chunks
  constexpr int KV_STAGE = KT_BYTES + V_BYTES;
  constexpr int P_BYTES = 2 * A_BYTES;        // [128, 128 keys] as two k-atoms
  constexpr uint32_t TMEM_COLS = 512;         // S0 | S1 | O

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = smem;
  uint8_t* skv = sq + Q_BYTES;                // 2 stages
  uint8_t* sp = skv + 2 * KV_STAGE;           // 2 P slabs
  uint64_t* bars = reinterpret_cast<uint64_t*>(sp + 2 * P_BYTES);
  uint64_t* qfull = bars;
  uint64_t* qempty = bars + 1;
  uint64_t* kfull = bars + 2;    // [2] k_t stages
  uint64_t* kempty = bars + 4;   // [2]
  uint64_t* vfull = bars + 6;    // [2] v stages
  uint64_t* vempty = bars + 8;   // [2]
  uint64_t* sfull = bars + 10;   // [2] TMEM score buffers
  uint64_t* sempty = bars + 12;  // [2]
  uint64_t* pfull = bars + 14;   // [2] P slabs
  uint64_t* pempty = bars + 16;  // [2]
  uint64_t* ofull = bars + 18;
  uint64_t* oempty = bars + 19;
  uint64_t* lbar = bars + 20;    // a unit's partial row sums are in place
  uint64_t* lfree = bars + 21;   // ... and have been read
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 22);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* issued = reinterpret_cast<int*>(tmem_slot + 2);  // [4]: k_t stages, v stages
  int* consumed = issued + 4;                           // [4]
  int* q_issued = consumed + 4;
  float* lred = reinterpret_cast<float*>(bars + 32);  // [key quarters 1..3][128 rows]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = (p.s + 127) / 128;
  const int nkb = (p.s + 127) / 128;
  const int units = nq * p.splits;
  auto unit_range = [&](int u, int& qb, int& j0, int& j1) {
    qb = u / p.splits;
    j0 = (u % p.splits) * p.kblk_per_split;
    j1 = j0 + p.kblk_per_split < nkb ? j0 + p.kblk_per_split : nkb;
  };

  if (threadIdx.x == 0) {
    mbar_init(qfull, 1);
    mbar_init(qempty, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&kfull[b], 1);
      mbar_init(&kempty[b], 1);
      mbar_init(&vfull[b], 1);
      mbar_init(&vempty[b], 1);
      mbar_init(&sfull[b], 1);
      mbar_init(&sempty[b], kAttnSoftmaxWarps);  // one arrival per softmax warp
      mbar_init(&pfull[b], kAttnSoftmaxWarps);
      mbar_init(&pempty[b], 1);
    }
    for (int i = 0; i < 4; ++i) issued[i] = consumed[i] = 0;
    mbar_init(ofull, 1);
    mbar_init(oempty, 128);
    mbar_init(lbar, kAttnSoftmaxThreads);
    mbar_init(lfree, 128);
    *q_issued = 0;
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t t_s0 = tmem_base, t_o = tmem_base + 256;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    int stage = 0;
    uint32_t ph = 0;
    int uq = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++uq) {
      int qb, j0, j1;
      unit_range(u, qb, j0, j1);
      if (!mbar_wait(qempty, (uq & 1) ^ 1u, abort_flag)) break;
      mbar_expect_tx(qfull, Q_BYTES);
#pragma unroll
      for (int a = 0; a < KA; ++a) tma_load_2d(&tmQ, qfull, sq + a * A_BYTES, a * 64, qb * 128);
      *q_issued += 1;
      bool ok = true;
      for (int j = j0; j < j1; ++j) {
        uint8_t* st = skv + stage * KV_STAGE;
        if (!mbar_wait(&kempty[stage], ph ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        mbar_expect_tx(&kfull[stage], KT_BYTES);
#pragma unroll
        for (int a = 0; a < KA; ++a)
#pragma unroll
          for (int c = 0; c < 2; ++c)
            tma_load_2d(&tmK, &kfull[stage], st + (a * 2 + c) * B_CHUNK, j * 128 + c * 64, a * 64);
        issued[stage] += 1;
        if (++stage == 2) {
          stage = 0;
          ph ^= 1u;
        }
      }
      if (!ok) break;
    }
  } else if (warp == 2 + kAttnSoftmaxWarps && lane == 0) {
    // ---------------- TMA producer of v ----------------
    // Its own thread, so a k_t slab is refilled as soon as its scores are
    // computed instead of queueing behind the v slab of the block before,
    // which waits for that block's softmax and second product.
    int stage = 0;
    uint32_t ph = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      int qb, j0, j1;
      unit_range(u, qb, j0, j1);
      bool ok = true;
      for (int j = j0; j < j1; ++j) {
        uint8_t* st = skv + stage * KV_STAGE;
        if (!mbar_wait(&vempty[stage], ph ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        mbar_expect_tx(&vfull[stage], V_BYTES);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int c = 0; c < KA; ++c)
            tma_load_2d(&tmV, &vfull[stage], st + KT_BYTES + (kb * KA + c) * B_CHUNK, c * 64, j * 128 + kb * 64);
        issued[2 + stage] += 1;
        if (++stage == 2) {
          stage = 0;
          ph ^= 1u;
        }
      }
      if (!ok) break;
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    int stage = 0, sb = 0, pb = 0;
    uint32_t ph = 0, sph = 0, pph = 0;
    int uq = 0;
    bool ok = true;
    // O += P @ v for the block whose v sits in stage `st` (phase `vp`)
    auto mma2 = [&](int st, uint32_t vp, bool first) {
      if (!mbar_wait(&pfull[pb], pph, abort_flag) || !mbar_wait(&vfull[st], vp, abort_flag)) {
        ok = false;
        return;
      }
      if (first && !mbar_wait(oempty, (uq & 1) ^ 1u, abort_flag)) {
        ok = false;
        return;
      }
      tc_fence_after();
      const uint32_t pa = smem_u32(sp + pb * P_BYTES);
      const uint32_t vb = smem_u32(skv + st * KV_STAGE + KT_BYTES);
#pragma unroll
      for (int kb = 0; kb < 2; ++kb)
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc_mma(t_o, sdesc(pa + kb * A_BYTES + k * 32, 16, 1024), sdesc(vb + kb * KA * B_CHUNK + k * 2048, B_CHUNK, 1024),
                 p.idesc_o, (first && kb == 0 && k == 0) ? 0u : 1u);
      tc_commit(&pempty[pb]);
      tc_commit(&vempty[st]);
      consumed[2 + st] += 1;
      if (++pb == 2) {
        pb = 0;
        pph ^= 1u;
      }
    };
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++uq) {
      int qb, j0, j1;
      unit_range(u, qb, j0, j1);
      if (!mbar_wait(qfull, uq & 1, abort_flag)) break;
      int prev = -1;
      uint32_t prev_ph = 0;
      for (int j = j0; j < j1 && ok; ++j) {
        if (!mbar_wait(&kfull[stage], ph, abort_flag) || !mbar_wait(&sempty[sb], sph ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t qa = smem_u32(sq);
        const uint32_t kt = smem_u32(skv + stage * KV_STAGE);
#pragma unroll
        for (int a = 0; a < KA; ++a)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc_mma(t_s0 + sb * 128, sdesc(qa + a * A_BYTES + k * 32, 16, 1024),
                   sdesc(kt + a * 2 * B_CHUNK + k * 2048, B_CHUNK, 1024), p.idesc_s, (a | k) != 0 ? 1u : 0u);
        tc_commit(&sfull[sb]);
        tc_commit(&kempty[stage]);            // this k_t slab is read
        consumed[stage] += 1;
        if (j == j1 - 1) tc_commit(qempty);  // the unit's last read of Q
        if (++sb == 2) {
          sb = 0;
          sph ^= 1u;
        }
        if (prev >= 0) mma2(prev, prev_ph, j == j0 + 1);
        prev = stage;
        prev_ph = ph;
        if (++stage == 2) {
          stage = 0;
          ph ^= 1u;
        }
      }
      if (!ok) break;
      mma2(prev, prev_ph, j1 - j0 == 1);
      if (!ok) break;
      tc_commit(ofull);
    }
  } else if (warp >= 2 && warp < 2 + kAttnSoftmaxWarps) {
    // ---------------- softmax and output ----------------
    const int q = warp & 3;             // TMEM lane quarter this warp may access
    const int kq = (warp - 2) >> 2;     // its quarter of the block's keys / O's columns
    const int row = q * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    int sb = 0, pb = 0;
    uint32_t sph = 0, pph = 0;
    int uq = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++uq) {
      int qb, j0, j1;
      unit_range(u, qb, j0, j1);
      float l = 0.f;
      bool ok = true;
      for (int j = j0; j < j1; ++j) {
        if (!mbar_wait_backoff(&sfull[sb], sph, abort_flag) ||
            !mbar_wait_backoff(&pempty[pb], pph ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float v[32];
        __syncwarp();
        tmem_ld32(t_s0 + sb * 128 + lane_off + kq * 32, v);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();  // every lane's scores are in registers: one arrival for the warp
        if (lane == 0) mbar_arrive(&sempty[sb]);
        const int key0 = j * 128 + kq * 32;
        if (key0 + 32 > p.s) {  // the ragged last block: keys past s weigh nothing
#pragma unroll
          for (int kk = 0; kk < 32; ++kk)
            if (key0 + kk >= p.s) v[kk] = -INFINITY;
        }
        uint4 pk[4];
        float2 lsum = make_float2(0.f, 0.f);  // this block's exponentials, in fp32 before rounding
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 8; e += 2) {  // two exponentials, one packed multiply, add and conversion
            const float2 ex = exp_pair(v[t * 8 + e], v[t * 8 + e + 1]);
            add_pair(lsum, ex);
            w[e / 2] = cvt_pack2<TA>(ex.x, ex.y);
          }
          pk[t] = make_uint4(w[0], w[1], w[2], w[3]);
        }
        l += lsum.x + lsum.y;
        uint8_t* line = sp + pb * P_BYTES + (kq >> 1) * A_BYTES + row * 128;
        const int cb = (kq & 1) * 4;
#pragma unroll
        for (int t = 0; t < 4; ++t) *reinterpret_cast<uint4*>(line + (((cb + t) ^ (row & 7)) * 16)) = pk[t];
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // P -> the tensor cores' reads
        __syncwarp();  // the warp's P lines are written: one arrival for the warp
        if (lane == 0) mbar_arrive(&pfull[pb]);
        if (++sb == 2) {
          sb = 0;
          sph ^= 1u;
        }
        if (++pb == 2) {
          pb = 0;
          pph ^= 1u;
        }
      }
      if (!ok) break;
      // the row's four partial sums meet in shared memory; the key-quarter 0
      // warps add them in key order and write the output
      if (kq != 0) {
        if (!mbar_wait(lfree, (uq & 1) ^ 1u, abort_flag)) break;  // the last unit's sums were read
        lred[(kq - 1) * 128 + row] = l;
      }
      mbar_arrive(lbar);
      if (kq != 0) continue;
      if (!mbar_wait_backoff(lbar, uq & 1, abort_flag)) break;
      l = ((l + lred[row]) + lred[128 + row]) + lred[256 + row];
      mbar_arrive(lfree);
      if (!mbar_wait_backoff(ofull, uq & 1, abort_flag)) break;
      tc_fence_after();
      const int64_t grow = static_cast<int64_t>(qb) * 128 + row;
      const bool row_ok = grow < p.s;
      const int split = u % p.splits;
      const float inv_l = 1.0f / l;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        float v[32];
        __syncwarp();
        tmem_ld32(t_o + lane_off + c * 32, v);
        tmem_wait_ld();
        if (!row_ok) continue;
        if (p.splits == 1) {
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] *= inv_l;
          store32<TC>(static_cast<TC*>(p.y) + grow * D + c * 32, v, c * 32, D);
        } else {
          store32<float>(p.part + (static_cast<int64_t>(split) * p.s + grow) * D + c * 32, v, c * 32, D);
        }
      }
      if (p.splits > 1 && row_ok) p.lpart[static_cast<int64_t>(split) * p.s + grow] = l;
      tc_fence_before();
      mbar_arrive(oempty);
    }
  }

  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) {
    // copies issued but not consumed may still land: wait for them (bounded)
    for (int s = 0; s < 4; ++s) {
      if (issued[s] > consumed[s]) {
        volatile int never = 0;
        mbar_wait(s < 2 ? &kfull[s] : &vfull[s - 2], static_cast<uint32_t>((issued[s] - 1) & 1), &never);
      }
    }
    if (*q_issued > 0) {
      volatile int never = 0;
      mbar_wait(qfull, static_cast<uint32_t>((*q_issued - 1) & 1), &never);
    }
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
  }
}

// Split keys of attn_fused: y[i, :] = sum_s part[s][i, :] / sum_s l[s][i],
// splits added in order. Four outputs per thread.
template <typename TC>
__global__ void __launch_bounds__(256) attn_reduce_kernel(const float* __restrict__ part,
                                                          const float* __restrict__ lpart, TC* __restrict__ y,
                                                          int64_t s, int64_t d, int splits) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  pdl_wait();
  pdl_trigger();
  const int64_t per_row = d / 4;
  if (idx >= s * per_row) return;
  const int64_t i = idx / per_row, j = (idx - i * per_row) * 4;
  float l = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k = 0; k < splits; ++k) {
    l += lpart[static_cast<int64_t>(k) * s + i];
    const float4 v = *reinterpret_cast<const float4*>(part + (static_cast<int64_t>(k) * s + i) * d + j);
    acc.x += v.x;
    acc.y += v.y;
    acc.z += v.z;
    acc.w += v.w;
  }
  const float r = 1.0f / l;
  TC* dst = y + i * d + j;
  dst[0] = from_f<TC>(acc.x * r);
  dst[1] = from_f<TC>(acc.y * r);
  dst[2] = from_f<TC>(acc.z * r);
  dst[3] = from_f<TC>(acc.w * r);
}

// ---- variant 2: CTA pairs (tcgen05 cta_group::2) ------------------------------------
//
// A cluster of two CTAs on two SMs computes a 256 x BN tile with one
// tcgen05.mma.cta_group::2 (M = 256) per K = 16 step, issued by the even
// ("leader") CTA: CTA r holds A rows [128 r, 128 r + 128) and B columns
// [BN/2 r, BN/2 r + BN/2) of the tile in its own shared memory, and its TMEM
// receives its 128 rows of the fp32 accumulator. Each CTA therefore stages
// half of B per k-block, halving B's shared-memory and L2 traffic per CTA.
// For SILU_GATE the leader holds the gate columns and the peer the matching up
// columns, so each CTA's TMEM again holds gate | up for its rows.
//
// Synchronisation: both CTAs' TMA loads (cp.async.bulk.tensor ... cta_group::2,
// no multicast) complete transaction bytes on the leader's `full` barrier,
// which the leader's producer arms with both CTAs' bytes; the leader's MMA
// thread frees a stage by committing to the `empty` barrier of each CTA, and
// announces a finished accumulator by committing to each CTA's `tmem_full`;
// each CTA's epilogue warps release a TMEM buffer by arriving on the leader's
// `tmem_empty`. Every wait is bounded as in the one-CTA kernel. A cluster barrier
// precedes exit, so no CTA leaves while its peer may still address it.

__device__ __forceinline__ uint32_t mapa_u32(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr, uint32_t count) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(cluster_addr), "r"(count)
               : "memory");
}

__device__ __forceinline__ void tma_load_2d_pair(const CUtensorMap* map, uint32_t leader_bar, void* dst, int c0,
                                                 int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tc_commit_to(uint32_t cluster_bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_bar)
               : "memory");
}

__device__ __forceinline__ void tc_mma_pair(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}

template <int BN, int EPI, typename TC>
__global__ void __launch_bounds__(192, 1)
    gemm_tcgen05_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmB2, GemmParams p) {
  constexpr int BH = BN / 2;                 // B columns staged per CTA
  constexpr int B_BYTES = BH * BK * 2;
  constexpr int STAGE = A_BYTES + B_BYTES;
  constexpr int BN_OUT = EPI == AXON_EPI_SILU_GATE ? BN / 2 : BN;
  constexpr uint32_t TMEM_COLS = 2 * BN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * STAGE);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;  // leader: all issued MMAs have retired
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* issued = reinterpret_cast<int*>(tmem_slot + 2);

  uint32_t rank;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  const bool leader = rank == 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (p.m + 2 * BM - 1) / (2 * BM);
  const int num_n = (p.n + BN_OUT - 1) / BN_OUT;
  const int tiles = num_m * num_n;
  const int kblocks = (p.k + BK - 1) / BK;
  const int pair_id = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);  // one arrival per epilogue warp of each CTA
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    *issued = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    tc_fence_before();
  }
  __syncthreads();
  cluster_barrier();  // both CTAs' barriers are initialised before either is addressed remotely
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    int stage = 0;
    uint32_t phase = 0;
    for (int t = pair_id; t < tiles; t += num_pairs) {
      int tm, tn;
      tile_coords(t, num_m, num_n, p.raster, tm, tn);
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) goto producer_done;
        const uint32_t leader_full = mapa_u32(smem_u32(&full[stage]), 0);
        if (leader) mbar_expect_tx(&full[stage], 2 * STAGE);
        uint8_t* sa = smem + stage * STAGE;
        uint8_t* sb = sa + A_BYTES;
        tma_load_2d_pair(&tmA, leader_full, sa, kb * BK, tm * 2 * BM + static_cast<int>(rank) * BM);
        if constexpr (EPI == AXON_EPI_SILU_GATE) {
          const CUtensorMap* mp = leader ? &tmB : &tmB2;  // gate columns on the leader, up on the peer
#pragma unroll
          for (int j = 0; j < BH / 64; ++j)
            tma_load_2d_pair(mp, leader_full, sb + j * B_CHUNK, tn * BN_OUT + j * 64, kb * BK);
        } else {
          const int kb_b = p.b_kwrap > 0 ? (kb * BK) % p.b_kwrap : kb * BK;
#pragma unroll
          for (int j = 0; j < BH / 64; ++j)
            tma_load_2d_pair(&tmB, leader_full, sb + j * B_CHUNK, tn * BN + static_cast<int>(rank) * BH + j * 64,
                             kb_b);
        }
        *issued += 1;
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  producer_done:;
  } else if (warp == 1 && lane == 0 && leader) {
    // ---------------- MMA issuer (leader only) ----------------
    int stage = 0;
    uint32_t phase = 0;
    int local = 0;
    for (int t = pair_id; t < tiles; t += num_pairs, ++local) {
      const int buf = local & 1;
      if (!mbar_wait(&tempty[buf], ((local >> 1) & 1) ^ 1u, abort_flag)) break;
      tc_fence_after();
      const uint32_t d = tmem_base + static_cast<uint32_t>(buf * BN);
      bool ok = true;
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + stage * STAGE);
        const uint32_t sb = sa + A_BYTES;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          const uint64_t ad = sdesc(sa + k * 32, 16, 1024);
          const uint64_t bd = sdesc(sb + k * 2048, B_CHUNK, 1024);
          tc_mma_pair(d, ad, bd, p.idesc, (kb | k) != 0);
        }
        tc_commit_to(smem_u32(&empty[stage]));
        tc_commit_to(mapa_u32(smem_u32(&empty[stage]), 1));
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      tc_commit_to(smem_u32(&tfull[buf]));
      tc_commit_to(mapa_u32(smem_u32(&tfull[buf]), 1));
    }
    // TMEM is released only after every MMA this thread issued has retired
    tc_commit_to(smem_u32(drain));
    volatile int never = 0;
    mbar_wait(drain, 0, &never);
  } else if (warp >= 2) {
    // ---------------- epilogue (both CTAs, their own 128 rows) ----------------
    const int q = warp & 3;
    int local = 0;
    TC* C = static_cast<TC*>(p.c);
    for (int t = pair_id; t < tiles; t += num_pairs, ++local) {
      int tm, tn;
      tile_coords(t, num_m, num_n, p.raster, tm, tn);
      const int buf = local & 1;
      if (!mbar_wait(&tfull[buf], (local >> 1) & 1, abort_flag)) break;
      tc_fence_after();
      const int64_t row = static_cast<int64_t>(tm) * 2 * BM + static_cast<int64_t>(rank) * BM + q * 32 + lane;
      const bool row_ok = row < p.m;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * BN);
      TC* crow = out_row<EPI, TC>(p, C, row_ok ? row : 0);
      float scale = 1.f;
      if constexpr (EPI == AXON_EPI_ROWSCALE) scale = row_ok ? p.row_scale[row] : 0.f;
      if constexpr (EPI == AXON_EPI_SILU_GATE) {
#pragma unroll 1
        for (int c = 0; c < BN_OUT / 32; ++c) {
          float g[32], u[32];
          __syncwarp();
          tmem_ld32(tbase + c * 32, g);
          tmem_ld32(tbase + BN_OUT + c * 32, u);
          tmem_wait_ld();
          const int64_t col = static_cast<int64_t>(tn) * BN_OUT + c * 32;
#pragma unroll
          for (int j = 0; j < 32; ++j) g[j] = g[j] / (1.0f + __expf(-g[j])) * u[j];
          if (row_ok && col < p.n) {
            if (p.terms <= 1) {
              store32<TC>(crow + col, g, col, p.n);
            } else {
#pragma unroll 1
              for (int tt = 0; tt < p.terms; ++tt) {
                float part[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                  part[j] = to_f(from_f<TC>(g[j]));
                  g[j] -= part[j];
                }
                store32<TC>(crow + tt * p.term_stride + col, part, col, p.n);
              }
            }
          }
        }
      } else if constexpr (EPI == kEpiPeer) {
        __half* stg = reinterpret_cast<__half*>(smem + S * STAGE + 256) + q * 32 * kPeerStageHalves;
        peer_store_tile<BN>(p, stg,
                            tbase, static_cast<int64_t>(tm) * 2 * BM + static_cast<int64_t>(rank) * BM + q * 32,
                            static_cast<int64_t>(tn) * BN, lane);
      } else {
        float psum = 0.f;  // EXP: this row's sum over the tile, of the values as stored
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          __syncwarp();
          tmem_ld32(tbase + c * 32, v);
          tmem_wait_ld();
          const int64_t col = static_cast<int64_t>(tn) * BN + c * 32;
          if constexpr (EPI == AXON_EPI_ROWSCALE) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] *= scale;
          }
          if constexpr (EPI == AXON_EPI_EXP) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              v[j] = to_f(from_f<TC>(__expf(v[j])));
              if (col + j < p.n) psum += v[j];
            }
          }
          if (row_ok && col < p.n) store32<TC>(crow + col, v, col, p.n);
        }
        if constexpr (EPI == AXON_EPI_EXP) {
          if (row_ok && p.row_part != nullptr) p.row_part[tn * p.part_ld + row] = psum;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_u32(smem_u32(&tempty[buf]), 0), 1);
    }
  }

  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag && *issued > 0) {
    // copies issued by this CTA may still be landing: give them time before
    // the pair leaves (this path only runs after a wait gave up)
    for (int i = 0; i < 1000; ++i) __nanosleep(1000);
  }
  cluster_barrier();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
  }
}

// ---- fused SwiGLU: both GEMMs (and, for tensor parallelism, the reduction) in one kernel
//
// y = (silu(x @ W_gate) * (x @ W_up)) @ W_down with the f16 activation of
// precision mode 4. Phase-A tiles (256 rows x 128 activation columns: gate and
// up accumulators side by side in TMEM, as gemm_tcgen05_pair's SiLU-gate
// epilogue) write the activation to global memory; phase-B tiles (256 x 256
// of y, K = the intermediate size) read it back through TMA. Pairs claim tiles
// from one atomic counter, all phase-A tiles before any phase-B tile, so a
// pair that finishes its part of phase A moves straight on to phase B instead
// of idling through the last partial wave. A phase-B tile's producers wait
// (bounded) until every phase-A tile of its 256-row block has been written:
// each phase-A epilogue warp adds one to its row block's counter after its
// stores (8 per tile). Tiles are claimed in order by running CTAs and phase-A
// tiles never wait, so every wait ends without assuming co-residency.
//
// Modes: kMlpLocal writes y; kMlpScatter writes each f16 partial row of y to
// its owner rank's inbox (axon_tp_mlp_partial). kMlpStep (axon_tp_mlp_step)
// and kMlpStepMC (axon_tp_mlp_step_multicast) run a whole tensor-parallel
// step: rows are owned in 8-row granules dealt to the ranks in turn, and two
// reduction warps per CTA (warps 6 and 7, beside the tile roles) claim units
// of this rank's rows -- one row x kStepCols columns, in row-block order --
// wait (bounded) until every rank's partials of the unit's 256-row block have
// arrived, and resolve the all-reduce for them while the GEMM tiles go on:
//   kMlpStep    each phase-B epilogue warp writes its f16 partial rows into
//               the owners' inboxes over NVLink and releases them into the
//               owners' arrival counts; a reduction warp sums the world
//               inbox copies in fp32 in rank order, rounds once to bf16 and
//               stores the row into every rank's output;
//   kMlpStepMC  each phase-B epilogue warp writes its f16 partial rows into
//               this rank's own partial buffer (bound to an NVLink multicast
//               object) and releases them into every rank's arrival counts;
//               a reduction warp reads each 16-byte packet of an owned row
//               once through the multicast address with multimem.ld_reduce
//               (the NVSwitch adds the world copies, accumulating in fp32),
//               rounds to bf16 and stores it once with multimem.st to the
//               output's multicast address, which the switch writes into
//               every rank's output.
// At the end each reduction warp adds its unit count to every rank's done
// count. A reduction wait depends only on phase-B tiles (of every rank),
// which depend only on their own phase A: no cycle across GPUs. Arrival and
// done counts accumulate over steps (epoch * per-step count), so nothing is
// reset between steps.
//
// The leader's producer thread claims each tile and publishes its id to both
// CTAs through a ring of shared-memory slots (the peer's by a distributed
// shared-memory store and a remote mbarrier arrival); each consumer role
// (the peer's producer, the leader's MMA thread, the epilogue warps of both
// CTAs) frees a slot by arriving on the leader's slot barrier.

constexpr int kSchedRing = 8;
constexpr int kMlpLocal = 0, kMlpScatter = 1, kMlpStep = 2, kMlpStepMC = 3;
constexpr int kStepCols = 1024;      // reduction unit: one owned row x this many columns
constexpr int kStepWarps = 2;        // reduction warps per CTA (kMlpStep, kMlpStepMC)

__host__ __device__ constexpr int mlp_threads(int mode) { return mode >= kMlpStep ? 192 + 32 * kStepWarps : 192; }

struct MlpParams {
  void* c;                  // kMlpLocal: y [m, ldc]
  void* peers[kMaxPeers];   // kMlpScatter / kMlpStep: each owner's inbox [world][m / world][n2] f16
  int peer_rank;
  int rows_per_owner;
  int world;
  __half* act;              // [m, n1] f16
  int* ready;               // [row blocks] phase-A epilogue warps done, the tile counter, the
                            // reduction warps' unit counter, [row blocks] phase-B warps done
  int m, n1, k1, n2;
  int64_t ldc;
  int stages;
  uint32_t idesc_a, idesc_b;
  int max_ctas;
  // kMlpStep
  int* arrive[kMaxPeers];   // each owner's arrival counts [row blocks]
  int* done[kMaxPeers];     // each rank's done count
  const __half* inbox;      // this rank's inbox
  void* y[kMaxPeers];       // each rank's output [m, n2] bf16
  int epoch;
  int group;                // row blocks per group of the tile order
  // kMlpStepMC
  __half* part;             // this rank's partial of y [m, n2] f16 (bound to a multicast object)
  const __half* part_mc;    // the partials' multicast address
  __nv_bfloat16* y_mc;      // the outputs' multicast address
};

__device__ __forceinline__ int ld_acquire_gpu_s32(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_sys_add(int* p, int v) {
  asm volatile("red.release.sys.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void st_shared_cluster_s32(uint32_t addr, int v) {
  asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

// Bounded wait until *ctr (raised by other CTAs of this GPU) reaches target
// (wrap-safe).
__device__ __forceinline__ bool wait_count(const int* ctr, int target, volatile int* abort_flag) {
  if (ld_acquire_gpu_s32(ctr) - target >= 0) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (ld_acquire_gpu_s32(ctr) - target >= 0) return true;
    if ((i & 15) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > kTimeoutNs) {
        *abort_flag = 1;
        atomicExch(&g_gemm_error, AXON_E_TIMEOUT);
        return false;
      }
    }
    __nanosleep(64);
  }
}

// Bounded wait for the reduction warps, whose counters other GPUs raise
// late in the kernel: relaxed system-scope polls with a growing sleep (up to
// 2 us) so the waiting warps take next to no issue slots or memory
// bandwidth from the tile roles on the same SM, and one acquire fence once
// the count is reached.
__device__ __forceinline__ bool wait_count_idle(const int* ctr, int target, volatile int* abort_flag) {
  auto ld = [&]() {
    int v;
    asm volatile("ld.relaxed.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
    return v;
  };
  const uint64_t t0 = globaltimer();
  uint32_t nap = 64;
  for (uint32_t i = 0;; ++i) {
    if (ld() - target >= 0) {
      asm volatile("fence.acq_rel.sys;" ::: "memory");
      return true;
    }
    if ((i & 7) == 7) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > kTimeoutNs) {
        *abort_flag = 1;
        atomicExch(&g_gemm_error, AXON_E_TIMEOUT);
        return false;
      }
    }
    __nanosleep(nap);
    if (nap < 2048) nap <<= 1;
  }
}

// mbar_wait with cluster-scope acquire: for barriers a thread of the other
// CTA of the pair arrives on after writing this CTA's shared memory.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  auto try_once = [&]() {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
  };
  if (try_once()) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (try_once()) return true;
    if ((i & 127) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > kTimeoutNs) {
        *abort_flag = 1;
        atomicExch(&g_gemm_error, AXON_E_TIMEOUT);
        return false;
      }
    }
  }
}

struct MlpTile {
  int kind;    // 0 = phase A (gate/up), 1 = B (down)
  int r, c;    // 256-row block, column tile
};

struct MlpGrid {
  int rb, ta_row, tb_row, group;
  __device__ int tiles() const { return rb * (ta_row + tb_row); }  // phases A and B: the ring's tiles
};

// Row groups of `group` 256-row blocks; the tile sequence is A0, A1, B0, A2,
// B1, ..., A(n-1), B(n-2), B(n-1): a group's down-projection tiles come after
// the next group's gate/up tiles have been claimed, so their activation rows
// are complete by the time they are loaded, and the down projection of early
// groups (and, in a tensor-parallel step, its traffic over NVLink) overlaps
// later groups' gate/up tiles. Gate/up tiles are column-major inside a group
// (a wave shares weight columns among the group's row blocks), down tiles
// row-major.
__device__ __forceinline__ MlpTile mlp_tile(int t, const MlpGrid& g) {
  const int GR = g.group;
  const int ng = (g.rb + GR - 1) / GR;
  MlpTile x;
  x.kind = 1;
  x.r = 0;
  x.c = 0;
  for (int k = 0; k <= ng; ++k) {
    if (k < ng) {
      const int gr = g.rb - k * GR < GR ? g.rb - k * GR : GR;
      const int sz = gr * g.ta_row;
      if (t < sz) {
        x.kind = 0;
        x.r = k * GR + t % gr;
        x.c = t / gr;
        return x;
      }
      t -= sz;
    }
    if (k >= 1) {
      const int j = k - 1;
      const int gr = g.rb - j * GR < GR ? g.rb - j * GR : GR;
      const int sz = gr * g.tb_row;
      if (t < sz) {
        x.kind = 1;
        x.r = j * GR + t / g.tb_row;
        x.c = t % g.tb_row;
        return x;
      }
      t -= sz;
    }
  }
  return x;  // not reached for t < tiles()
}

// 16 bytes through a multicast address: the NVSwitch reads the packet from
// every GPU bound to the object and returns the sum (f16 pairs added in
// fp32, rounded once to f16).
__device__ __forceinline__ uint4 multimem_ld_add_f16x8(const __half* mc) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}

// 16 bytes stored once to a multicast address; the switch writes them into
// every GPU bound to the object (bits only: the .f32 form is the 16-byte
// store).
__device__ __forceinline__ void multimem_st_b128(void* mc, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// The reduction warps of a whole tensor-parallel step (kMlpStep, kMlpStepMC;
// see above). Units are claimed from counters[rb + 1] in order, so the
// row blocks a warp waits for only grow; a wait that gives up aborts the CTA
// and records AXON_E_TIMEOUT.
template <int MODE>
__device__ void mlp_step_reduce_warp(const MlpParams& p, int rb, int lane, volatile int* abort_flag) {
  const int W = p.world;
  const int rows_local = p.m / W;
  const int rows_per_block = 256 / W;
  const int chunks = (p.n2 + kStepCols - 1) / kStepCols;
  const int units = rows_local * chunks;
  const int tb_row = (p.n2 + 255) / 256;
  // arrival count of a complete row block: kMlpStep counts granules into the
  // owner (32 per tile, over the world ranks' tiles); kMlpStepMC counts one
  // per rank (its last warp of the block publishes it)
  const int per_block = MODE == kMlpStepMC ? W : 32 * tb_row;
  const int target = p.epoch * per_block;
  const int64_t slot = static_cast<int64_t>(rows_local) * p.n2;
  int* ctr = p.ready + rb + 1;
  int seen = -1, mine = 0;
  bool ok = true;
  for (;;) {
    int u = 0;
    if (lane == 0) u = *abort_flag ? units : atomicAdd(ctr, 1);
    u = __shfl_sync(0xffffffffu, u, 0);
    if (u >= units) break;
    const int lr = u / chunks, c = u - (u / chunks) * chunks;
    const int blk = lr / rows_per_block;
    if (blk > seen) {
      int got = 1;
      if (lane == 0) got = wait_count_idle(p.arrive[p.peer_rank] + blk, target, abort_flag) ? 1 : 0;
      got = __shfl_sync(0xffffffffu, got, 0);
      if (!got) {
        ok = false;
        break;
      }
      seen = blk;
      if constexpr (MODE == kMlpStepMC) asm volatile("fence.proxy.alias;" ::: "memory");
    }
    const int col0 = c * kStepCols;
    const int packets = (p.n2 - col0 < kStepCols ? p.n2 - col0 : kStepCols) / 8;
    const int64_t grow = (static_cast<int64_t>(lr >> 3) * W + p.peer_rank) * 8 + (lr & 7);
    if constexpr (MODE == kMlpStepMC) {
      // four packets per lane in flight, each the world-sum of one 16-byte piece
      for (int pk0 = lane; pk0 < packets; pk0 += 128) {
        uint4 v[4];
#pragma unroll
        for (int h = 0; h < 4; ++h)
          if (pk0 + 32 * h < packets) v[h] = multimem_ld_add_f16x8(p.part_mc + grow * p.n2 + col0 + (pk0 + 32 * h) * 8);
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          if (pk0 + 32 * h >= packets) break;
          const __half* hv = reinterpret_cast<const __half*>(&v[h]);
          Vec<__nv_bfloat16> o;
#pragma unroll
          for (int e = 0; e < 8; ++e) o.e[e] = __float2bfloat16_rn(__half2float(hv[e]));
          multimem_st_b128(p.y_mc + grow * p.n2 + col0 + (pk0 + 32 * h) * 8, o.u);
        }
      }
    } else {
      const int64_t lrow = static_cast<int64_t>(lr) * p.n2 + col0;
      // two packets per lane in flight, every rank's copy loaded before any sum
      for (int pk0 = lane; pk0 < packets; pk0 += 64) {
        Vec<__half> v[2][kMaxPeers];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int pk = pk0 + 32 * h;
#pragma unroll
          for (int s2 = 0; s2 < kMaxPeers; ++s2)  // written by other GPUs: loads that skip cached copies
            if (s2 < W && pk < packets)
              v[h][s2].u = __ldcv(reinterpret_cast<const uint4*>(p.inbox + s2 * slot + lrow + pk * 8));
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int pk = pk0 + 32 * h;
          if (pk >= packets) break;
          float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int s2 = 0; s2 < kMaxPeers; ++s2)  // fixed rank order: the same sum on every run
            if (s2 < W)
#pragma unroll
              for (int e = 0; e < 8; ++e) acc[e] += __half2float(v[h][s2].e[e]);
          Vec<__nv_bfloat16> o;
#pragma unroll
          for (int e = 0; e < 8; ++e) o.e[e] = __float2bfloat16_rn(acc[e]);
          for (int d = 0; d < W; ++d)
            st_vec(static_cast<__nv_bfloat16*>(p.y[d]) + grow * p.n2 + col0 + pk * 8, o);
        }
      }
    }
    ++mine;
  }
  // publish this warp's rows: every store before the done counts (system scope)
  if constexpr (MODE == kMlpStepMC) asm volatile("fence.proxy.alias;" ::: "memory");
  __threadfence_system();
  __syncwarp();
  if (ok && mine > 0 && lane < W && !*abort_flag)
    asm volatile("red.relaxed.sys.global.add.s32 [%0], %1;" ::"l"(p.done[lane]), "r"(mine) : "memory");
}

template <typename TC, int MODE>
__global__ void __launch_bounds__(mlp_threads(MODE), 1)
    swiglu_fused_pair(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmWg,
                      const __grid_constant__ CUtensorMap tmWu, const __grid_constant__ CUtensorMap tmAct,
                      const __grid_constant__ CUtensorMap tmWd, MlpParams p) {
  constexpr int BN = 256, BH = 128;
  constexpr int B_BYTES = BH * BK * 2;
  constexpr int STAGE = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = 2 * BN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * STAGE);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* sfull = drain + 1;              // schedule ring: tile id published
  uint64_t* sempty = sfull + kSchedRing;    // leader only: every consumer has read the slot
  int* sched = reinterpret_cast<int*>(sempty + kSchedRing);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sched + kSchedRing);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  uint32_t rank;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  const bool leader = rank == 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  MlpGrid grid;
  grid.rb = (p.m + 2 * BM - 1) / (2 * BM);
  grid.ta_row = (p.n1 + BH - 1) / BH;
  grid.tb_row = (p.n2 + BN - 1) / BN;
  grid.group = p.group;
  const int tiles = grid.tiles();
  const int kb_a = (p.k1 + BK - 1) / BK, kb_b = (p.n1 + BK - 1) / BK;
  int* counter = p.ready + grid.rb;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
    }
    mbar_init(drain, 1);
    for (int s = 0; s < kSchedRing; ++s) {
      mbar_init(&sfull[s], 1);
      mbar_init(&sempty[s], 10);  // leader MMA + 4 + 4 epilogue warps + the peer's producer
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    tc_fence_before();
  }
  __syncthreads();
  cluster_barrier();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Consumer side of the schedule ring: the id of this role's i-th tile (-1 = done).
  auto next_tile = [&](int i, bool arrive_lane) -> int {
    const int slot = i % kSchedRing;
    if (!mbar_wait_cluster(&sfull[slot], static_cast<uint32_t>((i / kSchedRing) & 1), abort_flag)) return -1;
    const int t = *reinterpret_cast<volatile int*>(&sched[slot]);
    if (arrive_lane) mbar_arrive_cluster(mapa_u32(smem_u32(&sempty[slot]), 0), 1);
    return t;
  };

  if (warp == 0 && lane == 0) {
    // ---------------- producers (the leader's also claims tiles) ----------------
    int stage = 0;
    uint32_t phase = 0;
    for (int i = 0;; ++i) {
      int t;
      if (leader) {
        const int slot = i % kSchedRing;
        if (!mbar_wait_cluster(&sempty[slot], static_cast<uint32_t>(((i / kSchedRing) & 1) ^ 1), abort_flag)) break;
        t = atomicAdd(counter, 1);
        if (t >= tiles) t = -1;
        sched[slot] = t;
        st_shared_cluster_s32(mapa_u32(smem_u32(&sched[slot]), 1), t);
        mbar_arrive(&sfull[slot]);
        mbar_arrive_cluster(mapa_u32(smem_u32(&sfull[slot]), 1), 1);
      } else {
        t = next_tile(i, true);
      }
      if (t < 0) break;
      const MlpTile x = mlp_tile(t, grid);
      if (x.kind == 1) {
        if (!wait_count(p.ready + x.r, 8 * grid.ta_row, abort_flag)) break;
        asm volatile("fence.proxy.async.global;" ::: "memory");  // generic-proxy activation stores -> TMA reads
      }
      const int kblocks = x.kind == 0 ? kb_a : kb_b;
      const int row = x.r * 2 * BM + static_cast<int>(rank) * BM;
      bool ok = true;
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t leader_full = mapa_u32(smem_u32(&full[stage]), 0);
        if (leader) mbar_expect_tx(&full[stage], 2 * STAGE);
        uint8_t* sa = smem + stage * STAGE;
        uint8_t* sb = sa + A_BYTES;
        if (x.kind == 0) {
          tma_load_2d_pair(&tmX, leader_full, sa, kb * BK, row);
          const CUtensorMap* mp = leader ? &tmWg : &tmWu;  // gate columns on the leader, up on the peer
#pragma unroll
          for (int j = 0; j < BH / 64; ++j) tma_load_2d_pair(mp, leader_full, sb + j * B_CHUNK, x.c * BH + j * 64, kb * BK);
        } else {
          tma_load_2d_pair(&tmAct, leader_full, sa, kb * BK, row);
#pragma unroll
          for (int j = 0; j < BH / 64; ++j)
            tma_load_2d_pair(&tmWd, leader_full, sb + j * B_CHUNK, x.c * BN + static_cast<int>(rank) * BH + j * 64,
                             kb * BK);
        }
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
    }
  } else if (warp == 1 && lane == 0 && leader) {
    // ---------------- MMA issuer (leader only) ----------------
    int stage = 0;
    uint32_t phase = 0;
    int mm = 0;  // tiles that use TMEM (phases A and B)
    for (int i = 0;; ++i) {
      const int t = next_tile(i, true);
      if (t < 0) break;
      const MlpTile x = mlp_tile(t, grid);
      const int buf = mm & 1;
      if (!mbar_wait(&tempty[buf], ((mm >> 1) & 1) ^ 1u, abort_flag)) break;
      ++mm;
      tc_fence_after();
      const uint32_t d = tmem_base + static_cast<uint32_t>(buf * BN);
      const int kblocks = x.kind == 0 ? kb_a : kb_b;
      const uint32_t idesc = x.kind == 0 ? p.idesc_a : p.idesc_b;
      bool ok = true;
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + stage * STAGE);
        const uint32_t sb = sa + A_BYTES;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          const uint64_t ad = sdesc(sa + k * 32, 16, 1024);
          const uint64_t bd = sdesc(sb + k * 2048, B_CHUNK, 1024);
          tc_mma_pair(d, ad, bd, idesc, (kb | k) != 0);
        }
        tc_commit_to(smem_u32(&empty[stage]));
        tc_commit_to(mapa_u32(smem_u32(&empty[stage]), 1));
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      tc_commit_to(smem_u32(&tfull[buf]));
      tc_commit_to(mapa_u32(smem_u32(&tfull[buf]), 1));
    }
    tc_commit_to(smem_u32(drain));
    volatile int never = 0;
    mbar_wait(drain, 0, &never);
  } else if (warp >= 2 && warp < 6) {
    // ---------------- epilogue (both CTAs, their own 128 rows) ----------------
    const int q = warp & 3;
    int mm = 0;
    for (int i = 0;; ++i) {
      const int t = next_tile(i, false);  // every lane reads the slot ...
      __syncwarp();                       // ... before one arrival frees it for the whole warp
      if (lane == 0) mbar_arrive_cluster(mapa_u32(smem_u32(&sempty[i % kSchedRing]), 0), 1);
      if (t < 0) break;
      const MlpTile x = mlp_tile(t, grid);
      const int buf = mm & 1;
      const uint32_t tph = (mm >> 1) & 1;
      ++mm;
      if (!mbar_wait(&tfull[buf], tph, abort_flag)) break;
      tc_fence_after();
      const int64_t row0 = static_cast<int64_t>(x.r) * 2 * BM + static_cast<int64_t>(rank) * BM + q * 32;
      const int64_t row = row0 + lane;
      const bool row_ok = row < p.m;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * BN);
      if (x.kind == 0) {
        __half* arow = p.act + (row_ok ? row : 0) * static_cast<int64_t>(p.n1);
#pragma unroll 1
        for (int c = 0; c < BH / 32; ++c) {
          float g[32], u[32];
          __syncwarp();
          tmem_ld32(tbase + c * 32, g);
          tmem_ld32(tbase + BH + c * 32, u);
          tmem_wait_ld();
          const int64_t col = static_cast<int64_t>(x.c) * BH + c * 32;
#pragma unroll
          for (int j = 0; j < 32; ++j) g[j] = g[j] / (1.0f + __expf(-g[j])) * u[j];
          if (row_ok && col < p.n1) store32<__half>(arow + col, g, col, p.n1);
        }
        // this warp's rows of the activation are written: publish them to the
        // phase-B producers (TMA reads them through the async proxy)
        asm volatile("fence.proxy.async.global;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          __threadfence();
          atomicAdd(p.ready + x.r, 1);
        }
      } else if constexpr (MODE == kMlpStepMC) {
        // this rank's partial rows into its own (multicast-bound) buffer, then
        // released into every rank's arrival count of the row block
        __half* prow = p.part + (row_ok ? row : 0) * static_cast<int64_t>(p.n2);
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          __syncwarp();
          tmem_ld32(tbase + c * 32, v);
          tmem_wait_ld();
          const int64_t col = static_cast<int64_t>(x.c) * BN + c * 32;
          if (row_ok && col < p.n2) store32<__half>(prow + col, v, col, p.n2);
        }
        // Count the warp's rows into this rank's row-block count (GPU scope,
        // release); the warp that completes the block's count acquires the
        // other warps' stores and alone publishes the block to every rank
        // with one system-scope fence -- a system fence per warp and tile
        // stalls the epilogues and, through them, the tiles.
        __syncwarp();
        if (lane == 0) {
          int old;
          asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(p.ready + grid.rb + 2 + x.r)
                       : "memory");
          if (old == 8 * grid.tb_row - 1) {
            asm volatile("fence.proxy.alias;" ::: "memory");  // unicast stores -> the switch's multicast reads
            __threadfence_system();
            for (int d = 0; d < p.world; ++d)
              asm volatile("red.relaxed.sys.global.add.s32 [%0], 1;" ::"l"(p.arrive[d] + x.r) : "memory");
          }
        }
      } else if constexpr (MODE != kMlpLocal) {
        __half* stg = reinterpret_cast<__half*>(smem + S * STAGE + 512) + q * 32 * kPeerStageHalves;
        GemmParams gp{};
        for (int o = 0; o < kMaxPeers; ++o) gp.peers[o] = p.peers[o];
        gp.peer_rank = p.peer_rank;
        gp.rows_per_owner = p.rows_per_owner;
        gp.world = p.world;
        gp.interleave = MODE == kMlpStep;
        gp.m = p.m;
        gp.n = p.n2;
        gp.ldc = p.ldc;
        peer_store_tile<BN>(gp, stg, tbase, row0, static_cast<int64_t>(x.c) * BN, lane);
        if constexpr (MODE == kMlpStep) {
          // release this warp's 32 rows (4 granules) into their owners' counts
          __threadfence_system();
          __syncwarp();
          if (lane < p.world) {
            int k = 0;
#pragma unroll
            for (int g = 0; g < 4; ++g) k += ((row0 >> 3) + g) % p.world == lane;
            if (k) red_release_sys_add(p.arrive[lane] + x.r, k);
          }
        }
      } else {
        TC* crow = static_cast<TC*>(p.c) + (row_ok ? row : 0) * p.ldc;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          __syncwarp();
          tmem_ld32(tbase + c * 32, v);
          tmem_wait_ld();
          const int64_t col = static_cast<int64_t>(x.c) * BN + c * 32;
          if (row_ok && col < p.n2) store32<TC>(crow + col, v, col, p.n2);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_u32(smem_u32(&tempty[buf]), 0), 1);
    }
  } else if (warp >= 6) {
    // ---------------- reduction warps (kMlpStep, kMlpStepMC) ----------------
    if constexpr (MODE >= kMlpStep) mlp_step_reduce_warp<MODE>(p, grid.rb, lane, abort_flag);
  }

  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) {
    // copies issued by this CTA may still be landing (failure path only)
    for (int k = 0; k < 1000; ++k) __nanosleep(1000);
  }
  cluster_barrier();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
  }
}

// ---- host side -------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D tensor map over a row-major [outer, inner] matrix with 128-byte swizzle.
int make_map(CUtensorMap* map, const void* base, int32_t dtype, uint64_t inner, uint64_t outer, uint64_t ld,
             uint32_t box_inner, uint32_t box_outer, const char* what) {
  auto fn = encode_fn();
  if (!fn) return fail(AXON_E_CUDA, "axon_gemm: cuTensorMapEncodeTiled unavailable");
  const CUtensorMapDataType dt =
      dtype == AXON_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AXON_E_ARG, "axon_gemm: tensor map for %s rejected (CUresult %d)", what, (int)r);
  return AXON_OK;
}

// Persistent grid for `tiles` tiles on at most `cap` workers: the fewest
// workers that finish in the same number of rounds as `cap` would (224 pair
// tiles on 74 pairs take 4 rounds either way, so 56 pairs run them and the
// other SMs stay free for kernels that overlap the GEMM, such as the
// tensor-parallel reduction).
int64_t balanced_grid(int64_t tiles, int64_t cap) {
  if (tiles <= cap) return tiles;
  const int64_t rounds = (tiles + cap - 1) / cap;
  return (tiles + rounds - 1) / rounds;
}

template <int BN, int EPI, typename TC>
int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mb2, const GemmParams& gp,
                cudaStream_t s) {
  constexpr int STAGE = A_BYTES + BN * BK * 2;
  const size_t smem = static_cast<size_t>(gp.stages) * STAGE + 1024 + 256 + (EPI == kEpiPeer ? kPeerStageBytes : 0);
  auto kern = gemm_tcgen05<BN, EPI, TC>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return fail(AXON_E_LAUNCH, "axon_gemm: smem attribute: %s", cudaGetErrorString(e));
  constexpr int BN_OUT = EPI == AXON_EPI_SILU_GATE ? BN / 2 : BN;
  const int64_t tiles = static_cast<int64_t>((gp.m + BM - 1) / BM) * ((gp.n + BN_OUT - 1) / BN_OUT);
  int64_t cap = sm_count();
  if (gp.max_ctas > 0 && gp.max_ctas < cap) cap = gp.max_ctas;
  const int grid = static_cast<int>(balanced_grid(tiles, cap));
  kern<<<grid, 192, smem, s>>>(ma, mb, mb2, gp);
  return launch_status("axon_gemm");
}

// Variant 2: clusters of two CTAs, one pair per 256-row tile. The grid is
// capped at the number of pairs the GPU holds at once (each CTA needs a whole
// SM), so the kernel stays persistent.
template <int BN, int EPI, typename TC>
int launch_gemm_pair(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mb2, const GemmParams& gp,
                     cudaStream_t s) {
  constexpr int STAGE = A_BYTES + (BN / 2) * BK * 2;
  const size_t smem = static_cast<size_t>(gp.stages) * STAGE + 1024 + 256 + (EPI == kEpiPeer ? kPeerStageBytes : 0);
  auto kern = gemm_tcgen05_pair<BN, EPI, TC>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return fail(AXON_E_LAUNCH, "axon_gemm: smem attribute: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // pairs resident at once, for this smem footprint (cached per footprint)
  static int cached_pairs[9] = {0};
  int& pairs_cap = cached_pairs[gp.stages > 8 ? 8 : gp.stages];
  if (pairs_cap == 0) {
    cfg.gridDim = dim3(2, 1, 1);
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
    if (e != cudaSuccess || clusters <= 0)
      return fail(AXON_E_LAUNCH, "axon_gemm: no room for a CTA pair (%s)", cudaGetErrorString(e));
    pairs_cap = clusters;
  }
  constexpr int BN_OUT = EPI == AXON_EPI_SILU_GATE ? BN / 2 : BN;
  const int64_t tiles = static_cast<int64_t>((gp.m + 2 * BM - 1) / (2 * BM)) * ((gp.n + BN_OUT - 1) / BN_OUT);
  int64_t cap = pairs_cap;
  if (gp.max_ctas > 0 && gp.max_ctas / 2 < cap) cap = gp.max_ctas / 2 > 0 ? gp.max_ctas / 2 : 1;
  const int pairs = static_cast<int>(balanced_grid(tiles, cap));
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  e = cudaLaunchKernelEx(&cfg, kern, ma, mb, mb2, gp);
  if (e != cudaSuccess) return fail(AXON_E_LAUNCH, "axon_gemm: %s", cudaGetErrorString(e));
  return launch_status("axon_gemm");
}

template <int BN, int EPI>
int dispatch_c(int32_t c_dtype, bool pair, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mb2,
               const GemmParams& gp, cudaStream_t s) {
  if (pair) {
    if constexpr (BN >= 128) {
      switch (c_dtype) {
        case AXON_BF16: return launch_gemm_pair<BN, EPI, __nv_bfloat16>(ma, mb, mb2, gp, s);
        case AXON_F16: return launch_gemm_pair<BN, EPI, __half>(ma, mb, mb2, gp, s);
        case AXON_F32: return launch_gemm_pair<BN, EPI, float>(ma, mb, mb2, gp, s);
        default: return fail(AXON_E_UNSUPPORTED, "axon_gemm: unsupported output dtype %d", c_dtype);
      }
    }
    return fail(AXON_E_ARG, "axon_gemm: the CTA-pair variant needs block_n >= 128");
  }
  switch (c_dtype) {
    case AXON_BF16: return launch_gemm<BN, EPI, __nv_bfloat16>(ma, mb, mb2, gp, s);
    case AXON_F16: return launch_gemm<BN, EPI, __half>(ma, mb, mb2, gp, s);
    case AXON_F32: return launch_gemm<BN, EPI, float>(ma, mb, mb2, gp, s);
    default: return fail(AXON_E_UNSUPPORTED, "axon_gemm: unsupported output dtype %d", c_dtype);
  }
}

// Deepest ring that fits the 227 KB of shared memory; `b_cols` = B columns
// staged per CTA (block_n, or block_n / 2 for a CTA pair).
int max_stages(int b_cols, int extra = 0) {
  const int stage = A_BYTES + b_cols * BK * 2;
  const int avail = 232448 - 1024 - 256 - extra;
  int s = avail / stage;
  return s > 8 ? 8 : s;
}

template <typename TC, int MODE>
int launch_swiglu_fused(const CUtensorMap& mx, const CUtensorMap& mg, const CUtensorMap& mu, const CUtensorMap& ma,
                        const CUtensorMap& md, const MlpParams& mp, cudaStream_t s) {
  constexpr int STAGE = A_BYTES + 128 * BK * 2;
  const size_t smem =
      static_cast<size_t>(mp.stages) * STAGE + 1024 + 512 + (MODE != kMlpLocal ? kPeerStageBytes : 0);
  auto kern = swiglu_fused_pair<TC, MODE>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return fail(AXON_E_LAUNCH, "axon_silu_mlp: smem attribute: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(mlp_threads(MODE), 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static int cached_pairs[9] = {0};
  int& pairs_cap = cached_pairs[mp.stages > 8 ? 8 : mp.stages];
  if (pairs_cap == 0) {
    cfg.gridDim = dim3(2, 1, 1);
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
    if (e != cudaSuccess || clusters <= 0)
      return fail(AXON_E_LAUNCH, "axon_silu_mlp: no room for a CTA pair (%s)", cudaGetErrorString(e));
    pairs_cap = clusters;
  }
  const int64_t rb = (mp.m + 2 * BM - 1) / (2 * BM);
  const int64_t tiles = rb * ((mp.n1 + 127) / 128 + (mp.n2 + 255) / 256);
  int64_t pairs = pairs_cap;
  if (mp.max_ctas > 0 && mp.max_ctas / 2 < pairs) pairs = mp.max_ctas / 2 > 0 ? mp.max_ctas / 2 : 1;
  if (tiles < pairs) pairs = tiles;
  // row-block counters and the tile counter start at zero every call
  e = cudaMemsetAsync(mp.ready, 0, static_cast<size_t>(2 * rb + 2) * sizeof(int), s);
  if (e != cudaSuccess) return fail(AXON_E_CUDA, "axon_silu_mlp: counter reset: %s", cudaGetErrorString(e));
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
  e = cudaLaunchKernelEx(&cfg, kern, mx, mg, mu, ma, md, mp);
  if (e != cudaSuccess) return fail(AXON_E_LAUNCH, "axon_silu_mlp: %s", cudaGetErrorString(e));
  return launch_status("axon_silu_mlp");
}

// Bytes of the fused kernel's counters: one per 256-row block (activation
// written), the tile counter, the reduction warps' unit counter and one per
// 256-row block (down-projection partials written, kMlpStepMC).
int64_t swiglu_counter_bytes(int64_t m) { return (2 * ((m + 255) / 256) + 2) * 4; }

// The fused SwiGLU (precision 4): x [m, k1] bf16, w1/w2 [k1, n1] bf16, w3h [n1, n2]
// f16 (the caller's f16 copy of W_down), act [m, n1] f16 and counters from the
// caller's workspace; the output goes to c [m, ldc] (c_dtype) or, with
// `peers`, to the owners' inboxes as axon_tp_down_partial lays them out.
// `step` (with peers) selects the whole tensor-parallel step (kMlpStep).
struct StepArgs {
  int32_t* const* arrive;
  int32_t* const* done;
  const void* inbox;  // kMlpStep
  void* const* ys;    // kMlpStep
  int epoch;
  void* part;         // kMlpStepMC: this rank's partial buffer, its multicast address and the output's
  const void* part_mc;
  void* y_mc;
};

int swiglu_fused_impl(const void* x, const void* w1, const void* w2, const void* w3h, __half* act, int* counters,
                      void* c, int64_t ldc, int32_t c_dtype, int64_t m, int64_t n1, int64_t k1, int64_t n2,
                      const axon_tune_t& t, void* stream, void* const* peers = nullptr, int world = 0,
                      int peer_rank = 0, int64_t rows_per_owner = 0, const StepArgs* step = nullptr) {
  if (m > 0x7fffffff || n1 > 0x7fffffff || k1 > 0x7fffffff || n2 > 0x7fffffff)
    return fail(AXON_E_SHAPE, "axon_silu_mlp: sizes out of range");
  if (n1 % 8 || k1 % 8 || n2 % 8) return fail(AXON_E_SHAPE, "axon_silu_mlp: n, k and p must be multiples of 8");
  if (!aligned16(x) || !aligned16(w1) || !aligned16(w2) || !aligned16(w3h) || !aligned16(act) ||
      (c != nullptr && !aligned16(c)))
    return fail(AXON_E_ALIGN, "axon_silu_mlp: operands must be 16-byte aligned");
  const int extra = peers != nullptr || step != nullptr ? kPeerStageBytes : 0;
  const int smax = (232448 - 1024 - 512 - extra) / (A_BYTES + 128 * BK * 2) > 8
                       ? 8
                       : (232448 - 1024 - 512 - extra) / (A_BYTES + 128 * BK * 2);
  const int stages = t.stages > 0 ? t.stages : smax;
  if (stages < 2 || stages > smax) return fail(AXON_E_ARG, "axon_silu_mlp: stages must be in [2, %d]", smax);
  CUtensorMap mx, mg, mu, ma, md;
  int rc = make_map(&mx, x, AXON_BF16, k1, m, k1, BK, BM, "x");
  if (!rc) rc = make_map(&mg, w1, AXON_BF16, n1, k1, n1, 64, BK, "w1");
  if (!rc) rc = make_map(&mu, w2, AXON_BF16, n1, k1, n1, 64, BK, "w2");
  if (!rc) rc = make_map(&ma, act, AXON_F16, n1, m, n1, BK, BM, "activation");
  if (!rc) rc = make_map(&md, w3h, AXON_F16, n2, n1, n2, 64, BK, "w3");
  if (rc) return rc;
  MlpParams mp{};
  mp.c = c;
  if (peers != nullptr || step != nullptr) {
    if (peers != nullptr)
      for (int i = 0; i < world; ++i) mp.peers[i] = peers[i];
    mp.peer_rank = peer_rank;
    mp.rows_per_owner = static_cast<int>(rows_per_owner);
    mp.world = world;
  }
  if (step != nullptr) {
    for (int i = 0; i < world; ++i) {
      mp.arrive[i] = step->arrive[i];
      mp.done[i] = step->done[i];
      if (step->ys) mp.y[i] = step->ys[i];
    }
    mp.inbox = static_cast<const __half*>(step->inbox);
    mp.epoch = step->epoch;
    mp.part = static_cast<__half*>(step->part);
    mp.part_mc = static_cast<const __half*>(step->part_mc);
    mp.y_mc = static_cast<__nv_bfloat16*>(step->y_mc);
  }
  mp.act = act;
  mp.ready = counters;
  // tile order: two groups for one GPU (the weights are read twice), groups
  // of four row blocks for a tensor-parallel step (more overlap of the down
  // projection's traffic with gate/up tiles; the shard's weights are small);
  // tune.rows_per_cta overrides the group size of a step
  mp.group = step != nullptr ? (t.rows_per_cta > 0 ? t.rows_per_cta : 4) : 8;
  mp.m = static_cast<int>(m);
  mp.n1 = static_cast<int>(n1);
  mp.k1 = static_cast<int>(k1);
  mp.n2 = static_cast<int>(n2);
  mp.ldc = ldc;
  mp.stages = stages;
  mp.max_ctas = t.max_ctas;
  // M = 256 (pair), N = 256; A/B bf16 in phase A, f16 in phase B
  const uint32_t shape = (static_cast<uint32_t>(256 >> 3) << 17) | (static_cast<uint32_t>(256 >> 4) << 24);
  mp.idesc_a = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | shape;
  mp.idesc_b = (1u << 4) | (1u << 16) | shape;
  cudaStream_t s = as_stream(stream);
  if (step != nullptr && step->part != nullptr)
    return launch_swiglu_fused<__half, kMlpStepMC>(mx, mg, mu, ma, md, mp, s);
  if (step != nullptr) return launch_swiglu_fused<__half, kMlpStep>(mx, mg, mu, ma, md, mp, s);
  if (peers != nullptr) return launch_swiglu_fused<__half, kMlpScatter>(mx, mg, mu, ma, md, mp, s);
  switch (c_dtype) {
    case AXON_BF16: return launch_swiglu_fused<__nv_bfloat16, kMlpLocal>(mx, mg, mu, ma, md, mp, s);
    case AXON_F16: return launch_swiglu_fused<__half, kMlpLocal>(mx, mg, mu, ma, md, mp, s);
    case AXON_F32: return launch_swiglu_fused<float, kMlpLocal>(mx, mg, mu, ma, md, mp, s);
    default: return fail(AXON_E_UNSUPPORTED, "axon_silu_mlp: unsupported output dtype %d", c_dtype);
  }
}

}  // namespace
}  // namespace axon

using namespace axon;

namespace axon {
namespace {

// axon_gemm plus the two silu_mlp-internal knobs: `terms` (SILU_GATE writes
// the activation as that many split terms, `term_stride` columns apart) and
// `b_kwrap` (the k coordinate of B wraps modulo b_kwrap, so a K = terms * n
// contraction re-reads the same [n, p] weight once per term).
//
// `peers` (with world, peer_rank, rows_per_owner) switches the epilogue to the
// tensor-parallel inbox scatter of axon_tp_down_partial; C is then unused.
int gemm_impl(const void* a, const void* b, const void* b2, void* c, const float* row_scale, int64_t m, int64_t n,
              int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int32_t ab_dtype, int32_t c_dtype, int32_t epilogue,
              const axon_tune_t* tune, void* stream, int terms, int64_t term_stride, int64_t b_kwrap,
              void* const* peers = nullptr, int world = 0, int peer_rank = 0, int64_t rows_per_owner = 0,
              float* row_part = nullptr, int64_t part_ld = 0) {
  axon_tune_t t = tune_or_default(tune);
  if (m < 0 || n < 0 || k < 0) return fail(AXON_E_SHAPE, "axon_gemm: negative size");
  if (m == 0 || n == 0) return AXON_OK;  // empty output: nothing to launch, pointers may be NULL
  if (!a || !b || !c) return fail(AXON_E_ARG, "axon_gemm: NULL operand");
  if (ab_dtype != AXON_BF16 && ab_dtype != AXON_F16)
    return fail(AXON_E_UNSUPPORTED, "axon_gemm: A/B dtype must be bf16 or f16 (got %d)", ab_dtype);
  if (epilogue < AXON_EPI_NONE || epilogue > AXON_EPI_EXP)
    return fail(AXON_E_ARG, "axon_gemm: unknown epilogue %d", epilogue);
  if (epilogue == AXON_EPI_SILU_GATE && !b2) return fail(AXON_E_ARG, "axon_gemm: SILU_GATE needs b2");
  if (epilogue == AXON_EPI_ROWSCALE && !row_scale) return fail(AXON_E_ARG, "axon_gemm: ROWSCALE needs row_scale");
  if (m < 0 || n < 0 || k < 0 || m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff)
    return fail(AXON_E_SHAPE, "axon_gemm: sizes out of range");
  if (k % 8 || n % 8) return fail(AXON_E_SHAPE, "axon_gemm: k and n must be multiples of 8 (k=%lld n=%lld)",
                                  (long long)k, (long long)n);
  const int64_t b_rows = b_kwrap > 0 ? b_kwrap : k;
  if (lda < k || ldb < n || ldc < n) return fail(AXON_E_SHAPE, "axon_gemm: leading dimension too small");
  if (lda % 8 || ldb % 8 || ldc % 8) return fail(AXON_E_ALIGN, "axon_gemm: leading dimensions must be multiples of 8");
  if (!aligned16(a) || !aligned16(b) || !aligned16(c) || (b2 && !aligned16(b2)))
    return fail(AXON_E_ALIGN, "axon_gemm: operands must be 16-byte aligned");
  if (t.variant < 0 || t.variant > 2) return fail(AXON_E_ARG, "axon_gemm: unknown variant %d", t.variant);
  if (t.block_m != 0 && t.block_m != 128) return fail(AXON_E_ARG, "axon_gemm: block_m must be 128");
  if (t.block_k != 0 && t.block_k != 64) return fail(AXON_E_ARG, "axon_gemm: block_k must be 64");
  if (k == 0) return fail(AXON_E_SHAPE, "axon_gemm: k == 0 not supported");

  int bn = t.block_n;
  if (bn == 0) {
    // 256-column tiles: on B200 a 128-column tile runs at about two thirds
    // of the rate (4096 x 4096 x 14336: 791 vs 1175 TFLOP/s), which more than
    // pays for a ragged last wave of persistent CTAs.
    bn = epilogue == AXON_EPI_SILU_GATE ? 256 : (n <= 64 ? 64 : n <= 128 ? 128 : 256);
  }
  if (bn != 64 && bn != 128 && bn != 256) return fail(AXON_E_ARG, "axon_gemm: block_n must be 64, 128 or 256");
  if (epilogue == AXON_EPI_SILU_GATE && bn == 64) return fail(AXON_E_ARG, "axon_gemm: SILU_GATE needs block_n >= 128");
  // variant 1: one CTA per 128-row tile; 2: CTA pairs on 256-row tiles; 0
  // (default): pairs unless the 256-row tiling would add a mostly empty tile
  // (m % 256 in 1..128) or block_n is 64.
  const bool pair = t.variant == 2 || (t.variant == 0 && bn >= 128 && m >= 256 && (m % 256 == 0 || m % 256 > 128));
  if (pair && bn == 64) return fail(AXON_E_ARG, "axon_gemm: the CTA-pair variant needs block_n >= 128");
  const int smax = max_stages(pair ? bn / 2 : bn, peers != nullptr ? kPeerStageBytes : 0);
  int stages = t.stages > 0 ? t.stages : smax;
  if (stages < 2 || stages > smax) return fail(AXON_E_ARG, "axon_gemm: stages must be in [2, %d] for block_n %d", smax, bn);

  CUtensorMap ma, mb, mb2;
  int rc = make_map(&ma, a, ab_dtype, k, m, lda, BK, BM, "A");
  if (rc) return rc;
  rc = make_map(&mb, b, ab_dtype, n, b_rows, ldb, 64, BK, "B");
  if (rc) return rc;
  if (b2) {
    rc = make_map(&mb2, b2, ab_dtype, n, b_rows, ldb, 64, BK, "B2");
    if (rc) return rc;
  } else {
    mb2 = mb;
  }
  GemmParams gp{};
  if (peers != nullptr) {
    for (int i = 0; i < world; ++i) gp.peers[i] = peers[i];
    gp.peer_rank = peer_rank;
    gp.rows_per_owner = static_cast<int>(rows_per_owner);
  }
  gp.c = c;
  gp.row_scale = row_scale;
  gp.row_part = row_part;
  gp.part_ld = part_ld;
  if (row_part != nullptr && (epilogue != AXON_EPI_EXP || part_ld < m))
    return fail(AXON_E_ARG, "axon_gemm: row sums need the EXP epilogue and a tile stride of >= m");
  gp.m = static_cast<int>(m);
  gp.n = static_cast<int>(n);
  gp.k = static_cast<int>(k);
  gp.ldc = ldc;
  gp.stages = stages;
  gp.terms = terms;
  gp.term_stride = term_stride;
  gp.b_kwrap = static_cast<int>(b_kwrap);
  gp.max_ctas = t.max_ctas;
  gp.raster = t.split;  // tune.split: row tiles per raster band (0 = column-major)
  if (t.split < 0) return fail(AXON_E_ARG, "axon_gemm: split (raster band) must be >= 0");
  if (t.max_ctas < 0) return fail(AXON_E_ARG, "axon_gemm: max_ctas must be >= 0");
  const uint32_t fmt = ab_dtype == AXON_BF16 ? 1u : 0u;
  const uint32_t mma_m = pair ? 2 * BM : BM;  // a CTA pair issues M = 256
  gp.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | (0u << 15) | (1u << 16) |
             (static_cast<uint32_t>(bn >> 3) << 17) | ((mma_m >> 4) << 24);
  cudaStream_t s = as_stream(stream);
  if (peers != nullptr) {
    if (bn == 64) return fail(AXON_E_ARG, "axon_tp_down_partial: block_n must be 128 or 256");
    if (bn == 128)
      return pair ? launch_gemm_pair<128, kEpiPeer, __half>(ma, mb, mb2, gp, s)
                  : launch_gemm<128, kEpiPeer, __half>(ma, mb, mb2, gp, s);
    return pair ? launch_gemm_pair<256, kEpiPeer, __half>(ma, mb, mb2, gp, s)
                : launch_gemm<256, kEpiPeer, __half>(ma, mb, mb2, gp, s);
  }
  switch (epilogue * 4 + (bn == 64 ? 0 : bn == 128 ? 1 : 2)) {
    case 0: return dispatch_c<64, AXON_EPI_NONE>(c_dtype, pair, ma, mb, mb2, gp, s);
    case 1: return dispatch_c<128, AXON_EPI_NONE>(c_dtype, pair, ma, mb, mb2, gp, s);
    case 2: return dispatch_c<256, AXON_EPI_NONE>(c_dtype, pair, ma, mb, mb2, gp, s);
    case 4: return dispatch_c<64, AXON_EPI_ROWSCALE>(c_dtype, pair, ma, mb, mb2, gp, s);
    case 5: return dispatch_c<128, AXON_EPI_ROWSCALE>(c_dtype, pair, ma, mb, mb2, gp, s);
    case 6: return dispatch_c<256, AXON_EPI_ROWSCALE>(c_dtype, pair, ma, mb, mb2, gp, s);
    case 9: return dispatch_c<128, AXON_EPI_SILU_GATE>(c_dtype, pair, ma, mb, mb2, gp, s);
    case 10: return dispatch_c<256, AXON_EPI_SILU_GATE>(c_dtype, pair, ma, mb, mb2, gp, s);
    case 12: return dispatch_c<64, AXON_EPI_EXP>(c_dtype, pair, ma, mb, mb2, gp, s);
    case 13: return dispatch_c<128, AXON_EPI_EXP>(c_dtype, pair, ma, mb, mb2, gp, s);
    case 14: return dispatch_c<256, AXON_EPI_EXP>(c_dtype, pair, ma, mb, mb2, gp, s);
    default: return fail(AXON_E_ARG, "axon_gemm: unsupported tile/epilogue combination");
  }
}

}  // namespace
}  // namespace axon

namespace axon {
namespace {

// Tile width, k split and pipeline depth of gemm_resid3 for a shape.
struct Resid3Plan {
  int bn, splits, kb_per_split, stages;
  int64_t ws_bytes;
};

int resid3_plan(int64_t m, int64_t n, int64_t k, const axon_tune_t& t, Resid3Plan& pl) {
  int bn = t.block_n;
  if (bn == 0) {
    // the narrowest of 128 / 256 / 384 / 512 that covers n; wider outputs take
    // the width that wastes the fewest columns, then the fewest tiles
    bn = 512;
    for (int c : {128, 256, 384, 512})
      if (n <= c) {
        bn = c;
        break;
      }
    if (n > 512) {
      int64_t best = -1;
      for (int c : {512, 384, 256}) {
        const int64_t cols = (n + c - 1) / c * c;
        if (best < 0 || cols < best) {
          best = cols;
          bn = c;
        }
      }
    }
  }
  if (bn != 128 && bn != 256 && bn != 384 && bn != 512)
    return fail(AXON_E_ARG, "axon_gemm_resid3: block_n must be 128, 256, 384 or 512");
  const int64_t stage_bytes = static_cast<int64_t>(bn) * BK * 2;  // B slab; the h ring is fixed
  int smax = static_cast<int>((232448 - 1024 - 512 - 2 * BM * 4 - kResidHSlots * A_BYTES) / stage_bytes);
  if (smax > 4) smax = 4;
  const int stages = t.stages > 0 ? t.stages : smax;
  if (stages < 2 || stages > smax)
    return fail(AXON_E_ARG, "axon_gemm_resid3: stages must be in [2, %d] for block_n %d", smax, bn);
  const int64_t kblocks = (k + BK - 1) / BK;
  const int64_t tiles = (m + BM - 1) / BM * ((n + bn - 1) / bn);
  int64_t splits = t.split;
  if (splits < 0) return fail(AXON_E_ARG, "axon_gemm_resid3: split (k splits) must be >= 0");
  if (splits == 0) {
    // split k only while the tiles leave SMs idle, keeping >= 4 k-blocks a split
    splits = tiles >= sm_count() ? 1 : sm_count() / tiles;
    if (splits > kblocks / 4) splits = kblocks / 4;
    if (splits < 1) splits = 1;
  }
  if (splits > kblocks) splits = kblocks;
  const int64_t kbps = (kblocks + splits - 1) / splits;
  splits = (kblocks + kbps - 1) / kbps;  // no empty split
  pl.bn = bn;
  pl.splits = static_cast<int>(splits);
  pl.kb_per_split = static_cast<int>(kbps);
  pl.stages = stages;
  pl.ws_bytes = splits > 1 ? (splits * m * n * 4 + 255) / 256 * 256 + splits * m * 4 : 0;
  return AXON_OK;
}

template <int BN, typename TA, typename TC>
int launch_resid3(const void* x, const void* r1, const void* r2, const CUtensorMap& mb, const Resid3Params& rp,
                  int64_t cap, cudaStream_t s) {
  constexpr int STAGE = BN * BK * 2;
  const size_t smem = static_cast<size_t>(rp.stages) * STAGE + kResidHSlots * A_BYTES + 1024 + 512 + 2 * BM * 4;
  auto kern = gemm_resid3<BN, TA, TC>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return fail(AXON_E_LAUNCH, "axon_gemm_resid3: smem attribute: %s", cudaGetErrorString(e));
  const int64_t units = static_cast<int64_t>((rp.m + BM - 1) / BM) * ((rp.n + BN - 1) / BN) * rp.splits;
  const int grid = static_cast<int>(balanced_grid(units, cap));
  kern<<<grid, kResidThreads, smem, s>>>(static_cast<const TA*>(x), static_cast<const TA*>(r1),
                                         static_cast<const TA*>(r2), mb, rp);
  int rc = launch_status("axon_gemm_resid3");
  if (rc || rp.splits == 1) return rc;
  const int64_t packets = static_cast<int64_t>(rp.m) * (rp.n / 4);
  launch_k(resid3_reduce_kernel<TC>, dim3(static_cast<unsigned>((packets + 255) / 256)), dim3(256), 0, s,
           static_cast<const float*>(rp.part), static_cast<const float*>(rp.ss_part), static_cast<TC*>(rp.c),
           static_cast<int64_t>(rp.m), static_cast<int64_t>(rp.n), rp.ldc, rp.splits, rp.inv_k, rp.eps);
  return launch_status("axon_gemm_resid3");
}

template <int BN, typename TA>
int dispatch_resid3(int32_t c_dtype, const void* mx, const void* m1, const void* m2, const CUtensorMap& mb,
                    const Resid3Params& rp, int64_t cap, cudaStream_t s) {
  switch (c_dtype) {
    case AXON_BF16: return launch_resid3<BN, TA, __nv_bfloat16>(mx, m1, m2, mb, rp, cap, s);
    case AXON_F16: return launch_resid3<BN, TA, __half>(mx, m1, m2, mb, rp, cap, s);
    case AXON_F32: return launch_resid3<BN, TA, float>(mx, m1, m2, mb, rp, cap, s);
    default: return fail(AXON_E_UNSUPPORTED, "axon_gemm_resid3: unsupported output dtype %d", c_dtype);
  }
}

template <typename TA>
int dispatch_resid3_bn(int bn, int32_t c_dtype, const void* mx, const void* m1, const void* m2,
                       const CUtensorMap& mb, const Resid3Params& rp, int64_t cap, cudaStream_t s) {
  switch (bn) {
    case 128: return dispatch_resid3<128, TA>(c_dtype, mx, m1, m2, mb, rp, cap, s);
    case 256: return dispatch_resid3<256, TA>(c_dtype, mx, m1, m2, mb, rp, cap, s);
    case 384: return dispatch_resid3<384, TA>(c_dtype, mx, m1, m2, mb, rp, cap, s);
    default: return dispatch_resid3<512, TA>(c_dtype, mx, m1, m2, mb, rp, cap, s);
  }
}

uint32_t resid3_idesc(int32_t ab_dtype, int n) {
  const uint32_t fmt = ab_dtype == AXON_BF16 ? 1u : 0u;
  return (1u << 4) | (fmt << 7) | (fmt << 10) | (1u << 16) | (static_cast<uint32_t>(n >> 3) << 17) |
         ((static_cast<uint32_t>(BM) >> 4) << 24);
}

}  // namespace
}  // namespace axon

extern "C" int64_t axon_gemm_resid3_workspace_bytes(int64_t m, int64_t n, int64_t k, const axon_tune_t* tune) {
  if (m < 0 || n < 0 || k < 0) return fail(AXON_E_SHAPE, "axon_gemm_resid3_workspace_bytes: negative size");
  if (m == 0 || n == 0 || k == 0) return 0;
  Resid3Plan pl;
  const int rc = resid3_plan(m, n, k, tune_or_default(tune), pl);
  return rc ? rc : pl.ws_bytes;
}

extern "C" int axon_gemm_resid3(const void* x, const void* r1, const void* r2, const void* w, void* c,
                                void* workspace, int64_t workspace_bytes, int64_t m, int64_t n, int64_t k,
                                int32_t ab_dtype, int32_t c_dtype, float eps, const axon_tune_t* tune, void* stream) {
  const axon_tune_t t = tune_or_default(tune);
  if (m < 0 || n < 0 || k < 0) return fail(AXON_E_SHAPE, "axon_gemm_resid3: negative size");
  if (m == 0 || n == 0) return AXON_OK;
  if (!x || !r1 || !r2 || !w || !c) return fail(AXON_E_ARG, "axon_gemm_resid3: NULL operand");
  if (ab_dtype != AXON_BF16 && ab_dtype != AXON_F16)
    return fail(AXON_E_UNSUPPORTED, "axon_gemm_resid3: inputs must be bf16 or f16 (got %d)", ab_dtype);
  if (m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff || k == 0)
    return fail(AXON_E_SHAPE, "axon_gemm_resid3: sizes out of range");
  if (k % 8 || n % 8) return fail(AXON_E_SHAPE, "axon_gemm_resid3: k and n must be multiples of 8");
  if (!aligned16(x) || !aligned16(r1) || !aligned16(r2) || !aligned16(w) || !aligned16(c))
    return fail(AXON_E_ALIGN, "axon_gemm_resid3: operands must be 16-byte aligned");
  if (t.max_ctas < 0) return fail(AXON_E_ARG, "axon_gemm_resid3: max_ctas must be >= 0");
  Resid3Plan pl;
  int rc = resid3_plan(m, n, k, t, pl);
  if (rc) return rc;
  if (pl.ws_bytes > 0 && (!workspace || workspace_bytes < pl.ws_bytes || !aligned16(workspace)))
    return fail(AXON_E_ARG, "axon_gemm_resid3: %d k splits need a 16-byte aligned workspace of %lld bytes",
                pl.splits, (long long)pl.ws_bytes);
  CUtensorMap mb;
  rc = make_map(&mb, w, ab_dtype, n, k, n, 64, BK, "w");
  if (rc) return rc;
  Resid3Params rp{};
  rp.c = c;
  if (pl.splits > 1) {
    rp.part = static_cast<float*>(workspace);
    rp.ss_part = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) +
                                          (static_cast<int64_t>(pl.splits) * m * n * 4 + 255) / 256 * 256);
  }
  rp.m = static_cast<int>(m);
  rp.n = static_cast<int>(n);
  rp.k = static_cast<int>(k);
  rp.ldc = n;
  rp.stages = pl.stages;
  rp.idesc_lo = resid3_idesc(ab_dtype, pl.bn < 256 ? pl.bn : 256);
  rp.idesc_hi = resid3_idesc(ab_dtype, pl.bn > 256 ? pl.bn - 256 : 256);
  rp.splits = pl.splits;
  rp.kb_per_split = pl.kb_per_split;
  rp.raster = 1;  // a row block's column tiles side by side: its inputs come from L2 the second time
  rp.inv_k = 1.0f / static_cast<float>(k);
  rp.eps = eps;
  int64_t cap = sm_count();
  if (t.max_ctas > 0 && t.max_ctas < cap) cap = t.max_ctas;
  cudaStream_t s = as_stream(stream);
  return ab_dtype == AXON_BF16 ? dispatch_resid3_bn<__nv_bfloat16>(pl.bn, c_dtype, x, r1, r2, mb, rp, cap, s)
                               : dispatch_resid3_bn<__half>(pl.bn, c_dtype, x, r1, r2, mb, rp, cap, s);
}

namespace axon {
namespace {

struct AttnPlan {
  int splits, kblk_per_split;
  int64_t ws_bytes;
};

// Key splits: while the 128-row query blocks leave SMs idle, at least two
// key blocks a split.
AttnPlan attn_plan(int64_t s, int64_t d, const axon_tune_t& t) {
  const int64_t nb = (s + 127) / 128;
  int64_t splits = t.split;
  if (splits <= 0) {
    splits = nb >= sm_count() ? 1 : sm_count() / nb;
    if (splits > nb / 2) splits = nb / 2;
    if (splits < 1) splits = 1;
  }
  if (splits > nb) splits = nb;
  const int64_t per = (nb + splits - 1) / splits;
  splits = (nb + per - 1) / per;
  AttnPlan pl;
  pl.splits = static_cast<int>(splits);
  pl.kblk_per_split = static_cast<int>(per);
  pl.ws_bytes = splits > 1 ? (splits * s * d * 4 + 255) / 256 * 256 + splits * s * 4 : 0;
  return pl;
}

template <int D, typename TA, typename TC>
int launch_attn(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const AttnParams& ap,
                int64_t cap, cudaStream_t st) {
  constexpr int KA = D / 64;
  constexpr size_t smem = static_cast<size_t>(KA) * A_BYTES + 2 * (KA * 2 * B_CHUNK + 2 * KA * B_CHUNK) +
                          2 * 2 * A_BYTES + 32 * 8 + 3 * 128 * 4 + 1024;
  auto kern = attn_fused<D, TA, TC>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return fail(AXON_E_LAUNCH, "axon_attention: smem attribute: %s", cudaGetErrorString(e));
  const int64_t units = static_cast<int64_t>((ap.s + 127) / 128) * ap.splits;
  const int grid = static_cast<int>(balanced_grid(units, cap));
  kern<<<grid, kAttnThreads, smem, st>>>(mq, mk, mv, ap);
  int rc = launch_status("axon_attention");
  if (rc || ap.splits == 1) return rc;
  const int64_t packets = static_cast<int64_t>(ap.s) * (D / 4);
  launch_k(attn_reduce_kernel<TC>, dim3(static_cast<unsigned>((packets + 255) / 256)), dim3(256), 0, st,
           static_cast<const float*>(ap.part), static_cast<const float*>(ap.lpart), static_cast<TC*>(ap.y),
           static_cast<int64_t>(ap.s), static_cast<int64_t>(D), ap.splits);
  return launch_status("axon_attention");
}

template <int D, typename TA>
int dispatch_attn(int32_t c_dtype, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                  const AttnParams& ap, int64_t cap, cudaStream_t st) {
  switch (c_dtype) {
    case AXON_BF16: return launch_attn<D, TA, __nv_bfloat16>(mq, mk, mv, ap, cap, st);
    case AXON_F16: return launch_attn<D, TA, __half>(mq, mk, mv, ap, cap, st);
    case AXON_F32: return launch_attn<D, TA, float>(mq, mk, mv, ap, cap, st);
    default: return fail(AXON_E_UNSUPPORTED, "axon_attention: unsupported output dtype %d", c_dtype);
  }
}

}  // namespace
}  // namespace axon

extern "C" int64_t axon_attention_fused_workspace_bytes(int64_t s, int64_t d, const axon_tune_t* tune) {
  if (s < 0 || d < 0) return fail(AXON_E_SHAPE, "axon_attention_fused_workspace_bytes: negative size");
  if (s == 0 || d == 0) return 0;
  return attn_plan(s, d, tune_or_default(tune)).ws_bytes;
}

extern "C" int axon_attention_fused(const void* q, const void* k_t, const void* v, void* y, void* workspace,
                                    int64_t workspace_bytes, int64_t s, int64_t d, int32_t ab_dtype,
                                    int32_t c_dtype, const axon_tune_t* tune, void* stream) {
  const axon_tune_t t = tune_or_default(tune);
  if (s < 0 || d < 0) return fail(AXON_E_SHAPE, "axon_attention_fused: negative size");
  if (s == 0 || d == 0) return AXON_OK;
  if (d != 64 && d != 128) return fail(AXON_E_UNSUPPORTED, "axon_attention_fused: head dim must be 64 or 128");
  if (s % 8 || s > 0x7fffffff) return fail(AXON_E_SHAPE, "axon_attention_fused: s must be a multiple of 8");
  if (ab_dtype != AXON_BF16 && ab_dtype != AXON_F16)
    return fail(AXON_E_UNSUPPORTED, "axon_attention_fused: inputs must be bf16 or f16 (got %d)", ab_dtype);
  if (!q || !k_t || !v || !y) return fail(AXON_E_ARG, "axon_attention_fused: NULL tensor");
  if (!aligned16(q) || !aligned16(k_t) || !aligned16(v) || !aligned16(y))
    return fail(AXON_E_ALIGN, "axon_attention_fused: tensors must be 16-byte aligned");
  if (t.split < 0 || t.max_ctas < 0) return fail(AXON_E_ARG, "axon_attention_fused: negative tune field");
  const AttnPlan pl = attn_plan(s, d, t);
  if (pl.ws_bytes > 0 && (!workspace || workspace_bytes < pl.ws_bytes || !aligned16(workspace)))
    return fail(AXON_E_ARG, "axon_attention_fused: %d key splits need a 16-byte aligned workspace of %lld bytes",
                pl.splits, (long long)pl.ws_bytes);
  CUtensorMap mq, mk, mv;
  int rc = make_map(&mq, q, ab_dtype, d, s, d, 64, 128, "q");  // [s, d]: 128 rows x 64 of the head dim
  if (!rc) rc = make_map(&mk, k_t, ab_dtype, s, d, s, 64, 64, "k_t");  // [d, s]: 64 keys x 64 of the head dim
  if (!rc) rc = make_map(&mv, v, ab_dtype, d, s, d, 64, 64, "v");      // [s, d]: 64 of the head dim x 64 keys
  if (rc) return rc;
  AttnParams ap{};
  ap.y = y;
  if (pl.splits > 1) {
    ap.part = static_cast<float*>(workspace);
    ap.lpart = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) +
                                        (static_cast<int64_t>(pl.splits) * s * d * 4 + 255) / 256 * 256);
  }
  ap.s = static_cast<int>(s);
  ap.splits = pl.splits;
  ap.kblk_per_split = pl.kblk_per_split;
  const uint32_t fmt = ab_dtype == AXON_BF16 ? 1u : 0u;
  const uint32_t base = (1u << 4) | (fmt << 7) | (fmt << 10) | (1u << 16) | ((128u >> 4) << 24);
  ap.idesc_s = base | ((128u >> 3) << 17);
  ap.idesc_o = base | (static_cast<uint32_t>(d >> 3) << 17);
  int64_t cap = sm_count();
  if (t.max_ctas > 0 && t.max_ctas < cap) cap = t.max_ctas;
  cudaStream_t st = as_stream(stream);
  if (ab_dtype == AXON_BF16)
    return d == 64 ? dispatch_attn<64, __nv_bfloat16>(c_dtype, mq, mk, mv, ap, cap, st)
                   : dispatch_attn<128, __nv_bfloat16>(c_dtype, mq, mk, mv, ap, cap, st);
  return d == 64 ? dispatch_attn<64, __half>(c_dtype, mq, mk, mv, ap, cap, st)
                 : dispatch_attn<128, __half>(c_dtype, mq, mk, mv, ap, cap, st);
}

extern "C" int axon_gemm_exp(const void* a, const void* b, void* c, float* row_part, int64_t part_ld, int64_t m,
                             int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int32_t ab_dtype,
                             int32_t c_dtype, const axon_tune_t* tune, void* stream) {
  return gemm_impl(a, b, nullptr, c, nullptr, m, n, k, lda, ldb, ldc, ab_dtype, c_dtype, AXON_EPI_EXP, tune, stream,
                   1, 0, 0, nullptr, 0, 0, 0, row_part, part_ld);
}

extern "C" int axon_gemm(const void* a, const void* b, const void* b2, void* c, const float* row_scale, int64_t m,
                         int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int32_t ab_dtype,
                         int32_t c_dtype, int32_t epilogue, const axon_tune_t* tune, void* stream) {
  return gemm_impl(a, b, b2, c, row_scale, m, n, k, lda, ldb, ldc, ab_dtype, c_dtype, epilogue, tune, stream, 1, 0,
                   0);
}

extern "C" int axon_tp_down_partial(const void* act, const void* w, void* const* inboxes, int32_t world,
                                    int32_t rank, int64_t m, int64_t n, int64_t k, int64_t rows_per_owner,
                                    int32_t ab_dtype, const axon_tune_t* tune, void* stream) {
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world)
    return fail(AXON_E_ARG, "axon_tp_down_partial: world must be 1..%d and 0 <= rank < world", kMaxPeers);
  if (m < 0 || n < 0 || k < 0) return fail(AXON_E_SHAPE, "axon_tp_down_partial: negative size");
  if (m == 0 || n == 0) return AXON_OK;
  if (!inboxes) return fail(AXON_E_ARG, "axon_tp_down_partial: NULL inbox table");
  if (rows_per_owner <= 0 || rows_per_owner * world != m)
    return fail(AXON_E_SHAPE, "axon_tp_down_partial: m (%lld) must be world x rows_per_owner", (long long)m);
  for (int i = 0; i < world; ++i)
    if (!inboxes[i] || !aligned16(inboxes[i])) return fail(AXON_E_ALIGN, "axon_tp_down_partial: inbox %d NULL or unaligned", i);
  // C is never written on this path; pass a valid pointer for the argument checks
  return gemm_impl(act, w, nullptr, inboxes[0], nullptr, m, n, k, k, n, n, ab_dtype, AXON_F16, AXON_EPI_NONE, tune,
                   stream, 1, 0, 0, inboxes, world, rank, rows_per_owner);
}

extern "C" int64_t axon_tp_mlp_workspace_bytes(int64_t m, int64_t n) {
  if (m < 0 || n < 0) return fail(AXON_E_SHAPE, "axon_tp_mlp_workspace_bytes: negative size");
  return m * n * 2 + swiglu_counter_bytes(m);
}

extern "C" int axon_tp_mlp_partial(const void* x, const void* w_gate, const void* w_up, const void* w_down_h,
                                   void* workspace, int64_t workspace_bytes, void* const* inboxes, int32_t world,
                                   int32_t rank, int64_t m, int64_t n, int64_t k, int64_t p, int64_t rows_per_owner,
                                   const axon_tune_t* tune, void* stream) {
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world)
    return fail(AXON_E_ARG, "axon_tp_mlp_partial: world must be 1..%d and 0 <= rank < world", kMaxPeers);
  if (m < 0 || n < 0 || k < 0 || p < 0) return fail(AXON_E_SHAPE, "axon_tp_mlp_partial: negative size");
  if (m == 0 || p == 0) return AXON_OK;
  if (!x || !w_gate || !w_up || !w_down_h || !inboxes) return fail(AXON_E_ARG, "axon_tp_mlp_partial: NULL operand");
  if (rows_per_owner <= 0 || rows_per_owner * world != m)
    return fail(AXON_E_SHAPE, "axon_tp_mlp_partial: m (%lld) must be world x rows_per_owner", (long long)m);
  const int64_t need = m * n * 2 + swiglu_counter_bytes(m);
  if (!workspace || workspace_bytes < need)
    return fail(AXON_E_ARG, "axon_tp_mlp_partial: workspace of %lld bytes needed", (long long)need);
  for (int i = 0; i < world; ++i)
    if (!inboxes[i] || !aligned16(inboxes[i]))
      return fail(AXON_E_ALIGN, "axon_tp_mlp_partial: inbox %d NULL or unaligned", i);
  __half* act = static_cast<__half*>(workspace);
  int* counters = reinterpret_cast<int*>(static_cast<unsigned char*>(workspace) + m * n * 2);
  return swiglu_fused_impl(x, w_gate, w_up, w_down_h, act, counters, nullptr, p, AXON_F16, m, n, k, p,
                           tune_or_default(tune), stream, inboxes, world, rank, rows_per_owner);
}

extern "C" int64_t axon_tp_step_done_per_epoch(int32_t world, int64_t m, int64_t p) {
  if (world < 1 || m < 0 || p < 0) return fail(AXON_E_ARG, "axon_tp_step_done_per_epoch: bad argument");
  // every reduction unit (one owned row x kStepCols columns) counts once on
  // every rank: world owners x m / world rows x column chunks
  return m * ((p + kStepCols - 1) / kStepCols);
}

extern "C" int axon_tp_mlp_step(const void* x, const void* w_gate, const void* w_up, const void* w_down_h,
                                void* workspace, int64_t workspace_bytes, const void* inbox, void* const* inboxes,
                                int32_t* const* arrive, int32_t* const* done, void* const* ys, int32_t world,
                                int32_t rank, int32_t epoch, int64_t m, int64_t n, int64_t k, int64_t p,
                                const axon_tune_t* tune, void* stream) {
  if (world < 1 || world > kMaxPeers || (world & (world - 1)) || rank < 0 || rank >= world)
    return fail(AXON_E_ARG, "axon_tp_mlp_step: world must be 1, 2, 4 or 8 and 0 <= rank < world");
  if (m <= 0 || n <= 0 || k <= 0 || p <= 0) return fail(AXON_E_SHAPE, "axon_tp_mlp_step: sizes must be positive");
  if (m % 256) return fail(AXON_E_SHAPE, "axon_tp_mlp_step: m (%lld) must be a multiple of 256", (long long)m);
  if (!x || !w_gate || !w_up || !w_down_h || !inbox || !inboxes || !arrive || !done || !ys)
    return fail(AXON_E_ARG, "axon_tp_mlp_step: NULL argument");
  const int64_t need = m * n * 2 + swiglu_counter_bytes(m);
  if (!workspace || workspace_bytes < need)
    return fail(AXON_E_ARG, "axon_tp_mlp_step: workspace of %lld bytes needed", (long long)need);
  for (int i = 0; i < world; ++i)
    if (!inboxes[i] || !aligned16(inboxes[i]) || !ys[i] || !aligned16(ys[i]) || !arrive[i] || !done[i])
      return fail(AXON_E_ALIGN, "axon_tp_mlp_step: buffers of rank %d NULL or unaligned", i);
  if (!aligned16(inbox)) return fail(AXON_E_ALIGN, "axon_tp_mlp_step: inbox unaligned");
  __half* act = static_cast<__half*>(workspace);
  int* counters = reinterpret_cast<int*>(static_cast<unsigned char*>(workspace) + m * n * 2);
  StepArgs sa{arrive, done, inbox, ys, epoch, nullptr, nullptr, nullptr};
  return swiglu_fused_impl(x, w_gate, w_up, w_down_h, act, counters, nullptr, p, AXON_F16, m, n, k, p,
                           tune_or_default(tune), stream, inboxes, world, rank, m / world, &sa);
}

extern "C" int axon_tp_mlp_step_multicast(const void* x, const void* w_gate, const void* w_up,
                                          const void* w_down_h, void* workspace, int64_t workspace_bytes, void* part,
                                          const void* part_mc, void* y_mc, int32_t* const* arrive,
                                          int32_t* const* done, int32_t world, int32_t rank, int32_t epoch, int64_t m,
                                          int64_t n, int64_t k, int64_t p, const axon_tune_t* tune, void* stream) {
  if (world < 1 || world > kMaxPeers || (world & (world - 1)) || rank < 0 || rank >= world)
    return fail(AXON_E_ARG, "axon_tp_mlp_step_multicast: world must be 1, 2, 4 or 8 and 0 <= rank < world");
  if (m <= 0 || n <= 0 || k <= 0 || p <= 0)
    return fail(AXON_E_SHAPE, "axon_tp_mlp_step_multicast: sizes must be positive");
  if (m % 256) return fail(AXON_E_SHAPE, "axon_tp_mlp_step_multicast: m (%lld) must be a multiple of 256", (long long)m);
  if (!x || !w_gate || !w_up || !w_down_h || !part || !part_mc || !y_mc || !arrive || !done)
    return fail(AXON_E_ARG, "axon_tp_mlp_step_multicast: NULL argument");
  if (!aligned16(part) || !aligned16(part_mc) || !aligned16(y_mc))
    return fail(AXON_E_ALIGN, "axon_tp_mlp_step_multicast: partial and output buffers must be 16-byte aligned");
  const int64_t need = m * n * 2 + swiglu_counter_bytes(m);
  if (!workspace || workspace_bytes < need)
    return fail(AXON_E_ARG, "axon_tp_mlp_step_multicast: workspace of %lld bytes needed", (long long)need);
  for (int i = 0; i < world; ++i)
    if (!arrive[i] || !done[i]) return fail(AXON_E_ARG, "axon_tp_mlp_step_multicast: counters of rank %d NULL", i);
  __half* act = static_cast<__half*>(workspace);
  int* counters = reinterpret_cast<int*>(static_cast<unsigned char*>(workspace) + m * n * 2);
  StepArgs sa{arrive, done, nullptr, nullptr, epoch, part, part_mc, y_mc};
  return swiglu_fused_impl(x, w_gate, w_up, w_down_h, act, counters, nullptr, p, AXON_F16, m, n, k, p,
                           tune_or_default(tune), stream, nullptr, world, rank, m / world, &sa);
}

extern "C" int axon_gemm_status(void* stream) {
  int v = 0;
  cudaStream_t s = as_stream(stream);
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_gemm_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return fail(AXON_E_CUDA, "axon_gemm_status: %s", cudaGetErrorString(e));
  if (v != 0) {
    int zero = 0;
    cudaMemcpyToSymbolAsync(g_gemm_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
    cudaStreamSynchronize(s);
    return fail(v, "axon_gemm: a pipeline wait gave up (status %d)", v);
  }
  return AXON_OK;
}

extern "C" int axon_rmsnorm_matmul(const void* x, const void* w, void* y, void* workspace, int64_t m, int64_t n,
                                   int64_t k, int32_t ab_dtype, int32_t c_dtype, const axon_tune_t* tune,
                                   void* stream) {
  if (!workspace) return fail(AXON_E_ARG, "axon_rmsnorm_matmul: workspace (4*m bytes) required");
  int rc = axon_row_rsqrt(x, static_cast<float*>(workspace), m, k, k, ab_dtype, 1.0f, 0.0f, stream);
  if (rc) return rc;
  return axon_gemm(x, w, nullptr, y, static_cast<const float*>(workspace), m, n, k, k, n, n, ab_dtype, c_dtype,
                   AXON_EPI_ROWSCALE, tune, stream);
}

constexpr int kF16Act = 4;        // tune.precision value of the f16-activation mode
constexpr int kF16ActPrecast = 5;  // the same, with w3 passed as the caller's f16 copy
constexpr int64_t kFusedMaxTiles = 320;  // see axon_silu_mlp

static int silu_terms(const axon_tune_t* tune) {
  const int p = tune ? tune->precision : 0;
  return p <= 0 ? 1 : p;
}

static bool silu_f16(int terms) { return terms == kF16Act || terms == kF16ActPrecast; }

static bool silu_mode_ok(int terms) { return (terms >= 1 && terms <= 3) || silu_f16(terms); }

// precision 4 and 5 share one layout (the f16 copy of w3 goes unused at 5)
static int64_t silu_ws_bytes(int64_t m, int64_t n, int64_t p, int terms) {
  return silu_f16(terms) ? m * n * 2 + n * p * 2 + (swiglu_counter_bytes(m) + 255) / 256 * 256 : m * n * 2 * terms;
}

extern "C" int64_t axon_silu_mlp_workspace_bytes(int64_t m, int64_t n, int64_t p, int32_t ab_dtype,
                                                 const axon_tune_t* tune) {
  (void)ab_dtype;
  if (m < 0 || n < 0 || p < 0) return fail(AXON_E_SHAPE, "axon_silu_mlp_workspace_bytes: negative size");
  const int terms = silu_terms(tune);
  if (!silu_mode_ok(terms)) return fail(AXON_E_ARG, "axon_silu_mlp: precision must be 1, 2, 3, 4 or 5");
  return silu_ws_bytes(m, n, p, terms);
}

extern "C" int axon_silu_mlp(const void* x, const void* w1, const void* w2, const void* w3, void* y,
                             void* workspace, int64_t workspace_bytes, int64_t m, int64_t n, int64_t k, int64_t p,
                             int32_t ab_dtype, int32_t c_dtype, const axon_tune_t* tune, void* stream) {
  const int terms = silu_terms(tune);
  if (!silu_mode_ok(terms)) return fail(AXON_E_ARG, "axon_silu_mlp: precision must be 1, 2, 3, 4 or 5");
  if (m < 0 || n < 0 || k < 0 || p < 0) return fail(AXON_E_SHAPE, "axon_silu_mlp: negative size");
  if (m == 0 || p == 0) return AXON_OK;
  if (terms > 1 && terms <= 3 && n % 64)
    return fail(AXON_E_SHAPE, "axon_silu_mlp: split precision needs n %% 64 == 0 (n=%lld)", (long long)n);
  if (silu_f16(terms) && (ab_dtype != AXON_BF16 || p % 8))
    return fail(AXON_E_UNSUPPORTED, "axon_silu_mlp: the f16-activation mode takes bf16 operands and p %% 8 == 0");
  const int64_t need = silu_ws_bytes(m, n, p, terms);
  if (!workspace || workspace_bytes < need)
    return fail(AXON_E_ARG, "axon_silu_mlp: workspace of %lld bytes needed", (long long)need);
  axon_tune_t t = tune_or_default(tune);
  axon_tune_t up = t, down = t;
  up.block_n = t.block_n == 64 ? 0 : t.block_n;
  down.stages = 0;
  down.block_n = 0;
  if (silu_f16(terms)) {
    // The activation is written as f16 (8 more mantissa bits than bf16) and
    // the down projection runs f16 x f16, on an f16 copy of W_down: a tcgen05
    // f16-kind MMA takes both operands in one type. Precision 4 makes that
    // copy in the workspace on every call; at precision 5 w3 already is the
    // caller's f16 copy (made once, when the weights are loaded).
    __half* act = static_cast<__half*>(workspace);
    __half* w3h = reinterpret_cast<__half*>(static_cast<unsigned char*>(workspace) + m * n * 2);
    int* counters = reinterpret_cast<int*>(static_cast<unsigned char*>(workspace) + m * n * 2 + n * p * 2);
    int rc = AXON_OK;
    if (terms == kF16ActPrecast)
      w3h = static_cast<__half*>(const_cast<void*>(w3));
    else
      rc = cast_impl(w3, w3h, n * p, AXON_BF16, AXON_F16, as_stream(stream));
    if (rc) return rc;
    // variant 3: both GEMMs in one CTA-pair kernel; 1 / 2: two launches of
    // the one-CTA / CTA-pair GEMM; 0 (default): the fused kernel while the
    // gate/up GEMM has fewer than 320 pair tiles (about 4 waves on 74 pairs),
    // where filling the first GEMM's last partial wave with the second's
    // tiles pays; two launches above that. Measured on one B200, m = k = p =
    // 4096: n = 1792 (the 8-way shard of the BASELINE config, 224 tiles)
    // 156-169 us fused vs 182-194 us in two launches; n = 3584: 316-324 vs
    // 305-314; n = 7168: 631 vs 520-580; n = 14336: 1240 vs 1149-1185 (the
    // fused order reads the gate/up weights once per row group).
    const int64_t tiles_a = (m + 255) / 256 * ((n + 127) / 128);
    if (m >= 256 && (t.variant == 3 || (t.variant == 0 && tiles_a < kFusedMaxTiles)))
      return swiglu_fused_impl(x, w1, w2, w3h, act, counters, y, p, c_dtype, m, n, k, p, t, stream);
    if (t.variant == 3) return fail(AXON_E_SHAPE, "axon_silu_mlp: the fused variant needs m >= 256");
    rc = gemm_impl(x, w1, w2, act, nullptr, m, n, k, k, n, n, ab_dtype, AXON_F16, AXON_EPI_SILU_GATE, &up, stream, 1,
                   0, 0);
    if (rc) return rc;
    return gemm_impl(act, w3h, nullptr, y, nullptr, m, p, n, n, p, p, AXON_F16, c_dtype, AXON_EPI_NONE, &down,
                     stream, 1, 0, 0);
  }
  int rc = gemm_impl(x, w1, w2, workspace, nullptr, m, n, k, k, n, n * terms, ab_dtype, ab_dtype, AXON_EPI_SILU_GATE,
                     &up, stream, terms, n, 0);
  if (rc) return rc;
  return gemm_impl(workspace, w3, nullptr, y, nullptr, m, p, n * terms, n * terms, p, p, ab_dtype, c_dtype,
                   AXON_EPI_NONE, &down, stream, 1, 0, terms > 1 ? n : 0);
}
