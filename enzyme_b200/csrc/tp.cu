// Tensor-parallel SwiGLU over NVLink peer memory: the collective half of the
// fused down projection.
//
// The reference resolves the down projection's Partial(+) output with a
// terminal all-reduce (src/axon/sharding.py:380-384, :514-522). Here the
// all-reduce is split and fused around the GEMM instead of called as NCCL:
//
//   1. axon_tp_down_partial (gemm.cu): the down-projection GEMM's epilogue
//      writes each f16 partial row straight into the inbox of the rank that
//      owns the row, over NVLink, tile by tile while the mainloop runs
//      (reduce-scatter traffic overlapped with the tensor cores);
//   2. axon_tp_signal: after that GEMM, a system-scope fence and a release
//      store of the step's epoch into every owner's arrival flag;
//   3. axon_tp_reduce_gather: each owner waits (bounded) for all arrivals,
//      sums its rows' partials in fp32 in rank order, rounds once to the
//      output dtype and stores the rows into every rank's output buffer
//      (all-gather push), then axon_tp_signal raises the done flags;
//   4. axon_tp_wait: a rank waits (bounded) for every owner's done flag before
//      it reads the output.
//
// Peer buffers are ordinary device allocations shared with CUDA IPC
// (axon_ipc_handle / axon_ipc_open). The all-gather pushes rows with plain
// 16-byte peer stores or 1-D bulk copies (global <- shared) by default;
// axon_tp_reduce_multicast instead stores each row once with multimem.st to an
// NVLink multicast address (NVLS). No TMA tensor copy and no cluster-multicast
// load is used anywhere on this path, and NCCL is not called. Every wait
// gives up after about two seconds and records AXON_E_TIMEOUT, read and
// cleared by axon_tp_status, so a rank that never arrives ends the step with
// an error instead of a hung GPU.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>

#include "common.cuh"
#include "sm100.cuh"

namespace axon {

__device__ int g_tp_error;

namespace {

constexpr int kMaxWorld = 8;
constexpr uint64_t kTpWaitNs = 2000000000ull;

struct OutPtrs {
  void* p[kMaxWorld];
};
struct FlagPtrs {
  int* p[kMaxWorld];
};

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}


// Until flags[s] has reached `epoch` for every s < world (wrap-safe compare);
// false after about two seconds.
__device__ bool wait_flags(const int* flags, int world, int epoch) {
  const uint64_t t0 = sm100::globaltimer_ns();
  for (int s = 0; s < world; ++s) {
    while (ld_acquire_sys(flags + s) - epoch < 0) {
      if (sm100::globaltimer_ns() - t0 > kTpWaitNs) return false;
      __nanosleep(200);
    }
  }
  return true;
}

// One lane per destination rank, each with its own system-scope fence and a
// relaxed store (a release pattern): the world fences run side by side. A
// single thread storing world release flags one after another waits out a
// full NVLink round trip per flag (each release fences the previous store),
// which costs about 20 us at 8 ranks.
__global__ void tp_signal_kernel(FlagPtrs flags, int world, int rank, int epoch) {
  const int d = threadIdx.x;
  if (d >= world) return;
  __threadfence_system();  // this rank's earlier writes (previous grids) before the flag
  asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(flags.p[d] + rank), "r"(epoch) : "memory");
}

__global__ void tp_wait_kernel(const int* flags, int world, int epoch) {
  if (threadIdx.x != 0) return;
  if (!wait_flags(flags, world, epoch)) atomicExch(&g_tp_error, AXON_E_TIMEOUT);
  // outputs may have arrived through a multicast alias of this rank's buffer
  asm volatile("fence.proxy.alias;" ::: "memory");
}

__global__ void tp_wait_count_kernel(const int* counter, int target) {
  if (threadIdx.x != 0) return;
  if (!wait_flags(counter, 1, target)) atomicExch(&g_tp_error, AXON_E_TIMEOUT);
  // outputs may have arrived through a multicast alias of this rank's buffer
  asm volatile("fence.proxy.alias;" ::: "memory");
}

template <typename Tout>
__device__ __forceinline__ void store8(Tout* dst, const float* v) {
  if constexpr (sizeof(Tout) == 4) {
    reinterpret_cast<float4*>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    Vec<Tout> o;
#pragma unroll
    for (int e = 0; e < 8; ++e) o.e[e] = from_f<Tout>(v[e]);
    st_vec(dst, o);
  }
}

// Eight outputs as 16-byte multimem stores to a multicast address: the
// NVLink switch writes each store into every GPU bound to the multicast
// object, so one rank's output rows reach all ranks for one crossing of its
// own links. A store carries bits only (the .f32 vector form is the
// 16-byte store; no arithmetic is done on the values).
__device__ __forceinline__ void multimem_st16(void* mc, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

template <typename Tout>
__device__ __forceinline__ void store8_multicast(Tout* dst, const float* v) {
  if constexpr (sizeof(Tout) == 4) {
    multimem_st16(dst, make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]),
                                  __float_as_uint(v[3])));
    multimem_st16(dst + 4, make_uint4(__float_as_uint(v[4]), __float_as_uint(v[5]), __float_as_uint(v[6]),
                                      __float_as_uint(v[7])));
  } else {
    Vec<Tout> o;
#pragma unroll
    for (int e = 0; e < 8; ++e) o.e[e] = from_f<Tout>(v[e]);
    multimem_st16(dst, o.u);
  }
}

// inbox: [world][rows][n] f16 partials of this rank's rows; out row i of
// this rank goes to outs.p[d] + (out_row0 + rank * rows + i) * ld_out on every d.
// MC: outs.p[0] is a multicast address and n_outs is 1; the rows reach every
// rank through multimem stores, and each thread ends with an alias-proxy and a
// system-scope fence so the stores are ordered before the done flags that a
// later launch raises.
template <typename Tout, bool MC = false>
__global__ void __launch_bounds__(256) tp_reduce_gather_kernel(const __half* __restrict__ inbox, OutPtrs outs,
                                                               int n_outs, const int* arrive, int world, int rank,
                                                               int epoch, int64_t rows, int64_t n, int64_t out_row0,
                                                               int64_t ld_out) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = wait_flags(arrive, world, epoch);
    if (!ok) atomicExch(&g_tp_error, AXON_E_TIMEOUT);
  }
  __syncthreads();
  if (!ok) return;
  const int64_t slot = rows * n;
  const int64_t packets = slot / 8;
  const int64_t first_row = out_row0 + static_cast<int64_t>(rank) * rows;
  // Two packets per thread per iteration, all of their loads issued before
  // any sum, so each thread keeps 2 * world 16-byte loads in flight.
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t pk0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; pk0 < packets; pk0 += 2 * stride) {
    Vec<__half> v[2][kMaxWorld];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int64_t pk = pk0 + u * stride;
#pragma unroll
      for (int s = 0; s < kMaxWorld; ++s)
        if (s < world && pk < packets)  // written by peers: loads that bypass any cached copy
          v[u][s].u = __ldcv(reinterpret_cast<const uint4*>(inbox + s * slot + pk * 8));
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int64_t pk = pk0 + u * stride;
      if (pk >= packets) break;
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s = 0; s < kMaxWorld; ++s)  // fixed rank order: the sum is the same on every run
        if (s < world)
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] += __half2float(v[u][s].e[e]);
      const int64_t e0 = pk * 8;
      const int64_t i = e0 / n, j = e0 - i * n;
      if constexpr (MC) {
        store8_multicast(static_cast<Tout*>(outs.p[0]) + (first_row + i) * ld_out + j, acc);
      } else {
        for (int d = 0; d < n_outs; ++d) store8(static_cast<Tout*>(outs.p[d]) + (first_row + i) * ld_out + j, acc);
      }
    }
  }
  if constexpr (MC) {
    asm volatile("fence.proxy.alias;" ::: "memory");
    __threadfence_system();
  }
}

// The same reduction for contiguous outputs (ld_out == n), pushed by the bulk
// copy engine: a CTA sums a chunk of whole rows into shared memory, then one
// thread issues a 1-D bulk copy of the chunk to every rank's output
// (cp.async.bulk global <- shared, no multicast), so the all-gather crosses
// NVLink in long bursts instead of per-thread 16-byte stores. Two chunk
// buffers alternate: a buffer is refilled once its copies have read it.
template <typename Tout>
__global__ void __launch_bounds__(256) tp_reduce_push_kernel(const __half* __restrict__ inbox, OutPtrs outs,
                                                             int n_outs, const int* arrive, int world, int rank,
                                                             int epoch, int64_t rows, int64_t n, int64_t out_row0,
                                                             int chunk_rows) {
  extern __shared__ __align__(128) unsigned char cbuf[];
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = wait_flags(arrive, world, epoch);
    if (!ok) atomicExch(&g_tp_error, AXON_E_TIMEOUT);
  }
  __syncthreads();
  if (!ok) return;
  const int64_t slot = rows * n;
  const int64_t nchunks = (rows + chunk_rows - 1) / chunk_rows;
  const int64_t chunk_bytes = static_cast<int64_t>(chunk_rows) * n * sizeof(Tout);
  const int64_t first_row = out_row0 + static_cast<int64_t>(rank) * rows;
  int it = 0;
  for (int64_t ch = blockIdx.x; ch < nchunks; ch += gridDim.x, ++it) {
    Tout* buf = reinterpret_cast<Tout*>(cbuf + (it & 1) * chunk_bytes);
    if (threadIdx.x == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");  // buffer's copies have read it
    __syncthreads();
    const int64_t r0 = ch * chunk_rows;
    const int64_t nr = rows - r0 < chunk_rows ? rows - r0 : chunk_rows;
    const int64_t packets = nr * n / 8;
    const __half* src = inbox + r0 * n;
    for (int64_t pk0 = threadIdx.x; pk0 < packets; pk0 += 2 * blockDim.x) {
      Vec<__half> v[2][kMaxWorld];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int64_t pk = pk0 + u * blockDim.x;
#pragma unroll
        for (int s = 0; s < kMaxWorld; ++s)
          if (s < world && pk < packets) v[u][s].u = __ldcv(reinterpret_cast<const uint4*>(src + s * slot + pk * 8));
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int64_t pk = pk0 + u * blockDim.x;
        if (pk >= packets) break;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int s = 0; s < kMaxWorld; ++s)  // fixed rank order
          if (s < world)
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] += __half2float(v[u][s].e[e]);
        store8(buf + pk * 8, acc);
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // shared-memory writes -> bulk copy reads
    __syncthreads();
    if (threadIdx.x == 0) {
      const uint32_t bytes = static_cast<uint32_t>(nr * n * sizeof(Tout));
      const uint32_t saddr = static_cast<uint32_t>(__cvta_generic_to_shared(buf));
      for (int d = 0; d < n_outs; ++d) {
        Tout* dst = static_cast<Tout*>(outs.p[d]) + (first_row + r0) * n;
        asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(saddr), "r"(bytes)
                     : "memory");
      }
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
  }
  if (threadIdx.x == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // every copy complete
}

PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  }
  return fn;
}

int check_world(int32_t world, int32_t rank, const char* name) {
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world)
    return fail(AXON_E_ARG, "%s: world must be 1..%d and 0 <= rank < world (got %d, %d)", name, kMaxWorld, world,
                rank);
  return AXON_OK;
}

}  // namespace
}  // namespace axon

using namespace axon;

extern "C" int axon_ipc_handle(const void* dev_ptr, void* handle, int64_t* offset) {
  if (!dev_ptr || !handle || !offset) return fail(AXON_E_ARG, "axon_ipc_handle: NULL argument");
  auto range = address_range_fn();
  if (!range) return fail(AXON_E_CUDA, "axon_ipc_handle: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
    return fail(AXON_E_ARG, "axon_ipc_handle: not a device allocation");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return fail(AXON_E_CUDA, "axon_ipc_handle: %s", cudaGetErrorString(e));
  static_assert(sizeof(h) == AXON_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return AXON_OK;
}

extern "C" int axon_ipc_open(const void* handle, int64_t offset, void** dev_ptr) {
  if (!handle || !dev_ptr || offset < 0) return fail(AXON_E_ARG, "axon_ipc_open: bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(AXON_E_CUDA, "axon_ipc_open: %s", cudaGetErrorString(e));
  *dev_ptr = static_cast<unsigned char*>(base) + offset;
  return AXON_OK;
}

extern "C" int axon_ipc_close(void* dev_ptr, int64_t offset) {
  if (!dev_ptr || offset < 0) return fail(AXON_E_ARG, "axon_ipc_close: bad argument");
  cudaError_t e = cudaIpcCloseMemHandle(static_cast<unsigned char*>(dev_ptr) - offset);
  if (e != cudaSuccess) return fail(AXON_E_CUDA, "axon_ipc_close: %s", cudaGetErrorString(e));
  return AXON_OK;
}

extern "C" int axon_tp_signal(int32_t* const* flags, int32_t world, int32_t rank, int32_t epoch, void* stream) {
  int rc = check_world(world, rank, "axon_tp_signal");
  if (rc) return rc;
  if (!flags) return fail(AXON_E_ARG, "axon_tp_signal: NULL flag table");
  FlagPtrs f{};
  for (int d = 0; d < world; ++d) {
    if (!flags[d]) return fail(AXON_E_ARG, "axon_tp_signal: NULL flag array for rank %d", d);
    f.p[d] = flags[d];
  }
  tp_signal_kernel<<<1, 32, 0, as_stream(stream)>>>(f, world, rank, epoch);
  return launch_status("axon_tp_signal");
}

extern "C" int axon_tp_wait(const int32_t* flags, int32_t world, int32_t epoch, void* stream) {
  int rc = check_world(world, 0, "axon_tp_wait");
  if (rc) return rc;
  if (!flags) return fail(AXON_E_ARG, "axon_tp_wait: NULL flags");
  tp_wait_kernel<<<1, 32, 0, as_stream(stream)>>>(flags, world, epoch);
  return launch_status("axon_tp_wait");
}

extern "C" int axon_tp_wait_count(const int32_t* counter, int32_t target, void* stream) {
  if (!counter) return fail(AXON_E_ARG, "axon_tp_wait_count: NULL counter");
  tp_wait_count_kernel<<<1, 32, 0, as_stream(stream)>>>(counter, target);
  return launch_status("axon_tp_wait_count");
}

namespace axon {
namespace {

// The body of axon_tp_reduce_gather (n_outs = world), axon_tp_reduce_local
// (n_outs = 1) and axon_tp_reduce_multicast (n_outs = 1, multicast = true).
int reduce_impl(const void* inbox, void* const* outs, int n_outs, const int32_t* arrive, int32_t world,
                int32_t rank, int32_t epoch, int64_t rows, int64_t n, int64_t out_row0, int64_t ld_out,
                int32_t out_dtype, int32_t max_ctas, void* stream, bool multicast = false) {
  int rc = check_world(world, rank, "axon_tp_reduce_gather");
  if (rc) return rc;
  if (rows < 0 || n < 0 || out_row0 < 0) return fail(AXON_E_SHAPE, "axon_tp_reduce_gather: negative size");
  if (!inbox || !outs || !arrive) return fail(AXON_E_ARG, "axon_tp_reduce_gather: NULL argument");
  if (n % 8 || ld_out % 8 || ld_out < n)
    return fail(AXON_E_SHAPE, "axon_tp_reduce_gather: n and ld_out must be multiples of 8, ld_out >= n");
  if (out_dtype != AXON_BF16 && out_dtype != AXON_F32 && out_dtype != AXON_F16)
    return fail(AXON_E_UNSUPPORTED, "axon_tp_reduce_gather: unsupported output dtype %d", out_dtype);
  if (!aligned16(inbox)) return fail(AXON_E_ALIGN, "axon_tp_reduce_gather: inbox must be 16-byte aligned");
  OutPtrs o{};
  for (int d = 0; d < n_outs; ++d) {
    if (!outs[d] || !aligned16(outs[d])) return fail(AXON_E_ALIGN, "axon_tp_reduce_gather: output %d NULL or unaligned", d);
    o.p[d] = outs[d];
  }
  const int64_t packets = rows * n / 8;
  int64_t grid = (packets + 255) / 256;
  const int64_t cap = max_ctas > 0 ? max_ctas : 2 * sm_count();
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;  // still waits for the arrivals, so the done flags keep their meaning
  cudaStream_t s = as_stream(stream);
  const __half* in = static_cast<const __half*>(inbox);
  // contiguous outputs: whole-row chunks of about 8 KB pushed by bulk copies
  // (small chunks: every SM gets several, its loads and pushes overlap)
  if (multicast) {
    switch (out_dtype) {
      case AXON_BF16:
        tp_reduce_gather_kernel<__nv_bfloat16, true><<<static_cast<unsigned>(grid), 256, 0, s>>>(
            in, o, 1, arrive, world, rank, epoch, rows, n, out_row0, ld_out);
        break;
      case AXON_F16:
        tp_reduce_gather_kernel<__half, true><<<static_cast<unsigned>(grid), 256, 0, s>>>(
            in, o, 1, arrive, world, rank, epoch, rows, n, out_row0, ld_out);
        break;
      default:
        tp_reduce_gather_kernel<float, true><<<static_cast<unsigned>(grid), 256, 0, s>>>(
            in, o, 1, arrive, world, rank, epoch, rows, n, out_row0, ld_out);
        break;
    }
    return launch_status("axon_tp_reduce_multicast");
  }
  const int osize = out_dtype == AXON_F32 ? 4 : 2;
  if (ld_out == n && n * osize <= 32768) {
    const int chunk_rows = n * osize >= 8192 ? 1 : static_cast<int>(8192 / (n * osize));
    const int64_t nchunks = (rows + chunk_rows - 1) / chunk_rows;
    int64_t g2 = nchunks < cap ? nchunks : cap;
    if (g2 < 1) g2 = 1;
    const size_t smem = 2 * static_cast<size_t>(chunk_rows) * n * osize;
    switch (out_dtype) {
      case AXON_BF16: {
        auto k = tp_reduce_push_kernel<__nv_bfloat16>;
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        k<<<static_cast<unsigned>(g2), 256, smem, s>>>(in, o, n_outs, arrive, world, rank, epoch, rows, n,
                                                        out_row0, chunk_rows);
        break;
      }
      case AXON_F16: {
        auto k = tp_reduce_push_kernel<__half>;
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        k<<<static_cast<unsigned>(g2), 256, smem, s>>>(in, o, n_outs, arrive, world, rank, epoch, rows, n,
                                                        out_row0, chunk_rows);
        break;
      }
      default: {
        auto k = tp_reduce_push_kernel<float>;
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        k<<<static_cast<unsigned>(g2), 256, smem, s>>>(in, o, n_outs, arrive, world, rank, epoch, rows, n,
                                                        out_row0, chunk_rows);
        break;
      }
    }
    return launch_status("axon_tp_reduce_gather");
  }
  switch (out_dtype) {
    case AXON_BF16:
      tp_reduce_gather_kernel<__nv_bfloat16><<<static_cast<unsigned>(grid), 256, 0, s>>>(in, o, n_outs, arrive, world, rank,
                                                                                          epoch, rows, n, out_row0,
                                                                                          ld_out);
      break;
    case AXON_F16:
      tp_reduce_gather_kernel<__half><<<static_cast<unsigned>(grid), 256, 0, s>>>(in, o, n_outs, arrive, world, rank, epoch,
                                                                                   rows, n, out_row0, ld_out);
      break;
    default:
      tp_reduce_gather_kernel<float><<<static_cast<unsigned>(grid), 256, 0, s>>>(in, o, n_outs, arrive, world, rank, epoch,
                                                                                  rows, n, out_row0, ld_out);
      break;
  }
  return launch_status("axon_tp_reduce_gather");
}

}  // namespace
}  // namespace axon

extern "C" int axon_tp_reduce_gather(const void* inbox, void* const* outs, const int32_t* arrive, int32_t world,
                                     int32_t rank, int32_t epoch, int64_t rows, int64_t n, int64_t out_row0,
                                     int64_t ld_out, int32_t out_dtype, int32_t max_ctas, void* stream) {
  return reduce_impl(inbox, outs, world, arrive, world, rank, epoch, rows, n, out_row0, ld_out, out_dtype, max_ctas,
                     stream);
}

extern "C" int axon_tp_reduce_local(const void* inbox, void* out, const int32_t* arrive, int32_t world,
                                    int32_t rank, int32_t epoch, int64_t rows, int64_t n, int64_t out_row0,
                                    int64_t ld_out, int32_t out_dtype, int32_t max_ctas, void* stream) {
  void* one[1] = {out};
  return reduce_impl(inbox, one, 1, arrive, world, rank, epoch, rows, n, out_row0, ld_out, out_dtype, max_ctas,
                     stream);
}

extern "C" int axon_tp_reduce_multicast(const void* inbox, void* out_mc, const int32_t* arrive, int32_t world,
                                        int32_t rank, int32_t epoch, int64_t rows, int64_t n, int64_t out_row0,
                                        int64_t ld_out, int32_t out_dtype, int32_t max_ctas, void* stream) {
  void* one[1] = {out_mc};
  return reduce_impl(inbox, one, 1, arrive, world, rank, epoch, rows, n, out_row0, ld_out, out_dtype, max_ctas,
                     stream, true);
}

extern "C" int axon_tp_push_rows(const void* src, void* const* dsts, int64_t bytes, int32_t world, int32_t rank,
                                 void* stream) {
  int rc = check_world(world, rank, "axon_tp_push_rows");
  if (rc) return rc;
  if (bytes < 0 || !src || !dsts) return fail(AXON_E_ARG, "axon_tp_push_rows: bad argument");
  cudaStream_t s = as_stream(stream);
  // one copy per peer, in ring order from the next rank so that the ranks'
  // copies spread over the peers instead of all hitting rank 0 first
  for (int i = 1; i < world; ++i) {
    const int d = (rank + i) % world;
    if (!dsts[d]) return fail(AXON_E_ARG, "axon_tp_push_rows: NULL destination for rank %d", d);
    cudaError_t e = cudaMemcpyAsync(dsts[d], src, static_cast<size_t>(bytes), cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return fail(AXON_E_CUDA, "axon_tp_push_rows: %s", cudaGetErrorString(e));
  }
  return AXON_OK;
}

extern "C" int axon_tp_status(void* stream) {
  int v = 0;
  cudaStream_t s = as_stream(stream);
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_tp_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return fail(AXON_E_CUDA, "axon_tp_status: %s", cudaGetErrorString(e));
  if (v != 0) {
    int zero = 0;
    cudaMemcpyToSymbolAsync(g_tp_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
    cudaStreamSynchronize(s);
    return fail(v, "tensor-parallel step: a peer flag wait gave up (status %d)", v);
  }
  return AXON_OK;
}
