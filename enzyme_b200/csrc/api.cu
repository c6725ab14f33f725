// Library metadata and error plumbing shared by every entry point.
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace axon {

const char* last_error_cstr();

namespace {
thread_local std::string g_last_error;
}

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

void clear_error() { g_last_error.clear(); }

const char* last_error_cstr() { return g_last_error.c_str(); }

int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(AXON_E_LAUNCH, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return AXON_OK;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("AXON_B200_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace axon

// Variant catalogue: what each op accepts in axon_tune_t. Each entry is
// (op, JSON). The bench runner turns these into Axon's (hw_variant,
// TILES_IN_BLOCK_*) sweep.
static const char* kVariants[][2] = {
    {"rmsnorm",
     "{\"op\":\"rmsnorm\",\"variants\":[{\"id\":0,\"name\":\"auto_bulk_or_resident\",\"knobs\":{\"threads\":[0,64,128,256,512,1024]}},"
     "{\"id\":1,\"name\":\"row_streaming\",\"knobs\":{\"threads\":[0,128,256,512,1024]}},"
     "{\"id\":2,\"name\":\"row_bulk_warp\",\"knobs\":{\"threads\":[0,128,256,512,1024]}},"
     "{\"id\":3,\"name\":\"row_bulk_cta\",\"knobs\":{\"threads\":[0,256,512,1024],\"block_k\":[0,4,8,16,32]}}]}"},
    {"layernorm",
     "{\"op\":\"layernorm\",\"variants\":[{\"id\":0,\"name\":\"auto_bulk_or_resident\",\"knobs\":{\"threads\":[0,64,128,256,512,1024]}},"
     "{\"id\":1,\"name\":\"row_streaming\",\"knobs\":{\"threads\":[0,128,256,512,1024]}},"
     "{\"id\":2,\"name\":\"row_bulk_warp\",\"knobs\":{\"threads\":[0,128,256,512,1024]}},"
     "{\"id\":3,\"name\":\"row_bulk_cta\",\"knobs\":{\"threads\":[0,256,512,1024],\"block_k\":[0,4,8,16,32]}}]}"},
    {"softmax",
     "{\"op\":\"softmax\",\"variants\":[{\"id\":0,\"name\":\"auto_bulk_or_resident\",\"knobs\":{\"threads\":[0,64,128,256,512,1024]}},"
     "{\"id\":1,\"name\":\"row_streaming\",\"knobs\":{\"threads\":[0,128,256,512,1024]}},"
     "{\"id\":2,\"name\":\"row_bulk_warp\",\"knobs\":{\"threads\":[0,128,256,512,1024]}},"
     "{\"id\":3,\"name\":\"row_bulk_cta\",\"knobs\":{\"threads\":[0,256,512,1024],\"block_k\":[0,4,8,16,32]}}]}"},
    {"rope",
     "{\"op\":\"rope\",\"variants\":[{\"id\":0,\"name\":\"token_blocked\",\"knobs\":{}},"
     "{\"id\":1,\"name\":\"flat_vec16\",\"knobs\":{\"threads\":[0,128,256]}}]}"},
    {"cumsum",
     "{\"op\":\"cumsum\",\"variants\":[{\"id\":0,\"name\":\"decoupled_lookback\",\"knobs\":{\"split\":[0,2048,4096,8192,16384]}},"
     "{\"id\":1,\"name\":\"cluster_dsmem\",\"knobs\":{\"split\":[0,1,2,4,8]}},"
     "{\"id\":2,\"name\":\"row_stream\",\"knobs\":{\"stages\":[0,2,3,4],\"block_k\":[0,16,24,32,48],\"split\":[0,1,2]}},"
     "{\"id\":3,\"name\":\"balanced_ranges\",\"knobs\":{\"stages\":[0,2,3,4,6],\"block_k\":[0,16,32],\"max_ctas\":[0]}}]}"},
    {"adam",
     "{\"op\":\"adam\",\"variants\":[{\"id\":0,\"name\":\"grid_stride_vec\",\"knobs\":{\"threads\":[0,128,256,512]}}]}"},
    {"gemm",
     "{\"op\":\"gemm\",\"variants\":[{\"id\":0,\"name\":\"auto\",\"knobs\":{}},"
     "{\"id\":1,\"name\":\"tcgen05_ws_persistent\",\"knobs\":{\"block_m\":[0,128],"
     "\"block_n\":[0,64,128,256],\"block_k\":[0,64],\"stages\":[0,2,3,4,5,6,7,8],\"max_ctas\":[0],\"split\":[0,4,8,16]}},"
     "{\"id\":2,\"name\":\"tcgen05_cta_pair\",\"knobs\":{\"block_m\":[0,128],"
     "\"block_n\":[0,128,256],\"block_k\":[0,64],\"stages\":[0,2,3,4,5,6,7,8],\"max_ctas\":[0],\"split\":[0,4,8,16]}}]}"},
};

extern "C" {

const char* axon_version(void) { return "axon_b200 0.1.0 sm_100a"; }

const char* axon_last_error(void) { return axon::last_error_cstr(); }

int64_t axon_variants(const char* op, char* buf, int64_t len) {
  if (op == nullptr) return axon::fail(AXON_E_ARG, "axon_variants: op is NULL");
  for (auto& e : kVariants) {
    if (std::strcmp(e[0], op) == 0) {
      int64_t need = static_cast<int64_t>(std::strlen(e[1]));
      if (buf != nullptr && len > 0) {
        int64_t n = need < len - 1 ? need : len - 1;
        std::memcpy(buf, e[1], static_cast<size_t>(n));
        buf[n] = '\0';
      }
      return need;
    }
  }
  return axon::fail(AXON_E_UNSUPPORTED, "axon_variants: unknown op '%s'", op);
}

}  // extern "C"
