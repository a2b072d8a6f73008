// Residual-Consistency MLP without a caller workspace.
//
// ssam_rc_mlp_fwd() needs an intermediate buffer (the gathered, normalised rows
// and the fc1 activations) that the caller allocates. Some callers cannot
// allocate device memory at call time: a host that reserves its whole device
// memory budget up front and forbids allocation on the serving path, or a
// foreign-language binding (cgo, JNI, ctypes) that has no device allocator of
// its own. For them this file keeps a fixed scratch area inside the library
// image and runs the same RC-MLP kernels on it.
//
// The scratch is a file-scope device array of kNoAllocScratchBytes. Every GPU
// that loads the library holds it until the process exits. Host code cannot use
// the array's name as a device address, so the first call on each device looks
// the address up once with cudaGetSymbolAddress (with that device current) and
// caches it; make that first call before any stream capture begins.
#include <mutex>

#include "common.cuh"
#include "host_util.h"

namespace ssam {

// 32 MiB: enough for 2,600 rows of a ViT-H MLP (C = 1280, hidden = 5120) per call.
constexpr size_t kNoAllocScratchBytes = static_cast<size_t>(32) << 20;

static __device__ __align__(256) uint8_t g_rc_mlp_scratch[kNoAllocScratchBytes];

static std::mutex g_scratch_mutex;
static void* g_scratch_addr[64] = {nullptr};  // device address of g_rc_mlp_scratch, per device

// Device address of the scratch array on the current device (looked up once).
static int noalloc_scratch(void** addr) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return SSAM_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_rc_mlp_scratch) != cudaSuccess || p == nullptr) return SSAM_ERR_CUDA;
    g_scratch_addr[dev] = p;
  }
  *addr = g_scratch_addr[dev];
  return SSAM_OK;
}

}  // namespace ssam

extern "C" int ssam_rc_mlp_fwd_noalloc(float* x, int64_t ldx, const int32_t* rows, int n_rows, int C, int hidden,
                                       const float* ln_w, const float* ln_b, float eps, const void* w1,
                                       const float* b1, const void* w2, const float* b2, void* stream) {
  if (n_rows < 0 || C <= 0 || hidden <= 0) return SSAM_ERR_INVALID;
  if (n_rows == 0) return SSAM_OK;
  const size_t need = ssam::rc_mlp_workspace_size(n_rows, C, hidden);
  if (need > ssam::kNoAllocScratchBytes) return SSAM_ERR_UNSUPPORTED;  // beyond the fixed scratch capacity
  void* scratch = nullptr;
  const int st = ssam::noalloc_scratch(&scratch);
  if (st != SSAM_OK) return st;
  // Every intermediate is fully written before it is read, so nothing in the
  // scratch has to be cleared between calls.
  return ssam::rc_mlp_fwd(x, ldx, rows, n_rows, C, hidden, ln_w, ln_b, eps, w1, b1, w2, b2, scratch,
                          ssam::kNoAllocScratchBytes, static_cast<cudaStream_t>(stream));
}
