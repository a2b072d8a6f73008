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
// caches it; make that first call before any stream capture begins. The cache
// is keyed by the context's process-unique id as well: after cudaDeviceReset
// the device gets a new context with the array at a new address, and the next
// call looks it up again.
#include <mutex>

#include "common.cuh"
#include "host_util.h"

namespace ssam {

// 32 MiB: enough for 2,600 rows of a ViT-H MLP (C = 1280, hidden = 5120) per call.
constexpr size_t kNoAllocScratchBytes = static_cast<size_t>(32) << 20;

static __device__ __align__(256) uint8_t g_rc_mlp_scratch[kNoAllocScratchBytes];

struct ScratchSlot {
  unsigned long long ctx_id;  // cuCtxGetId of the context the address belongs to
  void* addr;                 // device address of g_rc_mlp_scratch in that context
};
static std::mutex g_scratch_mutex;
static ScratchSlot g_scratch[kMaxDevices] = {};

typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

// cuCtxGetId through the runtime's driver entry point (the library does not link libcuda).
static CtxGetIdFn ctx_get_id_fn() {
  static CtxGetIdFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetIdFn>(p);
  });
  return fn;
}

// Id of the current context; false when no context is current yet.
static bool current_ctx_id(unsigned long long* id) {
  CtxGetIdFn fn = ctx_get_id_fn();
  return fn != nullptr && fn(nullptr, id) == CUDA_SUCCESS;
}

// Device address of the scratch array in the current context of the current device.
static int noalloc_scratch(int dev, void** addr) {
  unsigned long long id = 0;
  const bool have_id = current_ctx_id(&id);
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  ScratchSlot& slot = g_scratch[dev];
  if (!have_id || slot.addr == nullptr || slot.ctx_id != id) {
    void* p = nullptr;  // (the lookup also creates the device's context if none is current)
    if (cudaGetSymbolAddress(&p, g_rc_mlp_scratch) != cudaSuccess || p == nullptr) return SSAM_ERR_CUDA;
    if (!current_ctx_id(&id)) return SSAM_ERR_CUDA;
    slot.ctx_id = id;
    slot.addr = p;
  }
  *addr = slot.addr;
  return SSAM_OK;
}

// A stream the caller passes must belong to the current device: the scratch
// address is that device's. NULL and the two special default-stream handles
// always refer to the current device.
static int check_stream_device(cudaStream_t stream, int dev) {
  if (stream == nullptr || stream == cudaStreamLegacy || stream == cudaStreamPerThread) return SSAM_OK;
  int sdev = -1;
  if (cudaStreamGetDevice(stream, &sdev) != cudaSuccess) return SSAM_ERR_INVALID;
  return sdev == dev ? SSAM_OK : SSAM_ERR_INVALID;
}

}  // namespace ssam

extern "C" int ssam_rc_mlp_fwd_noalloc(float* x, int64_t ldx, const int32_t* rows, int n_rows, int C, int hidden,
                                       const float* ln_w, const float* ln_b, float eps, const void* w1,
                                       const float* b1, const void* w2, const float* b2, void* stream) {
  if (n_rows < 0 || C <= 0 || hidden <= 0) return SSAM_ERR_INVALID;
  if (n_rows == 0) return SSAM_OK;
  const size_t need = ssam::rc_mlp_workspace_size(n_rows, C, hidden);
  if (need > ssam::kNoAllocScratchBytes) return SSAM_ERR_UNSUPPORTED;  // beyond the fixed scratch capacity
  const int dev = ssam::current_device();
  if (dev < 0) return SSAM_ERR_CUDA;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  int st = ssam::check_stream_device(s, dev);
  if (st != SSAM_OK) return st;
  void* scratch = nullptr;
  st = ssam::noalloc_scratch(dev, &scratch);
  if (st != SSAM_OK) return st;
  // Every intermediate is fully written before it is read, so nothing in the
  // scratch has to be cleared between calls.
  return ssam::rc_mlp_fwd(x, ldx, rows, n_rows, C, hidden, ln_w, ln_b, eps, w1, b1, w2, b2, scratch,
                          ssam::kNoAllocScratchBytes, s);
}
