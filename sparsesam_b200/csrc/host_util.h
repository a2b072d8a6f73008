// Host-side helpers shared by the launchers: alignment checks, SM count cache,
// TMA tensor-map encoding through the driver entry point (no -lcuda needed).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "../../include/sparsesam.h"

namespace ssam {

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

constexpr int kMaxDevices = 64;

// One-time, per-device launch set-up (cudaFuncSetAttribute and the like) that
// several host threads may reach at once: later calls read one atomic flag,
// first calls serialise on a mutex, and a set-up that failed runs again on the
// next call. `setup` returns an SSAM status.
class PerDeviceOnce {
 public:
  template <class F>
  int run(int dev, F&& setup) {
    if (dev < 0 || dev >= kMaxDevices) return SSAM_ERR_CUDA;
    if (done_[dev].load(std::memory_order_acquire)) return SSAM_OK;
    std::lock_guard<std::mutex> lock(mu_);
    if (done_[dev].load(std::memory_order_relaxed)) return SSAM_OK;
    const int st = setup();
    if (st == SSAM_OK) done_[dev].store(true, std::memory_order_release);
    return st;
  }

 private:
  std::atomic<bool> done_[kMaxDevices] = {};
  std::mutex mu_;
};

// The current device, or -1.
inline int current_device() {
  int dev = -1;
  return cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kMaxDevices ? dev : -1;
}

// Multiprocessor count of `dev` (cached; 148 on B200).
int num_sms(int dev);

// 2-D bf16 tensor map over a row-major [rows, cols] matrix with leading
// dimension `ld` (elements). Box = box_cols x box_rows; out-of-bounds reads fill 0.
int make_tmap_nhwc_bf16(CUtensorMap* map, const void* base, int B, int H, int W, int C, uint32_t box_c, uint32_t box_w,
                        uint32_t box_h);
int make_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                      uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle);

int status_from_cuda(cudaError_t e);

// Entry points implemented in the per-kernel translation units.
int conv3x3_nhwc(const void* in, int B, int H, int W, int Cin, const void* w, int Cout, const float* bias, void* out,
                 cudaStream_t stream);
int layernorm_half(const void* x, int64_t rows, int C, const void* w, const void* b, float eps, int gelu, int dtype,
                   void* out, cudaStream_t stream);
int gemm_bf16_addend(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K, const float* bias,
                     const float* addend, int addend_rows, float* out, cudaStream_t stream);
int gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K, const float* bias,
              int epilogue, void* out, int64_t ldo, const int32_t* out_rows, cudaStream_t stream);

int zorder(int H, int W, int32_t* perm, int32_t* inv_perm, cudaStream_t stream);
int stripe_sort_perm(const void* k, int64_t ld, int n_seq, int heads, int H, int W, int d, int gs, int layout,
                     int ranking, const int32_t* base_perm, int32_t* perm, int32_t* inv_perm, int32_t* inv_perm_group,
                     cudaStream_t stream);
int keep_select(const int32_t* inv_perm_group, int B, int heads, int N, int keep_n, int32_t* idx, int32_t* rows,
                cudaStream_t stream);
int a_shape_n_init(int N, int n_block, double ratio, int is_global);
int zstride_keep_n(int N, double ratio);
int zstride_keep(int H, int W, int keep_n, int B, int32_t* idx, int32_t* rows, cudaStream_t stream);
int a_shape_mask(int N, int m_block, int n_block, int n_init, int with_diag, uint8_t* mask);
size_t sparse_attn_workspace_size(int n_seq, int heads, int win);
int sparse_attn_fwd(const void* qkv, int64_t ld_qkv, int n_seq, int heads, int win, int d, const void* rel_pos_h,
                    const void* rel_pos_w, const int32_t* perm, int n_init_blocks, int n_block, int with_diag, float scale,
                    void* out, int64_t ld_out, const int32_t* out_rows, int grid_h, int grid_w, const void* pad_row,
                    void* workspace, size_t workspace_bytes, cudaStream_t stream);
int layernorm_gather(const float* x, int64_t ldx, const int32_t* src_rows, int n_rows, int C, const float* w,
                     const float* b, float eps, void* out, int64_t ld_out, cudaStream_t stream);
int hilbert_order(int H, int W, int32_t* perm, int32_t* inv_perm, cudaStream_t stream);
int layernorm_rows(const float* x, int n_rows, int C, const float* w, const float* b, float eps, void* out,
                   int out_mode, cudaStream_t stream);
int layernorm_nchw(const float* x, int B, int HW, int C, const float* w, const float* b, float eps, float* out,
                   cudaStream_t stream);
int layernorm_rows_copy(const float* x, int n_rows, int C, const float* w, const float* b, float eps, void* out,
                        float* copy, cudaStream_t stream);
int window_rows(int B, int H, int W, int ws, int32_t* rows, cudaStream_t stream);
int patch_im2col(const float* img, int B, int Cin, int H, int W, int p, void* out, cudaStream_t stream);
int broadcast_rows(const float* pos, int B, int T, int C, float* x, cudaStream_t stream);
int im2col3x3_nhwc(const void* in, int B, int H, int W, int C, void* out, cudaStream_t stream);
int nhwc_to_nchw(const float* in, int B, int HW, int C, float* out, cudaStream_t stream);
int split_bf16x2(const float* x, int n_rows, int C, void* out, cudaStream_t stream);
int split_bf16x3(const float* x, int n_rows, int C, void* out, cudaStream_t stream);
int window_of_raster(int B, int H, int W, int ws, int32_t* win_rows, cudaStream_t stream);
int fill_pad_rows(void* out, int64_t ld, const int32_t* rows, int n_rows, int C, const float* bias,
                  cudaStream_t stream);
int patch_im2col_split3(const float* img, int B, int Cin, int H, int W, int p, void* out, cudaStream_t stream);
size_t rc_mlp_workspace_size(int n_rows, int C, int hidden);
int rc_mlp_fwd(float* x, int64_t ldx, const int32_t* rows, int n_rows, int C, int hidden, const float* ln_w,
               const float* ln_b, float eps, const void* w1, const float* b1, const void* w2, const float* b2,
               void* workspace, size_t workspace_bytes, cudaStream_t stream);

}  // namespace ssam
