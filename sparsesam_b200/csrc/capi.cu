// extern "C" surface of libsparsesam_b200.so (declared in include/sparsesam.h).
// Each entry validates its arguments on the host, then enqueues kernels on the
// caller's stream and returns a status code.
#include "common.cuh"
#include "host_util.h"

using ssam::status_from_cuda;

namespace ssam {
// One CTA waits on an mbarrier phase that nothing completes: the bounded wait
// gives up (~2 s), raises SSAM_ERR_TIMEOUT on the device flag and returns.
__global__ void wait_timeout_check_kernel() {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0);
  __syncthreads();
}
}  // namespace ssam

extern "C" {

int ssam_version(void) { return 100; }

const char* ssam_status_string(int status) {
  switch (status) {
    case SSAM_OK:
      return "ok";
    case SSAM_ERR_INVALID:
      return "invalid argument";
    case SSAM_ERR_ALIGN:
      return "misaligned pointer or leading dimension";
    case SSAM_ERR_UNSUPPORTED:
      return "unsupported shape";
    case SSAM_ERR_CUDA:
      return "CUDA error";
    case SSAM_ERR_TIMEOUT:
      return "device wait timed out";
    default:
      return "unknown status";
  }
}

int ssam_device_error(int reset) {
  if (cudaDeviceSynchronize() != cudaSuccess) return SSAM_ERR_CUDA;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, ssam::g_device_error, sizeof(int)) != cudaSuccess) return SSAM_ERR_CUDA;
  if (reset) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(ssam::g_device_error, &zero, sizeof(int)) != cudaSuccess) return SSAM_ERR_CUDA;
  }
  return v;
}

int ssam_check_wait_timeout(void* stream) {
  ssam::wait_timeout_check_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>();
  return status_from_cuda(cudaGetLastError());
}

int ssam_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K, const float* bias,
                   int epilogue, void* out, int64_t ldo, const int32_t* out_rows, void* stream) {
  return ssam::gemm_bf16(A, lda, B, ldb, M, N, K, bias, epilogue, out, ldo, out_rows,
                         static_cast<cudaStream_t>(stream));
}

int ssam_hilbert_order(int H, int W, int32_t* perm, int32_t* inv_perm, void* stream) {
  return ssam::hilbert_order(H, W, perm, inv_perm, static_cast<cudaStream_t>(stream));
}

int ssam_zorder(int H, int W, int32_t* perm, int32_t* inv_perm, void* stream) {
  return ssam::zorder(H, W, perm, inv_perm, static_cast<cudaStream_t>(stream));
}

int ssam_stripe_sort_perm(const void* k, int64_t ld, int n_seq, int heads, int H, int W, int d, int group_size,
                          int layout, int ranking, const int32_t* base_perm, int32_t* perm, int32_t* inv_perm,
                          int32_t* inv_perm_group, void* stream) {
  return ssam::stripe_sort_perm(k, ld, n_seq, heads, H, W, d, group_size, layout, ranking, base_perm, perm, inv_perm,
                                inv_perm_group, static_cast<cudaStream_t>(stream));
}

int ssam_a_shape_n_init(int N, int n_block, double ratio, int is_global) {
  return ssam::a_shape_n_init(N, n_block, ratio, is_global);
}

int ssam_a_shape_mask(int N, int m_block, int n_block, int n_init, int with_diag, uint8_t* mask) {
  return ssam::a_shape_mask(N, m_block, n_block, n_init, with_diag, mask);
}

size_t ssam_sparse_attn_workspace_size(int n_seq, int heads, int win, int d) {
  (void)d;
  return ssam::sparse_attn_workspace_size(n_seq, heads, win);
}

int ssam_sparse_attn_fwd(const void* qkv, int64_t ld_qkv, int n_seq, int heads, int win, int d, const void* rel_pos_h,
                         const void* rel_pos_w, const int32_t* perm, int n_init_blocks, int n_block, int with_diag,
                         float scale, void* out, int64_t ld_out, const int32_t* out_rows, int grid_h, int grid_w,
                         const void* pad_row, void* workspace, size_t workspace_bytes, void* stream) {
  return ssam::sparse_attn_fwd(qkv, ld_qkv, n_seq, heads, win, d, rel_pos_h, rel_pos_w, perm, n_init_blocks, n_block,
                               with_diag, scale, out, ld_out, out_rows, grid_h, grid_w, pad_row, workspace,
                               workspace_bytes, static_cast<cudaStream_t>(stream));
}

int ssam_keep_select(const int32_t* inv_perm_group, int B, int heads, int N, int keep_n, int32_t* idx, int32_t* rows,
                     void* stream) {
  return ssam::keep_select(inv_perm_group, B, heads, N, keep_n, idx, rows, static_cast<cudaStream_t>(stream));
}

int ssam_zstride_keep_n(int N, double ratio) { return ssam::zstride_keep_n(N, ratio); }

int ssam_zstride_keep(int H, int W, int keep_n, int B, int32_t* idx, int32_t* rows, void* stream) {
  return ssam::zstride_keep(H, W, keep_n, B, idx, rows, static_cast<cudaStream_t>(stream));
}

int ssam_layernorm_gather(const float* x, int64_t ldx, const int32_t* src_rows, int n_rows, int C, const float* w,
                          const float* b, float eps, void* out, int64_t ld_out, void* stream) {
  return ssam::layernorm_gather(x, ldx, src_rows, n_rows, C, w, b, eps, out, ld_out, static_cast<cudaStream_t>(stream));
}

int ssam_window_rows(int B, int H, int W, int ws, int32_t* rows, void* stream) {
  return ssam::window_rows(B, H, W, ws, rows, static_cast<cudaStream_t>(stream));
}

size_t ssam_rc_mlp_workspace_size(int n_rows, int C, int hidden) {
  return ssam::rc_mlp_workspace_size(n_rows, C, hidden);
}

int ssam_rc_mlp_fwd(float* x, int64_t ldx, const int32_t* rows, int n_rows, int C, int hidden, const float* ln_w,
                    const float* ln_b, float eps, const void* w1, const float* b1, const void* w2, const float* b2,
                    void* workspace, size_t workspace_bytes, void* stream) {
  return ssam::rc_mlp_fwd(x, ldx, rows, n_rows, C, hidden, ln_w, ln_b, eps, w1, b1, w2, b2, workspace, workspace_bytes,
                          static_cast<cudaStream_t>(stream));
}

int ssam_patch_im2col(const float* img, int B, int Cin, int H, int W, int p, void* out, void* stream) {
  return ssam::patch_im2col(img, B, Cin, H, W, p, out, static_cast<cudaStream_t>(stream));
}

int ssam_broadcast_rows(const float* pos, int B, int T, int C, float* x, void* stream) {
  return ssam::broadcast_rows(pos, B, T, C, x, static_cast<cudaStream_t>(stream));
}

int ssam_im2col3x3_nhwc(const void* in, int B, int H, int W, int C, void* out, void* stream) {
  return ssam::im2col3x3_nhwc(in, B, H, W, C, out, static_cast<cudaStream_t>(stream));
}

int ssam_gemm_bf16_addend(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K,
                          const float* bias, const float* addend, int addend_rows, float* out, void* stream) {
  return ssam::gemm_bf16_addend(A, lda, B, ldb, M, N, K, bias, addend, addend_rows, out,
                                static_cast<cudaStream_t>(stream));
}

int ssam_conv3x3_nhwc(const void* in, int B, int H, int W, int Cin, const void* w, int Cout, const float* bias,
                      void* out, void* stream) {
  return ssam::conv3x3_nhwc(in, B, H, W, Cin, w, Cout, bias, out, static_cast<cudaStream_t>(stream));
}

int ssam_nhwc_to_nchw(const float* in, int B, int HW, int C, float* out, void* stream) {
  return ssam::nhwc_to_nchw(in, B, HW, C, out, static_cast<cudaStream_t>(stream));
}

int ssam_layernorm_rows(const float* x, int n_rows, int C, const float* w, const float* b, float eps, void* out,
                        int out_mode, void* stream) {
  return ssam::layernorm_rows(x, n_rows, C, w, b, eps, out, out_mode, static_cast<cudaStream_t>(stream));
}

int ssam_layernorm_nchw(const float* x, int B, int HW, int C, const float* w, const float* b, float eps, float* out,
                        void* stream) {
  return ssam::layernorm_nchw(x, B, HW, C, w, b, eps, out, static_cast<cudaStream_t>(stream));
}

int ssam_layernorm_gelu_half(const void* x, int64_t rows, int C, const void* w, const void* b, float eps, int gelu,
                             int dtype, void* out, void* stream) {
  return ssam::layernorm_half(x, rows, C, w, b, eps, gelu, dtype, out, static_cast<cudaStream_t>(stream));
}

int ssam_layernorm_rows_copy(const float* x, int n_rows, int C, const float* w, const float* b, float eps,
                             void* out_bf16, float* copy, void* stream) {
  return ssam::layernorm_rows_copy(x, n_rows, C, w, b, eps, out_bf16, copy, static_cast<cudaStream_t>(stream));
}

int ssam_split_bf16x2(const float* x, int n_rows, int C, void* out, void* stream) {
  return ssam::split_bf16x2(x, n_rows, C, out, static_cast<cudaStream_t>(stream));
}

int ssam_window_of_raster(int B, int H, int W, int ws, int32_t* win_rows, void* stream) {
  return ssam::window_of_raster(B, H, W, ws, win_rows, static_cast<cudaStream_t>(stream));
}

int ssam_fill_pad_rows(void* out, int64_t ld, const int32_t* rows, int n_rows, int C, const float* bias,
                       void* stream) {
  return ssam::fill_pad_rows(out, ld, rows, n_rows, C, bias, static_cast<cudaStream_t>(stream));
}

int ssam_split_bf16x3(const float* x, int n_rows, int C, void* out, void* stream) {
  return ssam::split_bf16x3(x, n_rows, C, out, static_cast<cudaStream_t>(stream));
}

int ssam_patch_im2col_split3(const float* img, int B, int Cin, int H, int W, int p, void* out, void* stream) {
  return ssam::patch_im2col_split3(img, B, Cin, H, W, p, out, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
