/*
 * sparsesam.h — C ABI of the B200 (sm_100a) SparseSAM image-encoder hot path.
 *
 * Conventions shared by every entry point:
 *   - All tensor arguments are caller-owned DEVICE pointers; nothing on the hot
 *     path allocates. Composite calls that need intermediates take a caller
 *     workspace whose size the matching *_workspace_size() query returns.
 *   - `stream` is a cudaStream_t passed as void*; NULL means the legacy stream.
 *   - Every call returns an int status (SSAM_OK or an SSAM_ERR_* code); no C++
 *     exception crosses this boundary. Calls only enqueue work: device-side
 *     failures (a bounded wait that ran out) are reported by ssam_device_error().
 *   - bf16 tensors are passed as `void*` holding IEEE bfloat16 values; fp32 as float*.
 *   - Calls are re-entrant: the only library globals are the device error flag
 *     and per-process caches of immutable launch configuration.
 *
 * Reference paths below are relative to the hchautran/SparseSAM repository.
 */
#ifndef SPARSESAM_B200_H_
#define SPARSESAM_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SSAM_OK 0
#define SSAM_ERR_INVALID 1     /* bad argument: null pointer, shape, ratio, mode   */
#define SSAM_ERR_ALIGN 2       /* pointer or leading dimension misaligned for TMA  */
#define SSAM_ERR_UNSUPPORTED 3 /* shape outside what the kernels implement         */
#define SSAM_ERR_CUDA 4        /* CUDA runtime / driver error while launching      */
#define SSAM_ERR_TIMEOUT 5     /* a bounded device-side wait ran out               */

/* GEMM epilogues (ssam_gemm_bf16). */
#define SSAM_EPI_BF16 0      /* out_bf16[r, n] = acc + bias[n]                         */
#define SSAM_EPI_GELU_BF16 1 /* out_bf16[r, n] = gelu_erf(acc + bias[n])               */
#define SSAM_EPI_ADD_F32 2   /* out_f32[rows[r], n] += acc + bias[n]; rows[r] < 0 skip */
#define SSAM_EPI_F32 3       /* out_f32[r, n] = acc + bias[n]                          */

/* Stripe-sort layouts and rankings (perm_mode = <space>_<layout>_<ranking>). */
#define SSAM_LAYOUT_INTERLEAVE 0
#define SSAM_LAYOUT_NAIVE 1
#define SSAM_RANKING_SORT 0
#define SSAM_RANKING_NOSORT 1

/* Library version (major*10000 + minor*100 + patch). */
int ssam_version(void);

/* Human-readable text for a status code. */
const char* ssam_status_string(int status);

/* Synchronises the current device and returns the device-side error flag
 * (SSAM_OK when no kernel raised one). `reset` != 0 clears it. */
int ssam_device_error(int reset);

/* Diagnostic for integrators (no counterpart in the reference): enqueues one
 * small kernel whose bounded wait nothing satisfies, so it gives up after about
 * two seconds, raises SSAM_ERR_TIMEOUT on the device flag and returns, the same
 * path every kernel of this library takes when a wait runs out. A following
 * ssam_device_error() reports SSAM_ERR_TIMEOUT; the context stays usable. */
int ssam_check_wait_timeout(void* stream);

/* ---------------------------------------------------------------------------
 * a1. Morton (Z-curve) raster->Z permutation of an H x W grid.
 * Replaces algos/sparsesam/z_utils.py:35-49 (encode), :65-85 (_compute_z_order),
 * :88-101 (get_z_order) and :104-113 (get_z_inverse).
 * perm[i] = raster index of the i-th token in Z order; inv_perm may be NULL.
 * ------------------------------------------------------------------------- */
int ssam_zorder(int H, int W, int32_t* perm, int32_t* inv_perm, void* stream);

/* Hilbert-curve raster->Hilbert permutation of an H x W grid, the base order of
 * the "hilbert" perm_mode space. Replaces algos/sparsesam/hilbert_utils.py:
 * 55-76 (_forward_hilbert_transform), :28-33 (_transposed_to_h), :108-129
 * (_compute_hilbert_order) and :132-147 (get_hilbert_order / _inverse), as
 * called at sam.py:131-132. Same outputs as ssam_zorder. */
int ssam_hilbert_order(int H, int W, int32_t* perm, int32_t* inv_perm, void* stream);

/* ---------------------------------------------------------------------------
 * a2. Stripe-Sort permutation of every (sequence, head) row of K.
 * Replaces algos/sparsesam/sam.py:105-164 (tile_stride_matching), as called at
 * sam.py:193-204.
 *   K of row r = s*heads + h, token t, channel c is read at
 *     k[(s*H*W + t)*ld + h*d + c]            (bf16; `k` already points at K)
 *   base_perm : int32[H*W] space-filling order (ssam_zorder output for "z",
 *               ssam_hilbert_order for "hilbert").
 *   Outputs (int32, [rows, H*W]): perm (interleave or naive layout), inv_perm,
 *   inv_perm_group. Group scores are computed in fp64; ties in the descending
 *   group ranking are broken by lowest group index.
 * ------------------------------------------------------------------------- */
int ssam_stripe_sort_perm(const void* k, int64_t ld, int n_seq, int heads, int H, int W, int d,
                          int group_size, int layout, int ranking, const int32_t* base_perm,
                          int32_t* perm, int32_t* inv_perm, int32_t* inv_perm_group, void* stream);

/* ---------------------------------------------------------------------------
 * a7. A-shape block-mask parameters. Replaces sam.py:219-223.
 * Returns n_init_blocks = int(ratio*ceil(N/n_block)) (+1 when !is_global), or
 * -1 on invalid input.
 * ------------------------------------------------------------------------- */
int ssam_a_shape_n_init(int N, int n_block, double ratio, int is_global);

/* Host-side (num_m x num_n) uint8 block mask equal to the inline predicate of
 * algos/kernels/flash_attn.py:132-145: enabled = n < n_init || (diag && n == m). */
int ssam_a_shape_mask(int N, int m_block, int n_block, int n_init, int with_diag, uint8_t* mask);

/* ---------------------------------------------------------------------------
 * a3+a4+a5+a6+a8. Stripe-Sort block-sparse attention with SAM's decomposed
 * relative-position bias, fused with the permutation gathers and the inverse
 * permutation / head merge.
 * Replaces sam.py:32-49 (get_rel_pos), sam.py:62-73 (compute_rel_bias),
 * sam.py:206-209 (q/k/v gathers), the kernel
 * algos/kernels/flash_attn.py:577-874 (call_a_shape / kernel_a_shape) with
 * :877-909 (_pos_modify_scores), and sam.py:231-232 (inverse gather + merge).
 *   qkv : bf16 [n_seq*win*win, 3*heads*d] rows, leading dim ld_qkv (elements);
 *         q | k | v column blocks, each head d contiguous (SAM qkv Linear order).
 *   rel_pos_h / rel_pos_w : bf16 [2*win-1, d] tables (Attention.rel_pos_h/w).
 *   perm  : int32 [n_seq*heads, win*win] permutation of every row.
 *   out   : bf16 [n_seq*win*win, heads*d] in raster token order, leading dim ld_out.
 *   n_init_blocks / n_block / with_diag : A-shape mask over n_block-token blocks
 *               (n_block 64, SparseSAM's choice at sam.py:52-57, or 128; query
 *               and key blocks have the same size, as the reference's
 *               get_compiled_a_shape(D, m_block, n_block, ...) is always called):
 *               query block m attends to key blocks n < n_init_blocks, and to
 *               n == m when with_diag != 0 (flash_attn.py:132-145).
 *   out_rows  : optional int32 [n_seq*N]: the output row of (sequence s,
 *               token t) is out_rows[s*N + t] (< 0: not stored); NULL stores it
 *               at row s*N + t. Windowed blocks pass the ssam_window_rows map,
 *               which fuses window_unpartition (sam.py:256) into the store.
 *   grid_h / grid_w : when both > 0 (windowed grids, win <= 16, without the
 *               diagonal), the n_seq sequences are the window_partition windows
 *               (sam.py:252; (image, window row, window column) order, zero
 *               padding at the bottom and right) of images of a grid_h x grid_w
 *               token grid, and only each window's real tokens are computed as
 *               queries: the padding tokens' outputs are discarded by
 *               window_unpartition (sam.py:256) in any case, and without the
 *               diagonal every query attends to the same key blocks, so the
 *               results of the real tokens are unchanged. Padding tokens remain
 *               keys. 0 / 0: every token is a query. n_seq must then be a
 *               multiple of the windows per image.
 *   pad_row   : optional bf16 [3*heads*d], with grid_h / grid_w given: the qkv
 *               projection of SAM's zero padding (the qkv bias in bf16). The
 *               kernel then reads it for the padding tokens' K and V and never
 *               reads their qkv rows (which need not be written). NULL: the
 *               padding rows of qkv hold those values (ssam_fill_pad_rows).
 *   workspace : ssam_sparse_attn_workspace_size() bytes (0 for windowed grids,
 *               win <= 16; global grids keep the per-query bias there).
 * d must be 64 or 80; n_block other than 64 / 128 returns SSAM_ERR_UNSUPPORTED.
 * ------------------------------------------------------------------------- */
size_t ssam_sparse_attn_workspace_size(int n_seq, int heads, int win, int d);
int ssam_sparse_attn_fwd(const void* qkv, int64_t ld_qkv, int n_seq, int heads, int win, int d,
                         const void* rel_pos_h, const void* rel_pos_w, const int32_t* perm,
                         int n_init_blocks, int n_block, int with_diag, float scale, void* out, int64_t ld_out,
                         const int32_t* out_rows, int grid_h, int grid_w, const void* pad_row, void* workspace,
                         size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * a10 (selection). Keep set of the Residual-Consistency MLP.
 * Replaces sam.py:277-280: avg_rank = mean over heads of inv_perm_group, then
 * topk(keep_n, largest=False). Ordering key is (sum of per-head ranks, token
 * index), i.e. ties go to the lowest token index.
 *   inv_perm_group : int32 [B*heads, N];  idx : int32 [B, keep_n] (token index,
 *   ascending key order);  rows (may be NULL): int32 [B*keep_n] = b*N + idx.
 * ------------------------------------------------------------------------- */
int ssam_keep_select(const int32_t* inv_perm_group, int B, int heads, int N, int keep_n, int32_t* idx,
                     int32_t* rows, void* stream);

/* ---------------------------------------------------------------------------
 * Static keep set of the SAM3 MLP-merge variant. Replaces
 * algos/sparsesam/sam3.py:49-71 (_get_keep_indices), as used by
 * ToMeSAM3Block.forward (sam3.py:96-109).
 * ssam_zstride_keep_n returns keep_n = min(max(1, round(ratio*N)), N) (Python
 * round: ties to even), or -1 when ratio is outside (0, 1].
 * ssam_zstride_keep writes idx[i] (i < keep_n) = the raster index of the token
 * at Morton position rint(f32(i) * f32(N / keep_n)) (clamped to [0, N)) of the
 * H x W grid, and, when rows != NULL, rows[b*keep_n + i] = b*H*W + idx[i] for
 * b < B (the row map ssam_rc_mlp_fwd takes).
 * ------------------------------------------------------------------------- */
int ssam_zstride_keep_n(int N, double ratio);
int ssam_zstride_keep(int H, int W, int keep_n, int B, int32_t* idx, int32_t* rows, void* stream);

/* ---------------------------------------------------------------------------
 * a9 / a10 data movement. Row-gathered LayerNorm:
 *   out[r, :] = bf16(LN(x[src_rows[r], :]) * w + b), or 0 when src_rows[r] < 0.
 * src_rows == NULL means identity. Covers norm1 + window_partition (sam.py:248,
 * 252), norm2 of the kept tokens (sam.py:282-283) and the dense norm2.
 * ------------------------------------------------------------------------- */
int ssam_layernorm_gather(const float* x, int64_t ldx, const int32_t* src_rows, int n_rows, int C,
                          const float* w, const float* b, float eps, void* out, int64_t ld_out, void* stream);

/* Row map of window_partition for a (B, H, W) token grid and window ws:
 * rows[(b*nwh*nww + wy*nww + wx)*ws*ws + ty*ws + tx] = b*H*W + y*W + x, or -1 in
 * the zero padding. The same map unpartitions (proj epilogue skips -1 rows). */
int ssam_window_rows(int B, int H, int W, int ws, int32_t* rows, void* stream);

/* Inverse of ssam_window_rows: win_rows[b*H*W + y*W + x] = the token's row in
 * the window layout. Lets the windowed blocks run LN1 and the qkv GEMM on the
 * B*H*W real tokens only, scattering qkv rows into the window layout. */
int ssam_window_of_raster(int B, int H, int W, int ws, int32_t* win_rows, void* stream);

/* out[i][0..C) = bf16(bias) for every window-layout row i with rows[i] < 0 (the
 * padding of window_partition, sam.py:252: zero tokens after norm1, whose qkv
 * is the Linear's bias). rows is the ssam_window_rows map. */
int ssam_fill_pad_rows(void* out, int64_t ld, const int32_t* rows, int n_rows, int C, const float* bias,
                       void* stream);

/* ---------------------------------------------------------------------------
 * GEMM on the 5th-generation tensor cores (tcgen05 + TMEM, TMA-fed):
 *   acc[r, n] = sum_k A[r, k] * B[n, k]        (A: M x K, B: N x K, bf16, K-major)
 * then the epilogue selected by `epilogue` (SSAM_EPI_*). `bias` may be NULL.
 * out_rows (NULL = identity) maps accumulator row r to output row out_rows[r]
 * for every epilogue; rows < 0 are skipped (window partition of qkv, keep-set
 * scatter of lin2). Output rows may repeat only with SSAM_EPI_ADD_F32.
 * Used for Attention.qkv / Attention.proj (sam.py:182, 233), MLPBlock lin1/lin2
 * (sam.py:283, 286), patch embedding and the neck convolutions.
 * Requirements: lda, ldb multiples of 8; K multiple of 8; N multiple of 32.
 * ------------------------------------------------------------------------- */
int ssam_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K,
                   const float* bias, int epilogue, void* out, int64_t ldo, const int32_t* out_rows,
                   void* stream);

/* ---------------------------------------------------------------------------
 * a10 (compute). Residual-Consistency MLP on a row subset, in place:
 *   x[rows[r]] += lin2(gelu(lin1(LN(x[rows[r]]))))   for r < n_rows
 * rows == NULL means the dense MLP over the first n_rows rows.
 * Replaces sam.py:281-288. Intermediates live in the caller workspace of
 * ssam_rc_mlp_workspace_size(n_rows, C, hidden) bytes.
 * ------------------------------------------------------------------------- */
size_t ssam_rc_mlp_workspace_size(int n_rows, int C, int hidden);
int ssam_rc_mlp_fwd(float* x, int64_t ldx, const int32_t* rows, int n_rows, int C, int hidden,
                    const float* ln_w, const float* ln_b, float eps, const void* w1, const float* b1,
                    const void* w2, const float* b2, void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Encoder stem and neck data movement (host model pieces kept by the patch).
 * ------------------------------------------------------------------------- */
/* Patch-embed im2col: img fp32 NCHW (B, Cin, H, W) -> bf16 [B*(H/p)*(W/p), Cin*p*p]
 * in (cin, ky, kx) column order, matching a Conv2d(Cin, C, p, stride p) weight view. */
int ssam_patch_im2col(const float* img, int B, int Cin, int H, int W, int p, void* out, void* stream);

/* x[b, t, :] = pos[t, :] for every image b (fp32, T tokens x C). */
int ssam_broadcast_rows(const float* pos, int B, int T, int C, float* x, void* stream);

/* 3x3 / pad 1 im2col over a channels-last bf16 grid (B, H, W, C) ->
 * bf16 [B*H*W, 9*C] in (ky, kx, c) column order, i.e. matching a Conv2d weight
 * permuted to (Cout, 3, 3, Cin). */
int ssam_im2col3x3_nhwc(const void* in, int B, int H, int W, int C, void* out, void* stream);

/* out fp32 [M, N] = A . B^T + bias + addend[(r % addend_rows), :] for every row r
 * (addend fp32 [addend_rows, N]; bias may be NULL): the SAM stem's patch
 * embedding with its positional embedding (addend_rows = tokens per image), x
 * written once. Operands as in ssam_gemm_bf16; M >= 256 (SSAM_ERR_UNSUPPORTED
 * below), N a multiple of 32. */
int ssam_gemm_bf16_addend(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K,
                          const float* bias, const float* addend, int addend_rows, float* out, void* stream);

/* 3x3 / pad 1 convolution of a channels-last bf16 grid in (B, H, W, Cin) as an
 * implicit GEMM on the tensor cores (the im2col is never written): out fp32
 * [B*H*W, Cout] = im2col3x3(in) . w^T (+ bias, which may be NULL), w bf16
 * [Cout, 9*Cin] in (ky, kx, cin) column order (a Conv2d weight permuted to
 * (Cout, 3, 3, Cin)); the results equal ssam_im2col3x3_nhwc followed by
 * ssam_gemm_bf16 with SSAM_EPI_F32 bit for bit. Needs Cin a multiple of 64,
 * Cout a multiple of 32, W dividing 128 and H*W a multiple of 128
 * (SSAM_ERR_UNSUPPORTED otherwise). */
int ssam_conv3x3_nhwc(const void* in, int B, int H, int W, int Cin, const void* w, int Cout, const float* bias,
                      void* out, void* stream);

/* Channels-last fp32 (B, H*W, C) -> channels-first fp32 (B, C, H*W). */
int ssam_nhwc_to_nchw(const float* in, int B, int HW, int C, float* out, void* stream);

/* Row LayerNorm of fp32 rows (nn.LayerNorm / the neck's LayerNorm2d over channels-last
 * rows). out_mode 0: fp32 [n_rows, C]; 1: bf16 [n_rows, C]; 2: the bf16 3-term split
 * [hi | lo | hi] of the result, [n_rows, 3*C] (the operand of the neck's 3x3
 * convolution, see ssam_split_bf16x3); other values return SSAM_ERR_INVALID. */
int ssam_layernorm_rows(const float* x, int n_rows, int C, const float* w, const float* b, float eps,
                        void* out, int out_mode, void* stream);

/* LayerNorm over C of channels-last fp32 rows (B, HW, C), stored channels-first
 * fp32 (B, C, HW): the neck's last LayerNorm2d and the NCHW features in one pass
 * (same arithmetic as ssam_layernorm_rows). C <= 256 (SSAM_ERR_UNSUPPORTED above). */
int ssam_layernorm_nchw(const float* x, int B, int HW, int C, const float* w, const float* b, float eps,
                        float* out, void* stream);

/* Channel LayerNorm (biased variance, eps) of half-precision channels-last rows
 * [rows, C], with an exact GELU after it when gelu = 1: the SAM-HQ mask decoder's
 * LayerNorm2d -> GELU pairs on its NHWC maps (replaces the torch LayerNorm2d and
 * nn.GELU that SAM-HQ's MaskDecoderHQ applies after its transposed convolutions,
 * called from tasks/sam_hq44k/eval_hq44k.py:87-129 through predict_torch).
 * dtype 0: fp16, 1: bf16 (x, w, b and out alike). C in {32, 64, 128, 256}
 * (SSAM_ERR_UNSUPPORTED otherwise); x, w, b, out 16-byte aligned and out not overlapping x. */
int ssam_layernorm_gelu_half(const void* x, int64_t rows, int C, const void* w, const void* b, float eps, int gelu,
                             int dtype, void* out, void* stream);

/* Row LayerNorm fp32 -> bf16 that also stores its input rows unchanged to
 * copy (fp32 [n_rows, C], 16-byte aligned). The encoder keeps its intermediate
 * embedding after a global-attention block (the token grid the SAM-HQ encoder
 * returns beside the features) this way: the next block's norm1 reads the
 * residual stream anyway, so the snapshot costs its writes only. */
int ssam_layernorm_rows_copy(const float* x, int n_rows, int C, const float* w, const float* b, float eps,
                             void* out_bf16, float* copy, void* stream);

/* ---------------------------------------------------------------------------
 * ssam_rc_mlp_fwd for callers that cannot allocate device memory at call time
 * (a host with a fixed, pre-reserved device memory budget, or a foreign-language
 * binding without a device allocator). Same arguments and result as
 * ssam_rc_mlp_fwd, minus the workspace: the intermediates live in a 32 MiB
 * scratch array inside the library that every device loading the library keeps
 * until process exit. No counterpart in the reference (its MLP path allocates
 * through PyTorch).
 *   - Returns SSAM_ERR_UNSUPPORTED when ssam_rc_mlp_workspace_size(n_rows, C,
 *     hidden) exceeds 32 MiB (about 2,600 rows at C = 1280, hidden = 5120).
 *   - The first call on a device resolves the scratch address for that device;
 *     make it before any CUDA stream capture starts. After cudaDeviceReset the
 *     device's next call resolves it again (the address is cached per context).
 *   - `stream` must belong to the current device (the scratch address is that
 *     device's); a stream of another device returns SSAM_ERR_INVALID.
 *   - All calls share the one scratch array: calls that may overlap on the GPU
 *     (different streams, or several host threads) race on it; serialise them.
 *   - Allocates nothing (no cudaMalloc / cudaFree, no library allocator).
 * ------------------------------------------------------------------------- */
int ssam_rc_mlp_fwd_noalloc(float* x, int64_t ldx, const int32_t* rows, int n_rows, int C, int hidden,
                            const float* ln_w, const float* ln_b, float eps, const void* w1, const float* b1,
                            const void* w2, const float* b2, void* stream);

/* hi/lo split of fp32 rows into bf16: out[r] = [bf16(x[r]) | bf16(x[r] - bf16(x[r]))]
 * (2*C columns). A GEMM of the split rows against [W | W] carries the fp32
 * activation into the tensor-core GEMM (used for the neck convolutions). */
int ssam_split_bf16x2(const float* x, int n_rows, int C, void* out, void* stream);

/* 3-term split of fp32 rows: out[r] = [hi | lo | hi] (3*C bf16 columns),
 * hi = bf16(x), lo = bf16(x - hi). A GEMM of the split rows against
 * [W_hi | W_hi | W_lo] (W_lo = bf16(W - W_hi)) carries both the fp32 activation
 * and the fp32 weight into the tensor-core GEMM up to the lo*lo term (about
 * 2^-16 relative); the neck convolutions use it. */
int ssam_split_bf16x3(const float* x, int n_rows, int C, void* out, void* stream);

/* Patch-embed im2col with the same 3-term split: rows of 3*Cin*p*p bf16 columns,
 * [hi | lo | hi], each part in (cin, ky, kx) order; against [W_hi | W_hi | W_lo]
 * the stem GEMM keeps fp32 accuracy. */
int ssam_patch_im2col_split3(const float* img, int B, int Cin, int H, int W, int p, void* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPARSESAM_B200_H_ */
