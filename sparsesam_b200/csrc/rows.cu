// Row-wise data movement around the GEMMs: gathered LayerNorm (norm1 +
// window_partition, norm2 of the keep set), window row maps, the stem im2col,
// the neck im2col / LayerNorm2d / NCHW transpose, and the Residual-Consistency
// MLP composite. These kernels are HBM-bound: vectorised 16-byte accesses,
// one warp per row, no shared-memory staging needed.
#include "common.cuh"
#include "host_util.h"

namespace ssam {

// ---------------------------------------------------------------------------
// LayerNorm over rows, optionally gathered through src_rows (-1 -> zero row).
// One warp per output row; the row lives in registers as float4 chunks.
// Matches torch.nn.LayerNorm: biased variance, (x - mean) * rsqrt(var + eps).
// COPY: the input row is also stored unchanged to copy[r] (fp32, C wide).
// OUT: 0 fp32, 1 bf16, 2 the bf16 3-term split [hi | lo | hi] (3C columns; the
// neck's 3x3 convolution operand, hi = bf16(y), lo = bf16(y - hi)).
// ---------------------------------------------------------------------------
enum { kLnF32 = 0, kLnBf16 = 1, kLnSplit3 = 2 };

// Mean and 1/std of one row held as float4 chunks (lane + 32 i) by a warp; the
// one reduction order every LayerNorm kernel here uses.
template <int CHUNKS>
__device__ __forceinline__ void ln_row_stats(const float4 (&v)[CHUNKS], int nc4, int C, float eps, float& mean,
                                             float& rstd) {
  const int lane = threadIdx.x & 31;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < CHUNKS; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  mean = s / C;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < CHUNKS; ++i) {
    const int c = lane + 32 * i;
    if (c < nc4) {
      const float a0 = v[i].x - mean, a1 = v[i].y - mean, a2 = v[i].z - mean, a3 = v[i].w - mean;
      q += (a0 * a0 + a1 * a1) + (a2 * a2 + a3 * a3);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  rstd = rsqrtf(q / C + eps);
}

template <int CHUNKS, int OUT, bool COPY = false>
__global__ void layernorm_rows_kernel(const float* __restrict__ x, int64_t ldx, const int32_t* __restrict__ src_rows,
                                      int n_rows, int C, const float* __restrict__ w, const float* __restrict__ b,
                                      float eps, void* __restrict__ out, int64_t ld_out, float* __restrict__ copy) {
  const int warps_per_block = blockDim.x >> 5;
  const int r = blockIdx.x * warps_per_block + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= n_rows) return;
  const int src = src_rows != nullptr ? __ldg(src_rows + r) : r;
  const int nc4 = C >> 2;
  if (src < 0) {
    for (int i = lane; i < (OUT == kLnSplit3 ? 3 * nc4 : nc4); i += 32) {
      if constexpr (OUT != kLnF32) {
        reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(out) + static_cast<int64_t>(r) * ld_out)[i] =
            make_uint2(0u, 0u);
      } else {
        reinterpret_cast<float4*>(static_cast<float*>(out) + static_cast<int64_t>(r) * ld_out)[i] =
            make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    return;
  }
  const float4* xr = reinterpret_cast<const float4*>(x + static_cast<int64_t>(src) * ldx);
  float4 v[CHUNKS];
#pragma unroll
  for (int i = 0; i < CHUNKS; ++i) {
    const int c = lane + 32 * i;
    v[i] = c < nc4 ? __ldg(xr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if constexpr (COPY) {
#pragma unroll
    for (int i = 0; i < CHUNKS; ++i) {
      const int c = lane + 32 * i;
      if (c < nc4) reinterpret_cast<float4*>(copy + static_cast<int64_t>(r) * C)[c] = v[i];
    }
  }
  float mean, rstd;
  ln_row_stats<CHUNKS>(v, nc4, C, eps, mean, rstd);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const float4* b4 = reinterpret_cast<const float4*>(b);
#pragma unroll
  for (int i = 0; i < CHUNKS; ++i) {
    const int c = lane + 32 * i;
    if (c < nc4) {
      const float4 ww = __ldg(w4 + c), bb = __ldg(b4 + c);
      const float y0 = (v[i].x - mean) * rstd * ww.x + bb.x;
      const float y1 = (v[i].y - mean) * rstd * ww.y + bb.y;
      const float y2 = (v[i].z - mean) * rstd * ww.z + bb.z;
      const float y3 = (v[i].w - mean) * rstd * ww.w + bb.w;
      if constexpr (OUT == kLnBf16) {
        reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(out) + static_cast<int64_t>(r) * ld_out)[c] =
            make_uint2(pack_bf16x2(y0, y1), pack_bf16x2(y2, y3));
      } else if constexpr (OUT == kLnSplit3) {
        const float h0 = __bfloat162float(__float2bfloat16_rn(y0)), h1 = __bfloat162float(__float2bfloat16_rn(y1));
        const float h2 = __bfloat162float(__float2bfloat16_rn(y2)), h3 = __bfloat162float(__float2bfloat16_rn(y3));
        uint2* row = reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(out) + static_cast<int64_t>(r) * ld_out);
        const uint2 hi = make_uint2(pack_bf16x2(h0, h1), pack_bf16x2(h2, h3));
        row[c] = hi;
        row[nc4 + c] = make_uint2(pack_bf16x2(y0 - h0, y1 - h1), pack_bf16x2(y2 - h2, y3 - h3));
        row[2 * nc4 + c] = hi;
      } else {
        reinterpret_cast<float4*>(static_cast<float*>(out) + static_cast<int64_t>(r) * ld_out)[c] =
            make_float4(y0, y1, y2, y3);
      }
    }
  }
}

template <int OUT, bool COPY = false>
static int launch_layernorm(const float* x, int64_t ldx, const int32_t* src_rows, int n_rows, int C, const float* w,
                            const float* b, float eps, void* out, int64_t ld_out, cudaStream_t stream,
                            float* copy = nullptr) {
  const int nc4 = C / 4;
  const int chunks = (nc4 + 31) / 32;
  const int wpb = 8;
  const dim3 grid((n_rows + wpb - 1) / wpb), block(32 * wpb);
#define SSAM_LN_CASE(K)                                                                                           \
  case K:                                                                                                         \
    layernorm_rows_kernel<K, OUT, COPY><<<grid, block, 0, stream>>>(x, ldx, src_rows, n_rows, C, w, b, eps, out, \
                                                                   ld_out, copy);                                 \
    break;
  switch (chunks) {
    SSAM_LN_CASE(1)
    SSAM_LN_CASE(2)
    SSAM_LN_CASE(4)
    SSAM_LN_CASE(8)
    SSAM_LN_CASE(16)
    case 3:
      layernorm_rows_kernel<4, OUT, COPY><<<grid, block, 0, stream>>>(x, ldx, src_rows, n_rows, C, w, b, eps, out,
                                                                     ld_out, copy);
      break;
    case 9: case 10:  // ViT-H (C = 1280): exactly 10 float4 per lane
      layernorm_rows_kernel<10, OUT, COPY><<<grid, block, 0, stream>>>(x, ldx, src_rows, n_rows, C, w, b, eps, out,
                                                                      ld_out, copy);
      break;
    case 5: case 6: case 7:
      layernorm_rows_kernel<8, OUT, COPY><<<grid, block, 0, stream>>>(x, ldx, src_rows, n_rows, C, w, b, eps, out,
                                                                     ld_out, copy);
      break;
    default:
      if (chunks > 16) return SSAM_ERR_UNSUPPORTED;
      layernorm_rows_kernel<16, OUT, COPY><<<grid, block, 0, stream>>>(x, ldx, src_rows, n_rows, C, w, b, eps, out,
                                                                      ld_out, copy);
  }
#undef SSAM_LN_CASE
  return status_from_cuda(cudaGetLastError());
}

int layernorm_gather(const float* x, int64_t ldx, const int32_t* src_rows, int n_rows, int C, const float* w,
                     const float* b, float eps, void* out, int64_t ld_out, cudaStream_t stream) {
  if (x == nullptr || w == nullptr || b == nullptr || out == nullptr || n_rows < 0 || C <= 0) return SSAM_ERR_INVALID;
  if (n_rows == 0) return SSAM_OK;
  if (C % 4 || ldx % 4 || ld_out % 4 || ldx < C || ld_out < C) return SSAM_ERR_ALIGN;
  if (!aligned16(x) || !aligned16(w) || !aligned16(b) || (reinterpret_cast<uintptr_t>(out) & 7)) return SSAM_ERR_ALIGN;
  return launch_layernorm<kLnBf16>(x, ldx, src_rows, n_rows, C, w, b, eps, out, ld_out, stream);
}

int layernorm_rows(const float* x, int n_rows, int C, const float* w, const float* b, float eps, void* out,
                   int out_mode, cudaStream_t stream) {
  if (x == nullptr || w == nullptr || b == nullptr || out == nullptr || n_rows < 0 || C <= 0) return SSAM_ERR_INVALID;
  if (out_mode < kLnF32 || out_mode > kLnSplit3) return SSAM_ERR_INVALID;
  if (n_rows == 0) return SSAM_OK;
  if (C % 4 || !aligned16(x) || !aligned16(w) || !aligned16(b) || !aligned16(out)) return SSAM_ERR_ALIGN;
  switch (out_mode) {
    case kLnF32:
      return launch_layernorm<kLnF32>(x, C, nullptr, n_rows, C, w, b, eps, out, C, stream);
    case kLnBf16:
      return launch_layernorm<kLnBf16>(x, C, nullptr, n_rows, C, w, b, eps, out, C, stream);
    default:
      return launch_layernorm<kLnSplit3>(x, C, nullptr, n_rows, C, w, b, eps, out, 3 * static_cast<int64_t>(C),
                                         stream);
  }
}

// LayerNorm of channels-last fp32 rows (B, HW, C), stored channels-first fp32
// (B, C, HW): the neck's last LayerNorm2d and the features' NCHW layout in one
// pass. A CTA normalises 32 consecutive pixels of one image (a warp per row, the
// reduction order of layernorm_rows) into a [C][32] shared-memory tile and writes
// it out as 128-byte channel rows.
constexpr int kLnNchwMaxC = 256;
__global__ void __launch_bounds__(256) layernorm_nchw_kernel(const float* __restrict__ x, int HW, int C,
                                                             const float* __restrict__ w, const float* __restrict__ b,
                                                             float eps, float* __restrict__ out) {
  __shared__ float tile[kLnNchwMaxC][33];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bimg = blockIdx.y, p0 = blockIdx.x * 32;
  const int nc4 = C >> 2;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const float4* b4 = reinterpret_cast<const float4*>(b);
  for (int j = warp; j < 32; j += 8) {
    const int p = p0 + j;
    if (p >= HW) break;
    const float4* xr = reinterpret_cast<const float4*>(x + (static_cast<int64_t>(bimg) * HW + p) * C);
    float4 v[kLnNchwMaxC / 128];
#pragma unroll
    for (int i = 0; i < kLnNchwMaxC / 128; ++i) {
      const int c = lane + 32 * i;
      v[i] = c < nc4 ? __ldg(xr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float mean, rstd;
    ln_row_stats<kLnNchwMaxC / 128>(v, nc4, C, eps, mean, rstd);
#pragma unroll
    for (int i = 0; i < kLnNchwMaxC / 128; ++i) {
      const int c = lane + 32 * i;
      if (c < nc4) {
        const float4 ww = __ldg(w4 + c), bb = __ldg(b4 + c);
        tile[4 * c][j] = (v[i].x - mean) * rstd * ww.x + bb.x;
        tile[4 * c + 1][j] = (v[i].y - mean) * rstd * ww.y + bb.y;
        tile[4 * c + 2][j] = (v[i].z - mean) * rstd * ww.z + bb.z;
        tile[4 * c + 3][j] = (v[i].w - mean) * rstd * ww.w + bb.w;
      }
    }
  }
  __syncthreads();
  const int p = p0 + lane;
  for (int c = warp; c < C; c += 8)
    if (p < HW) out[(static_cast<int64_t>(bimg) * C + c) * HW + p] = tile[c][lane];
}

int layernorm_nchw(const float* x, int B, int HW, int C, const float* w, const float* b, float eps, float* out,
                   cudaStream_t stream) {
  if (x == nullptr || w == nullptr || b == nullptr || out == nullptr || B <= 0 || HW <= 0 || C <= 0)
    return SSAM_ERR_INVALID;
  if (C > kLnNchwMaxC || B > 65535) return SSAM_ERR_UNSUPPORTED;
  if (C % 4 || !aligned16(x) || !aligned16(w) || !aligned16(b)) return SSAM_ERR_ALIGN;
  layernorm_nchw_kernel<<<dim3((HW + 31) / 32, B), 256, 0, stream>>>(x, HW, C, w, b, eps, out);
  return status_from_cuda(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// Channel LayerNorm (eps, biased variance) with an optional exact GELU after it,
// on half-precision channels-last rows (fp16 or bf16 in, weights and out): the
// SAM-HQ mask decoder's LayerNorm2d -> GELU pairs on its NHWC maps of 32 .. 256
// channels (millions of short rows, where a row per warp would leave most lanes
// idle). C / 8 threads per row, one 16-byte vector of 8 channels each; the row's
// sums are shuffle reductions inside its lane group, the mean first, then the
// mean of squared deviations from the registers. A grid-stride loop over row
// groups keeps every lane of a warp in the loop (rows past the end load zeros
// and store nothing), so the full-mask shuffles are always well defined.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void unpack8(uint4 r, float (&v)[8], const __half*) {
  const __half2* h = reinterpret_cast<const __half2*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void unpack8(uint4 r, float (&v)[8], const __nv_bfloat16*) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ uint4 pack8(const float (&v)[8], const __half*) {
  uint4 r;
  __half2* h = reinterpret_cast<__half2*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  return r;
}
__device__ __forceinline__ uint4 pack8(const float (&v)[8], const __nv_bfloat16*) {
  uint4 r;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  return r;
}

constexpr int kLnHalfThreads = 256;
template <typename T, int C, bool GELU>
__global__ void __launch_bounds__(kLnHalfThreads) layernorm_half_kernel(const T* __restrict__ x, int64_t rows,
                                                                         const T* __restrict__ w,
                                                                         const T* __restrict__ b, float eps,
                                                                         T* __restrict__ out) {
  constexpr int kTpr = C / 8;                    // threads per row
  constexpr int kRows = kLnHalfThreads / kTpr;   // rows per CTA per step
  const int sub = threadIdx.x % kTpr;
  float wv[8], bv[8];
  unpack8(__ldg(reinterpret_cast<const uint4*>(w) + sub), wv, w);
  unpack8(__ldg(reinterpret_cast<const uint4*>(b) + sub), bv, b);
  for (int64_t r0 = static_cast<int64_t>(blockIdx.x) * kRows; r0 < rows;
       r0 += static_cast<int64_t>(gridDim.x) * kRows) {
    const int64_t row = r0 + threadIdx.x / kTpr;
    const bool valid = row < rows;
    float v[8];
    const uint4 raw = valid ? __ldg(reinterpret_cast<const uint4*>(x + row * C) + sub) : make_uint4(0, 0, 0, 0);
    unpack8(raw, v, x);
    float s = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
#pragma unroll
    for (int o = kTpr / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / C;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[i] -= mean;
      q = fmaf(v[i], v[i], q);
    }
#pragma unroll
    for (int o = kTpr / 2; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float rstd = rsqrtf(q / C + eps);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float y = fmaf(v[i] * rstd, wv[i], bv[i]);
      v[i] = GELU ? gelu_exact(y) : y;
    }
    if (valid) reinterpret_cast<uint4*>(out + row * C)[sub] = pack8(v, out);
  }
}

template <typename T, int C>
static int launch_layernorm_half(const void* x, int64_t rows, const void* w, const void* b, float eps, int gelu,
                                 void* out, cudaStream_t stream) {
  constexpr int kRows = kLnHalfThreads / (C / 8);
  const int dev = current_device();
  const int64_t want = (rows + kRows - 1) / kRows;
  const int64_t cap = static_cast<int64_t>(dev >= 0 ? num_sms(dev) : 148) * 8;  // 8 resident CTAs per SM
  const int grid = static_cast<int>(want < cap ? want : cap);
  const T* xp = static_cast<const T*>(x);
  const T* wp = static_cast<const T*>(w);
  const T* bp = static_cast<const T*>(b);
  T* op = static_cast<T*>(out);
  if (gelu)
    layernorm_half_kernel<T, C, true><<<grid, kLnHalfThreads, 0, stream>>>(xp, rows, wp, bp, eps, op);
  else
    layernorm_half_kernel<T, C, false><<<grid, kLnHalfThreads, 0, stream>>>(xp, rows, wp, bp, eps, op);
  return status_from_cuda(cudaGetLastError());
}

template <typename T>
static int dispatch_layernorm_half(const void* x, int64_t rows, int C, const void* w, const void* b, float eps,
                                   int gelu, void* out, cudaStream_t stream) {
  switch (C) {
    case 32: return launch_layernorm_half<T, 32>(x, rows, w, b, eps, gelu, out, stream);
    case 64: return launch_layernorm_half<T, 64>(x, rows, w, b, eps, gelu, out, stream);
    case 128: return launch_layernorm_half<T, 128>(x, rows, w, b, eps, gelu, out, stream);
    case 256: return launch_layernorm_half<T, 256>(x, rows, w, b, eps, gelu, out, stream);
    default: return SSAM_ERR_UNSUPPORTED;
  }
}

int layernorm_half(const void* x, int64_t rows, int C, const void* w, const void* b, float eps, int gelu, int dtype,
                   void* out, cudaStream_t stream) {
  if (x == nullptr || w == nullptr || b == nullptr || out == nullptr || rows < 0 || C <= 0) return SSAM_ERR_INVALID;
  if ((dtype != 0 && dtype != 1) || (gelu != 0 && gelu != 1)) return SSAM_ERR_INVALID;
  if (C != 32 && C != 64 && C != 128 && C != 256) return SSAM_ERR_UNSUPPORTED;
  if (!aligned16(x) || !aligned16(w) || !aligned16(b) || !aligned16(out)) return SSAM_ERR_ALIGN;
  if (rows == 0) return SSAM_OK;
  return dtype == 0 ? dispatch_layernorm_half<__half>(x, rows, C, w, b, eps, gelu, out, stream)
                    : dispatch_layernorm_half<__nv_bfloat16>(x, rows, C, w, b, eps, gelu, out, stream);
}

int layernorm_rows_copy(const float* x, int n_rows, int C, const float* w, const float* b, float eps, void* out,
                        float* copy, cudaStream_t stream) {
  if (x == nullptr || w == nullptr || b == nullptr || out == nullptr || copy == nullptr || n_rows < 0 || C <= 0)
    return SSAM_ERR_INVALID;
  if (n_rows == 0) return SSAM_OK;
  if (C % 4 || !aligned16(x) || !aligned16(w) || !aligned16(b) || !aligned16(out) || !aligned16(copy))
    return SSAM_ERR_ALIGN;
  return launch_layernorm<kLnBf16, true>(x, C, nullptr, n_rows, C, w, b, eps, out, C, stream, copy);
}

// ---------------------------------------------------------------------------
// window_partition row map (host image_encoder window_partition, used at
// algos/sparsesam/sam.py:252 and :256).
// ---------------------------------------------------------------------------
__global__ void window_rows_kernel(int B, int H, int W, int ws, int nwh, int nww, int32_t* rows) {
  const int64_t total = static_cast<int64_t>(B) * nwh * nww * ws * ws;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int t = static_cast<int>(i % (ws * ws));
  const int64_t win = i / (ws * ws);
  const int wx = static_cast<int>(win % nww);
  const int wy = static_cast<int>((win / nww) % nwh);
  const int b = static_cast<int>(win / (static_cast<int64_t>(nww) * nwh));
  const int y = wy * ws + t / ws, x = wx * ws + t % ws;
  rows[i] = (y < H && x < W) ? b * H * W + y * W + x : -1;
}

int window_rows(int B, int H, int W, int ws, int32_t* rows, cudaStream_t stream) {
  if (B <= 0 || H <= 0 || W <= 0 || ws <= 0 || rows == nullptr) return SSAM_ERR_INVALID;
  const int nwh = (H + ws - 1) / ws, nww = (W + ws - 1) / ws;
  const int64_t total = static_cast<int64_t>(B) * nwh * nww * ws * ws;
  if (total > INT32_MAX) return SSAM_ERR_UNSUPPORTED;
  window_rows_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(B, H, W, ws, nwh, nww, rows);
  return status_from_cuda(cudaGetLastError());
}

// Inverse map: raster row (b, y, x) -> its row in the window layout.
__global__ void window_of_raster_kernel(int B, int H, int W, int ws, int nwh, int nww, int32_t* win_rows) {
  const int64_t total = static_cast<int64_t>(B) * H * W;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int x = static_cast<int>(i % W);
  const int y = static_cast<int>((i / W) % H);
  const int b = static_cast<int>(i / (static_cast<int64_t>(W) * H));
  const int64_t win = (static_cast<int64_t>(b) * nwh + y / ws) * nww + x / ws;
  win_rows[i] = static_cast<int32_t>(win * ws * ws + (y % ws) * ws + (x % ws));
}

int window_of_raster(int B, int H, int W, int ws, int32_t* win_rows, cudaStream_t stream) {
  if (B <= 0 || H <= 0 || W <= 0 || ws <= 0 || win_rows == nullptr) return SSAM_ERR_INVALID;
  const int nwh = (H + ws - 1) / ws, nww = (W + ws - 1) / ws;
  if (static_cast<int64_t>(B) * nwh * nww * ws * ws > INT32_MAX) return SSAM_ERR_UNSUPPORTED;
  const int64_t total = static_cast<int64_t>(B) * H * W;
  window_of_raster_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(B, H, W, ws, nwh, nww,
                                                                                         win_rows);
  return status_from_cuda(cudaGetLastError());
}

// Rows of the window layout that lie in the padding (rows[i] < 0) are set to
// bf16(bias): SAM pads the normalised tokens with zeros, so their qkv is the
// Linear's bias. One warp per row, 16 bytes per lane.
__global__ void fill_pad_rows_kernel(__nv_bfloat16* __restrict__ out, int64_t ld, const int32_t* __restrict__ rows,
                                     int n_rows, int C, const float* __restrict__ bias) {
  const int64_t wi = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wi >= n_rows || __ldg(rows + wi) >= 0) return;
  uint4* dst = reinterpret_cast<uint4*>(out + wi * ld);
  for (int c = lane * 8; c < C; c += 32 * 8) {
    const float4 b0 = __ldg(reinterpret_cast<const float4*>(bias + c));
    const float4 b1 = __ldg(reinterpret_cast<const float4*>(bias + c + 4));
    dst[c / 8] = make_uint4(pack_bf16x2(b0.x, b0.y), pack_bf16x2(b0.z, b0.w), pack_bf16x2(b1.x, b1.y),
                            pack_bf16x2(b1.z, b1.w));
  }
}

int fill_pad_rows(void* out, int64_t ld, const int32_t* rows, int n_rows, int C, const float* bias,
                  cudaStream_t stream) {
  if (out == nullptr || rows == nullptr || bias == nullptr || n_rows < 0 || C <= 0) return SSAM_ERR_INVALID;
  if (n_rows == 0) return SSAM_OK;
  if (C % 8 || ld % 8 || !aligned16(out) || !aligned16(bias)) return SSAM_ERR_ALIGN;
  const int64_t threads = static_cast<int64_t>(n_rows) * 32;
  fill_pad_rows_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, stream>>>(
      static_cast<__nv_bfloat16*>(out), ld, rows, n_rows, C, bias);
  return status_from_cuda(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// Stem / neck helpers.
// ---------------------------------------------------------------------------
// One thread per (output row, cin, ky): copies p contiguous pixels.
__global__ void patch_im2col_kernel(const float* __restrict__ img, int B, int Cin, int H, int W, int p,
                                    __nv_bfloat16* __restrict__ out) {
  const int gh = H / p, gw = W / p;
  const int64_t total = static_cast<int64_t>(B) * gh * gw * Cin * p;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int ky = static_cast<int>(i % p);
  const int cin = static_cast<int>((i / p) % Cin);
  const int64_t tok = i / (static_cast<int64_t>(p) * Cin);
  const int px = static_cast<int>(tok % gw), py = static_cast<int>((tok / gw) % gh);
  const int b = static_cast<int>(tok / (static_cast<int64_t>(gw) * gh));
  const float* src = img + ((static_cast<int64_t>(b) * Cin + cin) * H + (py * p + ky)) * W + px * p;
  __nv_bfloat16* dst = out + tok * (static_cast<int64_t>(Cin) * p * p) + (cin * p + ky) * p;
  for (int kx = 0; kx < p; kx += 2) {
    const float2 v = *reinterpret_cast<const float2*>(src + kx);
    *reinterpret_cast<uint32_t*>(dst + kx) = pack_bf16x2(v.x, v.y);
  }
}

int patch_im2col(const float* img, int B, int Cin, int H, int W, int p, void* out, cudaStream_t stream) {
  if (img == nullptr || out == nullptr || B <= 0 || Cin <= 0 || p <= 0 || H % p || W % p) return SSAM_ERR_INVALID;
  if (p % 2 || (reinterpret_cast<uintptr_t>(img) & 7) || (reinterpret_cast<uintptr_t>(out) & 3)) return SSAM_ERR_ALIGN;
  const int64_t total = static_cast<int64_t>(B) * (H / p) * (W / p) * Cin * p;
  patch_im2col_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(
      img, B, Cin, H, W, p, static_cast<__nv_bfloat16*>(out));
  return status_from_cuda(cudaGetLastError());
}

// Patch-embed im2col with the 3-term split of every pixel: a row holds
// [hi | lo | hi] (3 Cin p p columns, each part in (cin, ky, kx) order) with
// hi = bf16(x) and lo = bf16(x - hi); against [W_hi | W_hi | W_lo] the GEMM sums
// x_hi W_hi + x_lo W_hi + x_hi W_lo, i.e. the fp32 product up to the lo*lo term.
__global__ void patch_im2col_split3_kernel(const float* __restrict__ img, int B, int Cin, int H, int W, int p,
                                           __nv_bfloat16* __restrict__ out) {
  const int gh = H / p, gw = W / p;
  const int64_t total = static_cast<int64_t>(B) * gh * gw * Cin * p;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int ky = static_cast<int>(i % p);
  const int cin = static_cast<int>((i / p) % Cin);
  const int64_t tok = i / (static_cast<int64_t>(p) * Cin);
  const int px = static_cast<int>(tok % gw), py = static_cast<int>((tok / gw) % gh);
  const int b = static_cast<int>(tok / (static_cast<int64_t>(gw) * gh));
  const int K = Cin * p * p;
  const float* src = img + ((static_cast<int64_t>(b) * Cin + cin) * H + (py * p + ky)) * W + px * p;
  __nv_bfloat16* dst = out + tok * (3 * static_cast<int64_t>(K)) + (cin * p + ky) * p;
  for (int kx = 0; kx < p; kx += 2) {
    const float2 v = *reinterpret_cast<const float2*>(src + kx);
    const float h0 = __bfloat162float(__float2bfloat16_rn(v.x)), h1 = __bfloat162float(__float2bfloat16_rn(v.y));
    const uint32_t hi = pack_bf16x2(h0, h1);
    *reinterpret_cast<uint32_t*>(dst + kx) = hi;
    *reinterpret_cast<uint32_t*>(dst + K + kx) = pack_bf16x2(v.x - h0, v.y - h1);
    *reinterpret_cast<uint32_t*>(dst + 2 * K + kx) = hi;
  }
}

// Same output, one block per patch (grid px, py, b) and one thread per 8-pixel
// run of a patch row: two float4 loads, three 16-byte stores (p % 8 == 0).
__global__ void patch_im2col_split3_v8_kernel(const float* __restrict__ img, int Cin, int H, int W, int p,
                                              __nv_bfloat16* __restrict__ out) {
  const int px = blockIdx.x, py = blockIdx.y, b = blockIdx.z;
  const int gw = W / p, gh = H / p;
  const int runs = p / 8;
  const int K = Cin * p * p;
  const int64_t tok = (static_cast<int64_t>(b) * gh + py) * gw + px;
  for (int u = threadIdx.x; u < Cin * p * runs; u += blockDim.x) {
    const int run = u % runs, ky = (u / runs) % p, cin = u / (runs * p);
    const float4* src = reinterpret_cast<const float4*>(
        img + ((static_cast<int64_t>(b) * Cin + cin) * H + (py * p + ky)) * W + px * p + run * 8);
    const float4 v0 = __ldg(src), v1 = __ldg(src + 1);
    const float f[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    float h[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) h[e] = __bfloat162float(__float2bfloat16_rn(f[e]));
    const uint4 hi = make_uint4(pack_bf16x2(h[0], h[1]), pack_bf16x2(h[2], h[3]), pack_bf16x2(h[4], h[5]),
                                pack_bf16x2(h[6], h[7]));
    const uint4 lo = make_uint4(pack_bf16x2(f[0] - h[0], f[1] - h[1]), pack_bf16x2(f[2] - h[2], f[3] - h[3]),
                                pack_bf16x2(f[4] - h[4], f[5] - h[5]), pack_bf16x2(f[6] - h[6], f[7] - h[7]));
    __nv_bfloat16* dst = out + tok * (3 * static_cast<int64_t>(K)) + (cin * p + ky) * p + run * 8;
    *reinterpret_cast<uint4*>(dst) = hi;
    *reinterpret_cast<uint4*>(dst + K) = lo;
    *reinterpret_cast<uint4*>(dst + 2 * K) = hi;
  }
}

int patch_im2col_split3(const float* img, int B, int Cin, int H, int W, int p, void* out, cudaStream_t stream) {
  if (img == nullptr || out == nullptr || B <= 0 || Cin <= 0 || p <= 0 || H % p || W % p) return SSAM_ERR_INVALID;
  if (p % 2 || (reinterpret_cast<uintptr_t>(img) & 7) || (reinterpret_cast<uintptr_t>(out) & 3)) return SSAM_ERR_ALIGN;
  if (p % 8 == 0 && W % 4 == 0 && aligned16(img) && aligned16(out) && H / p <= 65535 && B <= 65535) {
    const int work = Cin * p * (p / 8);
    const int threads = work >= 128 ? 128 : ((work + 31) / 32) * 32;
    patch_im2col_split3_v8_kernel<<<dim3(W / p, H / p, B), threads, 0, stream>>>(img, Cin, H, W, p,
                                                                                 static_cast<__nv_bfloat16*>(out));
    return status_from_cuda(cudaGetLastError());
  }
  const int64_t total = static_cast<int64_t>(B) * (H / p) * (W / p) * Cin * p;
  patch_im2col_split3_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(
      img, B, Cin, H, W, p, static_cast<__nv_bfloat16*>(out));
  return status_from_cuda(cudaGetLastError());
}

__global__ void broadcast_rows_kernel(const float4* __restrict__ pos, int64_t per_image4, int64_t total4,
                                      float4* __restrict__ x) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < total4) x[i] = __ldg(pos + i % per_image4);
}

int broadcast_rows(const float* pos, int B, int T, int C, float* x, cudaStream_t stream) {
  if (pos == nullptr || x == nullptr || B <= 0 || T <= 0 || C <= 0) return SSAM_ERR_INVALID;
  if (C % 4 || !aligned16(pos) || !aligned16(x)) return SSAM_ERR_ALIGN;
  const int64_t per = static_cast<int64_t>(T) * C / 4, total = per * B;
  broadcast_rows_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<const float4*>(pos), per, total, reinterpret_cast<float4*>(x));
  return status_from_cuda(cudaGetLastError());
}

// 3x3 / pad 1 im2col, channels-last, (ky, kx, c) column order. One block per
// output pixel (grid x, y, b: no index division), 8 channels per thread and tap.
__global__ void im2col3x3_kernel(const __nv_bfloat16* __restrict__ in, int H, int W, int C,
                                 __nv_bfloat16* __restrict__ out) {
  const int x = blockIdx.x, y = blockIdx.y, b = blockIdx.z;
  const int c8 = C / 8;
  const int64_t pix = (static_cast<int64_t>(b) * H + y) * W + x;
  uint4* dst = reinterpret_cast<uint4*>(out + pix * (9 * static_cast<int64_t>(C)));
#pragma unroll
  for (int tap = 0; tap < 9; ++tap) {
    const int yy = y + tap / 3 - 1, xx = x + tap % 3 - 1;
    const bool inside = yy >= 0 && yy < H && xx >= 0 && xx < W;
    const uint4* src =
        inside ? reinterpret_cast<const uint4*>(in + ((static_cast<int64_t>(b) * H + yy) * W + xx) * C) : nullptr;
    for (int cc = threadIdx.x; cc < c8; cc += blockDim.x)
      dst[tap * c8 + cc] = inside ? __ldg(src + cc) : make_uint4(0u, 0u, 0u, 0u);
  }
}

int im2col3x3_nhwc(const void* in, int B, int H, int W, int C, void* out, cudaStream_t stream) {
  if (in == nullptr || out == nullptr || B <= 0 || H <= 0 || W <= 0 || C <= 0) return SSAM_ERR_INVALID;
  if (H > 65535 || B > 65535) return SSAM_ERR_UNSUPPORTED;
  if (C % 8 || !aligned16(in) || !aligned16(out)) return SSAM_ERR_ALIGN;
  const int threads = C / 8 >= 128 ? 128 : ((C / 8 + 31) / 32) * 32;
  im2col3x3_kernel<<<dim3(W, H, B), threads, 0, stream>>>(static_cast<const __nv_bfloat16*>(in), H, W, C,
                                                           static_cast<__nv_bfloat16*>(out));
  return status_from_cuda(cudaGetLastError());
}

// (B, HW, C) -> (B, C, HW), 32x32 tiles through shared memory.
__global__ void nhwc_to_nchw_kernel(const float* __restrict__ in, int HW, int C, float* __restrict__ out) {
  __shared__ float tile[32][33];
  const int b = blockIdx.z;
  const int p0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  const float* src = in + static_cast<int64_t>(b) * HW * C;
  float* dst = out + static_cast<int64_t>(b) * HW * C;
  for (int j = threadIdx.y; j < 32; j += blockDim.y) {
    const int p = p0 + j, c = c0 + threadIdx.x;
    if (p < HW && c < C) tile[j][threadIdx.x] = src[static_cast<int64_t>(p) * C + c];
  }
  __syncthreads();
  for (int j = threadIdx.y; j < 32; j += blockDim.y) {
    const int c = c0 + j, p = p0 + threadIdx.x;
    if (p < HW && c < C) dst[static_cast<int64_t>(c) * HW + p] = tile[threadIdx.x][j];
  }
}

int nhwc_to_nchw(const float* in, int B, int HW, int C, float* out, cudaStream_t stream) {
  if (in == nullptr || out == nullptr || B <= 0 || HW <= 0 || C <= 0) return SSAM_ERR_INVALID;
  const dim3 grid((HW + 31) / 32, (C + 31) / 32, B), block(32, 8);
  nhwc_to_nchw_kernel<<<grid, block, 0, stream>>>(in, HW, C, out);
  return status_from_cuda(cudaGetLastError());
}

// hi/lo bf16 split of fp32 rows: out[r] = [bf16(x) | bf16(x - bf16(x))] (2C columns).
// A GEMM over the split operand against a duplicated weight [W | W] reproduces the
// fp32 activation to ~2^-16 relative (used by the neck, right before LayerNorm2d).
__global__ void split_bf16x2_kernel(const float4* __restrict__ x, int64_t n4, int c4, uint2* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n4) return;
  const int64_t r = i / c4;
  const int c = static_cast<int>(i - r * c4);
  const float4 v = __ldg(x + i);
  const __nv_bfloat16 h0 = __float2bfloat16_rn(v.x), h1 = __float2bfloat16_rn(v.y);
  const __nv_bfloat16 h2 = __float2bfloat16_rn(v.z), h3 = __float2bfloat16_rn(v.w);
  uint2* row = out + r * 2 * c4;
  row[c] = make_uint2(pack_bf16x2(__bfloat162float(h0), __bfloat162float(h1)),
                      pack_bf16x2(__bfloat162float(h2), __bfloat162float(h3)));
  row[c4 + c] = make_uint2(pack_bf16x2(v.x - __bfloat162float(h0), v.y - __bfloat162float(h1)),
                           pack_bf16x2(v.z - __bfloat162float(h2), v.w - __bfloat162float(h3)));
}

int split_bf16x2(const float* x, int n_rows, int C, void* out, cudaStream_t stream) {
  if (x == nullptr || out == nullptr || n_rows < 0 || C <= 0) return SSAM_ERR_INVALID;
  if (n_rows == 0) return SSAM_OK;
  if (C % 4 || !aligned16(x) || (reinterpret_cast<uintptr_t>(out) & 7)) return SSAM_ERR_ALIGN;
  const int64_t n4 = static_cast<int64_t>(n_rows) * (C / 4);
  split_bf16x2_kernel<<<static_cast<unsigned>((n4 + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<const float4*>(x), n4, C / 4, static_cast<uint2*>(out));
  return status_from_cuda(cudaGetLastError());
}

// 3-term split of fp32 rows: out[r] = [hi | lo | hi] (3 C columns), hi = bf16(x),
// lo = bf16(x - hi); against [W_hi | W_hi | W_lo] a GEMM carries both the fp32
// activation and the fp32 weight up to the lo*lo term.
// One block per row (no index division).
__global__ void split_bf16x3_kernel(const float4* __restrict__ x, int c4, uint2* __restrict__ out) {
  const int64_t r = blockIdx.x;
  uint2* row = out + r * 3 * c4;
  for (int c = threadIdx.x; c < c4; c += blockDim.x) {
    const float4 v = __ldg(x + r * c4 + c);
    const float h0 = __bfloat162float(__float2bfloat16_rn(v.x)), h1 = __bfloat162float(__float2bfloat16_rn(v.y));
    const float h2 = __bfloat162float(__float2bfloat16_rn(v.z)), h3 = __bfloat162float(__float2bfloat16_rn(v.w));
    const uint2 hi = make_uint2(pack_bf16x2(h0, h1), pack_bf16x2(h2, h3));
    row[c] = hi;
    row[c4 + c] = make_uint2(pack_bf16x2(v.x - h0, v.y - h1), pack_bf16x2(v.z - h2, v.w - h3));
    row[2 * c4 + c] = hi;
  }
}

int split_bf16x3(const float* x, int n_rows, int C, void* out, cudaStream_t stream) {
  if (x == nullptr || out == nullptr || n_rows < 0 || C <= 0) return SSAM_ERR_INVALID;
  if (n_rows == 0) return SSAM_OK;
  if (C % 4 || !aligned16(x) || (reinterpret_cast<uintptr_t>(out) & 7)) return SSAM_ERR_ALIGN;
  const int c4 = C / 4;
  const int threads = c4 >= 256 ? 256 : ((c4 + 31) / 32) * 32;
  split_bf16x3_kernel<<<n_rows, threads, 0, stream>>>(reinterpret_cast<const float4*>(x), c4,
                                                      static_cast<uint2*>(out));
  return status_from_cuda(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// Residual-Consistency MLP (algos/sparsesam/sam.py:281-288):
//   xk = LN(x[rows]) (bf16) ; h = gelu(xk W1^T + b1) ; x[rows] += h W2^T + b2
// ---------------------------------------------------------------------------
static size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

size_t rc_mlp_workspace_size(int n_rows, int C, int hidden) {
  if (n_rows <= 0 || C <= 0 || hidden <= 0) return 0;
  return align256(static_cast<size_t>(n_rows) * C * 2) + align256(static_cast<size_t>(n_rows) * hidden * 2);
}

int rc_mlp_fwd(float* x, int64_t ldx, const int32_t* rows, int n_rows, int C, int hidden, const float* ln_w,
               const float* ln_b, float eps, const void* w1, const float* b1, const void* w2, const float* b2,
               void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (x == nullptr || ln_w == nullptr || ln_b == nullptr || w1 == nullptr || w2 == nullptr) return SSAM_ERR_INVALID;
  if (n_rows < 0 || C <= 0 || hidden <= 0) return SSAM_ERR_INVALID;
  if (n_rows == 0) return SSAM_OK;
  const size_t need = rc_mlp_workspace_size(n_rows, C, hidden);
  if (workspace == nullptr || workspace_bytes < need) return SSAM_ERR_INVALID;
  if (!aligned16(workspace)) return SSAM_ERR_ALIGN;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* xk = ws;
  void* h = ws + align256(static_cast<size_t>(n_rows) * C * 2);
  int st = layernorm_gather(x, ldx, rows, n_rows, C, ln_w, ln_b, eps, xk, C, stream);
  if (st != SSAM_OK) return st;
  st = gemm_bf16(xk, C, w1, C, n_rows, hidden, C, b1, SSAM_EPI_GELU_BF16, h, hidden, nullptr, stream);
  if (st != SSAM_OK) return st;
  return gemm_bf16(h, hidden, w2, hidden, n_rows, C, hidden, b2, SSAM_EPI_ADD_F32, x, ldx, rows, stream);
}

}  // namespace ssam
