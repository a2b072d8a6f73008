// Stripe-Sort block-sparse attention with SAM's decomposed relative-position
// bias, on the sm_100a tensor cores.
//
// Semantics (algos/kernels/flash_attn.py:577-909 with algos/sparsesam/sam.py:62-73,
// 206-233): for one (sequence, head) row with tokens in permuted order
// p = 0..N-1 (token perm[p]), query block m = p/64 attends to key blocks
// n < n_init (plus n == m when with_diag):
//   logit(p, k) = scale * <q_p, k_k> + relH[p][kh(k)] + relW[p][kw(k)]
//   relH[p][j]  = <q_p, Th[qh(p) - j + win - 1]>,  relW likewise with columns,
// keys past N are masked, rows are softmax-normalised (an empty row gives 0),
// and the result of permuted row p is written to raster token perm[p]
// (the inverse permutation and the head merge are fused into the store).
//
// One CTA = 128 permuted queries of one row, 4 warps, thread i owns query row i:
//   prologue : gather Q rows by perm (cp.async, UMMA SW128/SW32 layout), load the
//              rel-pos tables, P_H = Q Th^T and P_W = Q Tw^T on the tensor cores,
//              and scatter the per-row bias windows into shared memory;
//   per key block (64 keys, double-buffered cp.async gathers):
//              S = Q K^T (UMMA -> TMEM), row softmax from TMEM in registers
//              (online max/sum, exp2), P -> shared memory (bf16), O_blk = P V
//              (UMMA, V as an MN-major operand), O = alpha*O + O_blk in registers.
#include <cuda_fp16.h>

#include "common.cuh"
#include "host_util.h"

namespace ssam {

constexpr int kAttnThreads = 128;
constexpr int kAttnBM = 128;    // queries per CTA
constexpr int kAttnBN = 64;     // keys per block (the reference's 64-token mask granularity)
constexpr int kAttnTmemCols = 256;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Shared-memory geometry of a D-wide operand tile with R rows: the first 64
// channels in a 128B-swizzled region (R x 128 B), channels 64..79 (D == 80) in a
// 32B-swizzled region (R x 32 B) right after it.
template <int D>
struct TileGeom {
  static constexpr int kChunks = D / 8;  // 16-byte chunks per row
  static constexpr bool kTail = D > 64;
  static __host__ __device__ constexpr int bytes(int rows) { return rows * 128 + (kTail ? rows * 32 : 0); }
};

// Destination of 16-byte chunk c of row r inside a TileGeom region.
template <int D>
__device__ __forceinline__ uint32_t tile_chunk_addr(uint32_t base, int rows, int r, int c) {
  if (c < 8) return base + r * 128 + ((c ^ (r & 7)) << 4);
  return base + rows * 128 + r * 32 + (((c - 8) ^ ((r >> 2) & 1)) << 4);
}

// K-major operand descriptor for k-step ks (16 channels) of a TileGeom region.
template <int D>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int rows, int ks) {
  if (ks < 4) return make_smem_desc(base + ks * 32, 16, 1024, kSw128);
  return make_smem_desc(base + rows * 128, 16, 256, kSw32);
}

struct AttnParams {
  const __nv_bfloat16* qkv;
  int64_t ld_qkv;
  int heads, win, N, C;
  const __nv_bfloat16* th;  // (2win-1, D)
  const __nv_bfloat16* tw;
  const int32_t* perm;
  int n_init, with_diag;
  float scale_log2;  // scale * log2(e)
  __nv_bfloat16* out;
  int64_t ld_out;
  int nt;  // table rows padded to the MMA N (32 or 128)
};

template <int D>
struct AttnSmem {
  static constexpr int kQ = 0;
  static constexpr int kQBytes = TileGeom<D>::bytes(kAttnBM);
  static constexpr int kKVBytes = TileGeom<D>::bytes(kAttnBN);
  static constexpr int kK0 = kQ + kQBytes;           // K[2], V[2] (tables alias this region)
  static constexpr int kV0 = kK0 + 2 * kKVBytes;
  static constexpr int kP = kV0 + 2 * kKVBytes;      // 128 x 64 bf16, SW128
  static constexpr int kBias = kP + kAttnBM * 128;   // biasH[win][128], biasW[win][128] fp16
  static_assert(2 * TileGeom<D>::bytes(128) <= 4 * kKVBytes, "rel-pos tables must fit in the K/V region");
  static_assert(kK0 % 1024 == 0 && kKVBytes % 1024 == 0 && kP % 1024 == 0, "UMMA regions need 1 KB alignment");
  static __host__ __device__ constexpr int bias_bytes(int win) { return 2 * win * kAttnBM * 2; }
  static __host__ __device__ constexpr int kinfo_off(int win) { return kBias + bias_bytes(win); }
  static __host__ __device__ constexpr int total(int win) {
    return kinfo_off(win) + 2 * kAttnBN * 4 /*kinfo[2][64]*/ + kAttnBM * 4 /*tok*/ + 64 /*bar+tmem*/ + 1024;
  }
};

template <int D>
__global__ void __launch_bounds__(kAttnThreads, 2) sparse_attn_kernel(const AttnParams a) {
  using SM = AttnSmem<D>;
  using TG = TileGeom<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t s_base = smem_u32(smem);
  // Per-row bias windows, stored transposed ([j][row]) in fp16 like the
  // reference's sRelH / sRelW (flash_attn.py:838-839).
  __half* s_bias_h = reinterpret_cast<__half*>(smem + SM::kBias);
  __half* s_bias_w = s_bias_h + a.win * kAttnBM;
  int* s_kinfo = reinterpret_cast<int*>(smem + SM::kinfo_off(a.win));  // [2][64]
  int* s_tok = s_kinfo + 2 * kAttnBN;                                  // [128]
  uint64_t* bar = reinterpret_cast<uint64_t*>(s_tok + kAttnBM);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bar + 1);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int n_tiles = (a.N + kAttnBM - 1) / kAttnBM;
  const int tile = blockIdx.x % n_tiles;
  const int row = blockIdx.x / n_tiles;
  const int seq = row / a.heads, head = row - seq * a.heads;
  const int N = a.N, win = a.win;
  const int32_t* perm = a.perm + static_cast<int64_t>(row) * N;
  const __nv_bfloat16* q_base = a.qkv + static_cast<int64_t>(seq) * N * a.ld_qkv + head * D;
  const __nv_bfloat16* k_base = q_base + a.C;
  const __nv_bfloat16* v_base = q_base + 2 * a.C;
  const int nblk = (N + kAttnBN - 1) / kAttnBN;

  // Enabled key blocks of this tile: the keep bar, then the diagonal blocks.
  const int nk = a.n_init < nblk ? a.n_init : nblk;
  int n_diag = 0, diag0 = -1, diag1 = -1;
  if (a.with_diag) {
    for (int mb = 2 * tile; mb < 2 * tile + 2; ++mb) {
      if (mb < nblk && mb >= nk) {
        if (n_diag == 0) diag0 = mb; else diag1 = mb;
        ++n_diag;
      }
    }
  }
  const int n_blocks = nk + n_diag;
  auto block_at = [&](int i) { return i < nk ? i : (i == nk ? diag0 : diag1); };

  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_holder, kAttnTmemCols);
    tmem_relinquish();
  }

  // ---- prologue: Q rows (gathered by perm) and the two rel-pos tables ----
  {
    const int p = tile * kAttnBM + tid;
    s_tok[tid] = p < N ? __ldg(perm + p) : -1;
  }
  __syncthreads();
  const uint32_t sQ = s_base + SM::kQ;
  for (int idx = tid; idx < kAttnBM * TG::kChunks; idx += kAttnThreads) {
    const int r = idx / TG::kChunks, c = idx - r * TG::kChunks;
    const int t = s_tok[r];
    const void* src = t >= 0 ? static_cast<const void*>(q_base + static_cast<int64_t>(t) * a.ld_qkv + c * 8)
                             : static_cast<const void*>(a.qkv);
    cp_async16(tile_chunk_addr<D>(sQ, kAttnBM, r, c), src, t >= 0 ? 16u : 0u);
  }
  const uint32_t sTh = s_base + SM::kK0;
  const uint32_t sTw = sTh + TG::bytes(kAttnBM);
  const int trows = 2 * win - 1;
  for (int idx = tid; idx < a.nt * TG::kChunks; idx += kAttnThreads) {
    const int r = idx / TG::kChunks, c = idx - r * TG::kChunks;
    const bool ok = r < trows;
    cp_async16(tile_chunk_addr<D>(sTh, kAttnBM, r, c), ok ? static_cast<const void*>(a.th + r * D + c * 8) : a.th,
               ok ? 16u : 0u);
    cp_async16(tile_chunk_addr<D>(sTw, kAttnBM, r, c), ok ? static_cast<const void*>(a.tw + r * D + c * 8) : a.tw,
               ok ? 16u : 0u);
  }
  cp_async_commit();
  cp_async_wait_all();
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint32_t t_lane = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  uint32_t bar_phase = 0;
  bool ok = true;

  // P_H -> columns [0, nt), P_W -> columns [128, 128 + nt).
  if (tid == 0) {
    const uint32_t idesc_t = make_idesc_bf16(kAttnBM, a.nt, 0, 0);
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      umma_f16_ss(tmem, kmajor_desc<D>(sQ, kAttnBM, ks), kmajor_desc<D>(sTh, kAttnBM, ks), idesc_t, ks > 0);
      umma_f16_ss(tmem + 128, kmajor_desc<D>(sQ, kAttnBM, ks), kmajor_desc<D>(sTw, kAttnBM, ks), idesc_t, ks > 0);
    }
    umma_commit(bar);
  }
  ok = mbar_wait(bar, bar_phase);
  bar_phase ^= 1;
  ok = __syncthreads_and(ok);
  tc_fence_after();

  const int my_tok = s_tok[tid];
  const int qh = my_tok >= 0 ? my_tok / win : 0;
  const int qw = my_tok >= 0 ? my_tok - qh * win : 0;
  if (ok) {
    // relH[i][j] = P_H[i][qh - j + win - 1]: column c holds j = qh + win - 1 - c.
    for (int c0 = 0; c0 < a.nt; c0 += 32) {
      uint32_t rh[32], rw[32];
      tmem_ld_32x32b_x32(t_lane + c0, rh);
      tmem_ld_32x32b_x32(t_lane + 128 + c0, rw);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int jh = qh + win - 1 - (c0 + j);
        if (jh >= 0 && jh < win) s_bias_h[jh * kAttnBM + tid] = __float2half_rn(__uint_as_float(rh[j]));
        const int jw = qw + win - 1 - (c0 + j);
        if (jw >= 0 && jw < win) s_bias_w[jw * kAttnBM + tid] = __float2half_rn(__uint_as_float(rw[j]));
      }
    }
  }
  tc_fence_before();
  __syncthreads();  // tables consumed: the K/V region is free; bias visible to all threads

  // ---- main loop over enabled key blocks ----
  auto load_kv = [&](int i, int buf) {
    const int kb = block_at(i);
    const uint32_t sK = s_base + SM::kK0 + buf * SM::kKVBytes;
    const uint32_t sV = s_base + SM::kV0 + buf * SM::kKVBytes;
    if (tid < kAttnBN) {
      const int kp = kb * kAttnBN + tid;
      int info = -1;
      if (kp < N) {
        const int t = __ldg(perm + kp);
        const int kh = t / win;
        info = kh | ((t - kh * win) << 16);
      }
      s_kinfo[buf * kAttnBN + tid] = info;
    }
    for (int idx = tid; idx < kAttnBN * TG::kChunks; idx += kAttnThreads) {
      const int r = idx / TG::kChunks, c = idx - r * TG::kChunks;
      const int kp = kb * kAttnBN + r;
      const int t = kp < N ? __ldg(perm + kp) : -1;
      const int64_t off = static_cast<int64_t>(t) * a.ld_qkv + c * 8;
      cp_async16(tile_chunk_addr<D>(sK, kAttnBN, r, c), t >= 0 ? static_cast<const void*>(k_base + off) : a.qkv,
                 t >= 0 ? 16u : 0u);
      cp_async16(tile_chunk_addr<D>(sV, kAttnBN, r, c), t >= 0 ? static_cast<const void*>(v_base + off) : a.qkv,
                 t >= 0 ? 16u : 0u);
    }
    cp_async_commit();
  };

  float o[D];
#pragma unroll
  for (int c = 0; c < D; ++c) o[c] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;
  const int my_mb = 2 * tile + (tid >= 64 ? 1 : 0);
  const float log2e = 1.4426950408889634f;
  const uint32_t sP = s_base + SM::kP;
  const uint32_t idesc_s = make_idesc_bf16(kAttnBM, kAttnBN, 0, 0);
  const uint32_t idesc_o64 = make_idesc_bf16(kAttnBM, 64, 0, 1);
  const uint32_t idesc_o16 = make_idesc_bf16(kAttnBM, 16, 0, 1);

  if (ok && n_blocks > 0) load_kv(0, 0);
  for (int i = 0; i < n_blocks && ok; ++i) {
    const int buf = i & 1;
    const int kb = block_at(i);
    cp_async_wait_all();
    fence_proxy_async_smem();
    __syncthreads();
    if (i + 1 < n_blocks) load_kv(i + 1, buf ^ 1);
    const uint32_t sK = s_base + SM::kK0 + buf * SM::kKVBytes;
    const uint32_t sV = s_base + SM::kV0 + buf * SM::kKVBytes;

    // S = Q K^T -> TMEM columns [0, 64)
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks)
        umma_f16_ss(tmem, kmajor_desc<D>(sQ, kAttnBM, ks), kmajor_desc<D>(sK, kAttnBN, ks), idesc_s, ks > 0);
      umma_commit(bar);
    }
    ok = mbar_wait(bar, bar_phase);
    bar_phase ^= 1;
    ok = __syncthreads_and(ok);
    if (!ok) break;
    tc_fence_after();

    uint32_t s[64];
    {
      uint32_t (&s0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[0]);
      uint32_t (&s1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[32]);
      tmem_ld_32x32b_x32(t_lane, s0);
      tmem_ld_32x32b_x32(t_lane + 32, s1);
      tmem_ld_wait();
    }
    const bool row_on = (kb < nk) || (kb == my_mb);
    const int* kinfo = s_kinfo + buf * kAttnBN;
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      const int info = kinfo[j];
      float x = -INFINITY;
      if (row_on && info >= 0) {
        const float bh = __half2float(s_bias_h[(info & 0xffff) * kAttnBM + tid]);
        const float bw = __half2float(s_bias_w[(info >> 16) * kAttnBM + tid]);
        x = __uint_as_float(s[j]) * a.scale_log2 + (bh + bw) * log2e;
      }
      s[j] = __float_as_uint(x);
      mx = fmaxf(mx, x);
    }
    const float m_new = fmaxf(m_run, mx);
    const float m_use = m_new == -INFINITY ? 0.f : m_new;
    const float alpha = fast_exp2(m_run - m_use);
    float sum = 0.f;
    uint8_t* prow = smem + SM::kP + tid * 128;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float pv[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        pv[e] = fast_exp2(__uint_as_float(s[c * 8 + e]) - m_use);
        sum += pv[e];
      }
      uint4 w;
      w.x = pack_bf16x2(pv[0], pv[1]);
      w.y = pack_bf16x2(pv[2], pv[3]);
      w.z = pack_bf16x2(pv[4], pv[5]);
      w.w = pack_bf16x2(pv[6], pv[7]);
      *reinterpret_cast<uint4*>(prow + ((c ^ (tid & 7)) << 4)) = w;
    }
    l_run = l_run * alpha + sum;
    m_run = m_new;

    // O_blk = P V -> TMEM columns [128, 128 + D)
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < kAttnBN / 16; ++ks) {
        const uint64_t pd = make_smem_desc(sP + ks * 32, 16, 1024, kSw128);
        umma_f16_ss(tmem + 128, pd, make_smem_desc(sV + ks * 2048, 8192, 1024, kSw128), idesc_o64, ks > 0);
        if constexpr (TG::kTail)
          umma_f16_ss(tmem + 192, pd, make_smem_desc(sV + kAttnBN * 128 + ks * 512, 4096, 256, kSw32), idesc_o16,
                      ks > 0);
      }
      umma_commit(bar);
    }
    ok = mbar_wait(bar, bar_phase);
    bar_phase ^= 1;
    ok = __syncthreads_and(ok);
    if (!ok) break;
    tc_fence_after();
    {
      uint32_t r[32];
      tmem_ld_32x32b_x32(t_lane + 128, r);
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < 32; ++c) o[c] = o[c] * alpha + __uint_as_float(r[c]);
      tmem_ld_32x32b_x32(t_lane + 160, r);
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < 32; ++c) o[32 + c] = o[32 + c] * alpha + __uint_as_float(r[c]);
      if constexpr (D > 64) {
        uint32_t r16[16];
        tmem_ld_32x32b_x16(t_lane + 192, r16);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 16; ++c) o[64 + c] = o[64 + c] * alpha + __uint_as_float(r16[c]);
      }
    }
    tc_fence_before();
  }

  // ---- epilogue: normalise and store at the raster position (inverse permutation) ----
  if (ok && my_tok >= 0) {
    const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
    uint4* dst = reinterpret_cast<uint4*>(a.out + (static_cast<int64_t>(seq) * N + my_tok) * a.ld_out + head * D);
#pragma unroll
    for (int c = 0; c < D / 8; ++c) {
      uint4 w;
      w.x = pack_bf16x2(o[8 * c + 0] * inv_l, o[8 * c + 1] * inv_l);
      w.y = pack_bf16x2(o[8 * c + 2] * inv_l, o[8 * c + 3] * inv_l);
      w.z = pack_bf16x2(o[8 * c + 4] * inv_l, o[8 * c + 5] * inv_l);
      w.w = pack_bf16x2(o[8 * c + 6] * inv_l, o[8 * c + 7] * inv_l);
      dst[c] = w;
    }
  }

  // ---- teardown: drain copies and MMAs, free TMEM ----
  cp_async_wait_all();
  if (!ok && tid == 0) {
    umma_commit(bar);
    mbar_wait(bar, bar_phase);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, kAttnTmemCols);
}

template <int D>
static int launch_attn(const AttnParams& p, int n_rows, cudaStream_t stream) {
  using SM = AttnSmem<D>;
  // At least 96 KB so that no more than two CTAs share an SM: two CTAs x 256
  // TMEM columns fill the 512-column TMEM exactly.
  const int smem = SM::total(p.win) > 96 * 1024 ? SM::total(p.win) : 96 * 1024;
  static bool configured[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return SSAM_ERR_CUDA;
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(sparse_attn_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             SM::total(64) > 96 * 1024 ? SM::total(64) : 96 * 1024) != cudaSuccess)
      return SSAM_ERR_CUDA;
    configured[dev] = true;
  }
  const int64_t grid = static_cast<int64_t>((p.N + kAttnBM - 1) / kAttnBM) * n_rows;
  if (grid > INT32_MAX) return SSAM_ERR_UNSUPPORTED;
  sparse_attn_kernel<D><<<static_cast<unsigned>(grid), kAttnThreads, smem, stream>>>(p);
  return status_from_cuda(cudaGetLastError());
}

int sparse_attn_fwd(const void* qkv, int64_t ld_qkv, int n_seq, int heads, int win, int d, const void* rel_pos_h,
                    const void* rel_pos_w, const int32_t* perm, int n_init_blocks, int with_diag, float scale,
                    void* out, int64_t ld_out, cudaStream_t stream) {
  if (qkv == nullptr || rel_pos_h == nullptr || rel_pos_w == nullptr || perm == nullptr || out == nullptr)
    return SSAM_ERR_INVALID;
  if (n_seq <= 0 || heads <= 0 || win <= 0 || n_init_blocks < 0) return SSAM_ERR_INVALID;
  if (d != 64 && d != 80) return SSAM_ERR_UNSUPPORTED;
  if (win > 64) return SSAM_ERR_UNSUPPORTED;  // 2*win-1 table rows must fit one 128-wide MMA
  const int C = heads * d;
  if (ld_qkv < 3 * C || ld_out < C) return SSAM_ERR_INVALID;
  if (ld_qkv % 8 || ld_out % 8 || !aligned16(qkv) || !aligned16(out) || !aligned16(rel_pos_h) ||
      !aligned16(rel_pos_w))
    return SSAM_ERR_ALIGN;
  AttnParams p;
  p.qkv = static_cast<const __nv_bfloat16*>(qkv);
  p.ld_qkv = ld_qkv;
  p.heads = heads;
  p.win = win;
  p.N = win * win;
  p.C = C;
  p.th = static_cast<const __nv_bfloat16*>(rel_pos_h);
  p.tw = static_cast<const __nv_bfloat16*>(rel_pos_w);
  p.perm = perm;
  p.n_init = n_init_blocks;
  p.with_diag = with_diag ? 1 : 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ld_out = ld_out;
  p.nt = (2 * win - 1) <= 32 ? 32 : 128;
  const int n_rows = n_seq * heads;
  return d == 64 ? launch_attn<64>(p, n_rows, stream) : launch_attn<80>(p, n_rows, stream);
}

}  // namespace ssam
