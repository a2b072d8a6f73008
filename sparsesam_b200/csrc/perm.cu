// Token-order kernels: Morton order, Stripe-Sort permutation and the
// Residual-Consistency keep set. All outputs are integer index tensors and are
// produced bit-exactly: group scores are accumulated in fp64 and every ranking
// breaks ties by the lowest index.
#include "common.cuh"
#include "host_util.h"

namespace ssam {

constexpr int kMaxTokens = 16384;  // largest H*W handled by the permutation kernels

// ---------------------------------------------------------------------------
// a1. Morton order (algos/sparsesam/z_utils.py:35-49 encode, :65-85 _compute_z_order).
// Key of raster cell (r, c): bit i of r at position 2i+1, bit i of c at 2i,
// over num_bits = max(1, ceil(log2(max(H, W)))). perm = argsort(key); keys are
// unique, so the rank of a cell is the number of smaller keys.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t morton_key(uint32_t r, uint32_t c, int num_bits) {
  uint32_t z = 0;
  for (int i = 0; i < num_bits; ++i) {
    z |= ((r >> i) & 1u) << (2 * i + 1);
    z |= ((c >> i) & 1u) << (2 * i);
  }
  return z;
}

__global__ void zorder_kernel(int H, int W, int num_bits, int32_t* perm, int32_t* inv_perm) {
  const int N = H * W;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N) return;
  const uint32_t ki = morton_key(i / W, i % W, num_bits);
  int rank = 0;
  for (int j = 0; j < N; ++j) rank += morton_key(j / W, j % W, num_bits) < ki;
  perm[rank] = i;
  if (inv_perm != nullptr) inv_perm[i] = rank;
}

int zorder(int H, int W, int32_t* perm, int32_t* inv_perm, cudaStream_t stream) {
  if (H <= 0 || W <= 0 || perm == nullptr || H * W > kMaxTokens) return SSAM_ERR_INVALID;
  int m = H > W ? H : W;
  int num_bits = 0;
  while ((1 << num_bits) < m) ++num_bits;  // ceil(log2(m))
  if (num_bits < 1) num_bits = 1;
  const int N = H * W;
  zorder_kernel<<<(N + 255) / 256, 256, 0, stream>>>(H, W, num_bits, perm, inv_perm);
  return status_from_cuda(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// Hilbert order, the `hilbert` perm_mode space (algos/sparsesam/hilbert_utils.py:
// 55-76 _forward_hilbert_transform, :28-33 _transposed_to_h, :108-129 grid order).
// Skilling's transpose algorithm (J. Skilling, "Programming the Hilbert curve",
// AIP Conf. Proc. 707, 2004) in two dimensions, row = axis 0, column = axis 1,
// over p = max(1, ceil(log2(max(H, W)))) bits; the index interleaves the
// transposed bits with axis 0 the higher of each pair. Keys are unique, so the
// rank of a cell is the number of smaller keys.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t hilbert_key(uint32_t r, uint32_t c, int p) {
  uint32_t x0 = r, x1 = c;
  const uint32_t top = 1u << (p - 1);
  for (uint32_t q = top; q > 1; q >>= 1) {  // undo excess work: axis 0, then axis 1
    const uint32_t low = q - 1;
    if (x0 & q) x0 ^= low;
    if (x1 & q) {
      x0 ^= low;
    } else {
      const uint32_t t = (x0 ^ x1) & low;
      x0 ^= t;
      x1 ^= t;
    }
  }
  x1 ^= x0;  // Gray encode
  uint32_t t = 0;
  for (uint32_t q = top; q > 1; q >>= 1)
    if (x1 & q) t ^= q - 1;
  x0 ^= t;
  x1 ^= t;
  uint32_t h = 0;
  for (int i = 0; i < p; ++i) {
    h |= ((x0 >> (p - 1 - i)) & 1u) << (2 * p - 1 - 2 * i);
    h |= ((x1 >> (p - 1 - i)) & 1u) << (2 * p - 2 - 2 * i);
  }
  return h;
}

__global__ void hilbert_kernel(int H, int W, int num_bits, int32_t* perm, int32_t* inv_perm) {
  const int N = H * W;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N) return;
  const uint32_t ki = hilbert_key(i / W, i % W, num_bits);
  int rank = 0;
  for (int j = 0; j < N; ++j) rank += hilbert_key(j / W, j % W, num_bits) < ki;
  perm[rank] = i;
  if (inv_perm != nullptr) inv_perm[i] = rank;
}

int hilbert_order(int H, int W, int32_t* perm, int32_t* inv_perm, cudaStream_t stream) {
  if (H <= 0 || W <= 0 || perm == nullptr || H * W > kMaxTokens) return SSAM_ERR_INVALID;
  int m = H > W ? H : W;
  int num_bits = 0;
  while ((1 << num_bits) < m) ++num_bits;  // ceil(log2(m))
  if (num_bits < 1) num_bits = 1;
  const int N = H * W;
  hilbert_kernel<<<(N + 255) / 256, 256, 0, stream>>>(H, W, num_bits, perm, inv_perm);
  return status_from_cuda(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// a2. Stripe-Sort permutation (algos/sparsesam/sam.py:105-164, tile_stride_matching).
// One CTA per (sequence, head) row:
//   1. groups of `gs` consecutive tokens in base order (Z or Hilbert curve);
//   2. grp_std = mean over channels of the unbiased std over the group;
//      grp_mean normalised to unit L2 norm (eps 1e-12);
//   3. avg_sim_g = (sum_j <n_g, n_j> - 1) / max(G-1, 1) computed as
//      (<n_g, S> - 1)/(G-1) with S = sum_j n_j (the same sum, O(G d));
//   4. score = z(grp_std) + z(-avg_sim), z = (x - mean) / (unbiased std + 1e-6);
//   5. descending rank, ties -> lowest group index; layout interleave / naive.
// ---------------------------------------------------------------------------
struct StripeArgs {
  const __nv_bfloat16* k;
  int64_t ld;
  int heads, N, d, gs, G, layout, ranking;
  const int32_t* base_perm;
  int32_t* perm;
  int32_t* inv_perm;
  int32_t* inv_perm_group;
};

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide fp64 sum; `red` is a shared array of at least 32 doubles.
__device__ double block_sum_d(double v, double* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum_d(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double t = 0.0;
  for (int i = 0; i < nw; ++i) t += red[i];  // fixed order: identical on every thread
  return t;
}

constexpr int kStripeMaxChPerLane = 8;  // d <= 256

// x[i][j] = K[token j of group g][channel lane + 32 i] (0 past d): the group's
// tokens are read by GS lanes and shuffled, then all CH x GS values are loaded.
template <int GS, int CH>
__device__ __forceinline__ void stripe_group_values(const StripeArgs& a, const __nv_bfloat16* kr, int g, int lane,
                                                    int d, float (&x)[CH][GS]) {
  const int tk = lane < GS ? __ldg(a.base_perm + g * GS + lane) : 0;
  int t[GS];
#pragma unroll
  for (int j = 0; j < GS; ++j) t[j] = __shfl_sync(0xffffffffu, tk, j);
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int c = lane + 32 * i;
#pragma unroll
    for (int j = 0; j < GS; ++j)
      x[i][j] = c < d ? __bfloat162float(kr[static_cast<int64_t>(t[j]) * a.ld + c]) : 0.f;
  }
}

// GS > 0: group size known at compile time (SparseSAM uses 4): the tokens of a
// group are fetched once per warp and shuffled, the group's CH x GS values are
// loaded together (one memory round trip per group instead of one per value)
// and kept in registers for the variance. GS == 0: any group size (up to 32),
// values re-read per channel. The per-channel mean / variance follow
// np.std(ddof=1): sum in token order, mean = sum / gs, squared deviations
// rounded before they are summed (no fused multiply-add).
template <int GS, int CH>
__global__ void stripe_sort_kernel(const StripeArgs a) {
  extern __shared__ double sm_d[];
  double* s_std = sm_d;               // [G]
  double* s_inv = s_std + a.G;        // [G]  1 / max(||mean||, 1e-12)
  double* s_score = s_inv + a.G;      // [G]
  double* s_S = s_score + a.G;        // [d]
  double* s_red = s_S + a.d;          // [32]
  int* s_order = reinterpret_cast<int*>(s_red + 32);  // [G]

  const int row = blockIdx.x;
  const int seq = row / a.heads, head = row - seq * a.heads;
  const __nv_bfloat16* kr = a.k + static_cast<int64_t>(seq) * a.N * a.ld + static_cast<int64_t>(head) * a.d;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int G = a.G, gs = GS > 0 ? GS : a.gs, d = a.d, N = a.N;

  int32_t* perm = a.perm + static_cast<int64_t>(row) * N;
  int32_t* inv_perm = a.inv_perm + static_cast<int64_t>(row) * N;
  int32_t* inv_perm_group = a.inv_perm_group + static_cast<int64_t>(row) * N;

  if (a.ranking == SSAM_RANKING_SORT) {
    for (int c = threadIdx.x; c < d; c += blockDim.x) s_S[c] = 0.0;
    __syncthreads();
    // Pass 1: per-group std and norm, per-warp partial S.
    double Sp[CH];
#pragma unroll
    for (int i = 0; i < CH; ++i) Sp[i] = 0.0;
    for (int g = warp; g < G; g += nw) {
      double mean[CH];
      double std_sum = 0.0, sq = 0.0;
      if constexpr (GS > 0) {
        float x[CH][GS];
        stripe_group_values<GS, CH>(a, kr, g, lane, d, x);
#pragma unroll
        for (int i = 0; i < CH; ++i) {
          mean[i] = 0.0;
          if (lane + 32 * i < d) {
            double m = 0.0;
#pragma unroll
            for (int j = 0; j < GS; ++j) m = __dadd_rn(m, static_cast<double>(x[i][j]));
            m = m / GS;
            double v = 0.0;
#pragma unroll
            for (int j = 0; j < GS; ++j) {
              const double dx = __dsub_rn(static_cast<double>(x[i][j]), m);
              v = __dadd_rn(v, __dmul_rn(dx, dx));
            }
            std_sum += GS > 1 ? sqrt(v / (GS - 1)) : __longlong_as_double(0x7ff8000000000000ll);
            mean[i] = m;
            sq += m * m;
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < CH; ++i) {
          const int c = lane + 32 * i;
          mean[i] = 0.0;
          if (c < d) {
            double m = 0.0;
            for (int j = 0; j < gs; ++j) {
              const int t = __ldg(a.base_perm + g * gs + j);
              m = __dadd_rn(m, static_cast<double>(__bfloat162float(kr[static_cast<int64_t>(t) * a.ld + c])));
            }
            m /= gs;
            double v = 0.0;  // second pass re-reads the (L1-resident) group
            for (int j = 0; j < gs; ++j) {
              const int t = __ldg(a.base_perm + g * gs + j);
              const double dx =
                  __dsub_rn(static_cast<double>(__bfloat162float(kr[static_cast<int64_t>(t) * a.ld + c])), m);
              v = __dadd_rn(v, __dmul_rn(dx, dx));
            }
            std_sum += gs > 1 ? sqrt(v / (gs - 1)) : __longlong_as_double(0x7ff8000000000000ll);
            mean[i] = m;
            sq += m * m;
          }
        }
      }
      std_sum = warp_sum_d(std_sum);
      sq = warp_sum_d(sq);
      const double nrm = sqrt(sq);
      const double inv = 1.0 / (nrm > 1e-12 ? nrm : 1e-12);
      if (lane == 0) {
        s_std[g] = std_sum / d;
        s_inv[g] = inv;
      }
#pragma unroll
      for (int i = 0; i < CH; ++i) Sp[i] += mean[i] * inv;
    }
    // Reduce S over warps in a fixed warp order.
    for (int w = 0; w < nw; ++w) {
      __syncthreads();
      if (warp == w) {
#pragma unroll
        for (int i = 0; i < CH; ++i) {
          const int c = lane + 32 * i;
          if (c < d) s_S[c] += Sp[i];
        }
      }
    }
    __syncthreads();
    // Pass 2: <n_g, S> -> dissimilarity.
    for (int g = warp; g < G; g += nw) {
      double dot = 0.0;
      if constexpr (GS > 0) {
        float x[CH][GS];
        stripe_group_values<GS, CH>(a, kr, g, lane, d, x);
#pragma unroll
        for (int i = 0; i < CH; ++i) {
          const int c = lane + 32 * i;
          if (c < d) {
            double m = 0.0;
#pragma unroll
            for (int j = 0; j < GS; ++j) m = __dadd_rn(m, static_cast<double>(x[i][j]));
            dot += (m / GS) * s_S[c];
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < CH; ++i) {
          const int c = lane + 32 * i;
          if (c < d) {
            double m = 0.0;
            for (int j = 0; j < gs; ++j) {
              const int t = __ldg(a.base_perm + g * gs + j);
              m = __dadd_rn(m, static_cast<double>(__bfloat162float(kr[static_cast<int64_t>(t) * a.ld + c])));
            }
            dot += (m / gs) * s_S[c];
          }
        }
      }
      dot = warp_sum_d(dot);
      if (lane == 0) {
        const double avg_sim = (dot * s_inv[g] - 1.0) / (G > 1 ? G - 1 : 1);
        s_score[g] = -avg_sim;  // dissimilarity
      }
    }
    __syncthreads();
    // z-scores over groups (unbiased std, eps 1e-6).
    double ps = 0.0, pd = 0.0;
    for (int g = threadIdx.x; g < G; g += blockDim.x) {
      ps += s_std[g];
      pd += s_score[g];
    }
    const double mean_s = block_sum_d(ps, s_red) / G;
    const double mean_d = block_sum_d(pd, s_red) / G;
    double vs = 0.0, vd = 0.0;
    for (int g = threadIdx.x; g < G; g += blockDim.x) {
      vs += (s_std[g] - mean_s) * (s_std[g] - mean_s);
      vd += (s_score[g] - mean_d) * (s_score[g] - mean_d);
    }
    const double den = G > 1 ? G - 1 : 0;  // torch.std of one element is NaN
    const double sd_s = sqrt(block_sum_d(vs, s_red) / den);
    const double sd_d = sqrt(block_sum_d(vd, s_red) / den);
    __syncthreads();
    for (int g = threadIdx.x; g < G; g += blockDim.x) {
      const double zs = (s_std[g] - mean_s) / (sd_s + 1e-6);
      const double zd = (s_score[g] - mean_d) / (sd_d + 1e-6);
      s_inv[g] = zs + zd;  // reuse as the final score
    }
    __syncthreads();
    // Descending rank with lowest-index ties.
    for (int g = threadIdx.x; g < G; g += blockDim.x) {
      const double sg = s_inv[g];
      int r = 0;
      for (int j = 0; j < G; ++j) {
        const double sj = s_inv[j];
        r += (sj > sg) || (sj == sg && j < g);
      }
      s_order[r] = g;
    }
  } else {
    for (int g = threadIdx.x; g < G; g += blockDim.x) s_order[g] = g;
  }
  __syncthreads();

  // Emit perm (interleave or naive), inv_perm, inv_perm_group.
  for (int q = threadIdx.x; q < G; q += blockDim.x) {
    const int g = s_order[q];
    for (int t = 0; t < gs; ++t) {
      const int raster = __ldg(a.base_perm + g * gs + t);
      const int pg = q * gs + t;
      const int pi = a.layout == SSAM_LAYOUT_INTERLEAVE ? t * G + q : pg;
      perm[pi] = raster;
      inv_perm[raster] = pi;
      inv_perm_group[raster] = pg;
    }
  }
}

// threads: the block size for small rows (G <= 256); rows of more groups get as many
// warps as the variant's registers allow (up to 1024 threads): each warp walks its
// groups one at a time with one group's gathers in flight, so a row's two passes are
// latency chains whose length is groups per warp — with fewer rows than SMs (a
// global grid at small batches) nothing else hides them.
template <int GS, int CH>
static int launch_stripe(const StripeArgs& a, int rows, int threads, size_t smem, cudaStream_t stream) {
  static PerDeviceOnce configured;
  static std::atomic<int> max_threads{256};
  const int st = configured.run(current_device(), [] {
    cudaFuncAttributes attr;
    int e = status_from_cuda(cudaFuncGetAttributes(&attr, stripe_sort_kernel<GS, CH>));
    if (e != SSAM_OK) return e;
    const int by_regs = attr.numRegs > 0 ? (65536 / (attr.numRegs * 32)) * 32 : 256;
    int t = by_regs < attr.maxThreadsPerBlock ? by_regs : attr.maxThreadsPerBlock;
    t = t > 1024 ? 1024 : (t < 256 ? 256 : t);
    max_threads.store(t, std::memory_order_relaxed);
    return status_from_cuda(
        cudaFuncSetAttribute(stripe_sort_kernel<GS, CH>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
  });
  if (st != SSAM_OK) return st;
  if (a.G > 256) threads = max_threads.load(std::memory_order_relaxed);
  stripe_sort_kernel<GS, CH><<<rows, threads, smem, stream>>>(a);
  return status_from_cuda(cudaGetLastError());
}

int stripe_sort_perm(const void* k, int64_t ld, int n_seq, int heads, int H, int W, int d, int gs, int layout,
                     int ranking, const int32_t* base_perm, int32_t* perm, int32_t* inv_perm, int32_t* inv_perm_group,
                     cudaStream_t stream) {
  if (k == nullptr || base_perm == nullptr || perm == nullptr || inv_perm == nullptr || inv_perm_group == nullptr)
    return SSAM_ERR_INVALID;
  if (n_seq <= 0 || heads <= 0 || H <= 0 || W <= 0 || d <= 0 || gs <= 0) return SSAM_ERR_INVALID;
  if (layout != SSAM_LAYOUT_INTERLEAVE && layout != SSAM_LAYOUT_NAIVE) return SSAM_ERR_INVALID;
  if (ranking != SSAM_RANKING_SORT && ranking != SSAM_RANKING_NOSORT) return SSAM_ERR_INVALID;
  const int N = H * W;
  if (N % gs != 0) return SSAM_ERR_INVALID;  // sam.py:116
  if (N > kMaxTokens || d > 32 * kStripeMaxChPerLane || gs > 32) return SSAM_ERR_UNSUPPORTED;
  if (ld < static_cast<int64_t>(heads) * d) return SSAM_ERR_INVALID;
  StripeArgs a{static_cast<const __nv_bfloat16*>(k), ld, heads, N, d, gs, N / gs, layout, ranking, base_perm,
               perm, inv_perm, inv_perm_group};
  const int G = N / gs;
  const size_t smem = sizeof(double) * (3 * static_cast<size_t>(G) + d + 32) + sizeof(int) * G;
  int threads = 256;
  if (G <= 64) threads = 64;
  else if (G <= 256) threads = 128;
  if (gs == 4) {
    if (d <= 32) return launch_stripe<4, 1>(a, n_seq * heads, threads, smem, stream);
    if (d <= 64) return launch_stripe<4, 2>(a, n_seq * heads, threads, smem, stream);
    if (d <= 96) return launch_stripe<4, 3>(a, n_seq * heads, threads, smem, stream);
    if (d <= 128) return launch_stripe<4, 4>(a, n_seq * heads, threads, smem, stream);
    return launch_stripe<4, kStripeMaxChPerLane>(a, n_seq * heads, threads, smem, stream);
  }
  return launch_stripe<0, kStripeMaxChPerLane>(a, n_seq * heads, threads, smem, stream);
}

// ---------------------------------------------------------------------------
// a10 selection. Keep set (sam.py:277-280): avg_rank over heads of
// inv_perm_group, topk smallest keep_n. The key sum_h(rank) * N + token is
// unique and orders exactly like (mean rank, token index).
// ---------------------------------------------------------------------------
__global__ void keep_select_kernel(const int32_t* inv_perm_group, int heads, int N, int keep_n, int32_t* idx,
                                   int32_t* rows) {
  extern __shared__ uint64_t s_key[];
  const int b = blockIdx.x;
  const int32_t* ipg = inv_perm_group + static_cast<int64_t>(b) * heads * N;
  for (int t = threadIdx.x; t < N; t += blockDim.x) {
    uint64_t s = 0;
    for (int h = 0; h < heads; ++h) s += static_cast<uint64_t>(__ldg(ipg + static_cast<int64_t>(h) * N + t));
    s_key[t] = s * static_cast<uint64_t>(N) + static_cast<uint64_t>(t);
  }
  __syncthreads();
  // blockIdx.y selects this CTA's slice of the tokens to rank (every CTA of an
  // image builds all N keys: heads x N loads, cheap next to the N x N/slices compares)
  const int per = (N + gridDim.y - 1) / gridDim.y;
  const int t_end = min(N, (static_cast<int>(blockIdx.y) + 1) * per);
  for (int t = blockIdx.y * per + threadIdx.x; t < t_end; t += blockDim.x) {
    const uint64_t kt = s_key[t];
    int r = 0;
    for (int u = 0; u < N; ++u) r += s_key[u] < kt;
    if (r < keep_n) {
      idx[static_cast<int64_t>(b) * keep_n + r] = t;
      if (rows != nullptr) rows[static_cast<int64_t>(b) * keep_n + r] = b * N + t;
    }
  }
}

int keep_select(const int32_t* inv_perm_group, int B, int heads, int N, int keep_n, int32_t* idx, int32_t* rows,
                cudaStream_t stream) {
  if (inv_perm_group == nullptr || idx == nullptr) return SSAM_ERR_INVALID;
  if (B <= 0 || heads <= 0 || N <= 0 || keep_n <= 0 || keep_n > N) return SSAM_ERR_INVALID;
  if (N > kMaxTokens) return SSAM_ERR_UNSUPPORTED;
  static PerDeviceOnce configured;
  const int st = configured.run(current_device(), [] {
    return status_from_cuda(cudaFuncSetAttribute(keep_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 kMaxTokens * sizeof(uint64_t)));
  });
  if (st != SSAM_OK) return st;
  const int slices = N >= 4096 ? 4 : (N >= 1024 ? 2 : 1);
  keep_select_kernel<<<dim3(B, slices), 1024, N * sizeof(uint64_t), stream>>>(inv_perm_group, heads, N, keep_n, idx,
                                                                              rows);
  return status_from_cuda(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// a7. A-shape mask parameters (sam.py:219-223, flash_attn.py:132-145).
// ---------------------------------------------------------------------------
int a_shape_n_init(int N, int n_block, double ratio, int is_global) {
  if (N <= 0 || n_block <= 0 || !(ratio > 0.0) || ratio > 1.0) return -1;
  const int num_n = (N + n_block - 1) / n_block;
  const int n_keep = static_cast<int>(ratio * num_n);  // Python int() truncates toward zero
  return is_global ? n_keep : n_keep + 1;
}

// ---------------------------------------------------------------------------
// Static Z-stride keep set of the SAM3 MLP-merge variant
// (algos/sparsesam/sam3.py:49-71 _get_keep_indices): keep_n = min(max(1,
// round(ratio N)), N) Morton positions pos_i = rint(f32(i) * f32(N / keep_n))
// (fp32 product, ties to even, as torch.arange(float32) * (N / keep_n) and
// torch.round), clamped to [0, N), and idx[i] = the raster cell at Morton
// position pos_i. One thread per raster cell finds its Morton rank q (number
// of smaller keys) and stores itself at the i whose position is q; positions
// strictly increase with i (N / keep_n >= 1), so at most one i matches.
// ---------------------------------------------------------------------------
int zstride_keep_n(int N, double ratio) {
  if (N <= 0 || !(ratio > 0.0) || ratio > 1.0) return -1;
  double k = nearbyint(ratio * N);  // Python round(): ties to even (default rounding mode)
  if (k < 1.0) k = 1.0;
  return k > N ? N : static_cast<int>(k);
}

__device__ __forceinline__ int zstride_pos(int i, float step, int N) {
  const int p = static_cast<int>(rintf(__fmul_rn(static_cast<float>(i), step)));
  return p < 0 ? 0 : (p > N - 1 ? N - 1 : p);
}

__global__ void zstride_keep_kernel(int H, int W, int num_bits, int keep_n, float step, int B, int32_t* idx,
                                    int32_t* rows) {
  const int N = H * W;
  const int cell = blockIdx.x * blockDim.x + threadIdx.x;
  if (cell >= N) return;
  const uint32_t kc = morton_key(cell / W, cell % W, num_bits);
  int q = 0;
  for (int j = 0; j < N; ++j) q += morton_key(j / W, j % W, num_bits) < kc;
  // candidates around q / step; pos is strictly increasing in i
  const int i0 = static_cast<int>(static_cast<double>(q) / static_cast<double>(step));
  for (int i = i0 - 2; i <= i0 + 2; ++i) {
    if (i < 0 || i >= keep_n || zstride_pos(i, step, N) != q) continue;
    idx[i] = cell;
    if (rows != nullptr)
      for (int b = 0; b < B; ++b) rows[static_cast<int64_t>(b) * keep_n + i] = b * N + cell;
  }
}

int zstride_keep(int H, int W, int keep_n, int B, int32_t* idx, int32_t* rows, cudaStream_t stream) {
  if (H <= 0 || W <= 0 || idx == nullptr || B < 0 || (rows != nullptr && B <= 0)) return SSAM_ERR_INVALID;
  const int N = H * W;
  if (N > kMaxTokens) return SSAM_ERR_UNSUPPORTED;
  if (keep_n < 1 || keep_n > N) return SSAM_ERR_INVALID;
  if (rows != nullptr && static_cast<int64_t>(B) * N > INT32_MAX) return SSAM_ERR_UNSUPPORTED;
  int m = H > W ? H : W;
  int num_bits = 0;
  while ((1 << num_bits) < m) ++num_bits;  // ceil(log2(m)), z_utils.py:71
  if (num_bits < 1) num_bits = 1;
  const float step = static_cast<float>(static_cast<double>(N) / keep_n);  // Python float N / keep_n, then fp32
  zstride_keep_kernel<<<(N + 255) / 256, 256, 0, stream>>>(H, W, num_bits, keep_n, step, B, idx, rows);
  return status_from_cuda(cudaGetLastError());
}

int a_shape_mask(int N, int m_block, int n_block, int n_init, int with_diag, uint8_t* mask) {
  if (N <= 0 || m_block <= 0 || n_block <= 0 || mask == nullptr) return SSAM_ERR_INVALID;
  const int num_m = (N + m_block - 1) / m_block, num_n = (N + n_block - 1) / n_block;
  for (int m = 0; m < num_m; ++m)
    for (int n = 0; n < num_n; ++n) mask[m * num_n + n] = (n < n_init) || (with_diag && n == m);
  return SSAM_OK;
}

}  // namespace ssam
