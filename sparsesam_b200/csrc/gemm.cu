// Persistent, warp-specialised bf16 GEMM on the sm_100a tensor cores.
//
//   acc[r, n] = sum_k A[r, k] * B[n, k]      A: M x K, B: N x K (both K-major)
//
// Roles per CTA (one CTA per SM, 320 threads):
//   warp 0      : TMA producer — 128x64 A tile + 256x64 B tile per stage (SW128).
//   warp 1      : UMMA issuer  — tcgen05.mma M=128 N=256 K=16, fp32 accumulator
//                 in TMEM, two accumulator buffers (2 x 256 columns).
//   warps 2..9  : epilogue     — tcgen05.ld rows out of TMEM (two warps per TMEM
//                 sub-partition, each taking half of the 256 columns), fused
//                 bias / GELU / fp32 residual add through an optional row map.
// Every wait is bounded; on timeout the CTA records SSAM_ERR_TIMEOUT, drains the
// copies and MMAs it issued, frees TMEM and returns.
//
// Used for the SAM Attention.qkv / Attention.proj linears (algos/sparsesam/sam.py:182,233),
// MLPBlock lin1/lin2 (sam.py:283,286), the patch embedding and the neck convolutions.
#include "common.cuh"
#include "host_util.h"

namespace ssam {

constexpr int kGemmBM = 128;
constexpr int kGemmBN = 256;
constexpr int kGemmBK = 64;
constexpr int kGemmStages = 4;
constexpr int kGemmABytes = kGemmBM * kGemmBK * 2;  // 16 KB
constexpr int kGemmBBytes = kGemmBN * kGemmBK * 2;  // 32 KB
constexpr int kGemmStageBytes = kGemmABytes + kGemmBBytes;
constexpr int kGemmThreads = 320;
constexpr int kGemmEpiThreads = 256;
constexpr int kGemmTmemCols = 512;
constexpr int kEpiStageBytes = 32 * 32 * 4;  // per epilogue warp: one 32-row x 32-column fp32 chunk
constexpr int kEpiStageTotal = 8 * kEpiStageBytes;
constexpr int kGemmSmemBytes = kGemmStages * kGemmStageBytes + 1024 /*align slack*/ + 256 /*barriers*/ + kEpiStageTotal;

struct GemmParams {
  int M, N, K;
  const float* bias;
  void* out;
  int64_t ldo;
  const int32_t* out_rows;
  // implicit 3x3 convolution (pair kernel, CONV): A is a channels-last (B, H, W, Cin)
  // tensor map, K = 9 Cin in (ky, kx, cin) order, rows are the B*H*W output pixels
  int conv_w, conv_hw;
  // SSAM_EPI_F32: addend[(r % addend_rows) * N + n] is added to row r (may be null)
  const float* addend;
  int addend_rows;
};

template <int EPI>
__device__ __forceinline__ void gemm_epilogue_chunk(const GemmParams& p, int row, int col0, const uint32_t (&r)[32]) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
  if (p.bias != nullptr) {
    const float4* b4 = reinterpret_cast<const float4*>(p.bias + col0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 b = __ldg(b4 + i);
      const float2 lo = add2(make_float2(v[4 * i + 0], v[4 * i + 1]), make_float2(b.x, b.y));
      const float2 hi = add2(make_float2(v[4 * i + 2], v[4 * i + 3]), make_float2(b.z, b.w));
      v[4 * i + 0] = lo.x;
      v[4 * i + 1] = lo.y;
      v[4 * i + 2] = hi.x;
      v[4 * i + 3] = hi.y;
    }
  }
  if constexpr (EPI == SSAM_EPI_BF16 || EPI == SSAM_EPI_GELU_BF16) {
    if constexpr (EPI == SSAM_EPI_GELU_BF16) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float2 g = gelu_exact2(make_float2(v[2 * i], v[2 * i + 1]));
        v[2 * i] = g.x;
        v[2 * i + 1] = g.y;
      }
    }
    const int orow = p.out_rows != nullptr ? __ldg(p.out_rows + row) : row;
    if (orow < 0) return;
    uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + static_cast<int64_t>(orow) * p.ldo + col0);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 q;
      q.x = pack_bf16x2(v[8 * i + 0], v[8 * i + 1]);
      q.y = pack_bf16x2(v[8 * i + 2], v[8 * i + 3]);
      q.z = pack_bf16x2(v[8 * i + 4], v[8 * i + 5]);
      q.w = pack_bf16x2(v[8 * i + 6], v[8 * i + 7]);
      dst[i] = q;
    }
  } else if constexpr (EPI == SSAM_EPI_F32) {
    const int orow = p.out_rows != nullptr ? __ldg(p.out_rows + row) : row;
    if (orow < 0) return;
    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + static_cast<int64_t>(orow) * p.ldo + col0);
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[i] = make_float4(v[4 * i + 0], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  } else {
    const int orow = p.out_rows != nullptr ? __ldg(p.out_rows + row) : row;
    if (orow < 0) return;
    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + static_cast<int64_t>(orow) * p.ldo + col0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float4 o = dst[i];
      o.x += v[4 * i + 0];
      o.y += v[4 * i + 1];
      o.z += v[4 * i + 2];
      o.w += v[4 * i + 3];
      dst[i] = o;
    }
  }
}

// Coalesced form of gemm_epilogue_chunk for one epilogue warp: lane l holds
// row row0 + l, columns col0..col0+31 of the accumulator. The warp stages the
// 32 x 32 chunk (bias and GELU applied) in shared memory (16-byte units XOR
// swizzled by row) and reads it back so that eight lanes cover one row's
// 128-byte segment: each global load / store instruction then touches four
// rows instead of 32. Warp-collective (all 32 lanes, rows past M skipped).
template <int EPI>
__device__ __forceinline__ void gemm_epilogue_chunk_staged(const GemmParams& p, int row0, int lane, int col0,
                                                           const uint32_t (&r)[32], float4* stage) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
  if (p.bias != nullptr) {
    const float4* b4 = reinterpret_cast<const float4*>(p.bias + col0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 b = __ldg(b4 + i);
      const float2 lo = add2(make_float2(v[4 * i + 0], v[4 * i + 1]), make_float2(b.x, b.y));
      const float2 hi = add2(make_float2(v[4 * i + 2], v[4 * i + 3]), make_float2(b.z, b.w));
      v[4 * i + 0] = lo.x;
      v[4 * i + 1] = lo.y;
      v[4 * i + 2] = hi.x;
      v[4 * i + 3] = hi.y;
    }
  }
  if constexpr (EPI == SSAM_EPI_GELU_BF16) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float2 g = gelu_exact2(make_float2(v[2 * i], v[2 * i + 1]));
      v[2 * i] = g.x;
      v[2 * i + 1] = g.y;
    }
  }
  __syncwarp();  // the previous chunk's read-back is done
#pragma unroll
  for (int q = 0; q < 8; ++q)
    stage[lane * 8 + (q ^ (lane & 7))] = make_float4(v[4 * q + 0], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  const int row = row0 + lane;
  const int my_orow = row < p.M ? (p.out_rows != nullptr ? __ldg(p.out_rows + row) : row) : -1;
  __syncwarp();
  const int c4 = lane & 7;
  int orows[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) orows[i] = __shfl_sync(0xffffffffu, my_orow, 4 * i + (lane >> 3));
  if constexpr (EPI == SSAM_EPI_ADD_F32) {
    // all eight residual loads in flight before any store
    float4 o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      o[i] = orows[i] >= 0 ? reinterpret_cast<const float4*>(static_cast<const float*>(p.out) +
                                                             static_cast<int64_t>(orows[i]) * p.ldo + col0)[c4]
                           : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int rr = 4 * i + (lane >> 3);
      const float4 sv = stage[rr * 8 + (c4 ^ (rr & 7))];
      if (orows[i] < 0) continue;
      o[i].x += sv.x;
      o[i].y += sv.y;
      o[i].z += sv.z;
      o[i].w += sv.w;
      reinterpret_cast<float4*>(static_cast<float*>(p.out) + static_cast<int64_t>(orows[i]) * p.ldo + col0)[c4] = o[i];
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int rr = 4 * i + (lane >> 3);
      const float4 sv = stage[rr * 8 + (c4 ^ (rr & 7))];
      if (orows[i] < 0) continue;
      if constexpr (EPI == SSAM_EPI_BF16 || EPI == SSAM_EPI_GELU_BF16) {
        uint2* dst = reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.out) + static_cast<int64_t>(orows[i]) * p.ldo + col0);
        dst[c4] = make_uint2(pack_bf16x2(sv.x, sv.y), pack_bf16x2(sv.z, sv.w));
      } else {
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + static_cast<int64_t>(orows[i]) * p.ldo + col0);
        dst[c4] = sv;
      }
    }
  }
}

// Pair-kernel epilogue through the bulk-copy engine: lane l stages its row's
// 32 outputs in its own shared-memory row and one cp.async.bulk moves them
// (fp32 residual add: cp.reduce.async.bulk .add.f32, done at L2, so the SM never
// waits for the residual). Each lane reuses only its own row, so the only wait is
// for its previous copy to have read it.
template <int EPI>
__device__ __forceinline__ void gemm_epilogue_chunk_bulk(const GemmParams& p, int row, int col0, const uint32_t (&r)[32],
                                                         uint8_t* srow) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
  if (p.bias != nullptr) {
    const float4* b4 = reinterpret_cast<const float4*>(p.bias + col0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 b = __ldg(b4 + i);
      const float2 lo = add2(make_float2(v[4 * i + 0], v[4 * i + 1]), make_float2(b.x, b.y));
      const float2 hi = add2(make_float2(v[4 * i + 2], v[4 * i + 3]), make_float2(b.z, b.w));
      v[4 * i + 0] = lo.x;
      v[4 * i + 1] = lo.y;
      v[4 * i + 2] = hi.x;
      v[4 * i + 3] = hi.y;
    }
  }
  if constexpr (EPI == SSAM_EPI_GELU_BF16) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = gelu_exact(v[i]);
  }
  if constexpr (EPI == SSAM_EPI_F32) {
    if (p.addend != nullptr && row < p.M) {
      const float4* a4 = reinterpret_cast<const float4*>(p.addend + static_cast<int64_t>(row % p.addend_rows) * p.N +
                                                         col0);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 t = __ldg(a4 + i);
        const float2 lo = add2(make_float2(v[4 * i + 0], v[4 * i + 1]), make_float2(t.x, t.y));
        const float2 hi = add2(make_float2(v[4 * i + 2], v[4 * i + 3]), make_float2(t.z, t.w));
        v[4 * i + 0] = lo.x;
        v[4 * i + 1] = lo.y;
        v[4 * i + 2] = hi.x;
        v[4 * i + 3] = hi.y;
      }
    }
  }
  const int orow = row < p.M ? (p.out_rows != nullptr ? __ldg(p.out_rows + row) : row) : -1;
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
  if constexpr (EPI == SSAM_EPI_BF16 || EPI == SSAM_EPI_GELU_BF16) {
    uint4* sp = reinterpret_cast<uint4*>(srow);
#pragma unroll
    for (int q = 0; q < 4; ++q)
      sp[q] = make_uint4(pack_bf16x2(v[8 * q + 0], v[8 * q + 1]), pack_bf16x2(v[8 * q + 2], v[8 * q + 3]),
                         pack_bf16x2(v[8 * q + 4], v[8 * q + 5]), pack_bf16x2(v[8 * q + 6], v[8 * q + 7]));
  } else {
    float4* sp = reinterpret_cast<float4*>(srow);
#pragma unroll
    for (int q = 0; q < 8; ++q) sp[q] = make_float4(v[4 * q + 0], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  }
  fence_proxy_async_smem();
  if (orow >= 0) {
    if constexpr (EPI == SSAM_EPI_BF16 || EPI == SSAM_EPI_GELU_BF16) {
      asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], 64;" ::"l"(
                       static_cast<__nv_bfloat16*>(p.out) + static_cast<int64_t>(orow) * p.ldo + col0),
                   "r"(smem_u32(srow))
                   : "memory");
    } else if constexpr (EPI == SSAM_EPI_F32) {
      asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], 128;" ::"l"(
                       static_cast<float*>(p.out) + static_cast<int64_t>(orow) * p.ldo + col0),
                   "r"(smem_u32(srow))
                   : "memory");
    } else {
      asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], 128;" ::"l"(
                       static_cast<float*>(p.out) + static_cast<int64_t>(orow) * p.ldo + col0),
                   "r"(smem_u32(srow))
                   : "memory");
    }
  }
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kGemmStages * kGemmABytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + kGemmStages * kGemmStageBytes);
  uint64_t* empty_bar = full_bar + kGemmStages;
  uint64_t* tfull_bar = empty_bar + kGemmStages;  // [2]
  uint64_t* tempty_bar = tfull_bar + 2;           // [2]
  uint64_t* drain_bar = tempty_bar + 2;           // [1]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  // epilogue warp w (2..9): 4 KB chunk staging after the 256-byte barrier block
  float4* const epi_stage = reinterpret_cast<float4*>(smem + kGemmStages * kGemmStageBytes + 256) +
                            (threadIdx.x >> 5 >= 2 ? (threadIdx.x >> 5) - 2 : 0) * (kEpiStageBytes / 16);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_tiles = (p.M + kGemmBM - 1) / kGemmBM;
  const int n_tiles = (p.N + kGemmBN - 1) / kGemmBN;
  const int num_tiles = m_tiles * n_tiles;
  const int kblocks = (p.K + kGemmBK - 1) / kGemmBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemmStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], kGemmEpiThreads);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kGemmTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0;      // stages holding a load the MMA warp may not have consumed
      uint32_t issued_parity = 0;    // parity of the latest load per stage
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        const int mb = tile / n_tiles;
        const int nb = tile - mb * n_tiles;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1)) {
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], kGemmStageBytes);
          tma_load_2d(sA + stage * kGemmABytes, &tmA, &full_bar[stage], kb * kGemmBK, mb * kGemmBM);
          tma_load_2d(sB + stage * kGemmBBytes, &tmB, &full_bar[stage], kb * kGemmBK, nb * kGemmBN);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == kGemmStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (*abort_flag) {
        // Drain: every load this thread issued must land before the CTA exits.
        for (int s = 0; s < kGemmStages; ++s)
          if (issued_mask & (1u << s)) mbar_wait(&full_bar[s], (issued_parity >> s) & 1u);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- UMMA issuer ----------------
      const uint32_t idesc = make_idesc_bf16(kGemmBM, kGemmBN, 0, 0);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kGemmBN);
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * kGemmABytes);
          const uint32_t b0 = smem_u32(sB + stage * kGemmBBytes);
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k) {
            const uint64_t ad = make_smem_desc(a0 + k * 32, 16, 1024, kSw128);
            const uint64_t bd = make_smem_desc(b0 + k * 32, 16, 1024, kSw128);
            umma_f16_ss(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == kGemmStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        umma_commit(&tfull_bar[acc]);
      }
      // Make sure every MMA this thread issued has retired before TMEM is freed.
      umma_commit(drain_bar);
      mbar_wait(drain_bar, 0);
    }
  } else {
    // ---------------- epilogue warps 2..9 ----------------
    const int sp = warp & 3;                   // TMEM sub-partition this warp may access
    const int half = (warp - 2) >> 2;          // which 128-column half of the tile
    const int row_in_tile = sp * 32 + lane;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x, ++local) {
      const int mb = tile / n_tiles;
      const int nb = tile - mb * n_tiles;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_phase)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int row = mb * kGemmBM + row_in_tile;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(sp * 32) << 16) + static_cast<uint32_t>(acc * kGemmBN);
#pragma unroll 1
      for (int c = half * (kGemmBN / 2); c < (half + 1) * (kGemmBN / 2); c += 32) {
        const int col0 = nb * kGemmBN + c;
        if (col0 >= p.N) break;  // warp-uniform
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(c), r);
        tmem_ld_wait();
        gemm_epilogue_chunk_staged<EPI>(p, row - lane, lane, col0, r, epi_stage);
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kGemmTmemCols);
}

// ===========================================================================
// 2-SM variant: a cluster of two CTAs computes a 256x256 tile with
// tcgen05.mma.cta_group::2 (M=256, N=256, K=16). CTA r of the pair loads rows
// [r*128, r*128+128) of the A tile and of the B tile (PairCfg<EPI>::kStages stages of
// kSub 64-wide K sub-tiles, 32 KB each) and owns
// accumulator rows [r*128, r*128+128) in its TMEM. Both CTAs' TMA loads
// complete on the leader's (rank 0) full barrier; the leader's commits are
// multicast to both CTAs' empty / tmem-full barriers; both CTAs' epilogue
// threads release the accumulator on the leader's tmem-empty barrier.
// Per SM this halves the B tile held in shared memory and the TMA traffic per
// MMA compared with the 1-SM kernel.
// ===========================================================================
constexpr int kPairBM = 256;  // rows per CTA pair (128 per CTA)
constexpr int kPairRowStride = 144;  // bulk epilogue: per-lane output row staging (128 B + 16 B pad)
constexpr int kPairABytes = 128 * kGemmBK * 2;  // 16 KB
constexpr int kPairBBytes = 128 * kGemmBK * 2;  // 16 KB (half of the 256-column B tile)
constexpr int kPairStageBytes = kPairABytes + kPairBBytes;
// fp32 outputs leave through the bulk-copy engine (per-row staging, 36 KB: five
// 32 KB stages); bf16 outputs through the coalesced chunk staging (32 KB), with
// three 64 KB stages of two K sub-tiles each, so that one barrier round trip of
// the UMMA thread feeds eight MMAs instead of four (batch-64 qkv 2.14 -> 2.08 ms,
// fc1 0.951 -> 0.926 ms in a sustained loop). A sub-tile past K is zero-filled by TMA.
template <int EPI>
struct PairCfg {
  static constexpr bool kBulk = EPI == SSAM_EPI_ADD_F32 || EPI == SSAM_EPI_F32;
  static constexpr int kSub = kBulk ? 1 : 2;  // 64-wide K sub-tiles per stage
  static constexpr int kStages = kBulk ? 5 : 3;
  static constexpr int kStageABytes = kSub * kPairABytes;
  static constexpr int kStageBBytes = kSub * kPairBBytes;
  static constexpr int kStageBytes = kStageABytes + kStageBBytes;
  static constexpr int kEpiBytes = kBulk ? 8 * 32 * kPairRowStride : kEpiStageTotal;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256 + kEpiBytes;
  static_assert((2 * kStages + 5) * 8 + 8 <= 256, "mbarrier block overlaps the epilogue staging");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");
};
static_assert((2 * kGemmStages + 5) * 8 + 8 <= 256, "mbarrier block overlaps the epilogue staging");
static_assert(kGemmSmemBytes <= 227 * 1024, "shared memory per CTA");

template <int EPI, bool CONV = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const GemmParams p) {
  using PC = PairCfg<EPI>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + PC::kStages * PC::kStageABytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + PC::kStages * PC::kStageBytes);
  uint64_t* empty_bar = full_bar + PC::kStages;
  uint64_t* tfull_bar = empty_bar + PC::kStages;  // [2]
  uint64_t* tempty_bar = tfull_bar + 2;           // [2] (used on the leader)
  uint64_t* drain_bar = tempty_bar + 2;           // [1]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  // epilogue warp w (2..9): 4 KB chunk staging after the 256-byte barrier block
  uint8_t* const epi_row = smem + PC::kStages * PC::kStageBytes + 256 +
                          ((threadIdx.x >> 5 >= 2 ? (threadIdx.x >> 5) - 2 : 0) * 32 + (threadIdx.x & 31)) *
                              kPairRowStride;
  float4* const epi_stage = reinterpret_cast<float4*>(smem + PC::kStages * PC::kStageBytes + 256) +
                            (threadIdx.x >> 5 >= 2 ? (threadIdx.x >> 5) - 2 : 0) * (kEpiStageBytes / 16);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int n_pairs = gridDim.x >> 1;
  const int m_tiles = (p.M + kPairBM - 1) / kPairBM;
  const int n_tiles = (p.N + kGemmBN - 1) / kGemmBN;
  const int num_tiles = m_tiles * n_tiles;
  const int kblocks = (p.K + kGemmBK - 1) / kGemmBK;
  const int ksteps = (kblocks + PC::kSub - 1) / PC::kSub;  // stages per tile (a sub-tile past K reads zeros)

  if (threadIdx.x == 0) {
    for (int s = 0; s < PC::kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 2 * kGemmEpiThreads / 32);  // one arrive per epilogue warp of both CTAs
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, kGemmTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised before any cross-CTA use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs) ----------------
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      for (int tile = pair; tile < num_tiles && !*abort_flag; tile += n_pairs) {
        const int mb = tile / n_tiles;
        const int nb = tile - mb * n_tiles;
        for (int ks = 0; ks < ksteps; ++ks) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1)) {
            *abort_flag = 1;
            break;
          }
          const uint32_t bar = mapa_shared(smem_u32(&full_bar[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * PC::kStageBytes);
#pragma unroll
          for (int s = 0; s < PC::kSub; ++s) {
            const int kx = (ks * PC::kSub + s) * kGemmBK;
            if constexpr (CONV) {
              // this CTA's 128 output pixels are 128 / W whole rows of one image; the
              // 64 input channels of tap (ky, kx) are the same rows shifted by (ky - 1,
              // kx - 1), read as one 4-D box (outside the image: zeros, the padding)
              const int m0 = mb * kPairBM + rank * 128;
              const int img = m0 / p.conv_hw;
              const int y0 = (m0 - img * p.conv_hw) / p.conv_w;
              const int cin = p.K / 9;
              const int tap = kx / cin;
              tma_load_4d_pair(sA + stage * PC::kStageABytes + s * kPairABytes, &tmA, bar, kx - tap * cin,
                               tap % 3 - 1, y0 + tap / 3 - 1, img);
            } else {
              tma_load_2d_pair(sA + stage * PC::kStageABytes + s * kPairABytes, &tmA, bar, kx,
                               mb * kPairBM + rank * 128);
            }
            tma_load_2d_pair(sB + stage * PC::kStageBBytes + s * kPairBBytes, &tmB, bar, kx, nb * kGemmBN + rank * 128);
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == PC::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (*abort_flag && leader) {
        for (int s = 0; s < PC::kStages; ++s)
          if (issued_mask & (1u << s)) mbar_wait(&full_bar[s], (issued_parity >> s) & 1u);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- UMMA issuer (leader CTA) ----------------
      const uint32_t idesc = make_idesc_bf16(kPairBM, kGemmBN, 0, 0);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = pair; tile < num_tiles && !*abort_flag; tile += n_pairs, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kGemmBN);
        bool ok = true;
        for (int ks = 0; ks < ksteps; ++ks) {
          if (!mbar_wait(&full_bar[stage], phase)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * PC::kStageABytes);
          const uint32_t b0 = smem_u32(sB + stage * PC::kStageBBytes);
#pragma unroll
          for (int s = 0; s < PC::kSub; ++s)
#pragma unroll
            for (int k = 0; k < kGemmBK / 16; ++k) {
              const uint64_t ad = make_smem_desc(a0 + s * kPairABytes + k * 32, 16, 1024, kSw128);
              const uint64_t bd = make_smem_desc(b0 + s * kPairBBytes + k * 32, 16, 1024, kSw128);
              umma_f16_ss_pair(d_tmem, ad, bd, idesc, (ks | s | k) != 0 ? 1u : 0u);
            }
          umma_commit_pair(&empty_bar[stage], 0x3);
          if (++stage == PC::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        umma_commit_pair(&tfull_bar[acc], 0x3);
      }
      umma_commit_pair(drain_bar, 0x1);
      mbar_wait(drain_bar, 0);
    }
  } else {
    // ---------------- epilogue warps 2..9 (both CTAs) ----------------
    const int sp = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = static_cast<int>(rank) * 128 + sp * 32 + lane;
    const uint32_t tempty0 = mapa_shared(smem_u32(&tempty_bar[0]), 0);
    const uint32_t tempty1 = mapa_shared(smem_u32(&tempty_bar[1]), 0);
    int local = 0;
    for (int tile = pair; tile < num_tiles && !*abort_flag; tile += n_pairs, ++local) {
      const int mb = tile / n_tiles;
      const int nb = tile - mb * n_tiles;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_phase)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int row = mb * kPairBM + row_in_tile;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(sp * 32) << 16) + static_cast<uint32_t>(acc * kGemmBN);
#pragma unroll 1
      for (int c = half * (kGemmBN / 2); c < (half + 1) * (kGemmBN / 2); c += 32) {
        const int col0 = nb * kGemmBN + c;
        if (col0 >= p.N) break;  // warp-uniform
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(c), r);
        tmem_ld_wait();
        if constexpr (PC::kBulk) {
          gemm_epilogue_chunk_bulk<EPI>(p, row, col0, r, epi_row);
        } else {
          gemm_epilogue_chunk_staged<EPI>(p, row - lane, lane, col0, r, epi_stage);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc ? tempty1 : tempty0);  // one release per warp
    }
    if constexpr (PC::kBulk) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // copies done
  }

  tc_fence_before();
  cluster_sync_all();  // the leader's MMAs read the peer's shared memory until here
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, kGemmTmemCols);
}

template <int EPI, bool CONV = false>
static int launch_gemm_pair(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, cudaStream_t stream) {
  static PerDeviceOnce configured;
  const int dev = current_device();
  const int st = configured.run(dev, [] {
    return status_from_cuda(cudaFuncSetAttribute(gemm_bf16_pair_kernel<EPI, CONV>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 PairCfg<EPI>::kSmemBytes));
  });
  if (st != SSAM_OK) return st;
  const int m_tiles = (p.M + kPairBM - 1) / kPairBM;
  const int n_tiles = (p.N + kGemmBN - 1) / kGemmBN;
  const int tiles = m_tiles * n_tiles;
  const int max_pairs = num_sms(dev) / 2;
  const int pairs = tiles < max_pairs ? tiles : max_pairs;
  gemm_bf16_pair_kernel<EPI, CONV><<<2 * pairs, kGemmThreads, PairCfg<EPI>::kSmemBytes, stream>>>(ta, tb, p);
  return cudaGetLastError() == cudaSuccess ? SSAM_OK : SSAM_ERR_CUDA;
}

template <int EPI>
static int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, cudaStream_t stream) {
  static PerDeviceOnce configured;
  const int dev = current_device();
  const int st = configured.run(dev, [] {
    return status_from_cuda(
        cudaFuncSetAttribute(gemm_bf16_tn_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmemBytes));
  });
  if (st != SSAM_OK) return st;
  const int m_tiles = (p.M + kGemmBM - 1) / kGemmBM;
  const int n_tiles = (p.N + kGemmBN - 1) / kGemmBN;
  const int tiles = m_tiles * n_tiles;
  const int grid = tiles < num_sms(dev) ? tiles : num_sms(dev);
  gemm_bf16_tn_kernel<EPI><<<grid, kGemmThreads, kGemmSmemBytes, stream>>>(ta, tb, p);
  return cudaGetLastError() == cudaSuccess ? SSAM_OK : SSAM_ERR_CUDA;
}

// 3x3 / pad 1 convolution of a channels-last bf16 grid as an implicit GEMM on the
// pair kernel: out fp32 [B*H*W, Cout] = im2col3x3(in) . w^T (+ bias), the im2col
// never materialised. Needs whole image rows per CTA tile (W divides 128, H*W a
// multiple of 128) and 64-channel K steps within one tap (Cin a multiple of 64).
int conv3x3_nhwc(const void* in, int B, int H, int W, int Cin, const void* w, int Cout, const float* bias, void* out,
                 cudaStream_t stream) {
  if (in == nullptr || w == nullptr || out == nullptr || B <= 0 || H <= 0 || W <= 0 || Cin <= 0 || Cout <= 0)
    return SSAM_ERR_INVALID;
  if (Cin % kGemmBK != 0 || Cout % 32 != 0 || W > 128 || 128 % W != 0 || (static_cast<int64_t>(H) * W) % 128 != 0)
    return SSAM_ERR_UNSUPPORTED;
  const int64_t M64 = static_cast<int64_t>(B) * H * W, K64 = 9 * static_cast<int64_t>(Cin);
  if (M64 > INT32_MAX || K64 > INT32_MAX) return SSAM_ERR_UNSUPPORTED;
  if (!aligned16(in) || !aligned16(w) || !aligned16(out) || (bias != nullptr && !aligned16(bias))) return SSAM_ERR_ALIGN;
  CUtensorMap ta, tb;
  int st = make_tmap_nhwc_bf16(&ta, in, B, H, W, Cin, kGemmBK, static_cast<uint32_t>(W), static_cast<uint32_t>(128 / W));
  if (st != SSAM_OK) return st;
  st = make_tmap_2d_bf16(&tb, w, static_cast<uint64_t>(Cout), static_cast<uint64_t>(K64), static_cast<uint64_t>(K64),
                         kGemmBK, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != SSAM_OK) return st;
  GemmParams p{static_cast<int>(M64), Cout, static_cast<int>(K64), bias, out, Cout, nullptr, W, H * W, nullptr, 0};
  return launch_gemm_pair<SSAM_EPI_F32, true>(ta, tb, p, stream);
}

// out fp32 [M, N] = A . B^T + bias + addend[r % addend_rows] (the patch embedding
// plus its positional embedding, written once): the pair kernel's fp32 epilogue.
int gemm_bf16_addend(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K, const float* bias,
                     const float* addend, int addend_rows, float* out, cudaStream_t stream) {
  if (A == nullptr || B == nullptr || out == nullptr || addend == nullptr || addend_rows <= 0) return SSAM_ERR_INVALID;
  if (M <= 0 || N <= 0 || K <= 0 || lda < K || ldb < K) return SSAM_ERR_INVALID;
  if (N % 32 != 0 || K % 8 != 0 || M < kPairBM) return SSAM_ERR_UNSUPPORTED;
  if ((lda % 8) || (ldb % 8) || !aligned16(A) || !aligned16(B) || !aligned16(out) || !aligned16(addend) ||
      (bias != nullptr && !aligned16(bias)))
    return SSAM_ERR_ALIGN;
  CUtensorMap ta, tb;
  int st = make_tmap_2d_bf16(&ta, A, static_cast<uint64_t>(M), static_cast<uint64_t>(K), static_cast<uint64_t>(lda),
                             kGemmBK, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != SSAM_OK) return st;
  st = make_tmap_2d_bf16(&tb, B, static_cast<uint64_t>(N), static_cast<uint64_t>(K), static_cast<uint64_t>(ldb), kGemmBK,
                         128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != SSAM_OK) return st;
  GemmParams p{M, N, K, bias, out, N, nullptr, 0, 0, addend, addend_rows};
  return launch_gemm_pair<SSAM_EPI_F32>(ta, tb, p, stream);
}

int gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K, const float* bias,
              int epilogue, void* out, int64_t ldo, const int32_t* out_rows, cudaStream_t stream) {
  if (A == nullptr || B == nullptr || out == nullptr) return SSAM_ERR_INVALID;
  if (M < 0 || N <= 0 || K <= 0) return SSAM_ERR_INVALID;
  if (M == 0) return SSAM_OK;
  if (N % 32 != 0 || K % 8 != 0) return SSAM_ERR_UNSUPPORTED;
  if (lda < K || ldb < K || ldo < N) return SSAM_ERR_INVALID;
  if ((lda % 8) || (ldb % 8) || !aligned16(A) || !aligned16(B) || !aligned16(out)) return SSAM_ERR_ALIGN;
  if (bias != nullptr && !aligned16(bias)) return SSAM_ERR_ALIGN;
  if (epilogue == SSAM_EPI_ADD_F32 || epilogue == SSAM_EPI_F32) {
    if (ldo % 4) return SSAM_ERR_ALIGN;
  } else if (epilogue == SSAM_EPI_BF16 || epilogue == SSAM_EPI_GELU_BF16) {
    if (ldo % 8) return SSAM_ERR_ALIGN;
  } else {
    return SSAM_ERR_INVALID;
  }
  CUtensorMap ta, tb;
  int st = make_tmap_2d_bf16(&ta, A, static_cast<uint64_t>(M), static_cast<uint64_t>(K), static_cast<uint64_t>(lda),
                             kGemmBK, kGemmBM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != SSAM_OK) return st;
  st = make_tmap_2d_bf16(&tb, B, static_cast<uint64_t>(N), static_cast<uint64_t>(K), static_cast<uint64_t>(ldb), kGemmBK,
                         kGemmBN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != SSAM_OK) return st;
  GemmParams p{M, N, K, bias, out, ldo, out_rows, 0, 0, nullptr, 0};
  const int pair_tiles = ((M + kPairBM - 1) / kPairBM) * ((N + kGemmBN - 1) / kGemmBN);
  if (M >= kPairBM && pair_tiles >= 64) {
    // 2-SM kernel: 128-row boxes per CTA for both operands
    st = make_tmap_2d_bf16(&ta, A, static_cast<uint64_t>(M), static_cast<uint64_t>(K), static_cast<uint64_t>(lda),
                           kGemmBK, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != SSAM_OK) return st;
    st = make_tmap_2d_bf16(&tb, B, static_cast<uint64_t>(N), static_cast<uint64_t>(K), static_cast<uint64_t>(ldb),
                           kGemmBK, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != SSAM_OK) return st;
    switch (epilogue) {
      case SSAM_EPI_BF16:
        return launch_gemm_pair<SSAM_EPI_BF16>(ta, tb, p, stream);
      case SSAM_EPI_GELU_BF16:
        return launch_gemm_pair<SSAM_EPI_GELU_BF16>(ta, tb, p, stream);
      case SSAM_EPI_F32:
        return launch_gemm_pair<SSAM_EPI_F32>(ta, tb, p, stream);
      default:
        return launch_gemm_pair<SSAM_EPI_ADD_F32>(ta, tb, p, stream);
    }
  }
  switch (epilogue) {
    case SSAM_EPI_BF16:
      return launch_gemm<SSAM_EPI_BF16>(ta, tb, p, stream);
    case SSAM_EPI_GELU_BF16:
      return launch_gemm<SSAM_EPI_GELU_BF16>(ta, tb, p, stream);
    case SSAM_EPI_F32:
      return launch_gemm<SSAM_EPI_F32>(ta, tb, p, stream);
    default:
      return launch_gemm<SSAM_EPI_ADD_F32>(ta, tb, p, stream);
  }
}

}  // namespace ssam
