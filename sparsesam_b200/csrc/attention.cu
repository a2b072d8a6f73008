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
// Persistent, warp-specialised CTA (one per SM), 192 threads:
//   warps 0-3  softmax warpgroup: thread i owns query row i of the current
//              128-query tile; extracts its rel-pos bias windows, runs the online
//              softmax out of TMEM, writes P (bf16) and does the epilogue;
//   warp 4     loader: cp.async gathers of the permuted Q / K / V rows (64-key
//              blocks, 3 stages) and the rel-pos tables, signalled through
//              mbarriers (cp.async.mbarrier.arrive);
//   warp 5     UMMA issuer: P_H = Q Th^T and P_W = Q Tw^T for the next tile,
//              S(j+1) = Q K^T issued ahead of softmax(j) into a second TMEM
//              buffer, O += P V accumulated in TMEM (V as an MN-major operand).
// O is rescaled lazily: only when a row maximum grows by more than 2^8 is the
// TMEM row read, scaled and written back; otherwise the stale maximum is kept
// (probabilities stay below 2^8 and the final 1/l normalisation is consistent).
// Every wait is bounded; on timeout the CTA raises SSAM_ERR_TIMEOUT and unwinds.
#include <cuda_fp16.h>

#include "common.cuh"
#include "host_util.h"

namespace ssam {

constexpr int kAttnBM = 128;  // queries per tile
constexpr int kAttnBN = 64;   // keys per block (the reference's 64-token mask granularity)
constexpr int kAttnStages = 3;
constexpr int kAttnThreads = 192;
constexpr int kAttnTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Arrive on `bar` once every cp.async issued so far by this thread has landed.
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory geometry of a D-wide operand tile with R rows: channels 0..63 in
// a 128B-swizzled region (R x 128 B), channels 64..79 (D == 80) in a 32B-swizzled
// region (R x 32 B) right after it.
template <int D>
struct TileGeom {
  static constexpr int kChunks = D / 8;  // 16-byte chunks per row
  static constexpr bool kTail = D > 64;
  static __host__ __device__ constexpr int bytes(int rows) { return rows * 128 + (kTail ? rows * 32 : 0); }
};

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

__host__ __device__ constexpr int align1k(int v) { return (v + 1023) & ~1023; }

// Instruction descriptor for kind::f16 with fp16 A/B (formats 0), fp32 accumulator.
__host__ __device__ constexpr uint32_t make_idesc_f16(uint32_t M, uint32_t N) {
  return (1u << 4) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

// Two specialisations: SMALL for windowed grids (win <= 16, 32-row tables) and
// the global 64x64 grid. SMALL tiles have one or two key blocks, so they get a
// deeper S pipeline and double-buffered O / P_H / A_bias to remove tile bubbles.
template <int D, bool SMALL>
struct AttnCfg {
  static constexpr int kS = SMALL ? 3 : 2;        // S buffers in TMEM (QK^T lookahead)
  static constexpr int kO = SMALL ? 2 : 1;        // O accumulators in TMEM
  static constexpr int kPH = SMALL ? 2 : 1;       // P_H/P_W TMEM buffers
  static constexpr int kAB = SMALL ? 2 : 1;       // A_bias shared-memory buffers
  static constexpr int kStages = SMALL ? 3 : 2;   // K / V / one-hot stages
  static constexpr int kBW = SMALL ? 16 : 64;     // bias columns per table (>= win)
  static constexpr int kNT = SMALL ? 32 : 128;    // table rows padded to the MMA N
  static constexpr int kTmO = kS * kAttnBN;       // TMEM column of O[0]
  static constexpr int kTmPH = SMALL ? kTmO + kO * D : 256;
  static constexpr int kOHBytes = 2 * kAttnBN * kBW * 2;  // one-hot H | W regions per stage
  static constexpr int kABBytes = 2 * kAttnBM * kBW * 2;  // A_bias H | W regions
  static_assert(kTmPH + kPH * 2 * kNT <= kAttnTmemCols, "TMEM plan exceeds 512 columns");
};

// Byte offset of element (row r, column k) of a K-major fp16 bias operand region
// (128B swizzle for 64-wide rows, 32B swizzle for 16-wide rows).
template <bool SMALL>
__device__ __forceinline__ uint32_t bias_off(int r, int k) {
  if constexpr (SMALL) return r * 32 + ((((k >> 3) ^ ((r >> 2) & 1))) << 4) + (k & 7) * 2;
  return r * 128 + ((((k >> 3) ^ (r & 7))) << 4) + (k & 7) * 2;
}

// Shared-memory plan (bytes from a 1 KB-aligned base).
template <int D, bool SMALL>
struct AttnLayout {
  using C = AttnCfg<D, SMALL>;
  using TG = TileGeom<D>;
  static constexpr int kStage = 2 * TG::bytes(kAttnBN) + C::kOHBytes;  // K | V | one-hot
  int th, tw, q, kv, p, ab, kinfo, tok, bars, total;
  __host__ __device__ AttnLayout(int win) {
    th = 0;
    tw = align1k(th + TG::bytes(C::kNT));
    q = align1k(tw + TG::bytes(C::kNT));               // [2] x bytes(128)
    kv = q + 2 * TG::bytes(kAttnBM);                   // [stages] x kStage
    p = kv + C::kStages * kStage;                      // [2] x 128 x 128 B
    ab = p + 2 * kAttnBM * 128;                        // [kAB] x kABBytes
    kinfo = ab + C::kAB * C::kABBytes;                 // int [stages][64]
    tok = kinfo + C::kStages * kAttnBN * 4;            // int [2][128]
    bars = (tok + 2 * kAttnBM * 4 + 7) & ~7;           // mbarriers
    total = bars + 32 * 8 + 16 + 1024;                 // + alignment slack
    (void)win;
  }
};

struct AttnParams {
  const __nv_bfloat16* qkv;
  int64_t ld_qkv;
  int heads, win, N, C;
  const __nv_bfloat16* th;  // (2win-1, D)
  const __nv_bfloat16* tw;
  const int32_t* perm;
  int n_init, with_diag;
  float scale_log2;  // scale * log2(e)
  float inv_scale;   // 1 / scale
  __nv_bfloat16* out;
  int64_t ld_out;
  int n_tiles;  // 128-query tiles per row
  int total_tiles;
};

// Key blocks of one tile: the keep bar [0, nk), then the diagonal blocks of the
// two 64-query m-blocks of the tile that lie outside the bar.
struct TileBlocks {
  int nk, n, d0, d1;
  __device__ TileBlocks() : nk(0), n(0), d0(-1), d1(-1) {}
  __device__ TileBlocks(const AttnParams& a, int qtile) {
    const int nblk = (a.N + kAttnBN - 1) / kAttnBN;
    nk = a.n_init < nblk ? a.n_init : nblk;
    n = nk;
    d0 = d1 = -1;
    if (a.with_diag) {
      for (int mb = 2 * qtile; mb < 2 * qtile + 2; ++mb) {
        if (mb < nblk && mb >= nk) {
          if (n == nk) d0 = mb; else d1 = mb;
          ++n;
        }
      }
    }
  }
  __device__ int at(int i) const { return i < nk ? i : (i == nk ? d0 : d1); }
};

// Walks the flat (tile, key block) sequence of one persistent CTA.
struct BlockCursor {
  int tile, lt, j, g;
  bool done;
  TileBlocks tb;
  __device__ void start(const AttnParams& a) {
    tile = blockIdx.x;
    lt = 0;
    j = 0;
    g = 0;
    done = tile >= a.total_tiles;
    if (!done) tb = TileBlocks(a, tile % a.n_tiles);
  }
  __device__ void advance(const AttnParams& a) {
    ++j;
    ++g;
    if (j >= tb.n) {
      j = 0;
      ++lt;
      tile += gridDim.x;
      done = tile >= a.total_tiles;
      if (!done) tb = TileBlocks(a, tile % a.n_tiles);
    }
  }
};

// mbarrier indices
enum {
  kBarTab = 0,
  kBarQFull = 1,     // [2]
  kBarQEmpty = 3,    // [2]
  kBarKVFull = 5,    // [3]
  kBarKVEmpty = 8,   // [3]
  kBarPHFull = 11,   // [2]
  kBarPHFree = 13,   // [2]
  kBarABFull = 15,   // [2]
  kBarSFull = 17,    // [3]
  kBarSFree = 20,    // [3]
  kBarPFull = 23,    // [2]
  kBarODone = 25,    // [2]
  kBarOFree = 27,    // [2]
  kBarDrain = 29,
  kNumBars = 30
};

template <int D, bool SMALL>
__global__ void __launch_bounds__(kAttnThreads, 1) sparse_attn_kernel(const AttnParams a) {
  using TG = TileGeom<D>;
  using C = AttnCfg<D, SMALL>;
  using LAY = AttnLayout<D, SMALL>;
  const LAY L(a.win);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  int* s_kinfo = reinterpret_cast<int*>(smem + L.kinfo);
  int* s_tok = reinterpret_cast<int*>(smem + L.tok);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int N = a.N, win = a.win;

  if (tid == 0) {
    mbar_init(&bars[kBarTab], 64);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[kBarQFull + i], 64);
      mbar_init(&bars[kBarQEmpty + i], 1);
      mbar_init(&bars[kBarPHFull + i], 1);
      mbar_init(&bars[kBarPHFree + i], 128);
      mbar_init(&bars[kBarABFull + i], 128);
      mbar_init(&bars[kBarPFull + i], 128);
      mbar_init(&bars[kBarODone + i], 1);
      mbar_init(&bars[kBarOFree + i], 128);
    }
    for (int s = 0; s < 3; ++s) {
      mbar_init(&bars[kBarKVFull + s], 64);
      mbar_init(&bars[kBarKVEmpty + s], 1);
      mbar_init(&bars[kBarSFull + s], 1);
      mbar_init(&bars[kBarSFree + s], 128);
    }
    mbar_init(&bars[kBarDrain], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_holder, kAttnTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  auto wait_or_abort = [&](int bar, uint32_t parity) -> bool {
    if (*abort_flag) return false;
    if (!mbar_wait(&bars[bar], parity)) {
      *abort_flag = 1;
      return false;
    }
    return true;
  };
  auto tile_exists = [&](int lt_) { return static_cast<int>(blockIdx.x) + lt_ * static_cast<int>(gridDim.x) < a.total_tiles; };

  if (warp == 4) {
    // =========================== loader warp ===========================
    // Lane-per-row copies: a lane moves whole rows (kChunks x 16 B), so every
    // cp.async address is a row base plus a compile-time chunk offset. The
    // permutation indices of the next key block are fetched one block ahead.
    // Order: Q(0), then per tile t: Q(t+1), K/V(t, blocks) — the UMMA warp
    // computes P_H(t+1) from Q(t+1) while tile t runs.
    auto copy_row = [&](uint32_t region, int rows, int r, const __nv_bfloat16* src) {
      const uint32_t bytes = src != nullptr ? 16u : 0u;
      const uint8_t* s0 = reinterpret_cast<const uint8_t*>(src != nullptr ? src : a.qkv);
#pragma unroll
      for (int c = 0; c < TG::kChunks; ++c)
        cp_async16(tile_chunk_addr<D>(region, rows, r, c), s0 + (src != nullptr ? c * 16 : 0), bytes);
    };
    // one-hot regions start at zero; kinfo starts at -1 (nothing to clear)
    for (int s = 0; s < C::kStages; ++s) {
      uint4* oh = reinterpret_cast<uint4*>(smem + L.kv + s * LAY::kStage + 2 * TG::bytes(kAttnBN));
      for (int i = lane; i < C::kOHBytes / 16; i += 32) oh[i] = make_uint4(0u, 0u, 0u, 0u);
      for (int r = lane; r < kAttnBN; r += 32) s_kinfo[s * kAttnBN + r] = -1;
    }
    __syncwarp();
    // rel-pos tables, once per CTA
    const uint32_t sTh = sb + L.th, sTw = sb + L.tw;
    const int trows = 2 * win - 1;
    for (int r = lane; r < C::kNT; r += 32) {
      copy_row(sTh, C::kNT, r, r < trows ? a.th + r * D : nullptr);
      copy_row(sTw, C::kNT, r, r < trows ? a.tw + r * D : nullptr);
    }
    mbar_arrive(&bars[kBarTab]);
    cp_async_arrive_noinc(&bars[kBarTab]);

    auto load_q = [&](int lt_) -> bool {
      const int tile = blockIdx.x + lt_ * gridDim.x;
      const int row = tile / a.n_tiles, qtile = tile - row * a.n_tiles;
      const int seq = row / a.heads, head = row - seq * a.heads;
      const int32_t* perm = a.perm + static_cast<int64_t>(row) * N;
      const __nv_bfloat16* q_base = a.qkv + static_cast<int64_t>(seq) * N * a.ld_qkv + head * D;
      int qt[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int p = qtile * kAttnBM + lane + 32 * i;
        qt[i] = p < N ? __ldg(perm + p) : -1;
      }
      const int qb = lt_ & 1;
      if (!wait_or_abort(kBarQEmpty + qb, ((lt_ >> 1) & 1) ^ 1)) return false;
      const uint32_t sQ = sb + L.q + qb * TG::bytes(kAttnBM);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = lane + 32 * i;
        s_tok[qb * kAttnBM + r] = qt[i];
        copy_row(sQ, kAttnBM, r, qt[i] >= 0 ? q_base + static_cast<int64_t>(qt[i]) * a.ld_qkv : nullptr);
      }
      mbar_arrive(&bars[kBarQFull + qb]);
      cp_async_arrive_noinc(&bars[kBarQFull + qb]);
      return true;
    };

    int g = 0;
    bool ok = tile_exists(0) ? load_q(0) : true;
    for (int lt = 0; ok && tile_exists(lt) && !*abort_flag; ++lt) {
      if (tile_exists(lt + 1) && !(ok = load_q(lt + 1))) break;
      const int tile = blockIdx.x + lt * gridDim.x;
      const int row = tile / a.n_tiles, qtile = tile - row * a.n_tiles;
      const int seq = row / a.heads, head = row - seq * a.heads;
      const int32_t* perm = a.perm + static_cast<int64_t>(row) * N;
      const __nv_bfloat16* k_base = a.qkv + static_cast<int64_t>(seq) * N * a.ld_qkv + a.C + head * D;
      const TileBlocks tb(a, qtile);
      int nt0 = -1, nt1 = -1;
      if (tb.n > 0) {
        const int kp = tb.at(0) * kAttnBN + lane;
        nt0 = kp < N ? __ldg(perm + kp) : -1;
        nt1 = kp + 32 < N ? __ldg(perm + kp + 32) : -1;
      }
      for (int j = 0; j < tb.n; ++j, ++g) {
        const int t0 = nt0, t1 = nt1;
        if (j + 1 < tb.n) {  // prefetch the next block's tokens
          const int kp = tb.at(j + 1) * kAttnBN + lane;
          nt0 = kp < N ? __ldg(perm + kp) : -1;
          nt1 = kp + 32 < N ? __ldg(perm + kp + 32) : -1;
        }
        const int stage = g % C::kStages;
        if (!(ok = wait_or_abort(kBarKVEmpty + stage, ((g / C::kStages) & 1) ^ 1))) break;
        int* kinfo = s_kinfo + stage * kAttnBN;
        const uint32_t sK = sb + L.kv + stage * LAY::kStage;
        const uint32_t sV = sK + TG::bytes(kAttnBN);
        uint8_t* oh_h = smem + L.kv + stage * LAY::kStage + 2 * TG::bytes(kAttnBN);
        uint8_t* oh_w = oh_h + kAttnBN * C::kBW * 2;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int r = lane + 32 * i;
          const int t = i == 0 ? t0 : t1;
          int info = -1;
          if (t >= 0) {
            const int kh = t / win;
            info = kh | ((t - kh * win) << 16);
          }
          const int old = kinfo[r];
          if (old >= 0) {  // clear the previous one-hot entries of this row
            *reinterpret_cast<uint16_t*>(oh_h + bias_off<SMALL>(r, old & 0xffff)) = 0;
            *reinterpret_cast<uint16_t*>(oh_w + bias_off<SMALL>(r, old >> 16)) = 0;
          }
          if (info >= 0) {
            *reinterpret_cast<uint16_t*>(oh_h + bias_off<SMALL>(r, info & 0xffff)) = 0x3C00;  // fp16 1.0
            *reinterpret_cast<uint16_t*>(oh_w + bias_off<SMALL>(r, info >> 16)) = 0x3C00;
          }
          kinfo[r] = info;
          const __nv_bfloat16* krow = t >= 0 ? k_base + static_cast<int64_t>(t) * a.ld_qkv : nullptr;
          copy_row(sK, kAttnBN, r, krow);
          copy_row(sV, kAttnBN, r, krow != nullptr ? krow + a.C : nullptr);
        }
        fence_proxy_async_smem();  // one-hot rows (generic stores) -> UMMA reads
        mbar_arrive(&bars[kBarKVFull + stage]);
        cp_async_arrive_noinc(&bars[kBarKVFull + stage]);
      }
    }
    cp_async_wait_all();
  } else if (warp == 5) {
    // =========================== UMMA issuer ===========================
    if (lane == 0) {
      const uint32_t sTh = sb + L.th, sTw = sb + L.tw;
      const uint32_t idesc_t = make_idesc_bf16(kAttnBM, C::kNT, 0, 0);
      const uint32_t idesc_s = make_idesc_bf16(kAttnBM, kAttnBN, 0, 0);
      const uint32_t idesc_b = make_idesc_f16(kAttnBM, kAttnBN);
      const uint32_t idesc_o64 = make_idesc_bf16(kAttnBM, 64, 0, 1);
      const uint32_t idesc_o16 = make_idesc_bf16(kAttnBM, 16, 0, 1);
      bool ok = wait_or_abort(kBarTab, 0);
      fence_proxy_async_smem();

      auto issue_ph = [&](int lt_) -> bool {  // P_H / P_W of tile lt_
        const int qb = lt_ & 1, pb = lt_ % C::kPH;
        if (!wait_or_abort(kBarQFull + qb, (lt_ >> 1) & 1)) return false;
        if (!wait_or_abort(kBarPHFree + pb, ((lt_ / C::kPH) & 1) ^ 1)) return false;
        tc_fence_after();
        fence_proxy_async_smem();
        const uint32_t sQ = sb + L.q + qb * TG::bytes(kAttnBM);
        const uint32_t tPH = tmem + C::kTmPH + pb * 2 * C::kNT;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          umma_f16_ss(tPH, kmajor_desc<D>(sQ, kAttnBM, ks), kmajor_desc<D>(sTh, C::kNT, ks), idesc_t, ks > 0);
          umma_f16_ss(tPH + C::kNT, kmajor_desc<D>(sQ, kAttnBM, ks), kmajor_desc<D>(sTw, C::kNT, ks), idesc_t,
                      ks > 0);
        }
        umma_commit(&bars[kBarPHFull + pb]);
        return true;
      };
      auto issue_qk = [&](const BlockCursor& c) -> bool {
        if (c.j == 0) {
          if constexpr (SMALL) {
            if (tile_exists(c.lt + 1) && !issue_ph(c.lt + 1)) return false;
          } else {
            if (!issue_ph(c.lt)) return false;
          }
          if (!wait_or_abort(kBarABFull + c.lt % C::kAB, (c.lt / C::kAB) & 1)) return false;
        }
        const int st = c.g % C::kStages, sbuf = c.g % C::kS;
        if (!wait_or_abort(kBarKVFull + st, (c.g / C::kStages) & 1)) return false;
        if (!wait_or_abort(kBarSFree + sbuf, ((c.g / C::kS) & 1) ^ 1)) return false;
        tc_fence_after();
        fence_proxy_async_smem();
        const uint32_t sQ = sb + L.q + (c.lt & 1) * TG::bytes(kAttnBM);
        const uint32_t sK = sb + L.kv + st * LAY::kStage;
        const uint32_t sOH = sK + 2 * TG::bytes(kAttnBN);
        const uint32_t sAB = sb + L.ab + (c.lt % C::kAB) * C::kABBytes;
        const uint32_t tS = tmem + sbuf * kAttnBN;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks)
          umma_f16_ss(tS, kmajor_desc<D>(sQ, kAttnBM, ks), kmajor_desc<D>(sK, kAttnBN, ks), idesc_s, ks > 0);
        // + A_bias . onehot^T  (relH / scale at kh, relW / scale at kw)
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          const uint32_t ab = sAB + part * kAttnBM * C::kBW * 2;
          const uint32_t oh = sOH + part * kAttnBN * C::kBW * 2;
          if constexpr (SMALL) {
            umma_f16_ss(tS, make_smem_desc(ab, 16, 256, kSw32), make_smem_desc(oh, 16, 256, kSw32), idesc_b, 1u);
          } else {
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              umma_f16_ss(tS, make_smem_desc(ab + ks * 32, 16, 1024, kSw128),
                          make_smem_desc(oh + ks * 32, 16, 1024, kSw128), idesc_b, 1u);
          }
        }
        umma_commit(&bars[kBarSFull + sbuf]);
        if (c.j == c.tb.n - 1) umma_commit(&bars[kBarQEmpty + (c.lt & 1)]);
        return true;
      };
      auto issue_pv = [&](const BlockCursor& c) -> bool {
        if (!wait_or_abort(kBarPFull + (c.g & 1), (c.g >> 1) & 1)) return false;
        const int ob = c.lt % C::kO;
        if (c.j == 0 && !wait_or_abort(kBarOFree + ob, ((c.lt / C::kO) & 1) ^ 1)) return false;
        tc_fence_after();
        fence_proxy_async_smem();
        const int st = c.g % C::kStages;
        const uint32_t sP = sb + L.p + (c.g & 1) * (kAttnBM * 128);
        const uint32_t sV = sb + L.kv + st * LAY::kStage + TG::bytes(kAttnBN);
        const uint32_t tO = tmem + C::kTmO + ob * D;
#pragma unroll
        for (int ks = 0; ks < kAttnBN / 16; ++ks) {
          const uint64_t pd = make_smem_desc(sP + ks * 32, 16, 1024, kSw128);
          const uint32_t acc = (c.j > 0 || ks > 0) ? 1u : 0u;
          umma_f16_ss(tO, pd, make_smem_desc(sV + ks * 2048, 8192, 1024, kSw128), idesc_o64, acc);
          if constexpr (TG::kTail)
            umma_f16_ss(tO + 64, pd, make_smem_desc(sV + kAttnBN * 128 + ks * 512, 4096, 256, kSw32), idesc_o16, acc);
        }
        umma_commit(&bars[kBarODone + (c.g & 1)]);
        umma_commit(&bars[kBarKVEmpty + st]);
        return true;
      };

      if (ok && SMALL && tile_exists(0)) ok = issue_ph(0);
      BlockCursor cq, cp;
      cq.start(a);
      cp.start(a);
      while (ok && !cp.done) {
        while (ok && !cq.done && cq.g < cp.g + C::kS) {
          ok = issue_qk(cq);
          cq.advance(a);
        }
        if (!ok) break;
        ok = issue_pv(cp);
        cp.advance(a);
      }
      umma_commit(&bars[kBarDrain]);
      mbar_wait(&bars[kBarDrain], 0);
    }
  } else {
    // ======================== softmax warpgroup ========================
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(warp * 32) << 16);

    // rel-pos bias of tile lt_ -> A_bias[lt_ % kAB] row tid (fp16, relH/scale at column j)
    auto extract_bias = [&](int lt_, int& tok_out) -> bool {
      const int qb = lt_ & 1, pb = lt_ % C::kPH;
      if (!wait_or_abort(kBarQFull + qb, (lt_ >> 1) & 1)) return false;
      const int t = s_tok[qb * kAttnBM + tid];
      tok_out = t;
      const int qh = t >= 0 ? t / win : 0;
      const int qw = t >= 0 ? t - qh * win : 0;
      if (!wait_or_abort(kBarPHFull + pb, (lt_ / C::kPH) & 1)) return false;
      tc_fence_after();
      uint8_t* ab_h = smem + L.ab + (lt_ % C::kAB) * C::kABBytes;
      uint8_t* ab_w = ab_h + kAttnBM * C::kBW * 2;
      const uint32_t tPH = t_lane + C::kTmPH + pb * 2 * C::kNT;
      for (int c0 = 0; c0 < C::kNT; c0 += 32) {
        uint32_t rh[32], rw[32];
        tmem_ld_32x32b_x32(tPH + c0, rh);
        tmem_ld_32x32b_x32(tPH + C::kNT + c0, rw);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int jh = qh + win - 1 - (c0 + j);
          if (jh >= 0 && jh < win)
            *reinterpret_cast<__half*>(ab_h + bias_off<SMALL>(tid, jh)) =
                __float2half_rn(__uint_as_float(rh[j]) * a.inv_scale);
          const int jw = qw + win - 1 - (c0 + j);
          if (jw >= 0 && jw < win)
            *reinterpret_cast<__half*>(ab_w + bias_off<SMALL>(tid, jw)) =
                __float2half_rn(__uint_as_float(rw[j]) * a.inv_scale);
        }
      }
      for (int j = win; j < C::kBW; ++j) {  // padding columns must not hold NaN/Inf
        *reinterpret_cast<__half*>(ab_h + bias_off<SMALL>(tid, j)) = __float2half_rn(0.f);
        *reinterpret_cast<__half*>(ab_w + bias_off<SMALL>(tid, j)) = __float2half_rn(0.f);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars[kBarABFull + lt_ % C::kAB]);
      mbar_arrive(&bars[kBarPHFree + pb]);
      return true;
    };
    // O / l of tile lt_, stored at the raster token (inverse permutation and head merge)
    auto epilogue = [&](int lt_, int g_last, int tok, float l) -> bool {
      const int tile = blockIdx.x + lt_ * gridDim.x;
      const int row = tile / a.n_tiles;
      const int seq = row / a.heads, head = row - seq * a.heads;
      if (g_last >= 0 && !wait_or_abort(kBarODone + (g_last & 1), (g_last >> 1) & 1)) return false;
      tc_fence_after();
      const float inv_l = l > 0.f ? 1.f / l : 0.f;
      uint4* dst = tok >= 0 ? reinterpret_cast<uint4*>(a.out + (static_cast<int64_t>(seq) * N + tok) * a.ld_out +
                                                       head * D)
                            : nullptr;
      const uint32_t tO = t_lane + C::kTmO + (lt_ % C::kO) * D;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 16) {
        uint32_t r16[16];
        tmem_ld_32x32b_x16(tO + c0, r16);
        tmem_ld_wait();
        if (dst != nullptr) {
          float o[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) o[e] = g_last >= 0 ? __uint_as_float(r16[e]) * inv_l : 0.f;
          dst[c0 / 8] = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                                   pack_bf16x2(o[6], o[7]));
          dst[c0 / 8 + 1] = make_uint4(pack_bf16x2(o[8], o[9]), pack_bf16x2(o[10], o[11]),
                                       pack_bf16x2(o[12], o[13]), pack_bf16x2(o[14], o[15]));
        }
      }
      tc_fence_before();
      mbar_arrive(&bars[kBarOFree + lt_ % C::kO]);
      return true;
    };

    bool ok = true;
    int tok_cur = -1, tok_next = -1;
    if (tile_exists(0)) ok = extract_bias(0, tok_cur);
    int pend_lt = -1, pend_g = -1, pend_tok = -1;  // deferred epilogue
    float pend_l = 0.f;
    int g = 0;
    for (int lt = 0; ok && tile_exists(lt); ++lt) {
      const int tile = blockIdx.x + lt * gridDim.x;
      const int qtile = tile % a.n_tiles;
      const TileBlocks tb(a, qtile);
      const int my_mb = 2 * qtile + (tid >= 64 ? 1 : 0);
      const uint32_t tO = t_lane + C::kTmO + (lt % C::kO) * D;
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; j < tb.n; ++j, ++g) {
        const int st = g % C::kStages, sbuf = g % C::kS;
        const int kb = tb.at(j);
        if (!(ok = wait_or_abort(kBarKVFull + st, (g / C::kStages) & 1))) break;  // kinfo visibility
        if (!(ok = wait_or_abort(kBarSFull + sbuf, (g / C::kS) & 1))) break;
        tc_fence_after();
        uint32_t s[64];
        {
          uint32_t (&s0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[0]);
          uint32_t (&s1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[32]);
          tmem_ld_32x32b_x32(t_lane + sbuf * kAttnBN, s0);
          tmem_ld_32x32b_x32(t_lane + sbuf * kAttnBN + 32, s1);
          tmem_ld_wait();
        }
        tc_fence_before();
        mbar_arrive(&bars[kBarSFree + sbuf]);

        const bool full = kb < tb.nk && (kb + 1) * kAttnBN <= N;
        float mx = -INFINITY;
        if (full) {
#pragma unroll
          for (int jj = 0; jj < 64; ++jj) {
            const float x = __uint_as_float(s[jj]) * a.scale_log2;
            s[jj] = __float_as_uint(x);
            mx = fmaxf(mx, x);
          }
        } else {
          const int* kinfo = s_kinfo + st * kAttnBN;
          const bool row_on = (kb < tb.nk) || (kb == my_mb);
#pragma unroll
          for (int jj = 0; jj < 64; ++jj) {
            const float x = (row_on && kinfo[jj] >= 0) ? __uint_as_float(s[jj]) * a.scale_log2 : -INFINITY;
            s[jj] = __float_as_uint(x);
            mx = fmaxf(mx, x);
          }
        }
        const float m_new = fmaxf(m_run, mx);
        float m_use = m_run;
        bool rescale = false;
        if (j == 0) {
          m_use = m_new;
        } else if (m_new > m_run + kRescaleThreshold) {
          m_use = m_new;
          rescale = true;
        }
        const float m_off = m_use == -INFINITY ? 0.f : m_use;
        const float alpha = rescale ? fast_exp2(m_run - m_use) : 1.f;
        float sum = 0.f;
        uint32_t pk[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float p0 = fast_exp2(__uint_as_float(s[2 * e]) - m_off);
          const float p1 = fast_exp2(__uint_as_float(s[2 * e + 1]) - m_off);
          sum += p0 + p1;
          pk[e] = pack_bf16x2(p0, p1);
        }
        l_run = (j == 0 ? 0.f : l_run * alpha) + sum;
        m_run = m_use;
        // P buffer g&1 was last read by PV(g-2)
        if (g >= 2 && !(ok = wait_or_abort(kBarODone + (g & 1), ((g >> 1) - 1) & 1))) break;
        // tcgen05.ld/st are warp-collective (.sync.aligned): the O rescale runs on
        // the whole warp when any of its rows needs it (the others scale by 1).
        if (__any_sync(0xffffffffu, rescale)) {
          if (!(ok = wait_or_abort(kBarODone + ((g - 1) & 1), ((g - 1) >> 1) & 1))) break;
          tc_fence_after();
#pragma unroll
          for (int c0 = 0; c0 < D; c0 += 16) {
            uint32_t r16[16];
            tmem_ld_32x32b_x16(tO + c0, r16);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) r16[e] = __float_as_uint(__uint_as_float(r16[e]) * alpha);
            tmem_st_32x32b_x16(tO + c0, r16);
          }
          tmem_st_wait();
        }
        uint8_t* prow = smem + L.p + (g & 1) * (kAttnBM * 128) + tid * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(prow + ((c ^ (tid & 7)) << 4)) =
              make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&bars[kBarPFull + (g & 1)]);

        if (SMALL && j == 0) {
          // bias of the next tile and the previous tile's epilogue, off the critical path
          if (tile_exists(lt + 1) && !(ok = extract_bias(lt + 1, tok_next))) break;
          if (pend_lt >= 0 && !(ok = epilogue(pend_lt, pend_g, pend_tok, pend_l))) break;
          pend_lt = -1;
        }
      }
      if (!ok) break;
      if constexpr (SMALL) {
        pend_lt = lt;
        pend_g = tb.n > 0 ? g - 1 : -1;
        pend_tok = tok_cur;
        pend_l = l_run;
      } else {
        if (tile_exists(lt + 1) && !(ok = extract_bias(lt + 1, tok_next))) break;
        if (!(ok = epilogue(lt, tb.n > 0 ? g - 1 : -1, tok_cur, l_run))) break;
      }
      tok_cur = tok_next;
    }
    if (ok && pend_lt >= 0) epilogue(pend_lt, pend_g, pend_tok, pend_l);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) tmem_dealloc(tmem, kAttnTmemCols);
}

template <int D, bool SMALL>
static int launch_attn(const AttnParams& p, cudaStream_t stream) {
  const AttnLayout<D, SMALL> L(p.win);
  static bool configured[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return SSAM_ERR_CUDA;
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(sparse_attn_kernel<D, SMALL>, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total) !=
        cudaSuccess)
      return SSAM_ERR_CUDA;
    configured[dev] = true;
  }
  // One persistent CTA per SM (the plan exceeds half the SM's shared memory),
  // so its 512 TMEM columns are always available.
  const int smem = L.total > 116 * 1024 ? L.total : 116 * 1024;
  const int sms = num_sms(dev);
  const int grid = p.total_tiles < sms ? p.total_tiles : sms;
  sparse_attn_kernel<D, SMALL><<<grid, kAttnThreads, smem, stream>>>(p);
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
  if (!(scale > 0.f)) return SSAM_ERR_INVALID;
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
  p.inv_scale = 1.0f / scale;
  p.n_tiles = (p.N + kAttnBM - 1) / kAttnBM;
  const int64_t total = static_cast<int64_t>(p.n_tiles) * n_seq * heads;
  if (total > INT32_MAX) return SSAM_ERR_UNSUPPORTED;
  p.total_tiles = static_cast<int>(total);
  const bool small = win <= 16;  // 32-row tables, 16-wide bias operands
  if (d == 64) return small ? launch_attn<64, true>(p, stream) : launch_attn<64, false>(p, stream);
  return small ? launch_attn<80, true>(p, stream) : launch_attn<80, false>(p, stream);
}

}  // namespace ssam
