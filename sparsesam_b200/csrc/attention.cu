// Stripe-Sort block-sparse attention with SAM's decomposed relative-position
// bias, on the sm_100a tensor cores.
//
// Semantics (algos/kernels/flash_attn.py:577-909 with algos/sparsesam/sam.py:62-73,
// 206-233): for one (sequence, head) row with tokens in permuted order
// p = 0..N-1 (token perm[p]), query block m = p/n_block attends to key blocks
// n < n_init (plus n == m when with_diag), n_block = 64 (SparseSAM's own
// choice, sam.py:52-57) or 128:
//   logit(p, k) = scale * <q_p, k_k> + relH[p][kh(k)] + relW[p][kw(k)]
//   relH[p][j]  = <q_p, Th[qh(p) - j + win - 1]>,  relW likewise with columns,
// keys past N are masked, rows are softmax-normalised (an empty row gives 0),
// and the result of permuted row p is written to raster token perm[p]
// (the inverse permutation and the head merge are fused into the store).
//
// Persistent, warp-specialised CTA (one per SM), 512 threads (16 warps; 640 in
// 20 warps for windowed grids):
//   warps 0-7   softmax: warps w and w+4 share TMEM lane quarter w % 4 (query
//               rows 32(w%4)..+31 of the tile) and split each 128-key block
//               into two 64-key halves; the row maxima are exchanged through
//               shared memory. For the global grid they also place the next
//               tile's rel-pos bias operand in TMEM and run the deferred
//               epilogue, split the same way;
//   warps 8-14  loaders: coalesced cp.async gathers (eight lanes per 128-byte row
//               segment) of the permuted K rows with the one-hot key-position
//               operand (warps 8-11, 32 rows each), the V rows (warps 12-13,
//               64 rows each; for global grids also the bias rows) and the Q
//               rows (warp 14);
//   warp 15     UMMA issuer: S = Q K^T + A_bias onehot^T (A_bias from TMEM),
//               O += P V (P from TMEM, V as one N = D operand); for windowed
//               grids also [P_H | P_W] = Q [Th ; Tw]^T of the next tile;
//   warps 16-19 (windowed grids) epilogue: O / l of lane quarter w % 4, all D
//               columns, stored at the raster rows.
// Windowed grids run each role's per-tile code once per tile, so it is fetched
// anew every tile: loops that run once per tile stay rolled and each role keeps
// one copy of its code (instruction fetch, not FLOPs or bandwidth, bounds them).
// Blocks are 128 keys wide (one N = 128 MMA per 16 channels of QK^T) and P.V
// is one MMA per 16 keys. The loaders are latency-bound gathers, so the key rows
// are spread over four warps, and the copy loop is kept rolled (one body shared
// by every loader role): the kernel's hot code is instruction-cache sensitive.
// O is rescaled lazily: only when a row maximum grows by more than 2^8 is the
// TMEM row read, scaled and written back; otherwise the stale maximum is kept
// (probabilities stay below 2^8 and the final 1/l normalisation is consistent).
// Every wait is bounded; on timeout the CTA raises SSAM_ERR_TIMEOUT and unwinds.
#include <cuda_fp16.h>

#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "host_util.h"

namespace ssam {

constexpr int kAttnBM = 128;   // queries per tile
constexpr int kAttnBN = 128;   // keys per block
constexpr int kMaskBlk = 64;   // keep-bar unit inside the kernel (64-token blocks; 128-token masks are converted)
constexpr int kAttnKW = 4;      // K loader warps (128 / kAttnKW key rows each)
constexpr int kAttnVW = 2;      // V loader warps
constexpr int kAttnLW = kAttnKW + kAttnVW + 1;  // loader warps 8 .. 8 + kAttnLW - 1 (last: Q rows)
constexpr int kAttnMmaWarp = 8 + kAttnLW;
constexpr int kAttnEpiWarp = kAttnMmaWarp + 1;  // windowed grids: epilogue warps 16 .. 19
// threads per CTA: windowed grids add the four epilogue warps
__host__ __device__ constexpr int attn_threads(bool small) { return 32 * (kAttnMmaWarp + 1 + (small ? 4 : 0)); }
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

// TMA copy of a 2-D tile into this CTA's shared memory (no multicast); completion
// is counted in bytes on `bar`.
__device__ __forceinline__ void tma_tile_2d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
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
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_32x32b_x8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D(tmem) (+)= A(tmem) * B(smem): A is K-major in TMEM (row m in lane m, two
// 16-bit elements per 32-bit column), B described by a shared-memory descriptor.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Shared-memory geometry of a D-wide operand tile with R rows, in 16-channel
// chunks: chunk region k (channels 16k..16k+15) holds R rows of 32 bytes with the
// 32-byte swizzle (16-byte half h of row r at h ^ ((r >> 2) & 1)). The same
// bytes serve as a K-major operand (one region per 16-wide k-step) and, for V,
// as an MN-major operand with N = D (regions are the N atoms, LBO = R * 32).
template <int D>
struct TileGeom {
  static constexpr int kChunks = D / 8;  // 16-byte chunks per row
  static __host__ __device__ constexpr int bytes(int rows) { return rows * D * 2; }
};

template <int D>
__device__ __forceinline__ uint32_t tile_chunk_addr(uint32_t base, int rows, int r, int c) {
  return base + (c >> 1) * rows * 32 + r * 32 + ((((c & 1) ^ ((r >> 2) & 1))) << 4);
}

// K-major operand descriptor for k-step ks (16 channels) of a TileGeom region.
template <int D>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int rows, int ks) {
  return make_smem_desc(base + ks * rows * 32, 16, 256, kSw32);
}

__host__ __device__ constexpr int align1k(int v) { return (v + 1023) & ~1023; }

// Instruction descriptor for kind::f16 with fp16 A/B (formats 0), fp32 accumulator.
__host__ __device__ constexpr uint32_t make_idesc_f16(uint32_t M, uint32_t N) {
  return (1u << 4) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

// Two specialisations.
//   SMALL (windowed grids, win <= 16): the rel-pos bias of the next tile
//   ([P_H | P_W] on the tensor cores + band extraction) is computed inside the
//   kernel while the current tile runs.
//   LARGE (the global grid): the bias of every query is computed once by
//   relbias_kernel into a workspace (in permuted query order); a loader stages
//   the rows of the next tile and the softmax warps move them into TMEM.
// TMEM plan (512 columns): S[2] (128 fp32 columns each; P overwrites the first
// 64 as bf16 pairs), O[kO] (D columns each), A_bias[2] (kBW columns each: relH
// pairs then relW pairs), and for SMALL [P_H | P_W] (64 columns).
template <int D, bool SMALL>
struct AttnCfg {
  static constexpr int kS = 2;                    // S / P buffers in TMEM
  static constexpr int kTileGroup = SMALL ? 2 : 1;  // consecutive query tiles per CTA (tile_of)
  // Q buffers: a tile's Q rows load while the two before it hold theirs (windowed
  // tiles are one key block long, so the UMMA thread needs the next tile's Q for
  // its [P_H | P_W] while the current tile's QK^T is being issued)
  static constexpr int kQBuf = SMALL ? 3 : 2;
  static constexpr int kStages = 2;               // K / V / one-hot stages (3 measured slower for windows)
  static_assert(kStages == kS && kS == 2, "stage and S / O indices are g % 2 (one fill per block)");
  static constexpr int kBW = SMALL ? 16 : 64;     // bias columns per table (>= win)
  static constexpr int kNT = 32;                  // rows per table (SMALL), stacked Th ; Tw
  static constexpr int kABCols = kBW;             // 2 x kBW fp16 = kBW columns
  static constexpr int kPHCols = SMALL ? 2 * kNT : 0;
  static constexpr int kTmO = kS * kAttnBN;       // TMEM column of O[0]
  static constexpr int kO = (kTmO + 2 * D + 2 * kABCols + kPHCols <= kAttnTmemCols) ? 2 : 1;
  static constexpr int kTmAB = kTmO + kO * D;     // TMEM column of A_bias[0]
  static constexpr int kTmPH = kTmAB + 2 * kABCols;
  static constexpr int kOHBytes = 2 * kAttnBN * kBW * 2;  // one-hot H | W regions per stage
  static constexpr int kABRow = 80;  // SMALL: a query's fp16 P row (64 B) + 16 B (conflict-free 16-byte stores)
  static constexpr int kOSplit = D == 80 ? 48 : D / 2;    // O columns of the first softmax half
  // SMALL epilogue staging: per lane-quarter block, 32 bf16 rows of D columns; the
  // row stride padded by 16 B (an odd number of 16-byte units: 16-byte stores of
  // 8 lanes hit 32 banks)
  static constexpr int kOStride = 2 * D + 16;
  static_assert(!SMALL || kO == 2, "the epilogue warps pair O buffer, l slot and tile parity");
  static_assert(kTmPH + kPHCols <= kAttnTmemCols, "TMEM plan exceeds 512 columns");
};

// Byte offset of element (row r, column k) of a K-major fp16 one-hot operand
// region (128B swizzle for 64-wide rows, 32B swizzle for 16-wide rows).
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
  static constexpr int kTables = SMALL ? TG::bytes(2 * C::kNT) : 0;
  static constexpr int kABStage = SMALL ? kAttnBM * C::kABRow : kAttnBM * 256;  // band scratch / staged bias rows
  int tab, q, kv, ab, ostage, xchg, lsum, tinfo, bars, total;
  __host__ __device__ AttnLayout() {
    tab = 0;
    q = align1k(tab + kTables);                   // [kQBuf] x bytes(128)
    kv = align1k(q + C::kQBuf * TG::bytes(kAttnBM));  // [stages] x kStage
    ab = align1k(kv + C::kStages * kStage);       // kABStage
    ostage = ab + kABStage;                       // SMALL: epilogue staging, 128 rows x kOStride
    xchg = ostage + (SMALL ? kAttnBM * C::kOStride : 0);  // float [2][2 halves][2 values][128]
    lsum = xchg + 2 * 2 * 2 * kAttnBM * 4;        // SMALL: float [2 slots][2 halves][128] row-sum shares
    tinfo = lsum + (SMALL ? 2 * 2 * kAttnBM * 4 : 0);  // SMALL: int [2]: the next tile shares the K / V fill
    bars = (tinfo + (SMALL ? 8 : 0) + 7) & ~7;    // mbarriers
    total = bars + 64 * 8 + 16 + 1024;            // mbarriers, TMEM address, abort flag + alignment slack
  }
};

struct AttnParams {
  const __nv_bfloat16* qkv;
  int64_t ld_qkv;
  int heads, win, N, C;
  const __nv_bfloat16* th;  // (2win-1, D)
  const __nv_bfloat16* tw;
  const int32_t* perm;
  int n_init;     // keep bar in 64-token blocks
  int with_diag;  // 0: none, 1: 64-token diagonal blocks, 2: 128-token diagonal blocks (the whole tile)
  float scale_log2;  // scale * log2(e)
  float inv_scale;   // 1 / scale
  __nv_bfloat16* out;
  int64_t ld_out;
  const int32_t* out_rows;  // optional output row of (sequence, token)
  int n_tiles;  // 128-query tiles per row (without query compaction)
  int total_tiles;
  // Query compaction of windowed grids (wpi > 0): the sequences are the windows of
  // images of a grid_h x grid_w token grid (window_partition order, padding at the
  // bottom / right), and only each window's real tokens are queries.
  int wpi;        // windows per image (0: every token of every sequence is a query)
  int nww;        // windows per image row
  int grid_h, grid_w;
  int img_tiles;  // query tiles per image
  int row_tiles;  // query tiles of a window row of an image that is not the last
  int kt_in, kt_col, kt_row, kt_corner;  // tiles per window-head: inner, last column, last row, corner (1 or 2)
  int nwh;        // windows per image column
  // fp32 reciprocals of the compaction divisors (fast_div)
  float r_img_tiles, r_row_tiles, r_span_in, r_span_row, r_win, r_wlast;
  int w_last;     // real width of the last window column
  // with compaction: bf16 qkv row of SAM's zero padding, read for padding keys (null:
  // the padding rows of qkv hold it)
  const __nv_bfloat16* pad_row;
  __half* bias_ws;  // LARGE: [rows][n_tiles*128][128] fp16 = relH/scale | relW/scale
};

// Token of permuted query position p of (sequence, head) row `row`, or -1 past N.
// Without the diagonal every query block attends to the same key blocks
// (n < n_init), so a query's result does not depend on its place in the
// permutation: the queries are then taken in raster order (token p) and no
// permutation entry is read. With the diagonal, position p holds token perm[p].
//
// With query compaction the window's real tokens (the top-left h_real x w_real
// block of the win x win window) are taken in raster order: query p is token
// (p / w_real) win + p % w_real, and tiles past the real tokens do not exist.
// x / d for 0 <= x < 2^24 and d >= 1 with r = fp32(1 / d): the fp32 product errs
// by less than one (exact for d = 1), so one correction step gives the quotient.
__device__ __forceinline__ int fast_div(int x, int d, float r) {
  int q = __float2int_rz(__int2float_rn(x) * r);
  const int rem = x - q * d;
  q += (rem >= d) - (rem < 0);
  return q;
}

// A query tile: its (sequence, head) row, sequence, head, query tile, and the real tokens
// of the row's window (n_real of them, w_real per window row; all N tokens and
// w_real = win without compaction).
struct TileDesc {
  int row, seq, head, qtile, n_real, w_real, h_real;
};

// Token of query position p (= qtile * 128 + tile row) of a tile, or -1.
template <bool CP>
__device__ __forceinline__ int query_tok(const AttnParams& a, const TileDesc& d, int p) {
  if (!CP) {
    if (p >= a.N) return -1;
    return a.with_diag ? __ldg(a.perm + static_cast<int64_t>(d.row) * a.N + p) : p;
  }
  if (p >= d.n_real) return -1;
  const int ty = fast_div(p, d.w_real, d.w_real == a.win ? a.r_win : a.r_wlast);
  return ty * a.win + (p - ty * d.w_real);
}

// Descriptor of global tile `tile`. Without compaction every row has n_tiles
// tiles. With it, tiles are numbered image by image, window by window (window
// rows of the image first), head by head, a window-head holding kt = ceil(real
// tokens / 128) tiles (1 or 2), where the class of a window is inner, last
// column, last row or corner. Arithmetic only, with reciprocal divisions: each
// role decodes every tile once.
template <bool CP>
__device__ __forceinline__ TileDesc tile_desc(const AttnParams& a, int tile) {
  TileDesc d;
  if (!CP) {
    d.row = tile / a.n_tiles;
    d.qtile = tile - d.row * a.n_tiles;
    d.seq = d.row / a.heads;
    d.head = d.row - d.seq * a.heads;
    d.n_real = a.N;
    d.w_real = a.win;
    d.h_real = a.win;
    return d;
  }
  const int img = fast_div(tile, a.img_tiles, a.r_img_tiles);
  int rem = tile - img * a.img_tiles;
  int wy = fast_div(rem, a.row_tiles, a.r_row_tiles);
  if (wy > a.nwh - 1) wy = a.nwh - 1;
  rem -= wy * a.row_tiles;
  const bool last_row = wy == a.nwh - 1;
  const int k_in = last_row ? a.kt_row : a.kt_in, k_col = last_row ? a.kt_corner : a.kt_col;
  const int span = a.heads * k_in;  // tiles of one window before the last column
  int wx = fast_div(rem, span, last_row ? a.r_span_row : a.r_span_in);
  int k = k_in;
  const bool last_col = wx >= a.nww - 1;
  if (last_col) {
    wx = a.nww - 1;
    k = k_col;
  }
  rem -= wx * span;
  d.head = k == 2 ? rem >> 1 : rem;
  d.qtile = k == 2 ? rem & 1 : 0;
  d.seq = img * a.wpi + wy * a.nww + wx;
  d.row = d.seq * a.heads + d.head;
  d.w_real = last_col ? a.w_last : a.win;
  d.h_real = last_row ? a.grid_h - (a.nwh - 1) * a.win : a.win;
  d.n_real = d.h_real * d.w_real;
  return d;
}

// Output row of token `tok` of sequence `seq` (-1: not stored); n_seq * N fits
// int32 (checked on the host).
__device__ __forceinline__ int query_out_row(const AttnParams& a, int seq, int tok) {
  if (tok < 0) return -1;
  const int i = seq * a.N + tok;
  return a.out_rows != nullptr ? __ldg(a.out_rows + i) : i;
}

// Key blocks of one tile. The mask enables 64-key block m for query m-block mb
// when m < nk, or m == mb with the diagonal. Processed 128-key blocks: those
// covering the keep bar [0, 64 nk), then block qtile (it holds the tile's two
// diagonal 64-key blocks) when the bar does not reach it.
struct TileBlocks {
  int nk, nkb, n, qt;
  __device__ TileBlocks() : nk(0), nkb(0), n(0), qt(0) {}
  __device__ TileBlocks(const AttnParams& a, int qtile) {
    const int nblk = (a.N + kMaskBlk - 1) / kMaskBlk;
    nk = a.n_init < nblk ? a.n_init : nblk;
    nkb = (nk + 1) / 2;
    qt = qtile;
    n = nkb + ((a.with_diag && qtile >= nkb) ? 1 : 0);
  }
  __device__ int at(int i) const { return i < nkb ? i : qt; }
};

// Whether local tile lt + 1 reads local tile lt's K / V fill: lt is the first query
// tile of a window-head with a second one (query compaction, one key block).
template <bool SMALL, bool CP>
__device__ __forceinline__ bool next_shares(int lt, const TileDesc& d, const TileBlocks& tb) {
  return SMALL && CP && !(lt & 1) && d.qtile == 0 && d.n_real > kAttnBM && tb.n == 1;
}

// A persistent CTA's local tile lt covers global tile tile_of<GT>(lt): groups of
// GT consecutive tiles, group index blockIdx.x + k gridDim.x. Windowed grids use
// GT = 2: a window-head's two query tiles read the same key block, so the
// second finds K / V in L2 (measured 1.79 -> 1.72 ms per layer). The global grid
// keeps GT = 1 (CTAs running side by side then share a row's key blocks; GT = 2
// measured 5.29 -> 5.60 ms).
template <int GT>
__device__ __forceinline__ int tile_of(int lt) {
  return GT * (static_cast<int>(blockIdx.x) + (lt / GT) * static_cast<int>(gridDim.x)) + lt % GT;
}

// Walks the flat (tile, key block) sequence of one persistent CTA.
template <int GT, bool CP>
struct BlockCursor {
  int tile, lt, j, g;
  bool done;
  TileBlocks tb;
  // the block list depends on the query tile only with the diagonal (never with
  // query compaction): the UMMA thread decodes no tile otherwise
  __device__ void set_blocks(const AttnParams& a) {
    tb = TileBlocks(a, (!CP && a.with_diag) ? tile_desc<CP>(a, tile).qtile : 0);
  }
  __device__ void start(const AttnParams& a) {
    lt = 0;
    tile = tile_of<GT>(0);
    j = 0;
    g = 0;
    done = tile >= a.total_tiles;
    if (!done) set_blocks(a);
  }
  __device__ void advance(const AttnParams& a) {
    ++j;
    ++g;
    if (j >= tb.n) {
      j = 0;
      ++lt;
      tile = tile_of<GT>(lt);
      done = tile >= a.total_tiles;
      if (!done) set_blocks(a);
    }
  }
};

// mbarrier indices
// K (with its one-hot rows) and V of a stage are released separately: K once
// QK^T of the block has completed, V once P.V has, so the K loads of block g+2
// overlap the softmax of blocks g and g+1.
enum {
  kBarTab = 0,
  kBarQFull = 1,     // [kQBuf <= 3]  loader lanes (cp.async)
  kBarQEmpty = 4,    // [kQBuf <= 3]  UMMA commit after the tile's last QK^T
  kBarKFull = 7,     // [3]  K loader lanes (cp.async)
  kBarKEmpty = 10,   // [3]  compaction: UMMA commit after the fill's last QK^T (else S-full frees K)
  kBarVFull = 13,    // [3]  V loader lanes (cp.async)
  kBarVEmpty = 16,   // [3]  compaction: UMMA commit after the fill's last P.V (else O-done frees V)
  kBarPHFull = 19,   //      UMMA commit (SMALL)
  kBarPHFree = 20,   //      K loaders (SMALL)
  kBarABFull = 21,   // [2]  A_bias of the tile is in TMEM (SMALL: K loaders; LARGE: softmax)
  kBarABSFull = 23,  //      LARGE: bias rows staged (cp.async)
  kBarABSFree = 24,  //      LARGE: softmax copied the staged rows
  kBarSFull = 25,    // [2]  UMMA commit after QK^T
  kBarSFree = 27,    // [2]  unused: O-done frees the S block (P lives in its columns)
  kBarPFull = 29,    // [2]  softmax
  kBarODone = 31,    // [2]  UMMA commit after P.V of block g (index g & 1)
  kBarOFree = 33,    // [2]  epilogue (LARGE: softmax warps; SMALL: epilogue warps)
  kBarXchg = 35,     // [2 rounds][4 lane quarters]  the two softmax warps of a quarter
  kBarDrain = 43,
  kBarOFull = 44,    // [2]  SMALL: UMMA commit after the tile's last P.V (index tile & 1)
  kBarLFull = 46,    // [2]  SMALL: softmax row-sum shares of the tile (index tile & 1)
  kNumBars = 48
};
static_assert(kNumBars * 8 + 8 <= 64 * 8, "mbarrier region of AttnLayout too small");

// Band of one table: the BW/2 output words (fp16 pairs) relX[j] = S[qc + win - 1 - j]
// (j < win, zero above) for the fp16 row S staged at `srow`. With
// base = qc + win - BW the band is the reversed window S[base .. base + BW - 1]:
// it is read as BW/2 + 1 consecutive words from word base >> 1 (the words before
// the row only feed entries that are masked) and re-paired with byte permutes.
template <int BW>
__device__ __forceinline__ void relbias_band(const uint8_t* srow, int qc, int win, uint32_t (&out)[BW / 2]) {
  const int base = qc + win - BW;
  const int w0 = base >> 1;  // arithmetic shift: floor
  const uint32_t* sw = reinterpret_cast<const uint32_t*>(srow) + w0;
  uint32_t u[BW / 2 + 1];
#pragma unroll
  for (int i = 0; i <= BW / 2; ++i) u[i] = sw[i];
  const bool odd = base & 1;
#pragma unroll
  for (int k = 0; k < BW / 2; ++k) {
    // word k = (relX[2k], relX[2k+1]) = (S[base + BW - 1 - 2k], S[base + BW - 2 - 2k])
    const int m = BW / 2 - 1 - k;
    uint32_t w = odd ? __byte_perm(u[m + 1], u[m], 0x7610) : __byte_perm(u[m], 0u, 0x1032);
    if (2 * k >= win) w = 0u;
    else if (2 * k + 1 >= win) w &= 0xffffu;
    out[k] = w;
  }
}

// Writes the NV fp32 values v (times `mul`) as fp16 to `dst` (16-byte aligned).
template <int NV>
__device__ __forceinline__ void stage_f16_row(uint8_t* dst, const uint32_t* v, float mul) {
  static_assert(NV % 8 == 0, "whole 16-byte units");
  uint4* sp = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < NV / 8; ++i) {
    uint32_t h[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __half2 h2 = __floats2half2_rn(__uint_as_float(v[8 * i + 2 * j]) * mul,
                                           __uint_as_float(v[8 * i + 2 * j + 1]) * mul);
      h[j] = *reinterpret_cast<const uint32_t*>(&h2);
    }
    sp[i] = make_uint4(h[0], h[1], h[2], h[3]);
  }
}

// Epilogue of one softmax warp for nc16 16-column chunks of O starting at TMEM
// column tO: each lane's row, times `scale`, as bf16 into its `stride`-byte row of
// the warp's staging block; then the warp stores the block row segment by row
// segment (2 nc16 lanes of 16 bytes per row) to out row orow of each lane (< 0: not
// stored), columns starting at obase. Both loops stay rolled: the epilogue runs once
// per tile, and its code is fetched anew each time.
__device__ __forceinline__ void stage_out_rows(uint32_t tO, int nc16, uint8_t* stage, int stride, int orow,
                                               float scale, __nv_bfloat16* obase, int64_t ld_out) {
  const int lane = static_cast<int>(threadIdx.x & 31);
  __syncwarp();  // the previous tile's row segments have been read out of the block
  uint8_t* srow = stage + lane * stride;
  const float2 sc2 = make_float2(scale, scale);
#pragma unroll 1
  for (int c = 0; c < nc16; ++c) {
    uint32_t v[16];
    tmem_ld_32x32b_x16(tO + 16 * c, v);
    tmem_ld_wait();
    uint32_t w[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float2 o = mul2(make_float2(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1])), sc2);
      w[e] = pack_bf16x2(o.x, o.y);
    }
    uint4* d = reinterpret_cast<uint4*>(srow + 32 * c);
    d[0] = make_uint4(w[0], w[1], w[2], w[3]);
    d[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
  __syncwarp();
  // round k: lane l moves chunk (l + 32 k) % kch of block row (l + 32 k) / kch
  const int kch = 2 * nc16;
  int rr = lane / kch, c = lane - rr * kch;
  const int drr = 32 / kch, dc = 32 - drr * kch;
#pragma unroll 1
  for (int k = 0; k < kch; ++k) {
    const int dst_row = __shfl_sync(0xffffffffu, orow, rr);
    const uint4 val = *reinterpret_cast<const uint4*>(stage + rr * stride + c * 16);
    if (dst_row >= 0) *reinterpret_cast<uint4*>(obase + static_cast<int64_t>(dst_row) * ld_out + c * 8) = val;
    rr += drr;
    c += dc;
    if (c >= kch) {
      c -= kch;
      ++rr;
    }
  }
}

// tm_tile: qkv as a [n_seq*N, 3C] bf16 tensor with a 16-channel x 128-row box, the
// 32-byte swizzle (one box lands as one TileGeom chunk region): a windowed tile's
// consecutive Q rows.
template <int D, bool SMALL, bool CP>
__global__ void __launch_bounds__(attn_threads(SMALL), 1)
    sparse_attn_kernel(const AttnParams a, const __grid_constant__ CUtensorMap tm_tile) {
  using TG = TileGeom<D>;
  using C = AttnCfg<D, SMALL>;
  using LAY = AttnLayout<D, SMALL>;
  const LAY L;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int N = a.N, win = a.win;

  if (tid == 0) {
    mbar_init(&bars[kBarTab], 64);
    for (int i = 0; i < C::kQBuf; ++i) {
      mbar_init(&bars[kBarQFull + i], 32);  // one arrival per lane of the Q warp
      mbar_init(&bars[kBarQEmpty + i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[kBarABFull + i], SMALL ? 128 : 256);
      mbar_init(&bars[kBarSFull + i], 1);
      mbar_init(&bars[kBarSFree + i], 1);
      mbar_init(&bars[kBarPFull + i], 256);
      mbar_init(&bars[kBarODone + i], 1);
      mbar_init(&bars[kBarOFree + i], SMALL ? 128 : 256);
      mbar_init(&bars[kBarOFull + i], 1);
      mbar_init(&bars[kBarLFull + i], 256);
      for (int w = 0; w < 4; ++w) mbar_init(&bars[kBarXchg + 4 * i + w], 64);
    }
    mbar_init(&bars[kBarPHFull], 1);
    mbar_init(&bars[kBarPHFree], 128);
    mbar_init(&bars[kBarABSFull], kAttnVW * 64);
    mbar_init(&bars[kBarABSFree], 256);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&bars[kBarKFull + s], kAttnKW * 64);
      mbar_init(&bars[kBarKEmpty + s], 1);
      mbar_init(&bars[kBarVFull + s], kAttnVW * 64);
      mbar_init(&bars[kBarVEmpty + s], 1);
    }
    mbar_init(&bars[kBarDrain], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kAttnMmaWarp) {
    tmem_alloc(tmem_holder, kAttnTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  // Fast path: one try_wait (usually the phase has completed); the abort flag is
  // read only when the wait has to sleep.
  // (the bounded wait stays a call here: inlining its first test measured slower
  // for this kernel, whose loader and softmax paths sit at the register limit)
  auto wait_or_abort = [&](int bar, uint32_t parity) -> bool {
    if (mbar_try_wait(&bars[bar], parity)) return true;
    if (*abort_flag) return false;
    if (!mbar_wait_slow(&bars[bar], parity)) {
      *abort_flag = 1;
      return false;
    }
    return true;
  };
  auto tile_exists = [&](int lt_) { return tile_of<C::kTileGroup>(lt_) < a.total_tiles; };

  if (warp >= 8 && warp < kAttnMmaWarp) {
    // =========================== loader warps ===========================
    // Warp 8 + w (w < kAttnKW): K rows 32w..32w+31 of each block with their
    // one-hot rows and, for windowed grids, each tile's rel-pos bias operand; warp
    // 8 also the rel-pos tables. Warp 8 + kAttnKW + h: V rows 64h..64h+63 of each
    // block and (LARGE) the staged bias rows 64h..64h+63 of each tile. The last
    // loader warp: the 128 Q rows of each tile, as soon as its Q buffer is free.
    // Key rows (in permuted order) and gathered Q rows: a copy instruction moves
    // 16 bytes per lane with eight lanes on one 128-byte row segment (four rows
    // per instruction), then the 32-byte tails (sixteen rows); lane l holds the
    // tokens of rows l, l+32, ... and hands them out with shuffles; rows of padded
    // positions (token < 0) are zero-filled. A windowed tile's consecutive Q rows
    // (raster query order) arrive by TMA, one tile copy per 16-channel chunk.
    const int lw = warp - 8;
    const int kv = lw < kAttnKW ? 0 : (lw < kAttnKW + kAttnVW ? 1 : 2);  // 0: K, 1: V, 2: Q
    const int part = kv == 0 ? lw : lw - kAttnKW;
    constexpr int kKRows = kAttnBN / kAttnKW, kVRows = kAttnBN / kAttnVW;
    const int my_rows = kv == 0 ? kKRows : kVRows;
    const int row0 = part * my_rows;   // this warp's first key row of a block
    const bool q_warp = kv == 2;       // all Q rows of each tile
    // nrows (a multiple of 32, at most 128) rows starting at tile row r0, channel
    // offset xcol of each token row; tok[s] holds the token of row r0 + 32 s + lane
    // (-1: zero-filled, -2 - t: padding key t, read from pad_row).
    // One 32-row group per iteration (kept rolled: the loop body is shared by all
    // loader roles, which keeps the kernel's hot code small).
    auto copy_rows = [&](uint32_t region, int R, int r0, int nrows, const int (&tok)[4], const __nv_bfloat16* base,
                         int xcol) {
      const int c = lane & 7;
      const int ct = 8 + (lane & 1);
#pragma unroll 1
      for (int s = 0; s < nrows / 32; ++s) {
        const int tk = s == 0 ? tok[0] : s == 1 ? tok[1] : s == 2 ? tok[2] : tok[3];
        const int rb = r0 + 32 * s;
#pragma unroll
        for (int i = 0; i < 8; ++i) {  // 4 rows per instruction
          const int rr = 4 * i + (lane >> 3);
          const int t = __shfl_sync(0xffffffffu, tk, rr);
          const __nv_bfloat16* src = t >= 0 ? base + static_cast<int64_t>(t) * a.ld_qkv + xcol + c * 8
                                            : (t < -1 ? a.pad_row + xcol + c * 8 : a.qkv);
          cp_async16(tile_chunk_addr<D>(region, R, rb + rr, c), src, t != -1 ? 16u : 0u);
        }
        if constexpr (D > 64) {
#pragma unroll
          for (int i = 0; i < 2; ++i) {  // 16 rows per instruction
            const int rr = 16 * i + (lane >> 1);
            const int t = __shfl_sync(0xffffffffu, tk, rr);
            const __nv_bfloat16* src = t >= 0 ? base + static_cast<int64_t>(t) * a.ld_qkv + xcol + ct * 8
                                              : (t < -1 ? a.pad_row + xcol + ct * 8 : a.qkv);
            cp_async16(tile_chunk_addr<D>(region, R, rb + rr, ct), src, t != -1 ? 16u : 0u);
          }
        }
      }
    };
    constexpr int kMaxKV = (kKRows > kVRows ? kKRows : kVRows) / 32;  // tokens per lane

    // previous one-hot entries (kh | kw << 16, -1: none) of this K-loader lane's
    // two rows in each stage
    int oh_prev[C::kStages][kKRows / 32];
#pragma unroll
    for (int s2 = 0; s2 < C::kStages; ++s2)
#pragma unroll
      for (int i = 0; i < kKRows / 32; ++i) oh_prev[s2][i] = -1;
    if (lw == 0) {
      // one-hot regions start at zero
      for (int s2 = 0; s2 < C::kStages; ++s2) {
        uint4* oh = reinterpret_cast<uint4*>(smem + L.kv + s2 * LAY::kStage + 2 * TG::bytes(kAttnBN));
        for (int i = lane; i < C::kOHBytes / 16; i += 32) oh[i] = make_uint4(0u, 0u, 0u, 0u);
      }
      if constexpr (SMALL) {  // [Th ; Tw] stacked, rows past 2win-1 zero
        const int trows = 2 * win - 1;
        for (int r = lane; r < 2 * C::kNT; r += 32) {
          const int tr = r & (C::kNT - 1);
          const __nv_bfloat16* src = (r < C::kNT ? a.th : a.tw) + tr * D;
#pragma unroll
          for (int c = 0; c < TG::kChunks; ++c)
            cp_async16(tile_chunk_addr<D>(sb + L.tab, 2 * C::kNT, r, c), tr < trows ? src + c * 8 : a.th,
                       tr < trows ? 16u : 0u);
        }
      }
      __syncwarp();
      mbar_arrive(&bars[kBarTab]);
      cp_async_arrive_noinc(&bars[kBarTab]);
    }

    int q_last[C::kQBuf];  // last tile loaded into each Q buffer (-1: none)
#pragma unroll
    for (int i = 0; i < C::kQBuf; ++i) q_last[i] = -1;

    auto load_q = [&](int lt_) -> bool {
      const TileDesc td = tile_desc<CP>(a, tile_of<C::kTileGroup>(lt_));
      const int row = td.row, qtile = td.qtile, seq = td.seq, head = td.head;
      const int qb = lt_ % C::kQBuf;
      if (q_warp) {
        // raster query order over whole window rows: the tile's Q rows are consecutive
        const bool tiled = SMALL && !a.with_diag && td.w_real == win;
        int qt[4];  // rows 32 i + lane of the tile
#pragma unroll
        for (int i = 0; i < 4; ++i) qt[i] = tiled ? -1 : query_tok<CP>(a, td, qtile * kAttnBM + 32 * i + lane);
        if (!wait_or_abort(kBarQEmpty + qb, ((lt_ / C::kQBuf) & 1) ^ 1)) return false;
        const uint32_t dst = sb + L.q + qb * TG::bytes(kAttnBM);
        uint64_t* fb = &bars[kBarQFull + qb];
        if (tiled) {
          // one tile copy per 16-channel chunk (lanes 0 .. D/16 - 1); rows past the
          // tensor read as zero, rows of the next window are computed but not stored
          if (lane == 0) mbar_arrive_expect_tx(fb, TG::bytes(kAttnBM));
          __syncwarp();
          if (lane < D / 16)
            tma_tile_2d(dst + lane * kAttnBM * 32, &tm_tile, fb, head * D + 16 * lane, seq * N + qtile * kAttnBM);
          if (lane != 0) mbar_arrive(fb);
        } else {
          copy_rows(dst, kAttnBM, 0, 128, qt, a.qkv + static_cast<int64_t>(seq) * N * a.ld_qkv, head * D);
          cp_async_arrive_noinc(fb);
        }
#pragma unroll
        for (int i = 0; i < C::kQBuf; ++i)
          if (i == qb) q_last[i] = lt_;
      }
      if (!SMALL && kv == 1) {  // bias rows row0 .. row0 + kVRows - 1 of the tile (256 B each), two rows per instruction
        if (!wait_or_abort(kBarABSFree, (lt_ & 1) ^ 1)) return false;
        const uint8_t* src = reinterpret_cast<const uint8_t*>(
            a.bias_ws + (static_cast<int64_t>(row) * a.n_tiles + qtile) * kAttnBM * 128);
        const int c = lane & 15;
#pragma unroll 8
        for (int i = 0; i < kVRows / 2; ++i) {
          const int r = row0 + 2 * i + (lane >> 4);
          cp_async16(sb + L.ab + (c >> 3) * (kAttnBM * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4),
                     src + r * 256 + c * 16, 16u);
        }
        mbar_arrive(&bars[kBarABSFull]);
        cp_async_arrive_noinc(&bars[kBarABSFull]);
      }
      return true;
    };

    // SMALL, K warps: the rel-pos bias operand of tile lt_ (thread = query row
    // 32 (warp % 4) + lane, both tables). [P_H | P_W] of the tile comes from the
    // UMMA thread; each table row is staged as fp16 (x 1 / scale) and its band
    // relX[j] = P_X[qc - j + win - 1] read as a reversed window, then the two
    // bands go to A_bias[lt_ & 1] in TMEM. The buffer's previous reader, QK^T of
    // tile lt_ - 2, completed before the [P_H | P_W] commit of tile lt_.
    auto stage_bias_rows = [&](int lt_, const TileDesc& td, bool next_share) -> bool {
      if constexpr (!SMALL) {
        return true;
      } else {
      const int r = (warp & 3) * 32 + lane;
      const uint32_t t_lane = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
      const int t = query_tok<CP>(a, td, td.qtile * kAttnBM + r);
      const int qh = t >= 0 ? t / win : 0;
      const int qw = t >= 0 ? t - qh * win : 0;
      if (!wait_or_abort(kBarPHFull, lt_ & 1)) return false;
      tc_fence_after();
      uint32_t ph[C::kNT], pw[C::kNT];
      tmem_ld_32x32b_x32(t_lane + C::kTmPH, ph);
      tmem_ld_32x32b_x32(t_lane + C::kTmPH + C::kNT, pw);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&bars[kBarPHFree]);
      uint8_t* srow = smem + L.ab + r * C::kABRow;
      uint32_t v[2 * (C::kBW / 2)];
      uint32_t (&vh)[C::kBW / 2] = *reinterpret_cast<uint32_t(*)[C::kBW / 2]>(&v[0]);
      uint32_t (&vw)[C::kBW / 2] = *reinterpret_cast<uint32_t(*)[C::kBW / 2]>(&v[C::kBW / 2]);
      stage_f16_row<C::kNT>(srow, ph, a.inv_scale);
      relbias_band<C::kBW>(srow, qh, win, vh);
      stage_f16_row<C::kNT>(srow, pw, a.inv_scale);
      relbias_band<C::kBW>(srow, qw, win, vw);
      tmem_st_32x32b_x16(t_lane + C::kTmAB + (lt_ & 1) * C::kABCols, v);
      tmem_st_wait();
      tc_fence_before();
      // the UMMA thread reads whether the next tile shares this one's K / V fill once
      // A_bias is in (the slot's next write, for tile lt_ + 2, waits for [P_H | P_W]
      // of that tile, which the UMMA thread issues after reading this one)
      if (warp == 8 && lane == 0) reinterpret_cast<volatile int*>(smem + L.tinfo)[lt_ & 1] = next_share ? 1 : 0;
      mbar_arrive(&bars[kBarABFull + (lt_ & 1)]);
      return true;
      }
    };

    int g = 0;  // stage fills of this loader (stage g % kStages)
    bool share = false;  // the tile reads the previous tile's fill
    bool ok = true;
    if (kv == 2) {  // Q warp: every tile as soon as its Q buffer is free
      for (int lt = 0; ok && tile_exists(lt) && !*abort_flag; ++lt) ok = load_q(lt);
    }
    // (K / V warps of windowed grids load no Q and no staged bias rows: they skip
    // load_q, whose code would otherwise be inlined into their loop)
    if (!SMALL && kv < 2 && tile_exists(0)) ok = load_q(0);
    for (int lt = 0; kv < 2 && ok && tile_exists(lt) && !*abort_flag; ++lt) {
      if (!SMALL && tile_exists(lt + 1) && !(ok = load_q(lt + 1))) break;
      const TileDesc td = tile_desc<CP>(a, tile_of<C::kTileGroup>(lt));
      const int row = td.row, qtile = td.qtile, seq = td.seq, head = td.head;
      const int32_t* perm = a.perm + static_cast<int64_t>(row) * N;
      const __nv_bfloat16* base = a.qkv + static_cast<int64_t>(seq) * N * a.ld_qkv;
      const int xcol = (kv == 0 ? a.C : 2 * a.C) + head * D;
      const TileBlocks tb(a, qtile);
      // With query compaction a window-head with more than 128 real tokens has two
      // query tiles, global tiles 2m and 2m + 1 (a window's tiles start at an even
      // index), hence local tiles lt and lt + 1 of one CTA: with one key block, the
      // second reads the first one's K / V fill instead of gathering it again. Each
      // fill gets one empty commit, after its last reader.
      const bool next_share = next_shares<SMALL, CP>(lt, td, tb);
      int nt[4] = {-1, -1, -1, -1};  // tokens of keys row0 + lane + 32 i of the next block
      // keys of the window's padding (outside its h_real x w_real top-left block)
      // are read from pad_row when given
      const bool sub_pad = CP && a.pad_row != nullptr && td.n_real < N;
      auto fetch = [&](int jb) {
        const int kp = tb.at(jb) * kAttnBN + row0 + lane;
#pragma unroll
        for (int i = 0; i < kMaxKV; ++i) {
          int t = (32 * i < my_rows && kp + 32 * i < N) ? __ldg(perm + kp + 32 * i) : -1;
          if (sub_pad && t >= 0) {
            const int ty = fast_div(t, win, a.r_win);
            if (ty >= td.h_real || t - ty * win >= td.w_real) t = -2 - t;
          }
          nt[i] = t;
        }
      };
      if (tb.n > 0 && !share) fetch(0);
      for (int j = 0; j < (share ? 0 : tb.n); ++j, ++g) {
        int t[4] = {-1, -1, -1, -1};
#pragma unroll
        for (int i = 0; i < kMaxKV; ++i) t[i] = nt[i];
        if (j + 1 < tb.n) fetch(j + 1);  // the next block's tokens, one block ahead
        const int stage = g % C::kStages;
        const int full_bar = (kv == 0 ? kBarKFull : kBarVFull) + stage;
        // the stage is free once the QK^T (K) or P.V (V) that read its previous
        // fill last has completed: its K- / V-empty commit where fills can be
        // shared, else the S-full / O-done commit of that block (one fill per block)
        const int empty_bar = (SMALL && CP) ? (kv == 0 ? kBarKEmpty : kBarVEmpty) + stage
                                            : (kv == 0 ? kBarSFull : kBarODone) + stage;
        if (!(ok = wait_or_abort(empty_bar, ((g / C::kStages) & 1) ^ 1))) break;
        const uint32_t sK = sb + L.kv + stage * LAY::kStage;
        if (kv == 0) {  // one-hot rows of this lane's two keys
          uint8_t* oh_h = smem + L.kv + stage * LAY::kStage + 2 * TG::bytes(kAttnBN);
          uint8_t* oh_w = oh_h + kAttnBN * C::kBW * 2;
#pragma unroll
          for (int s2 = 0; s2 < C::kStages; ++s2) {
            if (s2 != stage) continue;  // keeps oh_prev in registers
#pragma unroll
            for (int i = 0; i < kKRows / 32; ++i) {
              const int r = row0 + lane + 32 * i;
              int info = -1;
              const int tk = t[i] >= 0 ? t[i] : (t[i] < -1 ? -2 - t[i] : -1);  // padding keys keep their place
              if (tk >= 0) {
                const int kh = tk / win;
                info = kh | ((tk - kh * win) << 16);
              }
              const int old = oh_prev[s2][i];
              if (old >= 0) {  // clear the previous one-hot entries of this row
                *reinterpret_cast<uint16_t*>(oh_h + bias_off<SMALL>(r, old & 0xffff)) = 0;
                *reinterpret_cast<uint16_t*>(oh_w + bias_off<SMALL>(r, old >> 16)) = 0;
              }
              if (info >= 0) {
                *reinterpret_cast<uint16_t*>(oh_h + bias_off<SMALL>(r, info & 0xffff)) = 0x3C00;  // fp16 1.0
                *reinterpret_cast<uint16_t*>(oh_w + bias_off<SMALL>(r, info >> 16)) = 0x3C00;
              }
              oh_prev[s2][i] = info;
            }
          }
          fence_proxy_async_smem();  // one-hot rows (generic stores) -> UMMA reads
        }
        copy_rows(kv == 0 ? sK : sK + TG::bytes(kAttnBN), kAttnBN, row0, my_rows, t, base, xcol);
        mbar_arrive(&bars[full_bar]);
        cp_async_arrive_noinc(&bars[full_bar]);
      }
      // the tile's bias operand once its key rows are on their way
      if constexpr (SMALL) {
        if (ok && kv == 0 && !(ok = stage_bias_rows(lt, td, next_share))) break;
      }
      share = next_share;
    }
    cp_async_wait_all();
    // No TMA copy of the Q warp may still be landing when the CTA exits: wait
    // (bounded) for the last phase of each Q buffer (whichever path filled it);
    // already complete unless the kernel is unwinding.
    if (q_warp && lane == 0) {
#pragma unroll
      for (int i = 0; i < C::kQBuf; ++i)
        if (q_last[i] >= 0) mbar_wait(&bars[kBarQFull + i], (q_last[i] / C::kQBuf) & 1);
    }
  } else if (warp == kAttnMmaWarp) {
    // =========================== UMMA issuer ===========================
    if (lane == 0) {
      const uint32_t idesc_t = make_idesc_bf16(kAttnBM, 2 * C::kNT, 0, 0);
      const uint32_t idesc_s = make_idesc_bf16(kAttnBM, kAttnBN, 0, 0);
      const uint32_t idesc_b = make_idesc_f16(kAttnBM, kAttnBN);
      const uint32_t idesc_o = make_idesc_bf16(kAttnBM, D, 0, 1);
      bool ok = !SMALL || wait_or_abort(kBarTab, 0);
      // K / V fill read by the current QK^T (fq) and P.V (fp): a new fill per block,
      // except a window-head's second tile, which shares its first tile's; bit
      // lt & 3 of nexts = tile lt + 1 shares tile lt's fill (read with A_bias of
      // tile lt; tile lt shares when bit (lt - 1) & 3 is set)
      int fq = -1, fp = -1;
      uint32_t nexts = 0;
      const volatile int* tinfo = reinterpret_cast<const volatile int*>(smem + L.tinfo);

      auto issue_ph = [&](int lt_) -> bool {  // [P_H | P_W] of tile lt_ (SMALL)
        const int qb = lt_ % C::kQBuf;
        if (!wait_or_abort(kBarQFull + qb, (lt_ / C::kQBuf) & 1)) return false;
        if (!wait_or_abort(kBarPHFree, (lt_ & 1) ^ 1)) return false;
        tc_fence_after();
        fence_proxy_async_smem();
        const uint64_t dq = kmajor_desc<D>(sb + L.q + qb * TG::bytes(kAttnBM), kAttnBM, 0);
        const uint64_t dt = kmajor_desc<D>(sb + L.tab, 2 * C::kNT, 0);
#pragma unroll 1
        for (int ks = 0; ks < D / 16; ++ks)
          umma_f16_ss(tmem + C::kTmPH, dq + ks * (kAttnBM * 2), dt + ks * (2 * C::kNT * 2), idesc_t, ks > 0);
        umma_commit(&bars[kBarPHFull]);
        return true;
      };
      auto issue_qk = [&](const BlockCursor<C::kTileGroup, CP>& c) -> bool {
        if (c.j == 0) {
          if constexpr (SMALL) {
            if (tile_exists(c.lt + 1) && !issue_ph(c.lt + 1)) return false;
          } else {
            if (!wait_or_abort(kBarQFull + c.lt % C::kQBuf, (c.lt / C::kQBuf) & 1)) return false;
          }
          if (!wait_or_abort(kBarABFull + (c.lt & 1), (c.lt >> 1) & 1)) return false;
        }
        if (SMALL && CP && c.j == 0)
          nexts = (nexts & ~(1u << (c.lt & 3))) | (static_cast<uint32_t>(tinfo[c.lt & 1] != 0) << (c.lt & 3));
        const bool share = SMALL && CP && c.j == 0 && ((nexts >> ((c.lt - 1) & 3)) & 1u);
        const bool shared_next = SMALL && CP && ((nexts >> (c.lt & 3)) & 1u);
        if (!share) ++fq;
        const int st = fq % C::kStages, sbuf = c.g % C::kS;
        if (!wait_or_abort(kBarKFull + st, (fq / C::kStages) & 1)) return false;
        // S block free once P.V of block g - kS (which reads P from it) completed
        if (!wait_or_abort(kBarODone + sbuf, ((c.g / C::kS) & 1) ^ 1)) return false;
        tc_fence_after();
        fence_proxy_async_smem();
        const uint32_t sQ = sb + L.q + (c.lt % C::kQBuf) * TG::bytes(kAttnBM);
        const uint32_t sK = sb + L.kv + st * LAY::kStage;
        const uint32_t sOH = sK + 2 * TG::bytes(kAttnBN);
        const uint32_t tAB = tmem + C::kTmAB + (c.lt & 1) * C::kABCols;
        const uint32_t tS = tmem + sbuf * kAttnBN;
        // (windowed grids issue each MMA once per tile: rolled loops keep the UMMA
        // thread's code, fetched anew every tile, short; descriptors step by the
        // 16-byte-unit offset of a 16-channel chunk)
        const uint64_t dq = kmajor_desc<D>(sQ, kAttnBM, 0), dk = kmajor_desc<D>(sK, kAttnBN, 0);
#pragma unroll(SMALL ? 1 : D / 16)
        for (int ks = 0; ks < D / 16; ++ks)
          umma_f16_ss(tS, dq + ks * (kAttnBM * 2), dk + ks * (kAttnBN * 2), idesc_s, ks > 0);
        // + A_bias . onehot^T  (relH / scale at kh, relW / scale at kw); A_bias from TMEM
#pragma unroll(SMALL ? 1 : 2)
        for (int part = 0; part < 2; ++part) {
          const uint32_t ab = tAB + part * (C::kBW / 2);
          const uint32_t oh = sOH + part * kAttnBN * C::kBW * 2;
          if constexpr (SMALL) {
            umma_f16_ts(tS, ab, make_smem_desc(oh, 16, 256, kSw32), idesc_b, 1u);
          } else {
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              umma_f16_ts(tS, ab + ks * 8, make_smem_desc(oh + ks * 32, 16, 1024, kSw128), idesc_b, 1u);
          }
        }
        umma_commit(&bars[kBarSFull + sbuf]);
        if (SMALL && CP && !shared_next) umma_commit(&bars[kBarKEmpty + st]);  // the fill's last QK^T
        if (c.j == c.tb.n - 1) umma_commit(&bars[kBarQEmpty + c.lt % C::kQBuf]);
        return true;
      };
      auto issue_pv = [&](const BlockCursor<C::kTileGroup, CP>& c) -> bool {
        if (!wait_or_abort(kBarPFull + (c.g & 1), (c.g >> 1) & 1)) return false;
        const int ob = c.lt % C::kO;
        if (c.j == 0 && !wait_or_abort(kBarOFree + ob, ((c.lt / C::kO) & 1) ^ 1)) return false;
        if (!(SMALL && CP && c.j == 0 && ((nexts >> ((c.lt - 1) & 3)) & 1u))) ++fp;
        const int st = fp % C::kStages, sbuf = c.g % C::kS;
        if (!wait_or_abort(kBarVFull + st, (fp / C::kStages) & 1)) return false;
        tc_fence_after();
        fence_proxy_async_smem();
        const uint32_t tP = tmem + sbuf * kAttnBN;
        const uint32_t sV = sb + L.kv + st * LAY::kStage + TG::bytes(kAttnBN);
        const uint32_t tO = tmem + C::kTmO + ob * D;
        // V as an MN-major operand with N = D: 32B-swizzled atoms of 8 keys x 16
        // channels, the D/16 channel regions LBO = 128 * 32 bytes apart; 16 keys = 512 B.
        // P of keys 0..63 sits in columns 0..31 of the S block, keys 64..127 in 64..95
        const uint64_t dv = make_smem_desc(sV, kAttnBN * 32, 256, kSw32);
#pragma unroll(SMALL ? 1 : kAttnBN / 16)
        for (int ks = 0; ks < kAttnBN / 16; ++ks)
          umma_f16_ts(tO, tP + ks * 8 + (ks >= kAttnBN / 32 ? 32 : 0), dv + ks * 32, idesc_o,
                      (c.j > 0 || ks > 0) ? 1u : 0u);
        umma_commit(&bars[kBarODone + (c.g & 1)]);  // also frees S block sbuf (and, without compaction, V)
        if (SMALL && CP && !((nexts >> (c.lt & 3)) & 1u)) umma_commit(&bars[kBarVEmpty + st]);  // last P.V
        if (SMALL && c.j == c.tb.n - 1) umma_commit(&bars[kBarOFull + ob]);
        return true;
      };

      if (ok && SMALL && tile_exists(0)) ok = issue_ph(0);
      BlockCursor<C::kTileGroup, CP> cq, cp;
      cq.start(a);
      cp.start(a);
      while (ok && !cp.done) {
        // QK^T of block g+1 goes ahead of P.V of block g, no further: a deeper
        // lookahead would make P.V(g) wait for a K/V stage that only P.V(g-1) frees.
        while (ok && !cq.done && cq.g <= cp.g + 1) {
          ok = issue_qk(cq);
          cq.advance(a);
        }
        if (!ok) break;
        ok = issue_pv(cp);
        cp.advance(a);
      }
      umma_commit(&bars[kBarDrain]);
      mbar_wait_slow(&bars[kBarDrain], 0);
    }
  } else if (warp >= kAttnEpiWarp) {
    if constexpr (SMALL) {
      // ===================== epilogue warps (windowed grids) =====================
      // Warp kAttnEpiWarp + q: query rows 32q .. 32q + 31 of every tile (TMEM lane
      // quarter q), all D columns: O / l as bf16, stored at the raster token of
      // the row (inverse permutation and head merge). The tile's O buffer and
      // row-sum slot are tile & 1; both are released through O-free.
      const int q4 = warp & 3;
      const int r = q4 * 32 + lane;
      const uint32_t t_lane = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
      uint8_t* stage = smem + L.ostage + q4 * 32 * C::kOStride;
      const float* lsum = reinterpret_cast<const float*>(smem + L.lsum);
      uint32_t ofull_par = 0;  // bit b: parity of the next O-full phase of buffer b
      bool ok = true;
      for (int lt = 0; ok && tile_exists(lt) && !*abort_flag; ++lt) {
        const TileDesc td = tile_desc<CP>(a, tile_of<C::kTileGroup>(lt));
        const int orow = query_out_row(a, td.seq, query_tok<CP>(a, td, td.qtile * kAttnBM + r));
        const bool any = TileBlocks(a, td.qtile).n > 0;
        const int ob = lt & 1;
        if (any) {  // O-full commits only for tiles with key blocks
          if (!(ok = wait_or_abort(kBarOFull + ob, (ofull_par >> ob) & 1))) break;
          ofull_par ^= 1u << ob;
        }
        if (!(ok = wait_or_abort(kBarLFull + ob, (lt >> 1) & 1))) break;
        tc_fence_after();
        const float l = lsum[(2 * ob) * kAttnBM + r] + lsum[(2 * ob + 1) * kAttnBM + r];
        stage_out_rows(t_lane + C::kTmO + ob * D, D / 16, stage, C::kOStride, orow, (any && l > 0.f) ? 1.f / l : 0.f,
                       a.out + td.head * D, a.ld_out);
        tc_fence_before();
        mbar_arrive(&bars[kBarOFree + ob]);
      }
    }
  } else {
    // ========================= softmax warps =========================
    // Thread (row r, half h): query row r = tid % 128 of the tile, keys 64h..64h+63
    // of every block, O columns [h ? kOSplit : 0, h ? D : kOSplit) (their
    // rescale; the epilogue of windowed grids runs on the epilogue warps).
    const int r = tid & (kAttnBM - 1);
    const int h = tid >> 7;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const int oc0 = h ? C::kOSplit : 0, oc1 = h ? D : C::kOSplit;
    float* xchg = reinterpret_cast<float*>(smem + L.xchg);  // [round & 1][half][value][row]
    int xround = 0;
    // Publish (max, sum) of this half and read the other half's, through a
    // 256-thread mbarrier round (bounded wait; double-buffered by round parity).
    auto exchange = [&](float my_max, float my_sum, float& other_max, float& other_sum) -> bool {
      float* buf = xchg + (xround & 1) * (4 * kAttnBM);
      buf[(h * 2 + 0) * kAttnBM + r] = my_max;
      buf[(h * 2 + 1) * kAttnBM + r] = my_sum;
      const int xb = kBarXchg + 4 * (xround & 1) + (warp & 3);
      mbar_arrive(&bars[xb]);
      if (!wait_or_abort(xb, (xround >> 1) & 1)) return false;
      other_max = buf[((h ^ 1) * 2 + 0) * kAttnBM + r];
      other_sum = buf[((h ^ 1) * 2 + 1) * kAttnBM + r];
      ++xround;
      return true;
    };

    // LARGE: A_bias of tile lt_ -> TMEM buffer lt_ & 1 (row r): the staged fp16
    // [relH/scale | relW/scale] row, half h's 32 words. Called once S of the current
    // tile's first block is in, so every QK^T that read the buffer's previous
    // contents has completed. (Windowed grids: the K-loader warps stage it.)
    auto stage_bias = [&](int lt_) -> bool {
      const uint32_t tAB = t_lane + C::kTmAB + (lt_ & 1) * C::kABCols;
      if (!wait_or_abort(kBarABSFull, lt_ & 1)) return false;
      const uint8_t* hrow = smem + L.ab + h * (kAttnBM * 128) + r * 128;
      uint32_t v[32];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 x = *reinterpret_cast<const uint4*>(hrow + ((c ^ (r & 7)) << 4));
        v[4 * c] = x.x;
        v[4 * c + 1] = x.y;
        v[4 * c + 2] = x.z;
        v[4 * c + 3] = x.w;
      }
      tmem_st_32x32b_x32(tAB + h * 32, v);
      mbar_arrive(&bars[kBarABSFree]);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bars[kBarABFull + (lt_ & 1)]);
      return true;
    };
    // This half's O columns / l of tile lt_, stored at the raster token
    // (inverse permutation and head merge)
    // (orow: the output row of this thread's query, looked up a tile ahead)
    auto epilogue = [&](int lt_, int g_last, int orow, int head, float l) -> bool {
      if (g_last >= 0 && !wait_or_abort(kBarODone + (g_last & 1), (g_last >> 1) & 1)) return false;
      tc_fence_after();
      const float inv_l = l > 0.f ? 1.f / l : 0.f;
      const uint32_t tO = t_lane + C::kTmO + (lt_ % C::kO) * D;
      {
        uint4* dst = orow >= 0 ? reinterpret_cast<uint4*>(a.out + static_cast<int64_t>(orow) * a.ld_out + head * D)
                               : nullptr;
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 16) {
          if (c0 < oc0 || c0 >= oc1) continue;
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
      }
      tc_fence_before();
      mbar_arrive(&bars[kBarOFree + lt_ % C::kO]);
      return true;
    };
    // Tile lt_ once per tile (decoded a tile ahead): its query tile, its head and
    // the output row of this thread's query.
    auto tile_info = [&](int lt_, int& qtile, int& head) -> int {
      const TileDesc td = tile_desc<CP>(a, tile_of<C::kTileGroup>(lt_));
      qtile = td.qtile;
      head = td.head;
      return query_out_row(a, td.seq, query_tok<CP>(a, td, td.qtile * kAttnBM + r));
    };

    // SMALL: this half's row-sum shares go to the epilogue warps; the query tile
    // matters to the block list and the mask only with the diagonal
    float* lsum = reinterpret_cast<float*>(smem + L.lsum);
    bool ok = true;
    int orow_cur = -1, orow_next = -1, qt_cur = 0, qt_next = 0, hd_cur = 0, hd_next = 0;
    if (tile_exists(0)) {
      if constexpr (!SMALL) {
        ok = stage_bias(0);
        orow_cur = tile_info(0, qt_cur, hd_cur);
      } else {
        qt_cur = (CP || !a.with_diag) ? 0 : tile_desc<CP>(a, tile_of<C::kTileGroup>(0)).qtile;
      }
    }
    int pend_lt = -1, pend_g = -1, pend_orow = -1, pend_head = 0;  // deferred epilogue
    float pend_l = 0.f;  // this half's share of the pending tile's row sum
    int g = 0;
    for (int lt = 0; ok && tile_exists(lt); ++lt) {
      const int qtile = qt_cur;
      const TileBlocks tb(a, qtile);
      const int my_mb = 2 * qtile + (r >= 64 ? 1 : 0);
      const uint32_t tO = t_lane + C::kTmO + (lt % C::kO) * D;
      if (tile_exists(lt + 1)) {
        if constexpr (SMALL)
          qt_next = (CP || !a.with_diag) ? 0 : tile_desc<CP>(a, tile_of<C::kTileGroup>(lt + 1)).qtile;
        else
          orow_next = tile_info(lt + 1, qt_next, hd_next);
      }
      float m_run = -INFINITY, l_run = 0.f;  // l_run: this half's share of the row sum
      for (int j = 0; j < tb.n; ++j, ++g) {
        const int sbuf = g % C::kS;
        const int kb = tb.at(j);
        if (!(ok = wait_or_abort(kBarSFull + sbuf, (g / C::kS) & 1))) break;
        tc_fence_after();
        // this half's 64 keys: 64-key mask block 2 kb + h
        const int mh = 2 * kb + h;
        // 64-token masks enable the query's own 64-block on the diagonal, 128-token
        // masks the tile's whole diagonal block
        const bool diag_tile = a.with_diag == 2 && kb == tb.qt;
        const bool full = (2 * kb + 1 < tb.nk || diag_tile) && (kb + 1) * kAttnBN <= N;
        const int kvalid = N - kb * kAttnBN - 64 * h;  // keys of this half inside the sequence
        const bool on = full || mh < tb.nk || diag_tile || (a.with_diag == 1 && mh == my_mb);
        // this half's 64 S columns; P of these keys is written back over their first 32
        const uint32_t tSh = t_lane + sbuf * kAttnBN + 64 * h;
        // pass 1: row maximum of the raw logits over both halves (scale > 0 commutes
        // with max); masked keys (off the mask, past N) do not take part
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        {
          uint32_t s[64];
          tmem_ld_32x32b_x32(tSh, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
          tmem_ld_32x32b_x32(tSh + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32]));
          tmem_ld_wait();
          if (full) {
#pragma unroll
            for (int jj = 0; jj < 64; ++jj) mx4[jj & 3] = fmaxf(mx4[jj & 3], __uint_as_float(s[jj]));
          } else if (on) {
#pragma unroll
            for (int jj = 0; jj < 64; ++jj)
              if (jj < kvalid) mx4[jj & 3] = fmaxf(mx4[jj & 3], __uint_as_float(s[jj]));
          }
        }
        float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
        float mx_other, l_other;
        // block 0's exchange also hands over the pending tile's row-sum shares
        if (!(ok = exchange(mx, (!SMALL && j == 0) ? pend_l : 0.f, mx_other, l_other))) break;
        if (!SMALL && j == 0) pend_l += l_other;
        mx = fmaxf(mx, mx_other);
        mx = mx == -INFINITY ? -INFINITY : mx * a.scale_log2;
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
        // tcgen05.ld/st are warp-collective (.sync.aligned): the O rescale runs on
        // the whole warp when any of its rows needs it (the others scale by 1).
        if (__any_sync(0xffffffffu, rescale)) {
          if (!(ok = wait_or_abort(kBarODone + ((g - 1) & 1), ((g - 1) >> 1) & 1))) break;
          tc_fence_after();
#pragma unroll
          for (int c0 = 0; c0 < D; c0 += 16) {
            if (c0 < oc0 || c0 >= oc1) continue;
            uint32_t r16[16];
            tmem_ld_32x32b_x16(tO + c0, r16);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) r16[e] = __float_as_uint(__uint_as_float(r16[e]) * alpha);
            tmem_st_32x32b_x16(tO + c0, r16);
          }
        }
        // pass 2: P = exp2(s * scale log2e - m) as bf16 pairs, 32 keys at a time (S re-read
        // from TMEM): keys 32c .. 32c + 31 of this half go to its columns 16c .. 16c + 15,
        // which pass 2 has already read
        float2 sum2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        float sum4[4] = {0.f, 0.f, 0.f, 0.f};
        const float2 sl2 = make_float2(a.scale_log2, a.scale_log2), nm2 = make_float2(-m_off, -m_off);
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t sc[32];
          tmem_ld_32x32b_x32(tSh + 32 * c, sc);
          tmem_ld_wait();
          uint32_t pk[16];
          if (full) {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const float2 x = fma2(make_float2(__uint_as_float(sc[2 * e]), __uint_as_float(sc[2 * e + 1])), sl2, nm2);
              const float2 p = make_float2(fast_exp2(x.x), fast_exp2(x.y));
              sum2[e & 1] = add2(sum2[e & 1], p);
              pk[e] = pack_bf16x2(p.x, p.y);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const int jj = 32 * c + 2 * e;
              const bool v0 = on && jj < kvalid;
              const bool v1 = on && jj + 1 < kvalid;
              const float p0 = v0 ? fast_exp2(fmaf(__uint_as_float(sc[2 * e]), a.scale_log2, -m_off)) : 0.f;
              const float p1 = v1 ? fast_exp2(fmaf(__uint_as_float(sc[2 * e + 1]), a.scale_log2, -m_off)) : 0.f;
              sum4[e & 3] += p0 + p1;
              pk[e] = pack_bf16x2(p0, p1);
            }
          }
          tmem_st_32x32b_x16(tSh + 16 * c, pk);
        }
        const float2 s2 = add2(sum2[0], sum2[1]);
        const float sum = ((sum4[0] + sum4[1]) + (sum4[2] + sum4[3])) + (s2.x + s2.y);
        l_run = (j == 0 ? 0.f : l_run * alpha) + sum;
        m_run = m_use;
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&bars[kBarPFull + (g & 1)]);

        if (!SMALL && j == 0) {
          // next tile's bias operand and the previous tile's epilogue, off the critical path
          if (tile_exists(lt + 1) && !(ok = stage_bias(lt + 1))) break;
          if (pend_lt >= 0 && !(ok = epilogue(pend_lt, pend_g, pend_orow, pend_head, pend_l))) break;
          pend_lt = -1;
        }
      }
      if (!ok) break;
      if constexpr (SMALL) {
        // this half's row-sum share of tile lt for the epilogue warps; the slot's
        // previous tile (lt - 2) was read before its O buffer was released
        if (!(ok = wait_or_abort(kBarOFree + (lt & 1), ((lt >> 1) & 1) ^ 1))) break;
        lsum[(2 * (lt & 1) + h) * kAttnBM + r] = l_run;
        mbar_arrive(&bars[kBarLFull + (lt & 1)]);
        qt_cur = qt_next;
        continue;
      }
      pend_lt = lt;
      pend_g = tb.n > 0 ? g - 1 : -1;
      pend_orow = orow_cur;
      pend_head = hd_cur;
      pend_l = l_run;
      orow_cur = orow_next;
      qt_cur = qt_next;
      hd_cur = hd_next;
    }
    if (ok && pend_lt >= 0) {  // the last tile's row-sum shares
      float m_unused, l_other;
      if (exchange(0.f, pend_l, m_unused, l_other)) epilogue(pend_lt, pend_g, pend_orow, pend_head, pend_l + l_other);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kAttnMmaWarp) tmem_dealloc(tmem, kAttnTmemCols);
}

// ---------------------------------------------------------------------------
// Global-grid bias pre-pass (below). Windowed grids compute their 16-column
// bands inside the attention kernel, which measured faster than a separate
// pass for 14x14 windows.
// ---------------------------------------------------------------------------
constexpr int kRelThreads = 128;

template <int D, int BW>
struct RelCfg {
  static_assert(BW == 64, "the bias pre-pass serves the global grid (64-wide bands)");
  static constexpr int kNT = 128;                    // table rows (2 win - 1 <= 127)
  static constexpr int kRowBytes = 4 * BW;           // [BW fp16 | BW fp16]
  static constexpr int kStageStride = 2 * kNT + 16;  // per-thread fp16 row of P (+16 B: conflict-free 16-byte ops)
  static constexpr int kTmemCols = 256;
  static constexpr int kSmem = 2 * TileGeom<D>::bytes(kNT) + TileGeom<D>::bytes(kAttnBM) +
                               kAttnBM * kStageStride + 64 + 1024;
};

// relbias_kernel: the rel-pos bias operand of every query, once per query.
// Persistent, two CTAs per SM, tables loaded once per CTA; per 128-query tile of
// an (image, head) row: P_H = Q Th^T and P_W = Q Tw^T on the tensor cores, each
// thread stages its query's P row as fp16 (relX / scale) in shared memory and
// extracts its bands relH[j] = P_H[qh - j + win - 1], relW likewise
// (sam.py:62-73); the tile's 128 output rows ([relH | relW], 256 B each, in
// permuted query order, zero rows for queries past N) are contiguous in
// bias_ws, so each warp copies its 32 rows out with coalesced 16-byte stores.
// The next tile's Q rows load while the current tile's bands are extracted.
template <int D, int BW>
__global__ void __launch_bounds__(kRelThreads) relbias_kernel(const AttnParams a) {
  using TG = TileGeom<D>;
  using RC = RelCfg<D, BW>;
  constexpr int kNT = RC::kNT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  const uint32_t sTh = sb, sTw = sb + TG::bytes(kNT), sQ = sb + 2 * TG::bytes(kNT);
  uint8_t* stage = smem + 2 * TG::bytes(kNT) + TG::bytes(kAttnBM);  // per-thread rows
  uint64_t* bar = reinterpret_cast<uint64_t*>(stage + kAttnBM * RC::kStageStride);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bar + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int N = a.N, win = a.win;

  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_holder, RC::kTmemCols);
    tmem_relinquish();
  }
  // tables, once per CTA (rows past 2 win - 1 zero)
  const int trows = 2 * win - 1;
  if (tid < kNT) {
#pragma unroll
    for (int c = 0; c < TG::kChunks; ++c) {
      cp_async16(tile_chunk_addr<D>(sTh, kNT, tid, c), tid < trows ? a.th + tid * D + c * 8 : a.th,
                 tid < trows ? 16u : 0u);
      cp_async16(tile_chunk_addr<D>(sTw, kNT, tid, c), tid < trows ? a.tw + tid * D + c * 8 : a.tw,
                 tid < trows ? 16u : 0u);
    }
  }
  // this thread's query token of a tile, and its Q row into sQ
  auto tile_token = [&](int tile) -> int {
    const int row = tile / a.n_tiles, qtile = tile - row * a.n_tiles;
    const int p = qtile * kAttnBM + tid;
    return p < N ? __ldg(a.perm + static_cast<int64_t>(row) * N + p) : -1;
  };
  auto load_q = [&](int tile, int t) {
    const int row = tile / a.n_tiles;
    const int seq = row / a.heads, head = row - seq * a.heads;
    const __nv_bfloat16* q_src =
        t >= 0 ? a.qkv + (static_cast<int64_t>(seq) * N + t) * a.ld_qkv + head * D : nullptr;
#pragma unroll
    for (int c = 0; c < TG::kChunks; ++c)
      cp_async16(tile_chunk_addr<D>(sQ, kAttnBM, tid, c), q_src != nullptr ? q_src + c * 8 : a.qkv,
                 q_src != nullptr ? 16u : 0u);
  };
  int t_cur = -1;
  if (static_cast<int>(blockIdx.x) < a.total_tiles) {
    t_cur = tile_token(blockIdx.x);
    load_q(blockIdx.x, t_cur);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint32_t t_lane = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  uint8_t* my_stage = stage + tid * RC::kStageStride;
  bool ok = true;
  int iter = 0;
  for (int tile = blockIdx.x; ok && tile < a.total_tiles; tile += gridDim.x, ++iter) {
    cp_async_wait_all();
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();  // Q (and, the first time, the tables) of every thread are in
    tc_fence_after();
    if (tid == 0) {
      const uint32_t idesc = make_idesc_bf16(kAttnBM, kNT, 0, 0);
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        umma_f16_ss(tmem, kmajor_desc<D>(sQ, kAttnBM, ks), kmajor_desc<D>(sTh, kNT, ks), idesc, ks > 0);
        umma_f16_ss(tmem + kNT, kmajor_desc<D>(sQ, kAttnBM, ks), kmajor_desc<D>(sTw, kNT, ks), idesc, ks > 0);
      }
      umma_commit(bar);
    }
    ok = __syncthreads_and(mbar_wait_slow(bar, iter & 1));
    tc_fence_after();
    // sQ is free again: the next tile's Q rows load during the extraction
    const int t = t_cur;
    const int next = tile + static_cast<int>(gridDim.x);
    if (ok && next < a.total_tiles) {
      t_cur = tile_token(next);
      load_q(next, t_cur);
    }
    if (ok) {
      const int qh = t >= 0 ? t / win : 0;
      const int qw = t >= 0 ? t - qh * win : 0;
      uint32_t bh[32], bw[32];
#pragma unroll
      for (int tab = 0; tab < 2; ++tab) {
        // P row of this table -> fp16 (x 1/scale) in my_stage; all four loads in flight before the wait
        uint32_t rr[kNT / 32][32];
#pragma unroll
        for (int q = 0; q < kNT / 32; ++q) tmem_ld_32x32b_x32(t_lane + tab * kNT + 32 * q, rr[q]);
        tmem_ld_wait();
#pragma unroll
        for (int q = 0; q < kNT / 32; ++q) {
          uint32_t hw[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const __half2 h2 = __floats2half2_rn(__uint_as_float(rr[q][2 * i]) * a.inv_scale,
                                                 __uint_as_float(rr[q][2 * i + 1]) * a.inv_scale);
            hw[i] = *reinterpret_cast<const uint32_t*>(&h2);
          }
          uint4* sp = reinterpret_cast<uint4*>(my_stage + q * 64);
#pragma unroll
          for (int i = 0; i < 4; ++i) sp[i] = make_uint4(hw[4 * i], hw[4 * i + 1], hw[4 * i + 2], hw[4 * i + 3]);
        }
        if (tab == 0) relbias_band<64>(my_stage, qh, win, bh);
        else relbias_band<64>(my_stage, qw, win, bw);
      }
      // output row [relH | relW] (zero for queries past N) back into my_stage
      uint4* sp = reinterpret_cast<uint4*>(my_stage);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        sp[i] = t >= 0 ? make_uint4(bh[4 * i], bh[4 * i + 1], bh[4 * i + 2], bh[4 * i + 3]) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        sp[8 + i] =
            t >= 0 ? make_uint4(bw[4 * i], bw[4 * i + 1], bw[4 * i + 2], bw[4 * i + 3]) : make_uint4(0u, 0u, 0u, 0u);
      __syncwarp();
      // the warp's 32 rows are contiguous in bias_ws: 16 lanes per 256-byte row
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(a.bias_ws) +
                                            (static_cast<int64_t>(tile) * kAttnBM + warp * 32) * RC::kRowBytes);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int rr = 2 * i + (lane >> 4), c16 = lane & 15;
        dst[rr * 16 + c16] =
            *reinterpret_cast<const uint4*>(stage + (warp * 32 + rr) * RC::kStageStride + c16 * 16);
      }
    }
    tc_fence_before();
    __syncthreads();  // TMEM and the staging rows are reused by the next tile
    tc_fence_after();
  }
  cp_async_wait_all();
  if (warp == 0) tmem_dealloc(tmem, RC::kTmemCols);
}

size_t sparse_attn_workspace_size(int n_seq, int heads, int win) {
  if (n_seq <= 0 || heads <= 0 || win <= 16) return 0;  // windowed grids compute the bias in-kernel
  const int64_t n_tiles = (static_cast<int64_t>(win) * win + kAttnBM - 1) / kAttnBM;
  return static_cast<size_t>(n_seq) * heads * n_tiles * kAttnBM * 128 * 2;
}

template <int D, bool SMALL, bool CP>
static int launch_attn(const AttnParams& p, const CUtensorMap& tm_tile, cudaStream_t stream) {
  const AttnLayout<D, SMALL> L;
  using RC = RelCfg<D, 64>;
  static PerDeviceOnce configured;
  const int dev = current_device();
  const int st = configured.run(dev, [&L] {
    if (cudaFuncSetAttribute(sparse_attn_kernel<D, SMALL, CP>, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total) !=
        cudaSuccess)
      return SSAM_ERR_CUDA;
    if (!SMALL && cudaFuncSetAttribute(relbias_kernel<D, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       RC::kSmem) != cudaSuccess)
      return SSAM_ERR_CUDA;
    return SSAM_OK;
  });
  if (st != SSAM_OK) return st;
  const int sms = num_sms(dev);
  if (!SMALL) {
    // persistent bias pre-pass, two CTAs per SM (256 TMEM columns each)
    const int want = sms * (512 / RC::kTmemCols);
    relbias_kernel<D, 64><<<p.total_tiles < want ? p.total_tiles : want, kRelThreads, RC::kSmem, stream>>>(p);
    if (cudaGetLastError() != cudaSuccess) return SSAM_ERR_CUDA;
  }
  // One persistent CTA per SM (the plan exceeds half the SM's shared memory),
  // so its 512 TMEM columns are always available.
  const int smem = L.total > 116 * 1024 ? L.total : 116 * 1024;
  const int grid = p.total_tiles < sms ? p.total_tiles : sms;
  sparse_attn_kernel<D, SMALL, CP><<<grid, attn_threads(SMALL), smem, stream>>>(p, tm_tile);
  return status_from_cuda(cudaGetLastError());
}

int sparse_attn_fwd(const void* qkv, int64_t ld_qkv, int n_seq, int heads, int win, int d, const void* rel_pos_h,
                    const void* rel_pos_w, const int32_t* perm, int n_init_blocks, int n_block, int with_diag,
                    float scale, void* out, int64_t ld_out, const int32_t* out_rows, int grid_h, int grid_w,
                    const void* pad_row, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (qkv == nullptr || rel_pos_h == nullptr || rel_pos_w == nullptr || perm == nullptr || out == nullptr)
    return SSAM_ERR_INVALID;
  if (n_seq <= 0 || heads <= 0 || win <= 0 || n_init_blocks < 0) return SSAM_ERR_INVALID;
  if (n_block != 64 && n_block != 128) return SSAM_ERR_UNSUPPORTED;
  if (n_init_blocks == 0 && !with_diag) return SSAM_ERR_INVALID;  // every query would have no key
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
  // the kernel's keep bar counts 64-token blocks (n < n_init of 128 tokens = n64 < 2 n_init)
  const int nblk64 = (p.N + kMaskBlk - 1) / kMaskBlk;
  p.n_init = n_block == 128 ? (n_init_blocks < nblk64 ? 2 * n_init_blocks : nblk64) : n_init_blocks;
  p.with_diag = with_diag ? (n_block == 128 ? 2 : 1) : 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ld_out = ld_out;
  p.out_rows = out_rows;
  p.pad_row = static_cast<const __nv_bfloat16*>(pad_row);
  if (pad_row != nullptr && !aligned16(pad_row)) return SSAM_ERR_ALIGN;
  p.inv_scale = 1.0f / scale;
  p.n_tiles = (p.N + kAttnBM - 1) / kAttnBM;
  const bool small = win <= 16;
  int64_t total = static_cast<int64_t>(p.n_tiles) * n_seq * heads;
  // query compaction: windowed grids without the diagonal whose image grid is known
  p.wpi = p.nww = p.grid_h = p.grid_w = p.img_tiles = p.row_tiles = 0;
  p.kt_in = p.kt_col = p.kt_row = p.kt_corner = 0;
  if (grid_h < 0 || grid_w < 0) return SSAM_ERR_INVALID;
  if (small && !with_diag && grid_h > 0 && grid_w > 0) {
    const int64_t nwh = (grid_h + win - 1) / win, nww = (grid_w + win - 1) / win;
    if (nwh * nww > INT32_MAX / 4) return SSAM_ERR_UNSUPPORTED;
    const int wpi = static_cast<int>(nwh * nww);
    if (n_seq % wpi != 0) return SSAM_ERR_INVALID;  // whole images of windows
    const int h_last = grid_h - static_cast<int>(nwh - 1) * win, w_last = grid_w - static_cast<int>(nww - 1) * win;
    auto tiles = [](int hr, int wr) { return (hr * wr + kAttnBM - 1) / kAttnBM; };
    p.kt_in = tiles(win, win);
    p.nwh = static_cast<int>(nwh);
    p.w_last = w_last;
    p.kt_col = tiles(win, w_last);
    p.kt_row = tiles(h_last, win);
    p.kt_corner = tiles(h_last, w_last);
    const int64_t row_tiles = heads * ((nww - 1) * p.kt_in + p.kt_col);
    const int64_t img_tiles = (nwh - 1) * row_tiles + heads * ((nww - 1) * p.kt_row + p.kt_corner);
    if (img_tiles > INT32_MAX) return SSAM_ERR_UNSUPPORTED;
    p.wpi = wpi;
    p.nww = static_cast<int>(nww);
    p.grid_h = grid_h;
    p.grid_w = grid_w;
    p.row_tiles = static_cast<int>(row_tiles);
    p.img_tiles = static_cast<int>(img_tiles);
    auto rcp = [](int64_t v) { return static_cast<float>(1.0 / static_cast<double>(v)); };
    p.r_img_tiles = rcp(img_tiles);
    p.r_row_tiles = rcp(row_tiles);
    p.r_span_in = rcp(static_cast<int64_t>(heads) * p.kt_in);
    p.r_span_row = rcp(static_cast<int64_t>(heads) * p.kt_row);
    p.r_win = rcp(win);
    p.r_wlast = rcp(w_last);
    // the decode's fp32 divisions are exact below 2^24
    if (static_cast<int64_t>(n_seq) * heads * 2 >= (1 << 24)) return SSAM_ERR_UNSUPPORTED;
    total = img_tiles * (n_seq / wpi);
  }
  if (total > INT32_MAX || static_cast<int64_t>(n_seq) * p.N > INT32_MAX) return SSAM_ERR_UNSUPPORTED;
  p.total_tiles = static_cast<int>(total);
  p.bias_ws = nullptr;
  if (!small) {
    const size_t need = sparse_attn_workspace_size(n_seq, heads, win);
    if (workspace == nullptr || workspace_bytes < need) return SSAM_ERR_INVALID;
    if (!aligned16(workspace)) return SSAM_ERR_ALIGN;
    p.bias_ws = static_cast<__half*>(workspace);
  }
  // qkv as a [n_seq * N, 3C] tensor for the windowed tiles' Q rows (TMA tile copies)
  CUtensorMap tm_tile;
  const int st = make_tmap_2d_bf16(&tm_tile, qkv, static_cast<uint64_t>(n_seq) * p.N, 3 * static_cast<uint64_t>(C),
                                   ld_qkv, 16, kAttnBM, CU_TENSOR_MAP_SWIZZLE_32B);
  if (st != SSAM_OK) return st;
  const bool cp = p.wpi > 0;  // query compaction (windowed grids with an image grid)
  if (d == 64)
    return small ? (cp ? launch_attn<64, true, true>(p, tm_tile, stream) : launch_attn<64, true, false>(p, tm_tile, stream))
                 : launch_attn<64, false, false>(p, tm_tile, stream);
  return small ? (cp ? launch_attn<80, true, true>(p, tm_tile, stream) : launch_attn<80, true, false>(p, tm_tile, stream))
               : launch_attn<80, false, false>(p, tm_tile, stream);
}

}  // namespace ssam
