"""Token-order restatements (numpy) — test infrastructure only.

Each function cites the reference code it restates. Scores are computed in
fp64; every ranking is stable (ties -> lowest index), which is the tie rule
the B200 kernels implement. The reference's own torch.argsort / topk are not
stable (F6 in the survey): inside exactly tied runs it may order differently.
"""
from __future__ import annotations

import math

import numpy as np


def morton_keys(H: int, W: int) -> np.ndarray:
    """Z-curve key of every raster cell: row bit i -> 2i+1, col bit i -> 2i
    (algos/sparsesam/z_utils.py:35-49 with num_dims=2, :71 for num_bits)."""
    num_bits = max(1, math.ceil(math.log2(max(H, W))))
    r, c = np.meshgrid(np.arange(H, dtype=np.int64), np.arange(W, dtype=np.int64), indexing="ij")
    r, c = r.ravel(), c.ravel()
    z = np.zeros(H * W, dtype=np.int64)
    for i in range(num_bits):
        z |= ((r >> i) & 1) << (2 * i + 1)
        z |= ((c >> i) & 1) << (2 * i)
    return z


def zorder(H: int, W: int) -> tuple[np.ndarray, np.ndarray]:
    """(perm, inv_perm): perm = argsort(key), inv = argsort(perm) (z_utils.py:65-85)."""
    perm = np.argsort(morton_keys(H, W), kind="stable")
    inv = np.argsort(perm, kind="stable")
    return perm, inv


def hilbert_keys(H: int, W: int) -> np.ndarray:
    """Hilbert index of every raster cell, row as axis 0 and column as axis 1.

    Skilling's transpose algorithm (J. Skilling, "Programming the Hilbert
    curve", AIP Conf. Proc. 707, 2004) as the reference applies it: the axes to
    transposed form (algos/sparsesam/hilbert_utils.py:55-76), then the bits
    interleaved with axis 0 the higher of each pair (:28-33), over
    p = max(1, ceil(log2(max(H, W)))) bits (:118)."""
    p = max(1, math.ceil(math.log2(max(H, W))))
    r, c = np.meshgrid(np.arange(H, dtype=np.int64), np.arange(W, dtype=np.int64), indexing="ij")
    x0, x1 = r.ravel().copy(), c.ravel().copy()
    top = 1 << (p - 1)
    q = top
    while q > 1:                                     # undo excess work, axis 0 then axis 1
        low = q - 1
        x0 = np.where((x0 & q) != 0, x0 ^ low, x0)
        hi = (x1 & q) != 0
        t = (x0 ^ x1) & low
        x0, x1 = np.where(hi, x0 ^ low, x0 ^ t), np.where(hi, x1, x1 ^ t)
        q >>= 1
    x1 = x1 ^ x0                                     # Gray encode
    t = np.zeros_like(x0)
    q = top
    while q > 1:
        t = np.where((x1 & q) != 0, t ^ (q - 1), t)
        q >>= 1
    x0, x1 = x0 ^ t, x1 ^ t
    h = np.zeros_like(x0)
    for i in range(p):
        h |= ((x0 >> (p - 1 - i)) & 1) << (2 * p - 1 - 2 * i)
        h |= ((x1 >> (p - 1 - i)) & 1) << (2 * p - 2 - 2 * i)
    return h


def hilbert_order(H: int, W: int) -> tuple[np.ndarray, np.ndarray]:
    """(perm, inv_perm) of the Hilbert curve (hilbert_utils.py:108-129); keys are unique."""
    perm = np.argsort(hilbert_keys(H, W), kind="stable")
    inv = np.argsort(perm, kind="stable")
    return perm, inv


def stripe_sort(k: np.ndarray, H: int, W: int, group_size: int = 4,
                perm_mode: str = "z_interleave_sort",
                base_perm: np.ndarray | None = None):
    """Restatement of tile_stride_matching (algos/sparsesam/sam.py:105-164).

    k: (R, H*W, C) values (any float dtype; promoted to fp64).
    Returns int64 (perm, inv_perm, inv_perm_group), each (R, H*W).
    """
    space, layout, ranking = perm_mode.split("_")
    assert space in ("z", "hilbert") and layout in ("interleave", "naive") and ranking in ("sort", "nosort")
    N = H * W
    assert N % group_size == 0
    G, gs = N // group_size, group_size
    if base_perm is None:
        base_perm = zorder(H, W)[0] if space == "z" else hilbert_order(H, W)[0]   # sam.py:128-132
    k = np.asarray(k, dtype=np.float64)
    R = k.shape[0]
    xg = k[:, base_perm, :].reshape(R, G, gs, -1)
    if ranking == "sort":
        score = _group_score(xg)
        grp_rank = np.argsort(-score, axis=-1, kind="stable")              # sam.py:150, stable ties
    else:
        grp_rank = np.broadcast_to(np.arange(G), (R, G))
    all_raster = base_perm.reshape(G, gs)[grp_rank]                       # (R, G, gs), sam.py:155-156
    perm_group = all_raster.reshape(R, N)
    perm = all_raster.transpose(0, 2, 1).reshape(R, N) if layout == "interleave" else perm_group.copy()
    inv = np.argsort(perm, axis=1, kind="stable")                          # sam.py:162
    inv_group = np.argsort(perm_group, axis=1, kind="stable")              # sam.py:163
    return perm, inv, inv_group


def _group_score(xg: np.ndarray) -> np.ndarray:
    """fp64 group score of tile_stride_matching (sam.py:139-149) for xg (R, G, gs, C).

    The row sum of the cosine-similarity matrix sim = n n^T (sam.py:142-143) is
    computed as <n_g, sum_j n_j>, which is the same sum in exact arithmetic;
    evaluated elementwise it gives exactly equal scores to exactly equal groups
    (a BLAS product can round identical rows differently)."""
    G = xg.shape[1]
    grp_std = xg.std(axis=2, ddof=1).mean(axis=-1)                        # sam.py:139
    grp_mean = xg.mean(axis=2)                                             # sam.py:140
    nrm = np.sqrt((grp_mean * grp_mean).sum(-1, keepdims=True))
    gm = grp_mean / np.maximum(nrm, 1e-12)                                 # F.normalize, sam.py:141
    rowsum = (gm * gm.sum(axis=1, keepdims=True)).sum(-1)                  # sim.sum(-1), sam.py:142-143
    avg_sim = (rowsum - 1.0) / max(G - 1, 1)
    dissim = -avg_sim
    eps = 1e-6
    std_n = (grp_std - grp_std.mean(-1, keepdims=True)) / (grp_std.std(-1, ddof=1, keepdims=True) + eps)
    dis_n = (dissim - dissim.mean(-1, keepdims=True)) / (dissim.std(-1, ddof=1, keepdims=True) + eps)
    return std_n + dis_n                                                   # sam.py:147-149


def group_scores(k: np.ndarray, H: int, W: int, group_size: int = 4) -> np.ndarray:
    """The fp64 group scores of stripe_sort for K rows (R, H*W, C) (tie diagnostics)."""
    N = H * W
    G = N // group_size
    base = zorder(H, W)[0]
    xg = np.asarray(k, dtype=np.float64)[:, base, :].reshape(k.shape[0], G, group_size, -1)
    return _group_score(xg)


def a_shape_n_init(N: int, n_block: int, ratio: float, is_global: bool) -> int:
    """n_init_blocks of the A-shape mask (sam.py:219-223)."""
    num_n = (N + n_block - 1) // n_block
    n_keep = int(ratio * num_n)
    return n_keep if is_global else n_keep + 1


def a_shape_mask(N: int, m_block: int, n_block: int, n_init: int, with_diag: bool) -> np.ndarray:
    """Enabled (m, n) block pairs: n < n_init or (diag and n == m) (flash_attn.py:132-145)."""
    nm, nn = -(-N // m_block), -(-N // n_block)
    m = np.arange(nm)[:, None]
    n = np.arange(nn)[None, :]
    return ((n < n_init) | (with_diag & (n == m))).astype(np.uint8)


def keep_select(inv_perm_group: np.ndarray, B: int, heads: int, keep_n: int) -> np.ndarray:
    """Keep set of the Residual-Consistency MLP (sam.py:277-280): the keep_n tokens
    with the smallest head-mean rank, ties -> lowest token index. (B, keep_n) int64."""
    N = inv_perm_group.shape[-1]
    sums = np.asarray(inv_perm_group, dtype=np.int64).reshape(B, heads, N).sum(1)
    return np.argsort(sums, axis=1, kind="stable")[:, :keep_n]


def keep_n_for(ratio: float, N: int) -> int:
    """keep_n = max(1, round(ratio * N)) (sam.py:277; Python round-half-even)."""
    return max(1, round(ratio * N))


def zstride_keep(H: int, W: int, ratio: float) -> np.ndarray:
    """Static keep set of the SAM3 MLP-merge variant (algos/sparsesam/sam3.py:49-71):
    keep_n = min(max(1, round(ratio N)), N) Morton positions at a uniform stride,
    pos_i = round(float32(i) * float32(N / keep_n)) (ties to even, as torch.round),
    clamped to [0, N - 1], mapped to raster indices through the Morton order. int64."""
    N = H * W
    keep_n = min(max(1, round(ratio * N)), N)
    zperm = zorder(H, W)[0]
    pos = np.rint(np.arange(keep_n, dtype=np.float32) * np.float32(N / keep_n)).astype(np.int64)
    return zperm[np.clip(pos, 0, N - 1)]
