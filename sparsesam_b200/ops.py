"""Torch-facing wrappers over the C ABI (include/sparsesam.h).

Each wrapper checks dtypes/devices/contiguity, passes raw device pointers and
torch's current CUDA stream to the shared library, and raises SparseSAMError on
a non-zero status. There is no CPU or PyTorch fallback: a tensor that is not on
a CUDA device is rejected.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import SSAM_EPI_ADD_F32, SSAM_EPI_BF16, SSAM_EPI_F32, SSAM_EPI_GELU_BF16  # noqa: F401


class KernelTimer:
    """Optional CUDA-event timing of GEMM / attention launches on the launching
    stream. Inactive by default; bench.py turns it on to measure per-kernel time."""

    active = False
    records: list = []   # (kind, flops, start_event, end_event)

    @classmethod
    def begin(cls):
        if not cls.active:
            return None
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        return ev

    @classmethod
    def end(cls, start, kind: str, flops: float):
        if start is None:
            return
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        cls.records.append((kind, flops, start, ev))


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _check_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("sparsesam_b200 ops run on CUDA tensors only (no CPU fallback)")


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _rowmajor(t: torch.Tensor, name: str) -> int:
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be a 2-D row-major tensor (unit column stride)")
    return t.stride(0)


def gemm_bf16(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor | None = None, *,
              epilogue: int = SSAM_EPI_BF16, out: torch.Tensor | None = None,
              out_rows: torch.Tensor | None = None, k_split: int = 1) -> torch.Tensor:
    """acc = a @ b.T (a: M x K bf16, b: N x K bf16) with a fused epilogue.

    SSAM_EPI_BF16 / SSAM_EPI_GELU_BF16 write bf16 `out` (M x N, allocated when
    None), SSAM_EPI_F32 fp32 `out`; SSAM_EPI_ADD_F32 accumulates into the fp32
    `out`. With `out_rows` (int32) accumulator row r goes to out[out_rows[r]]
    (-1 skips the row) for every epilogue. `k_split` > 1 marks a GEMM whose K
    holds that many terms of one product (the fp32-accurate [hi | lo | hi]
    split): its algorithmic work, as KernelTimer records it, is 2*M*N*K/k_split.
    """
    _check_cuda(a, b, bias, out, out_rows)
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise TypeError("gemm_bf16 takes bf16 operands")
    M, K = a.shape
    N, K2 = b.shape
    if K != K2:
        raise ValueError(f"inner dimensions differ: {K} vs {K2}")
    lda, ldb = _rowmajor(a, "a"), _rowmajor(b, "b")
    if bias is not None and (bias.dtype != torch.float32 or bias.numel() != N or not bias.is_contiguous()):
        raise ValueError("bias must be a contiguous fp32 vector of length N")
    if epilogue == SSAM_EPI_F32:
        if out is None:
            out = torch.empty(M, N, device=a.device, dtype=torch.float32)
        elif out.dtype != torch.float32 or out.shape[0] < M:
            raise ValueError("out must be fp32 with at least M rows")
    elif epilogue == SSAM_EPI_ADD_F32:
        if out is None or out.dtype != torch.float32:
            raise ValueError("SSAM_EPI_ADD_F32 needs an fp32 `out`")
        if out_rows is None and out.shape[0] < M:
            raise ValueError("out has fewer than M rows")
    else:
        if out is None:
            out = torch.empty(M, N, device=a.device, dtype=torch.bfloat16)
        elif out.dtype != torch.bfloat16 or out.shape[0] < M:
            raise ValueError("out must be bf16 with at least M rows")
    if out_rows is not None and (out_rows.dtype != torch.int32 or out_rows.numel() < M):
        raise ValueError("out_rows must be int32 with at least M entries")
    ldo = _rowmajor(out, "out")
    t0 = KernelTimer.begin()
    _lib.call("ssam_gemm_bf16", a.data_ptr(), lda, b.data_ptr(), ldb, M, N, K, _ptr(bias), epilogue,
              out.data_ptr(), ldo, _ptr(out_rows), _stream(a))
    KernelTimer.end(t0, "gemm", 2.0 * M * N * K / k_split)
    return out


def device_error(reset: bool = True) -> int:
    """Synchronise and return (optionally clearing) the library's device error flag."""
    return _lib.load().ssam_device_error(1 if reset else 0)


# ---------------------------------------------------------------------------
# Token order (a1, a2), mask parameters (a7), keep set (a10)
# ---------------------------------------------------------------------------
def zorder(H: int, W: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """Morton order of an H x W grid: (perm, inv_perm), int32 on `device`."""
    perm = torch.empty(H * W, dtype=torch.int32, device=device)
    inv = torch.empty_like(perm)
    _lib.call("ssam_zorder", H, W, perm.data_ptr(), inv.data_ptr(), torch.cuda.current_stream(perm.device).cuda_stream)
    return perm, inv


def hilbert_order(H: int, W: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """Hilbert-curve order of an H x W grid: (perm, inv_perm), int32 on `device`."""
    perm = torch.empty(H * W, dtype=torch.int32, device=device)
    inv = torch.empty_like(perm)
    _lib.call("ssam_hilbert_order", H, W, perm.data_ptr(), inv.data_ptr(),
              torch.cuda.current_stream(perm.device).cuda_stream)
    return perm, inv


_LAYOUTS = {"interleave": 0, "naive": 1}
_RANKINGS = {"sort": 0, "nosort": 1}


def parse_perm_mode(perm_mode: str) -> tuple[str, int, int]:
    """`<space>_<layout>_<ranking>` -> (space, layout code, ranking code) (sam.py:118-123)."""
    parts = perm_mode.split("_")
    if len(parts) != 3:
        raise ValueError(f"perm_mode must be <space>_<layout>_<ranking>, got {perm_mode!r}")
    space, layout, ranking = parts
    if space not in ("z", "hilbert"):
        raise ValueError(f"unknown space {space!r}")
    if layout not in _LAYOUTS:
        raise ValueError(f"unknown layout {layout!r}")
    if ranking not in _RANKINGS:
        raise ValueError(f"unknown ranking {ranking!r}")
    return space, _LAYOUTS[layout], _RANKINGS[ranking]


def stripe_sort_perm(k: torch.Tensor, n_seq: int, heads: int, H: int, W: int, d: int, base_perm: torch.Tensor,
                     group_size: int = 4, layout: int = 0, ranking: int = 0, ld: int | None = None):
    """Stripe-Sort permutation of every (sequence, head) row of K.

    `k` addresses K as k[(s*H*W + t)*ld + h*d + c] (a column view into a qkv
    buffer works). Returns int32 (perm, inv_perm, inv_perm_group) of shape
    (n_seq*heads, H*W)."""
    _check_cuda(k, base_perm)
    if k.dtype != torch.bfloat16 or base_perm.dtype != torch.int32:
        raise TypeError("k must be bf16 and base_perm int32")
    if ld is None:
        ld = k.stride(0) if k.dim() == 2 else heads * d
    rows, N = n_seq * heads, H * W
    perm = torch.empty(rows, N, dtype=torch.int32, device=k.device)
    inv = torch.empty_like(perm)
    inv_g = torch.empty_like(perm)
    _lib.call("ssam_stripe_sort_perm", k.data_ptr(), ld, n_seq, heads, H, W, d, group_size, layout, ranking,
              base_perm.data_ptr(), perm.data_ptr(), inv.data_ptr(), inv_g.data_ptr(), _stream(k))
    return perm, inv, inv_g


def a_shape_n_init(N: int, n_block: int, ratio: float, is_global: bool) -> int:
    v = _lib.load().ssam_a_shape_n_init(N, n_block, float(ratio), 1 if is_global else 0)
    if v < 0:
        raise ValueError(f"invalid A-shape parameters N={N} n_block={n_block} ratio={ratio}")
    return v


def a_shape_mask(N: int, m_block: int, n_block: int, n_init: int, with_diag: bool) -> torch.Tensor:
    num_m, num_n = -(-N // m_block), -(-N // n_block)
    mask = torch.empty(num_m, num_n, dtype=torch.uint8)
    _lib.call("ssam_a_shape_mask", N, m_block, n_block, n_init, 1 if with_diag else 0, mask.data_ptr())
    return mask


def keep_select(inv_perm_group: torch.Tensor, B: int, heads: int, keep_n: int):
    """(idx (B, keep_n), rows (B*keep_n,)) of the Residual-Consistency keep set."""
    _check_cuda(inv_perm_group)
    if inv_perm_group.dtype != torch.int32 or not inv_perm_group.is_contiguous():
        raise TypeError("inv_perm_group must be contiguous int32")
    N = inv_perm_group.shape[-1]
    idx = torch.empty(B, keep_n, dtype=torch.int32, device=inv_perm_group.device)
    rows = torch.empty(B * keep_n, dtype=torch.int32, device=inv_perm_group.device)
    _lib.call("ssam_keep_select", inv_perm_group.data_ptr(), B, heads, N, keep_n, idx.data_ptr(), rows.data_ptr(),
              _stream(inv_perm_group))
    return idx, rows


def zstride_keep_n(N: int, ratio: float) -> int:
    """keep_n of the SAM3 MLP-merge keep set: min(max(1, round(ratio*N)), N) (sam3.py:62-63)."""
    v = _lib.load().ssam_zstride_keep_n(N, float(ratio))
    if v < 0:
        raise ValueError(f"ratio must be in (0, 1], got {ratio}")
    return v


def zstride_keep(H: int, W: int, ratio: float, B: int, device):
    """(idx (keep_n,), rows (B*keep_n,)) of the SAM3 static keep set (sam3.py:49-71):
    raster indices of tokens sampled at a uniform stride along the Morton order,
    and their rows b*H*W + idx in a (B*H*W, C) token matrix."""
    keep_n = zstride_keep_n(H * W, ratio)
    idx = torch.empty(keep_n, dtype=torch.int32, device=device)
    rows = torch.empty(B * keep_n, dtype=torch.int32, device=device)
    _lib.call("ssam_zstride_keep", H, W, keep_n, B, idx.data_ptr(), rows.data_ptr(),
              torch.cuda.current_stream(idx.device).cuda_stream)
    return idx, rows


# ---------------------------------------------------------------------------
# Attention (a3-a6, a8)
# ---------------------------------------------------------------------------
def sparse_attn(qkv: torch.Tensor, n_seq: int, heads: int, win: int, d: int, rel_pos_h: torch.Tensor,
                rel_pos_w: torch.Tensor, perm: torch.Tensor, n_init_blocks: int, with_diag: bool, scale: float,
                out: torch.Tensor | None = None, out_rows: torch.Tensor | None = None,
                n_block: int = 64, grid: tuple[int, int] | None = None,
                pad_row: torch.Tensor | None = None) -> torch.Tensor:
    """Block-sparse attention of every (sequence, head) row; output in raster order (n_seq*N, heads*d),
    or, with `out_rows` (int32 [n_seq*N], -1 skips), (sequence, token) written to row out_rows[s*N + t].
    The A-shape mask is defined on n_block-token blocks (64 or 128). `grid` = (H, W): the
    sequences are the window_partition windows of H x W token grids, and only their real
    tokens are computed as queries (windowed grids without the diagonal). `pad_row` (bf16
    [3*heads*d], with `grid`): the qkv row of the windows' zero padding, read for padding keys
    instead of their qkv rows."""
    _check_cuda(qkv, rel_pos_h, rel_pos_w, perm, out, out_rows, pad_row)
    if pad_row is not None and (grid is None or pad_row.dtype != torch.bfloat16 or not pad_row.is_contiguous()
                                or pad_row.numel() != 3 * heads * d):
        raise ValueError("pad_row: contiguous bf16 [3*heads*d], with `grid`")
    if qkv.dtype != torch.bfloat16 or rel_pos_h.dtype != torch.bfloat16 or rel_pos_w.dtype != torch.bfloat16:
        raise TypeError("qkv and rel-pos tables must be bf16")
    if perm.dtype != torch.int32 or not perm.is_contiguous():
        raise TypeError("perm must be contiguous int32")
    if not (rel_pos_h.is_contiguous() and rel_pos_w.is_contiguous()):
        raise ValueError("rel-pos tables must be contiguous")
    ld = _rowmajor(qkv, "qkv")
    N = win * win
    if out_rows is not None and (out_rows.dtype != torch.int32 or out_rows.numel() < n_seq * N
                                 or not out_rows.is_contiguous()):
        raise ValueError("out_rows must be contiguous int32 with n_seq*N entries")
    if out is None:
        if out_rows is not None:
            raise ValueError("out_rows needs an explicit `out`")
        out = torch.empty(n_seq * N, heads * d, dtype=torch.bfloat16, device=qkv.device)
    ld_out = _rowmajor(out, "out")
    ws_bytes = int(_lib.load().ssam_sparse_attn_workspace_size(n_seq, heads, win, d))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=qkv.device) if ws_bytes else None
    t0 = KernelTimer.begin()
    _lib.call("ssam_sparse_attn_fwd", qkv.data_ptr(), ld, n_seq, heads, win, d, rel_pos_h.data_ptr(),
              rel_pos_w.data_ptr(), perm.data_ptr(), n_init_blocks, n_block, 1 if with_diag else 0, float(scale),
              out.data_ptr(), ld_out, _ptr(out_rows), grid[0] if grid else 0, grid[1] if grid else 0, _ptr(pad_row),
              _ptr(ws), ws_bytes, _stream(qkv), launches=2 if ws_bytes else 1)
    KernelTimer.end(t0, "attention_global" if ws_bytes else "attention_window",
                    attention_flops(n_seq * heads, N, d, n_init_blocks, with_diag, n_block))
    return out


def attention_flops(rows: int, N: int, d: int, n_init: int, with_diag: bool, block: int = 64) -> float:
    """4*d per enabled (query, key) pair: QK^T and PV of the A-shape mask over N tokens."""
    nb = -(-N // block)
    pairs = 0
    for m in range(nb):
        q = min(block, N - m * block)
        keys = min(min(n_init, nb) * block, N)
        if with_diag and m >= n_init:
            keys += min(block, N - m * block)
        pairs += q * keys
    return 4.0 * d * rows * pairs


# ---------------------------------------------------------------------------
# Rows: LayerNorm gathers, window maps, RC-MLP, stem/neck helpers
# ---------------------------------------------------------------------------
def layernorm_gather(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float,
                     src_rows: torch.Tensor | None = None, n_rows: int | None = None,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 LN(x[src_rows]) (zero rows where src_rows < 0); x is fp32 (rows, C)."""
    _check_cuda(x, w, b, src_rows, out)
    if x.dtype != torch.float32 or w.dtype != torch.float32 or b.dtype != torch.float32:
        raise TypeError("layernorm_gather takes fp32 x / w / b")
    x2 = x.reshape(-1, x.shape[-1])
    C = x2.shape[1]
    ldx = _rowmajor(x2, "x")
    if n_rows is None:
        n_rows = src_rows.numel() if src_rows is not None else x2.shape[0]
    if out is None:
        out = torch.empty(n_rows, C, dtype=torch.bfloat16, device=x.device)
    _lib.call("ssam_layernorm_gather", x2.data_ptr(), ldx, _ptr(src_rows), n_rows, C, w.data_ptr(), b.data_ptr(),
              float(eps), out.data_ptr(), _rowmajor(out, "out"), _stream(x))
    return out


def window_rows(B: int, H: int, W: int, ws: int, device) -> torch.Tensor:
    nwh, nww = -(-H // ws), -(-W // ws)
    rows = torch.empty(B * nwh * nww * ws * ws, dtype=torch.int32, device=device)
    _lib.call("ssam_window_rows", B, H, W, ws, rows.data_ptr(), torch.cuda.current_stream(rows.device).cuda_stream)
    return rows


def rc_mlp_workspace_size(n_rows: int, C: int, hidden: int) -> int:
    return int(_lib.load().ssam_rc_mlp_workspace_size(n_rows, C, hidden))


def rc_mlp(x: torch.Tensor, rows: torch.Tensor | None, n_rows: int, ln_w, ln_b, eps: float, w1, b1, w2, b2,
           workspace: torch.Tensor | None = None) -> torch.Tensor:
    """In place: x[rows] += lin2(gelu(lin1(LN(x[rows])))) (rows None -> first n_rows rows)."""
    _check_cuda(x, rows, ln_w, ln_b, w1, b1, w2, b2, workspace)
    x2 = x.view(-1, x.shape[-1])
    C = x2.shape[1]
    hidden = w1.shape[0]
    need = rc_mlp_workspace_size(n_rows, C, hidden)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    _lib.call("ssam_rc_mlp_fwd", x2.data_ptr(), _rowmajor(x2, "x"), _ptr(rows), n_rows, C, hidden, ln_w.data_ptr(),
              ln_b.data_ptr(), float(eps), w1.data_ptr(), _ptr(b1), w2.data_ptr(), _ptr(b2), workspace.data_ptr(),
              workspace.numel() * workspace.element_size(), _stream(x))
    return x


def patch_im2col(img: torch.Tensor, p: int, out: torch.Tensor | None = None) -> torch.Tensor:
    _check_cuda(img, out)
    img = img.contiguous().float()
    B, Cin, H, W = img.shape
    if out is None:
        out = torch.empty(B * (H // p) * (W // p), Cin * p * p, dtype=torch.bfloat16, device=img.device)
    _lib.call("ssam_patch_im2col", img.data_ptr(), B, Cin, H, W, p, out.data_ptr(), _stream(img))
    return out


def patch_im2col_split3(img: torch.Tensor, p: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 NCHW image -> bf16 (tokens, 3 Cin p p) = [hi | lo | hi] patch rows."""
    _check_cuda(img, out)
    img = img.contiguous().float()
    B, Cin, H, W = img.shape
    if out is None:
        out = torch.empty(B * (H // p) * (W // p), 3 * Cin * p * p, dtype=torch.bfloat16, device=img.device)
    _lib.call("ssam_patch_im2col_split3", img.data_ptr(), B, Cin, H, W, p, out.data_ptr(), _stream(img))
    return out


def broadcast_rows(pos: torch.Tensor, B: int, out: torch.Tensor) -> torch.Tensor:
    _check_cuda(pos, out)
    T, C = pos.shape[-3] * pos.shape[-2] if pos.dim() == 4 else pos.shape[0], pos.shape[-1]
    _lib.call("ssam_broadcast_rows", pos.data_ptr(), B, T, C, out.data_ptr(), _stream(out))
    return out


def im2col3x3_nhwc(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _check_cuda(x, out)
    B, H, W, C = x.shape
    if out is None:
        out = torch.empty(B * H * W, 9 * C, dtype=torch.bfloat16, device=x.device)
    _lib.call("ssam_im2col3x3_nhwc", x.data_ptr(), B, H, W, C, out.data_ptr(), _stream(x))
    return out


def gemm_bf16_addend(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor | None, addend: torch.Tensor,
                     k_split: int = 1) -> torch.Tensor:
    """fp32 (M, N) = a @ b.T + bias + addend[r % addend.shape[0]] for every row r
    (addend fp32 (rows, N), e.g. the positional embedding of each image's tokens)."""
    _check_cuda(a, b, bias, addend)
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise TypeError("gemm_bf16_addend takes bf16 operands")
    M, K = a.shape
    N = b.shape[0]
    if b.shape[1] != K:
        raise ValueError(f"inner dimensions differ: {K} vs {b.shape[1]}")
    if addend.dtype != torch.float32 or not addend.is_contiguous() or addend.dim() != 2 or addend.shape[1] != N:
        raise ValueError("addend must be contiguous fp32 (rows, N)")
    out = torch.empty(M, N, device=a.device, dtype=torch.float32)
    t0 = KernelTimer.begin()
    _lib.call("ssam_gemm_bf16_addend", a.data_ptr(), _rowmajor(a, "a"), b.data_ptr(), _rowmajor(b, "b"), M, N, K,
              _ptr(bias), addend.data_ptr(), addend.shape[0], out.data_ptr(), _stream(a))
    KernelTimer.end(t0, "gemm", 2.0 * M * N * K / k_split)
    return out


def conv3x3_supported(H: int, W: int, Cin: int, Cout: int) -> bool:
    """Whether conv3x3_nhwc takes this shape (else use im2col3x3_nhwc + gemm_bf16)."""
    return Cin % 64 == 0 and Cout % 32 == 0 and 0 < W <= 128 and 128 % W == 0 and (H * W) % 128 == 0


def conv3x3_nhwc(x: torch.Tensor, B: int, H: int, W: int, w: torch.Tensor,
                 bias: torch.Tensor | None = None, k_split: int = 1) -> torch.Tensor:
    """3x3 / pad 1 convolution of channels-last bf16 x (B*H*W, Cin) with w bf16
    (Cout, 9*Cin) in (ky, kx, cin) order -> fp32 (B*H*W, Cout), as an implicit GEMM
    (equal, bit for bit, to gemm_bf16(im2col3x3_nhwc(x), w, bias, SSAM_EPI_F32)).
    `k_split` as in gemm_bf16 (the channels are a k_split-term split operand)."""
    _check_cuda(x, w, bias)
    x2 = x.reshape(-1, x.shape[-1])
    if x2.dtype != torch.bfloat16 or not x2.is_contiguous() or x2.shape[0] != B * H * W:
        raise ValueError("x must be contiguous bf16 (B*H*W, Cin)")
    Cin = x2.shape[1]
    if w.dtype != torch.bfloat16 or not w.is_contiguous() or w.shape[1] != 9 * Cin:
        raise ValueError("w must be contiguous bf16 (Cout, 9*Cin)")
    Cout = w.shape[0]
    out = torch.empty(B * H * W, Cout, dtype=torch.float32, device=x.device)
    t0 = KernelTimer.begin()
    _lib.call("ssam_conv3x3_nhwc", x2.data_ptr(), B, H, W, Cin, w.data_ptr(), Cout, _ptr(bias), out.data_ptr(),
              _stream(x))
    KernelTimer.end(t0, "gemm", 2.0 * B * H * W * Cout * 9 * Cin / k_split)
    return out


def nhwc_to_nchw(x: torch.Tensor, B: int, H: int, W: int, C: int, out: torch.Tensor | None = None) -> torch.Tensor:
    _check_cuda(x, out)
    if out is None:
        out = torch.empty(B, C, H, W, dtype=torch.float32, device=x.device)
    _lib.call("ssam_nhwc_to_nchw", x.data_ptr(), B, H * W, C, out.data_ptr(), _stream(x))
    return out


def layernorm_rows(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float, out_bf16: bool,
                   out: torch.Tensor | None = None, copy_out: torch.Tensor | None = None,
                   split3: bool = False) -> torch.Tensor:
    """Row LayerNorm of fp32 x (rows, C). `copy_out` (fp32, x's shape; bf16 output only)
    also receives x unchanged, read once for both. `split3`: the bf16 3-term split
    [hi | lo | hi] of the result, (rows, 3C), as split_bf16x3 of the fp32 output."""
    _check_cuda(x, w, b, out, copy_out)
    x2 = x.reshape(-1, x.shape[-1])
    n, C = x2.shape
    if split3 and (out_bf16 or copy_out is not None):
        raise ValueError("split3 is its own output mode")
    if out is None:
        out = torch.empty(n, 3 * C if split3 else C, dtype=torch.bfloat16 if (out_bf16 or split3) else torch.float32,
                          device=x.device)
    if copy_out is None:
        _lib.call("ssam_layernorm_rows", x2.data_ptr(), n, C, w.data_ptr(), b.data_ptr(), float(eps),
                  out.data_ptr(), 2 if split3 else (1 if out_bf16 else 0), _stream(x))
        return out
    if not out_bf16:
        raise ValueError("copy_out is supported with the bf16 output")
    if copy_out.dtype != torch.float32 or not copy_out.is_contiguous() or copy_out.numel() != n * C:
        raise ValueError("copy_out must be a contiguous fp32 tensor with x's number of elements")
    _lib.call("ssam_layernorm_rows_copy", x2.data_ptr(), n, C, w.data_ptr(), b.data_ptr(), float(eps),
              out.data_ptr(), copy_out.data_ptr(), _stream(x))
    return out


def layernorm_nchw(x: torch.Tensor, B: int, H: int, W: int, w: torch.Tensor, b: torch.Tensor,
                   eps: float) -> torch.Tensor:
    """LayerNorm over C of channels-last fp32 rows (B*H*W, C) -> fp32 (B, C, H, W)."""
    _check_cuda(x, w, b)
    x2 = x.reshape(-1, x.shape[-1])
    if x2.dtype != torch.float32 or not x2.is_contiguous() or x2.shape[0] != B * H * W:
        raise ValueError("x must be contiguous fp32 (B*H*W, C)")
    C = x2.shape[1]
    out = torch.empty(B, C, H, W, dtype=torch.float32, device=x.device)
    _lib.call("ssam_layernorm_nchw", x2.data_ptr(), B, H * W, C, w.data_ptr(), b.data_ptr(), float(eps),
              out.data_ptr(), _stream(x))
    return out


LN_HALF_CHANNELS = (32, 64, 128, 256)


def layernorm_gelu_half(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float,
                        gelu: bool) -> torch.Tensor:
    """Channel LayerNorm (+ exact GELU) of fp16 / bf16 channels-last rows (..., C),
    C in LN_HALF_CHANNELS; w, b of x's dtype. Returns a new tensor of x's shape."""
    _check_cuda(x, w, b)
    if x.dtype not in (torch.float16, torch.bfloat16) or w.dtype != x.dtype or b.dtype != x.dtype:
        raise ValueError("x, w and b must share one half-precision dtype")
    if not x.is_contiguous() or not w.is_contiguous() or not b.is_contiguous():
        raise ValueError("x, w and b must be contiguous")
    C = x.shape[-1]
    out = torch.empty_like(x)
    if x.numel() == 0:
        return out
    _lib.call("ssam_layernorm_gelu_half", x.data_ptr(), x.numel() // C, C, w.data_ptr(), b.data_ptr(),
              float(eps), int(bool(gelu)), 0 if x.dtype == torch.float16 else 1, out.data_ptr(), _stream(x))
    return out


def split_bf16x2(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 (rows, C) -> bf16 (rows, 2C) = [hi | lo] with hi + lo ~= x."""
    _check_cuda(x, out)
    x2 = x.reshape(-1, x.shape[-1])
    if x2.dtype != torch.float32 or not x2.is_contiguous():
        raise TypeError("split_bf16x2 takes a contiguous fp32 tensor")
    n, C = x2.shape
    if out is None:
        out = torch.empty(n, 2 * C, dtype=torch.bfloat16, device=x.device)
    _lib.call("ssam_split_bf16x2", x2.data_ptr(), n, C, out.data_ptr(), _stream(x))
    return out


def split_bf16x3(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 (rows, C) -> bf16 (rows, 3C) = [hi | lo | hi]; pair with weights [W_hi | W_hi | W_lo]."""
    _check_cuda(x, out)
    x2 = x.reshape(-1, x.shape[-1])
    if x2.dtype != torch.float32 or not x2.is_contiguous():
        raise TypeError("split_bf16x3 takes a contiguous fp32 tensor")
    n, C = x2.shape
    if out is None:
        out = torch.empty(n, 3 * C, dtype=torch.bfloat16, device=x.device)
    _lib.call("ssam_split_bf16x3", x2.data_ptr(), n, C, out.data_ptr(), _stream(x))
    return out


def window_of_raster(B: int, H: int, W: int, ws: int, device) -> torch.Tensor:
    """int32 [B*H*W]: each raster token's row in the window layout (inverse of window_rows)."""
    out = torch.empty(B * H * W, dtype=torch.int32, device=device)
    _lib.call("ssam_window_of_raster", B, H, W, ws, out.data_ptr(), torch.cuda.current_stream(out.device).cuda_stream)
    return out


def fill_pad_rows(out: torch.Tensor, rows: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """out[i] = bf16(bias) for every window-layout row i with rows[i] < 0."""
    _check_cuda(out, rows, bias)
    if out.dtype != torch.bfloat16 or rows.dtype != torch.int32 or bias.dtype != torch.float32:
        raise TypeError("fill_pad_rows takes bf16 out, int32 rows, fp32 bias")
    n, C = out.shape
    if rows.numel() < n or bias.numel() != C:
        raise ValueError("rows / bias do not match out")
    _lib.call("ssam_fill_pad_rows", out.data_ptr(), _rowmajor(out, "out"), rows.data_ptr(), n, C, bias.data_ptr(),
              _stream(out))
    return out


def split_weight3(w: torch.Tensor) -> torch.Tensor:
    """fp32 weight (N, K) -> bf16 (N, 3K) = [W_hi | W_hi | W_lo] (setup-time, host side of the split GEMM)."""
    w = w.float()
    hi = w.to(torch.bfloat16)
    lo = (w - hi.float()).to(torch.bfloat16)
    return torch.cat([hi, hi, lo], dim=1).contiguous()
