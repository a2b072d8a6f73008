"""SparseSAM patch for SAM ViT image encoders, running on the B200 kernels.

Drop-in for algos/sparsesam/sam.py: the same `apply_patch(encoder, algo, ratio,
margin, mlp_merge, perm_mode)` entry point, the same `ToMeSAMBlock` /
`ToMeSAMAttention` classes installed by `__class__` reassignment, the same
`encoder.tome_info` dict ({ratio, mlp_merge, perm_mode, perm_cache}) and the
same per-forward permutation cache keyed (win, ratio, n_block, perm_mode).
Every step runs through the C ABI of libsparsesam_b200.so (sparsesam_b200.ops);
there is no CPU path — a patched encoder must live on a CUDA device.

Per block (sam.py:242-290), on an fp32 residual stream x (B*H*W, C):
  windowed  : LN1 on the real tokens -> qkv GEMM scattering rows into the
              window layout (padding rows = the qkv bias) -> Stripe-Sort
              permutation (first windowed block of the forward) -> block-sparse
              rel-pos attention storing raster rows (inverse permutation and
              window unpartition fused) -> proj GEMM adding into x
  global    : the same on the full grid, with the diagonal blocks enabled
  MLP       : Residual-Consistency MLP on the keep set (windowed blocks after the
              first global block, ratio < 1, mlp_merge) or the dense MLP; both
              are LN2 gather -> fc1+GELU GEMM -> fc2 GEMM scatter-adding into x.
"""
from __future__ import annotations

import types
from dataclasses import dataclass

import torch

from .. import ops
from ..host import resolve_host

ImageEncoderViT, Block, Attention = resolve_host()

_FA2_M_BLOCK_LOCAL = 64   # sam.py:52-57 (64-token mask granularity)
_FA2_N_BLOCK_LOCAL = 64
_FA2_M_BLOCK_GLOBAL = 64
_FA2_N_BLOCK_GLOBAL = 64
_FA2_THREADS_LOCAL = 128
_FA2_THREADS_GLOBAL = 128

_LN_EPS = 1e-6


# ---------------------------------------------------------------------------
# Device-side caches (static per grid / device)
# ---------------------------------------------------------------------------
_BASE_ORDER: dict = {}
_WINDOW_ROWS: dict = {}
_WINDOW_OF_RASTER: dict = {}


def _base_order(H: int, W: int, space: str, device) -> torch.Tensor:
    key = (H, W, space, str(device))
    if key not in _BASE_ORDER:
        order = ops.zorder if space == "z" else ops.hilbert_order   # sam.py:128-132
        _BASE_ORDER[key] = order(H, W, device)[0]
    return _BASE_ORDER[key]


def _window_rows(B: int, H: int, W: int, ws: int, device) -> torch.Tensor:
    key = (B, H, W, ws, str(device))
    if key not in _WINDOW_ROWS:
        _WINDOW_ROWS[key] = ops.window_rows(B, H, W, ws, device)
    return _WINDOW_ROWS[key]


def _window_of_raster(B: int, H: int, W: int, ws: int, device) -> torch.Tensor:
    key = (B, H, W, ws, str(device))
    if key not in _WINDOW_OF_RASTER:
        _WINDOW_OF_RASTER[key] = ops.window_of_raster(B, H, W, ws, device)
    return _WINDOW_OF_RASTER[key]


@dataclass
class _AttnWeights:
    qkv_w: torch.Tensor
    qkv_b: torch.Tensor
    proj_w: torch.Tensor
    proj_b: torch.Tensor
    rel_h: torch.Tensor
    rel_w: torch.Tensor
    pad_row: torch.Tensor   # bf16 qkv bias: the qkv row of SAM's zero window padding


@dataclass
class _BlockWeights:
    ln1_w: torch.Tensor
    ln1_b: torch.Tensor
    ln2_w: torch.Tensor
    ln2_b: torch.Tensor
    fc1_w: torch.Tensor
    fc1_b: torch.Tensor
    fc2_w: torch.Tensor
    fc2_b: torch.Tensor


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to(torch.bfloat16).contiguous()


def _f32(t: torch.Tensor | None, n: int, device) -> torch.Tensor:
    if t is None:
        return torch.zeros(n, dtype=torch.float32, device=device)
    return t.detach().to(torch.float32).contiguous()


def _attn_weights(attn) -> _AttnWeights:
    w = getattr(attn, "_ssam_w", None)
    if w is None:
        dev = attn.qkv.weight.device
        C = attn.qkv.weight.shape[1]
        if not attn.use_rel_pos:
            raise NotImplementedError("the SparseSAM B200 attention needs SAM's decomposed rel-pos tables")
        qkv_b = _f32(attn.qkv.bias, 3 * C, dev)
        w = _AttnWeights(_bf16(attn.qkv.weight), qkv_b, _bf16(attn.proj.weight), _f32(attn.proj.bias, C, dev),
                         _bf16(attn.rel_pos_h), _bf16(attn.rel_pos_w), _bf16(qkv_b))
        attn._ssam_w = w
    return w


def _block_weights(blk) -> _BlockWeights:
    w = getattr(blk, "_ssam_w", None)
    if w is None:
        dev = blk.norm1.weight.device
        C = blk.norm1.weight.shape[0]
        H = blk.mlp.lin1.weight.shape[0]
        w = _BlockWeights(_f32(blk.norm1.weight, C, dev), _f32(blk.norm1.bias, C, dev),
                          _f32(blk.norm2.weight, C, dev), _f32(blk.norm2.bias, C, dev),
                          _bf16(blk.mlp.lin1.weight), _f32(blk.mlp.lin1.bias, H, dev),
                          _bf16(blk.mlp.lin2.weight), _f32(blk.mlp.lin2.bias, C, dev))
        blk._ssam_w = w
    return w


def _require_cuda(t: torch.Tensor) -> None:
    if not t.is_cuda:
        raise RuntimeError("the SparseSAM B200 patch runs on CUDA tensors only (move the encoder and input "
                           "to a CUDA device); there is no CPU implementation")


# ---------------------------------------------------------------------------
# Attention
# ---------------------------------------------------------------------------
def _get_perm(info: dict, key: tuple, qkv: torch.Tensor, n_seq: int, heads: int, win: int, d: int):
    """(perm, inv_perm, inv_perm_group) for `key`, computed once per forward (sam.py:193-204)."""
    cache = info.setdefault("perm_cache", {})
    if key not in cache:
        space, layout, ranking = ops.parse_perm_mode(key[3])
        base = _base_order(win, win, space, qkv.device)
        C = heads * d
        cache[key] = ops.stripe_sort_perm(qkv[:, C:], n_seq, heads, win, win, d, base, group_size=4,
                                          layout=layout, ranking=ranking, ld=qkv.stride(0))
    return cache[key]


def _attention_core(attn, xn: torch.Tensor, n_seq: int, win: int, ratio: float, is_global: bool,
                    n_block: int, qkv: torch.Tensor | None = None, out: torch.Tensor | None = None,
                    out_rows: torch.Tensor | None = None, grid: tuple[int, int] | None = None,
                    pad_row: torch.Tensor | None = None):
    """xn: bf16 (n_seq*win*win, C) -> (o bf16 (rows, C) raster order, perm, inv_perm).

    With `qkv` given (already projected, e.g. from the real tokens only), xn is
    not used; `out` / `out_rows` place the attention rows and `grid` (the image token grid of
    windowed sequences) limits the queries to real tokens; `pad_row` stands for the qkv rows
    of the windows' padding keys (see ops.sparse_attn)."""
    w = _attn_weights(attn)
    heads = attn.num_heads
    C = w.proj_w.shape[1]
    d = C // heads
    N = win * win
    if qkv is None:
        qkv = ops.gemm_bf16(xn, w.qkv_w, w.qkv_b)                     # sam.py:182-184
    info = attn._tome_info
    perm_mode = info.get("perm_mode", "z_interleave_sort")
    perm, inv_perm, _ = _get_perm(info, (win, ratio, n_block, perm_mode), qkv, n_seq, heads, win, d)
    n_init = ops.a_shape_n_init(N, n_block, ratio, is_global)          # sam.py:219-223
    o = ops.sparse_attn(qkv, n_seq, heads, win, d, w.rel_h, w.rel_w, perm, n_init, is_global,
                        attn.scale, out=out, out_rows=out_rows, n_block=n_block, grid=grid,
                        pad_row=pad_row)                                                 # sam.py:206-232
    return o, perm, inv_perm


class ToMeSAMAttention(Attention):
    """Attention with Stripe-Sort block-sparse attention (sam.py:168-236).

    forward(x (B, H, W, C), ratio, ...) -> out (B, H, W, C) [, perm, inv_perm];
    perm / inv_perm are int32 (B*heads, H*W)."""

    def forward(self, x: torch.Tensor, ratio: float, use_fa2: bool = True,  # noqa: ARG002
                m_block: int = _FA2_M_BLOCK_LOCAL, n_block: int = _FA2_N_BLOCK_LOCAL,
                threads: int = _FA2_THREADS_LOCAL, is_global: bool = False, return_perm: bool = False):
        _require_cuda(x)
        if m_block != n_block or n_block not in (64, 128):
            raise NotImplementedError("the block mask is defined on equal query / key blocks of 64 or 128 tokens")
        B, H, W, C = x.shape
        if H != W:
            raise ValueError("SparseSAM attention expects square token grids")
        xn = x.reshape(B * H * W, C).to(torch.bfloat16).contiguous()
        o, perm, inv_perm = _attention_core(self, xn, B, H, ratio, is_global, n_block)
        w = _attn_weights(self)
        out = ops.gemm_bf16(o, w.proj_w, w.proj_b, epilogue=ops.SSAM_EPI_F32)
        out = out.view(B, H, W, C).to(x.dtype)
        if return_perm:
            return out, perm, inv_perm
        return out


# ---------------------------------------------------------------------------
# Block
# ---------------------------------------------------------------------------
def _keep_rows(info: dict, B: int, H: int, ratio: float, heads: int, device):
    """Keep set of the RC-MLP from the global permutation (sam.py:273-280), or None."""
    perm_mode = info.get("perm_mode", "z_interleave_sort")
    cache = info.get("perm_cache", {})
    g = cache.get((H, ratio, _FA2_N_BLOCK_GLOBAL, perm_mode))
    if g is None:
        return None
    key = ("keep", H, ratio, perm_mode, B)
    if key not in cache:
        keep_n = max(1, round(ratio * H * H))
        cache[key] = ops.keep_select(g[2], B, heads, keep_n)
    return cache[key]


class ToMeSAMBlock(Block):
    """Transformer block with Stripe-Sort attention and the Residual-Consistency MLP (sam.py:239-290)."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        _require_cuda(x)
        B, H, W, C = x.shape
        xr = x.detach().to(torch.float32).contiguous().clone()
        self._forward_residual(xr.view(B * H * W, C), B, H, W)
        return xr.view(B, H, W, C).to(x.dtype)

    def _forward_residual(self, xr: torch.Tensor, B: int, H: int, W: int,
                          snapshot: torch.Tensor | None = None) -> None:
        """In-place block update of the fp32 residual stream xr (B*H*W, C).

        `snapshot` (xr's shape) receives xr as it enters the block (the encoder's
        intermediate embedding of the previous, global block), written by norm1."""
        info = self._tome_info
        ratio = info["ratio"].pop(0) if isinstance(info["ratio"], list) else info["ratio"]
        C = xr.shape[1]
        bw = _block_weights(self)
        aw = _attn_weights(self.attn)
        if self.window_size > 0:
            # norm1 and the qkv projection on the B*H*W real tokens only; the GEMM
            # epilogue scatters qkv rows into the window layout (window_partition,
            # sam.py:252) and the padding rows get the qkv bias, the projection of
            # SAM's zero padding. The attention store fuses window_unpartition
            # (sam.py:256), so proj also runs on the real tokens only.
            ws = self.window_size
            rows = _window_rows(B, H, W, ws, xr.device)
            n_win = rows.numel() // (ws * ws)
            xn = ops.layernorm_rows(xr, bw.ln1_w, bw.ln1_b, _LN_EPS, out_bf16=True,
                                    copy_out=snapshot)                                      # norm1
            qkv = torch.empty(rows.numel(), 3 * C, dtype=torch.bfloat16, device=xr.device)
            ops.gemm_bf16(xn, aw.qkv_w, aw.qkv_b, out=qkv, out_rows=_window_of_raster(B, H, W, ws, xr.device))
            # the attention reads the padding keys' qkv from aw.pad_row; only the block
            # that computes the window permutation (from K of every window token) needs
            # the padding rows written
            perm_key = (ws, ratio, _FA2_N_BLOCK_LOCAL, info.get("perm_mode", "z_interleave_sort"))
            if perm_key not in info.get("perm_cache", {}):
                ops.fill_pad_rows(qkv, rows, aw.qkv_b)
            o = torch.empty(B * H * W, C, dtype=torch.bfloat16, device=xr.device)
            _attention_core(self.attn, None, n_win, ws, ratio, False, _FA2_N_BLOCK_LOCAL, qkv=qkv, out=o,
                            out_rows=rows, grid=(H, W), pad_row=aw.pad_row)
            ops.gemm_bf16(o, aw.proj_w, aw.proj_b, epilogue=ops.SSAM_EPI_ADD_F32, out=xr)     # + residual
        else:
            if H != W:
                raise ValueError("global SparseSAM attention expects a square grid")
            if snapshot is not None:
                snapshot.copy_(xr)
            xn = ops.layernorm_gather(xr, bw.ln1_w, bw.ln1_b, _LN_EPS)
            o, _, _ = _attention_core(self.attn, xn, B, H, ratio, True, _FA2_N_BLOCK_GLOBAL)
            ops.gemm_bf16(o, aw.proj_w, aw.proj_b, epilogue=ops.SSAM_EPI_ADD_F32, out=xr)

        keep = None
        if info.get("mlp_merge", True) and ratio < 1.0 and self.window_size > 0:
            keep = _keep_rows(info, B, H, ratio, self.attn.num_heads, xr.device)
        rows = keep[1] if keep is not None else None                                      # sam.py:277-282
        # x[rows] += lin2(gelu(lin1(norm2(x[rows])))); rows None -> dense MLP (sam.py:283-288)
        xk = ops.layernorm_gather(xr, bw.ln2_w, bw.ln2_b, _LN_EPS, src_rows=rows)
        h = ops.gemm_bf16(xk, bw.fc1_w, bw.fc1_b, epilogue=ops.SSAM_EPI_GELU_BF16)
        ops.gemm_bf16(h, bw.fc2_w, bw.fc2_b, epilogue=ops.SSAM_EPI_ADD_F32, out=xr, out_rows=rows)


# ---------------------------------------------------------------------------
# Encoder
# ---------------------------------------------------------------------------
@dataclass
class _StemNeckWeights:
    patch_w: torch.Tensor
    patch_b: torch.Tensor
    pos: torch.Tensor | None
    neck0_w: torch.Tensor
    ln_a_w: torch.Tensor
    ln_a_b: torch.Tensor
    neck2_w: torch.Tensor
    ln_b_w: torch.Tensor
    ln_b_b: torch.Tensor
    eps_a: float
    eps_b: float


def _stem_neck_weights(enc) -> _StemNeckWeights:
    w = getattr(enc, "_ssam_w", None)
    if w is None:
        conv = enc.patch_embed.proj
        C = conv.weight.shape[0]
        dev = conv.weight.device
        n = enc.neck
        pos = None
        if enc.pos_embed is not None:
            pos = enc.pos_embed.detach().to(torch.float32).reshape(-1, C).contiguous()
        # The stem and the neck run at fp32 accuracy on the tensor cores: their
        # activations enter as [hi | lo | hi] bf16 splits and the weights as
        # [W_hi | W_hi | W_lo] (ops.split_weight3), three times K. These few GEMMs
        # carry no sparsity and cost under 1% of the encoder's FLOPs; kept at bf16
        # the patch embedding alone adds about 5e-3 to the output embeddings.
        n2 = n[2].weight.detach().float().permute(0, 2, 3, 1)  # (out, ky, kx, cin)
        n2_hi = n2.to(torch.bfloat16)
        n2_lo = (n2 - n2_hi.float()).to(torch.bfloat16)
        w = _StemNeckWeights(
            patch_w=ops.split_weight3(conv.weight.detach().reshape(C, -1)),
            patch_b=_f32(conv.bias, C, dev), pos=pos,
            neck0_w=ops.split_weight3(n[0].weight.detach().reshape(n[0].weight.shape[0], -1)),
            ln_a_w=_f32(n[1].weight, 0, dev), ln_a_b=_f32(n[1].bias, 0, dev),
            neck2_w=torch.cat([n2_hi, n2_hi, n2_lo], dim=3).reshape(n2.shape[0], -1).contiguous(),
            ln_b_w=_f32(n[3].weight, 0, dev), ln_b_b=_f32(n[3].bias, 0, dev),
            eps_a=float(getattr(n[1], "eps", 1e-6)), eps_b=float(getattr(n[3], "eps", 1e-6)))
        enc._ssam_w = w
    return w


def encoder_forward(enc, img: torch.Tensor):
    """Patched ImageEncoderViT.forward: (features (B, 256, h, w) fp32, interm_embeddings).

    Stem: im2col + GEMM (+pos). Blocks: ToMeSAMBlock residual updates. Neck:
    1x1 conv GEMM -> LayerNorm2d -> 3x3 conv (im2col + GEMM) -> LayerNorm2d."""
    _require_cuda(img)
    w = _stem_neck_weights(enc)
    conv = enc.patch_embed.proj
    p = conv.kernel_size[0]
    B, _, Hi, Wi = img.shape
    gh, gw = Hi // p, Wi // p
    C = conv.weight.shape[0]
    T = gh * gw
    cols = ops.patch_im2col_split3(img.to(torch.float32), p)
    if w.pos is not None and B * T >= 256:
        # x = patches . W + b + pos, the positional embedding added in the GEMM epilogue
        x = ops.gemm_bf16_addend(cols, w.patch_w, w.patch_b, w.pos.view(T, C), k_split=3)
    elif w.pos is not None:
        x = torch.empty(B * T, C, dtype=torch.float32, device=img.device)
        ops.broadcast_rows(w.pos, B, x)
        ops.gemm_bf16(cols, w.patch_w, w.patch_b, epilogue=ops.SSAM_EPI_ADD_F32, out=x, k_split=3)
    else:
        x = torch.empty(B * T, C, dtype=torch.float32, device=img.device)
        ops.gemm_bf16(cols, w.patch_w, w.patch_b, epilogue=ops.SSAM_EPI_F32, out=x, k_split=3)
    interm = []
    n_blocks = len(enc.blocks)
    pending = None  # the snapshot of x after a global block, written by the next block's norm1
    for i, blk in enumerate(enc.blocks):
        blk._forward_residual(x, B, gh, gw, snapshot=pending)
        pending = None
        if blk.window_size == 0:
            # after the last block x itself (nothing updates it; the neck only reads it)
            if i == n_blocks - 1:
                interm.append(x.view(B, gh, gw, C))
            else:
                pending = torch.empty_like(x)
                interm.append(pending.view(B, gh, gw, C))
    # neck: fp32 activations and weights through the 3-term split (3x K); the first
    # LayerNorm2d writes the split operand of the 3x3 convolution, the second the
    # NCHW features
    y = ops.gemm_bf16(ops.split_bf16x3(x), w.neck0_w, None, epilogue=ops.SSAM_EPI_F32, k_split=3)
    ya3 = ops.layernorm_rows(y, w.ln_a_w, w.ln_a_b, w.eps_a, out_bf16=False, split3=True)
    if ops.conv3x3_supported(gh, gw, ya3.shape[1], w.neck2_w.shape[0]):
        z = ops.conv3x3_nhwc(ya3, B, gh, gw, w.neck2_w, k_split=3)   # implicit GEMM: no im2col buffer
    else:
        cols3 = ops.im2col3x3_nhwc(ya3.view(B, gh, gw, -1))
        z = ops.gemm_bf16(cols3, w.neck2_w, None, epilogue=ops.SSAM_EPI_F32, k_split=3)
    feats = ops.layernorm_nchw(z, B, gh, gw, w.ln_b_w, w.ln_b_b, w.eps_b)
    return feats, interm


def _warmup(encoder) -> None:
    """Build the device weight caches (bf16 GEMM operands, fp32 vectors) once,
    the B200 counterpart of _warmup_fa2_kernels (sam.py:293-345)."""
    if not next(encoder.parameters()).is_cuda:
        return  # built lazily at the first CUDA forward
    _stem_neck_weights(encoder)
    for blk in encoder.blocks:
        _block_weights(blk)
        _attn_weights(blk.attn)


def clear_caches(encoder) -> None:
    """Drop the device weight caches (call after changing the encoder's weights)."""
    for m in encoder.modules():
        if "_ssam_w" in m.__dict__:
            del m.__dict__["_ssam_w"]


def apply_patch(
    encoder,
    algo: str = "tome",
    ratio: float = 0.9,
    margin: float = 0.5,
    mlp_merge: bool = True,
    perm_mode: str = "z_interleave_sort",
    **_,
):
    """SparseSAM patch for the image encoder (sam.py:348-406).
    `mlp_merge=True` runs the per-block MLP only on the keep set of
    max(1, round(ratio*N)) tokens; `perm_mode` selects the Stripe-Sort ordering."""
    assert 0 < ratio <= 1.0, "ratio must be in (0, 1]"
    ops.parse_perm_mode(perm_mode)
    tome_info = {"ratio": ratio, "mlp_merge": bool(mlp_merge), "perm_mode": perm_mode}
    encoder.tome_info = tome_info

    def _patched_forward(self, x: torch.Tensor):
        n = len(self.blocks)
        r = self.tome_info["ratio"]
        self.tome_info["ratio"] = [r] * n
        self.tome_info["perm_cache"] = {}   # per forward: the permutation depends on K
        try:
            result = encoder_forward(self, x)
        finally:
            self.tome_info["ratio"] = r
        return result

    encoder.forward = types.MethodType(_patched_forward, encoder)

    for module in encoder.modules():
        if isinstance(module, Block) and not isinstance(module, ToMeSAMBlock):
            module.__class__ = ToMeSAMBlock
            module._tome_info = tome_info
        elif isinstance(module, Attention) and not isinstance(module, ToMeSAMAttention):
            module.__class__ = ToMeSAMAttention
            module._tome_info = tome_info
    clear_caches(encoder)
    _warmup(encoder)
    return encoder
