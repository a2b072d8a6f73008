"""SparseSAM MLP-merge patch for vitdet-style ViT blocks (the SAM3 variant), on
the B200 kernels.

Drop-in for algos/sparsesam/sam3.py: the same `apply_patch(encoder, ratio,
mlp_merge)` / `remove_patch(encoder)` entry points and the same
`ToMeSAM3Block` installed by `__class__` reassignment, sharing one
`encoder.tome_info` dict {ratio, mlp_merge}. Per block (sam3.py:83-109):

  attention  unchanged: the block's own attention module on every token (SAM3
             uses 2-D RoPE precomputed for the full grid, so the reference keeps
             attention dense and stock);
  MLP        only on the keep_n = round(ratio N) tokens sampled at a uniform
             stride along the Morton order of the grid (ssam_zstride_keep, static
             per grid, cached); the other tokens keep the residual. The keep-row
             LayerNorm gather, fc1 + GELU and fc2 scatter-add run as one
             ssam_rc_mlp_fwd call on an fp32 copy of the residual stream.

The block class patched is `sam3.model.vitdet.Block` when the SAM3 package is
importable, else the SAM encoder block of `sparsesam_b200.host` (the same
vitdet block structure: norm1, attn, norm2, mlp, window_size). A layer scale
after the MLP (`ls2` with a `gamma` vector) is folded into fc2's weights.
Inference only: dropout and drop path are identities (eval mode).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import ops
from ..host import resolve_host, window_partition, window_unpartition


def resolve_block():
    """The vitdet Block class the patch targets."""
    try:
        from sam3.model.vitdet import Block as _Block  # noqa: PLC0415
        return _Block
    except ImportError:
        return resolve_host()[1]


Block = resolve_block()

_KEEP_CACHE: dict = {}


def keep_rows(H: int, W: int, ratio: float, B: int, device) -> torch.Tensor:
    """Rows b*H*W + idx of the static keep set for B images (sam3.py:49-71), cached per grid."""
    key = (H, W, float(ratio), B, str(device))
    if key not in _KEEP_CACHE:
        _KEEP_CACHE[key] = ops.zstride_keep(H, W, ratio, B, device)[1]
    return _KEEP_CACHE[key]


@dataclass
class _MlpWeights:
    ln_w: torch.Tensor
    ln_b: torch.Tensor
    eps: float
    w1: torch.Tensor
    b1: torch.Tensor
    w2: torch.Tensor
    b2: torch.Tensor


def _mlp_layers(mlp):
    lin1 = getattr(mlp, "lin1", None) or getattr(mlp, "fc1", None)
    lin2 = getattr(mlp, "lin2", None) or getattr(mlp, "fc2", None)
    act = getattr(mlp, "act", None)
    if lin1 is None or lin2 is None:
        raise NotImplementedError("the MLP needs two Linear layers (lin1 / lin2 or fc1 / fc2)")
    if act is not None and not (isinstance(act, torch.nn.GELU) and act.approximate == "none"):
        raise NotImplementedError("the fused MLP implements the exact (erf) GELU only")
    return lin1, lin2


def _mlp_weights(blk) -> _MlpWeights:
    w = getattr(blk, "_ssam3_w", None)
    if w is None:
        lin1, lin2 = _mlp_layers(blk.mlp)
        dev = lin1.weight.device
        C, Hd = lin2.weight.shape[0], lin1.weight.shape[0]
        w2 = lin2.weight.detach().float()
        b2 = lin2.bias.detach().float() if lin2.bias is not None else torch.zeros(C, device=dev)
        gamma = getattr(getattr(blk, "ls2", None), "gamma", None)
        if gamma is not None:   # x + gamma * (W2 h + b2) = x + (gamma W2) h + gamma b2
            w2 = gamma.detach().float()[:, None] * w2
            b2 = gamma.detach().float() * b2
        n2 = blk.norm2
        w = _MlpWeights(n2.weight.detach().float().contiguous(), n2.bias.detach().float().contiguous(),
                        float(n2.eps), lin1.weight.detach().to(torch.bfloat16).contiguous(),
                        (lin1.bias.detach().float() if lin1.bias is not None else torch.zeros(Hd, device=dev))
                        .contiguous(), w2.to(torch.bfloat16).contiguous(), b2.contiguous())
        blk._ssam3_w = w
    return w


def _maybe(blk, name):
    m = getattr(blk, name, None)
    return m if m is not None else (lambda t: t)


class ToMeSAM3Block(Block):
    """Block forward with MLP-merge: stock attention, MLP on the keep set only (sam3.py:80-109)."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda:
            raise RuntimeError("the SparseSAM B200 patch runs on CUDA tensors only; there is no CPU implementation")
        if self.training:
            raise NotImplementedError("the SparseSAM B200 MLP-merge block is inference only (eval mode)")
        info = self._tome_info
        ratio = float(info["ratio"])
        mlp_merge = bool(info.get("mlp_merge", True))
        # attention, unchanged (the stock Block.forward's first half)
        shortcut = x
        h = self.norm1(x)
        if self.window_size > 0:
            H_w, W_w = h.shape[1], h.shape[2]
            h, pad_hw = window_partition(h, self.window_size)
        h = _maybe(self, "ls1")(self.attn(h))
        if self.window_size > 0:
            h = window_unpartition(h, self.window_size, pad_hw, (H_w, W_w))
        x = shortcut + _maybe(self, "dropout")(_maybe(self, "drop_path")(h))
        if x.ndim != 4:
            raise NotImplementedError("expects (B, H, W, C) token grids")
        # MLP on the keep set (or every token) through ssam_rc_mlp_fwd, in place on fp32 rows
        B, H, W, C = x.shape
        xr = x.detach().to(torch.float32).contiguous().clone().view(B * H * W, C)
        mw = _mlp_weights(self)
        if mlp_merge and ratio < 1.0:
            rows = keep_rows(H, W, ratio, B, x.device)
            n_rows = rows.numel()
        else:
            rows, n_rows = None, B * H * W
        ops.rc_mlp(xr, rows, n_rows, mw.ln_w, mw.ln_b, mw.eps, mw.w1, mw.b1, mw.w2, mw.b2)
        return xr.view(B, H, W, C).to(x.dtype)


def apply_patch(encoder: torch.nn.Module, ratio: float = 0.9, mlp_merge: bool = True, **_) -> torch.nn.Module:
    """Patch every vitdet Block of `encoder` with ToMeSAM3Block (sam3.py:112-157).
    `ratio` in (0, 1] is the fraction of tokens whose MLP update runs;
    `mlp_merge=False` runs the MLP on every token."""
    assert 0.0 < ratio <= 1.0, f"ratio must be in (0, 1], got {ratio}"
    info = {"ratio": float(ratio), "mlp_merge": bool(mlp_merge)}
    encoder.tome_info = info
    n_patched = 0
    for module in encoder.modules():
        if isinstance(module, Block) and not isinstance(module, ToMeSAM3Block):
            module.__class__ = ToMeSAM3Block
            module._tome_info = info
            module.__dict__.pop("_ssam3_w", None)
            n_patched += 1
    if n_patched == 0:
        raise RuntimeError("apply_patch(sam3): no vitdet Block found in encoder")
    return encoder


def remove_patch(encoder: torch.nn.Module) -> int:
    """Revert every patched block to the stock Block (sam3.py:160-169); returns the count."""
    n = 0
    for module in encoder.modules():
        if type(module) is ToMeSAM3Block:
            module.__class__ = Block
            module.__dict__.pop("_tome_info", None)
            module.__dict__.pop("_ssam3_w", None)
            n += 1
    encoder.__dict__.pop("tome_info", None)
    return n


__all__ = ["apply_patch", "remove_patch", "ToMeSAM3Block", "keep_rows"]
