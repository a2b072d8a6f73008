"""SAM-architecture ViT image encoder (host model of the hot path).

The reference patches `segment_anything.modeling.image_encoder` from the SAM-HQ
submodule (algos/sparsesam/sam.py:21-27), which is not vendored. This module is
an independent implementation of that architecture with the attribute names the
patch protocol touches:

  ImageEncoderViT: patch_embed.proj, pos_embed, blocks, neck
  Block:           norm1, attn, norm2, mlp (lin1, act, lin2), window_size
  Attention:       qkv, proj, num_heads, scale, use_rel_pos, rel_pos_h, rel_pos_w

`ImageEncoderViT.forward` returns `(features, interm_embeddings)` like SAM-HQ:
features (B, 256, H/16, W/16) from the neck, and the (B, H/16, W/16, C) token
grid after every global-attention block.

When the real `segment_anything` package is importable, `resolve_host()` returns
its classes instead so the patch can be applied to a user's own encoder.
"""
from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

SAM_PIXEL_MEAN = (123.675, 116.28, 103.53)
SAM_PIXEL_STD = (58.395, 57.12, 57.375)


class LayerNorm2d(nn.Module):
    """Channel LayerNorm of an NCHW map (eps 1e-6), as in SAM's neck."""

    def __init__(self, num_channels: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(num_channels))
        self.bias = nn.Parameter(torch.zeros(num_channels))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        mu = x.mean(1, keepdim=True)
        var = (x - mu).pow(2).mean(1, keepdim=True)
        y = (x - mu) / torch.sqrt(var + self.eps)
        return self.weight[:, None, None] * y + self.bias[:, None, None]


class MLPBlock(nn.Module):
    def __init__(self, embedding_dim: int, mlp_dim: int):
        super().__init__()
        self.lin1 = nn.Linear(embedding_dim, mlp_dim)
        self.lin2 = nn.Linear(mlp_dim, embedding_dim)
        self.act = nn.GELU()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.lin2(self.act(self.lin1(x)))


class PatchEmbed(nn.Module):
    def __init__(self, patch_size: int = 16, in_chans: int = 3, embed_dim: int = 768):
        super().__init__()
        self.proj = nn.Conv2d(in_chans, embed_dim, kernel_size=patch_size, stride=patch_size)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.proj(x).permute(0, 2, 3, 1)  # B, H, W, C


def window_partition(x: torch.Tensor, window_size: int) -> Tuple[torch.Tensor, Tuple[int, int]]:
    """Zero-pad (B, H, W, C) to window multiples and split into (B*nw, ws, ws, C) windows."""
    B, H, W, C = x.shape
    pad_h = (window_size - H % window_size) % window_size
    pad_w = (window_size - W % window_size) % window_size
    if pad_h or pad_w:
        x = F.pad(x, (0, 0, 0, pad_w, 0, pad_h))
    Hp, Wp = H + pad_h, W + pad_w
    x = x.view(B, Hp // window_size, window_size, Wp // window_size, window_size, C)
    windows = x.permute(0, 1, 3, 2, 4, 5).reshape(-1, window_size, window_size, C)
    return windows, (Hp, Wp)


def window_unpartition(windows: torch.Tensor, window_size: int, pad_hw: Tuple[int, int],
                       hw: Tuple[int, int]) -> torch.Tensor:
    """Inverse of window_partition followed by cropping the padding."""
    Hp, Wp = pad_hw
    H, W = hw
    B = windows.shape[0] // (Hp * Wp // window_size // window_size)
    x = windows.view(B, Hp // window_size, Wp // window_size, window_size, window_size, -1)
    x = x.permute(0, 1, 3, 2, 4, 5).reshape(B, Hp, Wp, -1)
    if Hp > H or Wp > W:
        x = x[:, :H, :W, :].contiguous()
    return x


def get_rel_pos(q_size: int, k_size: int, rel_pos: torch.Tensor) -> torch.Tensor:
    """(q_size, k_size, d) table: entry [i, j] = rel_pos[i - j + k_size - 1] (same-size grids).

    Linear interpolation is used when the table length differs from 2*max-1."""
    max_rel_dist = int(2 * max(q_size, k_size) - 1)
    if rel_pos.shape[0] != max_rel_dist:
        rel_pos = F.interpolate(rel_pos.reshape(1, rel_pos.shape[0], -1).permute(0, 2, 1),
                                size=max_rel_dist, mode="linear").reshape(-1, max_rel_dist).permute(1, 0)
    q_coords = torch.arange(q_size)[:, None] * max(k_size / q_size, 1.0)
    k_coords = torch.arange(k_size)[None, :] * max(q_size / k_size, 1.0)
    rel = (q_coords - k_coords) + (k_size - 1) * max(q_size / k_size, 1.0)
    return rel_pos[rel.long()]


def add_decomposed_rel_pos(attn: torch.Tensor, q: torch.Tensor, rel_pos_h: torch.Tensor,
                           rel_pos_w: torch.Tensor, q_size: Tuple[int, int],
                           k_size: Tuple[int, int]) -> torch.Tensor:
    q_h, q_w = q_size
    k_h, k_w = k_size
    Rh = get_rel_pos(q_h, k_h, rel_pos_h).to(q.dtype)
    Rw = get_rel_pos(q_w, k_w, rel_pos_w).to(q.dtype)
    B, _, dim = q.shape
    r_q = q.reshape(B, q_h, q_w, dim)
    rel_h = torch.einsum("bhwc,hkc->bhwk", r_q, Rh)
    rel_w = torch.einsum("bhwc,wkc->bhwk", r_q, Rw)
    attn = attn.view(B, q_h, q_w, k_h, k_w) + rel_h[:, :, :, :, None] + rel_w[:, :, :, None, :]
    return attn.view(B, q_h * q_w, k_h * k_w)


class Attention(nn.Module):
    """Multi-head attention with SAM's decomposed relative-position bias."""

    def __init__(self, dim: int, num_heads: int = 8, qkv_bias: bool = True, use_rel_pos: bool = True,
                 input_size: Optional[Tuple[int, int]] = None):
        super().__init__()
        self.num_heads = num_heads
        head_dim = dim // num_heads
        self.scale = head_dim ** -0.5
        self.qkv = nn.Linear(dim, dim * 3, bias=qkv_bias)
        self.proj = nn.Linear(dim, dim)
        self.use_rel_pos = use_rel_pos
        if use_rel_pos:
            assert input_size is not None
            self.rel_pos_h = nn.Parameter(torch.zeros(2 * input_size[0] - 1, head_dim))
            self.rel_pos_w = nn.Parameter(torch.zeros(2 * input_size[1] - 1, head_dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, H, W, _ = x.shape
        qkv = self.qkv(x).reshape(B, H * W, 3, self.num_heads, -1).permute(2, 0, 3, 1, 4)
        q, k, v = qkv.reshape(3, B * self.num_heads, H * W, -1).unbind(0)
        attn = (q * self.scale) @ k.transpose(-2, -1)
        if self.use_rel_pos:
            attn = add_decomposed_rel_pos(attn, q, self.rel_pos_h, self.rel_pos_w, (H, W), (H, W))
        attn = attn.softmax(dim=-1)
        x = (attn @ v).view(B, self.num_heads, H, W, -1).permute(0, 2, 3, 1, 4).reshape(B, H, W, -1)
        return self.proj(x)


class Block(nn.Module):
    """Pre-norm transformer block with windowed (window_size > 0) or global attention."""

    def __init__(self, dim: int, num_heads: int, mlp_ratio: float = 4.0, qkv_bias: bool = True,
                 use_rel_pos: bool = True, window_size: int = 0,
                 input_size: Optional[Tuple[int, int]] = None):
        super().__init__()
        self.norm1 = nn.LayerNorm(dim, eps=1e-6)
        self.attn = Attention(dim, num_heads=num_heads, qkv_bias=qkv_bias, use_rel_pos=use_rel_pos,
                              input_size=input_size if window_size == 0 else (window_size, window_size))
        self.norm2 = nn.LayerNorm(dim, eps=1e-6)
        self.mlp = MLPBlock(dim, int(dim * mlp_ratio))
        self.window_size = window_size

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shortcut = x
        x = self.norm1(x)
        if self.window_size > 0:
            H, W = x.shape[1], x.shape[2]
            x, pad_hw = window_partition(x, self.window_size)
        x = self.attn(x)
        if self.window_size > 0:
            x = window_unpartition(x, self.window_size, pad_hw, (H, W))
        x = shortcut + x
        return x + self.mlp(self.norm2(x))


class ImageEncoderViT(nn.Module):
    def __init__(self, img_size: int = 1024, patch_size: int = 16, in_chans: int = 3,
                 embed_dim: int = 768, depth: int = 12, num_heads: int = 12, mlp_ratio: float = 4.0,
                 out_chans: int = 256, qkv_bias: bool = True, use_abs_pos: bool = True,
                 use_rel_pos: bool = True, window_size: int = 14,
                 global_attn_indexes: Sequence[int] = ()):
        super().__init__()
        self.img_size = img_size
        self.patch_embed = PatchEmbed(patch_size, in_chans, embed_dim)
        grid = img_size // patch_size
        self.pos_embed = nn.Parameter(torch.zeros(1, grid, grid, embed_dim)) if use_abs_pos else None
        self.blocks = nn.ModuleList([
            Block(embed_dim, num_heads, mlp_ratio, qkv_bias, use_rel_pos,
                  window_size=window_size if i not in global_attn_indexes else 0,
                  input_size=(grid, grid))
            for i in range(depth)
        ])
        self.neck = nn.Sequential(
            nn.Conv2d(embed_dim, out_chans, kernel_size=1, bias=False),
            LayerNorm2d(out_chans),
            nn.Conv2d(out_chans, out_chans, kernel_size=3, padding=1, bias=False),
            LayerNorm2d(out_chans),
        )

    def forward(self, x: torch.Tensor):
        x = self.patch_embed(x)
        if self.pos_embed is not None:
            x = x + self.pos_embed
        interm_embeddings = []
        for blk in self.blocks:
            x = blk(x)
            if blk.window_size == 0:
                interm_embeddings.append(x)
        x = self.neck(x.permute(0, 3, 1, 2))
        return x, interm_embeddings


# ---------------------------------------------------------------------------
# Configurations and seeded random initialisation
# ---------------------------------------------------------------------------
VIT_CONFIGS = {
    "vit_b": dict(embed_dim=768, depth=12, num_heads=12, global_attn_indexes=(2, 5, 8, 11)),
    "vit_l": dict(embed_dim=1024, depth=24, num_heads=16, global_attn_indexes=(5, 11, 17, 23)),
    "vit_h": dict(embed_dim=1280, depth=32, num_heads=16, global_attn_indexes=(7, 15, 23, 31)),
}


def _trunc_normal_(t: torch.Tensor, std: float, gen: torch.Generator) -> None:
    # N(0, std) truncated at +-2 std, drawn by rejection with an explicit (CPU)
    # generator and copied to t's device, so a seed gives the same values on any device.
    with torch.no_grad():
        flat = t.view(-1)
        n = flat.numel()
        filled = 0
        while filled < n:
            draw = torch.randn(max(1024, int((n - filled) * 1.06)), generator=gen, device=gen.device) * std
            draw = draw[draw.abs() <= 2 * std][: n - filled]
            flat[filled:filled + draw.numel()] = draw.to(device=t.device, dtype=t.dtype)
            filled += draw.numel()


def init_weights(model: nn.Module, seed: int = 0) -> nn.Module:
    """Seeded random init used by every configuration of this build:
    trunc-normal(0.02) for Linear/Conv weights and pos_embed, zero biases,
    LayerNorm weight 1 / bias 0, rel-pos tables N(0, 0.02). Values are drawn on
    the CPU whatever the model's device, so a seed names the same weights everywhere."""
    dev = next(model.parameters()).device
    gen = torch.Generator(device="cpu").manual_seed(seed)
    with torch.no_grad():
        for name, mod in model.named_modules():
            if isinstance(mod, (nn.Linear, nn.Conv2d)):
                _trunc_normal_(mod.weight, 0.02, gen)
                if mod.bias is not None:
                    mod.bias.zero_()
            elif isinstance(mod, (nn.LayerNorm, LayerNorm2d)):
                mod.weight.fill_(1.0)
                mod.bias.zero_()
            if isinstance(mod, Attention) and mod.use_rel_pos:
                mod.rel_pos_h.copy_((torch.randn(mod.rel_pos_h.shape, generator=gen) * 0.02).to(dev))
                mod.rel_pos_w.copy_((torch.randn(mod.rel_pos_w.shape, generator=gen) * 0.02).to(dev))
        if getattr(model, "pos_embed", None) is not None:
            _trunc_normal_(model.pos_embed, 0.02, gen)
    return model


def build_image_encoder(arch: str = "vit_b", seed: int = 0, device: str | torch.device = "cpu",
                        dtype: torch.dtype = torch.float32, img_size: int = 1024) -> ImageEncoderViT:
    """SAM ViT-B/L/H image encoder with the seeded random weights described in init_weights."""
    cfg = VIT_CONFIGS[arch]
    with torch.device(device):
        enc = ImageEncoderViT(img_size=img_size, **cfg)
    init_weights(enc, seed)
    return enc.to(dtype)


def synthetic_images(batch: int, seed: int, img_size: int = 1024, device="cpu") -> torch.Tensor:
    """Uniform integer pixels in [0, 255] normalised with SAM's mean/std (NCHW fp32)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    px = torch.randint(0, 256, (batch, 3, img_size, img_size), generator=g, dtype=torch.int32).float()
    mean = torch.tensor(SAM_PIXEL_MEAN).view(1, 3, 1, 1)
    std = torch.tensor(SAM_PIXEL_STD).view(1, 3, 1, 1)
    return ((px - mean) / std).to(device)


def resolve_host():
    """(ImageEncoderViT, Block, Attention) of the installed SAM package, else of this module."""
    try:
        from segment_anything.modeling.image_encoder import Attention as A  # type: ignore
        from segment_anything.modeling.image_encoder import Block as B  # type: ignore
        from segment_anything.modeling.image_encoder import ImageEncoderViT as E  # type: ignore
        return E, B, A
    except Exception:
        return ImageEncoderViT, Block, Attention
