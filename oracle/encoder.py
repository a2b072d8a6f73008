"""SparseSAM-patched SAM ViT image encoder, restated in torch fp32 on CPU —
test infrastructure only. Also the SAM3 MLP-merge block (sam3_block).

Restates the reference's patched forward (algos/sparsesam/sam.py:371-380 for the
per-forward cache, :242-290 for ToMeSAMBlock.forward, :168-236 for
ToMeSAMAttention.forward) on top of the stock SAM encoder structure
(patch embed -> +pos -> blocks -> neck), reading only the parameters of the
module it is given. Discrete decisions (permutations) can be supplied by the
caller (`forced_perms`) so that a device run and this restatement can be
compared on the floating-point path with identical token orders.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import order
from .attention import sparse_attention

N_BLOCK = 64  # sam.py:52-55


def _ln(x, w, b, eps=1e-6):
    return F.layer_norm(x, (x.shape[-1],), w, b, eps)


def _window_partition(x, ws):
    B, H, W, C = x.shape
    ph, pw = (ws - H % ws) % ws, (ws - W % ws) % ws
    x = F.pad(x, (0, 0, 0, pw, 0, ph))
    Hp, Wp = H + ph, W + pw
    x = x.view(B, Hp // ws, ws, Wp // ws, ws, C).permute(0, 1, 3, 2, 4, 5).reshape(-1, ws, ws, C)
    return x, (Hp, Wp)


def _window_unpartition(xw, ws, pad_hw, hw):
    Hp, Wp = pad_hw
    H, W = hw
    B = xw.shape[0] // ((Hp // ws) * (Wp // ws))
    x = xw.view(B, Hp // ws, Wp // ws, ws, ws, -1).permute(0, 1, 3, 2, 4, 5).reshape(B, Hp, Wp, -1)
    return x[:, :H, :W, :]


def attention(attn, x, ratio, is_global, perm_cache, perm_mode, forced_perms=None):
    """ToMeSAMAttention.forward restated (sam.py:168-236). x: (B', h, w, C)."""
    B, H, W, C = x.shape
    heads = attn.num_heads
    d = C // heads
    N = H * W
    win = H
    qkv = F.linear(x.reshape(B, N, C), attn.qkv.weight.float(), attn.qkv.bias.float())
    qkv = qkv.view(B, N, 3, heads, d).permute(2, 0, 3, 1, 4).reshape(3, B * heads, N, d)
    q, k, v = qkv.unbind(0)
    key = (win, ratio, N_BLOCK, perm_mode)
    if key not in perm_cache:
        perm_cache[("k",) + key] = k.detach().clone()   # the K the permutation was ranked on
        if forced_perms is not None and key in forced_perms:
            perm_cache[key] = tuple(torch.as_tensor(t).long() for t in forced_perms[key])
        else:
            p, ip, ipg = order.stripe_sort(k.detach().numpy(), win, win, perm_mode=perm_mode)
            perm_cache[key] = (torch.from_numpy(p), torch.from_numpy(ip), torch.from_numpy(ipg))
    perm = perm_cache[key][0]
    n_init = order.a_shape_n_init(N, N_BLOCK, ratio, is_global)
    o = sparse_attention(q, k, v, attn.rel_pos_h.detach(), attn.rel_pos_w.detach(), perm, win, n_init,
                         with_diag=is_global, scale=attn.scale)
    o = o.reshape(B, heads, N, d).permute(0, 2, 1, 3).reshape(B, N, C)
    return F.linear(o, attn.proj.weight.float(), attn.proj.bias.float()).reshape(B, H, W, C)


def _mlp(blk, x):
    h = F.gelu(F.linear(x, blk.mlp.lin1.weight.float(), blk.mlp.lin1.bias.float()))
    return F.linear(h, blk.mlp.lin2.weight.float(), blk.mlp.lin2.bias.float())


def block(blk, x, ratio, perm_cache, perm_mode, mlp_merge, forced_perms=None, keep_log=None):
    """ToMeSAMBlock.forward restated (sam.py:242-290). x: (B, H, W, C) fp32."""
    B, H, W, C = x.shape
    shortcut = x
    xn = _ln(x, blk.norm1.weight.float(), blk.norm1.bias.float())
    if blk.window_size > 0:
        ws = blk.window_size
        xw, pad_hw = _window_partition(xn, ws)
        xa = attention(blk.attn, xw, ratio, False, perm_cache, perm_mode, forced_perms)
        xa = _window_unpartition(xa, ws, pad_hw, (H, W))
    else:
        xa = attention(blk.attn, xn, ratio, True, perm_cache, perm_mode, forced_perms)
    x = shortcut + xa
    xs = x.reshape(B, H * W, C)
    g = perm_cache.get((H, ratio, N_BLOCK, perm_mode))  # global-attention permutation of this grid
    if mlp_merge and ratio < 1.0 and blk.window_size > 0 and g is not None:
        heads = blk.attn.num_heads
        keep_n = order.keep_n_for(ratio, H * W)
        idx = torch.from_numpy(order.keep_select(g[2].numpy(), B, heads, keep_n))
        if keep_log is not None:
            keep_log.append(idx)
        xs = xs.clone()
        for b in range(B):
            kept = xs[b, idx[b]]
            kept = kept + _mlp(blk, _ln(kept, blk.norm2.weight.float(), blk.norm2.bias.float()))
            xs[b, idx[b]] = kept
    else:
        xs = xs + _mlp(blk, _ln(xs, blk.norm2.weight.float(), blk.norm2.bias.float()))
    return xs.reshape(B, H, W, C)


def _ln2d(x, w, b, eps=1e-6):
    mu = x.mean(1, keepdim=True)
    var = (x - mu).pow(2).mean(1, keepdim=True)
    return w[:, None, None] * ((x - mu) / torch.sqrt(var + eps)) + b[:, None, None]


def _stem(enc, img):
    x = F.conv2d(img.float(), enc.patch_embed.proj.weight.float(), enc.patch_embed.proj.bias.float(),
                 stride=enc.patch_embed.proj.stride)
    x = x.permute(0, 2, 3, 1)
    if enc.pos_embed is not None:
        x = x + enc.pos_embed.float()
    return x


def _neck(enc, x):
    n = enc.neck
    y = x.permute(0, 3, 1, 2)
    y = F.conv2d(y, n[0].weight.float())
    y = _ln2d(y, n[1].weight.float(), n[1].bias.float())
    y = F.conv2d(y, n[2].weight.float(), padding=1)
    return _ln2d(y, n[3].weight.float(), n[3].bias.float())


@torch.no_grad()
def encoder_forward(enc, img, ratio: float, mlp_merge: bool = True, perm_mode: str = "z_interleave_sort",
                    forced_perms=None, return_state: bool = False):
    """Patched encoder forward: (features (B,256,h,w), interm_embeddings[, state]).

    state = {"perm_cache": {...}, "keep": [idx per sparse-MLP block]}.
    """
    x = _stem(enc, img)
    perm_cache: dict = {}
    keep_log: list = []
    interm = []
    for blk in enc.blocks:
        x = block(blk, x, ratio, perm_cache, perm_mode, mlp_merge, forced_perms, keep_log)
        if blk.window_size == 0:
            interm.append(x)
    y = _neck(enc, x)
    if return_state:
        return y, interm, {"perm_cache": perm_cache, "keep": keep_log}
    return y, interm


def sam3_block(blk, x, ratio: float, mlp_merge: bool = True):
    """ToMeSAM3Block.forward restated (algos/sparsesam/sam3.py:83-109): the stock
    attention on every token (the block's own attention module, fp32), then the
    MLP on the static Z-stride keep set only (sam3.py:49-71); the other tokens keep
    the residual. x: (B, H, W, C) fp32."""
    B, H, W, C = x.shape
    shortcut = x
    xn = _ln(x, blk.norm1.weight.float(), blk.norm1.bias.float(), blk.norm1.eps)
    if blk.window_size > 0:
        ws = blk.window_size
        xw, pad_hw = _window_partition(xn, ws)
        xa = _window_unpartition(blk.attn(xw), ws, pad_hw, (H, W))
    else:
        xa = blk.attn(xn)
    x = shortcut + xa
    eps2 = blk.norm2.eps
    if mlp_merge and ratio < 1.0:
        idx = torch.from_numpy(order.zstride_keep(H, W, ratio))
        xs = x.reshape(B, H * W, C).clone()
        kept = xs[:, idx]
        xs[:, idx] = kept + _mlp(blk, _ln(kept, blk.norm2.weight.float(), blk.norm2.bias.float(), eps2))
        return xs.reshape(B, H, W, C)
    return x + _mlp(blk, _ln(x, blk.norm2.weight.float(), blk.norm2.bias.float(), eps2))


@torch.no_grad()
def sam3_encoder_forward(enc, img, ratio: float, mlp_merge: bool = True):
    """An encoder with every block patched as ToMeSAM3Block: (features, interm_embeddings)."""
    x = _stem(enc, img)
    interm = []
    for blk in enc.blocks:
        x = sam3_block(blk, x, ratio, mlp_merge)
        if blk.window_size == 0:
            interm.append(x)
    return _neck(enc, x), interm
