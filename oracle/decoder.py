"""SAM-HQ box-prompted decode restated functionally in fp64 — TEST INFRASTRUCTURE ONLY.

The checker for sparsesam_b200.hq (the caller of the encoder hot path in
tasks/sam_hq44k/eval_hq44k.py:87-129: predict_torch(boxes=..., hq_token_only=True)
after the encoder). The decoder itself belongs to SAM-HQ's `segment_anything`
package (algos/3rd_party/sam-hq, an unvendored submodule of unpinned version),
so this is a restatement of the published algorithm (SAM, Kirillov et al. 2023;
SAM-HQ, Ke et al. 2023), written in a different form from the module it checks
and reading only that module's parameters by name:

* attention as einsums over explicit head axes;
* each stride-2, 2x2 transposed convolution as the per-pixel linear map it is
  (every input pixel writes its own 2x2 output block);
* the 3x3 convolutions as nine shifted channel mixes;
* LayerNorms from their moments; bilinear resizing (align_corners=False, the
  half-pixel convention) from its index arithmetic.

SAM-HQ's own source and checkpoints are not available here; the product module
is also checked against the third-party SamModel / SamHQModel of the installed
transformers package (tests/test_hq_third_party.py). Parity of the product module
with this restatement, and of the GPU encoder + decoder with oracle.encoder + this
restatement, is what the other tests check.
"""
from __future__ import annotations

import math

import torch

D = torch.float64


def _p(sd, name):
    return sd[name].to(D)


def _linear(sd, pre, x):
    return x @ _p(sd, pre + ".weight").T + _p(sd, pre + ".bias")


def _ln_last(x, w, b, eps):
    mu = x.mean(-1, keepdim=True)
    var = ((x - mu) ** 2).mean(-1, keepdim=True)
    return (x - mu) / torch.sqrt(var + eps) * w + b


def _ln_channels(x, w, b, eps=1e-6):
    return _ln_last(x.permute(0, 2, 3, 1), w, b, eps).permute(0, 3, 1, 2)


def _gelu(x):
    return 0.5 * x * (1.0 + torch.erf(x / math.sqrt(2.0)))


def _up2x2(sd, pre, x):
    """Transposed convolution, kernel 2 stride 2: out[2i+a, 2j+b] = W[:, :, a, b]^T x[i, j] + bias."""
    w = _p(sd, pre + ".weight")                       # (Cin, Cout, 2, 2)
    y = torch.einsum("nchw,coab->nohawb", x, w)       # (N, Cout, H, 2, W, 2)
    B, O, H, _, W, _ = y.shape
    y = y.reshape(B, O, 2 * H, 2 * W)
    if pre + ".bias" in sd:
        y = y + _p(sd, pre + ".bias").view(1, -1, 1, 1)
    return y


def _conv3x3(sd, pre, x):
    """3x3 convolution with zero padding 1 as nine shifted channel mixes."""
    w = _p(sd, pre + ".weight")                       # (Cout, Cin, 3, 3)
    B, C, H, W = x.shape
    xp = torch.zeros(B, C, H + 2, W + 2, dtype=D)
    xp[:, :, 1:H + 1, 1:W + 1] = x
    y = torch.zeros(B, w.shape[0], H, W, dtype=D)
    for dy in range(3):
        for dx in range(3):
            y += torch.einsum("bchw,oc->bohw", xp[:, :, dy:dy + H, dx:dx + W], w[:, :, dy, dx])
    return y + _p(sd, pre + ".bias").view(1, -1, 1, 1)


def _attention(sd, pre, q, k, v, heads):
    qh = _linear(sd, pre + ".q_proj", q)
    kh = _linear(sd, pre + ".k_proj", k)
    vh = _linear(sd, pre + ".v_proj", v)
    B, Nq, Ci = qh.shape
    c = Ci // heads
    qh = qh.view(B, Nq, heads, c)
    kh = kh.view(B, -1, heads, c)
    vh = vh.view(B, -1, heads, c)
    s = torch.einsum("bqhc,bkhc->bhqk", qh, kh) / math.sqrt(c)
    s = s - s.amax(-1, keepdim=True)
    p = torch.exp(s)
    p = p / p.sum(-1, keepdim=True)
    o = torch.einsum("bhqk,bkhc->bqhc", p, vh).reshape(B, Nq, Ci)
    return _linear(sd, pre + ".out_proj", o)


def _mlp(sd, pre, x, n_layers):
    for i in range(n_layers):
        x = _linear(sd, f"{pre}.layers.{i}", x)
        if i + 1 < n_layers:
            x = torch.clamp(x, min=0.0)
    return x


def _fourier(G, p01):
    u = 2.0 * math.pi * ((2.0 * p01 - 1.0) @ G)
    return torch.cat([torch.sin(u), torch.cos(u)], dim=-1)


def dense_pe(sd, grid):
    G = _p(sd, "prompt_encoder.pe_layer.positional_encoding_gaussian_matrix")
    h, w = grid
    yy, xx = torch.meshgrid(torch.arange(h, dtype=D), torch.arange(w, dtype=D), indexing="ij")
    cells = torch.stack([(xx + 0.5) / w, (yy + 0.5) / h], dim=-1)        # (h, w, 2) = (x, y)
    return _fourier(G, cells).permute(2, 0, 1).unsqueeze(0)


def box_tokens(sd, boxes, image_size):
    """Two corner tokens per box: pe((corner + 0.5) / (w, h)) + corner-type embedding."""
    G = _p(sd, "prompt_encoder.pe_layer.positional_encoding_gaussian_matrix")
    h, w = image_size
    b = boxes.to(D) + 0.5
    c0 = torch.stack([b[:, 0] / w, b[:, 1] / h], dim=-1)
    c1 = torch.stack([b[:, 2] / w, b[:, 3] / h], dim=-1)
    t0 = _fourier(G, c0) + _p(sd, "prompt_encoder.point_embeddings.2.weight")
    t1 = _fourier(G, c1) + _p(sd, "prompt_encoder.point_embeddings.3.weight")
    return torch.stack([t0, t1], dim=1)


def _two_way(sd, src, pos, tokens, depth=2, heads=8):
    keys = src.flatten(2).transpose(1, 2)
    kpe = pos.flatten(2).transpose(1, 2)
    q = tokens
    for i in range(depth):
        pre = f"mask_decoder.transformer.layers.{i}"
        if i == 0:
            q = _attention(sd, pre + ".self_attn", q, q, q, heads)
        else:
            q = q + _attention(sd, pre + ".self_attn", q + tokens, q + tokens, q, heads)
        q = _ln_last(q, _p(sd, pre + ".norm1.weight"), _p(sd, pre + ".norm1.bias"), 1e-5)
        q = q + _attention(sd, pre + ".cross_attn_token_to_image", q + tokens, keys + kpe, keys, heads)
        q = _ln_last(q, _p(sd, pre + ".norm2.weight"), _p(sd, pre + ".norm2.bias"), 1e-5)
        hdn = torch.clamp(_linear(sd, pre + ".mlp.lin1", q), min=0.0)
        q = q + _linear(sd, pre + ".mlp.lin2", hdn)
        q = _ln_last(q, _p(sd, pre + ".norm3.weight"), _p(sd, pre + ".norm3.bias"), 1e-5)
        keys = keys + _attention(sd, pre + ".cross_attn_image_to_token", keys + kpe, q + tokens, q, heads)
        keys = _ln_last(keys, _p(sd, pre + ".norm4.weight"), _p(sd, pre + ".norm4.bias"), 1e-5)
    pre = "mask_decoder.transformer"
    q = q + _attention(sd, pre + ".final_attn_token_to_image", q + tokens, keys + kpe, keys, heads)
    q = _ln_last(q, _p(sd, pre + ".norm_final_attn.weight"), _p(sd, pre + ".norm_final_attn.bias"), 1e-5)
    return q, keys


def _seq(sd, pre, x, kinds):
    """A Sequential of 'up' (2x2 transposed conv), 'c3' (3x3 conv), 'ln' (LayerNorm2d), 'gelu'."""
    for i, k in enumerate(kinds):
        if k == "up":
            x = _up2x2(sd, f"{pre}.{i}", x)
        elif k == "c3":
            x = _conv3x3(sd, f"{pre}.{i}", x)
        elif k == "ln":
            x = _ln_channels(x, _p(sd, f"{pre}.{i}.weight"), _p(sd, f"{pre}.{i}.bias"))
        else:
            x = _gelu(x)
    return x


def decode_boxes(sd, features, interm0, boxes, image_size, multimask_output=False, hq_token_only=True):
    """Box i decoded against image i: (low-res logits (B, 1, 4h, 4w), IoU (B, 1)).

    features (B, 256, h, w), interm0 (B, h, w, C) (the first global block's output),
    boxes (B, 4) in the resized-input frame, image_size = the encoder's input size."""
    feats = features.to(D)
    B, C, h, w = feats.shape
    hq = (_seq(sd, "mask_decoder.embedding_encoder", feats, ["up", "ln", "gelu", "up"])
          + _seq(sd, "mask_decoder.compress_vit_feat", interm0.to(D).permute(0, 3, 1, 2),
                 ["up", "ln", "gelu", "up"]))
    out_tok = torch.cat([_p(sd, "mask_decoder.iou_token.weight"), _p(sd, "mask_decoder.mask_tokens.weight"),
                         _p(sd, "mask_decoder.hf_token.weight")], dim=0)
    n_mask = out_tok.shape[0] - 1                     # SAM mask tokens + the HQ token
    tokens = torch.cat([out_tok.unsqueeze(0).expand(B, -1, -1), box_tokens(sd, boxes, image_size)], dim=1)
    src = feats + _p(sd, "prompt_encoder.no_mask_embed.weight").view(1, -1, 1, 1)
    pos = dense_pe(sd, (h, w)).expand(B, -1, -1, -1)
    hs, keys = _two_way(sd, src, pos, tokens)
    up = _seq(sd, "mask_decoder.output_upscaling", keys.transpose(1, 2).reshape(B, C, h, w),
              ["up", "ln", "gelu", "up", "gelu"])
    up_hq = _seq(sd, "mask_decoder.embedding_maskfeature", up, ["c3", "ln", "gelu", "c3"]) + hq
    n_sam = n_mask - 1
    hyper = [_mlp(sd, f"mask_decoder.output_hypernetworks_mlps.{i}", hs[:, 1 + i], 3) for i in range(n_sam)]
    hyper_hq = _mlp(sd, "mask_decoder.hf_mlp", hs[:, 1 + n_sam], 3)
    m_sam = torch.einsum("bnc,bchw->bnhw", torch.stack(hyper, dim=1), up)
    m_hq = torch.einsum("bc,bchw->bhw", hyper_hq, up_hq).unsqueeze(1)
    iou = _mlp(sd, "mask_decoder.iou_prediction_head", hs[:, 0], 3)
    if multimask_output:
        scores = iou[:, 1:n_sam]
        best = scores.argmax(dim=1)
        iou_out = scores[torch.arange(B), best].unsqueeze(1)
        m_pick = m_sam[torch.arange(B), 1 + best].unsqueeze(1)
    else:
        iou_out = iou[:, 0:1]
        m_pick = m_sam[:, 0:1]
    return (m_hq if hq_token_only else m_pick + m_hq), iou_out


def _resize_axis(x, axis, n_out):
    """Bilinear resampling of one axis, half-pixel centres, edge-clamped (align_corners=False)."""
    n_in = x.shape[axis]
    scale = n_in / n_out
    src = (torch.arange(n_out, dtype=D) + 0.5) * scale - 0.5
    src = torch.clamp(src, min=0.0)
    i0 = torch.floor(src).long().clamp(max=n_in - 1)
    i1 = torch.clamp(i0 + 1, max=n_in - 1)
    lam = (src - i0.to(D))
    shape = [1] * x.dim()
    shape[axis] = n_out
    lam = lam.view(shape)
    return x.index_select(axis, i0) * (1 - lam) + x.index_select(axis, i1) * lam


def postprocess(low_res, img_size, input_size, original_size):
    """Low-res logits -> img_size^2 -> crop input_size -> original_size (bilinear)."""
    m = _resize_axis(_resize_axis(low_res.to(D), 2, img_size), 3, img_size)
    m = m[..., : input_size[0], : input_size[1]]
    return _resize_axis(_resize_axis(m, 2, original_size[0]), 3, original_size[1])
