"""SAM-HQ predictor around the encoder hot path: prompt encoder, HQ mask decoder,
the model's pre / post-processing, SamPredictor and the HQ-44K evaluation step.

The reference calls the encoder from tasks/sam_hq44k/eval_hq44k.py:87-129
(`process_batch`): predictor.model.preprocess -> predictor.model.image_encoder
-> for every image predictor.predict_torch(boxes=..., hq_token_only=True) ->
compute_iou / compute_boundary_iou, and builds the model with
`sam_model_registry[model_type](checkpoint=...)` (eval_hq44k.py:434). Those
classes come from SAM-HQ's `segment_anything` package (the
algos/3rd_party/sam-hq submodule: not vendored, version unpinned). This module
is an independent implementation of the published architecture:

* prompt encoder and two-way mask decoder of SAM (Kirillov et al., "Segment
  Anything", ICCV 2023): random Fourier position encoding of points and box
  corners, learned point-type embeddings, a dense "no mask" embedding, a
  two-layer two-way transformer between the prompt tokens and the 64x64 image
  tokens (token self-attention, token->image and image->token cross-attention
  at half width, a ReLU MLP on the tokens), 4x transposed-convolution
  upscaling, hypernetwork MLPs that turn the mask tokens into per-pixel linear
  classifiers, and an IoU head;
* SAM-HQ's additions (Ke et al., "Segment Anything in High Quality", NeurIPS
  2023): a learned high-quality output token with its own hypernetwork, and an
  HQ feature = upscaled image embedding + upscaled early ViT feature (the first
  global block's output, `interm_embeddings[0]`) added to a refined copy of the
  decoder's mask feature.

Parameter and buffer names follow SAM-HQ's checkpoint layout, so the state dict
of a `sam_hq_vit_*.pth` checkpoint loads into `SamHQ` (none is present here:
the weights are seeded random, `init_prompt_decoder_weights`). The arithmetic is
checked against the SamModel / SamHQModel implementations of the transformers
package with the same weights mapped onto their parameter names.

Differences by design:
* `SamPredictor.set_torch_image` takes a batch of images, and `predict_torch`
  decodes prompt i against image i in ONE decoder pass when the prompt batch
  equals the image batch (`process_batch` uses this instead of the
  reference's per-image decode loop); one image with several prompts is
  broadcast, as in SAM.
* the decoder computes in the dtype of its parameters; inputs (the encoder's
  fp32 features) are cast to it.
"""
from __future__ import annotations

import math
from functools import partial
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from . import host, ops
from .host import SAM_PIXEL_MEAN, SAM_PIXEL_STD


class LayerNorm2d(host.LayerNorm2d):
    """Channel LayerNorm of an NCHW map (eps 1e-6, parameters `weight` / `bias`),
    followed by the exact GELU when `gelu` (the decoder's LayerNorm2d -> GELU
    pairs; the GELU slot of the Sequential is then an nn.Identity, which keeps the
    checkpoint's parameter names). Computed on the channels-last view, which is
    contiguous for the decoder's channels-last maps: on CUDA half-precision maps
    by ssam_layernorm_gelu_half (one pass, GELU fused), elsewhere by torch."""

    def __init__(self, num_channels: int, eps: float = 1e-6, gelu: bool = False):
        super().__init__(num_channels, eps)
        self.gelu = gelu

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        nhwc = x.permute(0, 2, 3, 1)
        if (x.is_cuda and x.dtype in (torch.float16, torch.bfloat16) and self.weight.dtype == x.dtype
                and x.shape[1] in ops.LN_HALF_CHANNELS and nhwc.is_contiguous()):
            y = ops.layernorm_gelu_half(nhwc, self.weight, self.bias, self.eps, self.gelu)
        else:
            y = F.layer_norm(nhwc, (x.shape[1],), self.weight, self.bias, self.eps)
            if self.gelu:
                y = F.gelu(y)
        return y.permute(0, 3, 1, 2)


class RowLayerNorm(nn.LayerNorm):
    """nn.LayerNorm over the last dimension (same parameters); on CUDA
    half-precision rows of 32 .. 256 channels computed by ssam_layernorm_gelu_half
    (the two-way transformer's norm of the 4096 image tokens per prompt)."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if (x.is_cuda and x.dtype in (torch.float16, torch.bfloat16) and self.weight is not None
                and self.weight.dtype == x.dtype and x.shape[-1] in ops.LN_HALF_CHANNELS and x.is_contiguous()):
            return ops.layernorm_gelu_half(x, self.weight, self.bias, self.eps, False)
        return super().forward(x)


def _ln_gelu(c: int):
    """LayerNorm2d with the GELU fused, and the Identity that holds the GELU's slot."""
    return LayerNorm2d(c, gelu=True), nn.Identity()


def _channels_last(x: torch.Tensor) -> torch.Tensor:
    return x.contiguous(memory_format=torch.channels_last)


# ---------------------------------------------------------------------------
# Prompt encoder
# ---------------------------------------------------------------------------
class PositionEmbeddingRandom(nn.Module):
    """Random Fourier features of a position p = (x, y) in [0, 1]^2: with the fixed
    Gaussian matrix G (2 x F), u = 2*pi * (2p - 1) G and pe(p) = [sin u, cos u]
    (2F channels)."""

    def __init__(self, num_pos_feats: int = 128, scale: Optional[float] = None):
        super().__init__()
        s = 1.0 if scale is None or scale <= 0.0 else float(scale)
        self.register_buffer("positional_encoding_gaussian_matrix", s * torch.randn(2, num_pos_feats))

    def _fourier(self, p01: torch.Tensor) -> torch.Tensor:
        g = self.positional_encoding_gaussian_matrix
        u = (2.0 * p01.to(g.dtype) - 1.0) @ g
        u = (2.0 * math.pi) * u
        return torch.cat([torch.sin(u), torch.cos(u)], dim=-1)

    def forward(self, size: Tuple[int, int]) -> torch.Tensor:
        """Encoding of the cell centres of an h x w grid: (2F, h, w)."""
        h, w = size
        g = self.positional_encoding_gaussian_matrix
        ys = (torch.arange(h, device=g.device, dtype=g.dtype) + 0.5) / h
        xs = (torch.arange(w, device=g.device, dtype=g.dtype) + 0.5) / w
        pts = torch.stack([xs.view(1, w).expand(h, w), ys.view(h, 1).expand(h, w)], dim=-1)
        return self._fourier(pts).permute(2, 0, 1)

    def forward_with_coords(self, coords: torch.Tensor, image_size: Tuple[int, int]) -> torch.Tensor:
        """Encoding of pixel coordinates (..., 2) = (x, y) in an image of size (h, w)."""
        h, w = image_size
        g = self.positional_encoding_gaussian_matrix
        c = coords.to(g.dtype)
        # scalar divisors: no host-to-device copy (the step can be captured in a CUDA graph)
        return self._fourier(torch.stack([c[..., 0] / w, c[..., 1] / h], dim=-1))


class PromptEncoder(nn.Module):
    """Sparse (points, box corners) and dense (mask) prompt embeddings.

    Point labels: 1 foreground, 0 background, -1 padding (no point). Sparse
    embedding of a point = pe(point + 0.5) + the embedding of its label
    (`point_embeddings[0]` background, `[1]` foreground); a padding point is
    `not_a_point_embed` alone. A box (x0, y0, x1, y1) gives two tokens, its
    corners, with `point_embeddings[2]` / `[3]` added. Without a mask prompt the
    dense embedding is `no_mask_embed` at every image-token position."""

    def __init__(self, embed_dim: int = 256, image_embedding_size: Tuple[int, int] = (64, 64),
                 input_image_size: Tuple[int, int] = (1024, 1024), mask_in_chans: int = 16):
        super().__init__()
        self.embed_dim = embed_dim
        self.input_image_size = tuple(input_image_size)
        self.image_embedding_size = tuple(image_embedding_size)
        self.pe_layer = PositionEmbeddingRandom(embed_dim // 2)
        self.num_point_embeddings = 4
        self.point_embeddings = nn.ModuleList([nn.Embedding(1, embed_dim) for _ in range(4)])
        self.not_a_point_embed = nn.Embedding(1, embed_dim)
        self.mask_input_size = (4 * image_embedding_size[0], 4 * image_embedding_size[1])
        c4 = mask_in_chans // 4
        self.mask_downscaling = nn.Sequential(
            nn.Conv2d(1, c4, kernel_size=2, stride=2), *_ln_gelu(c4),
            nn.Conv2d(c4, mask_in_chans, kernel_size=2, stride=2), *_ln_gelu(mask_in_chans),
            nn.Conv2d(mask_in_chans, embed_dim, kernel_size=1),
        )
        self.no_mask_embed = nn.Embedding(1, embed_dim)

    def get_dense_pe(self) -> torch.Tensor:
        """Position encoding of the image tokens: (1, embed_dim, h, w)."""
        return self.pe_layer(self.image_embedding_size).unsqueeze(0)

    def _embed_points(self, points: torch.Tensor, labels: torch.Tensor, pad: bool) -> torch.Tensor:
        points = points + 0.5
        if pad:
            points = torch.cat([points, points.new_zeros(points.shape[0], 1, 2)], dim=1)
            labels = torch.cat([labels, labels.new_full((labels.shape[0], 1), -1)], dim=1)
        emb = self.pe_layer.forward_with_coords(points, self.input_image_size)
        lab = labels.unsqueeze(-1)
        none = self.not_a_point_embed.weight.view(1, 1, -1).to(emb.dtype).expand_as(emb)
        bg = emb + self.point_embeddings[0].weight.view(1, 1, -1).to(emb.dtype)
        fg = emb + self.point_embeddings[1].weight.view(1, 1, -1).to(emb.dtype)
        return torch.where(lab == -1, none, torch.where(lab == 0, bg, torch.where(lab == 1, fg, emb)))

    def _embed_boxes(self, boxes: torch.Tensor) -> torch.Tensor:
        corners = (boxes + 0.5).reshape(-1, 2, 2)
        emb = self.pe_layer.forward_with_coords(corners, self.input_image_size)
        corner_type = torch.cat([self.point_embeddings[2].weight, self.point_embeddings[3].weight], dim=0)
        return emb + corner_type.to(emb.dtype).unsqueeze(0)

    @staticmethod
    def _batch(points, boxes, masks) -> int:
        if points is not None:
            return points[0].shape[0]
        if boxes is not None:
            return boxes.shape[0]
        if masks is not None:
            return masks.shape[0]
        return 1

    def _device(self) -> torch.device:
        return self.point_embeddings[0].weight.device

    def forward(self, points: Optional[Tuple[torch.Tensor, torch.Tensor]], boxes: Optional[torch.Tensor],
                masks: Optional[torch.Tensor]) -> Tuple[torch.Tensor, torch.Tensor]:
        """(sparse (P, n_tokens, embed_dim), dense (P, embed_dim, h, w)) for P prompts."""
        bs = self._batch(points, boxes, masks)
        dt = self.no_mask_embed.weight.dtype
        parts = [torch.empty(bs, 0, self.embed_dim, device=self._device(), dtype=dt)]
        if points is not None:
            coords, labels = points
            parts.append(self._embed_points(coords, labels, pad=boxes is None).to(dt))
        if boxes is not None:
            parts.append(self._embed_boxes(boxes).to(dt))
        sparse = torch.cat(parts, dim=1)
        if masks is not None:
            dense = self.mask_downscaling(masks.to(dt))
        else:
            dense = self.no_mask_embed.weight.view(1, -1, 1, 1).expand(bs, -1, *self.image_embedding_size)
        return sparse, dense


# ---------------------------------------------------------------------------
# Two-way transformer
# ---------------------------------------------------------------------------
class DecoderAttention(nn.Module):
    """Multi-head attention whose q / k / v projections go down to
    embedding_dim / downsample_rate channels (the cross-attention layers use 2)."""

    def __init__(self, embedding_dim: int, num_heads: int, downsample_rate: int = 1):
        super().__init__()
        self.embedding_dim = embedding_dim
        self.internal_dim = embedding_dim // downsample_rate
        self.num_heads = num_heads
        if self.internal_dim % num_heads:
            raise ValueError("num_heads must divide embedding_dim / downsample_rate")
        self.q_proj = nn.Linear(embedding_dim, self.internal_dim)
        self.k_proj = nn.Linear(embedding_dim, self.internal_dim)
        self.v_proj = nn.Linear(embedding_dim, self.internal_dim)
        self.out_proj = nn.Linear(self.internal_dim, embedding_dim)

    def _split(self, x: torch.Tensor) -> torch.Tensor:
        b, n, c = x.shape
        return x.view(b, n, self.num_heads, c // self.num_heads).transpose(1, 2)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        qh, kh, vh = self._split(self.q_proj(q)), self._split(self.k_proj(k)), self._split(self.v_proj(v))
        o = F.scaled_dot_product_attention(qh, kh, vh)       # softmax(q k^T / sqrt(c)) v
        b, h, n, c = o.shape
        return self.out_proj(o.transpose(1, 2).reshape(b, n, h * c))


class DecoderMLPBlock(nn.Module):
    """lin2(ReLU(lin1(x))): the token MLP of a two-way block."""

    def __init__(self, embedding_dim: int, mlp_dim: int):
        super().__init__()
        self.lin1 = nn.Linear(embedding_dim, mlp_dim)
        self.lin2 = nn.Linear(mlp_dim, embedding_dim)
        self.act = nn.ReLU()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.lin2(self.act(self.lin1(x)))


class TwoWayAttentionBlock(nn.Module):
    """Token self-attention, token->image cross-attention, token MLP and
    image->token cross-attention, each followed by a residual add and a
    LayerNorm; the position encodings are added to the queries and keys of every
    attention (the first block's self-attention takes the tokens without them)."""

    def __init__(self, embedding_dim: int, num_heads: int, mlp_dim: int = 2048,
                 attention_downsample_rate: int = 2, skip_first_layer_pe: bool = False):
        super().__init__()
        self.self_attn = DecoderAttention(embedding_dim, num_heads)
        self.norm1 = nn.LayerNorm(embedding_dim)
        self.cross_attn_token_to_image = DecoderAttention(embedding_dim, num_heads, attention_downsample_rate)
        self.norm2 = nn.LayerNorm(embedding_dim)
        self.mlp = DecoderMLPBlock(embedding_dim, mlp_dim)
        self.norm3 = nn.LayerNorm(embedding_dim)
        self.norm4 = RowLayerNorm(embedding_dim)       # over the image tokens
        self.cross_attn_image_to_token = DecoderAttention(embedding_dim, num_heads, attention_downsample_rate)
        self.skip_first_layer_pe = skip_first_layer_pe

    def forward(self, queries: torch.Tensor, keys: torch.Tensor, query_pe: torch.Tensor,
                key_pe: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        if self.skip_first_layer_pe:
            queries = self.self_attn(queries, queries, queries)
        else:
            qp = queries + query_pe
            queries = queries + self.self_attn(qp, qp, queries)
        queries = self.norm1(queries)
        qp, kp = queries + query_pe, keys + key_pe
        queries = self.norm2(queries + self.cross_attn_token_to_image(qp, kp, keys))
        queries = self.norm3(queries + self.mlp(queries))
        qp, kp = queries + query_pe, keys + key_pe
        keys = self.norm4(keys + self.cross_attn_image_to_token(kp, qp, queries))
        return queries, keys


class TwoWayTransformer(nn.Module):
    """`depth` two-way blocks, then a final token->image attention and LayerNorm
    on the tokens. Returns (tokens (B, T, C), image tokens (B, h*w, C))."""

    def __init__(self, depth: int = 2, embedding_dim: int = 256, num_heads: int = 8, mlp_dim: int = 2048,
                 attention_downsample_rate: int = 2):
        super().__init__()
        self.depth = depth
        self.embedding_dim = embedding_dim
        self.num_heads = num_heads
        self.mlp_dim = mlp_dim
        self.layers = nn.ModuleList([
            TwoWayAttentionBlock(embedding_dim, num_heads, mlp_dim, attention_downsample_rate,
                                 skip_first_layer_pe=(i == 0))
            for i in range(depth)
        ])
        self.final_attn_token_to_image = DecoderAttention(embedding_dim, num_heads, attention_downsample_rate)
        self.norm_final_attn = nn.LayerNorm(embedding_dim)

    def forward(self, image_embedding: torch.Tensor, image_pe: torch.Tensor,
                point_embedding: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        keys = image_embedding.flatten(2).transpose(1, 2)
        key_pe = image_pe.flatten(2).transpose(1, 2)
        queries = point_embedding
        for layer in self.layers:
            queries, keys = layer(queries, keys, point_embedding, key_pe)
        attn = self.final_attn_token_to_image(queries + point_embedding, keys + key_pe, keys)
        return self.norm_final_attn(queries + attn), keys


class MLP(nn.Module):
    """num_layers Linear layers with ReLU between them (hypernetworks, IoU head)."""

    def __init__(self, input_dim: int, hidden_dim: int, output_dim: int, num_layers: int,
                 sigmoid_output: bool = False):
        super().__init__()
        dims = [input_dim] + [hidden_dim] * (num_layers - 1) + [output_dim]
        self.num_layers = num_layers
        self.layers = nn.ModuleList(nn.Linear(a, b) for a, b in zip(dims[:-1], dims[1:]))
        self.sigmoid_output = sigmoid_output

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        for i, layer in enumerate(self.layers):
            x = layer(x)
            if i + 1 < self.num_layers:
                x = F.relu(x)
        return torch.sigmoid(x) if self.sigmoid_output else x


# ---------------------------------------------------------------------------
# HQ mask decoder
# ---------------------------------------------------------------------------
class MaskDecoderHQ(nn.Module):
    """SAM's mask decoder with SAM-HQ's high-quality output token.

    Output tokens: IoU token, num_multimask_outputs + 1 SAM mask tokens, the HQ
    token. Low-resolution masks (4x the image-token grid) are the hypernetwork
    vector of each mask token dotted with the upscaled image tokens (SAM tokens)
    or with the HQ feature (HQ token)."""

    def __init__(self, *, transformer_dim: int = 256, transformer: Optional[nn.Module] = None,
                 num_multimask_outputs: int = 3, iou_head_depth: int = 3, iou_head_hidden_dim: int = 256,
                 vit_dim: int = 1024):
        super().__init__()
        c = transformer_dim
        self.transformer_dim = c
        self.transformer = transformer if transformer is not None else TwoWayTransformer(2, c, 8, 2048)
        self.num_multimask_outputs = num_multimask_outputs
        n_sam = num_multimask_outputs + 1
        self.iou_token = nn.Embedding(1, c)
        self.mask_tokens = nn.Embedding(n_sam, c)
        self.output_upscaling = nn.Sequential(
            nn.ConvTranspose2d(c, c // 4, kernel_size=2, stride=2), *_ln_gelu(c // 4),
            nn.ConvTranspose2d(c // 4, c // 8, kernel_size=2, stride=2), nn.GELU(),
        )
        self.output_hypernetworks_mlps = nn.ModuleList([MLP(c, c, c // 8, 3) for _ in range(n_sam)])
        self.iou_prediction_head = MLP(c, iou_head_hidden_dim, n_sam, iou_head_depth)
        # high-quality output token and the HQ feature path
        self.hf_token = nn.Embedding(1, c)
        self.hf_mlp = MLP(c, c, c // 8, 3)
        self.num_mask_tokens = n_sam + 1
        self.compress_vit_feat = nn.Sequential(
            nn.ConvTranspose2d(vit_dim, c, kernel_size=2, stride=2), *_ln_gelu(c),
            nn.ConvTranspose2d(c, c // 8, kernel_size=2, stride=2),
        )
        self.embedding_encoder = nn.Sequential(
            nn.ConvTranspose2d(c, c // 4, kernel_size=2, stride=2), *_ln_gelu(c // 4),
            nn.ConvTranspose2d(c // 4, c // 8, kernel_size=2, stride=2),
        )
        self.embedding_maskfeature = nn.Sequential(
            nn.Conv2d(c // 8, c // 4, 3, 1, 1), *_ln_gelu(c // 4),
            nn.Conv2d(c // 4, c // 8, 3, 1, 1),
        )

    def forward(self, image_embeddings: torch.Tensor, image_pe: torch.Tensor,
                sparse_prompt_embeddings: torch.Tensor, dense_prompt_embeddings: torch.Tensor,
                multimask_output: bool, hq_token_only: bool,
                interm_embeddings: Sequence[torch.Tensor]) -> Tuple[torch.Tensor, torch.Tensor]:
        """(low-res mask logits (P, 1, 4h, 4w), IoU predictions (P, 1)).

        multimask_output picks, per prompt, the SAM mask of the best predicted IoU
        among the multimask outputs (else the single-mask output); the HQ mask is
        returned alone (hq_token_only) or added to it."""
        dt = self.iou_token.weight.dtype
        image_embeddings = _channels_last(image_embeddings.to(dt))
        vit_features = _channels_last(interm_embeddings[0].to(dt).permute(0, 3, 1, 2))
        hq_features = self.embedding_encoder(image_embeddings) + self.compress_vit_feat(vit_features)
        masks, iou_pred = self.predict_masks(image_embeddings, image_pe.to(dt), sparse_prompt_embeddings.to(dt),
                                             dense_prompt_embeddings.to(dt), hq_features)
        n = self.num_mask_tokens
        if multimask_output:
            iou_pred, best = iou_pred[:, 1:n - 1].max(dim=1, keepdim=True)
            multi = masks[:, 1:n - 1]
            masks_sam = torch.gather(multi, 1, best.view(-1, 1, 1, 1).expand(-1, 1, *multi.shape[-2:]))
        else:
            iou_pred = iou_pred[:, 0:1]
            masks_sam = masks[:, 0:1]
        masks_hq = masks[:, n - 1:n]
        return (masks_hq if hq_token_only else masks_sam + masks_hq), iou_pred

    def predict_masks(self, image_embeddings: torch.Tensor, image_pe: torch.Tensor,
                      sparse_prompt_embeddings: torch.Tensor, dense_prompt_embeddings: torch.Tensor,
                      hq_features: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """All mask logits (P, num_mask_tokens, 4h, 4w) and IoU predictions (P, n_sam).
        Prompt i is decoded against image i when the image and prompt batches are
        equal; a single image is shared by all prompts."""
        P = sparse_prompt_embeddings.shape[0]
        out_tokens = torch.cat([self.iou_token.weight, self.mask_tokens.weight, self.hf_token.weight], dim=0)
        tokens = torch.cat([out_tokens.unsqueeze(0).expand(P, -1, -1), sparse_prompt_embeddings], dim=1)
        bi = image_embeddings.shape[0]
        if bi != P:
            if bi != 1:
                raise ValueError(f"{bi} images and {P} prompts: give one prompt per image or one image")
            image_embeddings = image_embeddings.expand(P, -1, -1, -1)
            hq_features = hq_features.expand(P, -1, -1, -1)
        src = image_embeddings + dense_prompt_embeddings
        pos_src = image_pe.expand(P, -1, -1, -1)
        b, c, h, w = src.shape
        hs, img_tokens = self.transformer(src, pos_src, tokens)
        iou_token_out = hs[:, 0]
        mask_tokens_out = hs[:, 1:1 + self.num_mask_tokens]
        # image tokens (b, h*w, c) are the channels-last memory of the (b, c, h, w) map
        up_sam = self.output_upscaling(img_tokens.reshape(b, h, w, c).permute(0, 3, 1, 2))
        up_hq = self.embedding_maskfeature(up_sam) + hq_features
        n_sam = self.num_mask_tokens - 1
        hyper = [mlp(mask_tokens_out[:, i]) for i, mlp in enumerate(self.output_hypernetworks_mlps)]
        hyper.append(self.hf_mlp(mask_tokens_out[:, n_sam]))
        hyper = torch.stack(hyper, dim=1)
        b, c8, uh, uw = up_sam.shape
        # per-pixel dot products on the channels-last maps: (b, uh*uw, c8) @ (b, c8, n)
        m_sam = _channels_last(up_sam).permute(0, 2, 3, 1).reshape(b, uh * uw, c8) @ hyper[:, :n_sam].transpose(1, 2)
        m_hq = _channels_last(up_hq).permute(0, 2, 3, 1).reshape(b, uh * uw, c8) @ hyper[:, n_sam:].transpose(1, 2)
        masks = torch.cat([m_sam, m_hq], dim=2).transpose(1, 2).reshape(b, n_sam + 1, uh, uw)
        return masks, self.iou_prediction_head(iou_token_out)


# ---------------------------------------------------------------------------
# Model, transforms, predictor
# ---------------------------------------------------------------------------
class SamHQ(nn.Module):
    """image_encoder + prompt_encoder + mask_decoder, with SAM's pixel
    normalisation and padding (`preprocess`) and mask resizing (`postprocess_masks`)."""

    mask_threshold: float = 0.0
    image_format: str = "RGB"

    def __init__(self, image_encoder: nn.Module, prompt_encoder: PromptEncoder, mask_decoder: MaskDecoderHQ,
                 pixel_mean: Sequence[float] = SAM_PIXEL_MEAN, pixel_std: Sequence[float] = SAM_PIXEL_STD):
        super().__init__()
        self.image_encoder = image_encoder
        self.prompt_encoder = prompt_encoder
        self.mask_decoder = mask_decoder
        self.register_buffer("pixel_mean", torch.tensor(pixel_mean, dtype=torch.float32).view(-1, 1, 1), False)
        self.register_buffer("pixel_std", torch.tensor(pixel_std, dtype=torch.float32).view(-1, 1, 1), False)

    @property
    def device(self) -> torch.device:
        return self.pixel_mean.device

    def preprocess(self, x: torch.Tensor) -> torch.Tensor:
        """Normalise pixels (0..255, NCHW) and zero-pad bottom / right to img_size."""
        x = (x.to(self.pixel_mean.dtype) - self.pixel_mean) / self.pixel_std
        s = self.image_encoder.img_size
        h, w = x.shape[-2:]
        return F.pad(x, (0, s - w, 0, s - h))

    def postprocess_masks(self, masks: torch.Tensor, input_size: Tuple[int, ...],
                          original_size: Tuple[int, ...]) -> torch.Tensor:
        """Low-res logits -> img_size x img_size -> crop the unpadded input -> original size (bilinear)."""
        s = self.image_encoder.img_size
        m = F.interpolate(masks, (s, s), mode="bilinear", align_corners=False)
        m = m[..., : input_size[0], : input_size[1]]
        if tuple(m.shape[-2:]) == tuple(original_size):
            return m        # a same-size bilinear resize samples every pixel at weight 1: the identity
        return F.interpolate(m, tuple(original_size), mode="bilinear", align_corners=False)

    @torch.no_grad()
    def forward(self, batched_input: List[Dict], multimask_output: bool, hq_token_only: bool = False) -> List[Dict]:
        """Per-image dicts ('image' 3xHxW resized, 'original_size', optional 'point_coords' /
        'point_labels' / 'boxes' / 'mask_inputs') -> dicts of 'masks', 'iou_predictions',
        'low_res_logits'. The images are encoded as one batch."""
        images = torch.stack([self.preprocess(r["image"]) for r in batched_input], dim=0)
        feats, interm = self.image_encoder(images)
        pe = self.prompt_encoder.get_dense_pe()
        out = []
        for i, rec in enumerate(batched_input):
            pts = (rec["point_coords"], rec["point_labels"]) if "point_coords" in rec else None
            sparse, dense = self.prompt_encoder(pts, rec.get("boxes"), rec.get("mask_inputs"))
            low, iou = self.mask_decoder(feats[i:i + 1], pe, sparse, dense, multimask_output, hq_token_only,
                                         [t[i:i + 1] for t in interm])
            masks = self.postprocess_masks(low, rec["image"].shape[-2:], rec["original_size"])
            out.append({"masks": masks > self.mask_threshold, "iou_predictions": iou, "low_res_logits": low})
        return out


class ResizeLongestSide:
    """Resizes images so that the longest side is target_length, and maps point /
    box coordinates accordingly (torch and numpy forms)."""

    def __init__(self, target_length: int):
        self.target_length = target_length

    @staticmethod
    def get_preprocess_shape(oldh: int, oldw: int, long_side_length: int) -> Tuple[int, int]:
        scale = long_side_length * 1.0 / max(oldh, oldw)
        return int(oldh * scale + 0.5), int(oldw * scale + 0.5)

    def apply_image_torch(self, image: torch.Tensor) -> torch.Tensor:
        """(B, 3, H, W) -> longest side target_length (bilinear, antialiased)."""
        size = self.get_preprocess_shape(image.shape[2], image.shape[3], self.target_length)
        return F.interpolate(image.float(), size, mode="bilinear", align_corners=False, antialias=True)

    def _scale(self, coords, original_size):
        oh, ow = original_size
        nh, nw = self.get_preprocess_shape(oh, ow, self.target_length)
        out = coords.clone() if isinstance(coords, torch.Tensor) else np.array(coords, dtype=np.float64, copy=True)
        if isinstance(out, torch.Tensor):
            out = out.to(torch.float32)
        out[..., 0] = out[..., 0] * (nw / ow)
        out[..., 1] = out[..., 1] * (nh / oh)
        return out

    def apply_coords(self, coords: np.ndarray, original_size: Tuple[int, int]) -> np.ndarray:
        return self._scale(coords, original_size)

    def apply_boxes(self, boxes: np.ndarray, original_size: Tuple[int, int]) -> np.ndarray:
        return self._scale(np.asarray(boxes).reshape(-1, 2, 2), original_size).reshape(-1, 4)

    def apply_coords_torch(self, coords: torch.Tensor, original_size: Tuple[int, int]) -> torch.Tensor:
        return self._scale(coords, original_size)

    def apply_boxes_torch(self, boxes: torch.Tensor, original_size: Tuple[int, int]) -> torch.Tensor:
        return self._scale(boxes.reshape(-1, 2, 2), original_size).reshape(-1, 4)


class SamPredictor:
    """set_image / set_torch_image computes the image embeddings once; predict /
    predict_torch decode prompts against them. Images may be batched (see the
    module docstring)."""

    def __init__(self, sam_model: SamHQ):
        self.model = sam_model
        self.transform = ResizeLongestSide(sam_model.image_encoder.img_size)
        self.reset_image()

    @property
    def device(self) -> torch.device:
        return self.model.device

    def reset_image(self) -> None:
        self.is_image_set = False
        self.features = None
        self.interm_features = None
        self.orig_h = self.orig_w = self.input_h = self.input_w = None
        self.original_size = None
        self.input_size = None

    def set_image(self, image: np.ndarray, image_format: str = "RGB") -> None:
        """HxWx3 uint8 image in `image_format` ('RGB' or 'BGR')."""
        if image_format not in ("RGB", "BGR"):
            raise ValueError("image_format must be 'RGB' or 'BGR'")
        if image_format != self.model.image_format:
            image = image[..., ::-1]
        t = torch.as_tensor(np.ascontiguousarray(image), device=self.device).permute(2, 0, 1)[None]
        self.set_torch_image(self.transform.apply_image_torch(t), image.shape[:2])

    @torch.no_grad()
    def set_torch_image(self, transformed_image: torch.Tensor, original_image_size: Tuple[int, ...]) -> None:
        """(B, 3, H, W) images already resized so that max(H, W) == img_size."""
        s = self.model.image_encoder.img_size
        if transformed_image.dim() != 4 or transformed_image.shape[1] != 3 or max(transformed_image.shape[2:]) != s:
            raise ValueError(f"set_torch_image takes (B, 3, H, W) with longest side {s}")
        self.reset_image()
        self.original_size = tuple(original_image_size)
        self.input_size = tuple(transformed_image.shape[-2:])
        self.features, self.interm_features = self.model.image_encoder(self.model.preprocess(transformed_image))
        self.is_image_set = True

    def predict(self, point_coords: Optional[np.ndarray] = None, point_labels: Optional[np.ndarray] = None,
                box: Optional[np.ndarray] = None, mask_input: Optional[np.ndarray] = None,
                multimask_output: bool = True, return_logits: bool = False, hq_token_only: bool = False):
        """numpy prompts in original-image coordinates -> numpy (masks, iou, low-res logits)."""
        if not self.is_image_set:
            raise RuntimeError("set an image with set_image before predict")
        dev = self.device
        coords = labels = boxes = masks = None
        if point_coords is not None:
            if point_labels is None:
                raise ValueError("point_labels must accompany point_coords")
            coords = torch.as_tensor(self.transform.apply_coords(point_coords, self.original_size),
                                     dtype=torch.float32, device=dev)[None]
            labels = torch.as_tensor(point_labels, dtype=torch.int64, device=dev)[None]
        if box is not None:
            boxes = torch.as_tensor(self.transform.apply_boxes(box, self.original_size),
                                    dtype=torch.float32, device=dev)[None].reshape(-1, 4)
        if mask_input is not None:
            masks = torch.as_tensor(mask_input, dtype=torch.float32, device=dev)[None]
        m, iou, low = self.predict_torch(coords, labels, boxes, masks, multimask_output, return_logits,
                                         hq_token_only)
        return m[0].cpu().numpy(), iou[0].float().cpu().numpy(), low[0].float().cpu().numpy()

    @torch.no_grad()
    def predict_torch(self, point_coords: Optional[torch.Tensor], point_labels: Optional[torch.Tensor],
                      boxes: Optional[torch.Tensor] = None, mask_input: Optional[torch.Tensor] = None,
                      multimask_output: bool = True, return_logits: bool = False,
                      hq_token_only: bool = False) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Prompts already in the resized-input frame (transform.apply_*_torch).
        Returns (masks (P, 1, H, W) bool or logits at the original size, IoU
        predictions (P, 1), low-res logits (P, 1, 4h, 4w))."""
        if not self.is_image_set:
            raise RuntimeError("set an image with set_image before predict")
        pts = (point_coords, point_labels) if point_coords is not None else None
        pe = self.model.prompt_encoder
        sparse, dense = pe(pts, boxes, mask_input)
        low, iou = self.model.mask_decoder(self.features, pe.get_dense_pe(), sparse, dense,
                                           multimask_output, hq_token_only, self.interm_features)
        masks = self.model.postprocess_masks(low.float(), self.input_size, self.original_size)
        if not return_logits:
            masks = masks > self.model.mask_threshold
        return masks, iou, low

    def get_image_embedding(self) -> torch.Tensor:
        if not self.is_image_set:
            raise RuntimeError("set an image with set_image before reading its embedding")
        return self.features


# ---------------------------------------------------------------------------
# Builders (seeded random weights; a checkpoint's state dict loads by name)
# ---------------------------------------------------------------------------
def init_prompt_decoder_weights(model: nn.Module, seed: int = 1) -> nn.Module:
    """Seeded random init of the prompt encoder and mask decoder: Linear / Conv /
    ConvTranspose weights N(0, 1/fan_in) truncated at 2 std (activations keep unit
    scale, so mask logits are O(1)), zero biases, LayerNorms 1 / 0, embeddings and
    the Fourier matrix N(0, 1). Drawn on the CPU, so a seed names the same weights
    on every device."""
    gen = torch.Generator(device="cpu").manual_seed(seed)
    with torch.no_grad():
        for mod in model.modules():
            if isinstance(mod, (nn.Linear, nn.Conv2d, nn.ConvTranspose2d)):
                w = mod.weight
                if isinstance(mod, nn.ConvTranspose2d):
                    fan_in = w.shape[0] * w.shape[2] * w.shape[3] // (mod.stride[0] * mod.stride[1])
                else:
                    fan_in = w[0].numel()
                host._trunc_normal_(w, 1.0 / math.sqrt(max(1, fan_in)), gen)
                if mod.bias is not None:
                    mod.bias.zero_()
            elif isinstance(mod, (nn.LayerNorm, LayerNorm2d)):      # RowLayerNorm included
                mod.weight.fill_(1.0)
                mod.bias.zero_()
            elif isinstance(mod, nn.Embedding):
                mod.weight.copy_(torch.randn(mod.weight.shape, generator=gen).to(mod.weight.device))
            elif isinstance(mod, PositionEmbeddingRandom):
                g = mod.positional_encoding_gaussian_matrix
                g.copy_(torch.randn(g.shape, generator=gen).to(g.device))
    return model


def build_sam_hq(arch: str = "vit_l", checkpoint: Optional[str] = None, seed: int = 0,
                 device: str | torch.device = "cpu", img_size: int = 1024,
                 decoder_dtype: torch.dtype = torch.float32) -> SamHQ:
    """SAM-HQ ViT-B / L / H: the host image encoder (seeded weights, seed), prompt
    encoder and HQ decoder (seed + 1), or the weights of `checkpoint` when given.
    decoder_dtype sets the prompt encoder's and decoder's parameter (and so compute)
    dtype; the reference runs the whole model in half precision (eval_hq44k.py:434)."""
    enc = host.build_image_encoder(arch, seed=seed, device=device, img_size=img_size)
    grid = img_size // 16
    with torch.device(device):
        prompt = PromptEncoder(256, (grid, grid), (img_size, img_size), 16)
        decoder = MaskDecoderHQ(transformer_dim=256, transformer=TwoWayTransformer(2, 256, 8, 2048),
                                num_multimask_outputs=3, iou_head_depth=3, iou_head_hidden_dim=256,
                                vit_dim=host.VIT_CONFIGS[arch]["embed_dim"])
    init_prompt_decoder_weights(nn.ModuleList([prompt, decoder]), seed + 1)
    sam = SamHQ(enc, prompt, decoder).to(device)
    if checkpoint is not None:
        state = torch.load(checkpoint, map_location=device)
        if isinstance(state, dict) and "model" in state:
            state = state["model"]
        # extra entries are tolerated; a parameter of this model left unset is an error
        missing = sam.load_state_dict(state, strict=False).missing_keys
        if missing:
            raise KeyError(f"checkpoint {checkpoint} lacks {len(missing)} parameters, e.g. {missing[:3]}")
    sam.prompt_encoder.to(decoder_dtype)
    sam.mask_decoder.to(decoder_dtype)
    return sam.eval()


sam_model_registry = {
    "default": partial(build_sam_hq, "vit_h"),
    "vit_h": partial(build_sam_hq, "vit_h"),
    "vit_l": partial(build_sam_hq, "vit_l"),
    "vit_b": partial(build_sam_hq, "vit_b"),
}


# ---------------------------------------------------------------------------
# HQ-44K evaluation helpers (SAM-HQ's train.utils.misc / train.train, restated)
# ---------------------------------------------------------------------------
def masks_to_boxes(masks: torch.Tensor) -> torch.Tensor:
    """(N, H, W) masks (nonzero = foreground) -> (N, 4) float boxes (x0, y0, x1, y1),
    the inclusive pixel extent of the foreground. An empty mask gives
    (1e8, 1e8, 0, 0)."""
    if masks.numel() == 0:
        return torch.zeros(0, 4, device=masks.device)
    fg = masks != 0
    n, h, w = fg.shape
    cols, rows = fg.any(dim=1), fg.any(dim=2)
    xi = torch.arange(w, device=masks.device, dtype=torch.float32)
    yi = torch.arange(h, device=masks.device, dtype=torch.float32)
    big = torch.tensor(1e8, device=masks.device)
    zero = torch.tensor(0.0, device=masks.device)
    x0 = torch.where(cols, xi, big).amin(dim=1)
    x1 = torch.where(cols, xi, zero).amax(dim=1)
    y0 = torch.where(rows, yi, big).amin(dim=1)
    y1 = torch.where(rows, yi, zero).amax(dim=1)
    return torch.stack([x0, y0, x1, y1], dim=1)


def _pred_fg(pred: torch.Tensor) -> torch.Tensor:
    return pred if pred.dtype == torch.bool else pred > 0


def _label_fg(label: torch.Tensor, threshold: float = 128) -> torch.Tensor:
    return label if label.dtype == torch.bool else label > threshold


def mask_iou(pred: torch.Tensor, label: torch.Tensor) -> torch.Tensor:
    """IoU of pred > 0 (logits or a bool mask) and label > 128 (0..255 labels)."""
    p, g = _pred_fg(pred), _label_fg(label)
    inter = (p & g).sum().float()
    union = (p | g).sum().float()
    return inter / union


def mask_to_boundary(mask: torch.Tensor, dilation_ratio: float = 0.02) -> torch.Tensor:
    """Boundary band of a bool (H, W) mask: the mask minus its erosion by a square of
    radius d = max(1, round(dilation_ratio * image diagonal)), with everything
    outside the image counted as background (Cheng et al., "Boundary IoU", CVPR 2021).
    d iterations of a 3x3 erosion equal one erosion by the (2d+1)^2 square; it is
    computed as two 1-D max filters of the complement."""
    h, w = mask.shape[-2:]
    d = max(1, int(round(dilation_ratio * math.sqrt(h * h + w * w))))
    k = 2 * d + 1
    bg = (~mask).to(torch.float32)[None, None]
    bg = F.pad(bg, (d, d, d, d), value=1.0)
    bg = F.max_pool2d(bg, (k, 1), stride=1)
    bg = F.max_pool2d(bg, (1, k), stride=1)
    eroded = bg[0, 0] < 0.5
    return mask & ~eroded


def boundary_iou(label: torch.Tensor, pred: torch.Tensor, dilation_ratio: float = 0.02) -> torch.Tensor:
    """Boundary IoU of label > 128 and pred > 0, (H, W) each."""
    g = mask_to_boundary(_label_fg(label), dilation_ratio)
    p = mask_to_boundary(_pred_fg(pred), dilation_ratio)
    return (g & p).sum().float() / (g | p).sum().float()


def _to_target_size(preds: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    if preds.shape[-2:] == target.shape[-2:]:
        return preds
    # bool masks resample as 0 / 1 and stay masks (> 0.5); logits resample as logits
    if preds.dtype == torch.bool:
        return F.interpolate(preds.float(), target.shape[-2:], mode="bilinear", align_corners=False) > 0.5
    return F.interpolate(preds.float(), target.shape[-2:], mode="bilinear", align_corners=False)


def compute_iou(preds: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    """Mean mask IoU over the batch; preds (N, 1, H, W) resized to target's size."""
    if target.shape[1] != 1:
        raise ValueError("one mask per image")
    p = _to_target_size(preds, target)
    return torch.stack([mask_iou(p[i, 0], target[i, 0]) for i in range(p.shape[0])]).mean()


def compute_boundary_iou(preds: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    """Mean boundary IoU over the batch; preds (N, 1, H, W) resized to target's size."""
    if target.shape[1] != 1:
        raise ValueError("one mask per image")
    p = _to_target_size(preds, target)
    return torch.stack([boundary_iou(target[i, 0], p[i, 0]) for i in range(p.shape[0])]).mean()


def process_batch(predictor: SamPredictor, images: torch.Tensor, labels_boxes: torch.Tensor,
                  labels_ori: torch.Tensor, hq_token_only: bool = True) -> Dict[str, float]:
    """One encoder forward of the batch and one box-prompted decode per image
    (eval_hq44k.py:87-129, same arguments and result keys). The decode of all the
    batch's boxes is a single decoder pass (box i on image i); the encoder time is
    taken with CUDA events on the current stream (host clock on a CPU model)."""
    device = predictor.device
    images = images.to(device)
    boxes = labels_boxes.to(device, dtype=torch.float32)
    labels_ori = labels_ori.to(device)
    model = predictor.model
    x = model.preprocess(images)
    cuda = device.type == "cuda"
    with torch.no_grad():
        if cuda:
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
            features, interm = model.image_encoder(x)
            ev1.record()
            ev1.synchronize()
            encoder_ms = ev0.elapsed_time(ev1)
        else:
            import time
            t0 = time.perf_counter()
            features, interm = model.image_encoder(x)
            encoder_ms = (time.perf_counter() - t0) * 1e3
    predictor.features, predictor.interm_features = features, interm
    predictor.original_size = tuple(images.shape[2:])
    predictor.input_size = tuple(x.shape[-2:])
    predictor.is_image_set = True
    masks, _, _ = predictor.predict_torch(None, None, boxes=boxes, hq_token_only=hq_token_only)
    b = images.shape[0]
    return {
        "encoder_ms": encoder_ms,
        "encoder_per_image_ms": encoder_ms / b,
        "iou": compute_iou(masks, labels_ori).item(),
        "boundary_iou": compute_boundary_iou(masks, labels_ori).item(),
    }


class GraphedBoxStep:
    """One predictor step for a fixed batch of square images — preprocess, image
    encoder, one box prompt per image through the prompt encoder and decoder, masks
    resized to the image size and thresholded — captured once as a CUDA graph and
    replayed. At small batches the eager step is launch-bound (the decoder alone is
    a few hundred short kernels); a replay issues them with one launch.

    step = GraphedBoxStep(sam, batch)
    masks, iou, low_res = step(images, boxes)   # images (B, 3, S, S) 0..255, boxes (B, 4)

    The outputs are the graph's own buffers, overwritten by the next call (clone to
    keep). The model's weights and the patch state are read when captured: capture
    again after changing either."""

    def __init__(self, sam: SamHQ, batch: int, hq_token_only: bool = True, multimask_output: bool = False,
                 image_dtype: torch.dtype = torch.uint8, warmup: int = 2):
        dev = sam.device
        if dev.type != "cuda":
            raise ValueError("GraphedBoxStep needs the model on a CUDA device")
        s = sam.image_encoder.img_size
        self.sam = sam
        self.images = torch.zeros(batch, 3, s, s, dtype=image_dtype, device=dev)
        self.boxes = torch.zeros(batch, 4, dtype=torch.float32, device=dev)
        self.boxes[:, 2:] = s - 1
        pred = SamPredictor(sam)

        def body():
            x = sam.preprocess(self.images)
            pred.features, pred.interm_features = sam.image_encoder(x)
            pred.original_size = pred.input_size = (s, s)
            pred.is_image_set = True
            return pred.predict_torch(None, None, boxes=self.boxes, multimask_output=multimask_output,
                                      hq_token_only=hq_token_only)

        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.no_grad(), torch.cuda.stream(side):
            for _ in range(warmup):   # library work spaces and autotuning outside the capture
                body()
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(self.graph):
            self.masks, self.iou, self.low_res = body()

    def __call__(self, images: torch.Tensor, boxes: torch.Tensor):
        self.images.copy_(images, non_blocking=True)
        self.boxes.copy_(boxes, non_blocking=True)
        self.graph.replay()
        return self.masks, self.iou, self.low_res


def synthetic_box_batch(batch: int, seed: int, img_size: int = 1024, device="cpu"):
    """Seeded stand-in for an HQ-44K batch (the dataset is not available): uniform
    noise pixels with one filled ellipse per image drawn in a random colour.
    Returns (images (B, 3, S, S) fp32 in 0..255, labels (B, 1, S, S) fp32 0 / 255,
    boxes (B, 4) = masks_to_boxes(labels), the reference's box prompt)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    s = img_size
    images = torch.randint(0, 256, (batch, 3, s, s), generator=g, dtype=torch.int32).float()
    yy, xx = torch.meshgrid(torch.arange(s, dtype=torch.float32), torch.arange(s, dtype=torch.float32),
                            indexing="ij")
    labels = torch.zeros(batch, 1, s, s)
    for i in range(batch):
        cx, cy = (torch.rand(2, generator=g) * 0.5 + 0.25) * s
        ax, ay = (torch.rand(2, generator=g) * 0.25 + 0.05) * s
        inside = ((xx - cx) / ax) ** 2 + ((yy - cy) / ay) ** 2 <= 1.0
        colour = torch.randint(0, 256, (3,), generator=g).float()
        images[i][:, inside] = colour.view(3, 1)
        labels[i, 0][inside] = 255.0
    boxes = masks_to_boxes(labels[:, 0])
    return images.to(device), labels.to(device), boxes.to(device)
