"""The SAM-HQ decoder (sparsesam_b200.hq) against third-party implementations of the
same published architectures: the installed transformers' SamModel (SAM's prompt
encoder and two-way mask decoder) and SamHQModel (SAM-HQ), with our weights mapped
onto their parameter names. SAM-HQ's own package (the reference's unvendored
algos/3rd_party/sam-hq submodule) is absent, so these pin the decoder's arithmetic.

transformers 5.5.0's SamHQMaskDecoder upscales its transformer's INPUT map (image
embedding + dense prompt embedding, H and W transposed) instead of the transformer's
image-token output, which it discards (`point_embedding, iou_token_out =
self.transformer(...)`, then overwritten); SAM and SAM-HQ upscale the output. The
SAM components are therefore pinned on SamModel, the HQ-specific stages on
SamHQModel one by one, and the whole HQ decode (tokens, IoU head and masks) on
SamHQModel with that one reading substituted.
"""
import pytest
import torch

from sparsesam_b200 import hq

pytest.importorskip("transformers.models.sam_hq")
from transformers import SamConfig, SamHQConfig, SamHQModel, SamModel  # noqa: E402
from transformers.models.sam.configuration_sam import (  # noqa: E402
    SamMaskDecoderConfig, SamPromptEncoderConfig, SamVisionConfig)
from transformers.models.sam_hq.configuration_sam_hq import (  # noqa: E402
    SamHQMaskDecoderConfig, SamHQPromptEncoderConfig, SamHQVisionConfig)

IMG = 256
G = IMG // 16
VIT = 768


def _hf_names():
    """transformers' parameter-name prefixes -> ours (SAM-HQ checkpoint names)."""
    m = {"prompt_encoder.shared_embedding.positional_embedding": "prompt_encoder.pe_layer.positional_encoding_gaussian_matrix",
         "shared_image_embedding.positional_embedding": "prompt_encoder.pe_layer.positional_encoding_gaussian_matrix"}
    pre = {
        "prompt_encoder.mask_embed.conv1": "prompt_encoder.mask_downscaling.0",
        "prompt_encoder.mask_embed.layer_norm1": "prompt_encoder.mask_downscaling.1",
        "prompt_encoder.mask_embed.conv2": "prompt_encoder.mask_downscaling.3",
        "prompt_encoder.mask_embed.layer_norm2": "prompt_encoder.mask_downscaling.4",
        "prompt_encoder.mask_embed.conv3": "prompt_encoder.mask_downscaling.6",
        "prompt_encoder.no_mask_embed": "prompt_encoder.no_mask_embed",
        "prompt_encoder.not_a_point_embed": "prompt_encoder.not_a_point_embed",
        "mask_decoder.iou_token": "mask_decoder.iou_token",
        "mask_decoder.mask_tokens": "mask_decoder.mask_tokens",
        "mask_decoder.hq_token": "mask_decoder.hf_token",
        "mask_decoder.transformer.final_attn_token_to_image": "mask_decoder.transformer.final_attn_token_to_image",
        "mask_decoder.transformer.layer_norm_final_attn": "mask_decoder.transformer.norm_final_attn",
        "mask_decoder.upscale_conv1": "mask_decoder.output_upscaling.0",
        "mask_decoder.upscale_layer_norm": "mask_decoder.output_upscaling.1",
        "mask_decoder.upscale_conv2": "mask_decoder.output_upscaling.3",
        "mask_decoder.compress_vit_conv1": "mask_decoder.compress_vit_feat.0",
        "mask_decoder.compress_vit_norm": "mask_decoder.compress_vit_feat.1",
        "mask_decoder.compress_vit_conv2": "mask_decoder.compress_vit_feat.3",
        "mask_decoder.encoder_conv1": "mask_decoder.embedding_encoder.0",
        "mask_decoder.encoder_norm": "mask_decoder.embedding_encoder.1",
        "mask_decoder.encoder_conv2": "mask_decoder.embedding_encoder.3",
        "mask_decoder.mask_conv1": "mask_decoder.embedding_maskfeature.0",
        "mask_decoder.mask_norm": "mask_decoder.embedding_maskfeature.1",
        "mask_decoder.mask_conv2": "mask_decoder.embedding_maskfeature.3",
    }

    def mlp(theirs, ours):
        pre.update({f"{theirs}.proj_in": f"{ours}.layers.0", f"{theirs}.layers.0": f"{ours}.layers.1",
                    f"{theirs}.proj_out": f"{ours}.layers.2"})

    for i in range(4):
        pre[f"prompt_encoder.point_embed.{i}"] = f"prompt_encoder.point_embeddings.{i}"
        mlp(f"mask_decoder.output_hypernetworks_mlps.{i}", f"mask_decoder.output_hypernetworks_mlps.{i}")
    mlp("mask_decoder.iou_prediction_head", "mask_decoder.iou_prediction_head")
    mlp("mask_decoder.hq_mask_mlp", "mask_decoder.hf_mlp")
    for layer in range(2):
        t = f"mask_decoder.transformer.layers.{layer}"
        for a in ("self_attn", "cross_attn_token_to_image", "cross_attn_image_to_token", "mlp"):
            pre[f"{t}.{a}"] = f"{t}.{a}"
        for n in range(1, 5):
            pre[f"{t}.layer_norm{n}"] = f"{t}.norm{n}"
    return m, pre


def _load_ours_into(model, ours_sd):
    full, pre = _hf_names()
    state = {}
    for k in model.state_dict():
        if k.startswith("vision_encoder"):
            continue
        if k in full:
            state[k] = ours_sd[full[k]]
            continue
        hit = [p for p in pre if k.startswith(p + ".")]
        assert len(hit) == 1, k
        state[k] = ours_sd[pre[hit[0]] + k[len(hit[0]):]]
    res = model.load_state_dict(state, strict=False)
    assert not [k for k in res.missing_keys if not k.startswith("vision_encoder")] and not res.unexpected_keys
    return model.eval()


@pytest.fixture(scope="module")
def setup():
    torch.manual_seed(0)
    ours = hq.build_sam_hq("vit_b", img_size=IMG)
    g = torch.Generator().manual_seed(11)
    feats = torch.randn(3, 256, G, G, generator=g)
    interm = [torch.randn(3, G, G, VIT, generator=g) for _ in range(4)]
    boxes = torch.tensor([[10.0, 20.0, 100.0, 200.0], [0.0, 0.0, 255.0, 255.0], [50.0, 60.0, 70.0, 80.0]])
    return ours, feats, interm, boxes


@torch.no_grad()
def test_sam_components_match_transformers_sam(setup):
    """SAM's parts of the decoder against SamModel on identical inputs: the prompt
    encoder (box corners, dense no-mask embedding, image-wide position encoding),
    the two-way transformer on SAM's seven tokens (IoU, four mask tokens, two box
    corners; SAM-HQ adds its HQ token to the same attention, so its SAM-token
    outputs are not SAM's), the upscaling and the hypernetwork / IoU heads."""
    ours, feats, interm, boxes = setup
    cfg = SamConfig(vision_config=SamVisionConfig(image_size=IMG, num_hidden_layers=1),
                    prompt_encoder_config=SamPromptEncoderConfig(image_size=IMG, image_embedding_size=G),
                    mask_decoder_config=SamMaskDecoderConfig())
    ref = _load_ours_into(SamModel(cfg), ours.state_dict())
    sparse, dense = ours.prompt_encoder(None, boxes, None)
    sp_ref, de_ref = ref.prompt_encoder(input_points=None, input_labels=None, input_boxes=boxes[:, None],
                                        input_masks=None)
    assert (sparse - sp_ref[:, 0]).abs().max().item() <= 1e-5
    assert torch.equal(dense, de_ref)
    pe = ours.prompt_encoder.get_dense_pe()
    assert (pe - ref.get_image_wide_positional_embeddings()).abs().max().item() <= 1e-5
    dec = ours.mask_decoder
    tokens = torch.cat([torch.cat([dec.iou_token.weight, dec.mask_tokens.weight], 0).unsqueeze(0).expand(3, -1, -1),
                        sparse], dim=1)
    src = feats + dense
    pos = pe.expand(3, -1, -1, -1)
    q, k = dec.transformer(src, pos, tokens)
    q_ref, k_ref = ref.mask_decoder.transformer(point_embeddings=tokens[:, None], image_embeddings=src,
                                                image_positional_embeddings=pos, attention_similarity=None)[:2]
    assert (q - q_ref[:, 0]).abs().max().item() <= 1e-4 * q_ref.abs().max().item()
    assert (k - k_ref[:, 0]).abs().max().item() <= 1e-4 * k_ref.abs().max().item()
    rd = ref.mask_decoder
    x = torch.randn(3, 256, G, G)
    up = dec.output_upscaling(x)
    up_ref = rd.activation(rd.upscale_conv2(rd.activation(rd.upscale_layer_norm(rd.upscale_conv1(x)))))
    assert (up - up_ref).abs().max().item() <= 1e-5 * up_ref.abs().max().item()
    t = torch.randn(3, 256)
    assert (dec.iou_prediction_head(t) - rd.iou_prediction_head(t)).abs().max().item() <= 1e-5
    for i in range(4):
        assert (dec.output_hypernetworks_mlps[i](t) - rd.output_hypernetworks_mlps[i](t)).abs().max().item() <= 1e-5


@torch.no_grad()
def test_hq_stages_match_transformers_sam_hq(setup):
    ours, feats, interm, boxes = setup
    cfg = SamHQConfig(vision_config=SamHQVisionConfig(image_size=IMG, num_hidden_layers=1),
                      prompt_encoder_config=SamHQPromptEncoderConfig(image_size=IMG, image_embedding_size=G),
                      mask_decoder_config=SamHQMaskDecoderConfig(vit_dim=VIT))
    ref = _load_ours_into(SamHQModel(cfg), ours.state_dict())
    dec, rd = ours.mask_decoder, ref.mask_decoder
    act = rd.activation
    vit = interm[0].permute(0, 3, 1, 2).contiguous()
    x = torch.randn(3, 256, G, G)
    y = torch.randn(3, 32, 4 * G, 4 * G)
    t = torch.randn(3, 256)
    pairs = [
        (dec.embedding_encoder(feats), rd.encoder_conv2(act(rd.encoder_norm(rd.encoder_conv1(feats))))),
        (dec.compress_vit_feat(vit), rd.compress_vit_conv2(act(rd.compress_vit_norm(rd.compress_vit_conv1(vit))))),
        (dec.output_upscaling(x), act(rd.upscale_conv2(act(rd.upscale_layer_norm(rd.upscale_conv1(x)))))),
        (dec.embedding_maskfeature(y), rd.mask_conv2(act(rd.mask_norm(rd.mask_conv1(y))))),
        (dec.hf_mlp(t), rd.hq_mask_mlp(t)),
    ]
    for a, b in pairs:
        assert (a - b).abs().max().item() <= 1e-5 * b.abs().max().item()
    # the whole decode, with transformers' reading of the upscaling input substituted
    orig = dec.transformer.forward

    def transposed_input(src, pos, tokens):
        q, _ = orig(src, pos, tokens)
        b, c, h, w = src.shape
        return q, src.transpose(2, 3).reshape(b, c, h * w).transpose(1, 2)

    dec.transformer.forward = transposed_input
    try:
        pred = hq.SamPredictor(ours)
        pred.features, pred.interm_features = feats, interm
        pred.original_size = pred.input_size = (IMG, IMG)
        pred.is_image_set = True
        for hq_only in (True, False):
            _, iou, low = pred.predict_torch(None, None, boxes=boxes, multimask_output=False, hq_token_only=hq_only)
            out = ref(image_embeddings=feats, intermediate_embeddings=interm, input_boxes=boxes[:, None],
                      multimask_output=False, hq_token_only=hq_only)
            want = out.pred_masks.reshape(low.shape)
            assert (low - want).abs().max().item() <= 1e-4 * want.abs().max().item()
            assert (iou - out.iou_scores.reshape(iou.shape)).abs().max().item() <= 1e-4
    finally:
        dec.transformer.forward = orig
