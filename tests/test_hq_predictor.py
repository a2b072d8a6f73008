"""SAM-HQ predictor host (sparsesam_b200.hq) on the CPU: the decoder module against
the fp64 restatement (oracle/decoder.py), batching and broadcast semantics, the
checkpoint parameter layout, and the HQ-44K helpers (masks_to_boxes, mask IoU,
boundary IoU) against plain numpy / scipy restatements.

The caller being mirrored is tasks/sam_hq44k/eval_hq44k.py:87-129 (process_batch:
encoder forward, predict_torch(boxes=..., hq_token_only=True), compute_iou /
compute_boundary_iou). SAM-HQ's own source and checkpoints are absent, so the
decoder's parity with SAM-HQ is unpinned; these tests pin the module to the
restatement and the helpers to their definitions.
"""
import math

import numpy as np
import pytest
import torch

from oracle import decoder as od
from sparsesam_b200 import hq

IMG = 256          # a 16 x 16 token grid keeps the CPU runs short
GRID = IMG // 16


@pytest.fixture(scope="module")
def sam():
    torch.manual_seed(0)
    return hq.build_sam_hq("vit_b", img_size=IMG)


def _inputs(B, seed=0, C=768):
    g = torch.Generator().manual_seed(seed)
    feats = torch.randn(B, 256, GRID, GRID, generator=g)
    interm0 = torch.randn(B, GRID, GRID, C, generator=g)
    xy0 = torch.rand(B, 2, generator=g) * (IMG / 2)
    wh = torch.rand(B, 2, generator=g) * (IMG / 2) + 4
    boxes = torch.cat([xy0, (xy0 + wh).clamp(max=IMG - 1)], dim=1).round()
    return feats, interm0, boxes


def _predictor(sam, feats, interm0):
    p = hq.SamPredictor(sam)
    p.features, p.interm_features = feats, [interm0]
    p.original_size = p.input_size = (IMG, IMG)
    p.is_image_set = True
    return p


@pytest.mark.parametrize("multimask", [False, True])
@pytest.mark.parametrize("hq_only", [True, False])
def test_decoder_matches_restatement(sam, multimask, hq_only):
    feats, interm0, boxes = _inputs(3)
    pred = _predictor(sam, feats, interm0)
    logits, iou, low = pred.predict_torch(None, None, boxes=boxes, multimask_output=multimask,
                                          hq_token_only=hq_only, return_logits=True)
    ref_low, ref_iou = od.decode_boxes(sam.state_dict(), feats, interm0, boxes, (IMG, IMG), multimask, hq_only)
    ref = od.postprocess(ref_low, IMG, (IMG, IMG), (IMG, IMG))
    scale = ref_low.abs().max().item()
    assert low.shape == (3, 1, 4 * GRID, 4 * GRID) and logits.shape == (3, 1, IMG, IMG)
    assert (low.double() - ref_low).abs().max().item() <= 1e-5 * scale + 1e-5
    assert (logits.double() - ref).abs().max().item() <= 1e-5 * scale + 1e-5
    assert (iou.double() - ref_iou).abs().max().item() <= 1e-5
    masks, _, _ = pred.predict_torch(None, None, boxes=boxes, multimask_output=multimask, hq_token_only=hq_only)
    assert masks.dtype == torch.bool and torch.equal(masks, logits > 0)


def test_batched_decode_equals_per_image(sam):
    feats, interm0, boxes = _inputs(4, seed=1)
    _, iou_b, low_b = _predictor(sam, feats, interm0).predict_torch(None, None, boxes=boxes,
                                                                    hq_token_only=True)
    for i in range(4):
        _, iou_i, low_i = _predictor(sam, feats[i:i + 1], interm0[i:i + 1]).predict_torch(
            None, None, boxes=boxes[i:i + 1], hq_token_only=True)
        assert torch.allclose(low_b[i:i + 1], low_i, rtol=1e-5, atol=1e-5)
        assert torch.allclose(iou_b[i:i + 1], iou_i, rtol=1e-5, atol=1e-6)


def test_one_image_many_prompts_broadcasts(sam):
    feats, interm0, boxes = _inputs(3, seed=2)
    _, _, low_bc = _predictor(sam, feats[:1], interm0[:1]).predict_torch(None, None, boxes=boxes,
                                                                         hq_token_only=False)
    _, _, low_rep = _predictor(sam, feats[:1].expand(3, -1, -1, -1).contiguous(),
                               interm0[:1].expand(3, -1, -1, -1).contiguous()).predict_torch(
        None, None, boxes=boxes, hq_token_only=False)
    assert torch.allclose(low_bc, low_rep, rtol=1e-5, atol=1e-5)
    with pytest.raises(ValueError):
        _predictor(sam, feats[:2], interm0[:2]).predict_torch(None, None, boxes=boxes)


def test_point_prompts(sam):
    """Point embeddings: pe(p + 0.5) + label embedding; a padding point (label -1,
    appended when no box is given) is not_a_point_embed alone."""
    pe = sam.prompt_encoder
    pts = torch.tensor([[[10.0, 20.0], [100.0, 5.0]]])
    lab = torch.tensor([[1, 0]])
    sparse, dense = pe((pts, lab), None, None)
    assert sparse.shape == (1, 3, 256) and dense.shape == (1, 256, GRID, GRID)
    G = pe.pe_layer.positional_encoding_gaussian_matrix.double()
    for j, (p, l) in enumerate(zip(pts[0], lab[0])):
        u = 2 * math.pi * ((2 * ((p.double() + 0.5) / IMG) - 1) @ G)
        want = torch.cat([u.sin(), u.cos()]) + pe.point_embeddings[int(l)].weight[0].double()
        assert torch.allclose(sparse[0, j].double(), want, atol=1e-5)
    assert torch.equal(sparse[0, 2], pe.not_a_point_embed.weight[0])
    # with a box the points are not padded; the box adds its two corner tokens
    sparse2, _ = pe((pts, lab), torch.tensor([[1.0, 2.0, 30.0, 40.0]]), None)
    assert sparse2.shape == (1, 4, 256)
    # a dense mask prompt replaces no_mask_embed
    _, dmask = pe(None, None, torch.randn(1, 1, 4 * GRID, 4 * GRID))
    assert dmask.shape == (1, 256, GRID, GRID)


def test_checkpoint_layout(sam):
    """Parameter names and shapes of SAM-HQ's checkpoints (so a state dict loads by name)."""
    sd = sam.state_dict()
    want = {
        "prompt_encoder.pe_layer.positional_encoding_gaussian_matrix": (2, 128),
        "prompt_encoder.point_embeddings.3.weight": (1, 256),
        "prompt_encoder.not_a_point_embed.weight": (1, 256),
        "prompt_encoder.mask_downscaling.6.weight": (256, 16, 1, 1),
        "prompt_encoder.no_mask_embed.weight": (1, 256),
        "mask_decoder.iou_token.weight": (1, 256),
        "mask_decoder.mask_tokens.weight": (4, 256),
        "mask_decoder.hf_token.weight": (1, 256),
        "mask_decoder.transformer.layers.0.self_attn.q_proj.weight": (256, 256),
        "mask_decoder.transformer.layers.1.cross_attn_token_to_image.k_proj.weight": (128, 256),
        "mask_decoder.transformer.layers.1.cross_attn_image_to_token.out_proj.weight": (256, 128),
        "mask_decoder.transformer.layers.0.mlp.lin1.weight": (2048, 256),
        "mask_decoder.transformer.final_attn_token_to_image.v_proj.weight": (128, 256),
        "mask_decoder.transformer.norm_final_attn.weight": (256,),
        "mask_decoder.output_upscaling.0.weight": (256, 64, 2, 2),
        "mask_decoder.output_upscaling.3.weight": (64, 32, 2, 2),
        "mask_decoder.output_hypernetworks_mlps.3.layers.2.weight": (32, 256),
        "mask_decoder.iou_prediction_head.layers.2.weight": (4, 256),
        "mask_decoder.hf_mlp.layers.0.weight": (256, 256),
        "mask_decoder.compress_vit_feat.0.weight": (768, 256, 2, 2),
        "mask_decoder.compress_vit_feat.3.weight": (256, 32, 2, 2),
        "mask_decoder.embedding_encoder.3.weight": (64, 32, 2, 2),
        "mask_decoder.embedding_maskfeature.0.weight": (64, 32, 3, 3),
        "mask_decoder.embedding_maskfeature.3.weight": (32, 64, 3, 3),
        "image_encoder.patch_embed.proj.weight": (768, 3, 16, 16),
    }
    for k, shape in want.items():
        assert k in sd and tuple(sd[k].shape) == shape, k
    assert "pixel_mean" not in sd  # non-persistent buffers, as in SAM
    # a state dict round-trips into a freshly built model
    other = hq.build_sam_hq("vit_b", img_size=IMG, seed=5)
    other.load_state_dict(sd)
    assert all(torch.equal(a, b) for a, b in zip(other.state_dict().values(), sd.values()))


def test_checkpoint_loading(sam, tmp_path):
    """sam_model_registry[arch](checkpoint=...) loads a saved state dict by name;
    extra entries are tolerated, a missing parameter is an error."""
    path = tmp_path / "sam_hq_vit_b.pth"
    sd = dict(sam.state_dict())
    sd["some_extra_buffer"] = torch.zeros(1)
    torch.save(sd, path)
    loaded = hq.sam_model_registry["vit_b"](checkpoint=str(path), img_size=IMG, seed=7)
    assert all(torch.equal(a, sd[k]) for k, a in loaded.state_dict().items())
    del sd["mask_decoder.hf_token.weight"]
    torch.save(sd, path)
    with pytest.raises(KeyError):
        hq.sam_model_registry["vit_b"](checkpoint=str(path), img_size=IMG)


def _np_boxes(m):
    out = []
    for mi in m:
        ys, xs = np.nonzero(mi)
        out.append([xs.min(), ys.min(), xs.max(), ys.max()] if len(xs) else [1e8, 1e8, 0, 0])
    return np.array(out, dtype=np.float32)


def test_masks_to_boxes():
    g = torch.Generator().manual_seed(3)
    m = (torch.rand(6, 40, 56, generator=g) > 0.97).float() * 255
    m[2] = 0                                            # empty mask
    m[3] = 0
    m[3, 7, 9] = 1                                      # single pixel, value 1
    got = hq.masks_to_boxes(m).numpy()
    assert np.array_equal(got, _np_boxes(m.numpy()))
    assert hq.masks_to_boxes(torch.zeros(0, 4, 4)).shape == (0, 4)


def _np_boundary(mask, ratio=0.02):
    from scipy import ndimage
    h, w = mask.shape
    d = max(1, int(round(ratio * math.sqrt(h * h + w * w))))
    # d iterations of a 3x3 erosion, background outside the image
    er = ndimage.binary_erosion(mask, structure=np.ones((3, 3), bool), iterations=d, border_value=0)
    return mask & ~er


def test_iou_and_boundary_iou():
    g = torch.Generator().manual_seed(4)
    yy, xx = torch.meshgrid(torch.arange(96.0), torch.arange(120.0), indexing="ij")
    for trial in range(4):
        c = torch.rand(4, generator=g)
        gt = (((xx - 30 - 60 * c[0]) / (10 + 20 * c[1])) ** 2 + ((yy - 30 - 40 * c[2]) / (8 + 20 * c[3])) ** 2 <= 1)
        noise = torch.rand(96, 120, generator=g) < 0.02
        logits = torch.where(gt ^ noise, torch.tensor(3.0), torch.tensor(-3.0))
        if trial == 3:
            logits[:, :] = -1.0
            logits[0, :] = 1.0                          # a foreground touching the image edge
        label = gt.float() * 255
        p, t = logits.numpy() > 0, label.numpy() > 128
        want = (p & t).sum() / (p | t).sum()
        assert abs(hq.mask_iou(logits, label).item() - want) < 1e-7
        bp, bt = _np_boundary(p), _np_boundary(t)
        want_b = (bp & bt).sum() / (bp | bt).sum()
        assert torch.equal(hq.mask_to_boundary(torch.from_numpy(p)), torch.from_numpy(bp))
        assert abs(hq.boundary_iou(label, logits).item() - want_b) < 1e-7
    # batch means, with and without a resize to the label's size
    preds = torch.stack([logits, -logits])[:, None]
    labels = torch.stack([label, label])[:, None]
    ious = [hq.mask_iou(preds[i, 0], labels[i, 0]).item() for i in range(2)]
    assert abs(hq.compute_iou(preds, labels).item() - sum(ious) / 2) < 1e-7
    assert hq.compute_boundary_iou(preds > 0, labels).item() >= 0
    small = hq.compute_iou(torch.nn.functional.interpolate(preds, scale_factor=0.5), labels)
    assert 0 <= small.item() <= 1


def test_process_batch_cpu_host_encoder():
    """The eval step on the stock (unpatched) host encoder: same arguments and
    result keys as the reference's process_batch."""
    sam = hq.build_sam_hq("vit_b", img_size=IMG)
    pred = hq.SamPredictor(sam)
    images, labels, boxes = hq.synthetic_box_batch(2, seed=0, img_size=IMG)
    assert torch.equal(boxes, hq.masks_to_boxes(labels[:, 0]))
    r = hq.process_batch(pred, images, boxes, labels)
    assert set(r) == {"encoder_ms", "encoder_per_image_ms", "iou", "boundary_iou"}
    assert 0.0 <= r["iou"] <= 1.0 and 0.0 <= r["boundary_iou"] <= 1.0
    # the batched decode inside process_batch equals set_torch_image + predict_torch per image
    batched = hq.SamPredictor(sam)
    batched.set_torch_image(images, (IMG, IMG))
    m_b, _, _ = batched.predict_torch(None, None, boxes=boxes, hq_token_only=True)
    for i in range(2):
        pred.set_torch_image(images[i:i + 1], (IMG, IMG))
        m_i, _, _ = pred.predict_torch(None, None, boxes=boxes[i:i + 1], hq_token_only=True)
        assert (m_i[0] ^ m_b[i]).float().mean().item() < 1e-3


def test_numpy_predict_and_transform():
    sam = hq.build_sam_hq("vit_b", img_size=IMG)
    pred = hq.SamPredictor(sam)
    img = np.random.default_rng(0).integers(0, 256, (100, 200, 3), dtype=np.uint8)
    pred.set_image(img)
    assert pred.input_size == (128, 256) and pred.original_size == (100, 200)
    masks, iou, low = pred.predict(box=np.array([10, 10, 120, 80]), hq_token_only=True)
    assert masks.shape == (1, 100, 200) and masks.dtype == bool and iou.shape == (1,)
    assert low.shape == (1, 4 * GRID, 4 * GRID)
    t = hq.ResizeLongestSide(1024)
    assert t.get_preprocess_shape(100, 200, 1024) == (512, 1024)
    b = t.apply_boxes(np.array([[10.0, 20.0, 30.0, 40.0]]), (100, 200))
    assert np.allclose(b, [[51.2, 102.4, 153.6, 204.8]])
    with pytest.raises(RuntimeError):
        hq.SamPredictor(sam).predict(box=np.array([1, 2, 3, 4]))
