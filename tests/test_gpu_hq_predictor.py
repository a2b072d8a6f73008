"""The SAM-HQ predictor end to end on the GPU: the patched encoder (B200 kernels)
and the HQ decoder (sparsesam_b200.hq) against the fp32 oracle encoder
(oracle/encoder.py, on the GPU's permutations) and the fp64 decoder restatement
(oracle/decoder.py), on SAM ViT-B 1024^2 at density 0.3 with box prompts — the
call sequence of tasks/sam_hq44k/eval_hq44k.py:87-129.

Tolerances come from the number format: running the fp32 oracle encoder with
bf16-rounded GEMM operands moves the low-res mask logits by 2.2e-2 (0.4 % of
their range), their cosine to 0.999995 and the thresholded masks to an IoU of
0.997 with the fp32 masks (ViT-B, these inputs, both decode modes). The GPU is
held to max-abs <= 1 % of the logit range, cosine >= 0.9999 and mask IoU >= 0.99,
with the decoder in fp32 and in fp16 (the reference runs its model in half
precision; an fp16 decoder moves the logits by about 0.2 % of their range).
"""
import pytest
import torch

from oracle import decoder as od
from oracle import encoder as oenc
from sparsesam_b200 import hq, registry

pytestmark = pytest.mark.gpu

RATIO = 0.3
_RUN: dict = {}


def _forced(enc):
    pc = enc.tome_info.get("perm_cache", {})
    return {k: tuple(t.long().cpu() for t in v) for k, v in pc.items() if isinstance(k[0], int) and len(v) == 3}


def _setup(cuda_device):
    if _RUN:
        return _RUN
    sam = hq.build_sam_hq("vit_b", img_size=1024, device=cuda_device)
    registry.apply_sam(sam.image_encoder, "sparsesam", ratio=RATIO)
    images, labels, boxes = hq.synthetic_box_batch(2, seed=0)
    pred = hq.SamPredictor(sam)
    pred.set_torch_image(images.to(cuda_device), (1024, 1024))
    forced = _forced(sam.image_encoder)
    cpu = hq.build_sam_hq("vit_b", img_size=1024)      # same seeds: the same weights
    feats, interm = oenc.encoder_forward(cpu.image_encoder, cpu.preprocess(images), RATIO, forced_perms=forced)
    # the same model with an fp16 prompt encoder / decoder, sharing the encoder's features
    half = hq.build_sam_hq("vit_b", img_size=1024, device=cuda_device, decoder_dtype=torch.float16)
    pred16 = hq.SamPredictor(half)
    pred16.features, pred16.interm_features = pred.features, pred.interm_features
    pred16.original_size, pred16.input_size, pred16.is_image_set = pred.original_size, pred.input_size, True
    _RUN.update(sam=sam, pred=pred, pred16=pred16, cpu=cpu, images=images, labels=labels, boxes=boxes,
                feats=feats, interm0=interm[0])
    return _RUN


@pytest.mark.parametrize("multimask,hq_only,decoder", [(False, True, "fp32"), (True, False, "fp32"),
                                                       (False, True, "fp16")])
def test_predictor_matches_oracle(cuda_device, multimask, hq_only, decoder):
    r = _setup(cuda_device)
    pred = r["pred"] if decoder == "fp32" else r["pred16"]
    logits, iou, low = pred.predict_torch(None, None, boxes=r["boxes"].to(cuda_device),
                                          multimask_output=multimask, hq_token_only=hq_only,
                                          return_logits=True)
    ref_low, ref_iou = od.decode_boxes(r["cpu"].state_dict(), r["feats"], r["interm0"], r["boxes"],
                                       (1024, 1024), multimask, hq_only)
    low = low.double().cpu()
    rng = ref_low.abs().max().item()
    err = (low - ref_low).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(low.flatten(), ref_low.flatten(), dim=0).item()
    assert err <= 1e-2 * rng and cos >= 0.9999, f"low-res logits: max-abs {err:.3e} (range {rng:.2f}) cos {cos:.6f}"
    assert (iou.double().cpu() - ref_iou).abs().max().item() <= 1e-2 * max(1.0, ref_iou.abs().max().item())
    m = logits.cpu() > 0
    m_ref = od.postprocess(ref_low, 1024, (1024, 1024), (1024, 1024)) > 0
    agree = ((m & m_ref).sum() / (m | m_ref).sum()).item()
    assert agree >= 0.99, f"mask IoU with the oracle's masks {agree:.4f}"


def test_decoder_alone_on_gpu_features(cuda_device):
    """The decoder's own GPU arithmetic: the GPU's features decoded on the GPU and
    by the fp64 restatement."""
    r = _setup(cuda_device)
    pred = r["pred"]
    _, _, low = pred.predict_torch(None, None, boxes=r["boxes"].to(cuda_device), hq_token_only=True)
    ref_low, _ = od.decode_boxes(r["cpu"].state_dict(), pred.features.cpu(), pred.interm_features[0].cpu(),
                                 r["boxes"], (1024, 1024), False, True)
    err = (low.double().cpu() - ref_low).abs().max().item()
    assert err <= 5e-3 * ref_low.abs().max().item(), err


def test_process_batch_on_gpu(cuda_device):
    r = _setup(cuda_device)
    pred = hq.SamPredictor(r["sam"])
    out = hq.process_batch(pred, r["images"], r["boxes"], r["labels"])
    assert set(out) == {"encoder_ms", "encoder_per_image_ms", "iou", "boundary_iou"}
    assert out["encoder_ms"] > 0 and 0 <= out["iou"] <= 1 and 0 <= out["boundary_iou"] <= 1
    # the batched decode equals a per-image decode (the reference's loop)
    m_b, _, low_b = pred.predict_torch(None, None, boxes=r["boxes"].to(cuda_device), hq_token_only=True)
    for i in range(2):
        p1 = hq.SamPredictor(r["sam"])
        p1.features = pred.features[i:i + 1]
        p1.interm_features = [t[i:i + 1] for t in pred.interm_features]
        p1.original_size, p1.input_size, p1.is_image_set = pred.original_size, pred.input_size, True
        _, _, low_i = p1.predict_torch(None, None, boxes=r["boxes"][i:i + 1].to(cuda_device), hq_token_only=True)
        assert torch.allclose(low_b[i:i + 1], low_i, rtol=1e-3, atol=1e-3 * low_i.abs().max().item())
    ious = [hq.mask_iou(m_b[i, 0], r["labels"][i, 0].to(cuda_device)).item() for i in range(2)]
    assert abs(out["iou"] - sum(ious) / 2) < 1e-6


@pytest.mark.parametrize("batch", [1, 2])
def test_graphed_step_replays_the_eager_step(cuda_device, batch):
    """GraphedBoxStep (the whole predictor step captured as one CUDA graph) gives the
    eager step's results, replay after replay, with new inputs copied in each time."""
    r = _setup(cuda_device)
    sam = r["sam"]
    step = hq.GraphedBoxStep(sam, batch)
    pred = hq.SamPredictor(sam)
    for trial in range(2):
        images, _, boxes = hq.synthetic_box_batch(batch, seed=10 + trial)
        images = images.to(torch.uint8).to(cuda_device)
        boxes = boxes.to(cuda_device)
        masks, iou, low = step(images, boxes)
        with torch.no_grad():
            pred.set_torch_image(images, (1024, 1024))
            m_e, iou_e, low_e = pred.predict_torch(None, None, boxes=boxes, multimask_output=False,
                                                   hq_token_only=True)
        torch.cuda.synchronize()
        assert torch.allclose(low, low_e, rtol=1e-4, atol=1e-4 * low_e.abs().max().item())
        assert torch.allclose(iou, iou_e, rtol=1e-4, atol=1e-5)
        assert (masks ^ m_e).float().mean().item() < 1e-4
