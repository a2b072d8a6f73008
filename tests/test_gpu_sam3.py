"""The SAM3 MLP-merge variant on the B200 kernels (algos/sparsesam/sam3.py).

ssam_zstride_keep must reproduce the reference's _get_keep_indices bit for bit
(fixtures from tests/golden/make_golden.py, which runs the reference's own
function); the patched blocks (stock attention, RC-MLP kernels on the keep set)
are compared with the oracle's ToMeSAM3Block restatement in fp32 under the
encoder tolerances of the north star (features max-abs 2e-2, cosine 0.999).
"""
import os

import numpy as np
import pytest
import torch

from oracle import encoder as oenc
from sparsesam_b200 import host, ops
from sparsesam_b200.sparsesam import sam3
from tests._golden import SAM3_E2E_RATIO, SAM3_GRIDS, SAM3_RATIOS, e2e_encoder, load

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("H,W", SAM3_GRIDS)
def test_zstride_keep_bit_exact(cuda_device, H, W):
    g = load("golden_sam3.npz")
    for r in SAM3_RATIOS:
        gold = g[f"keep_{H}x{W}_{r}"]
        idx, rows = ops.zstride_keep(H, W, r, 3, cuda_device)
        assert np.array_equal(idx.cpu().numpy(), gold), (H, W, r)
        want = (np.arange(3)[:, None] * H * W + gold[None, :]).reshape(-1)
        assert np.array_equal(rows.cpu().numpy(), want)
    assert ops.device_error() == 0


def _check(a, b, tag):
    err = (a - b).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(a.flatten().double(), b.flatten().double(), dim=0).item()
    bound = 2e-2 if tag == "features" else 5e-3 * b.abs().max().item()
    assert err <= bound and cos >= 0.999, f"{tag}: max-abs {err:.3e} (bound {bound:.3e}) cosine {cos:.6f}"


@pytest.mark.parametrize("ratio,mlp_merge", [(SAM3_E2E_RATIO, True), (0.5, True), (0.3, False), (1.0, True)])
def test_sam3_patch_small_encoder(cuda_device, ratio, mlp_merge):
    img = host.synthetic_images(2, seed=0, img_size=256)
    enc = e2e_encoder().to(cuda_device)
    sam3.apply_patch(enc, ratio=ratio, mlp_merge=mlp_merge)
    assert all(type(b).__name__ == "ToMeSAM3Block" for b in enc.blocks)
    with torch.no_grad():
        feats, interm = enc(img.to(cuda_device))
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    ref, ref_i = oenc.sam3_encoder_forward(e2e_encoder(), img, ratio, mlp_merge)
    _check(feats.cpu(), ref, "features")
    for a, b in zip(interm, ref_i):
        _check(a.cpu(), b, "interm")
    if ratio == SAM3_E2E_RATIO and mlp_merge:   # and against the reference's own run (first image)
        g = load("golden_sam3.npz")
        _check(feats[:1].cpu(), torch.from_numpy(g["e2e_features"]), "features")


def test_sam3_patch_skipped_tokens_keep_the_residual(cuda_device):
    """Tokens outside the keep set leave a patched block with the residual
    (shortcut + attention) unchanged; kept tokens get the MLP update."""
    enc = e2e_encoder().to(cuda_device)
    blk = enc.blocks[0]
    x = torch.randn(2, 16, 16, 128, device=cuda_device)
    with torch.no_grad():
        sc = x + host.window_unpartition(blk.attn(host.window_partition(blk.norm1(x), 14)[0]), 14, (28, 28), (16, 16))
    sam3.apply_patch(enc, ratio=0.25)
    with torch.no_grad():
        y = blk(x)
    idx = ops.zstride_keep(16, 16, 0.25, 1, cuda_device)[0].long()
    skipped = torch.ones(256, dtype=torch.bool, device=cuda_device)
    skipped[idx] = False
    ys, ss = y.reshape(2, 256, 128), sc.reshape(2, 256, 128)
    torch.testing.assert_close(ys[:, skipped], ss[:, skipped], atol=1e-5, rtol=1e-5)
    assert (ys[:, ~skipped] - ss[:, ~skipped]).abs().max().item() > 1e-3


def test_sam3_patch_vit_b(cuda_device):
    """A SAM ViT-B encoder (1024^2, seed-0 weights, one image) with every block
    patched at ratio 0.3, against the oracle's ToMeSAM3Block restatement."""
    torch.set_num_threads(max(1, len(os.sched_getaffinity(0))))
    img = host.synthetic_images(1, seed=0)
    enc = host.build_image_encoder("vit_b", seed=0, device=cuda_device).eval()
    sam3.apply_patch(enc, ratio=0.3)
    with torch.no_grad():
        feats, interm = enc(img.to(cuda_device))
    ref, ref_i = oenc.sam3_encoder_forward(host.build_image_encoder("vit_b", seed=0).eval(), img, 0.3)
    _check(feats.cpu(), ref, "features")
    for a, b in zip(interm, ref_i):
        _check(a.cpu(), b, "interm")


def test_sam3_remove_patch(cuda_device):
    enc = e2e_encoder().to(cuda_device)
    sam3.apply_patch(enc, ratio=0.5)
    assert sam3.remove_patch(enc) == len(enc.blocks)
    assert all(type(b).__name__ == "Block" for b in enc.blocks)
    assert not hasattr(enc, "tome_info")
