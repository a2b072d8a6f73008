"""The host SAM ViT encoder (sparsesam_b200/host.py, the model the patch is applied
to when SAM-HQ's segment_anything package is absent) against the SAM-HQ vision
encoder of the installed transformers package, with the same weights mapped onto
its parameter names: features (neck output) and the intermediate embeddings after
every global-attention block, on grids with and without window padding.

This pins the dense architecture the oracle (oracle/encoder.py) restates the
reference's patched forward on: patch embedding, absolute position embedding,
windowed / global attention with decomposed relative-position bias, MLP, neck.
"""
import pytest
import torch

from sparsesam_b200 import host

pytest.importorskip("transformers.models.sam_hq")
from transformers.models.sam_hq.configuration_sam_hq import SamHQVisionConfig  # noqa: E402
from transformers.models.sam_hq.modeling_sam_hq import SamHQVisionEncoder  # noqa: E402


def _theirs_name(k: str) -> str:
    k = k.replace("patch_embed.proj.", "patch_embed.projection.")
    k = k.replace("blocks.", "layers.").replace(".norm1.", ".layer_norm1.").replace(".norm2.", ".layer_norm2.")
    for ours, theirs in (("neck.0.", "neck.conv1."), ("neck.1.", "neck.layer_norm1."), ("neck.2.", "neck.conv2."),
                         ("neck.3.", "neck.layer_norm2.")):
        k = k.replace(ours, theirs)
    return k


@pytest.mark.parametrize("img", [256, 448])   # 16 x 16 tokens (windows padded to 28), 28 x 28 (no padding)
@torch.no_grad()
def test_host_encoder_matches_transformers_sam_hq(img):
    enc = host.build_image_encoder("vit_b", seed=3, img_size=img).eval()
    cfg = host.VIT_CONFIGS["vit_b"]
    ref = SamHQVisionEncoder(SamHQVisionConfig(image_size=img, hidden_size=cfg["embed_dim"],
                                               num_hidden_layers=cfg["depth"], num_attention_heads=cfg["num_heads"],
                                               global_attn_indexes=list(cfg["global_attn_indexes"]))).eval()
    state = {_theirs_name(k): v for k, v in enc.state_dict().items()}
    res = ref.load_state_dict(state, strict=True)
    assert not res.missing_keys and not res.unexpected_keys
    x = host.synthetic_images(2, seed=1, img_size=img)
    feats, interm = enc(x)
    out = ref(x)
    want = out.last_hidden_state
    assert feats.shape == want.shape and len(interm) == len(out.intermediate_embeddings) == 4
    assert (feats - want).abs().max().item() <= 1e-4 * want.abs().max().item()
    for a, b in zip(interm, out.intermediate_embeddings):
        assert (a - b).abs().max().item() <= 1e-4 * b.abs().max().item()
