"""The reference plugin API (AlgoSpec / register / apply_sam / remove_all_sam) on CPU."""
import pytest

from sparsesam_b200 import registry as R
from sparsesam_b200.sparsesam.sam import ToMeSAMAttention, ToMeSAMBlock
from tests._golden import e2e_encoder


class Args:
    ratios = [0.4]
    margin = 0.5
    mlp_merge = True


def test_choices_and_specs():
    assert R.choices("sam")[0] == "none"
    assert "sparsesam" in R.choices("sam")
    spec = R.spec_of("sam", "sparsesam")
    assert spec.block_class is ToMeSAMBlock and spec.attn_class is ToMeSAMAttention
    assert R.REGISTRATION_ERRORS == {}
    assert R.sam_algo_choices() == R.choices("sam")


def test_register_duplicate_raises():
    with pytest.raises(ValueError):
        R.register(R.AlgoSpec("sparsesam", "sam", lambda m, **k: m))


def test_apply_none_and_dense_are_noops():
    enc = e2e_encoder()
    assert R.apply_sam(enc, "none", ratio=0.3) is None
    assert R.apply_sam(enc, "sparsesam", ratio=1.0) is None   # registry.py:65-66
    assert not hasattr(enc, "tome_info")


def test_unknown_algorithm():
    with pytest.raises(KeyError):
        R.apply_sam(e2e_encoder(), "nope", ratio=0.5)


def test_apply_and_remove_roundtrip():
    enc = e2e_encoder()
    out = R.apply_sam(enc, "sparsesam", args=Args(), ratio=0.4)
    assert out is enc
    assert enc.tome_info == {"ratio": 0.4, "mlp_merge": True, "perm_mode": "z_interleave_sort"}
    assert all(type(b) is ToMeSAMBlock for b in enc.blocks)
    assert all(type(b.attn) is ToMeSAMAttention for b in enc.blocks)
    assert "forward" in enc.__dict__
    R.update_sam_ratio(enc, 0.3)
    assert enc.tome_info["ratio"] == 0.3
    n = R.remove_all_sam(enc)
    assert n == 2 * len(enc.blocks)
    assert not hasattr(enc, "tome_info") and "forward" not in enc.__dict__
    assert R.remove_all_sam(enc) == 0            # idempotent


def test_kwargs_forwarding_and_validation():
    enc = e2e_encoder()
    R.apply_sam(enc, "sparsesam", ratio=0.5, mlp_merge=False, perm_mode="z_naive_sort", unknown_kw=3)
    assert enc.tome_info == {"ratio": 0.5, "mlp_merge": False, "perm_mode": "z_naive_sort"}
    R.remove_all_sam(enc)
    with pytest.raises(AssertionError):
        R.apply_sam(enc, "sparsesam", ratio=0.0)
    with pytest.raises(ValueError):
        R.apply_sam(e2e_encoder(), "sparsesam", ratio=0.5, perm_mode="z_bad_sort")


def test_patched_forward_refuses_cpu():
    import torch
    enc = e2e_encoder()
    R.apply_sam(enc, "sparsesam", ratio=0.4)
    with pytest.raises(RuntimeError, match="CUDA"):
        enc(torch.zeros(1, 3, 256, 256))
    # the ratio list is restored even when the forward fails
    assert enc.tome_info["ratio"] == 0.4
