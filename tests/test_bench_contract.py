"""bench.py's FLOP convention and argument rules, on the CPU.

`tc_peak_frac` divides the encoder's algorithmic FLOPs by the measured peak,
so the per-image figure is pinned here: the valid-token convention (qkv / proj
on the real tokens, windowed attention over valid queries x enabled keys, global
attention over enabled 64x64 block pairs, the MLP on the keep set in the sparse
blocks, patch embedding and neck), which reproduces the per-image TFLOP of the
hot-path survey for every BASELINE architecture and density.
"""
import pytest

import bench


@pytest.mark.parametrize("arch,ratio,tflop", [
    ("vit_h", 0.3, 3.772), ("vit_h", 0.4, 4.029), ("vit_h", 1.0, 5.628),
    ("vit_l", 0.3, 1.893), ("vit_l", 1.0, 2.828),
    ("vit_b", 0.4, 0.663), ("vit_b", 1.0, 0.933),
])
def test_encoder_flops_per_image(arch, ratio, tflop):
    assert abs(bench.encoder_flops(arch, ratio) / 1e12 - tflop) <= 5e-4 * tflop


def test_sparse_mlp_only_after_the_first_global_block():
    # without the keep set every block runs the dense MLP: more FLOPs
    assert bench.encoder_flops("vit_h", 0.3, mlp_merge=False) > bench.encoder_flops("vit_h", 0.3)
    # density 1.0 enables every block pair and every key: the dense control
    assert bench.encoder_flops("vit_h", 1.0, mlp_merge=False) == bench.encoder_flops("vit_h", 1.0)


def test_warmup_is_at_least_three(monkeypatch):
    seen = {}
    monkeypatch.setattr(bench, "run_ours", lambda args: seen.setdefault("warmup", args.warmup))
    monkeypatch.setattr("sys.argv", ["bench.py", "--warmup", "1", "--steps", "2"])
    bench.main()
    assert seen["warmup"] == 3
