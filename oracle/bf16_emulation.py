"""bf16 operand emulation of the fp32 oracle encoder — TEST INFRASTRUCTURE.

Runs oracle.encoder.encoder_forward with every nn.Linear operand (input
activations and weights) rounded to bf16 and products accumulated in fp32, the
arithmetic the B200 GEMMs perform. The difference to the plain fp32 run is the
error a bf16 encoder carries before any kernel-specific approximation; the
tests use it to size the tolerance of the intermediate embeddings (residual
stream values) against the fp32 reference (algos/sparsesam/sam.py:242-290 path
restated in oracle/encoder.py).

Only tests/ import this module.
"""
from __future__ import annotations

import contextlib

import torch

from . import encoder as oenc


def _bf(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).float()


@contextlib.contextmanager
def bf16_gemm_operands():
    """Within the block, oracle linears round their inputs and weights to bf16."""
    orig = oenc.F.linear

    def linear(x, w, b=None):
        return orig(_bf(x), _bf(w), b)

    oenc.F.linear = linear
    try:
        yield
    finally:
        oenc.F.linear = orig


def emulated_errors(enc, img, ratio: float):
    """(features max-abs, [interm max-abs], [interm max |ref|]) of the bf16-operand
    run against the fp32 run, on the fp32 run's permutations."""
    ref, ri, st = oenc.encoder_forward(enc, img, ratio, return_state=True)
    forced = {k: v for k, v in st["perm_cache"].items() if isinstance(k[0], int)}
    with bf16_gemm_operands():
        out, oi = oenc.encoder_forward(enc, img, ratio, forced_perms=forced)
    return ((out - ref).abs().max().item(), [(a - b).abs().max().item() for a, b in zip(oi, ri)],
            [b.abs().max().item() for b in ri])
