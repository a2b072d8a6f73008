"""The bf16 arithmetic itself, emulated in the fp32 oracle, stays inside the
tolerances the GPU encoder tests apply (output embeddings max-abs 2e-2,
intermediate embeddings 0.5 % of their range): the bounds are achievable by a
correct bf16 implementation, and the intermediate bound is not looser than
what the format needs on the golden configuration."""
from oracle.bf16_emulation import emulated_errors
from sparsesam_b200 import host
from tests._golden import E2E_RATIO, e2e_encoder


def test_bf16_operand_emulation_within_tolerances():
    img = host.synthetic_images(2, seed=0, img_size=256)
    feat_err, interm_err, interm_scale = emulated_errors(e2e_encoder(), img, E2E_RATIO)
    assert feat_err <= 2e-2
    for e, sc in zip(interm_err, interm_scale):
        assert e <= 5e-3 * sc
        assert e > 0.0  # the emulation does round
