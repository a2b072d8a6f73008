"""Failure detection on the GPU without a fault.

Every wait in this library's kernels is bounded: when it runs out, the kernel
raises SSAM_ERR_TIMEOUT on a device flag, unwinds and returns, and the host
reads the flag through ssam_device_error(). Here a diagnostic kernel waits on a
barrier that nothing completes (no trap, no bad address, no endless loop): the
status must come back after about two seconds and the context must keep
running kernels correctly.
"""
import time

import pytest
import torch

from sparsesam_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def test_wait_timeout_reported_and_context_usable(cuda_device):
    lib = _lib.load()
    torch.cuda.synchronize()
    assert lib.ssam_device_error(1) == _lib.SSAM_OK
    t0 = time.monotonic()
    assert lib.ssam_check_wait_timeout(None) == _lib.SSAM_OK
    assert lib.ssam_device_error(1) == _lib.SSAM_ERR_TIMEOUT
    waited = time.monotonic() - t0
    assert 1.0 < waited < 30.0
    assert lib.ssam_device_error(0) == _lib.SSAM_OK  # cleared by the read above
    # the context keeps working: a GEMM afterwards is correct and raises nothing
    g = torch.Generator().manual_seed(0)
    a = torch.randn(512, 256, generator=g).to(torch.bfloat16).to(cuda_device)
    b = torch.randn(384, 256, generator=g).to(torch.bfloat16).to(cuda_device)
    out = ops.gemm_bf16(a, b, None, epilogue=ops.SSAM_EPI_F32)
    ref = a.float() @ b.float().t()
    assert (out - ref).abs().max().item() <= 1e-3 * ref.abs().max().item()
    assert ops.device_error() == _lib.SSAM_OK
