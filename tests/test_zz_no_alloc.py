"""ssam_rc_mlp_fwd_noalloc: the Residual-Consistency MLP for callers that cannot
allocate device memory at call time (a fixed, pre-reserved device memory budget,
or a foreign-language binding without a device allocator).

Called through the C ABI and compared with ssam_rc_mlp_fwd (caller workspace) on
two calls in a row, which also exercises the reuse of the library's shared
scratch array. Collected last so that a run stopping at the first failure has
already run every other test.
"""
import ctypes

import pytest
import torch

from sparsesam_b200 import _lib

pytestmark = pytest.mark.gpu

TOL = 3e-2  # the RC-MLP tolerance of tests/test_gpu_rows.py


def _inputs(seed, device, n_tok=4096, C=256, Hd=1024, n_rows=1500):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(n_tok, C, generator=g).to(device)
    rows = torch.randperm(n_tok, generator=g)[:n_rows].to(torch.int32).to(device)
    ln_w = (torch.rand(C, generator=g) + 0.5).to(device)
    ln_b = (torch.randn(C, generator=g) * 0.1).to(device)
    w1 = (torch.randn(Hd, C, generator=g) * 0.05).to(torch.bfloat16).to(device)
    b1 = (torch.randn(Hd, generator=g) * 0.1).to(device)
    w2 = (torch.randn(C, Hd, generator=g) * 0.05).to(torch.bfloat16).to(device)
    b2 = (torch.randn(C, generator=g) * 0.1).to(device)
    return x, rows, ln_w, ln_b, w1, b1, w2, b2


def _with_workspace(lib, x, rows, ln_w, ln_b, w1, b1, w2, b2, stream):
    C, Hd = x.shape[1], w1.shape[0]
    n = rows.numel()
    ws_bytes = lib.ssam_rc_mlp_workspace_size(n, C, Hd)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    st = lib.ssam_rc_mlp_fwd(x.data_ptr(), C, rows.data_ptr(), n, C, Hd, ln_w.data_ptr(), ln_b.data_ptr(), 1e-6,
                             w1.data_ptr(), b1.data_ptr(), w2.data_ptr(), b2.data_ptr(), ws.data_ptr(), ws_bytes,
                             stream)
    assert st == 0


def _no_alloc(lib, x, rows, ln_w, ln_b, w1, b1, w2, b2, stream):
    C, Hd = x.shape[1], w1.shape[0]
    st = lib.ssam_rc_mlp_fwd_noalloc(x.data_ptr(), C, rows.data_ptr(), rows.numel(), C, Hd, ln_w.data_ptr(),
                                     ln_b.data_ptr(), 1e-6, w1.data_ptr(), b1.data_ptr(), w2.data_ptr(),
                                     b2.data_ptr(), stream)
    assert st == 0


def test_no_alloc_matches_workspace_entry_two_calls(cuda_device):
    lib = _lib.load()
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    for call, seed in enumerate((11, 12)):
        x, *rest = _inputs(seed, cuda_device, n_rows=1500 if call == 0 else 900)
        ref = x.clone()
        out = x.clone()
        _with_workspace(lib, ref, *rest, stream)
        _no_alloc(lib, out, *rest, stream)
        torch.cuda.synchronize()
        err = (out - ref).abs().max().item()
        assert err <= TOL, f"call {call}: max-abs {err}"
        assert torch.equal(out, ref)  # same kernels on the same inputs
        # rows outside the keep set are untouched
        mask = torch.ones(x.shape[0], dtype=torch.bool, device=cuda_device)
        mask[rest[0].long()] = False
        assert torch.equal(out[mask], x[mask])
    assert lib.ssam_device_error(1) == 0


def test_no_alloc_allocates_nothing(cuda_device):
    """After a first call (which resolves the scratch address), further calls leave
    the device's free memory and torch's allocator exactly as they were."""
    lib = _lib.load()
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    x, *rest = _inputs(13, cuda_device)
    _no_alloc(lib, x, *rest, stream)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(cuda_device)
    reserved0 = torch.cuda.memory_reserved(cuda_device)
    for _ in range(3):
        _no_alloc(lib, x, *rest, stream)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(cuda_device)
    assert free1 == free0
    assert torch.cuda.memory_reserved(cuda_device) == reserved0
    assert lib.ssam_device_error(1) == 0


def test_no_alloc_rejects_a_stream_of_another_device(cuda_device):
    """The scratch address belongs to the current device; a stream created on
    another device is refused before anything is enqueued."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two devices")
    lib = _lib.load()
    other = torch.cuda.Stream(device=1)
    x, *rest = _inputs(14, cuda_device, n_rows=64)
    with torch.cuda.device(cuda_device):
        C, Hd = x.shape[1], rest[3].shape[0]
        st = lib.ssam_rc_mlp_fwd_noalloc(x.data_ptr(), C, rest[0].data_ptr(), 64, C, Hd, rest[1].data_ptr(),
                                         rest[2].data_ptr(), 1e-6, rest[3].data_ptr(), rest[4].data_ptr(),
                                         rest[5].data_ptr(), rest[6].data_ptr(), other.cuda_stream)
    assert st == _lib.SSAM_ERR_INVALID


def test_no_alloc_rejects_oversized_calls(cuda_device):
    lib = _lib.load()
    # 4096 rows x (1280 + 5120) x 2 B = 50 MiB > the 32 MiB scratch
    st = lib.ssam_rc_mlp_fwd_noalloc(ctypes.c_void_p(16), 1280, None, 4096, 1280, 5120, ctypes.c_void_p(16),
                                     ctypes.c_void_p(16), 1e-6, ctypes.c_void_p(16), None, ctypes.c_void_p(16),
                                     None, None)
    assert st == _lib.SSAM_ERR_UNSUPPORTED
