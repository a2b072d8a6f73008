"""The C-ABI shared library: loads, exports every declared symbol, validates
arguments on the host (no kernel launches; runs without a GPU)."""
import ctypes
import os
import re

import pytest

from sparsesam_b200 import _lib
from oracle import order

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "sparsesam.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(ssam_[a-z0-9_]+)\s*\(", text)))


def test_header_and_binding_agree():
    assert declared_symbols() == sorted(_lib.SIGNATURES)


def test_library_exports_every_symbol():
    lib = _lib.load()
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert missing == []
    assert _lib.missing_symbols() == []


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.ssam_version() >= 100
    for code in range(6):
        assert lib.ssam_status_string(code)


@pytest.mark.parametrize("N,ratio,is_global", [(196, 0.3, 0), (196, 0.5, 0), (4096, 0.3, 1), (4096, 0.4, 1),
                                                (4096, 0.5, 1), (256, 0.4, 1), (196, 1.0, 0), (4096, 0.01, 1)])
def test_a_shape_n_init_host(N, ratio, is_global):
    lib = _lib.load()
    assert lib.ssam_a_shape_n_init(N, 64, ratio, is_global) == order.a_shape_n_init(N, 64, ratio, bool(is_global))
    assert lib.ssam_a_shape_n_init(N, 64, 0.0, is_global) == -1


def test_a_shape_mask_host():
    import numpy as np
    lib = _lib.load()
    for N, n_init, diag in ((4096, 19, 1), (196, 2, 0), (256, 1, 1)):
        nm = -(-N // 64)
        buf = (ctypes.c_uint8 * (nm * nm))()
        assert lib.ssam_a_shape_mask(N, 64, 64, n_init, diag, buf) == 0
        got = np.frombuffer(buf, dtype=np.uint8).reshape(nm, nm)
        np.testing.assert_array_equal(got, order.a_shape_mask(N, 64, 64, n_init, bool(diag)))


def test_invalid_arguments_rejected_on_host():
    lib = _lib.load()
    nul = None
    # null pointers / bad shapes never reach the GPU
    assert lib.ssam_gemm_bf16(nul, 64, nul, 64, 128, 256, 64, nul, 0, nul, 256, nul, nul) == _lib.SSAM_ERR_INVALID
    assert lib.ssam_sparse_attn_fwd(1, 240, 1, 1, 14, 48, 16, 16, 16, 2, 64, 0, 1.0, 16, 48, nul, 0, 0, nul, nul, 0, nul) == \
        _lib.SSAM_ERR_UNSUPPORTED
    # global grids need the bias workspace; a query row without any key block is rejected
    assert lib.ssam_sparse_attn_fwd(16, 240, 1, 1, 64, 80, 16, 16, 16, 2, 64, 1, 1.0, 16, 80, nul, 0, 0, nul, nul, 0, nul) == \
        _lib.SSAM_ERR_INVALID
    assert lib.ssam_sparse_attn_fwd(16, 240, 1, 1, 14, 80, 16, 16, 16, 0, 64, 0, 1.0, 16, 80, nul, 0, 0, nul, nul, 0, nul) == \
        _lib.SSAM_ERR_INVALID
    # mask blocks other than 64 / 128 tokens are not implemented
    assert lib.ssam_sparse_attn_fwd(16, 240, 1, 1, 14, 80, 16, 16, 16, 2, 32, 0, 1.0, 16, 80, nul, 0, 0, nul, nul, 0, nul) == \
        _lib.SSAM_ERR_UNSUPPORTED
    assert lib.ssam_stripe_sort_perm(16, 64, 1, 1, 3, 3, 64, 4, 0, 0, 16, 16, 16, 16, nul) == _lib.SSAM_ERR_INVALID
    assert lib.ssam_keep_select(16, 1, 1, 16, 17, 16, nul, nul) == _lib.SSAM_ERR_INVALID
    assert lib.ssam_layernorm_rows_copy(16, 4, 64, 16, 16, 1e-6, 16, nul, nul) == _lib.SSAM_ERR_INVALID
    assert lib.ssam_layernorm_rows_copy(16, 4, 64, 16, 16, 1e-6, 16, 24, nul) == _lib.SSAM_ERR_ALIGN
    assert lib.ssam_stripe_sort_perm(16, 64, 1, 1, 4, 4, 64, 4, 7, 0, 16, 16, 16, 16, nul) == _lib.SSAM_ERR_INVALID


def test_sparse_attn_workspace_size():
    lib = _lib.load()
    assert lib.ssam_sparse_attn_workspace_size(4, 12, 14, 64) == 0          # windowed: bias in-kernel
    # global 64x64 grid: 32 query tiles x 128 rows x 128 fp16 per (image, head)
    assert lib.ssam_sparse_attn_workspace_size(2, 16, 64, 80) == 2 * 16 * 32 * 128 * 128 * 2
    assert lib.ssam_sparse_attn_workspace_size(1, 1, 17, 64) == 3 * 128 * 128 * 2
    assert lib.ssam_sparse_attn_workspace_size(0, 16, 64, 80) == 0


def test_rc_mlp_workspace_size():
    lib = _lib.load()
    n, C, Hd = 1229, 1280, 5120
    sz = lib.ssam_rc_mlp_workspace_size(n, C, Hd)
    assert sz >= n * (C + Hd) * 2 and sz % 256 == 0
    assert lib.ssam_rc_mlp_workspace_size(0, C, Hd) == 0
