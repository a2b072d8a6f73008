"""Row kernels (LayerNorm gathers, window maps, RC-MLP, stem/neck helpers) vs torch fp32."""
import pytest
import torch
import torch.nn.functional as F

from sparsesam_b200 import _lib, host, ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("C", [128, 768, 1024, 1280, 256])
def test_layernorm_gather(cuda_device, C):
    x = torch.randn(300, C, device=cuda_device) * 3 + 1
    w = torch.randn(C, device=cuda_device)
    b = torch.randn(C, device=cuda_device)
    src = torch.randint(-1, 300, (517,), device=cuda_device, dtype=torch.int32)
    out = ops.layernorm_gather(x, w, b, 1e-6, src_rows=src)
    ref = F.layer_norm(x[src.clamp(min=0).long()], (C,), w, b, 1e-6)
    ref[src < 0] = 0
    assert (out.float() - ref).abs().max().item() <= 2e-2 * ref.abs().max().item()
    assert torch.all(out[src < 0] == 0)


def test_window_rows_match_partition(cuda_device):
    B, H, W, ws, C = 2, 64, 64, 14, 4
    x = torch.randn(B, H, W, C, device=cuda_device)
    win, _ = host.window_partition(x, ws)
    rows = ops.window_rows(B, H, W, ws, cuda_device)
    flat = x.reshape(-1, C)
    got = torch.where((rows >= 0)[:, None], flat[rows.clamp(min=0).long()], torch.zeros((), device=cuda_device))
    assert torch.equal(got, win.reshape(-1, C))


@pytest.mark.parametrize("keep", [True, False])
def test_rc_mlp(cuda_device, keep):
    torch.manual_seed(0)
    n_tok, C, Hd = 2 * 4096, 256, 1024
    x = torch.randn(n_tok, C, device=cuda_device)
    ln_w, ln_b = torch.rand(C, device=cuda_device) + 0.5, torch.randn(C, device=cuda_device) * 0.1
    w1 = (torch.randn(Hd, C, device=cuda_device) * 0.05).to(torch.bfloat16)
    b1 = torch.randn(Hd, device=cuda_device) * 0.1
    w2 = (torch.randn(C, Hd, device=cuda_device) * 0.05).to(torch.bfloat16)
    b2 = torch.randn(C, device=cuda_device) * 0.1
    rows = torch.randperm(n_tok, device=cuda_device)[:2458].to(torch.int32) if keep else None
    x0 = x.clone()
    ref = x.clone()
    sel = rows.long() if keep else torch.arange(n_tok, device=cuda_device)
    xs = ref[sel]
    h = F.gelu(F.layer_norm(xs, (C,), ln_w, ln_b, 1e-6).to(torch.bfloat16).float() @ w1.float().T + b1)
    ref[sel] = xs + h.to(torch.bfloat16).float() @ w2.float().T + b2
    ops.rc_mlp(x, rows, sel.numel(), ln_w, ln_b, 1e-6, w1, b1, w2, b2)
    err = (x - ref).abs().max().item()
    assert err < 3e-2, err
    if keep:   # rows outside the keep set pass through unchanged, bit for bit (sam.py:284-288)
        skipped = torch.ones(n_tok, dtype=torch.bool, device=cuda_device)
        skipped[sel] = False
        assert int(skipped.sum()) == n_tok - 2458
        assert torch.equal(x[skipped], x0[skipped])


def test_patch_embed_im2col(cuda_device):
    img = torch.randn(2, 3, 64, 64, device=cuda_device)
    conv = torch.nn.Conv2d(3, 96, 16, 16).to(cuda_device)
    cols = ops.patch_im2col(img, 16)
    w = conv.weight.detach().reshape(96, -1).to(torch.bfloat16)
    out = ops.gemm_bf16(cols, w, conv.bias.detach().float().contiguous(), epilogue=ops.SSAM_EPI_F32)
    ref = conv(img).permute(0, 2, 3, 1).reshape(-1, 96)
    assert (out - ref).abs().max().item() < 3e-2


def test_neck_pieces(cuda_device):
    B, H, W, C = 2, 16, 16, 64
    x = torch.randn(B, H, W, C, device=cuda_device).to(torch.bfloat16)
    conv = torch.nn.Conv2d(C, 32, 3, padding=1, bias=False).to(cuda_device)
    cols = ops.im2col3x3_nhwc(x)
    w = conv.weight.detach().permute(0, 2, 3, 1).reshape(32, -1).to(torch.bfloat16)
    out = ops.gemm_bf16(cols, w, None, epilogue=ops.SSAM_EPI_F32)
    ref = conv(x.float().permute(0, 3, 1, 2)).permute(0, 2, 3, 1).reshape(-1, 32)
    assert (out - ref).abs().max().item() < 3e-2
    y = torch.randn(B * H * W, 32, device=cuda_device)
    lw, lb = torch.randn(32, device=cuda_device), torch.randn(32, device=cuda_device)
    ln = ops.layernorm_rows(y, lw, lb, 1e-6, out_bf16=False)
    assert (ln - F.layer_norm(y, (32,), lw, lb, 1e-6)).abs().max().item() < 1e-4
    t = ops.nhwc_to_nchw(y, B, H, W, 32)
    assert torch.equal(t, y.view(B, H, W, 32).permute(0, 3, 1, 2))
    pos = torch.randn(H * W, 32, device=cuda_device)
    xb = torch.empty(B * H * W, 32, device=cuda_device)
    ops.broadcast_rows(pos, B, xb)
    assert torch.equal(xb.view(B, H * W, 32), pos.expand(B, -1, -1))


@pytest.mark.parametrize("B,H,W,C", [(2, 64, 64, 256), (3, 7, 9, 32), (1, 5, 13, 256)])
def test_neck_layernorms_fused(cuda_device, B, H, W, C):
    """The neck's LayerNorm2d outputs: the 3-term split mode equals split_bf16x3 of
    the fp32 LayerNorm, and the NCHW mode equals the fp32 LayerNorm transposed, both
    bit for bit (one reduction order); pixel counts that are not multiples of 32
    exercise the last partial tile."""
    g = torch.Generator().manual_seed(3)
    y = (torch.randn(B * H * W, C, generator=g) * 2 + 0.5).to(cuda_device)
    lw = torch.randn(C, generator=g).to(cuda_device)
    lb = torch.randn(C, generator=g).to(cuda_device)
    ln = ops.layernorm_rows(y, lw, lb, 1e-6, out_bf16=False)
    assert torch.equal(ops.layernorm_rows(y, lw, lb, 1e-6, out_bf16=False, split3=True), ops.split_bf16x3(ln))
    assert torch.equal(ops.layernorm_nchw(y, B, H, W, lw, lb, 1e-6), ln.view(B, H, W, C).permute(0, 3, 1, 2))
    assert ops.device_error() == 0


def test_split_bf16x3_parts(cuda_device):
    x = torch.randn(37, 96, device=cuda_device) * 3
    out = ops.split_bf16x3(x).float()
    hi, lo, hi2 = out[:, :96], out[:, 96:192], out[:, 192:]
    assert torch.equal(hi, x.to(torch.bfloat16).float())
    assert torch.equal(hi2, hi)
    assert torch.equal(lo, (x - hi).to(torch.bfloat16).float())
    assert (hi + lo - x).abs().max().item() <= 2.0 ** -16 * x.abs().max().item()


def test_patch_embed_split3_matches_fp32_conv(cuda_device):
    """[hi | lo | hi] patches x [W_hi | W_hi | W_lo]: the stem GEMM at fp32 accuracy."""
    img = torch.randn(2, 3, 64, 64, device=cuda_device)
    conv = torch.nn.Conv2d(3, 96, 16, 16).to(cuda_device)
    cols = ops.patch_im2col_split3(img, 16)
    assert cols.shape == (2 * 16, 3 * 768)
    single = ops.patch_im2col(img, 16)
    assert torch.equal(cols[:, :768], single) and torch.equal(cols[:, 1536:], single)
    w3 = ops.split_weight3(conv.weight.detach().reshape(96, -1))
    out = ops.gemm_bf16(cols, w3, conv.bias.detach().float().contiguous(), epilogue=ops.SSAM_EPI_F32)
    with torch.backends.cudnn.flags(allow_tf32=False):
        ref = conv(img).permute(0, 2, 3, 1).reshape(-1, 96)
    assert (out - ref).abs().max().item() < 2e-4


def test_split3_gemm_matches_fp32_linear(cuda_device):
    x = torch.randn(300, 256, device=cuda_device)
    w = torch.randn(128, 256, device=cuda_device) * 0.05
    out = ops.gemm_bf16(ops.split_bf16x3(x), ops.split_weight3(w), None, epilogue=ops.SSAM_EPI_F32)
    ref = (x.double() @ w.double().T).float()
    assert (out - ref).abs().max().item() < 1e-4


def test_window_of_raster_inverts_window_rows(cuda_device):
    B, H, W, ws = 2, 64, 64, 14
    rows = ops.window_rows(B, H, W, ws, cuda_device).cpu()
    inv = ops.window_of_raster(B, H, W, ws, cuda_device).cpu()
    assert inv.numel() == B * H * W
    real = (rows >= 0).nonzero().flatten()
    assert torch.equal(inv[rows[real].long()], real.to(torch.int32))
    assert torch.equal(torch.sort(inv.long()).values, real)


@pytest.mark.parametrize("B,H,W,ws,C", [(1, 20, 20, 14, 96), (2, 64, 64, 14, 3840), (3, 9, 13, 7, 264)])
def test_fill_pad_rows_writes_bias_only_on_padding(cuda_device, B, H, W, ws, C):
    rows = ops.window_rows(B, H, W, ws, cuda_device)
    out = torch.randn(rows.numel(), C, device=cuda_device).to(torch.bfloat16)
    before = out.clone()
    bias = torch.randn(C, device=cuda_device)
    ops.fill_pad_rows(out, rows, bias)
    pad = rows < 0
    assert torch.equal(out[~pad], before[~pad])
    assert torch.equal(out[pad], bias.to(torch.bfloat16).expand(int(pad.sum()), C))


def test_gemm_bf16_scatters_rows(cuda_device):
    M, N, K = 300, 128, 64
    a = torch.randn(M, K, device=cuda_device).to(torch.bfloat16)
    b = torch.randn(N, K, device=cuda_device).to(torch.bfloat16)
    dst = torch.randperm(2 * M, device=cuda_device)[:M].to(torch.int32)
    dst[::7] = -1
    out = torch.zeros(2 * M, N, device=cuda_device, dtype=torch.bfloat16)
    ops.gemm_bf16(a, b, out=out, out_rows=dst)
    ref = (a.float() @ b.float().T).to(torch.bfloat16)
    keep = dst >= 0
    assert torch.allclose(out[dst[keep].long()].float(), ref[keep].float(), atol=6e-2, rtol=2e-2)
    written = torch.zeros(2 * M, dtype=torch.bool, device=cuda_device)
    written[dst[keep].long()] = True
    assert (out[~written] == 0).all()


@pytest.mark.parametrize("rows,C", [(1000, 1280), (37, 768), (5, 96)])
def test_layernorm_rows_copy_out(cuda_device, rows, C):
    """norm1 with the snapshot: the bf16 output equals the plain LayerNorm's and the
    copy holds the input rows bit for bit."""
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(rows, C, generator=g) * 3 + 1).to(cuda_device)
    w = torch.randn(C, generator=g).to(cuda_device)
    b = torch.randn(C, generator=g).to(cuda_device)
    ref = ops.layernorm_rows(x, w, b, 1e-6, out_bf16=True)
    snap = torch.full_like(x, float("nan"))
    out = ops.layernorm_rows(x, w, b, 1e-6, out_bf16=True, copy_out=snap)
    assert torch.equal(out, ref)
    assert torch.equal(snap, x)


@pytest.mark.parametrize("B,H,W,Cin,Cout", [(2, 64, 64, 768, 256), (1, 8, 32, 128, 64), (3, 16, 16, 64, 32)])
def test_conv3x3_implicit_matches_im2col(cuda_device, B, H, W, Cin, Cout):
    """The implicit-GEMM 3x3 convolution (4-D TMA boxes of the channels-last input,
    zeros outside the image) equals im2col + GEMM bit for bit, and the fp32
    convolution to bf16-operand accuracy; unsupported shapes are refused."""
    g = torch.Generator().manual_seed(9)
    x = torch.randn(B * H * W, Cin, generator=g).to(torch.bfloat16).to(cuda_device)
    w = (torch.randn(Cout, 9 * Cin, generator=g) * 0.05).to(torch.bfloat16).to(cuda_device)
    b = torch.randn(Cout, generator=g).to(cuda_device)
    assert ops.conv3x3_supported(H, W, Cin, Cout)
    got = ops.conv3x3_nhwc(x, B, H, W, w, b)
    ref = ops.gemm_bf16(ops.im2col3x3_nhwc(x.view(B, H, W, Cin)), w, b, epilogue=ops.SSAM_EPI_F32)
    assert ops.device_error() == 0
    assert torch.equal(got, ref)
    conv = torch.nn.functional.conv2d(x.float().view(B, H, W, Cin).permute(0, 3, 1, 2),
                                      w.float().view(Cout, 3, 3, Cin).permute(0, 3, 1, 2), b, padding=1)
    conv = conv.permute(0, 2, 3, 1).reshape(-1, Cout)
    assert (got - conv).abs().max().item() <= 1e-3 * conv.abs().max().item() + 1e-3


def test_conv3x3_implicit_refuses_unsupported(cuda_device):
    x = torch.zeros(1 * 9 * 9, 64, dtype=torch.bfloat16, device=cuda_device)
    w = torch.zeros(32, 9 * 64, dtype=torch.bfloat16, device=cuda_device)
    assert not ops.conv3x3_supported(9, 9, 64, 32)
    with pytest.raises(RuntimeError):
        ops.conv3x3_nhwc(x, 1, 9, 9, w)


@pytest.mark.parametrize("B,T,K,N", [(2, 4096, 2304, 1280), (16, 1024, 192, 512)])   # both GEMMs on the 2-SM kernel
def test_gemm_addend_is_broadcast_then_add(cuda_device, B, T, K, N):
    """The stem's GEMM with the positional embedding added in its epilogue equals
    the broadcast of the embedding followed by the accumulating GEMM, bit for bit
    (fp32 addition commutes)."""
    g = torch.Generator().manual_seed(13)
    a = torch.randn(B * T, K, generator=g).to(torch.bfloat16).to(cuda_device)
    w = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16).to(cuda_device)
    bias = torch.randn(N, generator=g).to(cuda_device)
    pos = torch.randn(T, N, generator=g).to(cuda_device)
    got = ops.gemm_bf16_addend(a, w, bias, pos)
    ref = torch.empty(B * T, N, device=cuda_device)
    ops.broadcast_rows(pos, B, ref)
    ops.gemm_bf16(a, w, bias, epilogue=ops.SSAM_EPI_ADD_F32, out=ref)
    assert ops.device_error() == 0
    assert torch.equal(got, ref)


@pytest.mark.parametrize("C", [32, 64, 128, 256])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("gelu", [False, True])
def test_layernorm_gelu_half_rows(cuda_device, C, dtype, gelu):
    """ssam_layernorm_gelu_half (the SAM-HQ decoder's LayerNorm2d -> GELU on
    channels-last maps) against torch fp32 LayerNorm (+ exact GELU) of the same
    half-precision inputs; rows not a multiple of a CTA's row group (the tail)."""
    g = torch.Generator().manual_seed(C)
    rows = 3 * 1184 * (256 // (C // 8)) + 37        # more row groups than the grid's CTAs, plus a tail
    x = (torch.randn(rows, C, generator=g) * 3 + 1.5).to(dtype).to(cuda_device)
    w = (torch.rand(C, generator=g) + 0.5).to(dtype).to(cuda_device)
    b = (torch.randn(C, generator=g) * 0.1).to(dtype).to(cuda_device)
    y = ops.layernorm_gelu_half(x, w, b, 1e-6, gelu)
    ref = torch.nn.functional.layer_norm(x.float(), (C,), w.float(), b.float(), 1e-6)
    if gelu:
        ref = torch.nn.functional.gelu(ref)
    # the output's own rounding (fp16: 2^-11, bf16: 2^-8 of the value) plus fp32 arithmetic
    rel = 2.0 ** -11 if dtype == torch.float16 else 2.0 ** -8
    err = (y.float() - ref).abs()
    assert (err <= rel * ref.abs() + 2e-4).all(), err.max().item()
    assert y.dtype == dtype and y.shape == x.shape


def test_layernorm_gelu_half_refuses(cuda_device):
    x = torch.zeros(10, 48, dtype=torch.float16, device=cuda_device)
    w = torch.ones(48, dtype=torch.float16, device=cuda_device)
    with pytest.raises(_lib.SparseSAMError):
        ops.layernorm_gelu_half(x, w, w.clone(), 1e-6, True)          # C = 48: unsupported
    x = torch.zeros(10, 64, dtype=torch.float16, device=cuda_device)
    w = torch.ones(64, dtype=torch.float16, device=cuda_device)
    with pytest.raises(ValueError):
        ops.layernorm_gelu_half(x, w.bfloat16(), w.bfloat16(), 1e-6, True)   # mixed dtypes
    assert ops.layernorm_gelu_half(x[:0], w, w.clone(), 1e-6, False).numel() == 0
