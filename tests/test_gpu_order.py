"""Z-order, Stripe-Sort permutation and keep set on the GPU vs the oracle: bit-exact."""
import numpy as np
import pytest
import torch

from oracle import order
from sparsesam_b200 import ops
from tests._golden import HILBERT_GRIDS, HILBERT_MODES, MODES, bf16_bits_to_f32, load

pytestmark = pytest.mark.gpu
GO = load("golden_order.npz")
GH = load("golden_hilbert.npz")


@pytest.mark.parametrize("H,W", [(4, 4), (14, 14), (64, 64), (16, 16), (7, 9), (1, 5)])
def test_zorder(cuda_device, H, W):
    p, inv = ops.zorder(H, W, cuda_device)
    op, oinv = order.zorder(H, W)
    np.testing.assert_array_equal(p.cpu().numpy(), op)
    np.testing.assert_array_equal(inv.cpu().numpy(), oinv)


def _gpu_perm(k_rows_f32: np.ndarray, win: int, mode: str, cuda_device, heads=1):
    """k_rows: (R, N, d) with R = n_seq*heads rows; laid out as a (n_seq*N, heads*d) buffer."""
    R, N, d = k_rows_f32.shape
    n_seq = R // heads
    buf = torch.from_numpy(k_rows_f32).view(n_seq, heads, N, d).permute(0, 2, 1, 3).reshape(n_seq * N, heads * d)
    buf = buf.to(cuda_device, torch.bfloat16).contiguous()
    space, layout, ranking = ops.parse_perm_mode(mode)
    base = (ops.zorder if space == "z" else ops.hilbert_order)(win, win, cuda_device)[0]
    p, ip, ipg = ops.stripe_sort_perm(buf, n_seq, heads, win, win, d, base, layout=layout, ranking=ranking)
    return p.cpu().numpy(), ip.cpu().numpy(), ipg.cpu().numpy()


@pytest.mark.parametrize("case,win", [("win", 14), ("winpad", 14), ("glob", 64)])
@pytest.mark.parametrize("mode", MODES)
def test_stripe_sort_golden_inputs(cuda_device, case, win, mode):
    k = bf16_bits_to_f32(GO[f"k_{case}"])
    p, ip, ipg = _gpu_perm(k, win, mode, cuda_device)
    op, oip, oipg = order.stripe_sort(k, win, win, perm_mode=mode)
    np.testing.assert_array_equal(p, op)
    np.testing.assert_array_equal(ip, oip)
    np.testing.assert_array_equal(ipg, oipg)


@pytest.mark.parametrize("H,W", list(HILBERT_GRIDS) + [(128, 128), (3, 1)])
def test_hilbert_order(cuda_device, H, W):
    p, inv = ops.hilbert_order(H, W, cuda_device)
    op, oinv = order.hilbert_order(H, W)
    np.testing.assert_array_equal(p.cpu().numpy(), op)
    np.testing.assert_array_equal(inv.cpu().numpy(), oinv)
    if (H, W) in HILBERT_GRIDS:  # the reference's own orders
        np.testing.assert_array_equal(p.cpu().numpy(), GH[f"horder_{H}x{W}"])


@pytest.mark.parametrize("case,win", [("win", 14), ("glob", 64)])
@pytest.mark.parametrize("mode", HILBERT_MODES)
def test_stripe_sort_hilbert_matches_reference(cuda_device, case, win, mode):
    """Hilbert base order: the GPU permutations equal the reference's own outputs."""
    k = bf16_bits_to_f32(GH[f"k_{case}"])
    p, ip, ipg = _gpu_perm(k, win, mode, cuda_device)
    np.testing.assert_array_equal(p, GH[f"{case}_{mode}_perm"].astype(np.int64))
    np.testing.assert_array_equal(ip, GH[f"{case}_{mode}_inv"].astype(np.int64))
    np.testing.assert_array_equal(ipg, GH[f"{case}_{mode}_invg"].astype(np.int64))


@pytest.mark.parametrize("heads,d", [(16, 80), (16, 64), (12, 64)])
def test_stripe_sort_global_multihead(cuda_device, heads, d):
    g = torch.Generator().manual_seed(heads * 100 + d)
    k = torch.randn(2 * heads, 4096, d, generator=g).to(torch.bfloat16).float().numpy()
    p, ip, ipg = _gpu_perm(k, 64, "z_interleave_sort", cuda_device, heads=heads)
    op, oip, oipg = order.stripe_sort(k, 64, 64)
    np.testing.assert_array_equal(p, op)
    np.testing.assert_array_equal(ipg, oipg)


def test_stripe_sort_padded_windows(cuda_device):
    # 64x64 grid -> 70x70 padded -> 25 windows; padded tokens carry the qkv bias
    g = torch.Generator().manual_seed(7)
    heads, d = 4, 80
    grid = torch.randn(1, 70, 70, heads * d, generator=g)
    bias = torch.randn(heads * d, generator=g) * 0.1
    grid[:, 64:, :, :] = bias
    grid[:, :, 64:, :] = bias
    win = grid.view(1, 5, 14, 5, 14, heads * d).permute(0, 1, 3, 2, 4, 5).reshape(25, 196, heads, d)
    rows = win.permute(0, 2, 1, 3).reshape(25 * heads, 196, d).to(torch.bfloat16).float().numpy()
    p, ip, ipg = _gpu_perm(rows, 14, "z_interleave_sort", cuda_device, heads=heads)
    op, oip, oipg = order.stripe_sort(rows, 14, 14)
    np.testing.assert_array_equal(p, op)
    np.testing.assert_array_equal(ipg, oipg)


@pytest.mark.parametrize("B,heads,N,keep_n", [(4, 16, 4096, 1229), (2, 12, 4096, 1638), (3, 2, 256, 102)])
def test_keep_select(cuda_device, B, heads, N, keep_n):
    g = torch.Generator().manual_seed(B + heads + keep_n)
    ipg = torch.stack([torch.randperm(N, generator=g) for _ in range(B * heads)]).to(torch.int32)
    if heads > 2:   # force exact ties of the head sums
        ipg[1] = ipg[0].flip(0)
    idx, rows = ops.keep_select(ipg.to(cuda_device), B, heads, keep_n)
    ref = order.keep_select(ipg.numpy(), B, heads, keep_n)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref)
    np.testing.assert_array_equal(rows.cpu().numpy(), (ref + np.arange(B)[:, None] * N).ravel())


def test_full_size_vit_h_properties(cuda_device):
    """ViT-H batch 64 global shapes: every row is a permutation, inverses agree,
    and sampled rows match the oracle bit-exactly."""
    n_seq, heads, d, win = 64, 16, 80, 64
    N = win * win
    g = torch.Generator(device=cuda_device).manual_seed(5)
    qkv_k = torch.randn(n_seq * N, heads * d, device=cuda_device, generator=g).to(torch.bfloat16)
    base = ops.zorder(win, win, cuda_device)[0]
    p, ip, ipg = ops.stripe_sort_perm(qkv_k, n_seq, heads, win, win, d, base)
    ar = torch.arange(N, device=cuda_device, dtype=torch.int32).expand(n_seq * heads, N)
    assert torch.equal(torch.sort(p, dim=1).values, ar)
    assert torch.equal(torch.gather(p, 1, ip.long()), ar)
    for r in (0, 517, n_seq * heads - 1):
        s, h = divmod(r, heads)
        rows = qkv_k[s * N:(s + 1) * N, h * d:(h + 1) * d].float().cpu().numpy()[None]
        op, _, oipg = order.stripe_sort(rows, win, win)
        np.testing.assert_array_equal(p[r].cpu().numpy(), op[0])
        np.testing.assert_array_equal(ipg[r].cpu().numpy(), oipg[0])
    keep_n = order.keep_n_for(0.3, N)
    idx, _ = ops.keep_select(ipg, n_seq, heads, keep_n)
    assert idx.shape == (n_seq, keep_n)
    srt = torch.sort(idx, dim=1).values
    assert bool((srt[:, 1:] > srt[:, :-1]).all())
    assert ops.device_error() == 0
