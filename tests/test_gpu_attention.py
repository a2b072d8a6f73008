"""Block-sparse rel-pos attention on the tensor cores vs the fp32 oracle.

Tolerance: bf16 operands, P rounded to bf16 before P.V and a bf16 output give a
max-abs error well below 3e-2 on O(1) outputs (the reference's own fp16 check
uses atol 1e-2, flash_attn.py:1553); the mean error must stay below 3e-3.
"""
import pytest
import torch

from oracle import order
from oracle.attention import sparse_attention
from sparsesam_b200 import ops

pytestmark = pytest.mark.gpu


def _case(cuda_device, n_seq, heads, win, d, ratio, is_global, table_std=0.3, seed=0):
    g = torch.Generator().manual_seed(seed)
    N, C = win * win, heads * d
    qkv = torch.randn(n_seq * N, 3 * C, generator=g).to(torch.bfloat16)
    th = (torch.randn(2 * win - 1, d, generator=g) * table_std).to(torch.bfloat16)
    tw = (torch.randn(2 * win - 1, d, generator=g) * table_std).to(torch.bfloat16)
    perm = torch.stack([torch.randperm(N, generator=g) for _ in range(n_seq * heads)]).to(torch.int32)
    n_init = order.a_shape_n_init(N, 64, ratio, is_global)
    scale = d ** -0.5
    out = ops.sparse_attn(qkv.to(cuda_device), n_seq, heads, win, d, th.to(cuda_device), tw.to(cuda_device),
                          perm.to(cuda_device), n_init, is_global, scale)
    # oracle on the same bf16 values, rows = (seq, head)
    q, k, v = qkv.float().view(n_seq, N, 3, heads, d).permute(2, 0, 3, 1, 4).reshape(3, n_seq * heads, N, d)
    ref = sparse_attention(q, k, v, th.float(), tw.float(), perm, win, n_init, is_global, scale,
                           round_tables_fp16=False)
    ref = ref.view(n_seq, heads, N, d).permute(0, 2, 1, 3).reshape(n_seq * N, C)
    err = (out.float().cpu() - ref).abs()
    return err, ref


@pytest.mark.parametrize("d", [64, 80])
@pytest.mark.parametrize("ratio", [0.2, 0.3, 0.5, 0.75, 1.0])
def test_window_attention(cuda_device, d, ratio):
    err, ref = _case(cuda_device, n_seq=6, heads=2, win=14, d=d, ratio=ratio, is_global=False)
    assert err.max().item() < 3e-2, err.max().item()
    assert err.mean().item() < 3e-3


@pytest.mark.parametrize("d", [64, 80])
@pytest.mark.parametrize("ratio", [0.01, 0.3, 0.4, 0.5, 1.0])
def test_global_attention(cuda_device, d, ratio):
    err, ref = _case(cuda_device, n_seq=1, heads=2, win=64, d=d, ratio=ratio, is_global=True)
    assert err.max().item() < 3e-2, err.max().item()
    assert err.mean().item() < 3e-3


@pytest.mark.parametrize("win,is_global", [(16, True), (16, False), (8, True)])
def test_small_grids(cuda_device, win, is_global):
    err, _ = _case(cuda_device, n_seq=3, heads=2, win=win, d=64, ratio=0.4, is_global=is_global)
    assert err.max().item() < 3e-2


def test_identity_perm_dense_matches_sdpa(cuda_device):
    """ratio 1.0, identity order, zero tables: plain softmax attention."""
    n_seq, heads, win, d = 4, 2, 14, 64
    N, C = win * win, heads * d
    qkv = torch.randn(n_seq * N, 3 * C, device=cuda_device).to(torch.bfloat16)
    z = torch.zeros(2 * win - 1, d, device=cuda_device, dtype=torch.bfloat16)
    perm = torch.arange(N, device=cuda_device, dtype=torch.int32).repeat(n_seq * heads, 1).contiguous()
    out = ops.sparse_attn(qkv, n_seq, heads, win, d, z, z, perm, 5, False, d ** -0.5)
    q, k, v = qkv.float().view(n_seq, N, 3, heads, d).permute(2, 0, 3, 1, 4)
    ref = torch.nn.functional.scaled_dot_product_attention(q, k, v).permute(0, 2, 1, 3).reshape(n_seq * N, C)
    assert (out.float() - ref).abs().max().item() < 2e-2
    assert ops.device_error() == 0


@pytest.mark.parametrize("d", [64, 80])
@pytest.mark.parametrize("win,n_seq,heads,is_global", [(14, 300, 2, False), (64, 3, 4, True)])
def test_persistent_ctas_run_many_tiles(cuda_device, d, win, n_seq, heads, is_global):
    """More query tiles than SMs: every CTA walks several tiles, which exercises the
    double-buffered O accumulators, the deferred epilogue and the Q/bias reuse."""
    err, _ = _case(cuda_device, n_seq=n_seq, heads=heads, win=win, d=d, ratio=0.3, is_global=is_global, seed=3)
    assert err.max().item() < 3e-2, err.max().item()
    assert err.mean().item() < 3e-3
    assert ops.device_error() == 0


def test_out_rows_places_rows(cuda_device):
    """out_rows stores (sequence, token) rows through a map (-1 drops the row), as
    the windowed blocks use it for window_unpartition."""
    n_seq, heads, win, d = 4, 2, 14, 64
    N, C = win * win, heads * d
    g = torch.Generator().manual_seed(5)
    qkv = torch.randn(n_seq * N, 3 * C, generator=g).to(torch.bfloat16).to(cuda_device)
    th = (torch.randn(2 * win - 1, d, generator=g) * 0.3).to(torch.bfloat16).to(cuda_device)
    tw = (torch.randn(2 * win - 1, d, generator=g) * 0.3).to(torch.bfloat16).to(cuda_device)
    perm = torch.stack([torch.randperm(N, generator=g) for _ in range(n_seq * heads)]).to(torch.int32)
    perm = perm.to(cuda_device)
    n_init = order.a_shape_n_init(N, 64, 0.4, False)
    base = ops.sparse_attn(qkv, n_seq, heads, win, d, th, tw, perm, n_init, False, d ** -0.5)
    dst = torch.randperm(2 * n_seq * N, generator=g)[: n_seq * N].to(torch.int32)
    dst[::5] = -1
    dst = dst.to(cuda_device)
    out = torch.zeros(2 * n_seq * N, C, device=cuda_device, dtype=torch.bfloat16)
    ops.sparse_attn(qkv, n_seq, heads, win, d, th, tw, perm, n_init, False, d ** -0.5, out=out, out_rows=dst)
    keep = dst >= 0
    assert torch.equal(out[dst[keep].long()], base[keep])
    assert ops.device_error() == 0


def _config1_inputs(cuda_device):
    """B=8, heads=16, N=4096 (64x64), d=64, Q/K/V ~ N(0, 1) from
    seed 1, rel-pos tables (127, 64) ~ N(0, 0.02), bf16; the permutation is
    Stripe-Sort (z_interleave_sort) of the same K, as sam.py:193-209 derives it."""
    B, heads, win, d = 8, 16, 64, 64
    N, C = win * win, heads * d
    g = torch.Generator().manual_seed(1)
    qkv = torch.randn(B * N, 3 * C, generator=g).to(torch.bfloat16).to(cuda_device)
    th = (torch.randn(2 * win - 1, d, generator=g) * 0.02).to(torch.bfloat16).to(cuda_device)
    tw = (torch.randn(2 * win - 1, d, generator=g) * 0.02).to(torch.bfloat16).to(cuda_device)
    base = ops.zorder(win, win, cuda_device)[0]
    perm, _, _ = ops.stripe_sort_perm(qkv[:, C:], B, heads, win, win, d, base, ld=qkv.stride(0))
    return qkv, th, tw, perm, (B, heads, win, d)


@pytest.mark.parametrize("n_block", [64, 128])
def test_config1_shape_stripe_sort_perms(cuda_device, n_block):
    """Config 1's exact shape on Stripe-Sort permutations of the same K, at
    densities 0.3 / 0.4 / 0.5 and the dense control, with the reference's 64-token
    mask and the 128-token mask BASELINE names. Every row runs on the GPU; rows
    sampled across images and heads are compared with the fp32 oracle on the same
    bf16 values, and their permutations with the oracle's Stripe-Sort (bit-exact)."""
    qkv, th, tw, perm, (B, heads, win, d) = _config1_inputs(cuda_device)
    N, C = win * win, heads * d
    sample = [0, 77, 127]   # (image, head) rows: b * heads + h
    qkv_c = qkv.float().cpu().view(B, N, 3, heads, d)
    perm_c = perm.cpu()
    for r in sample:
        b, h = divmod(r, heads)
        k_row = qkv_c[b, :, 1, h].numpy()[None]
        p_ref, _, _ = order.stripe_sort(k_row, win, win)
        assert (perm_c[r].numpy() == p_ref[0]).all(), f"row {r}: Stripe-Sort permutation differs"
    for ratio in (0.3, 0.4, 0.5, 1.0):
        n_init = order.a_shape_n_init(N, n_block, ratio, True)
        out = ops.sparse_attn(qkv, B, heads, win, d, th, tw, perm, n_init, True, d ** -0.5, n_block=n_block)
        assert ops.device_error() == 0
        out_c = out.float().cpu().view(B, N, heads, d)
        for r in sample:
            b, h = divmod(r, heads)
            q, k, v = (qkv_c[b, :, i, h][None] for i in range(3))
            ref = sparse_attention(q, k, v, th.float().cpu(), tw.float().cpu(), perm_c[r][None], win, n_init, True,
                                   d ** -0.5, m_block=n_block, n_block=n_block, round_tables_fp16=False)[0]
            err = (out_c[b, :, h] - ref).abs()
            assert err.max().item() < 3e-2, (ratio, r, err.max().item())
            assert err.mean().item() < 3e-3, (ratio, r, err.mean().item())


@pytest.mark.parametrize("d", [64, 80])
@pytest.mark.parametrize("win,is_global", [(14, False), (64, True), (16, True)])
@pytest.mark.parametrize("ratio", [0.3, 0.5])
def test_128_token_mask_blocks(cuda_device, d, win, is_global, ratio):
    """The A-shape mask on 128-token blocks (n_block = 128): the keep bar in
    128-token units and, for global grids, whole 128-token diagonal blocks."""
    g = torch.Generator().manual_seed(9)
    n_seq, heads = 2, 2
    N, C = win * win, heads * d
    qkv = torch.randn(n_seq * N, 3 * C, generator=g).to(torch.bfloat16)
    th = (torch.randn(2 * win - 1, d, generator=g) * 0.3).to(torch.bfloat16)
    tw = (torch.randn(2 * win - 1, d, generator=g) * 0.3).to(torch.bfloat16)
    perm = torch.stack([torch.randperm(N, generator=g) for _ in range(n_seq * heads)]).to(torch.int32)
    n_init = order.a_shape_n_init(N, 128, ratio, is_global)
    if n_init == 0 and not is_global:
        pytest.skip("no key block enabled")
    out = ops.sparse_attn(qkv.to(cuda_device), n_seq, heads, win, d, th.to(cuda_device), tw.to(cuda_device),
                          perm.to(cuda_device), n_init, is_global, d ** -0.5, n_block=128)
    q, k, v = qkv.float().view(n_seq, N, 3, heads, d).permute(2, 0, 3, 1, 4).reshape(3, n_seq * heads, N, d)
    ref = sparse_attention(q, k, v, th.float(), tw.float(), perm, win, n_init, is_global, d ** -0.5,
                           m_block=128, n_block=128, round_tables_fp16=False)
    ref = ref.view(n_seq, heads, N, d).permute(0, 2, 1, 3).reshape(n_seq * N, C)
    err = (out.float().cpu() - ref).abs()
    assert err.max().item() < 3e-2, err.max().item()
    assert err.mean().item() < 3e-3
    assert ops.device_error() == 0


@pytest.mark.parametrize("d", [64, 80])
@pytest.mark.parametrize("B,H,W,ws", [(2, 20, 20, 14), (1, 64, 64, 14), (3, 9, 13, 7), (2, 16, 30, 14)])
def test_query_compaction_matches_every_token(cuda_device, d, B, H, W, ws):
    """Windowed grids with the image grid given compute only the real tokens of each
    window as queries (padding tokens stay keys); every stored row equals the run that
    computes all tokens, bit for bit, and matches the fp32 oracle."""
    heads = 2
    g = torch.Generator().manual_seed(11)
    rows = ops.window_rows(B, H, W, ws, cuda_device)
    n_win, N, C = rows.numel() // (ws * ws), ws * ws, heads * d
    qkv = torch.randn(n_win * N, 3 * C, generator=g).to(torch.bfloat16).to(cuda_device)
    th = (torch.randn(2 * ws - 1, d, generator=g) * 0.3).to(torch.bfloat16).to(cuda_device)
    tw = (torch.randn(2 * ws - 1, d, generator=g) * 0.3).to(torch.bfloat16).to(cuda_device)
    perm = torch.stack([torch.randperm(N, generator=g) for _ in range(n_win * heads)]).to(torch.int32)
    n_init = order.a_shape_n_init(N, 64, 0.4, False)
    out_all = torch.full((B * H * W, C), 3.0, device=cuda_device, dtype=torch.bfloat16)
    out_cmp = out_all.clone()
    ops.sparse_attn(qkv, n_win, heads, ws, d, th, tw, perm.to(cuda_device), n_init, False, d ** -0.5,
                    out=out_all, out_rows=rows)
    ops.sparse_attn(qkv, n_win, heads, ws, d, th, tw, perm.to(cuda_device), n_init, False, d ** -0.5,
                    out=out_cmp, out_rows=rows, grid=(H, W))
    assert ops.device_error() == 0
    assert torch.equal(out_all, out_cmp)
    q, k, v = qkv.float().cpu().view(n_win, N, 3, heads, d).permute(2, 0, 3, 1, 4).reshape(3, n_win * heads, N, d)
    ref = sparse_attention(q, k, v, th.float().cpu(), tw.float().cpu(), perm, ws, n_init, False, d ** -0.5,
                           round_tables_fp16=False)
    ref = ref.view(n_win, heads, N, d).permute(0, 2, 1, 3).reshape(n_win * N, C)
    real = rows.cpu() >= 0
    got = torch.empty(n_win * N, C)
    got[real] = out_cmp.float().cpu()[rows.cpu()[real].long()]
    err = (got[real] - ref[real]).abs()
    assert err.max().item() < 3e-2 and err.mean().item() < 3e-3


def test_query_compaction_many_tiles_per_cta(cuda_device):
    """ViT-H's windowed shape (16 heads, d = 80, 64 x 64 grid, 3 images): 1,968 query
    tiles, about 13 per persistent CTA, so a CTA runs many window-heads whose two
    query tiles read one K / V fill, next to window-heads with a single tile. Every
    stored row equals the run without compaction bit for bit, and sampled windows
    match the fp32 oracle."""
    B, H, W, ws, heads, d = 3, 64, 64, 14, 16, 80
    g = torch.Generator().manual_seed(5)
    rows = ops.window_rows(B, H, W, ws, cuda_device)
    n_win, N, C = rows.numel() // (ws * ws), ws * ws, heads * d
    qkv = torch.randn(n_win * N, 3 * C, generator=g).to(torch.bfloat16).to(cuda_device)
    th = (torch.randn(2 * ws - 1, d, generator=g) * 0.3).to(torch.bfloat16).to(cuda_device)
    tw = (torch.randn(2 * ws - 1, d, generator=g) * 0.3).to(torch.bfloat16).to(cuda_device)
    perm = torch.stack([torch.randperm(N, generator=g) for _ in range(n_win * heads)]).to(torch.int32)
    n_init = order.a_shape_n_init(N, 64, 0.3, False)
    out_all = torch.full((B * H * W, C), 3.0, device=cuda_device, dtype=torch.bfloat16)
    out_cmp = out_all.clone()
    ops.sparse_attn(qkv, n_win, heads, ws, d, th, tw, perm.to(cuda_device), n_init, False, d ** -0.5,
                    out=out_all, out_rows=rows)
    ops.sparse_attn(qkv, n_win, heads, ws, d, th, tw, perm.to(cuda_device), n_init, False, d ** -0.5,
                    out=out_cmp, out_rows=rows, grid=(H, W))
    assert ops.device_error() == 0
    assert torch.equal(out_all, out_cmp)
    sample = [0, 4, 20, 24, 37, 74]   # inner, last-column, last-row and corner windows of images 0-2
    q, k, v = qkv.float().cpu().view(n_win, N, 3, heads, d)[sample].permute(2, 0, 3, 1, 4).reshape(3, -1, N, d)
    ps = perm.view(n_win, heads, N)[sample].reshape(-1, N)
    ref = sparse_attention(q, k, v, th.float().cpu(), tw.float().cpu(), ps, ws, n_init, False, d ** -0.5,
                           round_tables_fp16=False)
    ref = ref.view(len(sample), heads, N, d).permute(0, 2, 1, 3).reshape(len(sample) * N, C)
    r = rows.view(n_win, N)[sample].reshape(-1).cpu()
    real = r >= 0
    got = out_cmp.float().cpu()[r[real].long()]
    err = (got - ref[real]).abs()
    assert err.max().item() < 3e-2 and err.mean().item() < 3e-3


@pytest.mark.parametrize("B,H,W,heads,d", [(2, 64, 64, 4, 80), (3, 9, 13, 2, 64)])
def test_pad_row_stands_for_padding_keys(cuda_device, B, H, W, heads, d):
    """With `pad_row` the kernel reads the padding keys' K / V from that row and
    never their qkv rows: qkv whose padding rows are NaN gives, bit for bit, the
    output of the run whose padding rows hold the bias (ssam_fill_pad_rows)."""
    ws = 14 if H > 14 else 7
    g = torch.Generator().manual_seed(21)
    rows = ops.window_rows(B, H, W, ws, cuda_device)
    n_win, N, C = rows.numel() // (ws * ws), ws * ws, heads * d
    qkv = torch.randn(n_win * N, 3 * C, generator=g).to(torch.bfloat16).to(cuda_device)
    bias = torch.randn(3 * C, generator=g).to(cuda_device)
    th = (torch.randn(2 * ws - 1, d, generator=g) * 0.3).to(torch.bfloat16).to(cuda_device)
    tw = (torch.randn(2 * ws - 1, d, generator=g) * 0.3).to(torch.bfloat16).to(cuda_device)
    perm = torch.stack([torch.randperm(N, generator=g) for _ in range(n_win * heads)]).to(torch.int32)
    perm = perm.to(cuda_device)
    n_init = order.a_shape_n_init(N, 64, 0.3, False)
    filled = qkv.clone()
    ops.fill_pad_rows(filled, rows, bias)
    holes = qkv.clone()
    holes[rows < 0] = float("nan")
    out_a = torch.zeros(B * H * W, C, device=cuda_device, dtype=torch.bfloat16)
    out_b = out_a.clone()
    ops.sparse_attn(filled, n_win, heads, ws, d, th, tw, perm, n_init, False, d ** -0.5, out=out_a,
                    out_rows=rows, grid=(H, W))
    ops.sparse_attn(holes, n_win, heads, ws, d, th, tw, perm, n_init, False, d ** -0.5, out=out_b,
                    out_rows=rows, grid=(H, W), pad_row=bias.to(torch.bfloat16))
    assert ops.device_error() == 0
    assert torch.isfinite(out_b.float()).all()
    assert torch.equal(out_a, out_b)
