"""The CPU oracle against golden vectors from the reference's own code (CPU only)."""
import numpy as np
import pytest
import torch

from oracle import encoder as oenc
from oracle import order
from oracle.attention import sparse_attention
from tests._golden import (E2E_RATIO, HILBERT_GRIDS, HILBERT_MODES, MODES, bf16_bits_to_f32, e2e_encoder,
                           group_order, load, SAM3_E2E_RATIO, SAM3_GRIDS, SAM3_RATIOS)

GO = load("golden_order.npz")
GE = load("golden_e2e.npz")
GH = load("golden_hilbert.npz")


def test_zorder_kat():
    # 4x4 Morton order (known answer, z_utils.py:35-101)
    assert order.zorder(4, 4)[0].tolist() == [0, 1, 4, 5, 2, 3, 6, 7, 8, 9, 12, 13, 10, 11, 14, 15]
    for H, W in ((4, 4), (14, 14), (64, 64), (16, 16)):
        p, inv = order.zorder(H, W)
        np.testing.assert_array_equal(p, GO[f"zorder_{H}x{W}"])
        np.testing.assert_array_equal(inv, GO[f"zinv_{H}x{W}"])


def test_hilbert_order_matches_reference():
    # 4x4 Hilbert order (known answer from the reference's hilbert_utils.py)
    assert order.hilbert_order(4, 4)[0].tolist() == [0, 4, 5, 1, 2, 3, 7, 6, 10, 11, 15, 14, 13, 9, 8, 12]
    for H, W in HILBERT_GRIDS:
        p, inv = order.hilbert_order(H, W)
        np.testing.assert_array_equal(p, GH[f"horder_{H}x{W}"])
        np.testing.assert_array_equal(inv, GH[f"hinv_{H}x{W}"])


@pytest.mark.parametrize("case,win", [("win", 14), ("glob", 64)])
@pytest.mark.parametrize("mode", HILBERT_MODES)
def test_stripe_sort_hilbert_matches_reference(case, win, mode):
    k = bf16_bits_to_f32(GH[f"k_{case}"])
    p, ip, ipg = order.stripe_sort(k, win, win, perm_mode=mode)
    np.testing.assert_array_equal(p, GH[f"{case}_{mode}_perm"].astype(np.int64))
    np.testing.assert_array_equal(ip, GH[f"{case}_{mode}_inv"].astype(np.int64))
    np.testing.assert_array_equal(ipg, GH[f"{case}_{mode}_invg"].astype(np.int64))


CASES = [("win", 14, 64), ("winpad", 14, 64), ("glob", 64, 16)]


@pytest.mark.parametrize("case,win,d", CASES)
@pytest.mark.parametrize("mode", MODES)
def test_stripe_sort_matches_reference(case, win, d, mode):
    k = bf16_bits_to_f32(GO[f"k_{case}"])
    p, ip, ipg = order.stripe_sort(k, win, win, perm_mode=mode)
    gp, gip, gipg = (GO[f"{case}_{mode}_{s}"].astype(np.int64) for s in ("perm", "inv", "invg"))
    # inverses are consistent in both
    for perm, inv in ((p, ip), (gp, gip)):
        np.testing.assert_array_equal(np.take_along_axis(perm, inv, 1), np.broadcast_to(np.arange(win * win), perm.shape))
    if case != "winpad" or mode.endswith("nosort"):
        # no ties: bit-exact with the reference
        np.testing.assert_array_equal(p, gp)
        np.testing.assert_array_equal(ip, gip)
        np.testing.assert_array_equal(ipg, gipg)
        return
    # Exactly tied groups (zero-padded tokens): the reference's argsort is not
    # stable. The rank sequences must agree on scores, and differ only inside
    # runs of exactly equal score.
    N, gs = win * win, 4
    G = N // gs
    layout = mode.split("_")[1]
    zinv = order.zorder(win, win)[1]
    ours = group_order(p, layout, G, gs, zinv)
    gold = group_order(gp, layout, G, gs, zinv)
    sc = order.group_scores(k, win, win)
    for r in range(k.shape[0]):
        np.testing.assert_array_equal(sc[r, ours[r]], sc[r, gold[r]])
        differ = ours[r] != gold[r]
        if differ.any():
            # every differing rank position sits in a tied run of the score
            s_sorted = sc[r, ours[r]]
            for q in np.nonzero(differ)[0]:
                assert ((s_sorted == s_sorted[q]).sum()) > 1
        # our order is the stable one: within a tie, ascending group index
        s = sc[r, ours[r]]
        same = s[1:] == s[:-1]
        assert np.all(ours[r][1:][same] > ours[r][:-1][same])


def test_n_init_table_matches_reference():
    tab = GO["n_init_table"]
    ratios = GO["n_init_ratio"]
    for (N, is_global, n_init, with_diag), ratio in zip(tab, ratios):
        assert order.a_shape_n_init(int(N), 64, float(ratio), bool(is_global)) == n_init
        assert with_diag == is_global


def _forced_from_golden(mode="z_interleave_sort"):
    forced = {}
    for win in (14, 16):
        forced[(win, E2E_RATIO, 64, mode)] = tuple(GE[f"{s}_win{win}"].astype(np.int64) for s in ("perm", "inv", "invg"))
    return forced


def test_e2e_inputs_reproduce():
    from sparsesam_b200 import host
    enc = e2e_encoder()
    ws = sum(float(p.detach().double().sum()) for p in enc.parameters())
    assert abs(ws - float(GE["weights_checksum"][0])) <= 1e-9 * max(1.0, abs(ws))
    img = host.synthetic_images(1, seed=0, img_size=256)
    assert abs(float(img.double().sum()) - float(GE["img_checksum"][0])) < 1e-6


def _assert_same_up_to_ties(k, win, ours_perm, gold_perm, layout="interleave"):
    """Group rankings agree on scores and differ only inside exactly tied runs."""
    N, gs = win * win, 4
    G = N // gs
    zinv = order.zorder(win, win)[1]
    ours = group_order(ours_perm, layout, G, gs, zinv)
    gold = group_order(gold_perm, layout, G, gs, zinv)
    sc = order.group_scores(k, win, win)
    n_diff = 0
    for r in range(k.shape[0]):
        np.testing.assert_array_equal(sc[r, ours[r]], sc[r, gold[r]])
        s_sorted = sc[r, ours[r]]
        for q in np.nonzero(ours[r] != gold[r])[0]:
            assert (s_sorted == s_sorted[q]).sum() > 1
            n_diff += 1
    return n_diff


def test_e2e_permutations_match_reference():
    from sparsesam_b200 import host
    enc = e2e_encoder()
    img = host.synthetic_images(1, seed=0, img_size=256)
    _, _, state = oenc.encoder_forward(enc, img, E2E_RATIO, return_state=True)
    pc = state["perm_cache"]
    # global grid (16x16): no ties, bit-exact
    ours = pc[(16, E2E_RATIO, 64, "z_interleave_sort")]
    np.testing.assert_array_equal(ours[0].numpy(), GE["perm_win16"])
    np.testing.assert_array_equal(ours[2].numpy(), GE["invg_win16"])
    # windows (16x16 grid padded to 28x28): padded tokens tie exactly
    key = (14, E2E_RATIO, 64, "z_interleave_sort")
    k = pc[("k",) + key].numpy()
    _assert_same_up_to_ties(k, 14, pc[key][0].numpy(), GE["perm_win14"].astype(np.int64))


def test_e2e_keep_set_matches_reference():
    ipg = GE["invg_win16"].astype(np.int64)
    gold = GE["keep_0"].astype(np.int64)
    keep_n = order.keep_n_for(E2E_RATIO, 256)
    assert gold.shape == (1, keep_n)
    ours = order.keep_select(ipg, 1, 2, keep_n)
    sums = ipg.reshape(1, 2, 256).sum(1)
    # same multiset of keys; tokens strictly inside the cut are identical
    np.testing.assert_array_equal(np.sort(sums[0, ours[0]]), np.sort(sums[0, gold[0]]))
    cut = np.sort(sums[0])[keep_n - 1]
    inside = set(np.nonzero(sums[0] < cut)[0].tolist())
    assert inside <= set(ours[0].tolist()) and inside <= set(gold[0].tolist())


def test_e2e_features_match_reference():
    from sparsesam_b200 import host
    enc = e2e_encoder()
    img = host.synthetic_images(1, seed=0, img_size=256)
    feats, interm = oenc.encoder_forward(enc, img, E2E_RATIO, forced_perms=_forced_from_golden())
    np.testing.assert_allclose(feats.numpy(), GE["features"], atol=2e-4, rtol=0)
    for i, t in enumerate(interm):
        np.testing.assert_allclose(t.numpy(), GE[f"interm_{i}"], atol=2e-4, rtol=0)


def test_dense_control_matches_reference_and_stock():
    from sparsesam_b200 import host
    enc = e2e_encoder()
    img = host.synthetic_images(1, seed=0, img_size=256)
    feats, _ = oenc.encoder_forward(enc, img, 1.0)
    np.testing.assert_allclose(feats.numpy(), GE["dense_patched_features"], atol=2e-4, rtol=0)
    # ratio 1.0 enables every block: the patched path equals the stock encoder
    # up to the fp16 rounding of the rel-pos tables (sam.py:49).
    np.testing.assert_allclose(GE["dense_patched_features"], GE["stock_features"], atol=5e-3, rtol=0)


def test_attention_restatement_equals_stock_attention_when_dense():
    from sparsesam_b200 import host
    torch.manual_seed(0)
    attn = host.Attention(64, num_heads=2, input_size=(8, 8))
    torch.nn.init.normal_(attn.rel_pos_h, std=0.3)
    torch.nn.init.normal_(attn.rel_pos_w, std=0.3)
    x = torch.randn(2, 8, 8, 64)
    with torch.no_grad():
        ref = attn(x)
        B, N, C, h = 2, 64, 64, 2
        qkv = torch.nn.functional.linear(x.reshape(B, N, C), attn.qkv.weight, attn.qkv.bias)
        q, k, v = qkv.view(B, N, 3, h, C // h).permute(2, 0, 3, 1, 4).reshape(3, B * h, N, C // h).unbind(0)
        perm = torch.stack([torch.randperm(N) for _ in range(B * h)])
        o = sparse_attention(q, k, v, attn.rel_pos_h, attn.rel_pos_w, perm, 8, n_init=1, with_diag=False,
                             scale=attn.scale, round_tables_fp16=False)
        o = o.reshape(B, h, N, C // h).permute(0, 2, 1, 3).reshape(B, 8, 8, C)
        out = torch.nn.functional.linear(o, attn.proj.weight, attn.proj.bias)
    torch.testing.assert_close(out, ref, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("H,W", SAM3_GRIDS)
def test_zstride_keep_matches_reference(H, W):
    """The SAM3 keep set (sam3.py:49-71), bit-exact against the reference's own
    _get_keep_indices for every fixture grid and ratio."""
    g = load("golden_sam3.npz")
    for r in SAM3_RATIOS:
        np.testing.assert_array_equal(order.zstride_keep(H, W, r), g[f"keep_{H}x{W}_{r}"])


def test_zstride_keep_n_host_entry_point():
    """ssam_zstride_keep_n (host-only) equals min(max(1, round(r N)), N), Python's
    ties-to-even round included (r N = 2.5 -> 2, 3.5 -> 4)."""
    from sparsesam_b200 import _lib
    lib = _lib.load()
    for N in (1, 5, 9, 10, 196, 4096, 5184):
        for r in SAM3_RATIOS + (0.05, 0.35, 0.45, 0.75):
            assert lib.ssam_zstride_keep_n(N, r) == min(max(1, round(r * N)), N), (N, r)
    assert lib.ssam_zstride_keep_n(10, 0.25) == 2 and lib.ssam_zstride_keep_n(10, 0.35) == 4
    assert lib.ssam_zstride_keep_n(10, 0.0) == -1 and lib.ssam_zstride_keep_n(10, 1.5) == -1


def test_sam3_encoder_restatement_matches_reference():
    """The oracle's ToMeSAM3Block restatement on the small golden encoder equals the
    reference's own ToMeSAM3Block.forward run by make_golden.py."""
    from sparsesam_b200 import host
    g = load("golden_sam3.npz")
    img = host.synthetic_images(1, seed=0, img_size=256)
    feats, interm = oenc.sam3_encoder_forward(e2e_encoder(), img, SAM3_E2E_RATIO)
    np.testing.assert_allclose(feats.numpy(), g["e2e_features"], atol=2e-4, rtol=0)
    for i, t in enumerate(interm):
        np.testing.assert_allclose(t.numpy(), g[f"e2e_interm_{i}"], atol=2e-4, rtol=0)
