"""Generate the golden fixtures by running the reference's own SparseSAM code on CPU.

Usage:  python tests/golden/make_golden.py --reference <path to a hchautran/SparseSAM checkout>
        [--only hilbert]   (write golden_hilbert.npz alone)

What runs is the reference's unmodified algos/sparsesam/sam.py and z_utils.py.
Three things are supplied around it, because the reference cannot run on a CPU
host without them:
  * segment_anything.modeling.image_encoder (the un-vendored SAM-HQ submodule):
    provided by sparsesam_b200.host, an independent SAM-architecture encoder;
  * the CuTe-DSL kernel launch: replaced by a CPU function that computes what the
    reference's own kernel self-check computes (algos/kernels/flash_attn.py:1519-1551);
    the DLPack wrappers and stream lookup become identities;
  * get_rel_pos: its fp16 result is cast back to the query dtype so the fp32 run
    works (the fp16 rounding of the table is kept).
The reference's torch.argsort / topk are used as they are (not stable), so the
fixtures record the reference's own tie order.

Outputs (next to this script):
  golden_order.npz  Z-order KATs, tile_stride_matching outputs for window / padded
                    window / global inputs and four perm modes, A-shape n_init table
  golden_e2e.npz    a small SparseSAM-patched encoder forward (features,
                    intermediate embeddings, permutations, keep sets, dense control)
  golden_hilbert.npz  the reference's Hilbert orders (hilbert_utils.py) for seven
                    grids and tile_stride_matching in three Hilbert perm modes
  golden_sam3.npz   the SAM3 MLP-merge keep sets (sam3.py _get_keep_indices) for six
                    grids x ten ratios, and the small encoder with every block
                    patched by the reference's ToMeSAM3Block
"""
from __future__ import annotations

import argparse
import contextlib
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from sparsesam_b200 import host  # noqa: E402

# Small encoder used for the end-to-end fixture: 256x256 input -> 16x16 grid,
# 14x14 windows (padded to 28x28 -> 4 windows), heads of dim 64, blocks 1 and 3 global.
E2E_CFG = dict(img_size=256, embed_dim=128, depth=4, num_heads=2, global_attn_indexes=(1, 3), window_size=14)
E2E_RATIO = 0.4
E2E_SEED = 0


def e2e_encoder() -> host.ImageEncoderViT:
    enc = host.ImageEncoderViT(**E2E_CFG)
    host.init_weights(enc, E2E_SEED)
    return enc.float().eval()


def bf16_round(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).float()


def bf16_bits(x: torch.Tensor) -> np.ndarray:
    return x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def install_host_as_segment_anything() -> None:
    sa = types.ModuleType("segment_anything")
    sa.__path__ = []
    modeling = types.ModuleType("segment_anything.modeling")
    modeling.__path__ = []
    ie = types.ModuleType("segment_anything.modeling.image_encoder")
    for name in ("ImageEncoderViT", "Block", "Attention", "window_partition", "window_unpartition"):
        setattr(ie, name, getattr(host, name))
    sys.modules["segment_anything"] = sa
    sys.modules["segment_anything.modeling"] = modeling
    sys.modules["segment_anything.modeling.image_encoder"] = ie


class CpuKernel:
    """Stands in for FlashAttentionForwardAmpere: same call signature as the
    compiled a_shape kernel (sam.py:224-230), computing the dense masked softmax
    of the reference self-check (flash_attn.py:1519-1551). Records n_init_blocks."""

    calls: list = []

    @classmethod
    def get_compiled_a_shape(cls, D, m_block, n_block, threads, win, with_diagonal, *args):
        def run(q_c, k_c, v_c, o_c, rh_c, rw_c, pq_c, pk_c, n_init, scale, stream):
            cls.calls.append(dict(N=q_c.shape[1], win=win, with_diag=bool(with_diagonal), n_init=int(n_init)))
            q, k, v = q_c[:, :, 0].float(), k_c[:, :, 0].float(), v_c[:, :, 0].float()
            BH, N, _ = q.shape
            pq, pk = pq_c.long(), pk_c.long()
            rh, rw = rh_c[:, :, 0].float(), rw_c[:, :, 0].float()
            mb = torch.arange(N) // m_block
            nb = torch.arange(N) // n_block
            enabled = (nb[None, :] < n_init) | (bool(with_diagonal) & (mb[:, None] == nb[None, :]))
            for b in range(BH):
                bias = rh[b, pq[b]][:, pk[b] // win] + rw[b, pq[b]][:, pk[b] % win]
                s = q[b] @ k[b].T * scale + bias
                s = s.masked_fill(~enabled, float("-inf"))
                p = torch.softmax(s, dim=-1).nan_to_num(0.0)
                o_c[b, :, 0] = (p @ v[b]).to(o_c.dtype)
        return run


def load_reference(ref_root: str):
    sys.path.insert(0, ref_root)
    install_host_as_segment_anything()
    import algos.sparsesam.sam as ref_sam  # noqa: E402
    import algos.sparsesam.z_utils as ref_z  # noqa: E402
    orig_get_rel_pos = ref_sam.get_rel_pos
    ref_sam.get_rel_pos = lambda q, k, t: orig_get_rel_pos(q, k, t).to(t.dtype)
    ref_sam.FlashAttentionForwardAmpere = CpuKernel
    ref_sam._wrap_qkvo = lambda t, dtype: t
    ref_sam._wrap_bias = lambda t: t
    ref_sam._wrap_perm = lambda t: t
    ref_sam._get_cu_stream = lambda: None
    ref_sam._warmup_fa2_kernels = lambda enc: None
    return ref_sam, ref_z


@contextlib.contextmanager
def record_topk(log: list):
    orig = torch.Tensor.topk

    def topk(self, *a, **kw):
        res = orig(self, *a, **kw)
        log.append(res.indices.clone())
        return res

    torch.Tensor.topk = topk
    try:
        yield
    finally:
        torch.Tensor.topk = orig


def make_order(ref_sam, ref_z) -> dict:
    out = {}
    for H, W in ((4, 4), (14, 14), (64, 64), (16, 16)):
        out[f"zorder_{H}x{W}"] = ref_z.get_z_order(H, W).numpy().astype(np.int32)
        out[f"zinv_{H}x{W}"] = ref_z.get_z_inverse(H, W).numpy().astype(np.int32)
    g = torch.Generator().manual_seed(1234)
    cases = {}
    # Window rows: K of 8 (window, head) rows, 196 tokens, d = 64.
    cases["win"] = (bf16_round(torch.randn(8, 196, 64, generator=g)), 14)
    # Padded windows: bottom-right window of a 64x64 grid after 64->70 padding;
    # padded tokens have K = 0 (zero qkv bias), giving exactly tied groups.
    kp = bf16_round(torch.randn(4, 196, 64, generator=g))
    grid = kp.view(4, 14, 14, 64)
    grid[:, 8:, :, :] = 0
    grid[:, :, 8:, :] = 0
    cases["winpad"] = (kp, 14)
    # Global rows: 2 rows of a 64x64 grid, d = 16 (kept small for the fixture).
    cases["glob"] = (bf16_round(torch.randn(2, 4096, 16, generator=g)), 64)
    for name, (k, win) in cases.items():
        out[f"k_{name}"] = bf16_bits(k)
        modes = ("z_interleave_sort", "z_naive_sort", "z_interleave_nosort", "z_naive_nosort")
        for mode in modes:
            p, ip, ipg = ref_sam.tile_stride_matching(k, win, win, ratio=E2E_RATIO, perm_mode=mode)
            out[f"{name}_{mode}_perm"] = p.numpy().astype(np.int16)
            out[f"{name}_{mode}_inv"] = ip.numpy().astype(np.int16)
            out[f"{name}_{mode}_invg"] = ipg.numpy().astype(np.int16)
    # A-shape n_init from the reference attention forward (sam.py:219-223).
    rows = []
    for win, is_global in ((14, False), (16, True), (64, True), (16, False)):
        for ratio in (0.05, 0.1, 0.25, 0.3, 0.4, 0.5, 0.6, 0.75, 0.9, 1.0):
            attn = host.Attention(16, num_heads=1, input_size=(win, win))
            attn.__class__ = ref_sam.ToMeSAMAttention
            attn._tome_info = {"perm_mode": "z_interleave_sort"}
            CpuKernel.calls.clear()
            x = torch.randn(1, win, win, 16, generator=g)
            with torch.no_grad():
                attn(x, ratio, is_global=is_global, return_perm=True)
            c = CpuKernel.calls[-1]
            rows.append((win * win, int(is_global), ratio, c["n_init"], int(c["with_diag"])))
    out["n_init_table"] = np.array([(r[0], r[1], r[3], r[4]) for r in rows], dtype=np.int32)
    out["n_init_ratio"] = np.array([r[2] for r in rows], dtype=np.float64)
    return out


def make_hilbert(ref_sam) -> dict:
    import algos.sparsesam.hilbert_utils as ref_h  # noqa: E402
    out = {}
    for H, W in ((4, 4), (14, 14), (64, 64), (16, 16), (7, 9), (1, 5), (2, 2)):
        out[f"horder_{H}x{W}"] = ref_h.get_hilbert_order(H, W).numpy().astype(np.int32)
        out[f"hinv_{H}x{W}"] = ref_h.get_hilbert_inverse(H, W).numpy().astype(np.int32)
    g = torch.Generator().manual_seed(4321)
    cases = {"win": (bf16_round(torch.randn(6, 196, 64, generator=g)), 14),
             "glob": (bf16_round(torch.randn(2, 4096, 16, generator=g)), 64)}
    for name, (k, win) in cases.items():
        out[f"k_{name}"] = bf16_bits(k)
        for mode in ("hilbert_interleave_sort", "hilbert_naive_sort", "hilbert_interleave_nosort"):
            p, ip, ipg = ref_sam.tile_stride_matching(k, win, win, ratio=E2E_RATIO, perm_mode=mode)
            out[f"{name}_{mode}_perm"] = p.numpy().astype(np.int16)
            out[f"{name}_{mode}_inv"] = ip.numpy().astype(np.int16)
            out[f"{name}_{mode}_invg"] = ipg.numpy().astype(np.int16)
    return out


def make_e2e(ref_sam) -> dict:
    out = {}
    img = host.synthetic_images(1, seed=E2E_SEED, img_size=E2E_CFG["img_size"])
    out["img_checksum"] = np.array([float(img.double().sum())])
    enc = e2e_encoder()
    out["weights_checksum"] = np.array([sum(float(p.detach().double().sum()) for p in enc.parameters())])
    with torch.no_grad():
        dense_feat, dense_interm = enc(img)
    out["stock_features"] = dense_feat.numpy()

    ref_sam.apply_patch(enc, algo="tome", ratio=E2E_RATIO, mlp_merge=True)
    topk_log: list = []
    with torch.no_grad(), record_topk(topk_log):
        feat, interm = enc(img)
    out["features"] = feat.numpy()
    for i, t in enumerate(interm):
        out[f"interm_{i}"] = t.numpy()
    for key, val in enc.tome_info["perm_cache"].items():
        win = key[0]
        out[f"perm_win{win}"] = val[0].numpy().astype(np.int16)
        out[f"inv_win{win}"] = val[1].numpy().astype(np.int16)
        out[f"invg_win{win}"] = val[2].numpy().astype(np.int16)
    for i, idx in enumerate(topk_log):
        out[f"keep_{i}"] = idx.numpy().astype(np.int16)
    out["n_keep_calls"] = np.array([len(topk_log)])

    # Dense control: ratio 1.0 through the patch (all blocks enabled, dense MLP).
    enc2 = e2e_encoder()
    ref_sam.apply_patch(enc2, algo="tome", ratio=1.0, mlp_merge=True)
    with torch.no_grad():
        f1, _ = enc2(img)
    out["dense_patched_features"] = f1.numpy()
    return out


SAM3_GRIDS = ((64, 64), (72, 72), (14, 14), (7, 9), (1, 5), (3, 3))
SAM3_RATIOS = (0.001, 0.1, 0.25, 0.3, 0.4, 0.5, 0.7, 0.9, 0.99, 1.0)
SAM3_E2E_RATIO = 0.3


def load_sam3(ref_root: str, ref_z):
    """`_get_keep_indices` and `ToMeSAM3Block` of algos/sparsesam/sam3.py, unmodified.

    The module imports sam3.model.vitdet (the un-vendored SAM3 package) at load
    time, so the two definitions are taken from its source with `ast` and run in a
    namespace that supplies what they use: torch, get_z_order from the reference's
    z_utils, the host SAM Block as the base class (a vitdet-style block), and the
    host's window_partition / window_unpartition."""
    import ast
    path = os.path.join(ref_root, "algos", "sparsesam", "sam3.py")
    tree = ast.parse(open(path).read())
    keep = [n for n in tree.body if isinstance(n, (ast.FunctionDef, ast.ClassDef)) and
            n.name in ("_get_keep_indices", "ToMeSAM3Block")]
    assert len(keep) == 2
    ns = {"torch": torch, "nn": torch.nn, "Optional": None, "get_z_order": ref_z.get_z_order, "Block": host.Block,
          "window_partition": host.window_partition, "window_unpartition": host.window_unpartition,
          "_KEEP_PERM_CACHE": {}}
    exec(compile(ast.Module(body=keep, type_ignores=[]), path, "exec"), ns)
    return ns["_get_keep_indices"], ns["ToMeSAM3Block"]


def make_sam3(ref_root: str, ref_z) -> dict:
    get_keep, block_cls = load_sam3(ref_root, ref_z)
    out = {}
    for H, W in SAM3_GRIDS:
        for r in SAM3_RATIOS:
            out[f"keep_{H}x{W}_{r}"] = get_keep(H, W, r, "cpu").numpy().astype(np.int32)
    # The small golden encoder with every block patched by the reference's
    # ToMeSAM3Block (full attention, partial MLP on the keep set); SAM blocks carry
    # no layer scale, dropout or drop path, so those are identities here.
    img = host.synthetic_images(1, seed=E2E_SEED, img_size=E2E_CFG["img_size"])
    enc = e2e_encoder()
    info = {"ratio": SAM3_E2E_RATIO, "mlp_merge": True}
    for m in enc.modules():
        if isinstance(m, host.Block):
            m.__class__ = block_cls
            m._tome_info = info
            m.ls1 = m.ls2 = m.dropout = m.drop_path = torch.nn.Identity()
    with torch.no_grad():
        feat, interm = enc(img)
    out["e2e_features"] = feat.numpy()
    for i, t in enumerate(interm):
        out[f"e2e_interm_{i}"] = t.numpy()
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of a hchautran/SparseSAM checkout")
    ap.add_argument("--only", choices=("all", "hilbert", "sam3"), default="all")
    args = ap.parse_args()
    torch.manual_seed(0)
    ref_root = os.path.abspath(args.reference)
    ref_sam, ref_z = load_reference(ref_root)
    if args.only == "all":
        np.savez_compressed(os.path.join(HERE, "golden_order.npz"), **make_order(ref_sam, ref_z))
        np.savez_compressed(os.path.join(HERE, "golden_e2e.npz"), **make_e2e(ref_sam))
    if args.only in ("all", "hilbert"):
        np.savez_compressed(os.path.join(HERE, "golden_hilbert.npz"), **make_hilbert(ref_sam))
    if args.only in ("all", "sam3"):
        np.savez_compressed(os.path.join(HERE, "golden_sam3.npz"), **make_sam3(ref_root, ref_z))
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    main()
