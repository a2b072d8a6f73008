"""Dense restatement of the block-sparse rel-pos attention (torch fp32, CPU) —
test infrastructure only.

Follows the reference kernel's own self-check (algos/kernels/flash_attn.py:1519-1551):
scores of the permuted rows = (q_p k_p^T) * scale + relH[perm_q, kh(perm_k)] +
relW[perm_q, kw(perm_k)], block mask expanded to tokens, softmax with empty rows
-> 0, then P v_p. The result of permuted row p is written to raster row perm[p]
(the inverse gather at algos/sparsesam/sam.py:231-232).
"""
from __future__ import annotations

import torch


def rel_tables(table: torch.Tensor, win: int, round_fp16: bool = True) -> torch.Tensor:
    """(win, win, d): entry [i, j] = table[i - j + win - 1] (sam.py:32-49 for equal
    q/k sizes). The reference casts the result to fp16 (sam.py:49); with
    round_fp16 the values are rounded through fp16 and returned in fp32."""
    idx = torch.arange(win)[:, None] - torch.arange(win)[None, :] + win - 1
    t = table[idx]
    return t.half().float() if round_fp16 else t.float()


def rel_bias(q: torch.Tensor, Rh: torch.Tensor, Rw: torch.Tensor, win: int):
    """rel_h, rel_w of shape (R, N, win) from raster-order q (compute_rel_bias, sam.py:62-73)."""
    R, N, d = q.shape
    rq = q.reshape(R, win, win, d)
    rel_h = torch.einsum("bhwc,hkc->bhwk", rq, Rh).reshape(R, N, win)
    rel_w = torch.einsum("bhwc,wkc->bhwk", rq, Rw).reshape(R, N, win)
    return rel_h, rel_w


def sparse_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, rel_pos_h: torch.Tensor,
                     rel_pos_w: torch.Tensor, perm: torch.Tensor, win: int, n_init: int, with_diag: bool,
                     scale: float, m_block: int = 64, n_block: int = 64,
                     round_tables_fp16: bool = True) -> torch.Tensor:
    """q, k, v: (R, N, d) fp32 in raster order; perm: (R, N) int. Returns (R, N, d) raster order."""
    q, k, v = q.float(), k.float(), v.float()
    R, N, d = q.shape
    perm = perm.long()
    Rh = rel_tables(rel_pos_h.float(), win, round_tables_fp16)
    Rw = rel_tables(rel_pos_w.float(), win, round_tables_fp16)
    rel_h, rel_w = rel_bias(q, Rh, Rw, win)
    out = torch.empty_like(q)
    nm, nn = -(-N // m_block), -(-N // n_block)
    mb = torch.arange(N) // m_block
    nb = torch.arange(N) // n_block
    mask = (nb[None, :] < n_init) | (bool(with_diag) & (mb[:, None] == nb[None, :]))
    del nm, nn
    for r in range(R):
        p = perm[r]
        qp, kp, vp = q[r, p], k[r, p], v[r, p]
        kh, kw = p // win, p % win
        bias = rel_h[r, p][:, kh] + rel_w[r, p][:, kw]
        s = (qp @ kp.T) * scale + bias
        s = s.masked_fill(~mask, float("-inf"))
        a = torch.softmax(s, dim=-1).nan_to_num(0.0)
        out[r, p] = a @ vp
    return out
