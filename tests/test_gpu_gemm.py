"""tcgen05 GEMM parity against an fp64 matmul of the same bf16 operands.

Elementwise bound, from the arithmetic the kernel performs: products of bf16
operands are exact in fp32, the fp32 accumulation over K terms errs by at most
about K * 2^-24 * sum_k |a_k b_k| (taken 4x: K * 2^-22), and a bf16 output rounds
to nearest (half an ulp: 2^-8 relative). A GEMM that dropped or repeated a
16-wide K slice would miss this bound by an order of magnitude.
"""
import pytest
import torch

from sparsesam_b200 import ops

pytestmark = pytest.mark.gpu

SHAPES = [
    (128, 256, 64),
    (300, 256, 72),      # M tail, K tail inside one k-block
    (1000, 768, 1280),   # several n tiles, K multiple of 64
    (257, 96, 136),      # N not a multiple of 256, ragged everything
    (4900, 2304, 768),   # ViT-B windowed qkv shape (one image): 2-SM path
    (16384, 512, 128),   # 2-SM path, exact tiles
    (8192, 512, 320),    # 2-SM path, odd number of 64-wide K blocks (last stage half past K)
    (16384, 256, 136),   # 2-SM path, ragged K tail inside the last stage's first sub-tile
    (20000, 1280, 320),  # 2-SM path, M tail inside a CTA pair
    (16500, 768, 1280),  # 2-SM path, M tail in the second CTA of the last pair
    # small-batch ViT-L shapes (partial last wave of the 74 SM pairs)
    (16384, 1024, 1024),  # ViT-L batch-4 proj
    (4916, 1024, 512),    # ViT-L batch-4 fc2 on the keep rows (K shortened)
    (4916, 4096, 256),    # ViT-L batch-4 fc1 on the keep rows (K shortened)
    (16384, 992, 200),    # ragged last N tile, ragged K
]


def _ref(a, b, bias):
    r = a.double() @ b.double().T
    return (r + bias.double() if bias is not None else r).float()


def _bound(a, b, ref, out_bf16, slope=1.0):
    """Elementwise error bound (see the module docstring); `slope` bounds the
    derivative of the epilogue's activation (GELU: 1.13)."""
    K = a.shape[1]
    absprod = (a.double().abs() @ b.double().abs().T).float()
    acc = slope * K * 2.0 ** -22 * absprod
    rnd = 2.0 ** -8 * ref.abs() if out_bf16 else 2.0 ** -23 * ref.abs()
    return rnd + acc + 1e-6


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_bf16_epilogue(cuda_device, M, N, K):
    g = torch.Generator(device="cpu").manual_seed(M * 7 + N * 3 + K)
    a = torch.randn(M, K, generator=g).to(cuda_device, torch.bfloat16)
    b = (torch.randn(N, K, generator=g) * 0.05).to(cuda_device, torch.bfloat16)
    bias = torch.randn(N, generator=g).to(cuda_device)
    out = ops.gemm_bf16(a, b, bias)
    ref = _ref(a, b, bias)
    excess = ((out.float() - ref).abs() - _bound(a, b, ref, True)).max().item()
    assert excess <= 0, excess
    assert ops.device_error() == 0


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_gelu_epilogue(cuda_device, M, N, K):
    g = torch.Generator(device="cpu").manual_seed(11 + M)
    a = torch.randn(M, K, generator=g).to(cuda_device, torch.bfloat16)
    b = (torch.randn(N, K, generator=g) * 0.05).to(cuda_device, torch.bfloat16)
    bias = torch.randn(N, generator=g).to(cuda_device)
    out = ops.gemm_bf16(a, b, bias, epilogue=ops.SSAM_EPI_GELU_BF16)
    pre = _ref(a, b, bias)
    ref = torch.nn.functional.gelu(pre.double()).float()
    # + the erf approximation (|err| <= 1.5e-7, times |x| / 2) with headroom
    bound = _bound(a, b, ref, True, slope=1.13) + 1e-6 * (1.0 + pre.abs())
    excess = ((out.float() - ref).abs() - bound).max().item()
    assert excess <= 0, excess


def _written(rows, n_out):
    w = torch.zeros(n_out, dtype=torch.bool, device=rows.device)
    w[rows[rows >= 0].long()] = True
    return w


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_add_f32_rowmap(cuda_device, M, N, K):
    g = torch.Generator(device="cpu").manual_seed(23 + M)
    a = torch.randn(M, K, generator=g).to(cuda_device, torch.bfloat16)
    b = (torch.randn(N, K, generator=g) * 0.05).to(cuda_device, torch.bfloat16)
    bias = torch.randn(N, generator=g).to(cuda_device)
    n_out = M + 17
    rows = torch.randperm(n_out, generator=g)[:M].to(torch.int32)
    rows[::5] = -1                                  # skipped rows
    rows = rows.to(cuda_device)
    x0 = torch.randn(n_out, N, generator=g).to(cuda_device)
    x = x0.clone()
    ops.gemm_bf16(a, b, bias, epilogue=ops.SSAM_EPI_ADD_F32, out=x, out_rows=rows)
    ref = x0.clone()
    keep = rows >= 0
    acc = _ref(a, b, bias)
    ref[rows[keep].long()] += acc[keep]
    bound = torch.full_like(ref, 1e-6) + 2.0 ** -23 * ref.abs()
    bound[rows[keep].long()] += _bound(a, b, acc, False)[keep]
    excess = ((x - ref).abs() - bound).max().item()
    assert excess <= 0, excess
    assert torch.equal(x[~_written(rows, n_out)], x0[~_written(rows, n_out)])   # rows not addressed: untouched


@pytest.mark.parametrize("M", [256, 20480])
def test_gelu_epilogue_matches_exact_erf_gelu(cuda_device, M):
    """acc = 0, bias sweeps [-9, 9]: the GELU epilogue must reproduce the exact
    (erf) GELU of torch to within one bf16 ulp (its erf error is <= 1.5e-7)."""
    N, K = 2048, 64
    a = torch.zeros(M, K, device=cuda_device, dtype=torch.bfloat16)
    b = torch.zeros(N, K, device=cuda_device, dtype=torch.bfloat16)
    bias = torch.linspace(-9.0, 9.0, N, device=cuda_device)
    out = ops.gemm_bf16(a, b, bias, epilogue=ops.SSAM_EPI_GELU_BF16)
    exact = torch.nn.functional.gelu(bias.double()).float()
    got = out.float()
    # one bf16 ulp of the exact value (plus a tiny absolute floor near zero)
    ulp = torch.clamp(exact.abs(), min=2.0 ** -126) * 2.0 ** -7
    assert bool(((got - exact[None, :]).abs() <= ulp[None, :] + 1e-6).all())


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_bf16_rowmap(cuda_device, M, N, K):
    """bf16 epilogue through a row map (the window-partition scatter of qkv):
    row r lands at out[rows[r]], rows < 0 are skipped, untouched rows keep
    their contents."""
    g = torch.Generator(device="cpu").manual_seed(31 + M)
    a = torch.randn(M, K, generator=g).to(cuda_device, torch.bfloat16)
    b = (torch.randn(N, K, generator=g) * 0.05).to(cuda_device, torch.bfloat16)
    bias = torch.randn(N, generator=g).to(cuda_device)
    n_out = M + 23
    rows = torch.randperm(n_out, generator=g)[:M].to(torch.int32)
    rows[1::7] = -1
    rows = rows.to(cuda_device)
    out = torch.full((n_out, N), 7.0, device=cuda_device, dtype=torch.bfloat16)
    ops.gemm_bf16(a, b, bias, out=out, out_rows=rows)
    ref = torch.full((n_out, N), 7.0, device=cuda_device)
    keep = rows >= 0
    acc = _ref(a, b, bias)
    ref[rows[keep].long()] = acc[keep]
    bound = torch.zeros_like(ref)
    bound[rows[keep].long()] = _bound(a, b, acc, True)[keep]
    excess = ((out.float() - ref).abs() - bound).max().item()
    assert excess <= 0, excess


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("use_rows", [False, True])
def test_gemm_f32_epilogues(cuda_device, M, N, K, use_rows):
    """fp32 store and fp32 residual add, with and without a row map; the
    2-SM kernel moves these rows with bulk copies (the add as a bulk reduce)."""
    g = torch.Generator(device="cpu").manual_seed(41 + M + (1 if use_rows else 0))
    a = torch.randn(M, K, generator=g).to(cuda_device, torch.bfloat16)
    b = (torch.randn(N, K, generator=g) * 0.05).to(cuda_device, torch.bfloat16)
    bias = torch.randn(N, generator=g).to(cuda_device)
    n_out = M + 9 if use_rows else M
    rows = None
    if use_rows:
        rows = torch.randperm(n_out, generator=g)[:M].to(torch.int32)
        rows[2::9] = -1
        rows = rows.to(cuda_device)
    acc = _ref(a, b, bias)
    acc_bound = _bound(a, b, acc, False)
    keep = rows >= 0 if use_rows else slice(None)
    dst = rows[keep].long() if use_rows else slice(None)
    # plain fp32 store
    out = torch.full((n_out, N), -3.0, device=cuda_device)
    ops.gemm_bf16(a, b, bias, epilogue=ops.SSAM_EPI_F32, out=out, out_rows=rows)
    ref = torch.full((n_out, N), -3.0, device=cuda_device)
    ref[dst] = acc[keep]
    bound = torch.zeros_like(ref)
    bound[dst] = acc_bound[keep]
    assert ((out - ref).abs() - bound).max().item() <= 0
    # residual add
    x0 = torch.randn(n_out, N, generator=g).to(cuda_device)
    x = x0.clone()
    ops.gemm_bf16(a, b, bias, epilogue=ops.SSAM_EPI_ADD_F32, out=x, out_rows=rows)
    ref = x0.clone()
    ref[dst] += acc[keep]
    bound = 2.0 ** -23 * ref.abs() + 1e-6
    bound[dst] += acc_bound[keep]
    assert ((x - ref).abs() - bound).max().item() <= 0
    assert ops.device_error() == 0
