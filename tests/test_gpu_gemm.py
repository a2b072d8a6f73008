"""tcgen05 GEMM parity against an fp32 matmul of the same bf16 operands."""
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
]


def _ref(a, b, bias):
    r = a.float() @ b.float().T
    return r + bias if bias is not None else r


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_bf16_epilogue(cuda_device, M, N, K):
    g = torch.Generator(device="cpu").manual_seed(M * 7 + N * 3 + K)
    a = torch.randn(M, K, generator=g).to(cuda_device, torch.bfloat16)
    b = (torch.randn(N, K, generator=g) * 0.05).to(cuda_device, torch.bfloat16)
    bias = torch.randn(N, generator=g).to(cuda_device)
    out = ops.gemm_bf16(a, b, bias)
    ref = _ref(a, b, bias)
    err = (out.float() - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item() + 1e-3, err
    assert ops.device_error() == 0


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_gelu_epilogue(cuda_device, M, N, K):
    g = torch.Generator(device="cpu").manual_seed(11 + M)
    a = torch.randn(M, K, generator=g).to(cuda_device, torch.bfloat16)
    b = (torch.randn(N, K, generator=g) * 0.05).to(cuda_device, torch.bfloat16)
    bias = torch.randn(N, generator=g).to(cuda_device)
    out = ops.gemm_bf16(a, b, bias, epilogue=ops.SSAM_EPI_GELU_BF16)
    ref = torch.nn.functional.gelu(_ref(a, b, bias))
    err = (out.float() - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item() + 1e-3, err


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
    ref[rows[keep].long()] += _ref(a, b, bias)[keep]
    err = (x - ref).abs().max().item()
    assert err <= 1e-3 * ref.abs().max().item() + 1e-3, err


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
    ref[rows[keep].long()] = _ref(a, b, bias)[keep]
    err = (out.float() - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item() + 1e-3, err


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
    keep = rows >= 0 if use_rows else slice(None)
    dst = rows[keep].long() if use_rows else slice(None)
    # plain fp32 store
    out = torch.full((n_out, N), -3.0, device=cuda_device)
    ops.gemm_bf16(a, b, bias, epilogue=ops.SSAM_EPI_F32, out=out, out_rows=rows)
    ref = torch.full((n_out, N), -3.0, device=cuda_device)
    ref[dst] = acc[keep]
    assert (out - ref).abs().max().item() <= 1e-3 * ref.abs().max().item() + 1e-3
    # residual add
    x0 = torch.randn(n_out, N, generator=g).to(cuda_device)
    x = x0.clone()
    ops.gemm_bf16(a, b, bias, epilogue=ops.SSAM_EPI_ADD_F32, out=x, out_rows=rows)
    ref = x0.clone()
    ref[dst] += acc[keep]
    assert (x - ref).abs().max().item() <= 1e-3 * ref.abs().max().item() + 1e-3
    assert ops.device_error() == 0
