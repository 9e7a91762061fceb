"""tcgen05 GEMMs (``fuma_linear_f16x3``, ``fuma_linear``) vs fp64 torch matmul: forward and
input gradient.

f16x3 and 3xTF32 bound: max error <= (2e-6 + 1e-8 K) of the output's max magnitude. The K
term is the tensor core's fp32 accumulation, which truncates (~0.4 ulp toward zero per MMA
instruction, measured on B200 for 3xTF32: 1.1e-6 at K=128, 8e-6 at K=1024; f16x3 has one
truncating add per K=16 on the full-size accumulator instead of three per K=8). Single-pass
TF32 must be within TF32 rounding (2e-3)."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")

SHAPES = [  # (M, N, K): the model's forward and input-gradient shapes, ragged M, small widths, ragged K
    (1000, 128, 320), (4097, 1536, 128), (777, 640, 768), (130, 512, 1024), (129, 256, 512),
    (300, 384, 384), (1, 128, 128), (128, 64, 64), (513, 320, 128), (4096, 1024, 512), (2000, 128, 1536),
    (300, 80, 96), (257, 48, 40), (100, 16, 12), (65, 32, 160),
]


def tol(K):
    return 2e-6 + 1e-8 * K


def _lin(N, K, bias, mode, seed):
    from flash_uma_b200.linear import FrozenLinear
    g = torch.Generator().manual_seed(seed)
    W = torch.randn(N, K, generator=g) / K ** 0.5
    b = torch.randn(N, generator=g) if bias else None
    return W, b, FrozenLinear(W, b, mode=mode).to(DEV)


@pytest.mark.parametrize("mode", ["f16x3", "tf32x3"])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_linear_split_forward_backward(M, N, K, mode):
    from flash_uma_b200.linear import check_errors
    W, b, lin = _lin(N, K, True, mode, M + N + K)
    g = torch.Generator().manual_seed(K)
    x = torch.randn(M, K, generator=g)
    gy = torch.randn(M, N, generator=g)
    xd = x.to(DEV).requires_grad_(True)
    y = lin(xd)
    (gx,) = torch.autograd.grad(y, [xd], gy.to(DEV))
    torch.cuda.synchronize()
    check_errors()
    y_ref = x.double() @ W.double().t() + b.double()
    gx_ref = gy.double() @ W.double()
    assert (y.cpu().double() - y_ref).abs().max() <= tol(K) * y_ref.abs().max()
    assert (gx.cpu().double() - gx_ref).abs().max() <= tol(N) * gx_ref.abs().max()


@pytest.mark.parametrize("M,N,K", SHAPES[:4])
def test_linear_tf32(M, N, K):
    W, b, lin = _lin(N, K, False, "tf32", 7)
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(1))
    y = lin(x.to(DEV))
    y_ref = x.double() @ W.double().t()
    err = (y.cpu().double() - y_ref).abs().max() / y_ref.abs().max()
    assert err <= 2e-3
    assert err >= 1e-7   # it really is a reduced-precision product


@pytest.mark.parametrize("mode", ["f16x3", "tf32x3"])
def test_linear_strided_input_and_empty(mode):
    W, b, lin = _lin(128, 64, True, mode, 3)
    x = torch.randn(300, 320, generator=torch.Generator().manual_seed(2))
    xs = x.to(DEV)[:, :64]                      # row stride 320, view of a wider tensor
    y = lin(xs)
    y_ref = x[:, :64].double() @ W.double().t() + b.double()
    assert (y.cpu().double() - y_ref).abs().max() <= tol(64) * y_ref.abs().max()
    assert lin(torch.empty(0, 64, device=DEV)).shape == (0, 128)


@pytest.mark.parametrize("mode", ["f16x3", "tf32x3"])
def test_linear_deterministic(mode):
    W, b, lin = _lin(512, 1024, False, mode, 4)
    x = torch.randn(5000, 1024, device=DEV)
    assert torch.equal(lin(x), lin(x))


def test_f16x3_wide_dynamic_range():
    """Activations across eight decades, and weights far beyond the fp16 range (taken care of by
    the power-of-two weight scale), keep fp32-level relative accuracy row by row. Below ~1e-4
    the split has an absolute floor instead (2^-36 per activation, from fp16 subnormals in the
    scaled residual), checked on rows down to 1e-9."""
    from flash_uma_b200.linear import FrozenLinear, check_errors
    g = torch.Generator().manual_seed(9)
    K = 512
    W = torch.randn(256, K, generator=g) * 1e5
    scales = torch.cat([torch.logspace(-4, 4, 600), torch.logspace(-9, -4, 100)])
    x = torch.randn(700, K, generator=g) * scales[:, None]
    lin = FrozenLinear(W, None, mode="f16x3").to(DEV)
    y = lin(x.to(DEV))
    torch.cuda.synchronize()
    check_errors()
    y_ref = x.double() @ W.double().t()
    err = (y.cpu().double() - y_ref).abs().max(1).values
    rel = err / y_ref.abs().max(1).values
    assert rel[:600].max() <= tol(K)
    floor = K * 2.0 ** -36 * W.abs().max().item()
    assert (err[600:] <= tol(K) * y_ref[600:].abs().max(1).values + floor).all()


def test_f16x3_out_of_range_input_is_reported():
    """A finite activation beyond the fp16 range cannot be split: the kernel records it and
    the error check raises (the tf32x3 mode handles such data)."""
    from flash_uma_b200.linear import FrozenLinear, check_errors, poll_errors, snapshot_errors
    W = torch.randn(128, 64, generator=torch.Generator().manual_seed(5))
    lin = FrozenLinear(W, None, mode="f16x3").to(DEV)
    x = torch.randn(300, 64, device=DEV)
    x[17, 3] = 1.0e5
    lin(x)
    snapshot_errors()
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="fp16 range"):
        poll_errors()
    check_errors()                       # the flag was cleared by the raise
    lin(torch.randn(300, 64, device=DEV))
    check_errors()


@pytest.mark.parametrize("M,N,K", SHAPES[:11])
def test_linear_f16_single_product(M, N, K):
    """``fuma_linear_f16`` (the "f16" mode): C = fp16(A) . fp16(W s)^T / s, fp32 accumulation.
    Against fp64 arithmetic on the same fp16-rounded operands the only error is the tensor core's
    accumulation (bound as above); against the exact fp32 product it is within fp16 rounding
    (the TF32 accuracy class, 2e-3)."""
    from flash_uma_b200.linear import check_errors
    W, b, lin = _lin(N, K, True, "f16", M + 3 * N + K)
    g = torch.Generator().manual_seed(K + 1)
    x = torch.randn(M, K, generator=g)
    gy = torch.randn(M, N, generator=g)
    xd = x.to(DEV).requires_grad_(True)
    y = lin(xd)
    (gx,) = torch.autograd.grad(y, [xd], gy.to(DEV))
    torch.cuda.synchronize()
    check_errors()
    hi, _, inv, x1 = lin.w16
    assert x1
    w_r = hi[:N, :K].double().cpu() * inv
    y_rnd = x.half().double() @ w_r.t() + b.double()
    assert (y.cpu().double() - y_rnd).abs().max() <= tol(K) * y_rnd.abs().max()
    y_ref = x.double() @ W.double().t() + b.double()
    assert (y.cpu().double() - y_ref).abs().max() <= 2e-3 * y_ref.abs().max()
    gx_ref = gy.double() @ W.double()
    assert (gx.cpu().double() - gx_ref).abs().max() <= 2e-3 * gx_ref.abs().max()


@pytest.mark.parametrize("M,N,K", [(120000, 640, 768), (777, 640, 768), (300, 384, 384), (513, 128, 320),
                                   (4097, 1536, 128), (1, 128, 128), (2000, 128, 1536), (257, 384, 96)])
def test_linear_f16x3_transposed_tiles(M, N, K, monkeypatch):
    """The transposed 128 x 256 tiles (FUMA_GEMM_T=1, output features on the MMA's M side) on the
    pre-split operands give the same products as the row-major tiles: within the f16x3 bound of
    fp64, ragged edge counts included."""
    from flash_uma_b200.linear import _gemm16, _split16, check_errors, split_rows
    g = torch.Generator().manual_seed(M + N + K)
    W = (torch.randn(N, K, generator=g) / K ** 0.5).to(DEV)
    b = torch.randn(N, generator=g).to(DEV)
    x = torch.randn(M, K, generator=g).to(DEV)
    w16 = _split16(torch.nn.functional.pad(W, (0, (K + 7) // 8 * 8 - K)))
    xp = split_rows(x)
    monkeypatch.setenv("FUMA_GEMM_T", "0")
    y0 = _gemm16(xp, w16, b, K)
    monkeypatch.setenv("FUMA_GEMM_T", "1")
    y1 = _gemm16(xp, w16, b, K)
    torch.cuda.synchronize()
    check_errors()
    ref = x.double() @ W.double().t() + b.double()
    for y in (y0, y1):
        assert (y.double() - ref).abs().max() <= tol(K) * ref.abs().max()


@pytest.mark.parametrize("half", [False, True])
@pytest.mark.parametrize("M,N,K", [(120000, 640, 768), (777, 640, 768), (300, 384, 384), (513, 128, 320),
                                   (1, 128, 128), (257, 384, 96), (4097, 1536, 128)])
def test_linear_f16_transposed_tiles(M, N, K, half, monkeypatch):
    """Single-product mode on the transposed 128 x 256 tiles (two TMEM accumulators, fp32 or fp16
    results) and on the row-major tiles: both within the accumulation bound of fp64 arithmetic on
    the same fp16-rounded operands, plus one fp16 rounding of the result when it is stored as
    fp16 (relative 2^-11)."""
    from flash_uma_b200.linear import _gemm16, check_errors, split_rows
    W, b, lin = _lin(N, K, True, "f16", M + 5 * N + K)
    lin.prepare()
    g = torch.Generator().manual_seed(M + K)
    x = torch.randn(M, K, generator=g)
    xp = split_rows(x.to(DEV))
    ys = []
    for t in ("0", "1"):
        monkeypatch.setenv("FUMA_GEMM_T", t)
        ys.append(_gemm16(xp, lin.w16, lin.bias_p, K, out_half=half))
    torch.cuda.synchronize()
    check_errors()
    hi, _, inv, x1 = lin.w16
    assert x1
    ref = x.half().double() @ (hi[:N, :K].double().cpu() * inv).t() + b.double()
    for y in ys:
        assert y.dtype == (torch.float16 if half else torch.float32) and y.shape == (M, N)
        err = (y[:, :N].cpu().double() - ref).abs()
        bound = tol(K) * ref.abs().max() + (2.0 ** -11 * ref.abs() if half else 0.0)
        assert bool((err <= bound).all())
