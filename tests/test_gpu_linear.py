"""tcgen05 GEMM (``fuma_linear``) vs fp64 torch matmul: forward and input gradient.

3xTF32 bound: max error <= (2e-6 + 1e-8 K) of the output's max magnitude. The K term is
the tensor core's fp32 accumulation, which truncates (~0.4 ulp toward zero per MMA
instruction of K=8, measured on B200: 1.1e-6 at K=128, 8e-6 at K=1024). Single-pass
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


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_linear_tf32x3_forward_backward(M, N, K):
    from flash_uma_b200.linear import check_errors
    W, b, lin = _lin(N, K, True, "tf32x3", M + N + K)
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


def test_linear_strided_input_and_empty():
    W, b, lin = _lin(128, 64, True, "tf32x3", 3)
    x = torch.randn(300, 320, generator=torch.Generator().manual_seed(2))
    xs = x.to(DEV)[:, :64]                      # row stride 320, view of a wider tensor
    y = lin(xs)
    y_ref = x[:, :64].double() @ W.double().t() + b.double()
    assert (y.cpu().double() - y_ref).abs().max() <= tol(64) * y_ref.abs().max()
    assert lin(torch.empty(0, 64, device=DEV)).shape == (0, 128)


def test_linear_deterministic():
    W, b, lin = _lin(512, 1024, False, "tf32x3", 4)
    x = torch.randn(5000, 1024, device=DEV)
    assert torch.equal(lin(x), lin(x))
