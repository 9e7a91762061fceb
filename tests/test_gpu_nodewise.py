"""Fused node-wise kernels against the stand-in modules' own PyTorch definitions on the GPU
(fp32): forward values and input gradients."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


@pytest.mark.parametrize("N,C", [(1, 64), (333, 128), (4000, 128), (50, 256), (17, 32)])
def test_rms_norm_sh_matches_module(N, C):
    from flash_uma_b200 import ops
    from flash_uma_b200.linear import check_errors
    from flash_uma_b200.nodewise import EquivariantRMSNormSH
    g = torch.Generator().manual_seed(N * C)
    norm = EquivariantRMSNormSH(C)
    with torch.no_grad():
        norm.affine_weight.copy_(torch.rand(3, C, generator=g) + 0.5)
        norm.affine_bias.copy_(torch.randn(C, generator=g))
    norm = norm.to(DEV)
    x = (torch.randn(N, 9, C, generator=g) * torch.rand(N, 1, 1, generator=g) * 3 + 0.5).to(DEV)
    r = torch.randn(N, 9, C, generator=g).to(DEV)
    xa, xb = x.clone().requires_grad_(True), x.clone().requires_grad_(True)
    ya, yb = norm(xa), ops.rms_norm_sh(xb, norm)
    (ga,) = torch.autograd.grad((ya * r).sum(), xa)
    (gb,) = torch.autograd.grad((yb * r).sum(), xb)
    torch.cuda.synchronize()
    check_errors()
    assert (ya - yb).abs().max() <= 2e-6 * (1 + ya.abs().max())
    assert (ga - gb).abs().max() <= 1e-5 * (1 + ga.abs().max())


# tolerance relative to the largest value: fp32-accuracy modes (three fp16 products, or the
# batched fp32 GEMMs of the TF32 modes run with TF32 off) and the single-product mode
_ATOL = {"f16x3": 2e-5, "tf32x3": 2e-5, "f16": 4e-3}


@pytest.mark.parametrize("mode", ["f16x3", "f16", "tf32x3"])
@pytest.mark.parametrize("N,C,H", [(1, 64, 64), (333, 128, 128), (4000, 128, 128), (70, 64, 96)])
def test_atomwise_residual_matches_module(N, C, H, mode):
    from flash_uma_b200 import ops
    from flash_uma_b200.linear import check_errors
    from flash_uma_b200.nodewise import SpectralAtomwise
    g = torch.Generator().manual_seed(N + C + H)
    aw = SpectralAtomwise(C, H)
    with torch.no_grad():
        for p in aw.parameters():
            p.copy_(torch.randn(p.shape, generator=g) / (p.shape[-1] ** 0.5))
    aw = aw.to(DEV)
    xn = torch.randn(N, 9, C, generator=g).to(DEV)
    xm = torch.randn(N, 9, C, generator=g).to(DEV)
    r = torch.randn(N, 9, C, generator=g).to(DEV)
    a = [xn.clone().requires_grad_(True), xm.clone().requires_grad_(True)]
    b = [xn.clone().requires_grad_(True), xm.clone().requires_grad_(True)]
    ya = aw(a[0]) + a[1]
    yb = ops.atomwise_residual(aw, b[0], b[1], mode)
    ga = torch.autograd.grad((ya * r).sum(), a)
    gb = torch.autograd.grad((yb * r).sum(), b)
    torch.cuda.synchronize()
    check_errors()
    tol = _ATOL[mode]
    assert (ya - yb).abs().max() <= tol * (1 + ya.abs().max())
    for u, v in zip(ga, gb):
        assert (u - v).abs().max() <= tol * (1 + u.abs().max())
