"""Row-packed f16x3 split outputs (``*_f16x3`` entry points, ``fuma_split_rows_f16``): the
packed rows decode (hi + lo * 2^-11) to the plain entry point's fp32 output within the
split's precision, and feed ``fuma_linear_f16x3`` (a_split=1) like the fp32 data itself."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def decode(p: torch.Tensor) -> torch.Tensor:
    """fp32 values of a row-packed split [M, W] tensor."""
    M, W = p.shape
    h = p.view(torch.float16).view(M, 2, W).float()
    return h[:, 0] + h[:, 1] / 2048.0


def _close(x, y):
    # 22-bit pair: relative 2^-22 of each value, absolute floor 2^-36
    assert ((x - y).abs() <= x.abs() * 2.0 ** -21 + 2.0 ** -35).all()


def test_split_rows_roundtrip_and_range_flag():
    from flash_uma_b200.linear import check_errors, split_rows
    x = torch.randn(1000, 200, device=DEV) * torch.logspace(-6, 4, 200, device=DEV)
    _close(x, decode(split_rows(x)))
    check_errors()
    x[5, 7] = -7.0e4
    split_rows(x)
    with pytest.raises(RuntimeError, match="fp16 range"):
        check_errors()


def test_gating_and_ln_silu_split_outputs():
    from flash_uma_b200 import _native as nat
    from flash_uma_b200._native import ptr
    from flash_uma_b200.linear import check_errors, error_flag
    E, C = 777, 64
    s = torch.cuda.current_stream().cuda_stream
    err = error_flag(DEV)
    Y = [torch.randn(E, k * C, device=DEV) for k in (5, 4, 2)]
    plain = [torch.empty(E, k * C, device=DEV) for k in (3, 4, 2)]
    packed = [torch.empty(E, k * C, device=DEV) for k in (3, 4, 2)]
    nat.call("fuma_gating_fwd", *[ptr(t) for t in Y], E, C, *[ptr(t) for t in plain], s)
    nat.call("fuma_gating_fwd_f16x3", *[ptr(t) for t in Y], E, C, *[ptr(t) for t in packed], 2, ptr(err), s)
    for a, b in zip(plain, packed):
        _close(a, decode(b))
    gZ = [torch.randn_like(t) for t in plain]
    plain = [torch.empty_like(t) for t in Y]
    packed = [torch.empty_like(t) for t in Y]
    nat.call("fuma_gating_bwd", *[ptr(t) for t in gZ], *[ptr(t) for t in Y], E, C, *[ptr(t) for t in plain], s)
    nat.call("fuma_gating_bwd_f16x3", *[ptr(t) for t in gZ], *[ptr(t) for t in Y], E, C, *[ptr(t) for t in packed],
             2, ptr(err), s)
    for a, b in zip(plain, packed):
        _close(a, decode(b))
    D = 128
    x = torch.randn(E, D, device=DEV)
    gam, bet = torch.rand(D, device=DEV) + 0.5, torch.randn(D, device=DEV)
    out, out_p = torch.empty_like(x), torch.empty_like(x)
    mean, rstd = torch.empty(E, device=DEV), torch.empty(E, device=DEV)
    nat.call("fuma_ln_silu_fwd", ptr(x), ptr(gam), ptr(bet), 1e-7, E, D, ptr(out), ptr(mean), ptr(rstd), s)
    nat.call("fuma_ln_silu_fwd_f16x3", ptr(x), ptr(gam), ptr(bet), 1e-7, E, D, ptr(out_p), ptr(mean), ptr(rstd),
             2, ptr(err), s)
    _close(out, decode(out_p))
    g = torch.randn_like(x)
    gx, gx_p = torch.empty_like(x), torch.empty_like(x)
    nat.call("fuma_ln_silu_bwd", ptr(x), ptr(gam), ptr(bet), ptr(mean), ptr(rstd), ptr(g), E, D, ptr(gx), s)
    nat.call("fuma_ln_silu_bwd_f16x3", ptr(x), ptr(gam), ptr(bet), ptr(mean), ptr(rstd), ptr(g), E, D, ptr(gx_p),
             2, ptr(err), s)
    _close(gx, decode(gx_p))
    torch.cuda.synchronize()
    check_errors()


@pytest.mark.parametrize("M,N,K", [(1000, 128, 320), (777, 640, 768), (129, 256, 512), (5000, 1536, 128)])
def test_presplit_gemm_matches_fp32_operand(M, N, K):
    from flash_uma_b200.linear import FrozenLinear, _gemm16, check_errors, split_rows
    g = torch.Generator().manual_seed(M + K)
    W = torch.randn(N, K, generator=g) / K ** 0.5
    b = torch.randn(N, generator=g)
    x = torch.randn(M, K, generator=g)
    lin = FrozenLinear(W, b, mode="f16x3").to(DEV)
    lin.prepare()
    xd = x.to(DEV)
    y_pre = _gemm16(split_rows(xd), lin.w16, lin.bias_p, K)
    y_in = lin(xd)
    torch.cuda.synchronize()
    check_errors()
    assert torch.equal(y_pre, y_in)     # the same split values, the same products, the same order
    y_ref = x.double() @ W.double().t() + b.double()
    assert (y_pre.cpu().double() - y_ref).abs().max() <= (2e-6 + 1e-8 * K) * y_ref.abs().max()


def test_hi_only_split_outputs():
    """parts = 1 (the single-product mode's operands): the hi halves are those of parts = 2, bit
    for bit, and the lo halves of the rows are not written."""
    from flash_uma_b200 import _native as nat
    from flash_uma_b200._native import ptr
    from flash_uma_b200.linear import check_errors, error_flag
    E, C = 513, 64
    s = torch.cuda.current_stream().cuda_stream
    err = error_flag(DEV)
    Y = [torch.randn(E, k * C, device=DEV) for k in (5, 4, 2)]
    both = [torch.empty(E, k * C, device=DEV) for k in (3, 4, 2)]
    hi = [torch.full((E, k * C), 7.0, device=DEV) for k in (3, 4, 2)]
    nat.call("fuma_gating_fwd_f16x3", *[ptr(t) for t in Y], E, C, *[ptr(t) for t in both], 2, ptr(err), s)
    nat.call("fuma_gating_fwd_f16x3", *[ptr(t) for t in Y], E, C, *[ptr(t) for t in hi], 1, ptr(err), s)
    D = 128
    x = torch.randn(E, D, device=DEV)
    gam, bet = torch.rand(D, device=DEV) + 0.5, torch.randn(D, device=DEV)
    mean, rstd = torch.empty(E, device=DEV), torch.empty(E, device=DEV)
    o2, o1 = torch.empty_like(x), torch.full_like(x, 7.0)
    nat.call("fuma_ln_silu_fwd_f16x3", ptr(x), ptr(gam), ptr(bet), 1e-7, E, D, ptr(o2), ptr(mean), ptr(rstd), 2,
             ptr(err), s)
    nat.call("fuma_ln_silu_fwd_f16x3", ptr(x), ptr(gam), ptr(bet), 1e-7, E, D, ptr(o1), ptr(mean), ptr(rstd), 1,
             ptr(err), s)
    torch.cuda.synchronize()
    check_errors()
    for a, b in zip(both + [o2], hi + [o1]):
        W = a.shape[1]
        a16, b16 = a.view(torch.int16).view(a.shape[0], 2 * W), b.view(torch.int16).view(b.shape[0], 2 * W)
        assert torch.equal(a16[:, :W], b16[:, :W])                  # hi halves
        assert (b.view(b.shape[0], W)[:, W // 2:] == 7.0).all()     # lo halves untouched
