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
    nat.call("fuma_gating_fwd_f16x3", *[ptr(t) for t in Y], E, C, *[ptr(t) for t in packed], 2, 0, ptr(err), s)
    for a, b in zip(plain, packed):
        _close(a, decode(b))
    gZ = [torch.randn_like(t) for t in plain]
    plain = [torch.empty_like(t) for t in Y]
    packed = [torch.empty_like(t) for t in Y]
    nat.call("fuma_gating_bwd", *[ptr(t) for t in gZ], *[ptr(t) for t in Y], E, C, *[ptr(t) for t in plain], s)
    nat.call("fuma_gating_bwd_f16x3", *[ptr(t) for t in gZ], *[ptr(t) for t in Y], E, C, *[ptr(t) for t in packed],
             2, 0, ptr(err), s)
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
    nat.call("fuma_gating_fwd_f16x3", *[ptr(t) for t in Y], E, C, *[ptr(t) for t in both], 2, 0, ptr(err), s)
    nat.call("fuma_gating_fwd_f16x3", *[ptr(t) for t in Y], E, C, *[ptr(t) for t in hi], 1, 0, ptr(err), s)
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


def test_fp16_activation_inputs():
    """act_half (the single-product mode's 16-bit storage of the radial, conv1 and conv2 results
    and of the input gradients the backward kernels read): gather, gating and rotate-scatter fed
    fp16 arrays give exactly what they give on the same values in fp32 (the kernels convert each
    value on load and compute in fp32)."""
    from flash_uma_b200 import _native as nat
    from flash_uma_b200 import ops
    from flash_uma_b200._native import ptr
    from flash_uma_b200.linear import check_errors, error_flag
    from make_golden import small_op_inputs
    I = small_op_inputs(seed=4, C=32, N=60, E=500)
    d = {k: (v.to(DEV) if isinstance(v, torch.Tensor) else v) for k, v in I.items()}
    N, E, C = d["x"].shape[0], d["idx_i"].shape[0], 32
    s = torch.cuda.current_stream().cuda_stream
    err = error_flag(DEV)
    g = ops.build_graph_csr(d["idx_i"], d["idx_j"], N)
    wig = ops.precompute_geometry(d["pos"], d["Z"], d["idx_i"], d["idx_j"], d["shifts"], d["W_src"], d["W_tgt"],
                                  d["offset_g"], d["coeff_g"], d["cutoff"])[1].detach()
    env = torch.rand(E, device=DEV)
    rad_h = torch.randn(E, 12 * C, device=DEV).half()
    Y_h = [torch.randn(E, k * C, device=DEV).half() for k in (5, 4, 2)]
    O_h = [torch.randn(E, k * C, device=DEV).half() for k in (3, 4, 2)]
    gX_h = [torch.randn(E, k * C, device=DEV).half() for k in (6, 8, 4)]
    gZ_h = [torch.randn(E, k * C, device=DEV).half() for k in (3, 4, 2)]
    gout = torch.randn(N, 9, C, device=DEV)

    def both(name, args_h, args_f, outs_shapes, tail_h, tail_f):
        res = []
        for args, tail in ((args_h, tail_h), (args_f, tail_f)):
            outs = [torch.full(sh, float("nan"), device=DEV) for sh in outs_shapes]
            nat.call(name, *args, *[ptr(o) for o in outs], *tail)
            res.append(outs)
        torch.cuda.synchronize()
        for a, b in zip(*res):
            assert torch.equal(a.view(torch.int32), b.view(torch.int32)), name

    f32 = lambda ts: [t.float() for t in ts]   # noqa: E731
    ep = [ptr(d["x"]), ptr(d["idx_i"]), ptr(d["idx_j"]), ptr(wig)]
    rf = rad_h.float()   # kept alive: the kernels read it after this line
    both("fuma_gather_fwd_f16x3", ep + [ptr(rad_h), ptr(d["csd"]), ptr(d["batch"]), N, E, C],
         ep + [ptr(rf), ptr(d["csd"]), ptr(d["batch"]), N, E, C],
         [(E, 6 * C), (E, 8 * C), (E, 4 * C)], [2, 1, ptr(err), s], [2, 0, ptr(err), s])
    csr = [ptr(g.dst_row_ptr), ptr(g.dst_col), ptr(g.src_row_ptr), ptr(g.src_col)]
    gXf = f32(gX_h)
    both("fuma_gather_bwd_f16x3", [ptr(t) for t in gX_h] + ep[:2] + [ptr(wig), ptr(rad_h), ptr(d["csd"]),
                                                                    ptr(d["batch"])] + csr + [N, E, C, None, 0],
         [ptr(t) for t in gXf] + ep[:2] + [ptr(wig), ptr(rf), ptr(d["csd"]), ptr(d["batch"])] + csr + [N, E, C, None, 0],
         [(N, 9, C), (E, 34), (E, 12 * C)], [2, 1, ptr(err), s], [2, 0, ptr(err), s])
    Yf = f32(Y_h)
    both("fuma_gating_fwd_f16x3", [ptr(t) for t in Y_h] + [E, C], [ptr(t) for t in Yf] + [E, C],
         [(E, 3 * C), (E, 4 * C), (E, 2 * C)], [2, 1, ptr(err), s], [2, 0, ptr(err), s])
    gZf = f32(gZ_h)
    both("fuma_gating_bwd_f16x3", [ptr(t) for t in gZ_h] + [ptr(t) for t in Y_h] + [E, C],
         [ptr(t) for t in gZf] + [ptr(t) for t in Yf] + [E, C],
         [(E, 5 * C), (E, 4 * C), (E, 2 * C)], [2, 1, ptr(err), s], [2, 0, ptr(err), s])
    Of = f32(O_h)
    rs = [ptr(wig), ptr(env), ptr(d["x"]), ptr(g.dst_row_ptr), ptr(g.dst_col), N, E, C]
    both("fuma_rotate_scatter_fwd_f16x3", [ptr(t) for t in O_h] + rs, [ptr(t) for t in Of] + rs, [(N, 9, C)],
         [1, s], [0, s])
    rsb = [ptr(wig), ptr(env), ptr(g.dst_row_ptr), ptr(g.dst_col), N, E, C]
    both("fuma_rotate_scatter_bwd_f16x3", [ptr(gout)] + [ptr(t) for t in O_h] + rsb,
         [ptr(gout)] + [ptr(t) for t in Of] + rsb, [(E, 3 * C), (E, 4 * C), (E, 2 * C), (E, 34), (E,)],
         [2, 1, ptr(err), s], [2, 0, ptr(err), s])
    check_errors()


def test_linear_f16_half_output():
    """fuma_linear_f16 with c_half: the fp32 result rounded once to fp16 (equal to the fp32
    output's fp16 rounding), and the range flag for results beyond the fp16 limit."""
    from flash_uma_b200.linear import FrozenLinear, _gemm16, check_errors, split_rows
    for M, N, K in ((1000, 512, 1024), (777, 640, 768), (129, 128, 128), (300, 48, 96)):
        g = torch.Generator().manual_seed(M + N)
        W = torch.randn(N, K, generator=g) / K ** 0.5
        b = torch.randn(N, generator=g)
        lin = FrozenLinear(W, b, mode="f16").to(DEV)
        lin.prepare()
        xp = split_rows(torch.randn(M, K, generator=g).to(DEV))
        y32 = _gemm16(xp, lin.w16, lin.bias_p, K)
        y16 = _gemm16(xp, lin.w16, lin.bias_p, K, out_half=True)
        torch.cuda.synchronize()
        assert y16.dtype == torch.float16 and y16.shape == (M, N)
        assert torch.equal(y16, y32[:, :N].half())
    check_errors()
