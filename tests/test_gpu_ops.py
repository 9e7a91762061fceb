"""CUDA ops vs the CPU oracle (fp64 autograd) and vs the reference's golden vectors.

Tolerances: the kernels compute in fp32 (the scatters accumulate in fp64), the oracle
in fp64, so forward and backward agree to ~1e-6 relative; we assert 2e-5 relative to
the tensor's max magnitude (5e-5 for reductions over C such as g_wigner)."""
import os

import numpy as np
import pytest
import torch

from make_golden import csr_of, small_op_inputs
from oracle import ops as oops

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def rel(a, b):
    a = a.detach().double().cpu(); b = b.detach().double().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp(min=1.0)).item()


@pytest.fixture(scope="module")
def fops():
    from flash_uma_b200 import _native, ops
    _native.load()
    return ops


def rand_graph(N, E, seed, C=16, B=8, nsys=2):
    I = small_op_inputs(seed=seed, C=C, B=B, N=N, E=E)
    return I


def to_dev(*ts):
    return [t.to(DEV) for t in ts]


# ---------------------------------------------------------------------------- geometry
@pytest.mark.parametrize("seed,C,B,N,E", [(0, 16, 8, 40, 320), (1, 128, 64, 300, 5000), (2, 32, 12, 50, 7)])
def test_geometry(fops, seed, C, B, N, E):
    I = small_op_inputs(seed=seed, C=C, B=B, N=N, E=E)
    args = [I[k] for k in ("pos", "Z", "idx_i", "idx_j", "shifts", "W_src", "W_tgt", "offset_g")]
    pos, sh = I["pos"].double().requires_grad_(True), I["shifts"].double().requires_grad_(True)
    xe, wig, env = oops.precompute_geometry(pos, I["Z"], I["idx_i"], I["idx_j"], sh, I["W_src"].double(),
                                            I["W_tgt"].double(), I["offset_g"].double(), I["coeff_g"], I["cutoff"])
    gp, gs = torch.autograd.grad([xe, wig, env], [pos, sh], [I["g_xe"].double(), I["g_wig"].double(),
                                                             I["g_env"].double()])
    d = to_dev(*args)
    d[0].requires_grad_(True); d[4].requires_grad_(True)
    xe_c, wig_c, env_c = fops.precompute_geometry(*d, I["coeff_g"], I["cutoff"])
    assert rel(xe_c, xe) < 2e-5 and rel(wig_c, wig) < 2e-5 and rel(env_c, env) < 2e-5
    gp_c, gs_c = torch.autograd.grad([xe_c, wig_c, env_c], [d[0], d[4]],
                                     to_dev(I["g_xe"], I["g_wig"], I["g_env"]))
    assert rel(gs_c, gs) < 5e-5, rel(gs_c, gs)
    assert rel(gp_c, gp) < 5e-5, rel(gp_c, gp)


def test_geometry_matches_reference_golden(fops):
    g = dict(np.load(os.path.join(GOLD, "ops_small.npz")))
    I = small_op_inputs()
    d = to_dev(*[I[k] for k in ("pos", "Z", "idx_i", "idx_j", "shifts", "W_src", "W_tgt", "offset_g")])
    d[0].requires_grad_(True); d[4].requires_grad_(True)
    xe, wig, env = fops.precompute_geometry(*d, I["coeff_g"], I["cutoff"])
    np.testing.assert_allclose(xe.detach().cpu().numpy(), g["geom_xe"], atol=2e-6, rtol=1e-5)
    np.testing.assert_allclose(wig.detach().cpu().numpy(), g["geom_wig"], atol=3e-6)
    # env = 1 - 21u^5 + 35u^6 - 15u^7 cancels near the cutoff: fp32 terms of size ~70 leave an
    # absolute error of a few 1e-6 (FMA contraction differs between GPU and CPU)
    np.testing.assert_allclose(env.detach().cpu().numpy(), g["geom_env"], atol=1e-5)
    gp, gs = torch.autograd.grad([xe, wig, env], [d[0], d[4]], to_dev(I["g_xe"], I["g_wig"], I["g_env"]))
    np.testing.assert_allclose(gs.cpu().numpy(), g["geom_gshifts"], atol=2e-5 * np.abs(g["geom_gshifts"]).max())
    np.testing.assert_allclose(gp.cpu().numpy(), g["geom_gpos"], atol=5e-5 * np.abs(g["geom_gpos"]).max())


# ---------------------------------------------------------------------------- LN-SiLU
@pytest.mark.parametrize("M,D", [(64, 32), (1000, 128), (37, 1536), (5, 4), (0, 128)])
def test_ln_silu(fops, M, D):
    gen = torch.Generator().manual_seed(M + D)
    x = torch.randn(M, D, generator=gen) * 2 + 0.5
    gm = 1 + 0.1 * torch.randn(D, generator=gen); bt = 0.1 * torch.randn(D, generator=gen)
    go = torch.randn(M, D, generator=gen)
    xd = x.double().requires_grad_(True)
    y = oops.layer_norm_silu(xd, gm.double(), bt.double())
    xc = x.to(DEV).requires_grad_(True)
    yc = fops.layer_norm_silu(xc, gm.to(DEV), bt.to(DEV))
    if M == 0:
        assert yc.shape == (0, D)
        return
    assert rel(yc, y) < 2e-5
    (gx,) = torch.autograd.grad(y, [xd], go.double())
    (gxc,) = torch.autograd.grad(yc, [xc], go.to(DEV))
    assert rel(gxc, gx) < 5e-5


# ---------------------------------------------------------------------------- gather
@pytest.mark.parametrize("seed,C,N,E", [(0, 16, 40, 320), (1, 128, 200, 4000), (2, 144, 30, 200), (3, 32, 50, 0)])
def test_gather(fops, seed, C, N, E):
    I = small_op_inputs(seed=seed, C=C, N=N, E=max(E, 1))
    if E == 0:
        I["idx_i"] = I["idx_i"][:0]; I["idx_j"] = I["idx_j"][:0]; I["rad12"] = I["rad12"][:0]
        for k in ("g_X0", "g_X1", "g_X2"):
            I[k] = I[k][:0]
    wig = oops.precompute_geometry(I["pos"], I["Z"], I["idx_i"], I["idx_j"], I["shifts"][:E], I["W_src"],
                                   I["W_tgt"], I["offset_g"], I["coeff_g"], I["cutoff"])[1] if E else torch.zeros(0, 34)
    x = I["x"].double().requires_grad_(True); w = wig.double().requires_grad_(True)
    r = I["rad12"].double().requires_grad_(True)
    X = oops.gather_wigner_split(x, I["idx_i"], I["idx_j"], w, r, I["csd"].double(), I["batch"])
    xd, wd, rd = to_dev(I["x"], wig, I["rad12"])
    for t in (xd, wd, rd):
        t.requires_grad_(True)
    Xc = fops.gather_wigner_split(xd, *to_dev(I["idx_i"], I["idx_j"]), wd, rd, *to_dev(I["csd"], I["batch"]))
    for a, b in zip(Xc, X):
        assert a.shape == b.shape
        if E:
            assert rel(a, b) < 2e-5
    gouts = [I["g_X0"], I["g_X1"], I["g_X2"]]
    g = torch.autograd.grad(list(X), [x, w, r], [t.double() for t in gouts], allow_unused=True)
    gc = torch.autograd.grad(list(Xc), [xd, wd, rd], to_dev(*gouts), allow_unused=True)
    assert rel(gc[0], g[0] if g[0] is not None else torch.zeros_like(x)) < 5e-5
    if E:
        assert rel(gc[1], g[1]) < 5e-5 and rel(gc[2], g[2]) < 5e-5


def test_gather_matches_reference_golden(fops):
    g = dict(np.load(os.path.join(GOLD, "ops_small.npz")))
    I = small_op_inputs()
    wig = torch.tensor(g["geom_wig"])
    xd, wd, rd = to_dev(I["x"], wig, I["rad12"])
    for t in (xd, wd, rd):
        t.requires_grad_(True)
    X = fops.gather_wigner_split(xd, *to_dev(I["idx_i"], I["idx_j"]), wd, rd, *to_dev(I["csd"], I["batch"]))
    for k, t in enumerate(X):
        np.testing.assert_allclose(t.detach().cpu().numpy(), g[f"gat_X{k}"], atol=1e-5, rtol=1e-5)
    gx, gw, gr = torch.autograd.grad(list(X), [xd, wd, rd], to_dev(I["g_X0"], I["g_X1"], I["g_X2"]))
    np.testing.assert_allclose(gx.cpu().numpy(), g["gat_gx"], atol=5e-5, rtol=1e-5)
    np.testing.assert_allclose(gr.cpu().numpy(), g["gat_grad"], atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(gw.cpu().numpy(), g["gat_gwig"], atol=1e-4, rtol=1e-5)


# ---------------------------------------------------------------------------- gating
@pytest.mark.parametrize("C,E", [(16, 320), (128, 3000), (36, 1)])
def test_gating(fops, C, E):
    gen = torch.Generator().manual_seed(C * 7 + E)
    Y = [torch.randn(E, m * C, generator=gen) * 2 for m in (5, 4, 2)]
    G = [torch.randn(E, m * C, generator=gen) for m in (3, 4, 2)]
    Yd = [y.double().requires_grad_(True) for y in Y]
    Z = oops.fused_gating_split(*Yd, C)
    Yc = [y.to(DEV).requires_grad_(True) for y in Y]
    Zc = fops.fused_gating_split(*Yc, C)
    for a, b in zip(Zc, Z):
        assert rel(a, b) < 2e-5
    g = torch.autograd.grad(list(Z), Yd, [t.double() for t in G])
    gc = torch.autograd.grad(list(Zc), Yc, to_dev(*G))
    for a, b in zip(gc, g):
        assert rel(a, b) < 2e-5


# ---------------------------------------------------------------------------- rotate scatter
@pytest.mark.parametrize("seed,C,N,E", [(0, 16, 40, 320), (1, 128, 300, 6000), (2, 144, 25, 150), (3, 16, 10, 0)])
def test_rotate_scatter(fops, seed, C, N, E):
    I = small_op_inputs(seed=seed, C=C, N=N, E=max(E, 1))
    ii, jj = I["idx_i"][:E], I["idx_j"][:E]
    wig, env = oops.precompute_geometry(I["pos"], I["Z"], ii, jj, I["shifts"][:E], I["W_src"], I["W_tgt"],
                                        I["offset_g"], I["coeff_g"], I["cutoff"])[1:]
    rp, ci = csr_of(jj, N)
    Zo = [I[k][:E] for k in ("Zo0", "Zo1", "Zo2")]
    Zd = [z.double().requires_grad_(True) for z in Zo]
    wd, ed, xd = wig.double().requires_grad_(True), env.double().requires_grad_(True), I["x"].double().requires_grad_(True)
    out = oops.rotate_scatter_split(*Zd, wd, ed, xd, jj, rp, ci, N)
    Zc = [z.to(DEV).requires_grad_(True) for z in Zo]
    wc, ec, xc = [t.to(DEV).requires_grad_(True) for t in (wig, env, I["x"])]
    outc = fops.rotate_scatter_split(*Zc, wc, ec, xc, jj.to(DEV), rp.to(DEV), ci.to(DEV), N)
    assert rel(outc, out) < 2e-6
    g = torch.autograd.grad(out, Zd + [wd, ed, xd], I["g_node"].double(), allow_unused=True)
    gc = torch.autograd.grad(outc, Zc + [wc, ec, xc], I["g_node"].to(DEV), allow_unused=True)
    for a, b in zip(gc, g):
        if b is None or b.numel() == 0:
            continue
        assert rel(a, b) < 5e-5


def test_rotate_scatter_matches_reference_golden_and_is_deterministic(fops):
    g = dict(np.load(os.path.join(GOLD, "ops_small.npz")))
    I = small_op_inputs()
    rp, ci = csr_of(I["idx_j"], I["N"])
    args = to_dev(I["Zo0"], I["Zo1"], I["Zo2"], torch.tensor(g["geom_wig"]), torch.tensor(g["geom_env"]), I["x"])
    rest = to_dev(I["idx_j"], rp, ci)
    o1 = fops.rotate_scatter_split(*args, *rest, I["N"])
    o2 = fops.rotate_scatter_split(*args, *rest, I["N"])
    assert torch.equal(o1, o2)
    np.testing.assert_allclose(o1.cpu().numpy(), g["sc_out"], atol=1e-5, rtol=1e-6)


# ---------------------------------------------------------------------------- init scatter
@pytest.mark.parametrize("seed,C,N,E", [(0, 16, 40, 320), (1, 128, 300, 6000), (2, 144, 25, 150)])
def test_init_scatter(fops, seed, C, N, E):
    I = small_op_inputs(seed=seed, C=C, N=N, E=E)
    wig, env = oops.precompute_geometry(I["pos"], I["Z"], I["idx_i"], I["idx_j"], I["shifts"], I["W_src"],
                                        I["W_tgt"], I["offset_g"], I["coeff_g"], I["cutoff"])[1:]
    rp, ci = csr_of(I["idx_j"], N)
    rd, wd, ed = I["rad3"].double().requires_grad_(True), wig.double().requires_grad_(True), env.double().requires_grad_(True)
    out = oops.init_node_scatter(rd, wd, ed, I["Z"], I["batch"], I["W_sphere"].double(), I["csd"].double(),
                                 I["idx_j"], rp, ci, N)
    rc, wc, ec = [t.to(DEV).requires_grad_(True) for t in (I["rad3"], wig, env)]
    outc = fops.init_node_scatter(rc, wc, ec, *to_dev(I["Z"], I["batch"], I["W_sphere"], I["csd"], I["idx_j"], rp, ci), N)
    assert rel(outc, out) < 2e-6
    g = torch.autograd.grad(out, [rd, wd, ed], I["g_node"].double())
    gc = torch.autograd.grad(outc, [rc, wc, ec], I["g_node"].to(DEV))
    for a, b in zip(gc, g):
        assert rel(a, b) < 5e-5


def test_backward_is_deterministic(fops):
    """Gather backward (no atomics) and geometry backward give bitwise-identical results."""
    I = small_op_inputs(seed=5, C=128, N=200, E=6000)
    d = to_dev(*[I[k] for k in ("pos", "Z", "idx_i", "idx_j", "shifts", "W_src", "W_tgt", "offset_g")])
    outs = []
    for _ in range(2):
        pos = d[0].clone().requires_grad_(True)
        xe, wig, env = fops.precompute_geometry(pos, *d[1:], I["coeff_g"], I["cutoff"])
        x = I["x"].to(DEV).requires_grad_(True)
        X = fops.gather_wigner_split(x, d[2], d[3], wig, I["rad12"].to(DEV), *to_dev(I["csd"], I["batch"]))
        loss = sum((t * t).sum() for t in X) + (xe[:, :8] ** 2).sum()
        gp, gx = torch.autograd.grad(loss, [pos, x])
        outs.append((gp, gx))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])


def test_errors_are_raised_not_silent(fops):
    x = torch.randn(4, 6, device=DEV)   # D=6 not a multiple of 4
    with pytest.raises(RuntimeError, match="multiple of 4"):
        fops.layer_norm_silu(x, torch.ones(6, device=DEV), torch.zeros(6, device=DEV))
    with pytest.raises(TypeError):
        fops.layer_norm_silu(x.double()[:, :4], torch.ones(4, device=DEV), torch.zeros(4, device=DEV))
