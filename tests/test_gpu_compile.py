"""The ops under ``torch.compile``, as the reference publishes its timings (``readme.md:15,70``:
``torch.compile(model, dynamic=True)``).

* ``torch.library.opcheck`` on each ``fuma::`` custom operator: schema, fake (meta) kernel
  against the real one, autograd registration, dynamic-shape tracing.
* a reference-style message-passing layer written with the six ops and plain ``F.linear``
  compiles with ``fullgraph=True, dynamic=True`` (no graph break in the ops) and matches eager
  execution, forward and backward, at two edge counts (one compiled graph).
* the drop-in backbone (``ZeroAllocBackbone``) under ``torch.compile(dynamic=True)`` gives the
  eager energy and forces on benchmark config 1.
"""
import copy

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


@pytest.fixture(autouse=True)
def _no_tf32():
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = old


def _inputs(N=40, E=300, C=16, B=8, seed=0):
    from make_golden import small_op_inputs
    I = small_op_inputs(seed=seed, C=C, B=B, N=N, E=E)
    return {k: (v.to(DEV) if isinstance(v, torch.Tensor) else v) for k, v in I.items()}


def test_opcheck_every_op():
    from flash_uma_b200 import ops
    I = _inputs()
    N, C = I["x"].shape[0], I["x"].shape[2]
    E = I["idx_i"].shape[0]
    g = ops.build_graph_csr(I["idx_i"], I["idx_j"], N)
    xe, wig, env = ops.precompute_geometry(I["pos"], I["Z"], I["idx_i"], I["idx_j"], I["shifts"], I["W_src"],
                                           I["W_tgt"], I["offset_g"], I["coeff_g"], I["cutoff"])
    rg = lambda t: t.detach().clone().requires_grad_(True)   # noqa: E731
    csr = (g.dst_row_ptr, g.dst_col, g.src_row_ptr, g.src_col)
    cases = [
        (torch.ops.fuma.precompute_geometry.default,
         (rg(I["pos"]), I["Z"], I["idx_i"], I["idx_j"], rg(I["shifts"]), I["W_src"], I["W_tgt"], I["offset_g"],
          float(I["coeff_g"]), float(I["cutoff"]), *csr)),
        (torch.ops.fuma.layer_norm_silu.default,
         (rg(torch.randn(E, 32, device=DEV)), torch.ones(32, device=DEV), torch.zeros(32, device=DEV), 1e-7)),
        (torch.ops.fuma.gather_wigner_split.default,
         (rg(I["x"]), I["idx_i"], I["idx_j"], rg(wig), rg(I["rad12"]), I["csd"], I["batch"], *csr)),
        (torch.ops.fuma.fused_gating_split.default,
         (rg(torch.randn(E, 5 * C, device=DEV)), rg(torch.randn(E, 4 * C, device=DEV)),
          rg(torch.randn(E, 2 * C, device=DEV)), C)),
        (torch.ops.fuma.rotate_scatter_split.default,
         (rg(torch.randn(E, 3 * C, device=DEV)), rg(torch.randn(E, 4 * C, device=DEV)),
          rg(torch.randn(E, 2 * C, device=DEV)), rg(wig), rg(env), rg(I["x"]), g.dst_row_ptr, g.dst_col, N)),
        (torch.ops.fuma.init_node_scatter.default,
         (rg(torch.randn(E, 3 * C, device=DEV)), rg(wig), rg(env), I["Z"], I["batch"], I["W_sphere"], I["csd"],
          g.dst_row_ptr, g.dst_col, N)),
    ]
    for op, args in cases:
        torch.library.opcheck(op, args)


def _ref_style_layer(x, xe, wig, env, ii, jj, rp, ci, csd, batch, W, C):
    """One layer in the reference's formulation (model.py:143-157 without the node-wise modules):
    the six ops for the fused stages and F.linear for the dense contractions."""
    from flash_uma_b200 import ops
    h = ops.layer_norm_silu(F.linear(xe, W["r1"]), W["g"], W["b"])
    rad = F.linear(h, W["r3"])
    X0, X1, X2 = ops.gather_wigner_split(x, ii, jj, wig, rad, csd, batch)
    Z0, Z1, Z2 = ops.fused_gating_split(F.linear(X0, W["c10"]), F.linear(X1, W["c11"]), F.linear(X2, W["c12"]), C)
    return ops.rotate_scatter_split(F.linear(Z0, W["c20"]), F.linear(Z1, W["c21"]), F.linear(Z2, W["c22"]), wig, env,
                                    x, jj, rp, ci, x.shape[0])


def test_reference_style_layer_compiles_fullgraph():
    from flash_uma_b200 import ops
    C, B = 16, 8
    gen = torch.Generator().manual_seed(3)
    r = lambda *s: (torch.randn(*s, generator=gen) / s[-1] ** 0.5).to(DEV)   # noqa: E731
    W = {"r1": r(C, B + 2 * C), "g": torch.ones(C, device=DEV), "b": torch.zeros(C, device=DEV), "r3": r(12 * C, C),
         "c10": r(5 * C, 6 * C), "c11": r(4 * C, 8 * C), "c12": r(2 * C, 4 * C), "c20": r(3 * C, 3 * C),
         "c21": r(4 * C, 4 * C), "c22": r(2 * C, 2 * C)}
    compiled = torch.compile(_ref_style_layer, fullgraph=True, dynamic=True)
    for E, seed in ((300, 0), (517, 1)):
        I = _inputs(E=E, seed=seed)
        N = I["x"].shape[0]
        jj_sorted, order = torch.sort(I["idx_j"], stable=True)
        ii, jj = I["idx_i"][order], jj_sorted
        g = ops.build_graph_csr(ii, jj, N)
        xe, wig, env = ops.precompute_geometry(I["pos"], I["Z"], ii, jj, I["shifts"][order], I["W_src"], I["W_tgt"],
                                               I["offset_g"], I["coeff_g"], I["cutoff"])
        outs = []
        for fn in (_ref_style_layer, compiled):
            x = I["x"].detach().clone().requires_grad_(True)
            y = fn(x, xe, wig, env, ii, jj, g.dst_row_ptr, g.dst_col, I["csd"], I["batch"], W, C)
            (gx,) = torch.autograd.grad(y, [x], torch.ones_like(y))
            outs.append((y.detach(), gx))
        torch.testing.assert_close(outs[1][0], outs[0][0], rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(outs[1][1], outs[0][1], rtol=1e-5, atol=1e-5)


def test_backbone_under_torch_compile_matches_eager():
    """The drop-in backbone wrapped as the reference's users wrap theirs."""
    from flash_uma_b200.predict import Predictor
    from flash_uma_b200.synthetic import SyntheticESCNMDBackbone, make_energy_head
    from flash_uma_b200.systems import config1_system, to_graph
    from flash_uma_b200.wrapper import ZeroAllocBackbone
    data = to_graph([config1_system()]).to(DEV)
    off = SyntheticESCNMDBackbone(seed=0).to(DEV)
    head = make_energy_head(128, 128, seed=1).to(DEV)
    bb = ZeroAllocBackbone(off)
    eager = Predictor(bb, head)(data)
    comp = Predictor(torch.compile(bb, dynamic=True), head)(data)
    torch.testing.assert_close(comp["energy"], eager["energy"], rtol=1e-6, atol=1e-5)
    torch.testing.assert_close(comp["forces"], eager["forces"], rtol=0, atol=1e-5)
