"""Pin the CPU oracle to golden vectors produced by the reference implementation itself
(``tests/golden/make_golden.py`` runs the reference's Triton ops on CPU)."""
import os

import numpy as np
import pytest
import torch

from make_golden import csr_of, small_op_inputs
from oracle import model as omodel
from oracle import ops as oops

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def gold():
    return dict(np.load(os.path.join(GOLD, "ops_small.npz")))


@pytest.fixture(scope="module")
def inp():
    return small_op_inputs()


def close(a, b, atol, rtol=0.0):
    a = a.detach().cpu().numpy() if isinstance(a, torch.Tensor) else a
    np.testing.assert_allclose(a, b, atol=atol, rtol=rtol)


def test_geometry_forward_backward(gold, inp):
    I = inp
    pos = I["pos"].clone().requires_grad_(True)
    sh = I["shifts"].clone().requires_grad_(True)
    xe, wig, env = oops.precompute_geometry(pos, I["Z"], I["idx_i"], I["idx_j"], sh, I["W_src"], I["W_tgt"],
                                            I["offset_g"], I["coeff_g"], I["cutoff"])
    close(xe, gold["geom_xe"], 2e-6, 1e-5)
    close(env, gold["geom_env"], 1e-6)
    close(wig, gold["geom_wig"], 3e-6)
    gp, gs = torch.autograd.grad([xe, wig, env], [pos, sh], [I["g_xe"], I["g_wig"], I["g_env"]])
    scale = np.abs(gold["geom_gshifts"]).max()
    close(gs, gold["geom_gshifts"], 2e-5 * scale)
    close(gp, gold["geom_gpos"], 5e-5 * np.abs(gold["geom_gpos"]).max())


def test_wigner_blocks_orthogonal(gold):
    w = torch.tensor(gold["geom_wig"], dtype=torch.float64)
    D1 = w[:, :9].view(-1, 3, 3); D2 = w[:, 9:].view(-1, 5, 5)
    assert (D1 @ D1.transpose(1, 2) - torch.eye(3)).abs().max() < 5e-6
    assert (D2 @ D2.transpose(1, 2) - torch.eye(5)).abs().max() < 5e-6


def test_layer_norm_silu(gold, inp):
    x = inp["ln_x"].clone().requires_grad_(True)
    y = oops.layer_norm_silu(x, inp["ln_gamma"], inp["ln_beta"])
    close(y, gold["ln_out"], 2e-6, 1e-6)
    (gx,) = torch.autograd.grad(y, [x], inp["g_ln"])
    close(gx, gold["ln_gx"], 5e-6, 1e-5)


def test_gather(gold, inp):
    I = inp
    wig = torch.tensor(gold["geom_wig"])
    xin = I["x"].clone().requires_grad_(True)
    wg = wig.clone().requires_grad_(True)
    rad = I["rad12"].clone().requires_grad_(True)
    X = oops.gather_wigner_split(xin, I["idx_i"], I["idx_j"], wg, rad, I["csd"], I["batch"])
    for k, t in enumerate(X):
        close(t, gold[f"gat_X{k}"], 1e-5, 1e-5)
    gx, gw, gr = torch.autograd.grad(list(X), [xin, wg, rad], [I["g_X0"], I["g_X1"], I["g_X2"]])
    close(gx, gold["gat_gx"], 5e-5, 1e-5)
    close(gr, gold["gat_grad"], 1e-5, 1e-5)
    # the reference returns no gradient for the system embedding; the oracle's csd
    # gradient is irrelevant here, g_wigner is a sum over C
    close(gw, gold["gat_gwig"], 1e-4, 1e-5)


def test_gating(gold, inp):
    Y = [inp[k].clone().requires_grad_(True) for k in ("Y0", "Y1", "Y2")]
    Z = oops.fused_gating_split(*Y, inp["C"])
    for k, t in enumerate(Z):
        close(t, gold[f"gate_Z{k}"], 1e-6, 1e-6)
    g = torch.autograd.grad(list(Z), Y, [inp["g_Z0"], inp["g_Z1"], inp["g_Z2"]])
    for k, t in enumerate(g):
        close(t, gold[f"gate_gY{k}"], 1e-6, 1e-6)


def test_rotate_scatter(gold, inp):
    I = inp
    wig = torch.tensor(gold["geom_wig"]); env = torch.tensor(gold["geom_env"])
    rp, ci = csr_of(I["idx_j"], I["N"])
    Zo = [I[k].clone().requires_grad_(True) for k in ("Zo0", "Zo1", "Zo2")]
    wg = wig.clone().requires_grad_(True); en = env.clone().requires_grad_(True)
    xr = I["x"].clone().requires_grad_(True)
    out = oops.rotate_scatter_split(*Zo, wg, en, xr, I["idx_j"], rp, ci, I["N"])
    close(out, gold["sc_out"], 1e-5, 1e-6)
    g = torch.autograd.grad(out, Zo + [wg, en, xr], I["g_node"])
    names = ["sc_gZ0", "sc_gZ1", "sc_gZ2", "sc_gwig", "sc_genv", "sc_gxres"]
    for t, n in zip(g, names):
        close(t, gold[n], 5e-5, 1e-5)


def test_init_scatter(gold, inp):
    I = inp
    wig = torch.tensor(gold["geom_wig"]); env = torch.tensor(gold["geom_env"])
    rp, ci = csr_of(I["idx_j"], I["N"])
    rad = I["rad3"].clone().requires_grad_(True)
    wg = wig.clone().requires_grad_(True); en = env.clone().requires_grad_(True)
    out = oops.init_node_scatter(rad, wg, en, I["Z"], I["batch"], I["W_sphere"], I["csd"], I["idx_j"], rp, ci, I["N"])
    close(out, gold["init_out"], 1e-5, 1e-6)
    g = torch.autograd.grad(out, [rad, wg, en], I["g_node"])
    for t, n in zip(g, ["init_grad", "init_gwig", "init_genv"]):
        close(t, gold[n], 5e-5, 1e-5)


def _e2e(name, systems, dtype=torch.float32):
    from flash_uma_b200.predict import Predictor
    from flash_uma_b200.synthetic import SyntheticESCNMDBackbone, make_energy_head
    from flash_uma_b200.systems import to_graph
    g = dict(np.load(os.path.join(GOLD, name)))
    C, L, B = int(g["C"]), int(g["layers"]), int(g["B"])
    data = to_graph(systems)
    np.testing.assert_array_equal(data.edge_index.numpy(), g["edge_index"])
    np.testing.assert_array_equal(data.cell_offsets.numpy(), g["cell_offsets"])
    off = SyntheticESCNMDBackbone(num_layers=L, sphere_channels=C, hidden_channels=C, num_distance_basis=B,
                                  seed=0, stress=True)
    head = make_energy_head(C, C, seed=1)
    res = Predictor(omodel.OracleBackbone(off, dtype), head)(data, forces=True, stress=True)
    return g, res


@pytest.mark.slow
def test_end_to_end_batched_matches_reference():
    from flash_uma_b200.systems import config1_system, water_box
    g, res = _e2e("e2e_batched.npz", [config1_system(), water_box(n_mol=8, jitter=0.05, seed=3)])
    e = res["energy"].numpy()
    np.testing.assert_allclose(e, g["energy"], rtol=1e-5)
    assert np.abs(res["forces"].numpy() - g["forces"]).max() < 1e-4
    np.testing.assert_allclose(res["stress"].numpy(), g["stress"], atol=1e-4 * max(1.0, np.abs(g["stress"]).max()))


@pytest.mark.slow
def test_end_to_end_config1_matches_reference():
    from flash_uma_b200.systems import config1_system
    g, res = _e2e("e2e_config1.npz", [config1_system()])
    np.testing.assert_allclose(res["energy"].numpy(), g["energy"], rtol=1e-5)
    assert np.abs(res["forces"].numpy() - g["forces"]).max() < 1e-4
    np.testing.assert_allclose(res["node_embedding"].numpy(), g["node_embedding"], atol=2e-4, rtol=1e-4)
