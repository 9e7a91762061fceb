"""Generate the golden vectors in this directory by running the REFERENCE implementation.

Usage (only where the reference source tree is present; not on the GPU box):

    FLASHUMA_REFERENCE=<reference source tree> python tests/golden/make_golden.py [ops] [e2e]   # default: both

The reference's Triton kernels run on CPU tensors under the Triton interpreter
(see ``refharness.py``); autotune keeps each kernel's first config. Outputs:

* ``ops_small.npz``   - every op forward + backward on seeded small inputs (C=16,
                        B=8) with geometry edge cases (edges along +-y, edges at
                        the chart-blend boundaries e_y = +-0.9, an edge beyond the
                        cutoff, a very short edge, empty CSR rows).
* ``e2e_config1.npz`` - energy, forces, stress and node embedding of benchmark
                        config 1 (Cu fcc100 slab + CO, 29 atoms, C=128, 4 layers,
                        B=64, seed-0 weights) through the reference ``ZeroAllocBackbone``.
* ``e2e_batched.npz`` - a 2-system batch (slab + 8-molecule water box), C=32, 2 layers.

Weights are not stored: tests rebuild them from the seeds
(``SyntheticESCNMDBackbone(seed=0)``, ``make_energy_head(seed=1)``); the stored
graph arrays let the tests assert that the rebuild reproduces the same inputs.
"""
from __future__ import annotations

import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, HERE)

import refharness  # noqa: E402


def _np(t):
    return t.detach().cpu().numpy()


def small_op_inputs(seed: int = 0, C: int = 16, B: int = 8, N: int = 40, E: int = 320):
    """Seeded small inputs for the per-op fixtures (also used by the tests to rebuild them)."""
    g = torch.Generator().manual_seed(seed)
    pos = torch.randn(N, 3, generator=g) * 2.0
    idx_i = torch.randint(0, N, (E,), generator=g)
    idx_j = torch.randint(0, N, (E,), generator=g)
    idx_j[idx_j == 7] = 8                      # node 7 has no incoming edge (empty CSR row)
    idx_i[idx_i == idx_j] = (idx_i[idx_i == idx_j] + 1) % N
    shifts = torch.randint(-1, 2, (E, 3), generator=g).to(torch.float32) * 1.5
    # geometry edge cases: overwrite the vectors of the first edges via the shift
    special = torch.tensor([
        [0.0, 2.0, 0.0], [0.0, -2.0, 0.0],            # along +y / -y (chart singularities)
        [1.0, 0.9 * 2.0 / 1.0, 0.0],                   # generic
        [0.0, 0.0, 3.0], [3.0, 0.0, 0.0],              # along z / x
        [0.4358899, 0.9, 0.0], [0.4358899, -0.9, 0.0], # e_y = +-0.9 (blend boundaries)
        [0.0, 7.0, 0.5],                               # beyond the cutoff (env = 0)
        [0.05, 0.02, -0.03],                           # very short edge
        [1e-3, 1.5, 1e-3],                             # nearly +y
        [-1e-3, -1.5, 1e-3],                           # nearly -y
    ])
    ns = min(special.shape[0], E)
    shifts[:ns] = special[:ns] - (pos[idx_i[:ns]] - pos[idx_j[:ns]])
    Z = torch.randint(1, 90, (N,), generator=g)
    W_src = torch.randn(100, C, generator=g)
    W_tgt = torch.randn(100, C, generator=g)
    offset_g = torch.linspace(0.0, 6.0, B)
    coeff_g = float(-0.5 / (2.0 * (offset_g[1] - offset_g[0])) ** 2)
    nsys = 2
    batch = (torch.arange(N) >= N // 2).long()
    csd = torch.randn(nsys, C, generator=g)
    x = torch.randn(N, 9, C, generator=g)
    rad12 = torch.randn(E, 12 * C, generator=g)
    rad3 = torch.randn(E, 3 * C, generator=g)
    Y0 = torch.randn(E, 5 * C, generator=g) * 2
    Y1 = torch.randn(E, 4 * C, generator=g)
    Y2 = torch.randn(E, 2 * C, generator=g)
    Zo0 = torch.randn(E, 3 * C, generator=g)
    Zo1 = torch.randn(E, 4 * C, generator=g)
    Zo2 = torch.randn(E, 2 * C, generator=g)
    W_sphere = torch.randn(100, C, generator=g)
    ln_x = torch.randn(64, 32, generator=g) * 3 + 1
    ln_gamma = 1 + 0.1 * torch.randn(32, generator=g)
    ln_beta = 0.1 * torch.randn(32, generator=g)
    grads = dict(
        g_xe=torch.randn(E, B + 2 * C, generator=g), g_wig=torch.randn(E, 34, generator=g),
        g_env=torch.randn(E, generator=g),
        g_X0=torch.randn(E, 6 * C, generator=g), g_X1=torch.randn(E, 8 * C, generator=g),
        g_X2=torch.randn(E, 4 * C, generator=g),
        g_Z0=torch.randn(E, 3 * C, generator=g), g_Z1=torch.randn(E, 4 * C, generator=g),
        g_Z2=torch.randn(E, 2 * C, generator=g),
        g_node=torch.randn(N, 9, C, generator=g), g_ln=torch.randn(64, 32, generator=g),
    )
    return dict(C=C, B=B, N=N, E=E, pos=pos, idx_i=idx_i, idx_j=idx_j, shifts=shifts, Z=Z, W_src=W_src,
                W_tgt=W_tgt, offset_g=offset_g, coeff_g=coeff_g, cutoff=6.0, batch=batch, csd=csd, x=x,
                rad12=rad12, rad3=rad3, Y0=Y0, Y1=Y1, Y2=Y2, Zo0=Zo0, Zo1=Zo1, Zo2=Zo2, W_sphere=W_sphere,
                ln_x=ln_x, ln_gamma=ln_gamma, ln_beta=ln_beta, **grads)


def csr_of(idx, N):
    order = torch.argsort(idx, stable=True)
    counts = torch.bincount(idx, minlength=N)
    row_ptr = torch.zeros(N + 1, dtype=torch.int32)
    row_ptr[1:] = torch.cumsum(counts, 0).to(torch.int32)
    return row_ptr, order.to(torch.int32)


def make_ops_small(ref, path):
    I = small_op_inputs()
    out = {}
    # geometry
    pos = I["pos"].clone().requires_grad_(True)
    shifts = I["shifts"].clone().requires_grad_(True)
    xe, wig, env = ref.precompute_geometry(pos, I["Z"], I["idx_i"], I["idx_j"], shifts, I["W_src"], I["W_tgt"],
                                           I["offset_g"], I["coeff_g"], I["cutoff"])
    gp, gs = torch.autograd.grad([xe, wig, env], [pos, shifts], [I["g_xe"], I["g_wig"], I["g_env"]])
    out.update(geom_xe=_np(xe), geom_wig=_np(wig), geom_env=_np(env), geom_gpos=_np(gp), geom_gshifts=_np(gs))
    wig = wig.detach(); env = env.detach()
    # layer norm silu
    x = I["ln_x"].clone().requires_grad_(True)
    y = ref.layer_norm_silu(x, I["ln_gamma"], I["ln_beta"])
    (gx,) = torch.autograd.grad(y, [x], I["g_ln"])
    out.update(ln_out=_np(y), ln_gx=_np(gx))
    # gather
    xin = I["x"].clone().requires_grad_(True)
    wg = wig.clone().requires_grad_(True)
    rad = I["rad12"].clone().requires_grad_(True)
    X0, X1, X2 = ref.gather_wigner_split(xin, I["idx_i"], I["idx_j"], wg, rad, I["csd"], I["batch"])
    gx, gw, gr = torch.autograd.grad([X0, X1, X2], [xin, wg, rad], [I["g_X0"], I["g_X1"], I["g_X2"]])
    out.update(gat_X0=_np(X0), gat_X1=_np(X1), gat_X2=_np(X2), gat_gx=_np(gx), gat_gwig=_np(gw), gat_grad=_np(gr))
    # gating
    Y = [I[k].clone().requires_grad_(True) for k in ("Y0", "Y1", "Y2")]
    Zs = ref.fused_gating_split(*Y, I["C"])
    gY = torch.autograd.grad(list(Zs), Y, [I["g_Z0"], I["g_Z1"], I["g_Z2"]])
    out.update(gate_Z0=_np(Zs[0]), gate_Z1=_np(Zs[1]), gate_Z2=_np(Zs[2]),
               gate_gY0=_np(gY[0]), gate_gY1=_np(gY[1]), gate_gY2=_np(gY[2]))
    # rotate scatter
    row_ptr, col_idx = csr_of(I["idx_j"], I["N"])
    Zo = [I[k].clone().requires_grad_(True) for k in ("Zo0", "Zo1", "Zo2")]
    wg = wig.clone().requires_grad_(True); en = env.clone().requires_grad_(True)
    xres = I["x"].clone().requires_grad_(True)
    xo = ref.rotate_scatter_split(*Zo, wg, en, xres, I["idx_j"], row_ptr, col_idx, I["N"])
    g = torch.autograd.grad(xo, Zo + [wg, en, xres], I["g_node"])
    out.update(sc_out=_np(xo), sc_gZ0=_np(g[0]), sc_gZ1=_np(g[1]), sc_gZ2=_np(g[2]), sc_gwig=_np(g[3]),
               sc_genv=_np(g[4]), sc_gxres=_np(g[5]))
    # init scatter
    rad = I["rad3"].clone().requires_grad_(True)
    wg = wig.clone().requires_grad_(True); en = env.clone().requires_grad_(True)
    x0 = ref.init_node_scatter(rad, wg, en, I["Z"], I["batch"], I["W_sphere"], I["csd"], I["idx_j"], row_ptr,
                               col_idx, I["N"])
    g = torch.autograd.grad(x0, [rad, wg, en], I["g_node"])
    out.update(init_out=_np(x0), init_grad=_np(g[0]), init_gwig=_np(g[1]), init_genv=_np(g[2]))
    np.savez_compressed(path, **out)
    print("wrote", path, {k: v.shape for k, v in out.items()})


def make_e2e(ref_wrapper, path, systems, C, layers, B=64, stress=True):
    from flash_uma_b200.predict import Predictor
    from flash_uma_b200.synthetic import SyntheticESCNMDBackbone, make_energy_head
    from flash_uma_b200.systems import to_graph

    data = to_graph(systems)
    off = SyntheticESCNMDBackbone(num_layers=layers, sphere_channels=C, hidden_channels=C,
                                  num_distance_basis=B, seed=0, stress=stress)
    head = make_energy_head(C, C, seed=1)
    bb = ref_wrapper.ZeroAllocBackbone(off, dtype=torch.float32)
    t = time.time()
    res = Predictor(bb, head)(data, forces=True, stress=stress)
    print(f"reference e2e ({data.pos.shape[0]} atoms, {data.edge_index.shape[1]} edges) {time.time() - t:.1f}s")
    out = dict(energy=_np(res["energy"]), forces=_np(res["forces"]), node_embedding=_np(res["node_embedding"]),
               pos=_np(data.pos), edge_index=_np(data.edge_index), cell_offsets=_np(data.cell_offsets),
               C=C, layers=layers, B=B)
    if stress:
        out["stress"] = _np(res["stress"])
    np.savez_compressed(path, **out)
    print("wrote", path, "energy", out["energy"])


def main():
    torch.set_num_threads(os.cpu_count() or 1)
    ref, ref_model, ref_wrapper = refharness.load()
    which = set(sys.argv[1:]) or {"ops", "e2e"}
    if "ops" in which:
        make_ops_small(ref, os.path.join(HERE, "ops_small.npz"))
    if "e2e" not in which:
        return
    from flash_uma_b200.systems import config1_system, water_box
    make_e2e(ref_wrapper, os.path.join(HERE, "e2e_batched.npz"),
             [config1_system(), water_box(n_mol=8, jitter=0.05, seed=3)], C=32, layers=2)
    make_e2e(ref_wrapper, os.path.join(HERE, "e2e_config1.npz"), [config1_system()], C=128, layers=4)


if __name__ == "__main__":
    main()
