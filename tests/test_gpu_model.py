"""End-to-end parity of the CUDA path (``ZeroAllocBackbone``) with the reference implementation.

Bar (``north_star``): energy within 1e-5 relative and forces within 1e-4 eV/A max-abs of
the reference's own implementation on the same random-init weights and inputs. The
reference values are the golden vectors produced by running the reference's ops
(``tests/golden/make_golden.py``); the CPU oracle is checked alongside. Dense
contractions run in full fp32 (TF32 off) for these tests."""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
DEV = torch.device("cuda")


@pytest.fixture(autouse=True)
def _no_tf32():
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = old


def _run(systems, C, L, B, stress=True, seed=0, gemm=None, fused=True):
    from flash_uma_b200.predict import Predictor
    from flash_uma_b200.synthetic import SyntheticESCNMDBackbone, make_energy_head
    from flash_uma_b200.systems import to_graph
    from flash_uma_b200.wrapper import ZeroAllocBackbone
    data = to_graph(systems)
    off = SyntheticESCNMDBackbone(num_layers=L, sphere_channels=C, hidden_channels=C, num_distance_basis=B,
                                  seed=seed, stress=stress).to(DEV)
    head = make_energy_head(C, C, seed=1).to(DEV)
    bb = ZeroAllocBackbone(off, gemm=gemm)
    bb.ce.set_fused(fused)
    return data, Predictor(bb, head)(data.to(DEV), forces=True, stress=stress)


def _check(res, g, stress=True):
    e = res["energy"].cpu().numpy()
    np.testing.assert_allclose(e, g["energy"], rtol=1e-5, atol=0)
    ferr = np.abs(res["forces"].cpu().numpy() - g["forces"]).max()
    assert ferr < 1e-4, ferr
    if stress:
        np.testing.assert_allclose(res["stress"].cpu().numpy(), g["stress"],
                                   atol=1e-4 * max(1.0, np.abs(g["stress"]).max()))


@pytest.mark.parametrize("gemm,fused", [("f16x3", True), ("f16x3", False), ("tf32x3", False)])
def test_config1_matches_reference(gemm, fused):
    """Every dense-contraction path: fused f16x3 blocks (the default), f16x3 per op, 3xTF32."""
    from flash_uma_b200.systems import config1_system
    g = dict(np.load(os.path.join(GOLD, "e2e_config1.npz")))
    data, res = _run([config1_system()], int(g["C"]), int(g["layers"]), int(g["B"]), gemm=gemm, fused=fused)
    from flash_uma_b200.linear import check_errors
    check_errors()
    np.testing.assert_array_equal(data.edge_index.numpy(), g["edge_index"])
    _check(res, g)
    np.testing.assert_allclose(res["node_embedding"].cpu().numpy(), g["node_embedding"], atol=2e-4, rtol=1e-4)


def test_batched_systems_match_reference():
    from flash_uma_b200.systems import config1_system, water_box
    g = dict(np.load(os.path.join(GOLD, "e2e_batched.npz")))
    _, res = _run([config1_system(), water_box(n_mol=8, jitter=0.05, seed=3)], int(g["C"]), int(g["layers"]),
                  int(g["B"]))
    _check(res, g)


def test_forces_deterministic_and_invariant():
    """Run-to-run bitwise-identical forces (no atomics anywhere); energy invariant under a
    rigid rotation of the whole periodic system (cell rotated with it)."""
    from flash_uma_b200.predict import Predictor
    from flash_uma_b200.synthetic import SyntheticESCNMDBackbone, make_energy_head
    from flash_uma_b200.systems import bulk_fcc, to_graph
    from flash_uma_b200.wrapper import ZeroAllocBackbone
    data = to_graph([bulk_fcc(3, 3, 3, jitter=0.05, seed=4)]).to(DEV)
    off = SyntheticESCNMDBackbone(num_layers=2, sphere_channels=64, hidden_channels=64, seed=2).to(DEV)
    pred = Predictor(ZeroAllocBackbone(off), make_energy_head(64, 64).to(DEV))
    r1, r2 = pred(data), pred(data)
    assert torch.equal(r1["forces"], r2["forces"]) and torch.equal(r1["energy"], r2["energy"])
    q = torch.tensor([0.3, -0.5, 0.2, 0.7], dtype=torch.float64)
    q = q / q.norm()
    w, x, y, z = q
    R = torch.tensor([[1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)],
                      [2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)],
                      [2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)]])
    rot = data.clone()
    rot.pos = (data.pos.double() @ R.T.to(DEV)).float()
    rot.cell = (data.cell.double() @ R.T.to(DEV)).float()
    r3 = pred(rot)
    assert abs(r3["energy"].item() - r1["energy"].item()) < 2e-5 * max(1.0, abs(r1["energy"].item()))
    f_rot = (r1["forces"].double() @ R.T.to(DEV)).float()
    assert (r3["forces"] - f_rot).abs().max().item() < 2e-4


def test_gpu_matches_oracle_on_water():
    from flash_uma_b200.predict import Predictor
    from flash_uma_b200.synthetic import SyntheticESCNMDBackbone, make_energy_head
    from flash_uma_b200.systems import to_graph, water_box
    from flash_uma_b200.wrapper import ZeroAllocBackbone
    from oracle.model import OracleBackbone
    import copy
    data = to_graph([water_box(n_mol=40, seed=5)])
    off = SyntheticESCNMDBackbone(num_layers=2, sphere_channels=32, hidden_channels=32, num_distance_basis=16, seed=3)
    head = make_energy_head(32, 32)
    off64, head64 = copy.deepcopy(off).double(), copy.deepcopy(head).double()
    ref = Predictor(OracleBackbone(off64, torch.float64), head64)(
        type(data)(**{**data.__dict__, "pos": data.pos.double(), "cell": data.cell.double(),
                      "cell_offsets": data.cell_offsets.double()}), stress=True)
    res = Predictor(ZeroAllocBackbone(off.to(DEV)), head.to(DEV))(data.to(DEV), stress=True)
    e, er = res["energy"].cpu().double(), ref["energy"]
    assert ((e - er).abs() / er.abs().clamp(min=1)).max() < 1e-5
    assert (res["forces"].cpu().double() - ref["forces"]).abs().max() < 1e-4
    assert (res["stress"].cpu().double() - ref["stress"]).abs().max() < 1e-4 * max(1.0, ref["stress"].abs().max())


def test_lean_mode_is_bitwise_identical(monkeypatch):
    """The memory-lean backward (radial and conv2 outputs recomputed instead of saved) gives
    exactly the default mode's energy and forces: the recomputation runs the same kernels."""
    from flash_uma_b200.predict import Predictor
    from flash_uma_b200.synthetic import SyntheticESCNMDBackbone, make_energy_head
    from flash_uma_b200.systems import bulk_fcc, to_graph
    from flash_uma_b200.wrapper import ZeroAllocBackbone
    data = to_graph([bulk_fcc(3, 3, 3, jitter=0.05, seed=6)]).to(DEV)
    off = SyntheticESCNMDBackbone(num_layers=2, sphere_channels=64, hidden_channels=64, seed=7).to(DEV)
    pred = Predictor(ZeroAllocBackbone(off), make_energy_head(64, 64).to(DEV))
    monkeypatch.setenv("FUMA_LEAN", "0")
    ref = pred(data, stress=True)
    monkeypatch.setenv("FUMA_LEAN", "1")
    got = pred(data, stress=True)
    assert pred.backbone.ce.layers[0].lean
    for k in ("energy", "forces", "stress"):
        assert torch.equal(got[k], ref[k]), k


@pytest.mark.parametrize("N,E", [(1, 0), (7, 40), (500, 9000), (4000, 120000)])
def test_csr_permute_matches_sorted_build(N, E):
    """fuma_csr_permute: the renumbered CSRs equal the stable-argsort CSRs of the renumbered edges,
    bitwise, including empty rows (random graphs, random permutations)."""
    from flash_uma_b200 import ops
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(N + E)
    idx_i = torch.randint(0, N, (E,), generator=g).to(dev)
    idx_j = torch.randint(0, max(1, N // 2), (E,), generator=g).to(dev)   # half the nodes without in-edges
    perm = torch.randperm(N, generator=g).to(dev)
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(N, device=dev)
    base = ops.build_graph_csr(idx_i, idx_j, N)
    got = ops.permute_graph(base, perm)
    ref = ops.build_graph_csr(inv[idx_i], inv[idx_j], N)
    torch.cuda.synchronize()
    for f in ("dst_row_ptr", "dst_col", "src_row_ptr", "src_col"):
        assert torch.equal(getattr(got, f), getattr(ref, f)), f


@pytest.mark.parametrize("N,E,nsys", [(1, 0, 1), (29, 500, 1), (4000, 120000, 1), (3000, 50000, 3), (16384, 1000, 2),
                                      (16385, 5000, 1), (100800, 3024000, 1), (70000, 1000, 300),
                                      (40000, 100, 1 << 20), (50000, 10, -7)])
def test_native_morton_reorder_matches_torch(N, E, nsys):
    """fuma_morton_reorder against the torch statement of reorder_graph_morton (model.py:47-74)
    on the GPU: identical permutation (ties, e.g. duplicated positions, ordered by index), atom
    data and renumbered edges. Up to 16,384 atoms the one-block sort runs; above, the radix sort
    (config 5 has 100,800 atoms), with one or more system-id passes (300 and 2^20 systems), and
    with unsorted system ids (nsys < 0: |nsys| systems in random order)."""
    from flash_uma_b200.model import _reorder_native, _reorder_torch
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(N + E)
    pos = torch.rand(N, 3, generator=g) * 30.0
    if N > 10:
        pos[N // 2:N // 2 + 5] = pos[3]             # duplicated positions: equal keys
    if nsys < 0:
        batch = torch.randint(0, -nsys, (N,), generator=g)
    else:
        batch = torch.sort(torch.randint(0, nsys, (N,), generator=g))[0]
    Z = torch.randint(1, 90, (N,), generator=g)
    idx = torch.randint(0, N, (2, E), generator=g)
    args = [t.to(dev) for t in (pos, Z, batch, idx[0], idx[1])]
    got = _reorder_native(*args)
    ref = _reorder_torch(*args)
    torch.cuda.synchronize()
    for a, b in zip(got, ref):
        assert torch.equal(a, b)


def test_morton_reorder_flags_out_of_range_edges():
    """An edge index outside [0, N) is recorded (error code 32, raised by check_errors) and the
    edge is renumbered to atom 0 instead of being read out of bounds; valid edges are unaffected."""
    from flash_uma_b200.linear import check_errors
    from flash_uma_b200.model import _reorder_native, _reorder_torch
    dev = torch.device("cuda")
    for N in (100, 20000):   # both sort paths
        g = torch.Generator().manual_seed(N)
        pos = (torch.rand(N, 3, generator=g) * 20).to(dev)
        Z = torch.full((N,), 29, dtype=torch.long, device=dev)
        batch = torch.zeros(N, dtype=torch.long, device=dev)
        idx = torch.randint(0, N, (2, 50), generator=g).to(dev)
        bad = idx.clone()
        bad[0, 3] = N
        bad[1, 7] = -1
        got = _reorder_native(pos, Z, batch, bad[0], bad[1])
        ref = _reorder_torch(pos, Z, batch, idx[0], idx[1])
        torch.cuda.synchronize()
        with pytest.raises(RuntimeError, match="outside"):
            check_errors()
        ok = torch.ones(50, dtype=torch.bool, device=dev)
        ok[3] = ok[7] = False
        assert torch.equal(got[3][ok], ref[3][ok]) and torch.equal(got[4][ok], ref[4][ok])
        assert got[3][3].item() == 0 and got[4][7].item() == 0
        check_errors()   # the flag was cleared by the raise


@pytest.mark.parametrize("which", ["config1", "config3", "config4", "config5", "small_cell", "slab_open"])
def test_device_neighbor_list_matches_host(which):
    """fuma_neighbor_list gives exactly the host statement's edges (systems.neighbor_list): the
    same (source, destination, offset) triples in the same order, and the same fp64 distances,
    on the benchmark systems (configs 1, 3, 4, 5), on a cell smaller than the cutoff (many
    periodic images) and on a slab that is not periodic along z."""
    from flash_uma_b200.linear import check_errors
    from flash_uma_b200.neighbors import neighbor_list_device
    from flash_uma_b200 import systems as S
    sysm = {"config1": S.config1_system, "config3": S.config3_system, "config4": S.config4_system,
            "config5": S.config5_system, "small_cell": lambda: S.bulk_fcc(1, 1, 2, jitter=0.05, seed=3),
            "slab_open": lambda: S.AtomicSystem(S.bulk_fcc(4, 4, 3, jitter=0.05, seed=5).positions,
                                                np.full(192, 29), np.diag([14.44, 14.44, 30.0]),
                                                pbc=(True, True, False))}[which]()
    ei, off, dist = S.neighbor_list(sysm)
    pos = torch.tensor(sysm.positions, dtype=torch.float64, device="cuda")
    ei_d, off_d, dist_d = neighbor_list_device(pos, sysm.cell, sysm.pbc)
    torch.cuda.synchronize()
    check_errors()
    assert ei_d.shape == ei.shape
    assert np.array_equal(ei_d.cpu().numpy(), ei)
    assert np.array_equal(off_d.cpu().numpy(), off)
    np.testing.assert_array_equal(dist_d.cpu().numpy(), dist)


def test_config1_f16_mode_tf32_accuracy_class():
    """The single-product "f16" GEMM mode end to end on config 1 (fused blocks): within the TF32
    accuracy class of the reference's published setting, i.e. errors of fp16 operand rounding
    (about 5e-4 relative per operand), far below what separates physics (1e-3 relative energy,
    1e-2 eV/A forces), and deterministic run to run."""
    from flash_uma_b200.systems import config1_system
    g = dict(np.load(os.path.join(GOLD, "e2e_config1.npz")))
    data, res = _run([config1_system()], int(g["C"]), int(g["layers"]), int(g["B"]), stress=True, gemm="f16")
    from flash_uma_b200.linear import check_errors
    check_errors()
    e = res["energy"].cpu().numpy()
    assert np.abs(e - g["energy"]).max() <= 1e-3 * np.abs(g["energy"]).max()
    assert np.abs(res["forces"].cpu().numpy() - g["forces"]).max() < 1e-2
