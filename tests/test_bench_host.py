"""Host-side logic of the bench and of the lean-mode choice (no GPU)."""
import csv
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def test_lean_mode_threshold(monkeypatch):
    from flash_uma_b200.fused import lean_bytes_per_edge, lean_needed
    monkeypatch.delenv("FUMA_LEAN", raising=False)
    assert lean_bytes_per_edge(128, 128, 4) == 92672
    total = 178 * 2 ** 30   # a B200
    assert not lean_needed(1_512_000, 128, 128, 4, total_bytes=total)   # config 5 over 2 GPUs
    assert lean_needed(3_024_000, 128, 128, 4, total_bytes=total)       # config 5 on one GPU
    monkeypatch.setenv("FUMA_LEAN", "1")
    assert lean_needed(10, 128, 128, 4, total_bytes=total)
    monkeypatch.setenv("FUMA_LEAN", "0")
    assert not lean_needed(10 ** 9, 128, 128, 4, total_bytes=total)


@pytest.mark.parametrize("workload,world,atoms,stress,scaling", [
    ("default", 1, 4000, False, "weak"), ("default", 2, 8000, False, "weak"),
    ("config4", 1, 9999, True, "strong"), ("config5", 4, 100800, False, "strong")])
def test_workloads(workload, world, atoms, stress, scaling):
    import bench
    system, with_stress, sc, label = bench.workload_system(workload, world)
    assert system.natoms == atoms and with_stress == stress and sc == scaling and label


def test_summarize_launches(tmp_path, capsys):
    import bench
    p = tmp_path / "launches.csv"
    rows = [["ID", "Kernel Name", "Metric Name", "Metric Unit", "Metric Value"]]
    seq = [("void at::native::FillFunctor<float>(x)", "usecond", "40"), ("fuma::gemm_f16x3_kernel<128>(a)", "usecond", "100"),
           ("fuma::gather_fwd_kernel(b)", "nsecond", "50000"), ("fuma::gemm_f16x3_kernel<128>(c)", "msecond", "0.1"),
           ("void at::native::FillFunctor<float>(x)", "usecond", "40"), ("fuma::gather_fwd_kernel(b)", "usecond", "7")]
    for i, (n, u, v) in enumerate(seq):
        rows.append([str(i), n, "gpu__time_duration.sum", u, v])
    with open(p, "w", newline="") as f:
        csv.writer(f).writerows(rows)
    bench.summarize_launches(str(p))
    out = capsys.readouterr().out
    assert "one timed step: 3 launches, 0.25 ms" in out
    assert "fuma::gemm_f16x3_kernel<128>" in out and "80.0%" in out


@pytest.mark.parametrize("C,B,gemm,fused", [(128, 64, "f16x3", True), (32, 16, "f16x3", True),
                                            (16, 8, "f16x3", False), (128, 64, "tf32x3", False)])
def test_model_construction_and_path_choice(C, B, gemm, fused, monkeypatch):
    """Building the model needs no GPU; the fused blocks are chosen exactly when every GEMM
    width is a multiple of 16 in the f16x3 mode."""
    monkeypatch.delenv("FUMA_FUSED", raising=False)
    from flash_uma_b200.synthetic import SyntheticESCNMDBackbone
    from flash_uma_b200.wrapper import ZeroAllocBackbone
    off = SyntheticESCNMDBackbone(num_layers=2, sphere_channels=C, hidden_channels=C, num_distance_basis=B)
    bb = ZeroAllocBackbone(off, gemm=gemm)
    assert bb.ce.fused is fused
    assert all(lay.fused is fused for lay in bb.ce.layers)
    assert bb.ce.set_fused(False) is False and not bb.ce.layers[0].fused


def test_fused_module_surface():
    """Every entry point the model and the bench use exists (a missing one only fails on a GPU)."""
    from flash_uma_b200 import fused
    for name in ("geometry", "message_block", "init_block", "fusable", "lean_needed", "radial_fwd", "radial_bwd"):
        assert callable(getattr(fused, name)), name


def test_roofline_flops_match_the_model_gemms():
    """The bench's algorithmic FLOPs (``gemm_flops_per_step``) equal 2 N K per edge of every dense
    layer the model holds (radial MLPs, conv1 / conv2 m-blocks), forward plus the input
    gradients, minus the radial layer-1 columns of the embeddings (no position dependence), plus
    the atom-wise block's maps per atom (scalar MLP 2H x C, per-degree maps on 1 + 3 + 5 rows)."""
    import bench
    from flash_uma_b200.linear import FrozenLinear
    from flash_uma_b200.synthetic import SyntheticESCNMDBackbone
    from flash_uma_b200.wrapper import ZeroAllocBackbone
    C, B, L, E, N = 128, 64, 4, 1000, 100
    bb = ZeroAllocBackbone(SyntheticESCNMDBackbone(num_layers=L, sphere_channels=C, hidden_channels=C,
                                                   num_distance_basis=B), gemm="f16x3")
    ce = bb.ce
    per_edge = 0
    for mod in [ce.rad_init] + list(ce.layers):
        for lin in mod.modules():
            if isinstance(lin, FrozenLinear):
                per_edge += 2 * lin.N * lin.K
    fwd = E * per_edge
    bwd = fwd - E * (L + 1) * 2 * 2 * C * C           # radial layer-1 gradient: Gaussian columns only
    aw = 0
    for lay in ce.layers:
        a = lay.atom_wise
        H = a.hidden
        aw += 2 * N * C * 2 * H + 2 * (2 * 9 * N * C * H)   # scalar MLP, two per-degree maps (9 rows each)
    assert bench.gemm_flops_per_step(E, C, B, L) == fwd + bwd
    assert bench.gemm_flops_per_step(E, C, B, L, N_atomwise=N) == fwd + bwd + 2 * aw
