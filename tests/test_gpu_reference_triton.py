"""This build against the reference's own Triton path, both on the GPU, at full size.

The unmodified reference (installed into ``baseline/_ref`` by ``baseline/install_reference.py``)
runs its Triton kernels natively on the same device, on the same seed-0 weights, node-wise
stand-ins, energy head and inputs; TF32 is off for its ``F.linear`` calls (full fp32). Bars
(``north_star``): energy 1e-5 relative, forces 1e-4 eV/A max-abs. The reference's gather and
geometry backward use fp32 atomics, so its forces vary run to run at the 1e-6 level. Skipped
when the reference is not installed."""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


@pytest.fixture(scope="module")
def ref_wrapper():
    import bench
    w = bench.load_reference_gpu()
    if w is None:
        pytest.skip("reference not installed in baseline/_ref")
    return w


@pytest.fixture(autouse=True)
def _no_tf32():
    old = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old


def _both(ref_wrapper, system, stress):
    from flash_uma_b200.linear import check_errors
    from flash_uma_b200.predict import Predictor
    from flash_uma_b200.synthetic import SyntheticESCNMDBackbone, make_energy_head
    from flash_uma_b200.systems import to_graph
    from flash_uma_b200.wrapper import ZeroAllocBackbone
    data = to_graph([system]).to(DEV)
    off = SyntheticESCNMDBackbone(seed=0, stress=stress).to(DEV)
    head = make_energy_head(128, 128, seed=1).to(DEV)
    ours = Predictor(ZeroAllocBackbone(copy.deepcopy(off)), copy.deepcopy(head))(data, stress=stress)
    torch.cuda.synchronize()
    check_errors()
    ref = Predictor(ref_wrapper.ZeroAllocBackbone(off, dtype=torch.float32), head)(data, stress=stress)
    torch.cuda.synchronize()
    return ours, ref


def _check(ours, ref, stress):
    e, er = ours["energy"].double(), ref["energy"].double()
    assert ((e - er).abs() / er.abs().clamp(min=1.0)).max().item() < 1e-5
    assert (ours["forces"].double() - ref["forces"].double()).abs().max().item() < 1e-4
    if stress:
        s, sr = ours["stress"].double(), ref["stress"].double()
        assert (s - sr).abs().max().item() < 1e-4 * max(1.0, sr.abs().max().item())


def test_config1_matches_reference_triton(ref_wrapper):
    from flash_uma_b200.systems import config1_system
    ours, ref = _both(ref_wrapper, config1_system(), stress=True)
    _check(ours, ref, stress=True)


def test_config3_matches_reference_triton(ref_wrapper):
    """The bench workload (4,000 atoms, 120,000 edges), energy + forces."""
    from flash_uma_b200.systems import config3_system
    ours, ref = _both(ref_wrapper, config3_system(), stress=False)
    _check(ours, ref, stress=False)
