"""CUDA-graph replay of a whole energy + forces step (``predict.GraphedStep``) gives exactly the
eager step's results on new positions (the same kernels in the same order, deterministic)."""
import dataclasses

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


@pytest.mark.parametrize("C,B", [(128, 64), (32, 16)])
def test_graphed_step_matches_eager(C, B):
    from flash_uma_b200.predict import GraphedStep, Predictor
    from flash_uma_b200.synthetic import SyntheticESCNMDBackbone, make_energy_head
    from flash_uma_b200.systems import bulk_fcc, to_graph
    from flash_uma_b200.wrapper import ZeroAllocBackbone
    data = to_graph([bulk_fcc(3, 3, 3, jitter=0.05, seed=8)]).to(DEV)
    off = SyntheticESCNMDBackbone(num_layers=2, sphere_channels=C, hidden_channels=C, num_distance_basis=B,
                                  seed=4).to(DEV)
    pred = Predictor(ZeroAllocBackbone(off), make_energy_head(C, C).to(DEV))
    step = GraphedStep(pred, data)
    g = torch.Generator(device="cpu").manual_seed(0)
    for _ in range(3):
        pos = data.pos + 0.02 * torch.randn(data.pos.shape, generator=g).to(DEV)
        ref = pred(dataclasses.replace(data, pos=pos))
        out = step(pos)
        assert torch.equal(out["energy"], ref["energy"])
        assert torch.equal(out["forces"], ref["forces"])
