"""Spatial decomposition (CPU): plan invariants, and the partitioned driver over gloo ranks
(world sizes 2 and 4) reproducing the single-process energy, forces and stress. The CPU oracle runs
the model stages; the same driver runs the CUDA model over NCCL on GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flash_uma_b200 import partition as P
from flash_uma_b200.systems import bulk_fcc, neighbor_list


def _system():
    s = bulk_fcc(4, 4, 4, jitter=0.05, seed=7)
    ei, off, _ = neighbor_list(s, 6.0, 30)
    return s, ei, off


@pytest.mark.parametrize("world", [1, 2, 3, 4])
def test_plan_is_an_exact_partition(world):
    s, ei, _ = _system()
    plans = [P.make_plan(s.positions, s.cell, ei, world, r) for r in range(world)]
    all_edges = np.sort(np.concatenate([p.edges for p in plans]))
    assert np.array_equal(all_edges, np.arange(ei.shape[1]))          # every edge exactly once
    assert np.array_equal(np.sort(np.concatenate([p.owned for p in plans])), np.arange(s.natoms))
    for p in plans:
        src = ei[0, p.edges]
        assert set(np.unique(src[p.owner[src] != p.rank])) == set(p.halo)
        assert (p.owner[ei[1, p.edges]] == p.rank).all()
        # local indices point at the right global atoms
        loc = p.local_ids
        assert np.array_equal(loc[p.edge_index], ei[:, p.edges])
    for r in range(world):       # what r sends to q is what q expects from r
        for q in range(world):
            assert len(plans[r].send_idx[q]) == plans[q].recv_counts[r]
            if len(plans[r].send_idx[q]):
                sent = plans[r].owned[plans[r].send_idx[q]]
                expect = plans[q].halo[plans[q].owner[plans[q].halo] == r]
                assert np.array_equal(sent, expect)


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _backbone(balance: bool):
    from flash_uma_b200.synthetic import SyntheticESCNMDBackbone
    bb = SyntheticESCNMDBackbone(num_layers=2, sphere_channels=16, hidden_channels=16, num_distance_basis=8, seed=3)
    if balance:   # charge / spin channel balancing after every layer (model.py:213-216)
        bb.charge_channel_start, bb.charge_channel_end = 0, 4
        bb.spin_channel_start, bb.spin_channel_end = 4, 8
    return bb


def _data(balance: bool):
    from flash_uma_b200.systems import to_graph
    s, _, _ = _system()
    data = to_graph([s])
    if balance:
        data.charge, data.spin = torch.tensor([1]), torch.tensor([2])
    return s, data


def _worker(rank, world, port, out_path, balance=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.set_num_threads(1)
        import copy
        from flash_uma_b200.synthetic import SyntheticESCNMDBackbone, make_energy_head
        from flash_uma_b200.systems import to_graph
        from oracle.model import OracleBackbone
        s, data = _data(balance)
        bb = _backbone(balance)
        bb64 = copy.deepcopy(bb).double()
        head = make_energy_head(16, 16).double()
        model = OracleBackbone(bb64, torch.float64)
        csd = model.csd_embedding(data.charge, data.spin).double()
        plan = P.make_plan(s.positions, s.cell, data.edge_index.numpy(), world, rank)
        pm = P.PartitionedModel(model, plan, torch.device("cpu"))
        e, f, st = pm.energy_forces(head, data.pos.double(), data.atomic_numbers, data.batch,
                                    data.cell_offsets.double(), data.cell[0].double(), csd, stress=True,
                                    charge=data.charge, spin=data.spin, natoms=data.natoms)
        if rank == 0:
            torch.save({"energy": e, "forces": f, "stress": st}, out_path)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,balance", [(2, False), (4, False), (3, True)])
def test_partitioned_oracle_matches_single_process(world, balance, tmp_path):
    """``balance``: charge / spin channel balancing on, whose per-system sums span the ranks."""
    import copy
    from flash_uma_b200.predict import Predictor
    from flash_uma_b200.synthetic import make_energy_head
    from oracle.model import OracleBackbone
    out = str(tmp_path / "res.pt")
    mp.spawn(_worker, args=(world, _free_port(), out, balance), nprocs=world, join=True)
    got = torch.load(out)
    s, data = _data(balance)
    bb = _backbone(balance)
    ref = Predictor(OracleBackbone(copy.deepcopy(bb).double(), torch.float64), make_energy_head(16, 16).double())(
        type(data)(**{**data.__dict__, "pos": data.pos.double(), "cell": data.cell.double(),
                      "cell_offsets": data.cell_offsets.double()}), stress=True)
    assert torch.allclose(got["energy"], ref["energy"], rtol=1e-12, atol=1e-10)
    assert (got["forces"] - ref["forces"]).abs().max() < 1e-10
    assert (got["stress"] - ref["stress"]).abs().max() < 1e-10
