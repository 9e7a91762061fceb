"""Spatial domain decomposition of one periodic system over several GPUs (one process per GPU).

The reference is single-GPU. Here rank r owns the atoms whose fractional coordinate along
the longest cell axis lies in slab r, and the edges whose destination it owns (a
destination's messages come only from its own edges, so the per-destination FP64 scatter
sums are the single-GPU sums). Sources owned by other ranks are halo atoms: before every
message-passing layer each rank receives their current node embeddings from the owners
(one ``all_to_all_single``, NCCL over NVLink on GPUs), and in the backward pass the
gradients of those halo copies travel back to the owners and are added there in a fixed
peer order. Positions are replicated (every rank holds the global ``pos``); each rank's
partial position gradient is summed across ranks with one all-reduce, as is the energy.

Every rank builds every rank's plan from the same global neighbour list, so the edge sets
are exactly a partition of the single-GPU list and no setup communication is needed.

The driver works with any model object exposing the stage protocol ``build_graph``,
``geometry``, ``init_embedding``, ``layer_forward``, ``final`` (the CUDA model
:class:`~flash_uma_b200.model.ESCNInferenceModel`; the CPU tests drive the oracle through
the same protocol over gloo).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist


def slab_owner(positions: np.ndarray, cell: np.ndarray, world: int, axis: int | None = None) -> tuple[np.ndarray, int]:
    """Owner rank of every atom: slab of the wrapped fractional coordinate along ``axis``
    (default: the cell direction with the largest distance between opposite faces)."""
    cell = np.asarray(cell, dtype=np.float64)
    if axis is None:
        vol = abs(np.linalg.det(cell))
        face = [vol / np.linalg.norm(np.cross(cell[(k + 1) % 3], cell[(k + 2) % 3])) for k in range(3)]
        axis = int(np.argmax(face))
    frac = np.asarray(positions, dtype=np.float64) @ np.linalg.inv(cell)
    f = frac[:, axis] - np.floor(frac[:, axis])
    return np.minimum((f * world).astype(np.int64), world - 1), axis


@dataclass
class PartitionPlan:
    world: int
    rank: int
    axis: int
    owner: np.ndarray           # [N] owner rank of every atom
    owned: np.ndarray           # global ids owned here, ascending
    halo: np.ndarray            # global ids of halo atoms, ordered by (owner, id)
    edges: np.ndarray           # global ids of the edges handled here (destination owned), ascending
    edge_index: np.ndarray      # [2, E_r] local indices (owned atoms first, then halo)
    send_idx: list              # per peer: positions in ``owned`` to send (peer's halo order)
    recv_counts: list           # per peer: number of halo atoms received from it

    @property
    def local_ids(self) -> np.ndarray:
        return np.concatenate([self.owned, self.halo])


def _halo_of(p: int, owner: np.ndarray, src: np.ndarray, dst: np.ndarray) -> np.ndarray:
    sel = (owner[dst] == p) & (owner[src] != p)
    h = np.unique(src[sel])
    return h[np.lexsort((h, owner[h]))]


def make_plan(positions, cell, edge_index, world: int, rank: int, axis: int | None = None) -> PartitionPlan:
    """Deterministic plan of ``rank`` for the global ``edge_index`` [2, E] (row 0 source, row 1
    destination); identical on every rank for the same inputs."""
    edge_index = np.asarray(edge_index)
    src, dst = edge_index[0], edge_index[1]
    owner, axis = slab_owner(positions, cell, world, axis)
    N = owner.shape[0]
    owned = np.nonzero(owner == rank)[0]
    edges = np.nonzero(owner[dst] == rank)[0]
    halos = [_halo_of(p, owner, src, dst) for p in range(world)]
    halo = halos[rank]
    local = np.concatenate([owned, halo])
    g2l = np.full(N, -1, dtype=np.int64)
    g2l[local] = np.arange(local.shape[0])
    ei = g2l[edge_index[:, edges]]
    assert (ei >= 0).all()
    pos_in_owned = np.full(N, -1, dtype=np.int64)
    pos_in_owned[owned] = np.arange(owned.shape[0])
    send_idx = []
    for p in range(world):
        hp = halos[p]
        mine = hp[owner[hp] == rank] if p != rank else hp[:0]
        send_idx.append(pos_in_owned[mine])
    recv_counts = [int((owner[halo] == p).sum()) for p in range(world)]
    return PartitionPlan(world, rank, axis, owner, owned, halo, edges, ei, send_idx, recv_counts)


class HaloExchanger:
    """Device-side copy of a plan's exchange lists for one process group."""

    def __init__(self, plan: PartitionPlan, device, group=None):
        self.group = group
        self.send_idx = [torch.as_tensor(s, dtype=torch.long, device=device) for s in plan.send_idx]
        self.send_cat = torch.cat(self.send_idx) if self.send_idx else torch.zeros(0, dtype=torch.long, device=device)
        self.send_splits = [int(s.shape[0]) for s in plan.send_idx]
        self.recv_splits = list(plan.recv_counts)
        self.n_send = sum(self.send_splits)
        self.n_halo = sum(self.recv_splits)


# Optional timing of the collectives (bench breakdown): when a list, every collective of a step
# appends (name, start event, end event) recorded on the current stream around it.
collective_events: list | None = None


class _Timed:
    def __init__(self, name):
        self.name = name

    def __enter__(self):
        if collective_events is not None:
            self.e0 = torch.cuda.Event(enable_timing=True)
            self.e0.record()

    def __exit__(self, *exc):
        if collective_events is not None:
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record()
            collective_events.append((self.name, self.e0, e1))


def collective_times_ms() -> dict:
    """Total milliseconds per collective kind over the recorded events (synchronises)."""
    out: dict = {}
    for name, a, b in collective_events or []:
        b.synchronize()
        out[name] = out.get(name, 0.0) + a.elapsed_time(b)
    return out


class _HaloExchange(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_owned, ex: HaloExchanger):
        send = x_owned.index_select(0, ex.send_cat).contiguous()
        recv = x_owned.new_empty((ex.n_halo,) + tuple(x_owned.shape[1:]))
        with _Timed("halo_all_to_all_fwd"):
            dist.all_to_all_single(recv, send, ex.recv_splits, ex.send_splits, group=ex.group)
        ctx.ex, ctx.n_owned = ex, x_owned.shape[0]
        return recv

    @staticmethod
    def backward(ctx, g_recv):
        ex = ctx.ex
        g_send = g_recv.new_empty((ex.n_send,) + tuple(g_recv.shape[1:]))
        with _Timed("halo_all_to_all_bwd"):
            dist.all_to_all_single(g_send, g_recv.contiguous(), ex.send_splits, ex.recv_splits, group=ex.group)
        g_owned = g_recv.new_zeros((ctx.n_owned,) + tuple(g_recv.shape[1:]))
        off = 0
        for idx, n in zip(ex.send_idx, ex.send_splits):   # fixed peer order; indices unique per peer
            if n:
                g_owned.index_add_(0, idx, g_send[off: off + n])
                off += n
        return g_owned, None


def halo_exchange(x_owned: torch.Tensor, ex: HaloExchanger) -> torch.Tensor:
    """Node features of this rank's halo atoms, fetched from their owners (differentiable)."""
    return _HaloExchange.apply(x_owned, ex)


class PartitionedModel:
    """Runs a stage-protocol model on this rank's part of one periodic system."""

    def __init__(self, model, plan: PartitionPlan, device, group=None):
        self.model, self.plan, self.device, self.group = model, plan, device, group
        self.n_owned = int(plan.owned.shape[0])
        self.local_ids = torch.as_tensor(plan.local_ids, dtype=torch.long, device=device)
        self.edges = torch.as_tensor(plan.edges, dtype=torch.long, device=device)
        ei = torch.as_tensor(plan.edge_index, dtype=torch.long, device=device)
        self.idx_i, self.idx_j = ei[0].contiguous(), ei[1].contiguous()
        self.n_local = int(self.local_ids.shape[0])
        self.ex = HaloExchanger(plan, device, group)
        self.graph = model.build_graph(self.idx_i, self.idx_j, self.n_local)

    def node_embedding(self, pos, Z, batch, cell_offsets, cell, csd_emb, charge=None, spin=None, natoms=None):
        """Final node embedding of the owned atoms. ``pos``, ``Z``, ``batch`` are global [N];
        ``cell_offsets`` is the global [E, 3]; ``cell`` is [3, 3]; ``charge``, ``spin``, ``natoms``
        are per system (needed by models with charge / spin channel ranges, whose per-system
        channel sums are all-reduced across the ranks after every layer, ``model.py:213-216``)."""
        m = self.model
        pos_l = pos.index_select(0, self.local_ids)
        Z_l = Z.index_select(0, self.local_ids)
        b_l = batch.index_select(0, self.local_ids)
        shifts = cell_offsets.index_select(0, self.edges).to(cell.dtype) @ cell
        xe, wig, env = m.geometry(pos_l, Z_l, self.idx_i, self.idx_j, shifts, self.graph)
        x = m.init_embedding(xe, wig, env, Z_l, b_l, csd_emb, self.idx_j, self.graph, self.n_local)
        for k in range(len(m.layers)):
            x_owned = x[: self.n_owned]
            x = torch.cat([x_owned, halo_exchange(x_owned, self.ex)], 0)
            # owned rows out: the halo rows' layer outputs would be replaced by the next exchange
            x = m.layer_forward(k, x, xe, wig, env, self.idx_i, self.idx_j, self.graph, csd_emb, b_l, charge, spin,
                                natoms, n_out=self.n_owned, partitioned=True, group=self.group)
        return m.final(x[: self.n_owned])

    def energy_forces(self, head, pos, Z, batch, cell_offsets, cell, csd_emb, num_systems: int = 1,
                      stress: bool = False, charge=None, spin=None, natoms=None):
        """Global energy [num_systems] and forces [N, 3] (and, with ``stress``, the virial stress
        [1, 3, 3] of the one periodic system), identical on every rank.

        Stress follows the strain-displacement construction of the single-GPU predictor: a
        symmetric strain applied to the replicated positions and to the cell; every rank's
        gradient with respect to it covers its own edges and atoms, and one all-reduce sums them."""
        pos = pos.detach().requires_grad_(True)
        wrt = [pos]
        p, c = pos, cell
        if stress:
            if num_systems != 1:
                raise ValueError("the partitioned stress covers one periodic system")
            disp = torch.zeros(3, 3, dtype=pos.dtype, device=pos.device, requires_grad=True)
            sym = 0.5 * (disp + disp.t())
            p = pos + pos @ sym
            c = cell + cell @ sym
            wrt.append(disp)
        x = self.node_embedding(p, Z, batch, cell_offsets, c, csd_emb, charge, spin, natoms)
        b_owned = batch.index_select(0, self.local_ids[: self.n_owned])
        e_local = head(x, b_owned, num_systems)
        grads = torch.autograd.grad(e_local.sum(), wrt)
        energy = e_local.detach().clone()
        with _Timed("all_reduce_energy_forces"):
            dist.all_reduce(energy, group=self.group)
            g = grads[0]
            dist.all_reduce(g, group=self.group)
        if not stress:
            return energy, -g
        g_disp = grads[1].contiguous()
        with _Timed("all_reduce_stress"):
            dist.all_reduce(g_disp, group=self.group)
        vol = torch.linalg.det(cell.detach()).abs()
        return energy, -g, (g_disp / vol)[None]


class GraphedPartitionedStep:
    """:meth:`PartitionedModel.energy_forces` on a fixed partition (new positions every call),
    captured once as a CUDA graph together with its NCCL collectives (the per-layer halo
    exchanges in both directions and the energy / gradient all-reduces): a call copies the
    global positions into the captured input and replays the whole step with one launch.
    Every rank must construct it, call it and :meth:`release` it in the same order (the
    collectives inside are matched across ranks). Warm-up runs eagerly on a side stream first,
    so the NCCL communicators and every cached tensor exist before the capture. Returns the
    captured output tuple (overwritten by the next call). :meth:`release` frees the graph; do
    it before ``destroy_process_group``, which otherwise waits for the graph's NCCL work."""

    def __init__(self, pm: PartitionedModel, head, pos, Z, batch, cell_offsets, cell, csd_emb, num_systems: int = 1,
                 stress: bool = False, warmup: int = 3, capture_hook=None, charge=None, spin=None, natoms=None):
        self._pos = pos.detach().clone()
        args = (head, self._pos, Z, batch, cell_offsets, cell, csd_emb, num_systems, stress, charge, spin, natoms)
        dev = self._pos.device
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                pm.energy_forces(*args)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        dist.barrier(group=pm.group)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            if capture_hook is not None:
                capture_hook(True)
            try:
                self.out = pm.energy_forces(*args)
            finally:
                if capture_hook is not None:
                    capture_hook(False)
        torch.cuda.synchronize(dev)

    def __call__(self, pos: torch.Tensor):
        from . import linear
        linear.poll_errors()
        self._pos.copy_(pos, non_blocking=True)
        self.graph.replay()
        return self.out

    def release(self) -> None:
        if self.graph is not None:
            torch.cuda.synchronize(self._pos.device)
            self.graph.reset()
            self.graph = None
            self.out = None
