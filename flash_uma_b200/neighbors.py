"""The deterministic capped periodic neighbour list on the GPU (``fuma_neighbor_list``).

Same rule and output as the host statement :func:`flash_uma_b200.systems.neighbor_list`
(which documents it): per destination j, every (source i, integer offset s) with
``|pos_i - pos_j + s @ cell| < cutoff`` ordered by (distance, i, s) in fp64, the first
``max_neighbors`` kept, edges emitted by destination. The reference leaves graph generation
to FAIRChem / pymatgen outside its backbone (``readme.md:35-72``); this replaces the host
numpy pass (about 19 s for the 100,800-atom config 5) by one device pass.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _native as nat
from ._native import ptr, stream_of


def search_grid(cell: np.ndarray, pbc, cutoff: float):
    """(geom float64 [18]: cell then its inverse, grid int32 [12]: bins per axis, bin-offset
    range lo / hi, pbc) -- the binning and image ranges of the host statement."""
    cell = np.asarray(cell, dtype=np.float64).reshape(3, 3)
    inv = np.linalg.inv(cell)
    vol = abs(np.linalg.det(cell))
    face = np.array([vol / np.linalg.norm(np.cross(cell[(k + 1) % 3], cell[(k + 2) % 3])) for k in range(3)])
    reps = [int(np.ceil(cutoff / face[k])) if pbc[k] else 0 for k in range(3)]
    nb = np.maximum(1, np.floor(face / cutoff).astype(np.int64))
    lo, hi = [], []
    for k in range(3):
        if nb[k] > 2 or not pbc[k]:
            lo.append(-1), hi.append(1)
        else:
            lo.append(-reps[k] - 1), hi.append(reps[k] + 1)
    geom = np.concatenate([cell.reshape(-1), inv.reshape(-1)]).astype(np.float64)
    grid = np.array(list(nb) + lo + hi + [int(bool(p)) for p in pbc], dtype=np.int32)
    return geom, grid


def neighbor_list_device(pos: torch.Tensor, cell, pbc=(True, True, True), cutoff: float = 6.0,
                         max_neighbors: int = 30):
    """``edge_index`` [2, E] int64, ``cell_offsets`` [E, 3] int64 and ``distances`` [E] float64 on
    ``pos``'s device (pos [N, 3] float64; cell [3, 3] rows = lattice vectors). One synchronisation
    (the edge count)."""
    from .linear import error_flag
    nat.require_cuda(pos)
    pos = pos.to(torch.float64).contiguous()
    N = pos.shape[0]
    geom, grid = search_grid(np.asarray(cell.detach().cpu() if torch.is_tensor(cell) else cell), pbc, cutoff)
    lib = nat.load()
    gp = grid.ctypes.data_as(ctypes.c_void_p)
    nbytes = int(lib.fuma_neighbor_scratch_bytes(N, gp))
    dev = pos.device
    scratch = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    counts = torch.empty(N, dtype=torch.int32, device=dev)
    src = torch.empty(N, max_neighbors, dtype=torch.int64, device=dev)
    off = torch.empty(N, max_neighbors, 3, dtype=torch.int64, device=dev)
    dist = torch.empty(N, max_neighbors, dtype=torch.float64, device=dev)
    nat.call("fuma_neighbor_list", ptr(pos), N, geom.ctypes.data_as(ctypes.c_void_p), gp, float(cutoff),
             int(max_neighbors), ptr(scratch), nbytes, ptr(counts), ptr(src), ptr(off), ptr(dist),
             ptr(error_flag(dev)), stream_of(pos))
    mask = torch.arange(max_neighbors, device=dev)[None, :] < counts[:, None]
    dst = torch.arange(N, device=dev)[:, None].expand(N, max_neighbors)
    edge_index = torch.stack([src[mask], dst[mask]])
    return edge_index, off[mask], dist[mask]
