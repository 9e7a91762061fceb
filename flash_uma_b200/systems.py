"""Synthetic atomic systems and a deterministic capped periodic neighbour list.

The reference receives its graph from FAIRChem / pymatgen (``external_graph_gen``,
outside the backbone). Neither ASE nor pymatgen is available, so the systems of
the benchmark configurations are built here from crystallography, and the graph
is a deterministic capped neighbour list:

* every ordered pair (source i, destination j, integer cell offset s) with
  ``|pos_i - pos_j + s @ cell| < cutoff`` (self pairs only with s != 0) is a
  candidate edge, the edge vector being ``pos[i] - pos[j] + s @ cell``
  (the sign convention of ``ops/geom.py:72-74`` and ``wrapper.py:193-197``);
* per destination j, candidates are ordered by (distance, source index, offset)
  in float64 and the first ``max_neighbors`` are kept;
* edges are emitted sorted by destination, then by that order.

Distances use float64 so the selection is identical on every machine; a
spatially partitioned build that applies the same rule to the same global
coordinates gets the same edges.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch

CU_LATTICE = 3.61  # Angstrom
FCC_BASIS = np.array([[0.0, 0.0, 0.0], [0.5, 0.5, 0.0], [0.5, 0.0, 0.5], [0.0, 0.5, 0.5]])


@dataclass
class AtomicSystem:
    """Host-side description of one periodic system."""
    positions: np.ndarray        # [N, 3] float64, Angstrom
    numbers: np.ndarray          # [N] int64 atomic numbers
    cell: np.ndarray             # [3, 3] float64, rows are lattice vectors
    pbc: tuple = (True, True, True)
    name: str = ""
    charge: int = 0
    spin: int = 0

    @property
    def natoms(self) -> int:
        return int(self.positions.shape[0])


def bulk_fcc(nx: int, ny: int, nz: int, a: float = CU_LATTICE, z: int = 29, jitter: float = 0.0,
             seed: int = 0, name: str = "") -> AtomicSystem:
    """Conventional-cell fcc supercell (4 atoms per cell), periodic in 3D."""
    grid = np.stack(np.meshgrid(np.arange(nx), np.arange(ny), np.arange(nz), indexing="ij"), -1).reshape(-1, 3)
    frac = (grid[:, None, :] + FCC_BASIS[None]).reshape(-1, 3)
    pos = frac * a
    if jitter > 0:
        pos = pos + np.random.default_rng(seed).normal(0.0, jitter, pos.shape)
    cell = np.diag([nx * a, ny * a, nz * a]).astype(np.float64)
    return AtomicSystem(pos, np.full(len(pos), z, dtype=np.int64), cell, name=name or f"fcc{nx}x{ny}x{nz}")


def cu_fcc100_slab_co(size=(3, 3, 3), a: float = CU_LATTICE, vacuum: float = 8.0, height: float = 2.0,
                      co_bond: float = 1.13, jitter: float = 0.02, seed: int = 0) -> AtomicSystem:
    """Cu fcc(100) slab with a CO molecule at a bridge site (benchmark config 1).

    Surface cell: square lattice constant a/sqrt(2), layer spacing a/2, layer k
    shifted by (1/2, 1/2) of the surface cell on odd k, ``vacuum`` Angstrom of empty
    space below and above the slab. C sits ``height`` above the midpoint of two
    neighbouring top-layer atoms, O ``co_bond`` above C along z. Periodic in all
    three directions (vacuum separates the slab images along z)."""
    nx, ny, nl = size
    d = a / np.sqrt(2.0)
    dz = a / 2.0
    pos = []
    for k in range(nl):
        off = 0.5 * (k % 2)
        for ix in range(nx):
            for iy in range(ny):
                pos.append([(ix + off) * d, (iy + off) * d, vacuum + k * dz])
    pos = np.array(pos, dtype=np.float64)
    top = pos[-nx * ny:]
    z_top = top[0, 2]
    bridge = np.array([top[0, 0] + 0.5 * d, top[0, 1], z_top + height])
    pos = np.concatenate([pos, bridge[None], (bridge + np.array([0, 0, co_bond]))[None]])
    numbers = np.array([29] * (nx * ny * nl) + [6, 8], dtype=np.int64)
    cell = np.diag([nx * d, ny * d, (nl - 1) * dz + 2 * vacuum])
    if jitter > 0:
        pos = pos + np.random.default_rng(seed).normal(0.0, jitter, pos.shape)
    return AtomicSystem(pos, numbers, cell, name="cu_fcc100_3x3x3_co_bridge")


def water_box(n_mol: int = 3333, density: float = 1.0, oh: float = 0.96, angle_deg: float = 104.5,
              jitter: float = 0.1, seed: int = 0) -> AtomicSystem:
    """Periodic cubic water box: molecules on a jittered simple-cubic lattice with
    uniformly random orientations (benchmark config 4)."""
    rng = np.random.default_rng(seed)
    mass_g = n_mol * 18.015 / 6.02214076e23
    L = (mass_g / density * 1e24) ** (1.0 / 3.0)  # Angstrom
    m = int(np.ceil(n_mol ** (1.0 / 3.0)))
    sites = np.stack(np.meshgrid(np.arange(m), np.arange(m), np.arange(m), indexing="ij"), -1).reshape(-1, 3)
    sites = sites[rng.permutation(len(sites))[:n_mol]]
    centers = (sites + 0.5) * (L / m) + rng.normal(0.0, jitter, (n_mol, 3))
    half = np.deg2rad(angle_deg) / 2.0
    local = np.array([[0.0, 0.0, 0.0],
                      [oh * np.sin(half), oh * np.cos(half), 0.0],
                      [-oh * np.sin(half), oh * np.cos(half), 0.0]])
    # random rotations from uniformly distributed unit quaternions
    q = rng.normal(size=(n_mol, 4))
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    w, x, y, z = q.T
    R = np.stack([
        np.stack([1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)], -1),
        np.stack([2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)], -1),
        np.stack([2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)], -1),
    ], 1)
    pos = centers[:, None, :] + np.einsum("nij,kj->nki", R, local)
    pos = np.mod(pos.reshape(-1, 3), L)
    numbers = np.tile(np.array([8, 1, 1], dtype=np.int64), n_mol)
    return AtomicSystem(pos, numbers, np.diag([L, L, L]), name=f"water_{n_mol}")


def _sq3(v: np.ndarray) -> np.ndarray:
    """Squared length over the last axis (3) in a fixed order, (x^2 + z^2) + y^2, each operation
    rounded once (no fused multiply-add), so that the device list (fuma_neighbor_list) computes
    the same bits. (This is the order numpy's einsum("...k,...k") uses here, with which the
    committed fixtures' graphs were built.)"""
    return (v[..., 0] * v[..., 0] + v[..., 2] * v[..., 2]) + v[..., 1] * v[..., 1]


def neighbor_list(system: AtomicSystem, cutoff: float = 6.0, max_neighbors: int = 30):
    """Deterministic capped periodic neighbour list (see module docstring).

    Returns ``edge_index`` [2, E] int64 (row 0 source i, row 1 destination j),
    ``cell_offsets`` [E, 3] int64, ``distances`` [E] float64; edges sorted by
    destination then by (distance, source, offset)."""
    pos = np.asarray(system.positions, dtype=np.float64)
    cell = np.asarray(system.cell, dtype=np.float64)
    n = len(pos)
    inv = np.linalg.inv(cell)
    frac = pos @ inv
    # images needed along each lattice direction: cutoff / distance between opposite faces
    vol = abs(np.linalg.det(cell))
    face = np.array([vol / np.linalg.norm(np.cross(cell[(k + 1) % 3], cell[(k + 2) % 3])) for k in range(3)])
    reps = [int(np.ceil(cutoff / face[k])) if system.pbc[k] else 0 for k in range(3)]
    # bin atoms (wrapped into the cell) into cubes of side >= cutoff in fractional space
    wrapped = frac - np.floor(frac)
    wrap_shift = np.floor(frac).astype(np.int64)  # pos = wrapped@cell + wrap_shift@cell
    nb = np.maximum(1, np.floor(face / cutoff).astype(np.int64))
    b = np.minimum((wrapped * nb).astype(np.int64), nb - 1)
    bid = (b[:, 0] * nb[1] + b[:, 1]) * nb[2] + b[:, 2]
    order = np.argsort(bid, kind="stable")
    counts = np.bincount(bid, minlength=int(np.prod(nb)))
    starts = np.concatenate([[0], np.cumsum(counts)])
    wpos = wrapped @ cell

    src_l, dst_l, off_l, dist_l = [], [], [], []
    # for each destination bin, visit neighbouring bins (with periodic image shifts)
    rng_k = [range(-1, 2) if (nb[k] > 2 or not system.pbc[k]) else range(-reps[k] - 1, reps[k] + 2) for k in range(3)]
    for bx in range(nb[0]):
        for by in range(nb[1]):
            for bz in range(nb[2]):
                d_ids = order[starts[(bx * nb[1] + by) * nb[2] + bz]: starts[(bx * nb[1] + by) * nb[2] + bz + 1]]
                if len(d_ids) == 0:
                    continue
                for dx in rng_k[0]:
                    for dy in rng_k[1]:
                        for dz in rng_k[2]:
                            cx, cy, cz = bx + dx, by + dy, bz + dz
                            ix, iy, iz = cx % nb[0], cy % nb[1], cz % nb[2]
                            img = np.array([(cx - ix) // nb[0], (cy - iy) // nb[1], (cz - iz) // nb[2]])
                            if not system.pbc[0] and img[0] != 0: continue
                            if not system.pbc[1] and img[1] != 0: continue
                            if not system.pbc[2] and img[2] != 0: continue
                            s_bin = (ix * nb[1] + iy) * nb[2] + iz
                            s_ids = order[starts[s_bin]: starts[s_bin + 1]]
                            if len(s_ids) == 0:
                                continue
                            shift = img @ cell
                            vec = wpos[s_ids][None, :, :] + shift[None, None, :] - wpos[d_ids][:, None, :]
                            d2 = _sq3(vec)
                            dd, ss = np.nonzero(d2 < cutoff * cutoff)
                            si, di = s_ids[ss], d_ids[dd]
                            keep = ~((si == di) & np.all(img == 0))
                            if not keep.any():
                                continue
                            si, di = si[keep], di[keep]
                            # integer offset in terms of the ORIGINAL (unwrapped) positions
                            off = img[None, :] + wrap_shift[di] - wrap_shift[si]
                            src_l.append(si); dst_l.append(di); off_l.append(off)
                            dist_l.append(np.sqrt(d2[dd[keep], ss[keep]]))
    if not src_l:
        z = np.zeros(0, dtype=np.int64)
        return np.zeros((2, 0), np.int64), np.zeros((0, 3), np.int64), np.zeros(0)
    src = np.concatenate(src_l); dst = np.concatenate(dst_l)
    off = np.concatenate(off_l).astype(np.int64); dist = np.concatenate(dist_l)
    # recompute the distance from the unwrapped positions and offsets (what the model sees)
    vec = pos[src] - pos[dst] + off @ cell
    dist = np.sqrt(_sq3(vec))
    order = np.lexsort((off[:, 2], off[:, 1], off[:, 0], src, dist, dst))
    src, dst, off, dist = src[order], dst[order], off[order], dist[order]
    # rank within each destination and cap
    first = np.searchsorted(dst, np.arange(n))
    rank = np.arange(len(dst)) - first[dst]
    keep = (rank < max_neighbors) & (dist < cutoff)
    return np.stack([src[keep], dst[keep]]), off[keep], dist[keep]


@dataclass
class AtomicGraph:
    """Minimal stand-in for FAIRChem's ``AtomicData`` with the fields the backbone reads
    (``wrapper.py:171-210``): pos, atomic_numbers, cell [nsys,3,3], cell_offsets [E,3],
    edge_index [2,E], natoms, nedges, charge, spin, batch, optional dataset."""
    pos: torch.Tensor
    atomic_numbers: torch.Tensor
    cell: torch.Tensor
    cell_offsets: torch.Tensor
    edge_index: torch.Tensor
    natoms: torch.Tensor
    nedges: torch.Tensor
    charge: torch.Tensor
    spin: torch.Tensor
    batch: torch.Tensor
    dataset: Optional[list] = None
    extra: dict = field(default_factory=dict)

    def to(self, device) -> "AtomicGraph":
        kw = {k: (v.to(device) if isinstance(v, torch.Tensor) else v) for k, v in self.__dict__.items()}
        return AtomicGraph(**kw)

    def clone(self) -> "AtomicGraph":
        kw = {k: (v.clone() if isinstance(v, torch.Tensor) else v) for k, v in self.__dict__.items()}
        return AtomicGraph(**kw)


def to_graph(systems, cutoff: float = 6.0, max_neighbors: int = 30, dtype=torch.float32) -> AtomicGraph:
    """Batch one or more systems into an ``AtomicGraph`` (edges of system k point into system k)."""
    if isinstance(systems, AtomicSystem):
        systems = [systems]
    pos, Z, cells, offs, eidx, natoms, nedges, batch, charge, spin = [], [], [], [], [], [], [], [], [], []
    base = 0
    for k, s in enumerate(systems):
        ei, off, _ = neighbor_list(s, cutoff, max_neighbors)
        pos.append(s.positions); Z.append(s.numbers); cells.append(s.cell)
        offs.append(off); eidx.append(ei + base); natoms.append(s.natoms); nedges.append(ei.shape[1])
        batch.append(np.full(s.natoms, k)); charge.append(s.charge); spin.append(s.spin)
        base += s.natoms
    return AtomicGraph(
        pos=torch.tensor(np.concatenate(pos), dtype=dtype),
        atomic_numbers=torch.tensor(np.concatenate(Z), dtype=torch.long),
        cell=torch.tensor(np.stack(cells), dtype=dtype),
        cell_offsets=torch.tensor(np.concatenate(offs), dtype=dtype),
        edge_index=torch.tensor(np.concatenate(eidx, axis=1), dtype=torch.long),
        natoms=torch.tensor(natoms, dtype=torch.long),
        nedges=torch.tensor(nedges, dtype=torch.long),
        charge=torch.tensor(charge, dtype=torch.long),
        spin=torch.tensor(spin, dtype=torch.long),
        batch=torch.tensor(np.concatenate(batch), dtype=torch.long),
    )


def random_cluster_graph(num_atoms: int, degree: int = 50, cutoff: float = 6.0, seed: int = 0,
                         dtype=torch.float32) -> AtomicGraph:
    """Random non-periodic cluster with exactly ``num_atoms * degree`` directed edges: uniform
    positions in a cube, scaled so that the (N * degree)-th smallest distance between distinct
    atoms sits just inside the cutoff; every ordered pair closer than the cutoff is an edge (no
    per-atom cap), emitted by destination. Random atomic numbers 1..99. The same workload shape
    as the reference's atom-count sweep (random graphs of fixed mean degree); the cell is a
    cube enclosing the cluster (used only for the stress normalisation)."""
    rng = np.random.default_rng(seed)
    pos = rng.random((num_atoms, 3))
    d = np.sqrt(((pos[:, None, :] - pos[None, :, :]) ** 2).sum(-1))
    np.fill_diagonal(d, np.inf)
    k = min(num_atoms * degree, num_atoms * (num_atoms - 1))
    kth = np.partition(d.ravel(), k - 1)[k - 1]
    scale = (cutoff - 1e-4) / kth
    pos = pos * scale
    d = d * scale
    dst, src = np.nonzero(d.T < cutoff)          # rows of d.T are destinations: emitted by destination
    E = src.shape[0]
    side = float(pos.max() + cutoff)
    return AtomicGraph(
        pos=torch.tensor(pos, dtype=dtype),
        atomic_numbers=torch.tensor(rng.integers(1, 100, num_atoms), dtype=torch.long),
        cell=torch.tensor(np.eye(3)[None] * side, dtype=dtype),
        cell_offsets=torch.zeros(E, 3, dtype=dtype),
        edge_index=torch.tensor(np.stack([src, dst]), dtype=torch.long),
        natoms=torch.tensor([num_atoms], dtype=torch.long),
        nedges=torch.tensor([E], dtype=torch.long),
        charge=torch.zeros(1, dtype=torch.long),
        spin=torch.zeros(1, dtype=torch.long),
        batch=torch.zeros(num_atoms, dtype=torch.long),
    )


# ---- benchmark configurations (BASELINE.json "configs") --------------------------------------

def config1_system() -> AtomicSystem:
    """Cu fcc100 3x3x3 slab + CO at a bridge site, 29 atoms, jitter N(0, 0.02), seed 0."""
    return cu_fcc100_slab_co()


def config3_system() -> AtomicSystem:
    """Bulk fcc Cu 10x10x10 conventional (4,000 atoms), displacements N(0, 0.05), seed 0."""
    return bulk_fcc(10, 10, 10, jitter=0.05, seed=0, name="bulk_cu_4000")


def config4_system() -> AtomicSystem:
    """3,333 H2O at 1.0 g/cm^3 (~10k atoms), seed 0."""
    return water_box()


def config5_system() -> AtomicSystem:
    """Bulk fcc Cu 30x30x28 conventional (100,800 atoms), displacements N(0, 0.05), seed 0."""
    return bulk_fcc(30, 30, 28, jitter=0.05, seed=0, name="bulk_cu_100800")


def microbench_layer_inputs(N: int = 20000, E: int = 600000, C: int = 128, seed: int = 0):
    """Benchmark config 2 (one message-passing layer): src/dst uniform random int32 sorted
    by dst, unit edge vectors uniform on the sphere, distances U(0.8, 6.0). All atoms sit at
    the origin and the per-edge shift carries the edge vector, so the geometry stage sees
    exactly these vectors. Returns CPU tensors."""
    g = torch.Generator().manual_seed(seed)
    dst = torch.randint(0, N, (E,), generator=g, dtype=torch.int64)
    src = torch.randint(0, N, (E,), generator=g, dtype=torch.int64)
    dst, order = torch.sort(dst, stable=True)
    src = src[order]
    u = torch.randn(E, 3, generator=g, dtype=torch.float64)
    u = u / u.norm(dim=1, keepdim=True)
    d = torch.rand(E, generator=g, dtype=torch.float64) * (6.0 - 0.8) + 0.8
    shifts = (u * d[:, None]).to(torch.float32)
    x = torch.randn(N, 9, C, generator=g)
    return dict(N=N, E=E, C=C, idx_i=src, idx_j=dst, shifts=shifts, pos=torch.zeros(N, 3), x=x)
