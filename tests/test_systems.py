"""Structure generators and the deterministic capped periodic neighbour list (CPU)."""
import itertools

import numpy as np

from flash_uma_b200 import systems as S


def brute_force(system, cutoff, max_nb):
    pos, cell = system.positions, system.cell
    rows = []
    rng = range(-3, 4)
    for j in range(len(pos)):
        cand = []
        for i in range(len(pos)):
            for s in itertools.product(rng, rng, rng):
                if i == j and s == (0, 0, 0):
                    continue
                v = pos[i] - pos[j] + np.array(s) @ cell
                d = float(np.sqrt((v[0] * v[0] + v[2] * v[2]) + v[1] * v[1]))   # the rule's fixed order
                if d < cutoff:
                    cand.append((d, i, s))
        cand.sort()
        rows += [(i, j, s) for d, i, s in cand[:max_nb]]
    return rows


def test_neighbor_list_matches_brute_force():
    sysm = S.water_box(n_mol=6, seed=2)          # tiny periodic box: many periodic images
    ei, off, dist = S.neighbor_list(sysm, cutoff=4.0, max_neighbors=12)
    got = [(int(a), int(b), tuple(int(x) for x in o)) for a, b, o in zip(ei[0], ei[1], off)]
    assert got == brute_force(sysm, 4.0, 12)


def test_neighbor_list_properties_and_determinism():
    sysm = S.bulk_fcc(4, 4, 4, jitter=0.05, seed=1)
    ei, off, dist = S.neighbor_list(sysm, 6.0, 30)
    ei2, off2, _ = S.neighbor_list(sysm, 6.0, 30)
    assert np.array_equal(ei, ei2) and np.array_equal(off, off2)
    assert (dist < 6.0).all() and (dist > 0.5).all()
    assert np.all(np.diff(ei[1]) >= 0)                      # sorted by destination
    counts = np.bincount(ei[1], minlength=sysm.natoms)
    assert counts.max() == 30 and counts.min() == 30          # fcc has 78 neighbours inside 6 A
    vec = sysm.positions[ei[0]] - sysm.positions[ei[1]] + off @ sysm.cell
    np.testing.assert_allclose(np.linalg.norm(vec, axis=1), dist, rtol=1e-12)


def test_uncapped_list_is_symmetric():
    sysm = S.bulk_fcc(3, 3, 3, jitter=0.05, seed=3)
    ei, off, _ = S.neighbor_list(sysm, 5.0, 10_000)
    fwd = {(int(a), int(b), tuple(o)) for a, b, o in zip(ei[0], ei[1], off.tolist())}
    assert all((b, a, tuple(-x for x in o)) in fwd for a, b, o in fwd)


def test_benchmark_configs():
    c1 = S.config1_system()
    assert c1.natoms == 29 and list(c1.numbers[-2:]) == [6, 8]
    g1 = S.to_graph([c1])
    assert g1.edge_index.shape[1] <= 29 * 30
    c3 = S.config3_system()
    assert c3.natoms == 4000
    ei, _, _ = S.neighbor_list(c3, 6.0, 30)
    assert ei.shape[1] == 120_000
    w = S.water_box()
    assert w.natoms == 9999 and abs(w.cell[0, 0] - 46.4) < 0.1


def test_microbench_inputs():
    m = S.microbench_layer_inputs(N=2000, E=60000)
    assert m["idx_j"].shape == (60000,) and bool((m["idx_j"][1:] >= m["idx_j"][:-1]).all())
    d = m["shifts"].double().norm(dim=1)
    assert float(d.min()) >= 0.8 - 1e-5 and float(d.max()) <= 6.0 + 1e-5
