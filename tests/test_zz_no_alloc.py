"""fuma_morton_reorder_noalloc, the allocation-free Morton reorder, called through the C ABI.

Some callers cannot allocate device memory, or lend a device allocator, at the point where they
call in (host programs that own the whole device memory budget, steps that must not be
serialised by cudaMalloc, bindings that only pass the caller's arrays). For them this entry
point keeps the radix sort's scratch in an array built into the library instead of taking a
scratch buffer. The test calls it and the allocating entry point (fuma_morton_reorder, with a
scratch buffer from the caller) on the same inputs, twice in a row with different systems (the
built-in array keeps the first call's contents when the second one starts), above 16,384 atoms
so the multi-block radix sort (which uses the scratch) runs; the integer outputs must agree
bit for bit, as in the other Morton tests. It also checks that a system beyond the array's
524,288-atom limit is refused before anything is launched. Collected last on purpose (a failure
here leaves every other test already run) and independent of the other test files."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


@pytest.fixture(scope="module")
def lib():
    from flash_uma_b200 import _native
    return _native.load()


def _system(N, E, nsys, seed):
    g = torch.Generator().manual_seed(seed)
    pos = torch.rand(N, 3, generator=g) * 40.0
    pos[N // 3:N // 3 + 7] = pos[11]                                   # equal keys
    batch = torch.sort(torch.randint(0, nsys, (N,), generator=g))[0]
    Z = torch.randint(1, 90, (N,), generator=g)
    idx = torch.randint(0, N, (2, E), generator=g)
    return [t.to(DEV).contiguous() for t in (pos, Z, batch, idx[0], idx[1])]


def _outputs(N, E):
    i64 = dict(device=DEV, dtype=torch.int64)
    return [torch.full((N,), -5, **i64), torch.full((N,), -5, **i64), torch.full((N, 3), float("nan"), device=DEV),
            torch.full((N,), -5, **i64), torch.full((N,), -5, **i64), torch.full((E,), -5, **i64),
            torch.full((E,), -5, **i64)]


def _call(lib, inputs, noalloc):
    pos, Z, batch, ii, jj = inputs
    N, E = pos.shape[0], ii.shape[0]
    perm, inv, pos_s, Z_s, b_s, ii_s, jj_s = out = _outputs(N, E)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    p = lambda t: ctypes.c_void_p(t.data_ptr())   # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = [p(pos), p(Z), p(batch), p(ii), p(jj), ctypes.c_int64(N), ctypes.c_int64(E), p(perm), p(inv), p(pos_s),
            p(Z_s), p(b_s), p(ii_s), p(jj_s)]
    if noalloc:
        rc = lib.fuma_morton_reorder_noalloc(*args, p(err), stream)
        keep = None
    else:
        nbytes = int(lib.fuma_morton_scratch_bytes(N))
        keep = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=DEV)
        rc = lib.fuma_morton_reorder(*args, p(keep), ctypes.c_int64(nbytes), p(err), stream)
    assert rc == 0, lib.fuma_last_error()
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out


def test_noalloc_matches_allocating_entry_point_twice(lib):
    for N, E, nsys, seed in ((100800, 300000, 1, 1), (40000, 90000, 300, 2), (5000, 20000, 2, 3)):
        a = _call(lib, _system(N, E, nsys, seed), noalloc=True)
        b = _call(lib, _system(N, E, nsys, seed), noalloc=False)
        for x, y in zip(a, b):
            assert torch.equal(x, y)
        assert sorted(a[0].tolist()) == list(range(N))   # a permutation


def test_noalloc_refuses_systems_beyond_its_array(lib):
    N = (1 << 19) + 1
    rc = lib.fuma_morton_reorder_noalloc(*([ctypes.c_void_p(16)] * 5), ctypes.c_int64(N), ctypes.c_int64(0),
                                         *([ctypes.c_void_p(16)] * 8), ctypes.c_void_p(0))
    assert rc == -1
    assert b"524288" in lib.fuma_last_error()
