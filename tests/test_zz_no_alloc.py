"""fuma_gather_bwd_noalloc: the allocation-free gather backward, called through the C ABI.

This entry point serves callers that cannot let the library allocate device memory (for
example host frameworks that own the device memory budget, or steps that must not be
serialised by cudaMalloc): its scratch lives in a 32 MiB array built into the library. The
test checks it against fuma_gather_bwd, which takes a caller-provided scratch buffer, on
two consecutive calls with different inputs (the shared array keeps the previous call's
contents), and checks that oversized calls are refused. Collected last on purpose, and
independent of the other test files (passes alone or after them)."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
TOL = 2e-5  # same bound as the gather-backward parity tests (relative to the max magnitude)


def _inputs(seed, N=60, E=400, C=32):
    g = torch.Generator().manual_seed(seed)
    idx_i = torch.randint(0, N, (E,), generator=g)
    idx_j = torch.randint(0, N, (E,), generator=g)
    q = torch.randn(E, 4, generator=g)
    q = q / q.norm(dim=1, keepdim=True)
    w, x_, y, z = q.T
    R = torch.stack([1 - 2 * (y * y + z * z), 2 * (x_ * y - w * z), 2 * (x_ * z + w * y),
                     2 * (x_ * y + w * z), 1 - 2 * (x_ * x_ + z * z), 2 * (y * z - w * x_),
                     2 * (x_ * z - w * y), 2 * (y * z + w * x_), 1 - 2 * (x_ * x_ + y * y)], 1)
    wig = torch.cat([R, torch.randn(E, 25, generator=g) * 0.4], 1)
    return dict(
        N=N, E=E, C=C, idx_i=idx_i, idx_j=idx_j, wig=wig,
        x=torch.randn(N, 9, C, generator=g), rad=torch.randn(E, 12 * C, generator=g),
        csd=torch.randn(2, C, generator=g), batch=(torch.arange(N) >= N // 2).long(),
        g0=torch.randn(E, 6 * C, generator=g), g1=torch.randn(E, 8 * C, generator=g),
        g2=torch.randn(E, 4 * C, generator=g))


def _call_both(lib, I):
    from flash_uma_b200.ops import build_graph_csr
    d = {k: (v.to(DEV).contiguous() if isinstance(v, torch.Tensor) else v) for k, v in I.items()}
    gr = build_graph_csr(d["idx_i"], d["idx_j"], I["N"])
    N, E, C = I["N"], I["E"], I["C"]
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    common = [p(d["g0"]), p(d["g1"]), p(d["g2"]), p(d["x"]), p(d["idx_i"]), p(d["wig"]), p(d["rad"]), p(d["csd"]),
              p(d["batch"]), p(gr.dst_row_ptr), p(gr.dst_col), p(gr.src_row_ptr), p(gr.src_col),
              ctypes.c_int64(N), ctypes.c_int64(E), ctypes.c_int32(C)]
    outs = {}
    for name in ("ref", "noalloc"):
        gx = torch.full((N, 9, C), float("nan"), device=DEV)
        gw = torch.full((E, 34), float("nan"), device=DEV)
        grad = torch.full((E, 12 * C), float("nan"), device=DEV)
        if name == "ref":
            scratch = torch.empty(E * 9 * C, device=DEV)
            rc = lib.fuma_gather_bwd(*common, p(scratch), ctypes.c_int64(scratch.numel()), p(gx), p(gw), p(grad),
                                     stream)
        else:
            rc = lib.fuma_gather_bwd_noalloc(*common, p(gx), p(gw), p(grad), stream)
        assert rc == 0, lib.fuma_last_error()
        outs[name] = (gx, gw, grad)
    torch.cuda.synchronize()
    return outs


@pytest.fixture(scope="module")
def lib():
    from flash_uma_b200 import _native
    return _native.load()


def test_noalloc_matches_allocating_entry_point_twice(lib):
    for seed in (11, 12):   # two calls in a row: the shared scratch still holds the first call's rows
        outs = _call_both(lib, _inputs(seed))
        for a, b in zip(outs["noalloc"], outs["ref"]):
            assert torch.isfinite(a).all()
            assert (a - b).abs().max().item() <= TOL * max(1.0, b.abs().max().item())


def test_noalloc_refuses_oversized_calls(lib):
    from flash_uma_b200._native import _SIGS  # noqa: F401  (signatures set by load())
    C, E = 128, 8000                       # 8000 * 9 * 128 floats > 8 Mi-float capacity
    rc = lib.fuma_gather_bwd_noalloc(*([ctypes.c_void_p(16)] * 13), ctypes.c_int64(10), ctypes.c_int64(E),
                                     ctypes.c_int32(C), *([ctypes.c_void_p(16)] * 3), ctypes.c_void_p(0))
    assert rc == -1
    assert b"scratch" in lib.fuma_last_error()
