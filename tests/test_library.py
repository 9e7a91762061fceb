"""The ``fuma::`` custom operators (``flash_uma_b200.library``) without a GPU: every op and its
backward are registered with the reference's argument order, and their fake (meta)
implementations give the reference's output shapes, also with symbolic sizes, which is what
``torch.compile`` traces through."""
import torch
from torch._subclasses.fake_tensor import FakeTensorMode
from torch.fx.experimental.symbolic_shapes import ShapeEnv

import flash_uma_b200.library  # noqa: F401

OPS = ["precompute_geometry", "precompute_geometry_bwd", "layer_norm_silu", "layer_norm_silu_bwd",
       "gather_wigner_split", "gather_wigner_split_bwd", "fused_gating_split", "fused_gating_split_bwd",
       "rotate_scatter_split", "rotate_scatter_split_bwd", "init_node_scatter", "init_node_scatter_bwd"]


def test_all_ops_registered():
    for name in OPS:
        assert hasattr(torch.ops.fuma, name), name


def _shapes(mode, E, N, C=16, B=8):
    f, i64, i32 = torch.float32, torch.long, torch.int32
    with mode:
        pos, Z = torch.empty(N, 3), torch.zeros(N, dtype=i64)
        ii = torch.zeros(E, dtype=i64)
        xe, wig, env = torch.ops.fuma.precompute_geometry(pos, Z, ii, ii, torch.empty(E, 3), torch.empty(100, C),
                                                          torch.empty(100, C), torch.empty(B), -1.0, 6.0,
                                                          None, None, None, None)
        y, mean, rstd = torch.ops.fuma.layer_norm_silu(torch.empty(E, C), torch.empty(C), torch.empty(C), 1e-7)
        X = torch.ops.fuma.gather_wigner_split(torch.empty(N, 9, C), ii, ii, wig, torch.empty(E, 12 * C),
                                               torch.empty(1, C), Z, None, None, None, None)
        Zs = torch.ops.fuma.fused_gating_split(torch.empty(E, 5 * C), torch.empty(E, 4 * C), torch.empty(E, 2 * C), C)
        rp, ci = torch.zeros(N + 1, dtype=i32), torch.zeros(E, dtype=i32)
        out = torch.ops.fuma.rotate_scatter_split(*Zs, wig, env, torch.empty(N, 9, C), rp, ci, N)
        x0 = torch.ops.fuma.init_node_scatter(torch.empty(E, 3 * C), wig, env, Z, Z, torch.empty(100, C),
                                              torch.empty(1, C), rp, ci, N)
        gs = torch.ops.fuma.rotate_scatter_split_bwd(torch.empty(N, 9, C), *Zs, wig, env, rp, ci)
    return dict(xe=xe.shape, wig=wig.shape, env=env.shape, y=y.shape, mean=mean.shape, X=[t.shape for t in X],
                Z=[t.shape for t in Zs], out=out.shape, x0=x0.shape, gs=[t.shape for t in gs], dtype=out.dtype)


def test_fake_shapes():
    s = _shapes(FakeTensorMode(), E=40, N=10)
    assert s["xe"] == (40, 8 + 32) and s["wig"] == (40, 34) and s["env"] == (40,)
    assert s["y"] == (40, 16) and s["mean"] == (40,)
    assert s["X"] == [(40, 96), (40, 128), (40, 64)] and s["Z"] == [(40, 48), (40, 64), (40, 32)]
    assert s["out"] == (10, 9, 16) and s["x0"] == (10, 9, 16)
    assert s["gs"] == [(40, 48), (40, 64), (40, 32), (40, 34), (40,)] and s["dtype"] == torch.float32


def test_fake_shapes_symbolic():
    """Dynamic shapes: the edge and atom counts stay symbolic through every fake kernel."""
    mode = FakeTensorMode(shape_env=ShapeEnv())
    with mode:
        e = mode.shape_env.create_unbacked_symint()
    torch._check(e >= 0)
    s = _shapes(mode, E=e, N=10)
    assert str(s["X"][0][0]) == str(e) and s["X"][0][1] == 96
