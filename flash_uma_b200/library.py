"""The reference's six fused ops as ``torch.library`` custom operators (namespace ``fuma``).

The reference publishes its timings with ``torch.compile(dynamic=True)`` (``readme.md:15,70``).
Its ops are ``torch.autograd.Function``s launching Triton kernels, which Dynamo traces. Here the
kernels sit behind a C ABI (ctypes), which Dynamo cannot trace, so each op is registered as an
opaque custom operator with:

* a real implementation that calls the C ABI (``_native.call``) on the current stream,
* a fake (meta) implementation that only computes output shapes (symbolic sizes allowed), so
  ``torch.compile`` / ``torch.export`` can trace through it without running a kernel,
* an autograd formula that calls the op's backward, itself a custom operator.

Forward ops that need extra tensors for the backward (LN-SiLU statistics) return them as
additional outputs; the public wrappers in :mod:`flash_uma_b200.ops` hand back only the
reference's outputs. Shapes, dtypes and semantics follow the reference signatures
(``ops/geom.py:591``, ``ops/ln_silu.py:180``, ``ops/gather.py:516``, ``ops/gating.py:236``,
``ops/scatter.py:354``, ``ops/scatter.py:527``).
"""
from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor
from torch.library import custom_op

from . import _native as nat
from ._native import ptr, stream_of


def _csr(idx: Tensor, N: int):
    order = torch.argsort(idx, stable=True)
    bounds = torch.arange(N + 1, device=idx.device, dtype=idx.dtype)
    return torch.searchsorted(idx[order], bounds).to(torch.int32), order.to(torch.int32)


def _empty(shape, like, dtype=torch.float32):
    return torch.empty(shape, device=like.device, dtype=dtype)


# ---- geometry --------------------------------------------------------------------------------

@custom_op("fuma::precompute_geometry", mutates_args=())
def precompute_geometry(pos: Tensor, Z: Tensor, idx_i: Tensor, idx_j: Tensor, shifts: Tensor, W_src: Tensor,
                        W_tgt: Tensor, offset_g: Tensor, coeff_g: float, cutoff: float, dst_row_ptr: Optional[Tensor],
                        dst_col: Optional[Tensor], src_row_ptr: Optional[Tensor],
                        src_col: Optional[Tensor]) -> tuple[Tensor, Tensor, Tensor]:
    """(x_edge_raw [E, B+2C], wigner [E, 34], env [E]); the CSRs are only used by the backward."""
    nat.require_cuda(pos, Z, idx_i, idx_j, shifts, W_src, W_tgt, offset_g)
    N, E = pos.shape[0], idx_i.shape[0]
    B, C = offset_g.shape[0], W_src.shape[1]
    x_edge, wigner, env = _empty((E, B + 2 * C), pos), _empty((E, 34), pos), _empty((E,), pos)
    nat.call("fuma_geometry_fwd", ptr(pos), ptr(Z), ptr(idx_i), ptr(idx_j), ptr(shifts), ptr(W_src), ptr(W_tgt),
             ptr(offset_g), float(coeff_g), float(cutoff), N, E, B, C, ptr(x_edge), ptr(wigner), ptr(env),
             stream_of(pos))
    return x_edge, wigner, env


@precompute_geometry.register_fake
def _(pos, Z, idx_i, idx_j, shifts, W_src, W_tgt, offset_g, coeff_g, cutoff, dst_row_ptr, dst_col, src_row_ptr,
      src_col):
    E, B, C = idx_i.shape[0], offset_g.shape[0], W_src.shape[1]
    return pos.new_empty(E, B + 2 * C), pos.new_empty(E, 34), pos.new_empty(E)


@custom_op("fuma::precompute_geometry_bwd", mutates_args=())
def precompute_geometry_bwd(pos: Tensor, idx_i: Tensor, idx_j: Tensor, shifts: Tensor, offset_g: Tensor,
                            coeff_g: float, cutoff: float, g_x_edge: Tensor, g_wigner: Tensor, g_env: Tensor,
                            dst_row_ptr: Optional[Tensor], dst_col: Optional[Tensor], src_row_ptr: Optional[Tensor],
                            src_col: Optional[Tensor]) -> tuple[Tensor, Tensor]:
    """(g_pos [N, 3], g_shifts [E, 3]); CSRs of the edges (built here when not given)."""
    N, E, B = pos.shape[0], idx_i.shape[0], offset_g.shape[0]
    g_x_edge, g_wigner, g_env = g_x_edge.contiguous(), g_wigner.contiguous(), g_env.contiguous()
    g_vec = _empty((E, 3), pos)
    s = stream_of(pos)
    nat.call("fuma_geometry_bwd", ptr(pos), ptr(idx_i), ptr(idx_j), ptr(shifts), ptr(offset_g), float(coeff_g),
             float(cutoff), ptr(g_x_edge), g_x_edge.shape[1], ptr(g_wigner), ptr(g_env), E, B, ptr(g_vec), s)
    if dst_row_ptr is None:
        dst_row_ptr, dst_col = _csr(idx_j, N)
        src_row_ptr, src_col = _csr(idx_i, N)
    g_pos = torch.empty_like(pos)
    nat.call("fuma_edge_vec_to_nodes", ptr(src_row_ptr), ptr(src_col), ptr(dst_row_ptr), ptr(dst_col), ptr(g_vec), N,
             E, ptr(g_pos), s)
    return g_pos, g_vec


@precompute_geometry_bwd.register_fake
def _(pos, idx_i, idx_j, shifts, offset_g, coeff_g, cutoff, g_x_edge, g_wigner, g_env, dst_row_ptr, dst_col,
      src_row_ptr, src_col):
    return torch.empty_like(pos), pos.new_empty(idx_i.shape[0], 3)


def _geom_setup(ctx, inputs, output):
    pos, Z, idx_i, idx_j, shifts, W_src, W_tgt, offset_g, coeff_g, cutoff, dp, dc, sp, sc = inputs
    ctx.save_for_backward(pos, idx_i, idx_j, shifts, offset_g, dp, dc, sp, sc)
    ctx.coeff_g, ctx.cutoff = coeff_g, cutoff


def _geom_backward(ctx, g_xe, g_w, g_env):
    pos, idx_i, idx_j, shifts, offset_g, dp, dc, sp, sc = ctx.saved_tensors
    E, B = idx_i.shape[0], offset_g.shape[0]
    g_xe = g_xe if g_xe is not None else pos.new_zeros(E, B)
    g_w = g_w if g_w is not None else pos.new_zeros(E, 34)
    g_env = g_env if g_env is not None else pos.new_zeros(E)
    g_pos, g_sh = torch.ops.fuma.precompute_geometry_bwd(pos, idx_i, idx_j, shifts, offset_g, ctx.coeff_g, ctx.cutoff,
                                                         g_xe, g_w, g_env, dp, dc, sp, sc)
    return g_pos, None, None, None, g_sh, None, None, None, None, None, None, None, None, None


precompute_geometry.register_autograd(_geom_backward, setup_context=_geom_setup)


# ---- LayerNorm + SiLU --------------------------------------------------------------------------

@custom_op("fuma::layer_norm_silu", mutates_args=())
def layer_norm_silu(x: Tensor, gamma: Tensor, beta: Tensor, eps: float) -> tuple[Tensor, Tensor, Tensor]:
    """(out [M, D], mean [M], rstd [M])."""
    nat.require_cuda(x, gamma, beta)
    M, D = x.shape
    out, mean, rstd = torch.empty_like(x), _empty((M,), x), _empty((M,), x)
    nat.call("fuma_ln_silu_fwd", ptr(x), ptr(gamma), ptr(beta), float(eps), M, D, ptr(out), ptr(mean), ptr(rstd),
             stream_of(x))
    return out, mean, rstd


@layer_norm_silu.register_fake
def _(x, gamma, beta, eps):
    return torch.empty_like(x), x.new_empty(x.shape[0]), x.new_empty(x.shape[0])


@custom_op("fuma::layer_norm_silu_bwd", mutates_args=())
def layer_norm_silu_bwd(x: Tensor, gamma: Tensor, beta: Tensor, mean: Tensor, rstd: Tensor, g_out: Tensor) -> Tensor:
    M, D = x.shape
    g_out = g_out.contiguous()
    g_x = torch.empty_like(x)
    nat.call("fuma_ln_silu_bwd", ptr(x), ptr(gamma), ptr(beta), ptr(mean), ptr(rstd), ptr(g_out), M, D, ptr(g_x),
             stream_of(x))
    return g_x


@layer_norm_silu_bwd.register_fake
def _(x, gamma, beta, mean, rstd, g_out):
    return torch.empty_like(x)


def _ln_setup(ctx, inputs, output):
    x, gamma, beta, _ = inputs
    _, mean, rstd = output
    ctx.save_for_backward(x, gamma, beta, mean, rstd)


def _ln_backward(ctx, g_out, _g_mean, _g_rstd):
    x, gamma, beta, mean, rstd = ctx.saved_tensors
    return torch.ops.fuma.layer_norm_silu_bwd(x, gamma, beta, mean, rstd, g_out), None, None, None


layer_norm_silu.register_autograd(_ln_backward, setup_context=_ln_setup)


# ---- gather + rotate ---------------------------------------------------------------------------

@custom_op("fuma::gather_wigner_split", mutates_args=())
def gather_wigner_split(x_in: Tensor, idx_i: Tensor, idx_j: Tensor, wigner: Tensor, rad_out: Tensor, csd_emb: Tensor,
                        batch: Tensor, dst_row_ptr: Optional[Tensor], dst_col: Optional[Tensor],
                        src_row_ptr: Optional[Tensor], src_col: Optional[Tensor]) -> tuple[Tensor, Tensor, Tensor]:
    """(X_m0 [E, 6C], X_m1 [E, 8C], X_m2 [E, 4C]); the CSRs are only used by the backward."""
    nat.require_cuda(x_in, idx_i, idx_j, wigner, rad_out, csd_emb, batch)
    N, _, C = x_in.shape
    E = idx_i.shape[0]
    X0, X1, X2 = _empty((E, 6 * C), x_in), _empty((E, 8 * C), x_in), _empty((E, 4 * C), x_in)
    nat.call("fuma_gather_fwd", ptr(x_in), ptr(idx_i), ptr(idx_j), ptr(wigner), ptr(rad_out), ptr(csd_emb), ptr(batch),
             N, E, C, ptr(X0), ptr(X1), ptr(X2), stream_of(x_in))
    return X0, X1, X2


@gather_wigner_split.register_fake
def _(x_in, idx_i, idx_j, wigner, rad_out, csd_emb, batch, dst_row_ptr, dst_col, src_row_ptr, src_col):
    E, C = idx_i.shape[0], x_in.shape[2]
    return x_in.new_empty(E, 6 * C), x_in.new_empty(E, 8 * C), x_in.new_empty(E, 4 * C)


@custom_op("fuma::gather_wigner_split_bwd", mutates_args=())
def gather_wigner_split_bwd(g0: Tensor, g1: Tensor, g2: Tensor, x_in: Tensor, idx_i: Tensor, idx_j: Tensor,
                            wigner: Tensor, rad_out: Tensor, csd_emb: Tensor, batch: Tensor,
                            dst_row_ptr: Optional[Tensor], dst_col: Optional[Tensor], src_row_ptr: Optional[Tensor],
                            src_col: Optional[Tensor]) -> tuple[Tensor, Tensor, Tensor]:
    """(g_x [N, 9, C], g_wigner [E, 34], g_rad [E, 12C]), deterministic (no atomics)."""
    N, _, C = x_in.shape
    E = idx_i.shape[0]
    g0, g1, g2 = g0.contiguous(), g1.contiguous(), g2.contiguous()
    if dst_row_ptr is None:
        dst_row_ptr, dst_col = _csr(idx_j, N)
        src_row_ptr, src_col = _csr(idx_i, N)
    g_x, g_w, g_r = torch.empty_like(x_in), _empty((E, 34), x_in), torch.empty_like(rad_out)
    nat.call("fuma_gather_bwd", ptr(g0), ptr(g1), ptr(g2), ptr(x_in), ptr(idx_i), ptr(wigner), ptr(rad_out),
             ptr(csd_emb), ptr(batch), ptr(dst_row_ptr), ptr(dst_col), ptr(src_row_ptr), ptr(src_col), N, E, C, None, 0,
             ptr(g_x), ptr(g_w), ptr(g_r), stream_of(x_in))
    return g_x, g_w, g_r


@gather_wigner_split_bwd.register_fake
def _(g0, g1, g2, x_in, idx_i, idx_j, wigner, rad_out, csd_emb, batch, dst_row_ptr, dst_col, src_row_ptr, src_col):
    return torch.empty_like(x_in), x_in.new_empty(idx_i.shape[0], 34), torch.empty_like(rad_out)


def _gather_setup(ctx, inputs, output):
    ctx.save_for_backward(*inputs)


def _gather_backward(ctx, g0, g1, g2):
    (x_in, idx_i, idx_j, wigner, rad_out, csd_emb, batch, dst_row_ptr, dst_col, src_row_ptr,
     src_col) = ctx.saved_tensors
    E, C = idx_i.shape[0], x_in.shape[2]
    g0 = g0 if g0 is not None else x_in.new_zeros(E, 6 * C)
    g1 = g1 if g1 is not None else x_in.new_zeros(E, 8 * C)
    g2 = g2 if g2 is not None else x_in.new_zeros(E, 4 * C)
    g_x, g_w, g_r = torch.ops.fuma.gather_wigner_split_bwd(g0, g1, g2, x_in, idx_i, idx_j, wigner, rad_out, csd_emb,
                                                          batch, dst_row_ptr, dst_col, src_row_ptr, src_col)
    return g_x, None, None, g_w, g_r, None, None, None, None, None, None


gather_wigner_split.register_autograd(_gather_backward, setup_context=_gather_setup)


# ---- gating ------------------------------------------------------------------------------------

@custom_op("fuma::fused_gating_split", mutates_args=())
def fused_gating_split(Y0: Tensor, Y1: Tensor, Y2: Tensor, C: int) -> tuple[Tensor, Tensor, Tensor]:
    nat.require_cuda(Y0, Y1, Y2)
    E = Y0.shape[0]
    Z0, Z1, Z2 = _empty((E, 3 * C), Y0), _empty((E, 4 * C), Y0), _empty((E, 2 * C), Y0)
    nat.call("fuma_gating_fwd", ptr(Y0), ptr(Y1), ptr(Y2), E, C, ptr(Z0), ptr(Z1), ptr(Z2), stream_of(Y0))
    return Z0, Z1, Z2


@fused_gating_split.register_fake
def _(Y0, Y1, Y2, C):
    E = Y0.shape[0]
    return Y0.new_empty(E, 3 * C), Y0.new_empty(E, 4 * C), Y0.new_empty(E, 2 * C)


@custom_op("fuma::fused_gating_split_bwd", mutates_args=())
def fused_gating_split_bwd(g0: Tensor, g1: Tensor, g2: Tensor, Y0: Tensor, Y1: Tensor, Y2: Tensor,
                           C: int) -> tuple[Tensor, Tensor, Tensor]:
    E = Y0.shape[0]
    g0, g1, g2 = g0.contiguous(), g1.contiguous(), g2.contiguous()
    gY0, gY1, gY2 = torch.empty_like(Y0), torch.empty_like(Y1), torch.empty_like(Y2)
    nat.call("fuma_gating_bwd", ptr(g0), ptr(g1), ptr(g2), ptr(Y0), ptr(Y1), ptr(Y2), E, C, ptr(gY0), ptr(gY1),
             ptr(gY2), stream_of(Y0))
    return gY0, gY1, gY2


@fused_gating_split_bwd.register_fake
def _(g0, g1, g2, Y0, Y1, Y2, C):
    return torch.empty_like(Y0), torch.empty_like(Y1), torch.empty_like(Y2)


def _gating_setup(ctx, inputs, output):
    Y0, Y1, Y2, C = inputs
    ctx.save_for_backward(Y0, Y1, Y2)
    ctx.C = C


def _gating_backward(ctx, g0, g1, g2):
    Y0, Y1, Y2 = ctx.saved_tensors
    E, C = Y0.shape[0], ctx.C
    g0 = g0 if g0 is not None else Y0.new_zeros(E, 3 * C)
    g1 = g1 if g1 is not None else Y0.new_zeros(E, 4 * C)
    g2 = g2 if g2 is not None else Y0.new_zeros(E, 2 * C)
    gY0, gY1, gY2 = torch.ops.fuma.fused_gating_split_bwd(g0, g1, g2, Y0, Y1, Y2, C)
    return gY0, gY1, gY2, None


fused_gating_split.register_autograd(_gating_backward, setup_context=_gating_setup)


# ---- rotate back + scatter -----------------------------------------------------------------------

@custom_op("fuma::rotate_scatter_split", mutates_args=())
def rotate_scatter_split(Z0: Tensor, Z1: Tensor, Z2: Tensor, wigner: Tensor, env: Tensor, x_res: Tensor,
                         row_ptr: Tensor, col_idx: Tensor, N: int) -> Tensor:
    nat.require_cuda(Z0, Z1, Z2, wigner, env, x_res, row_ptr, col_idx)
    E, C = Z0.shape[0], Z0.shape[1] // 3
    x_out = _empty((N, 9, C), Z0)
    nat.call("fuma_rotate_scatter_fwd", ptr(Z0), ptr(Z1), ptr(Z2), ptr(wigner), ptr(env), ptr(x_res), ptr(row_ptr),
             ptr(col_idx), N, E, C, ptr(x_out), stream_of(Z0))
    return x_out


@rotate_scatter_split.register_fake
def _(Z0, Z1, Z2, wigner, env, x_res, row_ptr, col_idx, N):
    return Z0.new_empty(N, 9, Z0.shape[1] // 3)


@custom_op("fuma::rotate_scatter_split_bwd", mutates_args=())
def rotate_scatter_split_bwd(g_out: Tensor, Z0: Tensor, Z1: Tensor, Z2: Tensor, wigner: Tensor, env: Tensor,
                             row_ptr: Tensor, col_idx: Tensor) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """(g_Z0, g_Z1, g_Z2, g_wigner, g_env); the residual's gradient is g_out itself."""
    E, C, N = Z0.shape[0], Z0.shape[1] // 3, g_out.shape[0]
    g_out = g_out.contiguous()
    gZ0, gZ1, gZ2 = torch.empty_like(Z0), torch.empty_like(Z1), torch.empty_like(Z2)
    g_w, g_env = torch.empty_like(wigner), torch.empty_like(env)
    nat.call("fuma_rotate_scatter_bwd", ptr(g_out), ptr(Z0), ptr(Z1), ptr(Z2), ptr(wigner), ptr(env), ptr(row_ptr),
             ptr(col_idx), N, E, C, ptr(gZ0), ptr(gZ1), ptr(gZ2), ptr(g_w), ptr(g_env), stream_of(Z0))
    return gZ0, gZ1, gZ2, g_w, g_env


@rotate_scatter_split_bwd.register_fake
def _(g_out, Z0, Z1, Z2, wigner, env, row_ptr, col_idx):
    return (torch.empty_like(Z0), torch.empty_like(Z1), torch.empty_like(Z2), torch.empty_like(wigner),
            torch.empty_like(env))


def _scatter_setup(ctx, inputs, output):
    Z0, Z1, Z2, wigner, env, x_res, row_ptr, col_idx, N = inputs
    ctx.save_for_backward(Z0, Z1, Z2, wigner, env, row_ptr, col_idx)


def _scatter_backward(ctx, g_out):
    Z0, Z1, Z2, wigner, env, row_ptr, col_idx = ctx.saved_tensors
    gZ0, gZ1, gZ2, g_w, g_env = torch.ops.fuma.rotate_scatter_split_bwd(g_out, Z0, Z1, Z2, wigner, env, row_ptr,
                                                                       col_idx)
    return gZ0, gZ1, gZ2, g_w, g_env, g_out, None, None, None


rotate_scatter_split.register_autograd(_scatter_backward, setup_context=_scatter_setup)


# ---- initial node embedding ---------------------------------------------------------------------

@custom_op("fuma::init_node_scatter", mutates_args=())
def init_node_scatter(rad_out: Tensor, wigner: Tensor, env: Tensor, Z: Tensor, batch: Tensor, W_sphere: Tensor,
                      csd_emb: Tensor, row_ptr: Tensor, col_idx: Tensor, N: int) -> Tensor:
    nat.require_cuda(rad_out, wigner, env, Z, batch, W_sphere, csd_emb, row_ptr, col_idx)
    E, C = rad_out.shape[0], rad_out.shape[1] // 3
    x_out = _empty((N, 9, C), rad_out)
    nat.call("fuma_init_scatter_fwd", ptr(rad_out), ptr(wigner), ptr(env), ptr(Z), ptr(batch), ptr(W_sphere),
             ptr(csd_emb), ptr(row_ptr), ptr(col_idx), N, E, C, ptr(x_out), stream_of(rad_out))
    return x_out


@init_node_scatter.register_fake
def _(rad_out, wigner, env, Z, batch, W_sphere, csd_emb, row_ptr, col_idx, N):
    return rad_out.new_empty(N, 9, rad_out.shape[1] // 3)


@custom_op("fuma::init_node_scatter_bwd", mutates_args=())
def init_node_scatter_bwd(g_out: Tensor, rad_out: Tensor, wigner: Tensor, env: Tensor, row_ptr: Tensor,
                          col_idx: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """(g_rad [E, 3C], g_wigner [E, 34], g_env [E])."""
    E, C, N = rad_out.shape[0], rad_out.shape[1] // 3, g_out.shape[0]
    g_out = g_out.contiguous()
    g_rad, g_w, g_env = torch.empty_like(rad_out), torch.empty_like(wigner), torch.empty_like(env)
    nat.call("fuma_init_scatter_bwd", ptr(g_out), ptr(rad_out), ptr(wigner), ptr(env), ptr(row_ptr), ptr(col_idx), N,
             E, C, ptr(g_rad), ptr(g_w), ptr(g_env), stream_of(rad_out))
    return g_rad, g_w, g_env


@init_node_scatter_bwd.register_fake
def _(g_out, rad_out, wigner, env, row_ptr, col_idx):
    return torch.empty_like(rad_out), torch.empty_like(wigner), torch.empty_like(env)


def _init_setup(ctx, inputs, output):
    rad_out, wigner, env, Z, batch, W_sphere, csd_emb, row_ptr, col_idx, N = inputs
    ctx.save_for_backward(rad_out, wigner, env, Z, batch, row_ptr, col_idx)
    ctx.num_z, ctx.nsys = W_sphere.shape[0], csd_emb.shape[0]


def _init_backward(ctx, g_out):
    rad_out, wigner, env, Z, batch, row_ptr, col_idx = ctx.saved_tensors
    g_rad, g_w, g_env = torch.ops.fuma.init_node_scatter_bwd(g_out, rad_out, wigner, env, row_ptr, col_idx)
    C = rad_out.shape[1] // 3
    g_ws = g_csd = None
    if ctx.needs_input_grad[5]:
        g_ws = g_out.new_zeros(ctx.num_z, C).index_add_(0, Z, g_out[:, 0])
    if ctx.needs_input_grad[6]:
        g_csd = g_out.new_zeros(ctx.nsys, C).index_add_(0, batch, g_out[:, 0])
    return g_rad, g_w, g_env, None, None, g_ws, g_csd, None, None, None


init_node_scatter.register_autograd(_init_backward, setup_context=_init_setup)
