"""Fused message-passing blocks for the f16x3 GEMM mode.

The edge-wise part of one layer of the reference (``Packed_eSCN_Layer.forward``,
``model.py:143-157``: radial MLP, gather + rotate, SO(2) convolution 1, gating, SO(2)
convolution 2, rotate back + scatter) and the initial edge-degree embedding
(``model.py:203-206``) run here as ONE autograd Function each. Inside a block every dense
contraction reads its input in the row-packed f16x3 split layout, written directly by the
kernel that produces it (``*_f16x3`` entry points), so the fp16 tensor-core GEMM does no
conversion work; at the block boundary all tensors (inputs, outputs and their gradients)
are plain fp32, so autograd and the node-wise modules around the blocks see the same
interface as the per-op path. The arithmetic per element is the per-op path's; only the
GEMM operand format differs.

The blocks need every GEMM width to be a multiple of 16 (C, the radial hidden width and the
edge-feature width B + 2C); :func:`fusable` checks a model, which otherwise runs per op.
"""
from __future__ import annotations

import torch

from . import _native as nat
from ._native import ptr, stream_of
from .linear import _gemm16, error_flag

_EPS_LN = 1e-7   # LayerNorm epsilon of the radial MLPs (ops/ln_silu.py:180)


def _empty(shape, like):
    return torch.empty(shape, device=like.device, dtype=torch.float32)


class _GeometryFn(torch.autograd.Function):
    """Edge geometry for the fused blocks: the edge features come back as their row-packed
    split (a constant for autograd) plus ``x_gauss``, the Gaussian-basis columns [E, B] that
    carry the only position dependence of the edge features. The blocks return gradients for
    ``x_gauss`` alone: the embedding columns depend on the atomic numbers only."""

    @staticmethod
    def forward(ctx, pos, Z, idx_i, idx_j, shifts, W_src, W_tgt, offset_g, coeff_g, cutoff, graph):
        N, E = pos.shape[0], idx_i.shape[0]
        B, C = offset_g.shape[0], W_src.shape[1]
        x_edge = _empty((E, B + 2 * C), pos)
        wigner, env = _empty((E, 34), pos), _empty((E,), pos)
        s = stream_of(pos)
        nat.call("fuma_geometry_fwd", ptr(pos), ptr(Z), ptr(idx_i), ptr(idx_j), ptr(shifts), ptr(W_src), ptr(W_tgt),
                 ptr(offset_g), float(coeff_g), float(cutoff), N, E, B, C, ptr(x_edge), ptr(wigner), ptr(env), s)
        xe_p = _empty((E, B + 2 * C), pos)
        nat.call("fuma_split_rows_f16", ptr(x_edge), B + 2 * C, E, B + 2 * C, ptr(xe_p), B + 2 * C,
                 ptr(error_flag(pos.device)), s)
        ctx.mark_non_differentiable(xe_p)
        ctx.save_for_backward(pos, idx_i, idx_j, shifts, offset_g)
        ctx.coeff_g, ctx.cutoff, ctx.graph = float(coeff_g), float(cutoff), graph
        return xe_p, x_edge[:, :B].contiguous(), wigner, env   # x_edge itself is freed

    @staticmethod
    def backward(ctx, g_xe_p, g_gauss, g_wigner, g_env):
        pos, idx_i, idx_j, shifts, offset_g = ctx.saved_tensors
        E, B, N = idx_i.shape[0], offset_g.shape[0], pos.shape[0]
        g_gauss = g_gauss.contiguous() if g_gauss is not None else _empty((E, B), pos).zero_()
        g_wigner = g_wigner.contiguous() if g_wigner is not None else _empty((E, 34), pos).zero_()
        g_env = g_env.contiguous() if g_env is not None else _empty((E,), pos).zero_()
        g_vec = _empty((E, 3), pos)
        s = stream_of(pos)
        nat.call("fuma_geometry_bwd", ptr(pos), ptr(idx_i), ptr(idx_j), ptr(shifts), ptr(offset_g), ctx.coeff_g,
                 ctx.cutoff, ptr(g_gauss), g_gauss.shape[1], ptr(g_wigner), ptr(g_env), E, B, ptr(g_vec), s)
        g_pos = None
        if ctx.needs_input_grad[0]:
            g = ctx.graph
            g_pos = torch.empty_like(pos)
            nat.call("fuma_edge_vec_to_nodes", ptr(g.src_row_ptr), ptr(g.src_col), ptr(g.dst_row_ptr), ptr(g.dst_col),
                     ptr(g_vec), N, E, ptr(g_pos), s)
        g_shifts = g_vec if ctx.needs_input_grad[4] else None
        return g_pos, None, None, None, g_shifts, None, None, None, None, None, None


def geometry(pos, Z, idx_i, idx_j, shifts, W_src, W_tgt, offset_g, coeff_g, cutoff, graph):
    """(edge features as ((split [E, B+2C]), x_gauss [E, B]), wigner [E, 34], env [E]) for the
    fused blocks; same kernels and arguments as ``ops.precompute_geometry``."""
    nat.require_cuda(pos, Z, idx_i, idx_j, shifts, W_src, W_tgt, offset_g)
    f32 = lambda t: t.float().contiguous()
    i64 = lambda t: t.long().contiguous()
    xe_p, x_gauss, wigner, env = _GeometryFn.apply(f32(pos), i64(Z), i64(idx_i), i64(idx_j), f32(shifts), f32(W_src),
                                                   f32(W_tgt), f32(offset_g), coeff_g, cutoff, graph)
    return (xe_p, x_gauss), wigner, env


# ---- radial MLP on split operands ------------------------------------------------------------

def _parts(lin) -> int:
    """Halves of the split operand a producer writes for the GEMM that reads it: 2 (hi and lo)
    for the f16x3 products, 1 (hi only) for the single-product "f16" mode."""
    return 1 if lin.mode == "f16" else 2


def _ln_silu_split(y, gamma, beta, err, parts):
    M, D = y.shape
    out, mean, rstd = _empty((M, D), y), _empty((M,), y), _empty((M,), y)
    nat.call("fuma_ln_silu_fwd_f16x3", ptr(y), ptr(gamma), ptr(beta), _EPS_LN, M, D, ptr(out), ptr(mean), ptr(rstd),
             parts, ptr(err), stream_of(y))
    return out, mean, rstd


def _ln_silu_bwd_split(y, gamma, beta, mean, rstd, g, err, parts):
    M, D = y.shape
    gx = _empty((M, D), y)
    nat.call("fuma_ln_silu_bwd_f16x3", ptr(y), ptr(gamma), ptr(beta), ptr(mean), ptr(rstd), ptr(g), M, D, ptr(gx),
             parts, ptr(err), stream_of(y))
    return gx


def radial_fwd(rad, xe_p, err, half_out: bool = False):
    """Linear -> LN-SiLU -> Linear -> LN-SiLU -> Linear on the split edge features; returns the
    radial output (fp32; fp16 with ``half_out`` in the single-product mode) and what the
    backward needs."""
    Kx = xe_p.shape[1]
    y1 = _gemm16(xe_p, rad.l1.w16, rad.l1.bias_p, Kx)
    parts = _parts(rad.l1)
    h1, m1, r1 = _ln_silu_split(y1, rad.g1, rad.be1, err, parts)
    y2 = _gemm16(h1, rad.l2.w16, rad.l2.bias_p, h1.shape[1])
    del h1
    h2, m2, r2 = _ln_silu_split(y2, rad.g2, rad.be2, err, parts)
    out = _gemm16(h2, rad.l3.w16, rad.l3.bias_p, h2.shape[1], out_half=half_out)
    return out, (y1, m1, r1, y2, m2, r2)


def radial_bwd(rad, saved, g_out_p, err):
    """Input gradient of :func:`radial_fwd` from the split gradient of its output."""
    y1, m1, r1, y2, m2, r2 = saved
    g_h2 = _gemm16(g_out_p, rad.l3.wt16, None, g_out_p.shape[1])
    parts = _parts(rad.l1)
    g_y2 = _ln_silu_bwd_split(y2, rad.g2, rad.be2, m2, r2, g_h2, err, parts)
    del g_h2
    g_h1 = _gemm16(g_y2, rad.l2.wt16, None, g_y2.shape[1])
    del g_y2
    g_y1 = _ln_silu_bwd_split(y1, rad.g1, rad.be1, m1, r1, g_h1, err, parts)
    del g_h1
    # only the Gaussian-basis columns of the edge features depend on positions: rows :B of W1^T
    B = rad.n_gauss
    hi, lo, inv, x1 = rad.l1.wt16
    return _gemm16(g_y1, (hi[:B], lo[:B], inv, x1), None, g_y1.shape[1])


def _conv2(layer, Y0, Y1, Y2, C, err, s):
    """Gating (split outputs) then the three conv2 GEMMs: O0, O1, O2 fp32."""
    E = Y0.shape[0]
    parts = _parts(layer.conv2_m0)
    Z0, Z1, Z2 = _empty((E, 3 * C), Y0), _empty((E, 4 * C), Y0), _empty((E, 2 * C), Y0)
    half = parts == 1   # the single-product mode stores its GEMM results as fp16
    nat.call("fuma_gating_fwd_f16x3", ptr(Y0), ptr(Y1), ptr(Y2), E, C, ptr(Z0), ptr(Z1), ptr(Z2), parts, int(half),
             ptr(err), s)
    O0 = _gemm16(Z0, layer.conv2_m0.w16, layer.conv2_m0.bias_p, 3 * C, out_half=half)
    O1 = _gemm16(Z1, layer.conv2_m1.w16, None, 4 * C, out_half=half)
    O2 = _gemm16(Z2, layer.conv2_m2.w16, None, 2 * C, out_half=half)
    return O0, O1, O2


def _edge_forward(layer, x_norm, xe_p, wigner, csd, idx_i, idx_j, batch, N, C, err, s):
    """Radial MLP, gather, conv1, gating, conv2 of one block: (rad, radial saved, Y0..2, O0..2)."""
    E = idx_i.shape[0]
    parts = _parts(layer.conv1_m0)
    half = parts == 1   # the single-product mode: radial and conv results stored as fp16
    rad, rsaved = radial_fwd(layer.rad, xe_p, err, half_out=half)
    X0, X1, X2 = _empty((E, 6 * C), x_norm), _empty((E, 8 * C), x_norm), _empty((E, 4 * C), x_norm)
    nat.call("fuma_gather_fwd_f16x3", ptr(x_norm), ptr(idx_i), ptr(idx_j), ptr(wigner), ptr(rad), ptr(csd),
             ptr(batch), N, E, C, ptr(X0), ptr(X1), ptr(X2), parts, int(half), ptr(err), s)
    Y0 = _gemm16(X0, layer.conv1_m0.w16, layer.conv1_m0.bias_p, 6 * C, out_half=half)
    Y1 = _gemm16(X1, layer.conv1_m1.w16, None, 8 * C, out_half=half)
    Y2 = _gemm16(X2, layer.conv1_m2.w16, None, 4 * C, out_half=half)
    del X0, X1, X2
    O0, O1, O2 = _conv2(layer, Y0, Y1, Y2, C, err, s)
    return rad, rsaved, (Y0, Y1, Y2), (O0, O1, O2)


# ---- one message-passing block ---------------------------------------------------------------
# Saved for the backward per edge and layer: the radial output (12C), pre-activations (2H), Y
# (11C) and the conv2 outputs (9C), 17.4 KB at C = H = 128. With ``lean`` the block saves only
# its inputs and the backward recomputes the edge forward first (block-level recomputation:
# about 1.4x the step's work, for graphs whose activations would not fit in device memory).

class _MessageBlockFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_norm, x_in, xe_p, x_gauss, wigner, env, csd, layer, idx_i, idx_j, batch, graph, lean):
        N, _, C = x_in.shape
        E = idx_i.shape[0]
        err = error_flag(x_in.device)
        s = stream_of(x_in)
        rad, rsaved, (Y0, Y1, Y2), (O0, O1, O2) = _edge_forward(layer, x_norm, xe_p, wigner, csd, idx_i, idx_j,
                                                                 batch, N, C, err, s)
        x_mid = _empty((N, 9, C), x_in)
        nat.call("fuma_rotate_scatter_fwd_f16x3", ptr(O0), ptr(O1), ptr(O2), ptr(wigner), ptr(env), ptr(x_in),
                 ptr(graph.dst_row_ptr), ptr(graph.dst_col), N, E, C, ptr(x_mid), int(O0.dtype == torch.float16), s)
        if lean:
            ctx.save_for_backward(x_norm, wigner, env, csd, idx_i, batch, xe_p, idx_j)
        else:
            ctx.save_for_backward(x_norm, wigner, env, csd, idx_i, batch, rad, *rsaved, Y0, Y1, Y2, O0, O1, O2)
        ctx.layer, ctx.graph, ctx.lean = layer, graph, lean
        return x_mid

    @staticmethod
    def backward(ctx, g_mid):
        saved = ctx.saved_tensors
        x_norm, wigner, env, csd, idx_i, batch = saved[:6]
        layer, graph = ctx.layer, ctx.graph
        g_mid = g_mid.contiguous()
        N, _, C = x_norm.shape
        E = idx_i.shape[0]
        err = error_flag(x_norm.device)
        s = stream_of(x_norm)
        parts = _parts(layer.conv1_m0)
        if ctx.lean:
            xe_p, idx_j = saved[6:8]
            rad, rsaved, (Y0, Y1, Y2), (O0, O1, O2) = _edge_forward(layer, x_norm, xe_p, wigner, csd, idx_i, idx_j,
                                                                     batch, N, C, err, s)
        else:
            rad = saved[6]
            rsaved = saved[7:13]
            Y0, Y1, Y2, O0, O1, O2 = saved[13:19]
        # single-product mode: fp16 radial / conv results, and fp16 results of the two input-gradient
        # GEMMs read by the gating and gather backward (their operands are fp16 already)
        half = parts == 1
        gO0, gO1, gO2 = _empty((E, 3 * C), g_mid), _empty((E, 4 * C), g_mid), _empty((E, 2 * C), g_mid)
        g_w = _empty((E, 34), g_mid)
        g_env = _empty((E,), g_mid)
        nat.call("fuma_rotate_scatter_bwd_f16x3", ptr(g_mid), ptr(O0), ptr(O1), ptr(O2), ptr(wigner), ptr(env),
                 ptr(graph.dst_row_ptr), ptr(graph.dst_col), N, E, C, ptr(gO0), ptr(gO1), ptr(gO2), ptr(g_w),
                 ptr(g_env), parts, int(half), ptr(err), s)
        del O0, O1, O2
        gZ0 = _gemm16(gO0, layer.conv2_m0.wt16, None, 3 * C, out_half=half)
        gZ1 = _gemm16(gO1, layer.conv2_m1.wt16, None, 4 * C, out_half=half)
        gZ2 = _gemm16(gO2, layer.conv2_m2.wt16, None, 2 * C, out_half=half)
        del gO0, gO1, gO2
        gY0, gY1, gY2 = _empty((E, 5 * C), g_mid), _empty((E, 4 * C), g_mid), _empty((E, 2 * C), g_mid)
        nat.call("fuma_gating_bwd_f16x3", ptr(gZ0), ptr(gZ1), ptr(gZ2), ptr(Y0), ptr(Y1), ptr(Y2), E, C, ptr(gY0),
                 ptr(gY1), ptr(gY2), parts, int(half), ptr(err), s)
        del gZ0, gZ1, gZ2, Y0, Y1, Y2
        gX0 = _gemm16(gY0, layer.conv1_m0.wt16, None, 5 * C, out_half=half)
        gX1 = _gemm16(gY1, layer.conv1_m1.wt16, None, 4 * C, out_half=half)
        gX2 = _gemm16(gY2, layer.conv1_m2.wt16, None, 2 * C, out_half=half)
        del gY0, gY1, gY2
        g_x = torch.empty_like(x_norm)
        g_w2 = _empty((E, 34), g_mid)
        g_rad = _empty(tuple(rad.shape), g_mid)   # fp32 (split) whatever the radial rows' storage
        nat.call("fuma_gather_bwd_f16x3", ptr(gX0), ptr(gX1), ptr(gX2), ptr(x_norm), ptr(idx_i), ptr(wigner), ptr(rad),
                 ptr(csd), ptr(batch), ptr(graph.dst_row_ptr), ptr(graph.dst_col), ptr(graph.src_row_ptr),
                 ptr(graph.src_col), N, E, C, None, 0, ptr(g_x), ptr(g_w2), ptr(g_rad), parts, int(half), ptr(err), s)
        del gX0, gX1, gX2, rad
        g_xe = radial_bwd(layer.rad, rsaved, g_rad, err)
        g_w += g_w2
        return g_x, g_mid, None, g_xe, g_w, g_env, None, None, None, None, None, None, None


def message_block(layer, x_norm, x_in, xe, wigner, env, csd, idx_i, idx_j, batch, graph, lean: bool = False):
    """x_mid = x_in + scatter(SO(2) message of every edge) for one layer (fp32 in and out);
    ``xe`` = (split edge features, x_gauss) from :func:`geometry`; ``lean``: recompute instead
    of saving the radial and conv2 outputs."""
    xe_p, x_gauss = xe
    return _MessageBlockFn.apply(x_norm.contiguous(), x_in.contiguous(), xe_p, x_gauss, wigner, env,
                                 csd.contiguous(), layer, idx_i, idx_j, batch, graph, bool(lean))


def lean_bytes_per_edge(C: int, H: int, L: int) -> int:
    """Estimated device bytes per edge of a default-mode step (saved activations of L layers plus
    the largest transient of a layer's backward): 4 (L (32C + 2H) + 45C); 92,672 at C = H = 128,
    L = 4 (measured: 139 GB for 1.51M edges)."""
    return 4 * (L * (32 * C + 2 * H) + 45 * C)


def lean_needed(E: int, C: int, H: int, L: int, device=None, total_bytes: int | None = None) -> bool:
    """Whether the default-mode activations of an L-layer step over E edges would exceed 90% of
    the device memory (``total_bytes``, default: the device's). FUMA_LEAN=0/1 forces it."""
    import os
    force = os.environ.get("FUMA_LEAN")
    if force is not None:
        return force == "1"
    if total_bytes is None:
        total_bytes = torch.cuda.get_device_properties(device).total_memory
    return E * lean_bytes_per_edge(C, H, L) > 0.9 * total_bytes


# ---- initial edge-degree embedding -----------------------------------------------------------

class _InitBlockFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, xe_p, x_gauss, wigner, env, Z, batch, model, csd, graph, N):
        E = xe_p.shape[0]
        C = model.C
        err = error_flag(xe_p.device)
        rad, rsaved = radial_fwd(model.rad_init, xe_p, err)
        x = _empty((N, 9, C), xe_p)
        nat.call("fuma_init_scatter_fwd", ptr(rad), ptr(wigner), ptr(env), ptr(Z), ptr(batch), ptr(model.W_sphere),
                 ptr(csd), ptr(graph.dst_row_ptr), ptr(graph.dst_col), N, E, C, ptr(x), stream_of(xe_p))
        ctx.save_for_backward(rad, wigner, env, *rsaved)
        ctx.model, ctx.graph, ctx.N = model, graph, N
        return x

    @staticmethod
    def backward(ctx, g_out):
        rad, wigner, env, *rsaved = ctx.saved_tensors
        model, graph, N = ctx.model, ctx.graph, ctx.N
        g_out = g_out.contiguous()
        E, C = rad.shape[0], model.C
        err = error_flag(rad.device)
        parts = _parts(model.rad_init.l1)
        g_rad = torch.empty_like(rad)
        g_w, g_env = _empty((E, 34), rad), _empty((E,), rad)
        nat.call("fuma_init_scatter_bwd_f16x3", ptr(g_out), ptr(rad), ptr(wigner), ptr(env), ptr(graph.dst_row_ptr),
                 ptr(graph.dst_col), N, E, C, ptr(g_rad), ptr(g_w), ptr(g_env), parts, ptr(err), stream_of(rad))
        g_xe = radial_bwd(model.rad_init, rsaved, g_rad, err)
        return None, g_xe, g_w, g_env, None, None, None, None, None, None


def init_block(model, xe, wigner, env, Z, batch, csd, graph, N):
    """Initial node embedding from the split edge features (fp32 out)."""
    xe_p, x_gauss = xe
    return _InitBlockFn.apply(xe_p, x_gauss, wigner, env, Z.long().contiguous(), batch.long().contiguous(), model,
                              csd.contiguous(), graph, int(N))


def fusable(model) -> bool:
    """True if every dense contraction of ``model`` (an ESCNInferenceModel in f16x3 mode) has
    widths that are multiples of 16, so the fused blocks apply."""
    lins = [model.rad_init.l1, model.rad_init.l2, model.rad_init.l3]
    for lay in model.layers:
        lins += [lay.rad.l1, lay.rad.l2, lay.rad.l3, lay.conv1_m0, lay.conv1_m1, lay.conv1_m2, lay.conv2_m0,
                 lay.conv2_m1, lay.conv2_m2]
    modes = {l.mode for l in lins}
    return (len(modes) == 1 and modes <= {"f16x3", "f16"} and all(l.N % 16 == 0 and l.K % 16 == 0 for l in lins)
            and model.C % 16 == 0 and model.B % 16 == 0)
