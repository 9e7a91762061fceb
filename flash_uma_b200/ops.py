"""PyTorch autograd ops over the C ABI, mirroring the reference's op-level API.

Same names, argument order and meaning, return values and backward conventions
(one gradient per input, ``None`` for integer / frozen inputs) as the reference's
``ops/*.py`` Functions:

* ``precompute_geometry``   - ``ops/geom.py:591``
* ``layer_norm_silu``       - ``ops/ln_silu.py:180``
* ``gather_wigner_split``   - ``ops/gather.py:516``
* ``fused_gating_split``    - ``ops/gating.py:236``
* ``rotate_scatter_split``  - ``ops/scatter.py:354``
* ``init_node_scatter``     - ``ops/scatter.py:527``

Differences that callers may rely on: the backward passes are deterministic
(no atomics). ``precompute_geometry`` and ``gather_wigner_split`` accept an
optional keyword ``graph`` (a :class:`GraphCSR` of the same edges) so that the
backward can use the cached destination/source CSRs; without it they are built
on the fly. All feature tensors must be fp32 CUDA tensors; there is no CPU path.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native as nat
from ._native import ptr, stream_of


@dataclass
class GraphCSR:
    """Destination- and source-sorted CSR of one edge list (int32, on the device).

    dst_row_ptr[N+1], dst_col[E]: edges into node n are dst_col[dst_row_ptr[n]:dst_row_ptr[n+1]],
    in increasing edge order (stable, ``model.py:20-26``); src_* likewise for edges out of n."""
    N: int
    E: int
    dst_row_ptr: torch.Tensor
    dst_col: torch.Tensor
    src_row_ptr: torch.Tensor
    src_col: torch.Tensor


def _csr(idx: torch.Tensor, N: int):
    # stable sort + binary search of every row start: no device-to-host synchronisation
    order = torch.argsort(idx, stable=True)
    bounds = torch.arange(N + 1, device=idx.device, dtype=idx.dtype)
    row_ptr = torch.searchsorted(idx[order], bounds).to(torch.int32)
    return row_ptr, order.to(torch.int32)


def build_graph_csr(idx_i: torch.Tensor, idx_j: torch.Tensor, N: int) -> GraphCSR:
    d_ptr, d_col = _csr(idx_j, N)
    s_ptr, s_col = _csr(idx_i, N)
    return GraphCSR(N=N, E=int(idx_i.shape[0]), dst_row_ptr=d_ptr, dst_col=d_col, src_row_ptr=s_ptr, src_col=s_col)


def permute_graph(g: GraphCSR, perm: torch.Tensor) -> GraphCSR:
    """The CSRs of the same edges after renumbering the nodes (new node a = old node perm[a]),
    from ``g`` without a sort (``fuma_csr_permute``): bitwise ``build_graph_csr(inv[idx_i],
    inv[idx_j], N)`` for ``inv`` the inverse of ``perm``."""
    nat.require_cuda(g.dst_row_ptr, perm)
    perm = _i64(perm)
    N, E = g.N, g.E
    dev = g.dst_row_ptr.device
    i32 = dict(device=dev, dtype=torch.int32)
    d_ptr, s_ptr = torch.empty(N + 1, **i32), torch.empty(N + 1, **i32)
    d_col, s_col = torch.empty(E, **i32), torch.empty(E, **i32)
    nat.call("fuma_csr_permute", ptr(g.dst_row_ptr), ptr(g.dst_col), ptr(g.src_row_ptr), ptr(g.src_col), ptr(perm),
             N, E, ptr(d_ptr), ptr(d_col), ptr(s_ptr), ptr(s_col), stream_of(perm))
    return GraphCSR(N=N, E=E, dst_row_ptr=d_ptr, dst_col=d_col, src_row_ptr=s_ptr, src_col=s_col)


def _f32(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype != torch.float32:
        raise TypeError(f"{name} must be float32 (got {t.dtype})")
    return t.contiguous()


def _i64(t: torch.Tensor) -> torch.Tensor:
    return (t if t.dtype == torch.int64 else t.long()).contiguous()


def _i32(t: torch.Tensor) -> torch.Tensor:
    return (t if t.dtype == torch.int32 else t.int()).contiguous()


# ---------------------------------------------------------------------------------------------
class _RMSNormSH(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, aw, ab, bal, eps):
        nat.require_cuda(x)
        x = _f32(x, "x")
        N, K, C = x.shape
        if K != 9:
            raise ValueError(f"rms_norm_sh: x must be [N, 9, C], got {tuple(x.shape)}")
        out = torch.empty_like(x)
        rstd = torch.empty(N, device=x.device, dtype=torch.float32)
        nat.call("fuma_rmsnorm_sh_fwd", ptr(x), ptr(aw), ptr(ab), ptr(bal), eps, N, C, ptr(out), ptr(rstd),
                 stream_of(x))
        ctx.save_for_backward(x, aw, bal, rstd)
        return out

    @staticmethod
    def backward(ctx, g):
        x, aw, bal, rstd = ctx.saved_tensors
        N, _, C = x.shape
        g = _f32(g, "g")
        gx = torch.empty_like(x)
        nat.call("fuma_rmsnorm_sh_bwd", ptr(x), ptr(aw), ptr(bal), ptr(rstd), ptr(g), N, C, ptr(gx), stream_of(x))
        return gx, None, None, None, None


def rms_norm_sh(x: torch.Tensor, norm) -> torch.Tensor:
    """``norm(x)`` for an :class:`~flash_uma_b200.nodewise.EquivariantRMSNormSH` (lmax 2) in one
    CUDA kernel per direction (``fuma_rmsnorm_sh_fwd`` / ``_bwd``); its affine parameters are
    treated as constants (frozen, as in the inference model)."""
    if norm.lmax != 2:
        raise ValueError("rms_norm_sh: lmax must be 2")
    f = lambda t: t.detach().float().contiguous()   # noqa: E731
    return _RMSNormSH.apply(x, f(norm.affine_weight), f(norm.affine_bias), f(norm.balance_degree_weight),
                            float(norm.eps))


class _AtomwiseResidual(torch.autograd.Function):
    """y = x_mid + atom_wise(xn) for a SpectralAtomwise block (constants from atomwise_constants)."""

    @staticmethod
    def forward(ctx, xn, x_mid, prm):
        nat.require_cuda(xn, x_mid)
        Ws, bs, W1e, b1, W2e, b2 = prm
        xn, x_mid = _f32(xn, "xn"), _f32(x_mid, "x_mid")
        N, _, C = xn.shape
        H = b1.shape[0]
        s = stream_of(xn)
        u = torch.addmm(bs, xn[:, 0], Ws.t())                       # [N, 2H]
        h = torch.bmm(xn.transpose(0, 1), W1e.transpose(1, 2))      # [9, N, H], coefficient-major
        z = torch.empty_like(h)
        nat.call("fuma_atomwise_gate_fwd", ptr(h), ptr(u), ptr(b1), N, H, ptr(z), s)
        o = torch.bmm(z, W2e.transpose(1, 2))                       # [9, N, C]
        y = torch.empty_like(x_mid)
        nat.call("fuma_coef_to_node", ptr(o), ptr(x_mid), ptr(b2), 0, N, C, ptr(y), s)
        ctx.save_for_backward(h, u)
        ctx.prm = prm
        return y

    @staticmethod
    def backward(ctx, gy):
        h, u = ctx.saved_tensors
        Ws, bs, W1e, b1, W2e, b2 = ctx.prm
        gy = _f32(gy, "gy")
        _, N, H = h.shape
        C = gy.shape[2]
        s = stream_of(gy)
        gz = torch.bmm(gy.transpose(0, 1), W2e)                     # [9, N, H]
        gh, gu = torch.empty_like(h), torch.empty_like(u)
        nat.call("fuma_atomwise_gate_bwd", ptr(gz), ptr(h), ptr(u), ptr(b1), N, H, ptr(gh), ptr(gu), s)
        gx9 = torch.bmm(gh, W1e)                                    # [9, N, C]
        gu_x = torch.mm(gu, Ws)                                     # [N, C], into the l = 0 row
        gxn = torch.empty_like(gy)
        nat.call("fuma_coef_to_node", ptr(gx9), None, ptr(gu_x), 1, N, C, ptr(gxn), s)
        return gxn, gy, None


_DEG9 = [0, 1, 1, 1, 2, 2, 2, 2, 2]


def atomwise_constants(aw) -> tuple:
    """The frozen parameters of a SpectralAtomwise block as the fused path uses them, cached on
    the module: scalar MLP (W [2H, C], b [2H]), the two per-degree maps expanded to the 9
    coefficients (W1e [9, H, C], W2e [9, C, H]) and their l = 0 biases."""
    dev = aw.so3_linear_1.weight.device
    cached = getattr(aw, "_fuma_constants", None)
    if cached is not None and cached[0].device == dev:
        return cached
    f = lambda t: t.detach().float().contiguous()   # noqa: E731
    idx = torch.tensor(_DEG9, device=dev)
    lin = aw.scalar_mlp[0]
    prm = (f(lin.weight), f(lin.bias), f(aw.so3_linear_1.weight.index_select(0, idx)), f(aw.so3_linear_1.bias),
           f(aw.so3_linear_2.weight.index_select(0, idx)), f(aw.so3_linear_2.bias))
    aw._fuma_constants = prm
    return prm


def atomwise_residual(aw, xn: torch.Tensor, x_mid: torch.Tensor) -> torch.Tensor:
    """``x_mid + aw(xn)`` for a :class:`~flash_uma_b200.nodewise.SpectralAtomwise` (lmax 2): the
    per-coefficient linear maps as batched fp32 GEMMs on the coefficient-major view, the gating
    and the layout change (with residual and biases) as CUDA kernels. Frozen parameters."""
    if aw.lmax != 2 or (aw.hidden % 4) or (xn.shape[2] % 4):
        raise ValueError("atomwise_residual: lmax 2 and channel counts that are multiples of 4")
    return _AtomwiseResidual.apply(xn, x_mid, atomwise_constants(aw))


# ---------------------------------------------------------------------------------------------
class _PrecomputeGeometry(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pos, Z, idx_i, idx_j, shifts, W_src, W_tgt, offset_g, coeff_g, cutoff, graph):
        nat.require_cuda(pos, Z, idx_i, idx_j, shifts, W_src, W_tgt, offset_g)
        pos = _f32(pos, "pos"); shifts = _f32(shifts, "shifts")
        W_src = _f32(W_src, "W_src"); W_tgt = _f32(W_tgt, "W_tgt"); offset_g = _f32(offset_g, "offset_g")
        Z = _i64(Z); idx_i = _i64(idx_i); idx_j = _i64(idx_j)
        N, E = pos.shape[0], idx_i.shape[0]
        B, C = offset_g.shape[0], W_src.shape[1]
        dev = pos.device
        x_edge = torch.empty(E, B + 2 * C, device=dev, dtype=torch.float32)
        wigner = torch.empty(E, 34, device=dev, dtype=torch.float32)
        env = torch.empty(E, device=dev, dtype=torch.float32)
        nat.call("fuma_geometry_fwd", ptr(pos), ptr(Z), ptr(idx_i), ptr(idx_j), ptr(shifts), ptr(W_src), ptr(W_tgt),
                 ptr(offset_g), float(coeff_g), float(cutoff), N, E, B, C, ptr(x_edge), ptr(wigner), ptr(env),
                 stream_of(pos))
        ctx.save_for_backward(pos, idx_i, idx_j, shifts, offset_g)
        ctx.coeff_g, ctx.cutoff, ctx.graph, ctx.B = float(coeff_g), float(cutoff), graph, B
        return x_edge, wigner, env

    @staticmethod
    def backward(ctx, g_x_edge, g_wigner, g_env):
        pos, idx_i, idx_j, shifts, offset_g = ctx.saved_tensors
        E, B, N = idx_i.shape[0], ctx.B, pos.shape[0]
        dev = pos.device
        g_x_edge = g_x_edge.contiguous() if g_x_edge is not None else torch.zeros(E, B, device=dev)
        g_wigner = g_wigner.contiguous() if g_wigner is not None else torch.zeros(E, 34, device=dev)
        g_env = g_env.contiguous() if g_env is not None else torch.zeros(E, device=dev)
        g_vec = torch.empty(E, 3, device=dev, dtype=torch.float32)
        nat.call("fuma_geometry_bwd", ptr(pos), ptr(idx_i), ptr(idx_j), ptr(shifts), ptr(offset_g), ctx.coeff_g,
                 ctx.cutoff, ptr(g_x_edge), g_x_edge.shape[1], ptr(g_wigner), ptr(g_env), E, B, ptr(g_vec),
                 stream_of(pos))
        g_pos = None
        if ctx.needs_input_grad[0]:
            g = ctx.graph if ctx.graph is not None else build_graph_csr(idx_i, idx_j, N)
            g_pos = torch.empty_like(pos)
            nat.call("fuma_edge_vec_to_nodes", ptr(g.src_row_ptr), ptr(g.src_col), ptr(g.dst_row_ptr), ptr(g.dst_col),
                     ptr(g_vec), N, E, ptr(g_pos), stream_of(pos))
        g_shifts = g_vec if ctx.needs_input_grad[4] else None
        return g_pos, None, None, None, g_shifts, None, None, None, None, None, None


def precompute_geometry(pos, Z, idx_i, idx_j, shifts, W_src, W_tgt, offset_g, coeff_g, cutoff, *, graph=None):
    """Edge geometry -> (x_edge_raw [E, B+2C], wigner [E, 34], env [E]); see ``ops/geom.py:591``."""
    return _PrecomputeGeometry.apply(pos, Z, idx_i, idx_j, shifts, W_src, W_tgt, offset_g, coeff_g, cutoff, graph)


# ---------------------------------------------------------------------------------------------
class _LayerNormSiLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, gamma, beta, eps):
        nat.require_cuda(x, gamma, beta)
        x = _f32(x, "x"); gamma = _f32(gamma, "gamma"); beta = _f32(beta, "beta")
        M, D = x.shape
        out = torch.empty_like(x)
        mean = torch.empty(M, device=x.device, dtype=torch.float32)
        rstd = torch.empty(M, device=x.device, dtype=torch.float32)
        nat.call("fuma_ln_silu_fwd", ptr(x), ptr(gamma), ptr(beta), float(eps), M, D, ptr(out), ptr(mean), ptr(rstd),
                 stream_of(x))
        ctx.save_for_backward(x, gamma, beta, mean, rstd)
        return out

    @staticmethod
    def backward(ctx, g_out):
        x, gamma, beta, mean, rstd = ctx.saved_tensors
        g_out = g_out.contiguous()
        M, D = x.shape
        g_x = torch.empty_like(x)
        nat.call("fuma_ln_silu_bwd", ptr(x), ptr(gamma), ptr(beta), ptr(mean), ptr(rstd), ptr(g_out), M, D, ptr(g_x),
                 stream_of(x))
        return g_x, None, None, None


def layer_norm_silu(x, gamma, beta, eps=1e-7):
    """Fused row-wise LayerNorm + SiLU on [M, D]; see ``ops/ln_silu.py:180``."""
    return _LayerNormSiLU.apply(x, gamma, beta, eps)


# ---------------------------------------------------------------------------------------------
class _GatherWignerSplit(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_in, idx_i, idx_j, wigner, rad_out, csd_emb, batch, graph):
        nat.require_cuda(x_in, idx_i, idx_j, wigner, rad_out, csd_emb, batch)
        x_in = _f32(x_in, "x_in"); wigner = _f32(wigner, "wigner"); rad_out = _f32(rad_out, "rad_out")
        csd_emb = _f32(csd_emb, "csd_emb")
        idx_i = _i64(idx_i); idx_j = _i64(idx_j); batch = _i64(batch)
        N, _, C = x_in.shape
        E = idx_i.shape[0]
        dev = x_in.device
        X0 = torch.empty(E, 6 * C, device=dev, dtype=torch.float32)
        X1 = torch.empty(E, 8 * C, device=dev, dtype=torch.float32)
        X2 = torch.empty(E, 4 * C, device=dev, dtype=torch.float32)
        nat.call("fuma_gather_fwd", ptr(x_in), ptr(idx_i), ptr(idx_j), ptr(wigner), ptr(rad_out), ptr(csd_emb),
                 ptr(batch), N, E, C, ptr(X0), ptr(X1), ptr(X2), stream_of(x_in))
        ctx.save_for_backward(x_in, idx_i, idx_j, wigner, rad_out, csd_emb, batch)
        ctx.graph = graph
        return X0, X1, X2

    @staticmethod
    def backward(ctx, g0, g1, g2):
        x_in, idx_i, idx_j, wigner, rad_out, csd_emb, batch = ctx.saved_tensors
        N, _, C = x_in.shape
        E = idx_i.shape[0]
        dev = x_in.device
        g0 = g0.contiguous() if g0 is not None else torch.zeros(E, 6 * C, device=dev)
        g1 = g1.contiguous() if g1 is not None else torch.zeros(E, 8 * C, device=dev)
        g2 = g2.contiguous() if g2 is not None else torch.zeros(E, 4 * C, device=dev)
        g = ctx.graph if ctx.graph is not None else build_graph_csr(idx_i, idx_j, N)
        g_x = torch.empty_like(x_in)
        g_w = torch.empty(E, 34, device=dev, dtype=torch.float32)
        g_r = torch.empty_like(rad_out)
        nat.call("fuma_gather_bwd", ptr(g0), ptr(g1), ptr(g2), ptr(x_in), ptr(idx_i), ptr(wigner), ptr(rad_out),
                 ptr(csd_emb), ptr(batch), ptr(g.dst_row_ptr), ptr(g.dst_col), ptr(g.src_row_ptr), ptr(g.src_col),
                 N, E, C, None, 0, ptr(g_x), ptr(g_w), ptr(g_r), stream_of(x_in))
        return g_x, None, None, g_w, g_r, None, None, None


def gather_wigner_split(x_in, idx_i, idx_j, wigner, rad_out, csd_emb, batch, *, graph=None):
    """Gather + rotate into the edge frame + radial scale -> (X_m0, X_m1, X_m2); see ``ops/gather.py:516``."""
    return _GatherWignerSplit.apply(x_in, idx_i, idx_j, wigner, rad_out, csd_emb, batch, graph)


# ---------------------------------------------------------------------------------------------
class _FusedGatingSplit(torch.autograd.Function):
    @staticmethod
    def forward(ctx, Y0, Y1, Y2, C):
        nat.require_cuda(Y0, Y1, Y2)
        Y0 = _f32(Y0, "Y_m0"); Y1 = _f32(Y1, "Y_m1"); Y2 = _f32(Y2, "Y_m2")
        E = Y0.shape[0]
        dev = Y0.device
        Z0 = torch.empty(E, 3 * C, device=dev, dtype=torch.float32)
        Z1 = torch.empty(E, 4 * C, device=dev, dtype=torch.float32)
        Z2 = torch.empty(E, 2 * C, device=dev, dtype=torch.float32)
        nat.call("fuma_gating_fwd", ptr(Y0), ptr(Y1), ptr(Y2), E, C, ptr(Z0), ptr(Z1), ptr(Z2), stream_of(Y0))
        ctx.save_for_backward(Y0, Y1, Y2)
        ctx.C = C
        return Z0, Z1, Z2

    @staticmethod
    def backward(ctx, g0, g1, g2):
        Y0, Y1, Y2 = ctx.saved_tensors
        E, C, dev = Y0.shape[0], ctx.C, Y0.device
        g0 = g0.contiguous() if g0 is not None else torch.zeros(E, 3 * C, device=dev)
        g1 = g1.contiguous() if g1 is not None else torch.zeros(E, 4 * C, device=dev)
        g2 = g2.contiguous() if g2 is not None else torch.zeros(E, 2 * C, device=dev)
        gY0, gY1, gY2 = torch.empty_like(Y0), torch.empty_like(Y1), torch.empty_like(Y2)
        nat.call("fuma_gating_bwd", ptr(g0), ptr(g1), ptr(g2), ptr(Y0), ptr(Y1), ptr(Y2), E, C, ptr(gY0), ptr(gY1),
                 ptr(gY2), stream_of(Y0))
        return gY0, gY1, gY2, None


def fused_gating_split(Y_m0, Y_m1, Y_m2, C):
    """Split gating -> (Z_m0, Z_m1, Z_m2); see ``ops/gating.py:236``."""
    return _FusedGatingSplit.apply(Y_m0, Y_m1, Y_m2, int(C))


# ---------------------------------------------------------------------------------------------
class _RotateScatterSplit(torch.autograd.Function):
    @staticmethod
    def forward(ctx, Z0, Z1, Z2, wigner, env, x_res, idx_j, row_ptr, col_idx, N):
        nat.require_cuda(Z0, Z1, Z2, wigner, env, x_res, row_ptr, col_idx)
        Z0 = _f32(Z0, "Z_m0"); Z1 = _f32(Z1, "Z_m1"); Z2 = _f32(Z2, "Z_m2")
        wigner = _f32(wigner, "wigner"); env = _f32(env, "env"); x_res = _f32(x_res, "x_res")
        row_ptr = _i32(row_ptr); col_idx = _i32(col_idx)
        E = Z0.shape[0]
        C = Z0.shape[1] // 3
        x_out = torch.empty(N, 9, C, device=Z0.device, dtype=torch.float32)
        nat.call("fuma_rotate_scatter_fwd", ptr(Z0), ptr(Z1), ptr(Z2), ptr(wigner), ptr(env), ptr(x_res), ptr(row_ptr),
                 ptr(col_idx), N, E, C, ptr(x_out), stream_of(Z0))
        ctx.save_for_backward(Z0, Z1, Z2, wigner, env, row_ptr, col_idx)
        ctx.N, ctx.C = N, C
        return x_out

    @staticmethod
    def backward(ctx, g_out):
        Z0, Z1, Z2, wigner, env, row_ptr, col_idx = ctx.saved_tensors
        g_out = g_out.contiguous()
        E, N, C = Z0.shape[0], ctx.N, ctx.C
        gZ0, gZ1, gZ2 = torch.empty_like(Z0), torch.empty_like(Z1), torch.empty_like(Z2)
        g_w = torch.empty_like(wigner)
        g_env = torch.empty_like(env)
        nat.call("fuma_rotate_scatter_bwd", ptr(g_out), ptr(Z0), ptr(Z1), ptr(Z2), ptr(wigner), ptr(env), ptr(row_ptr),
                 ptr(col_idx), N, E, C, ptr(gZ0), ptr(gZ1), ptr(gZ2), ptr(g_w), ptr(g_env), stream_of(Z0))
        return gZ0, gZ1, gZ2, g_w, g_env, g_out, None, None, None, None


def rotate_scatter_split(Z_m0, Z_m1, Z_m2, wigner, env, x_res, idx_j, row_ptr, col_idx, N):
    """Rotate back + envelope + deterministic FP64 CSR sum + residual -> x_out [N, 9, C];
    see ``ops/scatter.py:354``."""
    return _RotateScatterSplit.apply(Z_m0, Z_m1, Z_m2, wigner, env, x_res, idx_j, row_ptr, col_idx, int(N))


# ---------------------------------------------------------------------------------------------
class _InitNodeScatter(torch.autograd.Function):
    @staticmethod
    def forward(ctx, rad_out, wigner, env, Z, batch, W_sphere, csd_emb, idx_j, row_ptr, col_idx, N):
        nat.require_cuda(rad_out, wigner, env, Z, batch, W_sphere, csd_emb, row_ptr, col_idx)
        rad_out = _f32(rad_out, "rad_out"); wigner = _f32(wigner, "wigner"); env = _f32(env, "env")
        W_sphere = _f32(W_sphere, "W_sphere"); csd_emb = _f32(csd_emb, "csd_emb")
        Z = _i64(Z); batch = _i64(batch); row_ptr = _i32(row_ptr); col_idx = _i32(col_idx)
        E, C = rad_out.shape[0], rad_out.shape[1] // 3
        x_out = torch.empty(N, 9, C, device=rad_out.device, dtype=torch.float32)
        nat.call("fuma_init_scatter_fwd", ptr(rad_out), ptr(wigner), ptr(env), ptr(Z), ptr(batch), ptr(W_sphere),
                 ptr(csd_emb), ptr(row_ptr), ptr(col_idx), N, E, C, ptr(x_out), stream_of(rad_out))
        ctx.save_for_backward(rad_out, wigner, env, Z, batch, row_ptr, col_idx)
        ctx.N, ctx.C, ctx.num_z, ctx.nsys = N, C, W_sphere.shape[0], csd_emb.shape[0]
        return x_out

    @staticmethod
    def backward(ctx, g_out):
        rad_out, wigner, env, Z, batch, row_ptr, col_idx = ctx.saved_tensors
        g_out = g_out.contiguous()
        E, N, C = rad_out.shape[0], ctx.N, ctx.C
        g_rad = torch.empty_like(rad_out)
        g_w = torch.empty_like(wigner)
        g_env = torch.empty_like(env)
        nat.call("fuma_init_scatter_bwd", ptr(g_out), ptr(rad_out), ptr(wigner), ptr(env), ptr(row_ptr), ptr(col_idx),
                 N, E, C, ptr(g_rad), ptr(g_w), ptr(g_env), stream_of(rad_out))
        g_ws = g_csd = None
        if ctx.needs_input_grad[5]:
            g_ws = torch.zeros(ctx.num_z, C, device=g_out.device).index_add_(0, Z, g_out[:, 0])
        if ctx.needs_input_grad[6]:
            g_csd = torch.zeros(ctx.nsys, C, device=g_out.device).index_add_(0, batch, g_out[:, 0])
        return g_rad, g_w, g_env, None, None, g_ws, g_csd, None, None, None, None


def init_node_scatter(rad_out, wigner, env, Z, batch, W_sphere, csd_emb, idx_j, row_ptr, col_idx, N):
    """Initial edge-degree node embedding -> x [N, 9, C]; see ``ops/scatter.py:527``."""
    return _InitNodeScatter.apply(rad_out, wigner, env, Z, batch, W_sphere, csd_emb, idx_j, row_ptr, col_idx, int(N))
