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
from . import library  # noqa: F401  (registers the fuma:: custom operators)
from ._native import ptr, stream_of
from .linear import _gemm16, error_flag


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


class _AtomwiseResidualTC(torch.autograd.Function):
    """y = x_mid + atom_wise(xn) with the per-degree maps on the fp16 tensor cores.

    The coefficient rows of xn (row k * N + n = xn[n, k]) are written as the row-packed split
    the GEMMs read; each per-degree map is one GEMM over all 9N rows against the three degree
    weights stacked, whose degree-blocked output the next kernel reads at the row's own degree
    (the unused two thirds of that product cost far less than two more launches)."""

    @staticmethod
    def forward(ctx, xn, x_mid, tc):
        nat.require_cuda(xn, x_mid)
        xn, x_mid = _f32(xn, "xn"), _f32(x_mid, "x_mid")
        N, _, C = xn.shape
        H = tc.H
        s, err, dev = stream_of(xn), ptr(error_flag(xn.device)), xn.device
        xs = torch.empty(9 * N, C, device=dev)
        nat.call("fuma_node_to_coef_f16x3", ptr(xn), N, C, ptr(xs), tc.parts, err, s)
        u = _gemm16(xs[:N], tc.scalar.w16, tc.scalar.bias_p, C)                  # [N, 2H]
        h = _gemm16(xs, tc.lin1.w16, None, C)                                    # [9N, 3H] degree-blocked
        zs = torch.empty(9 * N, H, device=dev)
        nat.call("fuma_atomwise_gate_fwd_f16x3", ptr(h), ptr(u), ptr(tc.b1), N, H, ptr(zs), tc.parts, err, s)
        o = _gemm16(zs, tc.lin2.w16, None, H)                                    # [9N, 3C] degree-blocked
        y = torch.empty_like(x_mid)
        nat.call("fuma_coef_to_node_blocked", ptr(o), ptr(x_mid), ptr(tc.b2), 0, N, C, ptr(y), s)
        ctx.save_for_backward(h, u)
        ctx.tc = tc
        return y

    @staticmethod
    def backward(ctx, gy):
        h, u = ctx.saved_tensors
        tc = ctx.tc
        gy = _f32(gy, "gy")
        N, _, C = gy.shape
        H = tc.H
        s, err, dev = stream_of(gy), ptr(error_flag(gy.device)), gy.device
        gs = torch.empty(9 * N, C, device=dev)
        nat.call("fuma_node_to_coef_f16x3", ptr(gy), N, C, ptr(gs), tc.parts, err, s)
        gz = _gemm16(gs, tc.lin2t.w16, None, C)                                  # [9N, 3H] degree-blocked
        ghs, gus = torch.empty(9 * N, H, device=dev), torch.empty(N, 2 * H, device=dev)
        nat.call("fuma_atomwise_gate_bwd_f16x3", ptr(gz), ptr(h), ptr(u), ptr(tc.b1), N, H, ptr(ghs), ptr(gus),
                 tc.parts, err, s)
        gx = _gemm16(ghs, tc.lin1t.w16, None, H)                                 # [9N, 3C] degree-blocked
        gu_x = _gemm16(gus, tc.scalar.wt16, None, 2 * H)                         # [N, C]
        gxn = torch.empty_like(gy)
        nat.call("fuma_coef_to_node_blocked", ptr(gx), None, ptr(gu_x), 1, N, C, ptr(gxn), s)
        return gxn, gy, None


class _AtomwiseTC:
    """Tensor-core constants of a SpectralAtomwise block for one GEMM mode (cached on it):
    FrozenLinear splits of the scalar MLP and of the stacked degree weights of both maps and
    their transposes."""

    def __init__(self, aw, mode: str):
        from .linear import FrozenLinear
        f = lambda t: t.detach().float()   # noqa: E731
        W1, W2 = f(aw.so3_linear_1.weight), f(aw.so3_linear_2.weight)   # [3, H, C], [3, C, H]
        lin = aw.scalar_mlp[0]
        self.H = W1.shape[1]
        self.mode = mode
        self.parts = 1 if mode == "f16" else 2
        self.scalar = FrozenLinear(lin.weight, lin.bias, mode)
        self.lin1 = FrozenLinear(W1.reshape(-1, W1.shape[2]), None, mode)                  # [3H, C]
        self.lin2 = FrozenLinear(W2.reshape(-1, W2.shape[2]), None, mode)                  # [3C, H]
        self.lin2t = FrozenLinear(W2.transpose(1, 2).reshape(-1, W2.shape[1]), None, mode)  # [3H, C]
        self.lin1t = FrozenLinear(W1.transpose(1, 2).reshape(-1, W1.shape[1]), None, mode)  # [3C, H]
        self.b1 = f(aw.so3_linear_1.bias).contiguous()
        self.b2 = f(aw.so3_linear_2.bias).contiguous()
        for m in (self.scalar, self.lin1, self.lin2, self.lin2t, self.lin1t):
            m.prepare()


def _atomwise_tc(aw, mode: str) -> _AtomwiseTC:
    dev = aw.so3_linear_1.weight.device
    cache = aw.__dict__.setdefault("_fuma_tc", {})
    tc = cache.get(mode)
    if tc is None or tc.b1.device != dev:
        tc = cache[mode] = _AtomwiseTC(aw, mode)
    return tc


def atomwise_residual(aw, xn: torch.Tensor, x_mid: torch.Tensor, mode: str | None = None) -> torch.Tensor:
    """``x_mid + aw(xn)`` for a :class:`~flash_uma_b200.nodewise.SpectralAtomwise` (lmax 2), frozen
    parameters. ``mode`` (default: the ``FUMA_GEMM`` mode) "f16x3" / "f16": the per-degree maps
    and the scalar MLP on the fp16 tensor cores (fp32 accuracy / single product), gating and the
    layout changes as CUDA kernels; "tf32x3" / "tf32": batched fp32 GEMMs (cuBLAS) between the
    same kernels."""
    from .linear import _F16_MODES, default_mode
    if aw.lmax != 2 or (aw.hidden % 4) or (xn.shape[2] % 4):
        raise ValueError("atomwise_residual: lmax 2 and channel counts that are multiples of 4")
    mode = mode or default_mode()
    if mode in _F16_MODES and aw.hidden % 16 == 0 and xn.shape[2] % 16 == 0:   # stacked widths 3H, 3C: GEMM tiles
        return _AtomwiseResidualTC.apply(xn, x_mid, _atomwise_tc(aw, mode))
    return _AtomwiseResidual.apply(xn, x_mid, atomwise_constants(aw))


# ---------------------------------------------------------------------------------------------
def _csr_args(graph):
    if graph is None:
        return None, None, None, None
    return graph.dst_row_ptr, graph.dst_col, graph.src_row_ptr, graph.src_col


def precompute_geometry(pos, Z, idx_i, idx_j, shifts, W_src, W_tgt, offset_g, coeff_g, cutoff, *, graph=None):
    """Edge geometry -> (x_edge_raw [E, B+2C], wigner [E, 34], env [E]); see ``ops/geom.py:591``.
    Custom operator ``fuma::precompute_geometry`` (:mod:`flash_uma_b200.library`)."""
    nat.require_cuda(pos, Z, idx_i, idx_j, shifts, W_src, W_tgt, offset_g)
    return torch.ops.fuma.precompute_geometry(_f32(pos, "pos"), _i64(Z), _i64(idx_i), _i64(idx_j),
                                              _f32(shifts, "shifts"), _f32(W_src, "W_src"), _f32(W_tgt, "W_tgt"),
                                              _f32(offset_g, "offset_g"), float(coeff_g), float(cutoff),
                                              *_csr_args(graph))


def layer_norm_silu(x, gamma, beta, eps=1e-7):
    """Fused row-wise LayerNorm + SiLU on [M, D]; see ``ops/ln_silu.py:180``. Custom operator
    ``fuma::layer_norm_silu`` (its row statistics, also returned, feed the backward)."""
    nat.require_cuda(x, gamma, beta)
    return torch.ops.fuma.layer_norm_silu(_f32(x, "x"), _f32(gamma, "gamma"), _f32(beta, "beta"), float(eps))[0]


def gather_wigner_split(x_in, idx_i, idx_j, wigner, rad_out, csd_emb, batch, *, graph=None):
    """Gather + rotate into the edge frame + radial scale -> (X_m0, X_m1, X_m2); see
    ``ops/gather.py:516``. Custom operator ``fuma::gather_wigner_split``; ``graph``: cached
    CSRs of the edges for the deterministic backward (built there otherwise)."""
    nat.require_cuda(x_in, idx_i, idx_j, wigner, rad_out, csd_emb, batch)
    return torch.ops.fuma.gather_wigner_split(_f32(x_in, "x_in"), _i64(idx_i), _i64(idx_j), _f32(wigner, "wigner"),
                                              _f32(rad_out, "rad_out"), _f32(csd_emb, "csd_emb"), _i64(batch),
                                              *_csr_args(graph))


def fused_gating_split(Y_m0, Y_m1, Y_m2, C):
    """Split gating -> (Z_m0, Z_m1, Z_m2); see ``ops/gating.py:236``. Custom operator
    ``fuma::fused_gating_split``."""
    nat.require_cuda(Y_m0, Y_m1, Y_m2)
    return torch.ops.fuma.fused_gating_split(_f32(Y_m0, "Y_m0"), _f32(Y_m1, "Y_m1"), _f32(Y_m2, "Y_m2"), int(C))


def rotate_scatter_split(Z_m0, Z_m1, Z_m2, wigner, env, x_res, idx_j, row_ptr, col_idx, N):
    """Rotate back + envelope + deterministic FP64 CSR sum + residual -> x_out [N, 9, C];
    see ``ops/scatter.py:354``. Custom operator ``fuma::rotate_scatter_split``."""
    nat.require_cuda(Z_m0, Z_m1, Z_m2, wigner, env, x_res, row_ptr, col_idx)
    return torch.ops.fuma.rotate_scatter_split(_f32(Z_m0, "Z_m0"), _f32(Z_m1, "Z_m1"), _f32(Z_m2, "Z_m2"),
                                               _f32(wigner, "wigner"), _f32(env, "env"), _f32(x_res, "x_res"),
                                               _i32(row_ptr), _i32(col_idx), int(N))


def init_node_scatter(rad_out, wigner, env, Z, batch, W_sphere, csd_emb, idx_j, row_ptr, col_idx, N):
    """Initial edge-degree node embedding -> x [N, 9, C]; see ``ops/scatter.py:527``. Custom
    operator ``fuma::init_node_scatter``."""
    nat.require_cuda(rad_out, wigner, env, Z, batch, W_sphere, csd_emb, row_ptr, col_idx)
    return torch.ops.fuma.init_node_scatter(_f32(rad_out, "rad_out"), _f32(wigner, "wigner"), _f32(env, "env"),
                                            _i64(Z), _i64(batch), _f32(W_sphere, "W_sphere"),
                                            _f32(csd_emb, "csd_emb"), _i32(row_ptr), _i32(col_idx), int(N))
