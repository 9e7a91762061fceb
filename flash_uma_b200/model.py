"""Model graph of the hot path: Morton reorder, cached CSRs, geometry, radial MLPs and the
message-passing layers, driving the CUDA ops of :mod:`flash_uma_b200.ops`.

Mirrors the reference ``model.py`` (``reorder_graph_morton`` :56-74, ``build_csr_cached``
:28-44, ``Packed_eSCN_Layer`` :81-157, ``eSCN_Inference_Model`` :160-221). The dense
contractions (radial MLP and SO(2) convolutions, ``F.linear`` / cuBLAS in the reference)
run on this library's tcgen05 tensor-core GEMMs (:class:`~flash_uma_b200.linear.FrozenLinear`),
f16x3 by default (``FUMA_GEMM=tf32x3`` / ``tf32`` select the TF32 kernels).
"""
from __future__ import annotations

from collections import OrderedDict

import torch
import torch.nn as nn
import torch.nn.functional as F

import os

from . import fused, ops
from .linear import FrozenLinear
from .nodewise import EquivariantRMSNormSH, SpectralAtomwise, balance_channels_batched

# ---- graph preparation ---------------------------------------------------------------------

_GRAPH_CACHE_CAPACITY = 8
_graph_cache: "OrderedDict[tuple, ops.GraphCSR]" = OrderedDict()


def _cache_key(idx_i: torch.Tensor, idx_j: torch.Tensor, N: int) -> tuple:
    # same invalidation rule as model.py:28-44: storage pointer, in-place version, size, device
    dev = idx_j.device.index if idx_j.device.type == "cuda" else -1
    return (idx_i.data_ptr(), idx_i._version, idx_j.data_ptr(), idx_j._version, idx_j.numel(), N, dev)


def build_graph_cached(idx_i: torch.Tensor, idx_j: torch.Tensor, N: int) -> ops.GraphCSR:
    """Destination + source CSR of the edges, LRU-cached on the index tensors (``model.py:28-44``)."""
    key = _cache_key(idx_i, idx_j, N)
    hit = _graph_cache.get(key)
    if hit is not None:
        _graph_cache.move_to_end(key)
        return hit
    g = ops.build_graph_csr(idx_i, idx_j, N)
    # keep the index tensors alive so their storage (and the key) cannot be recycled
    g.keepalive = (idx_i, idx_j)
    _graph_cache[key] = g
    if len(_graph_cache) > _GRAPH_CACHE_CAPACITY:
        _graph_cache.popitem(last=False)
    return g


def clear_graph_cache() -> None:
    _graph_cache.clear()


def _expand_bits(v: torch.Tensor) -> torch.Tensor:
    v = (v | (v << 16)) & 0x030000FF
    v = (v | (v << 8)) & 0x0300F00F
    v = (v | (v << 4)) & 0x030C30C3
    v = (v | (v << 2)) & 0x09249249
    return v


def reorder_graph_morton(pos, Z, batch, idx_i, idx_j):
    """Sort atoms by (system, 30-bit Morton code of the position quantised to 10 bits per
    axis over the bounding box) and remap the edges (``model.py:47-74``); stable sort. On the
    GPU ``fuma_morton_reorder`` does all but the position gather (kept in torch, so forces flow
    back through it): one shared-memory sort for up to 16,384 atoms, a multi-block radix sort
    on a scratch buffer above that."""
    if pos.is_cuda and pos.shape[0] > 0:
        return _reorder_native(pos, Z, batch, idx_i, idx_j)
    return _reorder_torch(pos, Z, batch, idx_i, idx_j)


def _reorder_torch(pos, Z, batch, idx_i, idx_j):
    pos_min = pos.min(dim=0, keepdim=True)[0]
    pos_max = pos.max(dim=0, keepdim=True)[0]
    scale = 1023.0 / torch.clamp(pos_max - pos_min, min=1e-5)
    q = ((pos - pos_min) * scale).to(torch.int32)
    code = _expand_bits(q[:, 0]) | (_expand_bits(q[:, 1]) << 1) | (_expand_bits(q[:, 2]) << 2)
    keys = code.to(torch.int64) | (batch.to(torch.int64) << 32)
    perm = torch.argsort(keys, stable=True)
    inv_perm = torch.empty_like(perm)
    inv_perm[perm] = torch.arange(len(perm), device=pos.device)
    return pos[perm], Z[perm], batch[perm], inv_perm[idx_i], inv_perm[idx_j], perm, inv_perm


def _reorder_native(pos, Z, batch, idx_i, idx_j):
    from ._native import call, load, ptr, stream_of
    from .linear import error_flag
    N, E = pos.shape[0], idx_i.shape[0]
    p = pos.detach().float().contiguous()
    Z, batch = Z.long().contiguous(), batch.long().contiguous()
    idx_i, idx_j = idx_i.long().contiguous(), idx_j.long().contiguous()
    i64 = dict(device=pos.device, dtype=torch.int64)
    perm, inv_perm = torch.empty(N, **i64), torch.empty(N, **i64)
    Z_s, batch_s = torch.empty(N, **i64), torch.empty(N, **i64)
    ii, jj = torch.empty(E, **i64), torch.empty(E, **i64)
    nbytes = int(load().fuma_morton_scratch_bytes(N))
    scratch = torch.empty(max(nbytes, 1), device=pos.device, dtype=torch.uint8) if nbytes else None
    call("fuma_morton_reorder", ptr(p), ptr(Z), ptr(batch), ptr(idx_i), ptr(idx_j), N, E, ptr(perm), ptr(inv_perm),
         None, ptr(Z_s), ptr(batch_s), ptr(ii), ptr(jj), ptr(scratch), nbytes, ptr(error_flag(pos.device)), stream_of(p))
    return pos[perm], Z_s, batch_s, ii, jj, perm, inv_perm


# ---- layers ------------------------------------------------------------------------------------

def pack_complex(R: torch.Tensor, I: torch.Tensor) -> torch.Tensor:
    """Real block form [[R, -I], [I, R]] of the complex SO(2) map R + iI (``model.py:101-138``)."""
    return torch.cat([torch.cat([R, -I], 1), torch.cat([I, R], 1)], 0)


class RadialMLP(nn.Module):
    """Linear -> LN-SiLU -> Linear -> LN-SiLU -> Linear (``model.py:147-149``, ``:203-205``)."""

    def __init__(self, net, mode=None):
        super().__init__()
        g = lambda t: t.detach().clone().float()
        self.l1 = FrozenLinear(net[0].weight, net[0].bias, mode)
        self.register_buffer("g1", g(net[1].weight)); self.register_buffer("be1", g(net[1].bias))
        self.l2 = FrozenLinear(net[3].weight, net[3].bias, mode)
        self.register_buffer("g2", g(net[4].weight)); self.register_buffer("be2", g(net[4].bias))
        self.l3 = FrozenLinear(net[6].weight, net[6].bias, mode)

    def forward(self, x_edge):
        h1 = ops.layer_norm_silu(self.l1(x_edge), self.g1, self.be1)
        h2 = ops.layer_norm_silu(self.l2(h1), self.g2, self.be2)
        return self.l3(h2)


def apply_norm(norm, x):
    """``norm(x)``: the fused CUDA kernels for the :class:`EquivariantRMSNormSH` modules (the
    stand-in norms), the module itself for any other normalisation module."""
    if type(norm) is EquivariantRMSNormSH and x.is_cuda and norm.lmax == 2:
        return ops.rms_norm_sh(x, norm)
    return norm(x)


def apply_atomwise(aw, xn, x_mid, mode=None):
    """``aw(xn) + x_mid``: the fused CUDA path for the :class:`SpectralAtomwise` modules (the
    stand-in atom-wise blocks; its linear maps in the layer's GEMM ``mode``), the module itself
    for any other atom-wise module."""
    if type(aw) is SpectralAtomwise and xn.is_cuda and aw.lmax == 2:
        return ops.atomwise_residual(aw, xn, x_mid, mode)
    return (aw(xn) + x_mid).contiguous()


class PackedLayer(nn.Module):
    """One eSCN message-passing block (``Packed_eSCN_Layer``, ``model.py:81-157``)."""

    def __init__(self, blk, C: int, mode=None):
        super().__init__()
        c1, c2 = blk.edge_wise.so2_conv_1, blk.edge_wise.so2_conv_2
        g = lambda t: t.detach().clone().float()
        self.C = C
        self.rad = RadialMLP(c1.rad_func.net, mode)
        self.conv1_m0 = FrozenLinear(c1.fc_m0.weight, c1.fc_m0.bias, mode)
        w = g(c1.so2_m_conv[0].fc.weight); self.conv1_m1 = FrozenLinear(pack_complex(w[:2 * C], w[2 * C:]), None, mode)
        w = g(c1.so2_m_conv[1].fc.weight); self.conv1_m2 = FrozenLinear(pack_complex(w[:C], w[C:]), None, mode)
        self.conv2_m0 = FrozenLinear(c2.fc_m0.weight, c2.fc_m0.bias, mode)
        w = g(c2.so2_m_conv[0].fc.weight); self.conv2_m1 = FrozenLinear(pack_complex(w[:2 * C], w[2 * C:]), None, mode)
        w = g(c2.so2_m_conv[1].fc.weight); self.conv2_m2 = FrozenLinear(pack_complex(w[:C], w[C:]), None, mode)
        self.norm_1, self.norm_2, self.atom_wise = blk.norm_1, blk.norm_2, blk.atom_wise
        for m in (self.norm_1, self.norm_2, self.atom_wise):
            for p in m.parameters():
                p.requires_grad_(False)

    fused = False   # set by ESCNInferenceModel: x_edge is then the row-packed split of the edge features
    lean = False    # set per step by ESCNInferenceModel for graphs too large to keep every activation

    def forward(self, x_in, x_edge, wigner, env, idx_i, idx_j, graph, csd_emb, batch, n_out=None):
        """``n_out``: return only the first ``n_out`` atoms' outputs (the partitioned model's owned
        atoms; the node-wise tail then skips the halo rows, whose messages are not computed here)."""
        x_norm = apply_norm(self.norm_1, x_in)
        if self.fused:
            x_mid = fused.message_block(self, x_norm, x_in, x_edge, wigner, env, csd_emb, idx_i, idx_j, batch, graph,
                                        self.lean)
            if n_out is not None:
                x_mid = x_mid[:n_out]
            return apply_atomwise(self.atom_wise, apply_norm(self.norm_2, x_mid), x_mid, self.conv1_m0.mode)
        rad_out = self.rad(x_edge)
        X0, X1, X2 = ops.gather_wigner_split(x_norm, idx_i, idx_j, wigner, rad_out, csd_emb, batch, graph=graph)
        Z0, Z1, Z2 = ops.fused_gating_split(self.conv1_m0(X0), self.conv1_m1(X1), self.conv1_m2(X2), self.C)
        O0, O1, O2 = self.conv2_m0(Z0), self.conv2_m1(Z1), self.conv2_m2(Z2)
        x_mid = ops.rotate_scatter_split(O0, O1, O2, wigner, env, x_in, idx_j, graph.dst_row_ptr, graph.dst_col,
                                         x_in.shape[0])
        if n_out is not None:
            x_mid = x_mid[:n_out]
        return apply_atomwise(self.atom_wise, apply_norm(self.norm_2, x_mid), x_mid, self.conv1_m0.mode)


class ESCNInferenceModel(nn.Module):
    """``eSCN_Inference_Model`` (``model.py:160-221``) built from a FAIRChem-layout backbone."""

    def __init__(self, off_bb, mode=None):
        super().__init__()
        self.C = int(off_bb.sphere_channels)
        self.B = int(off_bb.num_distance_basis)
        self.cutoff = float(off_bb.cutoff)
        offset = torch.linspace(0.0, self.cutoff, self.B)
        self.coeff_g = float(-0.5 / (2.0 * (offset[1] - offset[0])) ** 2)  # wrapper.py:122-125
        g = lambda t: t.detach().clone().float()
        self.register_buffer("offset_g", offset)
        self.register_buffer("W_sphere", g(off_bb.sphere_embedding.weight))
        self.register_buffer("W_src", g(off_bb.source_embedding.weight))
        self.register_buffer("W_tgt", g(off_bb.target_embedding.weight))
        self.rad_init = RadialMLP(off_bb.edge_degree_embedding.rad_func.net, mode)
        self.layers = nn.ModuleList([PackedLayer(b, self.C, mode) for b in off_bb.blocks])
        for rad in [self.rad_init] + [lay.rad for lay in self.layers]:
            rad.n_gauss = self.B   # leading edge-feature columns that depend on positions
        self.final_norm = off_bb.norm
        for p in self.final_norm.parameters():
            p.requires_grad_(False)
        self.charge_start, self.charge_end = off_bb.charge_channel_start, off_bb.charge_channel_end
        self.spin_start, self.spin_end = off_bb.spin_channel_start, off_bb.spin_channel_end
        # f16x3 with GEMM widths that are multiples of 16: fused blocks on split operands
        # (FUMA_FUSED=0 keeps the per-op path, for comparisons)
        self.set_fused(os.environ.get("FUMA_FUSED", "1") != "0")

    def set_fused(self, enable: bool) -> bool:
        """Use the fused f16x3 blocks when possible (``enable``) or the per-op path; returns the mode."""
        self.fused = bool(enable) and fused.fusable(self)
        for lay in self.layers:
            lay.fused = self.fused
        return self.fused

    def _linears(self):
        return [m for m in self.modules() if isinstance(m, FrozenLinear)]

    # ---- stages (also driven one by one by the spatially partitioned model, partition.py) ----
    def build_graph(self, idx_i, idx_j, N):
        return build_graph_cached(idx_i, idx_j, N)

    def build_graph_renumbered(self, edge_index, perm, N):
        """CSRs of the Morton-renumbered edges (``model.py:189-191``): the CSRs of the caller's
        numbering are cached on the caller's edge list, which stays the same across MD steps,
        and renumbered on every call without a sort (:func:`ops.permute_graph`); the result is
        bitwise the stable-argsort CSR of the renumbered edges."""
        return ops.permute_graph(build_graph_cached(edge_index[0], edge_index[1], N), perm)

    def geometry(self, pos, Z, idx_i, idx_j, shifts, graph):
        """(x_edge, wigner, env); in the fused mode x_edge comes back as (its row-packed split,
        its Gaussian-basis columns), see :func:`flash_uma_b200.fused.geometry`."""
        if self.fused:
            for lin in self._linears():
                lin.prepare()
            lean = fused.lean_needed(int(idx_i.shape[0]), self.C, self.layers[0].rad.l1.N if len(self.layers) else 0,
                                     len(self.layers), pos.device)
            for lay in self.layers:
                lay.lean = lean
            return fused.geometry(pos, Z, idx_i, idx_j, shifts, self.W_src, self.W_tgt, self.offset_g, self.coeff_g,
                                  self.cutoff, graph)
        return ops.precompute_geometry(pos, Z, idx_i, idx_j, shifts, self.W_src, self.W_tgt, self.offset_g,
                                       self.coeff_g, self.cutoff, graph=graph)

    def init_embedding(self, x_edge, wigner, env, Z, batch, csd_emb, idx_j, graph, N):
        if self.fused:
            return fused.init_block(self, x_edge, wigner, env, Z, batch, csd_emb, graph, N)
        rad0 = self.rad_init(x_edge)
        return ops.init_node_scatter(rad0, wigner, env, Z, batch, self.W_sphere, csd_emb, idx_j, graph.dst_row_ptr,
                                     graph.dst_col, N)

    def layer_forward(self, k, x, x_edge, wigner, env, idx_i, idx_j, graph, csd_emb, batch, charge=None, spin=None,
                      natoms=None, n_out=None, partitioned: bool = False, group=None):
        """``partitioned``: x holds one rank's atoms of systems spread over ``group`` (the channel
        balancing then sums over all ranks)."""
        x = self.layers[k](x, x_edge, wigner, env, idx_i, idx_j, graph, csd_emb, batch, n_out)
        if n_out is not None:
            batch = batch[:n_out]
        if self.charge_end > self.charge_start:
            x = balance_channels_batched(x, charge, natoms, batch, self.charge_start, self.charge_end, 0.0,
                                         partitioned, group)
        if self.spin_end > self.spin_start:
            x = balance_channels_batched(x, spin, natoms, batch, self.spin_start, self.spin_end, 1.0, partitioned,
                                         group)
        return x

    def final(self, x):
        return apply_norm(self.final_norm, x)

    def forward(self, pos, Z, batch, edge_index, shifts, csd_emb, charge=None, spin=None, natoms=None):
        pos_s, Z_s, batch_s, ii, jj, perm, inv_perm = reorder_graph_morton(pos, Z, batch, edge_index[0], edge_index[1])
        N = pos_s.shape[0]
        graph = self.build_graph_renumbered(edge_index, perm, N)
        x_edge, wigner, env = self.geometry(pos_s, Z_s, ii, jj, shifts, graph)
        x = self.init_embedding(x_edge, wigner, env, Z_s, batch_s, csd_emb, jj, graph, N)
        for k in range(len(self.layers)):
            x = self.layer_forward(k, x, x_edge, wigner, env, ii, jj, graph, csd_emb, batch_s, charge, spin, natoms)
        return self.final(x)[inv_perm]
