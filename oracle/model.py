"""CPU restatement of the reference model graph and drop-in wrapper (test infrastructure).

Follows ``model.py:17-74`` (Morton reorder, CSR), ``model.py:101-157`` (weight
packing, layer forward), ``model.py:187-221`` (model forward) and
``wrapper.py:22-85,122-125,163-169,192-210`` (weight transfer, Gaussian
coefficient, csd embedding, PBC shifts), using ``oracle.ops`` for the fused ops
and plain ``F.linear`` for the dense contractions. The node-wise FAIRChem modules
are shared by reference (the same objects the CUDA path uses).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import ops


def expand_bits(v: torch.Tensor) -> torch.Tensor:
    """Spread the low 10 bits of v so that two zero bits follow each (``model.py:47-53``)."""
    v = (v | (v << 16)) & 0x030000FF
    v = (v | (v << 8)) & 0x0300F00F
    v = (v | (v << 4)) & 0x030C30C3
    v = (v | (v << 2)) & 0x09249249
    return v


def morton3d(x, y, z):
    """30-bit Morton code, x in the lowest bit of each triple (``model.py:55-57``)."""
    return expand_bits(x) | (expand_bits(y) << 1) | (expand_bits(z) << 2)


def reorder_graph_morton(pos, Z, batch, idx_i, idx_j):
    """Quantise positions to 10 bits per axis over the bounding box, sort atoms by
    (batch << 32) | morton and remap the edge endpoints (``model.py:60-74``).
    A stable sort is used; ties do not change results (everything is mapped back)."""
    pos_min = pos.min(dim=0, keepdim=True)[0]
    pos_max = pos.max(dim=0, keepdim=True)[0]
    scale = 1023.0 / torch.clamp(pos_max - pos_min, min=1e-5)
    q = ((pos - pos_min) * scale).to(torch.int32)
    code = morton3d(q[:, 0], q[:, 1], q[:, 2])
    keys = code.to(torch.int64) | (batch.to(torch.int64) << 32)
    perm = torch.argsort(keys, stable=True)
    inv_perm = torch.empty_like(perm)
    inv_perm[perm] = torch.arange(len(perm))
    return pos[perm], Z[perm], batch[perm], inv_perm[idx_i], inv_perm[idx_j], perm, inv_perm


def build_csr(idx: torch.Tensor, N: int):
    """Destination CSR: row_ptr[N+1] int32 (exclusive prefix of counts), col_idx[E] int32 =
    stable argsort of idx (``model.py:20-26``)."""
    order = torch.argsort(idx, stable=True)
    counts = torch.bincount(idx, minlength=N)
    row_ptr = torch.zeros(N + 1, dtype=torch.int32)
    row_ptr[1:] = torch.cumsum(counts, 0).to(torch.int32)
    return row_ptr, order.to(torch.int32)


def pack_complex(R: torch.Tensor, I: torch.Tensor) -> torch.Tensor:
    """[[R, -I], [I, R]]: the real form of the complex SO(2) map R + iI (``model.py:101-138``)."""
    return torch.cat([torch.cat([R, -I], 1), torch.cat([I, R], 1)], 0)


class _Radial:
    def __init__(self, net, dtype):
        self.W1, self.b1 = net[0].weight.detach().to(dtype), net[0].bias.detach().to(dtype)
        self.g1, self.be1 = net[1].weight.detach().to(dtype), net[1].bias.detach().to(dtype)
        self.W2, self.b2 = net[3].weight.detach().to(dtype), net[3].bias.detach().to(dtype)
        self.g2, self.be2 = net[4].weight.detach().to(dtype), net[4].bias.detach().to(dtype)
        self.W3, self.b3 = net[6].weight.detach().to(dtype), net[6].bias.detach().to(dtype)

    def __call__(self, x_edge):
        h1 = ops.layer_norm_silu(F.linear(x_edge, self.W1, self.b1), self.g1, self.be1)
        h2 = ops.layer_norm_silu(F.linear(h1, self.W2, self.b2), self.g2, self.be2)
        return F.linear(h2, self.W3, self.b3)


class OracleLayer:
    """``Packed_eSCN_Layer`` (``model.py:81-157``) with weights copied from a FAIRChem-layout block."""

    def __init__(self, blk, C, dtype):
        c1, c2 = blk.edge_wise.so2_conv_1, blk.edge_wise.so2_conv_2
        self.C = C
        self.rad = _Radial(c1.rad_func.net, dtype)
        d = lambda t: t.detach().to(dtype)
        self.W1_m0, self.b1_m0 = d(c1.fc_m0.weight), d(c1.fc_m0.bias)
        w = d(c1.so2_m_conv[0].fc.weight); self.W1_m1 = pack_complex(w[:2 * C], w[2 * C:])
        w = d(c1.so2_m_conv[1].fc.weight); self.W1_m2 = pack_complex(w[:C], w[C:])
        self.W2_m0, self.b2_m0 = d(c2.fc_m0.weight), d(c2.fc_m0.bias)
        w = d(c2.so2_m_conv[0].fc.weight); self.W2_m1 = pack_complex(w[:2 * C], w[2 * C:])
        w = d(c2.so2_m_conv[1].fc.weight); self.W2_m2 = pack_complex(w[:C], w[C:])
        self.norm_1, self.norm_2, self.atom_wise = blk.norm_1, blk.norm_2, blk.atom_wise

    def __call__(self, x_in, x_edge, wigner, env, idx_i, idx_j, row_ptr, col_idx, csd_emb, batch, n_out=None):
        x_norm = self.norm_1(x_in)
        rad_out = self.rad(x_edge)
        X0, X1, X2 = ops.gather_wigner_split(x_norm, idx_i, idx_j, wigner, rad_out, csd_emb, batch)
        Y0, Y1, Y2 = F.linear(X0, self.W1_m0, self.b1_m0), F.linear(X1, self.W1_m1), F.linear(X2, self.W1_m2)
        Z0, Z1, Z2 = ops.fused_gating_split(Y0, Y1, Y2, self.C)
        O0, O1, O2 = F.linear(Z0, self.W2_m0, self.b2_m0), F.linear(Z1, self.W2_m1), F.linear(Z2, self.W2_m2)
        x_mid = ops.rotate_scatter_split(O0, O1, O2, wigner, env, x_in, idx_j, row_ptr, col_idx, x_in.shape[0])
        if n_out is not None:   # only the first n_out atoms' outputs are wanted (partitioned model)
            x_mid = x_mid[:n_out]
        return self.atom_wise(self.norm_2(x_mid)) + x_mid


class OracleBackbone:
    """CPU oracle of ``ZeroAllocBackbone`` (``wrapper.py:88-211``) + ``eSCN_Inference_Model``."""

    def __init__(self, off_bb, dtype=torch.float32, checkpoint_layers: bool = False):
        """``checkpoint_layers``: keep only each layer's input for the backward and recompute the
        layer there (torch.utils.checkpoint), which bounds host memory by one layer's activations
        (the full-size configurations); the arithmetic is unchanged."""
        self.dtype = dtype
        self.checkpoint_layers = checkpoint_layers
        self.C = off_bb.sphere_channels
        self.B = off_bb.num_distance_basis
        self.cutoff = float(off_bb.cutoff)
        offset = torch.linspace(0.0, self.cutoff, self.B)
        self.coeff_g = float(-0.5 / (2.0 * (offset[1] - offset[0])) ** 2)   # wrapper.py:124-125
        self.offset_g = offset.to(dtype)
        d = lambda t: t.detach().to(dtype)
        self.W_sphere = d(off_bb.sphere_embedding.weight)
        self.W_src = d(off_bb.source_embedding.weight)
        self.W_tgt = d(off_bb.target_embedding.weight)
        self.rad_init = _Radial(off_bb.edge_degree_embedding.rad_func.net, dtype)
        self.layers = [OracleLayer(b, self.C, dtype) for b in off_bb.blocks]
        self.final_norm = off_bb.norm
        self.off_bb = off_bb
        self.charge_range = (off_bb.charge_channel_start, off_bb.charge_channel_end)
        self.spin_range = (off_bb.spin_channel_start, off_bb.spin_channel_end)
        self.regress_config = off_bb.regress_config

    def csd_embedding(self, charge, spin, dataset=None):
        """``wrapper.py:163-169``."""
        bb = self.off_bb
        chg, sp = bb.charge_embedding(charge), bb.spin_embedding(spin)
        if bb.use_dataset_embedding and dataset is not None:
            return F.silu(bb.mix_csd(torch.cat((chg, sp, bb.dataset_embedding(dataset)), dim=1)))
        return F.silu(bb.mix_csd(torch.cat((chg, sp), dim=1)))

    # ---- stages (the same protocol as the CUDA model; used by the partitioned driver) ----
    def build_graph(self, idx_i, idx_j, N):
        row_ptr, col_idx = build_csr(idx_j, N)
        return (row_ptr, col_idx)

    def geometry(self, pos, Z, idx_i, idx_j, shifts, graph):
        return ops.precompute_geometry(pos, Z, idx_i, idx_j, shifts, self.W_src, self.W_tgt, self.offset_g,
                                       self.coeff_g, self.cutoff)

    def init_embedding(self, x_edge, wigner, env, Z, batch, csd_emb, idx_j, graph, N):
        rad0 = self.rad_init(x_edge)
        return ops.init_node_scatter(rad0, wigner, env, Z, batch, self.W_sphere, csd_emb, idx_j, graph[0], graph[1], N)

    def layer_forward(self, k, x, x_edge, wigner, env, idx_i, idx_j, graph, csd_emb, batch, charge=None, spin=None,
                      natoms=None, n_out=None, partitioned: bool = False, group=None):
        from flash_uma_b200.nodewise import balance_channels_batched
        x = self.layers[k](x, x_edge, wigner, env, idx_i, idx_j, graph[0], graph[1], csd_emb, batch, n_out)
        if n_out is not None:
            batch = batch[:n_out]
        if self.charge_range[1] > self.charge_range[0]:
            x = balance_channels_batched(x, charge, natoms, batch, *self.charge_range, target_offset=0.0,
                                         partitioned=partitioned, group=group)
        if self.spin_range[1] > self.spin_range[0]:
            x = balance_channels_batched(x, spin, natoms, batch, *self.spin_range, target_offset=1.0,
                                         partitioned=partitioned, group=group)
        return x

    def final(self, x):
        return self.final_norm(x)

    def model_forward(self, pos, Z, batch, edge_index, shifts, csd_emb, charge=None, spin=None, natoms=None):
        """``model.py:187-221``."""
        pos_s, Z_s, batch_s, ii, jj, perm, inv_perm = reorder_graph_morton(pos, Z, batch, edge_index[0], edge_index[1])
        N = pos_s.shape[0]
        graph = self.build_graph(ii, jj, N)
        x_edge, wigner, env = self.geometry(pos_s, Z_s, ii, jj, shifts, graph)
        x = self.init_embedding(x_edge, wigner, env, Z_s, batch_s, csd_emb, jj, graph, N)
        for k in range(len(self.layers)):
            args = (k, x, x_edge, wigner, env, ii, jj, graph, csd_emb, batch_s, charge, spin, natoms)
            if self.checkpoint_layers and torch.is_grad_enabled():
                from torch.utils.checkpoint import checkpoint
                x = checkpoint(self.layer_forward, *args, use_reentrant=False)
            else:
                x = self.layer_forward(*args)
        return self.final(x)[inv_perm]

    def forward(self, data):
        """``wrapper.py:171-211``: enables pos/cell grads, builds csd embedding and shifts."""
        rc = self.regress_config
        if not rc.direct_forces:
            if getattr(rc, "forces", False) or getattr(rc, "stress", False):
                data.pos.requires_grad_(True)
            if getattr(rc, "stress", False) and data.cell is not None and data.cell.is_floating_point():
                data.cell.requires_grad_(True)
        csd = self.csd_embedding(data.charge, data.spin, getattr(data, "dataset", None)).to(self.dtype)
        if len(data.natoms) == 1:
            shifts = data.cell_offsets.to(data.cell.dtype) @ data.cell.squeeze(0)
        else:
            cpe = data.cell.repeat_interleave(data.nedges, dim=0)
            shifts = torch.einsum("ij,ijk->ik", data.cell_offsets.to(cpe.dtype), cpe)
        x = self.model_forward(data.pos.to(self.dtype), data.atomic_numbers.long(), data.batch, data.edge_index,
                               shifts.to(self.dtype), csd, data.charge, data.spin, data.natoms)
        return {"node_embedding": x, "batch": data.batch}

    __call__ = forward
