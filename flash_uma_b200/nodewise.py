"""Node-wise (O(N)) modules that sit around the message-passing hot path.

The reference attaches FAIRChem's own ``norm_1`` / ``norm_2`` / ``atom_wise`` /
``final_norm`` modules to its layers by reference (``wrapper.py:73-79``) and
calls them from ``Packed_eSCN_Layer.forward`` (``model.py:145,157``) and
``eSCN_Inference_Model.forward`` (``model.py:218``). ``fairchem-core`` is not
available here, so these are stand-ins written from the published UMA / eSCN-MD
description:

* ``EquivariantRMSNormSH`` - RMS norm over all spherical-harmonic coefficients,
  each degree l weighted by 1/((2l+1)(lmax+1)), l=0 centred over channels, one
  learned scale per (degree, channel) and a bias on l=0 only.
* ``SO3Linear`` - per-degree channel mixing, bias on l=0 only.
* ``SpectralAtomwise`` - gated feed-forward block: scalar MLP on l=0 produces one
  sigmoid gate per degree l>0; l=0 goes through SiLU.
* ``EnergyHead`` - MLP on the l=0 coefficients, summed per system.

Outputs are contiguous [N, 9, C] tensors, as FAIRChem's are: the reference's
rotate-scatter reads its residual input with the strides of a freshly allocated
contiguous output (``ops/scatter.py:302-310``).

The same module objects are used by the CUDA path and by the CPU oracle, so the
parity of the hot path is independent of how faithfully these copy FAIRChem.
They are ordinary PyTorch modules (cuBLAS GEMMs + elementwise kernels on the
GPU); they are outside the hot path.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

LMAX = 2
NUM_COEFFS = (LMAX + 1) ** 2  # 9
# degree of each of the 9 real-SH coefficients: [0, 1,1,1, 2,2,2,2,2]
COEFF_DEGREE = [0, 1, 1, 1, 2, 2, 2, 2, 2]


class EquivariantRMSNormSH(nn.Module):
    """Stand-in for FAIRChem's ``rms_norm_sh`` normalisation of [N, 9, C]."""

    def __init__(self, channels: int, lmax: int = LMAX, eps: float = 1e-5):
        super().__init__()
        self.lmax, self.channels, self.eps = lmax, channels, eps
        self.affine_weight = nn.Parameter(torch.ones(lmax + 1, channels))
        self.affine_bias = nn.Parameter(torch.zeros(channels))
        deg = torch.tensor(COEFF_DEGREE[: (lmax + 1) ** 2])
        w = 1.0 / ((2 * deg + 1).to(torch.float32) * (lmax + 1))
        self.register_buffer("balance_degree_weight", w, persistent=False)
        self.register_buffer("expand_index", deg, persistent=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        l0 = x[:, :1]
        l0 = l0 - l0.mean(dim=2, keepdim=True)
        feat = torch.cat([l0, x[:, 1:]], dim=1)
        w = self.balance_degree_weight.to(x.dtype)
        fnorm = (feat.pow(2) * w[None, :, None]).sum(dim=1, keepdim=True)
        fnorm = fnorm.mean(dim=2, keepdim=True)
        scale = torch.rsqrt(fnorm + self.eps)
        weight = self.affine_weight.index_select(0, self.expand_index)  # [9, C]
        out = feat * scale * weight[None]
        bias = torch.zeros_like(out[:1])
        bias[:, 0] = self.affine_bias
        return out + bias


class SO3Linear(nn.Module):
    """Per-degree linear map [N, 9, Cin] -> [N, 9, Cout]; bias on l=0 only."""

    def __init__(self, cin: int, cout: int, lmax: int = LMAX):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(lmax + 1, cout, cin))
        self.bias = nn.Parameter(torch.zeros(cout))
        self.register_buffer("expand_index", torch.tensor(COEFF_DEGREE[: (lmax + 1) ** 2]), persistent=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        w = self.weight.index_select(0, self.expand_index)  # [9, Cout, Cin]
        out = torch.einsum("nkc,koc->nko", x, w).contiguous()
        bias = torch.zeros_like(out[:1])
        bias[:, 0] = self.bias
        return out + bias


class SpectralAtomwise(nn.Module):
    """Gated atom-wise feed-forward block on [N, 9, C]."""

    def __init__(self, channels: int, hidden: int, lmax: int = LMAX):
        super().__init__()
        self.lmax, self.hidden = lmax, hidden
        self.scalar_mlp = nn.Sequential(nn.Linear(channels, lmax * hidden), nn.SiLU())
        self.so3_linear_1 = SO3Linear(channels, hidden, lmax)
        self.so3_linear_2 = SO3Linear(hidden, channels, lmax)
        self.register_buffer("gate_index", torch.tensor(COEFF_DEGREE[1: (lmax + 1) ** 2]) - 1, persistent=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        n = x.shape[0]
        gates = torch.sigmoid(self.scalar_mlp(x[:, 0])).view(n, self.lmax, self.hidden)
        h = self.so3_linear_1(x)
        h0 = F.silu(h[:, :1])
        hl = h[:, 1:] * gates.index_select(1, self.gate_index)
        return self.so3_linear_2(torch.cat([h0, hl], dim=1)).contiguous()


class EnergyHead(nn.Module):
    """Energy MLP on the l=0 coefficients, summed per system (FAIRChem-style head)."""

    def __init__(self, channels: int, hidden: int):
        super().__init__()
        self.energy_block = nn.Sequential(
            nn.Linear(channels, hidden), nn.SiLU(),
            nn.Linear(hidden, hidden), nn.SiLU(),
            nn.Linear(hidden, 1),
        )

    def forward(self, node_embedding: torch.Tensor, batch: torch.Tensor, num_systems: int) -> torch.Tensor:
        e_atom = self.energy_block(node_embedding[:, 0]).squeeze(-1)
        # per-system sum as a one-hot contraction: fixed reduction order (index_add on a
        # GPU uses atomics and is not run-to-run reproducible)
        onehot = F.one_hot(batch, num_systems).to(e_atom.dtype)
        return onehot.t() @ e_atom


def balance_channels_batched(emb, target, natoms, batch, start_idx, end_idx, target_offset=0.0,
                             partitioned: bool = False, group=None):
    """Shift channels [start_idx, end_idx) of l=0 so that their per-system sum
    equals ``target + target_offset`` (stand-in for FAIRChem's charge/spin
    channel balancing called at ``model.py:213-216``). ``partitioned``: ``emb`` holds this
    rank's atoms of systems spread over the ranks of ``group``; the per-system sums are
    all-reduced across them (differentiably) before the correction.

    The per-system sums and the broadcast back to the atoms are one-hot contractions rather
    than index_add / index_select, whose GPU implementations (and their backward) add with
    atomics: forces stay bitwise reproducible run to run."""
    chans = emb[:, 0, start_idx:end_idx]
    nsys = natoms.shape[0]
    onehot = torch.nn.functional.one_hot(batch, nsys).to(emb.dtype)          # [N, nsys]
    sums = onehot.t() @ chans
    if partitioned:
        import torch.distributed as dist
        import torch.distributed.nn.functional as dfn
        sums = dfn.all_reduce(sums, op=dist.ReduceOp.SUM, group=group if group is not None else dist.group.WORLD)
    tgt = (target.to(emb.dtype) + target_offset)[:, None]
    corr = onehot @ ((tgt - sums) / natoms.to(emb.dtype)[:, None])
    out = emb.clone()
    out[:, 0, start_idx:end_idx] = chans + corr
    return out
