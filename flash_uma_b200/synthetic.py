"""Random-init UMA-s-shaped backbone with FAIRChem's ``eSCNMDBackbone`` attribute layout.

``ZeroAllocBackbone(off_bb)`` reads a FAIRChem backbone object by attribute
(``wrapper.py:22-85``, ``:102-146``). Without ``fairchem-core`` or a checkpoint
this module builds an object with exactly those attributes so the drop-in API can
be exercised: ``sphere_embedding``, ``source_embedding``, ``target_embedding``,
``edge_degree_embedding.rad_func.net[0,1,3,4,6]``, ``blocks[k].edge_wise.
so2_conv_{1,2}.{rad_func.net, fc_m0, so2_m_conv[0,1].fc}``, ``blocks[k].norm_1 /
norm_2 / atom_wise``, ``norm``, charge/spin channel ranges, ``charge_embedding``,
``spin_embedding``, ``mix_csd``, ``regress_config``, ``lmax``, ``mmax``, ...

Weights: every Linear weight ~ N(0, 1/fan_in); embeddings ~ N(0, 1); biases,
LayerNorm affine and norm scales get small random perturbations so that every
term of the kernels is exercised. All draws come from one CPU ``torch.Generator``
seeded with ``seed`` (deterministic across machines for a given torch version).
"""
from __future__ import annotations

from types import SimpleNamespace

import torch
import torch.nn as nn

from .nodewise import EnergyHead, EquivariantRMSNormSH, SpectralAtomwise


class _Embed(nn.Module):
    """Embedding indexed by an integer quantity shifted by ``offset`` (charge can be negative)."""

    def __init__(self, num: int, dim: int, offset: int):
        super().__init__()
        self.offset = offset
        self.weight = nn.Parameter(torch.empty(num, dim))

    def forward(self, v: torch.Tensor) -> torch.Tensor:
        return self.weight[(v.long() + self.offset).clamp(0, self.weight.shape[0] - 1)]


def _radial_net(in_dim: int, hidden: int, out_dim: int) -> nn.Sequential:
    # indices 0, 1, 3, 4, 6 are the ones the weight transfer reads (wrapper.py:33-40)
    return nn.Sequential(
        nn.Linear(in_dim, hidden), nn.LayerNorm(hidden), nn.SiLU(),
        nn.Linear(hidden, hidden), nn.LayerNorm(hidden), nn.SiLU(),
        nn.Linear(hidden, out_dim),
    )


class _SO2Conv(nn.Module):
    def __init__(self, rad: nn.Module | None, m0_in: int, m0_out: int, m1_in: int, m1_out: int, m2_in: int, m2_out: int):
        super().__init__()
        if rad is not None:
            self.rad_func = SimpleNamespace(net=rad)
            self._rad = rad  # registered so .to()/parameters() see it
        self.fc_m0 = nn.Linear(m0_in, m0_out, bias=True)
        self.so2_m_conv = nn.ModuleList([
            nn.Module(), nn.Module(),
        ])
        self.so2_m_conv[0].fc = nn.Linear(m1_in, m1_out, bias=False)
        self.so2_m_conv[1].fc = nn.Linear(m2_in, m2_out, bias=False)


class _EdgeWise(nn.Module):
    def __init__(self, C: int, H: int, B: int):
        super().__init__()
        # conv1: m0 [6C -> 5C] + bias; m1 weight [4C, 4C] = [R; I] halves of [2C, 4C];
        # m2 weight [2C, 2C] = [R; I] halves of [C, 2C]  (wrapper.py:58-63, model.py:87-89)
        self.so2_conv_1 = _SO2Conv(_radial_net(B + 2 * C, H, 12 * C), 6 * C, 5 * C, 4 * C, 4 * C, 2 * C, 2 * C)
        # conv2: m0 [3C -> 3C] + bias; m1 [4C, 2C]; m2 [2C, C]  (wrapper.py:66-71, model.py:91-93)
        self.so2_conv_2 = _SO2Conv(None, 3 * C, 3 * C, 2 * C, 4 * C, C, 2 * C)


class _Block(nn.Module):
    def __init__(self, C: int, H: int, B: int):
        super().__init__()
        self.norm_1 = EquivariantRMSNormSH(C)
        self.edge_wise = _EdgeWise(C, H, B)
        self.norm_2 = EquivariantRMSNormSH(C)
        self.atom_wise = SpectralAtomwise(C, H)


class SyntheticESCNMDBackbone(nn.Module):
    """UMA-s-shaped (lmax=mmax=2) random-init backbone object."""

    def __init__(self, num_layers: int = 4, sphere_channels: int = 128, hidden_channels: int = 128,
                 num_distance_basis: int = 64, cutoff: float = 6.0, max_num_elements: int = 100,
                 seed: int = 0, forces: bool = True, stress: bool = False):
        super().__init__()
        C, H, B = sphere_channels, hidden_channels, num_distance_basis
        self.lmax = 2
        self.mmax = 2
        self.num_layers = num_layers
        self.sphere_channels = C
        self.edge_channels = H
        self.hidden_channels = H
        self.num_distance_basis = B
        self.cutoff = float(cutoff)
        self.sphere_embedding = nn.Embedding(max_num_elements, C)
        self.source_embedding = nn.Embedding(max_num_elements, C)
        self.target_embedding = nn.Embedding(max_num_elements, C)
        ede = nn.Module()
        ede.rad_func = SimpleNamespace(net=_radial_net(B + 2 * C, H, 3 * C))
        ede._rad = ede.rad_func.net
        self.edge_degree_embedding = ede
        self.blocks = nn.ModuleList([_Block(C, H, B) for _ in range(num_layers)])
        self.norm = EquivariantRMSNormSH(C)
        self.charge_embedding = _Embed(201, C, 100)
        self.spin_embedding = _Embed(101, C, 0)
        self.dataset_embedding = None
        self.use_dataset_embedding = False
        self.mix_csd = nn.Linear(2 * C, C)
        self.charge_channel_start = 0
        self.charge_channel_end = 0
        self.spin_channel_start = 0
        self.spin_channel_end = 0
        self.regress_config = SimpleNamespace(forces=forces, stress=stress, direct_forces=False, direct_stress=False)
        self.reset_parameters(seed)

    @torch.no_grad()
    def reset_parameters(self, seed: int = 0) -> None:
        g = torch.Generator().manual_seed(seed)

        def normal(t, std, mean=0.0):
            t.copy_(torch.randn(t.shape, generator=g, dtype=torch.float32) * std + mean)

        for name, mod in self.named_modules():
            if isinstance(mod, nn.Linear):
                normal(mod.weight, mod.in_features ** -0.5)
                if mod.bias is not None:
                    normal(mod.bias, 0.05)
            elif isinstance(mod, nn.LayerNorm):
                normal(mod.weight, 0.1, 1.0)
                normal(mod.bias, 0.1)
            elif isinstance(mod, (nn.Embedding, _Embed)):
                normal(mod.weight, 1.0)
            elif isinstance(mod, EquivariantRMSNormSH):
                normal(mod.affine_weight, 0.1, 1.0)
                normal(mod.affine_bias, 0.1)
            elif type(mod).__name__ == "SO3Linear":
                normal(mod.weight, mod.weight.shape[-1] ** -0.5)
                normal(mod.bias, 0.05)

    def extra_repr(self) -> str:
        return (f"lmax={self.lmax}, C={self.sphere_channels}, H={self.hidden_channels}, B={self.num_distance_basis}, "
                f"layers={self.num_layers}, cutoff={self.cutoff}")


def make_energy_head(channels: int = 128, hidden: int = 128, seed: int = 1) -> EnergyHead:
    head = EnergyHead(channels, hidden)
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for mod in head.modules():
            if isinstance(mod, nn.Linear):
                mod.weight.copy_(torch.randn(mod.weight.shape, generator=g) * mod.in_features ** -0.5)
                mod.bias.copy_(torch.randn(mod.bias.shape, generator=g) * 0.05)
    return head
