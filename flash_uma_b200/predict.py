"""Energy / forces / stress above the backbone (stand-in for FAIRChem's MLP_EFS heads).

The reference leaves this layer to FAIRChem (``readme.md:35-72``): the heads run an
energy MLP on the backbone's l=0 output, sum per system, and take conservative
forces and the virial stress from autograd on ``pos`` and on a symmetric strain
applied to ``pos`` and ``cell``. Works with any backbone callable (the CUDA
``ZeroAllocBackbone`` or the CPU oracle), which is how parity tests compare them.
"""
from __future__ import annotations

import dataclasses

import torch


class Predictor:
    def __init__(self, backbone, head):
        self.backbone = backbone
        self.head = head

    def __call__(self, data, forces: bool = True, stress: bool = False):
        nsys = len(data.natoms)
        pos = data.pos.detach().clone().requires_grad_(forces or stress)
        cell = data.cell.detach().clone()
        wrt = []
        if forces or stress:
            wrt.append(pos)
        p, c = pos, cell
        if stress:
            disp = torch.zeros(nsys, 3, 3, dtype=pos.dtype, device=pos.device, requires_grad=True)
            sym = 0.5 * (disp + disp.transpose(1, 2))
            p = pos + torch.einsum("ni,nij->nj", pos, sym[data.batch])
            c = cell + torch.bmm(cell, sym)
            wrt.append(disp)
        fields = {f.name: getattr(data, f.name) for f in dataclasses.fields(data)}
        fields.update(pos=p, cell=c)
        d2 = type(data)(**fields)
        out = self.backbone(d2)
        emb = out["node_embedding"]
        head_dtype = next(self.head.parameters()).dtype
        energy = self.head(emb.to(head_dtype), data.batch, nsys)
        res = {"energy": energy.detach(), "node_embedding": emb.detach()}
        if wrt:
            grads = torch.autograd.grad(energy.sum(), wrt)
            res["forces"] = -grads[0]
            if stress:
                vol = torch.linalg.det(cell).abs()
                res["stress"] = grads[1] / vol[:, None, None]
        return res
