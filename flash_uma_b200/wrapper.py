"""``ZeroAllocBackbone``: drop-in replacement for FAIRChem's ``eSCNMDBackbone``.

Same constructor, attributes and methods as the reference (``wrapper.py:88-211``):
``ZeroAllocBackbone(off_bb, dtype=torch.float32)`` copies the weights out of a
FAIRChem backbone (``transfer_weights``, ``wrapper.py:22-85``), keeps the charge /
spin / dataset embeddings and ``mix_csd``, and its ``forward(data)`` returns
``{"node_embedding": [N, 9, C] (input atom order), "batch": [N]}``. Forces and stress
come from autograd on ``data.pos`` / ``data.cell`` through the CUDA backward kernels.

Only lmax = mmax = 2 and fp32 are supported; other values raise ``ValueError`` at
construction (``wrapper.py:105-118``). Inference only: the transferred weights are
frozen buffers.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import linear
from .model import ESCNInferenceModel


def validate_atoms_data(self, atoms, task_name):
    """Default charge / spin in ``atoms.info`` (``wrapper.py:7-12``)."""
    if "charge" not in atoms.info:
        atoms.info["charge"] = 0
    if "spin" not in atoms.info:
        atoms.info["spin"] = 1 if task_name == "omol" else 0


class ZeroAllocBackbone(nn.Module):
    def __init__(self, off_bb, dtype=torch.float32, gemm: str | None = None):
        """``gemm``: "f16x3" (default; fp16 tensor cores with fp32-level accuracy, inputs of the
        dense layers inside the fp16 range), "tf32x3" (fp32-level accuracy, full fp32 range),
        "tf32" (single pass, as the reference runs with TF32 enabled) or "f16" (single fp16
        product, the same accuracy class as TF32, the fastest mode); default from the FUMA_GEMM
        environment variable."""
        super().__init__()
        lmax = getattr(off_bb, "lmax", None)
        if lmax is not None and lmax != 2:
            raise ValueError(f"ZeroAllocBackbone only supports lmax=2 (the kernels are written for the "
                             f"9-coefficient layout); got lmax={lmax}.")
        mmax = getattr(off_bb, "mmax", None)
        if mmax is not None and mmax != 2:
            raise ValueError(f"ZeroAllocBackbone only supports mmax=2; got mmax={mmax}.")
        if dtype != torch.float32:
            raise ValueError(f"ZeroAllocBackbone computes in float32 only; got dtype={dtype}.")
        if int(off_bb.sphere_channels) % 4 != 0 or int(off_bb.sphere_channels) > 512:
            raise ValueError("sphere_channels must be a multiple of 4 and <= 512")
        device = next(off_bb.parameters()).device
        self.dtype = dtype
        self.ce = ESCNInferenceModel(off_bb, gemm).to(device)
        self.charge_embedding = off_bb.charge_embedding
        self.spin_embedding = off_bb.spin_embedding
        self.dataset_embedding = getattr(off_bb, "dataset_embedding", None)
        self.mix_csd = off_bb.mix_csd
        self.use_dataset_embedding = getattr(off_bb, "use_dataset_embedding", False)
        self.regress_config = off_bb.regress_config

    def validate_atoms_data(self, atoms, task_name):
        validate_atoms_data(self, atoms, task_name)

    def on_predict_check(self, data):
        """No consistency check is needed (``wrapper.py:155-157``)."""

    def prepare_for_inference(self, data, settings):
        """The backbone needs no per-system preparation (``wrapper.py:159-161``)."""
        return self

    def csd_embedding(self, charge, spin, dataset=None):
        """System (charge / spin / dataset) embedding, ``wrapper.py:163-169``."""
        chg_emb = self.charge_embedding(charge)
        spin_emb = self.spin_embedding(spin)
        if self.use_dataset_embedding and dataset is not None:
            dataset_emb = self.dataset_embedding(dataset)
            return F.silu(self.mix_csd(torch.cat((chg_emb, spin_emb, dataset_emb), dim=1)))
        return F.silu(self.mix_csd(torch.cat((chg_emb, spin_emb), dim=1)))

    def forward(self, data):
        # errors recorded by earlier GEMMs (pipeline timeouts, f16x3 range) surface here, one
        # call late, without a synchronisation
        _poll()
        data.atomic_numbers = data.atomic_numbers.long()
        data.atomic_numbers_full = data.atomic_numbers
        data.batch_full = data.batch
        rc = self.regress_config
        if not rc.direct_forces:
            if getattr(rc, "forces", False) or getattr(rc, "stress", False):
                data.pos.requires_grad_(True)
            if getattr(rc, "stress", False):
                if data.cell is not None and data.cell.is_floating_point():
                    data.cell.requires_grad_(True)
        csd = self.csd_embedding(charge=data.charge, spin=data.spin, dataset=getattr(data, "dataset", None))
        if len(data.natoms) == 1:
            shifts = data.cell_offsets.to(data.cell.dtype) @ data.cell.squeeze(0)
        else:
            cell_per_edge = data.cell.repeat_interleave(data.nedges, dim=0)
            shifts = torch.einsum("ij,ijk->ik", data.cell_offsets.to(cell_per_edge.dtype), cell_per_edge)
        x_node = _run_model(self.ce, data.pos, data.atomic_numbers, data.batch, data.edge_index, shifts, csd.float(),
                            data.charge, data.spin, data.natoms)
        return {"node_embedding": x_node, "batch": data.batch}


@torch.compiler.disable
def _poll():
    linear.poll_errors()


@torch.compiler.disable
def _run_model(ce, pos, Z, batch, edge_index, shifts, csd, charge, spin, natoms):
    """The CUDA model (and the host-side error snapshot after it). Under ``torch.compile`` this is
    one opaque region: the compiler traces the embeddings and shifts around it (the reference's
    own ops compile through torch.library custom operators, see ``flash_uma_b200.library``);
    the model itself is captured whole with CUDA graphs (``predict.GraphedStep``) instead."""
    x_node = ce(pos=pos, Z=Z, batch=batch, edge_index=edge_index, shifts=shifts, csd_emb=csd, charge=charge,
                spin=spin, natoms=natoms)
    linear.snapshot_errors()
    return x_node
