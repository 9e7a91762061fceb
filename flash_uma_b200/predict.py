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

from . import linear


class Predictor:
    def __init__(self, backbone, head):
        self.backbone = backbone
        self.head = head

    def __call__(self, data, forces: bool = True, stress: bool = False, check: bool = False):
        """Energy [nsys] (+ forces [N, 3], stress [nsys, 3, 3]) of ``data``. On a GPU the result
        also holds ``status``: a 1-element device int32 tensor, 0 unless a GEMM of this step (or
        of an earlier step not yet reported) failed (f16x3 range error 16, pipeline timeout
        1-5). Copy it to the host with the results and pass it to ``linear.raise_status``, or
        call with ``check=True`` to synchronise and raise here, before the results are used."""
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
        if pos.is_cuda:
            res["status"] = linear.step_status(pos.device)
            if check:
                linear.raise_status(res["status"])
        return res


class GraphedStep:
    """``predictor(data)`` on one fixed graph (atoms, edges, cell; new positions every call),
    captured once as a CUDA graph: a call copies the positions into the captured input and
    replays every kernel of the forward and backward pass with one launch, so the host does
    no per-kernel work. The graph build, Morton order and CSRs are part of the capture and are
    recomputed from the positions on every replay, exactly as in an eager call. Returns the
    captured output tensors (overwritten by the next call), including ``status``, the GEMM
    error status of this replay (see :class:`Predictor`): ``check=True`` synchronises and raises
    on an error before returning; otherwise errors also surface at the next call's poll."""

    def __init__(self, predictor, data, forces: bool = True, stress: bool = False, warmup: int = 3,
                 capture_hook=None):
        self._pos = data.pos.detach().clone()
        self._data = dataclasses.replace(data, pos=self._pos)
        dev = self._pos.device
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):   # warm-up on a side stream (caches, weight splits, allocator)
            for _ in range(warmup):
                predictor(self._data, forces=forces, stress=stress)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            if capture_hook is not None:
                capture_hook(True)
            try:
                self.out = predictor(self._data, forces=forces, stress=stress)
            finally:
                if capture_hook is not None:
                    capture_hook(False)

    def __call__(self, pos: torch.Tensor, check: bool = False):
        linear.poll_errors()
        self._pos.copy_(pos, non_blocking=True)
        self.graph.replay()
        if check:
            linear.raise_status(self.out["status"])
        return self.out
