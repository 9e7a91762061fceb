"""Frozen linear maps on the tcgen05 GEMM of the C ABI (``fuma_linear``).

Replaces the reference's ``F.linear`` calls on packed frozen weights (``model.py:147-154``):
``y = x @ W^T + b`` in the forward and ``dx = dy @ W`` in the backward (weights and biases
are frozen, so no weight gradients). Precision modes:

* ``"tf32x3"`` (default): three TF32 tensor-core products per K step on hi/lo splits of
  both operands - fp32-level accuracy (the parity mode).
* ``"tf32"``: a single TF32 product (what the reference runs with ``allow_tf32``).

The weight splits (and the transposed weights for the backward) are built once, on the
device, when the module is created or moved.
"""
from __future__ import annotations

import os

import torch
import torch.nn as nn

from . import _native as nat
from ._native import ptr, stream_of

_MODES = ("tf32x3", "tf32")
_err_flags: dict[int, torch.Tensor] = {}


def default_mode() -> str:
    m = os.environ.get("FUMA_GEMM", "tf32x3")
    if m not in _MODES:
        raise ValueError(f"FUMA_GEMM must be one of {_MODES}, got {m!r}")
    return m


def error_flag(device: torch.device) -> torch.Tensor:
    """Per-device int32 flag that the GEMM kernel sets if one of its pipeline waits times out."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _err_flags.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _err_flags[idx] = t
    return t


def check_errors(device: torch.device | None = None) -> None:
    """Raise if any GEMM on ``device`` (default: all used devices) reported a timeout (synchronises)."""
    for idx, t in _err_flags.items():
        if device is not None and device.index not in (None, idx):
            continue
        code = int(t.item())
        if code:
            t.zero_()
            raise RuntimeError(f"fuma_linear: a tensor-core pipeline wait timed out (code {code}) on cuda:{idx}")


def _split(w: torch.Tensor):
    w = w.contiguous()
    hi, lo = torch.empty_like(w), torch.empty_like(w)
    nat.call("fuma_split_tf32", ptr(w), w.numel(), ptr(hi), ptr(lo), stream_of(w))
    return hi, lo


def _gemm(a: torch.Tensor, w_hi: torch.Tensor, w_lo: torch.Tensor | None, bias: torch.Tensor | None, split: bool):
    M, K = a.shape
    N = w_hi.shape[0]
    if a.stride(1) != 1 or a.stride(0) % 4 != 0 or a.data_ptr() % 16 != 0:
        a = a.contiguous()
    out = torch.empty(M, N, device=a.device, dtype=torch.float32)
    nat.call("fuma_linear", ptr(a), a.stride(0), ptr(w_hi), ptr(w_lo) if split else None, ptr(bias), M, N, K,
             1 if split else 0, ptr(out), N, ptr(error_flag(a.device)), stream_of(a))
    return out


def _ceil16(n: int) -> int:
    return (n + 15) // 16 * 16


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, mod):
        ctx.mod = mod
        y = _gemm(x, mod.w_hi, mod.w_lo, mod.bias_p, mod.mode == "tf32x3")
        return y if mod.Np == mod.N else y[:, : mod.N]

    @staticmethod
    def backward(ctx, g):
        mod = ctx.mod
        g = g.contiguous()
        if mod.Np != mod.N:
            g = torch.nn.functional.pad(g, (0, mod.Np - mod.N))
        gx = _gemm(g, mod.wt_hi, mod.wt_lo, None, mod.mode == "tf32x3")
        return (gx if mod.Kp == mod.K else gx[:, : mod.K]), None


class FrozenLinear(nn.Module):
    """y = x W^T + b for a frozen W [N, K]; x [M, K] fp32 CUDA with K a multiple of 4.

    Output widths that are not multiples of 16 (small test models only) run on zero-padded
    weights and return a column slice."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None = None, mode: str | None = None):
        super().__init__()
        self.mode = mode or default_mode()
        if self.mode not in _MODES:
            raise ValueError(f"mode must be one of {_MODES}")
        w = weight.detach().float().contiguous()
        self.N, self.K = w.shape
        if self.K % 4:
            raise ValueError(f"FrozenLinear needs K % 4 == 0 (got K={self.K})")
        self.Np, self.Kp = _ceil16(self.N), _ceil16(self.K)
        self.register_buffer("weight", w)
        self.register_buffer("bias", None if bias is None else bias.detach().float().contiguous())
        for name in ("bias_p", "w_hi", "w_lo", "wt_hi", "wt_lo"):
            self.register_buffer(name, None, persistent=False)
        self._prepared_on = None

    def prepare(self) -> None:
        """Build the padded TF32 splits of W and W^T on W's device (idempotent)."""
        if self._prepared_on == self.weight.device:
            return
        if not self.weight.is_cuda:
            raise RuntimeError("FrozenLinear runs on CUDA only; move the module to a GPU first")
        dev = self.weight.device
        wf = torch.zeros(self.Np, self.K, device=dev)
        wf[: self.N] = self.weight
        wt = torch.zeros(self.Kp, self.Np, device=dev)
        wt[: self.K, : self.N] = self.weight.t()
        self.w_hi, self.w_lo = _split(wf)
        self.wt_hi, self.wt_lo = _split(wt)
        if self.bias is not None:
            bp = torch.zeros(self.Np, device=dev)
            bp[: self.N] = self.bias
            self.bias_p = bp
        self._prepared_on = dev

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        nat.require_cuda(x)
        if x.dtype != torch.float32:
            raise TypeError(f"FrozenLinear input must be float32 (got {x.dtype})")
        self.prepare()
        return _LinearFn.apply(x, self)

    def extra_repr(self) -> str:
        return f"N={self.N}, K={self.K}, bias={self.bias is not None}, mode={self.mode}"
