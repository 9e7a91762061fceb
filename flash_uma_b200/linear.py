"""Frozen linear maps on the tcgen05 GEMMs of the C ABI (``fuma_linear_f16x3``, ``fuma_linear``).

Replaces the reference's ``F.linear`` calls on packed frozen weights (``model.py:147-154``):
``y = x @ W^T + b`` in the forward and ``dx = dy @ W`` in the backward (weights and biases
are frozen, so no weight gradients). Precision modes:

* ``"f16x3"`` (default): fp16 tensor cores, both operands split as hi + lo * 2^-11 with
  three products per K step - fp32-level accuracy at half the operand bytes of TF32. Inputs
  must stay inside the fp16 range (|x| < 65520); a GEMM that meets a larger value records
  it in the device error flag and the next :func:`poll_errors` / :func:`check_errors` raises.
* ``"tf32x3"``: three TF32 products on hi/lo TF32 splits - fp32-level accuracy, full fp32
  range.
* ``"tf32"``: a single TF32 product (what the reference runs with ``allow_tf32``).
* ``"f16"``: a single fp16 product A_hi . W_hi on the same split operands (``fuma_linear_f16``):
  the accuracy class of TF32 (about 11 significant bits per operand) at a third of the f16x3
  tensor work; the fast mode to set beside the reference's published TF32 setting.

The weight splits (and the transposed weights for the backward) are built once, on the
device, when the module is first used on a device.
"""
from __future__ import annotations

import math
import os

import torch
import torch.nn as nn

from . import _native as nat
from ._native import ptr, stream_of

_MODES = ("f16x3", "tf32x3", "tf32", "f16")
_F16_MODES = ("f16x3", "f16")   # fp16 tensor cores on the row-packed split operands
_err_flags: dict[int, torch.Tensor] = {}
_err_host: dict[int, torch.Tensor] = {}     # pinned mirrors, filled asynchronously by snapshot_errors()

_ERR_RANGE = 16
_ERR_INDEX = 32   # fuma_morton_reorder: an edge index outside [0, N)


def default_mode() -> str:
    m = os.environ.get("FUMA_GEMM", "f16x3")
    if m not in _MODES:
        raise ValueError(f"FUMA_GEMM must be one of {_MODES}, got {m!r}")
    return m


def error_flag(device: torch.device) -> torch.Tensor:
    """Per-device int32 flag (the first error recorded is kept): a GEMM pipeline wait timed out
    (codes 1-5), an f16x3 input is out of the fp16 range (code 16), or the Morton reorder met an
    edge index outside [0, N) (code 32)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _err_flags.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _err_flags[idx] = t
    return t


def _raise(idx: int, code: int):
    if code == _ERR_INDEX:
        raise RuntimeError(f"fuma_morton_reorder: an edge index on cuda:{idx} is outside [0, num_atoms); the edge "
                           "was renumbered to atom 0 and the results are invalid")
    if code == _ERR_RANGE:
        raise RuntimeError(f"fuma_linear_f16x3: an input value on cuda:{idx} is beyond the fp16 range of the f16x3 "
                           "split (|x| >= 65520); construct the model with gemm='tf32x3' for such data")
    raise RuntimeError(f"fuma_linear: a tensor-core pipeline wait timed out (code {code}) on cuda:{idx}")


def _reset(idx: int):
    _err_flags[idx].zero_()
    if idx in _err_host:
        _err_host[idx].zero_()


def check_errors(device: torch.device | None = None) -> None:
    """Raise if any GEMM on ``device`` (default: all used devices) reported an error (synchronises)."""
    for idx, t in _err_flags.items():
        if device is not None and device.index not in (None, idx):
            continue
        code = int(t.item())
        if code:
            _reset(idx)
            _raise(idx, code)


def snapshot_errors() -> None:
    """Queue an asynchronous copy of every device's error flag into pinned host memory (no sync)."""
    for idx, t in _err_flags.items():
        h = _err_host.get(idx)
        if h is None:
            h = torch.zeros(1, dtype=torch.int32, pin_memory=True)
            _err_host[idx] = h
        h.copy_(t, non_blocking=True)


def step_status(device: torch.device) -> torch.Tensor:
    """A device-side copy of ``device``'s GEMM error flag, taken on the current stream after
    everything queued so far (no synchronisation): the status of the step that was just queued,
    0 when every GEMM of it (and of earlier unreported steps) succeeded. Callers that copy a
    step's results to the host copy this 4-byte tensor with them and pass it to
    :func:`raise_status`."""
    return error_flag(device).clone()


def raise_status(status: torch.Tensor, device: torch.device | None = None) -> None:
    """Raise (and clear the device flag) if a :func:`step_status` value holds an error code.
    Reads the value: a device tensor synchronises, a host copy does not (``device``: the GPU
    the host copy came from, default the current one)."""
    code = int(status.reshape(-1)[0])
    if code:
        if device is not None and device.index is not None:
            idx = device.index
        else:
            idx = status.device.index if status.is_cuda else torch.cuda.current_device()
        if idx in _err_flags:
            _reset(idx)
        _raise(idx, code)


def poll_errors() -> None:
    """Raise if an earlier :func:`snapshot_errors` copy has landed with an error code (no sync:
    an error is seen at the first poll after its snapshot completed)."""
    for idx, h in _err_host.items():
        code = int(h[0])
        if code:
            _reset(idx)
            _raise(idx, code)


def _split(w: torch.Tensor):
    w = w.contiguous()
    hi, lo = torch.empty_like(w), torch.empty_like(w)
    nat.call("fuma_split_tf32", ptr(w), w.numel(), ptr(hi), ptr(lo), stream_of(w))
    return hi, lo


def _split16(w: torch.Tensor, x1: bool = False):
    """fp16 hi/lo split of ``w * scale`` (scale a power of two keeping |w * scale| < 2^14):
    (hi, lo, 1 / scale, x1); ``x1``: products use the hi halves only (the "f16" mode)."""
    w = w.contiguous()
    amax = float(w.abs().max()) if w.numel() else 0.0
    e = max(0, math.ceil(math.log2(amax)) - 14) if amax > 0 else 0
    scale = 2.0 ** -e
    hi = torch.empty(w.shape, device=w.device, dtype=torch.float16)
    lo = torch.empty_like(hi)
    nat.call("fuma_split_f16", ptr(w), w.numel(), scale, ptr(hi), ptr(lo), stream_of(w))
    return hi, lo, 1.0 / scale, x1


def _as_operand(a: torch.Tensor) -> torch.Tensor:
    if a.stride(1) != 1 or a.stride(0) % 4 != 0 or a.data_ptr() % 16 != 0:
        a = a.contiguous()
    return a


def _gemm(a: torch.Tensor, w_hi: torch.Tensor, w_lo: torch.Tensor | None, bias: torch.Tensor | None, split: bool):
    M, K = a.shape
    N = w_hi.shape[0]
    a = _as_operand(a)
    out = torch.empty(M, N, device=a.device, dtype=torch.float32)
    nat.call("fuma_linear", ptr(a), a.stride(0), ptr(w_hi), ptr(w_lo) if split else None, ptr(bias), M, N, K,
             1 if split else 0, ptr(out), N, ptr(error_flag(a.device)), stream_of(a))
    return out


def split_rows(x: torch.Tensor, ldp: int | None = None) -> torch.Tensor:
    """Row-packed f16x3 split of x [M, K] (``fuma_split_rows_f16``): an fp32-typed [M, ldp]
    tensor whose row r holds the fp16 hi values of x[r] in its first 2*ldp bytes and the scaled
    fp16 lo values in the next 2*ldp bytes. Row slices and row concatenations stay valid."""
    M, K = x.shape
    ldp = ldp or (K + 7) // 8 * 8
    x = _as_operand(x)
    out = torch.empty(M, ldp, device=x.device, dtype=torch.float32)
    nat.call("fuma_split_rows_f16", ptr(x), x.stride(0), M, K, ptr(out), ldp, ptr(error_flag(x.device)),
             stream_of(x))
    return out


def _gemm16(a: torch.Tensor, w16, bias: torch.Tensor | None, K: int | None = None, out_half: bool = False):
    """fp16 tensor-core product with a weight split ``w16 = (hi, lo, scale_inv, x1)`` of W [N, ldw]:
    three products (f16x3) or, with ``x1``, the single hi . hi product. ``K`` given: ``a`` is a
    row-packed split (:func:`split_rows`) of a [M, K] activation. ``out_half`` (single product
    only): the result is stored as fp16 (the 16-bit activation storage of the "f16" mode)."""
    hi, lo, inv, x1 = w16
    N, ldw = hi.shape
    if K is None:
        M, K = a.shape
        if x1:
            a = split_rows(a)
            pre = 1
        else:
            a = _as_operand(a)
            pre = 0
    else:
        M = a.shape[0]
        pre = 1
    half = bool(out_half and x1)
    out = torch.empty(M, N, device=a.device, dtype=torch.float16 if half else torch.float32)
    if x1:
        nat.call("fuma_linear_f16", ptr(a), a.stride(0), ptr(hi), ldw, inv, ptr(bias), M, N, K, ptr(out), N,
                 1 if half else 0, ptr(error_flag(a.device)), stream_of(a))
    else:
        nat.call("fuma_linear_f16x3", ptr(a), a.stride(0), pre, ptr(hi), ptr(lo), ldw, inv, ptr(bias), M, N, K,
                 ptr(out), N, ptr(error_flag(a.device)), stream_of(a))
    return out


def _ceil16(n: int) -> int:
    return (n + 15) // 16 * 16


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, mod):
        ctx.mod = mod
        if mod.mode in _F16_MODES:
            y = _gemm16(x, mod.w16, mod.bias_p)
        else:
            y = _gemm(x, mod.w_hi, mod.w_lo, mod.bias_p, mod.mode == "tf32x3")
        return y if mod.Np == mod.N else y[:, : mod.N]

    @staticmethod
    def backward(ctx, g):
        mod = ctx.mod
        g = g.contiguous()
        if mod.Np != mod.N:
            g = torch.nn.functional.pad(g, (0, mod.Np - mod.N))
        if mod.mode in _F16_MODES:
            gx = _gemm16(g, mod.wt16, None)
        else:
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
        self.w16 = self.wt16 = None   # (hi, lo, scale_inv) fp16 splits of W and W^T (f16x3)
        self._prepared_on = None

    def prepare(self) -> None:
        """Build the padded splits of W and W^T for this mode on W's device (idempotent)."""
        if self._prepared_on == self.weight.device:
            return
        if not self.weight.is_cuda:
            raise RuntimeError("FrozenLinear runs on CUDA only; move the module to a GPU first")
        dev = self.weight.device
        if self.mode in _F16_MODES:
            wf = torch.zeros(self.Np, (self.K + 7) // 8 * 8, device=dev)   # rows 16-byte aligned in fp16
            wf[: self.N, : self.K] = self.weight
            wt = torch.zeros(self.Kp, self.Np, device=dev)
            wt[: self.K, : self.N] = self.weight.t()
            x1 = self.mode == "f16"
            self.w16, self.wt16 = _split16(wf, x1), _split16(wt, x1)
        else:
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
