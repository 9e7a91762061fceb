"""ctypes binding of the C ABI in ``include/flash_uma_b200.h``.

There is no CPU fallback: if the library has not been built, or there is no CUDA
device, the first call raises. Tensors are passed as raw device pointers; the
stream is PyTorch's current stream on the tensors' device.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

from . import build as _build

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_F32 = ctypes.c_float

# name -> argument types (return type is int for all compute entry points)
_SIGS = {
    "fuma_geometry_fwd": [_P, _P, _P, _P, _P, _P, _P, _P, _F32, _F32, _I64, _I64, _I32, _I32, _P, _P, _P, _P],
    "fuma_geometry_bwd": [_P, _P, _P, _P, _P, _F32, _F32, _P, _I64, _P, _P, _I64, _I32, _P, _P],
    "fuma_edge_vec_to_nodes": [_P, _P, _P, _P, _P, _I64, _I64, _P, _P],
    "fuma_ln_silu_fwd": [_P, _P, _P, _F32, _I64, _I32, _P, _P, _P, _P],
    "fuma_ln_silu_bwd": [_P, _P, _P, _P, _P, _P, _I64, _I32, _P, _P],
    "fuma_gather_fwd": [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I32, _P, _P, _P, _P],
    "fuma_gather_bwd": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I32, _P, _I64, _P, _P, _P, _P],
    "fuma_gating_fwd": [_P, _P, _P, _I64, _I32, _P, _P, _P, _P],
    "fuma_gating_bwd": [_P, _P, _P, _P, _P, _P, _I64, _I32, _P, _P, _P, _P],
    "fuma_rotate_scatter_fwd": [_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I32, _P, _P],
    "fuma_rotate_scatter_bwd": [_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I32, _P, _P, _P, _P, _P, _P],
    "fuma_init_scatter_fwd": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I32, _P, _P],
    "fuma_init_scatter_bwd": [_P, _P, _P, _P, _P, _P, _I64, _I64, _I32, _P, _P, _P, _P],
    "fuma_linear": [_P, _I64, _P, _P, _P, _I64, _I32, _I32, _I32, _P, _I64, _P, _P],
    "fuma_split_tf32": [_P, _I64, _P, _P, _P],
    "fuma_linear_f16x3": [_P, _I64, _I32, _P, _P, _I64, _F32, _P, _I64, _I32, _I32, _P, _I64, _P, _P],
    "fuma_linear_f16": [_P, _I64, _P, _I64, _F32, _P, _I64, _I32, _I32, _P, _I64, _I32, _P, _P],
    "fuma_split_rows_f16": [_P, _I64, _I64, _I32, _P, _I64, _P, _P],
    "fuma_split_f16": [_P, _I64, _F32, _P, _P, _P],
    "fuma_neighbor_list": [_P, _I64, _P, _P, ctypes.c_double, _I32, _P, _I64, _P, _P, _P, _P, _P, _P],
    "fuma_csr_permute": [_P, _P, _P, _P, _P, _I64, _I64, _P, _P, _P, _P, _P],
    "fuma_morton_reorder": [_P, _P, _P, _P, _P, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _P, _P],
    "fuma_atomwise_gate_fwd": [_P, _P, _P, _I64, _I32, _P, _P],
    "fuma_atomwise_gate_bwd": [_P, _P, _P, _P, _I64, _I32, _P, _P, _P],
    "fuma_coef_to_node": [_P, _P, _P, _I32, _I64, _I32, _P, _P],
    "fuma_node_to_coef_f16x3": [_P, _I64, _I32, _P, _I32, _P, _P],
    "fuma_atomwise_gate_fwd_f16x3": [_P, _P, _P, _I64, _I32, _P, _I32, _P, _P],
    "fuma_atomwise_gate_bwd_f16x3": [_P, _P, _P, _P, _I64, _I32, _P, _P, _I32, _P, _P],
    "fuma_coef_to_node_blocked": [_P, _P, _P, _I32, _I64, _I32, _P, _P],
    "fuma_rmsnorm_sh_fwd": [_P, _P, _P, _P, _F32, _I64, _I32, _P, _P, _P],
    "fuma_rmsnorm_sh_bwd": [_P, _P, _P, _P, _P, _I64, _I32, _P, _P],
    "fuma_morton_reorder_noalloc": [_P, _P, _P, _P, _P, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P],
}

_lib = None
_lock = threading.Lock()


def lib_path() -> str:
    return _build.lib_path()


def load(allow_build: bool = False) -> ctypes.CDLL:
    """Load the shared library (building it first if ``allow_build`` and it is missing/stale)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if allow_build and _build.needs_build():
            _build.build()
        if not os.path.exists(path):
            raise RuntimeError(f"flash_uma_b200: CUDA library not built ({path}); run `python -m flash_uma_b200.build`")
        lib = ctypes.CDLL(path)
        for name, args in _SIGS.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        lib.fuma_version.restype = ctypes.c_int
        lib.fuma_morton_scratch_bytes.argtypes = [_I64]
        lib.fuma_morton_scratch_bytes.restype = ctypes.c_int64
        lib.fuma_neighbor_scratch_bytes.argtypes = [_I64, _P]
        lib.fuma_neighbor_scratch_bytes.restype = ctypes.c_int64
        lib.fuma_last_error.restype = ctypes.c_char_p
        _lib = lib
        return lib


def exported_symbols():
    return ["fuma_version", "fuma_last_error", "fuma_morton_scratch_bytes", "fuma_neighbor_scratch_bytes",
            *_SIGS.keys()]


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


# kernels each entry point launches (used by launch accounting)
# variants writing the GEMM-input outputs in the row-packed f16x3 split layout: same arguments
# plus the number of halves written (2: hi and lo, 1: hi only) and an error flag before the stream
for _name in ("fuma_ln_silu_fwd", "fuma_ln_silu_bwd", "fuma_gather_fwd", "fuma_gather_bwd", "fuma_gating_fwd",
              "fuma_gating_bwd", "fuma_rotate_scatter_bwd", "fuma_init_scatter_bwd"):
    _SIGS[_name + "_f16x3"] = _SIGS[_name][:-1] + [_I32, _P, _P]   # ..., parts, err_flag, stream
for _name in ("fuma_gather_fwd", "fuma_gather_bwd", "fuma_gating_fwd", "fuma_gating_bwd", "fuma_rotate_scatter_bwd"):
    # ..., parts, act_half (fp16 radial / conv results), err_flag, stream
    _SIGS[_name + "_f16x3"] = _SIGS[_name][:-1] + [_I32, _I32, _P, _P]
_SIGS["fuma_rotate_scatter_fwd_f16x3"] = _SIGS["fuma_rotate_scatter_fwd"][:-1] + [_I32, _P]

KERNELS_PER_CALL = {name: 1 for name in _SIGS}
KERNELS_PER_CALL["fuma_gather_bwd"] = 3
KERNELS_PER_CALL["fuma_gather_fwd"] = 2
KERNELS_PER_CALL["fuma_csr_permute"] = 2
KERNELS_PER_CALL["fuma_neighbor_list"] = 4
KERNELS_PER_CALL["fuma_morton_reorder"] = 2   # up to 16,384 atoms (launches_of)
KERNELS_PER_CALL["fuma_morton_reorder_noalloc"] = 2
KERNELS_PER_CALL["fuma_gather_fwd_f16x3"] = 2
KERNELS_PER_CALL["fuma_rotate_scatter_fwd"] = 2
KERNELS_PER_CALL["fuma_rotate_scatter_bwd"] = 2
KERNELS_PER_CALL["fuma_gather_bwd_f16x3"] = 3
KERNELS_PER_CALL["fuma_rotate_scatter_bwd_f16x3"] = 2
KERNELS_PER_CALL["fuma_rotate_scatter_fwd_f16x3"] = 2


def launches_of(name: str, args) -> int:
    """Kernel launches of one call of entry point ``name`` with arguments ``args``."""
    if name in ("fuma_morton_reorder", "fuma_morton_reorder_noalloc") and args[5] > 16384:
        return 28   # bounds, keys, 8 radix passes of 3 kernels, permutation, renumbering
    return KERNELS_PER_CALL.get(name, 1)


class LaunchProbe:
    """Optional per-call instrumentation: counts kernel launches per entry point and, for the
    names in ``timed``, brackets each call with CUDA events on the current stream so the
    kernel's device time can be measured inside a larger timed region."""

    def __init__(self, timed=(), pool: int = 0, external: bool = False):
        """``external``: events that record as nodes when the calls are captured in a CUDA graph
        (their elapsed times then read the last replay)."""
        self.external = external
        self.timed = set(timed)
        self.counts: dict[str, int] = {}
        self.launches = 0
        self.events: dict[str, list] = {}
        self.meta: dict[str, list] = {}
        self.timing = True          # bracket calls of ``timed`` entry points with events
        # pre-created events keep the per-call host cost to two cudaEventRecord calls
        self._pool = [self._new_event() for _ in range(pool)]

    def _new_event(self):
        if self.external:
            return torch.cuda.Event(enable_timing=True, external=True)
        return torch.cuda.Event(enable_timing=True)

    def _event(self):
        return self._pool.pop() if self._pool else self._new_event()

    def before(self, name, args):
        self.counts[name] = self.counts.get(name, 0) + 1
        self.launches += launches_of(name, args)
        if self.timing and name in self.timed:
            ev0 = self._event()
            ev0.record()
            return ev0
        return None

    def after(self, name, ev0, args):
        if ev0 is None:
            return
        ev1 = self._event()
        ev1.record()
        self.events.setdefault(name, []).append((ev0, ev1))

    def times_ms(self, name):
        return [a.elapsed_time(b) for a, b in self.events.get(name, [])]


_probe: LaunchProbe | None = None


def set_probe(p: LaunchProbe | None) -> None:
    global _probe
    _probe = p


def call(name: str, *args) -> None:
    lib = load()
    p = _probe
    ev = p.before(name, args) if p is not None else None
    rc = getattr(lib, name)(*args)
    if p is not None:
        p.after(name, ev, args)
    if rc != 0:
        msg = lib.fuma_last_error().decode(errors="replace")
        raise RuntimeError(f"{name} failed (code {rc}): {msg}")


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("flash_uma_b200 ops run on CUDA tensors only (no CPU fallback); "
                               f"got a tensor on {t.device}")
