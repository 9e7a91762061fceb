"""Load the reference implementation's own ops on CPU (fixture generation only).

Runs only where the reference source tree exists; its location comes from the
``FLASHUMA_REFERENCE`` environment variable (there is no default path). Never on
the GPU box and never from the tests themselves - the tests read the committed
``.npz`` fixtures this produces.

The reference ops are Triton kernels; with ``TRITON_INTERPRET=1`` they execute
on CPU tensors. Two patches make that possible:
(1) ``triton.autotune`` keeps only the first config of each list, because the
autotuner's benchmarker needs a GPU; (2) ``torch.cuda.synchronize`` becomes a
no-op, because the first-call warm-up paths call it (``ops/gather.py:472,500``,
``ops/geom.py:568``). ``model.py`` imports ``balance_channels_batched`` from
fairchem at module load (``model.py:11``); a stub module provides it.
"""
from __future__ import annotations

import os
import sys
import types

REFERENCE_DIR = os.environ.get("FLASHUMA_REFERENCE", "")


def available() -> bool:
    return bool(REFERENCE_DIR) and os.path.isfile(os.path.join(REFERENCE_DIR, "ops", "gather.py"))


def load():
    """Import and return the reference modules: (ops namespace, model module, wrapper module)."""
    if not available():
        raise RuntimeError("the reference source tree was not found: set FLASHUMA_REFERENCE to its path "
                           f"(got {REFERENCE_DIR!r})")
    os.environ["TRITON_INTERPRET"] = "1"
    import torch
    import triton

    if not getattr(triton, "_fuma_patched", False):
        orig = triton.autotune

        def first_config_only(configs, key, **kw):
            return orig(configs=configs[:1], key=key, **kw)

        triton.autotune = first_config_only
        triton._fuma_patched = True
        torch.cuda.synchronize = lambda *a, **k: None

    # stub for the fairchem import at model.py:11
    from flash_uma_b200.nodewise import balance_channels_batched
    for name in ["fairchem", "fairchem.core", "fairchem.core.models", "fairchem.core.models.uma",
                 "fairchem.core.models.uma.escn_md"]:
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.modules["fairchem.core.models.uma.escn_md"].balance_channels_batched = balance_channels_batched

    if REFERENCE_DIR not in sys.path:
        sys.path.insert(0, REFERENCE_DIR)
    import ops.geom as geom
    import ops.gather as gather
    import ops.gating as gating
    import ops.scatter as scatter
    import ops.ln_silu as ln_silu
    import model as ref_model
    import wrapper as ref_wrapper

    ns = types.SimpleNamespace(
        precompute_geometry=geom.precompute_geometry,
        gather_wigner_split=gather.gather_wigner_split,
        fused_gating_split=gating.fused_gating_split,
        rotate_scatter_split=scatter.rotate_scatter_split,
        init_node_scatter=scatter.init_node_scatter,
        layer_norm_silu=ln_silu.layer_norm_silu,
    )
    return ns, ref_model, ref_wrapper
