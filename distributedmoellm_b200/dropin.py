"""Put the B200 path behind moelan's own entry points.

moelan looks its kernels up as module attributes at call time
(moelan/experts.py:151, 153, 219, 221, 743, 752; gguf.py:263, 289, 293) and
imports its GPU tier inside ``ExpertStore.setup_gpu`` (experts.py:760) and the
node benchmarks (coordinator.py:268-271, worker.py:278-281), so replacing
those attributes is the whole integration: coordinator.py and worker.py run
unchanged, and ``--gpu cuda`` selects this library's tier.
"""

from __future__ import annotations

import importlib

KERNEL_NAMES = ("moe_q4", "q4_expert_ptrs", "q4_matmul_t", "q8_matmul_t", "gguf_matmul_t", "q4_dequant",
                "q8_dequant", "gguf_dequant")
ACCEL_NAMES = ("GpuTier", "bench_gpu")


def install(moelan_module=None) -> dict:
    """Patch ``moelan.kernels`` and ``moelan.accel`` (or the given package
    object's ``kernels`` / ``accel``) with this library's entry points.
    Raises RuntimeError, patching nothing, when no sm_100 CUDA device is
    usable (there is no CPU fallback).  Returns the replaced originals, for
    :func:`uninstall`."""
    from . import device as D
    D.require_device()
    from . import accel, kernels
    pkg = moelan_module if moelan_module is not None else importlib.import_module("moelan")
    mk = getattr(pkg, "kernels", None) or importlib.import_module(pkg.__name__ + ".kernels")
    ma = getattr(pkg, "accel", None) or importlib.import_module(pkg.__name__ + ".accel")
    saved = {}
    for mod, src, names in ((mk, kernels, KERNEL_NAMES), (ma, accel, ACCEL_NAMES)):
        for n in names:
            saved[(mod, n)] = getattr(mod, n, None)
            setattr(mod, n, getattr(src, n))
    return saved


def uninstall(saved: dict) -> None:
    """Put back what :func:`install` replaced."""
    for (mod, n), v in saved.items():
        setattr(mod, n, v)
