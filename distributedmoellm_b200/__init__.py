"""distributedmoellm_b200: moelan's routed-expert hot path on NVIDIA B200.

Hand-written sm_100a CUDA kernels (csrc/, built into _lib/libmoelan_b200.so
and bound with ctypes) for:

* bit-exact dequantisation of int4 / int8 / GGUF expert weights;
* the router (logits, softmax top-k), the stable permute by expert and the
  weighted combine;
* fused decode mat-vecs over packed experts (gate|up, SiLU, down);
* grouped GEMMs on the tcgen05 tensor cores for prefill-sized batches;
* expert parallelism over NCCL (ep.py).

``install()`` swaps them in behind moelan's own entry points (its kernels
module and its ``--gpu`` expert tier), so moelan's coordinator and workers
run them unchanged.  There is no CPU fallback: without a CUDA device the
entry points raise RuntimeError.
"""

from ._build import build  # noqa: F401

__version__ = "0.1.0"


def install(moelan_module=None):
    """Patch moelan's expert-compute entry points with the B200 path."""
    from .dropin import install as _install
    return _install(moelan_module)


def uninstall(saved):
    """Undo :func:`install` (``saved``: what it returned)."""
    from .dropin import uninstall as _uninstall
    return _uninstall(saved)
