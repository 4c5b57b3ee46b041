"""Generate tests/golden/config1.npz: the reference's own greedy run of the
config-1 model (tokens and the logits each token was chosen from).

    python tests/golden/make_config1_golden.py <moelan project root>

Imports moelan from the given source tree (numba kernels on, int8
activations off, as the other fixtures), writes the config-1 checkpoint with
tests/golden/config1.py into a temporary directory and runs moelan's
MoEModel on it.  The GPU box never runs this script; it only reads the .npz.
"""

from __future__ import annotations

import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def main(ref_root: str) -> None:
    os.environ.setdefault("MOELAN_INT8_ACT", "0")
    os.environ.setdefault("NUMBA_CACHE_DIR", tempfile.mkdtemp(prefix="numba_"))
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(Path(ref_root).resolve()))
    sys.path.insert(0, str(HERE))
    import config1 as C1
    from moelan import kernels
    from moelan.model import MoEModel
    with tempfile.TemporaryDirectory() as d:
        model = MoEModel(C1.write_model(d))
        toks, logits = C1.greedy(model)
    np.savez_compressed(HERE / "config1.npz", tokens=toks, logits=logits, kernels_enabled=np.int32(kernels.ENABLED))
    print("config-1 greedy tokens:", toks.tolist(), "numba kernels:", kernels.ENABLED)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python make_config1_golden.py <moelan project root>")
    main(sys.argv[1])
