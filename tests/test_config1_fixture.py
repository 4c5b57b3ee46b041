"""Pins the config-1 fixture on the CPU: the reference (installed under
baseline/_ref), run unpatched on the checkpoint that tests/golden/config1.py
writes, gives exactly the tokens and logits stored in
tests/golden/config1.npz.  Skips when the reference is not installed."""

import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"


def test_reference_reproduces_the_config1_golden(tmp_path):
    if not (REF / "moelan").is_dir():
        pytest.skip("the reference is not installed under baseline/_ref")
    os.environ.setdefault("MOELAN_INT8_ACT", "0")
    os.environ.setdefault("NUMBA_CACHE_DIR", tempfile.mkdtemp(prefix="numba_"))
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import config1 as C1
    from moelan.model import MoEModel
    toks, logits = C1.greedy(MoEModel(C1.write_model(tmp_path)))
    with np.load(ROOT / "tests" / "golden" / "config1.npz") as g:
        assert toks.tolist() == g["tokens"].tolist()
        assert np.array_equal(logits, g["logits"])


def test_config1_checkpoint_layout(tmp_path):
    """The writer's container: one safetensors file with the colibri int4
    expert tensors (packed gate | up | down nibbles and their f32 scales)."""
    import json
    import struct
    import config1 as C1
    d = C1.write_model(tmp_path)
    raw = (d / "model.safetensors").read_bytes()
    n = struct.unpack("<Q", raw[:8])[0]
    hdr = json.loads(raw[8:8 + n])
    e = hdr["model.layers.0.mlp.experts.3.merged_weight"]
    assert e["dtype"] == "U8" and e["shape"] == [(2 * C1.INTER * C1.HIDDEN + C1.HIDDEN * C1.INTER) // 2]
    s = hdr["model.layers.0.mlp.experts.3.qs"]
    assert s["dtype"] == "F32" and s["shape"] == [(2 * C1.INTER * C1.HIDDEN + C1.HIDDEN * C1.INTER) // C1.GS]
    meta = json.loads((d / "qwen36_meta.json").read_text())
    assert meta["ebits"] == 4 and meta["expert_gs"] == C1.GS
    assert len(C1.prompt()) == C1.PROMPT_LEN and max(C1.prompt()) < C1.VOCAB
