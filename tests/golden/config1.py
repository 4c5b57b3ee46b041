"""Config 1 of the benchmark: a tiny random-init Qwen3-MoE-shaped model that
the reference runs end to end on the CPU.

4 layers, d_model 256, 4 query heads and 2 key/value heads of dimension 64,
16 routed experts (top-2) with SwiGLU intermediate 512, vocabulary 1024.
Expert weights are drawn from N(0, 0.02) and quantised to symmetric int4 per
group of 32 inputs with one f32 scale per group (the scheme of
moelan/tiny.py:94-100), written in the colibri int4 container layout that
moelan reads (``merged_weight`` = packed gate | up | down nibbles, ``qs`` =
their scales, ``qwen36_meta.json``; moelan/experts.py:403-416,
config.py:185-195); router weights are N(0, 1).  The remaining weights
(embeddings, attention, norms, output head) follow the usual tiny-model
recipe (N(0, 1/fan_in) projections, norms near 1).  Everything comes from
numpy's PCG64 with seed 0, so the GPU box regenerates the same bytes.

The greedy run: 16 new tokens after a 32-token prompt of random ids.
"""

from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

LAYERS, HIDDEN, HEADS, KV_HEADS, HEAD_DIM = 4, 256, 4, 2, 64
EXPERTS, TOP_K, INTER, GS, VOCAB = 16, 2, 512, 32, 1024
PROMPT_LEN, NEW_TOKENS, SEED = 32, 16, 0


def prompt() -> list[int]:
    return [int(t) for t in np.random.default_rng(SEED + 1).integers(0, VOCAB, PROMPT_LEN)]


def _int4(m: np.ndarray, gs: int):
    """Symmetric int4 per group of gs inputs: values -8..7, f32 scale = absmax / 7."""
    O, I = m.shape
    g = m.reshape(O, I // gs, gs)
    s = (np.abs(g).max(2) / 7.0).astype(np.float32)
    s = np.where(s == 0, np.float32(1.0), s).astype(np.float32)
    v = np.clip(np.rint(g / s[:, :, None]), -8, 7).astype(np.int8).reshape(O, I)
    return v, s


def _pack(v: np.ndarray) -> np.ndarray:
    """Two's-complement nibbles, low nibble = even column."""
    n = (v & 15).astype(np.uint8)
    return np.ascontiguousarray(n[:, 0::2] | (n[:, 1::2] << 4))


def write_safetensors(tensors: dict, path: Path) -> None:
    """A .safetensors file (8-byte little-endian header length, JSON header of
    dtype / shape / byte range per tensor, then the raw bytes): f32 and u8."""
    tags = {np.dtype(np.float32): "F32", np.dtype(np.uint8): "U8"}
    header, blobs, off = {}, [], 0
    for name, a in tensors.items():
        a = np.ascontiguousarray(a)
        b = a.tobytes()
        header[name] = {"dtype": tags[a.dtype], "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def write_model(out_dir) -> Path:
    """Write the config-1 checkpoint into out_dir and return its path."""
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    rng = np.random.default_rng(SEED)

    def w(*shape, scale=None):
        s = 1.0 / np.sqrt(shape[-1]) if scale is None else scale
        return (rng.standard_normal(shape) * s).astype(np.float32)

    def norm(n):
        return (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)

    t = {"model.embed_tokens.weight": w(VOCAB, HIDDEN, scale=0.5), "model.norm.weight": norm(HIDDEN),
         "lm_head.weight": w(VOCAB, HIDDEN)}
    for i in range(LAYERS):
        p = f"model.layers.{i}"
        t.update({
            f"{p}.input_layernorm.weight": norm(HIDDEN),
            f"{p}.post_attention_layernorm.weight": norm(HIDDEN),
            f"{p}.self_attn.q_proj.weight": w(HEADS * HEAD_DIM, HIDDEN),
            f"{p}.self_attn.k_proj.weight": w(KV_HEADS * HEAD_DIM, HIDDEN),
            f"{p}.self_attn.v_proj.weight": w(KV_HEADS * HEAD_DIM, HIDDEN),
            f"{p}.self_attn.o_proj.weight": w(HIDDEN, HEADS * HEAD_DIM),
            f"{p}.self_attn.q_norm.weight": norm(HEAD_DIM),
            f"{p}.self_attn.k_norm.weight": norm(HEAD_DIM),
            f"{p}.mlp.gate.weight": w(EXPERTS, HIDDEN, scale=1.0),
        })
        for e in range(EXPERTS):
            q = [_int4(w(*shape, scale=0.02), GS) for shape in ((INTER, HIDDEN), (INTER, HIDDEN), (HIDDEN, INTER))]
            t[f"{p}.mlp.experts.{e}.merged_weight"] = np.concatenate([_pack(v).reshape(-1) for v, _ in q])
            t[f"{p}.mlp.experts.{e}.qs"] = np.concatenate([s.reshape(-1) for _, s in q])
    write_safetensors(t, out / "model.safetensors")
    (out / "config.json").write_text(json.dumps({
        "architectures": ["Qwen3MoeForCausalLM"], "model_type": "qwen3_moe",
        "vocab_size": VOCAB, "hidden_size": HIDDEN, "num_hidden_layers": LAYERS,
        "num_attention_heads": HEADS, "num_key_value_heads": KV_HEADS, "head_dim": HEAD_DIM,
        "num_experts": EXPERTS, "num_experts_per_tok": TOP_K, "moe_intermediate_size": INTER,
        "norm_topk_prob": True, "rms_norm_eps": 1e-6, "rope_theta": 10000.0,
        "bos_token_id": VOCAB - 2, "eos_token_id": VOCAB - 1, "tie_word_embeddings": False,
        "max_position_embeddings": 2048}, indent=2))
    (out / "qwen36_meta.json").write_text(json.dumps({
        "model_type": "qwen3_moe", "ebits": 4, "expert_gs": GS, "num_experts": EXPERTS, "topk": TOP_K,
        "moe_inter": INTER}))
    return out


def greedy(model, n: int = NEW_TOKENS):
    """Greedy tokens and the logits each was chosen from, through the model's
    own cache-based forward (moelan/model.py:698-713 with temperature 0 and no
    stop tokens)."""
    cache = model.new_cache()
    logits = model.forward(prompt(), cache)
    toks, all_logits = [], []
    for _ in range(n):
        all_logits.append(np.asarray(logits, np.float32).copy())
        tok = int(np.argmax(logits))
        toks.append(tok)
        logits = model.forward([tok], cache)
    return np.array(toks, np.int32), np.stack(all_logits)
