"""Seeded synthetic checkpoints and inputs for the five benchmark configurations.

No network and no real checkpoints are available, so every configuration runs
on random-init weights of the named architecture and seeded token ids:

* weights: numpy PCG64 ``default_rng(seed)`` (seed 0), tensors drawn in the
  order ``tensor_specs`` lists them; linear and embedding weights
  N(0, 0.02) as float32 (``standard_normal(dtype=float32) * 0.02``); norm
  weights 1.0 (``norm_jitter`` > 0 gives ``1 + norm_jitter * N(0,1)`` instead,
  used by the small test models so a mis-applied norm weight shows);
* inputs: ``default_rng(config seed)`` as each ``*_inputs`` function states.

Tensor names follow the Hugging Face checkpoints the reference loads
(crates/inl-text/src/qwen3/mod.rs:180-330), so the same dictionaries can be
written to safetensors and read by both the library and the CPU oracle.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

# --------------------------------------------------------------------- configs
# Config 1/3/5 tower: Qwen3-Embedding-0.6B architecture.
QWEN3_0_6B = {
    "model_type": "qwen3",
    "hidden_size": 1024,
    "intermediate_size": 3072,
    "num_attention_heads": 16,
    "num_key_value_heads": 8,
    "head_dim": 128,
    "num_hidden_layers": 28,
    "rms_norm_eps": 1e-6,
    "rope_theta": 1_000_000.0,
    "vocab_size": 151669,
    "hidden_act": "silu",
    "attention_bias": False,
    "max_position_embeddings": 32768,
}

# Small Qwen3-shaped models for fast kernel parity (same code paths).
QWEN3_TINY = dict(QWEN3_0_6B, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                  num_key_value_heads=2, head_dim=128, num_hidden_layers=2, vocab_size=1000,
                  rope_theta=10_000.0, max_position_embeddings=4096)
QWEN3_TINY_D64 = dict(QWEN3_TINY, hidden_size=192, num_attention_heads=6, num_key_value_heads=3, head_dim=64,
                      intermediate_size=384)

LATE_PROJ_OUT = 128

# Config 2: ModernBERT-style SPLADE encoder (KURE-Sparse-nano shapes, BASELINE vocabulary).
# The benchmark config pins: V = 36282 tied decoder with a zero-initialised
# decoder bias, logit shift 0, no prefix tokens, no vocabulary mask, no fold.
MODERNBERT_SPLADE = {
    "model_type": "modernbert",
    "vocab_size": 36282,
    "hidden_size": 768,
    "intermediate_size": 1152,
    "num_hidden_layers": 22,
    "num_attention_heads": 12,
    "norm_eps": 1e-5,
    "local_attention": 128,
    "global_attn_every_n_layers": 3,
    "global_rope_theta": 160000.0,
    "local_rope_theta": 10000.0,
    "max_position_embeddings": 8192,
    "decoder_bias": True,
    "splade": {"logit_shift": 0.0},
}
MODERNBERT_TINY = dict(MODERNBERT_SPLADE, vocab_size=1000, hidden_size=256, intermediate_size=384,
                       num_hidden_layers=4, num_attention_heads=4, local_attention=32,
                       splade={"logit_shift": 0.05, "prefix_token_ids": [5], "masked_vocab_ids": [7, 9],
                               "canonical_ids": [v % 900 for v in range(1000)]})

# Config 4: EmbeddingGemma-style text tower (BASELINE shapes); per-layer
# embeddings and layer scalars dropped, embedding_projection replaced by the
# dense 768 -> 3072 -> 768 chain.
GEMMA_STYLE = {
    "model_type": "gemma_style",
    "vocab_size": 262144,
    "hidden_size": 768,
    "intermediate_size": 1152,
    "num_hidden_layers": 24,
    "num_attention_heads": 3,
    "num_key_value_heads": 1,
    "head_dim": 256,
    "rms_norm_eps": 1e-6,
    "sliding_window": 512,
    "full_attention_every_n_layers": 6,
    "rope_theta": 1_000_000.0,
    "rope_local_base_freq": 10_000.0,
    "hidden_activation": "gelu_pytorch_tanh",
    "dense_dims": [3072, 768],
    "max_position_embeddings": 8192,
}
GEMMA_TINY = dict(GEMMA_STYLE, vocab_size=1000, hidden_size=256, intermediate_size=384, num_hidden_layers=4,
                  num_attention_heads=2, num_key_value_heads=1, head_dim=128, sliding_window=40,
                  full_attention_every_n_layers=2, dense_dims=[512, 256])
MATRYOSHKA_DIMS = (128, 256, 512, 768)

# EmbeddingGemma 2 text tower as the reference loads it
# (crates/inl-text/src/gemma2.rs:78-211): nested text_config, per-layer
# embeddings (PLE) and layer scalars, per_layer_config head overrides on the
# full layer, embedding_projection to embedding_dim. Small widths; the full
# layer's head_dim 256 and the sliding layers' 128 take different attention
# query blocks in bf16.
EMBEDDING_GEMMA2_SMALL = {
    "model_type": "embedding_gemma2",
    "text_config": {
        "vocab_size": 1000,
        "hidden_size": 256,
        "intermediate_size": 512,
        "num_hidden_layers": 4,
        "num_attention_heads": 4,
        "num_key_value_heads": 2,
        "head_dim": 128,
        "hidden_activation": "gelu_pytorch_tanh",
        "rms_norm_eps": 1e-6,
        "sliding_window": 24,
        "layer_types": ["sliding_attention", "sliding_attention", "full_attention", "sliding_attention"],
        "hidden_size_per_layer_input": 64,
        "embedding_dim": 128,
        "rope_parameters": {
            "sliding_attention": {"rope_type": "default", "rope_theta": 10_000.0},
            "full_attention": {"rope_type": "default", "rope_theta": 1_000_000.0},
        },
        "max_position_embeddings": 2048,
        "per_layer_config": {"02": {"head_dim": 256, "num_key_value_heads": 1}},
    },
}


@dataclass
class Spec:
    name: str
    shape: tuple
    kind: str  # "linear" | "norm"


def qwen3_specs(cfg: dict) -> list[Spec]:
    H, I = cfg["hidden_size"], cfg["intermediate_size"]
    hq, hkv = cfg["num_attention_heads"], cfg["num_key_value_heads"]
    d = cfg.get("head_dim") or H // hq
    specs = [Spec("embed_tokens.weight", (cfg["vocab_size"], H), "linear")]
    for i in range(cfg["num_hidden_layers"]):
        p = f"layers.{i}."
        specs += [
            Spec(p + "self_attn.q_proj.weight", (hq * d, H), "linear"),
            Spec(p + "self_attn.k_proj.weight", (hkv * d, H), "linear"),
            Spec(p + "self_attn.v_proj.weight", (hkv * d, H), "linear"),
            Spec(p + "self_attn.o_proj.weight", (H, hq * d), "linear"),
            Spec(p + "self_attn.q_norm.weight", (d,), "norm"),
            Spec(p + "self_attn.k_norm.weight", (d,), "norm"),
            Spec(p + "mlp.gate_proj.weight", (I, H), "linear"),
            Spec(p + "mlp.up_proj.weight", (I, H), "linear"),
            Spec(p + "mlp.down_proj.weight", (H, I), "linear"),
            Spec(p + "input_layernorm.weight", (H,), "norm"),
            Spec(p + "post_attention_layernorm.weight", (H,), "norm"),
        ]
    specs.append(Spec("norm.weight", (H,), "norm"))
    return specs


def modernbert_specs(cfg: dict) -> list[Spec]:
    """Tensor names of crates/inl-sparse/src/modernbert.rs:469-520 (decoder tied)."""
    H, I, V = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    specs = [Spec("model.embeddings.tok_embeddings.weight", (V, H), "linear"),
             Spec("model.embeddings.norm.weight", (H,), "norm")]
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}."
        if i > 0:
            specs.append(Spec(p + "attn_norm.weight", (H,), "norm"))
        specs += [Spec(p + "attn.Wqkv.weight", (3 * H, H), "linear"), Spec(p + "attn.Wo.weight", (H, H), "linear"),
                  Spec(p + "mlp_norm.weight", (H,), "norm"), Spec(p + "mlp.Wi.weight", (2 * I, H), "linear"),
                  Spec(p + "mlp.Wo.weight", (H, I), "linear")]
    specs += [Spec("model.final_norm.weight", (H,), "norm"), Spec("head.dense.weight", (H, H), "linear"),
              Spec("head.norm.weight", (H,), "norm"), Spec("decoder.bias", (V,), "zero")]
    return specs


def gemma_specs(cfg: dict) -> list[Spec]:
    """Tensor names of crates/inl-text/src/gemma2.rs:233-494 (no PLE, no layer
    scalar) plus the dense head chain ``dense_head.<j>.weight``."""
    H, I, V = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    hq, hkv, d = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
    specs = [Spec("embed_tokens.weight", (V, H), "linear")]
    for i in range(cfg["num_hidden_layers"]):
        p = f"layers.{i}."
        specs += [
            Spec(p + "self_attn.q_proj.weight", (hq * d, H), "linear"),
            Spec(p + "self_attn.k_proj.weight", (hkv * d, H), "linear"),
            Spec(p + "self_attn.v_proj.weight", (hkv * d, H), "linear"),
            Spec(p + "self_attn.o_proj.weight", (H, hq * d), "linear"),
            Spec(p + "self_attn.q_norm.weight", (d,), "norm"),
            Spec(p + "self_attn.k_norm.weight", (d,), "norm"),
            Spec(p + "mlp.gate_proj.weight", (I, H), "linear"),
            Spec(p + "mlp.up_proj.weight", (I, H), "linear"),
            Spec(p + "mlp.down_proj.weight", (H, I), "linear"),
            Spec(p + "input_layernorm.weight", (H,), "norm"),
            Spec(p + "post_attention_layernorm.weight", (H,), "norm"),
            Spec(p + "pre_feedforward_layernorm.weight", (H,), "norm"),
            Spec(p + "post_feedforward_layernorm.weight", (H,), "norm"),
        ]
    specs.append(Spec("norm.weight", (H,), "norm"))
    prev = H
    for j, out in enumerate(cfg.get("dense_dims", [])):
        specs.append(Spec(f"dense_head.{j}.weight", (out, prev), "linear"))
        prev = out
    return specs


def embedding_gemma2_specs(cfg: dict) -> list[Spec]:
    """Tensor names of crates/inl-text/src/gemma2.rs:233-560 (text tower with
    PLE, layer scalars, per-layer head shapes and embedding_projection)."""
    tc = cfg.get("text_config", cfg)
    H, I, V, L = tc["hidden_size"], tc["intermediate_size"], tc["vocab_size"], tc["num_hidden_layers"]
    hq, P = tc["num_attention_heads"], tc["hidden_size_per_layer_input"]
    over = {int(k): v for k, v in (tc.get("per_layer_config") or {}).items()}
    specs = [Spec("embed_tokens.weight", (V, H), "linear"),
             Spec("ple.per_layer_model_projection.weight", (L * P, H), "linear"),
             Spec("ple.per_layer_projection_norm.weight", (P,), "norm")]
    for i in range(L):
        d = over.get(i, {}).get("head_dim") or tc["head_dim"]
        kv = over.get(i, {}).get("num_key_value_heads") or tc["num_key_value_heads"]
        p = f"layers.{i}."
        specs += [
            Spec(p + "self_attn.q_proj.weight", (hq * d, H), "linear"),
            Spec(p + "self_attn.k_proj.weight", (kv * d, H), "linear"),
            Spec(p + "self_attn.v_proj.weight", (kv * d, H), "linear"),
            Spec(p + "self_attn.o_proj.weight", (H, hq * d), "linear"),
            Spec(p + "self_attn.q_norm.weight", (d,), "norm"),
            Spec(p + "self_attn.k_norm.weight", (d,), "norm"),
            Spec(p + "mlp.gate_proj.weight", (I, H), "linear"),
            Spec(p + "mlp.up_proj.weight", (I, H), "linear"),
            Spec(p + "mlp.down_proj.weight", (H, I), "linear"),
            Spec(p + "input_layernorm.weight", (H,), "norm"),
            Spec(p + "post_attention_layernorm.weight", (H,), "norm"),
            Spec(p + "pre_feedforward_layernorm.weight", (H,), "norm"),
            Spec(p + "post_feedforward_layernorm.weight", (H,), "norm"),
            Spec(p + "ple_block.per_layer_input_gate.weight", (P, H), "linear"),
            Spec(p + "ple_block.per_layer_projection.weight", (H, P), "linear"),
            Spec(p + "ple_block.post_per_layer_input_norm.weight", (H,), "norm"),
            Spec(p + "layer_scalar", (1,), "norm"),
        ]
    specs.append(Spec("norm.weight", (H,), "norm"))
    specs.append(Spec("embedding_projection.weight", (tc["embedding_dim"], H), "linear"))
    return specs


def generate(specs: list[Spec], seed: int = 0, std: float = 0.02, norm_jitter: float = 0.0) -> dict:
    """Draw every tensor of ``specs`` in order from one PCG64 stream."""
    rng = np.random.default_rng(seed)
    out = {}
    for s in specs:
        n = int(np.prod(s.shape))
        if s.kind == "zero":
            v = np.zeros(n, dtype=np.float32)
        elif s.kind == "norm":
            if norm_jitter > 0:
                v = 1.0 + norm_jitter * rng.standard_normal(n, dtype=np.float32)
            else:
                v = np.ones(n, dtype=np.float32)
        else:
            v = rng.standard_normal(n, dtype=np.float32)
            v *= np.float32(std)
        out[s.name] = v.astype(np.float32, copy=False).reshape(s.shape)
    return out


def qwen3_weights(cfg: dict = QWEN3_0_6B, seed: int = 0, norm_jitter: float = 0.0) -> dict:
    return generate(qwen3_specs(cfg), seed=seed, norm_jitter=norm_jitter)


def modernbert_weights(cfg: dict = MODERNBERT_SPLADE, seed: int = 0, norm_jitter: float = 0.0) -> dict:
    return generate(modernbert_specs(cfg), seed=seed, norm_jitter=norm_jitter)


def gemma_weights(cfg: dict = GEMMA_STYLE, seed: int = 0, norm_jitter: float = 0.0) -> dict:
    return generate(gemma_specs(cfg), seed=seed, norm_jitter=norm_jitter)


def embedding_gemma2_weights(cfg: dict = EMBEDDING_GEMMA2_SMALL, seed: int = 0, norm_jitter: float = 0.0) -> dict:
    return generate(embedding_gemma2_specs(cfg), seed=seed, norm_jitter=norm_jitter)


def late_projection(cfg: dict = QWEN3_0_6B, out: int = LATE_PROJ_OUT, seed: int = 0) -> np.ndarray:
    """Dense 1024->128 ``linear.weight`` [out, H], drawn from ``default_rng(seed + 1000)``
    so that it does not shift the tower's stream."""
    rng = np.random.default_rng(seed + 1000)
    w = rng.standard_normal(out * cfg["hidden_size"], dtype=np.float32) * np.float32(0.02)
    return w.reshape(out, cfg["hidden_size"])


# ---------------------------------------------------------------------- inputs
def packed(lengths: np.ndarray, ids: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    cu = np.zeros(len(lengths) + 1, dtype=np.int32)
    np.cumsum(lengths, out=cu[1:])
    return np.ascontiguousarray(ids, dtype=np.uint32), cu


def cfg1_inputs(vocab: int = QWEN3_0_6B["vocab_size"]):
    """Config 1: 8 texts x 128 ids uniform in [0, vocab), default_rng(1).integers."""
    rng = np.random.default_rng(1)
    ids = rng.integers(0, vocab, size=(8, 128))
    return packed(np.full(8, 128), ids.reshape(-1))


def cfg3_inputs(vocab: int = QWEN3_0_6B["vocab_size"]):
    """Config 3: 64 texts x 512 ids, default_rng(3).integers."""
    rng = np.random.default_rng(3)
    ids = rng.integers(0, vocab, size=(64, 512))
    return packed(np.full(64, 512), ids.reshape(-1))


def cfg5_corpus(n_texts: int = 65536, vocab: int = QWEN3_0_6B["vocab_size"], seed: int = 5):
    """Config 5: lengths clip(round(exp(ln 256 + 0.6 N(0,1))), 8, 2048) then ids
    uniform in [0, vocab), both from default_rng(5) in that order."""
    rng = np.random.default_rng(seed)
    z = rng.standard_normal(n_texts)
    lengths = np.clip(np.rint(np.exp(math.log(256.0) + 0.6 * z)), 8, 2048).astype(np.int64)
    ids = rng.integers(0, vocab, size=int(lengths.sum()), dtype=np.int64)
    return lengths, ids.astype(np.uint32)


def random_texts(n: int, lo: int, hi: int, vocab: int, seed: int):
    """Ragged test inputs: lengths uniform in [lo, hi], ids uniform."""
    rng = np.random.default_rng(seed)
    lengths = rng.integers(lo, hi + 1, size=n)
    ids = rng.integers(0, vocab, size=int(lengths.sum()))
    return packed(lengths, ids)


def cfg2_inputs(vocab: int = MODERNBERT_SPLADE["vocab_size"]):
    """Config 2: 32 texts, lengths uniform in [16, 256], ids uniform; default_rng(2)
    draws the lengths then the ids."""
    rng = np.random.default_rng(2)
    lengths = rng.integers(16, 257, size=32)
    ids = rng.integers(0, vocab, size=int(lengths.sum()))
    return packed(lengths, ids)


def cfg4_inputs(vocab: int = GEMMA_STYLE["vocab_size"], n_texts: int = 128):
    """Config 4: lengths log-uniform in [32, 2048] (round(exp(U(ln 32, ln 2048)))),
    ids uniform; default_rng(4) draws the lengths then the ids."""
    rng = np.random.default_rng(4)
    lengths = np.rint(np.exp(rng.uniform(math.log(32.0), math.log(2048.0), size=n_texts))).astype(np.int64)
    ids = rng.integers(0, vocab, size=int(lengths.sum()))
    return packed(lengths, ids)
