"""Pins the EmbeddingGemma oracle (oracle/gemma.py) against the reference's own
golden fixture tiny_embeddinggemma2 (copied by tests/golden/make_golden.py):
the assertion of crates/inl-text/src/gemma2.rs:941-967 — every vector within
2e-5 of the golden, batched and alone, at max_length 64 and 9 (truncation)."""
import json
import math
from pathlib import Path

import numpy as np

from oracle import gemma as G

GOLDEN = Path(__file__).resolve().parent / "golden" / "tiny_embeddinggemma2"


def tokenize(text: str, max_length: int, vocab: dict) -> list[int]:
    """The fixture's tokenizer.json: Lowercase normaliser, Whitespace
    pre-tokeniser, WordLevel model (<unk> = 3), template <bos> A <eos>,
    truncation of the content to leave room for the two special tokens."""
    words = [vocab.get(w, vocab["<unk>"]) for w in text.lower().split()]
    return [vocab["<bos>"]] + words[: max(0, max_length - 2)] + [vocab["<eos>"]]


def load():
    from safetensors.numpy import load_file

    cfg = json.loads((GOLDEN / "config.json").read_text())
    weights = load_file(str(GOLDEN / "model.safetensors"))
    golden = json.loads((GOLDEN / "golden.json").read_text())
    vocab = json.loads((GOLDEN / "tokenizer.json").read_text())["model"]["vocab"]
    return cfg, weights, golden, vocab


def test_tokenizer_restatement_matches_golden_lengths():
    cfg, weights, golden, vocab = load()
    for case in golden["cases"]:
        lens = [len(tokenize(t, case["max_length"], vocab)) for t in golden["texts"]]
        assert lens == case["lengths"]


def test_tiny_embeddinggemma2_golden_batched_and_alone():
    cfg, weights, golden, vocab = load()
    for case in golden["cases"]:
        rows = [tokenize(t, case["max_length"], vocab) for t in golden["texts"]]
        ids = np.concatenate([np.asarray(r, dtype=np.uint32) for r in rows])
        cu = np.concatenate([[0], np.cumsum([len(r) for r in rows])]).astype(np.int32)
        got = G.embed(weights, cfg, ids, cu)
        assert got.shape[1] == golden["dim"]
        for i, want in enumerate(case["batched"]):
            assert np.abs(got[i] - np.asarray(want)).max() < 2e-5, (case["max_length"], i)
        for i, r in enumerate(rows):
            alone = G.embed(weights, cfg, np.asarray(r, dtype=np.uint32), np.array([0, len(r)]))
            assert np.abs(alone[0] - np.asarray(case["alone"][i])).max() < 2e-5, (case["max_length"], i)


def test_layer_shapes_follow_per_layer_overrides():
    cfg, *_ = load()
    tc = cfg["text_config"]
    assert G.layer_shape(tc, 2) == ("full_attention", 32, 1)
    assert G.layer_shape(tc, 1) == ("sliding_attention", 16, 2)


def test_dense_head_variant_is_unit_length_and_matryoshka():
    rng = np.random.default_rng(0)
    tc = {"hidden_size": 32, "intermediate_size": 48, "num_hidden_layers": 2, "num_attention_heads": 3,
          "num_key_value_heads": 1, "head_dim": 16, "rms_norm_eps": 1e-6, "sliding_window": 4,
          "full_attention_every_n_layers": 2, "vocab_size": 50, "rope_theta": 1e6, "rope_local_base_freq": 1e4}
    w = {"embed_tokens.weight": rng.standard_normal((50, 32)).astype(np.float32) * 0.1,
         "norm.weight": np.ones(32, np.float32)}
    for i in range(2):
        p = f"layers.{i}."
        for n, s in [("self_attn.q_proj.weight", (48, 32)), ("self_attn.k_proj.weight", (16, 32)),
                     ("self_attn.v_proj.weight", (16, 32)), ("self_attn.o_proj.weight", (32, 48)),
                     ("mlp.gate_proj.weight", (48, 32)), ("mlp.up_proj.weight", (48, 32)),
                     ("mlp.down_proj.weight", (32, 48))]:
            w[p + n] = rng.standard_normal(s).astype(np.float32) * 0.1
        for n, d in [("self_attn.q_norm.weight", 16), ("self_attn.k_norm.weight", 16),
                     ("input_layernorm.weight", 32), ("post_attention_layernorm.weight", 32),
                     ("pre_feedforward_layernorm.weight", 32), ("post_feedforward_layernorm.weight", 32)]:
            w[p + n] = np.ones(d, np.float32)
    dense = [rng.standard_normal((64, 32)).astype(np.float32), rng.standard_normal((32, 64)).astype(np.float32)]
    ids = rng.integers(0, 50, 20).astype(np.uint32)
    cu = np.array([0, 7, 20])
    full = G.embed_dense_head(w, tc, dense, ids, cu)
    short = G.embed_dense_head(w, tc, dense, ids, cu, out_dim=16)
    assert np.allclose(np.linalg.norm(full, axis=1), 1, atol=1e-5)
    assert np.allclose(np.linalg.norm(short, axis=1), 1, atol=1e-5)
    ref = full[:, :16] / np.linalg.norm(full[:, :16], axis=1, keepdims=True)
    assert np.abs(short - ref).max() < 1e-6
    assert math.isclose(float(np.sqrt(32.0)), float(np.float32(np.sqrt(32.0))), rel_tol=1e-7)


def test_synthetic_embedding_gemma2_exercises_ple_and_layer_shapes():
    """The GPU test's synthetic EmbeddingGemma 2 is sensitive to what it
    checks: dropping the per-layer embeddings, or the layer scalars, moves
    the oracle's embeddings well beyond the bf16 floor (cosine 0.999)."""
    import im_not_llm_b200 as inl

    cfg = inl.synthetic.EMBEDDING_GEMMA2_SMALL
    w = inl.synthetic.embedding_gemma2_weights(cfg, seed=2, norm_jitter=0.1)
    assert G.layer_shape(cfg["text_config"], 2) == ("full_attention", 256, 1)
    ids, cu = inl.synthetic.random_texts(4, 20, 120, cfg["text_config"]["vocab_size"], seed=5)
    ref = G.embed(w, cfg, ids, cu, prefix="")
    no_ple = G.embed({k: v for k, v in w.items() if not k.startswith("ple.")}, cfg, ids, cu, prefix="")
    unit = {k: (np.ones_like(v) * 1.5 if k.endswith("layer_scalar") else v) for k, v in w.items()}
    scaled = G.embed(unit, cfg, ids, cu, prefix="")
    for other in (no_ple, scaled):
        assert ((ref * other).sum(-1)).min() < 0.999
