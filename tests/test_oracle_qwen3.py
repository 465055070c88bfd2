"""Pins the Qwen3 oracle (oracle/qwen3.py) against the reference's own unit-test
invariants and a second opinion from transformers' Qwen3Model.

The reference tests restated here:
  * fused_rms_norm_matches_the_textbook_definition   crates/inl-text/src/qwen3/mod.rs:705-730
  * fused_rope_matches_the_manual_half_split_rotation crates/inl-text/src/qwen3/mod.rs:677-703
  * embeddings_are_unit_length_and_independent_of_batch_padding  :646-669
  * additive_mask_matches_the_reference_formula       crates/inl-core/src/attention.rs:402-432
  * tiled_and_flash_match_eager_on_padded_batches     crates/inl-core/src/attention.rs:434-481
"""
import numpy as np
import pytest

import im_not_llm_b200 as inl
from oracle import common as C
from oracle import qwen3 as Q
from tests.conftest import cosine_rows


def pseudo(n, seed, mul=2654435761, add=7):
    """The reference tests' 32-bit LCG in [-0.5, 0.5) (crates/inl-text/src/qwen3/mod.rs:480-488)."""
    state = (seed * mul + add) & 0xFFFFFFFF
    out = np.empty(n, dtype=np.float32)
    for i in range(n):
        state = (state * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = np.float32(state >> 8) / np.float32(1 << 24) - np.float32(0.5)
    return out


def test_rms_norm_matches_textbook():
    x = pseudo(3 * 48, 9).reshape(3, 48)
    w = pseudo(48, 4)
    var = (x * x).mean(-1, keepdims=True)
    expected = x / np.sqrt(var + 1e-6) * w
    assert np.abs(C.rms_norm(x, w, 1e-6) - expected).max() < 1e-5


def test_rope_matches_manual_half_split_rotation():
    heads, seq, dim = 2, 5, 32
    x = pseudo(heads * seq * dim, 11).reshape(heads, seq, dim).transpose(1, 0, 2)  # [L, heads, d]
    cos, sin = C.rope_table(dim, 10_000.0, seq)
    got = C.apply_rope(x, cos, sin)
    # manual: x*[cos,cos] + rotate_half(x)*[sin,sin]
    c2 = np.concatenate([cos, cos], -1)[:, None]
    s2 = np.concatenate([sin, sin], -1)[:, None]
    rot = np.concatenate([-x[..., dim // 2:], x[..., :dim // 2]], -1)
    assert np.abs(got - (x * c2 + rot * s2)).max() < 1e-5


def test_rope_table_is_f64_then_f32():
    cos, sin = C.rope_table(128, 1e6, 2048)
    i = np.arange(64)
    ang = 2047 * (1.0 / 1e6 ** (2 * i / 128))
    assert np.array_equal(cos[2047], np.cos(ang).astype(np.float32))
    assert np.array_equal(sin[2047], np.sin(ang).astype(np.float32))


def _padded_attention(q, k, v, pads, scale):
    """Eager attention on a left-padded batch with the reference's additive mask
    (causal -1e4, padded keys -1e4, both summed): crates/inl-core/src/attention.rs:170-199,236-249."""
    B, S, hq, d = q.shape
    rep = hq // k.shape[2]
    kk = np.repeat(k, rep, axis=2)
    vv = np.repeat(v, rep, axis=2)
    out = np.zeros_like(q)
    qi = np.arange(S)[:, None]
    ki = np.arange(S)[None, :]
    for b in range(B):
        mask = np.where(ki > qi, C.MASK_VALUE, 0).astype(np.float32)
        mask += np.where(ki < pads[b], C.MASK_VALUE, 0).astype(np.float32)
        s = np.einsum("qhd,khd->hqk", q[b], kk[b]) * scale + mask[None]
        out[b] = np.einsum("hqk,khd->qhd", C.softmax(s), vv[b])
    return out


def test_packed_attention_equals_padded_reference_attention():
    rng = np.random.default_rng(0)
    pads, S, hq, hkv, d = [0, 5, 11, 2], 13, 4, 2, 32
    q = rng.standard_normal((4, S, hq, d)).astype(np.float32)
    k = rng.standard_normal((4, S, hkv, d)).astype(np.float32)
    v = rng.standard_normal((4, S, hkv, d)).astype(np.float32)
    ref = _padded_attention(q, k, v, pads, d ** -0.5)
    for b, p in enumerate(pads):
        got = C.attend_text(q[b, p:], k[b, p:], v[b, p:], d ** -0.5, causal=True)
        assert np.abs(got - ref[b, p:]).max() < 1e-5


def test_additive_mask_formula():
    seq, pads = 7, [0, 3, 7]
    qi = np.arange(seq)[:, None]
    ki = np.arange(seq)[None, :]
    for pad in pads:
        m = np.where(ki > qi, C.MASK_VALUE, 0) + np.where(ki < pad, C.MASK_VALUE, 0)
        for q in range(seq):
            for k in range(seq):
                exp = (C.MASK_VALUE if k > q else 0) + (C.MASK_VALUE if k < pad else 0)
                assert m[q, k] == exp


@pytest.fixture(scope="module")
def tiny():
    cfg = dict(inl.synthetic.QWEN3_TINY)
    w = inl.synthetic.qwen3_weights(cfg, seed=0, norm_jitter=0.1)
    # Larger weights than 0.02 so that every layer moves the residual stream.
    for k, v in w.items():
        if v.ndim == 2 and not k.startswith("embed"):
            w[k] = v * np.float32(5.0)
    return cfg, w


def test_embeddings_are_unit_length_and_independent_of_packing(tiny):
    cfg, w = tiny
    ids, cu = inl.synthetic.random_texts(5, 3, 40, cfg["vocab_size"], seed=3)
    batched = Q.embed_last(w, cfg, ids, cu)
    assert np.allclose(np.linalg.norm(batched, axis=-1), 1.0, atol=1e-5)
    for i in range(5):
        s, e = cu[i], cu[i + 1]
        alone = Q.embed_last(w, cfg, ids[s:e], np.array([0, e - s]))
        assert cosine_rows(alone, batched[i:i + 1])[0] > 0.99999


def test_oracle_matches_transformers_qwen3(tiny):
    """Second opinion: transformers' Qwen3Model (f32 CPU, eager attention) on the same weights."""
    torch = pytest.importorskip("torch")
    transformers = pytest.importorskip("transformers")
    cfg, w = tiny
    hf_cfg = transformers.Qwen3Config(
        vocab_size=cfg["vocab_size"], hidden_size=cfg["hidden_size"], intermediate_size=cfg["intermediate_size"],
        num_hidden_layers=cfg["num_hidden_layers"], num_attention_heads=cfg["num_attention_heads"],
        num_key_value_heads=cfg["num_key_value_heads"], head_dim=cfg["head_dim"], rms_norm_eps=cfg["rms_norm_eps"],
        rope_theta=cfg["rope_theta"], max_position_embeddings=cfg["max_position_embeddings"],
        attention_bias=False, tie_word_embeddings=False)
    hf_cfg._attn_implementation = "eager"
    model = transformers.Qwen3Model(hf_cfg).eval()
    sd = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in w.items()}
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not [m for m in missing if "rotary" not in m], missing
    ids, cu = inl.synthetic.random_texts(3, 5, 33, cfg["vocab_size"], seed=4)
    ours = Q.hidden_states(w, cfg, ids, cu)
    ours = C.rms_norm(ours, w["norm.weight"], cfg["rms_norm_eps"])
    with torch.no_grad():
        for i in range(3):
            s, e = cu[i], cu[i + 1]
            t = torch.from_numpy(ids[s:e].astype(np.int64))[None]
            hf = model(input_ids=t).last_hidden_state[0].numpy()
            assert np.abs(hf - ours[s:e]).max() < 2e-4, np.abs(hf - ours[s:e]).max()


def test_late_head_normalizes_every_token(tiny):
    cfg, w = tiny
    ids, cu = inl.synthetic.random_texts(3, 4, 20, cfg["vocab_size"], seed=5)
    proj = inl.synthetic.late_projection(cfg, out=32)
    out = Q.encode_late(w, cfg, proj, ids, cu)
    assert out.shape == (cu[-1], 32)
    assert np.allclose(np.linalg.norm(out, axis=-1), 1.0, atol=1e-5)


def test_torch_restatement_matches_the_numpy_oracle(tiny):
    """oracle/qwen3_torch.py (the fast CPU checker and the bench's CPU arm) is
    the same function as oracle/qwen3.py: dense last-token vectors and late
    per-token vectors, texts of 1 to 300 tokens, f32 throughout."""
    from oracle import qwen3_torch as QT

    cfg, w = tiny
    ids, cu = inl.synthetic.random_texts(6, 1, 300, cfg["vocab_size"], seed=6)
    m = QT.Qwen3Cpu(w, cfg)
    dense = m.embed_last(ids, cu)
    want = Q.embed_last(w, cfg, ids, cu)
    assert cosine_rows(dense, want).min() > 0.99999
    assert np.abs(dense - want).max() < 1e-5
    proj = inl.synthetic.late_projection(cfg, out=32)
    late = m.encode_late(proj, ids, cu)
    want_late = Q.encode_late(w, cfg, proj, ids, cu)
    assert cosine_rows(late, want_late).min() > 0.99999
