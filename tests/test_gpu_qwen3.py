"""Model-level parity of the Qwen3 tower through the C ABI against the CPU
oracle (oracle/qwen3.py), on the same seeded weights and inputs.

Tolerances: f32 cosine >= 0.99999 per vector;
bf16 cosine >= 0.999 per vector; late-interaction bf16 per-token cosine >= 0.999.
"""
import numpy as np
import pytest

import im_not_llm_b200 as inl
from oracle import qwen3 as Q
from tests.conftest import cosine_rows

pytestmark = pytest.mark.gpu

F32_COS = 0.99999
BF16_COS = 0.999


def _tiny(cfg, scale=5.0):
    w = inl.synthetic.qwen3_weights(cfg, seed=0, norm_jitter=0.1)
    for k, v in w.items():
        if v.ndim == 2 and not k.startswith("embed"):
            w[k] = v * np.float32(scale)
    return w


@pytest.fixture(scope="module")
def tiny_pair():
    cfg = dict(inl.synthetic.QWEN3_TINY)
    return cfg, _tiny(cfg)


@pytest.mark.parametrize("dtype,floor", [("f32", F32_COS), ("bf16", BF16_COS)])
@pytest.mark.parametrize("cfg_name", ["QWEN3_TINY", "QWEN3_TINY_D64"])
def test_tiny_dense_matches_oracle(gpu, dtype, floor, cfg_name):
    cfg = dict(getattr(inl.synthetic, cfg_name))
    w = _tiny(cfg)
    ids, cu = inl.synthetic.random_texts(9, 1, 300, cfg["vocab_size"], seed=11)
    ref = Q.embed_last(w, cfg, ids, cu)
    m = inl.CudaModel(cfg, w, dtype=dtype)
    got = m.embed(ids, cu)
    m.close()
    cos = cosine_rows(got, ref)
    assert cos.min() >= floor, cos
    assert np.allclose(np.linalg.norm(got, axis=-1), 1.0, atol=1e-4)


@pytest.mark.parametrize("dtype,floor", [("f32", F32_COS), ("bf16", BF16_COS)])
def test_tiny_hidden_states_match_oracle(gpu, tiny_pair, dtype, floor):
    cfg, w = tiny_pair
    ids, cu = inl.synthetic.random_texts(4, 50, 200, cfg["vocab_size"], seed=12)
    from oracle import common as C

    ref = C.rms_norm(Q.hidden_states(w, cfg, ids, cu), w["norm.weight"], cfg["rms_norm_eps"])
    m = inl.CudaModel(cfg, w, dtype=dtype)
    got = m.hidden(ids, cu)
    m.close()
    assert cosine_rows(got, ref).min() >= floor


@pytest.mark.parametrize("dtype,floor", [("f32", F32_COS), ("bf16", BF16_COS)])
def test_tiny_late_matches_oracle(gpu, tiny_pair, dtype, floor):
    cfg = dict(tiny_pair[0], is_causal=False)
    w = tiny_pair[1]
    proj = inl.synthetic.late_projection(cfg, out=128)
    ids, cu = inl.synthetic.random_texts(5, 20, 150, cfg["vocab_size"], seed=13)
    ref = Q.encode_late(w, cfg, proj, ids, cu)
    m = inl.CudaModel(cfg, w, dtype=dtype)
    m.set_dense_head(proj)
    got = m.encode_multivector(ids, cu)
    m.close()
    cos = cosine_rows(got, ref)
    assert cos.min() >= floor, cos.min()
    assert np.allclose(np.linalg.norm(got, axis=-1), 1.0, atol=1e-4)


def test_packing_order_does_not_change_embeddings(gpu, tiny_pair):
    cfg, w = tiny_pair
    ids, cu = inl.synthetic.random_texts(12, 1, 400, cfg["vocab_size"], seed=14)
    m = inl.CudaModel(cfg, w, dtype="bf16")
    batched = m.embed(ids, cu)
    for i in (0, 5, 11):
        alone = m.embed(ids[cu[i]:cu[i + 1]], np.array([0, cu[i + 1] - cu[i]]))
        assert cosine_rows(alone, batched[i:i + 1])[0] > 0.99999
    m.close()


def test_engine_returns_input_order(gpu, tiny_pair):
    cfg, w = tiny_pair
    ids, cu = inl.synthetic.random_texts(40, 1, 120, cfg["vocab_size"], seed=15)
    texts = [ids[cu[i]:cu[i + 1]] for i in range(40)]
    emb = inl.TextEmbedder(lambda: inl.CudaModel(cfg, w, dtype="bf16"),
                           inl.TextOptions(max_batch_tokens=700, batch_size=9))
    out = emb.embed(texts)
    ref = Q.embed_last(w, cfg, ids, cu)
    assert cosine_rows(np.stack(out), ref).min() >= BF16_COS
    assert emb.unload() and not emb.is_loaded()


def test_invalid_inputs_are_rejected(gpu, tiny_pair):
    cfg, w = tiny_pair
    m = inl.CudaModel(cfg, w, dtype="bf16")
    with pytest.raises(inl.InvalidInputError):
        m.embed(np.array([1, 2, cfg["vocab_size"]], dtype=np.uint32), np.array([0, 3]))
    with pytest.raises(inl.InvalidInputError):
        m.embed(np.array([1, 2, 3], dtype=np.uint32), np.array([0, 2, 1, 3]))
    with pytest.raises(inl.InvalidInputError):
        long = np.zeros(cfg["max_position_embeddings"] + 1, dtype=np.uint32)
        m.embed(long, np.array([0, len(long)]))
    # the model stays usable after rejected calls
    ids, cu = inl.synthetic.random_texts(3, 5, 9, cfg["vocab_size"], seed=16)
    assert np.isfinite(m.embed(ids, cu)).all()
    assert m.embed(np.zeros(0, dtype=np.uint32), np.array([0])).shape == (0, cfg["hidden_size"])
    m.close()


@pytest.fixture(scope="module")
def qwen3_full():
    cfg = dict(inl.synthetic.QWEN3_0_6B)
    return cfg, inl.synthetic.qwen3_weights(cfg, seed=0)


@pytest.mark.slow
@pytest.mark.parametrize("dtype,floor", [("f32", F32_COS), ("bf16", BF16_COS)])
def test_config1_full_size(gpu, qwen3_full, dtype, floor):
    """Config 1 (8 x 128 ids, seed 1) on the full Qwen3-0.6B architecture."""
    cfg, w = qwen3_full
    ids, cu = inl.synthetic.cfg1_inputs()
    ref = Q.embed_last(w, cfg, ids, cu)
    m = inl.CudaModel(cfg, w, dtype=dtype)
    got = m.embed(ids, cu)
    m.close()
    cos = cosine_rows(got, ref)
    assert cos.min() >= floor, cos


@pytest.mark.slow
def test_config3_late_full_size_subset(gpu, qwen3_full):
    """Config 3 tower + head (bidirectional, 1024->128, per-token L2) on the first
    8 of its 64 x 512 texts (the oracle's cost bound); bf16 per-token cosine."""
    cfg, w = qwen3_full
    cfg = dict(cfg, is_causal=False)
    ids, cu = inl.synthetic.cfg3_inputs()
    ids, cu = ids[: cu[8]], cu[:9]
    proj = inl.synthetic.late_projection(cfg)
    ref = Q.encode_late(w, cfg, proj, ids, cu)
    m = inl.CudaModel(cfg, w, dtype="bf16")
    m.set_dense_head(proj)
    got = m.encode_multivector(ids, cu)
    m.close()
    cos = cosine_rows(got, ref)
    assert cos.min() >= BF16_COS, cos.min()


@pytest.mark.slow
def test_config5_batch_properties(gpu, qwen3_full):
    """A full ~64k-token packed batch of the config-5 corpus: finite unit
    vectors, short texts match the oracle computed alone, and embedding a text
    alone equals embedding it inside the packed batch."""
    cfg, w = qwen3_full
    lengths, ids = inl.synthetic.cfg5_corpus(n_texts=2048)
    order = inl.planner.longest_first(lengths)
    texts_all = np.split(ids, np.cumsum(lengths)[:-1])
    batch = [order[k] for k in inl.planner.plan_packed([lengths[i] for i in order], 65536)[0]]
    pids, pcu = inl.planner.pack(texts_all, batch)
    m = inl.CudaModel(cfg, w, dtype="bf16")
    got = m.embed(pids, pcu)
    assert np.isfinite(got).all()
    assert np.allclose(np.linalg.norm(got, axis=-1), 1.0, atol=1e-4)
    # the shortest texts of the batch against the oracle, and alone vs packed
    short = np.argsort(np.diff(pcu))[:3]
    for j in short:
        t = pids[pcu[j]:pcu[j + 1]]
        ref = Q.embed_last(w, cfg, t, np.array([0, len(t)]))
        alone = m.embed(t, np.array([0, len(t)]))
        assert cosine_rows(got[j:j + 1], ref)[0] >= BF16_COS
        assert cosine_rows(got[j:j + 1], alone)[0] > 0.99999
    m.close()
