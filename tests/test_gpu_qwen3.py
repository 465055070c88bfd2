"""Model-level parity of the Qwen3 tower through the C ABI against the CPU
oracle (oracle/qwen3.py, and its torch-CPU restatement oracle/qwen3_torch.py
for the full-size cases), on the same seeded weights and inputs.

Tolerances: f32 cosine >= 0.99999 per vector;
bf16 cosine >= 0.999 per vector; late-interaction per-token cosine >= 0.9999
in f32 and >= 0.999 in bf16.
"""
import numpy as np
import pytest

import im_not_llm_b200 as inl
from oracle import qwen3 as Q
from tests.conftest import cosine_rows

pytestmark = pytest.mark.gpu

F32_COS = 0.99999
BF16_COS = 0.999
LATE_F32_COS = 0.9999


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


@pytest.fixture(scope="module")
def qwen3_cpu(qwen3_full):
    from oracle import qwen3_torch as QT

    cfg, w = qwen3_full
    return QT.Qwen3Cpu(w, cfg)


@pytest.mark.slow
def test_config3_late_full_size_all_texts_bf16(gpu, qwen3_full, qwen3_cpu):
    """Config 3 tower + head (bidirectional, 1024->128, per-token L2) on all
    64 of its 512-token texts in one packed forward (32768 token vectors);
    bf16 per-token cosine."""
    cfg, w = qwen3_full
    cfg = dict(cfg, is_causal=False)
    ids, cu = inl.synthetic.cfg3_inputs()
    proj = inl.synthetic.late_projection(cfg)
    ref = qwen3_cpu.encode_late(proj, ids, cu)
    m = inl.CudaModel(cfg, w, dtype="bf16")
    m.set_dense_head(proj)
    got = m.encode_multivector(ids, cu)
    m.close()
    assert got.shape == ref.shape == (64 * 512, 128)
    cos = cosine_rows(got, ref)
    assert cos.min() >= BF16_COS, cos.min()


@pytest.mark.slow
def test_config3_late_full_size_f32(gpu, qwen3_full, qwen3_cpu):
    """Config 3 in f32 at the full architecture on 8 of its texts: every
    token vector at the late-interaction f32 floor (cosine >= 0.9999)."""
    cfg, w = qwen3_full
    cfg = dict(cfg, is_causal=False)
    ids, cu = inl.synthetic.cfg3_inputs()
    ids, cu = ids[: cu[8]], cu[:9]
    proj = inl.synthetic.late_projection(cfg)
    ref = qwen3_cpu.encode_late(proj, ids, cu)
    m = inl.CudaModel(cfg, w, dtype="f32")
    m.set_dense_head(proj)
    got = m.encode_multivector(ids, cu)
    m.close()
    cos = cosine_rows(got, ref)
    assert cos.min() >= LATE_F32_COS, cos.min()


def _cfg5_mixed_batch(budget=65536):
    """A ~64k-token packed batch of config-5 texts whose lengths span the
    corpus: its longest text (2048, the clip), the rest drawn in corpus order
    (lognormal, median 256) until the budget is full."""
    lengths, ids = inl.synthetic.cfg5_corpus(n_texts=16384)  # holds three texts at the 2048 clip
    texts = np.split(ids, np.cumsum(lengths)[:-1])
    first = int(np.argmax(lengths))
    batch, total = [first], int(lengths[first])
    for i in range(len(lengths)):
        if i != first and total + int(lengths[i]) <= budget:
            batch.append(i)
            total += int(lengths[i])
    return inl.planner.pack(texts, batch)


@pytest.mark.slow
def test_config5_packed_batch_across_lengths(gpu, qwen3_full, qwen3_cpu):
    """A full ~64k-token packed batch of the config-5 corpus in bf16: finite
    unit vectors; the longest text (2048 tokens: multi-tile causal attention
    and the far rows of the RoPE table), two texts at the median length and
    the shortest text against the oracle; and the longest and shortest
    embedded alone equal to their vectors in the packed batch."""
    cfg, w = qwen3_full
    pids, pcu = _cfg5_mixed_batch()
    L = np.diff(pcu)
    assert L.max() == 2048 and pcu[-1] > 60000
    m = inl.CudaModel(cfg, w, dtype="bf16")
    got = m.embed(pids, pcu)
    assert np.isfinite(got).all()
    assert np.allclose(np.linalg.norm(got, axis=-1), 1.0, atol=1e-4)
    order = np.argsort(L, kind="stable")
    median = order[len(order) // 2: len(order) // 2 + 2]
    picks = [int(np.argmax(L)), int(median[0]), int(median[1]), int(order[0])]
    rows = [pids[pcu[j]:pcu[j + 1]] for j in picks]
    sub_cu = np.concatenate([[0], np.cumsum([len(r) for r in rows])]).astype(np.int32)
    ref = qwen3_cpu.embed_last(np.concatenate(rows), sub_cu)
    cos = cosine_rows(got[picks], ref)
    assert cos.min() >= BF16_COS, dict(zip([int(L[j]) for j in picks], cos))
    for j in (picks[0], picks[-1]):
        t = pids[pcu[j]:pcu[j + 1]]
        alone = m.embed(t, np.array([0, len(t)]))
        assert cosine_rows(got[j:j + 1], alone)[0] > 0.99999
    m.close()


@pytest.mark.slow
def test_config5_longest_texts_f32(gpu, qwen3_full, qwen3_cpu):
    """The same long and median texts through the f32 tower: the f32 floor
    (cosine >= 0.99999) at 2048 tokens."""
    cfg, w = qwen3_full
    pids, pcu = _cfg5_mixed_batch()
    L = np.diff(pcu)
    order = np.argsort(L, kind="stable")
    picks = [int(np.argmax(L)), int(order[len(order) // 2]), int(order[0])]
    rows = [pids[pcu[j]:pcu[j + 1]] for j in picks]
    sub_cu = np.concatenate([[0], np.cumsum([len(r) for r in rows])]).astype(np.int32)
    sub_ids = np.concatenate(rows)
    ref = qwen3_cpu.embed_last(sub_ids, sub_cu)
    m = inl.CudaModel(cfg, w, dtype="f32")
    got = m.embed(sub_ids, sub_cu)
    m.close()
    cos = cosine_rows(got, ref)
    assert cos.min() >= F32_COS, cos


@pytest.mark.parametrize("cfg_name", ["QWEN3_TINY", "QWEN3_TINY_D64"])
def test_pruned_last_layer_equals_the_full_layer(gpu, cfg_name):
    """Causal last-token pooling prunes the last layer to the rows the pooled
    vector reads (the query tile of each text's last row for attention, the
    last rows for o / gate-up / down). The embeddings equal those of the
    unpruned layer: every row's arithmetic is the same, only other rows are
    skipped."""
    cfg = dict(getattr(inl.synthetic, cfg_name))
    w = _tiny(cfg)
    ids, cu = inl.synthetic.random_texts(37, 1, 700, cfg["vocab_size"], seed=17)
    m = inl.CudaModel(cfg, w, dtype="bf16")
    pruned = m.embed(ids, cu)
    m.set_prune_last(False)
    full = m.embed(ids, cu)
    m.set_prune_last(True)
    again = m.embed(ids, cu)
    m.close()
    assert np.abs(pruned - full).max() < 1e-6, np.abs(pruned - full).max()
    assert np.array_equal(pruned, again)
    assert cosine_rows(pruned, Q.embed_last(w, cfg, ids, cu)).min() >= BF16_COS


@pytest.mark.slow
def test_pruned_last_layer_full_size_batch(gpu, qwen3_full):
    """The same on a full ~64k-token config-5 batch (about 200 last rows: the
    pruned projections run on partial M tiles)."""
    cfg, w = qwen3_full
    pids, pcu = _cfg5_mixed_batch()
    m = inl.CudaModel(cfg, w, dtype="bf16")
    pruned = m.embed(pids, pcu)
    m.set_prune_last(False)
    full = m.embed(pids, pcu)
    m.close()
    assert cosine_rows(pruned, full).min() > 0.999999
    assert np.abs(pruned - full).max() < 1e-5, np.abs(pruned - full).max()
