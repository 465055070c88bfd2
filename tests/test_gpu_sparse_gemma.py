"""Model-level parity of the ModernBERT + SPLADE and EmbeddingGemma-style
towers through the C ABI against the CPU oracles (oracle/modernbert.py,
oracle/gemma.py), on the same seeded weights and inputs.

Tolerances. SPLADE f32: weights within 1e-4 and identical active term sets
(weight > 0), the assertion of the reference's golden test. SPLADE bf16:
cosine >= 0.999 of the dense term-weight rows. Dense f32: cosine >= 0.99999; bf16: >= 0.999.
"""
import numpy as np
import pytest

import im_not_llm_b200 as inl
from oracle import gemma as G
from oracle import modernbert as MB
from oracle.common import truncate_and_normalize
from tests.conftest import cosine_rows

pytestmark = pytest.mark.gpu


def _scaled(weights, scale):
    return {k: (v * np.float32(scale) if v.ndim == 2 and "embed" not in k else v) for k, v in weights.items()}


def assert_splade_f32(got, ref, tol=1e-4):
    """Weights within ``tol`` and identical active term sets (weight > 0, the
    SparseVector rule, crates/inl-sparse/src/lib.rs:51-62), as the
    reference's golden test asserts them (modernbert.rs:1014-1057); a flip
    reports its two weights."""
    assert got.shape == ref.shape
    assert np.abs(got - ref).max() <= tol, np.abs(got - ref).max()
    for i in range(len(ref)):
        a, b = got[i] > 0, ref[i] > 0
        flips = np.nonzero(a != b)[0]
        assert len(flips) == 0, (i, [(int(v), float(got[i, v]), float(ref[i, v])) for v in flips[:8]])


@pytest.fixture(scope="module")
def mb_tiny():
    cfg = dict(inl.synthetic.MODERNBERT_TINY)
    w = _scaled(inl.synthetic.modernbert_weights(cfg, seed=0, norm_jitter=0.1), 4.0)
    w["decoder.bias"] = (np.random.default_rng(9).standard_normal(cfg["vocab_size"]) * 0.05).astype(np.float32)
    return cfg, w


def _pooling(cfg):
    return cfg.get("splade", {})


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_sparse_compaction_equals_the_dense_rows(gpu, mb_tiny, dtype):
    """inl_cuda_forward_sparse_compact: per text the ascending term ids with
    weight > 0 and their weights, bit for bit the nonzeros of the dense rows;
    a prefix-only text is an empty vector; a capacity below the batch's term
    count is refused with the size needed in offsets[n]."""
    import ctypes

    from im_not_llm_b200 import _native as N_

    cfg, w = mb_tiny
    ids, cu = inl.synthetic.random_texts(9, 1, 200, cfg["vocab_size"], seed=23)
    ids[cu[3]:cu[4]] = 5  # prefix tokens only
    m = inl.CudaModel(cfg, w, dtype=dtype)
    dense = m.encode_sparse(ids, cu)
    pairs = m.encode_sparse_compact(ids, cu)
    assert len(pairs) == len(dense)
    for row, (idx, val) in zip(dense, pairs):
        nz = np.nonzero(row > 0)[0]
        assert np.array_equal(idx, nz) and np.array_equal(val, row[nz])
    assert len(pairs[3][0]) == 0
    total = sum(len(p[0]) for p in pairs)
    offsets = np.zeros(len(cu), dtype=np.int64)
    small = np.empty(max(total - 1, 1), dtype=np.int32)
    smallv = np.empty(max(total - 1, 1), dtype=np.float32)
    st = N_.lib().inl_cuda_forward_sparse_compact(m.handle, ids.ctypes.data, N_.INL_MEM_HOST, cu.ctypes.data,
                                                  len(cu) - 1, offsets.ctypes.data, small.ctypes.data,
                                                  smallv.ctypes.data, total - 1, N_.INL_MEM_HOST)
    assert st == 4 and offsets[-1] == total and "capacity" in N_.last_error()
    m.close()


def test_modernbert_tiny_f32_matches_oracle(gpu, mb_tiny):
    cfg, w = mb_tiny
    ids, cu = inl.synthetic.random_texts(7, 1, 200, cfg["vocab_size"], seed=21)
    ids[cu[2]] = 5  # a prefix token inside a text
    ids[cu[3]:cu[4]] = 5  # a text made only of prefix tokens pools to zero
    ref = MB.splade(w, cfg, _pooling(cfg), ids, cu)
    m = inl.CudaModel(cfg, w, dtype="f32")
    got = m.encode_sparse(ids, cu)
    m.close()
    assert got.shape[1] == MB.pooling_dimension(_pooling(cfg), cfg["vocab_size"]) == 900
    assert not got[3].any()
    assert_splade_f32(got, ref)


def test_modernbert_tiny_bf16_matches_oracle(gpu, mb_tiny):
    cfg, w = mb_tiny
    ids, cu = inl.synthetic.random_texts(7, 1, 300, cfg["vocab_size"], seed=22)
    ref = MB.splade(w, cfg, _pooling(cfg), ids, cu)
    m = inl.CudaModel(cfg, w, dtype="bf16")
    got = m.encode_sparse(ids, cu)
    m.close()
    assert cosine_rows(got, ref).min() >= 0.999


@pytest.mark.parametrize("dtype,floor", [("f32", 0.99999), ("bf16", 0.999)])
def test_modernbert_tiny_hidden_states(gpu, mb_tiny, dtype, floor):
    cfg, w = mb_tiny
    ids, cu = inl.synthetic.random_texts(5, 10, 150, cfg["vocab_size"], seed=23)
    ref = MB.hidden_states(w, cfg, ids, cu)
    m = inl.CudaModel(cfg, w, dtype=dtype)
    got = m.hidden(ids, cu)
    m.close()
    assert cosine_rows(got, ref).min() >= floor


def test_sparse_engine_returns_sorted_positive_terms(gpu, mb_tiny):
    cfg, w = mb_tiny
    ids, cu = inl.synthetic.random_texts(9, 1, 80, cfg["vocab_size"], seed=24)
    texts = [ids[cu[i]:cu[i + 1]] for i in range(9)]
    enc = inl.SparseEncoder(lambda: inl.CudaModel(cfg, w, dtype="f32"), inl.TextOptions(max_batch_tokens=200))
    out = enc.encode(texts)
    ref = MB.splade(w, cfg, _pooling(cfg), ids, cu)
    for i, sv in enumerate(out):
        assert np.all(np.diff(sv.indices.astype(np.int64)) > 0) and np.all(sv.values > 0)
        assert np.abs(sv.values - ref[i][sv.indices]).max(initial=0) < 1e-4
    assert enc.load().dimension == 900


@pytest.mark.slow
def test_config2_splade_full_size_f32(gpu):
    """Config 2: 22-layer ModernBERT, V = 36282, 32 texts of 16-256 tokens (seed 2), f32."""
    cfg = dict(inl.synthetic.MODERNBERT_SPLADE)
    w = inl.synthetic.modernbert_weights(cfg, seed=0)
    ids, cu = inl.synthetic.cfg2_inputs()
    ref = MB.splade(w, cfg, _pooling(cfg), ids, cu)
    m = inl.CudaModel(cfg, w, dtype="f32")
    got = m.encode_sparse(ids, cu)
    m.close()
    assert_splade_f32(got, ref)


# ------------------------------------------------------------------ Gemma-style
# The reference scores attention UNSCALED over RMS-normed q and k
# (crates/inl-text/src/gemma2.rs:14-16), so with unit q/k norm weights the logits
# have a standard deviation of sqrt(head_dim) and the softmax is nearly one-hot:
# rounding q and k to bf16 then moves whole attention rows. A numpy emulation of
# bf16 storage lands at cosine ~0.98 against the f32 oracle on such weights, so
# the bf16 checks scale the q/k norm weights by QK_NORM (logit spread ~1, as in
# trained checkpoints), where the same emulation reaches 0.99996. At config 4's
# depth (24 layers, head_dim 256) unit weights make the tower chaotic even in
# f32: perturbing every weight by 1e-6 relative moves the f32 oracle's embedding
# to cosine 0.98. So the full-size checks use QK_NORM in both dtypes, and the
# sharp case is covered on the 4-layer tiny tower in f32.
QK_NORM = np.float32(0.3)


def _gemma_weights(cfg, seed=0, scale=1.0, qk=1.0, norm_jitter=0.0):
    w = inl.synthetic.gemma_weights(cfg, seed=seed, norm_jitter=norm_jitter)
    if scale != 1.0:
        w = _scaled(w, scale)
    for k in list(w):
        if qk != 1.0 and ("q_norm" in k or "k_norm" in k):
            w[k] = w[k] * np.float32(qk)
    return w, [w[f"dense_head.{j}.weight"] for j in range(len(cfg["dense_dims"]))]


@pytest.fixture(scope="module")
def gemma_tiny():
    cfg = dict(inl.synthetic.GEMMA_TINY)
    return (cfg,) + _gemma_weights(cfg, scale=3.0, qk=QK_NORM, norm_jitter=0.1)


@pytest.mark.parametrize("dtype,floor", [("f32", 0.99999), ("bf16", 0.999)])
@pytest.mark.parametrize("out_dim", [0, 128])
def test_gemma_tiny_matches_oracle(gpu, gemma_tiny, dtype, floor, out_dim):
    cfg, w, dense = gemma_tiny
    ids, cu = inl.synthetic.random_texts(6, 1, 260, cfg["vocab_size"], seed=31)
    ref = G.embed_dense_head(w, cfg, dense, ids, cu, out_dim=out_dim, prefix="")
    m = inl.CudaModel(cfg, w, dtype=dtype)
    got = m.embed(ids, cu, out_dim=out_dim)
    m.close()
    assert got.shape == ref.shape
    assert cosine_rows(got, ref).min() >= floor
    assert np.allclose(np.linalg.norm(got, axis=1), 1.0, atol=1e-4)


def test_gemma_tiny_sharp_attention_f32(gpu):
    """Unit q/k norm weights: near one-hot unscaled attention, f32 end to end."""
    cfg = dict(inl.synthetic.GEMMA_TINY)
    w, dense = _gemma_weights(cfg, scale=3.0, norm_jitter=0.1)
    ids, cu = inl.synthetic.random_texts(5, 30, 200, cfg["vocab_size"], seed=32)
    ref = G.embed_dense_head(w, cfg, dense, ids, cu, prefix="")
    m = inl.CudaModel(cfg, w, dtype="f32")
    got = m.embed(ids, cu)
    m.close()
    assert cosine_rows(got, ref).min() >= 0.99999


def test_gemma_rejects_missing_per_layer_embeddings_and_bad_dims(gpu, gemma_tiny):
    """A config with per-layer embeddings needs their weights (a load error,
    as the reference's VarBuilder gives); an output dim above the model's is
    a config error."""
    cfg, w, _ = gemma_tiny
    with pytest.raises(inl.InferenceError, match="missing weight"):
        inl.CudaModel(dict(cfg, hidden_size_per_layer_input=16), w, dtype="bf16")
    m = inl.CudaModel(cfg, w, dtype="bf16")
    ids, cu = inl.synthetic.random_texts(2, 3, 9, cfg["vocab_size"], seed=3)
    with pytest.raises(inl.ConfigError):
        m.embed(ids, cu, out_dim=4096)
    m.close()


@pytest.fixture(scope="module")
def config4_case():
    """Config 4 architecture (24 layers, 3q/1kv x 256, window 512 on 5 of 6
    layers, V = 262144, dense 768->3072->768) on the first 12 of its 128
    log-uniform texts (seed 4), with the oracle's embeddings computed once."""
    cfg = dict(inl.synthetic.GEMMA_STYLE)
    w, dense = _gemma_weights(cfg, qk=QK_NORM)
    ids, cu = inl.synthetic.cfg4_inputs()
    ids, cu = ids[: cu[12]], cu[:13]
    return cfg, w, ids, cu, G.embed_dense_head(w, cfg, dense, ids, cu, prefix="")


@pytest.mark.slow
@pytest.mark.parametrize("dtype,floor", [("f32", 0.99999), ("bf16", 0.999)])
def test_config4_gemma_full_size_subset(gpu, config4_case, dtype, floor):
    """Full width and Matryoshka 256 (truncate, then renormalise)."""
    cfg, w, ids, cu, ref = config4_case
    m = inl.CudaModel(cfg, w, dtype=dtype)
    assert cosine_rows(m.embed(ids, cu), ref).min() >= floor
    got = m.embed(ids, cu, out_dim=256)
    m.close()
    assert cosine_rows(got, truncate_and_normalize(ref, 256)).min() >= floor


@pytest.mark.slow
@pytest.mark.parametrize("mode,eps", [("ffma", 1e-6), ("3xbf16", 5e-6)])
def test_config4_unscaled_weights_f32_within_the_oracles_own_f32_spread(gpu, mode, eps):
    """Config 4 with its BASELINE weights as drawn (unit q/k norm weights, no
    scaling) in f32, on its four shortest texts (33 to 43 tokens).

    Unscaled attention over RMS-normed q / k (crates/inl-text/src/gemma2.rs:14-16)
    at this depth is ill-conditioned: perturbing every weight matrix by one
    f32 rounding step (relative 1e-7) already moves the f32 oracle's own
    embeddings to cosine ~0.9994, below the 0.99999 floor. A GPU evaluation
    rounds differently, so the check is the oracle's own spread under
    perturbations of the size of the GPU's arithmetic error: the GPU's
    deviation 1 - cosine is at most the largest deviation of three oracle runs
    with every weight matrix perturbed by relative noise eps. For the SIMT
    FFMA GEMMs eps = 1e-6, the typical difference between two summation orders
    of a dot product of K ~ 10^3 terms (sqrt(K) u, u = 2^-24); for the 3xBF16
    tensor-core GEMMs eps = 5e-6, the size of their operand splitting error
    (|x - hi - lo| <= 2^-17 |x|). Measured on a B200 (FFMA): deviations 6e-4 to
    3.1e-3 against spreads of 2.2e-3 to 7.7e-3."""
    cfg = dict(inl.synthetic.GEMMA_STYLE)
    w, dense = _gemma_weights(cfg)
    ids, cu = inl.synthetic.cfg4_inputs()
    L = np.diff(cu)
    pick = np.argsort(L, kind="stable")[:4]
    rows = [ids[cu[i]:cu[i + 1]] for i in pick]
    pid = np.concatenate(rows).astype(np.uint32)
    pcu = np.concatenate([[0], np.cumsum([len(r) for r in rows])]).astype(np.int32)
    ref = G.embed_dense_head(w, cfg, dense, pid, pcu, prefix="")
    spread = np.zeros(len(rows))
    rng = np.random.default_rng(9)
    for _ in range(3):
        wp = {k: (v * (1 + eps * rng.standard_normal(v.shape))).astype(np.float32) if v.ndim == 2 else v
              for k, v in w.items()}
        dp = [wp[f"dense_head.{j}.weight"] for j in range(len(cfg["dense_dims"]))]
        spread = np.maximum(spread, 1 - cosine_rows(G.embed_dense_head(wp, cfg, dp, pid, pcu, prefix=""), ref))
    m = inl.CudaModel(cfg, w, dtype="f32")
    m.set_f32_gemm(mode)
    got = m.embed(pid, pcu)
    m.close()
    dev = 1 - cosine_rows(got, ref)
    assert (dev <= np.maximum(spread, 1e-5)).all(), {"gpu_deviation": dev.tolist(), "oracle_spread": spread.tolist()}


@pytest.mark.slow
def test_config2_splade_f32_both_gemm_modes_agree(gpu):
    """Config 2 in f32 through the SIMT FFMA GEMMs and through the 3xBF16
    tensor-core GEMMs: identical active term sets and weights within 1e-4
    of each other (each is also held to the oracle by
    test_config2_splade_full_size_f32 in the default mode)."""
    cfg = dict(inl.synthetic.MODERNBERT_SPLADE)
    w = inl.synthetic.modernbert_weights(cfg, seed=0)
    ids, cu = inl.synthetic.cfg2_inputs()
    m = inl.CudaModel(cfg, w, dtype="f32")
    split = m.encode_sparse(ids, cu)
    m.set_f32_gemm("ffma")
    ffma = m.encode_sparse(ids, cu)
    m.close()
    assert_splade_f32(split, ffma)
