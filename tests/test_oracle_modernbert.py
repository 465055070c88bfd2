"""Pins the ModernBERT + SPLADE oracle (oracle/modernbert.py) against the
reference's own golden fixture tiny_splade (copied by tests/golden/make_golden.py):
the same assertion as crates/inl-sparse/src/modernbert.rs:1014-1057 — identical
active term sets and |dw| <= 1e-4, for every case batched and alone — plus the
reference's pooling-formula and LayerNorm textbook tests restated."""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import common as C
from oracle import modernbert as MB

GOLDEN = Path(__file__).resolve().parent / "golden" / "tiny_splade"


def load_tiny_splade():
    from safetensors.numpy import load_file

    cfg = json.loads((GOLDEN / "config.json").read_text())
    pooling = json.loads((GOLDEN / "1_ShiftedTopKSpladePooling" / "config.json").read_text())
    weights = load_file(str(GOLDEN / "model.safetensors"))
    golden = json.loads((GOLDEN / "golden.json").read_text())
    return cfg, pooling, weights, golden


def _pack(rows):
    ids = np.concatenate([np.asarray(r, dtype=np.uint32) for r in rows])
    cu = np.concatenate([[0], np.cumsum([len(r) for r in rows])]).astype(np.int32)
    return ids, cu


def assert_matches(dense_row, want, tol, label):
    idx, vals = MB.sparse(dense_row)
    assert idx == want["indices"], f"{label}: active terms differ"
    assert np.max(np.abs(np.array(vals) - np.array(want["values"])), initial=0) <= tol, label


def test_tiny_splade_golden_batched_and_alone():
    cfg, pooling, weights, golden = load_tiny_splade()
    assert MB.pooling_dimension(pooling, cfg["vocab_size"]) == golden["dim"]
    for case in golden["cases"]:
        label = f'{case["kind"]}/{case["max_length"]}'
        ids, cu = _pack([r["ids"] for r in case["batched"]])
        got = MB.splade(weights, cfg, pooling, ids, cu)
        for i, want in enumerate(case["batched"]):
            assert_matches(got[i], want, 1e-4, f"{label} batched[{i}]")
        for i, want in enumerate(case["alone"]):
            ids, cu = _pack([want["ids"]])
            got = MB.splade(weights, cfg, pooling, ids, cu)
            assert_matches(got[0], want, 1e-4, f"{label} alone[{i}]")


def test_pooling_blocks_do_not_change_the_result():
    # crates/inl-sparse/src/modernbert.rs:1339-1393: block sizes 1/2/3/7/large
    cfg, pooling, weights, golden = load_tiny_splade()
    rows = [r["ids"] for r in golden["cases"][0]["batched"]]
    ids, cu = _pack(rows)
    ref = MB.splade(weights, cfg, pooling, ids, cu, block=10000)
    for block in (1, 2, 3, 7):
        assert np.abs(MB.splade(weights, cfg, pooling, ids, cu, block=block) - ref).max() < 1e-5


def test_splade_formula_on_random_logits():
    # crates/inl-sparse/src/modernbert.rs:1298-1337: max, bias, shift, relu, log1p, mask, fold
    rng = np.random.default_rng(0)
    logits = rng.standard_normal((7, 12)).astype(np.float32)
    bias = rng.standard_normal(12).astype(np.float32) * 0.1
    shift, masked = 0.3, [2, 5]
    m = logits.max(0) + bias - shift
    w = np.log(1 + np.maximum(m, 0))
    w[masked] = 0
    canon = [0, 1, 2, 3, 4, 5, 0, 1, 2, 3, 4, 5]
    folded = np.zeros(6, dtype=np.float32)
    for v, t in enumerate(canon):
        folded[t] = max(folded[t], w[v])
    # the same formula as oracle.splade's finish/fold steps
    open_ = np.ones(12, dtype=np.float32)
    open_[masked] = 0
    w2 = np.log(np.float32(1) + np.maximum(logits.max(0) + bias - np.float32(shift), 0) * open_)
    f2 = np.zeros(6, dtype=np.float32)
    for v, t in enumerate(canon):
        f2[t] = max(f2[t], w2[v])
    assert np.abs(f2 - folded).max() < 1e-6


def test_layer_norm_textbook():
    # crates/inl-sparse/src/modernbert.rs:1551-1584
    rng = np.random.default_rng(1)
    x = rng.standard_normal((5, 32)).astype(np.float32) * 3 + 1
    w = rng.standard_normal(32).astype(np.float32)
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    assert np.abs(C.layer_norm(x, w, None, 1e-5) - (x - mu) / np.sqrt(var + 1e-5) * w).max() < 1e-4


def test_sliding_window_changes_long_inputs_only():
    # crates/inl-sparse/src/modernbert.rs:1060-1098: a window narrower than the text matters
    cfg, pooling, weights, golden = load_tiny_splade()
    long_ids = golden["cases"][0]["alone"][1]["ids"]
    assert len(long_ids) > cfg["local_attention"]
    ids, cu = _pack([long_ids])
    base = MB.splade(weights, cfg, pooling, ids, cu)
    wide = MB.splade(weights, dict(cfg, local_attention=4096), pooling, ids, cu)
    assert np.abs(base - wide).max() > 1e-4
