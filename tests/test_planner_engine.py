"""Host logic: batch planners (restating the reference's planner tests,
crates/inl-text/src/native.rs:911-1108 and the sparse/late planners), the
packed planner and LPT assignment, the BatchDeadline semantics
(crates/inl-core/src/deadline.rs:71-130) and the engine facade contract
(crates/inl-text/src/native.rs:1368-1547) on a fake model (no GPU)."""
import threading
import time

import numpy as np
import pytest

import im_not_llm_b200 as inl
from im_not_llm_b200 import planner as P


def test_longest_first_is_stable():
    assert P.longest_first([3, 5, 3, 9, 5]) == [3, 1, 4, 0, 2]


def test_plan_batches_contiguous_cover_and_caps():
    lengths = [10, 9, 9, 8, 3, 3, 2, 1, 1]
    b = P.plan_batches(lengths, batch_size=3, max_batch_tokens=20)
    flat = [i for r in b for i in r]
    assert flat == list(range(len(lengths)))
    for r in b:
        assert len(r) <= 3
        if len(r) > 1:
            assert len(r) * max(lengths[i] for i in r) <= 20


def test_single_oversized_input_forms_its_own_batch():
    assert P.plan_batches([50, 1], batch_size=8, max_batch_tokens=10) == [range(0, 1), range(1, 2)]
    assert P.plan_packed([50, 1], 10) == [range(0, 1), range(1, 2)]


def test_empty_input_plans_no_batches():
    assert P.plan_batches([], 4, 10) == []
    assert P.plan_packed([], 10) == []
    assert P.plan_dense_batches([], 4, 10, 1, 1, 10) == []


def test_dense_planner_pads_to_longest_member():
    # crates/inl-text/src/native.rs:1034-1051: budget checked against the padded longest member
    b = P.plan_dense_batches([100, 1, 1, 1], batch_size=64, max_length=2048, per_row_bytes=64,
                             budget_bytes=1 << 30, max_batch_tokens=300, slack=8)
    assert b == [range(0, 2), range(2, 4)]


def test_plan_packed_counts_real_tokens():
    lengths = [1000, 600, 500, 300, 100, 50]
    b = P.plan_packed(lengths, 1100)
    assert [list(r) for r in b] == [[0], [1, 2], [3, 4, 5]]
    for r in b:
        assert sum(lengths[i] for i in r) <= 1100 or len(r) == 1


def test_lpt_balances_and_covers():
    costs = [10, 9, 8, 7, 6, 5, 4, 3, 2, 1]
    plan = P.assign_lpt(costs, 3)
    assert sorted(i for w in plan for i in w) == list(range(10))
    loads = [sum(costs[i] for i in w) for w in plan]
    assert max(loads) - min(loads) <= max(costs)


def test_pack_roundtrip():
    texts = [np.arange(n, dtype=np.uint32) + 10 * n for n in (3, 0, 5)]
    ids, cu = P.pack(texts, [2, 0, 1])
    assert cu.tolist() == [0, 5, 8, 8]
    assert ids[:5].tolist() == texts[2].tolist() and ids[5:8].tolist() == texts[0].tolist()


def test_cfg5_corpus_shape_and_determinism():
    lengths, ids = inl.synthetic.cfg5_corpus(n_texts=4096)
    assert lengths.min() >= 8 and lengths.max() <= 2048
    assert 200 < np.median(lengths) < 320
    assert len(ids) == lengths.sum() and ids.max() < inl.synthetic.QWEN3_0_6B["vocab_size"]
    l2, i2 = inl.synthetic.cfg5_corpus(n_texts=4096)
    assert np.array_equal(lengths, l2) and np.array_equal(ids, i2)


def test_weights_are_seeded_and_named_like_the_checkpoint():
    cfg = inl.synthetic.QWEN3_TINY
    a = inl.synthetic.qwen3_weights(cfg, seed=0)
    b = inl.synthetic.qwen3_weights(cfg, seed=0)
    assert a.keys() == b.keys() and all(np.array_equal(a[k], b[k]) for k in a)
    assert "layers.1.self_attn.q_norm.weight" in a and a["norm.weight"].tolist() == [1.0] * cfg["hidden_size"]
    assert abs(float(a["layers.0.mlp.up_proj.weight"].std()) - 0.02) < 1e-3


# ------------------------------------------------------------------ deadline
def test_stuck_batch_returns_timeout_within_deadline_and_wedges():
    d = inl.BatchDeadline()
    ran = []
    t0 = time.time()
    with pytest.raises(inl.TimeoutError_):
        d.run("batch", 0.2, lambda: time.sleep(3))
    assert time.time() - t0 < 0.4
    with pytest.raises(inl.TimeoutError_):
        d.run("batch", 5, lambda: ran.append(1))
    assert not ran  # later calls fail fast without running


def test_healthy_batches_return_values_and_errors_propagate():
    d = inl.BatchDeadline()
    assert d.run("x", 1, lambda: 42) == 42
    with pytest.raises(inl.InferenceError):
        d.run("x", 1, lambda: 1 / 0)
    with pytest.raises(inl.InvalidInputError):
        d.run("x", 1, lambda: (_ for _ in ()).throw(inl.InvalidInputError("bad")))
    assert not d.wedged


# ------------------------------------------------------------------ facade
class FakeModel:
    """Stands in for CudaModel: embeds a text as [len, first id, 0...]."""

    def __init__(self, delay=0.0, drop=False):
        self.delay = delay
        self.drop = drop
        self.dtype = "bf16"
        self.device = 0
        self.calls = 0
        self.closed = False

    def info(self):
        return {"dense_dim": 4, "arch": 0, "multivector_dim": 2, "is_causal": 1}

    def embed(self, ids, cu, out_dim=0):
        self.calls += 1
        time.sleep(self.delay)
        n = len(cu) - 1 - (1 if self.drop else 0)
        out = np.zeros((n, 4), dtype=np.float32)
        for i in range(n):
            out[i, 0] = cu[i + 1] - cu[i]
            out[i, 1] = ids[cu[i]] if cu[i + 1] > cu[i] else -1
        return out

    def close(self):
        self.closed = True


def _texts(n, seed=0):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, 100, size=int(rng.integers(1, 30))).astype(np.uint32) for _ in range(n)]


def test_embedder_returns_vectors_in_input_order():
    texts = _texts(50)
    e = inl.TextEmbedder(lambda: FakeModel(), inl.TextOptions(max_batch_tokens=64, batch_size=7))
    out = e.embed(texts)
    for t, v in zip(texts, out):
        assert v[0] == len(t) and v[1] == t[0]
    assert e.embed([]) == []


def test_truncation_to_max_length():
    e = inl.TextEmbedder(lambda: FakeModel(), inl.TextOptions(max_length=5))
    out = e.embed([np.arange(20, dtype=np.uint32)])
    assert out[0][0] == 5


def test_vector_count_mismatch_is_an_inference_error():
    e = inl.TextEmbedder(lambda: FakeModel(drop=True), inl.TextOptions())
    with pytest.raises(inl.InferenceError):
        e.embed(_texts(3))


def test_stuck_forward_times_out_and_later_calls_fail_fast():
    model = FakeModel(delay=2.0)
    e = inl.TextEmbedder(lambda: model, inl.TextOptions(per_batch_timeout_seconds=0.2))
    with pytest.raises(inl.TimeoutError_):
        e.embed(_texts(2))
    calls = model.calls
    with pytest.raises(inl.TimeoutError_):
        e.embed(_texts(2))
    assert model.calls == calls


def test_waiting_for_the_gate_does_not_count_against_the_deadline():
    model = FakeModel(delay=0.3)
    e = inl.TextEmbedder(lambda: model, inl.TextOptions(per_batch_timeout_seconds=0.5))
    errs = []

    def call():
        try:
            e.embed(_texts(1))
        except Exception as x:  # pragma: no cover - failure path
            errs.append(x)

    ts = [threading.Thread(target=call) for _ in range(3)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errs and model.calls == 3


def test_zero_timeout_and_output_dim_are_validated():
    with pytest.raises(inl.ConfigError):
        inl.TextEmbedder(lambda: FakeModel(), inl.TextOptions(timeout_seconds=0)).embed(_texts(1))
    with pytest.raises(inl.ConfigError):  # output_dim refused for Qwen3
        inl.TextEmbedder(lambda: FakeModel(), inl.TextOptions(output_dim=128)).embed(_texts(1))


def test_unload_releases_and_next_call_reloads():
    made = []

    def loader():
        made.append(FakeModel())
        return made[-1]

    e = inl.TextEmbedder(loader, inl.TextOptions())
    e.embed(_texts(2))
    assert e.is_loaded() and e.unload() and made[0].closed and not e.is_loaded()
    assert not e.unload()
    e.embed(_texts(2))
    assert len(made) == 2


def test_failed_load_is_not_cached():
    state = {"n": 0}

    def loader():
        state["n"] += 1
        if state["n"] == 1:
            raise inl.InferenceError("boom")
        return FakeModel()

    e = inl.TextEmbedder(loader, inl.TextOptions())
    with pytest.raises(inl.InferenceError):
        e.embed(_texts(1))
    assert len(e.embed(_texts(1))) == 1


def test_data_parallel_embedder_gathers_by_index():
    models = [FakeModel(), FakeModel(), FakeModel()]
    dp = inl.DataParallelEmbedder(models, max_batch_tokens=40)
    texts = _texts(60, seed=3)
    out = dp.embed(texts)
    for t, v in zip(texts, out):
        assert v[0] == len(t) and v[1] == t[0]
    assert all(m.calls > 0 for m in models)


def test_sparse_vector_contract():
    """crates/inl-sparse/src/lib.rs:258-318 restated: new validates, from_pairs
    sorts / merges by max / drops unusable weights, dot sums shared terms, the
    JSON form round-trips and re-validates."""
    SV = inl.SparseVector
    v = SV.new([1, 4, 9], [0.5, 2.0, 0.25])
    assert v.indices.tolist() == [1, 4, 9] and v.values.tolist() == [0.5, 2.0, 0.25]
    assert len(v) == 3 and not v.is_empty()
    for idx, val in [([1, 2], [1.0]), ([2, 1], [1.0, 1.0]), ([1, 1], [1.0, 1.0]), ([1], [0.0]), ([1], [-0.5]),
                     ([1], [float("nan")]), ([1], [float("inf")])]:
        with pytest.raises(inl.InferenceError):
            SV.new(idx, val)
    p = SV.from_pairs([(7, 1.0), (3, 0.5), (7, 2.5), (5, 0.0), (6, -1.0), (8, float("nan"))])
    assert p.indices.tolist() == [3, 7] and p.values.tolist() == [0.5, 2.5]
    left, right = SV.new([1, 3, 5], [2.0, 1.0, 4.0]), SV.new([3, 4, 5], [10.0, 7.0, 0.5])
    assert left.dot(right) == 1.0 * 10.0 + 4.0 * 0.5 == right.dot(left)
    assert left.dot(SV.from_pairs([])) == 0.0
    w = SV.new([2, 9], [1.5, 0.5])
    assert SV.from_json(w.to_json()) == w
    with pytest.raises(inl.InferenceError):
        SV.from_json('{"indices":[2,1],"values":[1.0,1.0]}')


class _EchoReplica:
    """A GPU replica stand-in: sparse row = one-hot of (length % 4), late
    vectors = (token id, position); optional NaN output."""

    def __init__(self, nan=False):
        self.calls, self.nan = 0, nan

    def info(self):
        return {"is_causal": 0}

    def encode_sparse(self, ids, cu):
        self.calls += 1
        out = np.zeros((len(cu) - 1, 4), dtype=np.float32)
        for i in range(len(cu) - 1):
            out[i, (cu[i + 1] - cu[i]) % 4] = np.nan if self.nan else 1.0 + i * 0
        return out

    def encode_sparse_compact(self, ids, cu):
        dense = self.encode_sparse(ids, cu)
        if not np.all(np.isfinite(dense)):
            raise inl.InferenceError("non-finite SPLADE term weight")
        return [(np.nonzero(r > 0)[0].astype(np.uint32), r[r > 0]) for r in dense]

    def encode_multivector(self, ids, cu):
        self.calls += 1
        out = np.zeros((len(ids), 2), dtype=np.float32)
        out[:, 0] = ids
        for i in range(len(cu) - 1):
            out[cu[i]:cu[i + 1], 1] = np.arange(cu[i + 1] - cu[i])
        if self.nan:
            out[0, 0] = np.nan
        return out


def test_data_parallel_sparse_and_late_gather_by_index():
    reps = [_EchoReplica(), _EchoReplica(), _EchoReplica()]
    dp = inl.DataParallelEmbedder(reps, max_batch_tokens=30, max_length=50)
    texts = _texts(40, seed=5)
    sv = dp.encode_sparse(texts)
    for t, v in zip(texts, sv):
        assert v.indices.tolist() == [len(t) % 4] and v.values.tolist() == [1.0]
    task = inl.LateTask(length=6, skip=frozenset({3}))
    late = dp.encode_late(texts, task)
    for t, v in zip(texts, late):
        kept = [x for x in list(t)[:6] if x != 3]
        assert v[:, 0].tolist() == kept
    assert all(r.calls > 0 for r in reps)
    with pytest.raises(inl.InferenceError, match="non-finite"):
        inl.DataParallelEmbedder([_EchoReplica(nan=True)]).encode_sparse([[1, 2]])
    with pytest.raises(inl.InferenceError, match="non-finite"):
        inl.DataParallelEmbedder([_EchoReplica(nan=True)]).encode_late([[1, 2]])


from hypothesis import given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402


@settings(max_examples=200, deadline=None)
@given(lengths=st.lists(st.integers(0, 300), max_size=60), budget=st.integers(1, 800),
       max_texts=st.one_of(st.none(), st.integers(1, 10)))
def test_plan_packed_properties(lengths, budget, max_texts):
    """For any lengths: consecutive ranges covering every input once, each
    within the real-token budget and the text cap unless it is one input."""
    order = inl.planner.longest_first(lengths)
    sorted_lengths = [lengths[i] for i in order]
    plan = inl.planner.plan_packed(sorted_lengths, budget, max_texts)
    flat = [k for r in plan for k in r]
    assert flat == list(range(len(lengths)))
    for r in plan:
        assert len(r) >= 1
        if len(r) > 1:
            assert sum(sorted_lengths[k] for k in r) <= budget
            assert max_texts is None or len(r) <= max_texts
    # longest first, ties in input order
    assert all(sorted_lengths[i] >= sorted_lengths[i + 1] for i in range(len(sorted_lengths) - 1))


@settings(max_examples=100, deadline=None)
@given(costs=st.lists(st.floats(0, 100, allow_nan=False), max_size=40), workers=st.integers(1, 8))
def test_assign_lpt_properties(costs, workers):
    """Every batch assigned once; the heaviest worker is within the LPT bound
    (at most the average load plus the largest single cost)."""
    plan = inl.planner.assign_lpt(costs, workers)
    assert len(plan) == workers
    assert sorted(b for w in plan for b in w) == list(range(len(costs)))
    loads = [sum(costs[b] for b in w) for w in plan]
    if costs:
        assert max(loads) <= sum(costs) / workers + max(costs) + 1e-9


@settings(max_examples=200, deadline=None)
@given(a=st.lists(st.tuples(st.integers(0, 50), st.one_of(st.floats(-2, 5, width=32),
                                                          st.sampled_from([float("nan"), float("inf")]))),
                  max_size=30),
       b=st.lists(st.tuples(st.integers(0, 50), st.floats(0.125, 5, width=32)), max_size=30))
def test_sparse_vector_properties(a, b):
    """from_pairs always yields a vector new() accepts; the JSON form
    round-trips; dot is symmetric and equals the dense inner product."""
    va, vb = inl.SparseVector.from_pairs(a), inl.SparseVector.from_pairs(b)
    for v in (va, vb):
        assert inl.SparseVector.new(v.indices, v.values) == v
        assert inl.SparseVector.from_json(v.to_json()) == v
    dense = np.zeros((2, 51), dtype=np.float64)
    dense[0, va.indices] = va.values
    dense[1, vb.indices] = vb.values
    assert va.dot(vb) == pytest.approx(vb.dot(va)) == pytest.approx(float(dense[0] @ dense[1]), rel=1e-5, abs=1e-6)
