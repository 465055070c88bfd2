"""Pins the Qwen3.5 late-interaction oracle (oracle/qwen3_5.py) against the
reference's own golden fixture tiny_qwen3_5_late (copied by
tests/golden/make_golden.py): the assertion of
crates/inl-late/tests/tiny_golden.rs, every token vector within 1e-4 of the
golden, batched and alone, for the query and the document task. Inputs go
through the host's task handling (LateTask: prompt, cut at the task length,
skiplist)."""
import json
from pathlib import Path

import numpy as np

import im_not_llm_b200 as inl
from oracle import qwen3_5 as Q35

LATE = Path(__file__).resolve().parent / "golden" / "tiny_qwen3_5_late"
TOLERANCE = 1e-4  # crates/inl-late/tests/tiny_golden.rs:24-26


def _load():
    from safetensors.numpy import load_file

    cfg = json.loads((LATE / "config.json").read_text())
    weights = load_file(str(LATE / "model.safetensors"))
    dense = load_file(str(LATE / "1_Dense" / "model.safetensors"))
    golden = json.loads((LATE / "golden.json").read_text())
    tok = inl.TextTokenizer.from_file(LATE / "tokenizer.json")
    return cfg, weights, dense["linear.weight"], golden, tok, inl.LateTask.from_model_dir(LATE, tok)


def test_oracle_matches_the_references_golden_vectors():
    cfg, weights, proj, golden, tok, tasks = _load()
    for case in golden["cases"]:
        setup = tasks[case["task"]]
        rows = [ids[:setup.length] for ids in tok.encode_untruncated([setup.prompt + t for t in golden["texts"]])]
        for which in ("batched", "alone"):
            for i, (ids, want) in enumerate(zip(rows, case[which])):
                got = Q35.late_vectors(weights, cfg, proj, None, ids, skip=setup.skip)
                want = np.asarray(want, dtype=np.float32).reshape(len(want), -1)
                assert got.shape == want.shape, (case["task"], which, i)
                if got.size:
                    err = np.abs(got - want).max()
                    assert err < TOLERANCE, (case["task"], which, i, err)
                    assert got.shape[1] == golden["dim"]


def test_recurrent_delta_rule_on_a_hand_case():
    """One head, dk = dv = 1, unit keys and queries after the L2 norm: the
    state is a scalar, S_t = a_t S_{t-1} + u_t, u_t = b_t (v_t - a_t S_{t-1})."""
    q = np.ones((3, 1, 1), dtype=np.float32)
    k = np.ones((3, 1, 1), dtype=np.float32)
    v = np.array([1.0, 2.0, -1.0], dtype=np.float32).reshape(3, 1, 1)
    g = np.log(np.array([0.5, 0.25, 1.0], dtype=np.float32)).reshape(3, 1)
    beta = np.array([1.0, 0.5, 0.25], dtype=np.float32).reshape(3, 1)
    n = 1 / np.sqrt(1 + 1e-6)  # l2norm of a unit scalar
    S, want = 0.0, []
    for t in range(3):
        a = np.exp(g[t, 0])
        u = beta[t, 0] * (v[t, 0, 0] - a * S * n)
        S = a * S + n * u
        want.append(S * n)
    got = Q35.gated_delta_rule(q, k, v, g, beta)[:, 0, 0]
    assert np.allclose(got, want, atol=1e-6)


def test_chunked_form_equals_the_recurrence():
    """The chunked (WY) form, the structure of a tensor-core kernel, gives the
    recurrent rule's outputs for lengths below, at and across chunk sizes."""
    rng = np.random.default_rng(3)
    for T, chunk, dk, dv in [(1, 64, 8, 8), (5, 4, 8, 16), (64, 64, 16, 8), (65, 64, 8, 8), (200, 64, 32, 32),
                             (37, 8, 16, 16)]:
        q = rng.standard_normal((T, 2, dk)).astype(np.float32)
        k = rng.standard_normal((T, 2, dk)).astype(np.float32)
        v = rng.standard_normal((T, 2, dv)).astype(np.float32)
        g = -np.abs(rng.standard_normal((T, 2))).astype(np.float32)
        beta = Q35.sigmoid(rng.standard_normal((T, 2)).astype(np.float32))
        want = Q35.gated_delta_rule(q, k, v, g, beta)
        got = Q35.gated_delta_rule_chunked(q, k, v, g, beta, chunk=chunk)
        assert np.abs(got - want).max() < 1e-5, (T, chunk)


def test_bf16_operand_mode_rounds_like_torch():
    """oracle/qwen3_5.py's bf16 operand mode: round to nearest, ties to even
    (torch's float -> bfloat16 conversion), f32 sums."""
    import torch

    from oracle import qwen3_5 as Q35

    rng = np.random.default_rng(7)
    x = (rng.standard_normal(4096) * np.exp(rng.uniform(-20, 20, 4096))).astype(np.float32)
    ties = np.array([1 + 2 ** -8, 1 + 3 * 2 ** -8, -(1 + 2 ** -8), 1 + 2 ** -9], dtype=np.float32)
    for v in (x, ties):
        want = torch.from_numpy(v).to(torch.bfloat16).float().numpy()
        assert np.array_equal(Q35.bf16_round(v), want)
    a = rng.standard_normal((5, 24)).astype(np.float32)
    w = rng.standard_normal((7, 24)).astype(np.float32)
    assert np.array_equal(Q35.linear(a, w, "bf16"), Q35.bf16_round(a) @ Q35.bf16_round(w).T)
    assert np.array_equal(Q35.linear(a, w), a @ w.T)
