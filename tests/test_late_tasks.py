"""Late encoder tasks (LateTask, LateEncoder.encode(inputs, task)) pinned on
the reference's tiny_qwen3_5_late fixture.

Its golden.json records, per task, how many tokens each text has after the
task's prompt is put in front and the ids are cut at the task's length
(`lengths`), and how many vectors come back once the document skiplist is
applied (the rows of `batched` / `alone`). The host does all of this; the
fixture's Qwen3.5 tower is not built here, so a stand-in model returns one
vector per token (crates/inl-late/src/native.rs:292-305, 580-620, 631-683)."""
import json
from pathlib import Path

import numpy as np
import pytest

import im_not_llm_b200 as inl

LATE = Path(__file__).resolve().parent / "golden" / "tiny_qwen3_5_late"


def _setup():
    tok = inl.TextTokenizer.from_file(LATE / "tokenizer.json")
    return tok, inl.LateTask.from_model_dir(LATE, tok), json.loads((LATE / "golden.json").read_text())


def test_task_setups_from_the_model_directory():
    tok, tasks, _ = _setup()
    q, d = tasks["query"], tasks["document"]
    assert (q.prompt, q.length, q.skip) == ("[Q] ", 24, frozenset())
    assert (d.prompt, d.length) == ("[D] ", 160)
    want = {tok.token_to_id(w) for w in [".", ",", "!", "~"]} - {None}
    assert d.skip == frozenset(want) and len(want) > 0
    capped = inl.LateTask.from_model_dir(LATE, tok, max_length=10)
    assert capped["query"].length == 10 and capped["document"].length == 10


def test_prompt_cut_and_skiplist_reproduce_the_references_counts():
    tok, tasks, golden = _setup()
    for case in golden["cases"]:
        setup = tasks[case["task"]]
        rows = [ids[:setup.length] for ids in tok.encode_untruncated([setup.prompt + t for t in golden["texts"]])]
        assert [len(r) for r in rows] == case["lengths"], case["task"]
        kept = [int(np.sum(~np.isin(r, list(setup.skip)))) for r in rows]
        assert kept == [len(v) for v in case["batched"]] == [len(v) for v in case["alone"]], case["task"]


class TokenEchoModel:
    """Stands in for CudaModel: one vector (token id, position) per token."""

    dtype, device = "bf16", 0

    def info(self):
        return {"multivector_dim": 2}

    def encode_multivector(self, ids, cu):
        out = np.zeros((len(ids), 2), dtype=np.float32)
        for i in range(len(cu) - 1):
            out[cu[i]:cu[i + 1], 0] = ids[cu[i]:cu[i + 1]]
            out[cu[i]:cu[i + 1], 1] = np.arange(cu[i + 1] - cu[i])
        return out

    def close(self):
        pass


def test_late_encoder_keeps_the_references_vectors_per_task():
    tok, tasks, golden = _setup()
    enc = inl.LateEncoder(lambda: TokenEchoModel(), inl.TextOptions(max_batch_tokens=64), tokenizer=tok,
                          tasks=tasks)
    for case in golden["cases"]:
        setup = tasks[case["task"]]
        out = enc.encode(golden["texts"], task=case["task"])
        assert [len(m) for m in out] == [len(v) for v in case["batched"]], case["task"]
        for text, m in zip(golden["texts"], out):
            (ids,) = tok.encode_untruncated([setup.prompt + text])
            ids = ids[:setup.length]
            kept = ~np.isin(ids, list(setup.skip))
            # the surviving vectors are those of the non-skiplist tokens, in token order
            assert m[:, 0].tolist() == ids[kept].astype(np.float32).tolist()
            assert m[:, 1].tolist() == np.arange(len(ids))[kept].astype(np.float32).tolist()
    with pytest.raises(inl.InvalidInputError):
        enc.encode(["x"], task="passage")
    # token-id lists: cut at the task's length, skiplist applied
    ids = np.array([5] * 30, dtype=np.uint32)
    assert len(enc.encode([ids], task="query")[0]) == 24


def test_late_token_counts_per_task_match_the_references_lengths():
    """LateEngine::token_counts(texts, task) (crates/inl-late/src/lib.rs:44-46):
    prompt included, after the task's cut; the golden's recorded lengths."""
    tok, tasks, golden = _setup()
    enc = inl.LateEncoder(lambda: TokenEchoModel(), inl.TextOptions(), tokenizer=tok, tasks=tasks)
    for case in golden["cases"]:
        assert enc.token_counts(golden["texts"], task=case["task"]) == case["lengths"], case["task"]
    assert not enc.is_loaded()
    with pytest.raises(inl.InvalidInputError):
        enc.token_counts(["x"], task="passage")
