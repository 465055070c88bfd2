"""Text front end (im-not-llm_b200/text.py and the facades' string inputs).

The tokenizer path is pinned against two of the reference's own fixtures.

* tiny_embeddinggemma2: its golden.json records the token count of every
  text at max_length 64 and 9 (crates/inl-text/src/gemma2.rs:941-967), and
  tests/test_oracle_gemma.py restates the fixture's tokenizer.json by hand.
* tiny_splade: its golden.json records the ids the reference fed its model
  for documents and queries at max_length 64 and 12.

The library must give the same ids, keep the template's special tokens when
it truncates, and count tokens before truncation."""
import json
from pathlib import Path

import numpy as np
import pytest

import im_not_llm_b200 as inl

GOLDEN = Path(__file__).resolve().parent / "golden" / "tiny_embeddinggemma2"


def _tok():
    return inl.TextTokenizer.from_file(GOLDEN / "tokenizer.json")


def _restated(text, max_length, vocab):
    words = [vocab.get(w, vocab["<unk>"]) for w in text.lower().split()]
    return [vocab["<bos>"]] + words[: max(0, max_length - 2)] + [vocab["<eos>"]]


def test_library_ids_match_restatement_and_golden_lengths():
    golden = json.loads((GOLDEN / "golden.json").read_text())
    vocab = json.loads((GOLDEN / "tokenizer.json").read_text())["model"]["vocab"]
    tok = _tok()
    for case in golden["cases"]:
        ids = tok.encode(golden["texts"], case["max_length"])
        assert [len(x) for x in ids] == case["lengths"]
        for text, got in zip(golden["texts"], ids):
            assert got.dtype == np.uint32
            assert got.tolist() == _restated(text, case["max_length"], vocab)


def test_truncation_keeps_special_tokens_and_counts_are_untruncated():
    vocab = json.loads((GOLDEN / "tokenizer.json").read_text())["model"]["vocab"]
    tok = _tok()
    text = " ".join(["the"] * 40)
    (ids,) = tok.encode([text], 9)
    assert len(ids) == 9 and ids[0] == vocab["<bos>"] and ids[-1] == vocab["<eos>"]
    assert tok.counts([text]) == [42]
    # one truncating copy per max_length, independent of each other
    assert len(tok.encode([text], 5)[0]) == 5 and len(tok.encode([text], 64)[0]) == 42


def test_unparsable_tokenizer_is_an_inference_error(tmp_path):
    bad = tmp_path / "tokenizer.json"
    bad.write_text("{ not json")
    with pytest.raises(inl.InferenceError):
        inl.TextTokenizer.from_file(bad)
    with pytest.raises(inl.ConfigError):
        _tok().encode(["x"], 0)


class RecordingModel:
    """Stands in for CudaModel: records the id segments it receives."""

    def __init__(self):
        self.dtype, self.device, self.seen = "bf16", 0, []

    def info(self):
        return {"dense_dim": 2, "arch": 0, "multivector_dim": 2, "sparse_dim": 4, "is_causal": True}

    def _segments(self, ids, cu):
        segs = [ids[cu[i]:cu[i + 1]].tolist() for i in range(len(cu) - 1)]
        self.seen.extend(segs)
        return segs

    def embed(self, ids, cu, out_dim=0):
        return np.array([[len(s), s[0]] for s in self._segments(ids, cu)], dtype=np.float32)

    def encode_sparse(self, ids, cu):
        out = np.zeros((len(cu) - 1, 4), dtype=np.float32)
        for i, s in enumerate(self._segments(ids, cu)):
            out[i, len(s) % 4] = 1.0
        return out

    def encode_sparse_compact(self, ids, cu):
        return [(np.nonzero(r > 0)[0].astype(np.uint32), r[r > 0]) for r in self.encode_sparse(ids, cu)]

    def close(self):
        pass


def test_embedder_applies_passage_and_query_prefixes():
    tok = _tok()
    model = RecordingModel()
    opts = inl.TextOptions(max_length=64, passage_prefix="title: none | text: ", query_prefix="query: ")
    e = inl.TextEmbedder(lambda: model, opts, tokenizer=tok)
    out = e.embed(["A quick test", "b"])
    want = tok.encode(["title: none | text: A quick test", "title: none | text: b"], 64)
    assert model.seen == [w.tolist() for w in want]
    assert [v[0] for v in out] == [len(w) for w in want]
    model.seen.clear()
    e.embed_query("what is it")
    assert model.seen == [tok.encode(["query: what is it"], 64)[0].tolist()]
    # token_counts: as given, no prefix, before truncation
    assert e.token_counts(["A quick test"]) == tok.counts(["A quick test"])
    # token ids still work and skip the tokenizer
    model.seen.clear()
    e.embed([np.array([5, 6, 7], dtype=np.uint32)])
    assert model.seen == [[5, 6, 7]]


def test_sparse_encoder_markers_and_input_errors():
    tok = _tok()
    model = RecordingModel()
    s = inl.SparseEncoder(lambda: model, inl.TextOptions.sparse(max_length=9), tokenizer=tok)
    s.encode(["some document text"])
    s.encode_query("a query")
    assert model.seen == [tok.encode(["[D] some document text"], 9)[0].tolist(),
                          tok.encode(["[Q] a query"], 9)[0].tolist()]
    with pytest.raises(inl.InvalidInputError):
        s.encode(["text", [1, 2, 3]])
    with pytest.raises(inl.ConfigError):
        inl.TextEmbedder(lambda: model, inl.TextOptions()).embed(["no tokenizer"])


SPLADE = Path(__file__).resolve().parent / "golden" / "tiny_splade"


def test_sparse_markers_and_truncation_reproduce_the_references_recorded_ids():
    """tiny_splade's golden.json records, per case, the ids the reference fed
    its model: the "[D] " / "[Q] " marker prepended (SparseEncoder::encode /
    encode_query), special tokens added, the tokenizer truncating at
    max_length 64 and 12 with [SEP] kept (crates/inl-sparse/src/modernbert.rs:1014-1057)."""
    golden = json.loads((SPLADE / "golden.json").read_text())
    tok = inl.TextTokenizer.from_file(SPLADE / "tokenizer.json")
    opts = inl.TextOptions.sparse()
    for case in golden["cases"]:
        prefix = opts.passage_prefix if case["kind"] == "document" else opts.query_prefix
        got = tok.encode([prefix + t for t in case["texts"]], case["max_length"])
        for rows in (case["batched"], case["alone"]):
            assert [g.tolist() for g in got] == [r["ids"] for r in rows], case["kind"]


def test_count_truncated_dense_and_sparse():
    tok = _tok()
    model = RecordingModel()
    texts = ["a b c d e f g h i j k", "short", "x " * 3, "w1 w2 w3 w4 w5 w6 w7"]
    counts = tok.counts(texts)  # <bos> ... <eos>: 13, 3, 5, 9
    e = inl.TextEmbedder(lambda: model, inl.TextOptions(max_length=9), tokenizer=tok)
    assert e.count_truncated(texts) == sum(n >= 9 for n in counts) == 2
    # the passage prefix counts, and texts under max_length bytes are not tokenized
    e2 = inl.TextEmbedder(lambda: model, inl.TextOptions(max_length=9, passage_prefix="p q r s "), tokenizer=tok)
    assert e2.count_truncated(texts) == sum(n >= 9 for n in tok.counts(["p q r s " + t for t in texts]))
    s = inl.SparseEncoder(lambda: model, inl.TextOptions.sparse(max_length=9), tokenizer=tok)
    # sparse: the byte gate looks at the text without its marker
    want = sum(len(t.encode()) >= 9 and len(ids) >= 9
               for t, ids in zip(texts, tok.encode(["[D] " + t for t in texts], 9)))
    assert s.count_truncated(texts) == want == 2  # "short" and "x x x " are under 9 bytes
    assert model.seen == []  # nothing reached the model


def test_data_parallel_embedder_takes_strings_and_checks_counts():
    tok = _tok()
    models = [RecordingModel(), RecordingModel()]
    dp = inl.DataParallelEmbedder(models, max_batch_tokens=8, tokenizer=tok, max_length=9, passage_prefix="p ")
    texts = ["a b c", "d e f g h i j k l m", "x"]
    out = dp.embed(texts)
    want = tok.encode(["p " + t for t in texts], 9)
    assert [v[0] for v in out] == [len(w) for w in want]
    assert sorted(map(tuple, models[0].seen + models[1].seen)) == sorted(tuple(w.tolist()) for w in want)
    with pytest.raises(inl.ConfigError):
        inl.DataParallelEmbedder(models).embed(["no tokenizer"])
    with pytest.raises(inl.InvalidInputError):
        dp.embed(["a", [1, 2]])

    class Dropping(RecordingModel):
        def embed(self, ids, cu, out_dim=0):
            return super().embed(ids, cu)[:-1]

    with pytest.raises(inl.InferenceError):
        inl.DataParallelEmbedder([Dropping()]).embed([[1, 2], [3]])


def test_gemma2_task_prefixes_match_the_model_card():
    """crates/inl-text/src/gemma2.rs:1090-1122 restated."""
    T = inl.Gemma2Task
    assert T.SEARCH_QUERY.prefix == "task: search result | query: "
    assert T.SEARCH_QUERY.apply("what causes the northern lights?") == \
        "task: search result | query: what causes the northern lights?"
    assert T.DOCUMENT.prefix == "title: none | text: "
    assert T.DOCUMENT.apply("a passage") == "title: none | text: a passage"
    assert inl.gemma2_document("Guide", "a passage") == "title: Guide | text: a passage"
    assert T.SEARCH_QUERY.is_query and not T.DOCUMENT.is_query
    for task in (T.QUERY, T.QUESTION_ANSWERING, T.FACT_CHECKING, T.CLASSIFICATION, T.CLUSTERING, T.CODE_RETRIEVAL):
        assert task.prefix.startswith("task: ") and task.is_query
        assert task.template == task.prefix + "{text}"


def test_gemma2_task_prefix_through_the_embedder_options():
    """A task prefix set as the query / passage prefix reaches the tokenizer
    exactly as Gemma2Task.apply builds it."""
    tok = _tok()
    model = RecordingModel()
    opts = inl.TextOptions(query_prefix=inl.Gemma2Task.SEARCH_QUERY.prefix,
                           passage_prefix=inl.Gemma2Task.DOCUMENT.prefix)
    e = inl.TextEmbedder(lambda: model, opts, tokenizer=tok)
    e.embed_query("a b")
    e.embed(["c d"])
    want = tok.encode([inl.Gemma2Task.SEARCH_QUERY.apply("a b"), inl.Gemma2Task.DOCUMENT.apply("c d")],
                      opts.max_length)
    assert [list(s) for s in model.seen] == [w.tolist() for w in want]


def test_identity_and_output_dim_checked_at_load():
    """identity (crates/inl-text/src/native.rs:476-488; sparse :271-283, late
    :256-270) loads the model; an output_dim the model cannot give is a config
    error at load (native.rs:438-440)."""
    model = RecordingModel()
    e = inl.TextEmbedder(lambda: model, inl.TextOptions(id="m", max_length=9))
    ident = e.identity()
    assert (ident.id, ident.dimension, ident.dtype, ident.device, ident.max_length) == ("m", 2, "bf16", "cuda", 9)
    with pytest.raises(inl.ConfigError, match="only supported for EmbeddingGemma 2"):
        inl.TextEmbedder(lambda: RecordingModel(), inl.TextOptions(output_dim=128)).load()
    s = inl.SparseEncoder(lambda: RecordingModel(), inl.TextOptions.sparse(id="s"))
    assert s.identity().dimension == 4 and s.is_loaded()


def test_option_refusals_of_the_three_engines():
    """batch_size 0: an inference error when the dense engine embeds
    (crates/inl-text/src/native.rs:552-556); a config error when a sparse or
    late encoder is built, as are a zero timeout and late max_length 0
    (crates/inl-sparse/src/native.rs:197-210, crates/inl-late/src/native.rs:184-202)."""
    e = inl.TextEmbedder(lambda: RecordingModel(), inl.TextOptions(batch_size=0))
    assert e.embed([]) == []
    with pytest.raises(inl.InferenceError, match="batch_size must be greater than 0"):
        e.embed([[1, 2]])
    for bad in (dict(batch_size=0), dict(timeout_seconds=0), dict(per_batch_timeout_seconds=0)):
        with pytest.raises(inl.ConfigError):
            inl.SparseEncoder(lambda: RecordingModel(), inl.TextOptions.sparse(**bad))
        with pytest.raises(inl.ConfigError):
            inl.LateEncoder(lambda: RecordingModel(), inl.TextOptions(**bad))
    with pytest.raises(inl.ConfigError, match="max_length"):
        inl.LateEncoder(lambda: RecordingModel(), inl.TextOptions(max_length=0))
