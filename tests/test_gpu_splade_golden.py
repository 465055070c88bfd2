"""The ModernBERT + SPLADE tower on the GPU against the reference's own
tiny_splade golden (f32): identical active term sets and |dw| <= 1e-4 for
every case, batched and one text per forward (the assertion of
crates/inl-sparse/src/modernbert.rs:1014-1057). The fixture's pooling has a
logit shift of 2, two prefix tokens that are also masked, and a canonical
fold of 72 terms onto 62; its head_dim 8 runs on the narrow RoPE kernel and
the small f32 attention. Once through CudaModel on the recorded ids, once
through the SparseEncoder facade from the texts ("[D] " / "[Q] " markers,
the fixture's tokenizer)."""
import json
from pathlib import Path

import numpy as np
import pytest

import im_not_llm_b200 as inl

GOLDEN = Path(__file__).resolve().parent / "golden" / "tiny_splade"
TOLERANCE = 1e-4  # crates/inl-sparse/src/modernbert.rs:1014-1057

pytestmark = pytest.mark.gpu


def _config():
    cfg = json.loads((GOLDEN / "config.json").read_text())
    cfg["splade"] = json.loads((GOLDEN / "1_ShiftedTopKSpladePooling" / "config.json").read_text())
    return cfg


def _pack(rows):
    ids = np.concatenate([np.asarray(r, dtype=np.uint32) for r in rows])
    cu = np.concatenate([[0], np.cumsum([len(r) for r in rows])]).astype(np.int32)
    return ids, cu


def _assert_term_weights(indices, values, want, label):
    assert list(indices) == want["indices"], f"{label}: active terms differ"
    if len(values):
        assert np.abs(np.asarray(values) - np.asarray(want["values"], dtype=np.float32)).max() <= TOLERANCE, label


def test_tiny_splade_on_the_recorded_ids(gpu):
    golden = json.loads((GOLDEN / "golden.json").read_text())
    m = inl.CudaModel(_config(), str(GOLDEN / "model.safetensors"), dtype="f32")
    try:
        assert m.info()["sparse_dim"] == golden["dim"]
        for case in golden["cases"]:
            label = f'{case["kind"]}/{case["max_length"]}'
            got = m.encode_sparse(*_pack([r["ids"] for r in case["batched"]]))
            for i, want in enumerate(case["batched"]):
                v = inl.SparseVector.from_dense(got[i])
                _assert_term_weights(v.indices, v.values, want, f"{label} batched[{i}]")
            for i, want in enumerate(case["alone"]):
                v = inl.SparseVector.from_dense(m.encode_sparse(*_pack([want["ids"]]))[0])
                _assert_term_weights(v.indices, v.values, want, f"{label} alone[{i}]")
    finally:
        m.close()


@pytest.mark.parametrize("batch_size,which", [(64, "batched"), (1, "alone")])
def test_tiny_splade_through_the_sparse_encoder(gpu, batch_size, which):
    golden = json.loads((GOLDEN / "golden.json").read_text())
    tok = inl.TextTokenizer.from_file(GOLDEN / "tokenizer.json")
    model = inl.CudaModel(_config(), str(GOLDEN / "model.safetensors"), dtype="f32")
    for case in golden["cases"]:
        enc = inl.SparseEncoder(lambda: model, inl.TextOptions.sparse(max_length=case["max_length"],
                                                                       batch_size=batch_size), tokenizer=tok)
        if case["kind"] == "document":
            out = enc.encode(case["texts"])
        else:
            out = [enc.encode_query(t) for t in case["texts"]]
        for i, (v, want) in enumerate(zip(out, case[which])):
            _assert_term_weights(v.indices, v.values, want, f'{case["kind"]}/{case["max_length"]} {which}[{i}]')
    model.close()


def test_tiny_splade_from_the_model_dir(gpu):
    """SparseEncoder.from_model_dir on the fixture as the reference lays it
    out: modules.json names the pooling module, the markers are the
    defaults, the context is capped at max_position_embeddings (64)."""
    golden = json.loads((GOLDEN / "golden.json").read_text())
    case = next(c for c in golden["cases"] if c["kind"] == "document" and c["max_length"] == 64)
    enc = inl.SparseEncoder.from_model_dir(GOLDEN)
    assert enc.options.max_length == 64
    for i, (v, want) in enumerate(zip(enc.encode(case["texts"]), case["batched"])):
        _assert_term_weights(v.indices, v.values, want, f"from_model_dir[{i}]")
    enc.unload()
