"""The Qwen3.5 late-interaction tower on the GPU (f32) against the reference's
tiny_qwen3_5_late golden: every kept token vector within 1e-4, batched and
one text per forward, query and document tasks (the assertion of
crates/inl-late/tests/tiny_golden.rs), through the LateEncoder facade with
the fixture's tokenizer, prompts, lengths and skiplist. The oracle
(oracle/qwen3_5.py) is pinned on the same golden on the CPU."""
import json
from pathlib import Path

import numpy as np
import pytest

import im_not_llm_b200 as inl

LATE = Path(__file__).resolve().parent / "golden" / "tiny_qwen3_5_late"
TOLERANCE = 1e-4  # crates/inl-late/tests/tiny_golden.rs:24-26
BF16_COS = 0.999  # per-token cosine against the oracle in the same bf16 operand mode

pytestmark = pytest.mark.gpu


def _encoder(batch_size, dtype="f32"):
    from safetensors.numpy import load_file

    cfg = json.loads((LATE / "config.json").read_text())
    dense = load_file(str(LATE / "1_Dense" / "model.safetensors"))["linear.weight"]
    tok = inl.TextTokenizer.from_file(LATE / "tokenizer.json")

    def load():
        m = inl.CudaModel(cfg, str(LATE / "model.safetensors"), dtype=dtype)
        m.set_dense_head(dense)
        return m

    return inl.LateEncoder(load, inl.TextOptions(batch_size=batch_size), tokenizer=tok,
                           tasks=inl.LateTask.from_model_dir(LATE, tok))


@pytest.mark.parametrize("batch_size,which", [(64, "batched"), (1, "alone")])
def test_tiny_late_tower_matches_the_references_golden(gpu, batch_size, which):
    golden = json.loads((LATE / "golden.json").read_text())
    enc = _encoder(batch_size)
    for case in golden["cases"]:
        out = enc.encode(golden["texts"], task=case["task"])
        for i, (got, want) in enumerate(zip(out, case[which])):
            want = np.asarray(want, dtype=np.float32).reshape(len(want), -1)
            assert got.shape == want.shape, (case["task"], i)
            if got.size:
                assert np.abs(got - want).max() < TOLERANCE, (case["task"], which, i)
    enc.unload()


def test_dense_bias_and_a_model_without_normalize(gpu):
    """The late head's optional pieces (crates/inl-late/src/native.rs:650-656):
    a Dense bias, and no L2 when the model has no Normalize module; every
    token vector, skiplist not applied, against oracle/qwen3_5.py."""
    from safetensors.numpy import load_file

    from oracle import qwen3_5 as Q35

    cfg = json.loads((LATE / "config.json").read_text())
    weights = load_file(str(LATE / "model.safetensors"))
    dense = load_file(str(LATE / "1_Dense" / "model.safetensors"))["linear.weight"]
    bias = (np.random.default_rng(4).standard_normal(dense.shape[0]) * 0.1).astype(np.float32)
    tok = inl.TextTokenizer.from_file(LATE / "tokenizer.json")
    rows = tok.encode_untruncated(["a short text", "and a second, somewhat longer one"])
    ids = np.concatenate(rows)
    cu = np.concatenate([[0], np.cumsum([len(r) for r in rows])]).astype(np.int32)
    m = inl.CudaModel(cfg, str(LATE / "model.safetensors"), dtype="f32")
    try:
        for normalize in (True, False):
            m.set_dense_head(dense, bias, normalize=normalize)
            got = m.encode_multivector(ids, cu)
            want = np.concatenate([Q35.late_vectors(weights, cfg, dense, bias, r, normalize=normalize) for r in rows])
            assert got.shape == want.shape
            assert np.abs(got - want).max() < TOLERANCE * max(1.0, float(np.abs(want).max()))
    finally:
        m.close()


def test_tiny_late_tower_from_the_model_dir(gpu):
    """The same golden through LateEncoder.from_model_dir: modules, Dense,
    Normalize, prompts, lengths and skiplist read from the directory."""
    golden = json.loads((LATE / "golden.json").read_text())
    enc = inl.LateEncoder.from_model_dir(LATE)
    for case in golden["cases"]:
        out = enc.encode(golden["texts"], task=case["task"])
        for i, (got, want) in enumerate(zip(out, case["batched"])):
            want = np.asarray(want, dtype=np.float32).reshape(len(want), -1)
            assert got.shape == want.shape, (case["task"], i)
            if got.size:
                assert np.abs(got - want).max() < TOLERANCE, (case["task"], i)
    enc.unload()


def test_tiny_late_tower_in_bf16(gpu):
    """The tower requested in bf16 (the reference accepts it,
    crates/inl-late/src/native.rs:232): GEMMs on bf16-rounded operands with
    f32 sums, f32 activations, norms and recurrence. Every token vector of the
    golden's texts (query and document prompts, batched) against the oracle in
    the same operand mode (oracle/qwen3_5.py ``operands="bf16"``), and the
    model reports bf16. Against the f32 golden itself this random tiny tower
    loses up to half its cosine on a few tokens in both implementations alike
    (the oracle's bf16 mode shows the same worst token), so the f32 vectors
    are not the bound here."""
    from safetensors.numpy import load_file

    from oracle import qwen3_5 as Q35

    cfg = json.loads((LATE / "config.json").read_text())
    weights = load_file(str(LATE / "model.safetensors"))
    dense = load_file(str(LATE / "1_Dense" / "model.safetensors"))["linear.weight"]
    golden = json.loads((LATE / "golden.json").read_text())
    tok = inl.TextTokenizer.from_file(LATE / "tokenizer.json")
    tasks = inl.LateTask.from_model_dir(LATE, tok)
    m = inl.CudaModel(cfg, str(LATE / "model.safetensors"), dtype="bf16")
    try:
        assert m.info()["dtype"] == 1  # INL_DTYPE_BF16, as created
        m.set_dense_head(dense)
        worst = 1.0
        for task in ("query", "document"):
            setup = tasks[task]
            rows = [r[:setup.length] for r in tok.encode_untruncated([setup.prompt + t for t in golden["texts"]])]
            rows = [np.asarray(r, dtype=np.uint32) for r in rows if len(r)]
            ids = np.concatenate(rows)
            cu = np.concatenate([[0], np.cumsum([len(r) for r in rows])]).astype(np.int32)
            got = m.encode_multivector(ids, cu)
            want = np.concatenate([Q35.late_vectors(weights, cfg, dense, None, r, operands="bf16") for r in rows])
            assert got.shape == want.shape
            cos = (got * want).sum(-1) / (np.linalg.norm(got, axis=-1) * np.linalg.norm(want, axis=-1))
            worst = min(worst, float(cos.min()))
        assert worst >= BF16_COS, worst
    finally:
        m.close()
