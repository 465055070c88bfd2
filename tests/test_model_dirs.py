"""Model directories read as the reference's native engines read them
(im-not-llm_b200/loading.py and the engines' from_model_dir), on the CPU: the
lazy loader is called with a stand-in CudaModel that records what it would
load. Fixtures are the reference's tiny checkpoints (tests/golden/), in the
reference's directory layout."""
import json
import shutil
from pathlib import Path

import numpy as np
import pytest

import im_not_llm_b200 as inl
from im_not_llm_b200 import engine, loading

GOLDEN = Path(__file__).resolve().parent / "golden"


class RecordingModel:
    """Stands in for CudaModel inside the engines' loaders."""
    made: list = []

    def __init__(self, config, weights, device=0, dtype="bf16"):
        self.config, self.weights, self.device, self.dtype = config, Path(weights), device, dtype
        self.dense = None
        RecordingModel.made.append(self)

    def set_dense_head(self, weight, bias=None, normalize=True):
        self.dense = (np.asarray(weight).shape, None if bias is None else np.asarray(bias).shape, normalize)

    def close(self):
        pass


@pytest.fixture
def recording(monkeypatch):
    RecordingModel.made = []
    monkeypatch.setattr(engine, "CudaModel", RecordingModel)
    return RecordingModel


def _splade_dir(tmp_path):
    d = tmp_path / "splade"
    shutil.copytree(GOLDEN / "tiny_splade", d)
    return d


def _late_dir(tmp_path):
    d = tmp_path / "late"
    shutil.copytree(GOLDEN / "tiny_qwen3_5_late", d)
    return d


def test_dense_dir_gemma2_defaults_to_f32(recording):
    d = GOLDEN / "tiny_embeddinggemma2"
    spec = loading.dense_model(d)
    assert (spec.architecture, spec.dtype, spec.weights.name) == ("gemma2", "f32", "model.safetensors")
    e = inl.TextEmbedder.from_model_dir(d, inl.TextOptions(max_length=9))
    assert recording.made == []  # loaded on first use
    assert e.token_counts(["a b c"]) == [5]
    m = e._model().model
    assert (m.dtype, m.weights, m.config["model_type"]) == ("f32", d / "model.safetensors", "embedding_gemma2")


def test_dense_dir_qwen3_defaults_to_bf16_and_takes_a_sharded_index(tmp_path, recording):
    d = tmp_path / "qwen3"
    d.mkdir()
    (d / "config.json").write_text(json.dumps({"model_type": "qwen3", "hidden_size": 8}))
    (d / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {"a": "model-1.safetensors"}}))
    shutil.copy(GOLDEN / "tiny_embeddinggemma2" / "tokenizer.json", d / "tokenizer.json")
    e = inl.TextEmbedder.from_model_dir(d, device=3)
    m = e._model().model
    assert (m.dtype, m.device, m.weights.name) == ("bf16", 3, "model.safetensors.index.json")
    with pytest.raises(inl.ConfigError):
        loading.dense_model(d, dtype="f16")
    (d / "model.safetensors.index.json").unlink()
    with pytest.raises(inl.InferenceError, match="model.safetensors are missing"):
        loading.dense_model(d)


def test_sparse_dir_reads_the_pooling_module_and_caps_the_context(tmp_path, recording):
    d = _splade_dir(tmp_path)
    e = inl.SparseEncoder.from_model_dir(d)
    assert e.options.query_prefix == "[Q] " and e.options.passage_prefix == "[D] "
    assert e.options.max_length == 64  # max_position_embeddings of the fixture
    m = e._model().model
    pooling = json.loads((GOLDEN / "tiny_splade" / "1_ShiftedTopKSpladePooling" / "config.json").read_text())
    assert m.config["splade"] == pooling and m.dtype == "f32"
    (d / "modules.json").write_text(json.dumps([{"path": "", "type": "x.Transformer"}]))
    with pytest.raises(inl.InferenceError, match="no SPLADE pooling module"):
        inl.SparseEncoder.from_model_dir(d)


def test_late_dir_dense_head_normalize_and_tasks(tmp_path, recording):
    d = _late_dir(tmp_path)
    e = inl.LateEncoder.from_model_dir(d)
    assert (e.tasks["query"].length, e.tasks["document"].length) == (24, 160)
    m = e._model().model
    assert m.dense == ((12, 32), None, True) and m.dtype == "f32"
    # without the Normalize module the vectors stay unnormalised
    modules = json.loads((d / "modules.json").read_text())
    (d / "modules.json").write_text(json.dumps(modules[:3]))
    assert loading.late_model(d).normalize is False


@pytest.mark.parametrize("edit,message", [
    (lambda d, m: m.append({"path": "4_Pooling", "type": "sentence_transformers.models.Pooling"}), "is not supported"),
    (lambda d, m: m.pop(1), "has no Dense projection"),
    (lambda d, m: m.insert(0, m.pop(1)), "must start with a Transformer"),
])
def test_late_dir_refuses_other_module_layouts(tmp_path, edit, message):
    d = _late_dir(tmp_path)
    modules = json.loads((d / "modules.json").read_text())
    edit(d, modules)
    (d / "modules.json").write_text(json.dumps(modules))
    with pytest.raises(inl.InferenceError, match=message):
        loading.late_model(d)


@pytest.mark.parametrize("field,value", [("activation_function", "torch.nn.Tanh"), ("use_residual", True),
                                         ("in_features", 64)])
def test_late_dir_refuses_a_dense_that_is_not_a_plain_projection(tmp_path, field, value):
    d = _late_dir(tmp_path)
    cfg = json.loads((d / "1_Dense" / "config.json").read_text())
    cfg[field] = value
    (d / "1_Dense" / "config.json").write_text(json.dumps(cfg))
    with pytest.raises(inl.InferenceError, match="plain 32 -> n projection"):
        loading.late_model(d)


def test_late_dir_refuses_query_expansion(tmp_path):
    d = _late_dir(tmp_path)
    st = json.loads((d / "sentence_bert_config.json").read_text())
    st["query_expansion"] = {"n": 4}
    (d / "sentence_bert_config.json").write_text(json.dumps(st))
    with pytest.raises(inl.InferenceError, match="query expansion"):
        loading.late_model(d)


def test_missing_files_are_inference_errors(tmp_path):
    with pytest.raises(inl.InferenceError, match="config.json is missing"):
        loading.dense_model(tmp_path)
    (tmp_path / "config.json").write_text("{not json")
    with pytest.raises(inl.InferenceError, match="is invalid"):
        loading.dense_model(tmp_path)


def test_late_dir_dense_bias_must_be_in_the_weights(tmp_path, recording):
    """A Dense config with "bias": true needs linear.bias in its weights
    (crates/inl-late/src/native.rs:559-566); the error comes at load."""
    d = _late_dir(tmp_path)
    cfg = json.loads((d / "1_Dense" / "config.json").read_text())
    cfg["bias"] = True
    (d / "1_Dense" / "config.json").write_text(json.dumps(cfg))
    e = inl.LateEncoder.from_model_dir(d)
    assert loading.late_model(d).dense_bias
    with pytest.raises(inl.InferenceError, match="Dense weight load failed"):
        e._model()
    assert not e.is_loaded()
