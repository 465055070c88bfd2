"""Model directories as the reference's native engines read them, for the
``from_model_dir`` constructors of the engine facades. Host-side file logic
only: what to load, with which settings, and the reference's refusals. The
weights themselves are read by libinl_cuda when the engine loads.

* dense (crates/inl-text/src/native.rs:60-130, 406-470, 871-890): the
  architecture from config.json's model_type (``embedding_gemma2`` is
  EmbeddingGemma 2, anything else loads as Qwen3); default dtype bf16 for
  Qwen3 on a CUDA GPU, f32 for EmbeddingGemma 2.
* sparse (crates/inl-sparse/src/native.rs:424-500, 245): the SPLADE pooling
  module named by modules.json, its config.json; default dtype f32; the
  context capped by max_position_embeddings.
* late (crates/inl-late/src/native.rs:455-620): modules.json starts with a
  Transformer, then one Dense, an optional MultiVectorMask and an optional
  Normalize, nothing else; the Dense is a plain hidden_size -> n projection
  (Identity activation, no residual); query expansion is refused.
* weights: model.safetensors, else the shards of model.safetensors.index.json
  (crates/inl-core/src/hub.rs:324-353, resolved by libinl_cuda).
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

from .errors import InlError

GEMMA2_MODEL_TYPE = "embedding_gemma2"  # crates/inl-text/src/gemma2.rs:44


def read_json(model_dir: Path, name: str, what: str = "model"):
    """``name`` under ``model_dir``, parsed; a missing or invalid file is an
    inference error (ModelSource::fetch, crates/inl-core/src/hub.rs:374-389)."""
    f = Path(model_dir) / name
    if not f.is_file():
        raise InlError.inference(f"native {what} file {name} is missing from {model_dir}")
    try:
        return json.loads(f.read_text())
    except ValueError as e:
        raise InlError.inference(f"native {what} {name} is invalid: {e}") from e


def weights_path(model_dir: Path) -> Path:
    """model.safetensors, else a sharded checkpoint's index."""
    d = Path(model_dir)
    for name in ("model.safetensors", "model.safetensors.index.json"):
        if (d / name).is_file():
            return d / name
    raise InlError.inference(f"native model weights model.safetensors are missing from {d}")


def tokenizer_path(model_dir: Path, what: str = "model") -> Path:
    f = Path(model_dir) / "tokenizer.json"
    if not f.is_file():
        raise InlError.inference(f"native {what} file tokenizer.json is missing from {model_dir}")
    return f


def _text_config(config: dict) -> dict:
    return config.get("text_config", config) if isinstance(config.get("text_config"), dict) else config


@dataclass(frozen=True)
class DenseModel:
    config: dict
    weights: Path
    tokenizer: Path
    architecture: str  # "qwen3" or "gemma2"
    dtype: str


def dense_model(model_dir: str | Path, dtype: str | None = None) -> DenseModel:
    d = Path(model_dir)
    config = read_json(d, "config.json")
    arch = "gemma2" if config.get("model_type") == GEMMA2_MODEL_TYPE else "qwen3"
    if dtype is None:  # default_dtype (native.rs:871-890): B200 is a bf16-capable CUDA GPU
        dtype = "f32" if arch == "gemma2" else "bf16"
    if dtype not in ("bf16", "f32"):
        raise InlError.config(f"dtype {dtype!r} is not supported: use bf16 or f32")
    return DenseModel(config, weights_path(d), tokenizer_path(d), arch, dtype)


@dataclass(frozen=True)
class SparseModel:
    config: dict  # config.json with the pooling module's config under "splade"
    weights: Path
    tokenizer: Path
    positions: int  # max_position_embeddings (the context cap)


def sparse_model(model_dir: str | Path) -> SparseModel:
    d = Path(model_dir)
    config = read_json(d, "config.json", "sparse model")
    modules = read_json(d, "modules.json", "sparse model")
    module = next((m for m in modules if isinstance(m, dict) and "splade" in str(m.get("type", "")).lower()), None)
    if module is None:
        raise InlError.inference("native sparse model modules.json has no SPLADE pooling module")
    sub = str(module.get("path") or "").rstrip("/")
    pooling = read_json(d, f"{sub}/config.json" if sub else "config.json", "sparse model")
    config = dict(config, splade=pooling)
    positions = int(config.get("max_position_embeddings") or 0)
    return SparseModel(config, weights_path(d), tokenizer_path(d, "sparse model"), positions)


@dataclass(frozen=True)
class LateModel:
    config: dict
    weights: Path
    tokenizer: Path
    dense_weights: Path  # the Dense module's model.safetensors (linear.weight [out, in], linear.bias)
    dense_out: int
    dense_bias: bool
    normalize: bool


def late_model(model_dir: str | Path) -> LateModel:
    d = Path(model_dir)
    modules = read_json(d, "modules.json", "late model")
    if not modules or not str(modules[0].get("type", "")).endswith("Transformer"):
        raise InlError.inference("native late model modules.json must start with a Transformer module")
    dense_dir, normalize = None, False
    for module in modules[1:]:
        kind = str(module.get("type", "")).rsplit(".", 1)[-1]
        if kind == "Dense" and dense_dir is None:
            dense_dir = str(module.get("path") or "")
        elif kind == "MultiVectorMask":
            pass  # read with the tasks (LateTask.from_model_dir)
        elif kind == "Normalize":
            normalize = True
        else:
            raise InlError.inference(f"native late model module {module.get('type')} is not supported")
    if dense_dir is None:
        raise InlError.inference("native late model modules.json has no Dense projection")
    config = read_json(d, "config.json", "late model")
    st = read_json(d, "sentence_bert_config.json", "late model")
    if st.get("query_expansion") is not None:
        raise InlError.inference("native late model query expansion is not supported")
    hidden = int(_text_config(config).get("hidden_size") or 0)
    sub = dense_dir.rstrip("/")
    dense = read_json(d, f"{sub}/config.json" if sub else "config.json", "late model")
    act = dense.get("activation_function")
    identity = act is None or str(act).endswith("Identity")
    if not identity or dense.get("use_residual") or int(dense.get("in_features") or -1) != hidden:
        raise InlError.inference(f"native late model Dense must be a plain {hidden} -> n projection without "
                                 f"activation or residual")
    dense_weights = d / (f"{sub}/model.safetensors" if sub else "model.safetensors")
    if not dense_weights.is_file():
        raise InlError.inference(f"native late model file {dense_weights.relative_to(d)} is missing from {d}")
    return LateModel(config, weights_path(d), tokenizer_path(d, "late model"), dense_weights,
                     int(dense.get("out_features") or 0), bool(dense.get("bias", False)), normalize)
