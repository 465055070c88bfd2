"""A sharded checkpoint (model.safetensors.index.json) loads to the same
model as the single file: the tiny EmbeddingGemma 2 golden checkpoint split
in two shards, embeddings equal to the single-file load's bit for bit (the
shard list follows crates/inl-core/src/hub.rs:324-353); an index without a
weight_map is an inference error."""
import json
from pathlib import Path

import numpy as np
import pytest

import im_not_llm_b200 as inl

GOLDEN = Path(__file__).resolve().parent / "golden" / "tiny_embeddinggemma2"

pytestmark = pytest.mark.gpu


def test_sharded_checkpoint_loads_like_the_single_file(gpu, tmp_path):
    from safetensors.numpy import load_file, save_file

    cfg = json.loads((GOLDEN / "config.json").read_text())
    weights = load_file(str(GOLDEN / "model.safetensors"))
    names = sorted(weights)
    half = len(names) // 2
    shards = {"model-00001-of-00002.safetensors": names[:half], "model-00002-of-00002.safetensors": names[half:]}
    weight_map = {}
    for file, keys in shards.items():
        save_file({k: weights[k] for k in keys}, str(tmp_path / file))
        weight_map.update({k: file for k in keys})
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": weight_map}))
    ids = np.array([2, 5, 9, 11, 1, 2, 7, 1], dtype=np.uint32)
    cu = np.array([0, 5, 8], dtype=np.int32)
    single = inl.CudaModel(cfg, str(GOLDEN / "model.safetensors"), dtype="f32")
    sharded = inl.CudaModel(cfg, str(tmp_path / "model.safetensors.index.json"), dtype="f32")
    try:
        assert np.array_equal(single.embed(ids, cu), sharded.embed(ids, cu))
    finally:
        single.close()
        sharded.close()
    (tmp_path / "broken.index.json").write_text(json.dumps({"metadata": {}}))
    with pytest.raises(inl.InferenceError, match="weight_map"):
        inl.CudaModel(cfg, str(tmp_path / "broken.index.json"), dtype="f32")


def test_config_check_agrees_with_a_loaded_model(gpu):
    """inl_cuda_config_check reports what inl_cuda_model_info reports after
    the load (but the device and the late Dense width)."""
    cfg = json.loads((GOLDEN / "config.json").read_text())
    want = inl.config_check(cfg, "f32")
    m = inl.CudaModel(cfg, str(GOLDEN / "model.safetensors"), dtype="f32")
    try:
        got = m.info()
    finally:
        m.close()
    for key in ("arch", "dtype", "hidden_size", "num_layers", "vocab_size", "dense_dim", "sparse_dim",
                "max_text_tokens", "is_causal"):
        assert got[key] == want[key], key
