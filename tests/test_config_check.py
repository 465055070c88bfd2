"""The C config parser on the CPU, through inl_cuda_config_check: the checks
a model load makes before reading any weight (the reference's Config::parse /
validate of each tower, the SPLADE pooling block, the shapes the CUDA towers
take per dtype), on the reference's own fixture configs and edits of them."""
import copy
import json
from pathlib import Path

import pytest

import im_not_llm_b200 as inl

GOLDEN = Path(__file__).resolve().parent / "golden"


def _json(*parts):
    return json.loads(GOLDEN.joinpath(*parts).read_text())


def _gemma2():
    return _json("tiny_embeddinggemma2", "config.json")


def _splade():
    cfg = _json("tiny_splade", "config.json")
    cfg["splade"] = _json("tiny_splade", "1_ShiftedTopKSpladePooling", "config.json")
    return cfg


def _qwen35():
    return _json("tiny_qwen3_5_late", "config.json")


def _edit(cfg, path, value):
    out = copy.deepcopy(cfg)
    node = out
    for k in path[:-1]:
        node = node[k]
    if value is None:
        node.pop(path[-1], None)
    else:
        node[path[-1]] = value
    return out


def test_fixture_configs_parse_to_their_shapes():
    g = inl.config_check(_gemma2(), "f32")  # crates/inl-text/src/gemma2.rs:1074-1088
    assert (g["arch"], g["hidden_size"], g["num_layers"], g["dense_dim"], g["is_causal"]) == (2, 32, 6, 24, 0)
    s = inl.config_check(_splade(), "f32")
    assert (s["arch"], s["vocab_size"], s["sparse_dim"], s["max_text_tokens"]) == (1, 72, 62, 64)
    q = inl.config_check(_qwen35(), "f32")
    assert (q["arch"], q["is_causal"], q["device"], q["multivector_dim"]) == (3, 0, -1, 0)  # "is_causal": false
    d = inl.config_check(inl.synthetic.QWEN3_0_6B, "bf16")
    assert (d["arch"], d["dense_dim"], d["is_causal"]) == (0, 1024, 1)


@pytest.mark.parametrize("path,value", [
    (("text_config", "per_layer_config"), {"99": {"head_dim": 32}}),          # not a layer index
    (("text_config", "per_layer_config"), {"x": {"head_dim": 32}}),
    (("text_config", "per_layer_config"), {"02": {"head_dim": 33}}),          # odd head_dim
    (("text_config", "per_layer_config"), {"02": {"num_key_value_heads": 3}}),  # 4 heads over 3
    (("text_config", "per_layer_config"), {"02": {"head_dim": 64}}),          # full layers 2 and 5 differ
    (("text_config", "rope_parameters", "full_attention", "rope_type"), "yarn"),
    (("text_config", "hidden_activation"), "gelu"),
    (("text_config", "layer_types"), ["sliding_attention"] * 5),             # one short
    (("text_config", "hidden_size_per_layer_input"), -1),
])
def test_gemma2_config_refusals(path, value):
    """Config::validate (crates/inl-text/src/gemma2.rs:135-184)."""
    with pytest.raises(inl.ConfigError):
        inl.config_check(_edit(_gemma2(), path, value), "f32")


def test_gemma2_head_dims_per_dtype():
    """head_dim 16 / 32 run in f32 only; 64 / 128 / 256 in both."""
    with pytest.raises(inl.ConfigError, match="head_dim 16"):
        inl.config_check(_gemma2(), "bf16")
    wide = _edit(_edit(_gemma2(), ("text_config", "head_dim"), 64), ("text_config", "per_layer_config"),
                 {"02": {"head_dim": 128, "num_key_value_heads": 1}, "05": {"head_dim": 128, "num_key_value_heads": 1}})
    assert inl.config_check(wide, "bf16")["arch"] == 2


@pytest.mark.parametrize("path,value,message", [
    (("splade", "canonical_ids"), list(range(10)), "vocab_size entries"),
    (("splade", "prefix_token_ids"), [72], "outside the vocabulary"),
    (("splade", "masked_vocab_ids"), [500], "outside the vocabulary"),
    (("splade", "top_k"), 5, "top_k"),
    (("splade", "pooling_strategy"), "mean", "max pooling"),
    (("splade", "activation_function"), "softplus", "max pooling"),
    (("mlp_bias",), True, "biased"),
])
def test_splade_config_refusals(path, value, message):
    """SpladePooling::validate (crates/inl-sparse/src/modernbert.rs:747-775) and
    the ModernBERT config checks (:28-166)."""
    with pytest.raises(inl.ConfigError, match=message):
        inl.config_check(_edit(_splade(), path, value), "f32")


def test_splade_without_fold_and_head_dim_per_dtype():
    cfg = _edit(_splade(), ("splade", "canonical_ids"), None)
    assert inl.config_check(cfg, "f32")["sparse_dim"] == 72  # the vocabulary (:775-781)
    with pytest.raises(inl.ConfigError, match="head_dim 8"):  # 32 / 4 heads
        inl.config_check(_splade(), "bf16")


@pytest.mark.parametrize("path,value", [
    (("text_config", "rope_parameters", "rope_type"), "yarn"),
    (("text_config", "hidden_act"), "gelu"),
    (("text_config", "layer_types"), ["linear_attention"]),
])
def test_qwen35_config_refusals(path, value):
    """Qwen3.5 Config::validate (crates/inl-late/src/qwen3_5.rs:115-160)."""
    cfg = _qwen35()
    if "text_config" not in cfg:
        path = path[1:]
    with pytest.raises(inl.ConfigError):
        inl.config_check(_edit(cfg, path, value), "f32")


def test_qwen35_accepts_bf16_as_the_reference_does():
    """The reference's late engine takes f32 (default) or bf16
    (crates/inl-late/src/native.rs:232); the tower reports the dtype it was
    asked for."""
    from im_not_llm_b200 import _native as N

    assert inl.config_check(_qwen35(), "bf16")["dtype"] == N.INL_DTYPE_BF16
    assert inl.config_check(_qwen35(), "f32")["dtype"] == N.INL_DTYPE_F32


def test_malformed_configs():
    for bad in ({}, {"model_type": "llama", "hidden_size": 8}, {"model_type": "qwen3", "hidden_size": 12,
                                                                 "intermediate_size": 8, "num_attention_heads": 1,
                                                                 "num_hidden_layers": 1, "vocab_size": 8}):
        with pytest.raises(inl.ConfigError):
            inl.config_check(bad, "f32")
    with pytest.raises(inl.ConfigError):
        inl.config_check(inl.synthetic.QWEN3_TINY, "f16")


def test_null_arguments_are_config_errors():
    import ctypes

    from im_not_llm_b200 import _native as N

    info = N.ModelInfo()
    assert N.lib().inl_cuda_config_check(None, N.INL_DTYPE_F32, ctypes.byref(info)) == 1  # INL_ERR_CONFIG
    assert N.lib().inl_cuda_config_check(b"{}", N.INL_DTYPE_F32, None) == 1  # INL_ERR_CONFIG
    assert N.lib().inl_cuda_config_check(b"not json", N.INL_DTYPE_F32, ctypes.byref(info)) == 1  # INL_ERR_CONFIG
