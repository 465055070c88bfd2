"""ctypes binding of libinl_cuda.so (the C ABI in include/inl_cuda.h and
include/inl_cuda_kernels.h).

The library is the only compute path: when it is missing or fails to load,
every model call raises ``InferenceError``; nothing falls back to the CPU.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

from .errors import InlError, error_for_status

LIB_PATH = Path(os.environ.get("INL_CUDA_LIB", Path(__file__).with_name("libinl_cuda.so")))

INL_DTYPE_F32 = 0
INL_DTYPE_BF16 = 1
INL_MEM_HOST = 0
INL_MEM_DEVICE = 1

EPI_BF16, EPI_RESID, EPI_GATED, EPI_F32 = 0, 1, 2, 3
ACT_SILU, ACT_GELU_ERF, ACT_GELU_TANH = 0, 1, 2

# Every symbol the two public headers declare.
EXPORTED = (
    "inl_cuda_model_create", "inl_cuda_model_create_from_tensors", "inl_cuda_model_set_dense_head",
    "inl_cuda_forward_dense", "inl_cuda_forward_multivector", "inl_cuda_forward_sparse",
    "inl_cuda_forward_hidden", "inl_cuda_model_info", "inl_cuda_model_destroy", "inl_cuda_last_error",
    "inl_cuda_device_count", "inl_cuda_version", "inl_cuda_gemm_bf16", "inl_cuda_gemm_f32",
    "inl_cuda_attention", "inl_cuda_model_set_profiling", "inl_cuda_model_profile",
    "inl_cuda_model_launch_count", "inl_cuda_model_stream", "inl_cuda_embed_gather", "inl_cuda_norm",
    "inl_cuda_qk_norm_rope", "inl_cuda_token_positions", "inl_cuda_last_token_norm_l2", "inl_cuda_gemm_bf16_ex",
    "inl_cuda_attention_noalloc", "inl_cuda_causal_conv_silu", "inl_cuda_gated_delta_rule",
    "inl_cuda_model_set_dense_normalize", "inl_cuda_config_check", "inl_cuda_model_set_prune_last",
    "inl_cuda_forward_sparse_compact", "inl_cuda_model_set_f32_gemm",
)


class GemmEx(ctypes.Structure):
    """Mirror of inl_gemm_ex (include/inl_cuda_kernels.h)."""
    _fields_ = [
        ("A", ctypes.c_void_p), ("lda", ctypes.c_int64), ("W", ctypes.c_void_p), ("ldw", ctypes.c_int64),
        ("M", ctypes.c_int), ("N", ctypes.c_int), ("K", ctypes.c_int),
        ("epi", ctypes.c_int), ("act", ctypes.c_int), ("gate_block", ctypes.c_int),
        ("out", ctypes.c_void_p), ("ldo", ctypes.c_int64), ("resid", ctypes.c_void_p), ("ldr", ctypes.c_int64),
        ("ss_in", ctypes.c_void_p), ("ss_in_parts", ctypes.c_int), ("ss_dim", ctypes.c_int),
        ("ss_eps", ctypes.c_float), ("ss_out", ctypes.c_void_p),
        ("qn", ctypes.c_void_p), ("kn", ctypes.c_void_p), ("pos", ctypes.c_void_p), ("cos", ctypes.c_void_p),
        ("sin", ctypes.c_void_p), ("hq", ctypes.c_int), ("hkv", ctypes.c_int), ("d", ctypes.c_int),
        ("max_pos", ctypes.c_int), ("qk_eps", ctypes.c_float), ("force_bn", ctypes.c_int),
        ("status", ctypes.c_void_p),
    ]


class ModelInfo(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in (
        "arch", "dtype", "device", "hidden_size", "num_layers", "vocab_size", "dense_dim",
        "multivector_dim", "sparse_dim", "max_text_tokens", "is_causal")]


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None

c_int, c_void_p, c_float, c_double = ctypes.c_int, ctypes.c_void_p, ctypes.c_float, ctypes.c_double
c_i64, c_char_p = ctypes.c_int64, ctypes.c_char_p
P = ctypes.POINTER


def _declare(lib: ctypes.CDLL) -> None:
    sig = {
        "inl_cuda_model_create": (c_int, [c_char_p, c_char_p, c_int, c_int, P(c_void_p)]),
        "inl_cuda_model_create_from_tensors": (
            c_int, [c_char_p, c_int, P(c_char_p), P(c_void_p), P(c_i64), c_int, c_int, P(c_void_p)]),
        "inl_cuda_model_set_dense_head": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p]),
        "inl_cuda_model_set_dense_normalize": (c_int, [c_void_p, c_int]),
        "inl_cuda_config_check": (c_int, [c_char_p, c_int, c_void_p]),
        "inl_cuda_forward_dense": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_int]),
        "inl_cuda_forward_multivector": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int]),
        "inl_cuda_forward_sparse": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int]),
        "inl_cuda_forward_sparse_compact": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p,
                                                    c_void_p, c_i64, c_int]),
        "inl_cuda_forward_hidden": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_int]),
        "inl_cuda_model_info": (c_int, [c_void_p, P(ModelInfo)]),
        "inl_cuda_model_destroy": (None, [c_void_p]),
        "inl_cuda_last_error": (c_int, [ctypes.c_char_p, ctypes.c_size_t]),
        "inl_cuda_device_count": (c_int, []),
        "inl_cuda_version": (c_char_p, []),
        "inl_cuda_gemm_bf16": (c_int, [c_void_p, c_i64, c_void_p, c_i64, c_int, c_int, c_int, c_int, c_int, c_int,
                                       c_void_p, c_i64, c_void_p, c_i64, c_int, c_void_p, c_void_p]),
        "inl_cuda_gemm_f32": (c_int, [c_void_p, c_i64, c_void_p, c_i64, c_int, c_int, c_int, c_int, c_int,
                                      c_void_p, c_i64, c_void_p, c_i64, c_void_p]),
        "inl_cuda_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_i64, c_void_p, c_i64, c_int,
                                       c_int, c_int, c_int, c_float, c_int, c_int, c_void_p, c_int, c_void_p]),
        "inl_cuda_attention_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_i64, c_void_p, c_i64,
                                               c_int, c_int, c_int, c_int, c_float, c_int, c_int, c_void_p, c_int,
                                               c_void_p]),
        "inl_cuda_model_set_profiling": (c_int, [c_void_p, c_int]),
        "inl_cuda_model_set_prune_last": (c_int, [c_void_p, c_int]),
        "inl_cuda_model_set_f32_gemm": (c_int, [c_void_p, c_int]),
        "inl_cuda_model_profile": (c_int, [c_void_p, c_int, P(c_int), P(c_double), P(c_double)]),
        "inl_cuda_model_launch_count": (ctypes.c_longlong, [c_void_p, c_int]),
        "inl_cuda_model_stream": (c_void_p, [c_void_p]),
        "inl_cuda_gemm_bf16_ex": (c_int, [P(GemmEx), c_void_p]),
        "inl_cuda_embed_gather": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_float, c_void_p, c_int,
                                          c_void_p, c_void_p]),
        "inl_cuda_norm": (c_int, [c_void_p, c_int, c_i64, c_void_p, c_void_p, c_float, c_int, c_int, c_int, c_void_p,
                                  c_int, c_i64, c_void_p]),
        "inl_cuda_qk_norm_rope": (c_int, [c_void_p, c_int, c_i64, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                                          c_int, c_float, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p]),
        "inl_cuda_token_positions": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p]),
        "inl_cuda_last_token_norm_l2": (c_int, [c_void_p, c_int, c_i64, c_void_p, c_int, c_void_p, c_float, c_int,
                                                c_void_p, c_void_p]),
        "inl_cuda_causal_conv_silu": (c_int, [c_void_p, c_i64, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p,
                                              c_i64, c_void_p]),
        "inl_cuda_gated_delta_rule": (c_int, [c_void_p, c_i64, c_void_p, c_void_p, c_i64, c_void_p, c_i64, c_void_p,
                                              c_void_p, c_void_p, c_float, c_int, c_int, c_int, c_int, c_void_p,
                                              c_int, c_void_p, c_i64, c_void_p]),
    }
    for name, (res, args) in sig.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args


def lib() -> ctypes.CDLL:
    """Load libinl_cuda.so once; raise InferenceError if it is missing."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise InlError.inference(
                    f"libinl_cuda.so not found at {LIB_PATH}: build it with `python im-not-llm_b200/build.py`")
            try:
                handle = ctypes.CDLL(str(LIB_PATH))
            except OSError as e:  # pragma: no cover - depends on the host
                raise InlError.inference(f"cannot load {LIB_PATH}: {e}") from e
            _declare(handle)
            _lib = handle
        return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(4096)
    lib().inl_cuda_last_error(buf, len(buf))
    return buf.value.decode("utf-8", "replace")


def check(status: int, what: str) -> None:
    if status != 0:
        raise error_for_status(status, f"{what}: {last_error()}")
