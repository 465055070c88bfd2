"""One loaded model on one GPU, through the C ABI of libinl_cuda.so.

``CudaModel`` is the thin host handle the engine facades drive: it owns an
``inl_model*`` and turns packed token ids (``ids`` uint32 [T] and
``cu_seqlens`` int32 [n+1]) into dense embeddings, late-interaction vectors or
final hidden states. Host numpy arrays or device pointers (``int``) are both
accepted; device pointers let a caller keep inputs and outputs in HBM.
"""
from __future__ import annotations

import ctypes
import json
from pathlib import Path

import numpy as np

from . import _native as N
from .errors import InlError


def _dtype_code(dtype: str) -> int:
    if dtype in ("bf16", "bfloat16"):
        return N.INL_DTYPE_BF16
    if dtype in ("f32", "float32"):
        return N.INL_DTYPE_F32
    raise InlError.config(f"unsupported dtype '{dtype}': expected f32 or bf16")


def _ptr(a) -> tuple[int, int]:
    """(address, memory kind) of a numpy array or a raw device pointer."""
    if isinstance(a, int):
        return a, N.INL_MEM_DEVICE
    if isinstance(a, np.ndarray):
        return a.ctypes.data, N.INL_MEM_HOST
    raise TypeError(f"expected a numpy array or a device pointer, got {type(a).__name__}")


def config_check(config: dict, dtype: str = "bf16") -> dict:
    """Parse and validate ``config`` (a config.json dict; the SPLADE pooling
    block under "splade") for ``dtype`` without a GPU or weights, as a model
    load would before reading any weight. Returns the model's info fields
    (device -1, multivector_dim 0); a refused config raises its InlError."""
    i = N.ModelInfo()
    N.check(N.lib().inl_cuda_config_check(json.dumps(config).encode(), _dtype_code(dtype), ctypes.byref(i)),
            "config")
    return {f: getattr(i, f) for f, _ in N.ModelInfo._fields_}


class CudaModel:
    """A model resident on ``cuda:device``."""

    def __init__(self, config: dict, weights: dict | str | Path, device: int = 0, dtype: str = "bf16"):
        self.config = dict(config)
        self.dtype = dtype
        self.device = device
        lib = N.lib()
        handle = ctypes.c_void_p()
        cfg = json.dumps(self.config).encode()
        if isinstance(weights, (str, Path)):
            st = lib.inl_cuda_model_create(cfg, str(weights).encode(), device, _dtype_code(dtype),
                                           ctypes.byref(handle))
        else:
            names = list(weights.keys())
            arrays = [np.ascontiguousarray(weights[k], dtype=np.float32) for k in names]
            c_names = (ctypes.c_char_p * len(names))(*[k.encode() for k in names])
            c_data = (ctypes.c_void_p * len(names))(*[a.ctypes.data for a in arrays])
            c_numel = (ctypes.c_int64 * len(names))(*[a.size for a in arrays])
            st = lib.inl_cuda_model_create_from_tensors(cfg, len(names), c_names, c_data, c_numel, device,
                                                        _dtype_code(dtype), ctypes.byref(handle))
        N.check(st, "model load")
        self._h = handle

    # ------------------------------------------------------------------ info
    @property
    def handle(self) -> ctypes.c_void_p:
        if self._h is None:
            raise InlError.inference("model was unloaded")
        return self._h

    def info(self) -> dict:
        i = N.ModelInfo()
        N.check(N.lib().inl_cuda_model_info(self.handle, ctypes.byref(i)), "model info")
        return {f: getattr(i, f) for f, _ in N.ModelInfo._fields_}

    def set_dense_head(self, weight: np.ndarray, bias: np.ndarray | None = None, normalize: bool = True) -> None:
        """The late model's Dense projection [out, in] (+ bias); ``normalize``:
        whether the model has a Normalize module after it."""
        w = np.ascontiguousarray(weight, dtype=np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        N.check(N.lib().inl_cuda_model_set_dense_head(self.handle, w.ctypes.data, w.shape[0], w.shape[1],
                                                      None if b is None else b.ctypes.data), "Dense head")
        N.check(N.lib().inl_cuda_model_set_dense_normalize(self.handle, 1 if normalize else 0), "Dense head")

    @property
    def stream(self) -> int:
        return int(N.lib().inl_cuda_model_stream(self.handle) or 0)

    # --------------------------------------------------------------- forward
    @staticmethod
    def _inputs(ids, cu_seqlens):
        cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
        if isinstance(ids, int):
            return ids, N.INL_MEM_DEVICE, cu
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        return ids, N.INL_MEM_HOST, cu

    def embed(self, ids, cu_seqlens, out=None, out_dim: int = 0) -> np.ndarray | int:
        """Dense unit-length embeddings [n, H] f32 (last-token pooling)."""
        ids, ids_mem, cu = self._inputs(ids, cu_seqlens)
        n = len(cu) - 1
        if out is None:
            out = np.empty((n, out_dim or self.info()["dense_dim"]), dtype=np.float32)
        optr, omem = _ptr(out)
        iptr = ids if isinstance(ids, int) else ids.ctypes.data
        N.check(N.lib().inl_cuda_forward_dense(self.handle, iptr, ids_mem, cu.ctypes.data, n, out_dim, optr, omem),
                "dense forward")
        return out

    def encode_sparse(self, ids, cu_seqlens, out=None) -> np.ndarray | int:
        """SPLADE term weights, one dense row per text [n, sparse_dim] f32."""
        ids, ids_mem, cu = self._inputs(ids, cu_seqlens)
        n = len(cu) - 1
        if out is None:
            out = np.empty((n, self.info()["sparse_dim"]), dtype=np.float32)
        optr, omem = _ptr(out)
        iptr = ids if isinstance(ids, int) else ids.ctypes.data
        N.check(N.lib().inl_cuda_forward_sparse(self.handle, iptr, ids_mem, cu.ctypes.data, n, optr, omem),
                "sparse forward")
        return out

    def encode_sparse_compact(self, ids, cu_seqlens) -> list[tuple[np.ndarray, np.ndarray]]:
        """SPLADE terms compacted on the device: per text, (indices uint32
        ascending, weights f32) of its active terms (weight > 0). Only the
        active terms are copied to the host."""
        ids, ids_mem, cu = self._inputs(ids, cu_seqlens)
        n = len(cu) - 1
        offsets = np.zeros(n + 1, dtype=np.int64)
        cap = max(n * self.info()["sparse_dim"], 1)  # upper bound: every term of every text
        idx = np.empty(cap, dtype=np.int32)
        val = np.empty(cap, dtype=np.float32)
        iptr = ids if isinstance(ids, int) else ids.ctypes.data
        N.check(N.lib().inl_cuda_forward_sparse_compact(self.handle, iptr, ids_mem, cu.ctypes.data, n,
                                                        offsets.ctypes.data, idx.ctypes.data, val.ctypes.data, cap,
                                                        N.INL_MEM_HOST), "sparse forward")
        return [(idx[offsets[i]:offsets[i + 1]].astype(np.uint32), val[offsets[i]:offsets[i + 1]].copy())
                for i in range(n)]

    def encode_multivector(self, ids, cu_seqlens, out=None) -> np.ndarray | int:
        """Per-token late-interaction vectors [T, out_features] f32."""
        ids, ids_mem, cu = self._inputs(ids, cu_seqlens)
        n = len(cu) - 1
        if out is None:
            out = np.empty((int(cu[-1]), self.info()["multivector_dim"]), dtype=np.float32)
        optr, omem = _ptr(out)
        iptr = ids if isinstance(ids, int) else ids.ctypes.data
        N.check(N.lib().inl_cuda_forward_multivector(self.handle, iptr, ids_mem, cu.ctypes.data, n, optr, omem),
                "multivector forward")
        return out

    def hidden(self, ids, cu_seqlens, normalize_final: bool = True, out=None) -> np.ndarray | int:
        """Final hidden states [T, H] f32."""
        ids, ids_mem, cu = self._inputs(ids, cu_seqlens)
        n = len(cu) - 1
        if out is None:
            out = np.empty((int(cu[-1]), self.config["hidden_size"]), dtype=np.float32)
        optr, omem = _ptr(out)
        iptr = ids if isinstance(ids, int) else ids.ctypes.data
        N.check(N.lib().inl_cuda_forward_hidden(self.handle, iptr, ids_mem, cu.ctypes.data, n,
                                                1 if normalize_final else 0, optr, omem), "hidden forward")
        return out

    def set_f32_gemm(self, mode: str) -> None:
        """f32 models: "3xbf16" (default) runs the contractions on the tensor
        cores over split bf16 operands; "ffma" on the SIMT f32 kernels."""
        N.check(N.lib().inl_cuda_model_set_f32_gemm(self.handle, {"ffma": 0, "3xbf16": 1}[mode]), "f32 GEMM mode")

    def set_prune_last(self, enable: bool) -> None:
        """Causal last-token pooling runs the last layer's attention, o and
        MLP only where the pooled row needs them (default on); off runs that
        layer on every row."""
        N.check(N.lib().inl_cuda_model_set_prune_last(self.handle, 1 if enable else 0), "prune_last")

    # ----------------------------------------------------------- measurement
    def set_profiling(self, enable: bool) -> None:
        N.check(N.lib().inl_cuda_model_set_profiling(self.handle, 1 if enable else 0), "profiling")

    def profile(self, kind: int = -1) -> dict:
        n = ctypes.c_int()
        ms = ctypes.c_double()
        fl = ctypes.c_double()
        N.check(N.lib().inl_cuda_model_profile(self.handle, kind, ctypes.byref(n), ctypes.byref(ms),
                                               ctypes.byref(fl)), "profile")
        return {"launches": n.value, "ms": ms.value, "flops": fl.value}

    def launch_count(self, reset: bool = False) -> int:
        return int(N.lib().inl_cuda_model_launch_count(self.handle, 1 if reset else 0))

    # --------------------------------------------------------------- release
    def close(self) -> None:
        if self._h is not None:
            N.lib().inl_cuda_model_destroy(self._h)
            self._h = None

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass
