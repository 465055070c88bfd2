"""im-not-llm B200: the packed variable-length encoder forward of im-not-llm's
embedding engines on sm_100a, behind a C ABI (libinl_cuda.so) and a Python
host layer that mirrors the reference's engine API."""
from .errors import (ConfigError, InferenceError, InlError, InvalidInputError,  # noqa: F401
                     TimeoutError_)
from .model import CudaModel, config_check  # noqa: F401
from .engine import (BatchDeadline, DataParallelEmbedder, EngineInfo, LateEncoder, LateTask,  # noqa: F401
                     SparseEncoder, SparseVector, TextEmbedder, TextIdentity, TextOptions)
from .text import Gemma2Task, TextTokenizer, gemma2_document  # noqa: F401
from . import loading, planner, synthetic, text  # noqa: F401

__all__ = [
    "BatchDeadline", "ConfigError", "CudaModel", "DataParallelEmbedder", "EngineInfo", "Gemma2Task", "InferenceError",
    "InlError", "InvalidInputError", "LateEncoder", "LateTask", "SparseEncoder", "SparseVector", "TextEmbedder", "TextIdentity", "TextOptions",
    "TextTokenizer", "TimeoutError_", "config_check", "gemma2_document", "loading", "planner", "synthetic", "text",
]
