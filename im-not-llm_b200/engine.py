"""Engine facades over libinl_cuda, mirroring the reference's engine API.

* ``TextEmbedder`` — the DenseEngine contract (load / token_counts / embed /
  unload / is_loaded; crates/inl-core/src/engine.rs:66-84) as
  crates/inl-text/src/native.rs implements it: truncate to ``max_length``,
  plan batches, one forward at a time behind a gate, each forward under a
  ``BatchDeadline``, vectors returned in input order, count mismatch is an
  error, Matryoshka ``output_dim`` only for EmbeddingGemma-style models.
* ``LateEncoder`` — the LateEngine contract (crates/inl-late/src/lib.rs:38-55;
  encode path crates/inl-late/src/native.rs:317-374,631-683): longest-first
  planning, per-token vectors, non-finite output is an error.
* ``SparseEncoder`` — the SparseEngine contract (crates/inl-sparse/src/lib.rs:236-252;
  encode path crates/inl-sparse/src/native.rs:349-544): longest-first packed
  batches, ``SparseVector`` results (positive weights only, sorted term ids),
  non-finite output is an error.
* ``DataParallelEmbedder`` — one model per GPU, one host thread per GPU,
  packed batches assigned longest-processing-time first; no collective;
  dense ``embed``, ``encode_sparse`` and ``encode_late``.

Inputs are strings or token-id lists. Strings go through the model's
tokenizer.json (``text.TextTokenizer``, the reference's settings: special
tokens, truncation by the tokenizer) with the query / passage prefixes of the
reference's options. Token-id lists are truncated to ``max_length``.
"""
from __future__ import annotations

import dataclasses
import json
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from pathlib import Path
from typing import Callable, Sequence

import numpy as np

from . import loading
from .errors import InlError
from .model import CudaModel
from .planner import assign_lpt, batch_cost, longest_first, pack, plan_packed
from .text import TextTokenizer

DEFAULT_MAX_LENGTH = 2048          # crates/inl-text/src/native.rs:23
DEFAULT_BATCH_SIZE = 64            # crates/inl-text/src/native.rs:26
DEFAULT_TIMEOUT_SECONDS = 60       # crates/inl-text/src/native.rs:32
DEFAULT_PACKED_TOKENS = 65536      # packed real tokens per forward on one B200
MATRYOSHKA_DIMS = (128, 256, 512, 768)  # crates/inl-text/src/native.rs:82-88
SPARSE_QUERY_PREFIX = "[Q] "       # crates/inl-sparse/src/native.rs:44
SPARSE_PASSAGE_PREFIX = "[D] "     # crates/inl-sparse/src/native.rs:45


class BatchDeadline:
    """Deadline for non-cancellable forward passes (crates/inl-core/src/deadline.rs:17-60).

    ``run`` executes ``task`` on a worker thread and waits at most ``budget``
    seconds; after one expiry the deadline is wedged and every later call fails
    fast with a timeout error without running its task.
    """

    def __init__(self):
        self._wedged = threading.Event()

    def ensure_healthy(self, what: str) -> None:
        if self._wedged.is_set():
            raise InlError.timeout(
                f"{what}: an earlier call timed out and its thread is still stuck; restart the process")

    @property
    def wedged(self) -> bool:
        return self._wedged.is_set()

    def run(self, what: str, budget: float, task: Callable[[], object]):
        self.ensure_healthy(what)
        box: dict = {}

        def body():
            try:
                box["value"] = task()
            except BaseException as e:  # surfaced to the caller below
                box["error"] = e

        t = threading.Thread(target=body, name=f"inl-forward:{what}", daemon=True)
        t.start()
        t.join(budget)
        if t.is_alive():
            self._wedged.set()
            raise InlError.timeout(
                f"{what} exceeded {budget:.3f}s; its thread cannot be cancelled — restart the process")
        if "error" in box:
            e = box["error"]
            if isinstance(e, InlError):
                raise e
            raise InlError.inference(f"{what}: blocking task failed: {e}") from e
        return box.get("value")


@dataclass
class EngineInfo:
    """crates/inl-core/src/engine.rs:10-26."""
    model_id: str
    dimension: int
    dtype: str
    device: str
    attention: str
    max_length: int
    modalities: list = field(default_factory=lambda: ["text"])


@dataclass(frozen=True)
class TextIdentity:
    """The embedding space of a TextEmbedder (crates/inl-text/src/native.rs:156-167):
    model id, output dimension, resolved dtype, device kind, context."""
    id: str
    dimension: int
    dtype: str
    device: str
    max_length: int


@dataclass
class TextOptions:
    """Subset of TextOptions (crates/inl-text/src/native.rs:172-287) that the
    packed GPU path uses."""
    id: str = "synthetic"
    batch_size: int = 4096               # texts per packed forward
    max_batch_tokens: int = DEFAULT_PACKED_TOKENS
    max_length: int = DEFAULT_MAX_LENGTH
    timeout_seconds: float = DEFAULT_TIMEOUT_SECONDS
    per_batch_timeout_seconds: float | None = None
    output_dim: int | None = None
    query_prefix: str | None = None    # prepended to string queries (embed_query / encode_query)
    passage_prefix: str | None = None  # prepended to string inputs of embed / encode

    @classmethod
    def sparse(cls, **kw) -> "TextOptions":
        """The sparse encoder's defaults: the "[Q] " / "[D] " markers
        (SparseOptions::default, crates/inl-sparse/src/native.rs:80-95)."""
        kw.setdefault("query_prefix", SPARSE_QUERY_PREFIX)
        kw.setdefault("passage_prefix", SPARSE_PASSAGE_PREFIX)
        return cls(**kw)

    def batch_timeout(self) -> float:
        """crates/inl-text/src/native.rs:739-752."""
        s = self.per_batch_timeout_seconds if self.per_batch_timeout_seconds is not None else self.timeout_seconds
        if not s or s <= 0:
            raise InlError.config("timeout_seconds / per_batch_timeout_seconds must be greater than 0")
        return float(s)


def _truncate(tokens: Sequence[Sequence[int]], max_length: int) -> list[np.ndarray]:
    return [np.asarray(t, dtype=np.uint32)[:max_length] for t in tokens]


class _Loaded:
    def __init__(self, model: CudaModel):
        self.model = model
        self.gate = threading.Lock()


def _check_encoder_options(options: TextOptions) -> None:
    """The sparse and late encoders refuse these options when they are built
    (crates/inl-sparse/src/native.rs:197-210, crates/inl-late/src/native.rs:184-197)."""
    s = options.per_batch_timeout_seconds if options.per_batch_timeout_seconds is not None else options.timeout_seconds
    if not s or s <= 0:
        raise InlError.config("timeout_seconds / per_batch_timeout_seconds must be greater than 0 for the native "
                              "encoder")
    if options.batch_size <= 0:
        raise InlError.config("batch_size must be greater than 0")


class _EngineBase:
    def __init__(self, loader: Callable[[], CudaModel], options: TextOptions,
                 tokenizer: TextTokenizer | None = None):
        self._loader = loader
        self.options = options
        self.tokenizer = tokenizer
        self.deadline = BatchDeadline()
        self._load_lock = threading.Lock()
        self._loaded: _Loaded | None = None

    def _model(self) -> _Loaded:
        with self._load_lock:  # concurrent callers share one load; failures are not cached
            if self._loaded is None:
                self._loaded = _Loaded(self._loader())
            return self._loaded

    def is_loaded(self) -> bool:
        return self._loaded is not None

    def unload(self) -> bool:
        with self._load_lock:
            if self._loaded is None:
                return False
            with self._loaded.gate:
                self._loaded.model.close()
            self._loaded = None
            return True

    def _is_text(self, inputs: list) -> bool:
        kinds = {isinstance(x, str) for x in inputs}
        if len(kinds) > 1:
            raise InlError.invalid_input("inputs mix strings and token-id lists")
        if kinds == {True} and self.tokenizer is None:
            raise InlError.config("string inputs need a tokenizer (tokenizer=TextTokenizer.from_file(...))")
        return kinds == {True}

    def _prepare(self, inputs: Sequence, prefix: str | None) -> list[np.ndarray]:
        """Strings: prefix prepended, then tokenized (the tokenizer truncates
        to max_length). Token-id lists: truncated to max_length."""
        items = list(inputs)
        if self._is_text(items):
            if prefix:
                items = [prefix + t for t in items]
            return self.tokenizer.encode(items, self.options.max_length)
        return _truncate(items, self.options.max_length)

    def token_counts(self, inputs: Sequence) -> list[int]:
        """Tokens per input before truncation, as given (no prefix;
        crates/inl-text/src/native.rs:502-520)."""
        items = list(inputs)
        if self._is_text(items):
            return self.tokenizer.counts(items)
        return [len(t) for t in items]

    def _run_batches(self, what: str, texts: list[np.ndarray], forward) -> list:
        if not texts:
            return []
        if self.options.batch_size <= 0:  # crates/inl-text/src/native.rs:552-556
            raise InlError.inference("batch_size must be greater than 0")
        self.deadline.ensure_healthy(what)
        loaded = self._model()
        budget = self.options.batch_timeout()
        lengths = [len(t) for t in texts]
        order = longest_first(lengths)
        sorted_lengths = [lengths[i] for i in order]
        results: list = [None] * len(texts)
        for r in plan_packed(sorted_lengths, self.options.max_batch_tokens, self.options.batch_size):
            members = [order[k] for k in r]
            ids, cu = pack(texts, members)
            with loaded.gate:  # queue before the deadline starts (crates/inl-text/src/native.rs:668)
                out = self.deadline.run(f"{what} batch", budget, lambda: forward(loaded.model, ids, cu))
            if len(out) != len(members):
                raise InlError.inference(f"{what} returned {len(out)} results for {len(members)} inputs")
            for i, v in zip(members, out):
                results[i] = v
        return results


class TextEmbedder(_EngineBase):
    """DenseEngine over a CudaModel (Qwen3 last-token or Gemma-style mean pooling)."""

    @classmethod
    def from_model_dir(cls, model_dir: str | Path, options: TextOptions | None = None, device: int = 0,
                       dtype: str | None = None) -> "TextEmbedder":
        """A Qwen3 or EmbeddingGemma 2 model directory (config.json, weights,
        tokenizer.json), loaded on first use; dtype defaults to bf16 for Qwen3
        and f32 for EmbeddingGemma 2 (crates/inl-text/src/native.rs:406-470, 871-890)."""
        spec = loading.dense_model(model_dir, dtype)
        return cls(lambda: CudaModel(spec.config, spec.weights, device, spec.dtype), options or TextOptions(),
                   tokenizer=TextTokenizer.from_file(spec.tokenizer))

    def load(self) -> EngineInfo:
        """Loads the model; a requested output_dim the model cannot give is a
        config error here, as at the reference's load (native.rs:438-440)."""
        m = self._model().model
        dim = self._output_dim(m) or m.info()["dense_dim"]
        return EngineInfo(self.options.id, dim, m.dtype, f"cuda:{m.device}", "fused", self.options.max_length)

    def identity(self) -> "TextIdentity":
        """The embedding space this embedder produces; loads the model
        (crates/inl-text/src/native.rs:476-488)."""
        info = self.load()
        return TextIdentity(self.options.id, info.dimension, info.dtype, "cuda", self.options.max_length)

    def _output_dim(self, model: CudaModel) -> int:
        """resolve_output_dim (crates/inl-text/src/native.rs:793-817)."""
        dim = self.options.output_dim
        if dim is None:
            return 0
        if model.info()["arch"] != 2:
            raise InlError.config("output_dim is only supported for EmbeddingGemma 2 models")
        if dim not in MATRYOSHKA_DIMS:
            raise InlError.config(f"output_dim {dim} is not supported by EmbeddingGemma 2: use one of "
                                  f"{list(MATRYOSHKA_DIMS)}")
        if dim > model.info()["dense_dim"]:
            raise InlError.config(f"output_dim {dim} exceeds the model's embeddings")
        return dim

    def embed(self, inputs: Sequence) -> list[np.ndarray]:
        """Passages (strings get the passage prefix) or token-id lists."""
        return self._embed(self._prepare(inputs, self.options.passage_prefix))

    def count_truncated(self, texts: Sequence[str]) -> int:
        """How many of ``texts`` (passage prefix applied) reach ``max_length``
        tokens and are therefore truncated (crates/inl-text/src/native.rs:372-404).
        Texts shorter than ``max_length`` UTF-8 bytes are skipped untokenized,
        as there: byte-level BPE gives at most one token per byte."""
        prefix = self.options.passage_prefix or ""
        cands = [prefix + t for t in texts if len((prefix + t).encode()) >= self.options.max_length]
        if not cands:
            return 0
        if self.tokenizer is None:
            raise InlError.config("count_truncated needs a tokenizer")
        return sum(n >= self.options.max_length for n in self.tokenizer.counts(cands))

    def embed_query(self, text: str) -> np.ndarray:
        """One search query with the query prefix (crates/inl-text/src/native.rs:534-546)."""
        out = self._embed(self._prepare([text], self.options.query_prefix))
        if not out:
            raise InlError.inference("empty response")
        return out[0]

    def _embed(self, texts: list[np.ndarray]) -> list[np.ndarray]:
        if not texts:
            return []
        out_dim = self._output_dim(self._model().model)

        def forward(model: CudaModel, ids, cu):
            return list(model.embed(ids, cu, out_dim=out_dim))

        return self._run_batches("native embedding", texts, forward)


@dataclass(frozen=True)
class LateTask:
    """TaskSetup (crates/inl-late/src/native.rs:122-128): the prompt put in
    front of string inputs, the context in tokens (prompt included), and the
    token ids whose vectors are dropped from the output."""
    prompt: str = ""
    length: int = DEFAULT_MAX_LENGTH
    skip: frozenset = frozenset()

    @staticmethod
    def from_model_dir(model_dir: str | Path, tokenizer: TextTokenizer,
                       max_length: int | None = None) -> dict[str, "LateTask"]:
        """Query and document setups of a Sentence-Transformers late model
        directory, as crates/inl-late/src/native.rs:455-620 reads them:
        prompts from config_sentence_transformers.json; query_length /
        document_length from sentence_bert_config.json (else max_seq_length,
        else the model's max_position_embeddings), capped by ``max_length``
        and the positions; the MultiVectorMask module's skiplist (a word
        counts only when it is one vocabulary token; tasks default to
        ["document"]; keep_only_token_ids is not supported)."""
        d = Path(model_dir)

        def read(name, default):
            f = d / name
            return json.loads(f.read_text()) if f.exists() else default

        cfg = read("config.json", {})
        positions = cfg.get("max_position_embeddings") or cfg.get("text_config", {}).get("max_position_embeddings")
        st = read("sentence_bert_config.json", {})
        prompts = read("config_sentence_transformers.json", {}).get("prompts") or {}
        mask = {"skiplist_words": [], "skiplist_tasks": []}
        for module in read("modules.json", []):
            if module.get("type", "").rsplit(".", 1)[-1] == "MultiVectorMask":
                mask = read(str(Path(module.get("path", "")) / "config.json"), {})
        if mask.get("keep_only_token_ids") is not None:
            raise InlError.inference("native late model keep_only_token_ids is not supported")
        ids = (tokenizer.token_to_id(w) for w in mask.get("skiplist_words", []))
        skip = frozenset(i for i in ids if i is not None)
        skip_tasks = mask.get("skiplist_tasks", ["document"])
        fallback = st.get("max_seq_length") or positions or DEFAULT_MAX_LENGTH

        def cap(length):
            v = length if length is not None else fallback
            if max_length is not None:
                v = min(v, max_length)
            return min(v, positions) if positions else v

        return {name: LateTask(prompts.get(name) or "", cap(st.get(f"{name}_length")),
                               skip if name in skip_tasks else frozenset())
                for name in ("query", "document")}


class LateEncoder(_EngineBase):
    """LateEngine over a CudaModel with a Dense head attached:
    ``encode(inputs, task)`` with task "query" or "document"
    (crates/inl-late/src/native.rs:292-374, 631-683). String inputs get the
    task's prompt and are cut at the task's length after tokenizing (the
    tokenizer does not truncate); token-id lists are cut at the task's
    length. The vectors of the task's skiplist tokens are dropped, and a
    non-finite kept value is an error."""

    TASKS = ("query", "document")

    @classmethod
    def from_model_dir(cls, model_dir: str | Path, options: TextOptions | None = None, device: int = 0,
                       dtype: str = "f32", max_length: int | None = None) -> "LateEncoder":
        """A Sentence-Transformers late-interaction directory (Transformer,
        Dense, optional MultiVectorMask and Normalize modules), loaded on first
        use: the tower, its Dense head (+ bias) and the Normalize flag; task
        prompts, lengths and skiplist from the directory
        (crates/inl-late/src/native.rs:455-620)."""
        spec = loading.late_model(model_dir)
        tok = TextTokenizer.from_file(spec.tokenizer)
        tasks = LateTask.from_model_dir(model_dir, tok, max_length)

        def load() -> CudaModel:
            from safetensors.numpy import load_file

            try:
                dense = load_file(str(spec.dense_weights))
            except Exception as e:
                raise InlError.inference(f"native late model Dense weight load failed: {e}") from e
            if "linear.weight" not in dense or (spec.dense_bias and "linear.bias" not in dense):
                raise InlError.inference("native late model Dense weight load failed: linear.weight / linear.bias")
            m = CudaModel(spec.config, spec.weights, device, dtype)
            try:
                m.set_dense_head(dense["linear.weight"], dense["linear.bias"] if spec.dense_bias else None,
                                 normalize=spec.normalize)
            except BaseException:
                m.close()
                raise
            return m

        return cls(load, options or TextOptions(), tokenizer=tok, tasks=tasks)

    def __init__(self, loader: Callable[[], CudaModel], options: TextOptions,
                 tokenizer: TextTokenizer | None = None, tasks: dict[str, LateTask] | None = None):
        _check_encoder_options(options)
        if options.max_length <= 0:  # crates/inl-late/src/native.rs:198-202
            raise InlError.config("max_length must be greater than 0")
        super().__init__(loader, options, tokenizer)
        default = LateTask(length=options.max_length)
        self.tasks = {name: (tasks or {}).get(name, default) for name in self.TASKS}

    def load(self) -> EngineInfo:
        m = self._model().model
        return EngineInfo(self.options.id, m.info()["multivector_dim"], m.dtype, f"cuda:{m.device}", "fused",
                          self.tasks["document"].length)

    def identity(self) -> EngineInfo:
        """The token-vector space; loads the model; max_length is the
        document context (crates/inl-late/src/native.rs:256-270)."""
        return self.load()

    def _setup(self, task: str) -> LateTask:
        setup = self.tasks.get(task)
        if setup is None:
            raise InlError.invalid_input(f"unknown late task {task!r}: use 'query' or 'document'")
        return setup

    def _rows(self, inputs: Sequence, setup: LateTask) -> list[np.ndarray]:
        """Strings: the task's prompt in front, tokenized, cut at the task's
        length (native.rs:292-305); token-id lists: cut at the task's length."""
        items = list(inputs)
        if self._is_text(items):
            return [ids[:setup.length] for ids in self.tokenizer.encode_untruncated([setup.prompt + t for t in items])]
        return _truncate(items, setup.length)

    def token_counts(self, inputs: Sequence, task: str = "document") -> list[int]:
        """Tokens the model sees per input for ``task``: prompt included,
        after the task's truncation (LateEngine::token_counts,
        crates/inl-late/src/lib.rs:44-46, native.rs:727-735)."""
        return [len(r) for r in self._rows(inputs, self._setup(task))]

    def encode(self, inputs: Sequence, task: str = "document") -> list[np.ndarray]:
        setup = self._setup(task)
        rows = self._rows(inputs, setup)
        skip = np.fromiter(sorted(setup.skip), dtype=np.uint32) if setup.skip else None

        def forward(model: CudaModel, ids, cu):
            flat = model.encode_multivector(ids, cu)
            out = []
            for i in range(len(cu) - 1):
                m = flat[cu[i]:cu[i + 1]]
                if skip is not None:
                    m = m[~np.isin(ids[cu[i]:cu[i + 1]], skip)]
                if not np.all(np.isfinite(m)):  # crates/inl-late/src/native.rs:675-679
                    raise InlError.inference("native late encoder produced non-finite values")
                out.append(m)
            return out

        return self._run_batches("native late", rows, forward)


class SparseVector:
    """Term ids strictly ascending, every weight finite and > 0 (a zero weight
    is the absence of a term): SparseVector, crates/inl-sparse/src/lib.rs:13-90."""

    __slots__ = ("indices", "values")

    def __init__(self, indices: np.ndarray, values: np.ndarray):
        self.indices = indices
        self.values = values

    @classmethod
    def new(cls, indices, values) -> "SparseVector":
        """Validate and wrap parallel indices / values (lib.rs:24-46)."""
        idx = np.asarray(indices, dtype=np.uint32)
        val = np.asarray(values, dtype=np.float32)
        if idx.shape != val.shape or idx.ndim != 1:
            raise InlError.inference(f"sparse vector has {idx.size} indices but {val.size} values")
        bad = np.nonzero(idx[1:] <= idx[:-1])[0]
        if bad.size:
            raise InlError.inference(f"sparse vector indices must be strictly ascending (saw {idx[bad[0]]} then "
                                     f"{idx[bad[0] + 1]})")
        wrong = np.nonzero(~(np.isfinite(val) & (val > 0)))[0]
        if wrong.size:
            raise InlError.inference(f"sparse vector weights must be finite and positive (saw {val[wrong[0]]})")
        return cls(idx, val)

    @classmethod
    def from_pairs(cls, pairs) -> "SparseVector":
        """Sort by index, keep the largest weight of a repeated index, drop
        weights that are not finite and positive; never fails (lib.rs:48-62)."""
        best: dict[int, float] = {}
        for i, w in pairs:
            w = float(np.float32(w))
            if np.isfinite(w) and w > 0 and w > best.get(int(i), 0.0):
                best[int(i)] = w
        keys = sorted(best)
        return cls(np.asarray(keys, dtype=np.uint32), np.asarray([best[k] for k in keys], dtype=np.float32))

    def is_empty(self) -> bool:
        return len(self.indices) == 0

    def __eq__(self, other) -> bool:
        return (isinstance(other, SparseVector) and np.array_equal(self.indices, other.indices)
                and np.array_equal(self.values, other.values))

    def to_json(self) -> str:
        """{"indices": [...], "values": [...]} (the serde form of lib.rs:18)."""
        return json.dumps({"indices": [int(i) for i in self.indices], "values": [float(v) for v in self.values]})

    @classmethod
    def from_json(cls, text: str) -> "SparseVector":
        """Parses and re-validates (lib.rs:92-110)."""
        try:
            d = json.loads(text)
            return cls.new(d["indices"], d["values"])
        except (ValueError, KeyError, TypeError) as e:
            raise InlError.inference(f"sparse vector JSON is invalid: {e}") from e

    @classmethod
    def from_dense(cls, row: np.ndarray) -> "SparseVector":
        idx = np.nonzero(row > 0)[0].astype(np.uint32)
        return cls(idx, row[idx].astype(np.float32))

    def dot(self, other: "SparseVector") -> float:
        """dot_terms (crates/inl-sparse/src/lib.rs:64-90)."""
        common, ia, ib = np.intersect1d(self.indices, other.indices, assume_unique=True, return_indices=True)
        return float(np.dot(self.values[ia], other.values[ib])) if len(common) else 0.0

    def __len__(self) -> int:
        return len(self.indices)


def _sparse_forward(model, ids, cu) -> list[SparseVector]:
    """One batch of SPLADE vectors: the active terms are compacted on the
    device (ascending term ids, weights > 0) and only they cross to the host.
    A non-finite weight is an inference error, as in the reference
    (crates/inl-sparse/src/native.rs:536-540)."""
    try:
        pairs = model.encode_sparse_compact(ids, cu)
    except InlError as e:
        if "non-finite" in str(e):
            raise InlError.inference("native sparse encoder produced non-finite weights") from e
        raise
    return [SparseVector(idx, val) for idx, val in pairs]


class SparseEncoder(_EngineBase):
    """SparseEngine over a ModernBERT + SPLADE CudaModel."""

    def __init__(self, loader: Callable[[], CudaModel], options: TextOptions, tokenizer: TextTokenizer | None = None):
        _check_encoder_options(options)
        super().__init__(loader, options, tokenizer)

    @classmethod
    def from_model_dir(cls, model_dir: str | Path, options: TextOptions | None = None, device: int = 0,
                       dtype: str = "f32") -> "SparseEncoder":
        """A Sentence-Transformers SPLADE directory (config.json, modules.json
        and its SPLADE pooling module, weights, tokenizer.json), loaded on
        first use; the context is capped by max_position_embeddings
        (crates/inl-sparse/src/native.rs:245, 424-500)."""
        spec = loading.sparse_model(model_dir)
        opts = options or TextOptions.sparse()
        if spec.positions and opts.max_length > spec.positions:
            opts = dataclasses.replace(opts, max_length=spec.positions)
        return cls(lambda: CudaModel(spec.config, spec.weights, device, dtype), opts,
                   tokenizer=TextTokenizer.from_file(spec.tokenizer))

    def load(self) -> EngineInfo:
        m = self._model().model
        return EngineInfo(self.options.id, m.info()["sparse_dim"], m.dtype, f"cuda:{m.device}", "fused",
                          self.options.max_length)

    def identity(self) -> EngineInfo:
        """The sparse space; loads the model (crates/inl-sparse/src/native.rs:271-283)."""
        return self.load()

    def encode(self, inputs: Sequence) -> list[SparseVector]:
        """Documents (strings get the passage marker) or token-id lists."""
        return self._encode(self._prepare(inputs, self.options.passage_prefix))

    def count_truncated(self, texts: Sequence[str]) -> int:
        """How many of ``texts`` reach the context limit once the passage
        marker and special tokens are counted (crates/inl-sparse/src/native.rs:319-348):
        texts shorter than ``max_length`` UTF-8 bytes are skipped, the rest are
        tokenized with truncation and counted when they come back at the limit."""
        cands = [(self.options.passage_prefix or "") + t for t in texts
                 if len(t.encode()) >= self.options.max_length]
        if not cands:
            return 0
        if self.tokenizer is None:
            raise InlError.config("count_truncated needs a tokenizer")
        return sum(len(ids) >= self.options.max_length
                   for ids in self.tokenizer.encode(cands, self.options.max_length))

    def encode_query(self, text: str) -> SparseVector:
        """One query with the query marker (crates/inl-sparse/src/native.rs:310-317)."""
        out = self._encode(self._prepare([text], self.options.query_prefix))
        if not out:
            raise InlError.inference("empty response")
        return out[0]

    def _encode(self, texts: list[np.ndarray]) -> list[SparseVector]:
        return self._run_batches("native sparse", texts, _sparse_forward)


class DataParallelEmbedder:
    """Dense, sparse or late encoding over several GPUs: one CudaModel replica
    and one host thread per device, batches assigned longest-processing-time
    first, no collective; results gathered on the host by input index. The
    per-batch checks are those of the single-GPU engines (result count,
    finite sparse and late outputs)."""

    def __init__(self, models: Sequence[CudaModel], max_batch_tokens: int = DEFAULT_PACKED_TOKENS,
                 tokenizer: TextTokenizer | None = None, max_length: int = DEFAULT_MAX_LENGTH,
                 passage_prefix: str | None = None):
        self.models = list(models)
        self.max_batch_tokens = max_batch_tokens
        self.tokenizer = tokenizer
        self.max_length = max_length
        self.passage_prefix = passage_prefix

    def _texts(self, inputs: Sequence, prefix: str | None, max_length: int, cut_after: bool = False) -> list:
        """Strings (prefix, tokenized and truncated by the tokenizer, or cut
        after tokenizing for the late tasks) or token-id lists (truncated)."""
        items = list(inputs)
        kinds = {isinstance(x, str) for x in items}
        if len(kinds) > 1:
            raise InlError.invalid_input("inputs mix strings and token-id lists")
        if kinds == {True}:
            if self.tokenizer is None:
                raise InlError.config("string inputs need a tokenizer (tokenizer=TextTokenizer.from_file(...))")
            prefixed = [(prefix or "") + t for t in items]
            if cut_after:
                return [ids[:max_length] for ids in self.tokenizer.encode_untruncated(prefixed)]
            return self.tokenizer.encode(prefixed, max_length)
        return _truncate(items, max_length)

    def _run(self, what: str, texts: list, forward) -> list:
        lengths = [len(t) for t in texts]
        order = longest_first(lengths)
        batches = [[order[k] for k in r] for r in plan_packed([lengths[i] for i in order], self.max_batch_tokens)]
        causal = bool(self.models[0].info()["is_causal"]) if self.models else True
        costs = [batch_cost([lengths[i] for i in b], causal) for b in batches]
        plan = assign_lpt(costs, len(self.models))
        results: list = [None] * len(texts)
        errors: list = []

        def worker(w: int):
            # The next batch is packed on a helper thread while this one runs:
            # the forward call releases the GIL for its whole duration.
            try:
                mine = plan[w]
                with ThreadPoolExecutor(max_workers=1) as packer:
                    nxt = packer.submit(pack, texts, batches[mine[0]]) if mine else None
                    for k, b in enumerate(mine):
                        ids, cu = nxt.result()
                        if k + 1 < len(mine):
                            nxt = packer.submit(pack, texts, batches[mine[k + 1]])
                        out = forward(self.models[w], ids, cu)
                        if len(out) != len(batches[b]):  # crates/inl-text/src/native.rs:674-679
                            raise InlError.inference(f"{what} returned {len(out)} results for {len(batches[b])} inputs")
                        for i, v in zip(batches[b], out):
                            results[i] = v
            except BaseException as e:
                errors.append(e)

        threads = [threading.Thread(target=worker, args=(w,)) for w in range(len(self.models))]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        if errors:
            raise errors[0]
        return results

    def embed(self, inputs: Sequence) -> list[np.ndarray]:
        """Dense unit vectors, one per input."""
        texts = self._texts(inputs, self.passage_prefix, self.max_length)
        return self._run("native embedding", texts, lambda m, ids, cu: m.embed(ids, cu))

    def encode_sparse(self, inputs: Sequence) -> list[SparseVector]:
        """SPLADE vectors, one per input (passage_prefix is the "[D] " marker
        for sparse models); non-finite weights are an error
        (crates/inl-sparse/src/native.rs:536-540)."""
        texts = self._texts(inputs, self.passage_prefix, self.max_length)

        return self._run("native sparse", texts, _sparse_forward)

    def encode_late(self, inputs: Sequence, task: LateTask | None = None) -> list[np.ndarray]:
        """Per-token vectors for one late task: its prompt in front, the ids
        cut at its length, its skiplist tokens' vectors dropped; non-finite
        values are an error (crates/inl-late/src/native.rs:631-683)."""
        setup = task or LateTask(length=self.max_length)
        texts = self._texts(inputs, setup.prompt, setup.length, cut_after=True)
        skip = np.fromiter(sorted(setup.skip), dtype=np.uint32) if setup.skip else None

        def forward(m, ids, cu):
            flat = m.encode_multivector(ids, cu)
            out = []
            for i in range(len(cu) - 1):
                v = flat[cu[i]:cu[i + 1]]
                if skip is not None:
                    v = v[~np.isin(ids[cu[i]:cu[i + 1]], skip)]
                if not np.all(np.isfinite(v)):
                    raise InlError.inference("native late encoder produced non-finite values")
                out.append(v)
            return out

        return self._run("native late", texts, forward)
