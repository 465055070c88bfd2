"""Text front end: strings to token ids with a model's ``tokenizer.json``.

The reference links the Rust ``tokenizers`` crate and loads the model repo's
tokenizer.json (crates/inl-text/src/qwen3/mod.rs:403-427,
crates/inl-text/src/native.rs:345-370, crates/inl-sparse/src/native.rs:501-513).
This module loads the same file through the Python binding of that library,
with the reference's settings:

* encode with special tokens (``encode(text, true)``);
* truncation to ``max_length`` done by the tokenizer (``TruncationParams
  { max_length, .. }``), so the template's special tokens (the trailing EOS of
  Qwen3, ``<bos> … <eos>`` of EmbeddingGemma) survive and the content is cut;
* token counts are taken without truncation, as ``token_counts`` is
  (crates/inl-text/src/native.rs:507-520).

There is no padding: each text is its own segment of a packed batch, and the
reference's left / right padding does not change a text's result.
"""
from __future__ import annotations

import enum

import threading
from pathlib import Path
from typing import Sequence

import numpy as np

from .errors import InlError


class TextTokenizer:
    """A tokenizer.json with one truncating copy per ``max_length`` in use."""

    def __init__(self, tokenizer):
        self._json = tokenizer.to_str()
        self._plain = self._copy(None)
        self._by_length: dict[int, object] = {}
        self._lock = threading.Lock()

    @classmethod
    def from_file(cls, path: str | Path) -> "TextTokenizer":
        try:
            from tokenizers import Tokenizer
        except ImportError as e:  # pragma: no cover - the image ships the package
            raise InlError.config(f"string inputs need the `tokenizers` package: {e}") from e
        try:
            return cls(Tokenizer.from_file(str(path)))
        except Exception as e:  # the binding raises a plain Exception on parse errors
            raise InlError.inference(f"native tokenizer parse failed: {e}") from e

    def _copy(self, max_length: int | None):
        from tokenizers import Tokenizer

        t = Tokenizer.from_str(self._json)
        t.no_padding()
        if max_length is None:
            t.no_truncation()
        else:
            t.enable_truncation(max_length)
        return t

    def _truncating(self, max_length: int):
        if max_length <= 0:
            raise InlError.config("max_length must be greater than 0")
        with self._lock:
            t = self._by_length.get(max_length)
            if t is None:
                t = self._by_length[max_length] = self._copy(max_length)
            return t

    def encode(self, texts: Sequence[str], max_length: int) -> list[np.ndarray]:
        """Ids per text: special tokens added, at most ``max_length`` of them."""
        try:
            encs = self._truncating(max_length).encode_batch(list(texts), add_special_tokens=True)
        except InlError:
            raise
        except Exception as e:
            raise InlError.inference(f"native tokenizer encode failed: {e}") from e
        return [np.asarray(e.ids, dtype=np.uint32) for e in encs]

    def encode_untruncated(self, texts: Sequence[str]) -> list[np.ndarray]:
        """Ids per text with special tokens and no truncation (the late
        encoder cuts them itself, crates/inl-late/src/native.rs:292-305)."""
        try:
            encs = self._plain.encode_batch(list(texts), add_special_tokens=True)
        except Exception as e:
            raise InlError.inference(f"native tokenizer encode failed: {e}") from e
        return [np.asarray(e.ids, dtype=np.uint32) for e in encs]

    def counts(self, texts: Sequence[str]) -> list[int]:
        """Tokens per text as the model would see them before truncation."""
        return [len(x) for x in self.encode_untruncated(texts)]

    def token_to_id(self, token: str) -> int | None:
        """The id of ``token`` if it is one vocabulary entry, else None."""
        return self._plain.token_to_id(token)


class Gemma2Task(enum.Enum):
    """EmbeddingGemma 2 prompt templates from the model card
    (crates/inl-text/src/gemma2.rs:802-857). The prompts are caller-controlled:
    ``TextEmbedder`` applies none on its own. Use ``apply`` to build the
    prefixed text, or set ``TextOptions.query_prefix`` / ``passage_prefix`` to
    ``Gemma2Task.<task>.prefix``."""
    SEARCH_QUERY = "task: search result | query: {text}"
    QUERY = "task: query | query: {text}"
    QUESTION_ANSWERING = "task: question answering | query: {text}"
    FACT_CHECKING = "task: fact checking | query: {text}"
    CLASSIFICATION = "task: classification | query: {text}"
    CLUSTERING = "task: clustering | query: {text}"
    CODE_RETRIEVAL = "task: code retrieval | query: {text}"
    DOCUMENT = "title: none | text: {text}"

    @property
    def template(self) -> str:
        return self.value

    @property
    def prefix(self) -> str:
        """The constant text the template puts before ``{text}``."""
        return self.value[: -len("{text}")]

    def apply(self, text: str) -> str:
        return self.prefix + text

    @property
    def is_query(self) -> bool:
        """Every task but DOCUMENT is query-side."""
        return self is not Gemma2Task.DOCUMENT


def gemma2_document(title: str, text: str) -> str:
    """``title: {title} | text: {text}`` for a titled document
    (crates/inl-text/src/gemma2.rs:859-862)."""
    return f"title: {title} | text: {text}"
