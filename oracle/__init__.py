"""CPU oracle for the encoder forward hot path: TEST INFRASTRUCTURE ONLY.

Plain numpy (f32) restatements of the reference's CPU forward code, used by
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` as the checker and the timed CPU
baseline. The shipped library never imports this package: the product path is
the CUDA library ``libinl_cuda.so`` and fails loudly when it is missing.

The reference (NomaDamas/im-not-llm) is Rust on candle 0.11.1 and cannot be
built in this image (no cargo/rustc, candle un-vendored), so it cannot be run
here. Each function cites the reference file:line it restates. Parity pins:

* ModernBERT + SPLADE pooling: the reference's ``tiny_splade`` golden fixture
  (``crates/inl-sparse/tests/fixtures/tiny_splade/golden.json``), copied into
  ``tests/golden/`` by ``tests/golden/make_golden.py``.
* EmbeddingGemma-style tower: the reference's ``tiny_embeddinggemma2`` golden
  (``crates/inl-text/tests/fixtures/tiny_embeddinggemma2/golden.json``).
* Qwen3.5 late tower (``qwen3_5.py``): the reference's ``tiny_qwen3_5_late``
  golden (``crates/inl-late/tests/fixtures/tiny_qwen3_5_late/golden.json``).
* Qwen3: parity unpinned by golden vectors (partial). No golden vector exists
  without the real checkpoint; the oracle is checked against the reference's
  own unit-test invariants (textbook RMSNorm, manual half-split RoPE, padding
  invariance, backend agreement) restated in ``tests/test_oracle_qwen3.py``,
  and against a second opinion, ``transformers`` ``Qwen3Model`` on the same
  random weights.
"""
