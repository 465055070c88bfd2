"""DataParallelEmbedder with real models: two replicas on cuda:0 driven by
two host threads give the single model's embeddings (same texts, other
batch compositions), and the sparse path the single model's SPLADE rows."""
import numpy as np
import pytest

import im_not_llm_b200 as inl
from tests.conftest import cosine_rows

pytestmark = pytest.mark.gpu


def test_two_replicas_match_one_model(gpu):
    cfg = dict(inl.synthetic.QWEN3_TINY)
    w = inl.synthetic.qwen3_weights(cfg, seed=0, norm_jitter=0.1)
    ids, cu = inl.synthetic.random_texts(40, 3, 300, cfg["vocab_size"], seed=11)
    texts = np.split(ids, cu[1:-1])
    models = [inl.CudaModel(cfg, w, device=0, dtype="bf16") for _ in range(2)]
    try:
        want = models[0].embed(ids, cu)
        got = np.stack(inl.DataParallelEmbedder(models, max_batch_tokens=1500).embed(texts))
        assert cosine_rows(got, want).min() >= 0.9999
    finally:
        for m in models:
            m.close()


def test_two_replicas_sparse(gpu):
    cfg = dict(inl.synthetic.MODERNBERT_TINY)
    w = inl.synthetic.modernbert_weights(cfg, seed=0, norm_jitter=0.1)
    ids, cu = inl.synthetic.random_texts(12, 2, 120, cfg["vocab_size"], seed=12)
    texts = np.split(ids, cu[1:-1])
    models = [inl.CudaModel(cfg, w, device=0, dtype="f32") for _ in range(2)]
    try:
        want = models[0].encode_sparse(ids, cu)
        got = inl.DataParallelEmbedder(models, max_batch_tokens=300).encode_sparse(texts)
        for row, v in zip(want, got):
            ref = inl.SparseVector.from_dense(row)
            assert v.indices.tolist() == ref.indices.tolist()
            assert np.abs(v.values - ref.values).max(initial=0) <= 1e-4
    finally:
        for m in models:
            m.close()
