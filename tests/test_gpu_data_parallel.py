"""DataParallelEmbedder with real models: two replicas on cuda:0 driven by
two host threads give the single model's embeddings (same texts, other
batch compositions), and the sparse path the single model's SPLADE rows;
with two or more GPUs visible, one replica per device gives device 0's
embeddings."""
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


@pytest.mark.parametrize("dtype,head_dim", [("bf16", 256), ("f32", 128)])
def test_replicas_on_every_device(gpu, dtype, head_dim):
    """One replica per visible GPU (the data-parallel layout of a node): the
    per-device kernel attributes (shared-memory limits of the tcgen05 GEMMs
    and attention, the f32 attention kernel) are set on each device, so every
    replica gives device 0's embeddings. Gemma-style tower: bf16 attention at
    head_dim 256 and the f32 SIMT attention."""
    import torch

    n_dev = torch.cuda.device_count()
    if n_dev < 2:
        pytest.skip("one CUDA device visible")
    cfg = dict(inl.synthetic.GEMMA_TINY, head_dim=head_dim)
    w = inl.synthetic.gemma_weights(cfg, seed=3, norm_jitter=0.1)
    ids, cu = inl.synthetic.random_texts(48, 3, 200, cfg["vocab_size"], seed=13)
    texts = np.split(ids, cu[1:-1])
    models = [inl.CudaModel(cfg, w, device=d, dtype=dtype) for d in range(n_dev)]
    try:
        want = models[0].embed(ids, cu)
        for m in models[1:]:
            assert cosine_rows(m.embed(ids, cu), want).min() >= 0.99999
        got = np.stack(inl.DataParallelEmbedder(models, max_batch_tokens=800).embed(texts))
        assert cosine_rows(got, want).min() >= 0.9999
    finally:
        for m in models:
            m.close()
