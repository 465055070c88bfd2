"""inl_cuda_attention_noalloc, the attention entry point for callers that may
not allocate device memory, against inl_cuda_attention on the same inputs.

Two calls in a row with different shapes: the second call finds the first
call's cu_seqlens and work list still in the shared device array (more texts,
more query blocks) and must not be affected by them. Outputs start as NaN so a
row the kernel skipped shows up. Tolerances are the attention tests': max
|diff| < 2e-2 for bf16, 2e-5 for f32.

This file is collected last so that it runs both after the other GPU tests
(the library's other entry points have already allocated on the device) and
alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

TOL = {"bf16": 2e-2, "f32": 2e-5}


def _cu(lengths):
    cu = np.zeros(len(lengths) + 1, dtype=np.int32)
    np.cumsum(lengths, out=cu[1:])
    return cu


def _run_both(torch, N_, dtype, lengths, hq, hkv, d, causal, window, seed):
    cu = _cu(lengths)
    T = int(cu[-1])
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    g = torch.Generator(device="cuda").manual_seed(seed)
    ld = (hq + 2 * hkv) * d
    qkv = torch.randn(T, ld, device="cuda", generator=g).to(tdt)
    q, k, v = qkv[:, :hq * d], qkv[:, hq * d:(hq + hkv) * d], qkv[:, (hq + hkv) * d:]
    outs = []
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for fn in (N_.lib().inl_cuda_attention_noalloc, N_.lib().inl_cuda_attention):
        out = torch.full((T, hq * d), float("nan"), device="cuda", dtype=tdt)
        st = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), ld, ld, ld, out.data_ptr(), hq * d,
                1 if dtype == "bf16" else 0, hq, hkv, d, d ** -0.5, causal, window, cu.ctypes.data, len(lengths),
                stream)
        N_.check(st, "attention")
        torch.cuda.synchronize()
        outs.append(out)
    return outs


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,d", [("bf16", 128), ("bf16", 64), ("f32", 64)])
def test_noalloc_attention_matches_allocating_entry_point_twice(gpu, dtype, d):
    import torch

    from im_not_llm_b200 import _native as N_

    calls = [
        # first call: long texts, many query blocks, GQA 16/8 (Qwen3-0.6B heads)
        dict(lengths=[2048, 1537, 129, 5, 1, 300, 0, 700], hq=16, hkv=8, causal=0, window=-1, seed=11),
        # second call: fewer and shorter texts, causal + window, GQA 4/1
        dict(lengths=[7, 64, 65, 33, 130], hq=4, hkv=1, causal=1, window=16, seed=12),
    ]
    for c in calls:
        got, want = _run_both(torch, N_, dtype, c["lengths"], c["hq"], c["hkv"], d, c["causal"], c["window"],
                              c["seed"])
        assert not torch.isnan(got.float()).any()
        err = (got.double() - want.double()).abs().max().item()
        assert err < TOL[dtype], (c, err)


def test_noalloc_attention_rejects_calls_over_its_limits():
    """Size checks run on the host before any CUDA call, so this needs no GPU."""
    from im_not_llm_b200 import _native as N_

    lib = N_.lib()
    too_many_texts = _cu(np.ones(8193, dtype=np.int64))
    st = lib.inl_cuda_attention_noalloc(None, None, None, 128, 128, 128, None, 128, 1, 1, 1, 128, 1.0, 0, -1,
                                        too_many_texts.ctypes.data, 8193, None)
    assert st == 4 and "8192" in N_.last_error()
    # 300 texts x 128 blocks of 128 rows = 38400 query blocks > 32768
    too_many_blocks = _cu(np.full(300, 128 * 128, dtype=np.int64))
    st = lib.inl_cuda_attention_noalloc(None, None, None, 128, 128, 128, None, 128, 1, 1, 1, 128, 1.0, 0, -1,
                                        too_many_blocks.ctypes.data, 300, None)
    assert st == 4 and "32768" in N_.last_error()
    bad = np.array([0, 5, 3], dtype=np.int32)
    st = lib.inl_cuda_attention_noalloc(None, None, None, 128, 128, 128, None, 128, 1, 1, 1, 128, 1.0, 0, -1,
                                        bad.ctypes.data, 2, None)
    assert st == 4 and "non-decreasing" in N_.last_error()
