"""inl_cuda_attention_noalloc, the attention entry point for callers that may
not allocate device memory, against inl_cuda_attention on the same inputs.

Two calls in a row with different shapes: the second call finds the first
call's cu_seqlens and work list still in the shared device array (more texts,
more query blocks) and must not be affected by them. Outputs start as NaN so a
row the kernel skipped shows up. Tolerances are the attention tests': max
|diff| < 2e-2 for bf16, 2e-5 for f32.

This file is collected last so that its GPU tests run after the other GPU
tests (the library's other entry points have already allocated on the
device); one of them repeats the two calls in a child process whose first
call into the library is the no-allocation one, so the per-device lookup of
the array's address is covered on a fresh process too.
"""
import ctypes
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]

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


CALLS = [
    # first call: long texts, many query blocks, GQA 16/8 (Qwen3-0.6B heads)
    dict(lengths=[2048, 1537, 129, 5, 1, 300, 0, 700], hq=16, hkv=8, causal=0, window=-1, seed=11),
    # second call: fewer and shorter texts, causal + window, GQA 4/1
    dict(lengths=[7, 64, 65, 33, 130], hq=4, hkv=1, causal=1, window=16, seed=12),
    # third call: causal, texts of equal and different block counts, an empty one
    dict(lengths=[640, 129, 640, 0, 1, 257, 1000, 3], hq=16, hkv=8, causal=1, window=-1, seed=13),
]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,d", [("bf16", 128), ("bf16", 64), ("f32", 64)])
def test_noalloc_attention_matches_allocating_entry_point_twice(gpu, dtype, d):
    import torch

    from im_not_llm_b200 import _native as N_

    for c in CALLS:
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


@pytest.mark.gpu
def test_noalloc_attention_in_a_fresh_process(gpu):
    """The same calls in a child process whose first call into the library is
    the no-allocation entry point (the array's device address is looked up
    there)."""
    code = (
        "import sys, torch; sys.path.insert(0, %r); sys.path.insert(0, %r)\n"
        "import test_zz_no_alloc as t\n"
        "from im_not_llm_b200 import _native as N_\n"
        "for c in t.CALLS:\n"
        "    got, want = t._run_both(torch, N_, 'bf16', c['lengths'], c['hq'], c['hkv'], 128, c['causal'],"
        " c['window'], c['seed'])\n"
        "    assert not torch.isnan(got.float()).any()\n"
        "    assert (got.double() - want.double()).abs().max().item() < t.TOL['bf16']\n"
        "print('fresh ok')\n" % (str(ROOT), str(ROOT / "tests")))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "fresh ok" in r.stdout, r.stdout + r.stderr


@pytest.mark.gpu
def test_noalloc_attention_refuses_a_capturing_stream(gpu):
    """It waits for its stream before returning, so a stream in capture is
    refused (INL_ERR_CONFIG) before anything is queued, and the capture stays
    valid."""
    import torch

    from im_not_llm_b200 import _native as N_

    cu = _cu([100, 28])
    qkv = torch.zeros(128, 3 * 128, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(128, 128, device="cuda", dtype=torch.bfloat16)
    side = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        st = N_.lib().inl_cuda_attention_noalloc(
            qkv.data_ptr(), qkv.data_ptr() + 256, qkv.data_ptr() + 512, 384, 384, 384, out.data_ptr(), 128, 1, 1,
            1, 128, 1.0, 1, -1, cu.ctypes.data, 2, ctypes.c_void_p(side.cuda_stream))
        out.add_(1)  # the capture is still usable after the refusal
    assert st == 1 and "capturing" in N_.last_error()
    graph.replay()
    torch.cuda.synchronize()
    assert out.float().eq(1).all()


def _work_order(cu, qb, causal):
    """The heaviest-first order of the allocating entry point: (text, block)
    items, stably sorted by the key blocks a causal block attends to (b + 1)
    or by the text's block count (csrc/model.cu attention_work)."""
    items = []
    for i in range(len(cu) - 1):
        nb = -(-(cu[i + 1] - cu[i]) // qb)
        items += [((b + 1) if causal else nb, i, b) for b in range(nb)]
    return [(i, b) for _, i, b in sorted(items, key=lambda x: -x[0])]


def _build_kernel_order(cu, qb, causal):
    """The slot arithmetic of build_work_kernel (csrc/attention_noalloc.cu),
    restated on the CPU: texts sorted by block count (ties in text order),
    exclusive prefix of the sorted counts, then each slot found by search."""
    n = len(cu) - 1
    nb = [-(-(cu[i + 1] - cu[i]) // qb) for i in range(n)]
    order = sorted(range(n), key=lambda i: (-nb[i], i))
    snb = [nb[i] for i in order]
    pre = np.concatenate([[0], np.cumsum(snb)]).astype(np.int64)
    n_work = int(pre[-1])
    out = []
    for p in range(n_work):
        if not causal:
            r = max(r for r in range(n) if pre[r] <= p)
            b = p - pre[r]
        else:
            def above(b):  # items on levels above b
                c = sum(1 for x in snb if x > b + 1)
                return pre[c] - (b + 1) * c
            b = min(b for b in range(snb[0]) if above(b) <= p)
            r = p - above(b)
        out.append((order[r], int(b)))
    return out


@pytest.mark.parametrize("causal", [0, 1])
def test_device_work_list_arithmetic_is_heaviest_first(causal):
    """CPU check of the build kernel's slot arithmetic: every (text, block)
    item exactly once, in non-increasing weight, the same weights slot by
    slot as the allocating entry point's list."""
    rng = np.random.default_rng(3)
    for lengths in ([2048, 1537, 129, 5, 1, 300, 0, 700], [640, 129, 640, 0, 1, 257, 1000, 3],
                    list(rng.integers(0, 3000, 200))):
        cu = _cu(lengths)
        got = _build_kernel_order(cu, 128, causal)
        want = _work_order(cu, 128, causal)
        assert sorted(got) == sorted(want) and len(set(got)) == len(got)
        nbs = [-(-(cu[i + 1] - cu[i]) // 128) for i in range(len(lengths))]
        weight = [(b + 1) if causal else nbs[i] for i, b in got]
        assert weight == [(b + 1) if causal else nbs[i] for i, b in want]
