"""Kernel-level parity on the GPU: the tcgen05 GEMM and the attention kernels
against fp32 references of the same op, called through the C ABI
(include/inl_cuda_kernels.h) with device pointers.

Tolerances: bf16-output GEMMs are compared relative to the largest reference
magnitude, bounded by one bf16 rounding (2^-8) plus slack: 8e-3. f32 kernels:
2e-5 relative. bf16 attention: 2e-2 absolute on O(1) values (P is rounded to
bf16 before the PV product, as in every bf16 flash kernel).
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

EPI_BF16, EPI_RESID, EPI_GATED, EPI_F32 = 0, 1, 2, 3


def _lib():
    from im_not_llm_b200 import _native

    return _native


def _stream(torch):
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _gemm(torch, A, W, epi=EPI_BF16, act=0, gate_block=128, resid=None, out_dtype=None, bn=0):
    N_ = _lib()
    M, K = A.shape
    N = W.shape[0]
    if epi == EPI_GATED:
        out = torch.empty(M, N // 2, dtype=torch.bfloat16, device="cuda")
    elif epi == EPI_F32:
        out = torch.empty(M, N, dtype=torch.float32, device="cuda")
    else:
        out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = N_.lib().inl_cuda_gemm_bf16(
        A.data_ptr(), A.stride(0), W.data_ptr(), W.stride(0), M, N, K, epi, act, gate_block,
        out.data_ptr(), out.stride(0), None if resid is None else resid.data_ptr(),
        0 if resid is None else resid.stride(0), bn, status.data_ptr(), _stream(torch))
    N_.check(st, "gemm")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return out


@pytest.mark.parametrize("M,N,K,bn", [
    (128, 256, 64, 0), (300, 512, 1024, 0), (1000, 4096, 1024, 0), (77, 128, 192, 0),
    (4096, 1024, 3072, 0), (513, 1024, 2048, 128), (129, 384, 1024, 0), (1, 256, 1024, 256),
    (2048, 6144, 1024, 256), (20000, 1024, 1024, 0),
])
def test_gemm_bf16_plain(gpu, M, N, K, bn):
    import torch

    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    W = (torch.randn(N, K, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    ref = A.float() @ W.float().T
    out = _gemm(torch, A, W, bn=bn)
    err = (out.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 8e-3, err


def test_gemm_bf16_f32_epilogue(gpu):
    import torch

    A = torch.randn(333, 1024, device="cuda").to(torch.bfloat16)
    W = (torch.randn(128, 1024, device="cuda") * 0.05).to(torch.bfloat16)
    ref = A.float() @ W.float().T
    out = _gemm(torch, A, W, epi=EPI_F32)
    err = (out - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-4, err


def test_gemm_bf16_residual_in_place(gpu):
    import torch

    A = torch.randn(700, 2048, device="cuda").to(torch.bfloat16)
    W = (torch.randn(1024, 2048, device="cuda") * 0.02).to(torch.bfloat16)
    h = torch.randn(700, 1024, device="cuda").to(torch.bfloat16)
    ref = (A.float() @ W.float().T).to(torch.bfloat16).float() + h.float()
    N_ = _lib()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = N_.lib().inl_cuda_gemm_bf16(A.data_ptr(), 2048, W.data_ptr(), 2048, 700, 1024, 2048, EPI_RESID, 0, 128,
                                     h.data_ptr(), 1024, h.data_ptr(), 1024, 0, status.data_ptr(), _stream(torch))
    N_.check(st, "gemm")
    torch.cuda.synchronize()
    err = (h.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 8e-3, err


@pytest.mark.parametrize("act", [0, 1, 2])
def test_gemm_bf16_gated(gpu, act):
    import torch
    import torch.nn.functional as F

    M, K, I, gb = 517, 1024, 768, 128
    A = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    gate = (torch.randn(I, K, device="cuda") * 0.03).to(torch.bfloat16)
    up = (torch.randn(I, K, device="cuda") * 0.03).to(torch.bfloat16)
    W = torch.empty(2 * I, K, device="cuda", dtype=torch.bfloat16)
    for b in range(I // gb):
        W[2 * b * gb:(2 * b + 1) * gb] = gate[b * gb:(b + 1) * gb]
        W[(2 * b + 1) * gb:(2 * b + 2) * gb] = up[b * gb:(b + 1) * gb]
    g = A.float() @ gate.float().T
    u = A.float() @ up.float().T
    fn = {0: F.silu, 1: lambda x: F.gelu(x), 2: lambda x: F.gelu(x, approximate="tanh")}[act]
    ref = fn(g) * u
    out = _gemm(torch, A, W, epi=EPI_GATED, act=act, gate_block=gb)
    err = (out.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1.5e-2, err


def test_gemm_rejects_misaligned_shapes(gpu):
    import torch

    from im_not_llm_b200 import InvalidInputError

    A = torch.randn(64, 100, device="cuda").to(torch.bfloat16)  # K % 8 != 0
    W = torch.randn(128, 100, device="cuda").to(torch.bfloat16)
    with pytest.raises(InvalidInputError):
        _gemm(torch, A, W)


def test_gemm_f32(gpu):
    import torch

    N_ = _lib()
    M, N, K = 300, 384, 520
    A = torch.randn(M, K, device="cuda")
    W = torch.randn(N, K, device="cuda") * 0.05
    out = torch.empty(M, N, device="cuda")
    st = N_.lib().inl_cuda_gemm_f32(A.data_ptr(), K, W.data_ptr(), K, M, N, K, EPI_F32, 0, out.data_ptr(), N,
                                    None, 0, _stream(torch))
    N_.check(st, "gemm_f32")
    torch.cuda.synchronize()
    ref = (A.double() @ W.double().T)
    err = (out.double() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 2e-6, err


def _attn_ref(torch, q, k, v, cu, hq, hkv, d, scale, causal, window):
    out = torch.zeros(q.shape[0], hq, d, dtype=torch.float64, device=q.device)
    rep = hq // hkv
    for i in range(len(cu) - 1):
        s, e = int(cu[i]), int(cu[i + 1])
        if e == s:
            continue
        qq = q[s:e].double().view(e - s, hq, d)
        kk = k[s:e].double().view(e - s, hkv, d).repeat_interleave(rep, dim=1)
        vv = v[s:e].double().view(e - s, hkv, d).repeat_interleave(rep, dim=1)
        sc = torch.einsum("qhd,khd->hqk", qq, kk) * scale
        qi = torch.arange(e - s, device=q.device)[:, None]
        ki = torch.arange(e - s, device=q.device)[None, :]
        mask = torch.zeros(e - s, e - s, dtype=torch.bool, device=q.device)
        if causal:
            mask |= ki > qi
        if window is not None and window >= 0:
            mask |= (qi - ki).abs() > window
        sc = sc.masked_fill(mask[None], float("-inf"))
        out[s:e] = torch.einsum("hqk,khd->qhd", torch.softmax(sc, -1), vv)
    return out.view(q.shape[0], hq * d)


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("d,hq,hkv,causal,window", [
    (128, 16, 8, 1, -1), (128, 4, 4, 0, -1), (64, 12, 12, 0, 64), (256, 3, 1, 0, 512), (64, 4, 2, 1, -1),
    (256, 3, 1, 0, -1), (128, 2, 1, 0, 40),
])
def test_attention_varlen(gpu, dtype, d, hq, hkv, causal, window):
    import torch

    N_ = _lib()
    lengths = [1, 7, 64, 65, 130, 300, 1000, 33]
    cu = np.zeros(len(lengths) + 1, dtype=np.int32)
    np.cumsum(lengths, out=cu[1:])
    T = int(cu[-1])
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    g = torch.Generator(device="cuda").manual_seed(d + hq)
    q = torch.randn(T, hq * d, device="cuda", generator=g).to(tdt)
    k = torch.randn(T, hkv * d, device="cuda", generator=g).to(tdt)
    v = torch.randn(T, hkv * d, device="cuda", generator=g).to(tdt)
    out = torch.full((T, hq * d), float("nan"), device="cuda", dtype=tdt)
    scale = d ** -0.5
    st = N_.lib().inl_cuda_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), hq * d, hkv * d, hkv * d,
                                     out.data_ptr(), hq * d, 1 if dtype == "bf16" else 0, hq, hkv, d, scale,
                                     causal, window, cu.ctypes.data, len(lengths), _stream(torch))
    N_.check(st, "attention")
    torch.cuda.synchronize()
    ref = _attn_ref(torch, q, k, v, cu, hq, hkv, d, scale, causal, window)
    err = (out.double() - ref).abs().max().item()
    assert err < (2e-2 if dtype == "bf16" else 2e-5), err
