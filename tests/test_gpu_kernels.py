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
EPI_RESID_F32, EPI_GATED_F32 = 6, 7


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
    elif epi == EPI_GATED_F32:
        out = torch.empty(M, N // 2, dtype=torch.float32, device="cuda")
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


@pytest.mark.parametrize("M,N,K,bn", [
    (333, 128, 1024, 0),   # one CTA, 128-wide tiles
    (333, 200, 1024, 0),   # a last chunk of 8 columns (the ragged store)
    (700, 768, 2304, 0),   # 256-wide tiles on CTA pairs, K as in a 3xBF16 product
    (700, 768, 2304, 128),  # the same on single CTAs
])
def test_gemm_bf16_f32_epilogue(gpu, M, N, K, bn):
    import torch

    A = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    W = (torch.randn(N, K, device="cuda") * 0.05).to(torch.bfloat16)
    ref = A.float() @ W.float().T
    out = _gemm(torch, A, W, epi=EPI_F32, bn=bn)
    err = (out - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-4, err


def test_gemm_bf16_residual_in_place(gpu):
    import torch

    A = torch.randn(700, 2048, device="cuda").to(torch.bfloat16)
    W = (torch.randn(1024, 2048, device="cuda") * 0.02).to(torch.bfloat16)
    h = torch.randn(700, 1024, device="cuda").to(torch.bfloat16)
    ref = (A.float() @ W.float().T) + h.float()
    N_ = _lib()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = N_.lib().inl_cuda_gemm_bf16(A.data_ptr(), 2048, W.data_ptr(), 2048, 700, 1024, 2048, EPI_RESID, 0, 128,
                                     h.data_ptr(), 1024, h.data_ptr(), 1024, 0, status.data_ptr(), _stream(torch))
    N_.check(st, "gemm")
    torch.cuda.synchronize()
    err = (h.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 8e-3, err


@pytest.mark.parametrize("M,N,K,bn", [(700, 1024, 2048, 0), (700, 1024, 2048, 128), (129, 200, 512, 0)])
def test_gemm_bf16_resid_f32_in_place(gpu, M, N, K, bn):
    """The 3xBF16 residual epilogue: f32 out = acc + f32 resid, in place
    (CTA pairs at N = 1024, single CTAs at 128, a ragged last chunk at 200)."""
    import torch

    N_ = _lib()
    A = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    W = (torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16)
    h = torch.randn(M, N, device="cuda")
    ref = (A.float() @ W.float().T) + h
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = N_.lib().inl_cuda_gemm_bf16(A.data_ptr(), K, W.data_ptr(), K, M, N, K, EPI_RESID_F32, 0, 128,
                                     h.data_ptr(), N, h.data_ptr(), N, bn, status.data_ptr(), _stream(torch))
    N_.check(st, "gemm")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    err = (h - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-5, err


@pytest.mark.parametrize("act,gb", [(0, 64), (1, 64), (2, 128), (0, 128)])
def test_gemm_bf16_gated_f32(gpu, act, gb):
    """The gated epilogue with an f32 output (gate/up blocks of 64 on
    128-wide tiles, of 128 on CTA pairs)."""
    import torch
    import torch.nn.functional as F

    M, K, I = 517, 1024, 768
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
    out = _gemm(torch, A, W, epi=EPI_GATED_F32, act=act, gate_block=gb)
    assert out.dtype == torch.float32
    err = (out - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-4, err


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
    (256, 3, 1, 0, -1), (128, 2, 1, 0, 40), (128, 8, 2, 1, -1), (64, 6, 2, 0, -1),
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


# ---------------------------------------------------------------- fused epilogues
def _ex(torch, **kw):
    N_ = _lib()
    a = N_.GemmEx()
    for k, v in kw.items():
        if hasattr(v, "data_ptr"):
            v = v.data_ptr()
        setattr(a, k, v)
    if not a.ldw:
        a.ldw = a.K
    N_.check(N_.lib().inl_cuda_gemm_bf16_ex(ctypes.byref(a), _stream(torch)), "gemm_ex")
    torch.cuda.synchronize()


def _row_scale(ss_parts, dim, eps):
    return torch_rsqrt(ss_parts.double().sum(-1, keepdim=True) / dim + eps)


def torch_rsqrt(x):
    return 1.0 / x.sqrt()


def test_gemm_residual_writes_row_sums_of_squares(gpu):
    import torch

    M, N, K = 777, 1024, 2048
    A = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    W = (torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16)
    h = torch.randn(M, N, device="cuda").to(torch.bfloat16)
    ref = (A.float() @ W.float().T) + h.float()
    ss = torch.full((M, N // 64), -1.0, device="cuda")
    _ex(torch, A=A, lda=K, W=W, M=M, N=N, K=K, epi=EPI_RESID, out=h, ldo=N, resid=h, ldr=N, ss_out=ss)
    err = (h.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 8e-3, err
    ss_ref = (h.double() ** 2).view(M, N // 64, 64).sum(-1)
    assert torch.allclose(ss.double(), ss_ref, rtol=1e-5, atol=1e-6)


def test_gemm_gated_with_folded_norm(gpu):
    import torch
    import torch.nn.functional as F

    M, K, I, gb = 300, 1024, 512, 128
    x = (torch.randn(M, K, device="cuda") * 3).to(torch.bfloat16)
    nw = torch.rand(K, device="cuda") + 0.5
    gate = torch.randn(I, K, device="cuda") * 0.03
    up = torch.randn(I, K, device="cuda") * 0.03
    ss = (x.double() ** 2).view(M, K // 64, 64).sum(-1).float()
    W = torch.empty(2 * I, K, device="cuda")
    for b in range(I // gb):
        W[2 * b * gb:(2 * b + 1) * gb] = gate[b * gb:(b + 1) * gb]
        W[(2 * b + 1) * gb:(2 * b + 2) * gb] = up[b * gb:(b + 1) * gb]
    Wf = (W * nw[None]).to(torch.bfloat16)  # norm weight folded into the columns
    out = torch.empty(M, I, device="cuda", dtype=torch.bfloat16)
    _ex(torch, A=x, lda=K, W=Wf, M=M, N=2 * I, K=K, epi=EPI_GATED, act=0, gate_block=gb, out=out, ldo=I,
        ss_in=ss, ss_in_parts=K // 64, ss_dim=K, ss_eps=1e-6)
    xn = x.double() / (x.double().pow(2).mean(-1, keepdim=True) + 1e-6).sqrt() * nw.double()
    ref = F.silu(xn @ gate.double().T) * (xn @ up.double().T)
    err = (out.double() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 2e-2, err


@pytest.mark.parametrize("d,hq,hkv", [(128, 16, 8), (64, 6, 3), (128, 4, 4)])
def test_gemm_qkv_epilogue(gpu, d, hq, hkv):
    import torch

    M, K = 333, 1024
    N = (hq + 2 * hkv) * d
    x = (torch.randn(M, K, device="cuda") * 2).to(torch.bfloat16)
    W = (torch.randn(N, K, device="cuda") * 0.03).to(torch.bfloat16)
    qn = torch.rand(d, device="cuda") + 0.5
    kn = torch.rand(d, device="cuda") + 0.5
    ss = (x.double() ** 2).view(M, K // 64, 64).sum(-1).float()
    max_pos = 1024
    pos = torch.randint(0, max_pos, (M,), device="cuda", dtype=torch.int32)
    half = d // 2
    inv = 1.0 / (1e6 ** (torch.arange(half, dtype=torch.float64) * 2 / d))
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None]
    cos, sin = ang.cos().float().cuda(), ang.sin().float().cuda()
    # packed by frequency pairs for the epilogue: [d/4, max_pos, (cos f, cos f+1, sin f, sin f+1)]
    pairs = torch.stack([cos[:, 0::2], cos[:, 1::2], sin[:, 0::2], sin[:, 1::2]], -1).transpose(0, 1).contiguous()
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    _ex(torch, A=x, lda=K, W=W, M=M, N=N, K=K, epi=4, out=out, ldo=N, ss_in=ss, ss_in_parts=K // 64, ss_dim=K,
        ss_eps=1e-6, qn=qn, kn=kn, pos=pos, cos=pairs, hq=hq, hkv=hkv, d=d, max_pos=max_pos, qk_eps=1e-6,
        status=st)
    assert st.item() == 0
    r = 1.0 / (x.double().pow(2).mean(-1, keepdim=True) + 1e-6).sqrt()
    y = (x.double() @ W.double().T) * r

    def norm(t, w):
        return t / (t.pow(2).mean(-1, keepdim=True) + 1e-6).sqrt() * w.double()

    def rope(t):
        c = cos.double()[pos.long()][:, None]
        s_ = sin.double()[pos.long()][:, None]
        return torch.cat([t[..., :half] * c - t[..., half:] * s_, t[..., half:] * c + t[..., :half] * s_], -1)

    q = rope(norm(y[:, :hq * d].view(M, hq, d), qn)).reshape(M, -1)
    k = rope(norm(y[:, hq * d:(hq + hkv) * d].view(M, hkv, d), kn)).reshape(M, -1)
    v = y[:, (hq + hkv) * d:]
    ref = torch.cat([q, k, v], -1)
    for name, sl in (("q", slice(0, hq * d)), ("k", slice(hq * d, (hq + hkv) * d)), ("v", slice((hq + hkv) * d, N))):
        err = (out[:, sl].double() - ref[:, sl]).abs().max().item() / ref[:, sl].abs().max().item()
        assert err < 1e-2, (name, err)


@pytest.mark.parametrize("d,hq,hkv,causal,window", [(128, 16, 8, 1, -1), (128, 16, 8, 0, -1), (128, 16, 8, 0, 300),
                                                    (256, 3, 1, 0, 512), (256, 3, 1, 0, -1), (64, 12, 12, 1, -1)])
def test_attention_long_texts(gpu, d, hq, hkv, causal, window):
    """Several 128-key blocks per query tile, texts up to 2048 tokens: GQA
    16/8 x 128 (Qwen3-0.6B), 3/1 x 256 with and without the 512 window
    (the EmbeddingGemma-style config), 12 x 64 causal."""
    import torch

    N_ = _lib()
    lengths = [2048, 1537, 129, 5]
    cu = np.zeros(len(lengths) + 1, dtype=np.int32)
    np.cumsum(lengths, out=cu[1:])
    T = int(cu[-1])
    g = torch.Generator(device="cuda").manual_seed(7)
    qkv = torch.randn(T, (hq + 2 * hkv) * d, device="cuda", generator=g).to(torch.bfloat16)
    q, k, v = qkv[:, :hq * d], qkv[:, hq * d:(hq + hkv) * d], qkv[:, (hq + hkv) * d:]
    out = torch.full((T, hq * d), float("nan"), device="cuda", dtype=torch.bfloat16)
    ld = (hq + 2 * hkv) * d
    st = N_.lib().inl_cuda_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), ld, ld, ld, out.data_ptr(), hq * d, 1,
                                     hq, hkv, d, d ** -0.5, causal, window, cu.ctypes.data, len(lengths),
                                     _stream(torch))
    N_.check(st, "attention")
    torch.cuda.synchronize()
    ref = _attn_ref(torch, q, k, v, cu, hq, hkv, d, d ** -0.5, causal, window)
    err = (out.double() - ref).abs().max().item()
    assert err < 2e-2, err
