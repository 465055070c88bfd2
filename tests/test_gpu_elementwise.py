"""Parity of the bandwidth-bound kernels (embedding gather, RMSNorm /
LayerNorm, per-head q/k norm + RoPE, token positions, last-token head) against
torch fp32/f64 references of the same op, through the C ABI with device
pointers. Tolerances: f32 1e-5 relative; bf16 outputs one bf16 rounding
(2^-8 relative) plus slack: 1e-2."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

F32, BF16 = 0, 1


def _n():
    from im_not_llm_b200 import _native

    return _native


def _s(torch):
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _tdt(torch, code):
    return torch.bfloat16 if code == BF16 else torch.float32


@pytest.mark.parametrize("tab,out", [(F32, F32), (BF16, BF16), (BF16, F32), (F32, BF16)])
@pytest.mark.parametrize("H", [1024, 768, 36])
def test_embed_gather(gpu, tab, out, H):
    import torch

    N = _n()
    V, T = 5000, 777
    table = torch.randn(V, H, device="cuda").to(_tdt(torch, tab))
    ids = torch.randint(0, V, (T,), device="cuda", dtype=torch.int32)
    o = torch.empty(T, H, device="cuda", dtype=_tdt(torch, out))
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    N.check(N.lib().inl_cuda_embed_gather(ids.data_ptr(), T, table.data_ptr(), tab, V, H, 2.5, o.data_ptr(), out,
                                          st.data_ptr(), _s(torch)), "embed")
    torch.cuda.synchronize()
    ref = table.float()[ids.long()] * 2.5
    tol = 1e-2 if out == BF16 else 1e-6
    assert ((o.float() - ref).abs() <= tol * ref.abs() + 1e-6).all()
    assert st.item() == 0


def test_embed_gather_flags_out_of_range_ids(gpu):
    import torch

    N = _n()
    table = torch.randn(10, 64, device="cuda")
    ids = torch.tensor([1, 10, 3], device="cuda", dtype=torch.int32)
    o = torch.full((3, 64), 7.0, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    N.check(N.lib().inl_cuda_embed_gather(ids.data_ptr(), 3, table.data_ptr(), F32, 10, 64, 1.0, o.data_ptr(), F32,
                                          st.data_ptr(), _s(torch)), "embed")
    torch.cuda.synchronize()
    assert st.item() != 0 and (o[1] == 0).all() and torch.equal(o[0], table[1])


@pytest.mark.parametrize("x,out", [(F32, F32), (BF16, BF16), (BF16, F32)])
@pytest.mark.parametrize("H", [1024, 768, 48])
@pytest.mark.parametrize("ln", [0, 1])
def test_norms(gpu, x, out, H, ln):
    import torch

    N = _n()
    rows = 1000
    X = (torch.randn(rows, H, device="cuda") * 3 + 0.5).to(_tdt(torch, x))
    w = torch.randn(H, device="cuda")
    b = torch.randn(H, device="cuda") if ln else None
    o = torch.empty(rows, H, device="cuda", dtype=_tdt(torch, out))
    N.check(N.lib().inl_cuda_norm(X.data_ptr(), x, H, w.data_ptr(), None if b is None else b.data_ptr(), 1e-5, ln,
                                  rows, H, o.data_ptr(), out, H, _s(torch)), "norm")
    torch.cuda.synchronize()
    xf = X.double()
    if ln:
        ref = torch.nn.functional.layer_norm(xf, (H,), w.double(), b.double(), 1e-5)
    else:
        ref = xf / torch.sqrt((xf * xf).mean(-1, keepdim=True) + 1e-5) * w.double()
    if out == BF16:
        err = ((o.double() - ref).abs() / (ref.abs() + 1e-3)).max().item()
        assert err < 1e-2, err
    else:
        err = (o.double() - ref).abs().max().item() / ref.abs().max().item()
        assert err < 2e-6, err


# head_dim 8 / 16 / 32: the narrow warp layout (EmbeddingGemma 2 tiny checkpoints)
@pytest.mark.parametrize("dt", [F32, BF16])
@pytest.mark.parametrize("d,hq,hkv,v_norm", [(128, 16, 8, 0), (64, 12, 12, 0), (256, 3, 1, 1),
                                             (16, 4, 2, 1),
                                             (32, 4, 1, 1),
                                             (8, 2, 2, 0)])
def test_qk_norm_rope(gpu, dt, d, hq, hkv, v_norm):
    import torch

    N = _n()
    T, max_pos = 300, 512
    ld = (hq + 2 * hkv) * d
    qkv = torch.randn(T, ld, device="cuda").to(_tdt(torch, dt))
    orig = qkv.double().clone()
    qw = torch.randn(d, device="cuda")
    kw = torch.randn(d, device="cuda")
    pos = torch.randint(0, max_pos, (T,), device="cuda", dtype=torch.int32)
    half = d // 2
    inv = 1.0 / (1e4 ** (torch.arange(half, dtype=torch.float64) * 2 / d))
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None]
    cos = ang.cos().float().cuda()
    sin = ang.sin().float().cuda()
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    N.check(N.lib().inl_cuda_qk_norm_rope(qkv.data_ptr(), dt, ld, T, hq, hkv, d, qw.data_ptr(), kw.data_ptr(), v_norm,
                                          1e-6, pos.data_ptr(), cos.data_ptr(), sin.data_ptr(), max_pos,
                                          st.data_ptr(), _s(torch)), "qk_norm_rope")
    torch.cuda.synchronize()
    assert st.item() == 0

    def norm(x, w):
        y = x / torch.sqrt((x * x).mean(-1, keepdim=True) + 1e-6)
        return y * w.double() if w is not None else y

    def rope(x):
        c = cos.double()[pos.long()][:, None]
        s = sin.double()[pos.long()][:, None]
        x1, x2 = x[..., :half], x[..., half:]
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)

    q = rope(norm(orig[:, :hq * d].view(T, hq, d), qw))
    k = rope(norm(orig[:, hq * d:(hq + hkv) * d].view(T, hkv, d), kw))
    v = orig[:, (hq + hkv) * d:].view(T, hkv, d)
    if v_norm:
        v = norm(v, None)
    ref = torch.cat([q.reshape(T, -1), k.reshape(T, -1), v.reshape(T, -1)], -1)
    tol = 1e-2 if dt == BF16 else 2e-6
    err = (qkv.double() - ref).abs().max().item() / ref.abs().max().item()
    assert err < tol, err


def test_token_positions(gpu):
    import torch

    N = _n()
    lengths = [3, 0, 5, 1, 0, 7]
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device="cuda")
    T = sum(lengths)
    pos = torch.full((T,), -1, dtype=torch.int32, device="cuda")
    N.check(N.lib().inl_cuda_token_positions(cu.data_ptr(), len(lengths), T, pos.data_ptr(), _s(torch)), "pos")
    torch.cuda.synchronize()
    assert pos.tolist() == [p for L in lengths for p in range(L)]


@pytest.mark.parametrize("dt", [F32, BF16])
def test_last_token_norm_l2(gpu, dt):
    import torch

    N = _n()
    lengths = [5, 1, 9, 2]
    cu_np = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    cu = torch.tensor(cu_np, device="cuda")
    H = 1024
    h = torch.randn(int(cu_np[-1]), H, device="cuda").to(_tdt(torch, dt))
    w = torch.rand(H, device="cuda") + 0.5
    out = torch.empty(4, H, device="cuda")
    N.check(N.lib().inl_cuda_last_token_norm_l2(h.data_ptr(), dt, H, cu.data_ptr(), 4, w.data_ptr(), 1e-6, H,
                                                out.data_ptr(), _s(torch)), "last")
    torch.cuda.synchronize()
    last = h.double()[torch.tensor(cu_np[1:] - 1).long()]
    y = last / torch.sqrt((last * last).mean(-1, keepdim=True) + 1e-6) * w.double()
    y = y / torch.sqrt((y * y).sum(-1, keepdim=True) + 1e-12)
    err = (out.double() - y).abs().max().item()
    assert err < (2e-3 if dt == BF16 else 1e-6), err
