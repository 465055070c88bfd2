"""Gated DeltaNet kernel hooks (im-not-llm_b200/csrc/deltanet.cu): the
Qwen3.5 linear-attention pieces, checked against oracle/qwen3_5.py, which is
itself pinned on the reference's tiny_qwen3_5_late golden.

The argument checks run on the host before any CUDA call, so they are tested
on CPU; the parity test against the oracle runs on the GPU."""
import ctypes

import numpy as np
import pytest

from oracle import qwen3_5 as Q35


def _cu(lengths):
    cu = np.zeros(len(lengths) + 1, dtype=np.int32)
    np.cumsum(lengths, out=cu[1:])
    return cu


def test_hook_argument_checks_need_no_gpu():
    from im_not_llm_b200 import _native as N_

    lib = N_.lib()
    bad = np.array([0, 5, 3], dtype=np.int32)
    # INL_ERR_INVALID_INPUT = 4
    assert lib.inl_cuda_causal_conv_silu(1, 8, 8, 1, 4, bad.ctypes.data, 2, 1, 8, None) == 4
    assert "non-decreasing" in N_.last_error()
    cu = _cu([3, 4])
    assert lib.inl_cuda_causal_conv_silu(1, 4, 8, 1, 4, cu.ctypes.data, 2, 1, 8, None) == 4  # ldx < C
    # nk 2, nv 4, dk 8, dv 8: mixed rows need 2*2*8 + 4*8 = 64 columns
    args = [1, 63, 1, 1, 4, 1, 32, 1, 1, 1, 1e-6, 2, 4, 8, 8, cu.ctypes.data, 2, 1, 32, None]
    assert lib.inl_cuda_gated_delta_rule(*args) == 4 and "strides" in N_.last_error()
    args[1] = 64
    args[2] = None
    assert lib.inl_cuda_gated_delta_rule(*args) == 1  # NULL argument: INL_ERR_CONFIG


@pytest.mark.gpu
@pytest.mark.parametrize("nk,nv,dk,dv", [(2, 4, 8, 8), (2, 2, 16, 64), (1, 2, 128, 128)])
def test_conv_and_delta_rule_match_the_oracle(gpu, nk, nv, dk, dv):
    import torch

    from im_not_llm_b200 import _native as N_

    lib = N_.lib()
    lengths = [1, 0, 7, 64, 65, 200, 3]
    cu = _cu(lengths)
    T, K = int(cu[-1]), 4
    C = 2 * nk * dk + nv * dv
    rng = np.random.default_rng(dk + dv)
    x = rng.standard_normal((T, C)).astype(np.float32)
    w = (rng.standard_normal((C, K)) * 0.5).astype(np.float32)
    ab = rng.standard_normal((T, 2 * nv)).astype(np.float32)  # b | a
    z = rng.standard_normal((T, nv * dv)).astype(np.float32)
    dt_bias = rng.standard_normal(nv).astype(np.float32)
    a_log = (rng.standard_normal(nv) * 0.5).astype(np.float32)
    norm_w = (1 + 0.1 * rng.standard_normal(dv)).astype(np.float32)
    eps = 1e-6
    dev = {k: torch.from_numpy(v).cuda() for k, v in
           dict(x=x, w=w, ab=ab, z=z, dt=dt_bias, al=a_log, nw=norm_w).items()}
    mixed = torch.empty(T, C, device="cuda")
    out = torch.full((T, nv * dv), float("nan"), device="cuda")
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    N_.check(lib.inl_cuda_causal_conv_silu(dev["x"].data_ptr(), C, C, dev["w"].data_ptr(), K, cu.ctypes.data,
                                           len(lengths), mixed.data_ptr(), C, s), "conv")
    N_.check(lib.inl_cuda_gated_delta_rule(mixed.data_ptr(), C, dev["ab"].data_ptr(), dev["ab"].data_ptr() + nv * 4,
                                           2 * nv, dev["z"].data_ptr(), nv * dv, dev["dt"].data_ptr(),
                                           dev["al"].data_ptr(), dev["nw"].data_ptr(), eps, nk, nv, dk, dv,
                                           cu.ctypes.data, len(lengths), out.data_ptr(), nv * dv, s), "delta rule")
    torch.cuda.synchronize()
    got_mixed, got = mixed.cpu().numpy(), out.cpu().numpy()
    for i in range(len(lengths)):
        a, b = int(cu[i]), int(cu[i + 1])
        if a == b:
            continue
        m = Q35.causal_conv_silu(x[a:b], w)
        assert np.abs(got_mixed[a:b] - m).max() < 1e-5
        q = m[:, :nk * dk].reshape(-1, nk, dk)
        k = m[:, nk * dk:2 * nk * dk].reshape(-1, nk, dk)
        v = m[:, 2 * nk * dk:].reshape(-1, nv, dv)
        q, k = np.repeat(q, nv // nk, axis=1), np.repeat(k, nv // nk, axis=1)
        beta = Q35.sigmoid(ab[a:b, :nv])
        g = Q35.softplus(ab[a:b, nv:] + dt_bias) * -np.exp(a_log)
        core = Q35.gated_delta_rule(q, k, v, g, beta)
        var = np.mean(core * core, axis=-1, keepdims=True)
        want = core / np.sqrt(var + eps) * norm_w * Q35.silu(z[a:b].reshape(-1, nv, dv))
        err = np.abs(got[a:b] - want.reshape(b - a, nv * dv)).max()
        assert err < 1e-4, (i, err)
