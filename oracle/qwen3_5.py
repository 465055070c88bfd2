"""Qwen3.5 text tower of the late-interaction engine on the CPU (numpy):
TEST INFRASTRUCTURE ONLY.

Restates crates/inl-late/src/qwen3_5.rs (Qwen35Text: Gated DeltaNet
"linear_attention" layers and gated "full_attention" layers) and the late
head of crates/inl-late/src/native.rs:631-683 (Dense projection,
F.normalize, task skiplist), over one text at a time (packed inputs: no
padding; the reference right-pads a batch, masks padded keys in full
attention, and its causal convolution and delta rule never look ahead, so a
text's rows are the same function).

The delta rule is restated in its recurrent form, the definition the
reference pins its chunked form against (the `recurrent` helper of its unit
tests, crates/inl-late/src/qwen3_5.rs:960-1000; the gated delta rule of
Yang, Kautz and Hatamizadeh, "Gated Delta Networks"): per value head, with
S_0 = 0 and alpha_t = exp(g_t),

    u_t = beta_t (v_t - alpha_t S_{t-1}^T k_t)
    S_t = alpha_t S_{t-1} + k_t u_t^T
    o_t = S_t^T q_t,

q and k L2-normalised (1e-6 inside the root), q scaled by dk^-1/2. The state
is kept in f64.

Parity is pinned on the reference's tiny_qwen3_5_late fixture (golden.json,
asserted by crates/inl-late/tests/tiny_golden.rs: max |d| < 1e-4 for every
token vector, batched and alone, query and document tasks).
"""
from __future__ import annotations

import numpy as np

from .common import softmax, silu


def _w(weights: dict, name: str) -> np.ndarray:
    return np.asarray(weights[name], dtype=np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """x rounded to the nearest bf16 (ties to even), as f32."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return (((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32)


def linear(x: np.ndarray, w: np.ndarray, operands: str = "f32") -> np.ndarray:
    """``x @ w^T`` in f32. ``operands="bf16"`` rounds both factors to bf16
    first and keeps the f32 sum: the CUDA tower's bf16 mode (bf16 products on
    the tensor cores, f32 activations, norms and recurrence). The reference's
    own bf16 tower has no golden vectors; this mode is what the CUDA bf16 path
    is checked against."""
    if operands == "bf16":
        return bf16_round(x) @ bf16_round(w).T
    return x @ w.T


def root_prefix(weights: dict) -> str:
    """The text model's root, as crates/inl-late/src/native.rs:519-531 finds it."""
    for p in ("language_model", "model.language_model", "model", ""):
        if (f"{p}.embed_tokens.weight" if p else "embed_tokens.weight") in weights:
            return f"{p}." if p else ""
    raise KeyError("no embed_tokens.weight")


def text_config(cfg: dict) -> dict:
    """A nested ``text_config`` or a flat one (Config::parse, qwen3_5.rs:90-103)."""
    return cfg.get("text_config", cfg)


def zc_rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """Zero-centred RMSNorm ``x / rms(x) * (1 + w)`` (qwen3_5.rs:188-206)."""
    x = x.astype(np.float32, copy=False)
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    return (x / np.sqrt(var + np.float32(eps)) * (np.float32(1) + w)).astype(np.float32)


def sigmoid(x: np.ndarray) -> np.ndarray:
    return (np.float32(1) / (np.float32(1) + np.exp(-x))).astype(np.float32)


def softplus(x: np.ndarray) -> np.ndarray:
    """``log(1 + exp(x))`` in the stable form of qwen3_5.rs:547-551."""
    return (np.maximum(x, 0) + np.log1p(np.exp(-np.abs(x)))).astype(np.float32)


def l2norm(x: np.ndarray) -> np.ndarray:
    """``x / sqrt(sum x^2 + 1e-6)`` over the last axis (qwen3_5.rs:553-557)."""
    return x / np.sqrt(np.sum(x * x, axis=-1, keepdims=True) + 1e-6)


def causal_conv_silu(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """Depthwise causal convolution then SiLU (qwen3_5.rs:463-479).

    x: [T, C]; w: [C, K]; out[t, c] = silu(sum_j x[t - K + 1 + j, c] w[c, j]),
    zero before the first token.
    """
    T, C = x.shape
    K = w.shape[1]
    xp = np.concatenate([np.zeros((K - 1, C), dtype=np.float32), x], axis=0)
    out = np.zeros((T, C), dtype=np.float32)
    for j in range(K):
        out += xp[j:j + T] * w[:, j]
    return silu(out)


def gated_delta_rule(q: np.ndarray, k: np.ndarray, v: np.ndarray, g: np.ndarray,
                     beta: np.ndarray) -> np.ndarray:
    """Recurrent gated delta rule. q, k: [T, H, dk]; v: [T, H, dv];
    g, beta: [T, H]. Returns [T, H, dv] (f32)."""
    T, H, dk = q.shape
    dv = v.shape[2]
    qn = l2norm(q.astype(np.float64)) * dk ** -0.5
    kn = l2norm(k.astype(np.float64))
    out = np.zeros((T, H, dv), dtype=np.float64)
    for h in range(H):
        S = np.zeros((dk, dv), dtype=np.float64)
        for t in range(T):
            S *= np.exp(np.float64(g[t, h]))
            u = np.float64(beta[t, h]) * (v[t, h].astype(np.float64) - S.T @ kn[t, h])
            S += np.outer(kn[t, h], u)
            out[t, h] = S.T @ qn[t, h]
    return out.astype(np.float32)


def gated_delta_rule_chunked(q: np.ndarray, k: np.ndarray, v: np.ndarray, g: np.ndarray,
                             beta: np.ndarray, chunk: int = 64) -> np.ndarray:
    """The same rule in its chunked (WY) form, the structure a tensor-core
    kernel computes (the reference's chunk_gated_delta_rule,
    crates/inl-late/src/qwen3_5.rs:612-739, restated; the WY form of Yang et
    al., "Parallelizing Linear Transformers with the Delta Rule over
    Sequence Length"). Per chunk of C tokens with local cumulative decay
    c_i = sum_{j<=i} g_j and D_ij = exp(c_i - c_j) (j <= i):

        A = strictly_lower((beta k) k^T * D)       U = (I + A)^-1 (beta v)
        W = (I + A)^-1 (beta k * exp(c))           u = U - W S
        o = (q * exp(c)) S + lower(q k^T * D) u
        S <- exp(c_C) S + (k * exp(c_C - c))^T u

    (I + A)^-1 by forward substitution. Same shapes and result as
    gated_delta_rule."""
    T, H, dk = q.shape
    dv = v.shape[2]
    qn = l2norm(q.astype(np.float64)) * dk ** -0.5
    kn = l2norm(k.astype(np.float64))
    out = np.zeros((T, H, dv), dtype=np.float64)
    for h in range(H):
        S = np.zeros((dk, dv), dtype=np.float64)
        for c0 in range(0, T, chunk):
            c1 = min(T, c0 + chunk)
            C = c1 - c0
            Q, K, V = qn[c0:c1, h], kn[c0:c1, h], v[c0:c1, h].astype(np.float64)
            b = beta[c0:c1, h].astype(np.float64)[:, None]
            cum = np.cumsum(g[c0:c1, h].astype(np.float64))
            D = np.tril(np.exp(np.minimum(cum[:, None] - cum[None, :], 0.0)))
            A = np.tril((b * K) @ K.T * D, -1)
            M = np.eye(C) + A  # unit lower triangular: solve by forward substitution
            Y = np.concatenate([b * V, b * K * np.exp(cum)[:, None]], axis=1)
            X = np.zeros_like(Y)
            for i in range(C):
                X[i] = Y[i] - M[i, :i] @ X[:i]
            U, W = X[:, :dv], X[:, dv:]
            u = U - W @ S
            out[c0:c1, h] = (Q * np.exp(cum)[:, None]) @ S + (Q @ K.T * D) @ u
            S = np.exp(cum[-1]) * S + (K * np.exp(cum[-1] - cum)[:, None]).T @ u
    return out.astype(np.float32)


def gated_deltanet(weights: dict, cfg: dict, p: str, x: np.ndarray, operands: str = "f32") -> np.ndarray:
    """GatedDeltaNet::forward (qwen3_5.rs:481-545) for one text; x: [T, H] normed."""
    T = x.shape[0]
    nk, nv = int(cfg["linear_num_key_heads"]), int(cfg["linear_num_value_heads"])
    dk, dv = int(cfg["linear_key_head_dim"]), int(cfg["linear_value_head_dim"])
    eps = float(cfg["rms_norm_eps"])
    conv_w = _w(weights, p + "conv1d.weight").reshape(2 * nk * dk + nv * dv, -1)
    mixed = causal_conv_silu(linear(x, _w(weights, p + "in_proj_qkv.weight"), operands), conv_w)
    beta = sigmoid(linear(x, _w(weights, p + "in_proj_b.weight"), operands))
    a = linear(x, _w(weights, p + "in_proj_a.weight"), operands) + _w(weights, p + "dt_bias")
    g = softplus(a) * -np.exp(_w(weights, p + "A_log"))
    q = mixed[:, :nk * dk].reshape(T, nk, dk)
    k = mixed[:, nk * dk:2 * nk * dk].reshape(T, nk, dk)
    v = mixed[:, 2 * nk * dk:].reshape(T, nv, dv)
    if nv > nk:  # value head j reads key head j // (nv / nk)
        q = np.repeat(q, nv // nk, axis=1)
        k = np.repeat(k, nv // nk, axis=1)
    core = gated_delta_rule(q, k, v, g, beta)
    # gated RMSNorm per value head with the plain weight, then silu(z)
    z = linear(x, _w(weights, p + "in_proj_z.weight"), operands).reshape(T, nv, dv)
    var = np.mean(core * core, axis=-1, keepdims=True, dtype=np.float32)
    normed = core / np.sqrt(var + np.float32(eps)) * _w(weights, p + "norm.weight")
    out = (normed * silu(z)).reshape(T, nv * dv)
    return linear(out, _w(weights, p + "out_proj.weight"), operands).astype(np.float32)


def rotary(cfg: dict, positions: int) -> tuple[np.ndarray, np.ndarray, int]:
    """cos / sin ``[positions, rotary_dim / 2]`` computed in f32 (qwen3_5.rs:940-958);
    rotary_dim = head_dim * partial_rotary_factor. Text inputs give the three
    M-RoPE axes one position, so it is plain partial RoPE."""
    rp = cfg["rope_parameters"]
    dim = int(int(cfg["head_dim"]) * float(rp.get("partial_rotary_factor", 1.0)))
    theta = np.float32(rp["rope_theta"])
    inv = np.array([np.float32(1) / theta ** np.float32((2 * i) / dim) for i in range(dim // 2)], dtype=np.float32)
    ang = np.arange(positions, dtype=np.float32)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32), dim


def rope_partial(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, dim: int) -> np.ndarray:
    """Half-split rotation of the first ``dim`` features of each head
    (FullAttention::rope, qwen3_5.rs:286-300). x: [T, heads, hd]."""
    half = dim // 2
    x1, x2 = x[..., :half], x[..., half:dim]
    c, s = cos[:, None, :], sin[:, None, :]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s, x[..., dim:]], axis=-1).astype(np.float32)


def full_attention(weights: dict, cfg: dict, p: str, x: np.ndarray, cos, sin, rdim: int,
                   operands: str = "f32") -> np.ndarray:
    """FullAttention::forward (qwen3_5.rs:302-350) for one text, no padding."""
    T = x.shape[0]
    hq, hkv, hd = int(cfg["num_attention_heads"]), int(cfg["num_key_value_heads"]), int(cfg["head_dim"])
    eps = float(cfg["rms_norm_eps"])
    qg = linear(x, _w(weights, p + "q_proj.weight"), operands).reshape(T, hq, 2 * hd)
    q = zc_rms_norm(qg[..., :hd], _w(weights, p + "q_norm.weight"), eps)
    gate = qg[..., hd:].reshape(T, hq * hd)
    k = zc_rms_norm(linear(x, _w(weights, p + "k_proj.weight"), operands).reshape(T, hkv, hd),
                    _w(weights, p + "k_norm.weight"), eps)
    v = linear(x, _w(weights, p + "v_proj.weight"), operands).reshape(T, hkv, hd)
    q = rope_partial(q, cos[:T], sin[:T], rdim)
    k = rope_partial(k, cos[:T], sin[:T], rdim)
    rep = hq // hkv
    kk, vv = np.repeat(k, rep, axis=1), np.repeat(v, rep, axis=1)
    s = np.einsum("qhd,khd->hqk", q, kk, dtype=np.float32) * np.float32(hd ** -0.5)
    if cfg.get("is_causal", True):  # additive -1e4 on future keys (qwen3_5.rs:16, 917-938)
        s = s + np.where(np.arange(T)[None, :] > np.arange(T)[:, None], np.float32(-1e4), np.float32(0))[None]
    o = np.einsum("hqk,khd->qhd", softmax(s, axis=-1), vv, dtype=np.float32).reshape(T, hq * hd)
    return linear(o * sigmoid(gate), _w(weights, p + "o_proj.weight"), operands).astype(np.float32)


def hidden(weights: dict, config: dict, ids: np.ndarray, operands: str = "f32") -> np.ndarray:
    """``last_hidden_state`` of one text (Qwen35Text::forward, qwen3_5.rs:893-915);
    ``operands`` as in :func:`linear`."""
    cfg = text_config(config)
    root = root_prefix(weights)
    eps = float(cfg["rms_norm_eps"])
    h = _w(weights, root + "embed_tokens.weight")[np.asarray(ids, dtype=np.int64)]
    cos, sin, rdim = rotary(cfg, max(len(ids), 1))
    for i, kind in enumerate(cfg["layer_types"]):
        p = f"{root}layers.{i}."
        x = zc_rms_norm(h, _w(weights, p + "input_layernorm.weight"), eps)
        if kind == "linear_attention":
            h = h + gated_deltanet(weights, cfg, p + "linear_attn.", x, operands)
        else:
            h = h + full_attention(weights, cfg, p + "self_attn.", x, cos, sin, rdim, operands)
        x = zc_rms_norm(h, _w(weights, p + "post_attention_layernorm.weight"), eps)
        m = silu(linear(x, _w(weights, p + "mlp.gate_proj.weight"), operands)) * linear(
            x, _w(weights, p + "mlp.up_proj.weight"), operands)
        h = h + linear(m, _w(weights, p + "mlp.down_proj.weight"), operands)
    return zc_rms_norm(h, _w(weights, root + "norm.weight"), eps)


def late_vectors(weights: dict, config: dict, projection: np.ndarray, bias: np.ndarray | None,
                 ids: np.ndarray, skip=frozenset(), normalize: bool = True, operands: str = "f32") -> np.ndarray:
    """One text's kept token vectors (encode_batch, crates/inl-late/src/native.rs:631-683):
    ``hidden @ W^T (+ b)``, ``x / max(|x|, 1e-12)``, skiplist tokens dropped;
    ``operands`` as in :func:`linear`."""
    y = linear(hidden(weights, config, ids, operands), projection.astype(np.float32), operands)
    if bias is not None:
        y = y + bias
    if normalize:
        y = y / np.maximum(np.sqrt(np.sum(y * y, axis=-1, keepdims=True)), np.float32(1e-12))
    keep = ~np.isin(np.asarray(ids), np.fromiter(skip, dtype=np.int64)) if skip else np.ones(len(ids), bool)
    return y[keep].astype(np.float32)
