"""Qwen3 encoder forward on the CPU in torch f32 (MKL): TEST INFRASTRUCTURE ONLY.

The same function as ``oracle/qwen3.py`` (numpy), restated with torch CPU
tensors so that long texts (2048 tokens) and whole configurations finish in
seconds: the checker for the model-level parity tests at full size, and the
timed CPU arm of ``bench.py`` (``cpu_baseline`` and ``--impl reference``).
It follows crates/inl-text/src/qwen3/mod.rs line for line:

* ``DecoderLayer::forward`` (:282-297): ``h += Attn(RMSNorm(h)); h += MLP(RMSNorm(h))``;
* ``Attention::forward`` (:227-254): q/k/v projections, per-head q/k RMSNorm
  (eps from the config), half-split RoPE from the f64 table stored as f32
  (``RotaryTable::new``, :129-153), GQA, scale ``d^-1/2``, o projection;
* ``Mlp::forward`` (:110-116): ``down(silu(gate(x)) * up(x))``;
* ``forward_last`` (:339-358) and the f32 L2 of ``Qwen3Embedder::embed``
  (:438-470): final RMSNorm of each text's last token, ``x / sqrt(sum x^2 + 1e-12)``.

Attention is f32 softmax(q k^T * scale + mask) v per text; the packed form
(positions 0..L-1, keys inside the text) is the reference's left-padded batch
by its padding-invariance test (:646-669). Softmax is evaluated by
``scaled_dot_product_attention`` on CPU f32 tensors, an exact f32 evaluation
of the same expression (not a reduced-precision kernel).

Parity: the same status as ``oracle/qwen3.py``, unpinned by golden vectors
(partial); ``tests/test_oracle_qwen3.py`` pins this file to the numpy
restatement on the tiny configuration.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F


def _t(weights: dict, name: str) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(weights[name], dtype=np.float32))


def _rms(x: torch.Tensor, w: torch.Tensor | None, eps: float) -> torch.Tensor:
    y = x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps)
    return y * w if w is not None else y


def _rope_table(d: int, theta: float, n: int) -> tuple[torch.Tensor, torch.Tensor]:
    # f64 angles, stored as f32 (RotaryTable::new, qwen3/mod.rs:129-153)
    inv = 1.0 / theta ** (torch.arange(0, d // 2, dtype=torch.float64) * 2.0 / d)
    ang = torch.arange(n, dtype=torch.float64)[:, None] * inv[None, :]
    return ang.cos().float(), ang.sin().float()


def _rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    # x [L, heads, d]; half-split rotation x*[cos,cos] + rotate_half(x)*[sin,sin]
    half = x.shape[-1] // 2
    c = torch.cat([cos, cos], -1)[:, None, :]
    s = torch.cat([sin, sin], -1)[:, None, :]
    rot = torch.cat([-x[..., half:], x[..., :half]], -1)
    return x * c + rot * s


class Qwen3Cpu:
    """The weights as torch CPU tensors, converted once (the bench times the
    forward only, as the reference's benchmarks time ``embed`` after load)."""

    def __init__(self, weights: dict, cfg: dict, threads: int | None = None):
        if threads:
            torch.set_num_threads(int(threads))
        self.cfg = cfg
        self.eps = float(cfg["rms_norm_eps"])
        self.hq, self.hkv = int(cfg["num_attention_heads"]), int(cfg["num_key_value_heads"])
        self.d = int(cfg.get("head_dim") or cfg["hidden_size"] // self.hq)
        self.theta = float(cfg["rope_theta"])
        self.embed = _t(weights, "embed_tokens.weight")
        self.norm = _t(weights, "norm.weight")
        self.layers = []
        for i in range(int(cfg["num_hidden_layers"])):
            p = f"layers.{i}."
            self.layers.append({
                "in": _t(weights, p + "input_layernorm.weight"),
                "post": _t(weights, p + "post_attention_layernorm.weight"),
                "qkv": torch.cat([_t(weights, p + "self_attn.q_proj.weight"), _t(weights, p + "self_attn.k_proj.weight"),
                                  _t(weights, p + "self_attn.v_proj.weight")], 0),
                "qn": _t(weights, p + "self_attn.q_norm.weight"),
                "kn": _t(weights, p + "self_attn.k_norm.weight"),
                "o": _t(weights, p + "self_attn.o_proj.weight"),
                "gu": torch.cat([_t(weights, p + "mlp.gate_proj.weight"), _t(weights, p + "mlp.up_proj.weight")], 0),
                "down": _t(weights, p + "mlp.down_proj.weight"),
            })

    @torch.no_grad()
    def hidden_states(self, ids: np.ndarray, cu_seqlens: np.ndarray, causal: bool = True) -> torch.Tensor:
        """Embedding + every layer, before the final norm: [T, H]
        (qwen3/mod.rs:339-358 without the final narrow/norm)."""
        cu = [int(c) for c in np.asarray(cu_seqlens)]
        T = cu[-1]
        hq, hkv, d, eps = self.hq, self.hkv, self.d, self.eps
        max_len = max((b - a for a, b in zip(cu[:-1], cu[1:])), default=1)
        cos, sin = _rope_table(d, self.theta, max(max_len, 1))
        h = self.embed[torch.from_numpy(np.asarray(ids, dtype=np.int64))]
        qo, ko = hq * d, hkv * d
        for w in self.layers:
            x = _rms(h, w["in"], eps)
            qkv = x @ w["qkv"].T
            q = _rms(qkv[:, :qo].reshape(T, hq, d), w["qn"], eps)
            k = _rms(qkv[:, qo:qo + ko].reshape(T, hkv, d), w["kn"], eps)
            v = qkv[:, qo + ko:].reshape(T, hkv, d)
            out = torch.empty(T, hq, d)
            for s, e in zip(cu[:-1], cu[1:]):
                L = e - s
                if L == 0:
                    continue
                qs = _rope(q[s:e], cos[:L], sin[:L]).transpose(0, 1)
                ks = _rope(k[s:e], cos[:L], sin[:L]).transpose(0, 1)
                vs = v[s:e].transpose(0, 1)
                o = F.scaled_dot_product_attention(qs[None], ks[None], vs[None], is_causal=causal,
                                                   scale=d ** -0.5, enable_gqa=True)[0]
                out[s:e] = o.transpose(0, 1)
            h = h + out.reshape(T, qo) @ w["o"].T
            x = _rms(h, w["post"], eps)
            gu = x @ w["gu"].T
            inter = gu.shape[1] // 2
            h = h + (F.silu(gu[:, :inter]) * gu[:, inter:]) @ w["down"].T
        return h

    @torch.no_grad()
    def embed_last(self, ids: np.ndarray, cu_seqlens: np.ndarray) -> np.ndarray:
        """Dense embeddings [n, H] (qwen3/mod.rs:339-358, :438-470)."""
        cu = np.asarray(cu_seqlens, dtype=np.int64)
        h = self.hidden_states(ids, cu, causal=True)
        last = _rms(h[torch.from_numpy(cu[1:] - 1)], self.norm, self.eps)
        return (last / torch.sqrt((last * last).sum(-1, keepdim=True) + 1e-12)).numpy()

    @torch.no_grad()
    def encode_late(self, projection: np.ndarray, ids: np.ndarray, cu_seqlens: np.ndarray) -> np.ndarray:
        """Per-token late vectors [T, out]: bidirectional tower, final RMSNorm
        on every token, projection, F.normalize with clamp 1e-12
        (crates/inl-late/src/native.rs:646-661; the non-causal mask branch of
        crates/inl-late/src/qwen3_5.rs:914-927)."""
        h = self.hidden_states(ids, cu_seqlens, causal=False)
        y = _rms(h, self.norm, self.eps) @ torch.from_numpy(np.asarray(projection, dtype=np.float32)).T
        return (y / y.norm(dim=-1, keepdim=True).clamp_min(1e-12)).numpy()
