"""Oracle: numpy restatement of the N730 decoder-layer math.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Follows the reference's own CPU restatement of each sub-step:

* RMSNorm: ``x / sqrt(mean(x64**2) + eps) * w`` (``src-code/diagnose_binary.py:160-162``,
  final norm ``src-code/inference.py:656-659``).
* RoPE: rotate_half pairs ``(i, i+hd/2)``, ``x0' = x0*c - x1*s``, ``x1' = x1*c + x0*s``,
  ``pos = s + offset`` (``diagnose_binary.py:164-180``); table in fp32 as
  ``freq = 1/powf(theta, 2i/hd)``, ``angle = pos*freq`` (``src-code/cpp/n730_cuda.cu:650-661``).
* Attention: GQA ``kv_h = h // (nh/nkv)``, ``S = QK^T/sqrt(hd)``, causal mask to
  -1e4 when ``seq_q > 1``, softmax ``exp(max(s-m, -50)) / (sum + 1e-9)``, ``O = PV``
  (``diagnose_binary.py:244-253``, clamp from ``n730_cuda.cu:238``, mask ``:259-275``).
* SwiGLU: ``g/(1+exp(-g)) * u`` (``diagnose_binary.py:306-307``).
* Residual adds and q/k/v biases as in ``inference.py:488-643``.
* Final RMSNorm + ``lm_head`` (tied to the embedding when absent), logits of the
  last position only (``inference.py:648-669``).
"""
from __future__ import annotations

import math

import numpy as np


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.asarray(x, np.float32)
    rms = np.sqrt((x.astype(np.float64) ** 2).mean(axis=-1, keepdims=True) + eps)
    return (x / rms * w).astype(np.float32)


def rope_table(max_pos: int, head_dim: int, theta: float):
    """fp32 cos/sin tables [max_pos, head_dim/2] following n730_cuda.cu:650-661."""
    h2 = head_dim // 2
    i = np.arange(h2, dtype=np.float32)
    expo = (np.float32(2) * i) / np.float32(head_dim)
    freq = np.float32(1.0) / np.power(np.float32(theta), expo).astype(np.float32)
    pos = np.arange(max_pos, dtype=np.float32)[:, None]
    ang = (pos * freq[None, :]).astype(np.float32)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def apply_rope(x: np.ndarray, n_heads: int, head_dim: int, offset: int,
               cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    sl = x.shape[0]
    x = x.reshape(sl, n_heads, head_dim).astype(np.float32)
    h2 = head_dim // 2
    c = cos[offset:offset + sl][:, None, :]
    s = sin[offset:offset + sl][:, None, :]
    x0, x1 = x[..., :h2].copy(), x[..., h2:].copy()
    out = np.empty_like(x)
    out[..., :h2] = x0 * c - x1 * s
    out[..., h2:] = x1 * c + x0 * s
    return out.reshape(sl, n_heads * head_dim)


def attention(q: np.ndarray, k_all: np.ndarray, v_all: np.ndarray,
              n_heads: int, n_kv: int, head_dim: int, offset: int) -> np.ndarray:
    """q [sq, nh*hd]; k_all/v_all [total, nkv*hd] -> [sq, nh*hd]."""
    sq = q.shape[0]
    total = k_all.shape[0]
    grp = n_heads // n_kv
    qr = q.reshape(sq, n_heads, head_dim).astype(np.float32)
    kr = np.repeat(k_all.reshape(total, n_kv, head_dim), grp, axis=1).astype(np.float32)
    vr = np.repeat(v_all.reshape(total, n_kv, head_dim), grp, axis=1).astype(np.float32)
    sc = np.einsum("shd,thd->sht", qr, kr) / np.float32(math.sqrt(head_dim))
    if sq > 1:
        qpos = offset + np.arange(sq)[:, None, None]
        kpos = np.arange(total)[None, None, :]
        sc = np.where(kpos > qpos, np.float32(-1e4), sc)
    sc = sc - sc.max(axis=-1, keepdims=True)
    p = np.exp(np.maximum(sc, -50.0)).astype(np.float32)
    p = p / (p.sum(axis=-1, keepdims=True) + np.float32(1e-9))
    return np.einsum("sht,thd->shd", p, vr).reshape(sq, n_heads * head_dim).astype(np.float32)


def swiglu(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = g.astype(np.float32)
    return (g / (np.float32(1.0) + np.exp(-g)) * u).astype(np.float32)


class _Cfg:
    """Reads either the reference ModelConfig names (inference.py:145-208) or
    the engine's shape names."""

    def __init__(self, c):
        g = lambda *names: next(getattr(c, n) for n in names if hasattr(c, n))
        self.hidden_size = g("hidden_size", "hidden")
        self.num_hidden_layers = g("num_hidden_layers", "layers")
        self.num_attention_heads = g("num_attention_heads", "heads")
        self.num_kv_heads = g("num_kv_heads", "kv_heads")
        self.head_dim = g("head_dim")
        self.rms_norm_eps = g("rms_norm_eps", "rms_eps")
        self.rope_theta = g("rope_theta")


class OracleDecoder:
    """Whole-model numpy forward with an fp32 KV cache (the reference keeps fp32 KV).

    ``weights`` maps HF tensor names to fp32 arrays (already dequantised with
    ``oracle.quant``); norms default to ones when absent
    (``inference.py:405-406``).
    """

    def __init__(self, cfg, weights: dict, max_pos: int = 4096):
        cfg = _Cfg(cfg)
        self.cfg = cfg
        self.w = weights
        self.cos, self.sin = rope_table(max_pos, cfg.head_dim, cfg.rope_theta)
        L = cfg.num_hidden_layers
        self.k = [np.zeros((0, cfg.num_kv_heads * cfg.head_dim), np.float32) for _ in range(L)]
        self.v = [np.zeros((0, cfg.num_kv_heads * cfg.head_dim), np.float32) for _ in range(L)]
        self.seq_len = 0
        self.last_hidden = None

    def _norm(self, name):
        return self.w.get(name, np.ones(self.cfg.hidden_size, np.float32))

    def _lin(self, x, name):
        y = x @ self.w[name + ".weight"].T
        b = self.w.get(name + ".bias")
        if b is not None:
            y = y + b
        return y.astype(np.float32)

    def layer(self, i: int, x: np.ndarray, offset: int) -> np.ndarray:
        c = self.cfg
        p = f"model.layers.{i}"
        h = rms_norm(x, self._norm(f"{p}.input_layernorm.weight"), c.rms_norm_eps)
        q = self._lin(h, f"{p}.self_attn.q_proj")
        k = self._lin(h, f"{p}.self_attn.k_proj")
        v = self._lin(h, f"{p}.self_attn.v_proj")
        q = apply_rope(q, c.num_attention_heads, c.head_dim, offset, self.cos, self.sin)
        k = apply_rope(k, c.num_kv_heads, c.head_dim, offset, self.cos, self.sin)
        self.k[i] = np.concatenate([self.k[i], k])
        self.v[i] = np.concatenate([self.v[i], v])
        a = attention(q, self.k[i], self.v[i], c.num_attention_heads, c.num_kv_heads,
                      c.head_dim, offset)
        x = (x + self._lin(a, f"{p}.self_attn.o_proj")).astype(np.float32)
        h2 = rms_norm(x, self._norm(f"{p}.post_attention_layernorm.weight"), c.rms_norm_eps)
        m = swiglu(self._lin(h2, f"{p}.mlp.gate_proj"), self._lin(h2, f"{p}.mlp.up_proj"))
        return (x + self._lin(m, f"{p}.mlp.down_proj")).astype(np.float32)

    def forward(self, token_ids) -> np.ndarray:
        c = self.cfg
        ids = np.asarray(token_ids, np.int64)
        offset = self.seq_len
        x = self.w["model.embed_tokens.weight"][ids].astype(np.float32)
        for i in range(c.num_hidden_layers):
            x = self.layer(i, x, offset)
        self.seq_len += len(ids)
        self.last_hidden = x
        last = rms_norm(x[-1], self._norm("model.norm.weight"), c.rms_norm_eps)
        lm = self.w.get("lm_head.weight", self.w["model.embed_tokens.weight"])
        return (last @ lm.T).astype(np.float32)
