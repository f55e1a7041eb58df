"""CPU oracle for the GLM-4 MoE attention block.

TEST INFRASTRUCTURE ONLY (see oracle/moe_oracle.py): imported by ``tests/`` as
the checker of the device attention path and as the host attention stand-in of
the runtime tests; the product package never imports it.

Restates, in the same numpy expression order (so the same bits on the same
numpy / OpenBLAS):

* ``glm4_attention_block`` -- offload_runtime/executors/glm4_moe.py:112-162
  (input RMSNorm, q/k/v projections with optional bias, per-head q/k RMS norm,
  partial rotary embedding, grouped-query repeat, causal softmax attention over
  the whole sequence at positions 0..T-1, o_proj, residual);
* ``rope`` / ``partial_rope`` / ``repeat_kv`` / ``rms_norm_no_weight`` --
  offload_runtime/executors/_common.py:106-155;
* ``glm4_decoder_layer`` -- glm4_moe.py:88-108 (attention, then the MoE block or
  the dense MLP by ``metadata["is_moe"]``).

``tests/golden/make_golden.py`` records the reference's own ``_attention_block``
outputs; ``tests/test_oracle_golden.py`` asserts this restatement reproduces
them bit for bit.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any

import numpy as np

from .moe_oracle import dense_mlp_block, moe_block, rms_norm


@dataclass
class AttnConfig:
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    eps: float = 1e-5
    rope_theta: float = 1_000_000.0
    partial_rotary_factor: float = 0.5

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    @classmethod
    def from_hf(cls, config: dict[str, Any]) -> "AttnConfig":
        """Same defaults as glm4_moe.py:70-84."""
        heads = config["num_attention_heads"]
        return cls(hidden=config["hidden_size"], heads=heads,
                   kv_heads=config.get("num_key_value_heads", heads),
                   head_dim=config.get("head_dim", config["hidden_size"] // heads),
                   eps=config.get("rms_norm_eps", 1e-5),
                   rope_theta=config.get("rope_theta", 1000000.0),
                   partial_rotary_factor=config.get("partial_rotary_factor", 0.5))


def rms_norm_no_weight(x: np.ndarray, eps: float) -> np.ndarray:
    """_common.py:139-142."""
    denom = np.sqrt(np.mean(x ** 2, axis=-1, keepdims=True) + eps)
    return x / denom


def rope_tables(positions: np.ndarray, dim: int, base: float) -> tuple[np.ndarray, np.ndarray]:
    """cos / sin of the rotary angles of _common.py:112-117: frequencies and angles
    in float64, rounded to float32 before cos / sin."""
    half = dim // 2
    freqs = 1.0 / (base ** (np.arange(0, half, dtype=np.float64) / half))
    angles = np.outer(positions.astype(np.float64), freqs).astype(np.float32)
    return np.cos(angles), np.sin(angles)


def rope(q: np.ndarray, k: np.ndarray, positions: np.ndarray, dim: int, base: float
         ) -> tuple[np.ndarray, np.ndarray]:
    """_common.py:106-126: rotate-half rotary embedding over the last axis."""
    half = dim // 2
    cos, sin = rope_tables(positions, dim, base)

    def rot(a: np.ndarray) -> np.ndarray:
        a1, a2 = a[..., :half], a[..., half:]
        return np.concatenate([a1 * cos - a2 * sin, a2 * cos + a1 * sin], axis=-1)

    return rot(q), rot(k)


def partial_rope(q: np.ndarray, k: np.ndarray, positions: np.ndarray, head_dim: int,
                 rotary_dim: int, base: float) -> tuple[np.ndarray, np.ndarray]:
    """_common.py:145-155: the rotary embedding on the first ``rotary_dim`` dims only."""
    qr, kr = rope(q[..., :rotary_dim], k[..., :rotary_dim], positions, rotary_dim, base)
    return (np.concatenate([qr, q[..., rotary_dim:]], axis=-1),
            np.concatenate([kr, k[..., rotary_dim:]], axis=-1))


def repeat_kv(a: np.ndarray, n_rep: int) -> np.ndarray:
    """_common.py:131-135."""
    return a if n_rep == 1 else np.repeat(a, n_rep, axis=0)


def softmax(x: np.ndarray) -> np.ndarray:
    """_common.py:87-90 over the last axis."""
    e = np.exp(x - x.max(axis=-1, keepdims=True))
    return e / e.sum(axis=-1, keepdims=True)


def glm4_attention_block(x: np.ndarray, t: Any, cfg: AttnConfig) -> np.ndarray:
    """``x + o_proj(attention(rms_norm(x)))``, glm4_moe.py:112-162."""
    T = x.shape[0]
    nh, nkv, hd = cfg.heads, cfg.kv_heads, cfg.head_dim
    h = rms_norm(x, t["input_layernorm.weight"], cfg.eps)
    proj = {}
    for name in ("q", "k", "v"):
        a = h @ t[f"self_attn.{name}_proj.weight"].T
        if f"self_attn.{name}_proj.bias" in t:
            a = a + t[f"self_attn.{name}_proj.bias"]
        proj[name] = a
    q = proj["q"].reshape(T, nh, hd).transpose(1, 0, 2)
    k = proj["k"].reshape(T, nkv, hd).transpose(1, 0, 2)
    v = proj["v"].reshape(T, nkv, hd).transpose(1, 0, 2)
    if "self_attn.q_norm.weight" in t:
        q = rms_norm_no_weight(q, cfg.eps) * t["self_attn.q_norm.weight"]
    if "self_attn.k_norm.weight" in t:
        k = rms_norm_no_weight(k, cfg.eps) * t["self_attn.k_norm.weight"]
    pos = np.arange(T, dtype=np.float32)
    if cfg.rotary_dim < hd:
        q, k = partial_rope(q, k, pos, hd, cfg.rotary_dim, cfg.rope_theta)
    else:
        q, k = rope(q, k, pos, hd, cfg.rope_theta)
    k = repeat_kv(k, nh // nkv)
    v = repeat_kv(v, nh // nkv)
    scores = (q @ k.transpose(0, 2, 1)) / math.sqrt(hd)
    scores = scores + np.triu(np.full((T, T), -1e10, dtype=np.float32), k=1)
    o = softmax(scores) @ v
    o = o.transpose(1, 0, 2).reshape(T, nh * hd)
    return x + o @ t["self_attn.o_proj.weight"].T


def glm4_decoder_layer(x: np.ndarray, t: Any, attn: AttnConfig, moe_cfg: Any,
                       is_moe: bool) -> np.ndarray:
    """glm4_moe.py:88-108: attention, then the MoE block or the dense MLP."""
    x = glm4_attention_block(x, t, attn)
    if is_moe:
        return moe_block(x, t, moe_cfg)[0]
    return dense_mlp_block(x, t, attn.eps)
