"""CPU oracle for the MoE feed-forward block.

TEST INFRASTRUCTURE ONLY.  This module is the checker, never the product:
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
``--impl reference`` leg may import it.  The product path (``moe_sm100``) never
imports anything under ``oracle/`` and fails loudly when its CUDA library is
missing.

What it restates (reference paths are relative to the disk-mem-off project):

* ``rms_norm``  -- offload_runtime/executors/_common.py:73-75
* ``silu``      -- offload_runtime/executors/_common.py:83-84
* ``softmax``   -- offload_runtime/executors/_common.py:87-90
* ``sigmoid``   -- offload_runtime/executors/qwen3_next.py:31-32
* ``route``     -- offload_runtime/executors/glm4_moe.py:180-200 (router logits, biased
  softmax, top-k, renormalise, routed_scaling_factor) and
  offload_runtime/executors/qwen3_next.py:277-293 (plain softmax, no scale)
* ``moe_block`` -- offload_runtime/executors/glm4_moe.py:176-240 and
  offload_runtime/executors/qwen3_next.py:273-333 (dispatch, SwiGLU experts, combine,
  shared expert, Qwen3 sigmoid shared gate, residual)
* ``int8_pc_*`` -- the per-output-channel INT8 format, an extension of
  offload_runtime/quantize.py:24-50 (``Int8Dequantizer``: ``(q - zero_point) * scale``)
  where ``scale`` becomes one fp16 value per output row.

The numpy call sequence of the reference is kept where it decides the bits of the
result (fp32 matmul shapes, the order in which expert contributions are added to
a token), so on the same numpy/OpenBLAS this oracle reproduces the reference
executor bit for bit.  ``tests/golden/`` pins it: the fixtures there were produced
by running the reference itself (``tests/golden/make_golden.py``).

Two routing contracts differ from the reference on purpose and are documented:

* ties: the reference selects with ``np.argpartition`` + an unstable
  ``np.argsort``, so equal scores resolve in a numpy-defined order.  This oracle
  (and the CUDA kernels) order slots by descending score and break exact ties by
  the lower expert id.  On tie-free inputs both agree exactly.
* ``score_func="sigmoid"`` is the HuggingFace GLM-4.x rule (sigmoid scores, bias
  added for selection only, unbiased weights), which the reference does not
  implement; it is pinned against transformers' ``Glm4MoeMoE.route_tokens_to_experts``.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import numpy as np

SCORE_SOFTMAX = "softmax"
SCORE_SIGMOID = "sigmoid"


@dataclass
class OracleConfig:
    hidden: int
    n_experts: int
    top_k: int
    inter: int
    shared_inter: int = 0
    score_func: str = SCORE_SOFTMAX
    use_bias: bool = True  # GLM adds e_score_correction_bias; Qwen3 has none
    norm_topk_prob: bool = True
    routed_scaling_factor: float = 1.0
    eps: float = 1e-6
    shared_prefix: str = "mlp.shared_experts."  # GLM; Qwen3 uses "mlp.shared_expert."
    extra: dict[str, Any] = field(default_factory=dict)


# ---------------------------------------------------------------------------
# elementwise primitives (same numpy expressions as the reference, so same bits)
# ---------------------------------------------------------------------------

def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """_common.py:73-75: ``w * (x / sqrt(mean(x**2) + eps))`` in fp32."""
    denom = np.sqrt(np.mean(x ** 2, axis=-1, keepdims=True) + eps)
    return w * (x / denom)


def silu(x: np.ndarray) -> np.ndarray:
    """_common.py:83-84."""
    return x / (1.0 + np.exp(-x))


def softmax(x: np.ndarray) -> np.ndarray:
    """_common.py:87-90 (last axis, max-subtracted)."""
    e = np.exp(x - x.max(axis=-1, keepdims=True))
    return e / e.sum(axis=-1, keepdims=True)


def sigmoid(x: np.ndarray) -> np.ndarray:
    """qwen3_next.py:31-32."""
    return 1.0 / (1.0 + np.exp(-x))


# ---------------------------------------------------------------------------
# routing
# ---------------------------------------------------------------------------

def select_topk(score: np.ndarray, k: int) -> np.ndarray:
    """Top-k expert ids per row, by descending score, exact ties -> lower id.

    Equals the reference's ``argpartition(-p, k)[:, :k]`` followed by
    ``argsort(-w)`` (glm4_moe.py:189-195) whenever the row has no exact ties.
    """
    n_rows, n_exp = score.shape
    ids = np.arange(n_exp)
    out = np.empty((n_rows, k), dtype=np.int64)
    for r in range(n_rows):
        # lexsort: last key is primary -> sort by -score, then by id
        order = np.lexsort((ids, -score[r].astype(np.float64)))
        out[r] = order[:k]
    return out


def route(h: np.ndarray, gate_w: np.ndarray, bias: np.ndarray | None, cfg: OracleConfig
          ) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Router + top-k + renormalise + scale.

    Returns ``(topk_ids [T,K] int64, topk_w [T,K] f32, logits [T,E] f32)``.
    softmax mode: glm4_moe.py:181-200 (bias added to the logits before the softmax;
    Qwen3 passes ``bias=None`` and scale 1.0, qwen3_next.py:278-293).
    sigmoid mode: scores = sigmoid(logits); selection on scores + bias; weights are
    the unbiased scores (transformers Glm4MoeMoE.route_tokens_to_experts).
    """
    logits = h @ gate_w.T
    k = cfg.top_k
    if cfg.score_func == SCORE_SOFTMAX:
        if bias is not None:
            logits = logits + bias
        probs = softmax(logits)
        ids = select_topk(probs, k)
        w = np.take_along_axis(probs, ids, axis=-1)
    elif cfg.score_func == SCORE_SIGMOID:
        scores = sigmoid(logits)
        choice = scores + bias if bias is not None else scores
        ids = select_topk(choice, k)
        w = np.take_along_axis(scores, ids, axis=-1)
    else:
        raise ValueError(f"unknown score_func {cfg.score_func!r}")
    if cfg.norm_topk_prob:
        w = w / (w.sum(axis=-1, keepdims=True) + 1e-20)
    w = w * np.float32(cfg.routed_scaling_factor)
    return ids, w.astype(np.float32, copy=False), logits


def permutation(ids: np.ndarray, n_experts: int) -> tuple[np.ndarray, np.ndarray]:
    """Expert-major dispatch order.

    Returns ``(expert_offsets [E+1], perm [T*K])`` where ``perm[r] = t*K + j`` lists the
    (token, slot) pairs of expert e in rows ``offsets[e]:offsets[e+1]``, tokens ascending.
    This is the order in which glm4_moe.py:208-215 gathers ``h[token_mask]``.
    """
    t_count, k = ids.shape
    flat = ids.reshape(-1)
    counts = np.bincount(flat, minlength=n_experts)
    offsets = np.zeros(n_experts + 1, dtype=np.int64)
    np.cumsum(counts, out=offsets[1:])
    # stable sort by expert keeps (token, slot) ascending inside an expert
    perm = np.argsort(flat, kind="stable")
    return offsets, perm


# ---------------------------------------------------------------------------
# the block
# ---------------------------------------------------------------------------

def _swiglu(xin: np.ndarray, wg: np.ndarray, wu: np.ndarray, wd: np.ndarray) -> np.ndarray:
    """glm4_moe.py:222-224: ``(silu(x Wg^T) * (x Wu^T)) Wd^T``."""
    return (silu(xin @ wg.T) * (xin @ wu.T)) @ wd.T


def dense_mlp_block(x: np.ndarray, t: dict[str, np.ndarray], eps: float) -> np.ndarray:
    """glm4_moe.py:166-172 (``_dense_mlp_block`` of first_k_dense_replace layers):
    ``x + (silu(h Wg^T) * (h Wu^T)) Wd^T`` with ``h = rms_norm(x)``."""
    h = rms_norm(x, t["post_attention_layernorm.weight"], eps)
    return x + _swiglu(h, t["mlp.gate_proj.weight"], t["mlp.up_proj.weight"],
                       t["mlp.down_proj.weight"])


def moe_block(x: np.ndarray, t: dict[str, np.ndarray], cfg: OracleConfig
              ) -> tuple[np.ndarray, dict[str, np.ndarray]]:
    """Full MoE block on fp32 numpy arrays; returns ``(x + moe(x), aux)``.

    ``t`` maps the reference's layer tensor names (``post_attention_layernorm.weight``,
    ``mlp.gate.weight``, ``mlp.experts.{e}.{gate,up,down}_proj.weight``, ...) to arrays.
    ``aux`` holds ``topk_ids``, ``topk_w``, ``logits``, ``offsets``, ``perm``.
    """
    h = rms_norm(x, t["post_attention_layernorm.weight"], cfg.eps)
    bias = t.get("mlp.gate.e_score_correction_bias") if cfg.use_bias else None
    ids, w, logits = route(h, t["mlp.gate.weight"], bias, cfg)

    out = np.zeros_like(h)
    # The reference visits experts in Python set order and adds one contribution per
    # (expert, token) into out[token]; keeping that order keeps the fp32 sums identical.
    for e in set(ids.ravel().tolist()):
        hit = ids == e
        rows = np.nonzero(hit.any(axis=-1))[0]
        y = _swiglu(h[rows], t[f"mlp.experts.{e}.gate_proj.weight"],
                    t[f"mlp.experts.{e}.up_proj.weight"], t[f"mlp.experts.{e}.down_proj.weight"])
        we = np.where(hit[rows], w[rows], np.float32(0)).sum(axis=-1)
        out[rows] += we[:, None] * y

    p = cfg.shared_prefix
    if f"{p}gate_proj.weight" in t:
        shared = _swiglu(h, t[f"{p}gate_proj.weight"], t[f"{p}up_proj.weight"],
                         t[f"{p}down_proj.weight"])
        if "mlp.shared_expert_gate.weight" in t:  # qwen3_next.py:327-329
            shared = shared * sigmoid(h @ t["mlp.shared_expert_gate.weight"].T)
        out = out + shared

    offsets, perm = permutation(ids, cfg.n_experts)
    aux = {"topk_ids": ids, "topk_w": w, "logits": logits, "offsets": offsets, "perm": perm}
    return x + out, aux


# ---------------------------------------------------------------------------
# INT8 per-output-channel format (extension of quantize.py:24-50)
# ---------------------------------------------------------------------------

def int8_pc_quantize(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Symmetric per-output-row INT8: ``s = fp16(max|w_row| / 127)``,
    ``q = clip(rint(w / f32(s)), -127, 127)``; rows whose scale is 0 quantise to 0."""
    w = np.asarray(w, dtype=np.float32)
    amax = np.abs(w).max(axis=1)
    s16 = (amax / np.float32(127.0)).astype(np.float16)
    s32 = s16.astype(np.float32)
    safe = np.where(s32 > 0, s32, np.float32(1.0))
    q = np.clip(np.rint(w / safe[:, None]), -127, 127)
    q = np.where(s32[:, None] > 0, q, 0).astype(np.int8)
    return q, s16


def int8_pc_dequantize(q: np.ndarray, s16: np.ndarray) -> np.ndarray:
    """``q.astype(f32) * f32(scale[row])`` -- the fp32 weights the reference executor sees."""
    return q.astype(np.float32) * s16.astype(np.float32)[:, None]


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 value (ties to even), returned as fp32."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32).reshape(np.shape(a))
