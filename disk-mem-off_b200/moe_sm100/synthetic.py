"""Seeded synthetic MoE layers built directly in device memory (benchmarks, full-size tests).

Full-size layers are too large to generate on the host (GLM-4.7 shape: 161 x 23.6 M
expert parameters), so the layer blob is assembled on the GPU with torch's
seeded generator, in the same ``metadata["tensors"]`` layout the loader uses
(names sorted, every tensor described by name/shape/dtype/offset/nbytes).
Distributions follow the benchmark configs: x ~ N(0,1), weights ~ N(0,0.02),
bias ~ N(0,0.01) plus an optional Zipf(s)-ranked skew.

``expert_dtype``: "bfloat16" (bf16-rounded N(0,0.02)) or "int8" (per-row
quantised from an fp32 N(0,0.02) source, fp16 scales = max|w|/127).

``experts = (lo, hi)`` materialises only routed experts [lo, hi) (the share of one
expert-parallel rank).  The router, bias, norm and shared expert are still built, the
router and bias from the same generator stream as a full layer; each routed expert and
the shared expert then come from their own generator (seeded from ``seed`` and the
expert id), so an expert's weights do not depend on which rank builds it.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import numpy as np


def _torch():
    import torch
    return torch


@dataclass
class SyntheticSpec:
    hidden: int
    n_experts: int
    top_k: int
    inter: int
    shared_inter: int
    family: str = "glm"              # "glm" | "qwen3"
    expert_dtype: str = "bfloat16"   # "bfloat16" | "int8"
    seed: int = 0
    bias_std: float = 0.01
    zipf_s: float = 0.0
    zipf_amp: float = 1.0
    experts: tuple[int, int] | None = None   # routed experts to materialise (None: all)


GLM47 = dict(hidden=5120, n_experts=160, top_k=8, inter=1536, shared_inter=1536, family="glm")
QWEN3_NEXT = dict(hidden=2048, n_experts=512, top_k=10, inter=512, shared_inter=512, family="qwen3")


def _tensor_list(spec: SyntheticSpec) -> list[tuple[str, list[int], str]]:
    H, I, SI, E = spec.hidden, spec.inter, spec.shared_inter, spec.n_experts
    ed = spec.expert_dtype
    out: list[tuple[str, list[int], str]] = [
        ("post_attention_layernorm.weight", [H], "float32"),
        ("mlp.gate.weight", [E, H], "float32"),
    ]
    if spec.family == "glm":
        out.append(("mlp.gate.e_score_correction_bias", [E], "float32"))

    def proj(prefix: str, rows_gu: int) -> None:
        for nm, shp in (("gate_proj", [rows_gu, H]), ("up_proj", [rows_gu, H]),
                        ("down_proj", [H, rows_gu])):
            out.append((f"{prefix}{nm}.weight", shp, ed))
            if ed == "int8":
                out.append((f"{prefix}{nm}.weight_scale", [shp[0]], "float16"))

    lo, hi = spec.experts if spec.experts is not None else (0, E)
    for e in range(lo, hi):
        proj(f"mlp.experts.{e}.", I)
    if SI > 0:
        proj("mlp.shared_experts." if spec.family == "glm" else "mlp.shared_expert.", SI)
        if spec.family == "qwen3":
            out.append(("mlp.shared_expert_gate.weight", [1, H], "float32"))
    out.sort(key=lambda r: r[0])
    return out


_ESIZE = {"float32": 4, "float16": 2, "bfloat16": 2, "int8": 1}


def build_device_layer(spec: SyntheticSpec, device: Any = "cuda") -> tuple[Any, list[dict[str, Any]]]:
    """Return ``(blob uint8 CUDA tensor, tensor metadata)`` for one synthetic MoE layer."""
    torch = _torch()
    items = _tensor_list(spec)
    meta: list[dict[str, Any]] = []
    off = 0
    for name, shape, dt in items:
        off = (off + 255) // 256 * 256
        nb = int(np.prod(shape)) * _ESIZE[dt]
        meta.append({"name": name, "shape": shape, "dtype": dt, "offset": off, "nbytes": nb})
        off += nb
    blob = torch.empty(off, dtype=torch.uint8, device=device)
    gen = torch.Generator(device=device)
    gen.manual_seed(spec.seed)
    by = {m["name"]: m for m in meta}

    def view(name: str, dtype: Any) -> Any:
        m = by[name]
        return blob[m["offset"]:m["offset"] + m["nbytes"]].view(dtype).view(m["shape"])

    H, E = spec.hidden, spec.n_experts
    view("post_attention_layernorm.weight", torch.float32).fill_(1.0)
    view("mlp.gate.weight", torch.float32).copy_(
        torch.randn((E, H), generator=gen, device=device) * 0.02)
    if spec.family == "glm":
        bias = torch.randn(E, generator=gen, device=device) * spec.bias_std
        if spec.zipf_s > 0:
            ranks = torch.arange(1, E + 1, device=device, dtype=torch.float64)
            skew = (spec.zipf_amp / ranks ** spec.zipf_s).float()
            perm = torch.randperm(E, generator=gen, device=device)
            bias = bias + skew[perm]
        view("mlp.gate.e_score_correction_bias", torch.float32).copy_(bias)
    if spec.family == "qwen3" and spec.shared_inter > 0:
        view("mlp.shared_expert_gate.weight", torch.float32).copy_(
            torch.randn((1, H), generator=gen, device=device) * 0.02)
    subset = spec.experts is not None
    if subset:
        lo, hi = spec.experts
        if not 0 <= lo < hi <= E:
            raise ValueError(f"expert range {spec.experts} outside [0, {E}]")
    gens: dict[int, Any] = {}

    def gen_for(name: str) -> Any:
        # full layers draw everything from one stream; subsets one stream per expert
        if not subset:
            return gen
        key = int(name.split(".")[2]) if name.startswith("mlp.experts.") else E
        if key not in gens:
            g = torch.Generator(device=device)
            g.manual_seed(spec.seed * 1_000_003 + 7919 * (key + 1))
            gens[key] = g
        return gens[key]

    for name, shape, dt in items:
        if dt not in ("bfloat16", "int8"):
            continue
        w = torch.randn(shape, generator=gen_for(name), device=device) * 0.02
        if dt == "bfloat16":
            view(name, torch.bfloat16).copy_(w.to(torch.bfloat16))
        else:
            s16 = (w.abs().amax(dim=1) / 127.0).to(torch.float16)
            s32 = s16.float()
            q = torch.round(w / torch.where(s32 > 0, s32, torch.ones_like(s32))[:, None])
            q = q.clamp_(-127, 127)
            q[s32 == 0] = 0
            view(name, torch.int8).copy_(q.to(torch.int8))
            view(name + "_scale", torch.float16).copy_(s16)
    return blob, meta


def host_tensor(blob: Any, meta: list[dict[str, Any]], name: str) -> np.ndarray:
    """fp32 host copy of one tensor of a device blob (int8 weights dequantised)."""
    torch = _torch()
    by = {m["name"]: m for m in meta}
    m = by[name]
    raw = blob[m["offset"]:m["offset"] + m["nbytes"]]
    if m["dtype"] == "float32":
        t = raw.view(torch.float32)
    elif m["dtype"] == "bfloat16":
        t = raw.view(torch.bfloat16).float()
    elif m["dtype"] == "float16":
        t = raw.view(torch.float16).float()
    else:
        s = by[name + "_scale"]
        sc = blob[s["offset"]:s["offset"] + s["nbytes"]].view(torch.float16).float()
        t = raw.view(torch.int8).float().view(m["shape"]) * sc[:, None]
    return t.reshape(m["shape"]).cpu().numpy()


class LazyHostTensors:
    """Mapping view of a device blob that copies a tensor to the host on first access.

    Lets a CPU executor run a full-size layer while fetching only the experts it
    touches.
    """

    def __init__(self, blob: Any, meta: list[dict[str, Any]]) -> None:
        self._blob = blob
        self._meta = meta
        self._names = {m["name"] for m in meta if not m["name"].endswith("_scale")}
        self._cache: dict[str, np.ndarray] = {}

    def __contains__(self, name: object) -> bool:
        return name in self._names

    def __getitem__(self, name: str) -> np.ndarray:
        if name not in self._names:
            raise KeyError(name)
        if name not in self._cache:
            self._cache[name] = host_tensor(self._blob, self._meta, name)
        return self._cache[name]

    def get(self, name: str, default: Any = None) -> Any:
        return self[name] if name in self._names else default

    def keys(self) -> Any:
        return iter(sorted(self._names))

    def __iter__(self) -> Any:
        return self.keys()

    def __len__(self) -> int:
        return len(self._names)

    def cached_bytes(self) -> int:
        return sum(a.nbytes for a in self._cache.values())


def build_device_attention(hidden: int, heads: int, kv_heads: int, head_dim: int, seed: int = 0,
                           device: Any = "cuda", bias: bool = True,
                           qk_norm: bool = True) -> tuple[Any, list[dict[str, Any]]]:
    """``(blob uint8 CUDA tensor, tensor metadata)`` of one synthetic GLM-4 attention
    block, named as the loader names them: bf16 projections N(0, 0.02), fp32 biases
    and norm weights (ones)."""
    torch = _torch()
    H, nh, nkv, hd = hidden, heads, kv_heads, head_dim
    items: list[tuple[str, list[int], str]] = [("input_layernorm.weight", [H], "float32")]
    for name, rows in (("q", nh * hd), ("k", nkv * hd), ("v", nkv * hd)):
        items.append((f"self_attn.{name}_proj.weight", [rows, H], "bfloat16"))
        if bias:
            items.append((f"self_attn.{name}_proj.bias", [rows], "float32"))
    if qk_norm:
        items += [("self_attn.q_norm.weight", [hd], "float32"), ("self_attn.k_norm.weight", [hd], "float32")]
    items.append(("self_attn.o_proj.weight", [H, nh * hd], "bfloat16"))
    meta: list[dict[str, Any]] = []
    off = 0
    for name, shape, dt in items:
        off = (off + 255) // 256 * 256
        nb = int(np.prod(shape)) * _ESIZE[dt]
        meta.append({"name": name, "shape": shape, "dtype": dt, "offset": off, "nbytes": nb})
        off += nb
    blob = torch.empty(off, dtype=torch.uint8, device=device)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    for m in meta:
        v = blob[m["offset"]:m["offset"] + m["nbytes"]]
        if m["dtype"] == "bfloat16":
            v.view(torch.bfloat16).view(m["shape"]).copy_(
                (torch.randn(m["shape"], generator=gen, device=device) * 0.02).to(torch.bfloat16))
        elif m["name"].endswith("_proj.bias"):
            v.view(torch.float32).copy_(torch.randn(m["shape"], generator=gen, device=device) * 0.02)
        else:
            v.view(torch.float32).fill_(1.0)
    return blob, meta
