"""GLM-4 MoE attention block on the device, behind the libmoe_sm100 C ABI.

``AttentionLayer.forward(x)`` is the device equivalent of
``GLM4MoeExecutor._attention_block(x, t)`` (offload_runtime/executors/glm4_moe.py:112-162):
``x + o_proj(causal softmax attention(rms_norm(x)))`` with the reference's q/k/v
biases, per-head q/k RMS norms, partial rotate-half RoPE and grouped-query heads,
over the whole sequence at positions 0..T-1.  PyTorch provides only buffers and
the current stream; the kernels are the library's (tcgen05 projections and a
tcgen05 flash-attention kernel).
"""
from __future__ import annotations

from ctypes import byref, c_void_p
from dataclasses import dataclass
from typing import Any, Iterable

from . import _lib
from ._lib import check, lib
from .layer import _descs, _stream_handle, _torch


@dataclass
class AttentionConfig:
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    rotary_dim: int
    rope_theta: float = 1_000_000.0
    rms_norm_eps: float = 1e-5
    max_tokens: int = 4096
    device: int = 0

    @classmethod
    def glm4_moe(cls, config: dict[str, Any], **overrides: Any) -> "AttentionConfig":
        """From the HF config with the reference's defaults (glm4_moe.py:70-84)."""
        heads = config["num_attention_heads"]
        head_dim = config.get("head_dim", config["hidden_size"] // heads)
        kw = dict(hidden=config["hidden_size"], heads=heads,
                  kv_heads=config.get("num_key_value_heads", heads), head_dim=head_dim,
                  rotary_dim=int(head_dim * config.get("partial_rotary_factor", 0.5)),
                  rope_theta=config.get("rope_theta", 1000000.0),
                  rms_norm_eps=config.get("rms_norm_eps", 1e-5))
        kw.update(overrides)
        return cls(**kw)

    def to_c(self) -> _lib.MoeAttnConfigC:
        return _lib.MoeAttnConfigC(hidden=self.hidden, heads=self.heads, kv_heads=self.kv_heads,
                                   head_dim=self.head_dim, rotary_dim=self.rotary_dim,
                                   rope_theta=self.rope_theta, rms_norm_eps=self.rms_norm_eps,
                                   max_tokens=self.max_tokens, device=self.device)


class AttentionLayer:
    """One layer's packed attention weights (f16, HBM-resident) and its forward."""

    def __init__(self, cfg: AttentionConfig) -> None:
        self.cfg = cfg
        h = c_void_p()
        check(lib().moe_attn_create(byref(cfg.to_c()), byref(h)))
        self._h = h
        self._ws: Any = None

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            lib().moe_attn_destroy(self._h)
            self._h = c_void_p()
        self._ws = None

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    def bind_device(self, blob_ptr: int, blob_bytes: int, tensor_meta: Iterable[dict[str, Any]],
                    stream: Any = None) -> None:
        descs, keep = _descs(tensor_meta)
        check(lib().moe_attn_bind(self._h, c_void_p(int(blob_ptr)), int(blob_bytes), descs,
                                  len(descs), c_void_p(_stream_handle(stream))))
        del keep

    def bind_host(self, blob: Any, tensor_meta: Iterable[dict[str, Any]]) -> None:
        torch = _torch()
        mv = memoryview(blob).cast("B")
        dev = torch.empty(mv.nbytes, dtype=torch.uint8, device=f"cuda:{self.cfg.device}")
        dev.copy_(torch.frombuffer(mv, dtype=torch.uint8))
        self.bind_device(dev.data_ptr(), mv.nbytes, tensor_meta)
        torch.cuda.current_stream().synchronize()

    @property
    def weight_bytes(self) -> int:
        return int(lib().moe_attn_weight_bytes(self._h))

    def workspace_bytes(self, tokens: int) -> int:
        return int(lib().moe_attn_workspace_bytes(self._h, int(tokens)))

    def forward(self, x: Any, out: Any = None, stream: Any = None) -> Any:
        """``x + attention(x)`` for a CUDA fp32 tensor ``x`` of shape [T, H]."""
        torch = _torch()
        if not (isinstance(x, torch.Tensor) and x.is_cuda and x.dtype == torch.float32):
            raise TypeError("AttentionLayer.forward expects a CUDA float32 tensor")
        if x.dim() != 2 or x.shape[1] != self.cfg.hidden:
            raise ValueError(f"x must be [T, {self.cfg.hidden}]")
        x = x.contiguous()
        out = torch.empty_like(x) if out is None else out
        t = x.shape[0]
        if t == 0:
            return out
        need = self.workspace_bytes(t)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(max(need, 256), dtype=torch.uint8, device=x.device)
        check(lib().moe_attn_forward(self._h, c_void_p(x.data_ptr()), c_void_p(out.data_ptr()), t,
                                     c_void_p(self._ws.data_ptr()), self._ws.numel(),
                                     c_void_p(_stream_handle(stream))))
        return out

    def status(self, stream: Any = None) -> None:
        check(lib().moe_attn_status(self._h, c_void_p(_stream_handle(stream))))
