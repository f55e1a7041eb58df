"""Device MoE path shared by the GLM-4 MoE and Qwen3-Next executors.

Drop-in for the reference executors' MoE block:

* ``_moe_mlp_block(x, t)`` keeps the reference signature (glm4_moe.py:176,
  qwen3_next.py:273): ``x`` is a host fp32 ``[T, H]`` array (or a CUDA fp32
  tensor), ``t`` the layer's named tensors.  ``t`` may be the reference's dict of
  host arrays (packed to the device once and cached) or a bound ``MoeLayer``.
* ``run_layer(layer, activations, device_weights, backend, stream)`` keeps the
  ``LayerExecutor`` protocol (runtime.py:15-26).  The MoE tensors are packed
  straight from the device blob; only the non-MoE tensors (attention, input
  norm) are read back to the host for the attention delegate, instead of the
  whole blob (_common.py:20-33).
* ``_dense_mlp_block(x, t)`` (glm4_moe.py:166) runs the dense MLP of
  ``first_k_dense_replace`` layers on the device too (a plan with no routed
  experts); ``run_layer`` uses it for non-MoE layers unless a ``dense_mlp=``
  callable is given.
* Attention is not part of this library: pass an ``attention=`` callable (for
  example the reference executor's own method, see ``reference_delegates``).
"""
from __future__ import annotations

import weakref
from collections import OrderedDict
from typing import Any, Callable

import numpy as np

from ..config import MoeLayerConfig
from ..layer import MoeLayer, _torch, layer_shapes
from ..packing import pack_layer

AttentionFn = Callable[[Any, Any, dict[str, Any]], Any]   # (layer, x, t_host) -> x
DenseFn = Callable[[Any, dict[str, Any]], Any]            # (x, t_host) -> x

_MOE_PREFIXES = ("mlp.", "post_attention_layernorm.")


def _short(name: str, layer: Any) -> str:
    prefix = layer.metadata.get("full_prefix", "") if hasattr(layer, "metadata") else ""
    return name[len(prefix):] if prefix and name.startswith(prefix) else name


def is_moe_tensor(short_name: str) -> bool:
    return short_name.startswith(_MOE_PREFIXES)


class DeviceMoeExecutor:
    """Common machinery; subclasses set the config parser and the block layout."""

    family = "glm"

    def __init__(self, config: dict[str, Any], *, score_func: str | None = None,
                 weight_format: str = "f16", max_tokens: int = 4096, device: int = 0,
                 resident: bool = True, attention: AttentionFn | None = None,
                 dense_mlp: DenseFn | None = None) -> None:
        self.config = dict(config)
        self.weight_format = weight_format
        self.max_tokens = max_tokens
        self.device = device
        self.resident = resident
        self.attention = attention
        self.dense_mlp = dense_mlp
        overrides: dict[str, Any] = dict(weight_format=weight_format, max_tokens=max_tokens,
                                         device=device)
        if score_func is not None:
            overrides["score_func"] = score_func
        self.moe_config = self._parse(self.config, overrides)
        self._bound: dict[Any, MoeLayer] = {}
        # per resident layer: (device AttentionLayer or None, host attention tensors)
        self._held: dict[int, tuple[Any, dict[str, Any]]] = {}
        # layers bound from host tensor dicts (the reference's ``_moe_mlp_block(x, t)``
        # call): a few most recent ones, each remembered by weak references to the
        # very arrays it was packed from
        self.tensor_cache_size = 2
        self._by_tensors: OrderedDict[tuple[int, bool], tuple[dict[str, Any], MoeLayer]] = OrderedDict()

    # -- overridden by the families --------------------------------------------------
    def _parse(self, config: dict[str, Any], overrides: dict[str, Any]) -> MoeLayerConfig:
        raise NotImplementedError

    def _is_moe_layer(self, layer: Any) -> bool:
        return True

    # -- binding ---------------------------------------------------------------------
    def _dense_config(self, tensor_meta: list[dict[str, Any]]) -> MoeLayerConfig:
        inter = next((int(m["shape"][0]) for m in tensor_meta
                      if str(m["name"]).endswith("mlp.gate_proj.weight")), 0)
        if inter <= 0:
            raise KeyError("mlp.gate_proj.weight")
        c = self.moe_config
        return MoeLayerConfig.dense_mlp({"hidden_size": c.hidden, "intermediate_size": inter},
                                        rms_norm_eps=c.rms_norm_eps,
                                        weight_format=c.weight_format, max_tokens=c.max_tokens,
                                        device=c.device)

    def _layer_config(self, tensor_meta: list[dict[str, Any]]) -> MoeLayerConfig:
        shp = layer_shapes(tensor_meta)
        return self.moe_config.with_shapes(shp["inter"] or self.moe_config.inter,
                                           shp["shared_inter"], shp["has_shared_gate"])

    def bind_device_blob(self, key: Any, blob_ptr: int, blob_bytes: int,
                         tensor_meta: list[dict[str, Any]], stream: Any = None,
                         dense: bool = False) -> MoeLayer:
        """Pack the MoE (or, with ``dense``, the dense-MLP) tensors of a
        device-resident layer blob (cached under ``key``)."""
        if self.resident and key in self._bound:
            return self._bound[key]
        ml = MoeLayer(self._dense_config(tensor_meta) if dense else self._layer_config(tensor_meta))
        ml.bind_device(blob_ptr, blob_bytes, tensor_meta, stream)
        if self.resident:
            self._bound[key] = ml
        return ml

    def bind_tensors(self, t: dict[str, Any], expert_format: str = "float32",
                     dense: bool = False) -> MoeLayer:
        """Pack a dict of host arrays (reference tensor names) and bind it."""
        moe_t = {k: np.asarray(v) for k, v in t.items() if is_moe_tensor(k)}
        blob, meta = pack_layer(moe_t, expert_format=expert_format)
        ml = MoeLayer(self._dense_config(meta) if dense else self._layer_config(meta))
        ml.bind_host(blob, meta)
        return ml

    # -- the block -------------------------------------------------------------------
    def _layer_for_tensors(self, t: dict[str, Any], dense: bool) -> MoeLayer:
        """The bound layer packed from the host tensor dict ``t``.

        The reference builds a fresh dict of numpy views for every call
        (_common.py:43-58), and CPython reuses the id of a collected dict, so the
        dict's id alone could name another layer's weights.  An entry therefore
        holds weak references to every array it was packed from and matches only
        when ``t`` maps the same names to those very (still alive) arrays; no
        host memory is kept alive by the cache, and at most
        ``tensor_cache_size`` packed layers stay bound."""
        names = sorted(k for k in t if is_moe_tensor(k))
        key = (id(t), dense)
        hit = self._by_tensors.get(key)
        if hit is not None:
            refs, ml = hit
            if refs.keys() == set(names) and all(refs[n]() is t[n] for n in names):
                self._by_tensors.move_to_end(key)
                return ml
            self._by_tensors.pop(key)
            ml.close()
        ml = self.bind_tensors(t, dense=dense)
        refs: dict[str, Any] = {}
        for n in names:
            try:
                refs[n] = weakref.ref(t[n])
            except TypeError:  # not weak-referenceable: never match this entry again
                refs[n] = lambda: None
        self._by_tensors[key] = (refs, ml)
        while len(self._by_tensors) > max(self.tensor_cache_size, 0):
            _k, (_r, old) = self._by_tensors.popitem(last=False)
            old.close()
        return ml

    def _moe_mlp_block(self, x: Any, t: Any) -> Any:
        """``x + MoE(rms_norm(x))`` on the device; same contract as the reference."""
        ml = t if isinstance(t, MoeLayer) else self._layer_for_tensors(t, dense=False)
        if isinstance(x, np.ndarray):
            return ml.forward_host(x)
        return ml.forward(x)

    def _dense_mlp_block(self, x: Any, t: Any) -> Any:
        """``x + down(silu(gate(h)) * up(h))``, ``h = rms_norm(x)``, on the device;
        same contract as the reference (glm4_moe.py:166-172)."""
        ml = t if isinstance(t, MoeLayer) else self._layer_for_tensors(t, dense=True)
        if isinstance(x, np.ndarray):
            return ml.forward_host(x)
        return ml.forward(x)

    # -- LayerExecutor protocol ----------------------------------------------------------
    def _device_attention_config(self) -> Any:
        """AttentionConfig for layers whose attention runs on the device, or None
        when attention goes to the host delegate (``attention=``)."""
        return None

    def run_layer(self, layer: Any, activations: Any, device_weights: Any, backend: Any,
                  stream: Any) -> Any:
        """One decoder layer (runtime.py:15-26).  ``device_weights`` is the layer blob
        the runtime copied to the device; ``None`` asks for a layer this executor
        holds from an earlier pass (``resident_nbytes`` is not None), which then
        runs without touching storage or the blob."""
        if getattr(backend, "name", None) != "cuda":
            raise ValueError("the sm_100a MoE executor runs on the 'cuda' backend only")
        lid = layer.layer_id
        if device_weights is None:
            held = self._held.get(lid)
            if held is None or not self._holds_block(layer):
                raise KeyError(f"layer {lid} is not resident in this executor")
        else:
            held = self._prepare_attention(layer, device_weights, backend, stream)
            if self.resident:
                self._held[lid] = held
        attn, t_host = held
        if not self._is_moe_layer(layer) and self.dense_mlp is not None:
            if device_weights is None:
                raise KeyError(f"layer {lid}: a host dense-MLP delegate needs the layer blob")
            x = self.attention(layer, activations, t_host) if t_host else activations
            return self.dense_mlp(x, _read_ranges(backend, device_weights, layer.metadata["tensors"], stream))
        ml = self._block_for(layer, device_weights, stream)
        if attn is not None:  # attention and MLP both on the device: one copy each way
            return self._device_layer(attn, ml, activations)
        x = activations
        if t_host:
            x = self.attention(layer, x, t_host)
        return self._moe_mlp_block(x, ml) if self._is_moe_layer(layer) else self._dense_mlp_block(x, ml)

    def _prepare_attention(self, layer: Any, device_weights: Any, backend: Any,
                           stream: Any) -> tuple[Any, dict[str, Any]]:
        """(device AttentionLayer or None, host tensors for the attention delegate)."""
        meta = layer.metadata["tensors"]
        host_meta = [m for m in meta if not is_moe_tensor(_short(m["name"], layer))]
        if not host_meta:
            return None, {}
        if self.attention is not None:
            return None, _read_ranges(backend, device_weights, host_meta, stream)
        acfg = self._device_attention_config()
        if acfg is None:
            raise NotImplementedError(
                "layer has attention tensors; pass attention=<callable(layer, x, t)> "
                "(e.g. moe_sm100.executors.reference_delegates(ref_executor))")
        from ..attention import AttentionLayer
        attn = AttentionLayer(acfg)
        attn.bind_device(int(device_weights.handle), int(device_weights.nbytes),
                         [dict(m, name=_short(m["name"], layer)) for m in host_meta],
                         getattr(stream, "value", stream))
        return attn, {}

    @staticmethod
    def _device_layer(attn: Any, ml: MoeLayer, x: Any) -> Any:
        torch = _torch()
        host = isinstance(x, np.ndarray)
        xd = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(
            f"cuda:{ml.cfg.device}") if host else x
        y = ml.forward(attn.forward(xd))
        return y.cpu().numpy() if host else y

    def _block_key(self, layer: Any) -> Any:
        return layer.layer_id if self._is_moe_layer(layer) else ("dense", layer.layer_id)

    def _holds_block(self, layer: Any) -> bool:
        if not self._is_moe_layer(layer) and self.dense_mlp is not None:
            return False  # the host delegate needs the blob on every pass
        return self._block_key(layer) in self._bound

    def _block_for(self, layer: Any, device_weights: Any, stream: Any) -> MoeLayer:
        key = self._block_key(layer)
        if device_weights is None:
            return self._bound[key]
        stream_handle = getattr(stream, "value", stream)
        meta = [dict(m, name=_short(m["name"], layer)) for m in layer.metadata["tensors"]]
        return self.bind_device_blob(key, int(device_weights.handle), int(device_weights.nbytes),
                                     meta, stream_handle, dense=not self._is_moe_layer(layer))

    # -- residency (used by moe_sm100.runtime.ResidentOffloadRuntime) -------------------
    def resident_nbytes(self, layer_id: int) -> int | None:
        """Device bytes this executor keeps for ``layer_id`` between passes (packed
        MLP / experts and, with device attention, the attention weights), or None
        when it cannot run the layer again without its blob."""
        held = self._held.get(layer_id) if self.resident else None
        if held is None:
            return None
        for key in (layer_id, ("dense", layer_id)):
            ml = self._bound.get(key)
            if ml is not None:
                return ml.weight_bytes + (held[0].weight_bytes if held[0] is not None else 0)
        return None

    def evict(self, key: Any) -> None:
        """Release what is kept for a layer id (or a bind key): its packed plans and
        the host copies of its attention tensors."""
        for k in (key, ("dense", key)):
            ml = self._bound.pop(k, None)
            if ml is not None:
                ml.close()
        held = self._held.pop(key, None)
        if held is not None and held[0] is not None:
            held[0].close()


def _read_ranges(backend: Any, buf: Any, metas: list[dict[str, Any]], stream: Any) -> dict[str, Any]:
    """Read only the listed tensors of a device blob back to host numpy arrays."""
    out: dict[str, Any] = {}
    for m in metas:
        dt = np.dtype("float32" if m["dtype"] in ("float32", "<f4") else
                      "float16" if m["dtype"] in ("float16", "<f2") else
                      "int8" if m["dtype"] in ("int8", "|i1") else "uint16")
        host = np.empty(int(m["nbytes"]), dtype=np.uint8)
        backend.copy_d2h_range(host, buf, int(m["offset"]), int(m["nbytes"]), stream)
        backend.synchronize_stream(stream)
        arr = host.view(dt).reshape(m["shape"])
        if dt == np.uint16:  # bfloat16 bits -> fp32, as the reference storage does
            arr = (arr.astype(np.uint32) << 16).view(np.float32)
        out[m["name"]] = arr
    return out


def reference_delegates(ref_executor: Any) -> dict[str, Any]:
    """The ``attention=`` callable built from a reference executor instance (dense
    MLP layers run on the device; pass the reference's ``_dense_mlp_block`` as
    ``dense_mlp=`` to keep them on the host instead).

    GLM-4 MoE: ``_attention_block`` (glm4_moe.py:112).
    Qwen3-Next: ``_full_attn_block`` / ``_linear_attn_block`` by ``metadata["attn_type"]``
    (qwen3_next.py:149-154).
    """
    def _strip(layer: Any, t: dict[str, Any]) -> dict[str, Any]:
        return {_short(k, layer): v for k, v in t.items()}

    if hasattr(ref_executor, "_attention_block"):
        def attention(layer: Any, x: Any, t: dict[str, Any]) -> Any:
            return ref_executor._attention_block(x, _strip(layer, t))
    else:
        def attention(layer: Any, x: Any, t: dict[str, Any]) -> Any:
            if layer.metadata.get("attn_type", "linear") == "full":
                return ref_executor._full_attn_block(x, _strip(layer, t))
            return ref_executor._linear_attn_block(x, _strip(layer, t))
    return {"attention": attention}
