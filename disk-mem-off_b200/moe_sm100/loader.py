"""Loader-side layer storage that keeps 16-bit weights and can write per-channel INT8.

The reference's ``SafetensorsStorage`` converts every tensor to ``compute_dtype``
(float32 by default) while packing a layer blob
(offload_runtime/loader/safetensors_storage.py:91-130), and the HF loader writes
the matching ``LayerSpec.metadata["tensors"]`` with that dtype
(offload_runtime/loader/huggingface.py:458-591).  For a bf16 checkpoint that
doubles the bytes of every layer that crosses PCIe and of every blob the device
path binds.

``PreservingSafetensorsStorage`` implements the same LayerStorage protocol
(``request`` / ``wait`` / ``get`` / ``release`` / ``close`` /
``get_disk_read_ms``) over the same files, but:

* a bf16 / f16 tensor keeps its checkpoint dtype, an f32 tensor stays f32;
* with ``expert_format="int8"`` every expert, shared-expert and dense-MLP
  projection (``mlp.experts.N.{gate,up,down}_proj.weight``,
  ``mlp.shared_expert(s).*``, ``mlp.{gate,up,down}_proj.weight``) is written as
  per-output-row INT8 plus an fp16 ``<name>_scale`` tensor (``s = fp16(max|w|/127)``,
  ``q = clip(rint(w / s), -127, 127)``), the format ``moe_bind_layer`` reads
  and ``Int8PerChannelDequantizer`` describes (``metadata["dtype"] ==
  "int8_per_channel"``);
* tensor offsets are 256-byte aligned.

It rewrites the layer specs it is given (from ``HuggingFaceLoader`` or any other
source of ``metadata["tensors"]`` with ``full_prefix``) into new ones that describe
its blobs; hand those to the runtime together with the storage.

The safetensors files are read directly (8-byte little-endian header length, a
JSON header of ``{name: {dtype, shape, data_offsets}}``, then the raw data), through
a memory map, so bf16 data needs no numpy bfloat16 support.
"""
from __future__ import annotations

import json
import mmap
import os
import struct
import threading
import time
from concurrent.futures import Future, ThreadPoolExecutor
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Iterable

import numpy as np

from .packing import is_expert_weight, quantize_int8_per_channel
from .types import HostBuffer, LayerSpec

_ST_DTYPES = {"BF16": ("bfloat16", 2), "F16": ("float16", 2), "F32": ("float32", 4),
              "I8": ("int8", 1), "F64": ("float64", 8)}
_NP = {"float16": np.float16, "float32": np.float32, "int8": np.int8, "float64": np.float64}
_ALIGN = 256


@dataclass(frozen=True)
class StoredTensor:
    path: Path
    dtype: str        # "bfloat16" | "float16" | "float32" | "int8" | "float64"
    shape: tuple[int, ...]
    start: int        # absolute byte offset of the data in the file
    nbytes: int


def read_safetensors_index(paths: Iterable[Path | str]) -> dict[str, StoredTensor]:
    """Name -> where its bytes are, for every tensor in the given files."""
    index: dict[str, StoredTensor] = {}
    for p in paths:
        path = Path(p)
        with open(path, "rb") as f:
            (hlen,) = struct.unpack("<Q", f.read(8))
            header = json.loads(f.read(hlen))
        base = 8 + hlen
        for name, info in header.items():
            if name == "__metadata__":
                continue
            st = info["dtype"]
            if st not in _ST_DTYPES:
                raise ValueError(f"{path.name}: tensor {name} has unsupported dtype {st}")
            b, e = info["data_offsets"]
            index[name] = StoredTensor(path, _ST_DTYPES[st][0], tuple(info["shape"]), base + b, e - b)
    return index


def _to_f32(raw: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bfloat16":
        return (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
    return raw.view(_NP[dtype]).astype(np.float32)


class PreservingSafetensorsStorage:
    """LayerStorage over safetensors files that keeps 16-bit (or writes INT8) weights."""

    def __init__(self, safetensors_paths: Iterable[Path | str], layer_specs: Iterable[LayerSpec],
                 *, expert_format: str = "bfloat16", max_workers: int = 2) -> None:
        if expert_format not in ("bfloat16", "int8"):
            raise ValueError("expert_format must be 'bfloat16' (keep checkpoint dtypes) or 'int8'")
        self.expert_format = expert_format
        self._index = read_safetensors_index(safetensors_paths)
        self._maps: dict[Path, mmap.mmap] = {}
        self._files: dict[Path, Any] = {}
        self._lock = threading.Lock()
        self._plans: dict[int, list[tuple[str, StoredTensor, str, int, int]]] = {}
        self.layers: list[LayerSpec] = [self._rewrite(spec) for spec in layer_specs]
        self._by_id = {spec.layer_id: spec for spec in self.layers}
        self._pool = ThreadPoolExecutor(max_workers=max_workers)
        self._pending: dict[int, Future[HostBuffer]] = {}
        self._done: dict[int, HostBuffer] = {}
        self._read_ms: dict[int, float] = {}

    @classmethod
    def from_model_dir(cls, model_dir: Path | str, layer_specs: Iterable[LayerSpec],
                       **kw: Any) -> "PreservingSafetensorsStorage":
        paths = sorted(Path(model_dir).glob("*.safetensors"))
        if not paths:
            raise FileNotFoundError(f"no .safetensors files in {model_dir}")
        return cls(paths, layer_specs, **kw)

    # -- layer description --------------------------------------------------------
    def _rewrite(self, spec: LayerSpec) -> LayerSpec:
        prefix = spec.metadata.get("full_prefix", "")
        plan: list[tuple[str, StoredTensor, str, int, int]] = []
        meta: list[dict[str, Any]] = []
        offset = 0
        has_int8 = False

        def place(name: str, shape: list[int], dtype: str, nbytes: int) -> int:
            nonlocal offset
            offset = (offset + _ALIGN - 1) // _ALIGN * _ALIGN
            at = offset
            meta.append({"name": name, "shape": shape, "dtype": dtype, "offset": at, "nbytes": nbytes})
            offset += nbytes
            return at

        for m in spec.metadata["tensors"]:
            name = m["name"]
            src = self._index.get(prefix + name) or self._index.get(name)
            if src is None:
                raise KeyError(prefix + name)
            shape = list(src.shape)
            if self.expert_format == "int8" and is_expert_weight(name) and len(shape) == 2:
                at = place(name, shape, "int8", shape[0] * shape[1])
                at_s = place(name + "_scale", [shape[0]], "float16", shape[0] * 2)
                plan.append((name, src, "int8", at, at_s))
                has_int8 = True
            else:
                plan.append((name, src, src.dtype, place(name, shape, src.dtype, src.nbytes), -1))
        md = dict(spec.metadata)
        md["tensors"] = meta
        if has_int8:
            md["dtype"] = "int8_per_channel"
        self._plans[spec.layer_id] = plan
        return LayerSpec(layer_id=spec.layer_id, name=spec.name, nbytes=offset, metadata=md)

    # -- reading --------------------------------------------------------------------
    def _map(self, path: Path) -> mmap.mmap:
        with self._lock:
            mm = self._maps.get(path)
            if mm is None:
                f = open(path, "rb")
                mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
                self._files[path] = f
                self._maps[path] = mm
            return mm

    def _load(self, layer_id: int) -> HostBuffer:
        spec = self._by_id[layer_id]
        blob = bytearray(spec.nbytes)
        out = np.frombuffer(blob, dtype=np.uint8)
        t0 = time.perf_counter()
        for _name, src, dtype, at, at_scale in self._plans[layer_id]:
            raw = np.frombuffer(self._map(src.path), dtype=np.uint8, count=src.nbytes, offset=src.start)
            if dtype == "int8" and src.dtype != "int8":
                q, s = quantize_int8_per_channel(_to_f32(raw, src.dtype).reshape(src.shape))
                out[at:at + q.nbytes] = q.view(np.uint8).ravel()
                out[at_scale:at_scale + s.nbytes] = s.view(np.uint8)
            else:
                out[at:at + src.nbytes] = raw
        self._read_ms[layer_id] = (time.perf_counter() - t0) * 1e3
        return HostBuffer(view=memoryview(blob), pinned=False)

    def get_disk_read_ms(self, layer_id: int) -> float:
        return self._read_ms.get(layer_id, 0.0)

    # -- LayerStorage protocol --------------------------------------------------------
    def request(self, layer_id: int) -> None:
        if layer_id not in self._pending and layer_id not in self._done:
            self._pending[layer_id] = self._pool.submit(self._load, layer_id)

    def wait(self, layer_id: int) -> None:
        fut = self._pending.pop(layer_id, None)
        if fut is not None:
            self._done[layer_id] = fut.result()

    def get(self, layer_id: int) -> HostBuffer:
        buf = self._done.pop(layer_id, None)
        return buf if buf is not None else self._load(layer_id)

    def release(self, layer_id: int) -> None:
        self._done.pop(layer_id, None)
        fut = self._pending.pop(layer_id, None)
        if fut is not None:
            fut.cancel()

    def close(self) -> None:
        self._pool.shutdown(wait=True, cancel_futures=True)
        self._pending.clear()
        self._done.clear()
        with self._lock:
            for mm in self._maps.values():
                mm.close()
            for f in self._files.values():
                f.close()
            self._maps.clear()
            self._files.clear()

    def __enter__(self) -> "PreservingSafetensorsStorage":
        return self

    def __exit__(self, *exc: Any) -> None:
        self.close()


def write_safetensors(path: Path | str, tensors: dict[str, tuple[str, np.ndarray]]) -> None:
    """Write ``{name: (dtype, array)}`` as a safetensors file (dtype "bfloat16" takes
    uint16 bit patterns).  Used to build checkpoints for tests and examples."""
    rev = {v[0]: k for k, v in _ST_DTYPES.items()}
    header: dict[str, Any] = {}
    chunks: list[bytes] = []
    pos = 0
    for name in sorted(tensors):
        dtype, arr = tensors[name]
        data = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": rev[dtype], "shape": list(arr.shape), "data_offsets": [pos, pos + len(data)]}
        chunks.append(data)
        pos += len(data)
    hdr = json.dumps(header, separators=(",", ":")).encode()
    hdr += b" " * ((8 - len(hdr) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hdr)))
        f.write(hdr)
        for c in chunks:
            f.write(c)
    os.chmod(path, 0o644)
