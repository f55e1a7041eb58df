"""Host-side logic of the resident-layer runtime and the dtype-preserving storage
(no GPU): a fake backend counts allocations and copies, a fake executor stands in
for the device MoE path."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from moe_sm100.loader import PreservingSafetensorsStorage, read_safetensors_index, write_safetensors
from moe_sm100.packing import bf16_bits, bf16_to_f32, quantize_int8_per_channel
from moe_sm100.quantize import Int8PerChannelDequantizer
from moe_sm100.runtime import ResidentOffloadRuntime
from moe_sm100.types import DeviceBuffer, HostBuffer, LayerSpec


class _CountingBackend:
    name = "fake"
    supports_pinned_host = False

    def __init__(self) -> None:
        self.mem: dict[int, bytes] = {}
        self.next = 1
        self.allocs = self.frees = 0
        self.h2d_bytes = 0

    def create_stream(self, purpose: str) -> str:
        return purpose

    def destroy_stream(self, stream: str) -> None:
        pass

    def alloc_device(self, nbytes: int) -> DeviceBuffer:
        self.allocs += 1
        h = self.next
        self.next += 1
        self.mem[h] = b""
        return DeviceBuffer(handle=h, nbytes=nbytes, backend=self.name)

    def free_device(self, buf: DeviceBuffer) -> None:
        self.frees += 1
        del self.mem[buf.handle]

    def copy_h2d_async(self, dst: DeviceBuffer, src: HostBuffer, stream: str) -> None:
        self.h2d_bytes += dst.nbytes
        self.mem[dst.handle] = bytes(src.view.cast("B")[: dst.nbytes])

    def record_event(self, stream: str) -> object:
        return object()

    def destroy_event(self, event: object) -> None:
        pass

    def wait_event(self, stream: str, event: object) -> None:
        pass

    def synchronize_stream(self, stream: str) -> None:
        pass


class _Storage:
    def __init__(self, blobs: dict[int, bytes]) -> None:
        self.blobs = blobs
        self.requested: list[int] = []
        self.got: list[int] = []

    def request(self, lid: int) -> None:
        self.requested.append(lid)

    def wait(self, lid: int) -> None:
        pass

    def get(self, lid: int) -> HostBuffer:
        self.got.append(lid)
        return HostBuffer(view=memoryview(bytearray(self.blobs[lid])))

    def release(self, lid: int) -> None:
        pass


class _Lookahead:
    def warmup_prefetch_ids(self, ids: list[int]) -> list[int]:
        return ids[:1]

    def next_prefetch_id(self, ids: list[int], i: int) -> int | None:
        return ids[i + 1] if i + 1 < len(ids) else None


class _Executor:
    """Adds the layer's first blob byte to x; keeps ``keep`` bytes per layer resident."""

    def __init__(self, backend: _CountingBackend, keep: int) -> None:
        self.backend, self.keep = backend, keep
        self.held: dict[int, int] = {}
        self.evicted: list[int] = []

    def run_layer(self, layer, activations, device_weights, backend, stream):  # noqa: ANN001, ANN201
        if device_weights is None:
            add = self.held[layer.layer_id]
        else:
            add = backend.mem[device_weights.handle][0]
            self.held[layer.layer_id] = add
        return activations + add

    def resident_nbytes(self, lid: int) -> int | None:
        return self.keep if lid in self.held else None

    def evict(self, lid: int) -> None:
        self.evicted.append(lid)
        self.held.pop(lid, None)


def _specs(n: int) -> list[LayerSpec]:
    return [LayerSpec(i, f"model.layers.{i}", 64, {"tensors": []}) for i in range(n)]


def test_second_pass_skips_storage_and_h2d_for_resident_layers() -> None:
    be = _CountingBackend()
    st = _Storage({i: bytes([i + 1]) * 64 for i in range(3)})
    ex = _Executor(be, keep=100)
    with ResidentOffloadRuntime(_specs(3), be, st, _Lookahead(), ex,
                                resident_budget_bytes=1000) as rt:
        out1, m1 = rt.run_inference([0, 1, 2], np.zeros(2))
        assert m1.transferred_bytes == 3 * 64 and m1.resident_layers == 0
        assert be.allocs == be.frees == 3  # blobs are never kept, only what the executor packed
        got_before = list(st.got)
        out2, m2 = rt.run_inference([0, 1, 2], np.zeros(2))
        assert m2.transferred_bytes == 0 and m2.resident_layers == 3
        assert st.got == got_before and be.h2d_bytes == 3 * 64
        assert all(lm.resident for lm in m2.layer_metrics)
        np.testing.assert_array_equal(out1, out2)
        np.testing.assert_array_equal(out1, np.full(2, 6.0))
    assert sorted(ex.evicted) == [0, 1, 2]  # close() releases what stayed resident


def test_budget_keeps_the_most_recent_layers() -> None:
    be = _CountingBackend()
    st = _Storage({i: bytes([1]) * 64 for i in range(4)})
    ex = _Executor(be, keep=100)
    rt = ResidentOffloadRuntime(_specs(4), be, st, _Lookahead(), ex, resident_budget_bytes=250)
    rt.run_inference([0, 1, 2, 3], np.zeros(1))
    assert ex.evicted == [0, 1] and rt.is_resident(2) and rt.is_resident(3)
    _, m = rt.run_inference([2, 3, 0], np.zeros(1))
    assert [lm.resident for lm in m.layer_metrics] == [True, True, False]
    assert m.transferred_bytes == 64
    # a layer larger than the whole budget is streamed every pass
    big = _Executor(be, keep=10_000)
    rt2 = ResidentOffloadRuntime(_specs(1), be, _Storage({0: b"\x01" * 64}), _Lookahead(), big,
                                 resident_budget_bytes=250)
    rt2.run_inference([0], np.zeros(1))
    assert big.evicted == [0] and not rt2.is_resident(0)
    rt.close()
    rt2.close()


def test_streaming_mode_and_one_staging_buffer() -> None:
    be = _CountingBackend()
    st = _Storage({i: bytes([1]) * (64 + 32 * i) for i in range(3)})
    specs = [LayerSpec(i, f"L{i}", 64 + 32 * i, {"tensors": []}) for i in range(3)]
    ex = _Executor(be, keep=1)
    with ResidentOffloadRuntime(specs, be, st, _Lookahead(), ex, use_buffer_pool=True) as rt:
        for _ in range(2):
            _, m = rt.run_inference([0, 1, 2], np.zeros(1))
            assert m.resident_layers == 0
        # growing layers: one buffer per new maximum, nothing else allocated
        assert be.allocs == 3 and be.frees == 2
        with pytest.raises(ValueError):
            rt.run_inference([7], np.zeros(1))
    assert be.frees == 3 and not be.mem


def test_residency_needs_an_executor_that_can_keep_layers() -> None:
    class _Plain:
        def run_layer(self, **kw):  # noqa: ANN003, ANN201
            return kw["activations"]

    with pytest.raises(TypeError):
        ResidentOffloadRuntime(_specs(1), _CountingBackend(), _Storage({}), _Lookahead(), _Plain(),
                               resident_budget_bytes=1)


# ------------------------------------------------------------------ preserving storage
def _checkpoint(tmp_path: Path) -> tuple[Path, dict[str, np.ndarray]]:
    rng = np.random.default_rng(9)
    f32 = {"model.layers.0.post_attention_layernorm.weight": rng.standard_normal(32).astype(np.float32),
           "model.layers.0.mlp.gate.weight": rng.standard_normal((4, 32)).astype(np.float32)}
    bf = {f"model.layers.0.mlp.experts.{e}.{p}_proj.weight":
          bf16_to_f32(bf16_bits(rng.standard_normal((16, 32)).astype(np.float32) * 0.02))
          for e in range(2) for p in ("gate", "up")}
    bf["model.layers.0.self_attn.q_proj.weight"] = bf16_to_f32(
        bf16_bits(rng.standard_normal((32, 32)).astype(np.float32)))
    tensors = {k: ("float32", v) for k, v in f32.items()}
    tensors.update({k: ("bfloat16", bf16_bits(v)) for k, v in bf.items()})
    path = tmp_path / "model.safetensors"
    write_safetensors(path, tensors)
    return path, {**f32, **bf}


def _loader_specs(values: dict[str, np.ndarray]) -> list[LayerSpec]:
    names = sorted(k[len("model.layers.0."):] for k in values)
    meta = [{"name": n, "shape": list(values["model.layers.0." + n].shape), "dtype": "float32",
             "offset": 0, "nbytes": 0} for n in names]
    return [LayerSpec(0, "model.layers.0", 0,
                      {"tensors": meta, "full_prefix": "model.layers.0.", "is_moe": True})]


def _read(blob: HostBuffer, m: dict) -> np.ndarray:  # noqa: ANN401
    raw = np.frombuffer(blob.view, dtype=np.uint8, count=m["nbytes"], offset=m["offset"])
    if m["dtype"] == "bfloat16":
        return bf16_to_f32(raw.view(np.uint16)).reshape(m["shape"])
    return raw.view({"float32": np.float32, "float16": np.float16, "int8": np.int8}[m["dtype"]]
                    ).reshape(m["shape"])


def test_preserving_storage_keeps_bf16(tmp_path: Path) -> None:
    path, values = _checkpoint(tmp_path)
    assert read_safetensors_index([path])["model.layers.0.mlp.gate.weight"].dtype == "float32"
    with PreservingSafetensorsStorage([path], _loader_specs(values)) as st:
        spec = st.layers[0]
        st.request(0)
        st.wait(0)
        blob = st.get(0)
        assert blob.nbytes == spec.nbytes
        dtypes = {m["name"]: m["dtype"] for m in spec.metadata["tensors"]}
        assert dtypes["mlp.experts.0.gate_proj.weight"] == "bfloat16"
        assert dtypes["self_attn.q_proj.weight"] == "bfloat16"
        assert dtypes["mlp.gate.weight"] == "float32"
        for m in spec.metadata["tensors"]:
            assert m["offset"] % 256 == 0
            np.testing.assert_array_equal(_read(blob, m), values["model.layers.0." + m["name"]])
        assert "dtype" not in spec.metadata and st.get_disk_read_ms(0) >= 0


def test_preserving_storage_writes_per_channel_int8(tmp_path: Path) -> None:
    path, values = _checkpoint(tmp_path)
    with PreservingSafetensorsStorage.from_model_dir(tmp_path, _loader_specs(values),
                                                     expert_format="int8") as st:
        spec = st.layers[0]
        blob = st.get(0)
        metas = {m["name"]: m for m in spec.metadata["tensors"]}
        assert spec.metadata["dtype"] == "int8_per_channel"
        assert Int8PerChannelDequantizer().is_per_channel(spec)
        q_ref, s_ref = quantize_int8_per_channel(values["model.layers.0.mlp.experts.1.up_proj.weight"])
        np.testing.assert_array_equal(_read(blob, metas["mlp.experts.1.up_proj.weight"]), q_ref)
        np.testing.assert_array_equal(_read(blob, metas["mlp.experts.1.up_proj.weight_scale"]), s_ref)
        # attention and router tensors keep their checkpoint dtypes
        assert metas["self_attn.q_proj.weight"]["dtype"] == "bfloat16"
        np.testing.assert_array_equal(_read(blob, metas["mlp.gate.weight"]),
                                      values["model.layers.0.mlp.gate.weight"])
    with pytest.raises(KeyError):
        bad = _loader_specs(values)
        bad[0].metadata["tensors"].append({"name": "mlp.missing.weight", "shape": [1],
                                           "dtype": "float32", "offset": 0, "nbytes": 4})
        PreservingSafetensorsStorage([path], bad)
