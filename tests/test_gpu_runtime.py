"""The drop-in path end to end on a B200: storage -> runtime -> executor.run_layer.

* ``ResidentOffloadRuntime`` + ``PreservingSafetensorsStorage`` (bf16 and
  per-channel INT8 blobs) + ``GLM4MoeExecutor`` on a small GLM-4 MoE checkpoint
  (a dense layer and two MoE layers), through ``moe_sm100.backends.CUDABackend``:
  the output matches the oracle's decoder layers, and the second pass moves no
  bytes over PCIe (every layer resident) and gives the same bits.
* The reference's own ``OffloadRuntime`` (when the reference package is installed
  under ``baseline/_ref``) driving the executor hook of INTEGRATION.md on the
  reference loader's fp32 blobs, against the reference executor on its
  ``NullBackend``.

Attention runs on the host through the attention delegate (the oracle's
restatement of glm4_moe.py:112-162, or the reference executor's own method), or on
the device (``moe_sm100.attention``, no delegate).
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

import tiny_glm  # noqa: E402
from moe_sm100.backends import CUDABackend  # noqa: E402
from moe_sm100.executors import GLM4MoeExecutor  # noqa: E402
from moe_sm100.loader import PreservingSafetensorsStorage  # noqa: E402
from moe_sm100.packing import dequantize_int8_per_channel, is_expert_weight  # noqa: E402
from moe_sm100.packing import quantize_int8_per_channel  # noqa: E402
from moe_sm100.runtime import ResidentOffloadRuntime  # noqa: E402
from oracle.attention_oracle import AttnConfig, glm4_attention_block, glm4_decoder_layer  # noqa: E402
from oracle.moe_oracle import OracleConfig  # noqa: E402

ROOT = Path(__file__).resolve().parents[1]
T = 24


class _CountingCUDABackend(CUDABackend):
    def __init__(self, device_id: int = 0) -> None:
        super().__init__(device_id)
        self.h2d_bytes = 0

    def copy_h2d_async(self, dst, src, stream):  # noqa: ANN001, ANN201
        self.h2d_bytes += dst.nbytes
        super().copy_h2d_async(dst, src, stream)


class _Lookahead:
    def warmup_prefetch_ids(self, ids: list[int]) -> list[int]:
        return ids[:1]

    def next_prefetch_id(self, ids: list[int], i: int) -> int | None:
        return ids[i + 1] if i + 1 < len(ids) else None


def _oracle_model(vals: dict, x: np.ndarray, int8: bool) -> np.ndarray:
    c = tiny_glm.CONFIG
    attn = AttnConfig.from_hf(c)
    moe = OracleConfig(hidden=c["hidden_size"], n_experts=c["n_routed_experts"],
                       top_k=c["num_experts_per_tok"], inter=c["moe_intermediate_size"],
                       shared_inter=c["moe_intermediate_size"],
                       routed_scaling_factor=c["routed_scaling_factor"], eps=c["rms_norm_eps"])
    for layer in range(c["num_hidden_layers"]):
        t = tiny_glm.layer_tensors(vals, layer)
        if int8:
            t = {k: (dequantize_int8_per_channel(*quantize_int8_per_channel(v))
                     if is_expert_weight(k) else v) for k, v in t.items()}
        x = glm4_decoder_layer(x, t, attn, moe, is_moe=layer >= c["first_k_dense_replace"])
    return x


def _rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b.astype(np.float64)))


@pytest.mark.parametrize("fmt,attention", [("bfloat16", "host"), ("int8", "host"),
                                           ("bfloat16", "device"), ("int8", "device")])
def test_resident_runtime_end_to_end(tmp_path: Path, fmt: str, attention: str) -> None:
    vals = tiny_glm.write_model(tmp_path)
    c = tiny_glm.CONFIG
    attn_cfg = AttnConfig.from_hf(c)
    x = np.random.default_rng(3).standard_normal((T, c["hidden_size"]), dtype=np.float32)
    ref = _oracle_model(vals, x, int8=fmt == "int8")
    backend = _CountingCUDABackend(0)
    storage = PreservingSafetensorsStorage.from_model_dir(tmp_path, tiny_glm.layer_specs(vals),
                                                          expert_format=fmt)
    # attention on the host through the delegate, or on the device (no delegate)
    delegate = {"attention": lambda layer, h, t: glm4_attention_block(h, t, attn_cfg)}
    ex = GLM4MoeExecutor(c, weight_format="int8" if fmt == "int8" else "f16", max_tokens=T,
                         **(delegate if attention == "host" else {}))
    ids = [s.layer_id for s in storage.layers]
    with ResidentOffloadRuntime(storage.layers, backend, storage, _Lookahead(), ex,
                                resident_budget_bytes=8 << 30) as rt:
        out1, m1 = rt.run_inference(ids, x)
        first = backend.h2d_bytes
        assert first == sum(s.nbytes for s in storage.layers) and m1.resident_layers == 0
        err = _rel_l2(out1, ref)
        assert err <= (5e-3 if fmt == "int8" else 2e-3), f"rel-L2 {err:.3e}"
        out2, m2 = rt.run_inference(ids, x)
        assert backend.h2d_bytes == first and m2.transferred_bytes == 0  # nothing re-streamed
        assert m2.resident_layers == len(ids)
        np.testing.assert_array_equal(out1, out2)
        assert rt.pool.resident_bytes > 0
    storage.close()


def _reference() -> object:
    ref_dir = ROOT / "baseline" / "_ref"
    if ref_dir.is_dir() and str(ref_dir) not in sys.path:
        sys.path.insert(0, str(ref_dir))
    return pytest.importorskip("offload_runtime", reason="reference package not installed")


def test_reference_offload_runtime_drives_the_device_executor(tmp_path: Path) -> None:
    """The reference runtime, loader and storage unchanged; only the executor hook
    and the backend are this package's."""
    _reference()
    from offload_runtime.backends.null_backend import NullBackend
    from offload_runtime.executors.glm4_moe import GLM4MoeExecutor as RefGLM4Moe
    from offload_runtime.loader.huggingface import HuggingFaceLoader
    from offload_runtime.runtime import OffloadRuntime
    from offload_runtime.scheduler.lookahead import LookaheadScheduler

    from moe_sm100.executors import reference_delegates

    tiny_glm.write_model(tmp_path)

    class GLM4MoeExecutorB200(RefGLM4Moe):
        def __init__(self, config: dict, **kw: object) -> None:
            super().__init__(config)
            self._dev = GLM4MoeExecutor(config, **kw, **reference_delegates(self))

        def run_layer(self, layer, activations, device_weights, backend, stream):  # noqa: ANN001, ANN201
            if backend.name == "cuda":
                return self._dev.run_layer(layer, activations, device_weights, backend, stream)
            return super().run_layer(layer, activations, device_weights, backend, stream)

    tokens = [3, 17, 5, 9, 60, 2, 33, 8]
    outs = {}
    for name in ("null", "cuda"):
        bundle = HuggingFaceLoader.load_from_dir(tmp_path)
        ids = [s.layer_id for s in bundle.layers]
        if name == "null":
            ex, be = RefGLM4Moe(bundle.config), NullBackend()
        else:
            ex, be = GLM4MoeExecutorB200(bundle.config, max_tokens=len(tokens)), CUDABackend(0)
        with OffloadRuntime(layers=bundle.layers, backend=be, storage=bundle.storage,
                            scheduler=LookaheadScheduler(lookahead=1), executor=ex) as rt:
            hidden = ex.embed(tokens, bundle.embed_weights["model.embed_tokens.weight"])
            hidden, metrics = rt.run_inference(ids, inputs=hidden)
            assert metrics.layer_count == len(ids)
            outs[name] = ex.lm_head(hidden, bundle.head_weights["model.norm.weight"],
                                    bundle.head_weights["lm_head.weight"])
        bundle.storage.close()
    err = _rel_l2(outs["cuda"], outs["null"])
    assert err <= 2e-3, f"logits rel-L2 {err:.3e}"
