"""Failure reporting on the device, without faulting the GPU (needs a B200).

* A bounded wait that runs out: ``moe_wait_probe`` waits, with the same bounded
  mbarrier wait the kernels use, on a barrier nothing arrives at; the wait gives
  up, the plan's status reads MOE_ERR_TIMEOUT, and the context stays usable (the
  next forward gives the same bits as before).
* An f16 activation that overflows: a layer whose expert weights drive
  silu(gate) * up past 65504 is reported as MOE_ERR_RANGE instead of flowing on
  as inf.
"""
from __future__ import annotations

from ctypes import c_void_p

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

from moe_sm100 import MoeLayer, MoeLayerConfig, _lib  # noqa: E402
from moe_sm100.packing import pack_layer  # noqa: E402

H, E, K, I = 256, 8, 2, 64


def _layer(scale: float) -> MoeLayer:
    rng = np.random.default_rng(5)
    t = {"post_attention_layernorm.weight": np.ones(H, np.float32),
         "mlp.gate.weight": (rng.standard_normal((E, H)) * 0.02).astype(np.float32)}
    for e in range(E):
        for name, shape in (("gate_proj", (I, H)), ("up_proj", (I, H)), ("down_proj", (H, I))):
            t[f"mlp.experts.{e}.{name}.weight"] = (rng.standard_normal(shape) * scale).astype(np.float32)
    blob, meta = pack_layer(t, expert_format="bfloat16")
    ml = MoeLayer(MoeLayerConfig(hidden=H, n_experts=E, top_k=K, inter=I, shared_inter=0,
                                 use_bias=False, routed_scaling_factor=1.0, max_tokens=16))
    ml.bind_host(blob, meta)
    return ml


def test_bounded_wait_runs_out_and_the_context_stays_usable() -> None:
    ml = _layer(0.02)
    x = torch.randn((9, H), generator=torch.Generator().manual_seed(1)).cuda()
    before = ml.forward(x).clone()
    ml.status()
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(_lib.lib().moe_wait_probe(ml._plan, 2_000_000, c_void_p(stream)))  # ~1 ms
    with pytest.raises(_lib.MoeError) as err:
        ml.status()
    assert err.value.code == _lib.MOE_ERR_TIMEOUT
    after = ml.forward(x)
    ml.status()  # the error word was cleared by the status read
    assert torch.equal(before, after)
    assert _lib.lib().moe_wait_probe(ml._plan, 0, c_void_p(stream)) == _lib.MOE_ERR_INVALID
    ml.close()


def test_f16_overflow_is_reported() -> None:
    ml = _layer(30.0)  # |gate|, |up| ~ 480 per token: silu(gate) * up far beyond 65504
    x = torch.randn((4, H), generator=torch.Generator().manual_seed(2)).cuda()
    ml.forward(x)
    with pytest.raises(_lib.MoeError) as err:
        ml.status()
    assert err.value.code == _lib.MOE_ERR_RANGE
    ml.close()
    ok = _layer(0.02)
    ok.forward(x)
    ok.status()
    ok.close()
