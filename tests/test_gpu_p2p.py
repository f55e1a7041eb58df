"""Peer-memory exchange on one GPU: the data path as a single rank, and a wait that runs out.

With one rank (world = 1) the packing kernel stores the records into the rank's own
receive buffer and the partial-sum kernel into its own partial buffer, so pack,
experts, partial sums and combine run exactly as on many GPUs; the waits find their
flags already set by the kernels before them on the stream.  Compared with the
single-GPU forward of the same plan.  The multi-GPU case is in test_ep_gpu.py.

The failure path: a wait for an epoch that no kernel publishes gives up after its
limit, records a timeout that moe_status reports as MOE_ERR_TIMEOUT, and the next
forward on the same plan is correct.
"""
from __future__ import annotations

import os
import socket

import pytest

torch = pytest.importorskip("torch")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]

TOL = 5e-4


@pytest.fixture(scope="module")
def one_rank_group():
    import datetime
    import torch.distributed as dist
    if dist.is_initialized():
        yield None
        return
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60))
    yield None
    dist.destroy_process_group()


@pytest.mark.parametrize("family,fmt", [("glm", "bfloat16"), ("qwen3", "int8")])
def test_peer_exchange_single_rank_matches_forward(one_rank_group, family: str, fmt: str) -> None:  # noqa: ANN001
    from moe_sm100 import MoeLayer, MoeLayerConfig
    from moe_sm100.ep import DeviceEPOps, ExpertParallelMoe
    from moe_sm100.synthetic import SyntheticSpec, build_device_layer
    glm = family == "glm"
    spec = SyntheticSpec(hidden=2048, n_experts=32, top_k=8, inter=512, shared_inter=512,
                         family=family, expert_dtype=fmt, seed=12)
    blob, meta = build_device_layer(spec, device="cuda:0")
    cfg = MoeLayerConfig(hidden=2048, n_experts=32, top_k=8, inter=512, shared_inter=512,
                         use_bias=glm, has_shared_gate=not glm,
                         weight_format="int8" if fmt == "int8" else "f16",
                         routed_scaling_factor=2.5 if glm else 1.0,
                         rms_norm_eps=1e-5, max_tokens=64, device=0)
    full = MoeLayer(cfg)
    full.bind_device(blob.data_ptr(), blob.numel(), meta)
    ops = DeviceEPOps(cfg, 0, 1)
    ops.bind_device(blob.data_ptr(), blob.numel(), meta)
    torch.cuda.synchronize()
    del blob
    try:
        ep = ExpertParallelMoe(ops, padded_tokens=32, small_exchange="p2p")
        gen = torch.Generator(device="cuda").manual_seed(9)
        for T in (1, 17, 32, 5):  # several epochs over the same buffers
            x = torch.randn((T, 2048), generator=gen, device="cuda")
            out = ep.forward(x)
            ops.status()
            ref = full.forward(x)
            full.status()
            err = float((out.double() - ref.double()).norm() / ref.double().norm())
            assert err <= TOL, (family, fmt, T, err)
        ep.forward(torch.randn((7, 2048), generator=gen, device="cuda"), timed=True)
        assert ep.last_timing["exchanged_rows"] == 32
        assert 0 < ep.last_timing["recv_rows"] <= 7 * 8
        # the pipelined serving loop through the same exchange: batches on two slots,
        # each output as the single-GPU forward of its batch
        pipe = ep.host_pipeline(24, depth=2)
        xs = [torch.randn((24, 2048), generator=gen, device="cuda") for _ in range(4)]
        pipe.x[0].copy_(xs[0])
        pipe.x[1].copy_(xs[1])
        for i in range(len(xs)):
            pipe.submit(i)
            if i >= 1:
                got = pipe.wait(i - 1).clone()
                if i + 1 < len(xs):
                    pipe.x[(i + 1) % 2].copy_(xs[i + 1])
                ref = full.forward(xs[i - 1]).cpu()
                err = float((got.double() - ref.double()).norm() / ref.double().norm())
                assert err <= TOL, (family, fmt, "pipeline", i - 1, err)
        got = pipe.wait(len(xs) - 1).clone()
        ref = full.forward(xs[-1]).cpu()
        assert float((got.double() - ref.double()).norm() / ref.double().norm()) <= TOL
        pipe.status()
        full.status()
    finally:
        ops.close()
        full.close()


def test_peer_wait_that_runs_out_reports_timeout(one_rank_group) -> None:  # noqa: ANN001
    from ctypes import c_void_p
    from moe_sm100 import MoeLayer, MoeLayerConfig
    from moe_sm100 import _lib
    from moe_sm100._lib import MoeError, lib
    from moe_sm100.synthetic import SyntheticSpec, build_device_layer
    spec = SyntheticSpec(hidden=1024, n_experts=8, top_k=2, inter=256, shared_inter=256,
                         family="glm", expert_dtype="bfloat16", seed=5)
    blob, meta = build_device_layer(spec, device="cuda:0")
    cfg = MoeLayerConfig(hidden=1024, n_experts=8, top_k=2, inter=256, shared_inter=256,
                         use_bias=True, routed_scaling_factor=2.5, max_tokens=8, device=0)
    ml = MoeLayer(cfg)
    ml.bind_device(blob.data_ptr(), blob.numel(), meta)
    flags = torch.zeros(16, dtype=torch.int32, device="cuda")  # nothing ever publishes
    try:
        rc = lib().moe_ep_p2p_wait(ml._plan, c_void_p(flags.data_ptr()), 2, 1, 2_000_000,
                                   c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 0
        with pytest.raises(MoeError) as ei:
            ml.status()
        assert ei.value.code == _lib.MOE_ERR_TIMEOUT
        # invalid requests are refused on the host
        assert lib().moe_ep_p2p_wait(ml._plan, c_void_p(flags.data_ptr()), 9, 1, 1000, c_void_p(0)) != 0
        assert lib().moe_ep_p2p_wait(ml._plan, c_void_p(flags.data_ptr()), 2, 0, 1000, c_void_p(0)) != 0
        # the context and the plan stay usable
        x = torch.randn((4, 1024), device="cuda")
        y = ml.forward(x)
        ml.status()
        assert bool(torch.isfinite(y).all())
    finally:
        ml.close()
