"""Expert-parallel forward on 2 GPUs over NCCL vs the single-GPU forward (needs >= 2 B200).

Two processes, one per GPU, each holding half of the routed experts.  Each rank
compares its expert-parallel output with a single-GPU plan holding all experts
on the same tokens: the only arithmetic difference is that expert outputs cross
the exchange as f16 (or are summed per rank before a reduce-scatter), so the
bound is the 16-bit parity tolerance.  All four exchanges run: exact (counts,
then rows and ids), fixed-capacity (equal row blocks, ids in the row tails),
token-replicated over NCCL (all-gather of token records, reduce-scatter of partial
sums) and the same over peer memory (NVLink stores and epoch flags, no NCCL).
"""
from __future__ import annotations

import os
import socket

import pytest

torch = pytest.importorskip("torch")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs 2 GPUs")]

TOL = 2e-3


def _worker(rank: int, world: int, port: int, q) -> None:  # noqa: ANN001
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device(f"cuda:{rank}"))
    try:
        from moe_sm100 import MoeLayer, MoeLayerConfig
        from moe_sm100.ep import DeviceEPOps, ExpertParallelMoe
        from moe_sm100.synthetic import SyntheticSpec, build_device_layer
        results = []
        for family, fmt in (("glm", "bfloat16"), ("qwen3", "int8")):
            spec = SyntheticSpec(hidden=2048, n_experts=32, top_k=8, inter=512, shared_inter=512,
                                 family=family, expert_dtype=fmt, seed=3)
            blob, meta = build_device_layer(spec, device=f"cuda:{rank}")
            glm = family == "glm"
            cfg = MoeLayerConfig(hidden=2048, n_experts=32, top_k=8, inter=512, shared_inter=512,
                                 use_bias=glm, has_shared_gate=not glm,
                                 weight_format="int8" if fmt == "int8" else "f16",
                                 routed_scaling_factor=2.5 if glm else 1.0,
                                 rms_norm_eps=1e-5, max_tokens=512, device=rank)
            ops = DeviceEPOps(cfg, rank, world)
            ops.bind_device(blob.data_ptr(), blob.numel(), meta)
            full = MoeLayer(cfg)
            full.bind_device(blob.data_ptr(), blob.numel(), meta)
            torch.cuda.synchronize()
            del blob
            ep = ExpertParallelMoe(ops)
            epp = ExpertParallelMoe(ops, padded_tokens=64)
            epg = ExpertParallelMoe(ops, padded_tokens=64, small_exchange="gathered")
            epp2p = ExpertParallelMoe(ops, padded_tokens=64, small_exchange="p2p")
            gen = torch.Generator(device=f"cuda:{rank}").manual_seed(100 + rank)
            for T in (1, 37, 300):
                x = torch.randn((T, 2048), generator=gen, device=f"cuda:{rank}")
                ref = full.forward(x)
                for mode, e in (("exact", ep), ("padded", epp), ("gathered", epg), ("p2p", epp2p)):
                    out = e.forward(x)  # T = 300 > 64 takes the exact path in all four
                    ops.status()
                    err = float((out.double() - ref.double()).norm() / ref.double().norm())
                    results.append((family, mode, T, err))
                full.status()
            # a capacity below the batch's worst case is refused on the host
            from ctypes import c_void_p
            from moe_sm100._lib import lib
            x = torch.randn((8, 2048), generator=gen, device=f"cuda:{rank}")
            send = torch.empty((2 * 8, 2048 + 8), dtype=torch.float16, device=f"cuda:{rank}")
            ws = torch.empty(int(lib().moe_workspace_bytes(ops.layer._plan, 8)), dtype=torch.uint8,
                             device=f"cuda:{rank}")
            rc = lib().moe_ep_dispatch_padded(ops.layer._plan, c_void_p(x.data_ptr()), 8, 8,
                                              c_void_p(send.data_ptr()), c_void_p(ws.data_ptr()),
                                              ws.numel(), c_void_p(0))
            results.append((family, "small_cap_rc", 8, 0.0 if rc != 0 else 1.0))
            ops.close()
            full.close()
        q.put((rank, results))
    finally:
        dist.destroy_process_group()


def test_expert_parallel_two_gpus_matches_single_gpu() -> None:
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        assert not p.is_alive(), "rank did not finish"
        assert p.exitcode == 0
    res = [q.get(timeout=10) for _ in procs]
    for _rank, rows in res:
        for family, mode, T, err in rows:
            assert err <= TOL, (family, mode, T, err)
