"""Token-replicated expert-parallel exchange on one GPU, with the ranks emulated in-process.

The exchange's two collectives are plain tensor operations: the all-gather is the
concatenation of the ranks' token records in rank order, the reduce-scatter the
sum of the ranks' partial sums cut into per-rank blocks.  With torch doing those on
one device, the device side of every rank -- moe_ep_token_pack, moe_ep_experts_gathered,
moe_ep_shared and moe_ep_combine_partial, each rank holding its own expert share --
runs here and is compared with a single plan holding all experts on the same
tokens.  The only arithmetic difference is the order of the fp32 sums over the
routed terms (per rank, then across ranks), so the bound is far below the 16-bit
parity tolerance.  Ragged batches: a full rank, an empty one, and partial ones.
"""
from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]

TOL = 5e-4
CAP = 16


@pytest.mark.parametrize("family,fmt,world", [("glm", "bfloat16", 2), ("qwen3", "int8", 4),
                                              ("glm", "int8", 8)])
def test_token_replicated_exchange_emulated_ranks(family: str, fmt: str, world: int) -> None:
    from moe_sm100 import MoeLayer, MoeLayerConfig
    from moe_sm100._lib import lib
    from moe_sm100.ep import DeviceEPOps
    from moe_sm100.synthetic import SyntheticSpec, build_device_layer
    glm = family == "glm"
    spec = SyntheticSpec(hidden=2048, n_experts=32, top_k=8, inter=512, shared_inter=512,
                         family=family, expert_dtype=fmt, seed=11)
    blob, meta = build_device_layer(spec, device="cuda:0")
    cfg = MoeLayerConfig(hidden=2048, n_experts=32, top_k=8, inter=512, shared_inter=512,
                         use_bias=glm, has_shared_gate=not glm,
                         weight_format="int8" if fmt == "int8" else "f16",
                         routed_scaling_factor=2.5 if glm else 1.0,
                         rms_norm_eps=1e-5, max_tokens=64, device=0)
    full = MoeLayer(cfg)
    full.bind_device(blob.data_ptr(), blob.numel(), meta)
    ranks = [DeviceEPOps(cfg, r, world) for r in range(world)]
    for o in ranks:
        o.bind_device(blob.data_ptr(), blob.numel(), meta)
    torch.cuda.synchronize()
    del blob
    try:
        counts = ([CAP, 0, 5, 1, 9, CAP, 2, 7] * 2)[:world]
        gen = torch.Generator(device="cuda").manual_seed(70 + world)
        xs = [torch.randn((n, 2048), generator=gen, device="cuda") for n in counts]
        sends = [o.token_pack(x, CAP) for o, x in zip(ranks, xs)]
        for o, x in zip(ranks, xs):
            o.start_shared(x)
        recv = torch.cat(sends)  # the all-gather, rank order
        width = int(lib().moe_ep_token_row_halves(ranks[0].layer._plan))
        assert width == 2048 + 4 * 8  # H values, 8 ids and 8 weights
        assert recv.shape == (world * CAP, width)
        ids = ranks[0].gathered_ids(recv)
        for r, n in enumerate(counts):
            assert bool((ids[r * CAP + n:(r + 1) * CAP] == -1).all())
            assert bool((ids[r * CAP:r * CAP + n] >= 0).all())
        partials = [o.experts_gathered(recv) for o in ranks]
        total = torch.stack(partials).sum(0)  # the reduce-scatter, before the cut
        # every record a rank has no expert for stays exactly zero in its partial
        e_loc = 32 // world
        for r, part in enumerate(partials):
            own = ((ids >= r * e_loc) & (ids < (r + 1) * e_loc)).any(dim=1)
            if bool((~own).any()):
                assert float(part[~own].abs().max()) == 0.0
        for r, (o, x) in enumerate(zip(ranks, xs)):
            out = o.combine_partial(x, total[r * CAP:(r + 1) * CAP].contiguous())
            o.status()
            if x.shape[0] == 0:
                assert out.shape == x.shape
                continue
            ref = full.forward(x)
            full.status()
            err = float((out.double() - ref.double()).norm() / ref.double().norm())
            assert err <= TOL, (family, fmt, world, r, err)
    finally:
        for o in ranks:
            o.close()
        full.close()
