"""Expert-parallel protocol on CPU ranks (gloo, world size 2).

moe_sm100.ep.ExpertParallelMoe is the product code that exchanges row counts,
rows, local expert ids and expert outputs between ranks (exact exchange),
fixed-capacity row blocks with the ids in their tails (padded exchange), or
token records and per-token partial sums (token-replicated exchange).  Here each rank plugs
in oracle-based stand-ins for the device ops, so the test checks the protocol
itself (splits, ordering, reverse exchange, combine indexing) against the
single-process oracle, and that malformed dispatch output fails on the host
before any collective runs.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle.cases import CaseSpec, make_case
from oracle.moe_oracle import moe_block, permutation, rms_norm, route, sigmoid, silu

SPEC = CaseSpec(hidden=128, n_experts=8, top_k=3, inter=32, shared_inter=32, tokens=24, seed=17,
                routed_scaling_factor=2.5, family="glm")
SPEC_QWEN = CaseSpec(hidden=128, n_experts=8, top_k=2, inter=32, shared_inter=48, tokens=9, seed=18,
                     family="qwen3", eps=1e-6)


class OracleEPOps:
    """CPU stand-in for DeviceEPOps built on the oracle's numpy arithmetic."""

    def __init__(self, t: dict, cfg, rank: int, world: int, corrupt: bool = False) -> None:  # noqa: ANN001
        self.t, self.cfg, self.rank, self.world = t, cfg, rank, world
        self.e_loc = cfg.n_experts // world
        self.corrupt = corrupt

    def _swiglu(self, x: np.ndarray, prefix: str) -> np.ndarray:
        t = self.t
        return (silu(x @ t[prefix + "gate_proj.weight"].T) * (x @ t[prefix + "up_proj.weight"].T)) @ \
            t[prefix + "down_proj.weight"].T

    def _route(self, x: torch.Tensor):  # noqa: ANN202
        cfg, t = self.cfg, self.t
        h = rms_norm(x.numpy(), t["post_attention_layernorm.weight"], cfg.eps)
        bias = t.get("mlp.gate.e_score_correction_bias") if cfg.use_bias else None
        ids, w, _ = route(h, t["mlp.gate.weight"], bias, cfg)
        offsets, perm = permutation(ids, cfg.n_experts)
        return h, w, ids, offsets, perm

    def dispatch(self, x: torch.Tensor):  # noqa: ANN201
        cfg = self.cfg
        h, w, ids, offsets, perm = self._route(x)
        slot_row = np.empty_like(perm)
        slot_row[perm] = np.arange(perm.size)
        self.state = (h, w, slot_row)
        rows = h[perm // cfg.top_k].astype(np.float32)
        experts = (ids.reshape(-1)[perm] % self.e_loc).astype(np.int32)
        d = np.minimum(np.arange(self.world + 1) * self.e_loc, cfg.n_experts)
        send_offsets = offsets[d].astype(np.int32)
        if self.corrupt:
            send_offsets[-1] += 1
        return torch.from_numpy(rows), torch.from_numpy(experts), torch.from_numpy(send_offsets)

    # fixed-capacity exchange: rows [world*cap, H + 1], the last column the local
    # expert id (-1 unused) standing in for the device format's f16 row + tail
    def capacity(self, tokens: int) -> int:
        return tokens * min(self.cfg.top_k, self.e_loc)

    def dispatch_padded(self, x: torch.Tensor, cap: int) -> torch.Tensor:
        cfg = self.cfg
        hdim = x.shape[1]
        send = np.zeros((self.world * cap, hdim + 1), dtype=np.float32)
        send[:, hdim] = -1
        if x.shape[0] == 0:
            self.state = (np.zeros((0, hdim), np.float32), np.zeros((0, cfg.top_k), np.float32),
                          np.zeros(0, np.int64))
            return torch.from_numpy(send)
        h, w, ids, offsets, perm = self._route(x)
        slot_row = np.empty_like(perm)
        flat = ids.reshape(-1)
        for d in range(self.world):
            beg, end = offsets[d * self.e_loc], offsets[(d + 1) * self.e_loc]
            assert end - beg <= cap
            for j, r in enumerate(range(beg, end)):
                q = perm[r]
                send[d * cap + j, :hdim] = h[q // cfg.top_k]
                send[d * cap + j, hdim] = flat[q] - d * self.e_loc
                slot_row[q] = d * cap + j
        self.state = (h, w, slot_row)
        return torch.from_numpy(send)

    def experts_padded(self, recv: torch.Tensor, cap: int) -> torch.Tensor:
        r = recv.numpy()
        hdim = r.shape[1] - 1
        ids = r[:, hdim].astype(np.int64)
        y = np.zeros((r.shape[0], hdim), dtype=np.float32)
        for le in np.unique(ids[ids >= 0]):
            sel = ids == le
            y[sel] = self._swiglu(r[sel, :hdim], f"mlp.experts.{self.rank * self.e_loc + int(le)}.")
        return torch.from_numpy(y)

    # token-replicated exchange: records [cap, H + 2K], the normalised row, then the
    # K global expert ids (-1: unused record) and the K routing weights, standing
    # in for the device format's f16 row + int32/fp32 tail
    @property
    def experts_per_rank(self) -> int:
        return self.e_loc

    def token_pack(self, x: torch.Tensor, cap: int) -> torch.Tensor:
        k = self.cfg.top_k
        hdim = x.shape[1]
        send = np.zeros((cap, hdim + 2 * k), dtype=np.float32)
        send[:, hdim:hdim + k] = -1
        self.state = (np.zeros((0, hdim), np.float32),)
        if x.shape[0] == 0:
            return torch.from_numpy(send)
        h, w, ids, _offsets, _perm = self._route(x)
        n = h.shape[0]
        send[:n, :hdim] = h
        send[:n, hdim:hdim + k] = ids
        send[:n, hdim + k:] = w
        self.state = (h,)
        return torch.from_numpy(send)

    def gathered_ids(self, recv: torch.Tensor) -> torch.Tensor:
        hdim = recv.shape[1] - 2 * self.cfg.top_k
        return recv[:, hdim:hdim + self.cfg.top_k].to(torch.int64)

    def experts_gathered(self, recv: torch.Tensor) -> torch.Tensor:
        k = self.cfg.top_k
        r = recv.numpy()
        hdim = r.shape[1] - 2 * k
        ids = r[:, hdim:hdim + k].astype(np.int64)
        w = r[:, hdim + k:]
        partial = np.zeros((r.shape[0], hdim), dtype=np.float32)
        lo, hi = self.rank * self.e_loc, (self.rank + 1) * self.e_loc
        for j in range(k):  # slot order, as the device sums
            for g in np.unique(ids[:, j]):
                if not lo <= g < hi:
                    continue
                sel = ids[:, j] == g
                y = self._swiglu(r[sel, :hdim], f"mlp.experts.{int(g)}.")
                partial[sel] += w[sel, j:j + 1] * y
        return torch.from_numpy(partial)

    def combine_partial(self, x: torch.Tensor, partial: torch.Tensor) -> torch.Tensor:
        (h,) = self.state
        if h.shape[0] == 0:
            return x.clone()
        acc = partial.numpy()[:h.shape[0]]
        p = self.cfg.shared_prefix
        if p + "gate_proj.weight" in self.t:
            sh = self._swiglu(h, p)
            if "mlp.shared_expert_gate.weight" in self.t:
                sh = sh * sigmoid(h @ self.t["mlp.shared_expert_gate.weight"].T)
            acc = acc + sh
        return torch.from_numpy(x.numpy() + acc)

    def experts(self, rows: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        r, e = rows.numpy(), ids.numpy()
        y = np.zeros_like(r)
        for le in np.unique(e):
            sel = e == le
            g = self.rank * self.e_loc + int(le)
            y[sel] = self._swiglu(r[sel], f"mlp.experts.{g}.")
        return torch.from_numpy(y)

    def combine(self, x: torch.Tensor, y_back: torch.Tensor) -> torch.Tensor:
        h, w, slot_row = self.state
        k = self.cfg.top_k
        if h.shape[0] == 0:
            return x.clone()
        yb = y_back.numpy()
        acc = np.zeros_like(h)
        for j in range(k):
            acc += w[:, j:j + 1] * yb[slot_row[np.arange(h.shape[0]) * k + j]]
        p = self.cfg.shared_prefix
        if p + "gate_proj.weight" in self.t:
            sh = self._swiglu(h, p)
            if "mlp.shared_expert_gate.weight" in self.t:
                sh = sh * sigmoid(h @ self.t["mlp.shared_expert_gate.weight"].T)
            acc = acc + sh
        return torch.from_numpy(x.numpy() + acc)


def _worker(rank: int, world: int, port: int, spec: CaseSpec, corrupt: bool, q,  # noqa: ANN001
            padded_tokens: int = 0, small_exchange: str = "padded") -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from moe_sm100.ep import ExpertParallelMoe
        x, t, _q, cfg = make_case(spec)
        # weak scaling: each rank routes its own half of the tokens
        mine = np.array_split(np.arange(spec.tokens), world)[rank]
        xr = x[mine]
        ep = ExpertParallelMoe(OracleEPOps(t, cfg, rank, world, corrupt=corrupt and rank == 0),
                               padded_tokens=padded_tokens, small_exchange=small_exchange)
        try:
            out = ep.forward(torch.from_numpy(xr)).numpy()
        except ValueError as err:
            q.put((rank, "ValueError", str(err)))
            return
        if xr.shape[0] == 0:
            q.put((rank, "ok", 0.0 if out.shape == xr.shape else 1.0))
            return
        ref, _ = moe_block(xr, t, cfg)
        err = float(np.linalg.norm(out - ref) / np.linalg.norm(ref))
        q.put((rank, "ok", err))
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(spec: CaseSpec, corrupt: bool = False, padded_tokens: int = 0,
         small_exchange: str = "padded") -> list:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker,
                         args=(r, 2, port, spec, corrupt, q, padded_tokens, small_exchange))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        if p.is_alive():
            p.kill()
            pytest.fail("gloo rank did not finish")
    return sorted(q.get(timeout=5) for _ in range(len(procs)) if not q.empty())


@pytest.mark.parametrize("spec", [SPEC, SPEC_QWEN], ids=["glm", "qwen3"])
def test_expert_parallel_protocol_matches_oracle(spec: CaseSpec) -> None:
    res = _run(spec)
    assert [r[1] for r in res] == ["ok", "ok"], res
    for _rank, _status, err in res:
        assert err < 1e-5


def test_malformed_dispatch_fails_on_host_before_exchange() -> None:
    res = _run(SPEC, corrupt=True)
    # rank 0 detects its own bad offsets and raises; rank 1 then finds its
    # count exchange partner gone and errors (or both raise) -- nobody hangs
    assert any(r[0] == 0 and r[1] == "ValueError" for r in res), res


@pytest.mark.parametrize("spec", [SPEC, SPEC_QWEN], ids=["glm", "qwen3"])
def test_fixed_capacity_exchange_matches_oracle(spec: CaseSpec) -> None:
    """Padded exchange: equal splits of cap rows, ids in the row tails, unused rows
    skipped by the experts and never read by combine."""
    res = _run(spec, padded_tokens=spec.tokens)
    assert [r[1] for r in res] == ["ok", "ok"], res
    for _rank, _status, err in res:
        assert err < 1e-5


def test_fixed_capacity_exchange_with_an_empty_rank() -> None:
    """One token over two ranks: rank 1 has no tokens, sends only unused rows and
    still serves rank 0's rows for its experts."""
    from dataclasses import replace
    res = _run(replace(SPEC, tokens=1), padded_tokens=4)
    assert [r[1] for r in res] == ["ok", "ok"], res
    for _rank, _status, err in res:
        assert err < 1e-5


@pytest.mark.parametrize("spec", [SPEC, SPEC_QWEN], ids=["glm", "qwen3"])
def test_token_replicated_exchange_matches_oracle(spec: CaseSpec) -> None:
    """Gathered exchange: all-gather of token records (ids and weights in the
    tails), per-rank partial sums over the resident experts, reduce-scatter sum.
    The ranks hold 12 and 12 (glm) / 5 and 4 (qwen3) tokens under a cap of 16."""
    res = _run(spec, padded_tokens=16, small_exchange="gathered")
    assert [r[1] for r in res] == ["ok", "ok"], res
    for _rank, _status, err in res:
        assert err < 1e-5


def test_token_replicated_exchange_with_an_empty_rank() -> None:
    """One token over two ranks: rank 1 sends only unused records, serves rank 0's
    slots for its experts and gets an empty partial back."""
    from dataclasses import replace
    res = _run(replace(SPEC, tokens=1), padded_tokens=4, small_exchange="gathered")
    assert [r[1] for r in res] == ["ok", "ok"], res
    for _rank, _status, err in res:
        assert err < 1e-5


class _RecordingP2POps:
    """Records the peer-memory exchange's calls (the device work itself needs GPUs)."""

    def __init__(self) -> None:
        self.calls: list = []

    def p2p_setup(self, cap: int, group) -> None:  # noqa: ANN001
        self.calls.append(("setup", cap))

    def p2p_pack(self, x: torch.Tensor, cap: int) -> None:
        self.calls.append(("pack", int(x.shape[0]), cap))

    def start_shared(self, x: torch.Tensor) -> None:
        self.calls.append(("shared",))

    def p2p_wait(self, which: int) -> None:
        self.calls.append(("wait", which))

    def p2p_experts(self) -> None:
        self.calls.append(("experts",))

    def p2p_combine(self, x: torch.Tensor) -> torch.Tensor:
        self.calls.append(("combine",))
        return x + 1


def test_peer_memory_exchange_protocol_order() -> None:
    """p2p exchange: buffers set up once at construction, then per forward pack,
    shared expert, wait for records, experts (+ partials to owners), wait for
    partials, combine; batches above padded_tokens take the exact path."""
    from moe_sm100.ep import ExpertParallelMoe
    ops = _RecordingP2POps()
    ep = ExpertParallelMoe(ops, padded_tokens=8, small_exchange="p2p")
    assert ops.calls == [("setup", 8)]
    out = ep.forward(torch.zeros(5, 4))
    assert torch.equal(out, torch.ones(5, 4))
    assert ops.calls[1:] == [("pack", 5, 8), ("shared",), ("wait", 0), ("experts",), ("wait", 1),
                             ("combine",)]
    with pytest.raises(ValueError):
        ExpertParallelMoe(ops, padded_tokens=8, small_exchange="bogus")
