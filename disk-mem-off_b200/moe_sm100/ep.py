"""Expert-parallel MoE layer: one process per GPU, experts sharded across ranks.

Rank r of N holds routed experts [r*E/N, (r+1)*E/N) (packed from the same layer
blob), the router and the shared expert are replicated, and every rank routes its
own tokens.  One forward (weak scaling: T tokens per rank):

  1. dispatch   route the local tokens; normalised f16 rows grouped by owner rank
  2. counts     all_to_all of the per-rank row counts (the only host sync)
  3. exchange   all_to_all of the rows and of their local expert ids; meanwhile
                the shared expert runs on a side stream when the ops provide it
                (``start_shared``).  (One batched group of point-to-point
                transfers for both was measured slower than two all_to_alls.)
  4. experts    grouped GEMMs of the resident experts on the received rows
  5. return     all_to_all of the f16 expert outputs back to their source rank
  6. combine    x + sum_k w * y + shared expert

Small batches can instead use the fixed-capacity exchange (``padded_tokens``): every
rank sends every rank exactly ``cap`` rows (cap = the most rows one batch of
``padded_tokens`` tokens can route to one rank), the local expert id travels in
each row's tail (-1 marks an unused row), and steps 2-3 become one all_to_all of
equal splits.  No counts cross and the host never waits, so the CPU runs ahead of
the device across layers; the price is moving cap rows per rank pair.

Or small batches replicate the tokens instead (``small_exchange="gathered"``):
every rank all-gathers fixed-size token records (normalised row, top-k expert ids
and weights; ``padded_tokens`` records per rank), applies its resident experts to
the slots of all gathered tokens that route to them, and one reduce-scatter (sum)
of per-token fp32 partial sums returns each rank the routed total for its own
tokens.  The host never waits either, and the bytes per rank are world * cap
records in and world * cap fp32 rows out, independent of top_k, where the padded
exchange moves world * cap * min(top_k, experts per rank) rows each way.

Or the same token-replicated exchange over peer memory (``small_exchange="p2p"``):
no collective library at all.  The packing kernel stores each rank's records
straight into every rank's receive buffer over NVLink, the partial-sum kernel
stores each record's partial sum straight into its owner's buffer, each publishing
an epoch flag when its stores are complete, and a bounded wait kernel on each rank
stands in for each collective (buffers mapped once with CUDA IPC, ``p2p.py``).

The collectives are torch.distributed (NCCL over NVLink on B200; gloo on CPU in
the tests).  The device work is libmoe_sm100's moe_ep_* entry points.
"""
from __future__ import annotations

from ctypes import c_void_p
from dataclasses import replace
from typing import Any, Protocol

from ._lib import check, lib
from .config import MoeLayerConfig
from .layer import MoeLayer, _stream_handle


def _torch():
    import torch
    return torch


class EPOps(Protocol):
    """Per-rank compute of the expert-parallel block (device or test stand-in).

    Optional: ``start_shared(x)`` (shared expert early, overlapping the exchange);
    for the fixed-capacity exchange ``capacity(tokens)``, ``dispatch_padded(x, cap)``
    (send rows [world*cap, ...] with the local expert id, -1 unused, in each row),
    ``experts_padded(recv, cap)`` and, for timed forwards, ``padded_ids(recv)``;
    for the token-replicated exchange ``token_pack(x, cap)`` (token records
    [cap, ...]), ``experts_gathered(recv)`` (fp32 partial sums [rows, H]),
    ``combine_partial(x, partial)`` and, for timed forwards, ``gathered_ids(recv)``
    (global expert ids [rows, top_k], -1 for unused records).
    """

    def dispatch(self, x: Any) -> tuple[Any, Any, Any]: ...      # rows, local expert ids, offsets

    def experts(self, rows: Any, expert_ids: Any) -> Any: ...   # expert outputs, same order

    def combine(self, x: Any, y_back: Any) -> Any: ...          # x + MoE(x)


class ExpertParallelMoe:
    """Runs the dispatch / expert / combine protocol of one rank.

    ``padded_tokens`` > 0 switches batches of at most that many tokens to a
    fixed-size exchange: ``small_exchange="padded"`` the fixed-capacity one (ops must
    provide ``capacity``, ``dispatch_padded`` and ``experts_padded``), "gathered" the
    token-replicated one (``token_pack``, ``experts_gathered``, ``combine_partial``).
    Every rank must take the same branch in the same forward: give all ranks the
    same ``padded_tokens`` and ``small_exchange`` and batches on the same side of it
    (decode steps below, prefill above).
    """

    def __init__(self, ops: EPOps, group: Any = None, padded_tokens: int = 0,
                 small_exchange: str = "padded") -> None:
        if small_exchange not in ("padded", "gathered", "p2p"):
            raise ValueError("small_exchange must be 'padded', 'gathered' or 'p2p'")
        self.ops = ops
        self.group = group
        self.last_timing: dict[str, float] = {}
        self.padded_tokens = int(padded_tokens)
        self.small_exchange = small_exchange
        self.cap = 0
        if self.padded_tokens > 0:
            self.cap = (int(ops.capacity(self.padded_tokens)) if small_exchange == "padded"
                        else self.padded_tokens)
            if self.cap <= 0:
                raise ValueError("no fixed capacity for padded_tokens")
            if small_exchange == "p2p":
                ops.p2p_setup(self.cap, group)

    def host_pipeline(self, tokens: int, depth: int = 2) -> Any:
        """Steps from pinned host memory with their copies overlapping the neighbouring
        steps' compute (``layer.HostPipeline``).  The step is this rank's forward,
        issued each step (not captured); every rank submits the same steps in order."""
        from .layer import HostPipeline

        def step(din: Any, dout: Any) -> None:
            dout.copy_(self.forward(din))
        return HostPipeline(step, tokens, self.ops.cfg.hidden, self.ops.cfg.device, depth,
                            graph=False, check=self.ops.status)

    def forward(self, x: Any, timed: bool = False) -> Any:
        torch = _torch()
        ev = {}

        def mark(name: str) -> None:
            if timed and x.is_cuda:
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                ev[name] = e

        if 0 < self.padded_tokens and x.shape[0] <= self.padded_tokens:
            if self.small_exchange == "gathered":
                out, n_recv = self._forward_gathered(x, mark)
            elif self.small_exchange == "p2p":
                out, n_recv = self._forward_p2p(x, mark)
            else:
                out, n_recv = self._forward_padded(x, mark)
        else:
            out, n_recv = self._forward_exact(x, mark)
        if timed and x.is_cuda:
            torch.cuda.synchronize()
            t = lambda a, b: ev[a].elapsed_time(ev[b])  # noqa: E731
            self.last_timing = {
                "dispatch_ms": t("start", "dispatched"),
                "a2a_ms": t("dispatched", "exchanged") + t("computed", "returned"),
                "experts_ms": t("exchanged", "computed"),
                "combine_ms": t("returned", "end"),
                "total_ms": t("start", "end"),
            }
            self.last_timing.update(n_recv())
        return out

    def _forward_padded(self, x: Any, mark: Any) -> tuple[Any, Any]:
        torch = _torch()
        import torch.distributed as dist
        g, cap = self.group, self.cap
        mark("start")
        send = self.ops.dispatch_padded(x, cap)
        mark("dispatched")
        start_shared = getattr(self.ops, "start_shared", None)
        if start_shared is not None:
            start_shared(x)
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=g)
        mark("exchanged")
        y = self.ops.experts_padded(recv, cap)
        mark("computed")
        y_back = torch.empty_like(y)
        dist.all_to_all_single(y_back, y, group=g)
        mark("returned")
        out = self.ops.combine(x, y_back)
        mark("end")

        def counts() -> dict[str, float]:
            ids = self.ops.padded_ids(recv)
            valid = ids[ids >= 0]
            return {"recv_rows": int(valid.numel()),
                    "recv_experts": int(torch.unique(valid).numel()) if valid.numel() else 0,
                    "exchanged_rows": int(recv.shape[0])}
        return out, counts

    def _forward_gathered(self, x: Any, mark: Any) -> tuple[Any, Any]:
        torch = _torch()
        import torch.distributed as dist
        g, cap = self.group, self.cap
        world = dist.get_world_size(g)
        mark("start")
        send = self.ops.token_pack(x, cap)
        mark("dispatched")
        start_shared = getattr(self.ops, "start_shared", None)
        if start_shared is not None:
            start_shared(x)
        recv = send.new_empty((world * cap,) + tuple(send.shape[1:]))
        dist.all_gather_into_tensor(recv, send, group=g)
        mark("exchanged")
        partial_all = self.ops.experts_gathered(recv)
        mark("computed")
        partial = partial_all.new_empty((cap,) + tuple(partial_all.shape[1:]))
        dist.reduce_scatter_tensor(partial, partial_all, op=dist.ReduceOp.SUM, group=g)
        mark("returned")
        out = self.ops.combine_partial(x, partial)
        mark("end")

        def counts() -> dict[str, float]:
            ids = self.ops.gathered_ids(recv)
            valid = ids[ids >= 0]
            rank = dist.get_rank(g)
            e_loc = self.ops.experts_per_rank
            mine = valid[(valid >= rank * e_loc) & (valid < (rank + 1) * e_loc)]
            return {"recv_rows": int(mine.numel()),
                    "recv_experts": int(torch.unique(mine).numel()) if mine.numel() else 0,
                    "exchanged_rows": int(recv.shape[0])}
        return out, counts

    def _forward_p2p(self, x: Any, mark: Any) -> tuple[Any, Any]:
        torch = _torch()
        cap = self.cap
        mark("start")
        self.ops.p2p_pack(x, cap)
        mark("dispatched")
        start_shared = getattr(self.ops, "start_shared", None)
        if start_shared is not None:
            start_shared(x)
        self.ops.p2p_wait(0)
        mark("exchanged")
        self.ops.p2p_experts()
        mark("computed")
        self.ops.p2p_wait(1)
        mark("returned")
        out = self.ops.p2p_combine(x)
        mark("end")

        def counts() -> dict[str, float]:
            ids = self.ops.p2p_ids()
            valid = ids[ids >= 0]
            e_loc = self.ops.experts_per_rank
            r = self.ops.rank
            mine = valid[(valid >= r * e_loc) & (valid < (r + 1) * e_loc)]
            return {"recv_rows": int(mine.numel()),
                    "recv_experts": int(torch.unique(mine).numel()) if mine.numel() else 0,
                    "exchanged_rows": int(ids.shape[0])}
        return out, counts

    def _forward_exact(self, x: Any, mark: Any) -> tuple[Any, Any]:
        torch = _torch()
        import torch.distributed as dist
        g = self.group
        mark("start")
        send_rows, send_experts, send_offsets = self.ops.dispatch(x)
        mark("dispatched")
        # counts go through the exchange on the device; the host reads the send
        # offsets and the received counts in one synchronisation
        world = dist.get_world_size(g)
        send_offsets = send_offsets.to(torch.int64)
        send_counts = send_offsets[1:] - send_offsets[:-1]
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=g)
        both = torch.cat([send_offsets, recv_counts]).tolist()
        offs, rc = both[:world + 1], both[world + 1:]
        if len(offs) != world + 1 or offs[0] != 0 or offs[-1] != send_rows.shape[0] \
                or any(b < a for a, b in zip(offs, offs[1:])):
            raise ValueError(f"malformed send offsets {offs} for {send_rows.shape[0]} rows")
        sc = [b - a for a, b in zip(offs, offs[1:])]
        n_recv = int(sum(rc))
        start_shared = getattr(self.ops, "start_shared", None)
        if start_shared is not None:
            start_shared(x)
        h = send_rows.shape[1]
        recv_rows = send_rows.new_empty((n_recv, h))
        recv_experts = send_experts.new_empty((n_recv,))
        dist.all_to_all_single(recv_rows, send_rows, rc, sc, group=g)
        dist.all_to_all_single(recv_experts, send_experts, rc, sc, group=g)
        mark("exchanged")
        y = self.ops.experts(recv_rows, recv_experts)
        mark("computed")
        y_back = y.new_empty((send_rows.shape[0], h))
        dist.all_to_all_single(y_back, y, sc, rc, group=g)
        mark("returned")
        out = self.ops.combine(x, y_back)
        mark("end")

        def counts() -> dict[str, float]:
            return {"recv_rows": n_recv,
                    "recv_experts": int(torch.unique(recv_experts).numel()) if n_recv else 0,
                    "exchanged_rows": n_recv}
        return out, counts


class DeviceEPOps:
    """EPOps over libmoe_sm100 for this rank's expert share (CUDA tensors).

    ``pool``: a dict shared by the layers of a stack that run one after another on
    the same stream.  Their workspaces and the shared-expert side stream then live
    in it once instead of once per layer (a forward's workspace is free again when
    its combine has been issued, and the next layer's dispatch is ordered after it).
    """

    def __init__(self, cfg: MoeLayerConfig, rank: int, world: int,
                 pool: dict[str, Any] | None = None) -> None:
        if cfg.n_experts % world:
            raise ValueError("n_experts must be divisible by the number of ranks")
        e_loc = cfg.n_experts // world
        self.cfg = replace(cfg, expert_begin=rank * e_loc, expert_end=(rank + 1) * e_loc)
        self.layer = MoeLayer(self.cfg)
        self.world = world
        self._pool: dict[str, Any] = pool if pool is not None else {}
        self._T = 0
        self._shared_done: Any = None  # event of a shared-expert pass started early

    @property
    def _ws(self) -> Any:
        return self._pool.get("ws")

    def bind_device(self, blob_ptr: int, blob_bytes: int, tensor_meta: list[dict[str, Any]],
                    stream: Any = None) -> None:
        self.layer.bind_device(blob_ptr, blob_bytes, tensor_meta, stream)

    def _buf(self, key: str, nbytes: int) -> Any:
        torch = _torch()
        cur = self._pool.get(key)
        if cur is None or cur.numel() < nbytes:
            cur = None  # drop the smaller buffer before allocating its successor
            self._pool.pop(key, None)
            cur = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=f"cuda:{self.cfg.device}")
            self._pool[key] = cur
        return cur

    def dispatch(self, x: Any) -> tuple[Any, Any, Any]:
        torch = _torch()
        t = x.shape[0]
        k, h = self.cfg.top_k, self.cfg.hidden
        plan = self.layer._plan
        ws = self._buf("ws", int(lib().moe_workspace_bytes(plan, max(t, 1))))
        rows = torch.empty((t * k, h), dtype=torch.float16, device=x.device)
        experts = torch.empty((t * k,), dtype=torch.int32, device=x.device)
        offsets = torch.empty((self.world + 1,), dtype=torch.int32, device=x.device)
        check(lib().moe_ep_dispatch(plan, c_void_p(x.data_ptr()), t, c_void_p(rows.data_ptr()),
                                    c_void_p(experts.data_ptr()), c_void_p(offsets.data_ptr()),
                                    c_void_p(ws.data_ptr()), ws.numel(),
                                    c_void_p(_stream_handle(None))))
        self._T = t
        return rows, experts, offsets

    def capacity(self, tokens: int) -> int:
        """Rows one rank may have to send one destination for `tokens` tokens."""
        return int(lib().moe_ep_capacity(self.layer._plan, int(tokens)))

    def dispatch_padded(self, x: Any, cap: int) -> Any:
        torch = _torch()
        t = x.shape[0]
        plan = self.layer._plan
        ws = self._buf("ws", int(lib().moe_workspace_bytes(plan, max(t, 1))))
        send = torch.empty((self.world * cap, self.cfg.hidden + 8), dtype=torch.float16,
                           device=x.device)
        check(lib().moe_ep_dispatch_padded(plan, c_void_p(x.data_ptr()), t, cap,
                                           c_void_p(send.data_ptr()), c_void_p(ws.data_ptr()),
                                           ws.numel(), c_void_p(_stream_handle(None))))
        self._T = t
        return send

    def experts_padded(self, recv: Any, cap: int) -> Any:
        torch = _torch()
        plan = self.layer._plan
        y = torch.empty((recv.shape[0], self.cfg.hidden), dtype=torch.float16, device=recv.device)
        ws = self._buf("ws_ep", int(lib().moe_ep_padded_workspace_bytes(plan, cap)))
        check(lib().moe_ep_experts_padded(plan, c_void_p(recv.data_ptr()), cap, c_void_p(y.data_ptr()),
                                          c_void_p(ws.data_ptr()), ws.numel(),
                                          c_void_p(_stream_handle(None))))
        return y

    def padded_ids(self, recv: Any) -> Any:
        """Local expert id of every received row (-1: unused), from the row tails."""
        h = self.cfg.hidden
        return recv[:, h:h + 8].contiguous().view(_torch().int32)[:, 0]

    @property
    def experts_per_rank(self) -> int:
        return self.cfg.expert_end - self.cfg.expert_begin

    def token_pack(self, x: Any, cap: int) -> Any:
        """Token records [cap, H + tail] f16 of the local tokens (token-replicated
        exchange): normalised row, top-k global expert ids and weights."""
        torch = _torch()
        t = x.shape[0]
        plan = self.layer._plan
        ws = self._buf("ws", int(lib().moe_workspace_bytes(plan, max(t, 1))))
        send = torch.empty((cap, int(lib().moe_ep_token_row_halves(plan))), dtype=torch.float16,
                           device=x.device)
        check(lib().moe_ep_token_pack(plan, c_void_p(x.data_ptr()), t, cap,
                                      c_void_p(send.data_ptr()), c_void_p(ws.data_ptr()),
                                      ws.numel(), c_void_p(_stream_handle(None))))
        self._T = t
        return send

    def experts_gathered(self, recv: Any) -> Any:
        """fp32 partial sums [rows, H] of this rank's experts over gathered records."""
        torch = _torch()
        rows = recv.shape[0]
        plan = self.layer._plan
        partial = torch.empty((rows, self.cfg.hidden), dtype=torch.float32, device=recv.device)
        ws = self._buf("ws_ep", int(lib().moe_ep_gathered_workspace_bytes(plan, rows)))
        check(lib().moe_ep_experts_gathered(plan, c_void_p(recv.data_ptr()), rows,
                                            c_void_p(partial.data_ptr()), c_void_p(ws.data_ptr()),
                                            ws.numel(), c_void_p(_stream_handle(None))))
        return partial

    def gathered_ids(self, recv: Any) -> Any:
        """Global expert ids [rows, top_k] of gathered token records (-1: unused)."""
        h, k = self.cfg.hidden, self.cfg.top_k
        return recv[:, h:].contiguous().view(_torch().int32)[:, :k]

    def combine_partial(self, x: Any, partial: Any) -> Any:
        torch = _torch()
        out = torch.empty_like(x)
        t = x.shape[0]
        if t == 0:
            return out
        plan = self.layer._plan
        ws = self._ws
        s = c_void_p(_stream_handle(None))
        self._join_shared(x, plan, ws, s)
        check(lib().moe_ep_combine_partial(plan, c_void_p(x.data_ptr()), t,
                                           c_void_p(partial.data_ptr()), c_void_p(out.data_ptr()),
                                           c_void_p(ws.data_ptr()), ws.numel(), s))
        return out

    def _join_shared(self, x: Any, plan: Any, ws: Any, s: Any) -> None:
        """Wait for the shared expert started early, or run it now."""
        torch = _torch()
        if self._shared_done is not None:
            torch.cuda.current_stream(x.device).wait_event(self._shared_done)
            self._shared_done = None
        else:
            check(lib().moe_ep_shared(plan, x.shape[0], c_void_p(ws.data_ptr()), ws.numel(), s))

    def experts(self, rows: Any, expert_ids: Any) -> Any:
        torch = _torch()
        r = rows.shape[0]
        y = torch.empty((r, self.cfg.hidden), dtype=torch.float16, device=rows.device)
        if r == 0:
            return y
        plan = self.layer._plan
        ws = self._buf("ws_ep", int(lib().moe_ep_workspace_bytes(plan, r)))
        check(lib().moe_ep_experts(plan, c_void_p(rows.data_ptr()), c_void_p(expert_ids.data_ptr()),
                                   r, c_void_p(y.data_ptr()), c_void_p(ws.data_ptr()), ws.numel(),
                                   c_void_p(_stream_handle(None))))
        return y

    def start_shared(self, x: Any) -> None:
        """Run the shared expert of the dispatched tokens on a side stream, so that
        it overlaps the row exchange; combine waits for it."""
        torch = _torch()
        t = x.shape[0]
        if t == 0 or self.cfg.shared_inter == 0:
            return
        side = self._pool.get("side")
        if side is None:
            side = self._pool["side"] = torch.cuda.Stream(device=x.device)
        main = torch.cuda.current_stream(x.device)
        side.wait_stream(main)  # after dispatch (its workspace holds the rows)
        ws = self._ws
        check(lib().moe_ep_shared(self.layer._plan, t, c_void_p(ws.data_ptr()), ws.numel(),
                                  c_void_p(side.cuda_stream)))
        self._shared_done = torch.cuda.Event()
        self._shared_done.record(side)

    def combine(self, x: Any, y_back: Any) -> Any:
        torch = _torch()
        out = torch.empty_like(x)
        t = x.shape[0]
        if t == 0:
            return out
        plan = self.layer._plan
        ws = self._ws
        s = c_void_p(_stream_handle(None))
        self._join_shared(x, plan, ws, s)
        check(lib().moe_ep_combine(plan, c_void_p(x.data_ptr()), t, c_void_p(y_back.data_ptr()),
                                   c_void_p(out.data_ptr()), c_void_p(ws.data_ptr()), ws.numel(), s))
        return out

    # ---------------------------------------------------------------- peer memory
    @property
    def rank(self) -> int:
        return self.cfg.expert_begin // self.experts_per_rank

    def p2p_setup(self, cap: int, group: Any = None) -> None:
        """Buffers of the peer-memory exchange for batches of at most `cap` tokens
        (a collective on first use per pool; layers sharing the pool share them)."""
        from .p2p import PeerExchange
        st = self._pool.get("p2p")
        if st is None or st.cap != cap:
            if st is not None:
                raise ValueError("layers sharing a pool must use one peer-exchange capacity")
            st = PeerExchange(self.rank, self.world, cap, self.cfg.hidden,
                              int(lib().moe_ep_token_row_halves(self.layer._plan)),
                              self.cfg.device, group)
            self._pool["p2p"] = st
        st.users += 1
        self._p2p = st
        self._p2p_group = group

    def p2p_pack(self, x: Any, cap: int) -> None:
        """Route the local tokens and store their records into every rank's buffer."""
        st = self._p2p
        st.epoch += 1
        t = x.shape[0]
        plan = self.layer._plan
        ws = self._buf("ws", int(lib().moe_workspace_bytes(plan, max(t, 1))))
        check(lib().moe_ep_p2p_pack(plan, c_void_p(x.data_ptr()), t, cap, self.rank, self.world,
                                    st.recv_arr, st.flags_arr, st.epoch, c_void_p(st.done_ptr),
                                    c_void_p(ws.data_ptr()), ws.numel(),
                                    c_void_p(_stream_handle(None))))
        self._T = t

    def p2p_wait(self, which: int) -> None:
        """Wait (bounded, on the device) until every rank's records (0) or partial
        sums (1) of this forward have arrived."""
        from .p2p import WAIT_LIMIT_CYCLES
        st = self._p2p
        check(lib().moe_ep_p2p_wait(self.layer._plan, c_void_p(st.flags_row(which)), self.world,
                                    st.epoch, WAIT_LIMIT_CYCLES, c_void_p(_stream_handle(None))))

    def p2p_experts(self) -> None:
        """Resident experts on every received record; partial sums to their owners."""
        st = self._p2p
        plan = self.layer._plan
        ws = self._buf("ws_ep", int(lib().moe_ep_gathered_workspace_bytes(plan, self.world * st.cap)))
        check(lib().moe_ep_p2p_experts(plan, c_void_p(st.recv), st.cap, self.rank, self.world,
                                       st.part_arr, st.flags_arr, st.epoch,
                                       c_void_p(st.done_ptr + 4), c_void_p(ws.data_ptr()),
                                       ws.numel(), c_void_p(_stream_handle(None))))

    def p2p_combine(self, x: Any) -> Any:
        torch = _torch()
        out = torch.empty_like(x)
        t = x.shape[0]
        if t == 0:
            return out
        st = self._p2p
        plan = self.layer._plan
        ws = self._ws
        s = c_void_p(_stream_handle(None))
        self._join_shared(x, plan, ws, s)
        check(lib().moe_ep_p2p_combine(plan, c_void_p(x.data_ptr()), t, c_void_p(st.part), st.cap,
                                       self.world, c_void_p(out.data_ptr()), c_void_p(ws.data_ptr()),
                                       ws.numel(), s))
        return out

    def p2p_ids(self) -> Any:
        return self._p2p.recv_ids()[:, :self.cfg.top_k]

    def status(self) -> None:
        self.layer.status()

    def close(self) -> None:
        st = getattr(self, "_p2p", None)
        if st is not None:
            st.users -= 1
            if st.users == 0:
                st.close(self._p2p_group)
                self._pool.pop("p2p", None)
            self._p2p = None
        self.layer.close()
