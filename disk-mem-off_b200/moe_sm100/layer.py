"""One HBM-resident MoE layer behind the libmoe_sm100 C ABI.

PyTorch is used only for device/pinned buffers and the current CUDA stream;
all compute is the library's sm_100a kernels.  ``MoeLayer.forward`` is the
device-side equivalent of ``_moe_mlp_block`` (glm4_moe.py:176-240,
qwen3_next.py:273-333) on a bound layer.
"""
from __future__ import annotations

import ctypes
from ctypes import byref, c_void_p
from typing import Any, Iterable

import numpy as np

from . import _lib
from ._lib import check, lib
from .config import MoeLayerConfig

_NP_DTYPE_NAMES = {
    "float32": "float32", "<f4": "float32", "float16": "float16", "<f2": "float16",
    "bfloat16": "bfloat16", "int8": "int8", "|i1": "int8",
}


def _torch():
    import torch  # deferred: tensor handles only
    return torch


def _stream_handle(stream: Any) -> int:
    if stream is None:
        return _torch().cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    if hasattr(stream, "cuda_stream"):
        return stream.cuda_stream
    if isinstance(stream, c_void_p):
        return stream.value or 0
    return int(stream)


def _descs(tensor_meta: Iterable[dict[str, Any]]) -> tuple[Any, list[bytes]]:
    metas = list(tensor_meta)
    arr = (_lib.MoeTensorDescC * len(metas))()
    keep: list[bytes] = []
    for i, m in enumerate(metas):
        name = str(m["name"]).encode()
        dt = _NP_DTYPE_NAMES.get(str(m["dtype"]), str(m["dtype"])).encode()
        keep += [name, dt]
        shape = list(m["shape"])
        if len(shape) == 0 or len(shape) > 2:
            # scalars / higher-rank tensors are never MoE tensors; describe them as 1-D
            shape = [int(np.prod(shape)) if shape else 1]
        arr[i].name = name
        arr[i].dtype = dt
        arr[i].shape[0] = int(shape[0])
        arr[i].shape[1] = int(shape[1]) if len(shape) == 2 else 1
        arr[i].ndim = len(shape)
        arr[i].offset = int(m["offset"])
        arr[i].nbytes = int(m["nbytes"])
    return arr, keep


class MoeLayer:
    """A plan + the packed, resident weights of one MoE layer."""

    def __init__(self, cfg: MoeLayerConfig) -> None:
        self.cfg = cfg
        plan = c_void_p()
        check(lib().moe_plan_create(byref(cfg.to_c()), byref(plan)))
        self._plan = plan
        self._ws: Any = None
        self._pinned: dict[str, Any] = {}

    # -- lifetime ---------------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_plan", None) is not None and self._plan.value:
            lib().moe_plan_destroy(self._plan)
            self._plan = c_void_p()
        self._ws = None

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    # -- binding ----------------------------------------------------------------
    def bind_device(self, blob_ptr: int, blob_bytes: int, tensor_meta: Iterable[dict[str, Any]],
                    stream: Any = None) -> None:
        """Pack the MoE tensors of a layer blob that is already in device memory."""
        descs, keep = _descs(tensor_meta)
        check(lib().moe_bind_layer(self._plan, c_void_p(int(blob_ptr)), int(blob_bytes), descs,
                                   len(descs), c_void_p(_stream_handle(stream))))
        del keep

    def bind_host(self, blob: Any, tensor_meta: Iterable[dict[str, Any]], stream: Any = None) -> None:
        """Copy a host blob to the device, pack it, and drop the staging copy."""
        torch = _torch()
        mv = memoryview(blob).cast("B")
        src = torch.frombuffer(mv, dtype=torch.uint8) if mv.nbytes else torch.empty(0, dtype=torch.uint8)
        dev = torch.empty(mv.nbytes, dtype=torch.uint8, device=f"cuda:{self.cfg.device}")
        dev.copy_(src)
        self.bind_device(dev.data_ptr(), mv.nbytes, tensor_meta, stream)
        _torch().cuda.current_stream().synchronize()
        del dev

    @property
    def weight_bytes(self) -> int:
        return int(lib().moe_plan_weight_bytes(self._plan))

    # -- compute ----------------------------------------------------------------
    def workspace_bytes(self, tokens: int) -> int:
        return int(lib().moe_workspace_bytes(self._plan, int(tokens)))

    def workspace(self, tokens: int) -> Any:
        need = self.workspace_bytes(tokens)
        if self._ws is None or self._ws.numel() < need:
            torch = _torch()
            self._ws = torch.empty(max(need, 256), dtype=torch.uint8, device=f"cuda:{self.cfg.device}")
        return self._ws

    def forward_ptr(self, x_ptr: int, out_ptr: int, tokens: int, ws_ptr: int, ws_bytes: int,
                    stream: Any = None) -> None:
        check(lib().moe_forward(self._plan, c_void_p(x_ptr), c_void_p(out_ptr), int(tokens),
                                c_void_p(ws_ptr), int(ws_bytes), c_void_p(_stream_handle(stream))))

    def forward_timed(self, x: Any, out: Any, stream: Any = None) -> list[float]:
        """Forward on CUDA tensors; returns device ms for [route, gate/up GEMM, down GEMM, combine]."""
        t = x.shape[0]
        ws = self.workspace(max(t, 1))
        ms = (ctypes.c_float * 4)()
        check(lib().moe_forward_timed(self._plan, c_void_p(x.data_ptr()), c_void_p(out.data_ptr()), t,
                                      c_void_p(ws.data_ptr()), ws.numel(), ms,
                                      c_void_p(_stream_handle(stream))))
        return [float(v) for v in ms]

    def forward(self, x: Any, out: Any = None, stream: Any = None) -> Any:
        """``x + MoE(x)`` for a CUDA fp32 tensor ``x`` of shape [T, H]."""
        torch = _torch()
        if not (isinstance(x, torch.Tensor) and x.is_cuda and x.dtype == torch.float32):
            raise TypeError("MoeLayer.forward expects a CUDA float32 tensor")
        if x.dim() != 2 or x.shape[1] != self.cfg.hidden:
            raise ValueError(f"x must be [T, {self.cfg.hidden}]")
        x = x.contiguous()
        if out is None:
            out = torch.empty_like(x)
        t = x.shape[0]
        if t == 0:
            return out
        ws = self.workspace(t)
        self.forward_ptr(x.data_ptr(), out.data_ptr(), t, ws.data_ptr(), ws.numel(), stream)
        return out

    def forward_host(self, x: Any, stream: Any = None, out: Any = None) -> Any:
        """Host fp32 in, host fp32 out: H2D, device forward, D2H (end-to-end path).

        ``x`` is a numpy array (staged through the layer's pinned buffers and
        answered with a new numpy array) or a pinned CPU torch tensor, which is
        copied to the device directly; the result then goes to ``out`` (a pinned
        CPU tensor of the same shape, allocated when omitted)."""
        torch = _torch()
        pinned_in = isinstance(x, torch.Tensor)
        if pinned_in:
            if x.device.type != "cpu" or x.dtype != torch.float32 or not x.is_contiguous():
                raise ValueError("x must be a contiguous fp32 CPU tensor")
            t, h = x.shape
        else:
            x = np.ascontiguousarray(x, dtype=np.float32)
            t, h = x.shape
        if h != self.cfg.hidden:
            raise ValueError(f"x must be [T, {self.cfg.hidden}]")
        if t == 0:
            return x.clone() if pinned_in else x.copy()
        pin_in, pin_out, dev_in, dev_out = self._staging(t)
        if pinned_in:
            src = x
            dst = out if out is not None else torch.empty((t, h), dtype=torch.float32,
                                                          pin_memory=True)
            if dst.shape != (t, h) or dst.dtype != torch.float32 or dst.device.type != "cpu":
                raise ValueError("out must be a [T, H] fp32 CPU tensor")
        else:
            np.copyto(pin_in[:t].numpy(), x)
            src, dst = pin_in[:t], pin_out[:t]
        s = torch.cuda.current_stream(self.cfg.device) if stream is None else stream
        dev_in[:t].copy_(src, non_blocking=True)
        ws = self.workspace(t)
        self.forward_ptr(dev_in.data_ptr(), dev_out.data_ptr(), t, ws.data_ptr(), ws.numel(), s)
        dst.copy_(dev_out[:t], non_blocking=True)
        s.synchronize()
        return dst if pinned_in else dst.numpy().copy()

    def host_runner(self, x_pinned: Any, out_pinned: Any) -> "HostRunner":
        """A reusable end-to-end step over fixed pinned host buffers (see HostRunner)."""
        return HostRunner(self, x_pinned, out_pinned)

    def host_pipeline(self, tokens: int, depth: int = 2) -> "HostPipeline":
        """Steps from pinned host memory with their copies overlapping the neighbouring
        steps' compute (see HostPipeline); each slot's layer step is one CUDA graph."""
        torch = _torch()
        if not 0 < tokens <= self.cfg.max_tokens:
            raise ValueError("tokens outside (0, max_tokens]")
        dev = torch.device(f"cuda:{self.cfg.device}")
        ws = torch.empty(max(self.workspace_bytes(tokens), 256), dtype=torch.uint8, device=dev)

        def step(din: Any, dout: Any) -> None:  # the slots share ws: steps run in order
            self.forward_ptr(din.data_ptr(), dout.data_ptr(), tokens, ws.data_ptr(), ws.numel())
        return HostPipeline(step, tokens, self.cfg.hidden, self.cfg.device, depth, graph=True,
                            check=self.status, keep=(ws,))

    def _staging(self, tokens: int) -> tuple[Any, Any, Any, Any]:
        torch = _torch()
        cap = self._pinned.get("cap", 0)
        if cap < tokens:
            h = self.cfg.hidden
            dev = f"cuda:{self.cfg.device}"
            self._pinned = {
                "cap": tokens,
                "in": torch.empty((tokens, h), dtype=torch.float32, pin_memory=True),
                "out": torch.empty((tokens, h), dtype=torch.float32, pin_memory=True),
                "din": torch.empty((tokens, h), dtype=torch.float32, device=dev),
                "dout": torch.empty((tokens, h), dtype=torch.float32, device=dev),
            }
        p = self._pinned
        return p["in"], p["out"], p["din"], p["dout"]

    def route(self, x: Any, stream: Any = None) -> dict[str, Any]:
        """Router + permutation only: topk_ids, topk_w, expert_offsets, perm (CUDA tensors)."""
        torch = _torch()
        x = x.contiguous()
        t = x.shape[0]
        k, e = self.cfg.top_k, self.cfg.n_experts
        dev = x.device
        ids = torch.empty((t, k), dtype=torch.int32, device=dev)
        w = torch.empty((t, k), dtype=torch.float32, device=dev)
        offs = torch.empty(e + 1, dtype=torch.int32, device=dev)
        perm = torch.empty(t * k, dtype=torch.int32, device=dev)
        if t > 0:
            ws = self.workspace(t)
            check(lib().moe_route(self._plan, c_void_p(x.data_ptr()), t, c_void_p(ids.data_ptr()),
                                  c_void_p(w.data_ptr()), c_void_p(offs.data_ptr()),
                                  c_void_p(perm.data_ptr()), c_void_p(ws.data_ptr()), ws.numel(),
                                  c_void_p(_stream_handle(stream))))
        else:
            offs.zero_()
        return {"topk_ids": ids, "topk_w": w, "expert_offsets": offs, "perm": perm}

    def status(self, stream: Any = None) -> None:
        """Synchronise and raise if a kernel reported a device-side error or timeout."""
        check(lib().moe_status(self._plan, c_void_p(_stream_handle(stream))))


def layer_shapes(tensor_meta: Iterable[dict[str, Any]]) -> dict[str, Any]:
    """Derive ``inter`` / ``shared_inter`` / shared-gate presence from layer metadata."""
    inter = shared = 0
    gate = False
    for m in tensor_meta:
        n = str(m["name"])
        if n.endswith("mlp.experts.0.gate_proj.weight"):
            inter = int(m["shape"][0])
        elif n.endswith(("mlp.shared_experts.gate_proj.weight", "mlp.shared_expert.gate_proj.weight")):
            shared = int(m["shape"][0])
        elif n.endswith("mlp.shared_expert_gate.weight"):
            gate = True
    return {"inter": inter, "shared_inter": shared, "has_shared_gate": gate}


class HostRunner:
    """One layer step from pinned host memory, for serving loops with fixed buffers.

    The step -- copy ``x_pinned`` to the device, ``moe_forward``, copy the result
    into ``out_pinned`` -- is captured once as a CUDA graph and replayed by each
    call, so a step costs one graph launch on the host instead of a dozen API
    calls.  The caller refills ``x_pinned`` before a call and reads
    ``out_pinned`` after it; the runner owns its device buffers and workspace.
    Capture needs one uncaptured warm-up step, which the constructor runs.
    """

    def __init__(self, layer: MoeLayer, x_pinned: Any, out_pinned: Any) -> None:
        torch = _torch()
        for name, tnsr in (("x_pinned", x_pinned), ("out_pinned", out_pinned)):
            if not (isinstance(tnsr, torch.Tensor) and tnsr.device.type == "cpu"
                    and tnsr.dtype == torch.float32 and tnsr.is_contiguous() and tnsr.is_pinned()):
                raise ValueError(f"{name} must be a contiguous pinned fp32 CPU tensor")
        if x_pinned.dim() != 2 or x_pinned.shape[1] != layer.cfg.hidden:
            raise ValueError(f"x_pinned must be [T, {layer.cfg.hidden}]")
        if out_pinned.shape != x_pinned.shape:
            raise ValueError("out_pinned must have the shape of x_pinned")
        t = x_pinned.shape[0]
        if not 0 < t <= layer.cfg.max_tokens:
            raise ValueError("T outside (0, max_tokens]")
        dev = torch.device(f"cuda:{layer.cfg.device}")
        self.layer, self.x, self.out = layer, x_pinned, out_pinned
        self._din = torch.empty_like(x_pinned, device=dev)
        self._dout = torch.empty_like(x_pinned, device=dev)
        self._ws = torch.empty(max(layer.workspace_bytes(t), 256), dtype=torch.uint8, device=dev)
        stream = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(stream):
            self._step()
        stream.synchronize()
        layer.status(stream)
        self._graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._graph, stream=stream):
            self._step()
        torch.cuda.current_stream(dev).synchronize()

    def _step(self) -> None:
        t = self.x.shape[0]
        self._din.copy_(self.x, non_blocking=True)
        self.layer.forward_ptr(self._din.data_ptr(), self._dout.data_ptr(), t, self._ws.data_ptr(),
                               self._ws.numel())
        self.out.copy_(self._dout, non_blocking=True)

    def __call__(self) -> Any:
        """Run one step and wait for it; returns ``out_pinned``."""
        torch = _torch()
        self._graph.replay()
        torch.cuda.current_stream(self._din.device).synchronize()
        return self.out


class HostPipeline:
    """Layer steps from pinned host memory, copies overlapped with compute.

    A serving loop that submits one batch per step: ``depth`` slots, each with its
    own pinned input / output buffers (``x[s]``, ``out[s]``) and device copies.
    ``submit(i)`` queues step i on slot ``i % depth``: the input copy on an H2D
    stream, the layer step (``step(din, dout)`` on a compute stream; with
    ``graph=True`` one CUDA graph per slot, captured at construction after one
    uncaptured run) once that copy lands, and the output copy on a D2H stream once
    the layer finishes.  ``wait(i)`` blocks until step i's output is in
    ``out[i % depth]``.  So while step i computes, step i + 1's input and step
    i - 1's output cross PCIe (in opposite directions).  A slot's device input is
    refilled only after the layer that read it finished, and its device output
    rewritten only after the copy that read it finished.  The caller fills
    ``x[s]`` for step i only after ``wait(i - depth)`` returned (or before the
    first ``depth`` submits) and reads ``out[s]`` after ``wait(i)``.  Steps compute
    one after another on the compute stream, so they may share a workspace.
    """

    def __init__(self, step: Any, tokens: int, hidden: int, device: int, depth: int = 2,
                 graph: bool = True, check: Any = None, keep: tuple = ()) -> None:
        torch = _torch()
        if tokens <= 0 or depth < 1:
            raise ValueError("tokens and depth must be positive")
        dev = torch.device(f"cuda:{device}")
        self.tokens, self.depth = tokens, depth
        self._step, self._check, self._keep = step, check, keep
        self.x = [torch.zeros((tokens, hidden), dtype=torch.float32, pin_memory=True)
                  for _ in range(depth)]
        self.out = [torch.empty((tokens, hidden), dtype=torch.float32, pin_memory=True)
                    for _ in range(depth)]
        self._din = [torch.zeros((tokens, hidden), dtype=torch.float32, device=dev)
                     for _ in range(depth)]
        self._dout = [torch.empty((tokens, hidden), dtype=torch.float32, device=dev)
                      for _ in range(depth)]
        self._h2d = torch.cuda.Stream(device=dev)
        self._d2h = torch.cuda.Stream(device=dev)
        self._comp = torch.cuda.Stream(device=dev)
        self._ev_in = [torch.cuda.Event() for _ in range(depth)]
        self._ev_out = [torch.cuda.Event() for _ in range(depth)]
        self._ev_done = [torch.cuda.Event() for _ in range(depth)]
        self._graphs = []
        if graph:
            for s in range(depth):  # one uncaptured step per slot, then its graph
                with torch.cuda.stream(self._comp):
                    step(self._din[s], self._dout[s])
                self._comp.synchronize()
                self.status()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=self._comp):
                    step(self._din[s], self._dout[s])
                self._graphs.append(g)
        torch.cuda.synchronize(dev)

    def submit(self, step: int) -> None:
        """Queue step ``step`` (input from ``x[step % depth]``); returns at once."""
        torch = _torch()
        s = step % self.depth
        self._h2d.wait_event(self._ev_out[s])  # the slot's previous layer read its input
        with torch.cuda.stream(self._h2d):
            self._din[s].copy_(self.x[s], non_blocking=True)
            self._ev_in[s].record(self._h2d)
        self._comp.wait_event(self._ev_in[s])
        self._comp.wait_event(self._ev_done[s])  # the slot's previous output was copied out
        with torch.cuda.stream(self._comp):
            if self._graphs:
                self._graphs[s].replay()
            else:
                self._step(self._din[s], self._dout[s])
        self._ev_out[s].record(self._comp)
        self._d2h.wait_event(self._ev_out[s])
        with torch.cuda.stream(self._d2h):
            self.out[s].copy_(self._dout[s], non_blocking=True)
            self._ev_done[s].record(self._d2h)

    def wait(self, step: int) -> Any:
        """Block until step ``step``'s output is in ``out[step % depth]``; returns it."""
        s = step % self.depth
        self._ev_done[s].synchronize()
        return self.out[s]

    def status(self) -> None:
        """Synchronise and raise if a kernel reported a device-side error or timeout."""
        self._comp.synchronize()
        if self._check is not None:
            self._check()
