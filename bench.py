"""MoE-layer benchmark (BASELINE.json metric: MoE-layer tokens/s, % of HBM roofline).

Default workload (N=1): BASELINE config 1 -- GLM-4.7-shape MoE layer (H 5120, 160
routed experts, top-8, I 1536, 1 shared expert of 1536), bf16-valued weights
~N(0,0.02) (stored as f16, lossless), reference softmax-biased routing with
routed_scaling_factor 2.5, decode batches of 1, 8 and 64 tokens; the headline
line is the 64-token batch, T=1 and T=8 are reported under "sub".

One step = one MoE-layer forward over one batch already resident in HBM.
Timing: W warm-up steps, then exactly K steps between CUDA events on the
launching stream, barrier + synchronize on both sides, max over ranks.  The
touched expert weights (>= 425 MB at T=1) are larger than the 126 MB L2, so no
flush is needed between steps.

e2e: the same metric through MoeLayer.host_pipeline (the library's serving-loop
calls over pinned host buffers) with host fp32 activations: every timed step
copies its input H2D, runs the layer (one CUDA graph) and copies its output D2H;
the copies run on H2D / D2H streams and overlap the neighbouring steps' compute, and
the host waits for each step's output.  e2e.serial: MoeLayer.host_runner, one
step at a time (H2D, layer, D2H, synchronise).

--impl reference: the CPU oracle port of the reference executor
(offload_runtime/executors/glm4_moe.py:176-240; same numpy expressions) on the
box's host cores, all BLAS threads, same config, metric and unit.

N > 1 (torchrun): expert parallel -- rank r holds routed experts
[r*160/N, (r+1)*160/N), router and shared expert replicated, 64 tokens per rank
(weak scaling).  Decode batches take by default the token-replicated exchange over
peer memory (each rank's token records and fp32 per-token partial sums stored over
NVLink by the kernels that produce them, epoch flags and bounded device waits, no
NCCL); --ep-exchange gathered: the same exchange as an NCCL all-gather and
reduce-scatter; padded: fixed-capacity all-to-all of f16 rows; exact: counts first,
then exactly the routed rows.  Prefill batches take the exact exchange.

--stack (torchrun, N = 2, 4 or 8): BASELINE config 4 -- 89 GLM-4.7-shape INT8 layers
(seed + layer each, Zipf-skewed routing) resident expert parallel, 160/N experts of
every layer per GPU; a 256-token decode batch and a 16384-token prefill batch split
evenly over the ranks (strong scaling); one JSON line with both workloads.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "disk-mem-off_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

PEAKS_FILE = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_HBM_GBS = 6650.0

GLM = dict(hidden=5120, n_experts=160, top_k=8, inter=1536, shared_inter=1536)


FALLBACK_BF16_TFLOPS = 1590.0


PROFILE_GEMM = os.path.join(os.path.dirname(os.path.abspath(__file__)), "profiles",
                            "moe_gemm_glm47_decode_T64.md")


def _traffic_ratio(kernel: str) -> float | None:
    """DRAM bytes / algorithmic bytes of a grouped GEMM launch, from the committed
    ncu summary (a 32-expert capture of the same kernel; traffic scales with the
    weights streamed, which the algorithmic count tracks)."""
    try:
        with open(PROFILE_GEMM) as f:
            for line in f:
                m = re.match(rf"traffic_ratio_{kernel}\s*=\s*([0-9.]+)", line.strip())
                if m:
                    return float(m.group(1))
    except OSError:
        return None
    return None


def _peaks() -> tuple[float, str]:
    try:
        with open(PEAKS_FILE) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def _tc_peak() -> float:
    try:
        with open(PEAKS_FILE) as f:
            return float(json.load(f)["bf16_tflops"])
    except Exception:
        return FALLBACK_BF16_TFLOPS


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Polls NVML (read-only) while the timed region runs."""

    def __init__(self, device_index: int) -> None:
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._ok = True
        except Exception:
            self._nv = None

    def _run(self) -> None:
        nv = self._nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((mhz, reasons))
            except Exception:
                pass
            time.sleep(0.005)

    def __enter__(self) -> "ClockSampler":
        if self._ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a: object) -> None:
        self._stop.set()
        if self._ok:
            self._t.join()

    def summary(self) -> dict:
        if not self._ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        nv = self._nv
        names = {
            "hw_slowdown": getattr(nv, "nvmlClocksEventReasonHwSlowdown", 0x8),
            "hw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
            "sw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
            "sw_power_cap": getattr(nv, "nvmlClocksEventReasonSwPowerCap", 0x4),
            "hw_power_brake_slowdown": getattr(nv, "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80),
        }
        seen = set()
        for _mhz, r in self.samples:
            for k, bit in names.items():
                if r & bit:
                    seen.add(k)
        mhz = [m for m, _ in self.samples]
        return {"sm_mhz": float(np.median(mhz)) if mhz else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(seen), "samples": len(mhz)}


# ------------------------------------------------------------------ distributed
def _dist_init():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device(f"cuda:{local}"))
    return world, rank, local


def _max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ------------------------------------------------------------------ CPU leg
def cpu_sample(blob, meta, x_np: np.ndarray, budget_s: float = 20.0) -> dict:
    """Time the oracle port of the reference executor on the host cores."""
    from moe_sm100.synthetic import LazyHostTensors
    from oracle.moe_oracle import OracleConfig, moe_block
    cfg = OracleConfig(hidden=GLM["hidden"], n_experts=GLM["n_experts"], top_k=GLM["top_k"],
                       inter=GLM["inter"], shared_inter=GLM["shared_inter"],
                       routed_scaling_factor=2.5, eps=1e-5)
    lazy = LazyHostTensors(blob, meta)
    moe_block(x_np, lazy, cfg)  # warm: fetches the touched experts once (fp32)
    times = []
    t_start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        moe_block(x_np, lazy, cfg)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > budget_s or len(times) >= 10:
            break
    try:
        from threadpoolctl import threadpool_info
        threads = max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    except Exception:
        threads = os.cpu_count() or 1
    med = float(np.median(times))
    return {"value": x_np.shape[0] / med, "unit": "tokens/s", "cores": threads,
            "kind": "port", "seconds_per_step": med, "reps": len(times),
            "sample": f"oracle port of GLM4MoeExecutor._moe_mlp_block (numpy fp32, "
                      f"weights = the bf16 values as fp32), T={x_np.shape[0]} decode batch, "
                      f"{len(times)} reps after 1 warm-up, median"}


# ------------------------------------------------------------------ helpers
def _algorithmic_bytes(ids: np.ndarray, T: int) -> dict:
    H, I, SI, E = GLM["hidden"], GLM["inter"], GLM["shared_inter"], GLM["n_experts"]
    U = len(np.unique(ids))
    w_gateup = (U * 2 * I * H + 2 * SI * H) * 2
    w_down = (U * H * I + H * SI) * 2
    rows = T * GLM["top_k"]
    act_gateup = (rows + T) * H * 2 + (rows * I + T * SI) * 2          # read x rows, write act
    act_down = (rows * I + T * SI) * 2 + (rows + T) * H * 4             # read act, write y
    layer = w_gateup + w_down + E * H * 4 + T * H * 8
    return {"unique_experts": int(U), "gateup": w_gateup + act_gateup,
            "down": w_down + act_down, "layer": layer}


def _make_layer(device: int, seed: int, max_tokens: int):
    import torch
    from moe_sm100 import MoeLayer, MoeLayerConfig
    from moe_sm100.synthetic import SyntheticSpec, build_device_layer
    spec = SyntheticSpec(**GLM, family="glm", expert_dtype="bfloat16", seed=seed)
    blob, meta = build_device_layer(spec, device=f"cuda:{device}")
    cfg = MoeLayerConfig(**GLM, routed_scaling_factor=2.5, rms_norm_eps=1e-5,
                         max_tokens=max_tokens, device=device)
    ml = MoeLayer(cfg)
    ml.bind_device(blob.data_ptr(), blob.numel(), meta)
    torch.cuda.synchronize()
    return ml, blob, meta


def _time_steps(fn, steps: int, warmup: int, world: int) -> float:
    import torch
    for _ in range(warmup):
        fn()
    _barrier(world)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        fn()
    e.record()
    torch.cuda.synchronize()
    _barrier(world)
    return _max_over_ranks(s.elapsed_time(e) / steps, world)


# ------------------------------------------------------------------ other configs
QWEN3 = dict(hidden=2048, n_experts=512, top_k=10, inter=512, shared_inter=512)


def _gemm_flops(T: int, k: int, H: int, I: int, SI: int) -> tuple[float, float]:
    gateup = 2.0 * T * k * 2 * I * H + 2.0 * T * 2 * SI * H
    down = 2.0 * T * k * I * H + 2.0 * T * SI * H
    return gateup, down


def _gemm_bytes(T: int, k: int, H: int, I: int, SI: int, unique: int, wbytes: int
                ) -> tuple[float, float]:
    """Algorithmic HBM bytes of the two grouped GEMMs: the touched experts' weights
    (and the shared expert's) once, the token rows in and the activations / expert
    outputs out (f16), the shared expert's output in fp32."""
    rows, srows = T * k, (T if SI else 0)
    gateup = (unique * 2 * I * H + 2 * SI * H) * wbytes + (rows + srows) * H * 2 \
        + (rows * I + srows * SI) * 2
    down = (unique * H * I + H * SI) * wbytes + (rows * I + srows * SI) * 2 + rows * H * 2 \
        + srows * H * 4
    return float(gateup), float(down)


def _measure(ml, T: int, H: int, steps: int, warmup: int, world: int, gen) -> dict:  # noqa: ANN001
    import torch
    x = torch.randn((T, H), generator=gen, device="cuda")
    out = torch.empty_like(x)
    ws = ml.workspace(T)
    stream = torch.cuda.current_stream().cuda_stream

    def step() -> None:
        ml.forward_ptr(x.data_ptr(), out.data_ptr(), T, ws.data_ptr(), ws.numel(), stream)

    ms = _time_steps(step, steps, warmup, world)
    ml.status()
    stage = np.zeros(4)
    for _ in range(steps):
        stage += np.array(ml.forward_timed(x, out))
    stage /= steps
    ids = ml.route(x)["topk_ids"].cpu().numpy()
    counts = np.bincount(ids.reshape(-1), minlength=ml.cfg.n_experts)
    return {"ms": ms, "stage": stage.tolist(), "unique": int((counts > 0).sum()),
            "max_load": int(counts.max())}


def run_other_configs(args, local: int, world: int, hbm: float, tflops: float) -> dict:  # noqa: ANN001
    """BASELINE config 2 (GLM-4.7 INT8, 4096-token prefill, Zipf routing; the same
    layer also at the 1-64-token decode batches the INT8 target names and at 32 and
    128 tokens, the per-rank decode batches of config 4) and config 3
    (Qwen3-Coder-Next shape, 1-token decode and 8192-token prefill)."""
    import torch
    from moe_sm100 import MoeLayer, MoeLayerConfig
    from moe_sm100.synthetic import SyntheticSpec, build_device_layer
    gen = torch.Generator(device="cuda").manual_seed(2000 + local)
    res: dict = {}
    runs = [
        ("cfg2_glm47_int8_prefill", dict(GLM, family="glm", expert_dtype="int8", seed=4321,
                                         zipf_s=1.1, zipf_amp=1.0),
         dict(weight_format="int8", routed_scaling_factor=2.5, rms_norm_eps=1e-5),
         [1, 8, 32, 64, 128, 4096]),
        ("cfg3_qwen3_next", dict(QWEN3, family="qwen3", expert_dtype="bfloat16", seed=5678),
         dict(use_bias=False, has_shared_gate=True, routed_scaling_factor=1.0,
              rms_norm_eps=1e-6), [1, 8192]),
    ]
    for name, spec_kw, cfg_kw, tokens in runs:
        if args.other_tokens:  # profiling aid: only the listed batch sizes
            keep = {int(v) for v in args.other_tokens.split(",")}
            tokens = [t for t in tokens if t in keep]
            if not tokens:
                continue
        spec = SyntheticSpec(**spec_kw)
        blob, meta = build_device_layer(spec, device=f"cuda:{local}")
        shape = {k: spec_kw[k] for k in ("hidden", "n_experts", "top_k", "inter", "shared_inter")}
        ml = MoeLayer(MoeLayerConfig(**shape, **cfg_kw, max_tokens=max(tokens), device=local))
        ml.bind_device(blob.data_ptr(), blob.numel(), meta)
        torch.cuda.synchronize()
        del blob
        H, I, SI, K = shape["hidden"], shape["inter"], shape["shared_inter"], shape["top_k"]
        wbytes = 1 if cfg_kw.get("weight_format") == "int8" else 2
        for T in tokens:
            steps = max(3, min(args.steps, 20 if T > 1024 else args.steps))
            m = _measure(ml, T, H, steps, args.warmup, world, gen)
            fg, fd = _gemm_flops(T, K, H, I, SI)
            entry = {"tokens_per_s": world * T / (m["ms"] * 1e-3), "ms_per_step": m["ms"],
                     "stage_ms": m["stage"], "unique_experts": m["unique"],
                     "max_expert_load": m["max_load"]}
            if T >= 1024:  # prefill
                entry["tc_frac_gateup"] = fg / (m["stage"][1] * 1e-3) / 1e12 / tflops
                entry["tc_frac_down"] = fd / (m["stage"][2] * 1e-3) / 1e12 / tflops
                entry["tc_frac_layer"] = (fg + fd) / (m["ms"] * 1e-3) / 1e12 / tflops
                entry["tflops_layer"] = (fg + fd) / (m["ms"] * 1e-3) / 1e12
                # each GEMM against the larger of its tensor and HBM floors: with few
                # tokens per expert (Qwen3 shape: ~160) the weights, not the FLOPs, bound it
                bg, bd = _gemm_bytes(T, K, H, I, SI, m["unique"], wbytes)
                for name_, fl, by, st in (("gateup", fg, bg, m["stage"][1]),
                                          ("down", fd, bd, m["stage"][2])):
                    t_tc, t_hbm = fl / (tflops * 1e12), by / (hbm * 1e9)
                    entry[f"roofline_{name_}"] = {
                        "bound": "tensor" if t_tc >= t_hbm else "hbm",
                        "frac": max(t_tc, t_hbm) / (st * 1e-3),
                        "flops": fl, "bytes": by, "launch_ms": st}
            else:  # decode: weight streaming
                wb = (m["unique"] + 1) * 3 * H * I * wbytes
                entry["layer_hbm_frac"] = wb / (m["ms"] * 1e-3) / 1e9 / hbm
            # the INT8 layer at decode sizes (the per-rank batches of BASELINE config 4)
            res[f"{name if T >= 1024 else name.replace('_prefill', '_decode')}_T{T}"] = entry
        ml.close()
        torch.cuda.empty_cache()
    if not args.other_tokens:
        res.update(run_attention(args, local, hbm, tflops))
    return res


GLM_ATTN = dict(hidden=5120, heads=96, kv_heads=8, head_dim=128)


def run_attention(args, local: int, hbm: float, tflops: float) -> dict:  # noqa: ANN001
    """The GLM-4.7-shape attention block on the device (scope row f3: x + o_proj(causal
    GQA attention(rms_norm(x))) over a whole sequence, as GLM4MoeExecutor._attention_block
    computes it): a 64-token and a 4096-token sequence, synthetic bf16-valued weights."""
    import torch
    from moe_sm100.attention import AttentionConfig, AttentionLayer
    from moe_sm100.synthetic import build_device_attention
    H, nh, nkv, hd = (GLM_ATTN[k] for k in ("hidden", "heads", "kv_heads", "head_dim"))
    blob, meta = build_device_attention(H, nh, nkv, hd, seed=99, device=f"cuda:{local}")
    cfg = AttentionConfig(hidden=H, heads=nh, kv_heads=nkv, head_dim=hd, rotary_dim=hd // 2,
                          rope_theta=1_000_000.0, rms_norm_eps=1e-5, max_tokens=4096, device=local)
    al = AttentionLayer(cfg)
    al.bind_device(blob.data_ptr(), blob.numel(), meta)
    torch.cuda.synchronize()
    del blob
    gen = torch.Generator(device="cuda").manual_seed(2500 + local)
    wbytes = ((nh + 2 * nkv) * hd * H + H * nh * hd) * 2
    res = {}
    for T in (64, 4096):
        x = torch.randn((T, H), generator=gen, device="cuda")
        out = torch.empty_like(x)
        steps = max(3, min(args.steps, 20))
        ms = _time_steps(lambda: al.forward(x, out), steps, args.warmup, 1)
        proj = 2.0 * T * H * (nh + 2 * nkv) * hd + 2.0 * T * nh * hd * H
        attn = 2.0 * 2 * nh * hd * T * (T + 1) / 2  # QK^T and PV over the causal half
        res[f"attn_glm47_T{T}"] = {
            "tokens_per_s": T / (ms * 1e-3), "ms_per_step": ms, "seq_len": T,
            "tflops": (proj + attn) / (ms * 1e-3) / 1e12,
            "tc_frac": (proj + attn) / (ms * 1e-3) / 1e12 / tflops,
            "weight_hbm_frac": wbytes / (ms * 1e-3) / 1e9 / hbm}
    al.status()
    al.close()
    torch.cuda.empty_cache()
    return res


# ------------------------------------------------------------------ expert parallel (N > 1)
def _timed_forward(ep, x):  # noqa: ANN001, ANN202
    """One instrumented forward (stage events) whose launches are all queued before
    the device reaches them: a ~2.5 ms spin on the stream first lets the host issue
    the whole forward, so the stage times are device time and not host issue gaps
    (a forward issued onto an idle device runs at the host's launch pace)."""
    import torch
    torch.cuda._sleep(5_000_000)
    return ep.forward(x, timed=True)


def run_ep_qwen3(args, world: int, rank: int, local: int, tflops: float) -> dict:  # noqa: ANN001
    """BASELINE config 3 across the ranks: Qwen3-Next shape, 512/N experts per rank,
    1-token decode and 8192-token prefill per rank (weak scaling)."""
    import torch
    from moe_sm100 import MoeLayerConfig
    from moe_sm100.ep import DeviceEPOps, ExpertParallelMoe
    from moe_sm100.synthetic import SyntheticSpec, build_device_layer
    spec = SyntheticSpec(**QWEN3, family="qwen3", expert_dtype="bfloat16", seed=5678)
    blob, meta = build_device_layer(spec, device=f"cuda:{local}")
    cfg = MoeLayerConfig(**QWEN3, use_bias=False, has_shared_gate=True, routed_scaling_factor=1.0,
                         rms_norm_eps=1e-6, max_tokens=8192, device=local)
    ops = DeviceEPOps(cfg, rank, world)
    ops.bind_device(blob.data_ptr(), blob.numel(), meta)
    torch.cuda.synchronize()
    del blob
    torch.cuda.empty_cache()
    # the 1-token decode uses the fixed-size exchange, the prefill the exact one
    ep = ExpertParallelMoe(ops, **_small_exchange(args, 1))
    gen = torch.Generator(device="cuda").manual_seed(3000 + rank)
    res = {}
    for T in (1, 8192):
        x = torch.randn((T, QWEN3["hidden"]), generator=gen, device="cuda")
        steps = max(3, min(args.steps, 10 if T > 1024 else args.steps))
        ms = _time_steps(lambda: ep.forward(x), steps, args.warmup, world)
        tim = []
        for _ in range(3):
            _timed_forward(ep, x)
            tim.append(ep.last_timing)
        a2a = float(np.median([t["a2a_ms"] for t in tim]))
        tot = float(np.median([t["total_ms"] for t in tim]))
        entry = {"tokens_per_s": world * T / (ms * 1e-3), "ms_per_step": ms,
                 "tokens_per_rank": T, "experts_per_rank": QWEN3["n_experts"] // world,
                 "a2a_frac_of_layer": _max_over_ranks(a2a / tot, world)}
        if T >= 1024:
            fg, fd = _gemm_flops(T, QWEN3["top_k"], QWEN3["hidden"], QWEN3["inter"],
                                 QWEN3["shared_inter"])
            entry["tc_frac_layer_per_gpu"] = (fg + fd) / (ms * 1e-3) / 1e12 / tflops
        res[f"cfg3_qwen3_next_ep{world}_T{T}"] = entry
    ops.status()
    ops.close()
    return res


def run_ep(args, world: int, rank: int, local: int) -> None:  # noqa: ANN001
    """N GPUs: experts sharded 160/N per rank, T tokens per rank, NCCL all-to-all."""
    import torch
    import torch.distributed as dist
    from moe_sm100 import MoeLayerConfig
    from moe_sm100.ep import DeviceEPOps, ExpertParallelMoe
    from moe_sm100.synthetic import SyntheticSpec, build_device_layer
    hbm, peak_kind = _peaks()
    T = args.tokens
    spec = SyntheticSpec(**GLM, family="glm", expert_dtype="bfloat16", seed=1234)
    blob, meta = build_device_layer(spec, device=f"cuda:{local}")
    cfg = MoeLayerConfig(**GLM, routed_scaling_factor=2.5, rms_norm_eps=1e-5, max_tokens=T,
                         device=local)
    ops = DeviceEPOps(cfg, rank, world)
    ops.bind_device(blob.data_ptr(), blob.numel(), meta)
    torch.cuda.synchronize()
    del blob
    torch.cuda.empty_cache()
    ep = ExpertParallelMoe(ops, **_small_exchange(args, T))
    gen = torch.Generator(device="cuda").manual_seed(1000 + rank)
    x = torch.randn((T, GLM["hidden"]), generator=gen, device="cuda")

    with ClockSampler(local) as clk:
        ms = _time_steps(lambda: ep.forward(x), args.steps, args.warmup, world)
    clocks = clk.summary()
    ops.status()
    # one instrumented forward per rank: share of the exchanges in the layer time
    tim = []
    for _ in range(max(3, min(args.steps, 10))):
        _timed_forward(ep, x)
        tim.append(ep.last_timing)
    a2a = float(np.median([t["a2a_ms"] for t in tim]))
    tot = float(np.median([t["total_ms"] for t in tim]))
    a2a_frac = _max_over_ranks(a2a / tot, world)
    recv = int(np.median([t["recv_rows"] for t in tim]))
    # end to end from pinned host memory through ExpertParallelMoe.host_pipeline: every
    # step copies its input H2D, runs the rank's forward and copies the output D2H,
    # the copies on their own streams overlapping the neighbouring steps' compute;
    # and one step at a time (H2D, forward, D2H, synchronise), reported as e2e.serial
    x_host = x.cpu().numpy()
    pipe = ep.host_pipeline(T, depth=2)
    for slot in pipe.x:
        slot.copy_(torch.from_numpy(x_host))
    for i in range(args.warmup):
        pipe.submit(i)
        pipe.wait(i)
    _barrier(world)
    t0 = time.perf_counter()
    for i in range(args.steps):
        pipe.submit(i)
        if i > 0:
            pipe.wait(i - 1)
    pipe.wait(args.steps - 1)
    e2e_s = _max_over_ranks((time.perf_counter() - t0) / args.steps, world)
    pipe.status()
    del pipe
    pin = torch.from_numpy(x_host).pin_memory()
    out_pin = torch.empty_like(pin).pin_memory()

    def e2e_step() -> None:
        xd = pin.to(f"cuda:{local}", non_blocking=True)
        out_pin.copy_(ep.forward(xd), non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for _ in range(args.warmup):
        e2e_step()
    _barrier(world)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    serial_s = _max_over_ranks((time.perf_counter() - t0) / args.steps, world)
    other = {}
    if not args.no_other:
        ops.close()
        del ep, ops
        torch.cuda.empty_cache()
        other = run_ep_qwen3(args, world, rank, local, _tc_peak())
    # expert weight bytes this rank streams per step (its touched local experts + shared)
    e_loc = GLM["n_experts"] // world
    layer_bytes = (min(e_loc, recv) + 1) * 3 * GLM["hidden"] * GLM["inter"] * 2
    frac = layer_bytes / (ms * 1e-3) / 1e9 / hbm
    if rank == 0:
        print(json.dumps({
            "metric": "MoE-layer tokens/s (GLM-4.7-shape decode) and % of HBM roofline",
            "value": world * T / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16 MMA / fp32 accumulate (bf16-valued weights); fp32 routing; "
                     + _exchange_dtype(args.ep_exchange),
            "data": "synthetic (seeded N(0,1) tokens, N(0,0.02) weights, random-init)",
            "config": {"workload": "BASELINE config 1 shape, expert parallel",
                       "tokens_per_rank": T, "experts_per_rank": e_loc,
                       "parallelism": f"ep{world} (" + ("NVLink peer stores" if args.ep_exchange == "p2p" else "NCCL collectives") + " dispatch/combine)",
                       "exchange": _exchange_name(args.ep_exchange),
                       "l2": "inputs larger than L2"},
            "roofline": {"bound": "hbm", "kernel": "whole expert-parallel layer (rank 0)",
                         "achieved": layer_bytes / (ms * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s",
                         "frac": frac, "peak_source": peak_kind, "traffic": None},
            "a2a_frac_of_layer": a2a_frac, "recv_rows_rank0": recv,
            "e2e": {"value": world * T / e2e_s, "unit": "tokens/s",
                    "h2d_bytes_per_step": T * GLM["hidden"] * 4,
                    "d2h_bytes_per_step": T * GLM["hidden"] * 4, "ms_per_step": e2e_s * 1e3,
                    "api": "ExpertParallelMoe.host_pipeline (2 slots, copies overlap compute)",
                    "serial": {"value": world * T / serial_s, "ms_per_step": serial_s * 1e3}},
            "cpu_baseline": None,
            "gpu_launches": _ep_launches(args.ep_exchange) * args.steps,
            "clocks": clocks,
            "other_configs": other,
        }))
    if args.no_other:
        ops.close()
    dist.barrier()
    dist.destroy_process_group()


def _exchange_name(kind: str) -> str:
    return {"padded": "fixed-capacity (one all-to-all of equal row blocks each way, no host sync)",
            "gathered": "token-replicated (all-gather of token records, reduce-scatter of fp32 "
                        "partial sums; no host sync)",
            "p2p": "token-replicated over peer memory (records and fp32 partial sums stored over "
                   "NVLink by the producing kernels, epoch flags, no NCCL)",
            "exact": "exact (counts, then rows and ids; one host sync)"}[kind]


def _exchange_dtype(kind: str) -> str:
    return ("f16 token rows and fp32 partial sums exchanged" if kind in ("gathered", "p2p")
            else "f16 rows exchanged")


def _small_exchange(args, tokens: int) -> dict:  # noqa: ANN001
    """ExpertParallelMoe keywords for batches of at most `tokens` tokens."""
    if args.ep_exchange == "exact":
        return {"padded_tokens": 0}
    return {"padded_tokens": tokens, "small_exchange": args.ep_exchange}


def _ep_launches(kind: str) -> int:
    """Kernels of one expert-parallel decode forward: routing (router, tail) and the
    send rows (dispatch, + send metadata on the exact exchange); hist, scan,
    scatter, gather, two GEMMs (experts; + the partial sums on the gathered
    exchange; + two flag waits on the peer-memory one); scan, two GEMMs (shared); combine."""
    return {"padded": 13, "gathered": 14, "exact": 14, "p2p": 16}[kind]


# ------------------------------------------------------------------ 89-layer stack (N > 1)
def _sum_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def _stack_resident_bytes(e_loc: int, layers: int) -> int:
    """Device bytes one rank keeps resident for the INT8 stack (packed weights,
    fp32 per-row scales, shared expert, norm, fp32 + f16 router, bias)."""
    H, I, SI, E = GLM["hidden"], GLM["inter"], GLM["shared_inter"], GLM["n_experts"]
    per_layer = (e_loc * (3 * H * I + (2 * I + H) * 4) + 3 * SI * H + (2 * SI + H) * 4
                 + H * 4 + E * H * 6 + E * 4)
    return layers * per_layer


def run_stack(args, world: int, rank: int, local: int) -> None:  # noqa: ANN001
    """a stack of GLM-4.7-shape INT8 MoE layers (seed + layer per
    layer, Zipf-skewed routing), resident expert parallel over the ranks (160/N
    experts of every layer per GPU), NCCL all-to-all dispatch and return.  The
    global batch is fixed (256-token decode, 16384-token prefill) and split evenly
    over the ranks: strong scaling."""
    import torch
    import torch.distributed as dist
    from moe_sm100 import MoeLayerConfig
    from moe_sm100.ep import DeviceEPOps, ExpertParallelMoe
    from moe_sm100.synthetic import SyntheticSpec, build_device_layer
    hbm, peak_kind = _peaks()
    tflops = _tc_peak()
    L = args.stack_layers
    H, E, K, I, SI = (GLM[k] for k in ("hidden", "n_experts", "top_k", "inter", "shared_inter"))
    batches = {"decode": args.stack_decode, "prefill": args.stack_prefill}
    head = {"metric": f"{L}-layer MoE stack tokens/s (GLM-4.7 shape, INT8 experts, expert parallel)",
            "unit": "tokens/s", "n_gpus": world, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None,
            "config": {"workload": "BASELINE config 4", "layers": L, "global_tokens": batches,
                       "experts_per_rank": E // world if world else None,
                       "parallelism": f"ep{world} (expert parallel; exchanges below)",
                       "exchange": {"decode": _exchange_name(args.ep_exchange), "prefill": "exact"}}}
    if world < 2 or E % world or any(t % world for t in batches.values()):
        if rank == 0:
            print(json.dumps({**head, "unavailable":
                              "the stack runs expert parallel on 2, 4 or 8 GPUs (160 experts and "
                              "the batches split evenly over the ranks)"}))
        return
    e_loc = E // world
    t_dec, t_pre = batches["decode"] // world, batches["prefill"] // world
    resident = _stack_resident_bytes(e_loc, L)
    # transient: dispatch and expert workspaces, exchanged rows and outputs of the
    # prefill batch (the hottest rank can receive about twice its share)
    transient = 16 * t_pre * K * H * 2 + (4 << 30)
    free, _total = torch.cuda.mem_get_info()
    fits = torch.tensor([1 if resident + transient <= free else 0], device="cuda")
    dist.all_reduce(fits, op=dist.ReduceOp.MIN)
    if int(fits.item()) == 0:
        if rank == 0:
            print(json.dumps({**head, "unavailable":
                              f"resident stack needs {resident / 2**30:.1f} GiB + "
                              f"{transient / 2**30:.1f} GiB transient per GPU; "
                              f"{free / 2**30:.1f} GiB free"}))
        dist.barrier()
        dist.destroy_process_group()
        return

    lo, hi = rank * e_loc, (rank + 1) * e_loc
    pool: dict = {}
    layers = []
    t0 = time.perf_counter()
    for layer in range(L):
        spec = SyntheticSpec(**GLM, family="glm", expert_dtype="int8", seed=args.stack_seed + layer,
                             zipf_s=1.1, zipf_amp=1.0, experts=(lo, hi))
        blob, meta = build_device_layer(spec, device=f"cuda:{local}")
        cfg = MoeLayerConfig(**GLM, weight_format="int8", routed_scaling_factor=2.5,
                             rms_norm_eps=1e-5, max_tokens=t_pre, device=local)
        ops = DeviceEPOps(cfg, rank, world, pool=pool)
        ops.bind_device(blob.data_ptr(), blob.numel(), meta)
        torch.cuda.synchronize()
        del blob
        # decode batches take the fixed-size exchange, prefill the exact one
        layers.append((ops, ExpertParallelMoe(ops, **_small_exchange(args, t_dec))))
    torch.cuda.empty_cache()
    build_s = time.perf_counter() - t0

    def stack(x):  # noqa: ANN001, ANN202
        for _ops, ep in layers:
            x = ep.forward(x)
        return x

    gen = torch.Generator(device="cuda").manual_seed(4000 + rank)
    results = {}
    clocks = None
    for name, t in (("decode", t_dec), ("prefill", t_pre)):
        x = torch.randn((t, H), generator=gen, device="cuda")
        steps = max(3, min(args.steps, 10))
        with ClockSampler(local) as clk:
            ms = _time_steps(lambda: stack(x), steps, args.warmup, world)
        if name == "decode":
            clocks = clk.summary()
        for ops, _ep in layers:
            ops.status()
        # one instrumented pass: exchange share and the experts each rank touched
        a2a = tot = 0.0
        touched = 0
        h = x
        for _ops, ep in layers:
            h = _timed_forward(ep, h)
            a2a += ep.last_timing["a2a_ms"]
            tot += ep.last_timing["total_ms"]
            touched += ep.last_timing["recv_experts"]
        g_tokens = t * world
        entry = {"tokens_per_s": g_tokens / (ms * 1e-3), "ms_per_step": ms,
                 "ms_per_layer": ms / L, "tokens_per_rank": t, "steps": steps,
                 "a2a_frac_of_layer": _max_over_ranks(a2a / tot, world)}
        if name == "decode":
            # INT8 weights (+ fp32 row scales) of the touched local experts and the
            # shared expert, streamed once per layer; mean over the GPUs
            wb = 3 * H * I + (2 * I + H) * 4
            rank_bytes = (touched + L) * wb
            achieved = _sum_over_ranks(rank_bytes, world) / world / (ms * 1e-3) / 1e9
            entry["roofline"] = {"bound": "hbm", "achieved": achieved, "peak": hbm,
                                 "unit": "GB/s", "frac": achieved / hbm, "peak_source": peak_kind,
                                 "per": "GPU (mean), expert weights of the stack"}
            entry["touched_local_experts_per_layer_rank0"] = touched / L
        else:
            fg, fd = _gemm_flops(g_tokens, K, H, I, SI)
            achieved = (fg + fd) * L / world / (ms * 1e-3) / 1e12
            entry["roofline"] = {"bound": "tensor", "achieved": achieved, "peak": tflops,
                                 "unit": "TFLOP/s", "frac": achieved / tflops,
                                 "peak_source": "MEASURED_PEAKS.json bf16 burst",
                                 "per": "GPU (mean), expert + shared GEMMs of the stack"}
        results[f"{name}_T{g_tokens}"] = entry
    if rank == 0:
        print(json.dumps({**head, "value": results[f"decode_T{batches['decode']}"]["tokens_per_s"],
                          "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": results[f"decode_T{batches['decode']}"]["ms_per_step"],
                          "dtype": "INT8 weights widened to f16 in shared memory, f16 MMA / fp32 "
                                   "accumulate; fp32 routing; " + _exchange_dtype(args.ep_exchange),
                          "data": "synthetic (seeded N(0,1) tokens; per-layer seeded N(0,0.02) "
                                  "weights quantised per row; Zipf(1.1) router bias)",
                          "resident_gib_per_gpu": resident / 2**30, "build_s": build_s,
                          "workloads": results, "clocks": clocks,
                          "gpu_launches_per_layer": {
                              "decode": _ep_launches(args.ep_exchange),
                              "prefill": 20}}))
    for ops, _ep in layers:
        ops.close()
    dist.barrier()
    dist.destroy_process_group()


# ------------------------------------------------------------------ arms
def _decode_batches(t_main: int, seed: int, with_sub: bool) -> dict:
    """The seeded input batches of the config-1 lines, drawn in a fixed order
    (T = 1, 8, then the headline batch) so both arms time the same tokens."""
    import torch
    gen = torch.Generator(device="cuda").manual_seed(seed)
    out = {}
    for T in (sorted({1, 8, t_main}) if with_sub else [t_main]):
        out[T] = torch.randn((T, GLM["hidden"]), generator=gen, device="cuda")
    return out


def _config1(t_main: int, world: int) -> dict:
    return {"workload": "BASELINE config 1: GLM-4.7-shape MoE layer, bf16 decode",
            "tokens_per_rank": t_main, "hidden": GLM["hidden"], "experts": GLM["n_experts"],
            "top_k": GLM["top_k"], "moe_intermediate": GLM["inter"],
            "shared_intermediate": GLM["shared_inter"],
            "routing": "reference softmax(logits+bias), scale 2.5",
            "parallelism": "replicas" if world > 1 else "single",
            "l2": "inputs larger than L2 (touched weights >= 425 MB)"}


def run_ours(args) -> None:  # noqa: ANN001
    import torch
    world, rank, local = _dist_init()
    torch.cuda.set_device(local)
    if args.stack:
        run_stack(args, world, rank, local)
        return
    if world > 1:
        run_ep(args, world, rank, local)
        return
    if args.only_attention:  # profiling aid: the attention block only
        print(json.dumps({"attention": run_attention(args, local, _peaks()[0], _tc_peak())}))
        return
    if args.only_other:  # profiling aid: BASELINE configs 2 and 3 only
        print(json.dumps({"other_configs": run_other_configs(args, local, world, _peaks()[0],
                                                              _tc_peak())}))
        return
    hbm, peak_kind = _peaks()
    T_main = args.tokens
    ml, blob, meta = _make_layer(local, seed=1234, max_tokens=max(64, T_main))

    results = {}
    for T, x in _decode_batches(T_main, 1000 + rank, not args.no_sub).items():
        out = torch.empty_like(x)
        ws = ml.workspace(T)
        stream = torch.cuda.current_stream().cuda_stream

        def step() -> None:
            ml.forward_ptr(x.data_ptr(), out.data_ptr(), T, ws.data_ptr(), ws.numel(), stream)

        if T == T_main:
            with ClockSampler(local) as clk:
                ms = _time_steps(step, args.steps, args.warmup, world)
            clocks = clk.summary()
        else:
            ms = _time_steps(step, args.steps, args.warmup, world)
        ml.status()
        # per-stage device times (events between the launches of one forward)
        stage = np.zeros(4)
        for _ in range(args.steps):
            stage += np.array(ml.forward_timed(x, out))
        stage /= args.steps
        ids = ml.route(x)["topk_ids"].cpu().numpy()
        ab = _algorithmic_bytes(ids, T)
        results[T] = dict(ms=ms, stage=stage.tolist(), bytes=ab, x=x)

    main = results[T_main]
    ms = main["ms"]
    stage = main["stage"]
    ab = main["bytes"]
    gate_gbs = ab["gateup"] / (stage[1] * 1e-3) / 1e9
    down_gbs = ab["down"] / (stage[2] * 1e-3) / 1e9
    layer_gbs = ab["layer"] / (ms * 1e-3) / 1e9

    # end to end from pinned host memory through the serving-loop calls: every step
    # copies its input to the device, runs the layer and copies its output back.
    # MoeLayer.host_pipeline (the headline e2e): two slots, each step's copies on
    # H2D / D2H streams overlapping the neighbouring steps' compute, the host waiting for
    # step i - 1's output after submitting step i, and for the last one at the end.
    # MoeLayer.host_runner (reported beside it): one step at a time, synchronised.
    x_host = main["x"].cpu().numpy()
    e2e_s = serial_s = float("nan")
    if not args.no_e2e:
        pipe = ml.host_pipeline(T_main, depth=2)
        for slot in pipe.x:
            slot.copy_(torch.from_numpy(x_host))
        for i in range(args.warmup):
            pipe.submit(i)
            pipe.wait(i)
        _barrier(world)
        t0 = time.perf_counter()
        for i in range(args.steps):
            pipe.submit(i)
            if i > 0:
                pipe.wait(i - 1)
        pipe.wait(args.steps - 1)
        e2e_s = _max_over_ranks((time.perf_counter() - t0) / args.steps, world)
        pipe.status()
        del pipe
        x_pin = torch.from_numpy(x_host).pin_memory()
        out_pin = torch.empty_like(x_pin).pin_memory()
        runner = ml.host_runner(x_pin, out_pin)
        for _ in range(args.warmup):
            runner()
        _barrier(world)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            runner()
        serial_s = _max_over_ranks((time.perf_counter() - t0) / args.steps, world)
        del runner

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_sample(blob, meta, x_host)
    other = {}
    if not args.no_sub and not args.no_other:
        ml.close()
        del blob
        torch.cuda.empty_cache()
        other = run_other_configs(args, local, world, hbm, _tc_peak())

    sub = {}
    for T, r in results.items():
        if T == T_main:
            continue
        b = r["bytes"]
        sub[f"T{T}"] = {
            "tokens_per_s": world * T / (r["ms"] * 1e-3), "ms_per_step": r["ms"],
            "stage_ms": r["stage"], "unique_experts": b["unique_experts"],
            "layer_hbm_frac": b["layer"] / (r["ms"] * 1e-3) / 1e9 / hbm,
            "gateup_hbm_frac": b["gateup"] / (r["stage"][1] * 1e-3) / 1e9 / hbm,
        }
    if rank == 0:
        line = {
            "metric": "MoE-layer tokens/s (GLM-4.7-shape decode) and % of HBM roofline",
            "value": world * T_main / (ms * 1e-3),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f16 MMA / fp32 accumulate (bf16-valued weights); fp32 routing",
            "data": "synthetic (seeded N(0,1) tokens, N(0,0.02) weights, random-init)",
            "config": _config1(T_main, world),
            "roofline": {"bound": "hbm", "kernel": "moe_gemm_kernel gate/up (swap-AB tcgen05)",
                         "achieved": gate_gbs, "peak": hbm, "unit": "GB/s",
                         "frac": gate_gbs / hbm, "peak_source": peak_kind,
                         "traffic": (_traffic_ratio("gateup") * ab["gateup"]
                                     if _traffic_ratio("gateup") else None),
                         "traffic_source": "profiles/moe_gemm_glm47_decode_T64.md: "
                                           "dram bytes / algorithmic bytes of an ncu capture "
                                           "(32 experts), times this launch's algorithmic bytes",
                         "algorithmic_bytes_per_launch": ab["gateup"],
                         "launch_ms": stage[1]},
            "roofline_down": {"achieved": down_gbs, "frac": down_gbs / hbm,
                              "traffic": (_traffic_ratio("down") * ab["down"]
                                          if _traffic_ratio("down") else None),
                              "algorithmic_bytes_per_launch": ab["down"], "launch_ms": stage[2]},
            "roofline_layer": {"achieved": layer_gbs, "frac": layer_gbs / hbm,
                               "algorithmic_bytes_per_step": ab["layer"],
                               "unique_experts": ab["unique_experts"]},
            "stage_ms": {"route": stage[0], "gemm_gateup": stage[1], "gemm_down": stage[2],
                         "combine": stage[3]},
            "e2e": {"value": world * T_main / e2e_s, "unit": "tokens/s",
                    "h2d_bytes_per_step": T_main * GLM["hidden"] * 4,
                    "d2h_bytes_per_step": T_main * GLM["hidden"] * 4,
                    "ms_per_step": e2e_s * 1e3,
                    "api": "MoeLayer.host_pipeline (2 slots, copies overlap compute)",
                    "serial": {"value": world * T_main / serial_s, "ms_per_step": serial_s * 1e3,
                               "api": "MoeLayer.host_runner (one step at a time)"}},
            "cpu_baseline": cpu,
            # our kernels per forward: router, decode tail, dispatch, two grouped
            # GEMMs, combine (T <= 256); prefill: prep, router GEMM, candidates,
            # fp32 recompute, final selection, histogram, scan, scatter, gather,
            # two grouped GEMMs, combine
            "gpu_launches": (6 if T_main <= 256 else 12) * args.steps,
            "clocks": clocks,
            "sub": sub,
            "other_configs": other,
        }
        print(json.dumps(line))
    ml.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_reference(args) -> None:  # noqa: ANN001
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import torch
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    from moe_sm100.synthetic import LazyHostTensors, SyntheticSpec, build_device_layer
    from oracle.moe_oracle import OracleConfig, moe_block
    spec = SyntheticSpec(**GLM, family="glm", expert_dtype="bfloat16", seed=1234)
    blob, meta = build_device_layer(spec, device=f"cuda:{local}")
    T = args.tokens
    # the same tokens the GPU arm times for its headline line (rank 0's batches)
    x = _decode_batches(T, 1000, not args.no_sub)[T].cpu().numpy()
    cfg = OracleConfig(hidden=5120, n_experts=160, top_k=8, inter=1536, shared_inter=1536,
                       routed_scaling_factor=2.5, eps=1e-5)
    # every host thread this process may use: torchrun sets OMP_NUM_THREADS=1 for its
    # ranks, and rank 0 runs the reference alone (the others have returned)
    try:
        from threadpoolctl import threadpool_limits
        _blas = threadpool_limits(limits=len(os.sched_getaffinity(0)) or os.cpu_count() or 1)
    except Exception:
        _blas = None
    lazy = LazyHostTensors(blob, meta)
    moe_block(x, lazy, cfg)  # fetch touched experts to host once (not timed)
    for _ in range(max(0, args.warmup - 1)):
        moe_block(x, lazy, cfg)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        moe_block(x, lazy, cfg)
    sec = (time.perf_counter() - t0) / args.steps
    try:
        from threadpoolctl import threadpool_info
        threads = max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    except Exception:
        threads = os.cpu_count() or 1
    value = T / sec
    print(json.dumps({
        "impl": "reference",
        "metric": "MoE-layer tokens/s (GLM-4.7-shape decode) and % of HBM roofline",
        "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (numpy)",
        "data": "synthetic (same seeds as the GPU arm)",
        "config": _config1(T, 1),
        "reference_run": "host cores, rank 0 only",
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"oracle port of GLM4MoeExecutor._moe_mlp_block, T={T}, "
                                   f"{args.steps} steps after {args.warmup} warm-up"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-sub", action="store_true", help="only the --tokens batch (no T=1/8 lines)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end timing")
    ap.add_argument("--only-other", action="store_true",
                    help="only BASELINE configs 2 and 3 (profiling aid)")
    ap.add_argument("--only-attention", action="store_true",
                    help="only the GLM-4.7-shape attention block (profiling aid)")
    ap.add_argument("--other-tokens", default="",
                    help="comma-separated batch sizes: run configs 2 and 3 only at these")
    ap.add_argument("--no-other", action="store_true",
                    help="skip BASELINE configs 2 and 3 (INT8 prefill, Qwen3 shape)")
    ap.add_argument("--experts", type=int, default=160,
                    help="routed experts (profiling uses fewer to stay within a few GB)")
    ap.add_argument("--ep-exchange", choices=["padded", "gathered", "p2p", "exact"], default="p2p",
                    help="N > 1 decode batches: fixed-capacity all-to-all, token-replicated "
                         "all-gather/reduce-scatter, or exact all-to-all")
    ap.add_argument("--stack", action="store_true",
                    help="BASELINE config 4: resident INT8 layer stack, expert parallel (N >= 2)")
    ap.add_argument("--stack-layers", type=int, default=89)
    ap.add_argument("--stack-seed", type=int, default=7000)
    ap.add_argument("--stack-decode", type=int, default=256, help="global decode batch")
    ap.add_argument("--stack-prefill", type=int, default=16384, help="global prefill batch")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    GLM["n_experts"] = args.experts
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
