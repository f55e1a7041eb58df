"""Generate the golden MoE fixtures under tests/golden/ from the reference itself.

Run in a container where the disk-mem-off reference is importable:

    python tests/golden/make_golden.py --reference /path/to/disk-mem-off

For every case in ``oracle.cases.GOLDEN_SPECS`` it builds the seeded inputs, runs the
reference executor's ``_moe_mlp_block`` (GLM4MoeExecutor or Qwen3NextExecutor,
unchanged) and stores its output plus the expert ids it selected.  The ids are
observed, not recomputed: the executor module's ``np`` is swapped for a proxy that
records the result of the ``take_along_axis`` call that reorders ``topk_indices``
(glm4_moe.py:194, qwen3_next.py:288).

For ``oracle.cases.SIGMOID_SPECS`` (HF GLM-4.x sigmoid routing, which the reference
does not implement) it records transformers' ``Glm4MoeMoE.route_tokens_to_experts``.

For ``oracle.cases.DENSE_SPECS`` it runs the reference ``_dense_mlp_block`` (the MLP
of GLM-4 first_k_dense_replace layers, glm4_moe.py:166-172) and stores its output.

For ``oracle.cases.ATTN_SPECS`` it runs the reference ``_attention_block`` (GLM-4 MoE
attention, glm4_moe.py:112-162) and stores its output.

``--only NAME ...`` regenerates just those fixtures (the manifest keeps the others).

Fixtures hold outputs and input checksums only; inputs are rebuilt from the seed.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle.cases import (ATTN_SPECS, DENSE_SPECS, GOLDEN_SPECS, SIGMOID_SPECS,  # noqa: E402
                          input_checksum, make_attn_case, make_case, make_dense_case)
from oracle.moe_oracle import rms_norm  # noqa: E402


class _RecordingNumpy:
    """Stands in for the executor module's ``np``; records take_along_axis results."""

    def __init__(self) -> None:
        self.calls: list[np.ndarray] = []

    def take_along_axis(self, arr, idx, axis):  # noqa: ANN001
        res = np.take_along_axis(arr, idx, axis=axis)
        self.calls.append(res)
        return res

    def __getattr__(self, name: str):  # noqa: ANN204
        return getattr(np, name)


def run_reference(spec, x, t):  # noqa: ANN001, ANN201
    if spec.family == "glm":
        import offload_runtime.executors.glm4_moe as mod
        ex = mod.GLM4MoeExecutor({
            "hidden_size": spec.hidden, "num_attention_heads": 8, "intermediate_size": spec.inter,
            "moe_intermediate_size": spec.inter, "rms_norm_eps": spec.eps,
            "num_experts_per_tok": spec.top_k, "n_routed_experts": spec.n_experts,
            "routed_scaling_factor": spec.routed_scaling_factor,
            "norm_topk_prob": spec.norm_topk_prob,
        })
    else:
        import offload_runtime.executors.qwen3_next as mod
        ex = mod.Qwen3NextExecutor({
            "hidden_size": spec.hidden, "num_attention_heads": 8, "rms_norm_eps": spec.eps,
            "num_experts": spec.n_experts, "num_experts_per_tok": spec.top_k,
            "moe_intermediate_size": spec.inter,
            "shared_expert_intermediate_size": spec.shared_inter,
            "norm_topk_prob": spec.norm_topk_prob,
        })
    rec = _RecordingNumpy()
    saved = mod.np
    mod.np = rec
    try:
        out = ex._moe_mlp_block(x, t)
    finally:
        mod.np = saved
    # calls: [0] weights gather, [1] reordered ids, [2] reordered weights
    ids = np.asarray(rec.calls[1], dtype=np.int64)
    return np.asarray(out, dtype=np.float32), ids


def run_reference_dense(spec, x, t):  # noqa: ANN001, ANN201
    import offload_runtime.executors.glm4_moe as mod
    ex = mod.GLM4MoeExecutor({
        "hidden_size": spec.hidden, "num_attention_heads": 8, "intermediate_size": spec.inter,
        "rms_norm_eps": spec.eps,
    })
    return np.asarray(ex._dense_mlp_block(x, t), dtype=np.float32)


def run_reference_attention(spec, x, t):  # noqa: ANN001, ANN201
    import offload_runtime.executors.glm4_moe as mod
    ex = mod.GLM4MoeExecutor(spec.hf_config())
    return np.asarray(ex._attention_block(x, t), dtype=np.float32)


def run_hf_sigmoid(spec, x, t):  # noqa: ANN001, ANN201
    import torch
    from transformers.models.glm4_moe.configuration_glm4_moe import Glm4MoeConfig
    from transformers.models.glm4_moe.modeling_glm4_moe import Glm4MoeMoE

    cfg = Glm4MoeConfig(hidden_size=spec.hidden, n_routed_experts=spec.n_experts,
                        num_experts_per_tok=spec.top_k, n_group=1, topk_group=1,
                        routed_scaling_factor=spec.routed_scaling_factor,
                        norm_topk_prob=spec.norm_topk_prob,
                        moe_intermediate_size=spec.inter, n_shared_experts=1)
    moe = Glm4MoeMoE(cfg).float()
    with torch.no_grad():
        moe.gate.weight.copy_(torch.from_numpy(t["mlp.gate.weight"]))
        moe.gate.e_score_correction_bias.copy_(torch.from_numpy(t["mlp.gate.e_score_correction_bias"]))
        h = rms_norm(x, t["post_attention_layernorm.weight"], spec.eps)
        logits = moe.gate(torch.from_numpy(h))
        ids, w = moe.route_tokens_to_experts(logits)
    return ids.numpy().astype(np.int64), w.numpy().astype(np.float32)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the disk-mem-off checkout")
    ap.add_argument("--out", default=str(Path(__file__).resolve().parent))
    ap.add_argument("--only", nargs="*", default=None, help="fixture names to regenerate")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    out_dir = Path(args.out)
    mpath = out_dir / "manifest.json"
    manifest = json.loads(mpath.read_text()) if args.only and mpath.exists() else {}
    want = (lambda n: True) if not args.only else (lambda n: n in args.only)
    for name, spec in GOLDEN_SPECS.items():
        if not want(name):
            continue
        x, t, _quant, _cfg = make_case(spec)
        out, ids = run_reference(spec, x, t)
        np.savez_compressed(out_dir / f"{name}.npz", out=out, topk_ids=ids,
                            checksum=input_checksum(x, t))
        manifest[name] = {"spec": spec.to_dict(), "source": "reference _moe_mlp_block"}
        print(name, out.shape, ids.shape)
    for name, spec in SIGMOID_SPECS.items():
        if not want(name):
            continue
        x, t, _quant, _cfg = make_case(spec)
        ids, w = run_hf_sigmoid(spec, x, t)
        np.savez_compressed(out_dir / f"{name}.npz", topk_ids=ids, topk_w=w,
                            checksum=input_checksum(x, t))
        manifest[name] = {"spec": spec.to_dict(),
                          "source": "transformers Glm4MoeMoE.route_tokens_to_experts"}
        print(name, ids.shape)
    for name, spec in DENSE_SPECS.items():
        if not want(name):
            continue
        x, t, _quant = make_dense_case(spec)
        out = run_reference_dense(spec, x, t)
        np.savez_compressed(out_dir / f"{name}.npz", out=out, checksum=input_checksum(x, t))
        manifest[name] = {"spec": spec.to_dict(), "source": "reference _dense_mlp_block"}
        print(name, out.shape)
    for name, spec in ATTN_SPECS.items():
        if not want(name):
            continue
        x, t = make_attn_case(spec)
        out = run_reference_attention(spec, x, t)
        np.savez_compressed(out_dir / f"{name}.npz", out=out, checksum=input_checksum(x, t))
        manifest[name] = {"spec": spec.to_dict(), "source": "reference _attention_block"}
        print(name, out.shape)
    mpath.write_text(json.dumps(manifest, indent=1, sort_keys=True))


if __name__ == "__main__":
    main()
