"""The oracle against the reference's own outputs (tests/golden, made by make_golden.py).

CPU only.  These pin the oracle: it must reproduce the reference executor
``_moe_mlp_block`` bit for bit on the fixtures, and the HF sigmoid router on the
sigmoid fixture, before any CUDA result is compared with it.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

from oracle.attention_oracle import AttnConfig, glm4_attention_block
from oracle.cases import (ATTN_SPECS, DENSE_SPECS, GOLDEN_SPECS, SIGMOID_SPECS, CaseSpec,
                          input_checksum, make_attn_case, make_case, make_dense_case)
from oracle.moe_oracle import (dense_mlp_block, int8_pc_dequantize, int8_pc_quantize, moe_block,
                               permutation, rms_norm, route, select_topk)

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _load(name: str) -> dict[str, np.ndarray]:
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as z:
        return {k: z[k] for k in z.files}


@pytest.mark.parametrize("name", sorted(GOLDEN_SPECS))
def test_oracle_reproduces_reference(name: str) -> None:
    spec = GOLDEN_SPECS[name]
    g = _load(name)
    x, t, _q, cfg = make_case(spec)
    np.testing.assert_array_equal(input_checksum(x, t), g["checksum"],
                                  err_msg="seeded inputs drifted from the fixture")
    out, aux = moe_block(x, t, cfg)
    np.testing.assert_array_equal(aux["topk_ids"], g["topk_ids"])
    np.testing.assert_array_equal(out, g["out"])  # bit-exact


@pytest.mark.parametrize("name", sorted(DENSE_SPECS))
def test_dense_oracle_reproduces_reference(name: str) -> None:
    """The dense MLP of first_k_dense_replace layers, against the reference's own
    ``_dense_mlp_block`` output (glm4_moe.py:166-172), bit for bit."""
    spec = DENSE_SPECS[name]
    g = _load(name)
    x, t, _q = make_dense_case(spec)
    np.testing.assert_array_equal(input_checksum(x, t), g["checksum"])
    np.testing.assert_array_equal(dense_mlp_block(x, t, spec.eps), g["out"])


@pytest.mark.parametrize("name", sorted(SIGMOID_SPECS))
def test_sigmoid_routing_matches_transformers(name: str) -> None:
    spec = SIGMOID_SPECS[name]
    g = _load(name)
    x, t, _q, cfg = make_case(spec)
    np.testing.assert_array_equal(input_checksum(x, t), g["checksum"])
    h = rms_norm(x, t["post_attention_layernorm.weight"], cfg.eps)
    ids, w, _ = route(h, t["mlp.gate.weight"], t["mlp.gate.e_score_correction_bias"], cfg)
    for r in range(ids.shape[0]):
        assert set(ids[r].tolist()) == set(g["topk_ids"][r].tolist())
        hf = dict(zip(g["topk_ids"][r].tolist(), g["topk_w"][r].tolist()))
        for e, wv in zip(ids[r].tolist(), w[r].tolist()):
            assert wv == pytest.approx(hf[e], rel=2e-6)


def test_tie_rule_lower_id_wins() -> None:
    score = np.array([[0.5, 0.9, 0.9, 0.1, 0.9]], dtype=np.float32)
    assert select_topk(score, 2).tolist() == [[1, 2]]
    assert select_topk(score, 4).tolist() == [[1, 2, 4, 0]]


def test_duplicate_router_rows_tie_deterministically() -> None:
    """Experts with identical router rows get identical scores; lower id is chosen first."""
    spec = CaseSpec(hidden=64, n_experts=8, top_k=2, inter=16, shared_inter=0, tokens=5, seed=11,
                    bias_std=0.0)
    x, t, _q, cfg = make_case(spec)
    t["mlp.gate.weight"][5] = t["mlp.gate.weight"][2]
    t["mlp.gate.e_score_correction_bias"][:] = 0
    h = rms_norm(x, t["post_attention_layernorm.weight"], cfg.eps)
    ids, _w, logits = route(h, t["mlp.gate.weight"], t["mlp.gate.e_score_correction_bias"], cfg)
    for r in range(ids.shape[0]):
        row = ids[r].tolist()
        if 5 in row:
            assert 2 in row and row.index(2) < row.index(5)


def test_permutation_is_expert_major_token_ascending() -> None:
    ids = np.array([[3, 1], [1, 0], [3, 2], [0, 1]])
    offsets, perm = permutation(ids, 4)
    assert offsets.tolist() == [0, 2, 5, 6, 8]
    # expert 0: (t1,s1),(t3,s0); expert 1: (t0,s1),(t1,s0),(t3,s1); expert 2: (t2,s1); expert 3: (t0,s0),(t2,s0)
    assert perm.tolist() == [3, 6, 1, 2, 7, 5, 0, 4]


def test_int8_per_channel_known_answers() -> None:
    w = np.array([[0.5, -1.27, 0.0, 0.635], [0.0, 0.0, 0.0, 0.0], [2.0, -2.0, 1.0, 0.004]],
                 dtype=np.float32)
    q, s = int8_pc_quantize(w)
    assert s.dtype == np.float16
    assert s[0] == np.float16(1.27 / 127) and s[1] == 0 and s[2] == np.float16(2.0 / 127)
    assert q[1].tolist() == [0, 0, 0, 0]
    assert q[0, 1] == -127 and q[2, 0] == 127 and q[2, 1] == -127
    deq = int8_pc_dequantize(q, s)
    assert np.max(np.abs(deq - w)) <= float(np.max(s.astype(np.float32))) * 0.5 + 1e-7


@pytest.mark.parametrize("name", sorted(ATTN_SPECS))
def test_attention_oracle_reproduces_reference(name: str) -> None:
    """glm4_attention_block against the reference's own _attention_block output."""
    spec = ATTN_SPECS[name]
    g = _load(name)
    x, t = make_attn_case(spec)
    np.testing.assert_array_equal(input_checksum(x, t), g["checksum"],
                                  err_msg="seeded inputs drifted from the fixture")
    out = glm4_attention_block(x, t, AttnConfig.from_hf(spec.hf_config()))
    np.testing.assert_array_equal(out, g["out"])  # bit-exact
