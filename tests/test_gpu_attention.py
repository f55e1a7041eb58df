"""GLM-4 MoE attention on the device vs the reference (needs a B200).

* every attention fixture in tests/golden (the reference's own
  ``_attention_block`` outputs, glm4_moe.py:112-162): block output within rel-L2
  2e-3, and the attention contribution alone (out - x) within 1e-2 (f16 tensor
  operands q, k, v and P against the reference's fp32);
* GLM-4.7 head geometry (head_dim 128, 96 query / 8 kv heads, hidden 5120) and
  longer sequences (many 128-key tiles, ragged last tile) against the oracle;
* deterministic (same bits on a second call) and causal (a prefix of the
  sequence gives the same rows as the whole sequence).
"""
from __future__ import annotations

import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

from moe_sm100.attention import AttentionConfig, AttentionLayer  # noqa: E402
from moe_sm100.packing import pack_layer  # noqa: E402
from oracle.attention_oracle import AttnConfig, glm4_attention_block  # noqa: E402
from oracle.cases import ATTN_SPECS, AttnSpec, make_attn_case  # noqa: E402

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
TOL_BLOCK = 2e-3
TOL_DELTA = 1e-2


def _rel(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b.astype(np.float64)))


def _layer(spec: AttnSpec, t: dict, max_tokens: int) -> AttentionLayer:
    blob, meta = pack_layer(t)  # attention tensors stay fp32 in the blob, as the loader writes them
    al = AttentionLayer(AttentionConfig.glm4_moe(spec.hf_config(), max_tokens=max_tokens))
    al.bind_host(blob, meta)
    return al


def _check(al: AttentionLayer, x: np.ndarray, ref: np.ndarray) -> np.ndarray:
    out = al.forward(torch.from_numpy(x).cuda())
    al.status()
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    eb, ed = _rel(got, ref), _rel(got - x, ref - x)
    assert eb <= TOL_BLOCK and ed <= TOL_DELTA, f"block rel-L2 {eb:.3e}, attention part {ed:.3e}"
    return got


@pytest.mark.parametrize("name", sorted(ATTN_SPECS))
def test_attention_matches_reference_fixture(name: str) -> None:
    spec = ATTN_SPECS[name]
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as z:
        gout = z["out"]
    x, t = make_attn_case(spec)
    al = _layer(spec, t, spec.tokens)
    got = _check(al, x, gout)
    again = al.forward(torch.from_numpy(x).cuda()).cpu().numpy()
    np.testing.assert_array_equal(got, again)  # deterministic
    al.close()


@pytest.mark.parametrize("spec", [
    AttnSpec(hidden=5120, heads=96, kv_heads=8, head_dim=128, tokens=300, seed=51),
    AttnSpec(hidden=1024, heads=16, kv_heads=2, head_dim=128, tokens=1500, seed=52),
    AttnSpec(hidden=512, heads=8, kv_heads=8, head_dim=64, tokens=700, seed=53, qk_norm=False,
             partial_rotary_factor=1.0, rope_theta=10000.0),
], ids=["glm47_heads_T300", "gqa8_T1500", "mha_hd64_T700"])
def test_attention_against_oracle(spec: AttnSpec) -> None:
    x, t = make_attn_case(spec)
    ref = glm4_attention_block(x, t, AttnConfig.from_hf(spec.hf_config()))
    al = _layer(spec, t, spec.tokens)
    got = _check(al, x, ref)
    # causal: the first rows of the sequence do not see the later ones.  The
    # projections split K by sequence length, so the shorter run adds the same
    # products in another order (f16 roundings of q / k / v may flip): equal to
    # ~1e-4, where a leak from later tokens would be O(1)
    n = spec.tokens // 3
    head = al.forward(torch.from_numpy(np.ascontiguousarray(x[:n])).cuda()).cpu().numpy()
    assert _rel(head - x[:n], got[:n] - x[:n]) <= 2e-3
    al.close()


def test_attention_limits() -> None:
    spec = ATTN_SPECS["attn_glm_small"]
    _x, t = make_attn_case(spec)
    al = _layer(spec, t, 8)
    with pytest.raises(ValueError):
        al.forward(torch.zeros((9, spec.hidden), device="cuda"))  # > max_tokens
    assert al.forward(torch.empty((0, spec.hidden), device="cuda")).shape == (0, spec.hidden)
    blob, meta = pack_layer(t)
    with pytest.raises(KeyError):
        bad = AttentionLayer(AttentionConfig.glm4_moe(spec.hf_config(), max_tokens=8))
        bad.bind_host(blob, [m for m in meta if m["name"] != "self_attn.o_proj.weight"])
    al.close()
