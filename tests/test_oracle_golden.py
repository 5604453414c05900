"""Pins the CPU oracle to the reference: every golden case (reference Triton
kernels run by the Triton interpreter, plus the literal vectors and expected
tensors of the reference operator tests) must match oracle/ops.py.

fp32 tolerance: rtol = atol = 1e-5 against the reference kernel outputs (the
interpreter accumulates in fp32, the oracle in fp64)."""
from __future__ import annotations

import numpy as np
import pytest

from golden_io import all_cases
from op_cases import oracle_outputs
from oracle import ops as O

CASES = list(all_cases())


def reference_defect(op: str, case: dict) -> bool:
    """Non-causal attention with Sk % 32 != 0: the reference kernel softmaxes over its
    zero-padded key block (oracle.ops.attention_reference_padded)."""
    return (op == "attention" and not case["attrs"].get("causal", False)
            and case["inputs"]["k"].shape[2] % 32 != 0)


@pytest.mark.parametrize("op,idx,case", CASES, ids=[f"{op}-{i}" for op, i, _ in CASES])
def test_oracle_matches_reference_kernel(op, idx, case):
    got = oracle_outputs(op, case["inputs"], case["attrs"])
    if reference_defect(op, case):
        inp = case["inputs"]
        padded = O.attention_reference_padded(inp["q"], inp["k"], inp["v"])
        np.testing.assert_allclose(padded, case["outputs"]["output"], rtol=1e-5, atol=1e-5)
        assert not np.allclose(got["output"], case["outputs"]["output"], rtol=1e-3, atol=1e-3)
        return
    for name, ref in case["outputs"].items():
        np.testing.assert_allclose(got[name], ref, rtol=1e-5, atol=1e-5, err_msg=f"{op} case {idx} {name}")
    for name, exp in case["expected"].items():
        # the reference tests' own expected values (rtol = atol = 1e-3 there)
        np.testing.assert_allclose(got[name], exp, rtol=1e-5, atol=1e-5, err_msg=f"{op} expected {name}")


def test_every_operator_has_golden_cases():
    ops = {op for op, _, _ in CASES}
    assert ops == {"linear", "matmul", "rms_norm", "rotary_embedding", "attention", "embedding",
                   "add", "mul", "silu", "relu", "softmax", "max_pool2d", "batch_norm2d",
                   "transpose", "conv2d", "reshape"}
    # the 16 reference operator tests are all captured (they carry expected tensors)
    with_expected = {op for op, _, c in CASES if c["expected"]}
    assert with_expected == ops


def test_reshape_shape_rules():
    assert O.reshape_shape([2, 3, 4], [4, -1]) == [4, 6]
    with pytest.raises(ValueError):
        O.reshape_shape([2, 3], [-1, -1])
    with pytest.raises(ValueError):
        O.reshape_shape([2, 3], [4, -1])
    with pytest.raises(ValueError):
        O.reshape_shape([2, 3], [0, 6])
    with pytest.raises(ValueError):
        O.reshape_shape([2, 3], [5])


def test_reference_flat_kv_append_differs_when_bh_gt_1():
    """The reference's flat append (src/kv_cache.cc:35-42) is not a sequence concat for B*H > 1;
    the oracle's kv_append is."""
    rng = np.random.default_rng(0)
    old = rng.standard_normal((1, 2, 3, 4))
    new = rng.standard_normal((1, 2, 1, 4))
    cat = np.concatenate([old, new], axis=2)
    assert not np.allclose(O.kv_append_reference_flat(old, new), cat)
    cache = np.zeros((1, 2, 8, 4))
    ck, _ = O.kv_append(cache, cache, old, old, 0)
    ck, _ = O.kv_append(ck, ck, new, new, 3)
    np.testing.assert_array_equal(ck[:, :, :4], cat)
    # with B*H == 1 the two agree (the only case the reference's single-token test exercises)
    np.testing.assert_array_equal(O.kv_append_reference_flat(old[:, :1], new[:, :1]),
                                  np.concatenate([old[:, :1], new[:, :1]], axis=2))


def test_gqa_attention_equals_repeated_kv():
    rng = np.random.default_rng(1)
    q = rng.standard_normal((2, 6, 5, 8))
    k = rng.standard_normal((2, 2, 7, 8))
    v = rng.standard_normal((2, 2, 7, 8))
    got = O.attention(q, k, v, causal=True)
    ref = O.attention(q, np.repeat(k, 3, axis=1), np.repeat(v, 3, axis=1), causal=True)
    np.testing.assert_allclose(got, ref, rtol=1e-12, atol=1e-12)


def test_rotary_positions_match_start_pos():
    rng = np.random.default_rng(2)
    q = rng.standard_normal((2, 3, 4, 8))
    k = rng.standard_normal((2, 1, 4, 8))
    ang = rng.standard_normal((16, 4))
    c, s = np.cos(ang), np.sin(ang)
    q1, k1 = O.rotary(q, k, c, s, start_pos=5)
    q2, k2 = O.rotary(q, k, c, s, positions=np.array([5, 5]))
    q3, k3 = O.rotary(q, k, c, s, positions=np.tile(np.arange(5, 9), (2, 1)))
    np.testing.assert_allclose(q1, q2)
    np.testing.assert_allclose(k1, k2)
    np.testing.assert_allclose(q1, q3)
    np.testing.assert_allclose(k1, k3)
