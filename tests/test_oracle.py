"""The CPU oracle against the reference's own golden vectors, and the
backend's own known-answer tests for the ops the reference does not have."""
import json
import math
import os

import numpy as np
import pytest

from oracle import oracle as ora

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "reference_kat.json")


def _kat_cases():
    with open(GOLDEN) as f:
        return json.load(f)


@pytest.mark.parametrize("case", _kat_cases(), ids=lambda c: c["id"])
def test_oracle_matches_reference_known_answers(case):
    op = case["op"]
    if op == "add":
        a, b = np.array(case["a"], np.float32), np.array(case["b"], np.float32)
        got = ora.elementwise("add", a, b, tuple(case["out_shape"])).ravel()
    elif op == "matmul":
        got = ora.matmul(np.array(case["a"], np.float32), np.array(case["b"], np.float32)).ravel()
    elif op == "softmax":
        got = ora.softmax(np.array(case["x"], np.float32)).ravel()
    elif op == "gelu":
        got = ora.gelu(np.array(case["x"], np.float32))
    elif op == "layer_norm":
        got = ora.layer_norm(np.array(case["x"], np.float32), np.array(case["gamma"], np.float32),
                             np.array(case["beta"], np.float32), case["eps"]).ravel()
    elif op == "linear":
        bias = None if case["bias"] is None else np.array(case["bias"], np.float32)
        got = ora.linear(np.array(case["x"], np.float32), np.array(case["w"], np.float32), bias).ravel()
    elif op == "transpose":
        got = ora.transpose2(np.array(case["x"], np.float32)).ravel()
    elif op == "expand":
        got = ora.broadcast_to(np.array(case["x"], np.float32), tuple(case["out_shape"])).ravel()
    elif op == "gelu_mul":
        x = np.array(case["x"], np.float32)
        got = ora.elementwise("mul", ora.gelu(x), x, x.shape).ravel()
        for g, w, t in zip(got[:2], case["want_first"], case["tol"]):
            assert abs(g - w) < t
        return
    else:
        raise AssertionError(op)
    want = np.array(case["want"], np.float32)
    assert np.all(np.abs(got - want) <= case["tol"]), (got, want)


def test_gelu_is_exact_form_not_tanh():
    # kernels.rs:234-251: the tanh approximation gives 0.8411920 at 1.0.
    assert abs(ora.gelu(np.array([1.0]))[0] - 0.8411920) > 1e-4
    g = ora.gelu(np.array([-1.0, 1.0], np.float32))
    assert abs(g[0] + g[1]) > 0.5


def test_bf16_round_to_nearest_even():
    vals = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38, 1e-40], np.float32)
    bits = ora.to_bf16(vals)
    assert bits[0] == 0x3F80
    assert bits[1] == 0x3F80  # halfway, rounds to even
    assert bits[2] == 0x3F82  # halfway, rounds up to even
    assert ora.from_bf16(bits)[3] == -2.5
    nan = ora.to_bf16(np.array([np.nan], np.float32))
    assert np.isnan(ora.from_bf16(nan))[0]


def test_int4_group_quantisation_known_answer():
    # One group of 32: w = (i - 16) / 10.  amax = 1.6, s = bf16(1.6 / 7).
    w = ((np.arange(32, dtype=np.float32) - 16) / 10).reshape(1, 32)
    packed, s = ora.quant_w4g32(w)
    sf = ora.from_bf16(s)[0, 0]
    assert s[0, 0] == ora.to_bf16(np.array([np.float32(1.6) / np.float32(7.0)]))[0]
    codes = []
    for byte in packed[0]:
        for nib in (int(byte) & 0xF, int(byte) >> 4):  # low nibble = even k
            codes.append(nib - 16 if nib >= 8 else nib)
    want = np.clip(np.rint(w[0] / np.float32(sf)), -8, 7)
    assert codes == list(want.astype(int))
    deq = ora.dequant_w4g32(packed, s)
    assert np.all(np.abs(deq - w) <= sf / 2 + 1e-7)


def test_int4_zero_group_has_zero_scale_and_codes():
    w = np.zeros((2, 64), np.float32)
    w[1, 32:] = 1.0
    packed, s = ora.quant_w4g32(w)
    assert s[0, 0] == 0 and s[0, 1] == 0 and s[1, 0] == 0
    assert np.all(packed[0] == 0) and np.all(packed[1, :16] == 0)
    assert np.all(packed[1, 16:] == 0x77)


def test_int8_per_channel_known_answer():
    w = np.array([[127.0, -63.5, 0.25, 0.0], [0, 0, 0, 0]], np.float32)
    q, s = ora.quant_w8pc(w)
    assert s[0] == np.float32(127.0) / np.float32(127.0) and s[1] == 0
    assert list(q[0]) == [127, -64, 0, 0]  # -63.5 rounds half to even
    assert np.all(q[1] == 0)


def test_rms_norm_known_answer():
    y = ora.rms_norm(np.array([[3.0, 4.0]], np.float32), np.array([1.0, 2.0], np.float32), 0.0)
    r = math.sqrt(12.5)
    assert np.allclose(y, [[3 / r, 8 / r]], rtol=1e-6)


def test_rope_position_zero_is_identity_and_rotates_pairs():
    x = ora.normal(5, (3, 2 * 8))
    assert np.array_equal(ora.rope(x, np.zeros(3, np.int32), 8), x)
    # head_dim 2: a single pair rotated by pos radians.
    y = ora.rope(np.array([[1.0, 0.0]], np.float32), np.array([3], np.int32), 2)
    assert np.allclose(y, [[math.cos(3), math.sin(3)]], atol=1e-7)


def test_silu_and_swiglu():
    assert ora.lib().ora_silu(0.0) == 0.0
    assert abs(ora.lib().ora_silu(1.0) - 0.7310586) < 1e-6
    assert np.allclose(ora.swiglu(np.array([1.0], np.float32), np.array([2.0], np.float32)), [1.4621172])


def test_attention_single_position_returns_v_and_ties_average():
    H, G, d, L = 2, 1, 4, 4
    kc = np.zeros((1, G, L, d), np.float32)
    vc = np.zeros((1, G, L, d), np.float32)
    vc[0, 0, 0] = [1, 2, 3, 4]
    vc[0, 0, 1] = [3, 2, 1, 0]
    q = ora.normal(1, (1, H * d))
    out = ora.attention(q, kc, vc, np.array([0]), np.array([0]), H, G, d)
    assert np.allclose(out.reshape(H, d), [[1, 2, 3, 4]] * H)
    out = ora.attention(q, kc, vc, np.array([0]), np.array([1]), H, G, d)  # equal scores
    assert np.allclose(out.reshape(H, d), [[2, 2, 2, 2]] * H)


def test_argmax_lowest_index_on_ties_and_skips_nan():
    x = np.array([[1, 3, 3, 2], [np.nan, -1, -1, np.nan], [np.nan] * 4], np.float32)
    assert list(ora.argmax(x)) == [1, 1, 0]


def test_embed_rejects_out_of_range_ids():
    table = ora.normal(2, (4, 3))
    out, rc = ora.embed(np.array([1, 4]), table)
    assert rc == -1 and np.array_equal(out[0], table[1]) and np.all(out[1] == 0)


def test_inputs_are_deterministic():
    a = ora.normal(7, (1000,))
    assert np.array_equal(a, ora.normal(7, (1000,)))
    big = ora.normal(0, (100000,))
    assert abs(big.mean()) < 0.02 and abs(big.std() - 1) < 0.02
    ids = ora.uniform_i32(2, 10000, 0, 32000)
    assert ids.min() >= 0 and ids.max() < 32000


def test_threaded_oracle_is_bit_identical():
    x = ora.round_bf16(ora.normal(0, (3, 256)))
    w = ora.normal(1, (64, 256), std=0.02)
    packed, s = ora.quant_w4g32(w)
    assert np.array_equal(ora.linear_w4g32(x, packed, s), ora.linear_w4g32(x, packed, s, threads=4))
