"""Pins the CPU oracle to the reference's own known-answer tests.

Each test cites the reference test it ports (paths inside win-directml-java,
``src/test/java/com/aresstack/windirectml/...``).  Inputs that the reference
draws from ``new java.util.Random(seed)`` are regenerated with the
:class:`oracle.JavaRandom` port, whose first outputs are themselves pinned
against the documented Java values.
"""
import math

import numpy as np
import pytest

import oracle


# --------------------------------------------------------------- java.util.Random
def test_java_random_matches_documented_sequence():
    # Widely published values of the JDK generator.
    r42 = oracle.JavaRandom(42)
    assert [r42.next_int() for _ in range(3)] == [-1170105035, 234785527, -1360544799]
    assert oracle.JavaRandom(0).next_int() == -1155484576
    assert oracle.JavaRandom(42).next_double() == 0.7275636800328681
    assert np.float32(oracle.JavaRandom(42).next_float()) == np.float32(0.7275637)
    r = oracle.JavaRandom(42)
    assert [r.next_int(10) for _ in range(5)] == [0, 3, 8, 4, 0]


# --------------------------------------------------------------- RoPE
def test_decoderonly_rope_position_zero_unchanged():
    # inference/decoderonly/DecoderOnlyRotaryEmbeddingTest.java:10-18
    v = np.array([1, 2, 3, 4], np.float32)
    out = oracle.rope_decoderonly(v, 1, 4, 0, 10000.0)
    np.testing.assert_allclose(out, v, atol=1e-6)


def test_decoderonly_rope_on_the_fly_angle():
    # inference/decoderonly/DecoderOnlyRotaryEmbeddingTest.java:20-29 (D=2, pos 2)
    out = oracle.rope_decoderonly(np.array([1, 0], np.float32), 1, 2, 2, 10000.0)
    assert abs(out[0] - np.float32(math.cos(2.0))) <= 1e-6
    assert abs(out[1] - np.float32(math.sin(2.0))) <= 1e-6


def test_gemma_rope_across_heads_matches_per_head():
    # inference/gemma/Gemma3RoPETest.java:27-48 (Random(101), 3 heads x 8, pos 5)
    packed = oracle.JavaRandom(101).floats_pm1(3 * 8)
    expected = np.concatenate([oracle.rope_half_gemma(packed[h * 8:(h + 1) * 8], 1, 8, 5, 10000.0)
                               for h in range(3)])
    got = oracle.rope_half_gemma(packed, 3, 8, 5, 10000.0)
    np.testing.assert_allclose(got, expected, atol=1e-6)


def test_gemma_rope_position_zero_identity():
    # inference/gemma/Gemma3RoPETest.java:50-61 (Random(103))
    packed = oracle.JavaRandom(103).floats_pm1(2 * 8)
    np.testing.assert_allclose(oracle.rope_half_gemma(packed, 2, 8, 0, 10000.0), packed, atol=1e-6)


def test_gemma_rope_preserves_pair_norm():
    # inference/gemma/Gemma3RoPETest.java:63-80 (D=256, Random(107), pos 9, theta 1e6)
    x = oracle.JavaRandom(107).floats_pm1(256)
    y = oracle.rope_half_gemma(x, 1, 256, 9, 1_000_000.0)
    nb = np.hypot(x[:128].astype(np.float64), x[128:].astype(np.float64))
    na = np.hypot(y[:128].astype(np.float64), y[128:].astype(np.float64))
    np.testing.assert_allclose(na, nb, atol=1e-4)


def test_gemma_math_rope_identity_norm_and_dual_theta():
    # inference/gemma/Gemma3ReferenceMathTest.java:48-72
    v = np.array([0.3, -0.7, 1.1, 0.2], np.float32)
    np.testing.assert_allclose(oracle.rope_half_gemma(v, 1, 4, 0, 10000.0), v, atol=1e-6)
    r = oracle.rope_half_gemma(v, 1, 4, 5, 10000.0)
    assert abs(np.linalg.norm(r.astype(np.float64)) - np.linalg.norm(v.astype(np.float64))) <= 1e-4
    local = oracle.rope_half_gemma(np.array([0, 1, 0, 0], np.float32), 1, 4, 3, 10000.0)
    glob = oracle.rope_half_gemma(np.array([0, 1, 0, 0], np.float32), 1, 4, 3, 1_000_000.0)
    assert abs(local[3] - glob[3]) > 1e-4


def test_decoderonly_and_gemma_rope_agree_to_float_rounding():
    x = oracle.JavaRandom(7).floats_pm1(4 * 64)
    a = oracle.rope_decoderonly(x, 4, 64, 4097, 1e6)
    b = oracle.rope_half_gemma(x, 4, 64, 4097, 1e6)
    np.testing.assert_allclose(a, b, atol=2e-6)


# --------------------------------------------------------------- RMSNorm
def test_zero_centered_rmsnorm_closed_form():
    # inference/gemma/Gemma3ReferenceMathTest.java:14-29
    v = np.array([1, 2, 3, 4], np.float32)
    out = oracle.rmsnorm_zero_centered(v, 1, 4, np.zeros(4, np.float32), 1e-6)
    rms = 1.0 / math.sqrt(30.0 / 4.0 + 1e-6)
    assert abs(out[0] - 1 * rms) <= 1e-5 and abs(out[3] - 4 * rms) <= 1e-5
    assert abs(math.sqrt(float(np.mean(out.astype(np.float64) ** 2))) - 1.0) <= 1e-4


def test_zero_centered_rmsnorm_adds_one_to_weight():
    # inference/gemma/Gemma3ReferenceMathTest.java:31-43
    v = np.array([1, 2, 3, 4], np.float32)
    one = oracle.rmsnorm_zero_centered(v, 1, 4, np.ones(4, np.float32), 1e-6)
    zero = oracle.rmsnorm_zero_centered(v, 1, 4, np.zeros(4, np.float32), 1e-6)
    np.testing.assert_allclose(one, 2.0 * zero, atol=1e-5)


# --------------------------------------------------------------- softmax
def test_softmax_distribution_and_order():
    # inference/decoderonly/DecoderOnlyMathTest.java:22-30 and qwen/Qwen2RuntimeMathTest.java:54-75
    x = oracle.softmax_decoderonly(np.array([1, 2, 3, 4, 0], np.float32))
    assert abs(float(np.sum(x)) - 1.0) <= 1e-5
    assert np.all(x > 0) and x[3] > x[2] > x[1] > x[0] > x[4]


def test_softmax_single_and_partial_length():
    # qwen/Qwen2RuntimeMathTest.java:77-96
    assert abs(oracle.softmax_decoderonly(np.array([5.0], np.float32))[0] - 1.0) <= 1e-6
    x = oracle.softmax_decoderonly(np.array([1, 2, 3, 100, 100], np.float32), 3)
    assert abs(float(x[:3].sum()) - 1.0) <= 1e-5
    assert x[3] == 100.0 and x[4] == 100.0


# --------------------------------------------------------------- layout
def test_gqa_mapping_14_2_contiguous_and_rejections():
    # inference/decoderonly/DecoderOnlyAttentionLayoutTest.java:9-30, qwen/Qwen2RuntimeMathTest.java:123-138
    for h in range(14):
        assert oracle.kv_head_for_query_head(14, 2, h) == (0 if h < 7 else 1)
    assert oracle.kv_head_for_query_head(14, 3, 0) == -1  # 14/3 rejected
    assert oracle.kv_head_for_query_head(14, 2, 14) == -1  # out of range


def test_gemma_gqa_mappings():
    # inference/gemma/Gemma3AttentionLayoutTest.java:18-25, Gemma3RoPETest.java:108-118
    assert all(oracle.kv_head_for_query_head(4, 1, h) == 0 for h in range(4))
    assert [oracle.kv_head_for_query_head(8, 2, h) for h in range(8)] == [0] * 4 + [1] * 4


def test_gemma_window_and_layer_plan():
    # inference/gemma/Gemma3AttentionLayoutTest.java:27-58, Gemma3RoPETest.java:84-134
    assert oracle.first_valid_key(False, 4, 10) == 7
    assert oracle.first_valid_key(True, 4, 100) == 0
    assert oracle.first_valid_key(False, 512, 1000) == 1000 - 512 + 1
    assert oracle.first_valid_key(False, 512, 100) == 0
    full = [layer for layer in range(18) if oracle.is_full_attention_layer(layer, 6)]
    assert full == [5, 11, 17]
    assert oracle.rope_theta_for_layer(5, 6, 1e6, 1e4) == 1e6
    assert oracle.rope_theta_for_layer(0, 6, 1e6, 1e4) == 1e4
    assert abs(oracle.attention_scale(256, 256) - np.float32(1.0 / math.sqrt(256))) <= 1e-7


# --------------------------------------------------------------- fp16 / bf16 rounding
def test_dtype_rounding_matches_numpy_fp16():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(10000).astype(np.float32) * s for s in (1e-6, 1e-3, 1, 100, 6e4)])
    np.testing.assert_array_equal(oracle.round_to(x, oracle.F16), x.astype(np.float16).astype(np.float32))


def test_bf16_rounding_is_nearest_even():
    x = np.array([1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -3.14159], np.float32)
    np.testing.assert_array_equal(oracle.round_to(x, oracle.BF16), np.array([1.0, 1.015625, -3.140625], np.float32))


def test_benchmark_generators_match_the_oracles():
    """The benchmark draws its inputs with b200attn.synthetic (so its GPU arm never loads the oracle); the
    values must be the ones the oracle's generators give the parity tests."""
    from b200attn import synthetic
    np.testing.assert_array_equal(synthetic.uniform_int(5, 256, 1024, 32768),
                                  oracle.splitmix_uniform_int(5, 256, 1024, 32768))
    np.testing.assert_array_equal(synthetic.uniform_int(2, 64, 16, 128, offset=3),
                                  oracle.splitmix_uniform_int(2, 64, 16, 128, offset=3))
    np.testing.assert_array_equal(synthetic.normal(7, 1000, offset=11), oracle.splitmix_normal(7, 1000, offset=11))
    lens = synthetic.uniform_int(5, 256, 1024, 32768)
    pick = synthetic.stratified_sample(lens, 16)
    assert len(set(pick.tolist())) == 16
    assert abs(lens[pick].mean() / lens.mean() - 1) < 0.03
