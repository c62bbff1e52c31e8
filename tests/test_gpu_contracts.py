"""The reference's own GPU tests, ported 1:1 onto the CUDA contracts.

* QwenAttentionShadersGpuTest (directml-windows-bindings/src/test/java/com/aresstack/windirectml/
  windows/QwenAttentionShadersGpuTest.java:34-323): rope_and_append and gqa_attention_decode,
  Random(42) / Random(123), tolerance 1e-4.
* Gemma3WarpFusedAttentionContextTest (directml-inference/src/test/java/com/aresstack/windirectml/
  inference/gemma/Gemma3WarpFusedAttentionContextTest.java:19-121): fused context vs the staged
  (scores -> softmax -> value) math, Random(1..5), tolerance 1e-3 abs + 1e-3 rel.
"""
import math

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

NUM_HEADS, KV_HEADS, HEAD_DIM, MAX_SEQ = 2, 1, 8, 4
Q_SIZE, KV_SIZE, CACHE_SIZE = NUM_HEADS * HEAD_DIM, KV_HEADS * HEAD_DIM, KV_HEADS * MAX_SEQ * HEAD_DIM
TOL = 1e-4


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def test_qwen_rope_and_append_matches_cpu_reference(ctx):
    import torch
    import b200attn
    rng = oracle.JavaRandom(42)
    q, k, v = rng.floats_pm1(Q_SIZE), rng.floats_pm1(KV_SIZE), rng.floats_pm1(KV_SIZE)
    pos = 2
    qd, kc, vc = _dev(q), torch.zeros(CACHE_SIZE, device="cuda"), torch.zeros(CACHE_SIZE, device="cuda")
    b200attn.QwenAttentionShaders(ctx).rope_and_append(qd, _dev(k), _dev(v), kc, vc, NUM_HEADS, KV_HEADS, HEAD_DIM,
                                                       pos, MAX_SEQ, 10000.0)
    torch.cuda.synchronize()
    q_want = oracle.rope_decoderonly(q, NUM_HEADS, HEAD_DIM, pos, 10000.0)
    k_rot = oracle.rope_decoderonly(k, KV_HEADS, HEAD_DIM, pos, 10000.0)
    np.testing.assert_allclose(qd.cpu().numpy(), q_want, atol=TOL)
    kc_want = np.zeros(CACHE_SIZE, np.float32)
    vc_want = np.zeros(CACHE_SIZE, np.float32)
    kc_want[pos * HEAD_DIM:(pos + 1) * HEAD_DIM] = k_rot
    vc_want[pos * HEAD_DIM:(pos + 1) * HEAD_DIM] = v
    np.testing.assert_allclose(kc.cpu().numpy(), kc_want, atol=TOL)
    np.testing.assert_allclose(vc.cpu().numpy(), vc_want, atol=TOL)


def test_qwen_gqa_attention_decode_matches_cpu_reference(ctx):
    import torch
    import b200attn
    rng = oracle.JavaRandom(123)
    seq_len = 3
    q = rng.floats_pm1(Q_SIZE)
    kc = np.zeros(CACHE_SIZE, np.float32)
    vc = np.zeros(CACHE_SIZE, np.float32)
    two, one = np.float32(2), np.float32(1)
    for kvh in range(KV_HEADS):
        for p in range(seq_len):
            base = (kvh * MAX_SEQ + p) * HEAD_DIM
            for d in range(HEAD_DIM):
                kc[base + d] = np.float32(rng.next_float()) * two - one
                vc[base + d] = np.float32(rng.next_float()) * two - one
    scale = float(np.float32(1.0 / math.sqrt(HEAD_DIM)))
    out = torch.zeros(Q_SIZE, device="cuda")
    b200attn.QwenAttentionShaders(ctx).gqa_attention_decode(_dev(q), _dev(kc), _dev(vc), out, NUM_HEADS, KV_HEADS,
                                                            HEAD_DIM, NUM_HEADS // KV_HEADS, seq_len, MAX_SEQ, scale)
    torch.cuda.synchronize()
    want = oracle.attend_cache(q.reshape(1, NUM_HEADS, HEAD_DIM), kc.reshape(1, KV_HEADS, MAX_SEQ, HEAD_DIM),
                               vc.reshape(1, KV_HEADS, MAX_SEQ, HEAD_DIM), [seq_len - 1], B=1, Hq=NUM_HEADS,
                               Hkv=KV_HEADS, D=HEAD_DIM, max_seq=MAX_SEQ, scale=scale, first_explicit=0)
    np.testing.assert_allclose(out.cpu().numpy(), want.ravel(), atol=TOL)


@pytest.mark.parametrize("num_heads,kv_heads,head_dim,max_seq,pos,bias,seed", [
    (NUM_HEADS, KV_HEADS, HEAD_DIM, MAX_SEQ, 2, True, 42),   # the shader test shapes, fused
    (14, 2, 64, 128, 77, True, 7),                           # a Qwen2.5-0.5B layer
    (14, 2, 64, 128, 0, False, 8),                           # first token, no bias
])
def test_qwen_decode_step_fused_matches_oracle(ctx, num_heads, kv_heads, head_dim, max_seq, pos, bias, seed):
    """b2a_qwen_decode_step = QwenGpuPipeline.decodeLayerGpuResident steps 1b-3 (fused bias Add,
    ROPE_AND_APPEND, GQA_ATTENTION_DECODE) on one fused [Q|K|V] row: the output within the shader
    tests' 1e-4, the appended rows within one float ulp, every other cache row untouched."""
    import torch
    import b200attn
    rng = oracle.JavaRandom(seed)
    q_size, kv_size = num_heads * head_dim, kv_heads * head_dim
    qkv = rng.floats_pm1(q_size + 2 * kv_size)
    qkv_bias = rng.floats_pm1(q_size + 2 * kv_size, 0.25) if bias else None
    kc = rng.floats_pm1(kv_heads * max_seq * head_dim)
    vc = rng.floats_pm1(kv_heads * max_seq * head_dim)
    scale = float(np.float32(1.0 / math.sqrt(head_dim)))
    theta = 1000000.0
    x = qkv + qkv_bias if bias else qkv.copy()  # the Add dispatch, in float32
    want, kc_want, vc_want = oracle.decode(
        x[:q_size].reshape(1, num_heads, head_dim), x[q_size:q_size + kv_size].reshape(1, kv_heads, head_dim),
        x[q_size + kv_size:].reshape(1, kv_heads, head_dim), kc.reshape(1, kv_heads, max_seq, head_dim),
        vc.reshape(1, kv_heads, max_seq, head_dim), [pos], B=1, Hq=num_heads, Hkv=kv_heads, D=head_dim,
        max_seq=max_seq, scale=scale, rope_theta=theta, rope_mode=oracle.ROPE_DECODERONLY,
        cache_layout=oracle.KV_HEAD_MAJOR, cache_dtype=oracle.F32)
    kcd, vcd = _dev(kc), _dev(vc)
    qkvd = _dev(qkv)
    out = torch.zeros(q_size, device="cuda")
    b200attn.QwenAttentionShaders(ctx).decode_step(qkvd, _dev(qkv_bias) if bias else None, kcd, vcd, out, num_heads,
                                                   kv_heads, head_dim, pos, max_seq, theta, scale)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), want.ravel(), atol=TOL)
    np.testing.assert_array_equal(qkvd.cpu().numpy(), qkv)  # the input row is not modified
    got_k, got_v = kcd.cpu().numpy(), vcd.cpu().numpy()
    kw, vw = kc_want.ravel(), vc_want.ravel()
    rows = np.zeros((kv_heads, max_seq), bool)
    rows[:, pos] = True
    rows = np.repeat(rows.ravel(), head_dim)
    np.testing.assert_array_equal(got_k[~rows], kc[~rows])
    np.testing.assert_array_equal(got_v[~rows], vc[~rows])
    ulp = np.spacing(np.abs(kw[rows]).astype(np.float32))
    assert np.all(np.abs(got_k[rows] - kw[rows]) <= ulp)
    np.testing.assert_array_equal(got_v[rows], vw[rows])


@pytest.mark.parametrize("num_heads,num_kv,head_dim,seq_len,first_valid,seed", [
    (4, 1, 256, 6, 0, 1),   # Gemma 270M shape, full attention
    (4, 1, 256, 12, 7, 2),  # local layer: firstValid > 0
    (2, 2, 8, 5, 0, 3),     # numKvHeads == numHeads
    (4, 2, 16, 8, 3, 4),
    (4, 1, 256, 1, 0, 5),   # queryPos = 0, one visible key
])
def test_gemma_fused_attention_context_matches_staged(ctx, num_heads, num_kv, head_dim, seq_len, first_valid, seed):
    import b200attn
    kv_dim = num_kv * head_dim
    query_pos = seq_len - 1
    scale = float(np.float32(1.0 / math.sqrt(head_dim)))
    rng = oracle.JavaRandom(seed)
    q = rng.floats_pm1(num_heads * head_dim, 0.1)
    keys = rng.floats_pm1(seq_len * kv_dim, 0.1)
    values = rng.floats_pm1(seq_len * kv_dim, 0.1)
    got = b200attn.Gemma3FusedAttentionContext(ctx).context(_dev(q), _dev(keys), _dev(values), num_heads, num_kv,
                                                            head_dim, kv_dim, query_pos, first_valid, scale)
    staged = oracle.attend_cache(q.reshape(1, num_heads, head_dim), keys.reshape(1, seq_len, num_kv, head_dim),
                                 values.reshape(1, seq_len, num_kv, head_dim), [query_pos], B=1, Hq=num_heads,
                                 Hkv=num_kv, D=head_dim, max_seq=seq_len, scale=scale, first_explicit=first_valid,
                                 cache_layout=oracle.KV_POS_MAJOR, softmax_mode=oracle.SOFTMAX_GEMMA).ravel()
    g = got.cpu().numpy()
    assert np.all(np.abs(g - staged) <= 1e-3 + 1e-3 * np.abs(staged))


def test_gemma_fused_context_rejects_large_head_dim(ctx):
    import b200attn
    z = _dev(np.zeros(4 * 512, np.float32))
    with pytest.raises(ValueError, match="exceeds fused-attention group size 256"):
        b200attn.Gemma3FusedAttentionContext(ctx).context(z, z, z, 4, 1, 512, 512, 0, 0, 0.05)
