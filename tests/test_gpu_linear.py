"""The projections around the attention on the tensor cores (b2a_linear: bias and residual
in the GEMM epilogue) and the decode attention block built from them (QKV projection + bias
-> fused decode step -> O projection + residual), against float64 numpy GEMMs and the oracle.
Reference: INF/qwen/Qwen2Runtime.java:693-777 (decode), 888-914 and 973-1000 (prefill)."""
import math

import numpy as np
import pytest

import oracle
from helpers import assert_close, normal, to_dev, to_np

pytestmark = pytest.mark.gpu

TORCH = {oracle.F32: "float32", oracle.F16: "float16", oracle.BF16: "bfloat16"}


def _gemm(x, w, bias=None, residual=None):
    y = x.astype(np.float64) @ w.astype(np.float64).T
    if bias is not None:
        y = y + bias.astype(np.float64)
    if residual is not None:
        y = y + residual.astype(np.float64)
    return y


@pytest.mark.parametrize("M,N,K,dtype,out_dtype,use_bias,use_res", [
    (64, 1152, 896, oracle.F16, oracle.F32, True, False),    # Qwen2.5-0.5B QKV projection, decode batch 64
    (64, 896, 896, oracle.BF16, oracle.BF16, False, True),   # O projection + residual, bf16
    (300, 200, 136, oracle.F16, oracle.F16, True, True),     # ragged M, N and a K that is not a multiple of 64
    (1, 72, 8, oracle.BF16, oracle.F32, False, False),       # one row, the smallest K
    (1024, 2048, 192, oracle.F16, oracle.F16, True, True),   # enough output tiles to fill the GPU: no split-K
])
def test_linear_matches_float64(ctx, M, N, K, dtype, out_dtype, use_bias, use_res):
    import torch
    import b200attn
    x = normal(900 + M, (M, K), dtype)
    w = oracle.round_to(normal(901 + N, (N, K), oracle.F32) / math.sqrt(K), dtype)
    bias = normal(902, (N,), oracle.F32) if use_bias else None
    res = normal(903, (M, N), out_dtype) if use_res else None
    want = _gemm(x, w, bias, res)
    y = torch.full((M, N), float("nan"), dtype=getattr(torch, TORCH[out_dtype]), device="cuda")
    b200attn.linear(ctx, to_dev(x, dtype), to_dev(w, dtype), y,
                    bias=None if bias is None else torch.from_numpy(bias).cuda(),
                    residual=None if res is None else to_dev(res, out_dtype))
    ctx.check_device_status()
    got = to_np(y)
    # fp32 accumulation of K products; a 16-bit output adds its own rounding (half an ulp)
    tol = 1e-4 if out_dtype == oracle.F32 else 2e-3 + np.abs(want) * (2.0 ** -8 if out_dtype == oracle.BF16
                                                                         else 2.0 ** -11)
    assert np.all(np.isfinite(got))
    assert np.all(np.abs(got - want) <= tol), float(np.max(np.abs(got - want) - tol))


def test_linear_split_k_shapes_back_to_back(ctx):
    """Decode-shaped projections split K over CTAs and meet in an fp32 accumulator that each tile's last
    CTA leaves at zero: launches of different shapes, queued without a synchronisation, must each be right."""
    import torch
    import b200attn
    runs = []
    for i, (M, N, K) in enumerate([(64, 1152, 896), (64, 896, 896), (8, 300, 2048), (64, 1152, 896)]):
        x = normal(950 + i, (M, K), oracle.F16)
        w = oracle.round_to(normal(960 + i, (N, K), oracle.F32) / math.sqrt(K), oracle.F16)
        bias = normal(970 + i, (N,), oracle.F32)
        y = torch.full((M, N), float("nan"), device="cuda")
        b200attn.linear(ctx, to_dev(x, oracle.F16), to_dev(w, oracle.F16), y, bias=torch.from_numpy(bias).cuda())
        runs.append((y, _gemm(x, w, bias)))
    torch.cuda.synchronize()
    ctx.check_device_status()
    for i, (y, want) in enumerate(runs):
        assert np.max(np.abs(to_np(y) - want)) < 1e-4, i


def test_linear_residual_in_place(ctx):
    """The residual may be the output buffer itself (hidden += o_proj)."""
    import torch
    import b200attn
    M, N, K = 40, 256, 128
    x = normal(910, (M, K), oracle.F16)
    w = oracle.round_to(normal(911, (N, K), oracle.F32) / math.sqrt(K), oracle.F16)
    h = normal(912, (M, N), oracle.F32)
    want = _gemm(x, w, None, h)
    y = to_dev(h, oracle.F32)
    b200attn.linear(ctx, to_dev(x, oracle.F16), to_dev(w, oracle.F16), y, residual=y)
    torch.cuda.synchronize()
    assert np.max(np.abs(to_np(y) - want)) < 1e-4


def _block_case(ctx, *, B, hidden, Hq, Hkv, D, max_seq, lens, dtype, seed):
    import torch
    import b200attn
    nqkv = (Hq + 2 * Hkv) * D
    x = normal(seed, (B, hidden), dtype)
    wqkv = oracle.round_to(normal(seed + 1, (nqkv, hidden), oracle.F32) / math.sqrt(hidden), dtype)
    bqkv = 0.1 * normal(seed + 2, (nqkv,), oracle.F32)
    wo = oracle.round_to(normal(seed + 3, (hidden, Hq * D), oracle.F32) / math.sqrt(Hq * D), dtype)
    res = normal(seed + 4, (B, hidden), dtype)
    kc = normal(seed + 5, (B, Hkv, max_seq, D), oracle.F16)
    vc = normal(seed + 6, (B, Hkv, max_seq, D), oracle.F16)
    lens = np.asarray(lens, np.int32)
    scale = float(np.float32(1 / math.sqrt(D)))
    # reference: fp32 projection rows (as the reference keeps them), the oracle's decode step, the
    # attention output rounded to the activation type (the O GEMM's operand type), then O proj + residual
    qkv = _gemm(x, wqkv, bqkv).astype(np.float32)
    q = qkv[:, :Hq * D].reshape(B, Hq, D)
    kn = qkv[:, Hq * D:(Hq + Hkv) * D].reshape(B, Hkv, D)
    vn = qkv[:, (Hq + Hkv) * D:].reshape(B, Hkv, D)
    attn, kc_w, vc_w = oracle.decode(q, kn, vn, kc, vc, lens, B=B, Hq=Hq, Hkv=Hkv, D=D, max_seq=max_seq, scale=scale,
                                     rope_theta=1e6, rope_mode=oracle.ROPE_DECODERONLY,
                                     cache_layout=oracle.KV_HEAD_MAJOR, cache_dtype=oracle.F16)
    want = _gemm(oracle.round_to(attn.reshape(B, Hq * D), dtype), wo, None, res)
    kcd, vcd = to_dev(kc, oracle.F16), to_dev(vc, oracle.F16)
    y = torch.full((B, hidden), float("nan"), dtype=getattr(torch, TORCH[dtype]), device="cuda")
    b200attn.decode_attention_block(ctx, to_dev(x, dtype), to_dev(wqkv, dtype), torch.from_numpy(bqkv).cuda(), kcd,
                                    vcd, torch.from_numpy(lens).cuda(), to_dev(wo, dtype), to_dev(res, dtype), y,
                                    num_q_heads=Hq, num_kv_heads=Hkv, scale=scale, rope_theta=1e6)
    ctx.check_device_status()
    got = to_np(y)
    # Tolerance: the 2e-3 bar, half an ulp of y's own rounding, and the attention output's rounding to
    # the activation type before the O projection: the GPU's and the oracle's attention outputs differ
    # (within the parity bar), so that rounding can land one ulp apart; each such half-ulp step is
    # weighted by w_o, and 4 sigma of their sum over the Hq*D inputs is allowed.
    mant = 7 if dtype == oracle.BF16 else 10
    a = np.abs(attn.reshape(B, Hq * D)).astype(np.float64)
    ulp_a = 2.0 ** (np.floor(np.log2(np.maximum(a, 2.0 ** -24))) - mant)
    flips = 4.0 * np.sqrt((ulp_a / 2) ** 2 @ (wo.astype(np.float64) ** 2).T)
    half_ulp = np.abs(want) * 2.0 ** -(mant + 1)
    tol = 2e-3 + half_ulp + flips
    assert np.all(np.abs(got - want) <= tol), float(np.max(np.abs(got - want) - tol))
    # the new k/v rows are in the caches (within one fp16 ulp: the fp32 rows are rotated, then rounded)
    for b, L in enumerate(lens):
        np.testing.assert_allclose(to_np(kcd[b, :, L]), kc_w[b, :, L], rtol=2 ** -10, atol=1e-6)
        np.testing.assert_allclose(to_np(vcd[b, :, L]), vc_w[b, :, L], rtol=2 ** -10, atol=1e-6)


def test_decode_attention_block_qwen_shape(ctx):
    """Qwen2.5-0.5B geometry (hidden 896, 14/2 heads, D 64, RoPE theta 1e6), fp16 activations."""
    _block_case(ctx, B=6, hidden=896, Hq=14, Hkv=2, D=64, max_seq=2000, lens=[0, 1, 700, 1999, 64, 1500],
                dtype=oracle.F16, seed=930)


def test_decode_attention_block_config_batch_bf16(ctx):
    """configs[2]'s batch of 64 with its context lengths (U[512, 8192]), bf16 activations."""
    lens = oracle.splitmix_uniform_int(3, 64, 512, 8192)
    _block_case(ctx, B=64, hidden=896, Hq=14, Hkv=2, D=64, max_seq=8193, lens=lens, dtype=oracle.BF16, seed=940)


def test_decode_attention_block_early_start(ctx):
    """Under b2a_set_decode_early_start the block's QKV GEMM, decode and O GEMM are launched with
    programmatic serialisation (each GEMM requests its weight panels before waiting for the kernel
    ahead); two blocks back to back, as two layers, both match the float64 reference."""
    try:
        ctx.set_decode_early_start(True)
        _block_case(ctx, B=6, hidden=896, Hq=14, Hkv=2, D=64, max_seq=2000, lens=[0, 1, 700, 1999, 64, 1500],
                    dtype=oracle.F16, seed=950)
        lens = oracle.splitmix_uniform_int(3, 64, 512, 8192)
        _block_case(ctx, B=64, hidden=896, Hq=14, Hkv=2, D=64, max_seq=8193, lens=lens, dtype=oracle.BF16, seed=960)
    finally:
        ctx.set_decode_early_start(False)
