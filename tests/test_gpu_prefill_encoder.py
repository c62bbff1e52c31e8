"""Prefill and encoder parity through the C ABI against the oracle."""
import math

import numpy as np
import pytest

import oracle
from helpers import assert_close, normal, to_dev, to_np

pytestmark = pytest.mark.gpu

TORCH = {oracle.F32: "float32", oracle.F16: "float16", oracle.BF16: "bfloat16"}


def _prefill_case(ctx, *, B, S, Hq, Hkv, D, dtype, out_dtype, theta, window=0, pos0=0, seed=1, rope=True):
    import torch
    import b200attn
    q = normal(seed, (B, S, Hq, D), dtype)
    k = normal(seed + 1, (B, S, Hkv, D), dtype)
    v = normal(seed + 2, (B, S, Hkv, D), dtype)
    scale = float(np.float32(1.0 / math.sqrt(D)))
    want = oracle.prefill(q, k, v, B=B, S=S, Hq=Hq, Hkv=Hkv, D=D, scale=scale, rope_theta=theta if rope else 0.0,
                          pos0=pos0, window=window)
    o = torch.empty((B, S, Hq, D), dtype=getattr(torch, TORCH[out_dtype]), device="cuda")
    b200attn.prefill_causal(ctx, to_dev(q, dtype), to_dev(k, dtype), to_dev(v, dtype), o, scale,
                            rope_mode=b200attn.ROPE_NEOX if rope else b200attn.ROPE_NONE, rope_theta=theta, pos0=pos0,
                            window=window)
    torch.cuda.synchronize()
    return to_np(o), want


def test_prefill_smollm2_config_fp32(ctx):
    """configs[0] exactly: B=1, S=256, 9/3 heads, D=64, NeoX RoPE theta 1e5, fp32 in/out."""
    got, want = _prefill_case(ctx, B=1, S=256, Hq=9, Hkv=3, D=64, dtype=oracle.F32, out_dtype=oracle.F32,
                              theta=1e5, seed=1)
    assert ctx.last_attention_kernel() == "f32_tiled"
    err, _ = assert_close(got, want, atol=2e-3, what="smollm2 prefill")
    assert err < 1e-4  # fp32 end to end


def test_prefill_phi3_shape_bf16(ctx):
    """configs[3] geometry (32 heads MHA, D=96, theta 1e4, bf16) at a reduced size."""
    got, want = _prefill_case(ctx, B=1, S=384, Hq=4, Hkv=4, D=96, dtype=oracle.BF16, out_dtype=oracle.F32,
                              theta=1e4, seed=5)
    assert_close(got, want, what="phi3-shaped prefill (fp32 out)")


def test_prefill_bf16_output_within_tolerance_plus_rounding(ctx):
    """A bf16 output cannot meet 2e-3 where |o| >= 0.5 (one ulp is 3.9e-3 there), so the bar is
    2e-3 plus half a bf16 ulp of the oracle value: the compute tolerance plus the output rounding."""
    got, want = _prefill_case(ctx, B=1, S=200, Hq=2, Hkv=2, D=96, dtype=oracle.BF16, out_dtype=oracle.BF16,
                              theta=1e4, seed=7)
    half_ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(want), 2.0 ** -126))) - 8)
    assert np.all(np.abs(got - want) <= 2e-3 + half_ulp)


@pytest.mark.parametrize("out_dtype", [oracle.F32, oracle.BF16])
def test_prefill_phi3_config_full_sequence(ctx, out_dtype):
    """configs[3] at its full sequence length: S = 4096, D = 96, MHA, NeoX RoPE theta 1e4, bf16 inputs, on
    a 2-head slice of one sequence (every query tile, the whole causal triangle, positions up to 4095).
    fp32 output: the 2e-3 / 0.9999 bar; bf16 output: 2e-3 plus half a bf16 ulp of the oracle value."""
    got, want = _prefill_case(ctx, B=1, S=4096, Hq=2, Hkv=2, D=96, dtype=oracle.BF16, out_dtype=out_dtype,
                              theta=1e4, seed=4096)
    if out_dtype == oracle.F32:
        assert_close(got, want, what="phi3 S=4096 prefill (fp32 out)")
    else:
        half_ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(want), 2.0 ** -126))) - 8)
        assert np.all(np.abs(got - want) <= 2e-3 + half_ulp), float(np.max(np.abs(got - want) - half_ulp))


def test_prefill_head_dim_256_tensor_cores(ctx):
    """head_dim 256 (Gemma-3): one 128-row query tile per work item on the tcgen05 kernel, causal GQA over
    several key tiles with a ragged last one."""
    got, want = _prefill_case(ctx, B=2, S=520, Hq=8, Hkv=2, D=256, dtype=oracle.F16, out_dtype=oracle.F32,
                              theta=1e4, seed=21)
    assert_close(got, want, what="fp16 prefill D=256")


@pytest.mark.parametrize("D", [32, 64, 128])
def test_prefill_fp16_gqa_window(ctx, D):
    got, want = _prefill_case(ctx, B=2, S=200, Hq=8, Hkv=2, D=D, dtype=oracle.F16, out_dtype=oracle.F32,
                              theta=1e4, window=50, seed=9 + D)
    assert_close(got, want, what=f"fp16 windowed prefill D={D}")


def test_prefill_position_offset_and_no_rope(ctx):
    got, want = _prefill_case(ctx, B=1, S=70, Hq=4, Hkv=1, D=64, dtype=oracle.F16, out_dtype=oracle.F32, theta=1e6,
                              pos0=1000, seed=13)
    assert_close(got, want, what="pos0 offset")
    got, want = _prefill_case(ctx, B=1, S=70, Hq=4, Hkv=1, D=64, dtype=oracle.F16, out_dtype=oracle.F32, theta=0,
                              rope=False, seed=14)
    assert_close(got, want, what="no rope")


def test_prefill_generic_path_head_dim_40(ctx):
    got, want = _prefill_case(ctx, B=1, S=90, Hq=3, Hkv=1, D=40, dtype=oracle.F16, out_dtype=oracle.F32, theta=1e4,
                              seed=15)
    assert_close(got, want, what="generic D=40")


# ------------------------------------------------------------------ encoder
def _encoder_case(ctx, *, B, H, S, D, dtype, lens, layout, seed):
    import torch
    import b200attn
    shape = (B, H, S, D) if layout == 0 else (B, S, H, D)
    q, k, v = (normal(seed + i, shape, dtype) for i in range(3))
    want = oracle.encoder_minilm(q, k, v, lens, B=B, H=H, S=S, D=D, layout=layout)
    y = torch.empty(shape, dtype=torch.float32, device="cuda")
    b200attn.mha(ctx, to_dev(q, dtype), to_dev(k, dtype), to_dev(v, dtype), y, 1.0 / math.sqrt(D),
                 key_lengths=torch.from_numpy(np.asarray(lens, np.int32)).cuda(),
                 layout=b200attn.HEAD_MAJOR if layout == 0 else b200attn.SEQ_MAJOR)
    torch.cuda.synchronize()
    return to_np(y), want


@pytest.mark.parametrize("layout", [0, 1])
def test_encoder_minilm_config_full_size(ctx, layout):
    """configs[1] at full size: B=64, S=128, H=12, D=32, fp16, key lengths ~ U[16,128]."""
    lens = oracle.splitmix_uniform_int(2, 64, 16, 128)
    got, want = _encoder_case(ctx, B=64, H=12, S=128, D=32, dtype=oracle.F16, lens=lens, layout=layout, seed=200)
    assert ctx.last_attention_kernel() == "tcgen05"  # head dim 32 runs on the tensor-core kernel
    assert_close(got, want, what="minilm encoder")


@pytest.mark.parametrize("layout,D", [(0, 64), (1, 96), (1, 128)])
def test_encoder_ragged_length_tensor_core_dims(ctx, layout, D):
    # head_dim 64/96/128 run on the tcgen05 kernel; S = 300 leaves a ragged last tile
    got, want = _encoder_case(ctx, B=3, H=2, S=300, D=D, dtype=oracle.F16, lens=[300, 129, 7], layout=layout,
                              seed=500 + D)
    assert_close(got, want, what=f"encoder D={D}")


@pytest.mark.parametrize("layout,D,S", [(0, 32, 128), (1, 64, 100), (1, 96, 77), (0, 128, 128)])
def test_encoder_short_sequences_two_heads_per_work_item(ctx, layout, D, S):
    """Bidirectional sequences of at most 128 keys take two (batch, head) pairs per tcgen05 work item
    (one per softmax group): an odd pair count leaves the last item with one tile, pairs straddle batch
    boundaries, and a sequence without valid keys (length 0) sits in either tile of an item."""
    B, H = 3, 3
    got, want = _encoder_case(ctx, B=B, H=H, S=S, D=D, dtype=oracle.F16, lens=[S, 0, 37], layout=layout,
                              seed=800 + D)
    assert ctx.last_attention_kernel() == "tcgen05"
    assert_close(got, want, what=f"packed encoder D={D} S={S}")


def test_encoder_zero_and_full_lengths(ctx):
    # a text with no valid key averages V (softmax of equal -1e9 scores), as the reference does
    got, want = _encoder_case(ctx, B=3, H=2, S=64, D=32, dtype=oracle.F16, lens=[0, 64, 1], layout=1, seed=300)
    assert_close(got, want, what="edge lengths")


def test_encoder_fp32_generic_odd_sequence(ctx):
    got, want = _encoder_case(ctx, B=2, H=3, S=37, D=24, dtype=oracle.F32, lens=[37, 5], layout=0, seed=310)
    assert_close(got, want, atol=1e-4, what="fp32 encoder")


@pytest.mark.parametrize("with_mask", [False, True])
def test_attention_kernel_contract_directml_cases(ctx, with_mask):
    """DirectMlAttentionKernelTest (runtime/kernels/DirectMlAttentionKernelTest.java:39-127):
    B=1,H=2,S=4,D=8 FLOAT32, Random(0xA77E47 / 0xDEC0DE) inputs, one blocked key per batch, tol 5e-4."""
    import torch
    import b200attn
    B, H, S, D = 1, 2, 4, 8
    scale = float(np.float32(1.0 / math.sqrt(D)))
    rng = oracle.JavaRandom(0xA77E47 if with_mask else 0xDEC0DE)
    q, k, v = (rng.floats_centered(B * H * S * D) for _ in range(3))
    mask = None
    if with_mask:
        mask = np.zeros(B * S, np.float32)
        for b in range(B):
            mask[b * S + rng.next_int(S)] = np.float32(-1e9)
    want = oracle.mha_additive(q, k, v, mask, B=B, H=H, S=S, D=D, scale=scale)
    kern = b200attn.CudaAttentionKernel(ctx, B, H, S, D, scale, with_mask)
    dev = lambda a: torch.from_numpy(a).cuda()
    y = torch.empty(B * H * S * D, device="cuda")
    kern.dispatch(dev(q), dev(k), dev(v), None if mask is None else dev(mask), y, scale)
    torch.cuda.synchronize()
    np.testing.assert_allclose(y.cpu().numpy(), want, atol=5e-4)
    with pytest.raises(b200attn.B200RuntimeException, match="scale mismatch"):
        kern.dispatch(dev(q), dev(k), dev(v), None, y, scale * 2)


def test_encoder_additive_mask_fp16(ctx):
    import torch
    import b200attn
    B, H, S, D = 4, 3, 96, 64
    lens = [96, 40, 1, 70]
    q, k, v = (normal(400 + i, (B, H, S, D), oracle.F16) for i in range(3))
    mask = np.zeros((B, S), np.float32)
    for b, L in enumerate(lens):
        mask[b, L:] = -1e9
    scale = float(np.float32(1.0 / math.sqrt(D)))
    want = oracle.mha_additive(q, k, v, mask, B=B, H=H, S=S, D=D, scale=scale)
    y = torch.empty((B, H, S, D), device="cuda")
    b200attn.mha(ctx, to_dev(q, oracle.F16), to_dev(k, oracle.F16), to_dev(v, oracle.F16), y, scale,
                 mask=torch.from_numpy(mask).cuda())
    torch.cuda.synchronize()
    assert ctx.last_attention_kernel() == "tcgen05"  # 12 heads of 96 keys: packed work items, additive mask
    assert_close(to_np(y), want, what="additive mask")


def _rotate_rows(x, *, B, S, H, D, pos0, theta, mode):
    """The oracle's rotation of every [b, s] row block at position pos0 + s."""
    fn = oracle.rope_half_gemma if mode == "gemma" else oracle.rope_decoderonly
    out = np.empty_like(x)
    for b in range(B):
        for s in range(S):
            out[b, s] = fn(np.ascontiguousarray(x[b, s]).reshape(-1), H, D, pos0 + s, theta).reshape(H, D)
    return out


@pytest.mark.parametrize("dtype,mode", [(oracle.BF16, "neox"), (oracle.F16, "neox"), (oracle.F32, "neox"),
                                        (oracle.BF16, "gemma")])
def test_prefill_rotated_keys_out_and_rope_modes(ctx, dtype, mode):
    """k_rot_out receives the rotated keys in the input type (the reference's rotated cache rows), and the
    Gemma rotation (double products) matches the oracle's applyRopeHalf restatement."""
    import torch
    import b200attn
    B, S, Hq, Hkv, D, pos0, theta = 2, 70, 4, 2, 64, 5, 1e4
    q = normal(31, (B, S, Hq, D), dtype)
    k = normal(32, (B, S, Hkv, D), dtype)
    v = normal(33, (B, S, Hkv, D), dtype)
    scale = float(np.float32(1.0 / math.sqrt(D)))
    q_rot = _rotate_rows(q, B=B, S=S, H=Hq, D=D, pos0=pos0, theta=theta, mode=mode)
    k_rot = _rotate_rows(k, B=B, S=S, H=Hkv, D=D, pos0=pos0, theta=theta, mode=mode)
    want = oracle.prefill(q_rot, k_rot, v, B=B, S=S, Hq=Hq, Hkv=Hkv, D=D, scale=scale, rope_theta=0.0)
    tdt = getattr(torch, TORCH[dtype])
    o = torch.empty((B, S, Hq, D), dtype=torch.float32, device="cuda")
    kr = torch.empty((B, S, Hkv, D), dtype=tdt, device="cuda")
    b200attn.prefill_causal(ctx, to_dev(q, dtype), to_dev(k, dtype), to_dev(v, dtype), o, scale,
                            rope_mode=b200attn.ROPE_GEMMA if mode == "gemma" else b200attn.ROPE_NEOX,
                            rope_theta=theta, pos0=pos0, k_rot_out=kr)
    torch.cuda.synchronize()
    assert_close(to_np(o), want, what=f"prefill {mode} {TORCH[dtype]}")
    # rotated keys: the oracle rotation rounded to the input type, within one ulp of that type
    got_k = to_np(kr)
    want_k = oracle.round_to(k_rot, dtype)
    ulp = {oracle.F16: 2.0 ** -10, oracle.BF16: 2.0 ** -7, oracle.F32: 2.0 ** -23}[dtype]
    bound = ulp * np.maximum(np.abs(want_k), 2.0 ** -14)
    assert np.all(np.abs(got_k - want_k) <= bound), float(np.max(np.abs(got_k - want_k) - bound))


@pytest.mark.parametrize("layout,S,D", [(0, 100, 64), (1, 100, 64), (1, 300, 32), (0, 600, 64), (1, 100, 96),
                                          (0, 300, 96)])
def test_encoder_bf16_inputs(ctx, layout, S, D):
    """bf16 encoder inputs on the tensor cores: up to 512 keys the kernel converts the staged tiles to
    fp16 itself (its two spare warps); longer sequences go through the conversion pre-pass."""
    lens = [S, 37, 1, 64]
    got, want = _encoder_case(ctx, B=4, H=3, S=S, D=D, dtype=oracle.BF16, lens=lens, layout=layout, seed=600 + S)
    assert ctx.last_attention_kernel() == "tcgen05"
    assert_close(got, want, what=f"bf16 encoder S={S}")


def test_encoder_bf16_beyond_the_fp16_range_is_flagged(ctx):
    """A bf16 value beyond the fp16 operand range cannot be multiplied: the in-kernel conversion raises
    the device status (B2A_EDEVICE), as the conversion pre-pass does."""
    import torch
    import b200attn
    B, H, S, D = 1, 2, 64, 32
    q = torch.zeros(B, S, H, D, dtype=torch.bfloat16, device="cuda")
    q[0, 3, 1, 5] = 1e6
    y = torch.empty(B, S, H, D, device="cuda")
    b200attn.mha(ctx, q, q.clone(), q.clone(), y, 0.125, layout=b200attn.SEQ_MAJOR)
    with pytest.raises(b200attn.B200RuntimeException) as ei:
        ctx.check_device_status()
    assert ei.value.status == b200attn.B2A_EDEVICE
    assert "fp16 operand range" in str(ei.value)


@pytest.mark.parametrize("tensor,value,flagged", [
    ("q", 65536.0, True),    # rotated at position 0 (identity): rounds to infinity in fp16
    ("k", -65536.0, True),
    ("v", 65536.0, True),    # converted without rotation
    ("v", 65280.0, False),   # the largest bf16 value below fp16's limit stays finite
    ("q", -65280.0, False),
])
def test_prefill_prepass_flags_values_beyond_the_fp16_range(ctx, tensor, value, flagged):
    """The bf16 pre-pass (RoPE of q, k; conversion of q, k, v to the fp16 operands) raises the device
    status (B2A_EDEVICE) exactly when a finite value rounds to infinity in fp16."""
    import torch
    import b200attn
    B, S, H, D = 1, 256, 2, 64
    t = {n: torch.zeros(B, S, H, D, dtype=torch.bfloat16, device="cuda") for n in "qkv"}
    t[tensor][0, 0, 1, 5] = value
    y = torch.empty(B, S, H, D, device="cuda")
    ctx.check_device_status()
    b200attn.prefill_causal(ctx, t["q"], t["k"], t["v"], y, 0.125, rope_mode=b200attn.ROPE_NEOX, rope_theta=1e4)
    torch.cuda.synchronize()
    if not flagged:
        ctx.check_device_status()
        return
    with pytest.raises(b200attn.B200RuntimeException) as ei:
        ctx.check_device_status()
    assert ei.value.status == b200attn.B2A_EDEVICE
    assert "fp16 operand range" in str(ei.value)


@pytest.mark.parametrize("dtype,window,theta,S,D", [
    (oracle.BF16, 32, 1e4, 96, 256),    # Gemma-3-270M local layer (4/1 heads, D 256)
    (oracle.BF16, 0, 1e6, 96, 256),     # global layer
    (oracle.F16, 40, 1e4, 130, 128),    # a tensor-core head dim, ragged last tile
    (oracle.F32, 0, 1e6, 48, 256),      # fp32 end to end
    (oracle.F32, 40, 1e4, 150, 128),    # fp32 on the tiled fp32 kernel, window inside a key tile
    (oracle.BF16, 512, 1e4, 700, 256),  # local layer over several 128-row tiles (tensor cores, one tile per item)
    (oracle.F16, 0, 1e6, 600, 256),     # global layer, fp16
])
def test_prefill_gemma_batched_matches_oracle(ctx, dtype, window, theta, S, D):
    """b2a_prefill_gemma: QK-norm (zero-centred RMSNorm, (1 + w)) and applyRopeHalf of every
    position, then one causal attention launch with the local-layer window, against the
    oracle's restatement of the same steps with the Gemma softmax (double exp-sum)."""
    import torch
    import b200attn
    B, Hq, Hkv, pos0, eps = 2, 4, 1, 3, 1e-6
    q = normal(41, (B, S, Hq, D), dtype)
    k = normal(42, (B, S, Hkv, D), dtype)
    v = normal(43, (B, S, Hkv, D), dtype)
    qw = (normal(44, (D,), oracle.F32) * 0.5).astype(np.float32)
    kw = (normal(45, (D,), oracle.F32) * 0.5).astype(np.float32)
    scale = float(np.float32(1.0 / math.sqrt(256.0)))  # 1/sqrt(query_pre_attn_scalar)

    def norm_rope(x, H, w):
        out = np.empty_like(x)
        for b in range(B):
            for s in range(S):
                r = oracle.rmsnorm_zero_centered(np.ascontiguousarray(x[b, s]).reshape(-1), H, D, w, eps)
                out[b, s] = oracle.rope_half_gemma(r, H, D, pos0 + s, theta).reshape(H, D)
        return out

    q_r, k_r = norm_rope(q, Hq, qw), norm_rope(k, Hkv, kw)
    want = oracle.prefill(q_r, k_r, v, B=B, S=S, Hq=Hq, Hkv=Hkv, D=D, scale=scale, rope_theta=0.0, window=window,
                          softmax_mode=oracle.SOFTMAX_GEMMA)
    o = torch.empty((B, S, Hq, D), dtype=torch.float32, device="cuda")
    kr = torch.empty((B, S, Hkv, D), dtype=getattr(torch, TORCH[dtype]), device="cuda")
    b200attn.prefill_gemma(ctx, to_dev(q, dtype), to_dev(k, dtype), to_dev(v, dtype), o, scale,
                           q_norm_w=torch.from_numpy(qw).cuda(), k_norm_w=torch.from_numpy(kw).cuda(), norm_eps=eps,
                           rope_mode=b200attn.ROPE_GEMMA, rope_theta=theta, pos0=pos0, window=window, k_rot_out=kr)
    torch.cuda.synchronize()
    assert_close(to_np(o), want, atol=1e-4 if dtype == oracle.F32 else 2e-3, what=f"gemma prefill {TORCH[dtype]}")
    want_k = oracle.round_to(k_r, dtype)
    ulp = {oracle.F16: 2.0 ** -10, oracle.BF16: 2.0 ** -7, oracle.F32: 2.0 ** -23}[dtype]
    assert np.all(np.abs(to_np(kr) - want_k) <= ulp * np.maximum(np.abs(want_k), 2.0 ** -14))


def test_generic_kernel_key_split_back_to_back(ctx):
    """fp32 launches too small to fill the GPU split each query block's keys over several CTAs and merge
    the chunks; launches of different shapes run back to back without a synchronisation in between, so a
    per-block counter left non-zero, or a merge reading another launch's slots, would show here."""
    import torch
    import b200attn
    cases = []
    for i, (S, Hq, Hkv, D, window) in enumerate([(300, 6, 2, 48, 100), (256, 9, 3, 64, 0), (130, 2, 2, 40, 0)]):
        q = normal(700 + i, (1, S, Hq, D), oracle.F32)
        k = normal(710 + i, (1, S, Hkv, D), oracle.F32)
        v = normal(720 + i, (1, S, Hkv, D), oracle.F32)
        scale = float(np.float32(1.0 / math.sqrt(D)))
        want = oracle.prefill(q, k, v, B=1, S=S, Hq=Hq, Hkv=Hkv, D=D, scale=scale, rope_theta=1e4, window=window)
        o = torch.full((1, S, Hq, D), float("nan"), dtype=torch.float32, device="cuda")
        b200attn.prefill_causal(ctx, to_dev(q, oracle.F32), to_dev(k, oracle.F32), to_dev(v, oracle.F32), o, scale,
                                rope_mode=b200attn.ROPE_NEOX, rope_theta=1e4, window=window)
        cases.append((o, want, f"fp32 prefill S={S} D={D} window={window}"))
    lens = [200, 17, 1]
    shape = (3, 4, 200, 48)  # head-major encoder, fp32, key padding (head dim 48: the generic kernel)
    q, k, v = (normal(730 + j, shape, oracle.F32) for j in range(3))
    want = oracle.encoder_minilm(q, k, v, lens, B=3, H=4, S=200, D=48, layout=0)
    y = torch.full(shape, float("nan"), dtype=torch.float32, device="cuda")
    b200attn.mha(ctx, to_dev(q, oracle.F32), to_dev(k, oracle.F32), to_dev(v, oracle.F32), y,
                 float(np.float32(1.0 / math.sqrt(48))),
                 key_lengths=torch.from_numpy(np.asarray(lens, np.int32)).cuda(), layout=b200attn.HEAD_MAJOR)
    cases.append((y, want, "fp32 encoder, key lengths"))
    torch.cuda.synchronize()
    ctx.check_device_status()
    for got, want, what in cases:
        err, _ = assert_close(to_np(got), want, what=what)
        assert err < 1e-4, what  # fp32 end to end


def test_generic_kernel_runs_unsplit_without_room_for_the_split_workspace():
    """Under a context workspace limit too small for the key-split workspace, a launch that would split
    runs unsplit instead of failing, and its results are the same."""
    import torch
    import b200attn
    lens = [200, 60]
    shape = (2, 2, 200, 48)  # head-major fp32 encoder, head dim 48 (the generic kernel): would split
    q, k, v = (normal(760 + j, shape, oracle.F32) for j in range(3))
    want = oracle.encoder_minilm(q, k, v, lens, B=2, H=2, S=200, D=48, layout=0)
    with b200attn.Context(0) as small:
        small.set_workspace_limit(4096)
        y = torch.full(shape, float("nan"), dtype=torch.float32, device="cuda")
        b200attn.mha(small, to_dev(q, oracle.F32), to_dev(k, oracle.F32), to_dev(v, oracle.F32), y,
                     float(np.float32(1.0 / math.sqrt(48))),
                     key_lengths=torch.from_numpy(np.asarray(lens, np.int32)).cuda(), layout=b200attn.HEAD_MAJOR)
        torch.cuda.synchronize()
        small.check_device_status()
        assert small.last_attention_kernel() == "generic"
        assert small.workspace_bytes() <= 4096
        err, _ = assert_close(to_np(y), want, what="unsplit fp32 encoder under a workspace limit")
        assert err < 1e-4


def test_fp32_prefill_rotates_in_kernel_from_the_cached_table(ctx):
    """fp32 NeoX prefill runs as one launch that rotates q and k inside the attention kernel, from a
    float (cos, sin) table the context keeps across calls: a change of theta, of head dim and a position
    range beyond the cached one each rebuild it, and every result matches the oracle exactly enough for
    fp32 end to end."""
    import torch
    import b200attn
    for i, (S, Hq, Hkv, D, theta, pos0) in enumerate([(256, 9, 3, 64, 1e5, 0), (100, 4, 2, 64, 1e4, 300),
                                                      (300, 4, 1, 64, 1e5, 50), (90, 2, 2, 32, 1e5, 7),
                                                      (256, 9, 3, 64, 1e5, 0)]):
        q = normal(600 + i, (1, S, Hq, D), oracle.F32)
        k = normal(610 + i, (1, S, Hkv, D), oracle.F32)
        v = normal(620 + i, (1, S, Hkv, D), oracle.F32)
        scale = float(np.float32(1.0 / math.sqrt(D)))
        want = oracle.prefill(q, k, v, B=1, S=S, Hq=Hq, Hkv=Hkv, D=D, scale=scale, rope_theta=theta, pos0=pos0)
        o = torch.full((1, S, Hq, D), float("nan"), dtype=torch.float32, device="cuda")
        b200attn.prefill_causal(ctx, to_dev(q, oracle.F32), to_dev(k, oracle.F32), to_dev(v, oracle.F32), o, scale,
                                rope_mode=b200attn.ROPE_NEOX, rope_theta=theta, pos0=pos0)
        torch.cuda.synchronize()
        assert ctx.last_attention_kernel() == ("f32_tiled" if D in (64, 128) else "generic")
        err, _ = assert_close(to_np(o), want, what=f"fused-rope fp32 prefill {i}")
        assert err < 1e-4


# ------------------------------------------------------------------ fp32 tiled kernel
@pytest.mark.parametrize("D,S,window,pos0,rope", [(64, 200, 0, 0, True), (128, 333, 0, 17, True),
                                                   (64, 300, 100, 5, True), (128, 150, 40, 0, False),
                                                   (64, 1, 0, 0, True), (64, 1040, 0, 0, True)])
def test_fp32_tiled_causal_prefill(ctx, D, S, window, pos0, rope):
    """fp32 causal prefill on the tiled fp32 kernel (16 query rows per CTA, key tiles alternating between two
    warp halves): GQA, ragged last query block and key tile, a sliding window whose start moves inside a tile,
    a position offset into the rotation table, no RoPE, one row, and a sequence whose 17 key tiles give the
    halves unequal tile counts."""
    got, want = _prefill_case(ctx, B=2, S=S, Hq=6, Hkv=2, D=D, dtype=oracle.F32, out_dtype=oracle.F32,
                              theta=1e4, window=window, pos0=pos0, seed=900 + D + S, rope=rope)
    assert ctx.last_attention_kernel() == "f32_tiled"
    err, _ = assert_close(got, want, what=f"fp32 tiled prefill D={D} S={S} window={window}")
    assert err < 1e-4  # fp32 end to end


@pytest.mark.parametrize("out_dtype", [oracle.BF16, oracle.F16])
def test_fp32_tiled_prefill_16bit_output(ctx, out_dtype):
    """fp32 inputs with a 16-bit output: the tiled fp32 kernel rounds its fp32 result once on store."""
    got, want = _prefill_case(ctx, B=1, S=130, Hq=4, Hkv=2, D=64, dtype=oracle.F32, out_dtype=out_dtype,
                              theta=1e4, seed=970)
    assert ctx.last_attention_kernel() == "f32_tiled"
    ulp = 2.0 ** -8 if out_dtype == oracle.BF16 else 2.0 ** -11
    assert_close(got, want, atol=2e-3 + ulp * np.abs(want).max(), what=f"fp32 in, {TORCH[out_dtype]} out")


@pytest.mark.parametrize("layout,D,S", [(0, 64, 150), (1, 128, 77), (1, 64, 256)])
def test_fp32_tiled_encoder_key_lengths(ctx, layout, D, S):
    """Bidirectional fp32 encoder on the tiled kernel: key lengths of 0 (every key masked: the mean of V),
    1, a ragged one and the full sequence, in both layouts."""
    got, want = _encoder_case(ctx, B=4, H=3, S=S, D=D, dtype=oracle.F32, lens=[S, 0, 1, S // 2 + 3], layout=layout,
                              seed=950 + D)
    assert ctx.last_attention_kernel() == "f32_tiled"
    err, _ = assert_close(got, want, what=f"fp32 tiled encoder D={D} S={S}")
    assert err < 1e-4


def test_fp32_tiled_additive_mask(ctx):
    import torch
    import b200attn
    B, H, S, D = 3, 2, 130, 64
    q, k, v = (normal(980 + i, (B, H, S, D), oracle.F32) for i in range(3))
    mask = (normal(985, (B, S), oracle.F32) * 2.0).astype(np.float32)
    mask[1, 7:] = -1e9
    scale = float(np.float32(1.0 / math.sqrt(D)))
    want = oracle.mha_additive(q, k, v, mask, B=B, H=H, S=S, D=D, scale=scale)
    y = torch.full((B, H, S, D), float("nan"), device="cuda")
    b200attn.mha(ctx, to_dev(q, oracle.F32), to_dev(k, oracle.F32), to_dev(v, oracle.F32), y, scale,
                 mask=torch.from_numpy(mask).cuda())
    torch.cuda.synchronize()
    assert ctx.last_attention_kernel() == "f32_tiled"
    err, _ = assert_close(to_np(y), want, what="fp32 tiled additive mask")
    assert err < 1e-4
