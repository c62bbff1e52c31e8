"""Decode parity: the CUDA decode step through the C ABI against the oracle.

Each case draws seeded inputs rounded to the cache dtype, runs
``b2a_decode`` (fused QK-norm + RoPE + KV append + split-KV attention) and
compares the output with ``oracle.decode`` (max abs <= 2e-3, cosine >=
0.9999) and the appended cache rows with the oracle's (one ulp of the cache
type); every other cache row must be untouched (bit-exact).
"""
import math

import numpy as np
import pytest

import oracle
from helpers import assert_close, normal, to_dev, to_np

pytestmark = pytest.mark.gpu


def _run_case(ctx, *, B, Hq, Hkv, D, max_seq, lens, cache_dtype=oracle.F16, q_dtype=oracle.F16,
              layout=oracle.KV_HEAD_MAJOR, rope_mode="neox", theta=1e6, window=0, qk_norm=False, seed=11,
              out_dtype=oracle.F32):
    import torch
    import b200attn
    lens = np.asarray(lens, np.int32)
    q = normal(seed, (B, Hq, D), q_dtype)
    kn = normal(seed + 1, (B, Hkv, D), q_dtype)
    vn = normal(seed + 2, (B, Hkv, D), q_dtype)
    shape = (B, Hkv, max_seq, D) if layout == oracle.KV_HEAD_MAJOR else (B, max_seq, Hkv, D)
    kc = normal(seed + 3, shape, cache_dtype)
    vc = normal(seed + 4, shape, cache_dtype)
    qw = kw = None
    if qk_norm:
        qw = (0.5 * normal(seed + 5, (D,), oracle.F32)).astype(np.float32)
        kw = (0.5 * normal(seed + 6, (D,), oracle.F32)).astype(np.float32)
    scale = float(np.float32(1.0 / np.sqrt(D)))
    orc_rope = oracle.ROPE_GEMMA if rope_mode == "gemma" else oracle.ROPE_DECODERONLY
    want, kc_want, vc_want = oracle.decode(
        q, kn, vn, kc, vc, lens, B=B, Hq=Hq, Hkv=Hkv, D=D, max_seq=max_seq, scale=scale,
        rope_theta=theta if rope_mode else 0.0, rope_mode=orc_rope, window=window, cache_layout=layout,
        cache_dtype=cache_dtype, q_norm_w=qw, k_norm_w=kw, norm_eps=1e-6,
        softmax_mode=oracle.SOFTMAX_GEMMA if rope_mode == "gemma" else oracle.SOFTMAX_DECODERONLY)

    kc_d, vc_d = to_dev(kc, cache_dtype), to_dev(vc, cache_dtype)
    out = torch.empty((B, Hq, D), dtype={oracle.F32: torch.float32, oracle.F16: torch.float16,
                                          oracle.BF16: torch.bfloat16}[out_dtype], device="cuda")
    b_rope = {None: b200attn.ROPE_NONE, "neox": b200attn.ROPE_NEOX, "gemma": b200attn.ROPE_GEMMA}[rope_mode]
    b200attn.decode(ctx, to_dev(q, q_dtype), to_dev(kn, q_dtype), to_dev(vn, q_dtype), kc_d, vc_d,
                    torch.from_numpy(lens).cuda(), out, scale,
                    kv_layout=b200attn.KV_HEAD_MAJOR if layout == oracle.KV_HEAD_MAJOR else b200attn.KV_POS_MAJOR,
                    rope_mode=b_rope, rope_theta=theta, window=window,
                    q_norm_w=None if qw is None else torch.from_numpy(qw).cuda(),
                    k_norm_w=None if kw is None else torch.from_numpy(kw).cuda(), norm_eps=1e-6)
    ctx.check_device_status()
    got = to_np(out)
    err, cos = assert_close(got, want, what="decode output")
    # appended rows: within one ulp of the cache type; everything else untouched
    kc_got, vc_got = to_np(kc_d), to_np(vc_d)
    ulp = {oracle.F16: 2 ** -10, oracle.BF16: 2 ** -7, oracle.F32: 2 ** -23}[cache_dtype]
    np.testing.assert_allclose(kc_got, kc_want, rtol=ulp, atol=1e-6)
    np.testing.assert_array_equal(vc_got, vc_want)
    return err, cos


def test_decode_qwen_shape_head_major(ctx):
    # configs[2] geometry (14/2 heads, D=64, theta 1e6) at a small batch
    lens = [0, 1, 63, 64, 65, 600, 699, 317]
    _run_case(ctx, B=8, Hq=14, Hkv=2, D=64, max_seq=700, lens=lens, theta=1e6)


def test_decode_qwen_shape_bf16_cache(ctx):
    _run_case(ctx, B=5, Hq=14, Hkv=2, D=64, max_seq=300, lens=[5, 128, 299, 0, 77], cache_dtype=oracle.BF16,
              q_dtype=oracle.BF16, seed=21)


@pytest.mark.parametrize("window,theta", [(512, 1e4), (0, 1e6)])
def test_decode_gemma_shape_local_and_global(ctx, window, theta):
    # configs[4] geometry: 4/1 heads, D=256, QK-norm, Gemma RoPE, position-major cache
    lens = [0, 511, 512, 513, 1500, 1999]
    _run_case(ctx, B=6, Hq=4, Hkv=1, D=256, max_seq=2000, lens=lens, layout=oracle.KV_POS_MAJOR,
              rope_mode="gemma", theta=theta, window=window, qk_norm=True, seed=31)


def test_decode_equal_units_take_whole_units_per_cta(ctx):
    """Every unit the same length (contexts past the window) and at least one unit per CTA: CTAs take
    whole units instead of cutting them (no partial slots, no merges). D = 64 (296 CTAs, 320 units) and a
    Gemma-local-shaped D = 256 case (148 CTAs, 150 units; QK-norm, Gemma RoPE)."""
    rng = np.random.default_rng(5)
    _run_case(ctx, B=160, Hq=4, Hkv=2, D=64, max_seq=320, lens=rng.integers(150, 319, 160), window=100, seed=81)
    _run_case(ctx, B=150, Hq=4, Hkv=1, D=256, max_seq=200, lens=rng.integers(64, 199, 150), window=64,
              layout=oracle.KV_POS_MAJOR, rope_mode="gemma", theta=1e4, qk_norm=True, seed=91)


def test_decode_batch_sizes_shrinking_and_growing_on_one_context(ctx):
    """The workspace's merge counters must stay zero between calls whatever the batch order: a large batch,
    then a small one whose partial slots must not land where a larger batch keeps counters, then a medium
    one, all with contexts long enough that units are split across CTAs and merged."""
    rng = np.random.default_rng(11)
    for i, B in enumerate([160, 4, 64]):
        _run_case(ctx, B=B, Hq=4, Hkv=2, D=64, max_seq=2048, lens=rng.integers(1000, 2047, B), seed=120 + i)


def test_decode_pos_major_multi_kv_head(ctx):
    _run_case(ctx, B=3, Hq=8, Hkv=2, D=128, max_seq=400, lens=[10, 399, 200], layout=oracle.KV_POS_MAJOR, seed=41)


def test_decode_more_than_eight_heads_per_kv_head(ctx):
    _run_case(ctx, B=2, Hq=16, Hkv=1, D=128, max_seq=300, lens=[150, 299], seed=51)


def test_decode_mha_head_dim_96(ctx):
    _run_case(ctx, B=3, Hq=4, Hkv=4, D=96, max_seq=260, lens=[0, 100, 259], seed=61)


def test_decode_long_sequence_splits_and_merges(ctx):
    # few sequences with long contexts force many chunks per sequence and the log-sum-exp merge
    _run_case(ctx, B=2, Hq=7, Hkv=1, D=64, max_seq=40000, lens=[39999, 3], seed=71)


def test_decode_no_rope(ctx):
    _run_case(ctx, B=2, Hq=4, Hkv=2, D=64, max_seq=100, lens=[50, 99], rope_mode=None, seed=81)


def test_decode_fp16_output(ctx):
    _run_case(ctx, B=4, Hq=14, Hkv=2, D=64, max_seq=500, lens=[1, 2, 400, 499], out_dtype=oracle.F16, seed=91)


def test_decode_generic_kernel_float32_cache(ctx):
    # float32 caches and head_dim 8 take the generic warp-per-head kernel
    _run_case(ctx, B=3, Hq=2, Hkv=1, D=8, max_seq=40, lens=[0, 17, 39], cache_dtype=oracle.F32,
              q_dtype=oracle.F32, theta=1e4, seed=101)


def test_decode_generic_kernel_odd_head_dim(ctx):
    _run_case(ctx, B=2, Hq=6, Hkv=3, D=48, max_seq=90, lens=[33, 89], seed=111)


def test_decode_rejects_out_of_range_ctx_len(ctx):
    import torch
    import b200attn
    B, Hq, Hkv, D, S = 2, 2, 1, 64, 16
    z = lambda *s: torch.zeros(*s, dtype=torch.float16, device="cuda")
    out = torch.zeros(B, Hq, D, device="cuda")
    lens = torch.tensor([3, 16], dtype=torch.int32, device="cuda")  # 16 == max_seq: invalid
    b200attn.decode(ctx, z(B, Hq, D), z(B, Hkv, D), z(B, Hkv, D), z(B, Hkv, S, D), z(B, Hkv, S, D), lens, out,
                    0.125)
    with pytest.raises(b200attn.B200RuntimeException, match="B2A_EDEVICE"):
        ctx.check_device_status()
    o = out.cpu().numpy()
    assert np.all(np.isnan(o[1])) and np.all(np.isfinite(o[0]))


def test_decode_argument_validation(ctx):
    import torch
    import b200attn
    z = lambda *s: torch.zeros(*s, dtype=torch.float16, device="cuda")
    lens = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError, match="divisible"):
        b200attn.decode(ctx, z(1, 14, 64), z(1, 3, 64), z(1, 3, 64), z(1, 3, 8, 64), z(1, 3, 8, 64), lens,
                        torch.zeros(1, 14, 64, device="cuda"), 0.125)
    with pytest.raises(ValueError, match="together"):
        b200attn.decode(ctx, z(1, 2, 64), z(1, 1, 64), z(1, 1, 64), z(1, 1, 8, 64), z(1, 1, 8, 64), lens,
                        torch.zeros(1, 2, 64, device="cuda"), 0.125, q_norm_w=torch.ones(64, device="cuda"))


def test_decode_full_size_qwen_config(ctx):
    """configs[2] at full size: B=64, 14/2, D=64, fp16 cache, ctx ~ U[512, 8192]."""
    lens = oracle.splitmix_uniform_int(3, 64, 512, 8192)
    _run_case(ctx, B=64, Hq=14, Hkv=2, D=64, max_seq=8193, lens=lens, theta=1e6, seed=3000)


def _long_context_case(ctx, *, lens, Hq, Hkv, D, max_seq, layout, rope_mode, theta, window, qk_norm, seed,
                       q_dtype=oracle.F16, cache_dtype=oracle.F16):
    """Parity at the benchmarked context lengths.  The caches are too large for the splitmix generator
    and for whole-cache comparisons, so they are drawn with numpy's seeded normal generator (rounded to
    the cache type), the output is compared with the oracle, the appended rows are compared within one
    ulp, and every other row is checked unchanged through a per-sequence checksum."""
    import torch
    import b200attn
    B = len(lens)
    lens = np.asarray(lens, np.int32)
    rng = np.random.default_rng(seed)
    q = normal(seed, (B, Hq, D), q_dtype)
    kn = normal(seed + 1, (B, Hkv, D), q_dtype)
    vn = normal(seed + 2, (B, Hkv, D), q_dtype)
    shape = (B, Hkv, max_seq, D) if layout == oracle.KV_HEAD_MAJOR else (B, max_seq, Hkv, D)
    assert cache_dtype == oracle.F16  # numpy's float16 cast rounds to nearest even, as the cache type does
    kc = rng.standard_normal(shape, dtype=np.float32).astype(np.float16).astype(np.float32)
    vc = rng.standard_normal(shape, dtype=np.float32).astype(np.float16).astype(np.float32)
    qw = kw = None
    if qk_norm:
        qw = (0.5 * normal(seed + 5, (D,), oracle.F32)).astype(np.float32)
        kw = (0.5 * normal(seed + 6, (D,), oracle.F32)).astype(np.float32)
    kc_d, vc_d = to_dev(kc, cache_dtype), to_dev(vc, cache_dtype)
    sums_before = [(kc_d[b].double().sum().item(), vc_d[b].double().sum().item()) for b in range(B)]
    scale = float(np.float32(1.0 / np.sqrt(D)))
    out = torch.empty((B, Hq, D), dtype=torch.float32, device="cuda")
    b200attn.decode(ctx, to_dev(q, q_dtype), to_dev(kn, q_dtype), to_dev(vn, q_dtype), kc_d, vc_d,
                    torch.from_numpy(lens).cuda(), out, scale,
                    kv_layout=b200attn.KV_HEAD_MAJOR if layout == oracle.KV_HEAD_MAJOR else b200attn.KV_POS_MAJOR,
                    rope_mode=b200attn.ROPE_GEMMA if rope_mode == "gemma" else b200attn.ROPE_NEOX,
                    rope_theta=theta, window=window,
                    q_norm_w=None if qw is None else torch.from_numpy(qw).cuda(),
                    k_norm_w=None if kw is None else torch.from_numpy(kw).cuda(), norm_eps=1e-6)
    ctx.check_device_status()
    # the oracle appends in place into the host caches (the device copies were taken above)
    old_rows = [(kc[b, :, L].copy(), vc[b, :, L].copy()) if layout == oracle.KV_HEAD_MAJOR else
                (kc[b, L].copy(), vc[b, L].copy()) for b, L in enumerate(lens)]
    want, _, _ = oracle.decode(
        q, kn, vn, kc, vc, lens, B=B, Hq=Hq, Hkv=Hkv, D=D, max_seq=max_seq, scale=scale, rope_theta=theta,
        rope_mode=oracle.ROPE_GEMMA if rope_mode == "gemma" else oracle.ROPE_DECODERONLY, window=window,
        cache_layout=layout, cache_dtype=cache_dtype, q_norm_w=qw, k_norm_w=kw, norm_eps=1e-6,
        softmax_mode=oracle.SOFTMAX_GEMMA if rope_mode == "gemma" else oracle.SOFTMAX_DECODERONLY, inplace=True)
    err, cos = assert_close(to_np(out), want, what="long-context decode output")
    ulp = {oracle.F16: 2 ** -10, oracle.BF16: 2 ** -7}[cache_dtype]
    for b, L in enumerate(lens):
        if layout == oracle.KV_HEAD_MAJOR:
            got_k, got_v, want_k, want_v = to_np(kc_d[b, :, L]), to_np(vc_d[b, :, L]), kc[b, :, L], vc[b, :, L]
        else:
            got_k, got_v, want_k, want_v = to_np(kc_d[b, L]), to_np(vc_d[b, L]), kc[b, L], vc[b, L]
        np.testing.assert_allclose(got_k, want_k, rtol=ulp, atol=1e-6)
        np.testing.assert_array_equal(got_v, want_v)
        # rows other than L unchanged: the sequence's sum moved by exactly (new row - old row)
        dk = float(got_k.astype(np.float64).sum() - old_rows[b][0].astype(np.float64).sum())
        dv = float(got_v.astype(np.float64).sum() - old_rows[b][1].astype(np.float64).sum())
        assert abs(kc_d[b].double().sum().item() - (sums_before[b][0] + dk)) < 1e-6
        assert abs(vc_d[b].double().sum().item() - (sums_before[b][1] + dv)) < 1e-6
    return err, cos


@pytest.mark.parametrize("window,theta", [(512, 1e4), (0, 1e6)])
def test_decode_gemma_config_full_context_range(ctx, window, theta):
    """configs[4] at its real context lengths: 12 of the benchmark's sequences (contexts drawn from
    U[1024, 32768] with the bench seed, the shortest and longest among them) plus one at the maximum
    32768, 4/1 heads, D = 256, QK-norm, Gemma RoPE, fp16 position-major cache; the local W512 / theta 1e4
    layer and the global theta 1e6 layer."""
    all_lens = oracle.splitmix_uniform_int(5, 256, 1024, 32768)
    order = np.argsort(all_lens)
    pick = order[np.linspace(0, 255, 12).astype(int)]
    lens = np.concatenate([all_lens[pick], [32768]]).astype(np.int32)
    _long_context_case(ctx, lens=lens, Hq=4, Hkv=1, D=256, max_seq=32769, layout=oracle.KV_POS_MAJOR,
                       rope_mode="gemma", theta=theta, window=window, qk_norm=True, seed=5000 + window)


def test_decode_qwen_config_longest_contexts(ctx):
    """configs[2] geometry at the top of its context range, 8192 included (14/2 heads, D = 64,
    head-major fp16 cache, NeoX RoPE theta 1e6)."""
    lens = np.array([8192, 8191, 7000, 512, 4096, 8000], np.int32)
    _long_context_case(ctx, lens=lens, Hq=14, Hkv=2, D=64, max_seq=8193, layout=oracle.KV_HEAD_MAJOR,
                       rope_mode="neox", theta=1e6, window=0, qk_norm=False, seed=5100)


def test_decode_early_start_layers_back_to_back(ctx):
    """b2a_set_decode_early_start: a chain of decode layers (each with its own caches, as in a model
    step; Qwen-shaped head-major and Gemma-shaped position-major with QK-norm) launched directly and
    replayed from a CUDA graph gives the same bits as the same chain without early start, and the
    first layer equals the oracle."""
    import torch
    import b200attn
    L, B, S = 4, 24, 1200
    lens = torch.from_numpy(np.asarray([(37 * i * i + 11) % (S - 1) for i in range(B)], np.int32)).cuda()
    cases = []
    for name, Hq, Hkv, D, layout, rope, norm in (("qwen", 14, 2, 64, b200attn.KV_HEAD_MAJOR, b200attn.ROPE_NEOX, False),
                                                 ("gemma", 4, 1, 256, b200attn.KV_POS_MAJOR, b200attn.ROPE_GEMMA, True)):
        shape = (B, Hkv, S, D) if layout == b200attn.KV_HEAD_MAJOR else (B, S, Hkv, D)
        layers = []
        for l in range(L):
            seed = 1500 + 10 * l + (0 if name == "qwen" else 500)
            q, kn, vn = (to_dev(normal(seed + i, s, oracle.F16), oracle.F16)
                         for i, s in enumerate([(B, Hq, D), (B, Hkv, D), (B, Hkv, D)]))
            kc, vc = to_dev(normal(seed + 3, shape, oracle.F16), oracle.F16), to_dev(normal(seed + 4, shape, oracle.F16), oracle.F16)
            layers.append(dict(q=q, kn=kn, vn=vn, kc=kc, vc=vc, out=torch.empty((B, Hq, D), device="cuda")))
        qw = torch.from_numpy((0.5 * normal(1590, (D,), oracle.F32)).astype(np.float32)).cuda() if norm else None
        kw = torch.from_numpy((0.5 * normal(1591, (D,), oracle.F32)).astype(np.float32)).cuda() if norm else None
        cases.append((name, Hq, Hkv, D, layout, rope, layers, qw, kw))

    def chain(case):
        name, Hq, Hkv, D, layout, rope, layers, qw, kw = case
        for l, t in enumerate(layers):
            b200attn.decode(ctx, t["q"], t["kn"], t["vn"], t["kc"], t["vc"], lens, t["out"], 1.0 / math.sqrt(D),
                            kv_layout=layout, rope_mode=rope, rope_theta=1e4 if l % 2 else 1e6,
                            window=512 if (name == "gemma" and l % 2) else 0, q_norm_w=qw, k_norm_w=kw,
                            norm_eps=1e-6)

    for case in cases:
        layers = case[6]
        ctx.set_decode_early_start(False)
        chain(case)
        torch.cuda.synchronize()
        ctx.check_device_status()
        ref = [t["out"].clone() for t in layers]
        try:
            ctx.set_decode_early_start(True)
            for t in layers:
                t["out"].fill_(float("nan"))
            chain(case)  # direct launches
            torch.cuda.synchronize()
            ctx.check_device_status()
            for l, t in enumerate(layers):
                assert torch.equal(t["out"], ref[l]), f"{case[0]} layer {l}: early start changed the output"
            for t in layers:
                t["out"].fill_(float("nan"))
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(s):
                with torch.cuda.graph(g, stream=s):
                    chain(case)
            torch.cuda.current_stream().wait_stream(s)
            for _ in range(3):
                g.replay()
            torch.cuda.synchronize()
            ctx.check_device_status()
            for l, t in enumerate(layers):
                assert torch.equal(t["out"], ref[l]), f"{case[0]} layer {l}: graph replay with early start differs"
            del g
        finally:
            ctx.set_decode_early_start(False)
    # the first Qwen layer against the oracle (the chain's caches have the new rows appended; the
    # oracle's append writes the same rows, so it starts from the appended caches as well)
    name, Hq, Hkv, D, layout, rope, layers, qw, kw = cases[0]
    t = layers[0]
    want, _, _ = oracle.decode(to_np(t["q"]), to_np(t["kn"]), to_np(t["vn"]), to_np(t["kc"]), to_np(t["vc"]),
                               lens.cpu().numpy(), B=B, Hq=Hq, Hkv=Hkv, D=D, max_seq=S,
                               scale=float(np.float32(1.0 / math.sqrt(D))), rope_theta=1e6,
                               rope_mode=oracle.ROPE_DECODERONLY, cache_layout=oracle.KV_HEAD_MAJOR,
                               cache_dtype=oracle.F16)
    assert_close(to_np(t["out"]), want, what="early-start chain, layer 0 against the oracle")
