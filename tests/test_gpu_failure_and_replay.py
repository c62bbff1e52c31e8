"""Failure detection without a GPU fault, and launches that reuse device state.

* A bounded wait inside the tensor-core prefill kernel is made to run out (the test
  hook of include/b200attn_testing.h leaves one K/V copy unissued): the launch
  returns, the device status reports it (B2A_ETIMEOUT), and the same context then
  computes correct results -- also when the next launch comes before anyone read
  the status.  The AttentionKernel mirror raises at the dispatch (or when its
  GpuBatch closes) instead of returning undefined output.
* A decode whose workspace would exceed the context's limit fails with B2A_EOOM.
* The persistent prefill takes work items from a counter that its last CTA resets:
  back-to-back launches with different item counts, and CUDA-graph replays of one
  launch, must each compute every item.
* Decode replays from a CUDA graph recompute the step (its split-merge counters are
  reset by the last piece of each unit).
"""
import math

import numpy as np
import pytest

import oracle
from helpers import assert_close, normal, to_dev, to_np

pytestmark = pytest.mark.gpu


def _prefill_inputs(B, S, Hq, Hkv, D, seed):
    q = normal(seed, (B, S, Hq, D), oracle.F16)
    k = normal(seed + 1, (B, S, Hkv, D), oracle.F16)
    v = normal(seed + 2, (B, S, Hkv, D), oracle.F16)
    scale = float(np.float32(1.0 / math.sqrt(D)))
    want = oracle.prefill(q, k, v, B=B, S=S, Hq=Hq, Hkv=Hkv, D=D, scale=scale, rope_theta=1e4)
    return q, k, v, scale, want


def test_bounded_wait_timeout_is_reported_and_the_context_stays_usable(ctx):
    import torch
    import b200attn
    B, S, Hq, Hkv, D = 1, 512, 2, 2, 64  # fp16, head dim 64: the tcgen05 kernel
    q, k, v, scale, want = _prefill_inputs(B, S, Hq, Hkv, D, seed=31)
    qd, kd, vd = to_dev(q, oracle.F16), to_dev(k, oracle.F16), to_dev(v, oracle.F16)
    o = torch.empty((B, S, Hq, D), dtype=torch.float32, device="cuda")
    ctx.check_device_status()  # nothing pending from earlier tests
    ctx.inject_wait_timeout()
    b200attn.prefill_causal(ctx, qd, kd, vd, o, scale, rope_mode=b200attn.ROPE_NEOX, rope_theta=1e4)
    torch.cuda.synchronize()  # the launch ends: its roles gave up after the bounded wait
    with pytest.raises(b200attn.B200RuntimeException) as ei:
        ctx.check_device_status()
    assert ei.value.status == b200attn.B2A_ETIMEOUT
    assert "bounded device wait ran out" in str(ei.value)
    ctx.check_device_status()  # reading the status cleared it
    # the context, its workspaces and the work-item counter are intact
    o.zero_()
    b200attn.prefill_causal(ctx, qd, kd, vd, o, scale, rope_mode=b200attn.ROPE_NEOX, rope_theta=1e4)
    torch.cuda.synchronize()
    ctx.check_device_status()
    assert_close(to_np(o), want, what="prefill after a timed-out launch")


def test_launch_after_a_timed_out_one_runs_normally_before_the_status_is_read(ctx):
    """The abort of a timed-out launch is per launch: the next launch, queued before anyone read the
    status, computes every item; the timeout is still reported afterwards."""
    import torch
    import b200attn
    B, S, Hq, Hkv, D = 2, 640, 4, 2, 96
    q, k, v, scale, want = _prefill_inputs(B, S, Hq, Hkv, D, seed=37)
    qd, kd, vd = to_dev(q, oracle.F16), to_dev(k, oracle.F16), to_dev(v, oracle.F16)
    o1 = torch.empty((B, S, Hq, D), dtype=torch.float32, device="cuda")
    o2 = torch.full((B, S, Hq, D), float("nan"), dtype=torch.float32, device="cuda")
    ctx.check_device_status()
    ctx.inject_wait_timeout()
    b200attn.prefill_causal(ctx, qd, kd, vd, o1, scale, rope_mode=b200attn.ROPE_NEOX, rope_theta=1e4)
    b200attn.prefill_causal(ctx, qd, kd, vd, o2, scale, rope_mode=b200attn.ROPE_NEOX, rope_theta=1e4)
    torch.cuda.synchronize()
    assert_close(to_np(o2), want, what="launch queued behind a timed-out one")
    with pytest.raises(b200attn.B200RuntimeException) as ei:
        ctx.check_device_status()
    assert ei.value.status == b200attn.B2A_ETIMEOUT


def test_attention_kernel_dispatch_raises_on_a_device_timeout(ctx):
    """CudaAttentionKernel.dispatch outside a batch waits and raises (the reference's dispatch waits on
    its fence); inside a GpuBatch the dispatch returns and the batch's close raises."""
    import torch
    import b200attn
    B, H, S, D = 1, 2, 256, 64  # fp16 head-major, head dim 64: the tcgen05 kernel
    shape = (B, H, S, D)
    q, k, v = (to_dev(normal(80 + i, shape, oracle.F16), oracle.F16) for i in range(3))
    y = torch.empty(shape, dtype=torch.float32, device="cuda")
    kern = b200attn.CudaAttentionKernel(ctx, B, H, S, D, 0.125, False)
    ctx.check_device_status()
    ctx.inject_wait_timeout()
    with pytest.raises(b200attn.B200RuntimeException) as ei:
        kern.dispatch(q, k, v, None, y, 0.125)
    assert ei.value.status == b200attn.B2A_ETIMEOUT
    kern.dispatch(q, k, v, None, y, 0.125)  # the context recovered
    ctx.inject_wait_timeout()
    with pytest.raises(b200attn.B200RuntimeException) as ei:
        with b200attn.GpuBatch.begin(ctx):
            kern.dispatch(q, k, v, None, y, 0.125)  # returns at once
            with b200attn.GpuBatch.begin(ctx):  # nested: shares the outer batch
                kern.dispatch(q, k, v, None, y, 0.125)
    assert ei.value.status == b200attn.B2A_ETIMEOUT
    assert b200attn.GpuBatch.current() is None
    ctx.check_device_status()


def test_decode_workspace_beyond_the_context_limit_is_b2a_eoom():
    """The decode's split workspace counts against the context's cap: a cap below it fails the call with
    B2A_EOOM (the reference has no cap; its allocation failures surface as DirectMlRuntimeException)."""
    import torch
    import b200attn
    B, Hq, Hkv, D, S = 4, 8, 2, 64, 256
    z = lambda *s: torch.zeros(*s, dtype=torch.float16, device="cuda")
    lens = torch.full((B,), 100, dtype=torch.int32, device="cuda")
    out = torch.empty(B, Hq, D, device="cuda")
    with b200attn.Context(0) as small:
        small.set_workspace_limit(1024)
        with pytest.raises(b200attn.B200RuntimeException) as ei:
            b200attn.decode(small, z(B, Hq, D), z(B, Hkv, D), z(B, Hkv, D), z(B, Hkv, S, D), z(B, Hkv, S, D), lens,
                            out, 0.125)
        assert ei.value.status == b200attn.B2A_EOOM
        assert "exceeds the context limit" in str(ei.value)
        assert small.workspace_bytes() <= 1024
        small.set_workspace_limit(0)  # no cap: the same call runs
        b200attn.decode(small, z(B, Hq, D), z(B, Hkv, D), z(B, Hkv, D), z(B, Hkv, S, D), z(B, Hkv, S, D), lens,
                        out, 0.125)
        small.check_device_status()


def test_persistent_prefill_back_to_back_launches_with_different_item_counts(ctx):
    import torch
    import b200attn
    shapes = [(1, 640, 4, 4, 64), (2, 384, 2, 1, 96), (1, 640, 4, 4, 64), (3, 256, 2, 2, 128)]
    runs = []
    for i, (B, S, Hq, Hkv, D) in enumerate(shapes):
        q, k, v, scale, want = _prefill_inputs(B, S, Hq, Hkv, D, seed=41 + 5 * i)
        o = torch.full((B, S, Hq, D), float("nan"), dtype=torch.float32, device="cuda")
        b200attn.prefill_causal(ctx, to_dev(q, oracle.F16), to_dev(k, oracle.F16), to_dev(v, oracle.F16), o, scale,
                                rope_mode=b200attn.ROPE_NEOX, rope_theta=1e4)
        runs.append((o, want))  # no synchronisation between the launches
    torch.cuda.synchronize()
    ctx.check_device_status()
    for i, (o, want) in enumerate(runs):
        assert_close(to_np(o), want, what=f"back-to-back prefill {i}")


def test_persistent_prefill_graph_replays_recompute_every_item(ctx):
    import torch
    import b200attn
    B, S, Hq, Hkv, D = 2, 512, 4, 2, 96
    q, k, v, scale, want = _prefill_inputs(B, S, Hq, Hkv, D, seed=61)
    qd, kd, vd = to_dev(q, oracle.F16), to_dev(k, oracle.F16), to_dev(v, oracle.F16)
    o = torch.empty((B, S, Hq, D), dtype=torch.float32, device="cuda")
    run = lambda: b200attn.prefill_causal(ctx, qd, kd, vd, o, scale, rope_mode=b200attn.ROPE_NEOX, rope_theta=1e4)
    run()  # workspaces reach their final size before capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
        run()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    for rep in range(3):
        o.fill_(float("nan"))  # a replay that skipped items would leave NaN behind
        g.replay()
        torch.cuda.synchronize()
        assert_close(to_np(o), want, what=f"graph replay {rep}")
    del g
    ctx.check_device_status()


def test_decode_graph_replays_recompute_the_step(ctx):
    import torch
    import b200attn
    B, Hq, Hkv, D, max_seq = 6, 14, 2, 64, 3000
    lens = np.array([5, 2900, 17, 1200, 2999, 640], np.int32)
    q = normal(71, (B, Hq, D), oracle.F16)
    kn, vn = normal(72, (B, Hkv, D), oracle.F16), normal(73, (B, Hkv, D), oracle.F16)
    kc, vc = normal(74, (B, Hkv, max_seq, D), oracle.F16), normal(75, (B, Hkv, max_seq, D), oracle.F16)
    scale = float(np.float32(1.0 / math.sqrt(D)))
    want, _, _ = oracle.decode(q, kn, vn, kc, vc, lens, B=B, Hq=Hq, Hkv=Hkv, D=D, max_seq=max_seq, scale=scale,
                               rope_theta=1e6, rope_mode=oracle.ROPE_DECODERONLY, window=0,
                               cache_layout=oracle.KV_HEAD_MAJOR, cache_dtype=oracle.F16,
                               softmax_mode=oracle.SOFTMAX_DECODERONLY)
    qd, knd, vnd = to_dev(q, oracle.F16), to_dev(kn, oracle.F16), to_dev(vn, oracle.F16)
    kcd, vcd = to_dev(kc, oracle.F16), to_dev(vc, oracle.F16)
    lens_d = torch.from_numpy(lens).cuda()
    out = torch.empty((B, Hq, D), dtype=torch.float32, device="cuda")
    run = lambda: b200attn.decode(ctx, qd, knd, vnd, kcd, vcd, lens_d, out, scale, kv_layout=b200attn.KV_HEAD_MAJOR,
                                  rope_mode=b200attn.ROPE_NEOX, rope_theta=1e6)
    run()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
        run()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    for rep in range(3):  # the appended row is the same every time, so every replay has one answer
        out.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        assert_close(to_np(out), want, what=f"decode graph replay {rep}")
    del g
    ctx.check_device_status()
