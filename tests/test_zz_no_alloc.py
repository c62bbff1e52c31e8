"""b2a_decode_noalloc: the decode step for callers that cannot allocate.

Some hosts own all device memory through their own arena or caching pool (a
JVM or serving runtime); for them a cudaMalloc inside the library can fail or
stall the device.  This entry point takes no context and uses a static device
scratch instead.  The test calls it through the C ABI twice in a row and
checks both results against the regular b2a_decode on identical inputs, with
the parity tolerance used everywhere else (max abs 2e-3, cosine 0.9999).
It lives in its own file so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest

import oracle
from helpers import assert_close, normal, to_dev, to_np

pytestmark = pytest.mark.gpu


def _noalloc_fn():
    import b200attn
    f = b200attn.lib().b2a_decode_noalloc
    vp, i, fl, d = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_double
    f.argtypes = [i, i, i, vp, vp, vp, vp, vp, i, vp, i, i, i, i, i, fl, i, d, i, vp, vp, fl, vp, vp]
    f.restype = i
    return f


def _case(ctx, *, B, Hq, Hkv, D, max_seq, lens, layout, rope, theta, window, norm, seed):
    import torch
    import b200attn
    ptr = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
    q = to_dev(normal(seed, (B, Hq, D), oracle.F16), oracle.F16)
    kn = to_dev(normal(seed + 1, (B, Hkv, D), oracle.F16), oracle.F16)
    vn = to_dev(normal(seed + 2, (B, Hkv, D), oracle.F16), oracle.F16)
    shape = (B, Hkv, max_seq, D) if layout == b200attn.KV_HEAD_MAJOR else (B, max_seq, Hkv, D)
    kc0 = to_dev(normal(seed + 3, shape, oracle.F16), oracle.F16)
    vc0 = to_dev(normal(seed + 4, shape, oracle.F16), oracle.F16)
    lens_d = torch.tensor(lens, dtype=torch.int32, device="cuda")
    qw = kw = None
    if norm:
        qw = torch.from_numpy((0.5 * normal(seed + 5, (D,), oracle.F32)).astype(np.float32)).cuda()
        kw = torch.from_numpy((0.5 * normal(seed + 6, (D,), oracle.F32)).astype(np.float32)).cuda()
    scale = 1.0 / np.sqrt(D)

    ref = torch.empty(B, Hq, D, device="cuda")
    kc, vc = kc0.clone(), vc0.clone()
    b200attn.decode(ctx, q, kn, vn, kc, vc, lens_d, ref, scale, kv_layout=layout, rope_mode=rope, rope_theta=theta,
                    window=window, q_norm_w=qw, k_norm_w=kw)
    torch.cuda.synchronize()

    f = _noalloc_fn()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    outs = []
    kc2, vc2 = kc0.clone(), vc0.clone()
    for _ in range(2):  # two calls in a row share (and reuse) the static scratch
        out = torch.full((B, Hq, D), float("nan"), device="cuda")
        rc = f(oracle.F16, oracle.F16, oracle.F32, ptr(q), ptr(kn), ptr(vn), ptr(kc2), ptr(vc2), layout, ptr(lens_d),
               B, Hq, Hkv, D, max_seq, scale, rope, theta, window, ptr(qw), ptr(kw), 1e-6, ptr(out), stream)
        assert rc == b200attn.B2A_OK, rc
        torch.cuda.synchronize()
        outs.append(to_np(out))
    want = to_np(ref)
    for got in outs:
        assert_close(got, want, what="no-alloc decode vs b2a_decode")
    # the appended cache rows match too
    assert torch.equal(kc2, kc) and torch.equal(vc2, vc)


def test_noalloc_decode_matches_regular_decode_qwen_shape(ctx):
    import b200attn
    _case(ctx, B=6, Hq=14, Hkv=2, D=64, max_seq=3000, lens=[0, 63, 64, 1000, 2999, 1500],
          layout=b200attn.KV_HEAD_MAJOR, rope=b200attn.ROPE_NEOX, theta=1e6, window=0, norm=False, seed=901)


def test_noalloc_decode_matches_regular_decode_gemma_shape_long_context(ctx):
    # few long sequences: units are cut across many CTAs and merged through the scratch slots
    import b200attn
    _case(ctx, B=2, Hq=4, Hkv=1, D=256, max_seq=40000, lens=[39999, 20000], layout=b200attn.KV_POS_MAJOR,
          rope=b200attn.ROPE_GEMMA, theta=1e6, window=0, norm=True, seed=911)


def test_noalloc_decode_rejects_requests_beyond_the_scratch(ctx):
    import b200attn
    f = _noalloc_fn()
    dummy = ctypes.c_void_p(16)  # never dereferenced: the size check fails first
    rc = f(oracle.F16, oracle.F16, oracle.F32, dummy, dummy, dummy, dummy, dummy, 0, dummy,
           2048, 64, 16, 64, 128, 0.125, 0, 0.0, 0, None, None, 1e-6, dummy, None)
    assert rc == b200attn.B2A_EINVAL
    buf = ctypes.create_string_buffer(512)
    b200attn.lib().b2a_last_error(None, buf, 512)
    assert b"static scratch limit" in buf.value
