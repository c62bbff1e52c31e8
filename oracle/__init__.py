"""CPU parity oracle for the attention hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline / reference
arm of ``bench.py`` may import this package.  The product library
(``win-directml-java_b200``) never calls it and has no CPU fallback.

Contents
--------
* ctypes bindings to ``liboracle.so`` (the C restatement in ``attn_oracle.c``
  of the reference's Java CPU attention; see that file for the citations);
* :class:`JavaRandom`, a port of ``java.util.Random``'s documented 48-bit LCG
  (``nextInt``, ``nextInt(bound)``, ``nextFloat``, ``nextDouble``) so the
  reference tests' seeded inputs (``new Random(42)`` ...) can be regenerated;
* :func:`splitmix_normal`, the seeded splitmix64 + Box-Muller N(0,1) generator
  used for the benchmark-shaped synthetic inputs;
* dtype rounding helpers (round-to-nearest-even to fp16 / bf16).
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

F32, F16, BF16 = 0, 1, 2
SOFTMAX_DECODERONLY, SOFTMAX_GEMMA = 0, 1
ROPE_DECODERONLY, ROPE_GEMMA = 0, 1
KV_HEAD_MAJOR, KV_POS_MAJOR = 0, 1

_fp = ctypes.POINTER(ctypes.c_float)
_ip = ctypes.POINTER(ctypes.c_int32)


def build() -> str:
    """Compile liboracle.so with the committed Makefile (system gcc + OpenMP)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
                os.path.join(_HERE, "attn_oracle.c")):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.orc_f32_to_f16_bits.restype = ctypes.c_uint16
        L.orc_f32_to_f16_bits.argtypes = [ctypes.c_float]
        L.orc_f16_bits_to_f32.restype = ctypes.c_float
        L.orc_f16_bits_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_f32_to_bf16_bits.restype = ctypes.c_uint16
        L.orc_f32_to_bf16_bits.argtypes = [ctypes.c_float]
        L.orc_round_to.restype = ctypes.c_float
        L.orc_round_to.argtypes = [ctypes.c_float, ctypes.c_int]
        L.orc_round_array.argtypes = [_fp, ctypes.c_int64, ctypes.c_int]
        L.orc_rope_decoderonly.argtypes = [_fp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_double]
        L.orc_rope_half_gemma.argtypes = [_fp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_double]
        L.orc_rmsnorm_zero_centered.argtypes = [_fp, ctypes.c_int, ctypes.c_int, _fp, ctypes.c_float]
        L.orc_softmax_decoderonly.argtypes = [_fp, ctypes.c_int]
        L.orc_prefill.restype = ctypes.c_int
        L.orc_prefill.argtypes = [_fp, _fp, _fp, _fp] + [ctypes.c_int] * 5 + [
            ctypes.c_float, ctypes.c_double] + [ctypes.c_int] * 6
        L.orc_decode.restype = ctypes.c_int
        L.orc_decode.argtypes = [_fp, _fp, _fp, _fp, _fp, ctypes.c_int, ctypes.c_int, _ip] + [
            ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_double, ctypes.c_int, ctypes.c_int, _fp, _fp,
                                 ctypes.c_float, ctypes.c_int, ctypes.c_int, _fp, ctypes.c_int]
        L.orc_attend_cache.restype = ctypes.c_int
        L.orc_attend_cache.argtypes = [_fp, _fp, _fp, ctypes.c_int, _ip] + [ctypes.c_int] * 5 + [
            ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int, _fp, ctypes.c_int]
        L.orc_encoder_minilm.restype = ctypes.c_int
        L.orc_encoder_minilm.argtypes = [_fp, _fp, _fp, _ip, _fp] + [ctypes.c_int] * 6
        L.orc_mha_additive.restype = ctypes.c_int
        L.orc_mha_additive.argtypes = [_fp, _fp, _fp, _fp, _fp] + [ctypes.c_int] * 4 + [ctypes.c_float,
                                                                                       ctypes.c_int]
        L.orc_kv_head_for_query_head.restype = ctypes.c_int
        L.orc_kv_head_for_query_head.argtypes = [ctypes.c_int] * 3
        L.orc_first_valid_key.restype = ctypes.c_int
        L.orc_first_valid_key.argtypes = [ctypes.c_int] * 3
        L.orc_max_threads.restype = ctypes.c_int
        L.orc_is_full_attention_layer.restype = ctypes.c_int
        L.orc_is_full_attention_layer.argtypes = [ctypes.c_int, ctypes.c_int]
        L.orc_rope_theta_for_layer.restype = ctypes.c_double
        L.orc_rope_theta_for_layer.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_double, ctypes.c_double]
        L.orc_attention_scale.restype = ctypes.c_float
        L.orc_attention_scale.argtypes = [ctypes.c_double, ctypes.c_int]
        _lib = L
    return _lib


def _f(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_fp)


def _i(a: np.ndarray):
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(_ip)


# --------------------------------------------------------------------------
# dtype rounding
# --------------------------------------------------------------------------
def round_to(x: np.ndarray, dtype: int) -> np.ndarray:
    """Round float32 values to fp16/bf16 (RNE) and widen back to float32."""
    out = np.ascontiguousarray(x, dtype=np.float32).copy()
    lib().orc_round_array(_f(out), out.size, dtype)
    return out


# --------------------------------------------------------------------------
# java.util.Random (the documented 48-bit linear congruential generator)
# --------------------------------------------------------------------------
class JavaRandom:
    """Port of ``java.util.Random`` as specified in its Javadoc.

    seed scrambling ``(seed ^ 0x5DEECE66D) & (2^48-1)``; ``next(bits)`` steps
    ``seed = seed * 0x5DEECE66D + 0xB mod 2^48`` and returns the top ``bits``.
    """
    MULT = 0x5DEECE66D
    MASK = (1 << 48) - 1

    def __init__(self, seed: int):
        self.seed = (seed ^ self.MULT) & self.MASK

    def next(self, bits: int) -> int:
        self.seed = (self.seed * self.MULT + 0xB) & self.MASK
        r = self.seed >> (48 - bits)
        if r >= 1 << 31:  # Java int cast
            r -= 1 << 32
        return r

    def next_int(self, bound: int | None = None) -> int:
        if bound is None:
            return self.next(32)
        if bound <= 0:
            raise ValueError("bound must be positive")
        if bound & (-bound) == bound:
            return (bound * self.next(31)) >> 31
        while True:
            bits = self.next(31)
            val = bits % bound
            if bits - val + (bound - 1) < (1 << 31):
                return val

    def next_float(self) -> float:
        return float(np.float32(self.next(24)) / np.float32(1 << 24))

    def next_double(self) -> float:
        return ((self.next(26) << 27) + self.next(27)) * 2.0 ** -53

    def floats_pm1(self, n: int, scale: float = 1.0) -> np.ndarray:
        """``rng.nextFloat() * 2 - 1`` (times ``scale``), evaluated in float as in Java."""
        out = np.empty(n, dtype=np.float32)
        two, one, s = np.float32(2), np.float32(1), np.float32(scale)
        for i in range(n):
            out[i] = (np.float32(self.next_float()) * two - one) * s
        return out

    def floats_centered(self, n: int) -> np.ndarray:
        """``(rng.nextFloat() - 0.5f) * 2.0f`` (DirectMlAttentionKernelTest.randomFloats)."""
        out = np.empty(n, dtype=np.float32)
        h, two = np.float32(0.5), np.float32(2)
        for i in range(n):
            out[i] = (np.float32(self.next_float()) - h) * two
        return out


# --------------------------------------------------------------------------
# splitmix64 + Box-Muller N(0,1)
# --------------------------------------------------------------------------
_SM_GAMMA = np.uint64(0x9E3779B97F4A7C15)


def _splitmix64(seed: int, idx: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + (idx.astype(np.uint64) + np.uint64(1)) * _SM_GAMMA
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def splitmix_normal(seed: int, n: int, offset: int = 0) -> np.ndarray:
    """n standard normals; element i uses splitmix64 draws 2(i+offset), 2(i+offset)+1."""
    i = np.arange(offset, offset + n, dtype=np.uint64)
    a = _splitmix64(seed, 2 * i)
    b = _splitmix64(seed, 2 * i + 1)
    u1 = ((a >> np.uint64(11)).astype(np.float64) + 1.0) * 2.0 ** -53  # (0, 1]
    u2 = (b >> np.uint64(11)).astype(np.float64) * 2.0 ** -53  # [0, 1)
    return (np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * math.pi * u2)).astype(np.float32)


def splitmix_uniform_int(seed: int, n: int, lo: int, hi: int, offset: int = 0) -> np.ndarray:
    """n integers uniform in [lo, hi] (inclusive)."""
    i = np.arange(offset, offset + n, dtype=np.uint64)
    z = _splitmix64(seed ^ 0x5EED, i)
    return (lo + (z % np.uint64(hi - lo + 1)).astype(np.int64)).astype(np.int32)


# --------------------------------------------------------------------------
# oracle entry points (numpy in, numpy out)
# --------------------------------------------------------------------------
def rope_decoderonly(x: np.ndarray, n_heads: int, head_dim: int, pos: int, theta: float) -> np.ndarray:
    out = np.ascontiguousarray(x, dtype=np.float32).copy()
    lib().orc_rope_decoderonly(_f(out), n_heads, head_dim, pos, theta)
    return out


def rope_half_gemma(x: np.ndarray, n_heads: int, head_dim: int, pos: int, theta: float) -> np.ndarray:
    out = np.ascontiguousarray(x, dtype=np.float32).copy()
    lib().orc_rope_half_gemma(_f(out), n_heads, head_dim, pos, theta)
    return out


def rmsnorm_zero_centered(x: np.ndarray, n_heads: int, head_dim: int, w: np.ndarray, eps: float) -> np.ndarray:
    out = np.ascontiguousarray(x, dtype=np.float32).copy()
    w = np.ascontiguousarray(w, dtype=np.float32)
    lib().orc_rmsnorm_zero_centered(_f(out), n_heads, head_dim, _f(w), eps)
    return out


def softmax_decoderonly(x: np.ndarray, length: int | None = None) -> np.ndarray:
    """DecoderOnlyMath.softmax(values, length): only the first `length` entries change."""
    out = np.ascontiguousarray(x, dtype=np.float32).copy()
    lib().orc_softmax_decoderonly(_f(out), out.size if length is None else length)
    return out


def prefill(q, k, v, *, B, S, Hq, Hkv, D, scale, rope_theta=0.0, pos0=0, window=0, causal=True,
            softmax_mode=SOFTMAX_DECODERONLY, skip_small=False, n_threads=0) -> np.ndarray:
    """Causal (or bidirectional) GQA attention; q [B,S,Hq,D], k/v [B,S,Hkv,D] float32."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    out = np.zeros((B, S, Hq, D), dtype=np.float32)
    rc = lib().orc_prefill(_f(q), _f(k), _f(v), _f(out), B, S, Hq, Hkv, D, scale, rope_theta, pos0, window,
                           int(causal), softmax_mode, int(skip_small), n_threads)
    if rc != 0:
        raise ValueError(f"orc_prefill failed: {rc}")
    return out


def decode(q_new, k_new, v_new, k_cache, v_cache, ctx_lens, *, B, Hq, Hkv, D, max_seq, scale,
           rope_theta=0.0, rope_mode=ROPE_DECODERONLY, window=0, cache_layout=KV_HEAD_MAJOR,
           cache_dtype=F16, q_norm_w=None, k_norm_w=None, norm_eps=1e-6,
           softmax_mode=SOFTMAX_DECODERONLY, skip_small=False, n_threads=0, inplace=False):
    """Decode one token per sequence.  Returns (out [B,Hq,D], k_cache', v_cache').

    With inplace=True the float32 caches passed in receive the appended rows
    (no copy), as the reference's caches do."""
    q_new = np.ascontiguousarray(q_new, dtype=np.float32)
    k_new = np.ascontiguousarray(k_new, dtype=np.float32)
    v_new = np.ascontiguousarray(v_new, dtype=np.float32)
    if inplace:
        assert k_cache.dtype == np.float32 and k_cache.flags.c_contiguous
        assert v_cache.dtype == np.float32 and v_cache.flags.c_contiguous
        kc, vc = k_cache, v_cache
    else:
        kc = np.ascontiguousarray(k_cache, dtype=np.float32).copy()
        vc = np.ascontiguousarray(v_cache, dtype=np.float32).copy()
    lens = np.ascontiguousarray(ctx_lens, dtype=np.int32)
    qw = None if q_norm_w is None else np.ascontiguousarray(q_norm_w, dtype=np.float32)
    kw = None if k_norm_w is None else np.ascontiguousarray(k_norm_w, dtype=np.float32)
    out = np.zeros((B, Hq, D), dtype=np.float32)
    rc = lib().orc_decode(_f(q_new), _f(k_new), _f(v_new), _f(kc), _f(vc), cache_layout, cache_dtype, _i(lens),
                          B, Hq, Hkv, D, max_seq, scale, rope_theta, rope_mode, window,
                          None if qw is None else _f(qw), None if kw is None else _f(kw), norm_eps,
                          softmax_mode, int(skip_small), _f(out), n_threads)
    if rc != 0:
        raise ValueError(f"orc_decode failed: {rc}")
    return out, kc, vc


def attend_cache(q, k_cache, v_cache, last_pos, *, B, Hq, Hkv, D, max_seq, scale, window=0, first_explicit=-1,
                 cache_layout=KV_HEAD_MAJOR, softmax_mode=SOFTMAX_DECODERONLY, n_threads=0) -> np.ndarray:
    """Attention over an existing cache (no append); q [B,Hq,D] float32."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    kc = np.ascontiguousarray(k_cache, dtype=np.float32)
    vc = np.ascontiguousarray(v_cache, dtype=np.float32)
    lp = np.ascontiguousarray(last_pos, dtype=np.int32)
    out = np.zeros((B, Hq, D), dtype=np.float32)
    rc = lib().orc_attend_cache(_f(q), _f(kc), _f(vc), cache_layout, _i(lp), B, Hq, Hkv, D, max_seq, scale, window,
                                first_explicit, softmax_mode, _f(out), n_threads)
    if rc != 0:
        raise ValueError(f"orc_attend_cache failed: {rc}")
    return out


def encoder_minilm(q, k, v, key_len, *, B, H, S, D, layout=0, n_threads=0) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    out = np.zeros_like(q)
    kl = None if key_len is None else np.ascontiguousarray(key_len, dtype=np.int32)
    lib().orc_encoder_minilm(_f(q), _f(k), _f(v), None if kl is None else _i(kl), _f(out), B, H, S, D, layout,
                             n_threads)
    return out


def mha_additive(q, k, v, mask, *, B, H, S, D, scale, n_threads=0) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.float32)
    y = np.zeros_like(q)
    lib().orc_mha_additive(_f(q), _f(k), _f(v), None if m is None else _f(m), _f(y), B, H, S, D, scale, n_threads)
    return y


def kv_head_for_query_head(n_q: int, n_kv: int, q_head: int) -> int:
    return lib().orc_kv_head_for_query_head(n_q, n_kv, q_head)


def first_valid_key(full_attention: bool, window: int, query_pos: int) -> int:
    return lib().orc_first_valid_key(int(full_attention), window, query_pos)


def is_full_attention_layer(layer: int, pattern: int) -> bool:
    return bool(lib().orc_is_full_attention_layer(layer, pattern))


def rope_theta_for_layer(layer: int, pattern: int, theta_global: float, theta_local: float) -> float:
    return lib().orc_rope_theta_for_layer(layer, pattern, theta_global, theta_local)


def attention_scale(query_pre_attn_scalar: float, head_dim: int) -> float:
    return lib().orc_attention_scale(query_pre_attn_scalar, head_dim)


def max_threads() -> int:
    return lib().orc_max_threads()
