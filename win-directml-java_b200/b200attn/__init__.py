"""Python host bindings of libb200attn.so, the B200 (sm_100a) attention backend.

The native library is the product; this module only marshals torch device
tensors into the C ABI declared in ``include/b200attn.h`` and maps status
codes to exceptions the way the reference's Java bindings do:

* ``B2A_EINVAL``               -> :class:`ValueError` (the reference throws
  ``IllegalArgumentException`` for bad shapes);
* every other non-zero status  -> :class:`B200RuntimeException` (the
  reference's unchecked ``DirectMlRuntimeException``,
  ``WB/runtime/DirectMlRuntimeException.java``).

There is no CPU fallback: if the shared library or a CUDA device is missing,
every call fails loudly.

Operator mirrors
----------------
* :class:`CudaAttentionKernel` -- ``AttentionKernel`` / ``DirectMlAttentionKernel``
  (``WB/runtime/kernels/AttentionKernel.java:19-24``,
  ``WB/runtime/kernels/DirectMlAttentionKernel.java:99-210,370-420``).
* :func:`prefill_causal` -- the causal GQA prefill of the decoder runtimes.
* :func:`decode` -- the fused decode step (QK-norm, RoPE, KV append, attention).
* :class:`QwenAttentionShaders` -- ``rope_and_append`` / ``gqa_attention_decode``
  (``WB/windows/QwenAttentionShaders.java:82-263``).
* :class:`Gemma3FusedAttentionContext` -- ``Gemma3WarpFusedAttentionContextKernel.context``
  (``INF/gemma/Gemma3WarpFusedAttentionContextKernel.java:111-135``).
"""
from __future__ import annotations

import ctypes
import os
import re
import subprocess
import threading

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(_PKG_DIR)
LIB_PATH = os.path.join(ROOT, "lib", "libb200attn.so")
HEADER_PATH = os.path.join(os.path.dirname(ROOT), "include", "b200attn.h")

B2A_OK, B2A_EINVAL, B2A_ECUDA, B2A_ENCCL, B2A_ETIMEOUT, B2A_EOOM, B2A_ENOTSUP, B2A_EDEVICE = range(8)
FLOAT32, FLOAT16, BFLOAT16 = 0, 1, 2
HEAD_MAJOR, SEQ_MAJOR = 0, 1
KV_HEAD_MAJOR, KV_POS_MAJOR = 0, 1
ROPE_NONE, ROPE_NEOX, ROPE_GEMMA = 0, 1, 2

_lib = None
_lib_lock = threading.Lock()


class B200RuntimeException(RuntimeError):
    """Unchecked runtime failure of the CUDA backend (mirror of DirectMlRuntimeException)."""

    def __init__(self, message: str, status: int = B2A_ECUDA):
        super().__init__(message)
        self.status = status


def build(verbose: bool = False) -> str:
    """Compile lib/libb200attn.so for sm_100a with the committed Makefile."""
    cmd = ["make", "-C", ROOT, "-j", str(max(1, min(16, os.cpu_count() or 1)))]
    if not verbose:
        cmd.insert(1, "-s")
    subprocess.run(cmd, check=True)
    return LIB_PATH


_vp = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float
_d = ctypes.c_double


def lib() -> ctypes.CDLL:
    """Load the shared library (raises if it has not been built)."""
    global _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise B200RuntimeException(
                f"{LIB_PATH} is missing: build the CUDA library first (make -C {ROOT}); "
                "there is no CPU fallback", B2A_ENOTSUP)
        L = ctypes.CDLL(LIB_PATH)
        L.b2a_create.argtypes = [_i, ctypes.POINTER(_vp)]
        L.b2a_destroy.argtypes = [_vp]
        L.b2a_last_error.argtypes = [_vp, ctypes.c_char_p, ctypes.c_size_t]
        L.b2a_status_string.restype = ctypes.c_char_p
        L.b2a_status_string.argtypes = [_i]
        L.b2a_abi_version.restype = _i
        L.b2a_build_info.restype = ctypes.c_char_p
        L.b2a_set_workspace_limit.argtypes = [_vp, ctypes.c_size_t]
        L.b2a_set_decode_early_start.argtypes = [_vp, _i]
        L.b2a_workspace_bytes.argtypes = [_vp, ctypes.POINTER(ctypes.c_size_t)]
        L.b2a_reserve_decode.argtypes = [_vp, _i, _i, _i, _i]
        L.b2a_check_device_status.argtypes = [_vp, _vp]
        L.b2a_test_inject_wait_timeout.argtypes = [_vp]
        L.b2a_test_last_attention_kernel.argtypes = [_vp]
        L.b2a_test_last_attention_kernel.restype = _i
        L.b2a_mha.argtypes = [_vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _i, _vp]
        L.b2a_prefill_causal.argtypes = [_vp, _i, _i, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _i, _d, _i, _i,
                                         _vp, _vp]
        L.b2a_decode.argtypes = [_vp, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _i, _i, _f, _i, _d,
                                 _i, _vp, _vp, _f, _vp, _vp]
        L.b2a_qwen_rope_and_append.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _vp]
        L.b2a_qwen_gqa_attention_decode.argtypes = [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _vp]
        L.b2a_qwen_decode_step.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _f, _vp]
        L.b2a_prefill_gemma.argtypes = [_vp, _i, _i, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _i, _d, _i, _i, _vp,
                                        _vp, _f, _vp, _vp]
        L.b2a_gemma_fused_attention_context.argtypes = [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _vp]
        L.b2a_partition_units.argtypes = [_i, _i, _vp, _vp]
        L.b2a_linear.argtypes = [_vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp]
        L.b2a_decode_attention_block.argtypes = [_vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _i, _i,
                                                 _i, _i, _i, _i, _f, _d, _i, _vp]
        L.b2a_group_create.argtypes = [_i, _vp, ctypes.POINTER(_vp)]
        L.b2a_group_destroy.argtypes = [_vp]
        L.b2a_group_last_error.argtypes = [_vp, ctypes.c_char_p, ctypes.c_size_t]
        L.b2a_group_size.argtypes = [_vp]
        L.b2a_group_context.argtypes = [_vp, _i, ctypes.POINTER(_vp)]
        L.b2a_group_check_device_status.argtypes = [_vp, _vp]
        L.b2a_sharded_decode.argtypes = [_vp, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _i, _i, _f, _i,
                                         _d, _i, _vp, _vp, _f, _vp, _vp, _vp]
        L.b2a_sharded_mha.argtypes = [_vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _i, _vp]
        for name in ("b2a_create", "b2a_destroy", "b2a_last_error", "b2a_set_workspace_limit",
                     "b2a_set_decode_early_start", "b2a_workspace_bytes",
                     "b2a_reserve_decode", "b2a_check_device_status", "b2a_mha", "b2a_prefill_causal", "b2a_decode",
                     "b2a_qwen_rope_and_append", "b2a_qwen_gqa_attention_decode", "b2a_qwen_decode_step", "b2a_prefill_gemma",
                     "b2a_gemma_fused_attention_context", "b2a_partition_units", "b2a_test_inject_wait_timeout",
                     "b2a_linear", "b2a_decode_attention_block", "b2a_group_create", "b2a_group_destroy", "b2a_group_last_error", "b2a_group_size",
                     "b2a_group_context", "b2a_group_check_device_status", "b2a_sharded_decode", "b2a_sharded_mha"):
            getattr(L, name).restype = _i
        _lib = L
        return _lib


def declared_symbols() -> list[str]:
    """Function names declared with B2A_API in include/*.h (the boundary and its test hooks)."""
    import glob
    names = []
    for path in sorted(glob.glob(os.path.join(os.path.dirname(HEADER_PATH), "*.h"))):
        names += re.findall(r"B2A_API\s+[\w\s\*]+?\b(b2a_\w+)\s*\(", open(path).read())
    return names


def _dtype_code(t) -> int:
    import torch
    m = {torch.float32: FLOAT32, torch.float16: FLOAT16, torch.bfloat16: BFLOAT16}
    if t.dtype not in m:
        raise ValueError(f"unsupported element type {t.dtype}")
    return m[t.dtype]


def _ptr(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("tensors must live on the CUDA device (GpuBuffer); got a host tensor")
    if not t.is_contiguous():
        raise ValueError("tensors must be contiguous (row-major TensorLayout)")
    return ctypes.c_void_p(t.data_ptr())


def _stream(stream):
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


class Context:
    """One CUDA device context (mirror of DirectMlContextImpl's role)."""

    def __init__(self, device: int = 0):
        self._h = _vp()
        rc = lib().b2a_create(device, ctypes.byref(self._h))
        if rc != B2A_OK:
            raise _error(rc, _message(None))
        self.device = device

    @property
    def handle(self):
        return self._h

    def check(self, rc: int):
        if rc != B2A_OK:
            raise _error(rc, _message(self._h))

    def close(self):
        if self._h:
            lib().b2a_destroy(self._h)
            self._h = _vp()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_workspace_limit(self, nbytes: int):
        self.check(lib().b2a_set_workspace_limit(self._h, nbytes))

    def set_decode_early_start(self, enable: bool):
        """b2a_set_decode_early_start: tensor-core decodes overlap their plan and first cache
        tiles with the kernel ahead of them on the stream (which must not write ctx_lens or the
        cache rows the decode reads)."""
        self.check(lib().b2a_set_decode_early_start(self._h, 1 if enable else 0))

    def workspace_bytes(self) -> int:
        n = ctypes.c_size_t()
        self.check(lib().b2a_workspace_bytes(self._h, ctypes.byref(n)))
        return n.value

    def reserve_decode(self, max_batch: int, num_q_heads: int, num_kv_heads: int, head_dim: int):
        self.check(lib().b2a_reserve_decode(self._h, max_batch, num_q_heads, num_kv_heads, head_dim))

    def check_device_status(self, stream=None):
        self.check(lib().b2a_check_device_status(self._h, _stream(stream)))

    def last_attention_kernel(self) -> str:
        """Test hook (include/b200attn_testing.h): the kernel family of the last whole-sequence
        attention launch: "tcgen05", "warp_mma", "generic", "f32_tiled" or "" before any."""
        return {1: "tcgen05", 2: "warp_mma", 3: "generic", 4: "f32_tiled"}.get(
            lib().b2a_test_last_attention_kernel(self._h), "")

    def inject_wait_timeout(self):
        """Test hook (include/b200attn_testing.h): the next tcgen05 attention launch of this
        context leaves one K/V copy unissued, so a bounded device wait runs out."""
        self.check(lib().b2a_test_inject_wait_timeout(self._h))


def _message(h) -> str:
    buf = ctypes.create_string_buffer(2048)
    lib().b2a_last_error(h, buf, len(buf))
    return buf.value.decode(errors="replace")


def _error(rc: int, msg: str) -> Exception:
    name = lib().b2a_status_string(rc).decode()
    if rc == B2A_EINVAL:
        return ValueError(f"{name}: {msg}")
    return B200RuntimeException(f"{name}: {msg}", rc)


# ---------------------------------------------------------------- operators
def mha(ctx: Context, q, k, v, y, scale: float, mask=None, key_lengths=None, layout: int = HEAD_MAJOR, stream=None):
    """Bidirectional MHA with optional key padding (AttentionKernel.dispatch semantics).

    q, k, v, y: [B,H,S,D] (HEAD_MAJOR) or [B,S,H,D] (SEQ_MAJOR) device tensors.
    mask: float32 [B,S] additive (0 / -1e9), key_lengths: int32 [B]; at most one.
    """
    if q.dim() != 4:
        raise ValueError("q must be 4-D")
    if layout == HEAD_MAJOR:
        B, H, S, D = q.shape
    else:
        B, S, H, D = q.shape
    for name, t in (("k", k), ("v", v), ("y", y)):
        if tuple(t.shape) != tuple(q.shape):
            raise ValueError(f"{name} expected shape {tuple(q.shape)}, got {tuple(t.shape)}")
    if mask is not None and mask.numel() != B * S:
        raise ValueError(f"mask expected {B * S} elements ([B,1,1,S]), got {mask.numel()}")
    ctx.check(lib().b2a_mha(ctx.handle, _dtype_code(q), _dtype_code(y), _ptr(q), _ptr(k), _ptr(v), _ptr(mask),
                            _ptr(key_lengths), _ptr(y), B, H, S, D, scale, layout, _stream(stream)))
    return y


def prefill_causal(ctx: Context, q, k, v, o, scale: float, rope_mode: int = ROPE_NEOX, rope_theta: float = 10000.0,
                   pos0: int = 0, window: int = 0, k_rot_out=None, stream=None):
    """Causal GQA prefill with fused RoPE; q [B,S,Hq,D], k/v [B,S,Hkv,D], o [B,S,Hq,D]."""
    B, S, Hq, D = q.shape
    Hkv = k.shape[2]
    if tuple(k.shape) != (B, S, Hkv, D) or tuple(v.shape) != (B, S, Hkv, D):
        raise ValueError("k and v must be [B,S,Hkv,D] matching q")
    if tuple(o.shape) != (B, S, Hq, D):
        raise ValueError("o must be [B,S,Hq,D]")
    ctx.check(lib().b2a_prefill_causal(ctx.handle, _dtype_code(q), _dtype_code(o), _ptr(q), _ptr(k), _ptr(v), _ptr(o),
                                       B, S, Hq, Hkv, D, scale, rope_mode, rope_theta, pos0, window, _ptr(k_rot_out),
                                       _stream(stream)))
    return o


def prefill_gemma(ctx: Context, q, k, v, o, scale: float, *, q_norm_w=None, k_norm_w=None, norm_eps: float = 1e-6,
                  rope_mode: int = ROPE_GEMMA, rope_theta: float = 10000.0, pos0: int = 0, window: int = 0,
                  k_rot_out=None, stream=None):
    """Batched Gemma-3 prefill: QK-norm + RoPE of every position and one causal attention
    launch (sliding window when window > 0); q [B,S,Hq,D], k/v [B,S,Hkv,D], o [B,S,Hq,D]."""
    B, S, Hq, D = q.shape
    Hkv = k.shape[2]
    if tuple(k.shape) != (B, S, Hkv, D) or tuple(v.shape) != (B, S, Hkv, D):
        raise ValueError("k and v must be [B,S,Hkv,D] matching q")
    if tuple(o.shape) != (B, S, Hq, D):
        raise ValueError("o must be [B,S,Hq,D]")
    ctx.check(lib().b2a_prefill_gemma(ctx.handle, _dtype_code(q), _dtype_code(o), _ptr(q), _ptr(k), _ptr(v), _ptr(o),
                                      B, S, Hq, Hkv, D, scale, rope_mode, rope_theta, pos0, window, _ptr(q_norm_w),
                                      _ptr(k_norm_w), norm_eps, _ptr(k_rot_out), _stream(stream)))
    return o


def decode(ctx: Context, q_new, k_new, v_new, k_cache, v_cache, ctx_lens, o, scale: float, *,
           kv_layout: int = KV_HEAD_MAJOR, rope_mode: int = ROPE_NEOX, rope_theta: float = 10000.0, window: int = 0,
           q_norm_w=None, k_norm_w=None, norm_eps: float = 1e-6, stream=None):
    """Fused decode step.  q_new [B,Hq,D]; k_new/v_new [B,Hkv,D]; caches
    [B,Hkv,max_seq,D] (KV_HEAD_MAJOR) or [B,max_seq,Hkv,D] (KV_POS_MAJOR);
    ctx_lens int32 [B] on the device; o [B,Hq,D]."""
    B, Hq, D = q_new.shape
    Hkv = k_new.shape[1]
    if kv_layout == KV_HEAD_MAJOR:
        max_seq = k_cache.shape[2]
        expect = (B, Hkv, max_seq, D)
    else:
        max_seq = k_cache.shape[1]
        expect = (B, max_seq, Hkv, D)
    if tuple(k_cache.shape) != expect or tuple(v_cache.shape) != expect:
        raise ValueError(f"caches must have shape {expect}")
    if ctx_lens.dtype.__str__() != "torch.int32" or ctx_lens.numel() != B:
        raise ValueError("ctx_lens must be int32 [B]")
    ctx.check(lib().b2a_decode(ctx.handle, _dtype_code(q_new), _dtype_code(k_cache), _dtype_code(o), _ptr(q_new),
                               _ptr(k_new), _ptr(v_new), _ptr(k_cache), _ptr(v_cache), kv_layout, _ptr(ctx_lens), B, Hq,
                               Hkv, D, max_seq, scale, rope_mode, rope_theta, window, _ptr(q_norm_w), _ptr(k_norm_w),
                               norm_eps, _ptr(o), _stream(stream)))
    return o


def linear(ctx: Context, x, w, y, bias=None, residual=None, stream=None):
    """y = x w^T + bias + residual on the tensor cores (x [M,K], w [N,K] fp16/bf16; bias float [N];
    residual and y [M,N]); the O projection with its residual add, the QKV projection with its bias."""
    M, K = x.shape
    N = w.shape[0]
    if tuple(w.shape) != (N, K) or tuple(y.shape) != (M, N):
        raise ValueError("w must be [N,K] and y [M,N] for x [M,K]")
    if residual is not None and tuple(residual.shape) != (M, N):
        raise ValueError("residual must be [M,N]")
    ctx.check(lib().b2a_linear(ctx.handle, _dtype_code(x), _dtype_code(y), _ptr(x), _ptr(w), _ptr(bias),
                               _ptr(residual), _ptr(y), M, N, K, _stream(stream)))
    return y


def decode_attention_block(ctx: Context, x, w_qkv, b_qkv, k_cache, v_cache, ctx_lens, w_o, residual, y, *,
                           num_q_heads: int, num_kv_heads: int, scale: float, rope_theta: float,
                           kv_layout: int = KV_HEAD_MAJOR, window: int = 0, stream=None):
    """One decode-layer attention block (Qwen2Runtime.processLayerDecode, normed input to residual 1):
    QKV projection + bias, NeoX RoPE at ctx_lens, KV append, GQA attention, O projection + residual."""
    B, hidden = x.shape
    D = w_qkv.shape[0] // (num_q_heads + 2 * num_kv_heads)
    max_seq = k_cache.shape[2] if kv_layout == KV_HEAD_MAJOR else k_cache.shape[1]
    ctx.check(lib().b2a_decode_attention_block(
        ctx.handle, _dtype_code(x), _dtype_code(k_cache), _ptr(x), _ptr(w_qkv), _ptr(b_qkv), _ptr(k_cache),
        _ptr(v_cache), kv_layout, _ptr(ctx_lens), _ptr(w_o), _ptr(residual), _ptr(y), B, hidden, num_q_heads,
        num_kv_heads, D, max_seq, scale, rope_theta, window, _stream(stream)))
    return y


def _ptr_array(tensors):
    """A C array of device pointers (None -> NULL entry) kept alive by the caller."""
    arr = (ctypes.c_void_p * len(tensors))()
    for i, t in enumerate(tensors):
        arr[i] = None if t is None else _ptr(t).value
    return arr


class Group:
    """Several GPUs driven from one process: one Context per device and an NCCL clique
    (b2a_group_create).  The sharded calls run each rank's equal shard on its own device
    and reassemble the outputs with one grouped ncclAllGather."""

    def __init__(self, devices):
        devs = (ctypes.c_int * len(devices))(*devices)
        self._h = _vp()
        rc = lib().b2a_group_create(len(devices), devs, ctypes.byref(self._h))
        if rc != B2A_OK:
            raise _error(rc, self._message(None))
        self.devices = list(devices)

    @staticmethod
    def _message(h) -> str:
        buf = ctypes.create_string_buffer(2048)
        lib().b2a_group_last_error(h, buf, len(buf))
        return buf.value.decode(errors="replace")

    def check(self, rc: int):
        if rc != B2A_OK:
            raise _error(rc, self._message(self._h))

    def size(self) -> int:
        return lib().b2a_group_size(self._h)

    def close(self):
        if self._h:
            lib().b2a_group_destroy(self._h)
            self._h = _vp()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _streams(self, streams):
        import torch
        if streams is None:
            streams = [torch.cuda.current_stream(d) for d in self.devices]
        arr = (ctypes.c_void_p * len(streams))()
        for i, s in enumerate(streams):
            arr[i] = s.cuda_stream
        return arr

    def check_device_status(self, streams=None):
        self.check(lib().b2a_group_check_device_status(self._h, self._streams(streams)))

    def decode(self, q_new, k_new, v_new, k_cache, v_cache, ctx_lens, o_shard, o_gathered, scale: float, *,
               kv_layout: int = KV_HEAD_MAJOR, rope_mode: int = ROPE_NEOX, rope_theta: float = 10000.0,
               window: int = 0, q_norm_w=None, k_norm_w=None, norm_eps: float = 1e-6, streams=None):
        """Per-rank lists of tensors (rank r's on device r): b2a_decode of every shard, then
        o_gathered[r] = concatenation of all ranks' o_shard (rank-major)."""
        B, Hq, D = q_new[0].shape
        Hkv = k_new[0].shape[1]
        max_seq = k_cache[0].shape[2] if kv_layout == KV_HEAD_MAJOR else k_cache[0].shape[1]
        keep = [_ptr_array(x) for x in (q_new, k_new, v_new, k_cache, v_cache, ctx_lens, o_shard, o_gathered)]
        qw = _ptr_array(q_norm_w) if q_norm_w is not None else None
        kw = _ptr_array(k_norm_w) if k_norm_w is not None else None
        self.check(lib().b2a_sharded_decode(
            self._h, _dtype_code(q_new[0]), _dtype_code(k_cache[0]), _dtype_code(o_shard[0]), *keep[:5], kv_layout,
            keep[5], B, Hq, Hkv, D, max_seq, scale, rope_mode, rope_theta, window, qw, kw, norm_eps, keep[6], keep[7],
            self._streams(streams)))

    def mha(self, q, k, v, y_shard, y_gathered, scale: float, *, mask=None, key_lengths=None,
            layout: int = HEAD_MAJOR, streams=None):
        """Per-rank lists: b2a_mha of every shard, then y_gathered[r] = all ranks' y_shard (batch-major)."""
        if layout == HEAD_MAJOR:
            B, H, S, D = q[0].shape
        else:
            B, S, H, D = q[0].shape
        keep = [_ptr_array(x) for x in (q, k, v)]
        m = _ptr_array(mask) if mask is not None else None
        kl = _ptr_array(key_lengths) if key_lengths is not None else None
        self.check(lib().b2a_sharded_mha(self._h, _dtype_code(q[0]), _dtype_code(y_shard[0]), *keep, m, kl,
                                         _ptr_array(y_shard), _ptr_array(y_gathered), B, H, S, D, scale, layout,
                                         self._streams(streams)))


def partition_units(unit_cost, n_ranks: int):
    """Equal-count, cost-balanced assignment of independent units to ranks (host only)."""
    import numpy as np
    cost = np.ascontiguousarray(unit_cost, dtype=np.int64)
    out = np.zeros(cost.size, dtype=np.int32)
    rc = lib().b2a_partition_units(cost.size, n_ranks, cost.ctypes.data_as(_vp), out.ctypes.data_as(_vp))
    if rc != B2A_OK:
        raise ValueError(f"partition_units: n_units ({cost.size}) must be a positive multiple of n_ranks ({n_ranks})")
    return out


_batch_local = threading.local()


class GpuBatch:
    """Submission coalescing, the mirror of DirectMlGpuBatch (WB/runtime/DirectMlGpuBatch.java):
    outside a batch every CudaAttentionKernel.dispatch waits for its launch and checks the
    device status (as DirectMlAttentionKernel.dispatch waits on a fence through
    D3D12Bindings.executeAndWait); inside one, dispatches return at once and close()
    synchronises once and raises the first device failure (B2A_ETIMEOUT, B2A_EDEVICE).
    Thread-bound and re-entrant: a nested begin() shares the outer batch and only the
    outermost close() drains."""

    def __init__(self, ctx: "Context", stream=None):
        self.ctx, self.stream, self._outer = ctx, stream, None

    @classmethod
    def begin(cls, ctx: "Context", stream=None) -> "GpuBatch":
        b = cls(ctx, stream)
        b._outer = getattr(_batch_local, "current", None)
        if b._outer is None:
            _batch_local.current = b
        return b

    @staticmethod
    def current():
        return getattr(_batch_local, "current", None)

    def close(self):
        if self._outer is not None:
            return  # nested: the outermost batch drains
        if getattr(_batch_local, "current", None) is self:
            _batch_local.current = None
            self.ctx.check_device_status(self.stream)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class CudaAttentionKernel:
    """AttentionKernel for the CUDA backend, shaped like DirectMlAttentionKernel:
    fixed (B, H, S, D, scale, hasMask) at construction, dispatch(q, k, v, mask, y, scale).
    Unlike the DirectML kernel it keeps no [B,H,S,S] intermediates.  A dispatch outside a
    GpuBatch waits for the launch and raises B200RuntimeException if the device flagged a
    failure (a bounded wait that ran out: B2A_ETIMEOUT), so it never returns with undefined
    output; inside a batch the check happens when the batch closes."""

    def __init__(self, ctx: Context, batch: int, heads: int, seq: int, head_dim: int, scale: float, has_mask: bool):
        if batch <= 0 or heads <= 0 or seq <= 0 or head_dim <= 0:
            raise ValueError("batch, heads, seq, headDim must be > 0")
        self.ctx, self.B, self.H, self.S, self.D = ctx, batch, heads, seq, head_dim
        self.scale, self.has_mask = scale, has_mask
        self.closed = False

    def dispatch(self, q, k, v, mask, y, scale: float, stream=None):
        if self.closed:
            raise B200RuntimeException("CudaAttentionKernel already closed")
        if scale != self.scale:
            raise B200RuntimeException(f"scale mismatch: kernel compiled with {self.scale}, got {scale}")
        expected = self.B * self.H * self.S * self.D
        for name, t in (("q", q), ("k", k), ("v", v), ("y", y)):
            if t is None:
                raise B200RuntimeException(f"{name} tensor is null")
            if t.numel() != expected:
                raise B200RuntimeException(
                    f"{name} expected {expected} elements ([B,H,S,D]=[{self.B},{self.H},{self.S},{self.D}]), "
                    f"got {t.numel()}")
        if self.has_mask and mask is None:
            raise B200RuntimeException("kernel was built with hasMask=true but mask=null")
        if not self.has_mask and mask is not None:
            raise B200RuntimeException("kernel was built with hasMask=false but mask!=null")
        shape = (self.B, self.H, self.S, self.D)
        mha(self.ctx, q.view(shape), k.view(shape), v.view(shape), y.view(shape), scale,
            mask=mask if self.has_mask else None, layout=HEAD_MAJOR, stream=stream)
        if GpuBatch.current() is None:  # executeAndWait: wait and surface device failures now
            self.ctx.check_device_status(stream)

    def close(self):
        self.closed = True


class QwenAttentionShaders:
    """The Qwen GPU decode pair with the HLSL root-constant contract (float32 buffers)."""

    def __init__(self, ctx: Context):
        self.ctx = ctx

    def rope_and_append(self, q, k, v, k_cache, v_cache, num_heads, kv_heads, head_dim, pos, max_seq_len,
                        rope_theta, stream=None):
        self.ctx.check(lib().b2a_qwen_rope_and_append(self.ctx.handle, _ptr(q), _ptr(k), _ptr(v), _ptr(k_cache),
                                                      _ptr(v_cache), num_heads, kv_heads, head_dim, pos, max_seq_len,
                                                      rope_theta, _stream(stream)))

    def gqa_attention_decode(self, q, k_cache, v_cache, attn_out, num_heads, kv_heads, head_dim, q_heads_per_kv_head,
                             seq_len, max_seq_len, scale, stream=None):
        self.ctx.check(lib().b2a_qwen_gqa_attention_decode(self.ctx.handle, _ptr(q), _ptr(k_cache), _ptr(v_cache),
                                                           _ptr(attn_out), num_heads, kv_heads, head_dim,
                                                           q_heads_per_kv_head, seq_len, max_seq_len, scale,
                                                           _stream(stream)))

    def decode_step(self, qkv, qkv_bias, k_cache, v_cache, attn_out, num_heads, kv_heads, head_dim, pos, max_seq_len,
                    rope_theta, scale, stream=None):
        """Bias + RoPE + KV append + GQA attention of one token from the fused [Q|K|V] row
        (QwenGpuPipeline.decodeLayerGpuResident steps 1b-3) in one launch."""
        self.ctx.check(lib().b2a_qwen_decode_step(self.ctx.handle, _ptr(qkv), _ptr(qkv_bias), _ptr(k_cache),
                                                  _ptr(v_cache), _ptr(attn_out), num_heads, kv_heads, head_dim, pos,
                                                  max_seq_len, rope_theta, scale, _stream(stream)))


class Gemma3FusedAttentionContext:
    """Gemma3WarpFusedAttentionContextKernel.context with the same arguments (float32)."""

    def __init__(self, ctx: Context):
        self.ctx = ctx

    def context(self, q, keys, values, num_heads, num_kv_heads, head_dim, kv_dim, query_pos, first_valid, scale,
                out=None, stream=None):
        import torch
        if num_kv_heads <= 0 or num_heads % num_kv_heads != 0:
            raise ValueError("numHeads must be a multiple of numKvHeads")
        if q.numel() != num_heads * head_dim:
            raise ValueError(f"q length mismatch: {q.numel()} != {num_heads * head_dim}")
        visible = (query_pos + 1) * kv_dim
        if keys.numel() < visible or values.numel() < visible:
            raise ValueError(f"keys/values too small for queryPos {query_pos}")
        if out is None:
            out = torch.empty(num_heads * head_dim, dtype=torch.float32, device=q.device)
        self.ctx.check(lib().b2a_gemma_fused_attention_context(self.ctx.handle, _ptr(q), _ptr(keys), _ptr(values),
                                                               _ptr(out), num_heads, num_heads // num_kv_heads,
                                                               head_dim, kv_dim, first_valid, query_pos, scale,
                                                               _stream(stream)))
        return out
