// api.cpp -- the C ABI of libb200attn.so (include/b200attn.h): contexts,
// argument validation with the reference's error wording, workspace
// management and kernel dispatch.  No exception crosses the boundary and no
// call falls back to the CPU.
#include <cuda_runtime.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <numeric>
#include <string>
#include <vector>

#include "../../include/b200attn.h"
#include "../../include/b200attn_testing.h"
#include "internal.h"

using namespace b2a;

struct b2a_context {
    int device = 0;
    int sm_count = 0;
    std::string last_error;
    size_t ws_limit = 0;  // 0: unlimited
    int* status = nullptr;  // device int[kStatusBufferInts]: error flags, prefill work-item counters
    int* status_host = nullptr;  // pinned int[kStatusWords]: where b2a_check_device_status reads the flags
    // decode workspace: [counters][partials]
    void* dec_ws = nullptr;
    size_t dec_ws_bytes = 0;
    // counter region at the start of dec_ws, partial slots after it; the region never
    // shrinks (a later, smaller batch's slots would otherwise land on counters a larger
    // batch relies on being zero) and is zeroed whenever it grows or the buffer is new
    size_t dec_counter_bytes = 0;
    // prefill workspace: rope table + rotated q/k staging
    void* pf_ws = nullptr;
    size_t pf_ws_bytes = 0;
    // float NeoX (cos, sin) table [position][D/2] for positions [0, rope_npos), reused by later
    // calls with the same theta and head dim (rebuilt, on the calling stream, when it does not cover)
    void* rope_tab = nullptr;
    size_t rope_tab_bytes = 0;
    double rope_theta = 0.0;
    int rope_D = 0;
    int rope_npos = 0;
    // attention block: the QKV projection's fp32 rows and the attention output
    void* blk_ws = nullptr;
    size_t blk_ws_bytes = 0;
    // split-K projections: [tile counters][fp32 accumulator], all zero between launches
    void* lin_ws = nullptr;
    size_t lin_ws_bytes = 0;
    size_t lin_region = 0;
    // generic-kernel key split: [counters][partial slots], the same layout rules as dec_ws
    void* split_ws = nullptr;
    size_t split_ws_bytes = 0;
    size_t split_counter_bytes = 0;
    // test hook (b2a_test_inject_wait_timeout): the next tcgen05 attention launch
    // leaves one K/V copy unissued
    bool inject_wait_timeout = false;
    // b2a_set_decode_early_start: tensor-core decodes launched with programmatic serialisation
    bool decode_early_start = false;
    // test hook (b2a_test_last_attention_kernel): the kernel the last whole-sequence
    // attention launch took
    int last_attention_kernel = 0;
};

namespace {

thread_local std::string g_create_error;

int fail(b2a_context* ctx, int status, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    if (ctx) ctx->last_error = buf;
    else g_create_error = buf;
    return status;
}

int cuda_fail(b2a_context* ctx, cudaError_t e, const char* what) {
    if (e == cudaErrorMemoryAllocation) return fail(ctx, B2A_EOOM, "%s: %s", what, cudaGetErrorString(e));
    return fail(ctx, B2A_ECUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

// Makes ctx->device current for the duration of a call.
struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

bool valid_dtype(int d) { return d == B2A_FLOAT32 || d == B2A_FLOAT16 || d == B2A_BFLOAT16; }
size_t dtype_size(int d) { return d == B2A_FLOAT32 ? 4 : 2; }

int ensure_buffer(b2a_context* ctx, void** buf, size_t* have, size_t need, const char* what) {
    if (*have >= need) return B2A_OK;
    const size_t other =
        ctx->dec_ws_bytes + ctx->pf_ws_bytes + ctx->split_ws_bytes + ctx->blk_ws_bytes + ctx->rope_tab_bytes +
        ctx->lin_ws_bytes - *have;
    if (ctx->ws_limit != 0 && need + other > ctx->ws_limit)
        return fail(ctx, B2A_EOOM, "%s workspace of %zu bytes exceeds the context limit of %zu bytes", what,
                    need + other, ctx->ws_limit);
    if (*buf) {
        cudaFree(*buf);  // implicitly waits for work that may still use it
        *buf = nullptr;
        *have = 0;
    }
    cudaError_t e = cudaMalloc(buf, need);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return cuda_fail(ctx, e, what);
    }
    *have = need;
    return B2A_OK;
}

// Sizes a [counters][partial slots] workspace: the counter region keeps the largest size
// any call needed, the partial slots start after it, and the counters are zeroed (on
// `stream`, or synchronously when it is null and `sync`) when the buffer is new or the
// region grows.  Returns the counter region's size in *counter_bytes.
int ensure_counted_buffer(b2a_context* ctx, void** buf, size_t* have, size_t* region, size_t counter_ints,
                          size_t partial_bytes, const char* what, cudaStream_t stream, bool sync,
                          size_t* counter_bytes) {
    const size_t need_counters = (counter_ints * sizeof(int) + 255) / 256 * 256;
    const size_t cb = std::max(need_counters, *region);
    const bool grow = cb + partial_bytes > *have;
    const int rc = ensure_buffer(ctx, buf, have, cb + partial_bytes, what);
    if (rc != B2A_OK) return rc;
    if (grow || cb > *region) {
        const cudaError_t e = sync ? cudaMemset(*buf, 0, cb) : cudaMemsetAsync(*buf, 0, cb, stream);
        if (e != cudaSuccess) return cuda_fail(ctx, e, what);
        *region = cb;
    }
    *counter_bytes = cb;
    return B2A_OK;
}

void inv_freq_table(double theta, int D, double* out) {
    // 1 / theta^(2i/D) in double (INF/decoderonly/DecoderOnlyRotaryEmbedding.java:57-59,
    // INF/gemma/Gemma3ReferenceMath.java:74)
    for (int i = 0; i < D / 2; ++i) out[i] = 1.0 / pow(theta, (2.0 * i) / D);
}

// The context's NeoX table covering positions [0, npos) for (theta, D); built on `stream` when the
// cached one does not cover them.  Calls on other streams must be ordered after this one (the
// same rule as every workspace of a context).
int neox_table(b2a_context* ctx, double theta, int D, int npos, cudaStream_t stream, const float2** out) {
    if (!(ctx->rope_tab != nullptr && ctx->rope_theta == theta && ctx->rope_D == D && ctx->rope_npos >= npos)) {
        const int n = (npos + 255) / 256 * 256;
        const int rc = ensure_buffer(ctx, &ctx->rope_tab, &ctx->rope_tab_bytes, (size_t)n * (D / 2) * sizeof(float2),
                                     "rope table");
        if (rc) return rc;
        double inv[kMaxHeadDim / 2];
        inv_freq_table(theta, D, inv);
        const cudaError_t e =
            launch_rope_table_f32(static_cast<float2*>(ctx->rope_tab), n, D / 2, 0, inv, stream);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "rope table launch");
        ctx->rope_theta = theta;
        ctx->rope_D = D;
        ctx->rope_npos = n;
    }
    *out = static_cast<const float2*>(ctx->rope_tab);
    return B2A_OK;
}

// Whether the tcgen05 kernel converts bf16 operands to fp16 itself instead of a pre-pass that
// writes fp16 copies.  In the kernel two otherwise idle warps convert each staged tile, so every
// work item converts the key/value tiles it reads: for sequences of at most 512 keys (at most two
// work items per head) that is cheaper than the extra launch and the copies' HBM round trip; for
// longer ones the repeated conversion costs more.  (Rotating q and k in the kernel the same way was
// slower at every length measured, so RoPE stays in the pre-pass.)
constexpr int kInKernelPrepMaxSeq = 512;

int check_heads(b2a_context* ctx, int Hq, int Hkv) {
    // DecoderOnlyAttentionLayout constructor (INF/decoderonly/DecoderOnlyAttentionLayout.java:12-22)
    if (Hq <= 0) return fail(ctx, B2A_EINVAL, "numQueryHeads must be positive");
    if (Hkv <= 0) return fail(ctx, B2A_EINVAL, "numKeyValueHeads must be positive");
    if (Hq % Hkv != 0)
        return fail(ctx, B2A_EINVAL, "numQueryHeads must be divisible by numKeyValueHeads for grouped-query attention");
    return B2A_OK;
}

int check_head_dim(b2a_context* ctx, int D) {
    // DecoderOnlyRotaryEmbedding constructor (INF/decoderonly/DecoderOnlyRotaryEmbedding.java:14-16)
    if (D <= 0 || D % 2 != 0) return fail(ctx, B2A_EINVAL, "headDim must be positive and even");
    if (D > kMaxHeadDim) return fail(ctx, B2A_ENOTSUP, "headDim %d exceeds the supported maximum %d", D, kMaxHeadDim);
    return B2A_OK;
}

// Whole-sequence attention: the tcgen05 kernel where its shape rules hold,
// else the warp-MMA kernel (16-bit, head_dim 32..128), else the tiled fp32 kernel
// (fp32, head_dim 64 / 128), else the generic one.
cudaError_t launch_attention(b2a_context* ctx, const AttnParams& p, cudaStream_t s) {
    if (attn_tcgen05_supported(p)) {
        const bool stall = ctx->inject_wait_timeout;
        ctx->inject_wait_timeout = false;
        ctx->last_attention_kernel = B2A_TEST_KERNEL_TCGEN05;
        return launch_attn_tcgen05(p, ctx->status, s, stall);
    }
    if (attn_tc_supported(p)) {
        ctx->last_attention_kernel = B2A_TEST_KERNEL_WARP_MMA;
        return launch_attn_tc(p, s);
    }
    if (attn_f32_supported(p)) {
        ctx->last_attention_kernel = B2A_TEST_KERNEL_F32_TILED;
        return launch_attn_f32(p, s);
    }
    ctx->last_attention_kernel = B2A_TEST_KERNEL_GENERIC;
    // generic kernel: launches too small to fill the GPU split each query block's keys
    // over several CTAs; without room for the split workspace they run unsplit
    size_t part_bytes = 0, counter_ints = 0;
    const int nsplit = attn_simt_split_plan(p, ctx->sm_count, &part_bytes, &counter_ints);
    if (nsplit > 1) {
        size_t counter_bytes = 0;
        if (ensure_counted_buffer(ctx, &ctx->split_ws, &ctx->split_ws_bytes, &ctx->split_counter_bytes, counter_ints,
                                  part_bytes, "attention split workspace", s, false, &counter_bytes) == B2A_OK) {
            const SimtSplit sp{reinterpret_cast<float*>(static_cast<char*>(ctx->split_ws) + counter_bytes),
                               static_cast<int*>(ctx->split_ws), nsplit, kSimtSplitKeys};
            return launch_attn_simt(p, s, &sp);
        }
        ctx->last_error.clear();  // the refused workspace is not an error of this call
    }
    return launch_attn_simt(p, s);
}

int run_decode(b2a_context* ctx, DecodeParams& p, cudaStream_t stream, bool allow_tc) {
    // 16-byte row loads need 16-byte aligned cache bases and row strides
    const bool aligned = ((uintptr_t)p.k_cache % 16 == 0) && ((uintptr_t)p.v_cache % 16 == 0) &&
                         p.stride_b % 8 == 0 && p.stride_h % 8 == 0 && p.stride_pos % 8 == 0;
    p.status = ctx->status;
    if (allow_tc && aligned && decode_tc_supported(p.D, p.cache_dtype)) {
        p.n_hg = (p.G + 7) / 8;
        int target = 0, cap = 0;
        size_t partial_bytes = 0;
        decode_tc_workspace(ctx->device, p.B, p.Hkv, p.n_hg, p.D, p.cache_dtype, &target, &cap, &partial_bytes);
        const int bmax = std::min(p.B, kDecodeMaxBatchPerLaunch);
        const size_t counter_ints = (size_t)bmax * p.Hkv * p.n_hg;
        size_t counter_bytes = 0;
        int rc = ensure_counted_buffer(ctx, &ctx->dec_ws, &ctx->dec_ws_bytes, &ctx->dec_counter_bytes, counter_ints,
                                       partial_bytes, "decode workspace", stream, false, &counter_bytes);
        if (rc != B2A_OK) return rc;
        p.counters = static_cast<int*>(ctx->dec_ws);
        p.partials = reinterpret_cast<float*>(static_cast<char*>(ctx->dec_ws) + counter_bytes);
        p.target_items = target;
        p.item_capacity = cap;
        p.early_start = ctx->decode_early_start ? 1 : 0;
        const int B = p.B;
        // one launch covers at most kDecodeMaxBatchPerLaunch sequences and a key
        // stream (visible keys plus per-unit overhead keys) below 2^31 (the kernel's int32 prefix)
        const int per_launch = (int)std::min<int64_t>(kDecodeMaxBatchPerLaunch,
                                                      INT32_MAX / ((int64_t)p.max_seq + 1 + kDecodeGapKeysMax));
        for (int b0 = 0; b0 < B; b0 += per_launch) {
            DecodeParams s = p;
            s.B = std::min(per_launch, B - b0);
            const size_t qe = dtype_size(p.q_dtype), oe = dtype_size(p.out_dtype), ce = dtype_size(p.cache_dtype);
            s.q = static_cast<const char*>(p.q) + (size_t)b0 * q_stride_of(p) * qe;
            if (p.k_new) s.k_new = static_cast<const char*>(p.k_new) + (size_t)b0 * kvn_stride_of(p) * qe;
            if (p.v_new) s.v_new = static_cast<const char*>(p.v_new) + (size_t)b0 * kvn_stride_of(p) * qe;
            s.k_cache = static_cast<char*>(p.k_cache) + (size_t)b0 * p.stride_b * ce;
            s.v_cache = static_cast<char*>(p.v_cache) + (size_t)b0 * p.stride_b * ce;
            if (p.ctx_lens) s.ctx_lens = p.ctx_lens + b0;
            s.out = static_cast<char*>(p.out) + (size_t)b0 * p.Hq * p.D * oe;
            cudaError_t e = launch_decode_tc(s, ctx->device, stream);
            if (e != cudaSuccess) return cuda_fail(ctx, e, "decode kernel launch");
        }
        return B2A_OK;
    }
    cudaError_t e = launch_decode_simt(p, stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "decode kernel launch");
    return B2A_OK;
}

}  // namespace

namespace b2a {
// Message for b2a_last_error(NULL, ...) from entry points that take no context.
void set_thread_error(const char* msg) { g_create_error = msg ? msg : ""; }
}  // namespace b2a

extern "C" {

B2A_API const char* b2a_status_string(int status) {
    switch (status) {
        case B2A_OK: return "B2A_OK";
        case B2A_EINVAL: return "B2A_EINVAL";
        case B2A_ECUDA: return "B2A_ECUDA";
        case B2A_ENCCL: return "B2A_ENCCL";
        case B2A_ETIMEOUT: return "B2A_ETIMEOUT";
        case B2A_EOOM: return "B2A_EOOM";
        case B2A_ENOTSUP: return "B2A_ENOTSUP";
        case B2A_EDEVICE: return "B2A_EDEVICE";
        default: return "B2A_UNKNOWN";
    }
}

B2A_API int b2a_abi_version(void) { return B2A_ABI_VERSION; }

B2A_API const char* b2a_build_info(void) {
    return "libb200attn sm_100a; CUDA " __DATE__ " " __TIME__;
}

B2A_API int b2a_create(int device, b2a_context** out) {
    if (!out) return fail(nullptr, B2A_EINVAL, "out must not be null");
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(nullptr, B2A_ECUDA, "no CUDA device available: %s", cudaGetErrorString(e));
    }
    if (device < 0 || device >= n) return fail(nullptr, B2A_EINVAL, "device %d out of range [0, %d)", device, n);
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, device);
    if (e != cudaSuccess) return fail(nullptr, B2A_ECUDA, "cudaGetDeviceProperties: %s", cudaGetErrorString(e));
    if (prop.major != 10 || prop.minor != 0)
        return fail(nullptr, B2A_ENOTSUP, "device %d is sm_%d%d; this library is built for sm_100a (B200) only",
                    device, prop.major, prop.minor);
    DeviceGuard guard(device);
    if (!guard.ok) return fail(nullptr, B2A_ECUDA, "cudaSetDevice(%d) failed", device);
    b2a_context* ctx = new (std::nothrow) b2a_context();
    if (!ctx) return fail(nullptr, B2A_EOOM, "host allocation failed");
    ctx->device = device;
    ctx->sm_count = prop.multiProcessorCount;
    e = cudaMalloc(&ctx->status, kStatusBufferInts * sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(ctx->status, 0, kStatusBufferInts * sizeof(int));
    if (e == cudaSuccess) e = cudaMallocHost(&ctx->status_host, kStatusWords * sizeof(int));
    if (e != cudaSuccess) {
        if (ctx->status) cudaFree(ctx->status);
        delete ctx;
        cudaGetLastError();
        return fail(nullptr, e == cudaErrorMemoryAllocation ? B2A_EOOM : B2A_ECUDA, "status buffer: %s",
                    cudaGetErrorString(e));
    }
    *out = ctx;
    return B2A_OK;
}

B2A_API int b2a_destroy(b2a_context* ctx) {
    if (!ctx) return B2A_OK;
    {
        DeviceGuard guard(ctx->device);
        if (ctx->status) cudaFree(ctx->status);
        if (ctx->status_host) cudaFreeHost(ctx->status_host);
        if (ctx->dec_ws) cudaFree(ctx->dec_ws);
        if (ctx->pf_ws) cudaFree(ctx->pf_ws);
        if (ctx->split_ws) cudaFree(ctx->split_ws);
        if (ctx->blk_ws) cudaFree(ctx->blk_ws);
        if (ctx->rope_tab) cudaFree(ctx->rope_tab);
        if (ctx->lin_ws) cudaFree(ctx->lin_ws);
    }
    delete ctx;
    return B2A_OK;
}

B2A_API int b2a_last_error(const b2a_context* ctx, char* buf, size_t n) {
    const std::string& s = ctx ? ctx->last_error : g_create_error;
    if (buf && n > 0) {
        size_t k = std::min(n - 1, s.size());
        memcpy(buf, s.data(), k);
        buf[k] = '\0';
    }
    return (int)s.size();
}

B2A_API int b2a_set_workspace_limit(b2a_context* ctx, size_t bytes) {
    if (!ctx) return B2A_EINVAL;
    ctx->ws_limit = bytes;
    return B2A_OK;
}

B2A_API int b2a_set_decode_early_start(b2a_context* ctx, int enable) {
    if (!ctx) return B2A_EINVAL;
    ctx->decode_early_start = enable != 0;
    return B2A_OK;
}

B2A_API int b2a_workspace_bytes(const b2a_context* ctx, size_t* bytes) {
    if (!ctx || !bytes) return B2A_EINVAL;
    *bytes = ctx->dec_ws_bytes + ctx->pf_ws_bytes + ctx->split_ws_bytes + ctx->blk_ws_bytes + ctx->rope_tab_bytes +
             ctx->lin_ws_bytes;
    return B2A_OK;
}

B2A_API int b2a_reserve_decode(b2a_context* ctx, int max_batch, int num_q_heads, int num_kv_heads, int head_dim) {
    if (!ctx) return B2A_EINVAL;
    int rc = check_heads(ctx, num_q_heads, num_kv_heads);
    if (rc) return rc;
    if ((rc = check_head_dim(ctx, head_dim))) return rc;
    if (max_batch <= 0) return fail(ctx, B2A_EINVAL, "max_batch must be positive");
    if (!decode_tc_supported(head_dim, B2A_FLOAT16)) return B2A_OK;  // generic kernel needs no workspace
    DeviceGuard guard(ctx->device);
    const int n_hg = (num_q_heads / num_kv_heads + 7) / 8;
    int target = 0, cap = 0;
    size_t partial_bytes = 0;
    decode_tc_workspace(ctx->device, max_batch, num_kv_heads, n_hg, head_dim, B2A_FLOAT16, &target, &cap,
                        &partial_bytes);
    const size_t counter_ints = (size_t)std::min(max_batch, kDecodeMaxBatchPerLaunch) * num_kv_heads * n_hg;
    size_t counter_bytes = 0;
    return ensure_counted_buffer(ctx, &ctx->dec_ws, &ctx->dec_ws_bytes, &ctx->dec_counter_bytes, counter_ints,
                                 partial_bytes, "decode workspace", nullptr, true, &counter_bytes);
}

B2A_API int b2a_test_inject_wait_timeout(b2a_context* ctx) {
    if (!ctx) return B2A_EINVAL;
    ctx->inject_wait_timeout = true;
    return B2A_OK;
}

B2A_API int b2a_test_last_attention_kernel(const b2a_context* ctx) {
    return ctx ? ctx->last_attention_kernel : 0;
}

B2A_API int b2a_check_device_status(b2a_context* ctx, void* stream) {
    if (!ctx) return B2A_EINVAL;
    DeviceGuard guard(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // one stream-ordered copy of the flags into pinned memory, one synchronisation
    cudaError_t e = cudaMemcpyAsync(ctx->status_host, ctx->status, kStatusWords * sizeof(int),
                                    cudaMemcpyDeviceToHost, s);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "status read");
    e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "stream synchronize");
    const int flags = ctx->status_host[0];
    if (flags == 0) return B2A_OK;
    e = cudaMemsetAsync(ctx->status, 0, kStatusWords * sizeof(int), s);  // ordered before later launches
    if (e != cudaSuccess) return cuda_fail(ctx, e, "status clear");
    std::string msg;
    if (flags & 8) msg += "a bounded device wait ran out (attention pipeline aborted; its outputs are undefined). ";
    if (flags & 1) msg += "a ctx_lens entry was outside [0, max_seq); its outputs are NaN. ";
    if (flags & 2) msg += "decode work items exceeded the workspace capacity. ";
    if (flags & 4) msg += "a bf16 input exceeded the fp16 operand range (|x| > 65504). ";
    // a timed-out pipeline is reported as such; the other flags are failed device-side argument checks
    return fail(ctx, (flags & 8) ? B2A_ETIMEOUT : B2A_EDEVICE, "%s", msg.c_str());
}

// ----------------------------------------------------------------- encoder
B2A_API int b2a_mha(b2a_context* ctx, int in_dtype, int out_dtype, const void* q, const void* k, const void* v,
                    const float* mask, const int32_t* key_lengths, void* y, int B, int H, int S, int D, float scale,
                    int layout, void* stream) {
    if (!ctx) return B2A_EINVAL;
    if (!valid_dtype(in_dtype) || !valid_dtype(out_dtype))
        return fail(ctx, B2A_EINVAL, "unsupported element type (in %d, out %d)", in_dtype, out_dtype);
    if (!q || !k || !v || !y) return fail(ctx, B2A_EINVAL, "q, k, v and y tensors must not be null");
    if (mask && key_lengths) return fail(ctx, B2A_EINVAL, "pass either an additive mask or key lengths, not both");
    // DirectMlAttentionKernel constructor (WB/runtime/kernels/DirectMlAttentionKernel.java:109-111)
    if (B <= 0 || H <= 0 || S <= 0 || D <= 0) return fail(ctx, B2A_EINVAL, "batch, heads, seq, headDim must be > 0");
    if (D > kMaxHeadDim || D % 2) return fail(ctx, B2A_ENOTSUP, "headDim %d not supported (even, <= %d)", D, kMaxHeadDim);
    if (layout != B2A_HEAD_MAJOR && layout != B2A_SEQ_MAJOR) return fail(ctx, B2A_EINVAL, "unknown layout %d", layout);
    if (!(scale == scale) || scale <= 0.f) return fail(ctx, B2A_EINVAL, "scale must be a positive number");
    DeviceGuard guard(ctx->device);
    AttnParams p{};
    p.q = q;
    p.k = k;
    p.v = v;
    p.in_dtype = in_dtype;
    p.o = y;
    p.out_dtype = out_dtype;
    p.B = B;
    p.S = S;
    p.Hq = H;
    p.Hkv = H;
    p.D = D;
    if (layout == B2A_HEAD_MAJOR) {
        p.q_sb = (int64_t)H * S * D;
        p.q_ss = D;
        p.q_sh = (int64_t)S * D;
    } else {
        p.q_sb = (int64_t)S * H * D;
        p.q_ss = (int64_t)H * D;
        p.q_sh = D;
    }
    p.k_sb = p.q_sb;
    p.k_ss = p.q_ss;
    p.k_sh = p.q_sh;
    p.causal = 0;
    p.window = 0;
    p.mask = mask;
    p.key_len = key_lengths;
    p.scale = scale;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSuccess;
    if (in_dtype == B2A_BFLOAT16) {
        // short sequences: the tensor-core kernel converts the staged bf16 tiles to fp16 itself
        // (no pre-pass; measured on B200, bf16 B=64 H=12 S=128 D=32: 30.2 vs 36.3 us; S=512 D=64:
        // 56.8 vs 69.0 us; at S=1024 D=128 the pre-pass is faster, 142 vs 151 us)
        AttnParams t = p;
        t.xform = 7;
        if (S <= kInKernelPrepMaxSeq && attn_tcgen05_supported(t)) {
            e = launch_attention(ctx, t, s);
            if (e != cudaSuccess) return cuda_fail(ctx, e, "attention kernel launch");
            return B2A_OK;
        }
    }
    if (in_dtype == B2A_BFLOAT16) {
        // same operand rule as the prefill: bf16 inputs are multiplied as fp16
        const size_t n = (size_t)B * H * S * D;
        const size_t one = (n * 2 + 255) / 256 * 256;
        int rc = ensure_buffer(ctx, &ctx->pf_ws, &ctx->pf_ws_bytes, 3 * one, "encoder");
        if (rc) return rc;
        char* base = static_cast<char*>(ctx->pf_ws);
        const void* ptrs[] = {q, k, v};
        if (prep_vectorizable(D, (int64_t)n, ptrs, 3)) {  // one launch for the three conversions
            const PrepJob jobs[3] = {PrepJob{q, base, nullptr, H, 0}, PrepJob{k, base + one, nullptr, H, 0},
                                     PrepJob{v, base + 2 * one, nullptr, H, 0}};
            e = launch_prep(jobs, 3, B, S, D, in_dtype, B2A_FLOAT16, 0, B2A_ROPE_NONE, nullptr, nullptr, ctx->status,
                            s);
        } else {
            e = launch_convert(q, in_dtype, base, B2A_FLOAT16, (int64_t)n, ctx->status, s);
            if (e == cudaSuccess) e = launch_convert(k, in_dtype, base + one, B2A_FLOAT16, (int64_t)n, ctx->status, s);
            if (e == cudaSuccess)
                e = launch_convert(v, in_dtype, base + 2 * one, B2A_FLOAT16, (int64_t)n, ctx->status, s);
        }
        if (e != cudaSuccess) return cuda_fail(ctx, e, "conversion kernel launch");
        p.q = base;
        p.k = base + one;
        p.v = base + 2 * one;
        p.in_dtype = B2A_FLOAT16;
    }
    e = launch_attention(ctx, p, s);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "attention kernel launch");
    return B2A_OK;
}

// ----------------------------------------------------------------- prefill
B2A_API int b2a_prefill_causal(b2a_context* ctx, int in_dtype, int out_dtype, const void* q, const void* k,
                               const void* v, void* o, int B, int S, int Hq, int Hkv, int D, float scale, int rope_mode,
                               double rope_theta, int pos0, int window, void* k_rot_out, void* stream) {
    if (!ctx) return B2A_EINVAL;
    if (!valid_dtype(in_dtype) || !valid_dtype(out_dtype))
        return fail(ctx, B2A_EINVAL, "unsupported element type (in %d, out %d)", in_dtype, out_dtype);
    if (!q || !k || !v || !o) return fail(ctx, B2A_EINVAL, "q, k, v and o must not be null");
    int rc = check_heads(ctx, Hq, Hkv);
    if (rc) return rc;
    if ((rc = check_head_dim(ctx, D))) return rc;
    if (B <= 0 || S <= 0) return fail(ctx, B2A_EINVAL, "batch and sequence length must be > 0");
    if (window < 0) return fail(ctx, B2A_EINVAL, "window must not be negative");
    if (pos0 < 0) return fail(ctx, B2A_EINVAL, "pos0 must not be negative");
    if (rope_mode != B2A_ROPE_NONE && rope_mode != B2A_ROPE_NEOX && rope_mode != B2A_ROPE_GEMMA)
        return fail(ctx, B2A_EINVAL, "unknown rope mode %d", rope_mode);
    if (rope_mode != B2A_ROPE_NONE && !(rope_theta > 0.0)) return fail(ctx, B2A_EINVAL, "rope theta must be > 0");
    if (!(scale == scale) || scale <= 0.f) return fail(ctx, B2A_EINVAL, "scale must be a positive number");
    DeviceGuard guard(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);

    AttnParams p{};
    p.q = q;
    p.k = k;
    p.v = v;
    p.in_dtype = in_dtype;
    p.o = o;
    p.out_dtype = out_dtype;
    p.B = B;
    p.S = S;
    p.Hq = Hq;
    p.Hkv = Hkv;
    p.D = D;
    p.q_sb = (int64_t)S * Hq * D;
    p.q_ss = (int64_t)Hq * D;
    p.q_sh = D;
    p.k_sb = (int64_t)S * Hkv * D;
    p.k_ss = (int64_t)Hkv * D;
    p.k_sh = D;
    p.causal = 1;
    p.window = window;
    p.scale = scale;

    const size_t nq = (size_t)B * S * Hq * D, nk = (size_t)B * S * Hkv * D;
    auto r256 = [](size_t x) { return (x + 255) / 256 * 256; };

    // fp32 inputs (the fp32 kernels) with the NeoX rotation and no rotated-key output: the
    // kernel rotates q and k itself from the context's cached table -- one launch, no pre-pass
    if (in_dtype == B2A_FLOAT32 && rope_mode == B2A_ROPE_NEOX && k_rot_out == nullptr) {
        const float2* tab = nullptr;
        if ((int64_t)pos0 + S > INT32_MAX) return fail(ctx, B2A_EINVAL, "pos0 + S exceeds the position range");
        if ((rc = neox_table(ctx, rope_theta, D, pos0 + S, s, &tab))) return rc;
        p.rope_table = tab;
        p.rope_pos0 = pos0;
        const cudaError_t e = launch_attention(ctx, p, s);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "attention kernel launch");
        return B2A_OK;
    }

    // bf16 inputs are multiplied as fp16 tensor-core operands: the rotated q/k,
    // P and V then carry 11 significant bits instead of 8, which keeps short
    // causal rows within the 2e-3 tolerance (bf16 -> fp16 is exact inside the
    // fp16 range; values beyond it raise device status bit 2).
    const int cdt = in_dtype == B2A_BFLOAT16 ? B2A_FLOAT16 : in_dtype;
    const size_t ce = dtype_size(cdt);
    const bool rope = rope_mode != B2A_ROPE_NONE;
    const bool conv = cdt != in_dtype;
    // the vectorised pre-pass reads NeoX (cos, sin) rows from the context's cached float table;
    // Gemma's double table (and the row-wise fallback's) is built per call into the workspace
    const bool cached_table = rope_mode == B2A_ROPE_NEOX;
    const size_t table_bytes = rope ? r256((size_t)S * (D / 2) * 16) : 0;
    const size_t q_bytes = (rope || conv) ? r256(nq * ce) : 0;
    const bool k_in_out = rope && !conv && k_rot_out != nullptr;  // rotated keys land in k_rot_out directly
    const size_t k_bytes = ((rope || conv) && !k_in_out) ? r256(nk * ce) : 0;
    const size_t v_bytes = conv ? r256(nk * ce) : 0;
    if (table_bytes + q_bytes + k_bytes + v_bytes > 0) {
        rc = ensure_buffer(ctx, &ctx->pf_ws, &ctx->pf_ws_bytes, table_bytes + q_bytes + k_bytes + v_bytes, "prefill");
        if (rc) return rc;
    }
    char* base = static_cast<char*>(ctx->pf_ws);
    double2* table = reinterpret_cast<double2*>(base);
    void* q_c = base + table_bytes;
    void* k_c = k_in_out ? k_rot_out : base + table_bytes + q_bytes;
    void* v_c = base + table_bytes + q_bytes + k_bytes;
    cudaError_t e = cudaSuccess;
    const void* prep_ptrs[] = {q, k, v, q_c, k_c, v_c, k_rot_out};
    const bool vec_prep = (rope || conv) && prep_vectorizable(D, (int64_t)std::max(nq, nk), prep_ptrs, 7);
    if (vec_prep) {
        // one launch: q and k rotated / converted, v converted (NeoX: from the cached table,
        // else after a table build)
        double inv[kMaxHeadDim / 2] = {};
        if (rope) inv_freq_table(rope_theta, D, inv);
        double2* prep_table = table;
        if (rope && cached_table) {
            const float2* tab = nullptr;
            if ((int64_t)pos0 + S > INT32_MAX) return fail(ctx, B2A_EINVAL, "pos0 + S exceeds the position range");
            if ((rc = neox_table(ctx, rope_theta, D, pos0 + S, s, &tab))) return rc;
            prep_table = reinterpret_cast<double2*>(const_cast<float2*>(tab + (size_t)pos0 * (D / 2)));
        }
        PrepJob jobs[3];
        int nj = 0;
        jobs[nj++] = PrepJob{q, q_c, nullptr, Hq, rope ? 1 : 0};
        jobs[nj++] = PrepJob{k, k_c, (rope && k_rot_out && !k_in_out) ? k_rot_out : nullptr, Hkv, rope ? 1 : 0};
        if (conv) jobs[nj++] = PrepJob{v, v_c, nullptr, Hkv, 0};
        e = launch_prep(jobs, nj, B, S, D, in_dtype, cdt, pos0, rope_mode, inv, prep_table, ctx->status, s,
                        rope && cached_table);
        if (e == cudaSuccess && !rope && k_rot_out)
            e = cudaMemcpyAsync(k_rot_out, k, nk * dtype_size(in_dtype), cudaMemcpyDeviceToDevice, s);
    } else if (rope) {
        double inv[kMaxHeadDim / 2];
        inv_freq_table(rope_theta, D, inv);
        e = launch_rope_rows_with_table(q, in_dtype, q_c, cdt, B, S, Hq, D, p.q_sb, p.q_ss, p.q_sh, p.q_sb, p.q_ss,
                                        p.q_sh, pos0, rope_mode, inv, table, true, ctx->status, s);
        if (e == cudaSuccess)
            e = launch_rope_rows_with_table(k, in_dtype, k_c, cdt, B, S, Hkv, D, p.k_sb, p.k_ss, p.k_sh, p.k_sb,
                                            p.k_ss, p.k_sh, pos0, rope_mode, inv, table, false, ctx->status, s);
        if (e == cudaSuccess && k_rot_out && !k_in_out)  // caller wants rotated keys in its own dtype
            e = launch_rope_rows_with_table(k, in_dtype, k_rot_out, in_dtype, B, S, Hkv, D, p.k_sb, p.k_ss, p.k_sh,
                                            p.k_sb, p.k_ss, p.k_sh, pos0, rope_mode, inv, table, false, nullptr, s);
    } else {
        if (conv) {
            e = launch_convert(q, in_dtype, q_c, cdt, (int64_t)nq, ctx->status, s);
            if (e == cudaSuccess) e = launch_convert(k, in_dtype, k_c, cdt, (int64_t)nk, ctx->status, s);
        }
        if (e == cudaSuccess && k_rot_out)
            e = cudaMemcpyAsync(k_rot_out, k, nk * dtype_size(in_dtype), cudaMemcpyDeviceToDevice, s);
    }
    if (e == cudaSuccess && conv && !vec_prep) e = launch_convert(v, in_dtype, v_c, cdt, (int64_t)nk, ctx->status, s);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "rope / conversion kernel launch");
    if (rope || conv) {
        p.q = q_c;
        p.k = k_c;
    }
    if (conv) p.v = v_c;
    p.in_dtype = cdt;
    e = launch_attention(ctx, p, s);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "attention kernel launch");
    return B2A_OK;
}

// ----------------------------------------------------------------- Gemma prefill
B2A_API int b2a_prefill_gemma(b2a_context* ctx, int in_dtype, int out_dtype, const void* q, const void* k, const void* v,
                              void* o, int B, int S, int Hq, int Hkv, int D, float scale, int rope_mode,
                              double rope_theta, int pos0, int window, const float* q_norm_w, const float* k_norm_w,
                              float norm_eps, void* k_rot_out, void* stream) {
    // Gemma3WarpLayer.forwardPrefillBatched steps 3-4 (INF/gemma/Gemma3WarpLayer.java:395-411): per position QK-norm,
    // RoPE at p, KV append, then one attention over [firstValid(p), p] per position; here the
    // norm + rotation of all positions is one pre-pass and the attention one launch.
    if (!ctx) return B2A_EINVAL;
    if (!valid_dtype(in_dtype) || !valid_dtype(out_dtype))
        return fail(ctx, B2A_EINVAL, "unsupported element type (in %d, out %d)", in_dtype, out_dtype);
    if (!q || !k || !v || !o) return fail(ctx, B2A_EINVAL, "q, k, v and o must not be null");
    int rc = check_heads(ctx, Hq, Hkv);
    if (rc) return rc;
    if ((rc = check_head_dim(ctx, D))) return rc;
    if (B <= 0 || S <= 0) return fail(ctx, B2A_EINVAL, "batch and sequence length must be > 0");
    if (window < 0) return fail(ctx, B2A_EINVAL, "window must not be negative");
    if (pos0 < 0) return fail(ctx, B2A_EINVAL, "pos0 must not be negative");
    if (rope_mode != B2A_ROPE_NONE && rope_mode != B2A_ROPE_NEOX && rope_mode != B2A_ROPE_GEMMA)
        return fail(ctx, B2A_EINVAL, "unknown rope mode %d", rope_mode);
    if (rope_mode != B2A_ROPE_NONE && !(rope_theta > 0.0)) return fail(ctx, B2A_EINVAL, "rope theta must be > 0");
    if (!(scale == scale) || scale <= 0.f) return fail(ctx, B2A_EINVAL, "scale must be a positive number");
    if (!(norm_eps >= 0.f)) return fail(ctx, B2A_EINVAL, "norm eps must not be negative");
    DeviceGuard guard(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);

    // same operand rule as b2a_prefill_causal: bf16 inputs are multiplied as fp16
    const int cdt = in_dtype == B2A_BFLOAT16 ? B2A_FLOAT16 : in_dtype;
    const size_t ce = dtype_size(cdt);
    const size_t nq = (size_t)B * S * Hq * D, nk = (size_t)B * S * Hkv * D;
    auto r256 = [](size_t x) { return (x + 255) / 256 * 256; };
    const bool rope = rope_mode != B2A_ROPE_NONE;
    const bool conv = cdt != in_dtype;
    const size_t table_bytes = rope ? r256((size_t)S * (D / 2) * 16) : 0;
    const size_t q_bytes = r256(nq * ce), k_bytes = r256(nk * ce), v_bytes = conv ? r256(nk * ce) : 0;
    rc = ensure_buffer(ctx, &ctx->pf_ws, &ctx->pf_ws_bytes, table_bytes + q_bytes + k_bytes + v_bytes, "prefill");
    if (rc) return rc;
    char* base = static_cast<char*>(ctx->pf_ws);
    double2* table = reinterpret_cast<double2*>(base);
    void* q_c = base + table_bytes;
    void* k_c = base + table_bytes + q_bytes;
    void* v_c = conv ? base + table_bytes + q_bytes + k_bytes : const_cast<void*>(v);
    double inv[kMaxHeadDim / 2] = {};
    if (rope) inv_freq_table(rope_theta, D, inv);
    cudaError_t e = launch_norm_rope_rows(q, q_c, nullptr, in_dtype, cdt, B, S, Hq, D, q_norm_w, norm_eps, rope_mode,
                                          pos0, inv, table, true, ctx->status, s);
    if (e == cudaSuccess)
        e = launch_norm_rope_rows(k, k_c, k_rot_out, in_dtype, cdt, B, S, Hkv, D, k_norm_w, norm_eps, rope_mode, pos0,
                                  inv, table, false, ctx->status, s);
    if (e == cudaSuccess && conv) e = launch_convert(v, in_dtype, v_c, cdt, (int64_t)nk, ctx->status, s);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "norm / rope / conversion kernel launch");

    AttnParams p{};
    p.q = q_c;
    p.k = k_c;
    p.v = v_c;
    p.in_dtype = cdt;
    p.o = o;
    p.out_dtype = out_dtype;
    p.B = B;
    p.S = S;
    p.Hq = Hq;
    p.Hkv = Hkv;
    p.D = D;
    p.q_sb = (int64_t)S * Hq * D;
    p.q_ss = (int64_t)Hq * D;
    p.q_sh = D;
    p.k_sb = (int64_t)S * Hkv * D;
    p.k_ss = (int64_t)Hkv * D;
    p.k_sh = D;
    p.causal = 1;
    p.window = window;
    p.scale = scale;
    e = launch_attention(ctx, p, s);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "attention kernel launch");
    return B2A_OK;
}

// ----------------------------------------------------------------- decode
B2A_API int b2a_decode(b2a_context* ctx, int q_dtype, int cache_dtype, int out_dtype, const void* q_new,
                       const void* k_new, const void* v_new, void* k_cache, void* v_cache, int kv_layout,
                       const int32_t* ctx_lens, int B, int Hq, int Hkv, int D, int max_seq, float scale,
                       int rope_mode, double rope_theta, int window, const float* q_norm_w, const float* k_norm_w,
                       float norm_eps, void* o, void* stream) {
    if (!ctx) return B2A_EINVAL;
    if (!valid_dtype(q_dtype) || !valid_dtype(cache_dtype) || !valid_dtype(out_dtype))
        return fail(ctx, B2A_EINVAL, "unsupported element type (q %d, cache %d, out %d)", q_dtype, cache_dtype,
                    out_dtype);
    if (!q_new || !k_new || !v_new || !k_cache || !v_cache || !ctx_lens || !o)
        return fail(ctx, B2A_EINVAL, "q_new, k_new, v_new, caches, ctx_lens and o must not be null");
    int rc = check_heads(ctx, Hq, Hkv);
    if (rc) return rc;
    if ((rc = check_head_dim(ctx, D))) return rc;
    if (B <= 0) return fail(ctx, B2A_EINVAL, "batch must be > 0");
    if (max_seq <= 0) return fail(ctx, B2A_EINVAL, "max_seq must be > 0");
    if (window < 0) return fail(ctx, B2A_EINVAL, "window must not be negative");
    if (kv_layout != B2A_KV_HEAD_MAJOR && kv_layout != B2A_KV_POS_MAJOR)
        return fail(ctx, B2A_EINVAL, "unknown kv layout %d", kv_layout);
    if (rope_mode != B2A_ROPE_NONE && rope_mode != B2A_ROPE_NEOX && rope_mode != B2A_ROPE_GEMMA)
        return fail(ctx, B2A_EINVAL, "unknown rope mode %d", rope_mode);
    if (rope_mode != B2A_ROPE_NONE && !(rope_theta > 0.0)) return fail(ctx, B2A_EINVAL, "rope theta must be > 0");
    if ((q_norm_w == nullptr) != (k_norm_w == nullptr))
        return fail(ctx, B2A_EINVAL, "q_norm_w and k_norm_w must be given together");
    if (!(scale == scale) || scale <= 0.f) return fail(ctx, B2A_EINVAL, "scale must be a positive number");
    if (q_norm_w && !(norm_eps >= 0.f)) return fail(ctx, B2A_EINVAL, "norm_eps must not be negative");
    DeviceGuard guard(ctx->device);
    DecodeParams p{};
    p.q = q_new;
    p.k_new = k_new;
    p.v_new = v_new;
    p.q_dtype = q_dtype;
    p.k_cache = k_cache;
    p.v_cache = v_cache;
    p.cache_dtype = cache_dtype;
    p.stride_b = (int64_t)Hkv * max_seq * D;
    if (kv_layout == B2A_KV_HEAD_MAJOR) {
        p.stride_h = (int64_t)max_seq * D;
        p.stride_pos = D;
    } else {
        p.stride_h = D;
        p.stride_pos = (int64_t)Hkv * D;
    }
    p.ctx_lens = ctx_lens;
    p.B = B;
    p.Hq = Hq;
    p.Hkv = Hkv;
    p.G = Hq / Hkv;
    p.D = D;
    p.max_seq = max_seq;
    p.window = window;
    p.first_explicit = -1;
    p.append = 1;
    p.rope_mode = rope_mode;
    p.scale = scale;
    p.q_norm_w = q_norm_w;
    p.k_norm_w = k_norm_w;
    p.norm_eps = norm_eps;
    p.out = o;
    p.out_dtype = out_dtype;
    if (rope_mode != B2A_ROPE_NONE) inv_freq_table(rope_theta, D, p.inv_freq);
    return run_decode(ctx, p, static_cast<cudaStream_t>(stream), true);
}

// ------------------------------------------------- reference GPU contracts
B2A_API int b2a_qwen_rope_and_append(b2a_context* ctx, float* q, const float* k, const float* v, float* k_cache,
                                     float* v_cache, int num_heads, int kv_heads, int head_dim, int pos,
                                     int max_seq_len, float rope_theta, void* stream) {
    if (!ctx) return B2A_EINVAL;
    if (!q || !k || !v || !k_cache || !v_cache) return fail(ctx, B2A_EINVAL, "buffers must not be null");
    if (num_heads <= 0 || kv_heads <= 0) return fail(ctx, B2A_EINVAL, "numHeads and kvHeads must be positive");
    int rc = check_head_dim(ctx, head_dim);
    if (rc) return rc;
    if (pos < 0 || pos >= max_seq_len) return fail(ctx, B2A_EINVAL, "pos %d outside [0, maxSeqLen=%d)", pos, max_seq_len);
    if (!(rope_theta > 0.f)) return fail(ctx, B2A_EINVAL, "rope theta must be > 0");
    DeviceGuard guard(ctx->device);
    double inv[kMaxHeadDim / 2];
    inv_freq_table((double)rope_theta, head_dim, inv);
    cudaError_t e = launch_qwen_rope_append(q, k, v, k_cache, v_cache, num_heads, kv_heads, head_dim, pos, max_seq_len,
                                            inv, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(ctx, e, "rope_and_append launch");
    return B2A_OK;
}

B2A_API int b2a_qwen_gqa_attention_decode(b2a_context* ctx, const float* q, const float* k_cache, const float* v_cache,
                                          float* attn_out, int num_heads, int kv_heads, int head_dim,
                                          int q_heads_per_kv_head, int seq_len, int max_seq_len, float scale,
                                          void* stream) {
    if (!ctx) return B2A_EINVAL;
    if (!q || !k_cache || !v_cache || !attn_out) return fail(ctx, B2A_EINVAL, "buffers must not be null");
    int rc = check_heads(ctx, num_heads, kv_heads);
    if (rc) return rc;
    if (q_heads_per_kv_head != num_heads / kv_heads)
        return fail(ctx, B2A_EINVAL, "qHeadsPerKvHead %d != numHeads / kvHeads = %d", q_heads_per_kv_head,
                    num_heads / kv_heads);
    if ((rc = check_head_dim(ctx, head_dim))) return rc;
    if (seq_len <= 0 || seq_len > max_seq_len)
        return fail(ctx, B2A_EINVAL, "seqLen %d outside [1, maxSeqLen=%d]", seq_len, max_seq_len);
    if (!(scale == scale) || scale <= 0.f) return fail(ctx, B2A_EINVAL, "scale must be a positive number");
    DeviceGuard guard(ctx->device);
    DecodeParams p{};
    p.q = q;
    p.q_dtype = B2A_FLOAT32;
    p.k_cache = const_cast<float*>(k_cache);
    p.v_cache = const_cast<float*>(v_cache);
    p.cache_dtype = B2A_FLOAT32;
    p.stride_b = 0;
    p.stride_h = (int64_t)max_seq_len * head_dim;
    p.stride_pos = head_dim;
    p.ctx_lens = nullptr;
    p.pos_scalar = seq_len - 1;
    p.B = 1;
    p.Hq = num_heads;
    p.Hkv = kv_heads;
    p.G = q_heads_per_kv_head;
    p.D = head_dim;
    p.max_seq = max_seq_len;
    p.first_explicit = 0;
    p.append = 0;
    p.scale = scale;
    p.out = attn_out;
    p.out_dtype = B2A_FLOAT32;
    return run_decode(ctx, p, static_cast<cudaStream_t>(stream), false);
}

B2A_API int b2a_qwen_decode_step(b2a_context* ctx, const float* qkv, const float* qkv_bias, float* k_cache,
                                 float* v_cache, float* attn_out, int num_heads, int kv_heads, int head_dim, int pos,
                                 int max_seq_len, float rope_theta, float scale, void* stream) {
    // QwenGpuPipeline.decodeLayerGpuResident steps 1b-3 in one launch
    // (INF/qwen/QwenGpuPipeline.java:647-691): bias add on the fused [Q|K|V] row, RoPE of q and k
    // at pos, k/v append at pos, GQA attention over cache positions [0, pos].
    if (!ctx) return B2A_EINVAL;
    if (!qkv || !k_cache || !v_cache || !attn_out)
        return fail(ctx, B2A_EINVAL, "qkv, caches and attn_out must not be null");
    int rc = check_heads(ctx, num_heads, kv_heads);
    if (rc) return rc;
    if ((rc = check_head_dim(ctx, head_dim))) return rc;
    if (pos < 0 || pos >= max_seq_len) return fail(ctx, B2A_EINVAL, "pos %d outside [0, maxSeqLen=%d)", pos, max_seq_len);
    if (!(rope_theta > 0.f)) return fail(ctx, B2A_EINVAL, "rope theta must be > 0");
    if (!(scale == scale) || scale <= 0.f) return fail(ctx, B2A_EINVAL, "scale must be a positive number");
    DeviceGuard guard(ctx->device);
    const int64_t q_size = (int64_t)num_heads * head_dim, kv_size = (int64_t)kv_heads * head_dim;
    DecodeParams p{};
    p.q = qkv;
    p.k_new = qkv + q_size;
    p.v_new = qkv + q_size + kv_size;
    p.q_dtype = B2A_FLOAT32;
    p.q_seq_stride = p.kv_new_seq_stride = q_size + 2 * kv_size;
    if (qkv_bias) {
        p.q_bias = qkv_bias;
        p.k_bias = qkv_bias + q_size;
        p.v_bias = qkv_bias + q_size + kv_size;
    }
    p.k_cache = k_cache;
    p.v_cache = v_cache;
    p.cache_dtype = B2A_FLOAT32;
    p.stride_b = 0;
    p.stride_h = (int64_t)max_seq_len * head_dim;
    p.stride_pos = head_dim;
    p.ctx_lens = nullptr;
    p.pos_scalar = pos;
    p.B = 1;
    p.Hq = num_heads;
    p.Hkv = kv_heads;
    p.G = num_heads / kv_heads;
    p.D = head_dim;
    p.max_seq = max_seq_len;
    p.first_explicit = 0;
    p.append = 1;
    p.rope_mode = B2A_ROPE_NEOX;
    inv_freq_table((double)rope_theta, head_dim, p.inv_freq);
    p.scale = scale;
    p.out = attn_out;
    p.out_dtype = B2A_FLOAT32;
    return run_decode(ctx, p, static_cast<cudaStream_t>(stream), false);
}

B2A_API int b2a_gemma_fused_attention_context(b2a_context* ctx, const float* q, const float* keys, const float* values,
                                              float* ctx_out, int num_heads, int groups_per_kv, int head_dim,
                                              int kv_dim, int first_valid, int query_pos, float scale, void* stream) {
    if (!ctx) return B2A_EINVAL;
    if (!q || !keys || !values || !ctx_out) return fail(ctx, B2A_EINVAL, "buffers must not be null");
    // Gemma3WarpFusedAttentionContextKernel.context (INF/gemma/Gemma3WarpFusedAttentionContextKernel.java:111-124)
    if (num_heads <= 0 || groups_per_kv <= 0 || num_heads % groups_per_kv != 0)
        return fail(ctx, B2A_EINVAL, "numHeads must be a multiple of numKvHeads");
    if (head_dim > 256)
        return fail(ctx, B2A_EINVAL, "headDim %d exceeds fused-attention group size 256", head_dim);
    int rc = check_head_dim(ctx, head_dim);
    if (rc) return rc;
    const int n_kv = num_heads / groups_per_kv;
    if (kv_dim < n_kv * head_dim) return fail(ctx, B2A_EINVAL, "kvDim %d < numKvHeads * headDim", kv_dim);
    if (query_pos < 0 || first_valid < 0 || first_valid > query_pos)
        return fail(ctx, B2A_EINVAL, "visible key range [%d, %d] is empty or negative", first_valid, query_pos);
    if (!(scale == scale) || scale <= 0.f) return fail(ctx, B2A_EINVAL, "scale must be a positive number");
    DeviceGuard guard(ctx->device);
    DecodeParams p{};
    p.q = q;
    p.q_dtype = B2A_FLOAT32;
    p.k_cache = const_cast<float*>(keys);
    p.v_cache = const_cast<float*>(values);
    p.cache_dtype = B2A_FLOAT32;
    p.stride_b = 0;
    p.stride_h = head_dim;
    p.stride_pos = kv_dim;
    p.ctx_lens = nullptr;
    p.pos_scalar = query_pos;
    p.B = 1;
    p.Hq = num_heads;
    p.Hkv = n_kv;
    p.G = groups_per_kv;
    p.D = head_dim;
    p.max_seq = query_pos + 1;
    p.first_explicit = first_valid;
    p.append = 0;
    p.scale = scale;
    p.out = ctx_out;
    p.out_dtype = B2A_FLOAT32;
    return run_decode(ctx, p, static_cast<cudaStream_t>(stream), false);
}

// ----------------------------------------------------------------- projections
namespace {
// b2a_linear; early: launched with programmatic serialisation (the projections of
// b2a_decode_attention_block under b2a_set_decode_early_start)
int run_linear(b2a_context* ctx, int in_dtype, int out_dtype, const void* x, const void* w, const float* bias,
               const void* residual, void* y, int M, int N, int K, void* stream, bool early) {
    if (!ctx) return B2A_EINVAL;
    if (!x || !w || !y) return fail(ctx, B2A_EINVAL, "x, w and y must not be null");
    if (in_dtype != B2A_FLOAT16 && in_dtype != B2A_BFLOAT16)
        return fail(ctx, B2A_ENOTSUP, "b2a_linear multiplies 16-bit operands (FLOAT16 or BFLOAT16), got %d", in_dtype);
    if (!valid_dtype(out_dtype)) return fail(ctx, B2A_EINVAL, "unsupported output element type %d", out_dtype);
    if (M <= 0 || N <= 0 || K <= 0) return fail(ctx, B2A_EINVAL, "M, N and K must be > 0");
    if (K % 8 != 0) return fail(ctx, B2A_EINVAL, "K must be a multiple of 8 (16-byte rows for the TMA loads)");
    DeviceGuard guard(ctx->device);
    if (!linear_tc_supported(in_dtype, K, K, K, x, w))
        return fail(ctx, B2A_EINVAL, "x and w must be 16-byte aligned");
    LinearArgs a{};
    a.x = x;
    a.ldx = K;
    a.w = w;
    a.ldw = K;
    a.in_dtype = in_dtype;
    a.bias = bias;
    a.residual = residual;
    a.ldr = N;
    a.y = y;
    a.ldy = N;
    a.out_dtype = out_dtype;
    a.M = M;
    a.N = N;
    a.K = K;
    a.ksplit = 1;
    a.early = early ? 1 : 0;
    // launches with too few output tiles to fill the GPU split K over CTAs (without room for the
    // split workspace under the context's limit they run unsplit)
    size_t acc_bytes = 0, counter_ints = 0;
    const int ks = linear_split_plan(M, N, K, ctx->sm_count, &acc_bytes, &counter_ints);
    if (ks > 1) {
        // the accumulator counts as counter region: zeroed when new or grown, kept zero by the kernel
        const size_t region_ints = counter_ints + (acc_bytes + sizeof(int) - 1) / sizeof(int) + 64;
        size_t region_bytes = 0;
        if (ensure_counted_buffer(ctx, &ctx->lin_ws, &ctx->lin_ws_bytes, &ctx->lin_region, region_ints, 0,
                                  "projection split workspace", static_cast<cudaStream_t>(stream), false,
                                  &region_bytes) == B2A_OK) {
            a.ksplit = ks;
            a.counters = static_cast<int*>(ctx->lin_ws);
            a.acc = reinterpret_cast<float*>(static_cast<char*>(ctx->lin_ws) + (counter_ints * sizeof(int) + 255) / 256 * 256);
        } else {
            ctx->last_error.clear();  // the refused workspace is not an error of this call
        }
    }
    const cudaError_t e = launch_linear_tc(a, ctx->status, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(ctx, e, "linear kernel launch");
    return B2A_OK;
}
}  // namespace

B2A_API int b2a_linear(b2a_context* ctx, int in_dtype, int out_dtype, const void* x, const void* w, const float* bias,
                       const void* residual, void* y, int M, int N, int K, void* stream) {
    return run_linear(ctx, in_dtype, out_dtype, x, w, bias, residual, y, M, N, K, stream, false);
}

B2A_API int b2a_decode_attention_block(b2a_context* ctx, int act_dtype, int cache_dtype, const void* x,
                                       const void* w_qkv, const float* b_qkv, void* k_cache, void* v_cache,
                                       int kv_layout, const int32_t* ctx_lens, const void* w_o, const void* residual,
                                       void* y, int B, int hidden, int Hq, int Hkv, int D, int max_seq, float scale,
                                       double rope_theta, int window, void* stream) {
    // Qwen2Runtime.processLayerDecode from the normed input to residual 1
    // (INF/qwen/Qwen2Runtime.java:693-777): QKV projection + bias, RoPE, KV append, GQA
    // attention, O projection + residual, in three launches -- the bias in the QKV GEMM's
    // epilogue, RoPE and the append in the attention's prologue, the residual in the O GEMM's
    // epilogue.
    if (!ctx) return B2A_EINVAL;
    if (!x || !w_qkv || !k_cache || !v_cache || !ctx_lens || !w_o || !y)
        return fail(ctx, B2A_EINVAL, "x, w_qkv, caches, ctx_lens, w_o and y must not be null");
    if (act_dtype != B2A_FLOAT16 && act_dtype != B2A_BFLOAT16)
        return fail(ctx, B2A_ENOTSUP, "activations and weights must be FLOAT16 or BFLOAT16");
    int rc = check_heads(ctx, Hq, Hkv);
    if (rc) return rc;
    if ((rc = check_head_dim(ctx, D))) return rc;
    if (B <= 0 || hidden <= 0 || max_seq <= 0) return fail(ctx, B2A_EINVAL, "B, hidden and max_seq must be > 0");
    if (hidden % 8 != 0 || (Hq * D) % 8 != 0)
        return fail(ctx, B2A_EINVAL, "hidden and Hq*D must be multiples of 8 (16-byte rows for the TMA loads)");
    if (!(rope_theta > 0.0)) return fail(ctx, B2A_EINVAL, "rope theta must be > 0");
    DeviceGuard guard(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int nqkv = (Hq + 2 * Hkv) * D;
    const size_t qkv_bytes = ((size_t)B * nqkv * 4 + 255) / 256 * 256;
    const size_t attn_bytes = (size_t)B * Hq * D * 2;
    rc = ensure_buffer(ctx, &ctx->blk_ws, &ctx->blk_ws_bytes, qkv_bytes + attn_bytes, "attention block");
    if (rc) return rc;
    float* qkv = static_cast<float*>(ctx->blk_ws);
    void* attn = static_cast<char*>(ctx->blk_ws) + qkv_bytes;
    // 1. qkv = x W_qkv^T + b (fp32 rows [Q | K | V], as the reference keeps them)
    if ((rc = run_linear(ctx, act_dtype, B2A_FLOAT32, x, w_qkv, b_qkv, nullptr, qkv, B, nqkv, hidden, stream,
                         ctx->decode_early_start)))
        return rc;
    // 2. RoPE of q and k at ctx_lens[b], k/v append, attention (the decode kernel reads the fused rows)
    DecodeParams p{};
    p.q = qkv;
    p.k_new = qkv + (int64_t)Hq * D;
    p.v_new = qkv + (int64_t)(Hq + Hkv) * D;
    p.q_dtype = B2A_FLOAT32;
    p.q_seq_stride = p.kv_new_seq_stride = nqkv;
    p.k_cache = k_cache;
    p.v_cache = v_cache;
    p.cache_dtype = cache_dtype;
    p.stride_b = (int64_t)Hkv * max_seq * D;
    if (kv_layout == B2A_KV_HEAD_MAJOR) {
        p.stride_h = (int64_t)max_seq * D;
        p.stride_pos = D;
    } else if (kv_layout == B2A_KV_POS_MAJOR) {
        p.stride_h = D;
        p.stride_pos = (int64_t)Hkv * D;
    } else {
        return fail(ctx, B2A_EINVAL, "unknown kv layout %d", kv_layout);
    }
    if (!valid_dtype(cache_dtype)) return fail(ctx, B2A_EINVAL, "unsupported cache element type %d", cache_dtype);
    p.ctx_lens = ctx_lens;
    p.B = B;
    p.Hq = Hq;
    p.Hkv = Hkv;
    p.G = Hq / Hkv;
    p.D = D;
    p.max_seq = max_seq;
    p.window = window;
    p.first_explicit = -1;
    p.append = 1;
    p.rope_mode = B2A_ROPE_NEOX;
    inv_freq_table(rope_theta, D, p.inv_freq);
    p.scale = scale;
    p.out = attn;
    p.out_dtype = act_dtype;
    if ((rc = run_decode(ctx, p, s, true))) return rc;
    // 3. y = attn W_o^T + residual
    return run_linear(ctx, act_dtype, act_dtype, attn, w_o, nullptr, residual, y, B, hidden, Hq * D, stream,
                      ctx->decode_early_start);
}

// ----------------------------------------------------------------- sharding
B2A_API int b2a_partition_units(int n_units, int n_ranks, const int64_t* unit_cost, int32_t* rank_of_unit) {
    if (n_units <= 0 || n_ranks <= 0 || !unit_cost || !rank_of_unit) return B2A_EINVAL;
    if (n_units % n_ranks != 0) return B2A_EINVAL;
    const int cap = n_units / n_ranks;
    std::vector<int> order(n_units);
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return unit_cost[a] > unit_cost[b]; });
    std::vector<int64_t> load(n_ranks, 0);
    std::vector<int> count(n_ranks, 0);
    for (int u : order) {
        int best = -1;
        for (int r = 0; r < n_ranks; ++r) {
            if (count[r] >= cap) continue;
            if (best < 0 || load[r] < load[best]) best = r;
        }
        rank_of_unit[u] = best;
        load[best] += unit_cost[u];
        ++count[best];
    }
    return B2A_OK;
}

}  // extern "C"
