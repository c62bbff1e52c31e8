// decode_noalloc.cu -- b2a_decode_noalloc: the fused decode step for callers
// that must not allocate device memory.
//
// Who needs it: hosts whose device memory is owned by another allocator -- a
// JVM or serving runtime that hands this library slices of its own arena or
// caching pool.  For them a cudaMalloc outside the arena can fail once the
// arena has reserved the device, and cudaMalloc / cudaFree synchronise the
// device, stalling the serving loop.  b2a_decode needs a context, whose
// creation and first decode call cudaMalloc their workspace; this entry point
// takes no context and allocates nothing.
//
// Its scratch (the split-KV partial slots, the per-unit merge counters and a
// status word) is the file-scope array g_decode_scratch below: a fixed
// kScratchBytes on every GPU that loads the library, held until the process
// exits.  Host code must not pass the array's name to a kernel (on the host
// it is only a stand-in for the symbol); the first call on each device, with
// that device current, resolves its device address with
// cudaGetSymbolAddress and caches it.  Make that first call before any
// stream capture begins.
//
// All calls share the one array and it keeps the last call's contents: each
// call clears the merge counters on its stream before the kernel, and calls
// whose kernels overlap on the GPU (different streams, or different host
// threads) race on the array -- serialise them.
#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>

#include <mutex>

#include "../../include/b200attn.h"
#include "internal.h"

namespace b2a {
namespace {

constexpr size_t kScratchBytes = size_t(4) << 20;  // 4 MiB per device
constexpr size_t kStatusBytes = 256;
constexpr int kMaxUnits = 16384;  // sequences x kv heads x head groups of 8, per call
constexpr size_t kCounterBytes = size_t(kMaxUnits) * sizeof(int);
constexpr size_t kPartialBytes = kScratchBytes - kStatusBytes - kCounterBytes;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_decode_scratch[kScratchBytes];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of g_decode_scratch on the current device (resolved once).
cudaError_t scratch_for(int device, unsigned char** out) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_scratch_ptr[device] == nullptr) {
        void* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_decode_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_ptr[device] = ptr;
    }
    *out = static_cast<unsigned char*>(g_scratch_ptr[device]);
    return cudaSuccess;
}

int reject(int status, const char* fmt, long long a = 0, long long b = 0) {
    char buf[512];
    snprintf(buf, sizeof(buf), fmt, a, b);
    set_thread_error(buf);
    return status;
}

}  // namespace
}  // namespace b2a

using namespace b2a;

extern "C" B2A_API int b2a_decode_noalloc(int q_dtype, int cache_dtype, int out_dtype, const void* q_new,
                                          const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                                          int kv_layout, const int32_t* ctx_lens, int B, int Hq, int Hkv, int D,
                                          int max_seq, float scale, int rope_mode, double rope_theta, int window,
                                          const float* q_norm_w, const float* k_norm_w, float norm_eps, void* o,
                                          void* stream) {
    auto ok_dtype = [](int d) { return d == B2A_FLOAT32 || d == B2A_FLOAT16 || d == B2A_BFLOAT16; };
    if (!ok_dtype(q_dtype) || !ok_dtype(out_dtype)) return reject(B2A_EINVAL, "unsupported element type");
    if (!q_new || !k_new || !v_new || !k_cache || !v_cache || !ctx_lens || !o)
        return reject(B2A_EINVAL, "q_new, k_new, v_new, caches, ctx_lens and o must not be null");
    if (Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0)
        return reject(B2A_EINVAL, "numQueryHeads must be divisible by numKeyValueHeads for grouped-query attention");
    if (B <= 0 || max_seq <= 0 || window < 0) return reject(B2A_EINVAL, "batch and max_seq must be > 0, window >= 0");
    if (kv_layout != B2A_KV_HEAD_MAJOR && kv_layout != B2A_KV_POS_MAJOR)
        return reject(B2A_EINVAL, "unknown kv layout %lld", kv_layout);
    if (rope_mode != B2A_ROPE_NONE && rope_mode != B2A_ROPE_NEOX && rope_mode != B2A_ROPE_GEMMA)
        return reject(B2A_EINVAL, "unknown rope mode %lld", rope_mode);
    if (rope_mode != B2A_ROPE_NONE && !(rope_theta > 0.0)) return reject(B2A_EINVAL, "rope theta must be > 0");
    if ((q_norm_w == nullptr) != (k_norm_w == nullptr))
        return reject(B2A_EINVAL, "q_norm_w and k_norm_w must be given together");
    if (!(scale > 0.f)) return reject(B2A_EINVAL, "scale must be a positive number");
    if (q_norm_w && !(norm_eps >= 0.f)) return reject(B2A_EINVAL, "norm_eps must not be negative");
    // only the tensor-core decode (16-bit caches, head_dim 64/96/128/256) uses scratch
    if (!decode_tc_supported(D, cache_dtype))
        return reject(B2A_ENOTSUP, "b2a_decode_noalloc needs an fp16/bf16 cache and head_dim 64, 96, 128 or 256 "
                                   "(got head_dim %lld)", D);
    if (((uintptr_t)k_cache | (uintptr_t)v_cache) % 16 != 0)
        return reject(B2A_EINVAL, "caches must be 16-byte aligned");
    const int n_hg = (Hq / Hkv + 7) / 8;
    const long long units = (long long)B * Hkv * n_hg;
    if (B > kDecodeMaxBatchPerLaunch || units > kMaxUnits)
        return reject(B2A_EINVAL, "b2a_decode_noalloc: batch x kv heads x ceil(G/8) = %lld exceeds the static "
                                  "scratch limit of %lld units (batch <= 2048)", units, kMaxUnits);
    static_assert(kDecodeGapKeysMax == 640, "the message below names max_seq + 641");
    if ((long long)B * ((long long)max_seq + 1 + kDecodeGapKeysMax) >= INT32_MAX)
        return reject(B2A_EINVAL, "b2a_decode_noalloc: batch x (max_seq + 641) = %lld must stay below %lld",
                      (long long)B * ((long long)max_seq + 1 + kDecodeGapKeysMax), INT32_MAX);

    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess || device < 0 || device >= kMaxDevices)
        return reject(B2A_ECUDA, "no current CUDA device (%lld)", device);
    int target = 0, cap = 0;
    size_t partial_bytes = 0;
    decode_tc_workspace(device, B, Hkv, n_hg, D, cache_dtype, &target, &cap, &partial_bytes);
    if (partial_bytes > kPartialBytes)
        return reject(B2A_ENOTSUP, "b2a_decode_noalloc: %lld bytes of partial slots exceed the static scratch (%lld)",
                      (long long)partial_bytes, (long long)kPartialBytes);
    unsigned char* scratch = nullptr;
    e = scratch_for(device, &scratch);
    if (e != cudaSuccess) return reject(B2A_ECUDA, "cudaGetSymbolAddress failed (%lld)", (long long)e);

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // counters must start at zero; the status word is cleared with them
    e = cudaMemsetAsync(scratch, 0, kStatusBytes + (size_t)units * sizeof(int), s);
    if (e != cudaSuccess) return reject(B2A_ECUDA, "cudaMemsetAsync on the scratch failed (%lld)", (long long)e);

    DecodeParams p{};
    p.q = q_new;
    p.k_new = k_new;
    p.v_new = v_new;
    p.q_dtype = q_dtype;
    p.k_cache = k_cache;
    p.v_cache = v_cache;
    p.cache_dtype = cache_dtype;
    p.stride_b = (int64_t)Hkv * max_seq * D;
    p.stride_h = kv_layout == B2A_KV_HEAD_MAJOR ? (int64_t)max_seq * D : D;
    p.stride_pos = kv_layout == B2A_KV_HEAD_MAJOR ? D : (int64_t)Hkv * D;
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
    p.status = reinterpret_cast<int*>(scratch);
    p.counters = reinterpret_cast<int*>(scratch + kStatusBytes);
    p.partials = reinterpret_cast<float*>(scratch + kStatusBytes + kCounterBytes);
    p.n_hg = n_hg;
    p.target_items = target;
    p.item_capacity = cap;
    if (rope_mode != B2A_ROPE_NONE)
        for (int i = 0; i < D / 2; ++i) p.inv_freq[i] = 1.0 / pow(rope_theta, (2.0 * i) / D);
    e = launch_decode_tc(p, device, s);
    if (e != cudaSuccess) return reject(B2A_ECUDA, "decode kernel launch failed (%lld)", (long long)e);
    return B2A_OK;
}
