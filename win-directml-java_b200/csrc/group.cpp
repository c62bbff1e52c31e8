// group.cpp -- b2a_group: one process driving several GPUs of a node, one context
// per device plus an NCCL communicator clique (ncclCommInitAll), and the sharded
// entry points that run every device's shard and reassemble the outputs with one
// grouped ncclAllGather over NVLink.
//
// The reference runs on one GPU and has no counterpart; the attention units
// (sequence, kv head) are independent, so a batch is split into equal shards, one
// per device, with no exchange while they are computed -- the all-gather only
// collects the finished outputs.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, or the file the
// B2A_NCCL_LIBRARY environment variable names), so single-GPU users of the
// library need no NCCL; every NCCL failure, a missing library included, is
// reported as B2A_ENCCL.  nccl.h is used for its types only.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/b200attn.h"
#include "internal.h"

namespace {

struct NcclApi {
    void* handle = nullptr;
    ncclResult_t (*CommInitAll)(ncclComm_t*, int, const int*) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    ncclResult_t (*GetVersion)(int*) = nullptr;
};

// Resolves the NCCL entry points; empty string on success, else the reason.
std::string load_nccl(NcclApi* api) {
    const char* env = getenv("B2A_NCCL_LIBRARY");
    const char* path = (env && *env) ? env : "libnccl.so.2";
    void* h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
    if (!h) {
        const char* e = dlerror();
        return std::string("NCCL could not be loaded (") + path + "): " + (e ? e : "unknown error");
    }
    auto sym = [&](const char* name) { return dlsym(h, name); };
    api->handle = h;
    api->CommInitAll = reinterpret_cast<decltype(api->CommInitAll)>(sym("ncclCommInitAll"));
    api->CommDestroy = reinterpret_cast<decltype(api->CommDestroy)>(sym("ncclCommDestroy"));
    api->AllGather = reinterpret_cast<decltype(api->AllGather)>(sym("ncclAllGather"));
    api->GroupStart = reinterpret_cast<decltype(api->GroupStart)>(sym("ncclGroupStart"));
    api->GroupEnd = reinterpret_cast<decltype(api->GroupEnd)>(sym("ncclGroupEnd"));
    api->GetErrorString = reinterpret_cast<decltype(api->GetErrorString)>(sym("ncclGetErrorString"));
    api->GetVersion = reinterpret_cast<decltype(api->GetVersion)>(sym("ncclGetVersion"));
    if (!api->CommInitAll || !api->CommDestroy || !api->AllGather || !api->GroupStart || !api->GroupEnd ||
        !api->GetErrorString) {
        dlclose(h);
        api->handle = nullptr;
        return std::string(path) + " lacks an NCCL entry point (ncclCommInitAll, ncclAllGather, ...)";
    }
    return std::string();
}

thread_local std::string g_group_create_error;

}  // namespace

struct b2a_group {
    NcclApi nccl;
    std::vector<int> devices;
    std::vector<b2a_context*> ctx;
    std::vector<ncclComm_t> comms;
    std::string last_error;
};

namespace {

int gfail(b2a_group* g, int status, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    (g ? g->last_error : g_group_create_error) = buf;
    return status;
}

// A failing rank's status, with its context's message.
int rank_fail(b2a_group* g, int r, int status, const char* what) {
    char msg[768];
    b2a_last_error(g->ctx[r], msg, sizeof(msg));
    return gfail(g, status, "%s on rank %d (device %d): %s: %s", what, r, g->devices[r], b2a_status_string(status),
                 msg);
}

size_t dtype_bytes(int d) { return d == B2A_FLOAT32 ? 4 : 2; }

// One grouped all-gather of every rank's `bytes` from send[r] into recv[r] (rank-major).
int gather(b2a_group* g, void* const* send, void* const* recv, size_t bytes, void* const* streams) {
    const int n = (int)g->devices.size();
    ncclResult_t rc = g->nccl.GroupStart();
    for (int r = 0; r < n && rc == ncclSuccess; ++r) {
        if (cudaSetDevice(g->devices[r]) != cudaSuccess) return gfail(g, B2A_ECUDA, "cudaSetDevice(%d)", g->devices[r]);
        rc = g->nccl.AllGather(send[r], recv[r], bytes, ncclInt8, g->comms[r],
                               static_cast<cudaStream_t>(streams ? streams[r] : nullptr));
    }
    const ncclResult_t end = g->nccl.GroupEnd();
    if (rc == ncclSuccess) rc = end;
    if (rc != ncclSuccess) return gfail(g, B2A_ENCCL, "ncclAllGather: %s", g->nccl.GetErrorString(rc));
    return B2A_OK;
}

struct DevRestore {
    int prev = -1;
    DevRestore() {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    }
    ~DevRestore() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

}  // namespace

extern "C" {

B2A_API int b2a_group_create(int ndev, const int* devices, b2a_group** out) {
    if (!out) return gfail(nullptr, B2A_EINVAL, "out must not be null");
    *out = nullptr;
    if (!devices) return gfail(nullptr, B2A_EINVAL, "devices must not be null");
    b2a_group* g = new (std::nothrow) b2a_group();
    if (!g) return gfail(nullptr, B2A_EOOM, "host allocation failed");
    const std::string why = load_nccl(&g->nccl);
    if (!why.empty()) {
        delete g;
        return gfail(nullptr, B2A_ENCCL, "%s", why.c_str());
    }
    auto give_up = [&](int status) {
        b2a_group_destroy(g);
        return status;
    };
    DevRestore restore;
    // the communicator clique first: NCCL validates the rank count and the device list
    g->comms.assign(ndev > 0 ? ndev : 0, nullptr);
    const ncclResult_t rc = g->nccl.CommInitAll(ndev > 0 ? g->comms.data() : nullptr, ndev, devices);
    if (rc != ncclSuccess) {
        g->comms.clear();
        gfail(nullptr, B2A_ENCCL, "ncclCommInitAll(%d ranks): %s", ndev, g->nccl.GetErrorString(rc));
        return give_up(B2A_ENCCL);
    }
    for (int r = 0; r < ndev; ++r) {
        b2a_context* c = nullptr;
        const int st = b2a_create(devices[r], &c);
        if (st != B2A_OK) {
            char msg[512];
            b2a_last_error(nullptr, msg, sizeof(msg));
            gfail(nullptr, st, "rank %d (device %d): %s", r, devices[r], msg);
            return give_up(st);
        }
        g->devices.push_back(devices[r]);
        g->ctx.push_back(c);
    }
    *out = g;
    return B2A_OK;
}

B2A_API int b2a_group_destroy(b2a_group* g) {
    if (!g) return B2A_OK;
    {
        DevRestore restore;
        for (ncclComm_t c : g->comms)
            if (c) g->nccl.CommDestroy(c);
        for (b2a_context* c : g->ctx) b2a_destroy(c);
    }
    if (g->nccl.handle) dlclose(g->nccl.handle);
    delete g;
    return B2A_OK;
}

B2A_API int b2a_group_last_error(const b2a_group* g, char* buf, size_t n) {
    const std::string& s = g ? g->last_error : g_group_create_error;
    if (buf && n > 0) {
        const size_t k = std::min(n - 1, s.size());
        memcpy(buf, s.data(), k);
        buf[k] = '\0';
    }
    return (int)s.size();
}

B2A_API int b2a_group_size(const b2a_group* g) { return g ? (int)g->devices.size() : 0; }

B2A_API int b2a_group_context(b2a_group* g, int rank, b2a_context** ctx) {
    if (!g || !ctx) return B2A_EINVAL;
    if (rank < 0 || rank >= (int)g->ctx.size()) return gfail(g, B2A_EINVAL, "rank %d outside [0, %zu)", rank,
                                                             g->ctx.size());
    *ctx = g->ctx[rank];
    return B2A_OK;
}

B2A_API int b2a_group_check_device_status(b2a_group* g, void* const* streams) {
    if (!g) return B2A_EINVAL;
    for (int r = 0; r < (int)g->ctx.size(); ++r) {
        const int st = b2a_check_device_status(g->ctx[r], streams ? streams[r] : nullptr);
        if (st != B2A_OK) return rank_fail(g, r, st, "device status");
    }
    return B2A_OK;
}

B2A_API int b2a_sharded_decode(b2a_group* g, int q_dtype, int cache_dtype, int out_dtype,
                               const void* const* q_new, const void* const* k_new, const void* const* v_new,
                               void* const* k_cache, void* const* v_cache, int kv_layout,
                               const int32_t* const* ctx_lens, int B_shard, int Hq, int Hkv, int D, int max_seq,
                               float scale, int rope_mode, double rope_theta, int window,
                               const float* const* q_norm_w, const float* const* k_norm_w, float norm_eps,
                               void* const* o_shard, void* const* o_gathered, void* const* streams) {
    if (!g) return B2A_EINVAL;
    if (!q_new || !k_new || !v_new || !k_cache || !v_cache || !ctx_lens || !o_shard || !o_gathered)
        return gfail(g, B2A_EINVAL, "per-rank pointer arrays must not be null");
    if ((q_norm_w == nullptr) != (k_norm_w == nullptr))
        return gfail(g, B2A_EINVAL, "q_norm_w and k_norm_w must be given together");
    DevRestore restore;
    const int n = (int)g->ctx.size();
    for (int r = 0; r < n; ++r) {
        const int st = b2a_decode(g->ctx[r], q_dtype, cache_dtype, out_dtype, q_new[r], k_new[r], v_new[r],
                                  k_cache[r], v_cache[r], kv_layout, ctx_lens[r], B_shard, Hq, Hkv, D, max_seq, scale,
                                  rope_mode, rope_theta, window, q_norm_w ? q_norm_w[r] : nullptr,
                                  k_norm_w ? k_norm_w[r] : nullptr, norm_eps, o_shard[r],
                                  streams ? streams[r] : nullptr);
        if (st != B2A_OK) return rank_fail(g, r, st, "b2a_decode");
    }
    return gather(g, o_shard, o_gathered, (size_t)B_shard * Hq * D * dtype_bytes(out_dtype), streams);
}

B2A_API int b2a_sharded_mha(b2a_group* g, int in_dtype, int out_dtype, const void* const* q, const void* const* k,
                            const void* const* v, const float* const* mask, const int32_t* const* key_lengths,
                            void* const* y_shard, void* const* y_gathered, int B_shard, int H, int S, int D,
                            float scale, int layout, void* const* streams) {
    if (!g) return B2A_EINVAL;
    if (!q || !k || !v || !y_shard || !y_gathered) return gfail(g, B2A_EINVAL, "per-rank pointer arrays must not be null");
    DevRestore restore;
    const int n = (int)g->ctx.size();
    for (int r = 0; r < n; ++r) {
        const int st = b2a_mha(g->ctx[r], in_dtype, out_dtype, q[r], k[r], v[r], mask ? mask[r] : nullptr,
                               key_lengths ? key_lengths[r] : nullptr, y_shard[r], B_shard, H, S, D, scale, layout,
                               streams ? streams[r] : nullptr);
        if (st != B2A_OK) return rank_fail(g, r, st, "b2a_mha");
    }
    return gather(g, y_shard, y_gathered, (size_t)B_shard * H * S * D * dtype_bytes(out_dtype), streams);
}

}  // extern "C"
