// sm100.cuh -- sm_100a building blocks shared by the tensor-core kernels: mbarrier
// waits bounded by %globaltimer, TMA tile loads, tcgen05 MMA issue / commit, TMEM
// loads and stores, shared-memory matrix and instruction descriptors, and the host's
// access to cuTensorMapEncodeTiled.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace b2a {
namespace {

constexpr uint64_t kWaitNs = 1000000000ull;  // 1 s: the bound of every mbarrier wait

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// try_wait without a suspend-time hint: the thread retries at the hardware's
// own short interval.
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred P1;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, P1;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: false when kWaitNs elapse or another role / another CTA of this launch
// already aborted.  A timeout raises status bit 3 (the sticky report b2a_check_device_status
// reads) and the launch's abort word (status[kStatusAbortWord]), which the other CTAs poll;
// the abort word is reset by the launch's last CTA, so later launches run normally.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status) {
    if (mbar_test(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_test(bar, parity)) return true;
        if ((i & 1023u) == 0) {
            if (*abort_flag) return false;
            if (*(volatile int*)(status + kStatusAbortWord)) {
                *abort_flag = 1;
                return false;
            }
            if (global_ns() - t0 > kWaitNs) {
                *abort_flag = 1;
                atomicOr(status, 8);
                atomicExch(status + kStatusAbortWord, 1);
                return false;
            }
        }
    }
}
// Bounded wait on the exit path (no abort short-cut).
__device__ __forceinline__ void mbar_drain(uint32_t bar, uint32_t parity) {
    const uint64_t t0 = global_ns();
    while (!mbar_test(bar, parity))
        if (global_ns() - t0 > kWaitNs) return;
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1, int c2,
                                            int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];" ::"r"(dst),
        "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// MMA issue and commit, warp-wide: the whole warp computes the (warp-uniform)
// operands and lane 0 alone issues, so the descriptors stay in the uniform
// datapath instead of being moved there for every instruction.
// Descriptors travel as two 32-bit words: only the low word (start address and
// LBO fields) changes between K steps, tiles and stages; the high word (SBO,
// version, layout) is one constant per operand.
template <int kAcc>  // 0: overwrite, 1: accumulate, -1: the runtime flag `acc`
__device__ __forceinline__ void umma_ss_w(uint32_t lane, uint32_t d_tmem, uint32_t a_lo, uint32_t a_hi, uint32_t b_lo,
                                          uint32_t b_hi, uint32_t idesc, uint32_t acc = 0) {
    asm volatile(
        "{\n\t.reg .pred p, l0;\n\t.reg .b64 da, db;\n\t"
        "setp.eq.u32 l0, %7, 0;\n\t"
        "setp.ne.b32 p, %6, 0;\n\t"
        "mov.b64 da, {%1, %2};\n\t"
        "mov.b64 db, {%3, %4};\n\t"
        "@l0 tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %5, p;\n\t}" ::"r"(d_tmem),
        "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(kAcc < 0 ? acc : (uint32_t)kAcc), "r"(lane));
}
template <int kAcc>
__device__ __forceinline__ void umma_ts_w(uint32_t lane, uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo,
                                          uint32_t b_hi, uint32_t idesc, uint32_t acc = 0) {
    asm volatile(
        "{\n\t.reg .pred p, l0;\n\t.reg .b64 db;\n\t"
        "setp.eq.u32 l0, %6, 0;\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "mov.b64 db, {%2, %3};\n\t"
        "@l0 tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], db, %4, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(kAcc < 0 ? acc : (uint32_t)kAcc), "r"(lane));
}
__device__ __forceinline__ void umma_commit_w(uint32_t lane, uint32_t bar) {
    asm volatile(
        "{\n\t.reg .pred l0;\n\t"
        "setp.eq.u32 l0, %1, 0;\n\t"
        "@l0 tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(bar),
        "r"(lane)
        : "memory");
}

#define B2A_R32(r) \
    "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), \
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), \
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), \
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])

// 32 consecutive 32-bit TMEM columns of this thread's lane (asynchronous until tmem_wait_ld).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : B2A_R32(r)
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
    tmem_st16(taddr, r);
    tmem_st16(taddr + 16, r + 16);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor, sm_100 version 1: 128-byte swizzle (layout type 2) unless
// another layout is given (4: 64-byte swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t layout = 2u) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)layout << 61;  // 2: 128-byte swizzle, 4: 64-byte swizzle
    return d;
}

// Instruction descriptor, kind::f16, fp32 accumulate.
__host__ __device__ constexpr uint32_t make_idesc(int fmt, int M, int N, int a_mn_major, int b_mn_major) {
    return (1u << 4) | ((uint32_t)fmt << 7) | ((uint32_t)fmt << 10) | ((uint32_t)a_mn_major << 15) |
           ((uint32_t)b_mn_major << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}


__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(map), "r"(c0), "r"(c1), "r"(bar)
        : "memory");
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// 8 consecutive output elements (16-byte aligned for 16-bit types, 32-byte for fp32) in `dtype`.
__device__ __forceinline__ void store8(void* out, int64_t off, const float* v, int dtype) {
    if (dtype == kF32) {
        float4* o = reinterpret_cast<float4*>(static_cast<float*>(out) + off);
        o[0] = make_float4(v[0], v[1], v[2], v[3]);
        o[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else if (dtype == kF16) {
        uint4 u;
        u.x = pack_half2(v[0], v[1]);
        u.y = pack_half2(v[2], v[3]);
        u.z = pack_half2(v[4], v[5]);
        u.w = pack_half2(v[6], v[7]);
        *reinterpret_cast<uint4*>(static_cast<__half*>(out) + off) = u;
    } else {
        uint4 u;
        uint32_t* w = &u.x;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
            w[i] = *reinterpret_cast<uint32_t*>(&h);
        }
        *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + off) = u;
    }
}

// ---------------------------------------------------------------- host
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeFn encode_fn() {
    static std::once_flag once;
    static EncodeFn fn = nullptr;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeFn>(ptr);
    });
    return fn;
}

}  // namespace
}  // namespace b2a
