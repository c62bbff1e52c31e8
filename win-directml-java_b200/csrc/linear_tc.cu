// linear_tc.cu -- y = x W^T + bias + residual on the tcgen05 tensor cores: the
// projections either side of the attention with their elementwise steps fused
// into the GEMM epilogue (the QKV projection's bias, the O projection's residual
// add; INF/qwen/Qwen2Runtime.java:693-716 / 888-914 and 756-777 / 973-1000).
//
// CTA = one 128-row x BN-column output tile (and, split-K, one range of its K panels), 128 threads:
//   warp 0, lane 0  TMA producer: x and W tiles of 64 K-columns (128-byte swizzle)
//                   into a 4-stage ring;
//   warp 1          MMA issuer (lane 0 issues): per K panel four
//                   tcgen05.mma kind::f16 (M 128, N BN, K 16) into one TMEM
//                   accumulator of BN fp32 columns;
//   all four warps  epilogue: thread t owns output row t (TMEM lane t) and adds
//                   the bias and the residual to its accumulator row.
// Rows past M and K columns past K are zero-filled by the TMA loads; columns past
// N are not stored.  Every mbarrier wait is bounded (status bit 3 on a timeout).
// Split-K (launches with too few output tiles to fill the GPU, e.g. decode projections with
// M = batch <= 128): the K panels are cut into ksplit ranges, one CTA each; each CTA adds its
// partial tile into an fp32 accumulator (vector atomics), and the tile's last CTA (a per-tile
// counter) adds bias and residual, stores y, and leaves the accumulator rows and the counter at
// zero for the next launch.  The accumulation order, and so the last bits of y, may differ
// between runs.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "internal.h"
#include "sm100.cuh"

namespace b2a {
namespace {

constexpr int kLBM = 128;      // output rows per CTA (the MMA's M)
constexpr int kLBK = 64;       // K columns per stage (one 128-byte swizzle panel)
constexpr int kLStages = 4;
constexpr int kLThreads = 128;

template <int BN>
struct LinGeo {
    static constexpr int kATile = kLBM * kLBK * 2;
    static constexpr int kWTile = BN * kLBK * 2;
    static constexpr int kStage = kATile + kWTile;
    static constexpr int oBar = kLStages * kStage;
    static constexpr int kBytes = oBar + 256;  // barriers, TMEM address, abort flag
    static_assert(kBytes + 1024 <= 227 * 1024, "shared memory budget");
};

struct LinParams {
    int M, N, K;
    const float* bias;     // [N] fp32 or NULL
    const void* residual;  // [M][ldr] of out_dtype or NULL
    int64_t ldr;
    void* y;               // [M][ldy] of out_dtype
    int64_t ldy;
    int out_dtype;
    int fmt;               // MMA operand type: 0 fp16, 1 bf16
    int* status;
    int ksplit;            // K ranges per output tile (1: no split)
    int panels_per_split;  // K panels (64 columns) per range
    float* acc;            // split-K: fp32 [M][N] accumulator, zero between launches
    int* counters;         // split-K: [tiles], zero between launches
    int early;             // launched with programmatic serialisation: wait before reading x / residual
};

__device__ __forceinline__ float lin_load(const void* p, int64_t i, int dtype) { return load_as_float(p, i, dtype); }

// Fire-and-forget fp32 adds in L2 (red, no value returned): four consecutive floats (16-byte aligned) or one.
__device__ __forceinline__ void red_add4(float* a, float x, float y, float z, float w) {
    asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(a), "f"(x), "f"(y), "f"(z), "f"(w)
                 : "memory");
}
__device__ __forceinline__ void red_add1(float* a, float x) {
    asm volatile("red.relaxed.gpu.global.add.f32 [%0], %1;" ::"l"(a), "f"(x) : "memory");
}

template <int BN>
__global__ void __launch_bounds__(kLThreads, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                     const __grid_constant__ LinParams p) {
    using Gm = LinGeo<BN>;
    // a decode launched after this GEMM with early start (b2a_set_decode_early_start) may be
    // scheduled from now on: it waits for this grid's completion before reading its output
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    extern __shared__ unsigned char smem_raw[];
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    unsigned char* base_ptr = smem_raw + (base - smem_u32(smem_raw));
    const uint32_t bar0 = base + Gm::oBar;
    auto bFull = [&](int s) { return bar0 + 8u * s; };
    auto bEmpty = [&](int s) { return bar0 + 8u * (kLStages + s); };
    const uint32_t bDone = bar0 + 8u * (2 * kLStages);
    const uint32_t bDrain = bar0 + 8u * (2 * kLStages + 1);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(base_ptr + Gm::oBar + 128);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(base_ptr + Gm::oBar + 136);
    volatile int* last_flag = reinterpret_cast<volatile int*>(base_ptr + Gm::oBar + 140);  // split-K
    auto sX = [&](int s) { return base + (uint32_t)(s * Gm::kStage); };
    auto sW = [&](int s) { return base + (uint32_t)(s * Gm::kStage + Gm::kATile); };

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int* const status = p.status;
    const int nk_all = (p.K + kLBK - 1) / kLBK;
    const int kt0 = (int)blockIdx.z * p.panels_per_split;
    const int nk = min(nk_all, kt0 + p.panels_per_split) - kt0;  // this CTA's K panels: kt0 .. kt0 + nk - 1
    const int m0 = blockIdx.x * kLBM, n0 = blockIdx.y * BN;

    if (tid == 0) {
        for (int s = 0; s < kLStages; ++s) {
            mbar_init(bFull(s), 1);
            mbar_init(bEmpty(s), 1);
        }
        mbar_init(bDone, 1);
        mbar_init(bDrain, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        __syncwarp();
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                     "r"((uint32_t)BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 0) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            int issued = 0;
            // early start: the weight panels of the first stages are requested while the kernel
            // ahead (which produces x) finishes; each stage's barrier expects x and w bytes alike
            const int pre = p.early ? min(nk, kLStages) : 0;
            for (int kt = 0; kt < pre; ++kt) {
                mbar_expect_tx(bFull(kt), Gm::kStage);
                tma_load_2d(sW(kt), &tmW, bFull(kt), (kt0 + kt) * kLBK, n0);
            }
            if (p.early) asm volatile("griddepcontrol.wait;" ::: "memory");
            for (int kt = 0; kt < nk; ++kt) {
                const int st = kt % kLStages;
                if (kt >= kLStages && !mbar_wait(bEmpty(st), ((kt / kLStages) - 1) & 1, abort_flag, status)) break;
                if (kt >= pre) {
                    mbar_expect_tx(bFull(st), Gm::kStage);
                    tma_load_2d(sW(st), &tmW, bFull(st), (kt0 + kt) * kLBK, n0);
                }
                tma_load_2d(sX(st), &tmX, bFull(st), (kt0 + kt) * kLBK, m0);
                issued = kt + 1;
            }
            // every copy issued lands before the CTA may exit
            for (int kt = issued > kLStages ? issued - kLStages : 0; kt < issued; ++kt)
                mbar_drain(bFull(kt % kLStages), (kt / kLStages) & 1);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        const uint32_t ln = (uint32_t)lane;
        const uint32_t idesc = make_idesc(p.fmt, kLBM, BN, 0, 0);
        const uint64_t dX = smem_desc(sX(0), 16, 1024), dW = smem_desc(sW(0), 16, 1024);
        const uint32_t x_lo = (uint32_t)dX, w_lo = (uint32_t)dW, hi = (uint32_t)(dX >> 32);
        for (int kt = 0; kt < nk; ++kt) {
            const int st = kt % kLStages;
            if (!__all_sync(0xffffffffu, mbar_wait(bFull(st), (kt / kLStages) & 1, abort_flag, status))) break;
            tc_fence_after();
            const uint32_t so = (uint32_t)(st * Gm::kStage) >> 4;
#pragma unroll
            for (int ks = 0; ks < kLBK / 16; ++ks) {
                const uint32_t ko = (uint32_t)(ks * 32) >> 4;  // 16 K columns = 32 bytes inside the swizzled row
                umma_ss_w<-1>(ln, tmem, x_lo + so + ko, hi, w_lo + so + ko, hi, idesc, (kt | ks) ? 1u : 0u);
            }
            umma_commit_w(ln, bEmpty(st));
        }
        umma_commit_w(ln, bDone);
        umma_commit_w(ln, bDrain);
    }

    // ---------------------------------------------------------------- epilogue
    // Thread t reads TMEM lane t (output row t), 32 columns at a time.  Split-K launches stage each
    // chunk in shared memory and walk it row-major, four columns per thread, so that the reductions
    // and the final pass are coalesced (eight threads cover a 128-byte row segment).
    __syncwarp();
    const bool ok = __all_sync(0xffffffffu, mbar_wait(bDone, 0, abort_flag, status));
    tc_fence_after();
    if (p.early) asm volatile("griddepcontrol.wait;" ::: "memory");  // before reading residual / bias, writing
    constexpr int kPitch = 36;  // staged row pitch (floats): 16-byte aligned, conflict-free float4 writes
    float* const stage = reinterpret_cast<float*>(base_ptr);  // the ring is idle once every MMA is done
    const int rows = min(kLBM, p.M - m0);
    const bool vec_y = (p.ldy % 4 == 0) && (p.residual == nullptr || p.ldr % 4 == 0);
    // bias, residual and the store of 4 consecutive columns n .. n+3 (cnt of them valid) of row m
    auto finish4 = [&](int m, int n, float4 v, int cnt) {
        float x[4] = {v.x, v.y, v.z, v.w};
        if (p.bias != nullptr) {
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (e < cnt) x[e] += __ldg(p.bias + n + e);
        }
        if (p.residual != nullptr) {
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (e < cnt) x[e] += lin_load(p.residual, (int64_t)m * p.ldr + n + e, p.out_dtype);
        }
        const int64_t off = (int64_t)m * p.ldy + n;
        if (cnt == 4 && vec_y) {
            if (p.out_dtype == kF32) {
                *reinterpret_cast<float4*>(static_cast<float*>(p.y) + off) = make_float4(x[0], x[1], x[2], x[3]);
            } else {
                uint2 u;
                if (p.out_dtype == kF16) {
                    u.x = pack_half2(x[0], x[1]);
                    u.y = pack_half2(x[2], x[3]);
                } else {
                    __nv_bfloat162 a = __floats2bfloat162_rn(x[0], x[1]), b = __floats2bfloat162_rn(x[2], x[3]);
                    u.x = *reinterpret_cast<uint32_t*>(&a);
                    u.y = *reinterpret_cast<uint32_t*>(&b);
                }
                *reinterpret_cast<uint2*>(static_cast<unsigned short*>(p.y) + off) = u;
            }
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (e < cnt) store_from_float(p.y, off + e, x[e], p.out_dtype);
        }
    };
    if (ok && p.ksplit == 1) {
        // one output tile per CTA: each thread stores its own row (16-byte stores); a CTA-wide staging
        // pass would add two barriers per 32 columns to every tile of a large GEMM
        const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
        const int m = m0 + warp * 32 + lane;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(lane_base + 32 * c, r);
            tmem_wait_ld();
            const int nc = n0 + 32 * c;
            if (m >= p.M || nc >= p.N) continue;
            const int cnt = min(32, p.N - nc);
            float v[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(r[e]);
            if (p.bias != nullptr) {
#pragma unroll
                for (int e = 0; e < 32; ++e)
                    if (e < cnt) v[e] += __ldg(p.bias + nc + e);
            }
            if (p.residual != nullptr) {
#pragma unroll
                for (int e = 0; e < 32; ++e)
                    if (e < cnt) v[e] += lin_load(p.residual, (int64_t)m * p.ldr + nc + e, p.out_dtype);
            }
            const int64_t off = (int64_t)m * p.ldy + nc;
            if (cnt == 32 && off % 8 == 0) {
#pragma unroll
                for (int e = 0; e < 32; e += 8) store8(p.y, off + e, v + e, p.out_dtype);
            } else {
#pragma unroll
                for (int e = 0; e < 32; ++e)
                    if (e < cnt) store_from_float(p.y, off + e, v[e], p.out_dtype);
            }
        }
    } else if (ok) {
        // split-K: the partial tile goes through the staging tile so that its vector reductions into
        // the accumulator are coalesced
        const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
        const int row = warp * 32 + lane;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
            const int nc = n0 + 32 * c;
            if (nc >= p.N) break;  // uniform across the CTA
            uint32_t r[32];
            tmem_ld32(lane_base + 32 * c, r);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; e += 4)
                *reinterpret_cast<float4*>(stage + row * kPitch + e) =
                    make_float4(__uint_as_float(r[e]), __uint_as_float(r[e + 1]), __uint_as_float(r[e + 2]),
                                __uint_as_float(r[e + 3]));
            __syncthreads();
            const int cols = min(32, p.N - nc);
            for (int idx = tid; idx < rows * 8; idx += kLThreads) {
                const int rr = idx >> 3, c4 = (idx & 7) * 4;
                if (c4 >= cols) continue;
                const float4 v = *reinterpret_cast<const float4*>(stage + rr * kPitch + c4);
                const int m = m0 + rr, n = nc + c4, cnt = min(4, cols - c4);
                float* a = p.acc + (int64_t)m * p.N + n;
                if (cnt == 4 && ((uintptr_t)a & 15) == 0) {
                    red_add4(a, v.x, v.y, v.z, v.w);
                } else {
                    const float x[4] = {v.x, v.y, v.z, v.w};
                    for (int e = 0; e < cnt; ++e) red_add1(a + e, x[e]);
                }
            }
            __syncthreads();  // the staging tile is rewritten by the next chunk
        }
    }
    if (p.ksplit > 1) {
        // the tile's last range to finish completes it: bias, residual, store, and the accumulator
        // rows and the counter back to zero
        __threadfence();
        __syncthreads();
        int* const counter = p.counters + blockIdx.y * gridDim.x + blockIdx.x;
        if (tid == 0) *last_flag = atomicAdd(counter, 1) == p.ksplit - 1;
        __syncthreads();
        if (*last_flag) {
            __threadfence();
            const int cols = min(BN, p.N - n0);
            const int c4n = (cols + 3) / 4;
            for (int idx = tid; idx < rows * c4n; idx += kLThreads) {
                const int rr = idx / c4n, c4 = (idx - rr * c4n) * 4;
                const int m = m0 + rr, n = n0 + c4, cnt = min(4, cols - c4);
                float* a = p.acc + (int64_t)m * p.N + n;
                float4 v;
                if (cnt == 4 && ((uintptr_t)a & 15) == 0) {
                    v = __ldcg(reinterpret_cast<const float4*>(a));
                    *reinterpret_cast<float4*>(a) = make_float4(0.f, 0.f, 0.f, 0.f);
                } else {
                    float x[4] = {0.f, 0.f, 0.f, 0.f};
                    for (int e = 0; e < cnt; ++e) {
                        x[e] = __ldcg(a + e);
                        a[e] = 0.f;
                    }
                    v = make_float4(x[0], x[1], x[2], x[3]);
                }
                finish4(m, n, v, cnt);
            }
            if (tid == 0) *counter = 0;
        }
    }
    // all MMAs this CTA issued are complete before TMEM is released
    if (warp == 1) mbar_drain(bDrain, 0);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)BN));
}

// [rows][cols] 16-bit matrix with row stride ld (elements), box kLBK x box_rows, 128-byte swizzle.
bool make_map_2d(CUtensorMap* m, const void* ptr, int fmt, int rows, int cols, int64_t ld, int box_rows) {
    EncodeFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kLBK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, fmt ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr),
              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

constexpr int kLinBN = 128;
constexpr int kMaxDevicesL = 64;

cudaError_t linear_ready() {
    static std::once_flag once[kMaxDevicesL];
    static cudaError_t err[kMaxDevicesL];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevicesL) return cudaErrorInvalidDevice;
    std::call_once(once[dev], [dev] {
        err[dev] = cudaFuncSetAttribute(linear_tc_kernel<kLinBN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        LinGeo<kLinBN>::kBytes + 1024);
    });
    return err[dev];
}

}  // namespace

bool linear_tc_supported(int in_dtype, int K, int64_t ldx, int64_t ldw, const void* x, const void* w) {
    if (in_dtype != kF16 && in_dtype != kBF16) return false;
    if (K <= 0 || ldx % 8 != 0 || ldw % 8 != 0 || ldx < K || ldw < K) return false;
    if ((uintptr_t)x % 16 != 0 || (uintptr_t)w % 16 != 0) return false;
    return encode_fn() != nullptr;
}

int linear_split_plan(int M, int N, int K, int sm_count, size_t* acc_bytes, size_t* counter_ints) {
    const int tiles = ((M + kLBM - 1) / kLBM) * ((N + kLinBN - 1) / kLinBN);
    const int nk = (K + kLBK - 1) / kLBK;
    int ks = 1;
    if (2 * tiles <= sm_count) ks = std::min(nk, std::max(1, sm_count / tiles));
    const int pps = (nk + ks - 1) / ks;
    ks = (nk + pps - 1) / pps;  // no empty ranges
    *acc_bytes = ks > 1 ? (size_t)M * N * sizeof(float) : 0;
    *counter_ints = ks > 1 ? (size_t)tiles : 0;
    return ks;
}

cudaError_t launch_linear_tc(const LinearArgs& a, int* status, cudaStream_t stream) {
    const cudaError_t ready = linear_ready();
    if (ready != cudaSuccess) return ready;
    const int fmt = a.in_dtype == kBF16 ? 1 : 0;
    CUtensorMap mx, mw;
    if (!make_map_2d(&mx, a.x, fmt, a.M, a.K, a.ldx, kLBM) || !make_map_2d(&mw, a.w, fmt, a.N, a.K, a.ldw, kLinBN))
        return cudaErrorInvalidValue;
    LinParams p{};
    p.M = a.M;
    p.N = a.N;
    p.K = a.K;
    p.bias = a.bias;
    p.residual = a.residual;
    p.ldr = a.ldr;
    p.y = a.y;
    p.ldy = a.ldy;
    p.out_dtype = a.out_dtype;
    p.fmt = fmt;
    p.status = status;
    const int nk = (a.K + kLBK - 1) / kLBK;
    p.ksplit = a.ksplit > 1 ? a.ksplit : 1;
    p.panels_per_split = (nk + p.ksplit - 1) / p.ksplit;
    p.acc = a.acc;
    p.counters = a.counters;
    p.early = a.early;
    const dim3 grid((unsigned)((a.M + kLBM - 1) / kLBM), (unsigned)((a.N + kLinBN - 1) / kLinBN), (unsigned)p.ksplit);
    if (!a.early) {
        linear_tc_kernel<kLinBN><<<grid, kLThreads, LinGeo<kLinBN>::kBytes + 1024, stream>>>(mx, mw, p);
        return cudaGetLastError();
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kLThreads);
    cfg.dynamicSmemBytes = LinGeo<kLinBN>::kBytes + 1024;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, linear_tc_kernel<kLinBN>, mx, mw, p);
}

}  // namespace b2a
