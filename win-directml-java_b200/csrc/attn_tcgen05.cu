// attn_tcgen05.cu -- whole-sequence attention (causal prefill, bidirectional
// encoder) on the 5th-generation tensor cores: tcgen05.mma with TMEM
// accumulators, TMA-staged Q/K/V tiles, mbarrier pipeline.
//
// CTA = two tiles of 128 query rows (A and B) of one (batch, head), 384 threads
// in three warpgroups:
//   warps 0-3  softmax of tile A, warps 4-7 softmax of tile B: thread t of a
//              group owns query row t = TMEM lane t (tcgen05.ld/st 32x32b);
//   warp 8     TMA producer: Q_A, Q_B once, then ring items of two 128-key
//              tiles, K(i) and V(i-1), into a 2-3 stage ring (plain tiled
//              loads, 128-byte swizzle, 64-element panels of the head dim);
//   warp 9     MMA issuer (the whole warp runs the loop, lane 0 issues).  Per
//              key tile j: O_A += P_A(j) V_j, S_A = Q_A K_{j+1}^T, then the same
//              for B, so the tensor core works on one tile while the softmax
//              group of the other runs (ping-pong).  Its per-step overhead
//              (barrier waits, commits) sits between MMA runs with the tensor
//              core idle -- issue blocks while earlier MMAs execute -- so it
//              waits once per step for the ring item and commits O only after
//              a tile's last PV;
//   warps 10-11 idle.
// setmaxnreg moves registers from the control warpgroup (8-11) to the softmax
// warpgroups, which keep a whole score row (128 fp32) in registers.
// TMEM (512 columns): S_A 0..127, S_B 128..255 (fp32 scores; the softmax
// writes P as fp16 pairs over the first 64 columns, and the PV MMA reads it
// from TMEM), O_A at 256, O_B at 384.
// Softmax per tile: one TMEM read of the score row, row max (3-input max),
// exp2 + row sum + P (f32x2 FMA/add); masks only on tiles that touch the
// causal diagonal, the window start or the key end (a per-row visible key
// range); the scale is folded into one FMA per score; a quarter of the exp2
// run on the FMA pipe as a polynomial (exp2_poly_pair) next to the 16/clk/SM
// MUFU.  The running maximum moves lazily: O is rescaled only when a row's
// maximum grows by more than 8 (log2 units), so P <= 2^8.
//
// Every mbarrier wait is bounded by %globaltimer (kWaitNs).  On a timeout the
// kernel sets status bit 3; other roles stop at their next wait; the producer
// waits (bounded) for its own TMA copies, the MMA thread drains its MMAs,
// TMEM is freed and the CTA returns.
//
// Same semantics as attn_simt.cu / attn_mma.cu (the reference citations are
// there); operands are fp16 (bf16 callers are converted by the host layer).
// The additive [B][S] key mask has its own instantiation (kAdditive).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace b2a {
namespace {

constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kThreadsTc = 384;
// Register split between the warpgroups (setmaxnreg): the kernel launches with
// kRegsLaunch per thread (ptxas' limit for 384 threads and one CTA per SM, which
// the host checks before launching); the control warpgroup returns registers so
// the two softmax warpgroups can keep a whole 128-column score row resident.
// 2 * kRegsSoftmax + kRegsControl == 3 * kRegsLaunch: the pool is used exactly.
constexpr int kRegsLaunch = 168;
constexpr int kRegsSoftmax = 224;
constexpr int kRegsControl = 56;
static_assert(2 * kRegsSoftmax + kRegsControl == 3 * kRegsLaunch, "register split must equal the launch pool");
constexpr uint64_t kWaitNs = 1000000000ull;  // 1 s
constexpr float kRescaleThreshold = 8.0f;
#ifndef B2A_POLY_PAIRS
#define B2A_POLY_PAIRS 2
#endif
constexpr int kPolyPairs = B2A_POLY_PAIRS;  // of every 8 exp2 pairs, on the FMA pipe
constexpr uint32_t kTmemCols = 512;

struct TcParams {
    int B, S, Hq, Hkv, G, D;
    int causal, window;
    const float* mask;
    const int32_t* key_len;
    float scale;
    float scale_log2;
    void* out;
    int out_dtype;
    int64_t o_sb, o_ss, o_sh;
    int* status;
    int fmt;  // 0 = fp16, 1 = bf16 operands
};

template <int D>
struct TcGeo {
    static constexpr int NP = (D + 63) / 64;      // 128-byte panels per row
    static constexpr int kPanelBytes = 128 * 128;  // 128 rows x 128 B
    static constexpr int kTileBytes = NP * kPanelBytes;
    static constexpr int kStages = D <= 64 ? 3 : 2;
    static constexpr int oQ = 0;                   // Q_A, Q_B
    static constexpr int oK = 2 * kTileBytes;
    static constexpr int oV = oK + kStages * kTileBytes;
    static constexpr int oBar = oV + kStages * kTileBytes;
    static constexpr int kBytes = oBar + 512;
    static constexpr uint32_t kTxTile = kTileBytes;  // bytes one K or V tile load delivers (zero fill included)
    static_assert(kBytes + 1024 <= 227 * 1024, "shared memory budget");
};

// ---------------------------------------------------------------- PTX helpers
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
// Bounded wait: false when kWaitNs elapse (status bit 3) or another role /
// another CTA already aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status) {
    if (mbar_test(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_test(bar, parity)) return true;
        if ((i & 1023u) == 0) {
            if (*abort_flag) return false;
            if (*(volatile int*)status & 8) {
                *abort_flag = 1;
                return false;
            }
            if (global_ns() - t0 > kWaitNs) {
                *abort_flag = 1;
                atomicOr(status, 8);
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

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), sm_100 version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor, kind::f16, fp32 accumulate.
__host__ __device__ constexpr uint32_t make_idesc(int fmt, int M, int N, int a_mn_major, int b_mn_major) {
    return (1u << 4) | ((uint32_t)fmt << 7) | ((uint32_t)fmt << 10) | ((uint32_t)a_mn_major << 15) |
           ((uint32_t)b_mn_major << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// 2^x on the FMA pipe instead of the MUFU: x = n + f with n = round(x) taken by adding 1.5 * 2^23 (the FP adder
// rounds to an integer; n is then in the low mantissa bits), f in
// [-0.5, 0.5]; 2^f by a degree-4 polynomial fitted here to 2^f on
// [-0.5, 0.5] (least squares on Chebyshev nodes with relative-error
// reweighting; max relative error 8.5e-6, far below the fp16 rounding of P);
// 2^n added to the exponent field.  x is clamped at -126 so the exponent
// stays non-negative: masked scores (-inf) give 2^-126, which is 0 in fp16.

// Pairs of fp32 in one 64-bit register: the f32x2 instructions of sm_100 do two
// lanes per issue slot on the FMA pipe.
typedef unsigned long long f32x2;
__device__ __forceinline__ f32x2 f2_make(float lo, float hi) {
    f32x2 d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
    return d;
}
__device__ __forceinline__ void f2_split(f32x2 v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f32x2 f2_fma(f32x2 a, f32x2 b, f32x2 c) {
    f32x2 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ f32x2 f2_add(f32x2 a, f32x2 b) {
    f32x2 d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
// Two of them per call, two lanes per f32x2 instruction.
__device__ __forceinline__ void exp2_poly_pair(float x0, float x1, float& e0, float& e1) {
    const f32x2 x = f2_make(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
    const f32x2 t = f2_add(x, f2_make(12582912.f, 12582912.f));
    const f32x2 f = f2_fma(f2_add(t, f2_make(-12582912.f, -12582912.f)), f2_make(-1.f, -1.f), x);  // x - round(x)
    f32x2 p = f2_fma(f2_make(0.009254964f, 0.009254964f), f, f2_make(0.05585603f, 0.05585603f));
    p = f2_fma(p, f, f2_make(0.24031252f, 0.24031252f));
    p = f2_fma(p, f, f2_make(0.6931306f, 0.6931306f));
    p = f2_fma(p, f, f2_make(0.9999978f, 0.9999978f));
    float p0, p1, t0, t1;
    f2_split(p, p0, p1);
    f2_split(t, t0, t1);
    // the low mantissa bits of t hold round(x); shifted by 23 they land in the exponent
    e0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
    e1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
}

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

// ---------------------------------------------------------------- kernel
// kAdditive: the additive [B][S] key mask is applied (its own instantiation, so the
// mask loads do not weigh on the register budget of the unmasked kernels).
template <int D, bool kAdditive>
__global__ void __launch_bounds__(kThreadsTc, 1)
    attn_tcgen05_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ TcParams p) {
    using Gm = TcGeo<D>;
    constexpr int NP = Gm::NP;
    constexpr int ST = Gm::kStages;
    extern __shared__ unsigned char smem_raw[];
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    unsigned char* base_ptr = smem_raw + (base - smem_u32(smem_raw));
    const uint32_t sQ = base + Gm::oQ, sK = base + Gm::oK, sV = base + Gm::oV;
    const uint32_t bar0 = base + Gm::oBar;
    // barriers, 8 bytes each
    const uint32_t bQ = bar0;
    // Ring item i holds K(i) (i < n_max) and V(i-1) (i >= 1): step j reads V(j) and then
    // K(j+1), both last in the same step, so one stage, one full and one empty barrier
    // serve the pair (one wait and one release per step on the MMA thread).  K(i) sits
    // in stage i % ST of the K ring, V(i-1) in stage i % ST of the V ring.
    auto bKVfull = [&](int s) { return bar0 + 8u * (1 + s); };
    auto bKVempty = [&](int s) { return bar0 + 8u * (1 + ST + s); };
    auto bSfull = [&](int t) { return bar0 + 8u * (1 + 2 * ST + t); };
    auto bPfull = [&](int t) { return bar0 + 8u * (3 + 2 * ST + t); };
    auto bOdone = [&](int t) { return bar0 + 8u * (5 + 2 * ST + t); };
    const uint32_t bDrain = bar0 + 8u * (7 + 2 * ST);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(base_ptr + Gm::oBar + 256);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(base_ptr + Gm::oBar + 264);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // parameter fields copied to registers once: the asm statements below clobber
    // memory, which would otherwise force a reload through a generic pointer at
    // every use (a 25x slower masked softmax tile when the mask test read them)
    const int S = p.S, causal = p.causal, window = p.window;
    const float* const mask = kAdditive ? p.mask : nullptr;
    const float scale = p.scale;
    int* const status = p.status;
    const int n_pairs = (S + 2 * kBM - 1) / (2 * kBM);
    const int pair = causal ? n_pairs - 1 - (int)blockIdx.x : (int)blockIdx.x;
    const int h = blockIdx.y, b = blockIdx.z;
    const int kvh = h / p.G;
    const int qbase = pair * 2 * kBM;

    // per query tile: first row, key range, number of key tiles
    int q0t[2], kb[2], ke[2], nt[2];
    bool uniform = false;
    for (int t = 0; t < 2; ++t) {
        q0t[t] = qbase + t * kBM;
        kb[t] = 0;
        ke[t] = S;
        if (causal) {
            ke[t] = min(S, q0t[t] + kBM);
            if (window > 0) kb[t] = max(0, q0t[t] - window + 1);
        } else if (p.key_len != nullptr) {
            const int kl = p.key_len[b];
            if (kl <= 0) uniform = true;
            else ke[t] = min(kl, S);
        }
    }
    const int t_begin = kb[0] / kBN;  // tile A starts no later than tile B
    for (int t = 0; t < 2; ++t) nt[t] = q0t[t] < S ? (ke[t] + kBN - 1) / kBN - t_begin : 0;
    // scalars: the roles' loops select between them instead of indexing the arrays with
    // a runtime tile index (which would put the arrays in local memory)
    const int nt0 = nt[0], nt1 = nt[1];
    const int n_max = max(nt0, nt1);

    if (tid == 0) {
        mbar_init(bQ, 1);
        for (int s = 0; s < ST; ++s) {
            mbar_init(bKVfull(s), 1);
            mbar_init(bKVempty(s), 1);
        }
        for (int t = 0; t < 2; ++t) {
            mbar_init(bSfull(t), 1);
            mbar_init(bPfull(t), 128);
            mbar_init(bOdone(t), 1);
        }
        mbar_init(bDrain, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        __syncwarp();  // lane 0 ran the init branch alone; the allocation is warp-collective
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp >= 8) {
      asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
      if (warp == 8) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            mbar_expect_tx(bQ, 2 * Gm::kTileBytes);
            for (int t = 0; t < 2; ++t)
                for (int pn = 0; pn < NP; ++pn)
                    tma_load_4d(sQ + t * Gm::kTileBytes + pn * Gm::kPanelBytes, &tmQ, bQ, 64 * pn, h, q0t[t], b);
            // ring items 0..n_max: K(i) and V(i-1), each into its stage after the stage's
            // previous item was released
            int issued = 0;
            for (int i = 0; n_max > 0 && i <= n_max; ++i) {
                const int st = i % ST;
                if (i >= ST && !mbar_wait(bKVempty(st), ((i / ST) - 1) & 1, abort_flag, status)) break;
                const bool has_k = i < n_max, has_v = i >= 1;
                mbar_expect_tx(bKVfull(st), (has_k ? Gm::kTxTile : 0u) + (has_v ? Gm::kTxTile : 0u));
                if (has_k)
                    for (int pn = 0; pn < NP; ++pn)
                        tma_load_4d(sK + st * Gm::kTileBytes + pn * Gm::kPanelBytes, &tmK, bKVfull(st), 64 * pn, kvh,
                                    (t_begin + i) * kBN, b);
                if (has_v)
                    for (int pn = 0; pn < NP; ++pn)
                        tma_load_4d(sV + st * Gm::kTileBytes + pn * Gm::kPanelBytes, &tmV, bKVfull(st), 64 * pn, kvh,
                                    (t_begin + i - 1) * kBN, b);
                issued = i + 1;
            }
            // every copy this thread issued lands before the CTA may exit
            mbar_drain(bQ, 0);
            for (int i = (issued > ST ? issued - ST : 0); i < issued; ++i) mbar_drain(bKVfull(i % ST), (i / ST) & 1);
        }
    } else if (warp == 9) {
        // ------------------------------------------------------------ MMA issuer
        // The whole warp runs this loop with warp-uniform waits (vote.all); lane 0
        // issues the MMAs and commits.
        {
            const uint32_t ln = (uint32_t)lane;
            const uint32_t idq = make_idesc(p.fmt, kBM, kBN, 0, 0);
            const uint32_t idp = make_idesc(p.fmt, kBM, D, 0, 1);
            int item_ready = -1;  // highest ring item whose full wait was observed
            bool ok = __all_sync(0xffffffffu, mbar_wait(bQ, 0, abort_flag, status));
            auto wait_item = [&](int i) -> bool {
                if (item_ready >= i) return true;
                if (!__all_sync(0xffffffffu, mbar_wait(bKVfull(i % ST), (i / ST) & 1, abort_flag, status)))
                    return false;
                tc_fence_after();
                item_ready = i;
                return true;
            };
            // descriptors of each buffer's start: a K step, tile or stage offset only moves the
            // 14-bit start-address field (addr >> 4) of the low word, and every offset here stays inside it
            const uint64_t dQ = smem_desc(sQ, 16, 1024), dK = smem_desc(sK, 16, 1024);
            const uint64_t dV = smem_desc(sV, Gm::kPanelBytes, 1024);
            const uint32_t q_lo = (uint32_t)dQ, k_lo = (uint32_t)dK, v_lo = (uint32_t)dV;
            const uint32_t qk_hi = (uint32_t)(dQ >> 32), v_hi = (uint32_t)(dV >> 32);  // dK's high word is dQ's
            auto issue_qk = [&](int t, int j) {
                const uint32_t a0 = q_lo + (uint32_t)(t * Gm::kTileBytes >> 4);
                const uint32_t b0 = k_lo + (uint32_t)((j % ST) * Gm::kTileBytes >> 4);
                const uint32_t d = tmem + 128u * t;
#pragma unroll
                for (int ks = 0; ks < D / 16; ++ks) {
                    const uint32_t koff = ((uint32_t)(ks >> 2) * Gm::kPanelBytes + (uint32_t)(ks & 3) * 32u) >> 4;
                    if (ks == 0) umma_ss_w<0>(ln, d, a0, qk_hi, b0, qk_hi, idq);
                    else umma_ss_w<1>(ln, d, a0 + koff, qk_hi, b0 + koff, qk_hi, idq);
                }
                umma_commit_w(ln, bSfull(t));
            };
            auto issue_pv = [&](int t, int j) {
                // V(j) (ring item j+1), MN-major: 8-key atoms 1024 B apart (SBO), 64-column panels kPanelBytes
                // apart (LBO)
                const uint32_t b0 = v_lo + (uint32_t)(((j + 1) % ST) * Gm::kTileBytes >> 4);
                const uint32_t d = tmem + 256u + 128u * t, a = tmem + 128u * t;
                umma_ts_w<-1>(ln, d, a, b0, v_hi, idp, j > 0 ? 1u : 0u);
#pragma unroll
                for (int kk = 1; kk < kBN / 16; ++kk) umma_ts_w<1>(ln, d, a + kk * 8u, b0 + kk * 128u, v_hi, idp);
            };
            if (ok && n_max > 0) {
                ok = wait_item(0);
                if (ok && nt0 > 0) issue_qk(0, 0);
                if (ok && nt1 > 0) issue_qk(1, 0);
                if (ok) umma_commit_w(ln, bKVempty(0));  // item 0 (K(0)) read by both tiles
            }
            for (int j = 0; j < n_max && ok; ++j) {
                // the tile whose part of this step reads item j+1 last: tile B whenever it takes
                // part (its rows follow tile A's, so nt0 <= nt1 unless tile B is empty)
                const int rel = j < nt1 ? 1 : 0;
                // rolled over the two tiles: unrolled, each tile's per-step descriptor words
                // would be loop-invariant and hoisted into (spilled) registers
#pragma unroll 1
                for (int t = 0; t < 2 && ok; ++t) {
                    const int ntt = t ? nt1 : nt0;
                    if (j >= ntt) continue;
                    if (!__all_sync(0xffffffffu, mbar_wait(bPfull(t), j & 1, abort_flag, status))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (!wait_item(j + 1)) {  // V(j), K(j+1)
                        ok = false;
                        break;
                    }
                    issue_pv(t, j);
                    // O_t is complete after its last PV; earlier PVs need no signal of their own:
                    // S_t(j+1) is committed after PV_t(j), and a commit tracks every earlier MMA
                    if (j + 1 == ntt) umma_commit_w(ln, bOdone(t));
                    if (j + 1 < ntt) issue_qk(t, j + 1);
                    if (t == rel) umma_commit_w(ln, bKVempty((j + 1) % ST));
                }
            }
            // all MMAs lane 0 issued are complete before TMEM is released
            umma_commit_w(ln, bDrain);
            mbar_drain(bDrain, 0);
        }
      }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
        // ------------------------------------------------------------ softmax groups
        const int t = warp >> 2;       // 0: tile A, 1: tile B
        const int row = tid & 127;     // TMEM lane within the group
        // this group's tile bounds as scalars (no dynamically indexed arrays in the hot loop)
        const int my_q0 = t ? q0t[1] : q0t[0];
        const int my_kb = t ? kb[1] : kb[0];
        const int my_ke = t ? ke[1] : ke[0];
        const int my_nt = t ? nt[1] : nt[0];
        const int q = my_q0 + row;
        const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        const uint32_t s_addr = lane_base + (t ? 128u : 0u);
        const uint32_t o_addr = lane_base + (t ? 384u : 256u);
        const float sl2 = p.scale_log2;
        const int q_lo = my_q0, q_hi = my_q0 + kBM - 1;
        // keys this row sees: [row_lo, row_hi); a uniform row (no valid key) weights all keys equally
        int row_lo = my_kb, row_hi = my_ke;
        if (causal) {
            row_hi = min(row_hi, q + 1);
            if (window > 0) row_lo = max(row_lo, q - window + 1);
        }
        const float edge_mult = uniform ? 0.f : sl2;
        const bool additive = kAdditive && !uniform;
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        for (int j = 0; j < my_nt && ok; ++j) {
            if (!__all_sync(0xffffffffu, mbar_wait(bSfull(t), j & 1, abort_flag, status))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int n0 = (t_begin + j) * kBN;
            // a tile needs per-element masks when it touches the diagonal, the window start or the key end
            const bool edge = uniform || kAdditive || n0 + kBN > my_ke || n0 < my_kb ||
                              (causal && n0 + kBN - 1 > q_lo) || (causal && window > 0 && n0 <= q_hi - window);
            // the whole score row in registers: one TMEM read serves both passes
            uint32_t r[kBN];
#pragma unroll
            for (int c = 0; c < kBN / 32; ++c) tmem_ld32(s_addr + 32 * c, r + 32 * c);
            tmem_wait_ld();
            if (edge) {
                // masked tiles become log2-domain scores (-inf outside the row's keys)
                const int lo = row_lo - n0, hi = row_hi - n0;
                if (additive) {
                    const float* mrow = mask + (int64_t)b * S + n0;
#pragma unroll
                    for (int i = 0; i < kBN; ++i)
                        r[i] = __float_as_uint(i >= lo && i < hi
                                                   ? (__uint_as_float(r[i]) * scale + __ldg(mrow + i)) * kLog2e
                                                   : -INFINITY);
                } else {
#pragma unroll
                    for (int i = 0; i < kBN; ++i)
                        r[i] = __float_as_uint(i >= lo && i < hi ? __uint_as_float(r[i]) * edge_mult : -INFINITY);
                }
            }
            // pass 1: row maximum (raw scores on interior tiles, scaled after)
            float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
            for (int i = 0; i < kBN; i += 8) {
                mx0 = max3f(mx0, __uint_as_float(r[i]), __uint_as_float(r[i + 1]));
                mx1 = max3f(mx1, __uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
                mx2 = max3f(mx2, __uint_as_float(r[i + 4]), __uint_as_float(r[i + 5]));
                mx3 = max3f(mx3, __uint_as_float(r[i + 6]), __uint_as_float(r[i + 7]));
            }
            float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
            if (!edge) mx *= sl2;
            // lazy rescale: move the reference maximum only when it grew by > threshold
            const bool need = mx > m_run + kRescaleThreshold;
            if (__any_sync(0xffffffffu, need)) {
                const float m_new = need ? mx : m_run;
                const float alpha = (m_run == -INFINITY) ? 0.f : fast_exp2(m_run - m_new);
                l_run *= alpha;
                // O_t holds PV(j-1) complete: S_t(j), waited for above, was committed after it
                if (j > 0) {
#pragma unroll
                    for (int c = 0; c < D / 32; ++c) {
                        uint32_t o[32];
                        tmem_ld32(o_addr + 32 * c, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_st32(o_addr + 32 * c, o);
                    }
                }
                m_run = m_new;
            }
            const float mb = m_run == -INFINITY ? 0.f : m_run;
            // pass 2: P = 2^(s - m) as fp16 pairs over the first 64 S columns, row sum
            const float mul = edge ? 1.f : sl2;
            const f32x2 mul2 = f2_make(mul, mul), nmb2 = f2_make(-mb, -mb);
            f32x2 sum0 = 0ull, sum1 = 0ull;
            uint32_t pk[kBN / 2];
#pragma unroll
            for (int i = 0; i < kBN; i += 2) {
                float x0, x1, e0, e1;
                f2_split(f2_fma(f2_make(__uint_as_float(r[i]), __uint_as_float(r[i + 1])), mul2, nmb2), x0, x1);
                // kPolyPairs of every 8 pairs on the FMA pipe, the rest on the MUFU
                if (((i >> 1) & 7) >= 8 - kPolyPairs) {
                    exp2_poly_pair(x0, x1, e0, e1);
                } else {
                    e0 = fast_exp2(x0);
                    e1 = fast_exp2(x1);
                }
                if ((i >> 1) & 1) sum1 = f2_add(sum1, f2_make(e0, e1));
                else sum0 = f2_add(sum0, f2_make(e0, e1));
                pk[i >> 1] = pack_half2(e0, e1);
                if (((i >> 1) & 15) == 15) tmem_st16(s_addr + (uint32_t)((i >> 1) - 15), pk + (i >> 1) - 15);
            }
            float a0, a1, b0, b1;
            f2_split(sum0, a0, a1);
            f2_split(sum1, b0, b1);
            l_run += (a0 + a1) + (b0 + b1);
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bPfull(t));
        }
        // epilogue: O / l for rows inside the sequence
        if (ok && my_nt > 0 && __all_sync(0xffffffffu, mbar_wait(bOdone(t), 0, abort_flag, status))) {
            tc_fence_after();
            const float inv = 1.f / l_run;
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
                uint32_t r[32];
                tmem_ld32(o_addr + 32 * c, r);
                tmem_wait_ld();
                if (q < S) {
                    const int64_t off = b * p.o_sb + (int64_t)q * p.o_ss + h * p.o_sh + 32 * c;
#pragma unroll
                    for (int i = 0; i < 32; i += 8) {
                        float v[8];
#pragma unroll
                        for (int k = 0; k < 8; ++k) v[k] = __uint_as_float(r[i + k]) * inv;
                        store8(p.out, off + i, v, p.out_dtype);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

// ---------------------------------------------------------------- host side
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
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

// [B][S][H][D] tensor (element strides sb, ss, sh; d contiguous), box 64 x 1 x 128 x 1.
bool make_map(CUtensorMap* m, const void* ptr, int fmt, int B, int S, int H, int D, int64_t sb, int64_t ss,
              int64_t sh) {
    EncodeFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)S, (cuuint64_t)B};
    const cuuint64_t strides[3] = {(cuuint64_t)sh * 2, (cuuint64_t)ss * 2, (cuuint64_t)sb * 2};
    const cuuint32_t box[4] = {64, 1, 128, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = fn(m, fmt ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                          const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int D>
constexpr int smem_request() {
    // at least 116 KB so no two CTAs share an SM: each one allocates all 512 TMEM columns
    return TcGeo<D>::kBytes + 1024 > 116 * 1024 ? TcGeo<D>::kBytes + 1024 : 116 * 1024;
}

// One-time setup of an instantiation on the current device: the shared-memory
// opt-in, and the check that ptxas gave it exactly kRegsLaunch registers per
// thread, the pool the setmaxnreg split in the kernel divides (with any other
// count the softmax warpgroups' increase could not be met, so the kernel is
// reported unsupported and the caller takes another path).
constexpr int kMaxDevices = 64;
template <int D, bool kAdditive>
cudaError_t kernel_ready() {
    static std::once_flag once[kMaxDevices];
    static cudaError_t err[kMaxDevices];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::call_once(once[dev], [dev] {
        cudaFuncAttributes fa{};
        cudaError_t e = cudaFuncGetAttributes(&fa, attn_tcgen05_kernel<D, kAdditive>);
        if (e == cudaSuccess && fa.numRegs != kRegsLaunch) e = cudaErrorInvalidDeviceFunction;
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(attn_tcgen05_kernel<D, kAdditive>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     smem_request<D>());
        err[dev] = e;
    });
    return err[dev];
}
template <int D>
cudaError_t kernel_ready_for(const AttnParams& p) {
    return p.mask != nullptr ? kernel_ready<D, true>() : kernel_ready<D, false>();
}

template <int D>
cudaError_t launch_impl(const AttnParams& a, int* status, cudaStream_t stream) {
    const bool additive = a.mask != nullptr;
    const cudaError_t ready = kernel_ready_for<D>(a);
    if (ready != cudaSuccess) return ready;
    const int fmt = 0;  // fp16 operands (attn_tcgen05_supported)
    CUtensorMap mq, mk, mv;
    if (!make_map(&mq, a.q, fmt, a.B, a.S, a.Hq, a.D, a.q_sb, a.q_ss, a.q_sh) ||
        !make_map(&mk, a.k, fmt, a.B, a.S, a.Hkv, a.D, a.k_sb, a.k_ss, a.k_sh) ||
        !make_map(&mv, a.v, fmt, a.B, a.S, a.Hkv, a.D, a.k_sb, a.k_ss, a.k_sh))
        return cudaErrorInvalidValue;
    TcParams p{};
    p.B = a.B;
    p.S = a.S;
    p.Hq = a.Hq;
    p.Hkv = a.Hkv;
    p.G = a.Hq / a.Hkv;
    p.D = a.D;
    p.causal = a.causal;
    p.window = a.window;
    p.mask = a.mask;
    p.key_len = a.key_len;
    p.scale = a.scale;
    p.scale_log2 = a.scale * kLog2e;
    p.out = a.o;
    p.out_dtype = a.out_dtype;
    p.o_sb = a.q_sb;
    p.o_ss = a.q_ss;
    p.o_sh = a.q_sh;
    p.status = status;
    p.fmt = fmt;
    dim3 grid((a.S + 2 * kBM - 1) / (2 * kBM), a.Hq, a.B);
    if (additive)
        attn_tcgen05_kernel<D, true><<<grid, kThreadsTc, smem_request<D>(), stream>>>(mq, mk, mv, p);
    else
        attn_tcgen05_kernel<D, false><<<grid, kThreadsTc, smem_request<D>(), stream>>>(mq, mk, mv, p);
    return cudaGetLastError();
}

}  // namespace

bool attn_tcgen05_supported(const AttnParams& p) {
    // fp16 operands only: P goes to TMEM as fp16 and both MMA operands share one type
    if (p.in_dtype != kF16) return false;
    if (!(p.D == 64 || p.D == 96 || p.D == 128)) return false;
    const int64_t strides[] = {p.q_sb, p.q_ss, p.q_sh, p.k_sb, p.k_ss, p.k_sh};
    for (int64_t s : strides)
        if (s % 8 != 0 || s <= 0) return false;
    const uintptr_t ptrs[] = {(uintptr_t)p.q, (uintptr_t)p.k, (uintptr_t)p.v, (uintptr_t)p.o};
    for (uintptr_t x : ptrs)
        if (x % 16 != 0) return false;
    if (p.Hq > 65535 || p.B > 65535 || encode_fn() == nullptr) return false;
    const cudaError_t ready = p.D == 64 ? kernel_ready_for<64>(p) : p.D == 96 ? kernel_ready_for<96>(p)
                                                                               : kernel_ready_for<128>(p);
    return ready == cudaSuccess;
}

cudaError_t launch_attn_tcgen05(const AttnParams& p, int* status, cudaStream_t stream) {
    switch (p.D) {
        case 64: return launch_impl<64>(p, status, stream);
        case 96: return launch_impl<96>(p, status, stream);
        case 128: return launch_impl<128>(p, status, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace b2a
