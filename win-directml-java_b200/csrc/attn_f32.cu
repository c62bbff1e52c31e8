// attn_f32.cu -- fp32 whole-sequence attention for head_dim 64 and 128: causal
// prefill (optional sliding window and NeoX RoPE applied inside), bidirectional
// encoder with per-sequence key lengths or an additive key mask.  It is the
// FLOAT32 path of the reference's attention contract
// (WB/runtime/kernels/AttentionKernel.java:19-24) and of fp32 causal prefill
// (SmolLM2ReferenceForwardPass.runSelfAttention,
// INF/smollm2/SmolLM2ReferenceForwardPass.java:167-210), laid out for short,
// latency-bound launches: every CTA owns whole query rows, so no CTA waits on
// another and nothing is merged across CTAs.
//
// CTA = 16 query rows of one (batch, q head) and kParts groups of four warps (4 at
// head_dim 64, 2 at 128, where a thread needs twice the registers).  The block's key
// tiles (64 keys) are dealt round-robin to the groups; each group streams its tiles
// through its own shared K and V buffers (16-byte cp.async; the next K is requested
// as soon as the current scores are formed, the next V as soon as P.V is done).
// Warp w of a group owns keys [16w, 16w + 16) of each of the group's tiles and keeps
// its own online softmax for the 16 rows; at the end every warp's (max, sum, O)
// rows are combined (log-sum-exp) in shared memory.
//
// Products: m16n8k8 TF32 warp MMAs in three passes, a_hi*b_hi + a_hi*b_lo +
// a_lo*b_hi, with x_hi = tf32(x) and x_lo = tf32(x - x_hi) (round to nearest): each
// product keeps ~21 significant bits (the dropped a_lo*b_lo term is below 2^-21
// relative) and accumulates in fp32.  Measured on B200 against the fp32 FMA form of
// this kernel: 14.1 against 16.3 us per configs[0] step (warm), the three passes
// costing less issue than 1024 FMAs per MMA; outputs stay within the 1e-4 the fp32
// tests hold them to.
//   S = Q K^T   A = q rows (split once when staged), B = the warp's 16 keys;
//   O += P V    A = P (through a per-warp shared tile), B = V.
// K rows are padded to D + 4 floats and V rows to D + 8, so the fragment reads
// (8 rows x 4 columns of K, 4 rows x 8 columns of V) hit 32 distinct banks.
// RoPE: q rows are rotated as they are staged; each K tile is rotated in shared
// memory with (cos, sin) values fetched into registers with the tile (float
// products of the float (cos, sin) of a double angle: the same arithmetic as the
// generic kernel and the pre-pass).
#include <math.h>

#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace b2a {
namespace {

constexpr int kBM = 16;      // query rows per CTA
constexpr int kBN = 64;      // keys per tile
constexpr int kGroup = 128;  // threads of one warp group
constexpr int kPP = 20;      // pitch of a warp's P tile (16 x 16): conflict-free fragment reads

template <int D>
struct F32Geo {
    static constexpr int kParts = D <= 64 ? 4 : 2;  // warp groups
    static constexpr int kThreads = kParts * kGroup;
    static constexpr int kWarps = kThreads / 32;
    static constexpr int kKP = D + 4;  // K / Q row pitch: 4g + t banks for an 8 x 4 fragment
    static constexpr int kVP = D + 8;  // V row pitch: 8t + g banks for a 4 x 8 fragment
    static constexpr int kGroupFloats = kBN * kKP + kBN * kVP + 4 * kBM * kPP;  // K, V, P of one group
    static constexpr int kQFloats = 2 * kBM * kKP;                              // q hi and lo parts
    static constexpr size_t kBytes = size_t(kParts * kGroupFloats + kQFloats) * sizeof(float);
    static constexpr int kRot = kBN * (D / 2) / kGroup;  // K rotation pairs per thread and tile
    // combine area (after the loop, over the groups' buffers): per warp 16 rows of O and (m, l),
    // then one weight per (warp, row)
    static constexpr int kOP = D + 4;
    static constexpr int kWarpOut = kBM * kOP + 2 * kBM;
    static_assert(kWarps * kWarpOut + kWarps * kBM + kBM <= kParts * kGroupFloats, "combine area fits");
};

__device__ __forceinline__ void bar_part(int part) {  // the 128 threads of one warp group
    asm volatile("bar.sync %0, %1;" ::"r"(1 + part), "n"(kGroup) : "memory");
}

__device__ __forceinline__ uint32_t to_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}
// x = hi + lo, both TF32 (the three-pass split)
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
    hi = to_tf32(x);
    lo = to_tf32(x - __uint_as_float(hi));
}
__device__ __forceinline__ void mma_tf32(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// d += a * b in three passes (small terms first)
__device__ __forceinline__ void mma3(float (&d)[4], const uint32_t (&ah)[4], const uint32_t (&al)[4], uint32_t bh0,
                                     uint32_t bh1, uint32_t bl0, uint32_t bl1) {
    mma_tf32(d, al[0], al[1], al[2], al[3], bh0, bh1);
    mma_tf32(d, ah[0], ah[1], ah[2], ah[3], bl0, bl1);
    mma_tf32(d, ah[0], ah[1], ah[2], ah[3], bh0, bh1);
}

template <int D>
__global__ void __launch_bounds__(F32Geo<D>::kThreads) attn_f32_kernel(const __grid_constant__ AttnParams p) {
    using Gm = F32Geo<D>;
    constexpr int kKP = Gm::kKP, kVP = Gm::kVP, kParts = Gm::kParts, kThreads = Gm::kThreads;
    // launched with programmatic serialisation: placed while the kernel ahead finishes, every global
    // access waits for it
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    constexpr int kHalfD = D / 2;
    extern __shared__ __align__(16) float fsm[];
    const int tid = threadIdx.x, part = tid >> 7, ht = tid & (kGroup - 1);
    const int lane = tid & 31, wg = ht >> 5;  // warp within the group
    const int g = lane >> 2, t4 = lane & 3;   // MMA fragment coordinates
    float* const ks = fsm + part * Gm::kGroupFloats;
    float* const vs = ks + kBN * kKP;
    float* const ps = vs + kBN * kVP + wg * kBM * kPP;  // this warp's P tile
    float* const qhi = fsm + kParts * Gm::kGroupFloats;
    float* const qlo = qhi + kBM * kKP;

    const int S = p.S;
    const int nblk = (S + kBM - 1) / kBM;
    const int blk = nblk - 1 - (int)blockIdx.x;  // longest causal blocks first
    const int h = blockIdx.y, b = blockIdx.z;
    const int kvh = h / (p.Hq / p.Hkv);
    const int r0 = blk * kBM, r1 = min(S, r0 + kBM);
    const float2* const rope = p.rope_table;

    // key range of the block: causal [window start of row r0, r1), else the sequence's keys
    bool uniform = false;
    int kf = 0, ke = S;
    if (p.causal) {
        ke = r1;
        if (p.window > 0) kf = max(0, r0 - p.window + 1);
    } else if (p.key_len != nullptr) {
        const int kl = p.key_len[b];
        if (kl <= 0) uniform = true;  // every key masked: equal scores, the mean of V
        else ke = min(kl, S);
    }
    const int t_begin = kf / kBN, t_end = (ke + kBN - 1) / kBN;

    const float* const kg = static_cast<const float*>(p.k) + b * p.k_sb + (int64_t)kvh * p.k_sh;
    const float* const vg = static_cast<const float*>(p.v) + b * p.k_sb + (int64_t)kvh * p.k_sh;
    auto load_rows = [&](float* dst, int pitch, const float* src, int t) {
        const int n0 = t * kBN;
#pragma unroll
        for (int i = 0; i < kBN * D / 4 / kGroup; ++i) {
            const int e = ht + i * kGroup, key = e / (D / 4), c = e - key * (D / 4);
            const bool in = n0 + key < S;
            const float* src_row = src + (int64_t)(in ? n0 + key : 0) * p.k_ss + 4 * c;
            cp_async_16(smem_u32(dst + key * pitch + 4 * c), src_row, in ? 16 : 0);
        }
        cp_async_commit();
    };
    float2 trot[Gm::kRot];
    auto fetch_rot = [&](int t) {  // (cos, sin) of this thread's K pairs of tile t
        const int n0 = t * kBN;
#pragma unroll
        for (int i = 0; i < Gm::kRot; ++i) {
            const int e = ht + i * kGroup, key = e / kHalfD, j = e - key * kHalfD;
            trot[i] = n0 + key < S ? __ldg(rope + (int64_t)(p.rope_pos0 + n0 + key) * kHalfD + j)
                                   : make_float2(1.f, 0.f);
        }
    };

    // this group's first tile in flight before the q rows are prepared
    const int t0 = t_begin + part;
    if (t0 < t_end) {
        if (rope != nullptr) fetch_rot(t0);
        load_rows(ks, kKP, kg, t0);
        load_rows(vs, kVP, vg, t0);
    }

    // q rows (rotated at positions rope_pos0 + row; zeros past the sequence), stored as
    // their TF32 hi and lo parts
    const float* const qg = static_cast<const float*>(p.q) + b * p.q_sb + (int64_t)h * p.q_sh;
    auto put_q = [&](int r, int d, float4 v) {
        const float x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint32_t hi, lo;
            split_tf32(x[i], hi, lo);
            qhi[r * kKP + d + i] = __uint_as_float(hi);
            qlo[r * kKP + d + i] = __uint_as_float(lo);
        }
    };
    if (rope != nullptr) {
        for (int e = tid; e < kBM * (D / 8); e += kThreads) {
            const int r = e / (D / 8), c = e - r * (D / 8);  // float4 c and its partner c + D/8
            float4 lo = make_float4(0.f, 0.f, 0.f, 0.f), hi = lo;
            if (r0 + r < S) {
                const float* row = qg + (int64_t)(r0 + r) * p.q_ss;
                const float4 a = *reinterpret_cast<const float4*>(row + 4 * c);
                const float4 z = *reinterpret_cast<const float4*>(row + 4 * c + kHalfD);
                const float2* cs = rope + (int64_t)(p.rope_pos0 + r0 + r) * kHalfD + 4 * c;
                const float av[4] = {a.x, a.y, a.z, a.w}, zv[4] = {z.x, z.y, z.z, z.w};
                float lv[4], hv[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 t = __ldg(cs + i);
                    lv[i] = __fsub_rn(__fmul_rn(av[i], t.x), __fmul_rn(zv[i], t.y));
                    hv[i] = __fadd_rn(__fmul_rn(av[i], t.y), __fmul_rn(zv[i], t.x));
                }
                lo = make_float4(lv[0], lv[1], lv[2], lv[3]);
                hi = make_float4(hv[0], hv[1], hv[2], hv[3]);
            }
            put_q(r, 4 * c, lo);
            put_q(r, 4 * c + kHalfD, hi);
        }
    } else {
        for (int e = tid; e < kBM * (D / 4); e += kThreads) {
            const int r = e / (D / 4), c = e - r * (D / 4);
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (r0 + r < S) v = *reinterpret_cast<const float4*>(qg + (int64_t)(r0 + r) * p.q_ss + 4 * c);
            put_q(r, 4 * c, v);
        }
    }
    __syncthreads();

    // this thread's rows g and g + 8: keys [lo, hi) visible to each
    const float sl2 = p.scale * kLog2e;
    const float* const mrow = p.mask != nullptr ? p.mask + (int64_t)b * S : nullptr;
    int lo_key[2], hi_key[2];
#pragma unroll
    for (int a = 0; a < 2; ++a) {
        const int q = r0 + g + 8 * a;
        lo_key[a] = 0;
        hi_key[a] = ke;
        if (p.causal) {
            hi_key[a] = min(ke, q + 1);
            if (p.window > 0) lo_key[a] = max(0, q - p.window + 1);
        }
    }
    // keys any row of the block sees (a warp whose 16 keys lie outside skips the tile)
    const int blk_lo = p.causal && p.window > 0 ? kf : 0, blk_hi = ke;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    float o[D / 8][4];
#pragma unroll
    for (int nb = 0; nb < D / 8; ++nb) o[nb][0] = o[nb][1] = o[nb][2] = o[nb][3] = 0.f;

    for (int t = t0; t < t_end; t += kParts) {
        const int n0 = t * kBN;
        cp_async_wait<1>();  // K(t) landed (V(t) may still be in flight)
        bar_part(part);
        if (rope != nullptr) {
#pragma unroll
            for (int i = 0; i < Gm::kRot; ++i) {
                const int e = ht + i * kGroup, key = e / kHalfD, j = e - key * kHalfD;
                float* row = ks + key * kKP;
                const float a = row[j], z = row[j + kHalfD];
                row[j] = __fsub_rn(__fmul_rn(a, trot[i].x), __fmul_rn(z, trot[i].y));
                row[j + kHalfD] = __fadd_rn(__fmul_rn(a, trot[i].y), __fmul_rn(z, trot[i].x));
            }
            bar_part(part);
        }
        const int wk0 = n0 + 16 * wg;  // this warp's keys [wk0, wk0 + 16)
        const bool active = wk0 < blk_hi && wk0 + 16 > blk_lo;
        // S = Q K^T for the warp's 16 keys: two n-blocks of 8 keys
        float s[2][4];
#pragma unroll
        for (int nb = 0; nb < 2; ++nb) s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.f;
        if (active && !uniform) {
#pragma unroll
            for (int kk = 0; kk < D / 8; ++kk) {
                uint32_t ah[4], al[4];
                const int c = 8 * kk + t4;
                ah[0] = __float_as_uint(qhi[g * kKP + c]);
                ah[1] = __float_as_uint(qhi[(g + 8) * kKP + c]);
                ah[2] = __float_as_uint(qhi[g * kKP + c + 4]);
                ah[3] = __float_as_uint(qhi[(g + 8) * kKP + c + 4]);
                al[0] = __float_as_uint(qlo[g * kKP + c]);
                al[1] = __float_as_uint(qlo[(g + 8) * kKP + c]);
                al[2] = __float_as_uint(qlo[g * kKP + c + 4]);
                al[3] = __float_as_uint(qlo[(g + 8) * kKP + c + 4]);
#pragma unroll
                for (int nb = 0; nb < 2; ++nb) {
                    const float* kr = ks + (16 * wg + 8 * nb + g) * kKP + c;
                    uint32_t bh0, bl0, bh1, bl1;
                    split_tf32(kr[0], bh0, bl0);
                    split_tf32(kr[4], bh1, bl1);
                    mma3(s[nb], ah, al, bh0, bh1, bl0, bl1);
                }
            }
        }
        bar_part(part);  // every score read of K(t) is done: the buffer takes the group's next K
        if (t + kParts < t_end) {
            if (rope != nullptr) fetch_rot(t + kParts);
            load_rows(ks, kKP, kg, t + kParts);
        } else {
            cp_async_commit();  // an empty group keeps the wait counts uniform
        }
        // masked log2-domain scores; online softmax over the warp's keys (4 lanes per row)
        float corr[2];
#pragma unroll
        for (int a = 0; a < 2; ++a) {
            float mx = -INFINITY;
#pragma unroll
            for (int nb = 0; nb < 2; ++nb)
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const int key = wk0 + 8 * nb + 2 * t4 + i;
                    const float raw = s[nb][2 * a + i];
                    float v;
                    if (!active) v = -INFINITY;
                    else if (uniform) v = key < S ? 0.f : -INFINITY;
                    else if (key < lo_key[a] || key >= hi_key[a]) v = -INFINITY;
                    else if (mrow != nullptr) v = (raw * p.scale + __ldg(mrow + key)) * kLog2e;
                    else v = raw * sl2;
                    s[nb][2 * a + i] = v;
                    mx = fmaxf(mx, v);
                }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float mn = fmaxf(m[a], mx);
            corr[a] = mn == -INFINITY ? 1.f : fast_exp2(m[a] - mn);
            float sum = 0.f;
#pragma unroll
            for (int nb = 0; nb < 2; ++nb) {
                const float e0 = mn == -INFINITY ? 0.f : fast_exp2(s[nb][2 * a] - mn);
                const float e1 = mn == -INFINITY ? 0.f : fast_exp2(s[nb][2 * a + 1] - mn);
                *reinterpret_cast<float2*>(ps + (g + 8 * a) * kPP + 8 * nb + 2 * t4) = make_float2(e0, e1);
                sum += e0 + e1;
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            l[a] = l[a] * corr[a] + sum;
            m[a] = mn;
        }
#pragma unroll
        for (int nb = 0; nb < D / 8; ++nb) {
            o[nb][0] *= corr[0];
            o[nb][1] *= corr[0];
            o[nb][2] *= corr[1];
            o[nb][3] *= corr[1];
        }
        cp_async_wait<1>();  // V(t) landed (the next K may still be in flight)
        bar_part(part);      // V(t) visible to the group (P is the warp's own: __syncwarp suffices)
        // O += P V over the warp's 16 keys: two k-steps of 8 keys
        if (active) {
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
                uint32_t ah[4], al[4];
                split_tf32(ps[g * kPP + 8 * kk + t4], ah[0], al[0]);
                split_tf32(ps[(g + 8) * kPP + 8 * kk + t4], ah[1], al[1]);
                split_tf32(ps[g * kPP + 8 * kk + t4 + 4], ah[2], al[2]);
                split_tf32(ps[(g + 8) * kPP + 8 * kk + t4 + 4], ah[3], al[3]);
                const float* v0 = vs + (16 * wg + 8 * kk + t4) * kVP + g;
#pragma unroll
                for (int nb = 0; nb < D / 8; ++nb) {
                    uint32_t bh0, bl0, bh1, bl1;
                    split_tf32(v0[8 * nb], bh0, bl0);
                    split_tf32(v0[4 * kVP + 8 * nb], bh1, bl1);
                    mma3(o[nb], ah, al, bh0, bh1, bl0, bl1);
                }
            }
        }
        bar_part(part);  // V(t) consumed: V's buffer takes the group's next V
        if (t + kParts < t_end) load_rows(vs, kVP, vg, t + kParts);
        else cp_async_commit();
    }
    cp_async_wait<0>();

    // every warp's rows into the combine area (over the groups' buffers, now idle)
    __syncthreads();
    const int W = part * 4 + wg;
    float* const mine = fsm + W * Gm::kWarpOut;
#pragma unroll
    for (int nb = 0; nb < D / 8; ++nb) {
        *reinterpret_cast<float2*>(mine + g * Gm::kOP + 8 * nb + 2 * t4) = make_float2(o[nb][0], o[nb][1]);
        *reinterpret_cast<float2*>(mine + (g + 8) * Gm::kOP + 8 * nb + 2 * t4) = make_float2(o[nb][2], o[nb][3]);
    }
    if (t4 == 0) {
#pragma unroll
        for (int a = 0; a < 2; ++a) {
            mine[kBM * Gm::kOP + g + 8 * a] = m[a];
            mine[kBM * Gm::kOP + kBM + g + 8 * a] = l[a];
        }
    }
    __syncthreads();
    // per row: each warp's weight 2^(m_w - M) / sum_w 2^(m_w - M) l_w
    float* const wts = fsm + Gm::kWarps * Gm::kWarpOut;
    if (tid < kBM) {
        const int r = tid;
        float M = -INFINITY;
        for (int w = 0; w < Gm::kWarps; ++w) M = fmaxf(M, fsm[w * Gm::kWarpOut + kBM * Gm::kOP + r]);
        float den = 0.f;
        for (int w = 0; w < Gm::kWarps; ++w) {
            const float mw = fsm[w * Gm::kWarpOut + kBM * Gm::kOP + r];
            const float f = mw == -INFINITY ? 0.f : fast_exp2(mw - M);
            wts[w * kBM + r] = f;
            den += f * fsm[w * Gm::kWarpOut + kBM * Gm::kOP + kBM + r];
        }
        const float inv = 1.f / den;
        for (int w = 0; w < Gm::kWarps; ++w) wts[w * kBM + r] *= inv;
    }
    __syncthreads();
    float* const og = static_cast<float*>(p.o);
    for (int e4 = tid; e4 < kBM * (D / 4); e4 += kThreads) {
        const int r = e4 / (D / 4), d = 4 * (e4 - r * (D / 4));
        if (r0 + r >= S) continue;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
        for (int w = 0; w < Gm::kWarps; ++w) {
            const float f = wts[w * kBM + r];
            const float4 ow = *reinterpret_cast<const float4*>(fsm + w * Gm::kWarpOut + r * Gm::kOP + d);
            acc.x = fmaf(f, ow.x, acc.x);
            acc.y = fmaf(f, ow.y, acc.y);
            acc.z = fmaf(f, ow.z, acc.z);
            acc.w = fmaf(f, ow.w, acc.w);
        }
        const int64_t oi = b * p.q_sb + (int64_t)(r0 + r) * p.q_ss + (int64_t)h * p.q_sh + d;
        if (p.out_dtype == kF32) {
            *reinterpret_cast<float4*>(og + oi) = acc;
        } else {
            store_from_float(p.o, oi + 0, acc.x, p.out_dtype);
            store_from_float(p.o, oi + 1, acc.y, p.out_dtype);
            store_from_float(p.o, oi + 2, acc.z, p.out_dtype);
            store_from_float(p.o, oi + 3, acc.w, p.out_dtype);
        }
    }
}

template <int D>
cudaError_t launch_d(const AttnParams& p, cudaStream_t stream) {
    constexpr size_t smem = F32Geo<D>::kBytes;
    // the shared-memory opt-in is a per-device attribute: set once for each device
    constexpr int kMaxDevices = 64;
    static std::once_flag once[kMaxDevices];
    static cudaError_t attr[kMaxDevices];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::call_once(once[dev], [dev] {
        attr[dev] = cudaFuncSetAttribute(attn_f32_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    });
    if (attr[dev] != cudaSuccess) return attr[dev];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((p.S + kBM - 1) / kBM), (unsigned)p.Hq, (unsigned)p.B);
    cfg.blockDim = dim3(F32Geo<D>::kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, attn_f32_kernel<D>, p);
}

}  // namespace

bool attn_f32_supported(const AttnParams& p) {
    // float4 rows: head dim, strides and bases in whole 16-byte units; q and o share strides
    const bool al = p.q_sb % 4 == 0 && p.q_ss % 4 == 0 && p.q_sh % 4 == 0 && p.k_sb % 4 == 0 && p.k_ss % 4 == 0 &&
                    p.k_sh % 4 == 0 && (uintptr_t)p.q % 16 == 0 && (uintptr_t)p.k % 16 == 0 &&
                    (uintptr_t)p.v % 16 == 0 && (uintptr_t)p.o % 16 == 0;
    return p.in_dtype == kF32 && (p.D == 64 || p.D == 128) && al && p.S > 0 && p.Hkv > 0 && p.Hq % p.Hkv == 0 &&
           p.Hq <= 65535 && p.B <= 65535;
}

cudaError_t launch_attn_f32(const AttnParams& p, cudaStream_t stream) {
    return p.D == 64 ? launch_d<64>(p, stream) : launch_d<128>(p, stream);
}

}  // namespace b2a
