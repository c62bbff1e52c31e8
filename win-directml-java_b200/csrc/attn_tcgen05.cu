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
// from TMEM), O_A at 256, O_B at 384.  At head dim 256 a work item is one
// query tile (S_A 0..127, O_A 128..383; warps 4-7 have no tile) and the K/V
// ring has one stage (Q 64 KB + K 64 KB + V 64 KB of shared memory).
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
// Head dims 32, 64, 96, 128 and 256.  A K/V/Q row is staged as 64-element panels
// (the TMA box is 64 wide; dims past D are zero-filled): at D = 32 the QK MMAs read
// the first two 16-element K steps of each row and the PV MMAs have N = 32, so the
// zero half of the panel is never read.
// Same semantics as attn_simt.cu / attn_mma.cu (the reference citations are
// there); operands are fp16 (bf16 callers are converted by the host layer).
// The additive [B][S] key mask has its own instantiation (kAdditive).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "internal.h"
#include "sm100.cuh"

namespace b2a {
namespace {

constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kThreadsTc = 384;
// Register split between the warpgroups (setmaxnreg): the kernel launches with
// kRegsLaunch per thread (ptxas' limit for 384 threads and one CTA per SM, which
// the host checks before launching); the control warpgroup returns registers so
// the two softmax warpgroups can keep a whole 128-column score row resident.
// 2 * kSoftmax + kControl == 3 * kRegsLaunch: the pool is used exactly.  At D = 256
// the MMA issuer (16 QK and 8 PV MMAs per step) needs more of the control share.
constexpr int kRegsLaunch = 168;
template <int D>
struct RegSplit {
    static constexpr int kSoftmax = D <= 128 ? 216 : 208;
    static constexpr int kControl = 3 * kRegsLaunch - 2 * kSoftmax;
    static_assert(kControl % 8 == 0 && kSoftmax % 8 == 0, "setmaxnreg takes multiples of 8");
};
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
    int* sched;   // device int[2]: next work item, CTAs finished (zero between launches)
    int n_items;  // work items: query-tile pairs x heads x batch (packed: ceil(heads x batch / 2))
    int stall;    // test hook: the CTA of work item 0 does not issue that item's ring item 1 (V(0), K(1))
    // packed items (bidirectional, S <= 128, two query tiles per item): tile A and tile B are the
    // single query tiles of two consecutive (batch, head) pairs, so both softmax groups work
    int packed;
    // in-kernel operand conversion by warps 10 and 11 (kXformQ / K / V): the staged bf16 tile
    // becomes the fp16 operand in place
    int xform;
};
constexpr int kXformQ = 1, kXformK = 2, kXformV = 4;

template <int D>
struct TcGeo {
    // Panels of 64 elements with the 128-byte swizzle; at D = 96, panels of 32 elements with the
    // 64-byte swizzle: three of them hold a row without padding (a tile takes 24 KB, not 32 KB),
    // which leaves the shared memory for two Q buffers
    static constexpr int kPanelElems = D == 96 ? 32 : 64;
    static constexpr int kRowBytes = 2 * kPanelElems;             // one panel row
    static constexpr uint32_t kLayout = D == 96 ? 4u : 2u;        // UMMA descriptor layout: 64B / 128B swizzle
    static constexpr int NP = (D + kPanelElems - 1) / kPanelElems;  // panels per row
    static constexpr int kPanelBytes = 128 * kRowBytes;          // 128 rows
    static constexpr int kTileBytes = NP * kPanelBytes;
    // query tiles per work item: TMEM holds kTiles x (S 128 + O D) columns, two tiles up to D = 128
    static constexpr int kTiles = D <= 128 ? 2 : 1;
    static constexpr uint32_t kOcol = 128u * kTiles;  // first O column (the S tiles come first)
    // ring stages; at D = 256 one (a step's softmax + 24 MMAs outlast the next tiles' loads)
    static constexpr int kStages = D <= 64 ? 3 : (D <= 128 ? 2 : 1);
    // Q buffers per tile: two at D <= 64 and D = 96, so that the next work item's Q tiles load
    // while the current item still reads its own (short items would otherwise wait for Q after
    // every item)
    static constexpr int kQBuf = (D <= 64 || D == 96) ? 2 : 1;
    static constexpr int kQTiles = kQBuf * kTiles;
    static constexpr int oQ = 0;                   // Q tiles: buffer-major, tile-minor
    static constexpr int oK = kQTiles * kTileBytes;
    static constexpr int oV = oK + kStages * kTileBytes;
    static constexpr int oBar = oV + kStages * kTileBytes;
    static constexpr int kBytes = oBar + 512;  // barriers, TMEM address, abort flag, work-item mailbox
    static constexpr uint32_t kTxTile = kTileBytes;  // bytes one K or V tile load delivers (zero fill included)
    static_assert(kBytes + 1024 <= 227 * 1024, "shared memory budget");
};

// 8 bf16 values (one 16-byte chunk) as floats (exact), and 8 floats packed to fp16.
__device__ __forceinline__ void unpack8_bf16(uint4 r, float* x) {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        x[2 * i] = __uint_as_float(w[i] << 16);
        x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}
__device__ __forceinline__ uint4 pack8_f16(const float* x) {
    uint4 u;
    u.x = pack_half2(x[0], x[1]);
    u.y = pack_half2(x[2], x[3]);
    u.z = pack_half2(x[4], x[5]);
    u.w = pack_half2(x[6], x[7]);
    return u;
}

// In-kernel conversion of one staged bf16 tile (TMA layout: 128 rows of swizzled panels, TcGeo<D>:
// 64-element panels with the 128-byte swizzle, 32-element ones with the 64-byte swizzle at D = 96):
// rows [0, rows) become fp16 in place.  Thread tx of the 64 takes rows tx and tx + 64.  Returns the
// largest |value| (a value beyond the fp16 range becomes infinite: the caller flags it).
template <int D>
__device__ __forceinline__ float xform_tile(unsigned char* tile, int tx, int rows) {
    constexpr int kChunks = D / 8;                      // 16-byte chunks of a row that hold data
    constexpr int kPer = (D == 96 ? 32 : 64) / 8;       // chunks per panel row
    constexpr int kPanel = 128 * 16 * kPer;             // panel bytes
    float mx = 0.f;
    for (int rr = tx; rr < rows && rr < 128; rr += 64) {
        // 128-byte swizzle: chunk ^ (row & 7); 64-byte swizzle: chunk ^ ((row >> 1) & 3)
        const int sw = kPer == 8 ? (rr & 7) : ((rr >> 1) & 3);
#pragma unroll 4
        for (int c = 0; c < kChunks; ++c) {
            uint4* pc = reinterpret_cast<uint4*>(tile + (c / kPer) * kPanel + rr * 16 * kPer +
                                                 (((c % kPer) ^ sw) << 4));
            float x[8];
            unpack8_bf16(*pc, x);
#pragma unroll
            for (int i = 0; i < 8; ++i) mx = fmaxf(mx, fabsf(x[i]));
            *pc = pack8_f16(x);
        }
    }
    return mx;
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

// ---------------------------------------------------------------- kernel
// kAdditive: the additive [B][S] key mask is applied (its own instantiation, so the
// mask loads do not weigh on the register budget of the unmasked kernels).
// A work item is the group of `tiles` query tiles (A, B; one tile, A, when the head dim
// leaves TMEM room for one) starting at row 128 * tiles * pair of one (batch, head).
// Items are numbered pair-fastest, longest causal pair first within a head:
// w = x + n_pairs * (h + Hq * b), pair = n_pairs - 1 - x when causal.  CTAs take
// items in that order from a device counter, so the heads in flight at any time are a
// few consecutive ones (their K/V stay in L2) and the longest items start first.
struct ItemGeo {
    int b, h;         // tile A's batch and head
    int b1, h1;       // tile B's (packed items: the next (batch, head) pair; else b, h)
    int q0a, q0b;     // first query row of tile A / B
    int kb0, kb1;     // first visible key of tile A / B (sliding window)
    int ke0, ke1;     // key end of tile A / B
    int t_begin;      // first key tile (tile A's window start)
    int nt0, nt1;     // key tiles of tile A / B from t_begin (0: tile beyond S)
    int n_max;
    bool uniform;     // tile A has no valid key (key_len <= 0): every key weighs the same
    bool uniform1;    // the same for tile B
};

__device__ __forceinline__ ItemGeo item_geo(int w, int n_pairs, int tiles, int Hq, int S, int causal, int window,
                                            const int32_t* key_len, int packed, int n_heads_total) {
    ItemGeo g;
    if (packed) {
        // two (batch, head) pairs of one 128-row tile each, the whole (<= 128-key) sequence visible
        const int bh0 = 2 * w, bh1 = 2 * w + 1;
        g.b = bh0 / Hq;
        g.h = bh0 - g.b * Hq;
        const bool has1 = bh1 < n_heads_total;
        g.b1 = has1 ? bh1 / Hq : g.b;
        g.h1 = has1 ? bh1 - g.b1 * Hq : g.h;
        g.q0a = g.q0b = 0;
        g.kb0 = g.kb1 = 0;
        g.ke0 = g.ke1 = S;
        g.uniform = g.uniform1 = false;
        if (key_len != nullptr) {
            const int kl0 = key_len[g.b], kl1 = key_len[g.b1];
            if (kl0 <= 0) g.uniform = true;
            else g.ke0 = min(kl0, S);
            if (kl1 <= 0) g.uniform1 = true;
            else g.ke1 = min(kl1, S);
        }
        g.t_begin = 0;
        g.nt0 = 1;
        g.nt1 = has1 ? 1 : 0;
        g.n_max = 1;
        return g;
    }
    const int x = w % n_pairs, rest = w / n_pairs;
    g.h = rest % Hq;
    g.b = rest / Hq;
    g.b1 = g.b;
    g.h1 = g.h;
    const int pair = causal ? n_pairs - 1 - x : x;
    g.q0a = pair * tiles * kBM;
    g.q0b = tiles == 2 ? g.q0a + kBM : S;  // a single-tile item's tile B lies past the sequence
    g.kb0 = g.kb1 = 0;
    g.ke0 = g.ke1 = S;
    g.uniform = false;
    if (causal) {
        g.ke0 = min(S, g.q0a + kBM);
        g.ke1 = min(S, g.q0b + kBM);
        if (window > 0) {
            g.kb0 = max(0, g.q0a - window + 1);
            g.kb1 = max(0, g.q0b - window + 1);
        }
    } else if (key_len != nullptr) {
        const int kl = key_len[g.b];
        if (kl <= 0) g.uniform = true;
        else g.ke0 = g.ke1 = min(kl, S);
    }
    g.uniform1 = g.uniform;
    g.t_begin = g.kb0 / kBN;  // tile A starts no later than tile B
    g.nt0 = (g.ke0 + kBN - 1) / kBN - g.t_begin;  // q0a < S for every item
    g.nt1 = g.q0b < S ? (g.ke1 + kBN - 1) / kBN - g.t_begin : 0;
    g.n_max = max(g.nt0, g.nt1);
    return g;
}

// Work-item mailbox slot (ints): the producer computes an item's geometry once and
// publishes it; the MMA warp and the softmax groups read the fields they use from shared
// memory, so no role keeps the geometry's inputs or the whole geometry in registers.
constexpr int kSlotValid = 0;  // 0: no more items
constexpr int kSlotB = 1, kSlotH = 2, kSlotQ0a = 3, kSlotQ0b = 4;
constexpr int kSlotKb0 = 5, kSlotKb1 = 6, kSlotKe0 = 7, kSlotKe1 = 8;
constexpr int kSlotTBegin = 9, kSlotNt0 = 10, kSlotNt1 = 11, kSlotUniform = 12;
// key tiles starting in [kSlotIntLo_t, kSlotIntHi_t] are interior for every row of tile t
constexpr int kSlotIntLo0 = 13, kSlotIntHi0 = 14, kSlotIntLo1 = 15, kSlotIntHi1 = 16;
// tile B's batch, head and uniform flag (differ from tile A's for packed items)
constexpr int kSlotB1 = 17, kSlotH1 = 18, kSlotUniform1 = 19;
constexpr int kSlotInts = 24;

__device__ __forceinline__ void publish_item(volatile int* ms, bool valid, const ItemGeo& g, int causal, int window) {
    ms[kSlotValid] = valid ? 1 : 0;
    if (!valid) return;
    ms[kSlotB] = g.b;
    ms[kSlotH] = g.h;
    ms[kSlotQ0a] = g.q0a;
    ms[kSlotQ0b] = g.q0b;
    ms[kSlotKb0] = g.kb0;
    ms[kSlotKb1] = g.kb1;
    ms[kSlotKe0] = g.ke0;
    ms[kSlotKe1] = g.ke1;
    ms[kSlotTBegin] = g.t_begin;
    ms[kSlotNt0] = g.nt0;
    ms[kSlotNt1] = g.nt1;
    ms[kSlotUniform] = g.uniform ? 1 : 0;
    ms[kSlotB1] = g.b1;
    ms[kSlotH1] = g.h1;
    ms[kSlotUniform1] = g.uniform1 ? 1 : 0;
    // a key tile [n0, n0 + 128) needs no per-element mask when it lies inside the key range,
    // wholly at or below the diagonal of the tile's first row and wholly inside the window of
    // its last row
    for (int t = 0; t < 2; ++t) {
        const int q_first = t ? g.q0b : g.q0a, q_last = q_first + kBM - 1;
        int lo = t ? g.kb1 : g.kb0, hi = (t ? g.ke1 : g.ke0) - kBN;
        if (causal) {
            hi = min(hi, q_first - kBN + 1);
            if (window > 0) lo = max(lo, q_last - window + 1);
        }
        if (t ? g.uniform1 : g.uniform) {
            lo = 1;
            hi = 0;
        }
        ms[t ? kSlotIntLo1 : kSlotIntLo0] = lo;
        ms[t ? kSlotIntHi1 : kSlotIntHi0] = hi;
    }
}

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
    // barriers, 8 bytes each.  Every phase count runs on across the CTA's work items.
    // Q tile qs = (item % kQBuf) * kTiles + t: loaded per item, released by the commit after the
    // item's last QK of tile t
    auto bQfull = [&](int qs) { return bar0 + 8u * (0 + qs); };
    auto bQempty = [&](int qs) { return bar0 + 8u * (4 + qs); };
    // Ring item i of a work item holds K(i) (i < n_max) and V(i-1) (i >= 1): step j reads
    // V(j) and then K(j+1), both last in the same step, so one stage, one full and one
    // empty barrier serve the pair (one wait and one release per step on the MMA thread).
    // The ring's item count g runs across work items: K and V of ring item g sit in stage
    // g % ST of the K and V rings.
    auto bKVfull = [&](int s) { return bar0 + 8u * (8 + s); };
    auto bKVempty = [&](int s) { return bar0 + 8u * (8 + ST + s); };
    auto bSfull = [&](int t) { return bar0 + 8u * (8 + 2 * ST + t); };
    auto bPfull = [&](int t) { return bar0 + 8u * (10 + 2 * ST + t); };
    auto bOdone = [&](int t) { return bar0 + 8u * (12 + 2 * ST + t); };
    // work-item mailbox: the producer publishes item k in slot k % 2; the MMA warp and the
    // eight softmax warps each release it once read
    auto bItemFull = [&](int s) { return bar0 + 8u * (14 + 2 * ST + s); };
    auto bItemEmpty = [&](int s) { return bar0 + 8u * (16 + 2 * ST + s); };
    const uint32_t bDrain = bar0 + 8u * (18 + 2 * ST);
    // in-kernel preparation: a staged tile is an MMA operand once the preparing warps release it
    auto bQready = [&](int qs) { return bar0 + 8u * (19 + 2 * ST + qs); };
    auto bKVready = [&](int s) { return bar0 + 8u * (23 + 2 * ST + s); };
    static_assert(8 * (23 + 3 * ST) <= 256, "barriers fit below the TMEM address word");
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(base_ptr + Gm::oBar + 256);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(base_ptr + Gm::oBar + 264);
    // mailbox slot s: kSlotInts ints at oBar + 288 + 4 kSlotInts s, a work item's geometry
    volatile int* slots = reinterpret_cast<volatile int*>(base_ptr + Gm::oBar + 288);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // parameter fields copied to registers once: the asm statements below clobber
    // memory, which would otherwise force a reload through a generic pointer at
    // every use (a 25x slower masked softmax tile when the mask test read them)
    const int n_items = p.n_items;
    int* const status = p.status;
    // launched with programmatic serialisation: the set-up below (barriers, TMEM) overlaps the
    // kernel ahead; griddepcontrol.wait follows it, before any global read or write
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (tid == 0) {
        for (int qs = 0; qs < Gm::kQTiles; ++qs) {
            mbar_init(bQfull(qs), 1);
            mbar_init(bQempty(qs), 1);
            mbar_init(bQready(qs), 2);
        }
        for (int t = 0; t < 2; ++t) {
            mbar_init(bSfull(t), 1);
            mbar_init(bPfull(t), 128);
            mbar_init(bOdone(t), 1);
            mbar_init(bItemFull(t), 1);
            // readers of a mailbox slot: the MMA warp, the eight softmax warps (+ the two preparing warps)
            mbar_init(bItemEmpty(t), p.xform ? 11 : 9);
        }
        for (int s = 0; s < ST; ++s) {
            mbar_init(bKVfull(s), 1);
            mbar_init(bKVempty(s), 1);
            mbar_init(bKVready(s), 2);
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
    asm volatile("griddepcontrol.wait;" ::: "memory");

    if (warp >= 8) {
      asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(RegSplit<D>::kControl));
      if (warp == 8) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const int S = p.S, causal = p.causal, window = p.window, Hq = p.Hq, G = p.G;
            const int32_t* const key_len = p.key_len;
            int* const sched = p.sched;
            const int n_pairs = (S + Gm::kTiles * kBM - 1) / (Gm::kTiles * kBM);
            const int packed = Gm::kTiles == 2 ? p.packed : 0, n_heads_total = p.B * Hq;
            int k = 0;        // work items published
            int g = 0;        // ring items issued
            int q_items = 0;  // work items whose Q tiles were issued
            int skip_g = -1;  // test hook: the ring item of work item 0 whose copy is never issued
            // Packed items (uniform cost) are assigned statically, CTA c taking items c, c + grid, ...,
            // and their geometry (key-length reads, microseconds under load) is computed before the wait
            // for a free mailbox slot, so short items follow one another closely.  Other items come
            // from the counter when the CTA is ready for one, so that no CTA holds an item it has not
            // started while another has none.
            int w_static = (int)blockIdx.x;
            for (;; ++k) {
                const int slot = k & 1;
                int w;
                ItemGeo it;
                if (packed) {
                    w = w_static;
                    w_static += (int)gridDim.x;
                    it = item_geo(w < n_items ? w : 0, n_pairs, Gm::kTiles, Hq, S, causal, window, key_len, packed,
                                  n_heads_total);
                    // slot k % 2 is free once every reader of item k-2 is done with it
                    if (k >= 2 && !mbar_wait(bItemEmpty(slot), ((k >> 1) - 1) & 1, abort_flag, status)) break;
                } else {
                    if (k >= 2 && !mbar_wait(bItemEmpty(slot), ((k >> 1) - 1) & 1, abort_flag, status)) break;
                    w = atomicAdd(sched, 1);
                    it = item_geo(w < n_items ? w : 0, n_pairs, Gm::kTiles, Hq, S, causal, window, key_len, packed,
                                  n_heads_total);
                }
                if (p.stall && w == 0) skip_g = g + 1;
                publish_item(slots + kSlotInts * slot, w < n_items, it, causal, window);
                mbar_arrive(bItemFull(slot));  // release: the slot's values are visible to the waiters
                if (w >= n_items) break;
                const int kvh = it.h / G, kvh1 = it.h1 / G;
                bool ok = true;
                const int qb = k % Gm::kQBuf;
                for (int t = 0; t < Gm::kTiles && ok; ++t) {
                    const int qs = qb * Gm::kTiles + t;
                    if (k >= Gm::kQBuf && !mbar_wait(bQempty(qs), ((k / Gm::kQBuf) - 1) & 1, abort_flag, status)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(bQfull(qs), Gm::kTileBytes);
                    for (int pn = 0; pn < NP; ++pn)
                        tma_load_4d(sQ + qs * Gm::kTileBytes + pn * Gm::kPanelBytes, &tmQ, bQfull(qs),
                                    Gm::kPanelElems * pn,
                                    t ? it.h1 : it.h, t ? it.q0b : it.q0a, t ? it.b1 : it.b);
                }
                if (!ok) break;
                q_items = k + 1;
                // ring items 0..n_max of this work item (n_max >= 1), each into its stage after
                // the stage's previous ring item was released
                for (int i = 0; i <= it.n_max; ++i) {
                    const int st = g % ST;
                    if (g >= ST && !mbar_wait(bKVempty(st), ((g / ST) - 1) & 1, abort_flag, status)) {
                        ok = false;
                        break;
                    }
                    if (g == skip_g) {  // nothing is issued for it: its consumer's wait runs out
                        ++g;
                        continue;
                    }
                    if (packed) {
                        // ring item 0: K of tile A's head in the K slot, K of tile B's in the V slot;
                        // ring item 1: V of tile A's head in the V slot, V of tile B's in the K slot
                        const bool two = it.nt1 > 0;
                        mbar_expect_tx(bKVfull(st), two ? 2u * Gm::kTxTile : Gm::kTxTile);
                        const CUtensorMap* const m = i == 0 ? &tmK : &tmV;
                        const uint32_t dst_a = (i == 0 ? sK : sV) + st * Gm::kTileBytes;
                        const uint32_t dst_b = (i == 0 ? sV : sK) + st * Gm::kTileBytes;
                        for (int pn = 0; pn < NP; ++pn) {
                            tma_load_4d(dst_a + pn * Gm::kPanelBytes, m, bKVfull(st), Gm::kPanelElems * pn, kvh, 0,
                                        it.b);
                            if (two)
                                tma_load_4d(dst_b + pn * Gm::kPanelBytes, m, bKVfull(st), Gm::kPanelElems * pn, kvh1,
                                            0, it.b1);
                        }
                        ++g;
                        continue;
                    }
                    const bool has_k = i < it.n_max, has_v = i >= 1;
                    mbar_expect_tx(bKVfull(st), (has_k ? Gm::kTxTile : 0u) + (has_v ? Gm::kTxTile : 0u));
                    if (has_k)
                        for (int pn = 0; pn < NP; ++pn)
                            tma_load_4d(sK + st * Gm::kTileBytes + pn * Gm::kPanelBytes, &tmK, bKVfull(st),
                                        Gm::kPanelElems * pn, kvh, (it.t_begin + i) * kBN, it.b);
                    if (has_v)
                        for (int pn = 0; pn < NP; ++pn)
                            tma_load_4d(sV + st * Gm::kTileBytes + pn * Gm::kPanelBytes, &tmV, bKVfull(st),
                                        Gm::kPanelElems * pn, kvh, (it.t_begin + i - 1) * kBN, it.b);
                    ++g;
                }
                if (!ok) break;
            }
            // every copy this thread issued lands before the CTA may exit
            for (int j = q_items > Gm::kQBuf ? q_items - Gm::kQBuf : 0; j < q_items; ++j)
                for (int t = 0; t < Gm::kTiles; ++t)
                    mbar_drain(bQfull((j % Gm::kQBuf) * Gm::kTiles + t), (j / Gm::kQBuf) & 1);
            for (int i = (g > ST ? g - ST : 0); i < g; ++i)
                if (i != skip_g) mbar_drain(bKVfull(i % ST), (i / ST) & 1);
        }
    } else if (warp >= 10) {
        // ------------------------------------------------------------ operand conversion
        // Warps 10-11 follow the producer's sequence of work items and ring items: each staged bf16
        // tile is converted to fp16 in place, made visible to the tensor core's (async) proxy, and
        // released to the MMA warp.
        if (p.xform != 0) {
            const int tx = tid - 320;  // 0..63
            const int S = p.S, xform = p.xform;
            const bool packed = Gm::kTiles == 2 && p.packed != 0;
            float mx = 0.f;
            int g = 0;
            bool ok = true;
            auto release = [&](uint32_t bar) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(bar);
            };
            for (int k = 0; ok; ++k) {
                const int slot = k & 1;
                if (!__all_sync(0xffffffffu, mbar_wait(bItemFull(slot), (k >> 1) & 1, abort_flag, status))) break;
                volatile int* const ms = slots + kSlotInts * slot;
                if (!ms[kSlotValid]) break;
                const int nt1 = ms[kSlotNt1], n_max = max(ms[kSlotNt0], nt1), t_begin = ms[kSlotTBegin];
                const int qb = k % Gm::kQBuf, qpar = (k / Gm::kQBuf) & 1;
                for (int t = 0; t < Gm::kTiles && ok; ++t) {
                    const int qs = qb * Gm::kTiles + t;
                    if (!__all_sync(0xffffffffu, mbar_wait(bQfull(qs), qpar, abort_flag, status))) {
                        ok = false;
                        break;
                    }
                    if (xform & kXformQ) {
                        const int q0 = ms[t ? kSlotQ0b : kSlotQ0a];
                        if (q0 < S && (t == 0 || nt1 > 0))
                            mx = fmaxf(mx, xform_tile<D>(base_ptr + Gm::oQ + qs * Gm::kTileBytes, tx, S - q0));
                    }
                    release(bQready(qs));
                }
                for (int i = 0; i <= n_max && ok; ++i) {
                    const int st = (g + i) % ST;
                    if (!__all_sync(0xffffffffu, mbar_wait(bKVfull(st), ((g + i) / ST) & 1, abort_flag, status))) {
                        ok = false;
                        break;
                    }
                    unsigned char* const ks = base_ptr + Gm::oK + st * Gm::kTileBytes;
                    unsigned char* const vs = base_ptr + Gm::oV + st * Gm::kTileBytes;
                    if (packed) {
                        // ring item 0: K tiles in both slots; ring item 1: V tiles in both
                        if (xform & (i == 0 ? kXformK : kXformV)) {
                            mx = fmaxf(mx, xform_tile<D>(i == 0 ? ks : vs, tx, S));
                            if (nt1 > 0) mx = fmaxf(mx, xform_tile<D>(i == 0 ? vs : ks, tx, S));
                        }
                    } else {
                        if ((xform & kXformK) && i < n_max) mx = fmaxf(mx, xform_tile<D>(ks, tx, S - (t_begin + i) * kBN));
                        if ((xform & kXformV) && i >= 1)
                            mx = fmaxf(mx, xform_tile<D>(vs, tx, S - (t_begin + i - 1) * kBN));
                    }
                    release(bKVready(st));
                }
                g += n_max + 1;
                __syncwarp();
                if (lane == 0) mbar_arrive(bItemEmpty(slot));  // done with the slot
            }
            // a value beyond the fp16 operand range (|x| > 65504 rounds to infinity): status bit 2
            if (__any_sync(0xffffffffu, mx >= 65520.f) && lane == 0) atomicOr(status, 4);
        }
    } else if (warp == 9) {
        // ------------------------------------------------------------ MMA issuer
        // The whole warp runs this loop with warp-uniform waits (vote.all); lane 0
        // issues the MMAs and commits.
        {
            const uint32_t ln = (uint32_t)lane;
            // fp16 operands (attn_tcgen05_supported), fp32 accumulators
            constexpr uint32_t idq = make_idesc(0, kBM, kBN, 0, 0);
            constexpr uint32_t idp = make_idesc(0, kBM, D, 0, 1);
            int g = 0;                // ring items of earlier work items
            int item_ready = -1;      // highest ring item whose full wait was observed
            int cp0 = 0, cp1 = 0;     // P hand-overs consumed per tile
            bool ok = true;
            // tiles prepared in kernel are operands once the preparing warps release them
            const bool kv_prep = (p.xform & (kXformK | kXformV)) != 0, q_prep = (p.xform & kXformQ) != 0;
            auto wait_item = [&](int i) -> bool {
                if (item_ready >= i) return true;
                if (!__all_sync(0xffffffffu, mbar_wait(kv_prep ? bKVready(i % ST) : bKVfull(i % ST), (i / ST) & 1,
                                                       abort_flag, status)))
                    return false;
                tc_fence_after();
                item_ready = i;
                return true;
            };
            // descriptors of each buffer's start: a K step, tile or stage offset only moves the
            // 14-bit start-address field (addr >> 4) of the low word, and every offset here stays inside it
            constexpr uint32_t kSbo = 8 * Gm::kRowBytes;  // 8-row core-matrix groups
            const uint64_t dQ = smem_desc(sQ, 16, kSbo, Gm::kLayout), dK = smem_desc(sK, 16, kSbo, Gm::kLayout);
            const uint64_t dV = smem_desc(sV, Gm::kPanelBytes, kSbo, Gm::kLayout);
            const uint32_t q_lo = (uint32_t)dQ, v_lo = (uint32_t)dV;
            const uint32_t qk_hi = (uint32_t)(dQ >> 32), v_hi = (uint32_t)(dV >> 32);  // dK's high word is dQ's
            // packed items: tile B's K sits in the V slot (read K-major) and its V in the K slot (read MN-major)
            const bool packed = Gm::kTiles == 2 && p.packed != 0;
            const uint32_t k_lo_b = packed ? (uint32_t)smem_desc(sV, 16, kSbo, Gm::kLayout) : (uint32_t)dK;
            const uint32_t v_lo_b = packed ? (uint32_t)smem_desc(sK, Gm::kPanelBytes, kSbo, Gm::kLayout) : v_lo;
            const uint32_t k_lo = (uint32_t)dK;
            // S_t = Q_t K^T with K in ring stage st
            int qb = 0;  // Q buffer of the current item
            auto issue_qk = [&](int t, int st) {
                const uint32_t a0 = q_lo + (uint32_t)((qb * Gm::kTiles + t) * Gm::kTileBytes >> 4);
                const uint32_t b0 = (t ? k_lo_b : k_lo) + (uint32_t)(st * Gm::kTileBytes >> 4);
                const uint32_t d = tmem + 128u * t;
#pragma unroll
                for (int ks = 0; ks < D / 16; ++ks) {
                    constexpr int kSteps = Gm::kPanelElems / 16;  // 16-element K steps per panel
                    const uint32_t koff =
                        ((uint32_t)(ks / kSteps) * Gm::kPanelBytes + (uint32_t)(ks % kSteps) * 32u) >> 4;
                    if (ks == 0) umma_ss_w<0>(ln, d, a0, qk_hi, b0, qk_hi, idq);
                    else umma_ss_w<1>(ln, d, a0 + koff, qk_hi, b0 + koff, qk_hi, idq);
                }
                umma_commit_w(ln, bSfull(t));
            };
            // O_t (+)= P_t V with V in ring stage st, MN-major: 8-key atoms 8 panel rows apart (SBO),
            // panels kPanelBytes apart (LBO); a 16-key step moves 16 panel rows
            auto issue_pv = [&](int t, int st, uint32_t acc) {
                const uint32_t b0 = (t ? v_lo_b : v_lo) + (uint32_t)(st * Gm::kTileBytes >> 4);
                const uint32_t d = tmem + Gm::kOcol + 128u * t, a = tmem + 128u * t;
                umma_ts_w<-1>(ln, d, a, b0, v_hi, idp, acc);
#pragma unroll
                for (int kk = 1; kk < kBN / 16; ++kk)
                    umma_ts_w<1>(ln, d, a + kk * 8u, b0 + kk * (uint32_t)Gm::kRowBytes, v_hi, idp);
            };
            for (int k = 0; ok; ++k) {
                const int slot = k & 1;
                if (!__all_sync(0xffffffffu, mbar_wait(bItemFull(slot), (k >> 1) & 1, abort_flag, status))) {
                    ok = false;
                    break;
                }
                volatile int* const ms = slots + kSlotInts * slot;
                if (!ms[kSlotValid]) break;
                const int nt0 = ms[kSlotNt0], nt1 = ms[kSlotNt1], n_max = max(nt0, nt1);
                qb = k % Gm::kQBuf;
                const int qpar = (k / Gm::kQBuf) & 1, qs0 = qb * Gm::kTiles;
                ok = __all_sync(0xffffffffu,
                                mbar_wait(q_prep ? bQready(qs0) : bQfull(qs0), qpar, abort_flag, status) &&
                                    (Gm::kTiles == 1 ||
                                     mbar_wait(q_prep ? bQready(qs0 + 1) : bQfull(qs0 + 1), qpar, abort_flag, status)));
                if (ok) ok = wait_item(g);
                if (!ok) break;
                // S_t(0); a tile with at most one key tile reads Q_t for the last time here
                if (nt0 > 0) issue_qk(0, g % ST);
                if (nt0 <= 1) umma_commit_w(ln, bQempty(qs0));
                if (nt1 > 0) issue_qk(1, g % ST);
                if (Gm::kTiles == 2 && nt1 <= 1) umma_commit_w(ln, bQempty(qs0 + 1));
                umma_commit_w(ln, bKVempty(g % ST));  // ring item 0 (K(0)) read by both tiles
                for (int j = 0; j < n_max && ok; ++j) {
                    const int st = (g + j + 1) % ST;  // ring item j+1: V(j), K(j+1)
                    // the tile whose part of this step reads ring item j+1 last: tile B whenever it
                    // takes part (its rows follow tile A's, so nt0 <= nt1 unless tile B is empty)
                    const int rel = j < nt1 ? 1 : 0;
                    // rolled over the two tiles: unrolled, each tile's per-step descriptor words
                    // would be loop-invariant and hoisted into (spilled) registers
#pragma unroll 1
                    for (int t = 0; t < 2 && ok; ++t) {
                        const int ntt = t ? nt1 : nt0;
                        if (j >= ntt) continue;
                        const int cp = t ? cp1++ : cp0++;
                        if (!__all_sync(0xffffffffu, mbar_wait(bPfull(t), cp & 1, abort_flag, status))) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        if (!wait_item(g + j + 1)) {
                            ok = false;
                            break;
                        }
                        issue_pv(t, st, j > 0 ? 1u : 0u);
                        // O_t is complete after its last PV; earlier PVs need no signal of their own:
                        // S_t(j+1) is committed after PV_t(j), and a commit tracks every earlier MMA
                        if (j + 1 == ntt) umma_commit_w(ln, bOdone(t));
                        if (j + 1 < ntt) {
                            issue_qk(t, st);
                            if (j + 2 == ntt) umma_commit_w(ln, bQempty(qs0 + t));  // the item's last QK of tile t
                        }
                        if (t == rel) umma_commit_w(ln, bKVempty(st));
                    }
                }
                g += n_max + 1;
                __syncwarp();
                if (lane == 0) mbar_arrive(bItemEmpty(slot));  // done with the slot
            }
            // all MMAs lane 0 issued are complete before TMEM is released
            umma_commit_w(ln, bDrain);
            mbar_drain(bDrain, 0);
        }
      }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(RegSplit<D>::kSoftmax));
        // ------------------------------------------------------------ softmax groups
        const int t = warp >> 2;       // 0: tile A, 1: tile B
        const int row = tid & 127;     // TMEM lane within the group
        const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        const uint32_t s_addr = lane_base + (t ? 128u : 0u);
        const uint32_t o_addr = lane_base + Gm::kOcol + (t ? 128u : 0u);
        const int S = p.S, causal = p.causal, window = p.window;
        const float* const mask = kAdditive ? p.mask : nullptr;
        const float scale = p.scale;
        const float sl2 = p.scale_log2;
        int cs = 0, co = 0;  // S and O hand-overs consumed
        bool ok = true;
        for (int k = 0; ok; ++k) {
            const int slot = k & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(bItemFull(slot), (k >> 1) & 1, abort_flag, status))) {
                ok = false;
                break;
            }
            volatile int* const ms = slots + kSlotInts * slot;
            if (!ms[kSlotValid]) break;
            // this group's tile: key tiles, visible keys per row, interior key-tile starts
            const int my_nt = ms[t ? kSlotNt1 : kSlotNt0];
            const int q = ms[t ? kSlotQ0b : kSlotQ0a] + row;
            const int n_base = ms[kSlotTBegin] * kBN;
            // keys this row sees: [row_lo, row_hi); a uniform row (no valid key) weights all keys equally
            int row_lo = ms[t ? kSlotKb1 : kSlotKb0], row_hi = ms[t ? kSlotKe1 : kSlotKe0];
            if (causal) {
                row_hi = min(row_hi, q + 1);
                if (window > 0) row_lo = max(row_lo, q - window + 1);
            }
            // key tiles starting in [int_lo, int_hi] need no per-element mask
            const int int_lo = ms[t ? kSlotIntLo1 : kSlotIntLo0], int_hi = ms[t ? kSlotIntHi1 : kSlotIntHi0];
            const bool uniform = ms[t ? kSlotUniform1 : kSlotUniform] != 0;
            const float* const mrow0 = kAdditive ? mask + (int64_t)ms[t ? kSlotB1 : kSlotB] * S : nullptr;
            const float edge_mult = uniform ? 0.f : sl2;
            const bool additive = kAdditive && !uniform;
            float m_run = -INFINITY, l_run = 0.f;
            for (int j = 0; j < my_nt; ++j) {
                if (!__all_sync(0xffffffffu, mbar_wait(bSfull(t), cs & 1, abort_flag, status))) {
                    ok = false;
                    break;
                }
                ++cs;
                tc_fence_after();
                const int n0 = n_base + j * kBN;
                // a tile needs per-element masks when it touches the diagonal, the window start or the key end
                const bool edge = kAdditive || n0 < int_lo || n0 > int_hi;
                // the whole score row in registers: one TMEM read serves both passes
                uint32_t r[kBN];
#pragma unroll
                for (int c = 0; c < kBN / 32; ++c) tmem_ld32(s_addr + 32 * c, r + 32 * c);
                tmem_wait_ld();
                // scaled: the row holds log2-domain scores (else raw ones, scaled in the max and exponent)
                bool scaled = false;
                if (edge) {
                    // masked tiles: -inf outside the row's keys
                    const int lo = row_lo - n0, hi = row_hi - n0;
                    scaled = true;
                    if (!additive && !uniform && lo <= 0) {
                        // only an upper bound (key padding, the causal diagonal): one compare per score,
                        // raw scores kept like an interior tile's
                        scaled = false;
#pragma unroll
                        for (int i = 0; i < kBN; ++i) r[i] = i < hi ? r[i] : __float_as_uint(-INFINITY);
                    } else if (additive) {
                        const float* mrow = mrow0 + n0;
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
                if (!scaled) mx *= sl2;
                // lazy rescale: move the reference maximum only when it grew by > threshold;
                // O is multiplied after pass 2, when the score row no longer holds registers
                const bool need = mx > m_run + kRescaleThreshold;
                const bool rescale = __any_sync(0xffffffffu, need);
                float alpha = 1.f;
                if (rescale) {
                    const float m_new = need ? mx : m_run;
                    alpha = (m_run == -INFINITY) ? 0.f : fast_exp2(m_run - m_new);
                    l_run *= alpha;
                    m_run = m_new;
                }
                const float mb = m_run == -INFINITY ? 0.f : m_run;
                // pass 2: P = 2^(s - m) as fp16 pairs over the first 64 S columns, row sum
                const float mul = scaled ? 1.f : sl2;
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
                // O_t holds PV(j-1) complete: S_t(j), waited for above, was committed after it;
                // PV(j) adds to O only after the hand-over below
                if (rescale && j > 0) {
#pragma unroll 1
                    for (int c = 0; c < D / 32; ++c) {
                        uint32_t o[32];
                        tmem_ld32(o_addr + 32 * c, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_st32(o_addr + 32 * c, o);
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(bPfull(t));
            }
            // epilogue: O / l for rows inside the sequence.  O_t is read out (tcgen05.ld, waited
            // for) before this group hands over the next item's first P, the point after which
            // that item's first PV overwrites O_t.
            if (!ok) break;
            if (my_nt > 0) {
                if (!__all_sync(0xffffffffu, mbar_wait(bOdone(t), co & 1, abort_flag, status))) {
                    ok = false;
                    break;
                }
                ++co;
                tc_fence_after();
                const float inv = 1.f / l_run;
#pragma unroll
                for (int c = 0; c < D / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld32(o_addr + 32 * c, r);
                    tmem_wait_ld();
                    if (q < S) {
                        const int64_t off = ms[t ? kSlotB1 : kSlotB] * p.o_sb + (int64_t)q * p.o_ss +
                                            ms[t ? kSlotH1 : kSlotH] * p.o_sh + 32 * c;
#pragma unroll
                        for (int i = 0; i < 32; i += 8) {
                            float v[8];
#pragma unroll
                            for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(r[i + e]) * inv;
                            store8(p.out, off + i, v, p.out_dtype);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(bItemEmpty(slot));  // done with the slot
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    // the last CTA to finish resets the work-item counters and the abort word for the next
    // launch: every CTA has fetched its last item and passed its last wait (its roles are past
    // the barrier above) before it counts
    if (tid == 0) {
        int* const sched = p.sched;
        __threadfence();
        if (atomicAdd(sched + 1, 1) == (int)gridDim.x - 1) {
            atomicExch(sched, 0);
            atomicExch(sched + 1, 0);
            atomicExch(status + kStatusAbortWord, 0);
        }
    }
}

// ---------------------------------------------------------------- host side
// [B][S][H][D] tensor (element strides sb, ss, sh; d contiguous), box 64 x 1 x 128 x 1.
bool make_map(CUtensorMap* m, const void* ptr, int fmt, int B, int S, int H, int D, int64_t sb, int64_t ss,
              int64_t sh) {
    EncodeFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)S, (cuuint64_t)B};
    const cuuint64_t strides[3] = {(cuuint64_t)sh * 2, (cuuint64_t)ss * 2, (cuuint64_t)sb * 2};
    // the kernel's panels (TcGeo<D>): 32 elements with the 64-byte swizzle at D = 96, else 64 with the 128-byte one
    const bool narrow = D == 96;
    const cuuint32_t box[4] = {narrow ? 32u : 64u, 1, 128, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = fn(m, fmt ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                          const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          narrow ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
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

// Bidirectional sequences of at most one tile with two query tiles per item (head dim <= 128)
// pack two (batch, head) pairs into each item.
bool packed_items(const AttnParams& a) { return !a.causal && a.S <= kBM && a.D <= 128; }

// query-tile pairs x heads x batch, or (packed) pairs of (batch, head)
int64_t work_items(const AttnParams& a) {
    if (packed_items(a)) return ((int64_t)a.Hq * a.B + 1) / 2;
    const int rows = (a.D <= 128 ? 2 : 1) * kBM;  // TcGeo<D>::kTiles query tiles per item
    return (int64_t)((a.S + rows - 1) / rows) * a.Hq * a.B;
}

template <int D>
cudaError_t launch_impl(const AttnParams& a, int* status, cudaStream_t stream, bool stall) {
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
    // persistent: one CTA per SM (each holds all of TMEM), work items from the counter
    p.sched = status + kStatusSchedWord;
    p.n_items = (int)work_items(a);
    p.stall = stall ? 1 : 0;
    p.packed = packed_items(a) ? 1 : 0;
    p.xform = a.xform;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
                                                  cudaSuccess || sms <= 0)
        return cudaErrorInvalidDevice;
    const dim3 grid((unsigned)std::min(p.n_items, sms));
    // programmatic stream serialisation: the CTAs may be placed, and set up their barriers and
    // TMEM, while the kernel ahead finishes; they wait for it before touching global memory
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kThreadsTc);
    cfg.dynamicSmemBytes = smem_request<D>();
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (additive) return cudaLaunchKernelEx(&cfg, attn_tcgen05_kernel<D, true>, mq, mk, mv, p);
    return cudaLaunchKernelEx(&cfg, attn_tcgen05_kernel<D, false>, mq, mk, mv, p);
}

}  // namespace

bool attn_tcgen05_supported(const AttnParams& p) {
    // fp16 operands only: P goes to TMEM as fp16 and both MMA operands share one type; bf16 inputs
    // are converted by the kernel itself when it prepares all three tensors (xform 7)
    if (p.in_dtype != kF16 && !(p.in_dtype == kBF16 && p.xform == 7)) return false;
    if (p.in_dtype == kF16 && p.xform != 0) return false;
    if (!(p.D == 32 || p.D == 64 || p.D == 96 || p.D == 128 || p.D == 256)) return false;
    const int64_t strides[] = {p.q_sb, p.q_ss, p.q_sh, p.k_sb, p.k_ss, p.k_sh};
    for (int64_t s : strides)
        if (s % 8 != 0 || s <= 0) return false;
    const uintptr_t ptrs[] = {(uintptr_t)p.q, (uintptr_t)p.k, (uintptr_t)p.v, (uintptr_t)p.o};
    for (uintptr_t x : ptrs)
        if (x % 16 != 0) return false;
    // the work-item counter reaches items + grid within int32
    if (p.Hq > 65535 || p.B > 65535 || work_items(p) > INT32_MAX / 2 || encode_fn() == nullptr) return false;
    const cudaError_t ready = p.D == 32    ? kernel_ready_for<32>(p)
                              : p.D == 64  ? kernel_ready_for<64>(p)
                              : p.D == 96  ? kernel_ready_for<96>(p)
                              : p.D == 128 ? kernel_ready_for<128>(p)
                                           : kernel_ready_for<256>(p);
    return ready == cudaSuccess;
}

cudaError_t launch_attn_tcgen05(const AttnParams& p, int* status, cudaStream_t stream, bool stall) {
    switch (p.D) {
        case 32: return launch_impl<32>(p, status, stream, stall);
        case 64: return launch_impl<64>(p, status, stream, stall);
        case 96: return launch_impl<96>(p, status, stream, stall);
        case 128: return launch_impl<128>(p, status, stream, stall);
        case 256: return launch_impl<256>(p, status, stream, stall);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace b2a
