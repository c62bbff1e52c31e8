// decode_tc.cu -- split-KV single-token decode for fp16 / bf16 KV caches.
//
// One persistent launch per decode step (one CTA slot per resident CTA).
// Each CTA
//   1. plans from the device-resident ctx_lens: the visible keys of every
//      unit (sequence, kv head, head group of 8) form one key stream, and CTA
//      c owns the contiguous range [c*R, (c+1)*R) of it (stream-K split:
//      balanced to one key whatever the length mix);
//   2. walks the pieces of units inside its range.  Per piece it
//        - streams K and V tiles of 64 keys with 16-byte cp.async (3-4 stage
//          ring, padded rows so ldmatrix is bank-conflict free),
//        - builds the item's q rows in shared memory: optional zero-centred
//          RMS QK-norm and RoPE at position L (angles in double), and for
//          the chunk that ends at L the new key/value row, which it writes
//          to the cache and patches into its own tile (no other item reads
//          row L, so the append needs no grid-wide ordering),
//        - computes S^T = K Q^T and O^T += V^T P^T with m16n8k16 warp MMAs:
//          keys are the M dimension (16 per warp), the G <= 8 query heads of
//          a kv head the N = 8 dimension, so one K/V byte feeds every head;
//          online softmax in fp32 (base-2, one exp2 per key and head);
//        - merges its four warps and either writes the output (whole units)
//          or a partial (m, l, O) slot (at most two per CTA: a unit cut at
//          the start and one cut at the end of its range); the last piece of
//          a unit to finish merges the slots with a log-sum-exp combine and
//          resets its counter.
// The arithmetic intensity is 4-7 flop/byte, so the kernel is bound by HBM;
// warp MMAs are used because they cut the issue count per key ~10x against
// fp32 FMAs + shuffles (G=7, D=64 would otherwise be issue-bound), not for
// FLOPs.
//
// Semantics follow Qwen2Runtime.processLayerDecode (INF/qwen/Qwen2Runtime.java:723-766),
// the HLSL decode contracts (WB/windows/QwenAttentionShaders.java:82-263,
// INF/gemma/Gemma3WarpFusedAttentionContextKernel.java:32-86) and the Gemma
// decode prologue (INF/gemma/Gemma3ReferenceForwardPass.java:124-142).
#include <math.h>

#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "internal.h"

namespace b2a {
namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kTile = 16 * kWarps;  // keys per pipeline stage
constexpr int kHeads = 8;           // query heads per unit (MMA N)

template <int D>
struct Geo {
    static constexpr int kRow = D + 8;  // padded smem row (elements): odd number of 16 B units
    static constexpr int kStages = D <= 64 ? 4 : 3;
    // Fixed cost of one piece (tile issue, q prologue, epilogue and merge) in keys of
    // streaming time, measured on B200 with in-kernel timers: ~6 us per piece against
    // ~0.6 us per 64-key tile at D = 64, relatively less at larger D.  The stream-K
    // split charges it to every unit, so CTAs that cross unit boundaries take fewer keys.
    static constexpr int kGapKeys = D <= 64 ? 640 : (D <= 128 ? 384 : 256);
    static_assert(kGapKeys <= kDecodeGapKeysMax, "host launch split assumes this bound");
    static constexpr int kStageElems = 2 * kTile * kRow;  // K tile then V tile
    static constexpr int kChunks = D / 8;                 // 16-byte chunks per cache row
    static constexpr size_t kPipeBytes = size_t(kStages) * kStageElems * 2;
    static constexpr size_t kQBytes = size_t(kHeads) * kRow * 2;
    static constexpr size_t kNewBytes = size_t(2) * D * 2;
    static constexpr size_t kVecBytes = size_t(kWarps) * D * 4;
    static constexpr size_t kCsBytes = size_t(D / 2) * 2 * sizeof(double);
    static constexpr size_t kPrefixBytes = size_t(kDecodeMaxBatchPerLaunch + 1) * 4;
    static constexpr size_t kMlBytes = size_t(kWarps) * kHeads * 2 * 4;
    static constexpr size_t kMergeBytes = size_t(kWarps) * kHeads * D * 4;  // aliases the pipe
    static_assert(kMergeBytes <= kPipeBytes, "merge scratch must fit in the pipeline buffers");
    // every region starts on a 16-byte boundary (misc is read as 8-byte words,
    // cs as doubles, the pipe and q rows by 16-byte cp.async / ldmatrix)
    static constexpr size_t a16(size_t x) { return (x + 15) / 16 * 16; }
    static constexpr size_t oQ = a16(kPipeBytes);
    static constexpr size_t oQlo = a16(oQ + kQBytes);  // low parts of q (bf16 caches only)
    static constexpr size_t oNew = a16(oQlo + kQBytes);
    static constexpr size_t oVec = a16(oNew + kNewBytes);
    static constexpr size_t oCs = a16(oVec + kVecBytes);
    static constexpr size_t oPrefix = a16(oCs + kCsBytes);
    // context length per sequence, cached by the plan for the piece loop where it fits
    // (every head dim but 256, whose pipeline fills shared memory)
    static constexpr size_t kLensBytes = size_t(kDecodeMaxBatchPerLaunch) * 4;
    static constexpr size_t oLens = a16(oPrefix + kPrefixBytes);
    static constexpr bool kLensCached = a16(oLens + kLensBytes) + kMlBytes + 64 <= 227 * 1024;
    static constexpr size_t oMl = kLensCached ? a16(oLens + kLensBytes) : oLens;
    static constexpr size_t oMisc = a16(oMl + kMlBytes);
    static constexpr size_t kTotal = oMisc + 64;
    static_assert(oMisc % 16 == 0 && oCs % 16 == 0 && oMl % 16 == 0, "aligned shared regions");
    static_assert(kTotal <= 227 * 1024, "shared memory budget");
};

__device__ __forceinline__ int ctx_len_of(const DecodeParams& p, int b) {
    return p.ctx_lens ? p.ctx_lens[b] : p.pos_scalar;
}
// Visible key range [first, L] of a sequence whose context length is L_in.
__device__ __forceinline__ bool seq_range_of(const DecodeParams& p, int L_in, int& L, int& first) {
    L = L_in;
    if (L < 0 || L >= p.max_seq) {
        L = 0;
        first = 0;
        return false;
    }
    if (p.first_explicit >= 0) first = min(p.first_explicit, L);
    else if (p.window > 0) first = max(0, L - p.window + 1);
    else first = 0;
    return true;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// One head vector's elements d = lane + 32 j as loaded (raw bits) and its optional
// projection bias, requested early and converted later by prep_finish.
template <int D>
struct HeadLoad {
    uint32_t raw[D / 32];
    float bias[D / 32];
};
template <int D>
__device__ __forceinline__ void head_load(HeadLoad<D>& h, const void* src, int64_t off, int dtype, const float* bias,
                                          int lane) {
#pragma unroll
    for (int j = 0; j < D / 32; ++j) {
        h.raw[j] = load_raw(src, off + lane + 32 * j, dtype);
        h.bias[j] = bias != nullptr ? __ldg(bias + lane + 32 * j) : 0.f;
    }
}

// Converts a loaded head vector, adds its bias, applies the optional QK-norm, and
// writes it (rotated when requested) as float into vec[0..D).  Whole warp; vec is
// warp-private.
template <int D>
__device__ __forceinline__ void prep_finish(const DecodeParams& p, const HeadLoad<D>& h, int dtype, bool has_bias,
                                            bool has_norm, const float (&norm_w)[D / 32], bool rope, const double* cs,
                                            float* vec, int lane) {
    double ss = 0.0;
    float x[D / 32];
#pragma unroll
    for (int j = 0; j < D / 32; ++j) {
        x[j] = raw_to_float(h.raw[j], dtype);
        if (has_bias) x[j] = __fadd_rn(x[j], h.bias[j]);  // projection bias, fp32
        ss += (double)x[j] * (double)x[j];
    }
    if (has_norm) {
        // Gemma3ReferenceMath.rmsNormZeroCentered: double sum of squares,
        // float rms, (float)(x*rms * (1 + w)) (INF/gemma/Gemma3ReferenceMath.java:32-40).
        ss = warp_sum_d(ss);
        const float rms = (float)(1.0 / sqrt(__dadd_rn(ss / (double)D, (double)p.norm_eps)));
#pragma unroll
        for (int j = 0; j < D / 32; ++j)
            x[j] = (float)__dmul_rn((double)__fmul_rn(x[j], rms), __dadd_rn(1.0, (double)norm_w[j]));
    }
#pragma unroll
    for (int j = 0; j < D / 32; ++j) vec[lane + 32 * j] = x[j];
    __syncwarp();
    if (rope) {
        constexpr int H = D / 2;
        float y0[(H + 31) / 32], y1[(H + 31) / 32];
#pragma unroll
        for (int j = 0; j < (H + 31) / 32; ++j) {
            const int i = lane + 32 * j;
            if (i < H) {
                const float a = vec[i], b = vec[i + H];
                const double c = cs[2 * i], s = cs[2 * i + 1];
                if (p.rope_mode == 2) {
                    // applyRopeHalf: double products, float result (INF/gemma/Gemma3ReferenceMath.java:76-81)
                    y0[j] = (float)__dsub_rn(__dmul_rn((double)a, c), __dmul_rn((double)b, s));
                    y1[j] = (float)__dadd_rn(__dmul_rn((double)b, c), __dmul_rn((double)a, s));
                } else {
                    // DecoderOnlyRotaryEmbedding.rotate: float cos/sin, float products
                    // (INF/decoderonly/DecoderOnlyRotaryEmbedding.java:61-67)
                    const float cf = (float)c, sf = (float)s;
                    y0[j] = __fsub_rn(__fmul_rn(a, cf), __fmul_rn(b, sf));
                    y1[j] = __fadd_rn(__fmul_rn(a, sf), __fmul_rn(b, cf));
                }
            }
        }
        __syncwarp();
#pragma unroll
        for (int j = 0; j < (H + 31) / 32; ++j) {
            const int i = lane + 32 * j;
            if (i < H) {
                vec[i] = y0[j];
                vec[i + H] = y1[j];
            }
        }
    }
    __syncwarp();
}

template <int D, typename T>
__global__ void __launch_bounds__(kThreads) decode_tc_kernel(const __grid_constant__ DecodeParams p) {
    using Gm = Geo<D>;
    constexpr int kRow = Gm::kRow;
    constexpr int kStages = Gm::kStages;
    extern __shared__ __align__(128) unsigned char smem[];
    T* pipe = reinterpret_cast<T*>(smem);
    T* q_s = reinterpret_cast<T*>(smem + Gm::oQ);
    T* qlo_s = reinterpret_cast<T*>(smem + Gm::oQlo);
    // bf16 operands carry 8 mantissa bits: q and P are split into hi + lo
    // bf16 parts and both are multiplied, which restores ~16-bit operand
    // precision at twice the (idle) tensor work.
    constexpr bool kSplit = std::is_same<T, __nv_bfloat16>::value;
    T* knew_s = reinterpret_cast<T*>(smem + Gm::oNew);
    T* vnew_s = knew_s + D;
    float* vec_all = reinterpret_cast<float*>(smem + Gm::oVec);
    double* cs_s = reinterpret_cast<double*>(smem + Gm::oCs);
    int* prefix = reinterpret_cast<int*>(smem + Gm::oPrefix);
    int* lens_s = reinterpret_cast<int*>(smem + Gm::oLens);  // valid when Gm::kLensCached
    float* ml_s = reinterpret_cast<float*>(smem + Gm::oMl);
    int* misc = reinterpret_cast<int*>(smem + Gm::oMisc);
    float* merge_s = reinterpret_cast<float*>(smem);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    float* vec = vec_all + warp * D;
    // a decode launched after this one with early start may be scheduled from now on; it
    // still waits for this grid's completion before it reads its inputs or writes
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    // ---------------------------------------------------------------- plan
    // Stream-K split: the visible keys of all units (sequence, kv head, head
    // group), each followed by kGapKeys keys that stand for its fixed per-piece
    // cost, form one key stream; CTA c owns the contiguous range
    // [c*R, (c+1)*R), R = ceil(total / gridDim.x).  Work is balanced to about a
    // tile, and a unit is cut only where CTA ranges cross its real keys; a range
    // that falls on a unit's gap does no work there.
    // prefix[b] = stream length of sequences < b, per unit (int32: the host keeps
    // each launch's total below 2^31).
    // Unit-aligned ranges instead: when every unit has the same length (a sliding-window
    // layer whose contexts all exceed the window) and there are at least as many units as
    // CTAs, CTA c takes whole units [c*U/G, (c+1)*U/G) -- no unit is cut, so no partial
    // slots and no merges -- unless the uneven unit counts would cost more than the two
    // pieces' allowance that stream-K charges.
    int n_min = 0, n_max = 0;
    {
        const int per = (p.B + kThreads - 1) / kThreads;
        const int b0 = min(p.B, tid * per), b1 = min(p.B, b0 + per);
        int run = 0, bad = 0, lmin = INT32_MAX, lmax = 0;
        for (int b = b0; b < b1; ++b) {
            const int L_in = ctx_len_of(p, b);
            if (Gm::kLensCached) lens_s[b] = L_in;
            int L, first;
            if (!seq_range_of(p, L_in, L, first)) bad = 1;
            run += L - first + 1 + Gm::kGapKeys;
            lmin = min(lmin, L - first + 1);
            lmax = max(lmax, L - first + 1);
        }
        lmin = __reduce_min_sync(0xffffffffu, lmin);
        lmax = __reduce_max_sync(0xffffffffu, lmax);
        if (lane == 0) {
            misc[4 + warp] = lmin;
            misc[12 + warp] = lmax;
        }
        if (bad && blockIdx.x == 0) atomicOr(p.status, 1);
        int incl = run;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        if (lane == 31) misc[warp] = incl;
        __syncthreads();
        int warp_off = 0;
        for (int w = 0; w < warp; ++w) warp_off += misc[w];
        int acc = warp_off + incl - run;
        for (int b = b0; b < b1; ++b) {
            prefix[b] = acc;
            int L, first;
            seq_range_of(p, Gm::kLensCached ? lens_s[b] : ctx_len_of(p, b), L, first);
            acc += L - first + 1 + Gm::kGapKeys;
        }
        if (tid == kThreads - 1) prefix[p.B] = warp_off + incl;
        __syncthreads();
        n_min = misc[4];
        n_max = misc[12];
        for (int w = 1; w < kWarps; ++w) {
            n_min = min(n_min, misc[4 + w]);
            n_max = max(n_max, misc[12 + w]);
        }
    }
    const int per_chunk = p.Hkv * p.n_hg;  // units per sequence
    const long long total = (long long)prefix[p.B] * per_chunk;
    const long long R = (total + gridDim.x - 1) / gridDim.x;
    if (2 * (long long)gridDim.x > p.item_capacity) {  // never write past the partial slots
        if (tid == 0 && blockIdx.x == 0) atomicOr(p.status, 2);
        return;
    }
    const float scale_log2 = p.scale * kLog2e;
    constexpr float kNegInf = -INFINITY;
    const bool small = total <= (long long)INT32_MAX;
    const long long n_units = (long long)p.B * per_chunk, n_cta = gridDim.x;
    const long long unit_len = (long long)n_max + Gm::kGapKeys;
    const bool aligned = n_min == n_max && n_units >= n_cta &&
                         (n_units + n_cta - 1) / n_cta * unit_len <= R + 2 * Gm::kGapKeys;
    const long long range_lo = aligned ? blockIdx.x * n_units / n_cta * unit_len : (long long)blockIdx.x * R;
    const long long range_hi =
        aligned ? (blockIdx.x + 1) * n_units / n_cta * unit_len : min(total, range_lo + R);

    bool dep_done = false;  // early start: the kernel before this one has completed
    // Where shared memory holds no copy of the lengths (head dim 256), the next sequence's
    // length is requested one piece ahead: a global read made when the piece needs it
    // waits behind the other CTAs' streams for about a microsecond.
    int pf_b = -1, pf_len = 0;
    for (long long pos = range_lo; pos < range_hi;) {
        // unit containing pos: sequence b (prefix search), then (kv head, head group)
        int lo = 0, hi = p.B - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if ((long long)prefix[mid] * per_chunk <= pos) lo = mid;
            else hi = mid - 1;
        }
        const int b = lo;
        int L_in;
        if (Gm::kLensCached) {
            L_in = lens_s[b];
        } else {
            L_in = b == pf_b ? pf_len : ctx_len_of(p, b);
            if (b + 1 < p.B) {
                pf_b = b + 1;
                pf_len = ctx_len_of(p, b + 1);  // used by the next piece, if it is in sequence b + 1
            }
        }
        int L, first;
        const bool ok = seq_range_of(p, L_in, L, first);
        const int n_b = L - first + 1;
        const int n_v = n_b + Gm::kGapKeys;  // the unit's stream length
        const long long seq_base = (long long)prefix[b] * per_chunk;
        // 32-bit divisions when the whole stream fits (`small`)
        const int r = small ? (int)(pos - seq_base) / n_v : (int)((pos - seq_base) / n_v);
        const long long u_start = seq_base + (long long)r * n_v, u_end = u_start + n_b;
        if (pos >= u_end) {  // in the unit's gap: nothing to attend
            pos = u_start + n_v;
            continue;
        }
        const long long piece_end = min(range_hi, u_end);
        const int kvh = r / p.n_hg, hg = r - kvh * p.n_hg;
        const int k0 = first + (int)(pos - u_start);
        const int k1 = first + (int)(piece_end - u_start);
        const int c0 = small ? (int)u_start / (int)R : (int)(u_start / R);
        const int c1 = small ? (int)(u_end - 1) / (int)R : (int)((u_end - 1) / R);
        const int n_split = aligned ? 1 : c1 - c0 + 1;      // pieces of this unit
        const int my_slot = 2 * blockIdx.x + (pos == range_lo ? 0 : 1);
        const int unit = b * per_chunk + r;
        pos = piece_end;
        const int h0 = kvh * p.G + hg * kHeads;
        const int nh = min(kHeads, p.G - hg * kHeads);

        if (!ok) {
            if (p.early_start && !dep_done) {  // no write before the kernel ahead has completed
                asm volatile("griddepcontrol.wait;" ::: "memory");
                dep_done = true;
            }
            for (int e = tid; e < nh * D; e += kThreads)
                store_from_float(p.out, ((int64_t)b * p.Hq + h0 + e / D) * D + e % D, __int_as_float(0x7fc00000),
                                 p.out_dtype);
            continue;
        }

        const T* kc = static_cast<const T*>(p.k_cache) + b * p.stride_b + kvh * p.stride_h;
        const T* vc = static_cast<const T*>(p.v_cache) + b * p.stride_b + kvh * p.stride_h;
        const int n_tiles = (k1 - k0 + kTile - 1) / kTile;
        const bool has_new = p.append && k1 == L + 1;

        auto load_tile = [&](int tile, int stage) {
            const int ts = k0 + tile * kTile;
            T* ks = pipe + stage * Gm::kStageElems;
            T* vs = ks + kTile * kRow;
#pragma unroll 4
            for (int x = tid; x < kTile * Gm::kChunks; x += kThreads) {
                const int row = x / Gm::kChunks, cc = x - row * Gm::kChunks;
                const int key = ts + row;
                const bool in = key < k1;
                const int64_t off = (int64_t)(in ? key : k0) * p.stride_pos + cc * 8;
                cp_async_16(smem_u32(ks + row * kRow + cc * 8), kc + off, in ? 16 : 0);
                cp_async_16(smem_u32(vs + row * kRow + cc * 8), vc + off, in ? 16 : 0);
            }
        };

        // ------------------------------------------------ prologue loads
        // Every global read of the prologue (RoPE frequencies, this unit's q rows, the new
        // k/v row, biases) is requested before the first tiles' copies are issued and used
        // only after them: with HBM saturated by the other CTAs' streams each read takes
        // microseconds, and issued one after another they were most of a piece's fixed cost.
        const bool rope = p.append && p.rope_mode != 0;
        double inv_f = 0.0;
        if (rope && tid < D / 2) inv_f = p.inv_freq[tid];  // a kernel-parameter array: plain load
        // Early start (programmatic dependent launch): the first piece requests its cache tiles
        // (rows below L, which the kernel before it on the stream does not write), then waits
        // for that kernel to complete before reading anything it may have produced -- q, the
        // new k/v rows, biases, norm weights -- and before any write.
        const bool tiles_first = p.early_start && !dep_done;
        if (tiles_first) {
#pragma unroll
            for (int s = 0; s < kStages - 1; ++s) {
                if (s < n_tiles) load_tile(s, s);
                cp_async_commit();
            }
            asm volatile("griddepcontrol.wait;" ::: "memory");
            dep_done = true;
        }
        constexpr int kHeadsPerWarp = kHeads / kWarps;
        static_assert(kHeads % kWarps == 0 && D / 2 <= kThreads, "prologue work split");
        HeadLoad<D> qload[kHeadsPerWarp];
#pragma unroll
        for (int i = 0; i < kHeadsPerWarp; ++i) {
            const int hl = warp + kWarps * i;
            if (hl < nh)
                head_load<D>(qload[i], p.q, (int64_t)b * q_stride_of(p) + (int64_t)(h0 + hl) * D, p.q_dtype,
                             p.q_bias ? p.q_bias + (h0 + hl) * D : nullptr, lane);
        }
        // QK-norm weights, elements lane + 32 j: the q weights serve every q head of the warp
        float qnw[D / 32], knw[D / 32];
        const float* const qn = p.append ? p.q_norm_w : nullptr;
        const float* const kn = (has_new && warp == 0) ? p.k_norm_w : nullptr;
#pragma unroll
        for (int j = 0; j < D / 32; ++j) {
            qnw[j] = qn != nullptr ? __ldg(qn + lane + 32 * j) : 0.f;
            knw[j] = kn != nullptr ? __ldg(kn + lane + 32 * j) : 0.f;
        }
        HeadLoad<D> nload;  // warp 0: the new key row, warp 1: the new value row
        if (has_new && warp < 2)
            head_load<D>(nload, warp == 0 ? p.k_new : p.v_new, (int64_t)b * kvn_stride_of(p) + (int64_t)kvh * D,
                         p.q_dtype, warp == 0 ? (p.k_bias ? p.k_bias + kvh * D : nullptr)
                                              : (p.v_bias ? p.v_bias + kvh * D : nullptr),
                         lane);
        if (!tiles_first) {
#pragma unroll
            for (int s = 0; s < kStages - 1; ++s) {
                if (s < n_tiles) load_tile(s, s);
                cp_async_commit();
            }
        }

        // ------------------------------------------------ prologue (q, new k/v)
        if (rope && tid < D / 2) {
            double sn, cn;
            sincos((double)L * inv_f, &sn, &cn);
            cs_s[2 * tid] = cn;
            cs_s[2 * tid + 1] = sn;
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < kHeadsPerWarp; ++i) {
            const int hl = warp + kWarps * i;
            T* qrow = q_s + hl * kRow;
            T* qlo = qlo_s + hl * kRow;
            if (hl >= nh) {
                for (int d = lane; d < D; d += 32) qrow[d] = qlo[d] = Elem<T>::from_float(0.f);
                continue;
            }
            prep_finish<D>(p, qload[i], p.q_dtype, p.q_bias != nullptr, qn != nullptr, qnw, rope, cs_s, vec, lane);
            for (int d = lane; d < D; d += 32) {
                const T hi = Elem<T>::from_float(vec[d]);
                qrow[d] = hi;
                if (kSplit) qlo[d] = Elem<T>::from_float(vec[d] - Elem<T>::to_float(hi));
            }
            __syncwarp();
        }
        if (has_new) {
            if (warp == 0) {
                prep_finish<D>(p, nload, p.q_dtype, p.k_bias != nullptr, kn != nullptr, knw, rope, cs_s, vec, lane);
                T* dst = static_cast<T*>(p.k_cache) + b * p.stride_b + kvh * p.stride_h + (int64_t)L * p.stride_pos;
                for (int d = lane; d < D; d += 32) {
                    const T v = Elem<T>::from_float(vec[d]);
                    knew_s[d] = v;
                    if (hg == 0) dst[d] = v;
                }
            } else if (warp == 1) {
                T* dst = static_cast<T*>(p.v_cache) + b * p.stride_b + kvh * p.stride_h + (int64_t)L * p.stride_pos;
#pragma unroll
                for (int j = 0; j < D / 32; ++j) {
                    const int d = lane + 32 * j;
                    float vf = raw_to_float(nload.raw[j], p.q_dtype);
                    if (p.v_bias != nullptr) vf = __fadd_rn(vf, nload.bias[j]);
                    const T v = Elem<T>::from_float(vf);
                    vnew_s[d] = v;
                    if (hg == 0) dst[d] = v;
                }
            }
        }
        __syncthreads();

        uint32_t qb[D / 16][2];
        uint32_t qbl[kSplit ? D / 16 : 1][2];
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
            const T* base = q_s + g * kRow + 16 * ks + 2 * t;
            qb[ks][0] = *reinterpret_cast<const uint32_t*>(base);
            qb[ks][1] = *reinterpret_cast<const uint32_t*>(base + 8);
            if constexpr (kSplit) {
                const T* bl = qlo_s + g * kRow + 16 * ks + 2 * t;
                qbl[ks][0] = *reinterpret_cast<const uint32_t*>(bl);
                qbl[ks][1] = *reinterpret_cast<const uint32_t*>(bl + 8);
            }
        }

        // ------------------------------------------------------- main loop
        float acc[D / 16][4];
#pragma unroll
        for (int mt = 0; mt < D / 16; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
        float m0 = kNegInf, m1 = kNegInf, l0 = 0.f, l1 = 0.f;
        const int wrow = warp * 16;

        for (int tile = 0; tile < n_tiles; ++tile) {
            cp_async_wait<kStages - 2>();
            __syncthreads();
            const int stage = tile % kStages;
            T* ks = pipe + stage * Gm::kStageElems;
            T* vs = ks + kTile * kRow;
            const int ts = k0 + tile * kTile;
            if (has_new && L >= ts && L < ts + kTile) {
                const int row = L - ts;
                for (int d = tid; d < D; d += kThreads) {
                    ks[row * kRow + d] = knew_s[d];
                    vs[row * kRow + d] = vnew_s[d];
                }
                __syncthreads();
            }
            {
                const int nt = tile + kStages - 1;
                if (nt < n_tiles) load_tile(nt, nt % kStages);
                cp_async_commit();
            }
            if (ts + wrow >= k1) continue;  // this warp's 16 rows are all past the chunk

            float s[4] = {0.f, 0.f, 0.f, 0.f};
            const uint32_t ka = smem_u32(ks + (wrow + (lane & 15)) * kRow + 8 * (lane >> 4));
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
                uint32_t a[4];
                ldmatrix_x4(a[0], a[1], a[2], a[3], ka + kk * 32);
                Mma<T>::run(s, a, qb[kk][0], qb[kk][1]);
                if constexpr (kSplit) Mma<T>::run(s, a, qbl[kk][0], qbl[kk][1]);
            }
            const int key_a = ts + wrow + g, key_b = key_a + 8;
            const float sa0 = key_a < k1 ? s[0] * scale_log2 : kNegInf;
            const float sa1 = key_a < k1 ? s[1] * scale_log2 : kNegInf;
            const float sb0 = key_b < k1 ? s[2] * scale_log2 : kNegInf;
            const float sb1 = key_b < k1 ? s[3] * scale_log2 : kNegInf;
            float mt0 = fmaxf(sa0, sb0), mt1 = fmaxf(sa1, sb1);
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                mt0 = fmaxf(mt0, __shfl_xor_sync(0xffffffffu, mt0, o));
                mt1 = fmaxf(mt1, __shfl_xor_sync(0xffffffffu, mt1, o));
            }
            const float mn0 = fmaxf(m0, mt0), mn1 = fmaxf(m1, mt1);
            const float base0 = mn0 == kNegInf ? 0.f : mn0;
            const float base1 = mn1 == kNegInf ? 0.f : mn1;
            const float c0 = fast_exp2(m0 - base0), c1 = fast_exp2(m1 - base1);
            const float pa0 = fast_exp2(sa0 - base0), pa1 = fast_exp2(sa1 - base1);
            const float pb0 = fast_exp2(sb0 - base0), pb1 = fast_exp2(sb1 - base1);
            l0 = l0 * c0 + pa0 + pb0;
            l1 = l1 * c1 + pa1 + pb1;
            m0 = mn0;
            m1 = mn1;
#pragma unroll
            for (int mt = 0; mt < D / 16; ++mt) {
                acc[mt][0] *= c0;
                acc[mt][1] *= c1;
                acc[mt][2] *= c0;
                acc[mt][3] *= c1;
            }
            const uint32_t ph0 = Elem<T>::pack(pa0, pa1), ph1 = Elem<T>::pack(pb0, pb1);
            const uint32_t pf0 = movmatrix_trans(ph0);
            const uint32_t pf1 = movmatrix_trans(ph1);
            uint32_t pl0 = 0, pl1 = 0;
            if constexpr (kSplit) {
                const T* h0p = reinterpret_cast<const T*>(&ph0);
                const T* h1p = reinterpret_cast<const T*>(&ph1);
                pl0 = movmatrix_trans(Elem<T>::pack(pa0 - Elem<T>::to_float(h0p[0]), pa1 - Elem<T>::to_float(h0p[1])));
                pl1 = movmatrix_trans(Elem<T>::pack(pb0 - Elem<T>::to_float(h1p[0]), pb1 - Elem<T>::to_float(h1p[1])));
            }
            const uint32_t va = smem_u32(vs + (wrow + (lane & 7) + 8 * (lane >> 4)) * kRow + 8 * ((lane >> 3) & 1));
#pragma unroll
            for (int mt = 0; mt < D / 16; ++mt) {
                uint32_t a[4];
                ldmatrix_x4_trans(a[0], a[1], a[2], a[3], va + mt * 32);
                Mma<T>::run(acc[mt], a, pf0, pf1);
                if constexpr (kSplit) Mma<T>::run(acc[mt], a, pl0, pl1);
            }
        }
        cp_async_wait<0>();
        __syncthreads();  // pipeline drained: merge_s may alias it now

        // ------------------------------------------------------- epilogue
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            l0 += __shfl_xor_sync(0xffffffffu, l0, o);
            l1 += __shfl_xor_sync(0xffffffffu, l1, o);
        }
        {
            // The warp's unnormalised O as [d][head] float pairs (heads 2t, 2t+1 of row d),
            // the head index XOR-swizzled by (d >> 2) & 7: these pair stores and the merge's
            // reads along d (one head, consecutive d) are both free of bank conflicts.
            float* mw = merge_s + warp * kHeads * D;
#pragma unroll
            for (int mt = 0; mt < D / 16; ++mt) {
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    const int d = 16 * mt + g + 8 * hf, f = (d >> 2) & 7;
                    const float a = acc[mt][2 * hf], c = acc[mt][2 * hf + 1];
                    *reinterpret_cast<float2*>(mw + d * kHeads + ((2 * t) ^ (f & 6))) =
                        (f & 1) ? make_float2(c, a) : make_float2(a, c);
                }
            }
            if (g == 0) {
                ml_s[(warp * kHeads + 2 * t) * 2 + 0] = m0;
                ml_s[(warp * kHeads + 2 * t) * 2 + 1] = l0;
                ml_s[(warp * kHeads + 2 * t + 1) * 2 + 0] = m1;
                ml_s[(warp * kHeads + 2 * t + 1) * 2 + 1] = l1;
            }
        }
        __syncthreads();
        float* slot = p.partials + (int64_t)my_slot * kHeads * (D + 2);
        if (tid < kHeads) {
            // per head: the four warps' weights 2^(m_w - M) (in place of m_w) and the
            // combined sum (in place of warp 0's l); a split piece also publishes (M, sum)
            const int hl = tid;
            float M = kNegInf;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) M = fmaxf(M, ml_s[(w * kHeads + hl) * 2]);
            const float base = M == kNegInf ? 0.f : M;
            float l = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
                const float f = fast_exp2(ml_s[(w * kHeads + hl) * 2] - base);
                l += f * ml_s[(w * kHeads + hl) * 2 + 1];
                ml_s[(w * kHeads + hl) * 2] = f;
            }
            ml_s[hl * 2 + 1] = l;
            if (n_split > 1) {
                slot[kHeads * D + hl] = base;
                slot[kHeads * D + kHeads + hl] = l;
            }
        }
        __syncthreads();
        for (int e = tid; e < nh * D; e += kThreads) {
            const int hl = e / D, d = e - hl * D;
            const int sw = d * kHeads + (hl ^ ((d >> 2) & 7));
            float o = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) o += ml_s[(w * kHeads + hl) * 2] * merge_s[w * kHeads * D + sw];
            if (n_split == 1) store_from_float(p.out, ((int64_t)b * p.Hq + h0 + hl) * D + d, o / ml_s[hl * 2 + 1],
                                               p.out_dtype);
            else slot[hl * D + d] = o;
        }
        if (n_split > 1) {
            // publish the slot (one fence after the barrier orders every thread's stores
            // before the counter update), then count the unit's finished pieces
            __syncthreads();
            int* counter = p.counters + unit;
            if (tid == 0) {
                __threadfence();
                const int last = atomicAdd(counter, 1) == n_split - 1;
                if (last) __threadfence();
                misc[8] = last;
            }
            __syncthreads();
            if (misc[8]) {
                // Last piece of the unit: log-sum-exp combine of its n_split
                // partial slots.  The piece of CTA c sits in slot 2c, or 2c+1
                // when the unit starts inside c's range after its first piece.
                // A thread owns float4 groups of 4 consecutive d of one head; the loads of
                // up to kBatch slots are all issued before any is used (one L2 round trip
                // per batch).
                auto slot_of = [&](int c) {
                    const int sub = (c == c0 && u_start != (long long)c0 * R) ? 1 : 0;
                    return p.partials + (int64_t)(2 * c + sub) * kHeads * (D + 2);
                };
                constexpr int kQ4 = kHeads * D / 4;                     // float4 groups of a slot's O
                constexpr int kPer = (kQ4 + kThreads - 1) / kThreads;  // per thread: 1, 2, 2, 4
                constexpr int kBatch = kPer == 1 ? 8 : (kPer == 2 ? 4 : 2);
                float4 o[kPer];
                float lsum[kPer], mrun[kPer];
#pragma unroll
                for (int j = 0; j < kPer; ++j) {
                    o[j] = make_float4(0.f, 0.f, 0.f, 0.f);
                    lsum[j] = 0.f;
                    mrun[j] = kNegInf;
                }
                for (int cb = 0; cb < n_split; cb += kBatch) {
                    float4 ov[kBatch][kPer];
                    float mv[kBatch][kPer], lv[kBatch][kPer];
#pragma unroll
                    for (int i = 0; i < kBatch; ++i) {
                        if (cb + i >= n_split) break;
                        const float* sl = slot_of(c0 + cb + i);
#pragma unroll
                        for (int j = 0; j < kPer; ++j) {
                            const int q4 = tid + j * kThreads, hl = min(q4, kQ4 - 1) * 4 / D;
                            ov[i][j] = q4 < kQ4 ? __ldcg(reinterpret_cast<const float4*>(sl) + q4)
                                                : make_float4(0.f, 0.f, 0.f, 0.f);
                            mv[i][j] = __ldcg(sl + kHeads * D + hl);
                            lv[i][j] = __ldcg(sl + kHeads * D + kHeads + hl);
                        }
                    }
#pragma unroll
                    for (int j = 0; j < kPer; ++j) {
                        float M = mrun[j];
#pragma unroll
                        for (int i = 0; i < kBatch; ++i)
                            if (cb + i < n_split) M = fmaxf(M, mv[i][j]);
                        const float base = M == kNegInf ? 0.f : M;
                        const float keep = fast_exp2(mrun[j] - base);  // 0 for the first batch
                        o[j].x *= keep;
                        o[j].y *= keep;
                        o[j].z *= keep;
                        o[j].w *= keep;
                        lsum[j] *= keep;
#pragma unroll
                        for (int i = 0; i < kBatch; ++i) {
                            if (cb + i >= n_split) break;
                            const float f = fast_exp2(mv[i][j] - base);
                            o[j].x += f * ov[i][j].x;
                            o[j].y += f * ov[i][j].y;
                            o[j].z += f * ov[i][j].z;
                            o[j].w += f * ov[i][j].w;
                            lsum[j] += f * lv[i][j];
                        }
                        mrun[j] = M;
                    }
                }
#pragma unroll
                for (int j = 0; j < kPer; ++j) {
                    const int q4 = tid + j * kThreads;
                    if (q4 >= kQ4) break;
                    const int hl = q4 * 4 / D, d = q4 * 4 - hl * D;
                    if (hl < nh) {
                        const int64_t oi = ((int64_t)b * p.Hq + h0 + hl) * D + d;
                        store_from_float(p.out, oi + 0, o[j].x / lsum[j], p.out_dtype);
                        store_from_float(p.out, oi + 1, o[j].y / lsum[j], p.out_dtype);
                        store_from_float(p.out, oi + 2, o[j].z / lsum[j], p.out_dtype);
                        store_from_float(p.out, oi + 3, o[j].w / lsum[j], p.out_dtype);
                    }
                }
                if (tid == 0) *counter = 0;
            }
        }
        __syncthreads();  // shared buffers are reused by the next piece
    }
}

struct LaunchInfo {
    int grid = 0;
    size_t smem = 0;
};

// Kernel attributes are per device: set up once for each device (the caller has made
// `device` current).
template <int D, typename T>
LaunchInfo launch_info(int device) {
    constexpr int kMaxDevices = 64;
    static std::once_flag once[kMaxDevices];
    static LaunchInfo info[kMaxDevices];
    static cudaError_t err[kMaxDevices];
    if (device < 0 || device >= kMaxDevices) return LaunchInfo{};
    std::call_once(once[device], [device] {
        auto kern = decode_tc_kernel<D, T>;
        LaunchInfo li;
        li.smem = Geo<D>::kTotal;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)li.smem);
        int occ = 0, sms = 0;
        if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, li.smem);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
        li.grid = occ * sms;
        info[device] = li;
        err[device] = e;
    });
    if (err[device] != cudaSuccess) return LaunchInfo{};
    return info[device];
}

template <typename F>
bool dispatch_dim(int D, F&& f) {
    switch (D) {
        case 64: f(std::integral_constant<int, 64>{}); return true;
        case 96: f(std::integral_constant<int, 96>{}); return true;
        case 128: f(std::integral_constant<int, 128>{}); return true;
        case 256: f(std::integral_constant<int, 256>{}); return true;
        default: return false;
    }
}

}  // namespace

bool decode_tc_supported(int D, int cache_dtype) {
    return (cache_dtype == kF16 || cache_dtype == kBF16) && (D == 64 || D == 96 || D == 128 || D == 256);
}

void decode_tc_workspace(int device, int B, int Hkv, int n_hg, int D, int cache_dtype, int* target_items,
                         int* item_capacity, size_t* partial_bytes) {
    int grid = 0;
    dispatch_dim(D, [&](auto dc) {
        constexpr int kD = decltype(dc)::value;
        grid = cache_dtype == kBF16 ? launch_info<kD, __nv_bfloat16>(device).grid
                                    : launch_info<kD, __half>(device).grid;
    });
    if (grid <= 0) grid = 148;
    (void)B;
    (void)Hkv;
    (void)n_hg;
    *target_items = grid;
    *item_capacity = 2 * grid;  // two partial slots per CTA
    *partial_bytes = (size_t)(*item_capacity) * kHeads * (D + 2) * sizeof(float);
}

cudaError_t launch_decode_tc(const DecodeParams& p, int device, cudaStream_t stream) {
    cudaError_t err = cudaErrorInvalidValue;
    dispatch_dim(p.D, [&](auto dc) {
        constexpr int kD = decltype(dc)::value;
        auto go = [&](auto kern, const LaunchInfo& li) {
            if (li.grid <= 0) return cudaErrorInvalidConfiguration;
            if (!p.early_start) {
                kern<<<li.grid, kThreads, li.smem, stream>>>(p);
                return cudaGetLastError();
            }
            // programmatic stream serialisation: the launch may begin before the kernel ahead of
            // it completes; the kernel's griddepcontrol.wait orders its dependent reads and writes
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3((unsigned)li.grid);
            cfg.blockDim = dim3(kThreads);
            cfg.dynamicSmemBytes = li.smem;
            cfg.stream = stream;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            return cudaLaunchKernelEx(&cfg, kern, p);
        };
        if (p.cache_dtype == kBF16) err = go(decode_tc_kernel<kD, __nv_bfloat16>, launch_info<kD, __nv_bfloat16>(device));
        else err = go(decode_tc_kernel<kD, __half>, launch_info<kD, __half>(device));
    });
    return err;
}

}  // namespace b2a
