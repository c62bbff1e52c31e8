// attn_simt.cu -- generic whole-sequence attention (causal prefill and
// bidirectional encoder) for any element type and any even head_dim <= 256,
// computing in fp32.  It is the path of the reference's FLOAT32
// AttentionKernel contract (WB/runtime/kernels/AttentionKernel.java:19-24,
// DirectMlAttentionKernel validates FLOAT32 at L663-675) and of fp32 causal
// prefill (SmolLM2ReferenceForwardPass.runSelfAttention,
// INF/smollm2/SmolLM2ReferenceForwardPass.java:167-210); 16-bit inputs with a
// tensor-core instantiation take attn_tcgen05.cu / attn_mma.cu instead.
//
// CTA = 8 consecutive query positions of one (batch, kv head) and up to 8 of
// the kv head's query heads (its GQA group): warp w owns position s0 + w for
// every head of the group.  Keys go through shared memory 32 at a time (one
// coalesced load per tile, shared by all 8 positions and all heads of the
// group); scores are one key per lane, dot products over fp32 shared rows
// padded by one word (conflict-free); P·V is lanes over head dimensions with
// the probabilities read back from a per-warp shared row (one broadcast load
// per key for all heads).  Online softmax in exp2 with the scale folded in.
// q/k arrive already rotated when RoPE applies.
// When rows hold whole groups of 4 elements (kVec: head_dim, strides and bases
// multiples of 4 elements) each thread owns fixed 4-element groups of a tile and
// loads the next tile's groups into registers while the current tile is used, so a
// CTA's sequential key tiles do not each wait for a global load.
// Key split (launches too small to fill the GPU, e.g. one short causal prefill):
// each query block's key range is cut into chunks of SimtSplit::split_keys keys, one
// CTA per chunk; a chunk's CTA writes its rows' (max, sum, unnormalised O) to a slot,
// and the last CTA of the block to finish (a per-block counter) combines the slots
// (log-sum-exp) and resets the counter, so the counters are zero between launches.
#include <math.h>

#include <type_traits>

#include "common.cuh"
#include "internal.h"

namespace b2a {
namespace {

constexpr int kRows = 8;                     // query positions per CTA (one warp each)
constexpr int kHeads = 8;                    // at most this many query heads per CTA (a GQA group or a chunk)
constexpr int kTileKeys = 32;                // keys per shared-memory tile (one per lane)

// kHT: query heads per CTA rounded up to 1, 2, 4 or 8; every K and V element read from
// shared memory feeds all of them (independent FMA chains), padding heads are zeros.
// kNPL: head dimensions per lane, ceil(D / 32) rounded up to 1, 2, 3, 4 or 8.
// 4 consecutive elements, not yet converted (16-bit types use the first two words).
__device__ __forceinline__ uint4 load_raw4(const void* p, int64_t i, int dtype) {
    if (dtype == kF32) return __ldg(reinterpret_cast<const uint4*>(static_cast<const float*>(p) + i));
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(static_cast<const unsigned short*>(p) + i));
    return make_uint4(u.x, u.y, 0u, 0u);
}
__device__ __forceinline__ void raw4_store(float* dst, uint4 r, int dtype) {
    if (dtype == kF32) {
        dst[0] = __uint_as_float(r.x);
        dst[1] = __uint_as_float(r.y);
        dst[2] = __uint_as_float(r.z);
        dst[3] = __uint_as_float(r.w);
    } else {
        dst[0] = raw_to_float(r.x & 0xffffu, dtype);
        dst[1] = raw_to_float(r.x >> 16, dtype);
        dst[2] = raw_to_float(r.y & 0xffffu, dtype);
        dst[3] = raw_to_float(r.y >> 16, dtype);
    }
}

template <int kHT, int kNPL, bool kVec>
__global__ void __launch_bounds__(kRows * 32) attn_simt_kernel(const __grid_constant__ AttnParams p, int G,
                                                               const SimtSplit split) {
    extern __shared__ float sm[];
    const int D = p.D, Dp = D + 1;
    float* ks = sm;                          // [kTileKeys][D + 1]
    float* vs = ks + kTileKeys * Dp;         // [kTileKeys][D + 1]
    float* qs = vs + kTileKeys * Dp;         // [kRows][heads][D]
    float* ps = qs + kRows * kHT * D;        // [kRows][kTileKeys][kHT] this tile's probabilities
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int in_dtype = p.in_dtype;
    const float* const mask = p.mask;
    const int64_t k_ss = p.k_ss;
    const int S = p.S;
    const int nsplit = split.nsplit;
    const int qblk = (int)blockIdx.x / nsplit, part = (int)blockIdx.x - qblk * nsplit;
    const int s0 = qblk * kRows;
    const int chunks = (G + kHeads - 1) / kHeads;
    const int kvh = blockIdx.y / chunks, h0 = kvh * G + (blockIdx.y % chunks) * kHeads;
    const int nh = min(kHeads, kvh * G + G - h0);  // heads of this CTA
    const int b = blockIdx.z;
    const int s = s0 + warp;
    const bool row_valid = s < S;

    // visible keys of this row, and the CTA's union of them
    int first = 0, last = S - 1;
    bool uniform = false;  // every key masked: softmax over equal scores -> mean of V
    if (p.causal) {
        last = min(s, S - 1);
        if (p.window > 0) first = max(0, s - p.window + 1);
    } else if (p.key_len != nullptr) {
        const int kl = p.key_len[b];
        if (kl <= 0) uniform = true;
        else last = min(kl, S) - 1;
    }
    int cta_first = first, cta_last = last;
    if (p.causal) {
        const int s_hi = min(s0 + kRows - 1, S - 1);
        cta_last = s_hi;
        cta_first = p.window > 0 ? max(0, s0 - p.window + 1) : 0;
    }
    // key split: this CTA's chunk of the block's range (the block's chunk count from its whole range)
    int n_parts = 1;
    if (nsplit > 1) {
        n_parts = min(nsplit, (cta_last - cta_first + split.split_keys) / split.split_keys);
        if (part >= n_parts) return;  // past the block's keys (the whole CTA, before any barrier)
        const int lo = cta_first + part * split.split_keys;
        cta_last = min(cta_last, lo + split.split_keys - 1);
        cta_first = lo;
    }

    // this row's query vectors, as fp32 (padding heads zero)
    const float2* const rope = p.rope_table;
    const int half = D >> 1;
    if (rope != nullptr) {
        // NeoX rotation at position rope_pos0 + s, float products from the float (cos, sin) of a
        // double angle (INF/decoderonly/DecoderOnlyRotaryEmbedding.java:42-67)
        const float2* cs_row = rope + (int64_t)(p.rope_pos0 + (row_valid ? s : 0)) * half;
        for (int g = 0; g < kHT; ++g)
            for (int i = lane; i < half; i += 32) {
                float y0 = 0.f, y1 = 0.f;
                if (row_valid && g < nh) {
                    const int64_t qo = b * p.q_sb + (int64_t)s * p.q_ss + (int64_t)(h0 + g) * p.q_sh;
                    const float a = load_as_float(p.q, qo + i, p.in_dtype);
                    const float c = load_as_float(p.q, qo + i + half, p.in_dtype);
                    const float2 t = __ldg(cs_row + i);
                    y0 = __fsub_rn(__fmul_rn(a, t.x), __fmul_rn(c, t.y));
                    y1 = __fadd_rn(__fmul_rn(a, t.y), __fmul_rn(c, t.x));
                }
                qs[(warp * kHT + g) * D + i] = y0;
                qs[(warp * kHT + g) * D + i + half] = y1;
            }
    } else {
        for (int g = 0; g < kHT; ++g)
            for (int d = lane; d < D; d += 32)
                qs[(warp * kHT + g) * D + d] =
                    row_valid && g < nh
                        ? load_as_float(p.q, b * p.q_sb + (int64_t)s * p.q_ss + (int64_t)(h0 + g) * p.q_sh + d,
                                        p.in_dtype)
                        : 0.f;
    }
    const float sl2 = p.scale * kLog2e;
    float acc[kHT][kNPL];
    float m[kHT], l[kHT];
#pragma unroll
    for (int g = 0; g < kHT; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int i = 0; i < kNPL; ++i) acc[g][i] = 0.f;
    }
    const int64_t kbase = b * p.k_sb + (int64_t)kvh * p.k_sh;
    // vector path: this thread's 4-element groups of a tile (key within the tile, first dim);
    // a tile has kTileKeys * D / 4 <= kNPL * blockDim.x groups
    constexpr int kG = kVec ? kNPL : 1;
    int gkey[kG], goff[kG];
    uint4 kraw[kG], vraw[kG];
    if constexpr (kVec) {
        const int G4 = D / 4;
#pragma unroll
        for (int i = 0; i < kG; ++i) {
            const int x = threadIdx.x + i * (kRows * 32);
            gkey[i] = x < kTileKeys * G4 ? x / G4 : -1;
            goff[i] = (x % G4) * 4;
        }
    }
    // in-kernel RoPE of the staged keys: thread t rotates the pairs e = t + kRotPer * blockDim ... of a
    // tile; with half <= 32 their (cos, sin) are fetched with the tile (no dependent load after staging)
    constexpr int kRotPer = kTileKeys * 32 / (kRows * 32);
    const bool rot_prefetch = kVec && rope != nullptr && half <= 32;
    float2 trot[kRotPer];
    auto fetch = [&](int kb) {  // the tile at kb into registers (zeros past the CTA's last key)
        const int nk = min(kTileKeys, cta_last - kb + 1);
#pragma unroll
        for (int i = 0; i < kG; ++i) {
            if (gkey[i] >= 0 && gkey[i] < nk) {
                const int64_t r = kbase + (int64_t)(kb + gkey[i]) * k_ss + goff[i];
                kraw[i] = load_raw4(p.k, r, in_dtype);
                vraw[i] = load_raw4(p.v, r, in_dtype);
            } else {
                kraw[i] = vraw[i] = make_uint4(0u, 0u, 0u, 0u);
            }
        }
        if (rot_prefetch) {
#pragma unroll
            for (int r = 0; r < kRotPer; ++r) {
                const int e = (int)threadIdx.x + r * (int)blockDim.x, jj = e / half;
                trot[r] = jj < nk ? __ldg(rope + (int64_t)(p.rope_pos0 + kb + jj) * half + (e - jj * half))
                                  : make_float2(0.f, 0.f);
            }
        }
    };
    if (kVec && cta_first <= cta_last) fetch(cta_first);
    __syncthreads();
    for (int kb = cta_first; kb <= cta_last; kb += kTileKeys) {
        // stage 32 keys of K and V (fp32) for the whole CTA
        const int nk = min(kTileKeys, cta_last - kb + 1);
        if constexpr (kVec) {
#pragma unroll
            for (int i = 0; i < kG; ++i) {
                if (gkey[i] < 0) continue;
                raw4_store(ks + gkey[i] * Dp + goff[i], kraw[i], in_dtype);
                raw4_store(vs + gkey[i] * Dp + goff[i], vraw[i], in_dtype);
            }
        } else {
            for (int e = threadIdx.x; e < kTileKeys * D; e += blockDim.x) {
                const int j = e / D, d = e - j * D;
                float kv = 0.f, vv = 0.f;
                if (j < nk) {
                    const int64_t r = kbase + (int64_t)(kb + j) * k_ss + d;
                    kv = load_as_float(p.k, r, in_dtype);
                    vv = load_as_float(p.v, r, in_dtype);
                }
                ks[j * Dp + d] = kv;
                vs[j * Dp + d] = vv;
            }
        }
        if (rope != nullptr) {
            // rotate the staged keys in place at their positions (the same float rotation as q)
            __syncthreads();
            if (rot_prefetch) {
#pragma unroll
                for (int r = 0; r < kRotPer; ++r) {
                    const int e = (int)threadIdx.x + r * (int)blockDim.x, jj = e / half, i = e - jj * half;
                    if (jj < nk) {
                        const float a = ks[jj * Dp + i], c = ks[jj * Dp + i + half];
                        const float2 t = trot[r];
                        ks[jj * Dp + i] = __fsub_rn(__fmul_rn(a, t.x), __fmul_rn(c, t.y));
                        ks[jj * Dp + i + half] = __fadd_rn(__fmul_rn(a, t.y), __fmul_rn(c, t.x));
                    }
                }
            } else {
                for (int e = threadIdx.x; e < nk * half; e += blockDim.x) {
                    const int jj = e / half, i = e - jj * half;
                    const float a = ks[jj * Dp + i], c = ks[jj * Dp + i + half];
                    const float2 t = __ldg(rope + (int64_t)(p.rope_pos0 + kb + jj) * half + i);
                    ks[jj * Dp + i] = __fsub_rn(__fmul_rn(a, t.x), __fmul_rn(c, t.y));
                    ks[jj * Dp + i + half] = __fadd_rn(__fmul_rn(a, t.y), __fmul_rn(c, t.x));
                }
            }
        }
        __syncthreads();
        // the next tile's loads are in flight while this one is used
        if (kVec && kb + kTileKeys <= cta_last) fetch(kb + kTileKeys);
        const int j = kb + lane;
        const bool vis = row_valid && j >= first && j <= last && j - kb < nk;
        const bool any = row_valid && kb <= last && kb + kTileKeys - 1 >= first;
        if (any) {
            // scores of this lane's key for every head: one pass over the key row
            float sc[kHT];
#pragma unroll
            for (int g = 0; g < kHT; ++g) sc[g] = -INFINITY;
            if (vis) {
                if (uniform) {
#pragma unroll
                    for (int g = 0; g < kHT; ++g) sc[g] = 0.f;
                } else {
                    const float* qw = qs + warp * kHT * D;
                    const float* kr = ks + lane * Dp;
                    float dot[kHT];
#pragma unroll
                    for (int g = 0; g < kHT; ++g) dot[g] = 0.f;
                    // D is even and every q row starts 16-byte aligned when D % 4 == 0: q is read
                    // four dimensions at a time (a broadcast), K one word at a time (odd row pitch)
                    int d = 0;
                    if ((D & 3) == 0) {
#pragma unroll 2
                        for (; d < D; d += 4) {
                            const float k0 = kr[d], k1 = kr[d + 1], k2 = kr[d + 2], k3 = kr[d + 3];
#pragma unroll
                            for (int g = 0; g < kHT; ++g) {
                                const float4 q4 = *reinterpret_cast<const float4*>(qw + g * D + d);
                                dot[g] = fmaf(q4.x, k0, dot[g]);
                                dot[g] = fmaf(q4.y, k1, dot[g]);
                                dot[g] = fmaf(q4.z, k2, dot[g]);
                                dot[g] = fmaf(q4.w, k3, dot[g]);
                            }
                        }
                    }
                    for (; d < D; ++d) {
                        const float kv = kr[d];
#pragma unroll
                        for (int g = 0; g < kHT; ++g) dot[g] = fmaf(qw[g * D + d], kv, dot[g]);
                    }
#pragma unroll
                    for (int g = 0; g < kHT; ++g)
                        sc[g] = mask != nullptr ? (dot[g] * p.scale + mask[(int64_t)b * S + j]) * kLog2e
                                                : dot[g] * sl2;
                }
            }
            float pj[kHT];
#pragma unroll
            for (int g = 0; g < kHT; ++g) {
                const float mn = fmaxf(m[g], warp_max(sc[g]));
                // mn is -inf only while nothing is visible (warp-uniform): keep the state
                const float corr = mn == -INFINITY ? 1.f : fast_exp2(m[g] - mn);
                pj[g] = mn == -INFINITY ? 0.f : fast_exp2(sc[g] - mn);
                l[g] = l[g] * corr + warp_sum(pj[g]);
                m[g] = mn;
#pragma unroll
                for (int i = 0; i < kNPL; ++i) acc[g][i] *= corr;
            }
            // this lane's key's probabilities into the warp's row, read back per key as broadcasts
            float* prow = ps + warp * kTileKeys * kHT;
#pragma unroll
            for (int g = 0; g < kHT; ++g) prow[lane * kHT + g] = pj[g];
            __syncwarp();
            for (int jj = 0; jj < nk; ++jj) {
                float pw[kHT];
                if constexpr (kHT % 4 == 0) {
#pragma unroll
                    for (int g = 0; g < kHT; g += 4) {
                        const float4 t = *reinterpret_cast<const float4*>(prow + jj * kHT + g);
                        pw[g] = t.x;
                        pw[g + 1] = t.y;
                        pw[g + 2] = t.z;
                        pw[g + 3] = t.w;
                    }
                } else {
#pragma unroll
                    for (int g = 0; g < kHT; ++g) pw[g] = prow[jj * kHT + g];
                }
#pragma unroll
                for (int i = 0; i < kNPL; ++i) {
                    // dimensions beyond D read the tile's padding (zeros or the next row): their
                    // accumulators are never stored
                    const float vv = vs[jj * Dp + min(lane + 32 * i, D)];
#pragma unroll
                    for (int g = 0; g < kHT; ++g) acc[g][i] = fmaf(pw[g], vv, acc[g][i]);
                }
            }
        }
        __syncthreads();
    }
    if (n_parts == 1) {
        if (!row_valid) return;
#pragma unroll
        for (int g = 0; g < kHT; ++g) {
            if (g >= nh) break;
            const float inv = 1.f / l[g];
            const int64_t qo = b * p.q_sb + (int64_t)s * p.q_ss + (int64_t)(h0 + g) * p.q_sh;
#pragma unroll
            for (int i = 0; i < kNPL; ++i) {
                const int d = lane + 32 * i;
                if (d < D) store_from_float(p.o, qo + d, acc[g][i] * inv, p.out_dtype);
            }
        }
        return;
    }
    // this chunk's partial state: per row and head, O (unnormalised) [D], max, sum
    const int n_qblk = (int)gridDim.x / nsplit;
    const int blk = ((int)blockIdx.z * (int)gridDim.y + (int)blockIdx.y) * n_qblk + qblk;
    const int row_floats = D + 2;
    auto slot_of = [&](int pt) { return split.part + ((size_t)blk * nsplit + pt) * (kRows * kHT * row_floats); };
    if (row_valid) {
        float* mine = slot_of(part);
#pragma unroll
        for (int g = 0; g < kHT; ++g) {
            float* r = mine + (warp * kHT + g) * row_floats;
#pragma unroll
            for (int i = 0; i < kNPL; ++i) {
                const int d = lane + 32 * i;
                if (d < D) r[d] = acc[g][i];
            }
            if (lane == 0) {
                r[D] = m[g];
                r[D + 1] = l[g];
            }
        }
    }
    __threadfence();
    __syncthreads();
    __shared__ int is_last;
    if (threadIdx.x == 0) is_last = atomicAdd(split.cnt + blk, 1) == n_parts - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    if (row_valid) {
#pragma unroll
        for (int g = 0; g < kHT; ++g) {
            if (g >= nh) break;
            const int off = (warp * kHT + g) * row_floats;
            float M = -INFINITY;
            for (int pt = 0; pt < n_parts; ++pt) M = fmaxf(M, __ldcg(slot_of(pt) + off + D));
            const float base = M == -INFINITY ? 0.f : M;
            float L = 0.f, o[kNPL];
#pragma unroll
            for (int i = 0; i < kNPL; ++i) o[i] = 0.f;
            for (int pt = 0; pt < n_parts; ++pt) {
                const float* r = slot_of(pt) + off;
                const float f = fast_exp2(__ldcg(r + D) - base);  // 0 for a chunk with none of the row's keys
                L += f * __ldcg(r + D + 1);
#pragma unroll
                for (int i = 0; i < kNPL; ++i) {
                    const int d = lane + 32 * i;
                    if (d < D) o[i] += f * __ldcg(r + d);
                }
            }
            const float inv = 1.f / L;
            const int64_t qo = b * p.q_sb + (int64_t)s * p.q_ss + (int64_t)(h0 + g) * p.q_sh;
#pragma unroll
            for (int i = 0; i < kNPL; ++i) {
                const int d = lane + 32 * i;
                if (d < D) store_from_float(p.o, qo + d, o[i] * inv, p.out_dtype);
            }
        }
    }
    if (threadIdx.x == 0) split.cnt[blk] = 0;  // zero again for the next launch
}

}  // namespace

namespace {
int head_tile(const AttnParams& p) {
    const int G = p.Hq / p.Hkv;
    const int heads = G < kHeads ? G : kHeads;
    return heads <= 1 ? 1 : heads <= 2 ? 2 : heads <= 4 ? 4 : 8;
}
}  // namespace

int attn_simt_split_plan(const AttnParams& p, int sm_count, size_t* part_bytes, size_t* counter_ints) {
    *part_bytes = 0;
    *counter_ints = 0;
    const int G = p.Hq / p.Hkv;
    const int64_t blocks = (int64_t)((p.S + kRows - 1) / kRows) * p.Hkv * ((G + kHeads - 1) / kHeads) * p.B;
    // split only launches that leave SMs idle, into as many chunks as the longest range has
    const int nsplit = (p.S + kSimtSplitKeys - 1) / kSimtSplitKeys;
    if (blocks >= 2 * (int64_t)sm_count || nsplit <= 1 || blocks * nsplit > 65535) return 1;
    *part_bytes = (size_t)blocks * nsplit * kRows * head_tile(p) * (p.D + 2) * sizeof(float);
    *counter_ints = (size_t)blocks;
    return nsplit;
}

cudaError_t launch_attn_simt(const AttnParams& p, cudaStream_t stream, const SimtSplit* split) {
    const int G = p.Hq / p.Hkv;
    const int chunks = (G + kHeads - 1) / kHeads;
    const int ht = head_tile(p);
    const SimtSplit sp = split != nullptr ? *split : SimtSplit{nullptr, nullptr, 1, kSimtSplitKeys};
    const size_t smem =
        ((size_t)2 * kTileKeys * (p.D + 1) + (size_t)kRows * ht * p.D + (size_t)kRows * kTileKeys * ht) * sizeof(float);
    // 4-element groups: head dim, strides and bases in whole groups (16 B for fp32, 8 B for 16-bit)
    const size_t es = p.in_dtype == kF32 ? 4 : 2;
    const bool vec = p.D % 4 == 0 && p.k_ss % 4 == 0 && p.k_sh % 4 == 0 && p.k_sb % 4 == 0 &&
                     (uintptr_t)p.k % (4 * es) == 0 && (uintptr_t)p.v % (4 * es) == 0;
    const dim3 grid((p.S + kRows - 1) / kRows * sp.nsplit, p.Hkv * chunks, p.B);
    auto go = [&](auto kernel) {
        if (smem > 48 * 1024) {
            const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
        }
        kernel<<<grid, kRows * 32, smem, stream>>>(p, G, sp);
        return cudaGetLastError();
    };
    const int npl = (p.D + 31) / 32;
    auto by_dims = [&](auto ht_tag) {
        constexpr int HT = decltype(ht_tag)::value;
        auto pick = [&](auto npl_tag) {
            constexpr int NPL = decltype(npl_tag)::value;
            return vec ? go(attn_simt_kernel<HT, NPL, true>) : go(attn_simt_kernel<HT, NPL, false>);
        };
        if (npl <= 1) return pick(std::integral_constant<int, 1>{});
        if (npl <= 2) return pick(std::integral_constant<int, 2>{});
        if (npl <= 3) return pick(std::integral_constant<int, 3>{});
        if (npl <= 4) return pick(std::integral_constant<int, 4>{});
        return pick(std::integral_constant<int, 8>{});
    };
    switch (ht) {
        case 1: return by_dims(std::integral_constant<int, 1>{});
        case 2: return by_dims(std::integral_constant<int, 2>{});
        case 4: return by_dims(std::integral_constant<int, 4>{});
        default: return by_dims(std::integral_constant<int, 8>{});
    }
}

}  // namespace b2a
