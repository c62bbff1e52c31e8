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
// the probabilities broadcast by shuffles.  Online softmax in exp2 with the
// scale folded in.  q/k arrive already rotated when RoPE applies.
#include <math.h>

#include "common.cuh"
#include "internal.h"

namespace b2a {
namespace {

constexpr int kRows = 8;                     // query positions per CTA (one warp each)
constexpr int kHeads = 8;                    // query heads per CTA (a GQA group, or a chunk of one)
constexpr int kTileKeys = 32;                // keys per shared-memory tile (one per lane)
constexpr int kMaxPerLane = kMaxHeadDim / 32;

__global__ void __launch_bounds__(kRows * 32) attn_simt_kernel(const __grid_constant__ AttnParams p, int G,
                                                                int heads_here_max) {
    extern __shared__ float sm[];
    const int D = p.D, Dp = D + 1;
    float* ks = sm;                          // [kTileKeys][D + 1]
    float* vs = ks + kTileKeys * Dp;         // [kTileKeys][D + 1]
    float* qs = vs + kTileKeys * Dp;         // [kRows][heads][D]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = p.S;
    const int s0 = blockIdx.x * kRows;
    const int chunks = (G + kHeads - 1) / kHeads;
    const int kvh = blockIdx.y / chunks, h0 = kvh * G + (blockIdx.y % chunks) * kHeads;
    const int nh = min(kHeads, kvh * G + G - h0);  // heads of this CTA
    const int b = blockIdx.z;
    const int s = s0 + warp;
    const bool row_valid = s < S;

    // this row's query vectors, as fp32
    for (int g = 0; g < nh; ++g)
        for (int d = lane; d < D; d += 32)
            qs[(warp * heads_here_max + g) * D + d] =
                row_valid ? load_as_float(p.q, b * p.q_sb + (int64_t)s * p.q_ss + (int64_t)(h0 + g) * p.q_sh + d,
                                          p.in_dtype)
                          : 0.f;

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
    const float sl2 = p.scale * kLog2e;
    float acc[kHeads][kMaxPerLane];
    float m[kHeads], l[kHeads];
#pragma unroll
    for (int g = 0; g < kHeads; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) acc[g][i] = 0.f;
    }
    const int64_t kbase = b * p.k_sb + (int64_t)kvh * p.k_sh;
    __syncthreads();
    for (int kb = cta_first; kb <= cta_last; kb += kTileKeys) {
        // stage 32 keys of K and V (fp32) for the whole CTA
        const int nk = min(kTileKeys, cta_last - kb + 1);
        for (int e = threadIdx.x; e < kTileKeys * D; e += blockDim.x) {
            const int j = e / D, d = e - j * D;
            float kv = 0.f, vv = 0.f;
            if (j < nk) {
                const int64_t r = kbase + (int64_t)(kb + j) * p.k_ss + d;
                kv = load_as_float(p.k, r, p.in_dtype);
                vv = load_as_float(p.v, r, p.in_dtype);
            }
            ks[j * Dp + d] = kv;
            vs[j * Dp + d] = vv;
        }
        __syncthreads();
        const int j = kb + lane;
        const bool vis = row_valid && j >= first && j <= last && j - kb < nk;
        const bool any = row_valid && kb <= last && kb + kTileKeys - 1 >= first;
        if (any) {
#pragma unroll
            for (int g = 0; g < kHeads; ++g) {
                if (g >= nh) break;
                float sc = -INFINITY;
                if (vis) {
                    if (uniform) {
                        sc = 0.f;
                    } else {
                        const float* qg = qs + (warp * heads_here_max + g) * D;
                        const float* kr = ks + lane * Dp;
                        float dot = 0.f;
                        for (int d = 0; d < D; ++d) dot = fmaf(qg[d], kr[d], dot);
                        if (p.mask != nullptr) sc = (dot * p.scale + p.mask[(int64_t)b * S + j]) * kLog2e;
                        else sc = dot * sl2;
                    }
                }
                const float mn = fmaxf(m[g], warp_max(sc));
                if (mn == -INFINITY) continue;  // nothing visible yet for this head (warp-uniform)
                const float corr = exp2f(m[g] - mn);
                const float pj = exp2f(sc - mn);
                l[g] = l[g] * corr + warp_sum(pj);
                m[g] = mn;
#pragma unroll
                for (int i = 0; i < kMaxPerLane; ++i) acc[g][i] *= corr;
                for (int jj = 0; jj < nk; ++jj) {
                    const float pw = __shfl_sync(0xffffffffu, pj, jj);
#pragma unroll
                    for (int i = 0; i < kMaxPerLane; ++i) {
                        const int d = lane + 32 * i;
                        if (d < D) acc[g][i] = fmaf(pw, vs[jj * Dp + d], acc[g][i]);
                    }
                }
            }
        }
        __syncthreads();
    }
    if (!row_valid) return;
#pragma unroll
    for (int g = 0; g < kHeads; ++g) {
        if (g >= nh) break;
        const float inv = 1.f / l[g];
        const int64_t qo = b * p.q_sb + (int64_t)s * p.q_ss + (int64_t)(h0 + g) * p.q_sh;
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) {
            const int d = lane + 32 * i;
            if (d < D) store_from_float(p.o, qo + d, acc[g][i] * inv, p.out_dtype);
        }
    }
}

}  // namespace

cudaError_t launch_attn_simt(const AttnParams& p, cudaStream_t stream) {
    const int G = p.Hq / p.Hkv;
    const int chunks = (G + kHeads - 1) / kHeads;
    const int heads_here_max = G < kHeads ? G : kHeads;
    const size_t smem = ((size_t)2 * kTileKeys * (p.D + 1) + (size_t)kRows * heads_here_max * p.D) * sizeof(float);
    if (smem > 48 * 1024) {
        const cudaError_t e =
            cudaFuncSetAttribute(attn_simt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    const dim3 grid((p.S + kRows - 1) / kRows, p.Hkv * chunks, p.B);
    attn_simt_kernel<<<grid, kRows * 32, smem, stream>>>(p, G, heads_here_max);
    return cudaGetLastError();
}

}  // namespace b2a
