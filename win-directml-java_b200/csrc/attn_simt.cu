// attn_simt.cu -- generic whole-sequence attention (causal prefill and
// bidirectional encoder) for any element type and any even head_dim <= 256,
// computing in fp32.  It is the path of the reference's FLOAT32
// AttentionKernel contract (WB/runtime/kernels/AttentionKernel.java:19-24,
// DirectMlAttentionKernel validates FLOAT32 at L663-675) and of fp32 causal
// prefill (SmolLM2ReferenceForwardPass.runSelfAttention,
// INF/smollm2/SmolLM2ReferenceForwardPass.java:167-210); 16-bit inputs with a
// tensor-core instantiation take attn_mma.cu instead.
//
// One warp per (batch, query position, head).  Keys are processed 32 at a
// time, one key per lane; probabilities are folded into lane-owned output
// dimensions with shuffles.  q/k arrive already rotated when RoPE applies.
#include <math.h>

#include "common.cuh"
#include "internal.h"

namespace b2a {
namespace {

constexpr int kWarps = 4;
constexpr int kMaxPerLane = kMaxHeadDim / 32;

__global__ void __launch_bounds__(kWarps * 32) attn_simt_kernel(const __grid_constant__ AttnParams p) {
    extern __shared__ float sm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int D = p.D;
    float* qs = sm + warp * D;
    const int64_t task = (int64_t)blockIdx.x * kWarps + warp;
    if (task >= (int64_t)p.B * p.S * p.Hq) return;
    const int h = (int)(task % p.Hq);
    const int s = (int)((task / p.Hq) % p.S);
    const int b = (int)(task / ((int64_t)p.Hq * p.S));
    const int kvh = h / (p.Hq / p.Hkv);
    const int64_t qo = b * p.q_sb + s * p.q_ss + h * p.q_sh;
    const int64_t ko = b * p.k_sb + kvh * p.k_sh;
    for (int d = lane; d < D; d += 32) qs[d] = load_as_float(p.q, qo + d, p.in_dtype);
    __syncwarp();

    int first = 0, last = p.S - 1;
    bool uniform = false;  // every key masked: softmax over equal scores -> mean of V
    if (p.causal) {
        last = s;
        if (p.window > 0) first = max(0, s - p.window + 1);
    } else if (p.key_len != nullptr) {
        const int kl = p.key_len[b];
        if (kl <= 0) uniform = true;
        else last = min(kl, p.S) - 1;
    }
    const float sl2 = p.scale * kLog2e;
    float acc[kMaxPerLane];
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) acc[i] = 0.f;
    float m = -INFINITY, l = 0.f;
    for (int kb = first; kb <= last; kb += 32) {
        const int j = kb + lane;
        float sc = -INFINITY;
        if (j <= last) {
            if (uniform) {
                sc = 0.f;
            } else {
                const int64_t r = ko + (int64_t)j * p.k_ss;
                float dot = 0.f;
                for (int d = 0; d < D; ++d) dot += qs[d] * load_as_float(p.k, r + d, p.in_dtype);
                if (p.mask != nullptr) sc = (dot * p.scale + p.mask[(int64_t)b * p.S + j]) * kLog2e;
                else sc = dot * sl2;
            }
        }
        const float mb = warp_max(sc);
        const float mn = fmaxf(m, mb);
        const float corr = exp2f(m - mn);
        const float pj = exp2f(sc - mn);
        l = l * corr + warp_sum(pj);
        m = mn;
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) acc[i] *= corr;
        const int nk = min(32, last - kb + 1);
        for (int jj = 0; jj < nk; ++jj) {
            const float pw = __shfl_sync(0xffffffffu, pj, jj);
            const int64_t r = ko + (int64_t)(kb + jj) * p.k_ss;
#pragma unroll
            for (int i = 0; i < kMaxPerLane; ++i) {
                const int d = lane + 32 * i;
                if (d < D) acc[i] += pw * load_as_float(p.v, r + d, p.in_dtype);
            }
        }
    }
    const float inv = 1.f / l;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
        const int d = lane + 32 * i;
        if (d < D) store_from_float(p.o, qo + d, acc[i] * inv, p.out_dtype);
    }
}

}  // namespace

cudaError_t launch_attn_simt(const AttnParams& p, cudaStream_t stream) {
    const int64_t tasks = (int64_t)p.B * p.S * p.Hq;
    const int64_t grid = (tasks + kWarps - 1) / kWarps;
    const size_t smem = (size_t)kWarps * p.D * sizeof(float);
    attn_simt_kernel<<<(unsigned)grid, kWarps * 32, smem, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace b2a
