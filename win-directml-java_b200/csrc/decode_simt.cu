// decode_simt.cu -- generic decode kernels: any even head_dim <= 256 and any
// cache type (float32 caches included).  They serve the reference's exact GPU
// contracts, which use float caches and small head dims:
//   ROPE_AND_APPEND_HLSL and GQA_ATTENTION_DECODE_HLSL (WB/windows/QwenAttentionShaders.java:82-263),
//   FUSED_ATTENTION_HLSL (INF/gemma/Gemma3WarpFusedAttentionContextKernel.java:32-86),
// and every b2a_decode shape without a tensor-core instantiation.
//
// One warp per (sequence, query head).  Keys are taken 32 at a time, one key
// per lane (full dot product per lane, q broadcast from shared memory), then
// the block of 32 probabilities is folded into the lane-owned output
// dimensions with shuffles.  Online softmax in fp32, base 2.
#include <math.h>

#include "common.cuh"
#include "internal.h"

namespace b2a {
namespace {

constexpr int kWarps = 4;
constexpr int kMaxPerLane = kMaxHeadDim / 32;

__device__ __forceinline__ bool seq_range(const DecodeParams& p, int b, int& L, int& first) {
    L = p.ctx_lens ? p.ctx_lens[b] : p.pos_scalar;
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

// Norm + RoPE of one head vector into vec[0..D) (float), whole warp.
__device__ void prep_head_generic(const DecodeParams& p, const void* src, int64_t off, int dtype,
                                  const float* bias, const float* norm_w, bool rope, int L, float* vec, int lane) {
    const int D = p.D;
    double ss = 0.0;
    for (int d = lane; d < D; d += 32) {
        float x = load_as_float(src, off + d, dtype);
        if (bias != nullptr) x = __fadd_rn(x, bias[d]);  // projection bias, fp32
        vec[d] = x;
        ss += (double)x * (double)x;
    }
    __syncwarp();
    if (norm_w != nullptr) {
        ss = warp_sum_d(ss);
        const float rms = (float)(1.0 / sqrt(__dadd_rn(ss / (double)D, (double)p.norm_eps)));
        for (int d = lane; d < D; d += 32)
            vec[d] = (float)__dmul_rn((double)__fmul_rn(vec[d], rms), __dadd_rn(1.0, (double)norm_w[d]));
        __syncwarp();
    }
    if (rope) {
        const int H = D / 2;
        for (int i = lane; i < H; i += 32) {
            double s, c;
            sincos((double)L * p.inv_freq[i], &s, &c);
            const float a = vec[i], b = vec[i + H];
            float y0, y1;
            if (p.rope_mode == 2) {
                y0 = (float)__dsub_rn(__dmul_rn((double)a, c), __dmul_rn((double)b, s));
                y1 = (float)__dadd_rn(__dmul_rn((double)b, c), __dmul_rn((double)a, s));
            } else {
                const float cf = (float)c, sf = (float)s;
                y0 = __fsub_rn(__fmul_rn(a, cf), __fmul_rn(b, sf));
                y1 = __fadd_rn(__fmul_rn(a, sf), __fmul_rn(b, cf));
            }
            vec[i] = y0;  // each pair is owned by exactly one lane
            vec[i + H] = y1;
        }
        __syncwarp();
    }
}

__global__ void __launch_bounds__(kWarps * 32) decode_simt_kernel(const __grid_constant__ DecodeParams p) {
    extern __shared__ float sm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int D = p.D;
    float* qv = sm + warp * 3 * D;
    float* kn = qv + D;
    float* vn = kn + D;
    const int task = blockIdx.x * kWarps + warp;
    if (task >= p.B * p.Hq) return;
    const int b = task / p.Hq, h = task - b * p.Hq;
    const int kvh = h / p.G;
    int L, first;
    if (!seq_range(p, b, L, first)) {
        for (int d = lane; d < D; d += 32)
            store_from_float(p.out, ((int64_t)b * p.Hq + h) * D + d, __int_as_float(0x7fc00000), p.out_dtype);
        if (lane == 0 && h == 0) atomicOr(p.status, 1);
        return;
    }
    const bool rope = p.append && p.rope_mode != 0;
    prep_head_generic(p, p.q, (int64_t)b * q_stride_of(p) + (int64_t)h * D, p.q_dtype,
                      p.q_bias ? p.q_bias + h * D : nullptr, p.append ? p.q_norm_w : nullptr, rope, L, qv, lane);
    const int64_t row0 = b * p.stride_b + kvh * p.stride_h;
    if (p.append) {
        prep_head_generic(p, p.k_new, (int64_t)b * kvn_stride_of(p) + (int64_t)kvh * D, p.q_dtype,
                          p.k_bias ? p.k_bias + kvh * D : nullptr, p.k_norm_w, rope, L, kn, lane);
        for (int d = lane; d < D; d += 32) {
            kn[d] = round_through(kn[d], p.cache_dtype);
            float vf = load_as_float(p.v_new, (int64_t)b * kvn_stride_of(p) + (int64_t)kvh * D + d, p.q_dtype);
            if (p.v_bias != nullptr) vf = __fadd_rn(vf, p.v_bias[kvh * D + d]);
            vn[d] = round_through(vf, p.cache_dtype);
            if (h % p.G == 0) {  // one writer per kv head; readers use kn/vn for row L
                store_from_float(p.k_cache, row0 + (int64_t)L * p.stride_pos + d, kn[d], p.cache_dtype);
                store_from_float(p.v_cache, row0 + (int64_t)L * p.stride_pos + d, vn[d], p.cache_dtype);
            }
        }
        __syncwarp();
    }
    const float sl2 = p.scale * kLog2e;
    float acc[kMaxPerLane];
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) acc[i] = 0.f;
    float m = -INFINITY, l = 0.f;
    for (int kb = first; kb <= L; kb += 32) {
        const int j = kb + lane;
        float s = -INFINITY;
        if (j <= L) {
            float dot = 0.f;
            if (p.append && j == L) {
                for (int d = 0; d < D; ++d) dot += qv[d] * kn[d];
            } else {
                const int64_t r = row0 + (int64_t)j * p.stride_pos;
                for (int d = 0; d < D; ++d) dot += qv[d] * load_as_float(p.k_cache, r + d, p.cache_dtype);
            }
            s = dot * sl2;
        }
        const float mb = warp_max(s);
        const float mn = fmaxf(m, mb);
        const float corr = exp2f(m - mn);
        const float pj = exp2f(s - mn);
        l = l * corr + warp_sum(pj);
        m = mn;
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) acc[i] *= corr;
        const int nk = min(32, L - kb + 1);
        for (int jj = 0; jj < nk; ++jj) {
            const float pw = __shfl_sync(0xffffffffu, pj, jj);
            const int key = kb + jj;
            const bool is_new = p.append && key == L;
            const int64_t r = row0 + (int64_t)key * p.stride_pos;
#pragma unroll
            for (int i = 0; i < kMaxPerLane; ++i) {
                const int d = lane + 32 * i;
                if (d < D) acc[i] += pw * (is_new ? vn[d] : load_as_float(p.v_cache, r + d, p.cache_dtype));
            }
        }
    }
    const float inv = 1.f / l;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
        const int d = lane + 32 * i;
        if (d < D) store_from_float(p.out, ((int64_t)b * p.Hq + h) * D + d, acc[i] * inv, p.out_dtype);
    }
}

// ROPE_AND_APPEND_HLSL equivalent: blocks [0, num_heads) rotate q heads in
// place, blocks [num_heads, num_heads+kv_heads) rotate k and write k, v rows
// into the head-major float caches at `pos`.
__global__ void qwen_rope_append_kernel(float* q, const float* k, const float* v, float* k_cache, float* v_cache,
                                        int num_heads, int head_dim, int pos, int max_seq,
                                        const __grid_constant__ DecodeParams freq) {
    const int head = blockIdx.x;
    const int half = head_dim / 2;
    for (int t = threadIdx.x; t < half; t += blockDim.x) {
        double s, c;
        sincos((double)pos * freq.inv_freq[t], &s, &c);
        const float cf = (float)c, sf = (float)s;
        if (head < num_heads) {
            float* qh = q + (int64_t)head * head_dim;
            const float x0 = qh[t], x1 = qh[half + t];
            qh[t] = __fsub_rn(__fmul_rn(x0, cf), __fmul_rn(x1, sf));
            qh[half + t] = __fadd_rn(__fmul_rn(x0, sf), __fmul_rn(x1, cf));
        } else {
            const int kvh = head - num_heads;
            const float* kh = k + (int64_t)kvh * head_dim;
            const float* vh = v + (int64_t)kvh * head_dim;
            const int64_t base = ((int64_t)kvh * max_seq + pos) * head_dim;
            const float k0 = kh[t], k1 = kh[half + t];
            k_cache[base + t] = __fsub_rn(__fmul_rn(k0, cf), __fmul_rn(k1, sf));
            k_cache[base + half + t] = __fadd_rn(__fmul_rn(k0, sf), __fmul_rn(k1, cf));
            v_cache[base + t] = vh[t];
            v_cache[base + half + t] = vh[half + t];
        }
    }
}

}  // namespace

cudaError_t launch_decode_simt(const DecodeParams& p, cudaStream_t stream) {
    const int tasks = p.B * p.Hq;
    const int grid = (tasks + kWarps - 1) / kWarps;
    const size_t smem = (size_t)kWarps * 3 * p.D * sizeof(float);
    decode_simt_kernel<<<grid, kWarps * 32, smem, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_qwen_rope_append(float* q, const float* k, const float* v, float* k_cache, float* v_cache,
                                    int num_heads, int kv_heads, int head_dim, int pos, int max_seq,
                                    const double* inv_freq, cudaStream_t stream) {
    DecodeParams freq{};
    for (int i = 0; i < head_dim / 2; ++i) freq.inv_freq[i] = inv_freq[i];
    const int threads = head_dim / 2 < 32 ? 32 : (head_dim / 2 > 128 ? 128 : head_dim / 2);
    qwen_rope_append_kernel<<<num_heads + kv_heads, threads, 0, stream>>>(q, k, v, k_cache, v_cache, num_heads,
                                                                         head_dim, pos, max_seq, freq);
    return cudaGetLastError();
}

}  // namespace b2a
