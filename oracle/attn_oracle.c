/*
 * attn_oracle.c -- CPU restatement of win-directml-java's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library under win-directml-java_b200/.  Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline / reference arm may load it; the product path
 * never calls it and has no CPU fallback.
 *
 * Parity pinning.  The reference is Java 21 (no JDK exists on the build or GPU
 * machines), so this is a restatement, not the reference run.  It is pinned
 * against the reference's own known-answer tests (RoPE identity / on-the-fly
 * angle, zero-centred RMSNorm closed form, GQA and window layout values,
 * softmax properties) and against the in-test CPU references of its GPU tests,
 * re-run on inputs regenerated with a port of java.util.Random (same seeds).
 * The reference holds no numeric golden attention vectors.
 *
 * Float semantics.  Java float arithmetic is IEEE single precision without
 * fused multiply-add contraction; this file is compiled with
 * -ffp-contract=off so every `a * b + c` rounds twice, as in Java.  Where the
 * reference widens to double, the same expressions are written in double.
 *
 * Citations use paths inside the reference project with these prefixes:
 *   INF/ = directml-inference/src/main/java/com/aresstack/windirectml/inference/
 *   ENC/ = directml-encoder/src/main/java/com/aresstack/windirectml/encoder/
 *   WB/  = directml-windows-bindings/src/main/java/com/aresstack/windirectml/
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* dtype rounding (round-to-nearest-even), used to store appended cache rows */
/* ------------------------------------------------------------------------ */

enum { ORC_F32 = 0, ORC_F16 = 1, ORC_BF16 = 2 };

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* IEEE binary16 encode with round-to-nearest-even, written from the format
 * definition: 1 sign bit, 5 exponent bits (bias 15), 10 fraction bits. */
ORC_API uint16_t orc_f32_to_f16_bits(float f) {
    uint32_t x = f2u(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (exp == 0xffu) { /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0u));
    }
    int e = (int)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u); /* overflow -> inf */
    if (e <= 0) {
        /* subnormal half (or zero): value = man_with_hidden * 2^(e-1-10) */
        if (e < -10) return (uint16_t)sign;
        uint32_t m = man | 0x800000u;
        int shift = 14 - e; /* 24-bit mantissa down to the subnormal grid */
        uint32_t half = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t mid = 1u << (shift - 1);
        if (rem > mid || (rem == mid && (half & 1u))) half++;
        return (uint16_t)(sign | half);
    }
    uint32_t half = sign | ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (half & 1u))) half++; /* may carry into exp: correct */
    return (uint16_t)half;
}

ORC_API float orc_f16_bits_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    if (exp == 0) {
        if (man == 0) return u2f(sign);
        /* subnormal: man * 2^-24 */
        float v = (float)man * 5.9604644775390625e-8f;
        return sign ? -v : v;
    }
    if (exp == 31) return u2f(sign | 0x7f800000u | (man << 13));
    return u2f(sign | ((exp - 15 + 127) << 23) | (man << 13));
}

ORC_API uint16_t orc_f32_to_bf16_bits(float f) {
    uint32_t x = f2u(f);
    if ((x & 0x7f800000u) == 0x7f800000u && (x & 0x7fffffu)) return (uint16_t)((x >> 16) | 0x40u);
    uint32_t lsb = (x >> 16) & 1u;
    x += 0x7fffu + lsb;
    return (uint16_t)(x >> 16);
}

ORC_API float orc_bf16_bits_to_f32(uint16_t b) { return u2f((uint32_t)b << 16); }

ORC_API float orc_round_to(float f, int dtype) {
    if (dtype == ORC_F16) return orc_f16_bits_to_f32(orc_f32_to_f16_bits(f));
    if (dtype == ORC_BF16) return orc_bf16_bits_to_f32(orc_f32_to_bf16_bits(f));
    return f;
}

ORC_API void orc_round_array(float* x, int64_t n, int dtype) {
    if (dtype == ORC_F32) return;
    for (int64_t i = 0; i < n; ++i) x[i] = orc_round_to(x[i], dtype);
}

/* ------------------------------------------------------------------------ */
/* a1: DecoderOnlyRotaryEmbedding (INF/decoderonly/DecoderOnlyRotaryEmbedding.java:13-67)
 * NeoX half rotation over pairs (x[i], x[i+D/2]); angle = pos * (1/theta^(2i/D))
 * in double; cos/sin rounded to float (table or on the fly give the same
 * floats); the rotation itself is float arithmetic.                          */
/* ------------------------------------------------------------------------ */
static inline double decoderonly_angle(int pos, int i, int head_dim, double theta) {
    /* DecoderOnlyRotaryEmbedding.java:57-59 */
    return pos * (1.0 / pow(theta, (2.0 * i) / head_dim));
}

ORC_API void orc_rope_decoderonly(float* x, int n_heads, int head_dim, int pos, double theta) {
    int half = head_dim / 2;
    for (int h = 0; h < n_heads; ++h) {
        float* v = x + (int64_t)h * head_dim;
        for (int i = 0; i < half; ++i) {
            double a = decoderonly_angle(pos, i, head_dim, theta);
            float c = (float)cos(a), s = (float)sin(a);
            float x0 = v[i], x1 = v[half + i];
            /* DecoderOnlyRotaryEmbedding.java:61-67 */
            v[i] = x0 * c - x1 * s;
            v[half + i] = x0 * s + x1 * c;
        }
    }
}

/* a2: Gemma3ReferenceMath.applyRopeHalf (INF/gemma/Gemma3ReferenceMath.java:65-83):
 * cos/sin and the products in double, then rounded to float.               */
ORC_API void orc_rope_half_gemma(float* x, int n_heads, int head_dim, int pos, double theta) {
    int half = head_dim / 2;
    for (int h = 0; h < n_heads; ++h) {
        float* v = x + (int64_t)h * head_dim;
        for (int i = 0; i < half; ++i) {
            double inv_freq = 1.0 / pow(theta, (2.0 * i) / head_dim);
            double angle = pos * inv_freq;
            double c = cos(angle), s = sin(angle);
            float x1 = v[i], x2 = v[i + half];
            v[i] = (float)(x1 * c - x2 * s);
            v[i + half] = (float)(x2 * c + x1 * s);
        }
    }
}

/* a3: Gemma3ReferenceMath.rmsNormZeroCentered (INF/gemma/Gemma3ReferenceMath.java:25-46),
 * applied per head as QK-norm (INF/gemma/Gemma3ReferenceForwardPass.java:134-141). */
ORC_API void orc_rmsnorm_zero_centered(float* x, int n_heads, int head_dim, const float* w, float eps) {
    for (int h = 0; h < n_heads; ++h) {
        float* v = x + (int64_t)h * head_dim;
        double sum_sq = 0;
        for (int i = 0; i < head_dim; ++i) {
            double d = v[i];
            sum_sq += d * d;
        }
        float rms = (float)(1.0 / sqrt(sum_sq / head_dim + (double)eps));
        for (int i = 0; i < head_dim; ++i) v[i] = (float)((double)(v[i] * rms) * (1.0 + (double)w[i]));
    }
}

/* a5: DecoderOnlyMath.softmax (INF/decoderonly/DecoderOnlyMath.java:60-79):
 * float max, exp through double, FLOAT running sum, multiply by 1/sum.      */
ORC_API void orc_softmax_decoderonly(float* v, int n) {
    float mx = -INFINITY;
    for (int i = 0; i < n; ++i) if (v[i] > mx) mx = v[i];
    float sum = 0;
    for (int i = 0; i < n; ++i) {
        v[i] = (float)exp((double)(v[i] - mx));
        sum += v[i];
    }
    float inv = 1.0f / sum;
    for (int i = 0; i < n; ++i) v[i] *= inv;
}

/* scalar float dot in source order: SmolLM2ReferenceForwardPass.dotHead
 * (INF/smollm2/SmolLM2ReferenceForwardPass.java:292-300) and
 * Gemma3ReferenceForwardPass.dot (INF/gemma/Gemma3ReferenceForwardPass.java:211-217). */
static inline float dot_f(const float* a, const float* b, int n) {
    float s = 0.0f;
    for (int i = 0; i < n; ++i) s += a[i] * b[i];
    return s;
}

/* ------------------------------------------------------------------------ */
/* Softmax-accumulate semantics used by the decoder variants.                */
/* ------------------------------------------------------------------------ */
enum {
    /* SmolLM2 / Qwen2 / Phi-3: DecoderOnlyMath.softmax (float sum), then
     * context += p * V in float (SmolLM2ReferenceForwardPass.java:193-205,
     * Qwen2Runtime.java:756-764).                                          */
    ORC_SOFTMAX_DECODERONLY = 0,
    /* Gemma 3: float max, double exp sum, float 1/sum, float p * V
     * (INF/gemma/Gemma3ReferenceForwardPass.java:151-172).                 */
    ORC_SOFTMAX_GEMMA = 1
};

/* One query head attending keys [first, last] of a cache view.  kv_at(j)
 * returns the float row of key/value position j for this kv head.          */
static void attend_one(const float* q, int head_dim, float scale,
                       const float* k_base, const float* v_base, int64_t row_stride,
                       int first, int last, int softmax_mode, int skip_small,
                       float* scores, float* out) {
    int n = last - first + 1;
    for (int d = 0; d < head_dim; ++d) out[d] = 0.0f;
    if (n <= 0) return;
    if (softmax_mode == ORC_SOFTMAX_DECODERONLY) {
        for (int j = 0; j < n; ++j) scores[j] = dot_f(q, k_base + (int64_t)(first + j) * row_stride, head_dim) * scale;
        orc_softmax_decoderonly(scores, n);
        for (int j = 0; j < n; ++j) {
            float w = scores[j];
            if (skip_small && w < 1e-8f) continue; /* Qwen2Runtime.java:762 / Phi3Runtime.java:651 */
            const float* vr = v_base + (int64_t)(first + j) * row_stride;
            for (int d = 0; d < head_dim; ++d) out[d] += w * vr[d];
        }
    } else {
        float mx = -INFINITY;
        for (int j = 0; j < n; ++j) {
            float sc = dot_f(q, k_base + (int64_t)(first + j) * row_stride, head_dim) * scale;
            scores[j] = sc;
            if (sc > mx) mx = sc;
        }
        double sum = 0;
        for (int j = 0; j < n; ++j) {
            double e = exp((double)(scores[j] - mx));
            scores[j] = (float)e;
            sum += e;
        }
        float inv = (float)(1.0 / sum);
        for (int j = 0; j < n; ++j) {
            float a = scores[j] * inv;
            const float* vr = v_base + (int64_t)(first + j) * row_stride;
            for (int d = 0; d < head_dim; ++d) out[d] += a * vr[d];
        }
    }
}

/* ------------------------------------------------------------------------ */
/* a6/a7/a9: causal GQA prefill.                                             */
/* SmolLM2ReferenceForwardPass.runSelfAttention (INF/smollm2/SmolLM2ReferenceForwardPass.java:167-210):
 *   RoPE every q and k head at its position (DecoderOnlyRotaryEmbedding),
 *   kvHead = qHead / (Hq/Hkv) (INF/decoderonly/DecoderOnlyAttentionLayout.java:43-53),
 *   scores over source positions 0..pos, DecoderOnlyMath.softmax, float accumulation.
 * Qwen2Runtime.processLayerPrefill (INF/qwen/Qwen2Runtime.java:916-971) has the
 * same math with positions startPos+s, parallel over (s, h).
 * Layout: q [B][S][Hq][D], k/v [B][S][Hkv][D], out [B][S][Hq][D], all float.
 * rope_theta <= 0 disables RoPE.  window > 0 limits keys to
 * [max(0, t-window+1), t] (Gemma3AttentionLayout.firstValidKey,
 * INF/gemma/Gemma3AttentionLayout.java:57-62).  causal == 0 gives
 * bidirectional attention over all S keys.                                 */
/* ------------------------------------------------------------------------ */
ORC_API int orc_prefill(const float* q_in, const float* k_in, const float* v_in, float* out,
                        int B, int S, int Hq, int Hkv, int D, float scale,
                        double rope_theta, int pos0, int window, int causal,
                        int softmax_mode, int skip_small, int n_threads) {
    if (Hkv <= 0 || Hq % Hkv != 0 || D <= 0 || (D & 1)) return -1;
    int G = Hq / Hkv;
    int64_t q_row = (int64_t)Hq * D, kv_row = (int64_t)Hkv * D;
    float* q = (float*)malloc(sizeof(float) * (size_t)B * S * q_row);
    float* k = (float*)malloc(sizeof(float) * (size_t)B * S * kv_row);
    if (!q || !k) { free(q); free(k); return -2; }
    memcpy(q, q_in, sizeof(float) * (size_t)B * S * q_row);
    memcpy(k, k_in, sizeof(float) * (size_t)B * S * kv_row);
    if (rope_theta > 0) {
        for (int b = 0; b < B; ++b)
            for (int s = 0; s < S; ++s) {
                orc_rope_decoderonly(q + ((int64_t)b * S + s) * q_row, Hq, D, pos0 + s, rope_theta);
                orc_rope_decoderonly(k + ((int64_t)b * S + s) * kv_row, Hkv, D, pos0 + s, rope_theta);
            }
    }
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#endif
    int64_t tasks = (int64_t)B * S * Hq;
#pragma omp parallel
    {
        float* scores = (float*)malloc(sizeof(float) * (size_t)S);
#pragma omp for schedule(dynamic, 16)
        for (int64_t idx = 0; idx < tasks; ++idx) {
            int h = (int)(idx % Hq);
            int s = (int)((idx / Hq) % S);
            int b = (int)(idx / ((int64_t)Hq * S));
            int kvh = h / G;
            int first = 0, last = S - 1;
            if (causal) {
                last = s;
                if (window > 0) first = s - window + 1 > 0 ? s - window + 1 : 0;
            }
            const float* qr = q + ((int64_t)b * S + s) * q_row + (int64_t)h * D;
            const float* kb = k + (int64_t)b * S * kv_row + (int64_t)kvh * D;
            const float* vb = v_in + (int64_t)b * S * kv_row + (int64_t)kvh * D;
            attend_one(qr, D, scale, kb, vb, kv_row, first, last, softmax_mode, skip_small, scores,
                       out + ((int64_t)b * S + s) * q_row + (int64_t)h * D);
        }
        free(scores);
    }
    free(q);
    free(k);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* a7/a10/a14/a15: single-token decode over a KV cache.                      */
/* Per sequence b with L = ctx_lens[b] tokens already cached:
 *   optional QK-norm of the new q and k heads (Gemma3ReferenceForwardPass.java:134-141),
 *   RoPE at position L (DecoderOnly rotation for rope_mode 0,
 *   Gemma applyRopeHalf for rope_mode 1),
 *   append k, v at position L (Qwen2Runtime.java:733-738), the cache row
 *   rounded to the cache dtype,
 *   attention of every q head over keys [first, L] where first = 0 or
 *   max(0, L-window+1) (Gemma3AttentionLayout.java:57-62).
 * Cache layouts: 0 = head-major [B][Hkv][max_seq][D]
 * (INF/decoderonly/DecoderOnlyKvCacheLayout.java:53-59), 1 = position-major
 * [B][max_seq][Hkv][D] (INF/decoderonly/DecoderOnlyWarpLayerKvCache.java:13-45).
 * The caches are float arrays holding values already representable in
 * cache_dtype; they are modified in place (the appended row).              */
/* ------------------------------------------------------------------------ */
ORC_API int orc_decode(const float* q_new, const float* k_new, const float* v_new,
                       float* k_cache, float* v_cache, int cache_layout, int cache_dtype,
                       const int32_t* ctx_lens, int B, int Hq, int Hkv, int D, int max_seq,
                       float scale, double rope_theta, int rope_mode, int window,
                       const float* q_norm_w, const float* k_norm_w, float norm_eps,
                       int softmax_mode, int skip_small, float* out, int n_threads) {
    if (Hkv <= 0 || Hq % Hkv != 0 || D <= 0 || (D & 1)) return -1;
    int G = Hq / Hkv;
    for (int b = 0; b < B; ++b)
        if (ctx_lens[b] < 0 || ctx_lens[b] >= max_seq) return -3;
    int64_t seq_stride = (int64_t)Hkv * max_seq * D;
    int64_t head_stride = cache_layout == 0 ? (int64_t)max_seq * D : D;
    int64_t row_stride = cache_layout == 0 ? D : (int64_t)Hkv * D;
    float* qbuf = (float*)malloc(sizeof(float) * (size_t)B * Hq * D);
    float* kbuf = (float*)malloc(sizeof(float) * (size_t)Hkv * D);
    if (!qbuf || !kbuf) { free(qbuf); free(kbuf); return -2; }
    memcpy(qbuf, q_new, sizeof(float) * (size_t)B * Hq * D);
    for (int b = 0; b < B; ++b) {
        int L = ctx_lens[b];
        float* qb = qbuf + (int64_t)b * Hq * D;
        memcpy(kbuf, k_new + (int64_t)b * Hkv * D, sizeof(float) * (size_t)Hkv * D);
        if (q_norm_w) orc_rmsnorm_zero_centered(qb, Hq, D, q_norm_w, norm_eps);
        if (k_norm_w) orc_rmsnorm_zero_centered(kbuf, Hkv, D, k_norm_w, norm_eps);
        if (rope_theta > 0) {
            if (rope_mode == 1) {
                orc_rope_half_gemma(qb, Hq, D, L, rope_theta);
                orc_rope_half_gemma(kbuf, Hkv, D, L, rope_theta);
            } else {
                orc_rope_decoderonly(qb, Hq, D, L, rope_theta);
                orc_rope_decoderonly(kbuf, Hkv, D, L, rope_theta);
            }
        }
        for (int kvh = 0; kvh < Hkv; ++kvh) {
            float* kr = k_cache + b * seq_stride + kvh * head_stride + (int64_t)L * row_stride;
            float* vr = v_cache + b * seq_stride + kvh * head_stride + (int64_t)L * row_stride;
            for (int d = 0; d < D; ++d) {
                kr[d] = orc_round_to(kbuf[(int64_t)kvh * D + d], cache_dtype);
                vr[d] = orc_round_to(v_new[((int64_t)b * Hkv + kvh) * D + d], cache_dtype);
            }
        }
    }
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#endif
    int64_t tasks = (int64_t)B * Hq;
#pragma omp parallel
    {
        float* scores = (float*)malloc(sizeof(float) * (size_t)max_seq);
#pragma omp for schedule(dynamic, 1)
        for (int64_t idx = 0; idx < tasks; ++idx) {
            int b = (int)(idx / Hq), h = (int)(idx % Hq);
            int kvh = h / G;
            int L = ctx_lens[b];
            int first = window > 0 ? (L - window + 1 > 0 ? L - window + 1 : 0) : 0;
            const float* kb = k_cache + b * seq_stride + kvh * head_stride;
            const float* vb = v_cache + b * seq_stride + kvh * head_stride;
            attend_one(qbuf + ((int64_t)b * Hq + h) * D, D, scale, kb, vb, row_stride, first, L,
                       softmax_mode, skip_small, scores, out + ((int64_t)b * Hq + h) * D);
        }
        free(scores);
    }
    free(qbuf);
    free(kbuf);
    return 0;
}

/* Attention of q [B][Hq][D] over an existing cache with no append: keys
 * [first, last_pos[b]] where first = first_explicit (>= 0) or the window rule.
 * This is the CPU side of the reference's GPU decode contracts: the test
 * reference of GQA_ATTENTION_DECODE_HLSL (QwenAttentionShadersGpuTest.java:233-256,
 * directml-windows-bindings/src/test/java/com/aresstack/windirectml/windows/)
 * and the Gemma attention the fused context kernel is checked against
 * (INF/gemma/Gemma3ReferenceForwardPass.java:144-172).                     */
ORC_API int orc_attend_cache(const float* q, const float* k_cache, const float* v_cache, int cache_layout,
                             const int32_t* last_pos, int B, int Hq, int Hkv, int D, int max_seq, float scale,
                             int window, int first_explicit, int softmax_mode, float* out, int n_threads) {
    if (Hkv <= 0 || Hq % Hkv != 0 || D <= 0) return -1;
    int G = Hq / Hkv;
    for (int b = 0; b < B; ++b)
        if (last_pos[b] < 0 || last_pos[b] >= max_seq) return -3;
    int64_t seq_stride = (int64_t)Hkv * max_seq * D;
    int64_t head_stride = cache_layout == 0 ? (int64_t)max_seq * D : D;
    int64_t row_stride = cache_layout == 0 ? D : (int64_t)Hkv * D;
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#endif
#pragma omp parallel
    {
        float* scores = (float*)malloc(sizeof(float) * (size_t)max_seq);
#pragma omp for schedule(dynamic, 1)
        for (int64_t idx = 0; idx < (int64_t)B * Hq; ++idx) {
            int b = (int)(idx / Hq), h = (int)(idx % Hq);
            int kvh = h / G;
            int L = last_pos[b];
            int first;
            if (first_explicit >= 0) first = first_explicit < L ? first_explicit : L;
            else first = window > 0 ? (L - window + 1 > 0 ? L - window + 1 : 0) : 0;
            attend_one(q + idx * D, D, scale, k_cache + b * seq_stride + kvh * head_stride,
                       v_cache + b * seq_stride + kvh * head_stride, row_stride, first, L, softmax_mode, 0, scores,
                       out + idx * D);
        }
        free(scores);
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* a11: CpuMiniLmEncoder.multiHeadAttention (ENC/minilm/CpuMiniLmEncoder.java:318-375),
 * identical to CpuBertEncoder.multiHeadAttention (ENC/bert/CpuBertEncoder.java:193-235):
 * double dot of float products, score := -1e9 where the key is masked, float
 * max, double exp sum, inv = 1/max(sum,1e-12) in float, double P.V.
 * The reference runs one text at a time in [S][H*D]; here a batch of texts
 * with per-text key lengths (key j valid iff j < key_len[b]).  layout 0 =
 * head-major [B][H][S][D], 1 = sequence-major [B][S][H][D].               */
/* ------------------------------------------------------------------------ */
ORC_API int orc_encoder_minilm(const float* q, const float* k, const float* v,
                               const int32_t* key_len, float* out,
                               int B, int H, int S, int D, int layout, int n_threads) {
    double scale = 1.0 / sqrt((double)D);
    int64_t sS = layout == 0 ? D : (int64_t)H * D;    /* stride between positions */
    int64_t sH = layout == 0 ? (int64_t)S * D : D;    /* stride between heads */
    int64_t sB = (int64_t)H * S * D;
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#endif
#pragma omp parallel
    {
        float* sc = (float*)malloc(sizeof(float) * (size_t)S * S);
#pragma omp for schedule(dynamic, 1)
        for (int64_t bh = 0; bh < (int64_t)B * H; ++bh) {
            int b = (int)(bh / H), h = (int)(bh % H);
            const float* qb = q + b * sB + h * sH;
            const float* kb = k + b * sB + h * sH;
            const float* vb = v + b * sB + h * sH;
            float* ob = out + b * sB + h * sH;
            int kl = key_len ? key_len[b] : S;
            for (int i = 0; i < S; ++i)
                for (int j = 0; j < S; ++j) {
                    double sum = 0.0;
                    for (int d = 0; d < D; ++d) sum += qb[i * sS + d] * kb[j * sS + d];
                    double score = sum * scale;
                    if (j >= kl) score = -1e9;
                    sc[(int64_t)i * S + j] = (float)score;
                }
            for (int i = 0; i < S; ++i) {
                float* row = sc + (int64_t)i * S;
                float mx = -INFINITY;
                for (int j = 0; j < S; ++j) if (row[j] > mx) mx = row[j];
                double sum = 0.0;
                for (int j = 0; j < S; ++j) {
                    double e = exp((double)(row[j] - mx));
                    row[j] = (float)e;
                    sum += e;
                }
                float inv = (float)(1.0 / (sum > 1e-12 ? sum : 1e-12));
                for (int j = 0; j < S; ++j) row[j] *= inv;
            }
            for (int i = 0; i < S; ++i)
                for (int d = 0; d < D; ++d) {
                    double sum = 0.0;
                    for (int j = 0; j < S; ++j) sum += sc[(int64_t)i * S + j] * vb[j * sS + d];
                    ob[i * sS + d] = (float)sum;
                }
        }
        free(sc);
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* a12: AttentionKernel.dispatch contract (WB/runtime/kernels/AttentionKernel.java:19-24)
 * as pinned by DirectMlAttentionKernelTest.cpuAttention
 * (directml-windows-bindings/src/test/java/com/aresstack/windirectml/runtime/kernels/
 *  DirectMlAttentionKernelTest.java:129-175): [B,H,S,D] head-major, optional
 * additive mask [B,S] broadcast over heads and queries; score =
 * (float)(double-dot * scale) + mask; float max; double exp sum; float 1/sum;
 * double P.V.                                                              */
/* ------------------------------------------------------------------------ */
ORC_API int orc_mha_additive(const float* q, const float* k, const float* v, const float* mask,
                             float* y, int B, int H, int S, int D, float scale, int n_threads) {
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#endif
#pragma omp parallel
    {
        float* sc = (float*)malloc(sizeof(float) * (size_t)S * S);
#pragma omp for schedule(dynamic, 1)
        for (int64_t bh = 0; bh < (int64_t)B * H; ++bh) {
            int b = (int)(bh / H);
            const float* qb = q + bh * S * D;
            const float* kb = k + bh * S * D;
            const float* vb = v + bh * S * D;
            float* yb = y + bh * S * D;
            for (int i = 0; i < S; ++i)
                for (int j = 0; j < S; ++j) {
                    double s = 0.0;
                    for (int d = 0; d < D; ++d) s += qb[(int64_t)i * D + d] * kb[(int64_t)j * D + d];
                    float f = (float)(s * scale);
                    if (mask) f += mask[(int64_t)b * S + j];
                    sc[(int64_t)i * S + j] = f;
                }
            for (int i = 0; i < S; ++i) {
                float* row = sc + (int64_t)i * S;
                float mx = -INFINITY;
                for (int j = 0; j < S; ++j) mx = row[j] > mx ? row[j] : mx;
                double sum = 0.0;
                for (int j = 0; j < S; ++j) {
                    double e = exp((double)(row[j] - mx));
                    row[j] = (float)e;
                    sum += e;
                }
                float inv = (float)(1.0 / sum);
                for (int j = 0; j < S; ++j) row[j] *= inv;
            }
            for (int i = 0; i < S; ++i)
                for (int d = 0; d < D; ++d) {
                    double s = 0.0;
                    for (int j = 0; j < S; ++j) s += sc[(int64_t)i * S + j] * vb[(int64_t)j * D + d];
                    yb[(int64_t)i * D + d] = (float)s;
                }
        }
        free(sc);
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* a4: layout helpers (exposed so the known-answer tests can call them).     */
/* ------------------------------------------------------------------------ */
/* DecoderOnlyAttentionLayout.kvHeadForQueryHead (INF/decoderonly/DecoderOnlyAttentionLayout.java:12-53):
 * returns -1 where the reference throws IllegalArgumentException.          */
ORC_API int orc_kv_head_for_query_head(int n_q, int n_kv, int q_head) {
    if (n_q <= 0 || n_kv <= 0 || n_q % n_kv != 0) return -1;
    if (q_head < 0 || q_head >= n_q) return -1;
    return q_head / (n_q / n_kv);
}

/* Gemma3AttentionLayout.firstValidKey (INF/gemma/Gemma3AttentionLayout.java:57-62). */
ORC_API int orc_first_valid_key(int full_attention, int window, int query_pos) {
    if (full_attention || window <= 0) return 0;
    int f = query_pos - window + 1;
    return f > 0 ? f : 0;
}

/* Gemma3Config.isFullAttentionLayer without an explicit layer_types list
 * (INF/gemma/Gemma3Config.java:73-81): every pattern-th layer is global. */
ORC_API int orc_is_full_attention_layer(int layer, int pattern) {
    if (pattern > 0) return (layer + 1) % pattern == 0;
    return 1;
}

/* Gemma3Config.ropeThetaForLayer (INF/gemma/Gemma3Config.java:84-86). */
ORC_API double orc_rope_theta_for_layer(int layer, int pattern, double theta_global, double theta_local) {
    return orc_is_full_attention_layer(layer, pattern) ? theta_global : theta_local;
}

/* Gemma3Config.attentionScale (INF/gemma/Gemma3Config.java:57-61), as the
 * float Gemma3AttentionLayout.attentionScale returns (L49-51). */
ORC_API float orc_attention_scale(double query_pre_attn_scalar, int head_dim) {
    double scalar = query_pre_attn_scalar > 0 ? query_pre_attn_scalar : head_dim;
    return (float)(1.0 / sqrt(scalar));
}

ORC_API int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
