// rope.cu -- RoPE pre-pass for prefill: rotates q or k rows of a [B][S][H][D]
// tensor (any strides) at positions pos0 + s and writes them, possibly in
// another element type, to a destination (which may alias the source).
// Angles: pos * inv_freq[i] in double with inv_freq = 1 / theta^(2i/D) from
// the host, as DecoderOnlyRotaryEmbedding.positionAngle
// (INF/decoderonly/DecoderOnlyRotaryEmbedding.java:57-59).  cos/sin of each
// (position, pair) are taken once into a table, then applied to every head.
#include <math.h>

#include "common.cuh"
#include "internal.h"

namespace b2a {
namespace {

struct FreqTable {
    double inv_freq[kMaxHeadDim / 2];
};

// table[s][i] = (cos, sin) of (pos0 + s) * inv_freq[i], double.
__global__ void rope_table_kernel(double2* table, int S, int half, int pos0, const __grid_constant__ FreqTable f) {
    const int64_t n = (int64_t)S * half;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int s = (int)(e / half), i = (int)(e - (int64_t)s * half);
        double sn, cn;
        sincos((double)(pos0 + s) * f.inv_freq[i], &sn, &cn);
        table[e] = make_double2(cn, sn);
    }
}

// Same angles, stored as the float (cos, sin) the NeoX rotation multiplies with
// (the double values rounded to float): half the bytes of the double table.
__global__ void rope_table_f32_kernel(float2* table, int S, int half, int pos0, const __grid_constant__ FreqTable f) {
    const int64_t n = (int64_t)S * half;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int s = (int)(e / half), i = (int)(e - (int64_t)s * half);
        double sn, cn;
        sincos((double)(pos0 + s) * f.inv_freq[i], &sn, &cn);
        table[e] = make_float2((float)cn, (float)sn);
    }
}

// Flags (status bit 2) a finite input that became infinite in the
// destination type: bf16 operands above the fp16 range.
__device__ __forceinline__ void flag_overflow(float in, float out, int* status) {
    if (status != nullptr && isinf(out) && !isinf(in)) atomicOr(status, 4);
}

__global__ void convert_kernel(const void* src, int src_dtype, void* dst, int dst_dtype, int64_t n, int* status) {
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const float x = load_as_float(src, e, src_dtype);
        store_from_float(dst, e, x, dst_dtype);
        flag_overflow(x, round_through(x, dst_dtype), status);
    }
}

__global__ void rope_rows_kernel(const void* src, int src_dtype, void* dst, int dst_dtype, int S, int H, int D,
                                 int64_t sb, int64_t ss, int64_t sh, int64_t db, int64_t ds, int64_t dh,
                                 int64_t rows, int rope_mode, const double2* table, int* status) {
    const int half = D / 2;
    const int64_t pairs = rows * half;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < pairs; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = e / half;
        const int i = (int)(e - row * half);
        const int h = (int)(row % H);
        const int s = (int)((row / H) % S);
        const int64_t b = row / ((int64_t)H * S);
        const int64_t so = b * sb + s * ss + h * sh;
        const int64_t dofs = b * db + s * ds + h * dh;
        const float a = load_as_float(src, so + i, src_dtype);
        const float c2 = load_as_float(src, so + i + half, src_dtype);
        const double2 cs = table[(int64_t)s * half + i];
        float y0, y1;
        if (rope_mode == 2) {
            y0 = (float)__dsub_rn(__dmul_rn((double)a, cs.x), __dmul_rn((double)c2, cs.y));
            y1 = (float)__dadd_rn(__dmul_rn((double)c2, cs.x), __dmul_rn((double)a, cs.y));
        } else {
            const float cf = (float)cs.x, sf = (float)cs.y;
            y0 = __fsub_rn(__fmul_rn(a, cf), __fmul_rn(c2, sf));
            y1 = __fadd_rn(__fmul_rn(a, sf), __fmul_rn(c2, cf));
        }
        store_from_float(dst, dofs + i, y0, dst_dtype);
        store_from_float(dst, dofs + i + half, y1, dst_dtype);
        flag_overflow(y0, round_through(y0, dst_dtype), status);
        flag_overflow(y1, round_through(y1, dst_dtype), status);
    }
}

// ---------------------------------------------------------------- vectorised pre-pass
// One launch prepares all operands of a prefill: rows of q and k are rotated
// (and converted), v is converted; every thread moves 8 elements of each half
// of a row (16-byte accesses for 16-bit types).
struct PrepSeg {
    const void* src;
    void* dst;       // compute dtype
    void* dst_in;    // optional second copy in the input dtype (rotated keys for the caller)
    int64_t units;   // rotated: B * S * head groups * (D/2)/8; plain: elements / 8
    int H;
    int rotate;
};
struct PrepParams {
    PrepSeg seg[3];
    int n_seg;
    int S, D, half, chunks;
    int in_dtype, out_dtype, rope_mode;
    const void* table;  // float2 (NeoX) or double2 (Gemma) (cos, sin) per (position, pair)
    int* status;
};

// Out-of-range check (status bit 4 when a finite value rounds to infinity in the 16-bit
// type): one maximum of the 8 magnitudes against the type's largest finite value; only a
// group at or above it (rare: values in [max, rounding threshold) still round to a finite
// value) takes the per-element test.
__device__ __forceinline__ void store8(void* base, int64_t e, int dtype, const float* x, int* status) {
    if (dtype == kF32) {
        *reinterpret_cast<float4*>(static_cast<float*>(base) + e) = make_float4(x[0], x[1], x[2], x[3]);
        *reinterpret_cast<float4*>(static_cast<float*>(base) + e + 4) = make_float4(x[4], x[5], x[6], x[7]);
        return;
    }
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if (dtype == kBF16) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t*>(&h);
        } else {
            const __half2 h = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t*>(&h);
        }
    }
    if (status != nullptr) {
        const float m = fmaxf(fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3]))),
                              fmaxf(fmaxf(fabsf(x[4]), fabsf(x[5])), fmaxf(fabsf(x[6]), fabsf(x[7]))));
        if (m >= (dtype == kBF16 ? 3.38953139e38f : 65504.f)) {
            // per element, on the packed results: infinity in the 16-bit type from a finite input
            const uint32_t inf16 = dtype == kBF16 ? 0x7F80u : 0x7C00u;
            bool over = false;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                over |= ((w[i] & 0x7FFFu) == inf16 && !isinf(x[2 * i])) ||
                        (((w[i] >> 16) & 0x7FFFu) == inf16 && !isinf(x[2 * i + 1]));
            }
            if (over) atomicOr(status, 4);
        }
    }
    *reinterpret_cast<uint4*>(static_cast<uint16_t*>(base) + e) = make_uint4(w[0], w[1], w[2], w[3]);
}

// 8 raw elements (16 bytes of a 16-bit type, 32 of fp32), loaded before any
// arithmetic so that each thread has all its loads in flight at once.
template <bool kF32In>
struct Raw8 {
    uint4 w[kF32In ? 2 : 1];
};
template <bool kF32In>
__device__ __forceinline__ Raw8<kF32In> raw_load(const void* base, int64_t e) {
    Raw8<kF32In> r;
    if (kF32In) {
        r.w[0] = *reinterpret_cast<const uint4*>(static_cast<const float*>(base) + e);
        r.w[kF32In ? 1 : 0] = *reinterpret_cast<const uint4*>(static_cast<const float*>(base) + e + 4);
    } else {
        r.w[0] = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + e);
    }
    return r;
}
template <bool kF32In>
__device__ __forceinline__ void raw_unpack(const Raw8<kF32In>& r, int dtype, float* x) {
    if (kF32In) {
        const uint4 a = r.w[0], b = r.w[kF32In ? 1 : 0];
        x[0] = __uint_as_float(a.x); x[1] = __uint_as_float(a.y); x[2] = __uint_as_float(a.z); x[3] = __uint_as_float(a.w);
        x[4] = __uint_as_float(b.x); x[5] = __uint_as_float(b.y); x[6] = __uint_as_float(b.z); x[7] = __uint_as_float(b.w);
        return;
    }
    const uint32_t w[4] = {r.w[0].x, r.w[0].y, r.w[0].z, r.w[0].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if (dtype == kBF16) {
            x[2 * i] = __uint_as_float(w[i] << 16);
            x[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        } else {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
            x[2 * i] = f.x;
            x[2 * i + 1] = f.y;
        }
    }
}

// kMode 1: NeoX rotation in float; 2: Gemma rotation with double products.
// kF32In: fp32 inputs (else 16-bit).  kHeads head rows per rotated unit; plain
// conversion moves 2 * kHeads chunks per thread and pass.
template <int kMode, bool kF32In, int kHeads>
__global__ void __launch_bounds__(256, 2) prep_kernel(const __grid_constant__ PrepParams p) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t first = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    // the segments one after another, each over the whole grid
#pragma unroll 1
    for (int sgi = 0; sgi < p.n_seg; ++sgi) {
        const PrepSeg sg = p.seg[sgi];
        if (!sg.rotate) {
            // plain conversion: 2 * kHeads chunks of 8 per thread and pass, stride apart (coalesced)
            constexpr int kPlain = 2 * kHeads;
            for (int64_t u = first; u < sg.units; u += kPlain * stride) {
                Raw8<kF32In> r[kPlain];
#pragma unroll
                for (int k = 0; k < kPlain; ++k)
                    if (u + k * stride < sg.units) r[k] = raw_load<kF32In>(sg.src, (u + k * stride) * 8);
#pragma unroll
                for (int k = 0; k < kPlain; ++k) {
                    if (u + k * stride >= sg.units) break;
                    float x[8];
                    raw_unpack<kF32In>(r[k], p.in_dtype, x);
                    store8(sg.dst, (u + k * stride) * 8, p.out_dtype, x, p.status);
                }
            }
            continue;
        }
        // rotated: unit = (b, s, head group, chunk); the chunk's 8 (cos, sin) pairs are read
        // once and applied to the kHeads rows of the group
        // 32-bit index arithmetic (the host keeps units below 2^31): 64-bit division is a
        // long emulated sequence and dominated this loop
        const uint32_t groups = (uint32_t)(sg.H + kHeads - 1) / kHeads, chunks = (uint32_t)p.chunks;
        for (int64_t u = first; u < sg.units; u += stride) {
            const uint32_t uu = (uint32_t)u;
            const uint32_t rest = uu / chunks;
            const int chunk = (int)(uu - rest * chunks);
            const uint32_t bs32 = rest / groups;
            const int g = (int)(rest - bs32 * groups);
            const int64_t bs = bs32;
            const int i0 = chunk * 8;
            const int s = (int)(bs32 % (uint32_t)p.S);
            Raw8<kF32In> ra[kHeads], rc[kHeads];
#pragma unroll
            for (int k = 0; k < kHeads; ++k) {
                const int h = g * kHeads + k;
                if (h < sg.H) {
                    const int64_t e0 = (bs * sg.H + h) * p.D + i0;
                    ra[k] = raw_load<kF32In>(sg.src, e0);
                    rc[k] = raw_load<kF32In>(sg.src, e0 + p.half);
                }
            }
            // the chunk's 8 (cos, sin) pairs, once per unit, into registers
            float cf[8], sf[8];
            double cd[8], sd[8];
            if (kMode == 2) {
                const double2* cs = static_cast<const double2*>(p.table) + (int64_t)s * p.half + i0;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const double2 t = cs[i];
                    cd[i] = t.x;
                    sd[i] = t.y;
                }
            } else {
                const float4* cs = reinterpret_cast<const float4*>(static_cast<const float2*>(p.table) +
                                                                   (int64_t)s * p.half + i0);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float4 t = cs[i];
                    cf[2 * i] = t.x;
                    sf[2 * i] = t.y;
                    cf[2 * i + 1] = t.z;
                    sf[2 * i + 1] = t.w;
                }
            }
#pragma unroll
            for (int k = 0; k < kHeads; ++k) {
                const int h = g * kHeads + k;
                if (h >= sg.H) break;
                const int64_t e0 = (bs * sg.H + h) * p.D + i0, e1 = e0 + p.half;
                float a[8], c[8], y0[8], y1[8];
                raw_unpack<kF32In>(ra[k], p.in_dtype, a);
                raw_unpack<kF32In>(rc[k], p.in_dtype, c);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    if (kMode == 2) {
                        y0[i] = (float)__dsub_rn(__dmul_rn((double)a[i], cd[i]), __dmul_rn((double)c[i], sd[i]));
                        y1[i] = (float)__dadd_rn(__dmul_rn((double)c[i], cd[i]), __dmul_rn((double)a[i], sd[i]));
                    } else {
                        y0[i] = __fsub_rn(__fmul_rn(a[i], cf[i]), __fmul_rn(c[i], sf[i]));
                        y1[i] = __fadd_rn(__fmul_rn(a[i], sf[i]), __fmul_rn(c[i], cf[i]));
                    }
                }
                store8(sg.dst, e0, p.out_dtype, y0, p.status);
                store8(sg.dst, e1, p.out_dtype, y1, p.status);
                if (sg.dst_in != nullptr) {
                    store8(sg.dst_in, e0, p.in_dtype, y0, nullptr);
                    store8(sg.dst_in, e1, p.in_dtype, y1, nullptr);
                }
            }
        }
    }
}

// ---------------------------------------------------------------- QK-norm + RoPE rows
__device__ __forceinline__ double warp_sum_double(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// One warp per [b][s][h] row: zero-centred RMSNorm with (1 + w)
// (Gemma3ReferenceMath.rmsNormZeroCentered, INF/gemma/Gemma3ReferenceMath.java:25-46:
// double sum of squares, float rms, (float)(x * rms * (1 + w))), then the rotation at
// position pos0 + s from the double table (Gemma: double products; NeoX: float), into
// dst (out_dtype) and, when set, dst_in (the input dtype: the rows the KV cache keeps).
__global__ void __launch_bounds__(256) norm_rope_rows_kernel(const void* src, void* dst, void* dst_in, int in_dtype,
                                                            int out_dtype, int64_t rows, int S, int H, int D,
                                                            const float* norm_w, float eps, int rope_mode,
                                                            const double2* table, int* status) {
    extern __shared__ float nr_sm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* vec = nr_sm + warp * D;
    const int half = D / 2;
    for (int64_t row = (int64_t)blockIdx.x * 8 + warp; row < rows; row += (int64_t)gridDim.x * 8) {
        const int s = (int)((row / H) % S);
        const int64_t off = row * D;
        double ss = 0.0;
        for (int d = lane; d < D; d += 32) {
            const float x = load_as_float(src, off + d, in_dtype);
            vec[d] = x;
            ss += (double)x * (double)x;
        }
        __syncwarp();
        if (norm_w != nullptr) {
            ss = warp_sum_double(ss);
            const float rms = (float)(1.0 / sqrt(__dadd_rn(ss / (double)D, (double)eps)));
            for (int d = lane; d < D; d += 32)
                vec[d] = (float)__dmul_rn((double)__fmul_rn(vec[d], rms), __dadd_rn(1.0, (double)norm_w[d]));
            __syncwarp();
        }
        if (rope_mode != 0) {
            for (int i = lane; i < half; i += 32) {
                const double2 t = table[(int64_t)s * half + i];
                const float a = vec[i], b = vec[i + half];
                float y0, y1;
                if (rope_mode == 2) {
                    y0 = (float)__dsub_rn(__dmul_rn((double)a, t.x), __dmul_rn((double)b, t.y));
                    y1 = (float)__dadd_rn(__dmul_rn((double)b, t.x), __dmul_rn((double)a, t.y));
                } else {
                    const float cf = (float)t.x, sf = (float)t.y;
                    y0 = __fsub_rn(__fmul_rn(a, cf), __fmul_rn(b, sf));
                    y1 = __fadd_rn(__fmul_rn(a, sf), __fmul_rn(b, cf));
                }
                vec[i] = y0;  // each pair belongs to one lane
                vec[i + half] = y1;
            }
            __syncwarp();
        }
        for (int d = lane; d < D; d += 32) {
            store_from_float(dst, off + d, vec[d], out_dtype);
            flag_overflow(vec[d], round_through(vec[d], out_dtype), status);
            if (dst_in != nullptr) store_from_float(dst_in, off + d, vec[d], in_dtype);
        }
        __syncwarp();
    }
}

}  // namespace

// `table` is a device buffer of S * D/2 double2 entries owned by the caller;
// build_table == false reuses a table built by an earlier call with the same
// S, pos0 and frequencies (q and k of one prefill share it).
cudaError_t launch_rope_rows_with_table(const void* src, int src_dtype, void* dst, int dst_dtype, int B, int S, int H,
                                        int D, int64_t sb, int64_t ss, int64_t sh, int64_t db, int64_t ds, int64_t dh,
                                        int pos0, int rope_mode, const double* inv_freq, double2* table,
                                        bool build_table, int* status, cudaStream_t stream) {
    const int half = D / 2;
    if (build_table) {
        FreqTable f{};
        for (int i = 0; i < half; ++i) f.inv_freq[i] = inv_freq[i];
        const int64_t n = (int64_t)S * half;
        const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
        rope_table_kernel<<<grid, 256, 0, stream>>>(table, S, half, pos0, f);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    const int64_t rows = (int64_t)B * S * H;
    const int64_t pairs = rows * half;
    const int grid = (int)((pairs + 255) / 256 < 148 * 32 ? (pairs + 255) / 256 : 148 * 32);
    rope_rows_kernel<<<grid, 256, 0, stream>>>(src, src_dtype, dst, dst_dtype, S, H, D, sb, ss, sh, db, ds, dh, rows,
                                               rope_mode, table, status);
    return cudaGetLastError();
}

cudaError_t launch_rope_table_f32(float2* table, int npos, int half, int pos0, const double* inv_freq,
                                  cudaStream_t stream) {
    FreqTable f{};
    for (int i = 0; i < half; ++i) f.inv_freq[i] = inv_freq[i];
    const int64_t n = (int64_t)npos * half;
    const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    rope_table_f32_kernel<<<grid, 256, 0, stream>>>(table, npos, half, pos0, f);
    return cudaGetLastError();
}

cudaError_t launch_convert(const void* src, int src_dtype, void* dst, int dst_dtype, int64_t n, int* status,
                           cudaStream_t stream) {
    const int64_t blocks = (n + 255) / 256;
    const int grid = (int)(blocks < 148 * 32 ? blocks : 148 * 32);
    convert_kernel<<<grid, 256, 0, stream>>>(src, src_dtype, dst, dst_dtype, n, status);
    return cudaGetLastError();
}

bool prep_vectorizable(int D, int64_t elems, const void* const* ptrs, int n) {
    if (D % 16 != 0) return false;  // D/2 a multiple of 8
    if (elems / 16 >= (int64_t)1 << 31) return false;  // rotated units are counted in 32 bits
    for (int i = 0; i < n; ++i)
        if (ptrs[i] != nullptr && reinterpret_cast<uintptr_t>(ptrs[i]) % 16 != 0) return false;
    return true;
}

cudaError_t launch_prep(const PrepJob* jobs, int n_jobs, int B, int S, int D, int in_dtype, int out_dtype, int pos0,
                        int rope_mode, const double* inv_freq, double2* table, int* status, cudaStream_t stream,
                        bool table_ready) {
    const int half = D / 2;
    bool any_rotate = false;
    for (int i = 0; i < n_jobs; ++i) any_rotate |= jobs[i].rotate != 0;
    if (any_rotate && !table_ready) {
        FreqTable f{};
        for (int i = 0; i < half; ++i) f.inv_freq[i] = inv_freq[i];
        const int64_t n = (int64_t)S * half;
        const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
        if (rope_mode == 2) rope_table_kernel<<<grid, 256, 0, stream>>>(table, S, half, pos0, f);
        else rope_table_f32_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<float2*>(table), S, half, pos0, f);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    PrepParams p{};
    p.S = S;
    p.D = D;
    p.half = half;
    p.chunks = half / 8;
    p.in_dtype = in_dtype;
    p.out_dtype = out_dtype;
    p.rope_mode = rope_mode;
    p.table = table;
    p.status = status;
    // rotated rows per unit: fewer where the unit holds more registers (fp32 data, double cos/sin)
    const bool gemma = rope_mode == 2;
    const int heads = (in_dtype == kF32 ? 2 : 4) / (gemma ? 2 : 1);
    int64_t most = 0;
    for (int i = 0; i < n_jobs && i < 3; ++i) {
        PrepSeg& sg = p.seg[p.n_seg++];
        sg.src = jobs[i].src;
        sg.dst = jobs[i].dst;
        sg.dst_in = jobs[i].dst_in;
        sg.H = jobs[i].H;
        sg.rotate = jobs[i].rotate;
        const int64_t rows = (int64_t)B * S * jobs[i].H;
        sg.units = sg.rotate ? (int64_t)B * S * ((jobs[i].H + heads - 1) / heads) * p.chunks : rows * D / 8;
        const int64_t threads = sg.rotate ? sg.units : (sg.units + 2 * heads - 1) / (2 * heads);
        most = threads > most ? threads : most;
    }
    // 2 blocks of 256 per SM stay resident (about 128 registers a thread): one wave of them loops
    // over every segment (a grid of several waves measured 256 against 244 us for configs[3])
    const int64_t blocks = (most + 255) / 256;
    const int grid = (int)(blocks < 148 * 2 ? blocks : 148 * 2);
    if (in_dtype != kF32) {
        if (gemma) prep_kernel<2, false, 2><<<grid, 256, 0, stream>>>(p);
        else prep_kernel<1, false, 4><<<grid, 256, 0, stream>>>(p);
    } else {
        if (gemma) prep_kernel<2, true, 1><<<grid, 256, 0, stream>>>(p);
        else prep_kernel<1, true, 2><<<grid, 256, 0, stream>>>(p);
    }
    return cudaGetLastError();
}

cudaError_t launch_norm_rope_rows(const void* src, void* dst, void* dst_in, int in_dtype, int out_dtype, int B, int S,
                                  int H, int D, const float* norm_w, float eps, int rope_mode, int pos0,
                                  const double* inv_freq, double2* table, bool build_table, int* status,
                                  cudaStream_t stream) {
    const int half = D / 2;
    if (rope_mode != 0 && build_table) {
        FreqTable f{};
        for (int i = 0; i < half; ++i) f.inv_freq[i] = inv_freq[i];
        const int64_t n = (int64_t)S * half;
        const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
        rope_table_kernel<<<grid, 256, 0, stream>>>(table, S, half, pos0, f);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    const int64_t rows = (int64_t)B * S * H;
    const int64_t blocks = (rows + 7) / 8;
    const int grid = (int)(blocks < 148 * 16 ? blocks : 148 * 16);
    norm_rope_rows_kernel<<<grid, 256, (size_t)8 * D * sizeof(float), stream>>>(
        src, dst, dst_in, in_dtype, out_dtype, rows, S, H, D, norm_w, eps, rope_mode, table, status);
    return cudaGetLastError();
}

}  // namespace b2a
