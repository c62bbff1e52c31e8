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

cudaError_t launch_convert(const void* src, int src_dtype, void* dst, int dst_dtype, int64_t n, int* status,
                           cudaStream_t stream) {
    const int64_t blocks = (n + 255) / 256;
    const int grid = (int)(blocks < 148 * 32 ? blocks : 148 * 32);
    convert_kernel<<<grid, 256, 0, stream>>>(src, src_dtype, dst, dst_dtype, n, status);
    return cudaGetLastError();
}

}  // namespace b2a
