// attn_mma.cu -- whole-sequence attention (causal prefill, bidirectional
// encoder) for fp16 / bf16 inputs with m16n8k16 warp MMAs.
//
// CTA = 4 warps = 64 query rows of one (batch, head); key/value tiles of 64
// rows double-buffered with 16-byte cp.async into padded shared rows;
// S = Q K^T and O += P V on warp MMAs with fp32 accumulation; online softmax
// in fp32 (base 2).  P is rounded to the input type for the P.V product.
// Masks: causal (+ optional sliding window), per-batch key length, or an
// additive [B][S] float mask added to the scaled score.
// The semantics are the same as attn_simt.cu; see there for citations.
#include <math.h>

#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "internal.h"

namespace b2a {
namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kBM = 64;
constexpr int kBN = 64;

template <int D>
struct AGeo {
    static constexpr int kRow = D + 8;
    static constexpr int kChunks = D / 8;
    static constexpr size_t kTileBytes = size_t(kBM) * kRow * 2;
    static constexpr size_t kTotal = kTileBytes * 5;  // Q + 2 stages x (K, V)
};

template <int D, typename T>
__global__ void __launch_bounds__(kThreads) attn_mma_kernel(const __grid_constant__ AttnParams p) {
    using Gm = AGeo<D>;
    constexpr int kRow = Gm::kRow;
    extern __shared__ __align__(128) unsigned char smem[];
    T* q_s = reinterpret_cast<T*>(smem);
    T* kv_s = q_s + kBM * kRow;  // stage st: K at kv_s + (2*st)*kBM*kRow, V after it

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    // parameter fields in registers: the asm statements below (cp.async, ldmatrix) clobber
    // memory, which would otherwise reload each field through a generic pointer at every use
    const int S = p.S, causal = p.causal, window = p.window;
    const float* const mask = p.mask;
    const float scale = p.scale;
    const int n_mt = (S + kBM - 1) / kBM;
    const int mt_idx = n_mt - 1 - (int)blockIdx.x;  // heavy causal tiles first
    const int h = blockIdx.y, b = blockIdx.z;
    const int kvh = h / (p.Hq / p.Hkv);
    const int m0 = mt_idx * kBM;

    const T* qg = static_cast<const T*>(p.q) + b * p.q_sb + h * p.q_sh;
    const T* kg = static_cast<const T*>(p.k) + b * p.k_sb + kvh * p.k_sh;
    const T* vg = static_cast<const T*>(p.v) + b * p.k_sb + kvh * p.k_sh;

    // key range for this query tile
    int key_end = S;  // exclusive
    int key_begin = 0;
    bool uniform = false;
    if (causal) {
        key_end = min(S, m0 + kBM);
        if (window > 0) key_begin = max(0, m0 - window + 1);
    } else if (p.key_len != nullptr) {
        const int kl = p.key_len[b];
        if (kl <= 0) uniform = true;
        else key_end = min(kl, S);
    }
    const int t_begin = key_begin / kBN;
    const int n_tiles = (key_end + kBN - 1) / kBN - t_begin;

    auto load_rows = [&](T* dst, const T* src, int64_t row_stride, int row0, int nrows_valid) {
#pragma unroll 4
        for (int x = tid; x < kBM * Gm::kChunks; x += kThreads) {
            const int row = x / Gm::kChunks, cc = x - row * Gm::kChunks;
            const bool in = row0 + row < nrows_valid;
            const T* s = src + (int64_t)(in ? row0 + row : 0) * row_stride + cc * 8;
            cp_async_16(smem_u32(dst + row * kRow + cc * 8), s, in ? 16 : 0);
        }
    };
    auto load_kv = [&](int tile, int stage) {
        const int n0 = (t_begin + tile) * kBN;
        T* ks = kv_s + (2 * stage) * kBM * kRow;
        load_rows(ks, kg, p.k_ss, n0, S);
        load_rows(ks + kBM * kRow, vg, p.k_ss, n0, S);
    };

    load_rows(q_s, qg, p.q_ss, m0, S);
    if (n_tiles > 0) load_kv(0, 0);
    cp_async_commit();

    uint32_t qa[D / 16][4];
    float o[D / 8][4];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float mr0 = -INFINITY, mr1 = -INFINITY, lr0 = 0.f, lr1 = 0.f;
    const float sl2 = scale * kLog2e;
    const int qrow0 = m0 + warp * 16 + g, qrow1 = qrow0 + 8;

    for (int tile = 0; tile < n_tiles; ++tile) {
        if (tile + 1 < n_tiles) {
            load_kv(tile + 1, (tile + 1) & 1);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        if (tile == 0) {
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks)
                ldmatrix_x4(qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3],
                            smem_u32(q_s + (warp * 16 + (lane & 15)) * kRow + 16 * ks + 8 * (lane >> 4)));
        }
        const T* ks_ = kv_s + (2 * (tile & 1)) * kBM * kRow;
        const T* vs_ = ks_ + kBM * kRow;
        const int n0 = (t_begin + tile) * kBN;

        float s[kBN / 8][4];
#pragma unroll
        for (int i = 0; i < kBN / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
            for (int np = 0; np < kBN / 16; ++np) {
                const int mi = lane >> 3, r = lane & 7;
                uint32_t bf[4];
                ldmatrix_x4(bf[0], bf[1], bf[2], bf[3],
                            smem_u32(ks_ + (16 * np + r + 8 * (mi >> 1)) * kRow + 16 * ks + 8 * (mi & 1)));
                Mma<T>::run(s[2 * np], qa[ks], bf[0], bf[1]);
                Mma<T>::run(s[2 * np + 1], qa[ks], bf[2], bf[3]);
            }
        }
        // scale + mask, row max; tiles every key of which this warp's 16 rows see take the
        // scale alone
        const int wq0 = m0 + warp * 16;
        const bool edge = uniform || mask != nullptr || n0 < key_begin || n0 + kBN > key_end ||
                          (causal && n0 + kBN - 1 > wq0) || (causal && window > 0 && n0 <= wq0 + 15 - window);
        float mx0 = -INFINITY, mx1 = -INFINITY;
        if (!edge) {
#pragma unroll
            for (int nt = 0; nt < kBN / 8; ++nt) {
#pragma unroll
                for (int e = 0; e < 4; ++e) s[nt][e] *= sl2;
                mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
                mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
            }
        } else {
#pragma unroll
            for (int nt = 0; nt < kBN / 8; ++nt) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int kj = n0 + nt * 8 + 2 * t + (e & 1);
                    const int qi = (e < 2) ? qrow0 : qrow1;
                    bool vis = kj < key_end && kj >= key_begin;
                    if (causal) vis = vis && kj <= qi && (window <= 0 || kj > qi - window);
                    float v;
                    if (!vis) v = -INFINITY;
                    else if (uniform) v = 0.f;
                    else if (mask != nullptr) v = (s[nt][e] * scale + mask[(int64_t)b * S + kj]) * kLog2e;
                    else v = s[nt][e] * sl2;
                    s[nt][e] = v;
                }
                mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
                mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
            }
        }
#pragma unroll
        for (int off = 1; off < 4; off <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
        }
        const float mn0 = fmaxf(mr0, mx0), mn1 = fmaxf(mr1, mx1);
        const float b0 = mn0 == -INFINITY ? 0.f : mn0, b1 = mn1 == -INFINITY ? 0.f : mn1;
        const float c0 = fast_exp2(mr0 - b0), c1 = fast_exp2(mr1 - b1);
        mr0 = mn0;
        mr1 = mn1;
        float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
        for (int nt = 0; nt < kBN / 8; ++nt) {
            s[nt][0] = fast_exp2(s[nt][0] - b0);
            s[nt][1] = fast_exp2(s[nt][1] - b0);
            s[nt][2] = fast_exp2(s[nt][2] - b1);
            s[nt][3] = fast_exp2(s[nt][3] - b1);
            rs0 += s[nt][0] + s[nt][1];
            rs1 += s[nt][2] + s[nt][3];
        }
        lr0 = lr0 * c0 + rs0;
        lr1 = lr1 * c1 + rs1;
#pragma unroll
        for (int i = 0; i < D / 8; ++i) {
            o[i][0] *= c0;
            o[i][1] *= c0;
            o[i][2] *= c1;
            o[i][3] *= c1;
        }
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
            uint32_t pa[4];
            pa[0] = Elem<T>::pack(s[2 * kk][0], s[2 * kk][1]);
            pa[1] = Elem<T>::pack(s[2 * kk][2], s[2 * kk][3]);
            pa[2] = Elem<T>::pack(s[2 * kk + 1][0], s[2 * kk + 1][1]);
            pa[3] = Elem<T>::pack(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
            for (int dp = 0; dp < D / 16; ++dp) {
                const int mi = lane >> 3, r = lane & 7;
                uint32_t bf[4];
                ldmatrix_x4_trans(bf[0], bf[1], bf[2], bf[3],
                                  smem_u32(vs_ + (16 * kk + r + 8 * (mi & 1)) * kRow + 16 * dp + 8 * (mi >> 1)));
                Mma<T>::run(o[2 * dp], pa, bf[0], bf[1]);
                Mma<T>::run(o[2 * dp + 1], pa, bf[2], bf[3]);
            }
        }
        __syncthreads();  // stage (tile & 1) is refilled two iterations later
    }
    if (n_tiles <= 0) cp_async_wait<0>();

#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
        lr0 += __shfl_xor_sync(0xffffffffu, lr0, off);
        lr1 += __shfl_xor_sync(0xffffffffu, lr1, off);
    }
    const float i0 = 1.f / lr0, i1 = 1.f / lr1;
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt) {
        const int d = dt * 8 + 2 * t;
        if (qrow0 < S) {
            const int64_t off = b * p.q_sb + (int64_t)qrow0 * p.q_ss + h * p.q_sh + d;
            store_from_float(p.o, off, o[dt][0] * i0, p.out_dtype);
            store_from_float(p.o, off + 1, o[dt][1] * i0, p.out_dtype);
        }
        if (qrow1 < S) {
            const int64_t off = b * p.q_sb + (int64_t)qrow1 * p.q_ss + h * p.q_sh + d;
            store_from_float(p.o, off, o[dt][2] * i1, p.out_dtype);
            store_from_float(p.o, off + 1, o[dt][3] * i1, p.out_dtype);
        }
    }
}

template <int D, typename T>
cudaError_t launch_impl(const AttnParams& p, cudaStream_t stream) {
    // the dynamic shared-memory size is a per-device kernel attribute: set once per device
    constexpr int kMaxDevices = 64;
    static std::once_flag once[kMaxDevices];
    static cudaError_t err[kMaxDevices];
    const size_t smem = AGeo<D>::kTotal;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::call_once(once[dev], [dev, smem] {
        cudaError_t e = cudaFuncSetAttribute(attn_mma_kernel<D, T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        err[dev] = e;
    });
    if (err[dev] != cudaSuccess) return err[dev];
    dim3 grid((p.S + kBM - 1) / kBM, p.Hq, p.B);
    attn_mma_kernel<D, T><<<grid, kThreads, smem, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace

bool attn_tc_supported(const AttnParams& p) {
    if (p.in_dtype != kF16 && p.in_dtype != kBF16) return false;
    if (!(p.D == 32 || p.D == 64 || p.D == 96 || p.D == 128)) return false;
    // 16-byte cp.async rows: every row start must stay 16-byte aligned
    const int64_t strides[] = {p.q_sb, p.q_ss, p.q_sh, p.k_sb, p.k_ss, p.k_sh};
    for (int64_t s : strides)
        if (s % 8 != 0) return false;
    const uintptr_t ptrs[] = {(uintptr_t)p.q, (uintptr_t)p.k, (uintptr_t)p.v};
    for (uintptr_t a : ptrs)
        if (a % 16 != 0) return false;
    return p.Hq <= 65535 && p.B <= 65535;
}

cudaError_t launch_attn_tc(const AttnParams& p, cudaStream_t stream) {
    const bool bf = p.in_dtype == kBF16;
    switch (p.D) {
        case 32: return bf ? launch_impl<32, __nv_bfloat16>(p, stream) : launch_impl<32, __half>(p, stream);
        case 64: return bf ? launch_impl<64, __nv_bfloat16>(p, stream) : launch_impl<64, __half>(p, stream);
        case 96: return bf ? launch_impl<96, __nv_bfloat16>(p, stream) : launch_impl<96, __half>(p, stream);
        case 128: return bf ? launch_impl<128, __nv_bfloat16>(p, stream) : launch_impl<128, __half>(p, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace b2a
