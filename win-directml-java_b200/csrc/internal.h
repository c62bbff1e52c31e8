// internal.h -- launch parameters and launcher declarations shared between the
// C-ABI layer (api.cpp) and the CUDA translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b2a {

constexpr int kMaxHeadDim = 256;
constexpr int kDecodeMaxBatchPerLaunch = 2048;
// Largest per-unit overhead (in keys) the decode split adds to each unit's stream
// length; launches keep B * (max_seq + 1 + kDecodeGapKeysMax) below 2^31.
constexpr int kDecodeGapKeysMax = 640;

// One decode step (or one attention over an existing cache when append == 0).
struct DecodeParams {
    const void* q;       // [B][Hq][D] q_dtype
    const void* k_new;   // [B][Hkv][D] q_dtype (append mode)
    const void* v_new;   // [B][Hkv][D] q_dtype (append mode)
    int q_dtype;
    void* k_cache;       // cache_dtype
    void* v_cache;
    int cache_dtype;
    int64_t stride_b, stride_h, stride_pos;  // cache strides in elements
    const int* ctx_lens; // device [B]; NULL -> pos_scalar for every sequence
    int pos_scalar;
    int B, Hq, Hkv, G, D, max_seq;
    int window;          // > 0: sliding window
    int first_explicit;  // >= 0: first visible key (overrides window)
    int append;          // 1: norm + rope + append new k/v at position L, attend [first, L]
                         // 0: attend [first, L] of the cache with q as given
    int rope_mode;       // 0 none, 1 NeoX (float rotation), 2 Gemma (double rotation)
    float scale;
    const float* q_norm_w;
    const float* k_norm_w;
    float norm_eps;
    void* out;           // [B][Hq][D] out_dtype
    int out_dtype;
    // split-KV workspace
    float* partials;
    int* counters;       // [B * Hkv * n_hg], zero between launches
    int* status;         // device error flags (bit 0: ctx_len out of range)
    int n_hg;            // head groups of 8 per kv head
    int target_items;
    int item_capacity;
    // per-sequence element strides of q and of the new k/v rows; 0 means contiguous
    // (Hq * D and Hkv * D).  A fused [q | k | v] row per sequence sets both to (Hq + 2 Hkv) * D.
    int64_t q_seq_stride, kv_new_seq_stride;
    // optional float biases added to q, k and v before norm and RoPE ([Hq*D], [Hkv*D], [Hkv*D])
    const float* q_bias;
    const float* k_bias;
    const float* v_bias;
    // 1: launched with programmatic stream serialisation: the plan and the first piece's cache
    // tiles may overlap the kernel before it on the stream, which must not write ctx_lens or
    // the cache rows below ctx_lens[b] (tensor-core decode only)
    int early_start;
    double inv_freq[kMaxHeadDim / 2];
};
__host__ __device__ inline int64_t q_stride_of(const DecodeParams& p) {
    return p.q_seq_stride ? p.q_seq_stride : (int64_t)p.Hq * p.D;
}
__host__ __device__ inline int64_t kvn_stride_of(const DecodeParams& p) {
    return p.kv_new_seq_stride ? p.kv_new_seq_stride : (int64_t)p.Hkv * p.D;
}

// Tensor-core split-KV decode for 16-bit caches; returns false when the shape
// has no tensor-core instantiation (caller then uses the generic kernel).
bool decode_tc_supported(int D, int cache_dtype);
// Workspace geometry of the tensor-core decode for a batch of B sequences.
void decode_tc_workspace(int device, int B, int Hkv, int n_hg, int D, int cache_dtype, int* target_items,
                         int* item_capacity, size_t* partial_bytes);
cudaError_t launch_decode_tc(const DecodeParams& p, int device, cudaStream_t stream);

// Generic warp-per-head decode: any even D <= 256, any cache dtype.
cudaError_t launch_decode_simt(const DecodeParams& p, cudaStream_t stream);

// Qwen rope_and_append contract (float32, single sequence).
cudaError_t launch_qwen_rope_append(float* q, const float* k, const float* v, float* k_cache, float* v_cache,
                                    int num_heads, int kv_heads, int head_dim, int pos, int max_seq,
                                    const double* inv_freq, cudaStream_t stream);

// Attention over whole sequences (prefill / encoder).
struct AttnParams {
    const void* q;   // rotated already when the caller wants RoPE
    const void* k;
    const void* v;
    int in_dtype;
    void* o;
    int out_dtype;
    int B, S, Hq, Hkv, D;
    // element strides: [b][s][h][d] addressing for q/o and k/v
    int64_t q_sb, q_ss, q_sh;
    int64_t k_sb, k_ss, k_sh;
    int causal;
    int window;
    const float* mask;        // additive [B][S] or NULL
    const int32_t* key_len;   // [B] or NULL
    float scale;
    // NeoX RoPE applied inside the kernel to q and k at position rope_pos0 + s: float (cos, sin)
    // [position][D/2] covering positions [0, rope_pos0 + S), or NULL (q and k are used as given).
    // Only the fp32 kernels (attn_f32.cu, attn_simt.cu) take it.
    const float2* rope_table;
    int rope_pos0;
    // tcgen05 kernel only: 7 = q, k and v are bf16 (in_dtype) and the kernel converts each staged
    // tile to fp16 in shared memory; 0 = fp16 operands as given.
    int xform;
};

// Key split of the generic kernel: partial slots and per-query-block counters (zero
// between launches) in a caller-provided workspace; nsplit == 1 means no split.
constexpr int kSimtSplitKeys = 64;
struct SimtSplit {
    float* part;
    int* cnt;
    int nsplit;
    int split_keys;
};
// Chunks per query block for this launch (1: no split) and the workspace it needs.
int attn_simt_split_plan(const AttnParams& p, int sm_count, size_t* part_bytes, size_t* counter_ints);
cudaError_t launch_attn_simt(const AttnParams& p, cudaStream_t stream, const SimtSplit* split = nullptr);
// fp32 inputs at head_dim 64 / 128 (attn_f32.cu): 16 query rows per CTA, no key split.
bool attn_f32_supported(const AttnParams& p);
cudaError_t launch_attn_f32(const AttnParams& p, cudaStream_t stream);
// The context's device status buffer: words [0, kStatusWords) are the error flags
// b2a_check_device_status reports and clears; words kStatusSchedWord and the next one are
// the persistent prefill kernel's work-item counters, and word kStatusAbortWord its
// per-launch abort word (a CTA whose bounded wait ran out sets it so that the launch's other
// CTAs stop too).  All three are zero between launches: the last CTA of each launch resets
// them, so one timed-out launch does not abort the next ones (the sticky report stays in
// the error flags until they are read).
constexpr int kStatusWords = 4;
constexpr int kStatusSchedWord = 4;
constexpr int kStatusAbortWord = 6;
constexpr int kStatusBufferInts = 8;

// tcgen05 / TMEM / TMA kernel (fp16 operands, head_dim 64, 96, 128); status bit 3 = bounded wait ran out.
// `status` is the context's status buffer (kStatusBufferInts ints).
bool attn_tcgen05_supported(const AttnParams& p);
// stall (test hook): the CTA that takes work item 0 leaves one of its K/V copies unissued, so a
// bounded wait runs out (status bit 3).
cudaError_t launch_attn_tcgen05(const AttnParams& p, int* status, cudaStream_t stream, bool stall = false);
bool attn_tc_supported(const AttnParams& p);
cudaError_t launch_attn_tc(const AttnParams& p, cudaStream_t stream);

// RoPE pre-pass: dst[b][s][h][:] = rotate(src[b][s][h][:], pos0 + s); dst may alias src.
// `table` holds S * D/2 (cos, sin) pairs; build_table == false reuses it.
cudaError_t launch_rope_rows_with_table(const void* src, int src_dtype, void* dst, int dst_dtype, int B, int S, int H,
                                        int D, int64_t sb, int64_t ss, int64_t sh, int64_t db, int64_t ds, int64_t dh,
                                        int pos0, int rope_mode, const double* inv_freq, double2* table,
                                        bool build_table, int* status, cudaStream_t stream);

// table[s][i] = float (cos, sin) of (pos0 + s) * inv_freq[i] (angles in double), s < npos.
cudaError_t launch_rope_table_f32(float2* table, int npos, int half, int pos0, const double* inv_freq,
                                  cudaStream_t stream);

// Vectorised prefill pre-pass (D a multiple of 16, 16-byte aligned tensors):
// each job rotates (rope_mode 1/2) or converts a dense [B][S][H][D] tensor into
// out_dtype at dst, and, if dst_in is set, also writes the rotated rows in the
// input dtype there.  One table build plus one launch for all jobs (at most 3).
struct PrepJob {
    const void* src;
    void* dst;
    void* dst_in;
    int H;
    int rotate;
};
// elems: the largest tensor's element count.
bool prep_vectorizable(int D, int64_t elems, const void* const* ptrs, int n);
// table_ready: `table` already holds the (cos, sin) rows of positions pos0 .. pos0 + S - 1 (the
// context's cached NeoX table); otherwise the rows are built into it first.
cudaError_t launch_prep(const PrepJob* jobs, int n_jobs, int B, int S, int D, int in_dtype, int out_dtype, int pos0,
                        int rope_mode, const double* inv_freq, double2* table, int* status, cudaStream_t stream,
                        bool table_ready = false);

// QK-norm + RoPE pre-pass (one warp per [b][s][h] row of a dense tensor): zero-centred
// RMSNorm with (1 + w) when norm_w is set, rotation at pos0 + s (rope_mode 1 NeoX,
// 2 Gemma) from a double (cos, sin) table built here when build_table is set; writes
// dst in out_dtype and, when dst_in is set, the same rows in in_dtype.
cudaError_t launch_norm_rope_rows(const void* src, void* dst, void* dst_in, int in_dtype, int out_dtype, int B, int S,
                                  int H, int D, const float* norm_w, float eps, int rope_mode, int pos0,
                                  const double* inv_freq, double2* table, bool build_table, int* status,
                                  cudaStream_t stream);

// y[M][N] = x[M][K] w[N][K]^T (+ bias[N]) (+ residual[M][N]) on the tensor cores: 16-bit x and
// w of one type (row strides ldx, ldw, multiples of 8 elements), fp32 accumulation, y and the
// residual in out_dtype (row strides ldy, ldr).
struct LinearArgs {
    const void* x;
    int64_t ldx;
    const void* w;
    int64_t ldw;
    int in_dtype;
    const float* bias;
    const void* residual;
    int64_t ldr;
    void* y;
    int64_t ldy;
    int out_dtype;
    int M, N, K;
    // split-K (linear_split_plan): ksplit K ranges per output tile, an fp32 [M][N] accumulator and
    // per-tile counters, both zero between launches
    int ksplit;
    float* acc;
    int* counters;
    // early start (programmatic stream serialisation): the weight panels of the first stages are
    // requested before waiting for the kernel ahead, which must not write w
    int early;
};
bool linear_tc_supported(int in_dtype, int K, int64_t ldx, int64_t ldw, const void* x, const void* w);
// K ranges per output tile for a launch that leaves SMs idle (1: no split), and its workspace.
int linear_split_plan(int M, int N, int K, int sm_count, size_t* acc_bytes, size_t* counter_ints);
cudaError_t launch_linear_tc(const LinearArgs& a, int* status, cudaStream_t stream);

// Sets the message b2a_last_error(NULL, ...) returns on this thread.
void set_thread_error(const char* msg);

// Element-type conversion of n contiguous elements; sets status bit 2 when a
// finite value overflows the destination type.
cudaError_t launch_convert(const void* src, int src_dtype, void* dst, int dst_dtype, int64_t n, int* status,
                           cudaStream_t stream);

}  // namespace b2a
