/*
 * b200attn.h -- C ABI of libb200attn.so, the B200 (sm_100a) backend for the
 * attention hot path of win-directml-java: RoPE + scaled-dot-product attention
 * for causal GQA prefill, single-token decode over a KV cache, and masked
 * bidirectional encoder attention.
 *
 * Conventions
 *   - Plain C.  Every entry point returns an int status (b2a_status); no
 *     exception or C++ type crosses the boundary.  On failure the message is
 *     kept per context and read with b2a_last_error().
 *   - Tensor pointers are caller-owned DEVICE pointers unless a parameter
 *     says "host".  `stream` is a cudaStream_t passed as void* (NULL = the
 *     legacy default stream).  Calls are asynchronous on that stream.
 *   - A context is bound to one CUDA device.  It is not thread-safe: use one
 *     context per thread, as the reference's kernels are used per thread.
 *   - There is no CPU fallback: a call that cannot run on the GPU fails.
 *   - Element types follow the reference's TensorDataType names.
 *
 * Reference paths below are relative to the win-directml-java project:
 *   WB/  = directml-windows-bindings/src/main/java/com/aresstack/windirectml/
 *   INF/ = directml-inference/src/main/java/com/aresstack/windirectml/inference/
 *   ENC/ = directml-encoder/src/main/java/com/aresstack/windirectml/encoder/
 */
#ifndef B200ATTN_H
#define B200ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define B2A_API __attribute__((visibility("default")))
#else
#define B2A_API
#endif

#define B2A_ABI_VERSION 1

typedef struct b2a_context b2a_context;

/* Status codes.  The reference wraps native failures in the unchecked
 * DirectMlRuntimeException (WB/runtime/DirectMlRuntimeException.java) and
 * rejects bad shapes with IllegalArgumentException; a binding maps every
 * non-zero status to one of those with b2a_last_error() as the message. */
typedef enum b2a_status {
    B2A_OK = 0,
    B2A_EINVAL = 1,   /* bad shape, dtype, head divisibility, null or misaligned pointer */
    B2A_ECUDA = 2,    /* a CUDA runtime call failed */
    B2A_ENCCL = 3,    /* NCCL failed or could not be loaded (b2a_group_*, b2a_sharded_*) */
    B2A_ETIMEOUT = 4, /* a bounded device-side wait ran out (b2a_check_device_status) */
    B2A_EOOM = 5,     /* device allocation failed or exceeded the context's cap */
    B2A_ENOTSUP = 6,  /* valid arguments, but no kernel for this combination */
    B2A_EDEVICE = 7   /* a device-side argument check failed (see b2a_check_device_status) */
} b2a_status;

/* TensorDataType FLOAT32 / FLOAT16 / BFLOAT16 (WB/runtime/TensorDataType.java). */
typedef enum b2a_dtype {
    B2A_FLOAT32 = 0,
    B2A_FLOAT16 = 1,
    B2A_BFLOAT16 = 2
} b2a_dtype;

/* Activation layouts.
 * HEAD_MAJOR = [B, H, S, D] (AttentionKernel contract, WB/runtime/kernels/AttentionKernel.java:11-13).
 * SEQ_MAJOR  = [B, S, H, D] (the encoders' flat [seq][H*D] rows,
 *              ENC/minilm/CpuMiniLmEncoder.java:311-316). */
typedef enum b2a_layout {
    B2A_HEAD_MAJOR = 0,
    B2A_SEQ_MAJOR = 1
} b2a_layout;

/* KV cache layouts, per sequence.
 * KV_HEAD_MAJOR = [B][Hkv][max_seq][D] (INF/decoderonly/DecoderOnlyKvCacheLayout.java:53-59,
 *                 WB/windows/QwenAttentionShaders.java:73-75).
 * KV_POS_MAJOR  = [B][max_seq][Hkv][D] (INF/decoderonly/DecoderOnlyWarpLayerKvCache.java:13-45,
 *                 INF/gemma/Gemma3WarpFusedAttentionContextKernel.java:58). */
typedef enum b2a_kv_layout {
    B2A_KV_HEAD_MAJOR = 0,
    B2A_KV_POS_MAJOR = 1
} b2a_kv_layout;

/* Rotary embedding variants.  Both rotate the pairs (x[i], x[i+D/2]) by
 * angle = pos * theta^(-2i/D), the angle taken in double precision.
 * NEOX    : DecoderOnlyRotaryEmbedding (INF/decoderonly/DecoderOnlyRotaryEmbedding.java:42-67),
 *           cos/sin rounded to float, rotation in float.
 * GEMMA   : Gemma3ReferenceMath.applyRopeHalf (INF/gemma/Gemma3ReferenceMath.java:65-83),
 *           rotation in double, result rounded to float. */
typedef enum b2a_rope_mode {
    B2A_ROPE_NONE = 0,
    B2A_ROPE_NEOX = 1,
    B2A_ROPE_GEMMA = 2
} b2a_rope_mode;

/* ---------------------------------------------------------------- lifecycle */

/* Create a context on CUDA device `device` (replaces DirectMlContextImpl
 * initialisation, WB/runtime/DirectMlContextImpl.java). */
B2A_API int b2a_create(int device, b2a_context** out);

/* Destroy the context and free its workspace (AutoCloseable.close of the
 * reference kernels, WB/runtime/kernels/DirectMlAttentionKernel.java:592-617). */
B2A_API int b2a_destroy(b2a_context* ctx);

/* Copy the last error message of `ctx` into buf (NUL-terminated, truncated
 * to n bytes).  Returns the full message length.  ctx may be NULL for errors
 * of b2a_create. */
B2A_API int b2a_last_error(const b2a_context* ctx, char* buf, size_t n);

/* Static name of a status code. */
B2A_API const char* b2a_status_string(int status);

/* ABI version (B2A_ABI_VERSION) and build string. */
B2A_API int b2a_abi_version(void);
B2A_API const char* b2a_build_info(void);

/* Cap on the bytes of device workspace the context may allocate (0 = no
 * cap).  A call whose workspace would exceed it fails with B2A_EOOM, except
 * for the optional key-split workspace of the generic (fp32 / odd head dim)
 * attention kernel: without room for it the launch runs unsplit. */
B2A_API int b2a_set_workspace_limit(b2a_context* ctx, size_t bytes);

/* Early start for b2a_decode on the tensor-core path (enable != 0; off by default).
 * Each decode launch is then made with programmatic stream serialisation: it plans its
 * work from ctx_lens and requests its first KV-cache tiles while the kernel before it on
 * the stream finishes, and waits for that kernel to complete before it reads q, the new
 * k/v rows, biases or norm weights and before any write.  Contract: the kernel launched
 * immediately before a decode on the same stream must not write ctx_lens or the cache
 * rows below ctx_lens[b] (rows the decode reads) -- true of back-to-back decode layers and
 * of projections that produce q / k / v.  The two projections of b2a_decode_attention_block are
 * launched the same way: each requests its first weight panels before waiting for the kernel
 * ahead (which must not write the weights).  Returns B2A_OK, or B2A_EINVAL for a null context. */
B2A_API int b2a_set_decode_early_start(b2a_context* ctx, int enable);

/* Bytes of device workspace the context currently holds. */
B2A_API int b2a_workspace_bytes(const b2a_context* ctx, size_t* bytes);

/* Pre-allocate the decode workspace for batches up to max_batch with the
 * given head geometry, so later b2a_decode calls allocate nothing. */
B2A_API int b2a_reserve_decode(b2a_context* ctx, int max_batch, int num_q_heads, int num_kv_heads,
                               int head_dim);

/* Synchronise `stream` and report what the context's kernels flagged on the
 * device since the last call, then clear it:
 *   B2A_ETIMEOUT  a bounded device-side wait ran out and the launch aborted
 *                 (its outputs are undefined); takes precedence over the others;
 *   B2A_EDEVICE   a device-side argument check failed (a ctx_lens entry outside
 *                 [0, max_seq), a bf16 input beyond the fp16 operand range);
 *   B2A_OK        nothing was flagged.
 * The compute calls are asynchronous, as CUDA launches are; a binding that
 * mirrors the reference's synchronous dispatch (DirectMlAttentionKernel.dispatch
 * waits on a fence unless a DirectMlGpuBatch is open, WB/windows/D3D12Bindings.java:921-937)
 * calls this after each dispatch, or once when its batch closes, and throws on
 * a non-zero status. */
B2A_API int b2a_check_device_status(b2a_context* ctx, void* stream);

/* ------------------------------------------------------------ encoder MHA */

/* Multi-head scaled-dot-product attention, bidirectional, with an optional key
 * padding mask: the AttentionKernel.dispatch(q, k, v, mask, y, scale) contract
 * (WB/runtime/kernels/AttentionKernel.java:19-24; validation as
 * DirectMlAttentionKernel.recordOnto, WB/runtime/kernels/DirectMlAttentionKernel.java:401-420,663-685).
 *   q, k, v, y : [B,H,S,D] (HEAD_MAJOR) or [B,S,H,D] (SEQ_MAJOR), element type in_dtype for
 *                q/k/v and out_dtype for y.
 *   mask       : optional additive float mask [B,S] (0 or -1e9, the [B,1,1,S] tensor of
 *                BertPoolingWeights.additiveMask, ENC/bert/BertPoolingWeights.java:62-77), or NULL.
 *   key_lengths: optional int32 [B]; key j of batch b is masked iff j >= key_lengths[b]
 *                (the CPU encoders' int attention mask, ENC/minilm/CpuMiniLmEncoder.java:337).
 *                At most one of mask / key_lengths may be non-NULL.
 *   scale      : usually 1/sqrt(D).
 * A masked key contributes exactly zero weight; a row whose keys are all masked
 * yields the mean of V, as softmax over equal -1e9 scores does in the reference. */
B2A_API int b2a_mha(b2a_context* ctx, int in_dtype, int out_dtype,
                    const void* q, const void* k, const void* v,
                    const float* mask, const int32_t* key_lengths, void* y,
                    int B, int H, int S, int D, float scale, int layout, void* stream);

/* ------------------------------------------------------------ causal prefill */

/* Causal grouped-query attention over a whole prompt with RoPE fused
 * (SmolLM2ReferenceForwardPass.runSelfAttention, INF/smollm2/SmolLM2ReferenceForwardPass.java:167-210;
 *  Qwen2Runtime.processLayerPrefill attention, INF/qwen/Qwen2Runtime.java:916-971;
 *  Phi3Runtime prefill attention, INF/phi3/Phi3Runtime.java:609-697).
 *   q : [B,S,Hq,D], k/v : [B,S,Hkv,D] (in_dtype), o : [B,S,Hq,D] (out_dtype); Hq % Hkv == 0,
 *       query head h reads kv head h / (Hq/Hkv) (INF/decoderonly/DecoderOnlyAttentionLayout.java:43-53).
 *   rope_mode / rope_theta : rotation applied to q and k at positions pos0 + s
 *       (B2A_ROPE_NONE to skip).  q, k, v are not modified.
 *   window : 0 = full causal; > 0 = keys [max(0, t-window+1), t]
 *       (INF/gemma/Gemma3AttentionLayout.java:57-62).
 *   k_rot_out : optional [B,S,Hkv,D] (in_dtype) receiving the rotated keys (the KV-cache
 *       store of Qwen2Runtime.java:927-936), or NULL.  For f16/bf16 inputs on the
 *       tensor-core path it doubles as the rotated-key staging buffer; pass NULL to
 *       let the context hold that buffer. */
B2A_API int b2a_prefill_causal(b2a_context* ctx, int in_dtype, int out_dtype,
                               const void* q, const void* k, const void* v, void* o,
                               int B, int S, int Hq, int Hkv, int D, float scale,
                               int rope_mode, double rope_theta, int pos0, int window,
                               void* k_rot_out, void* stream);

/* ------------------------------------------------------------ decode */

/* One decode step for a batch of sequences, fused: optional per-head QK-norm
 * (zero-centred RMSNorm x*rsqrt(mean(x^2)+eps)*(1+w), INF/gemma/Gemma3ReferenceMath.java:25-46),
 * RoPE of the new q and k at position ctx_lens[b], append of k and v into the
 * cache at that position, then attention of every q head over the visible
 * keys [first, ctx_lens[b]] including the new one, first = 0 or
 * max(0, ctx_lens[b]-window+1).  Mirrors Qwen2Runtime.processLayerDecode
 * (INF/qwen/Qwen2Runtime.java:723-766), the Qwen GPU pair rope_and_append +
 * gqa_attention_decode (WB/windows/QwenAttentionShaders.java:82-263) and the
 * Gemma decode step (INF/gemma/Gemma3WarpLayer.java:263-281,
 * INF/gemma/Gemma3ReferenceForwardPass.java:124-182).
 *   q_new [B,Hq,D], k_new / v_new [B,Hkv,D] : element type q_dtype.
 *   k_cache / v_cache : cache_dtype, layout kv_layout, capacity max_seq positions.
 *   ctx_lens : DEVICE int32 [B], tokens already cached per sequence (the new
 *              token's position); each must lie in [0, max_seq).  Entries
 *              outside raise the device status (b2a_check_device_status) and that
 *              sequence's output is NaN.
 *   q_norm_w / k_norm_w : optional DEVICE float [D] QK-norm weights (both or neither).
 *   o [B,Hq,D] : out_dtype. */
B2A_API int b2a_decode(b2a_context* ctx, int q_dtype, int cache_dtype, int out_dtype,
                       const void* q_new, const void* k_new, const void* v_new,
                       void* k_cache, void* v_cache, int kv_layout, const int32_t* ctx_lens,
                       int B, int Hq, int Hkv, int D, int max_seq, float scale,
                       int rope_mode, double rope_theta, int window,
                       const float* q_norm_w, const float* k_norm_w, float norm_eps,
                       void* o, void* stream);

/* The b2a_decode step for callers that cannot allocate device memory: hosts
 * whose GPU memory belongs to another allocator (a JVM or serving runtime
 * that owns an arena or caching pool), where a cudaMalloc outside that pool
 * can fail and cudaMalloc/cudaFree would synchronise the device.  No
 * counterpart exists in the reference.  Same arguments and results as
 * b2a_decode, without a context: it runs on the current CUDA device and
 * allocates nothing; its scratch is a fixed 4 MiB static device array per GPU,
 * held until the process exits.  The first call on a device resolves that
 * array's address; make it before any stream capture.  Limits: fp16/bf16
 * caches, head_dim 64/96/128/256, batch <= 2048 and
 * batch * Hkv * ceil((Hq/Hkv)/8) <= 16384; larger requests fail with
 * B2A_EINVAL / B2A_ENOTSUP and a message in b2a_last_error(NULL, ...).
 * The split-KV partial slots take 2 * grid * 8 * (head_dim + 2) * 4 bytes of
 * the array, grid being the decode kernel's resident CTAs (SMs x CTAs per SM
 * for that head dim): on a B200 (148 SMs) every supported head dim fits (at
 * most about 2.5 MB); a GPU with more resident CTAs can exceed it, and then
 * every call at that head dim returns B2A_ENOTSUP.
 * All calls share the scratch: calls whose kernels overlap on the GPU race,
 * so serialise them (one stream).  An out-of-range ctx_lens entry gives NaN
 * outputs for that sequence; there is no device-status query. */
B2A_API int b2a_decode_noalloc(int q_dtype, int cache_dtype, int out_dtype, const void* q_new, const void* k_new,
                               const void* v_new, void* k_cache, void* v_cache, int kv_layout,
                               const int32_t* ctx_lens, int B, int Hq, int Hkv, int D, int max_seq, float scale,
                               int rope_mode, double rope_theta, int window, const float* q_norm_w,
                               const float* k_norm_w, float norm_eps, void* o, void* stream);

/* Batched Gemma-3 prefill: Gemma3WarpLayer.forwardPrefillBatched (INF/gemma/Gemma3WarpLayer.java:
 * 395-411) runs QK-norm, RoPE and the KV append per position and then one attention
 * dispatch per position over [firstValid(p), p]; here all positions take one norm +
 * rotation pre-pass and one attention launch.  q [B,S,Hq,D], k/v
 * [B,S,Hkv,D], o [B,S,Hq,D] dense.  q_norm_w / k_norm_w [D] (NULL: no norm) apply the
 * zero-centred RMSNorm x * rsqrt(mean(x^2) + eps) * (1 + w) with a double sum of
 * squares (Gemma3ReferenceMath.rmsNormZeroCentered, L25-46) to every q / k head before
 * the rotation at position pos0 + s (rope_mode GEMMA: applyRopeHalf's double products;
 * NEOX: float).  window > 0 is the local-layer sliding window (firstValidKey =
 * max(0, p - window + 1)); scale is 1/sqrt(query_pre_attn_scalar).  k_rot_out (or NULL)
 * receives the normed, rotated keys in the input type: the rows the KV cache keeps (the
 * values are appended unchanged). */
B2A_API int b2a_prefill_gemma(b2a_context* ctx, int in_dtype, int out_dtype, const void* q, const void* k,
                              const void* v, void* o, int B, int S, int Hq, int Hkv, int D, float scale,
                              int rope_mode, double rope_theta, int pos0, int window, const float* q_norm_w,
                              const float* k_norm_w, float norm_eps, void* k_rot_out, void* stream);

/* ------------------------------------------- reference GPU contracts, 1:1 */

/* ROPE_AND_APPEND_HLSL (WB/windows/QwenAttentionShaders.java:82-135), root
 * constants {numHeads, kvHeads, headDim, pos, maxSeqLen, ropeTheta}: rotates
 * q [numHeads*headDim] in place and writes the rotated k and the unchanged v
 * [kvHeads*headDim] into the float caches [kvHeads][maxSeqLen][headDim] at
 * position pos.  All float32.  The angle is taken in double precision. */
B2A_API int b2a_qwen_rope_and_append(b2a_context* ctx, float* q, const float* k, const float* v,
                                     float* k_cache, float* v_cache, int num_heads, int kv_heads,
                                     int head_dim, int pos, int max_seq_len, float rope_theta,
                                     void* stream);

/* One Qwen2 decode-layer attention step on the fused QKV projection output, in one
 * launch: QwenGpuPipeline.decodeLayerGpuResident steps 1b-3
 * (INF/qwen/QwenGpuPipeline.java:647-691), which dispatch the fused-bias Add,
 * ROPE_AND_APPEND_HLSL and GQA_ATTENTION_DECODE_HLSL.  qkv is one token's
 * [Q (numHeads*headDim) | K (kvHeads*headDim) | V (kvHeads*headDim)] row;
 * qkv_bias (same layout, or NULL) is added first; q and k are rotated at pos
 * (angles in double, as b2a_qwen_rope_and_append); k and v are written into the
 * float caches [kvHeads][maxSeqLen][headDim] at pos; attn_out [numHeads*headDim]
 * = softmax(scale * q.K[0..pos]) . V.  All float32.  qkv is not modified (the
 * reference rotates Q in place as an intermediate nothing reads afterwards). */
B2A_API int b2a_qwen_decode_step(b2a_context* ctx, const float* qkv, const float* qkv_bias, float* k_cache,
                                 float* v_cache, float* attn_out, int num_heads, int kv_heads, int head_dim, int pos,
                                 int max_seq_len, float rope_theta, float scale, void* stream);

/* GQA_ATTENTION_DECODE_HLSL (WB/windows/QwenAttentionShaders.java:168-263), root
 * constants {numHeads, kvHeads, headDim, qHeadsPerKvHead, seqLen, maxSeqLen, scale}:
 * attn_out[h] = softmax(scale * q[h].K[0..seqLen)) . V over the float caches
 * [kvHeads][maxSeqLen][headDim], kv head h / qHeadsPerKvHead. */
B2A_API int b2a_qwen_gqa_attention_decode(b2a_context* ctx, const float* q, const float* k_cache,
                                          const float* v_cache, float* attn_out, int num_heads,
                                          int kv_heads, int head_dim, int q_heads_per_kv_head,
                                          int seq_len, int max_seq_len, float scale, void* stream);

/* FUSED_ATTENTION_HLSL (INF/gemma/Gemma3WarpFusedAttentionContextKernel.java:32-86,
 * call contract L111-135), constants {numHeads, groupsPerKv, headDim, kvDim,
 * firstValid, queryPos, scale}: ctx_out[h] = softmax over keys
 * [firstValid, queryPos] of the position-major float caches keys/values
 * [pos][kvDim], kv head h / groupsPerKv.  head_dim <= 256. */
B2A_API int b2a_gemma_fused_attention_context(b2a_context* ctx, const float* q, const float* keys,
                                              const float* values, float* ctx_out, int num_heads,
                                              int groups_per_kv, int head_dim, int kv_dim,
                                              int first_valid, int query_pos, float scale, void* stream);

/* ------------------------------------------------ projections around attention */

/* y[M,N] = x[M,K] w[N,K]^T + bias[N] + residual[M,N] on the tensor cores (tcgen05, TMEM
 * accumulator, TMA-staged tiles), bias and residual fused into the epilogue: the O
 * projection with the residual add (residual1 = input + oProjOut; decode
 * INF/qwen/Qwen2Runtime.java:756-777, prefill L973-1000) and the QKV projection with its
 * bias (decode L693-716, prefill L888-914).  x and w: FLOAT16 or BFLOAT16 (one type), row-major, K a
 * multiple of 8; bias: float [N] or NULL; residual: [M,N] of out_dtype or NULL (may
 * alias y); fp32 accumulation. */
B2A_API int b2a_linear(b2a_context* ctx, int in_dtype, int out_dtype, const void* x, const void* w,
                       const float* bias, const void* residual, void* y, int M, int N, int K, void* stream);

/* One decode-layer attention block, Qwen2Runtime.processLayerDecode from the normed input
 * to the first residual (INF/qwen/Qwen2Runtime.java:693-777), in three launches: the QKV
 * projection with its bias (fp32 rows [Q | K | V]), the fused decode step (NeoX RoPE at
 * ctx_lens[b], KV append, GQA attention; as b2a_decode) reading those rows directly, and
 * the O projection with the residual add.
 *   x [B, hidden], w_qkv [(Hq + 2 Hkv) D, hidden], w_o [hidden, Hq D], residual / y
 *   [B, hidden]: act_dtype (FLOAT16 / BFLOAT16); b_qkv float [(Hq + 2 Hkv) D] or NULL;
 *   caches as b2a_decode.  The attention output feeding the O projection is rounded to
 *   act_dtype (the operand type of its tensor-core GEMM). */
B2A_API int b2a_decode_attention_block(b2a_context* ctx, int act_dtype, int cache_dtype, const void* x,
                                       const void* w_qkv, const float* b_qkv, void* k_cache, void* v_cache,
                                       int kv_layout, const int32_t* ctx_lens, const void* w_o, const void* residual,
                                       void* y, int B, int hidden, int Hq, int Hkv, int D, int max_seq, float scale,
                                       double rope_theta, int window, void* stream);

/* ------------------------------------------------------------ multi-GPU */

/* One process driving several GPUs of a node: the multi-device counterpart of
 * b2a_create (the reference's DirectMlContextImpl is single-device and the
 * reference has no multi-GPU path).  A group holds one context per device and an NCCL
 * communicator clique (ncclCommInitAll).  NCCL is loaded at run time
 * (libnccl.so.2, or the file named by the B2A_NCCL_LIBRARY environment variable);
 * a missing library and every NCCL failure -- a rank count below 1 or a device
 * list NCCL rejects included -- return B2A_ENCCL.  Not thread-safe. */
typedef struct b2a_group b2a_group;
B2A_API int b2a_group_create(int ndev, const int* devices, b2a_group** out);
B2A_API int b2a_group_destroy(b2a_group* g);
/* Message of the group's last failure (g may be NULL for b2a_group_create). */
B2A_API int b2a_group_last_error(const b2a_group* g, char* buf, size_t n);
B2A_API int b2a_group_size(const b2a_group* g);
/* The context of rank `rank` (owned by the group; do not destroy it). */
B2A_API int b2a_group_context(b2a_group* g, int rank, b2a_context** ctx);
/* b2a_check_device_status on every rank (streams[r] or the default stream). */
B2A_API int b2a_group_check_device_status(b2a_group* g, void* const* streams);

/* Sharded decode: every argument that is a tensor is a per-rank array of device
 * pointers (index r = rank r, memory on that rank's device); each rank holds an
 * equal shard of B_shard sequences and runs b2a_decode on it (same argument
 * meaning), then one grouped ncclAllGather copies every rank's o_shard
 * [B_shard, Hq, D] into o_gathered[r] [n_ranks * B_shard, Hq, D] on every rank,
 * rank-major.  Partitioning by (sequence, kv head): pass each unit as a sequence
 * with Hkv = 1 and Hq = Hq/Hkv (its cache rows and q heads), as planned by
 * b2a_partition_units.  streams: per-rank cudaStream_t array or NULL.
 * Asynchronous; a rank's argument failure returns its status with the rank named. */
B2A_API int b2a_sharded_decode(b2a_group* g, int q_dtype, int cache_dtype, int out_dtype,
                               const void* const* q_new, const void* const* k_new, const void* const* v_new,
                               void* const* k_cache, void* const* v_cache, int kv_layout,
                               const int32_t* const* ctx_lens, int B_shard, int Hq, int Hkv, int D, int max_seq,
                               float scale, int rope_mode, double rope_theta, int window,
                               const float* const* q_norm_w, const float* const* k_norm_w, float norm_eps,
                               void* const* o_shard, void* const* o_gathered, void* const* streams);

/* Sharded encoder attention: b2a_mha on every rank's B_shard sequences (per-rank
 * pointer arrays; mask / key_lengths arrays may be NULL), then one grouped
 * ncclAllGather of y_shard into y_gathered[r] (rank-major along the batch). */
B2A_API int b2a_sharded_mha(b2a_group* g, int in_dtype, int out_dtype, const void* const* q, const void* const* k,
                            const void* const* v, const float* const* mask, const int32_t* const* key_lengths,
                            void* const* y_shard, void* const* y_gathered, int B_shard, int H, int S, int D,
                            float scale, int layout, void* const* streams);

/* Partition `n_units` independent (sequence, kv-head) units over `n_ranks`
 * ranks with equal unit counts (n_units % n_ranks == 0 required), balancing
 * the per-unit cost `unit_cost` (host, e.g. KV bytes) by a longest-first
 * greedy assignment.  Writes rank_of_unit[n_units] (host).  No collective is
 * involved; outputs are reassembled by the caller (an all-gather). */
B2A_API int b2a_partition_units(int n_units, int n_ranks, const int64_t* unit_cost, int32_t* rank_of_unit);

#ifdef __cplusplus
}
#endif

#endif /* B200ATTN_H */
