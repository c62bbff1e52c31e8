/* b200attn_testing.h -- test hooks of libb200attn.so.  Not part of the
 * reference-facing boundary (b200attn.h); no reference interface corresponds.
 *
 * They exist so that the failure-detection path can be exercised without a GPU
 * fault: every wait inside the library's kernels is bounded, and when one runs
 * out the kernel raises device status bit 3, stops its roles, drains its own
 * copies and tensor-core work, frees its tensor memory and returns, leaving the
 * context usable.  b2a_check_device_status then returns B2A_EDEVICE with the
 * message "a bounded device wait ran out". */
#ifndef B200ATTN_TESTING_H
#define B200ATTN_TESTING_H

#include "b200attn.h"

#ifdef __cplusplus
extern "C" {
#endif

/* One-shot: the next whole-sequence attention launch of this context that takes
 * the tensor-core (tcgen05) kernel leaves one of its K/V tile copies unissued, so
 * the wait for it runs out after 1 s.  The outputs of that launch are undefined;
 * the context's next launches are unaffected.  Returns B2A_OK, or B2A_EINVAL for
 * a null context. */
B2A_API int b2a_test_inject_wait_timeout(b2a_context* ctx);

/* The kernel family the context's last whole-sequence attention launch (b2a_mha,
 * b2a_prefill_causal, b2a_prefill_gemma) took, so that tests can assert the path:
 * B2A_TEST_KERNEL_TCGEN05 (tensor cores, TMEM, TMA), B2A_TEST_KERNEL_WARP_MMA
 * (mma.sync), B2A_TEST_KERNEL_GENERIC (fp32 / odd head dims), B2A_TEST_KERNEL_F32_TILED
 * (fp32 at head_dim 64 / 128); 0 before any launch
 * or for a null context. */
#define B2A_TEST_KERNEL_TCGEN05 1
#define B2A_TEST_KERNEL_WARP_MMA 2
#define B2A_TEST_KERNEL_GENERIC 3
#define B2A_TEST_KERNEL_F32_TILED 4
B2A_API int b2a_test_last_attention_kernel(const b2a_context* ctx);

#ifdef __cplusplus
}
#endif

#endif /* B200ATTN_TESTING_H */
