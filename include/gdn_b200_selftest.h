/*
 * gdn_b200_selftest.h — hardware-layer self-test exported by libgdn_b200.so.
 *
 * Not part of the contest boundary (it has no counterpart in the reference):
 * it checks the tensor-core operand layouts the chunked prefill is built on.
 */
#ifndef GDN_B200_SELFTEST_H_
#define GDN_B200_SELFTEST_H_

#ifdef __cplusplus
extern "C" {
#endif

/*
 * D[128 x N] = A[128 x K] * B[N x K]^T on the tensor cores (tcgen05.mma,
 * kind::f16, fp32 accumulation).  A, B, D are row-major fp32 device arrays;
 * A and B are rounded to f16 (fmt 0) or bf16 (fmt 1) and staged K-major
 * (a_mn / b_mn = 0) or MN-major (1) with the 128-byte swizzle (the 64-byte
 * swizzle for an MN-major B with N = 32).
 * N in {16, ..., 128} (multiple of 16; 32 or a multiple of 64 when b_mn = 1),
 * K in {16, ..., 128} (multiple of 16).  Synchronises `stream`; returns
 * GDN_ERR_DEVICE if a bounded wait in the kernel timed out.
 */
int gdn_umma_selftest(const float *A, const float *B, float *D, int N, int K, int a_mn, int b_mn,
                      int fmt, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_SELFTEST_H_ */
