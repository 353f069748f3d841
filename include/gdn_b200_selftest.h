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

/* mode bits of gdn_umma_selftest_ex */
#define GDN_SELFTEST_A_TMEM 1    /* A staged in tensor memory (TMEM-A MMA form); needs a_mn == 0 */
#define GDN_SELFTEST_NO_ARRIVE 2 /* issue nothing: the kernel's bounded wait must run out */

/*
 * gdn_umma_selftest with a mode word and the budget of the kernel's one
 * bounded wait in SM clock cycles (0 = the default, ~1 s).  With
 * GDN_SELFTEST_NO_ARRIVE nothing ever arrives on the mbarrier the kernel
 * waits for: the wait gives up after wait_cycles, the kernel records the
 * timeout, frees its tensor memory and returns, D is left untouched and the
 * call returns GDN_ERR_DEVICE; the context stays usable.  The unit's status
 * word is cleared before every launch.
 */
int gdn_umma_selftest_ex(const float *A, const float *B, float *D, int N, int K, int a_mn, int b_mn,
                         int fmt, int mode, long long wait_cycles, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_SELFTEST_H_ */
