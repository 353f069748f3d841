// gdn_umma_selftest.cu — checks the tcgen05 operand layouts of umma.cuh.
//
// One CTA stages A [128 x K] and B [N x K] (given row-major in fp32) into
// shared memory in the requested 128-byte-swizzled K-major or MN-major
// layout, as f16 or bf16, runs K/16 tcgen05.mma instructions into TMEM and
// reads D = A * B^T [128 x N] back.  The test suite compares D with a torch
// matmul of the same rounded operands; the prefill kernel relies on every
// layout exercised here.
#include "gdn_common.cuh"
#include "umma.cuh"
#include "../../include/gdn_b200_selftest.h"

namespace gdn {

template <typename T>
__device__ __forceinline__ T cvt(float x);
template <>
__device__ __forceinline__ __half cvt<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 cvt<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

template <typename T>
__global__ void __launch_bounds__(128) umma_selftest_kernel(const float* A, const float* B, float* D,
                                                            int N, int K, int a_mn, int b_mn,
                                                            int fmt) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte align the operand tiles inside the dynamic allocation
    unsigned char* base = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* sA = base;                 // 128 x K  (<= 32 KiB)
    unsigned char* sB = base + 128 * 128 * 2; // N x K    (<= 32 KiB)
    __shared__ uint64_t mbar;
    __shared__ uint32_t tmem_base;
    const int tid = threadIdx.x, warp = tid >> 5;

    for (int i = tid; i < 128 * K; i += 128) {
        int m = i / K, k = i % K;
        uint32_t off = a_mn ? umma::mnmaj_off(m, k, K) : umma::kmaj_off(m, k, 128);
        *reinterpret_cast<T*>(sA + off) = cvt<T>(A[i]);
    }
    const bool b_sw64 = b_mn && N == 32;  // an MN extent of 32 uses the 64-byte swizzle
    for (int i = tid; i < N * K; i += 128) {
        int n = i / K, k = i % K;
        uint32_t off = b_sw64 ? umma::mnmaj64_off(n, k) : (b_mn ? umma::mnmaj_off(n, k, K) : umma::kmaj_off(n, k, N));
        *reinterpret_cast<T*>(sB + off) = cvt<T>(B[i]);
    }
    if (warp == 0) {
        umma::tmem_alloc(&tmem_base, 128);
        umma::tmem_relinquish();
    }
    if (tid == 0) {
        umma::mbar_init(&mbar, 1);
        umma::fence_mbar_init();
    }
    umma::fence_proxy_async_smem();
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = tmem_base;
    if (tid == 0) {
        const uint32_t idesc = umma::idesc_f16(128, N, fmt, fmt, a_mn, b_mn);
        const uint32_t a0 = umma::smem_u32(sA), b0 = umma::smem_u32(sB);
        for (int k0 = 0; k0 < K; k0 += 16) {
            uint64_t ad = a_mn ? umma::desc_mnmaj(a0, K, k0) : umma::desc_kmaj(a0, 128, k0);
            uint64_t bd = b_sw64 ? umma::desc_mnmaj64(b0, k0)
                                 : (b_mn ? umma::desc_mnmaj(b0, K, k0) : umma::desc_kmaj(b0, N, k0));
            umma::mma_f16(tmem, ad, bd, idesc, k0 > 0);
        }
        umma::mma_commit(&mbar);
    }
    umma::mbar_wait(&mbar, 0);
    umma::fence_after_sync();
    const int row = 32 * warp + (tid & 31);
    for (int c = 0; c < N; c += 16) {
        float v[16];
        umma::tmem_ld16(tmem + ((uint32_t)(32 * warp) << 16) + c, v);
#pragma unroll
        for (int j = 0; j < 16; ++j) D[row * N + c + j] = v[j];
    }
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 0) umma::tmem_dealloc(tmem, 128);
}

}  // namespace gdn

extern "C" int gdn_umma_selftest(const float* A, const float* B, float* D, int N, int K, int a_mn,
                                 int b_mn, int fmt, void* stream) {
    if (!A || !B || !D) return GDN_ERR_INVALID;
    if (N < 16 || N > 128 || N % 16 || K < 16 || K > 128 || K % 16) return GDN_ERR_UNSUPPORTED;
    if ((a_mn | b_mn | fmt) & ~1) return GDN_ERR_INVALID;
    if (b_mn && N % 64 && N != 32) return GDN_ERR_UNSUPPORTED;  // MN-major: 64-wide blocks, or one 32-wide
    const size_t smem = 2 * 128 * 128 * 2 + 1024;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (fmt) {
        auto kern = gdn::umma_selftest_kernel<__nv_bfloat16>;
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        kern<<<1, 128, smem, st>>>(A, B, D, N, K, a_mn, b_mn, fmt);
    } else {
        auto kern = gdn::umma_selftest_kernel<__half>;
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        kern<<<1, 128, smem, st>>>(A, B, D, N, K, a_mn, b_mn, fmt);
    }
    if (cudaGetLastError() != cudaSuccess) return GDN_ERR_CUDA;
    unsigned int status = 0;
    if (cudaMemcpyFromSymbolAsync(&status, gdn::g_device_status, sizeof(status), 0,
                                  cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return GDN_ERR_CUDA;
    return status ? GDN_ERR_DEVICE : GDN_OK;
}
