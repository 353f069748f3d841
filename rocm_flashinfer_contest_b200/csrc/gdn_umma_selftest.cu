// gdn_umma_selftest.cu — checks the tcgen05 operand layouts of umma.cuh.
//
// One CTA stages A [128 x K] and B [N x K] (given row-major in fp32) into
// shared memory in the requested 128-byte-swizzled K-major or MN-major
// layout, as f16 or bf16, runs K/16 tcgen05.mma instructions into TMEM and
// reads D = A * B^T [128 x N] back.  The test suite compares D with a torch
// matmul of the same rounded operands; the prefill kernels rely on every
// layout exercised here.
//
// Two further modes of gdn_umma_selftest_ex:
//  * GDN_SELFTEST_A_TMEM: A is staged in tensor memory instead (row m in
//    TMEM lane m, two 16-bit elements per 32-bit column) and the MMAs read it
//    from there (the TMEM-A form of tcgen05.mma);
//  * GDN_SELFTEST_NO_ARRIVE: no MMA is issued and nothing ever arrives on the
//    mbarrier the kernel waits for, so its bounded wait runs out after
//    `wait_cycles`; the kernel then records the timeout in the status word,
//    frees its TMEM and returns, and the call reports GDN_ERR_DEVICE.  This is
//    how the failure path of every bounded wait is exercised without a fault.
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
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    const T a = cvt<T>(lo), b = cvt<T>(hi);
    return (uint32_t)(*reinterpret_cast<const uint16_t*>(&a)) |
           ((uint32_t)(*reinterpret_cast<const uint16_t*>(&b)) << 16);
}

constexpr uint32_t kSelftestCols = 256;  // D in columns 0..N-1, a TMEM-resident A from column 128
constexpr uint32_t kTmemA = 128;

template <typename T>
__global__ void __launch_bounds__(128) umma_selftest_kernel(const float* A, const float* B, float* D,
                                                            int N, int K, int a_mn, int b_mn,
                                                            int fmt, int mode, long long wait_cycles) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte align the operand tiles inside the dynamic allocation
    unsigned char* base = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* sA = base;                 // 128 x K  (<= 32 KiB)
    unsigned char* sB = base + 128 * 128 * 2; // N x K    (<= 32 KiB)
    __shared__ uint64_t mbar;
    __shared__ uint32_t tmem_base;
    const int tid = threadIdx.x, warp = tid >> 5;
    const bool a_tmem = (mode & GDN_SELFTEST_A_TMEM) != 0;
    const bool no_arrive = (mode & GDN_SELFTEST_NO_ARRIVE) != 0;

    if (!a_tmem) {
        for (int i = tid; i < 128 * K; i += 128) {
            int m = i / K, k = i % K;
            uint32_t off = a_mn ? umma::mnmaj_off(m, k, K) : umma::kmaj_off(m, k, 128);
            *reinterpret_cast<T*>(sA + off) = cvt<T>(A[i]);
        }
    }
    const bool b_sw64 = b_mn && N == 32;  // an MN extent of 32 uses the 64-byte swizzle
    for (int i = tid; i < N * K; i += 128) {
        int n = i / K, k = i % K;
        uint32_t off = b_sw64 ? umma::mnmaj64_off(n, k) : (b_mn ? umma::mnmaj_off(n, k, K) : umma::kmaj_off(n, k, N));
        *reinterpret_cast<T*>(sB + off) = cvt<T>(B[i]);
    }
    if (warp == 0) {
        umma::tmem_alloc(&tmem_base, kSelftestCols);
        umma::tmem_relinquish();
    }
    if (tid == 0) {
        umma::mbar_init(&mbar, 1);
        umma::fence_mbar_init();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = tmem_base;
    const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
    const int row = 32 * warp + (tid & 31);
    if (a_tmem) {
        // row `row` of A into this thread's TMEM lane, 16 columns (32 elements) per store
        for (int c0 = 0; c0 < K / 2; c0 += 16) {
            float w[16];
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const int k = 2 * (c0 + c);
                w[c] = k < K ? __uint_as_float(pack2<T>(A[row * K + k], A[row * K + k + 1])) : 0.f;
            }
            umma::tmem_st16(tmem + lane_base + kTmemA + c0, w);
        }
    }
    umma::fence_proxy_async_smem();
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (tid == 0 && !no_arrive) {
        const uint32_t idesc = umma::idesc_f16(128, N, fmt, fmt, a_tmem ? 0 : a_mn, b_mn);
        const uint32_t a0 = umma::smem_u32(sA), b0 = umma::smem_u32(sB);
        for (int k0 = 0; k0 < K; k0 += 16) {
            uint64_t bd = b_sw64 ? umma::desc_mnmaj64(b0, k0)
                                 : (b_mn ? umma::desc_mnmaj(b0, K, k0) : umma::desc_kmaj(b0, N, k0));
            if (a_tmem) {
                umma::mma_f16_ts(tmem, tmem + kTmemA + (uint32_t)(k0 / 2), bd, idesc, k0 > 0);
            } else {
                uint64_t ad = a_mn ? umma::desc_mnmaj(a0, K, k0) : umma::desc_kmaj(a0, 128, k0);
                umma::mma_f16(tmem, ad, bd, idesc, k0 > 0);
            }
        }
        umma::mma_commit(&mbar);
    }
    // in NO_ARRIVE mode nothing arrives: the wait runs out, flags the timeout
    // and returns false; no MMA is in flight, so the TMEM is freed safely
    const bool ok = umma::mbar_wait(&mbar, 0, wait_cycles > 0 ? wait_cycles : (1ll << 31));
    umma::fence_after_sync();
    if (ok) {
        for (int c = 0; c < N; c += 16) {
            float v[16];
            umma::tmem_ld16(tmem + lane_base + c, v);
#pragma unroll
            for (int j = 0; j < 16; ++j) D[row * N + c + j] = v[j];
        }
    }
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 0) umma::tmem_dealloc(tmem, kSelftestCols);
}

}  // namespace gdn

extern "C" int gdn_umma_selftest_ex(const float* A, const float* B, float* D, int N, int K, int a_mn,
                                    int b_mn, int fmt, int mode, long long wait_cycles, void* stream) {
    if (!A || !B || !D) return GDN_ERR_INVALID;
    if (N < 16 || N > 128 || N % 16 || K < 16 || K > 128 || K % 16) return GDN_ERR_UNSUPPORTED;
    if ((a_mn | b_mn | fmt) & ~1) return GDN_ERR_INVALID;
    if (mode & ~(GDN_SELFTEST_A_TMEM | GDN_SELFTEST_NO_ARRIVE)) return GDN_ERR_INVALID;
    if ((mode & GDN_SELFTEST_A_TMEM) && a_mn) return GDN_ERR_UNSUPPORTED;  // TMEM holds A K-major
    if (wait_cycles < 0) return GDN_ERR_INVALID;
    if (b_mn && N % 64 && N != 32) return GDN_ERR_UNSUPPORTED;  // MN-major: 64-wide blocks, or one 32-wide
    const size_t smem = 2 * 128 * 128 * 2 + 1024;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // this unit's status word starts clear, so the result is this call's own
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbolAsync(gdn::g_device_status, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, st) !=
        cudaSuccess)
        return GDN_ERR_CUDA;
    if (fmt) {
        auto kern = gdn::umma_selftest_kernel<__nv_bfloat16>;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return GDN_ERR_CUDA;
        kern<<<1, 128, smem, st>>>(A, B, D, N, K, a_mn, b_mn, fmt, mode, wait_cycles);
    } else {
        auto kern = gdn::umma_selftest_kernel<__half>;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return GDN_ERR_CUDA;
        kern<<<1, 128, smem, st>>>(A, B, D, N, K, a_mn, b_mn, fmt, mode, wait_cycles);
    }
    if (cudaGetLastError() != cudaSuccess) return GDN_ERR_CUDA;
    unsigned int status = 0;
    if (cudaMemcpyFromSymbolAsync(&status, gdn::g_device_status, sizeof(status), 0,
                                  cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return GDN_ERR_CUDA;
    return status ? GDN_ERR_DEVICE : GDN_OK;
}

extern "C" int gdn_umma_selftest(const float* A, const float* B, float* D, int N, int K, int a_mn,
                                 int b_mn, int fmt, void* stream) {
    return gdn_umma_selftest_ex(A, B, D, N, K, a_mn, b_mn, fmt, 0, 0, stream);
}
