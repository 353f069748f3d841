// gdn_prefill_chunk.cu — chunk-parallel varlen GDN prefill on the sm_100a
// tensor cores (tcgen05.mma into TMEM).
//
// Plays the role of AITER's chunk_gated_delta_rule in the reference solution
// (solutions/gdn_prefill/main.py:62-74) for the contest definition
// gdn_prefill_*_k_last (flashinfer/trace/templates/gdn.py:189-273).  The
// chunked form is the WY/UT representation of the delta rule (Yang et al.,
// "Parallelizing Linear Transformers with the Delta Rule over Sequence
// Length", NeurIPS 2024; "Gated Delta Networks", ICLR 2025), arranged here so
// that every tensor-core product is an M = 128 tile.
//
// Notation for one chunk of C = 64 tokens of one (sequence, v-head), with the
// state S as a [K = 128] x [V] matrix (k-last storage is S^T) and rows
// i, j = tokens of the chunk:
//   gamma_i = sum_{j<=i} log g_j  (in-chunk cumulative log decay), gamma_C = gamma_63
//   A_ij = beta_i e^{gamma_i-gamma_j} k_i.k_j   (j < i, else 0)
//   P_ij = scale e^{gamma_i-gamma_j} q_i.k_j    (j <= i, else 0)
//   T    = (I + A)^-1,  P' = P T
//   Y    = diag(beta) (V - diag(e^gamma) K S)
//   Delta= T Y                                 (the per-token delta-rule updates)
//   O    = diag(scale e^gamma) Q S + P' Y      (= scale q_i^T S_i for every token)
//   S   <- e^{gamma_C} S + (diag(e^{gamma_C-gamma}) K)^T Delta
// Only factors e^{x} with x <= 0 appear, so nothing overflows however strong
// the decay.  Tokens past the end of the sequence get k = q = v = beta = 0 and
// log g = 0, which leaves every formula exact for a partial last chunk.
//
// Two kernels:
//  * prep  (one CTA per (chunk, v-head), all chunks of all sequences at once):
//      the state-independent part — gates, gamma, MMA [K ; Q] K^T (bf16 as
//      given), the decay masks, T = (I + A)^-1 by a blocked solve on the CUDA
//      cores in fp32, and P' = P T on the tensor cores — and writes the f16
//      operand tile [T ; P'] (already in its shared-memory swizzled layout)
//      and the chunk's gate factors into a workspace slot.
//  * chain (one CTA per (sequence, v-head, 64-wide V tile), 8 warps): walks
//      the chunks in order with the state resident in TMEM (fp32):
//        MMA_1 : [K ; Q] x S     -> KS (rows 0-63: Y = beta (V - e^gamma KS)), QS (rows 64-127)
//        MMA_2 : [T ; P'] x Y    -> Delta (rows 0-63), P'Y (rows 64-127);
//                                   O = scale e^gamma QS + P'Y
//        MMA_3 : K^T x Delta~ with Delta~ = diag(e^{gamma_C - gamma}) Delta,
//                S = e^{gamma_C} S + K^T Delta~  (= K~^T Delta)
//      The diagonal scalings of Q and K are applied to rows of the products
//      instead of to the operands, so [K ; Q] is a plain f16 copy of the
//      input rows; and since the K rows of that K-major tile have exactly the
//      bytes of an MN-major K^T tile whose two 64-wide blocks sit 16 KiB
//      apart, MMA_3 reads K^T from the same tile.  The next chunk's rows and
//      workspace slot stream in with cp.async and are converted while MMA_3
//      of the current chunk runs.
// Operands are f16 except in the prep MMA (bf16 inputs as given); every
// accumulation is fp32 and the state carried between chunks is fp32.
//
// Workspace slot of chunk j of sequence n: floor(cu[n] / 64) + n + j, which is
// below floor(T / 64) + N for every chunk, so the workspace holds
// (floor(T / 64) + N) * HV slots of kSlotBytes.
#include "gdn_prefill_common.cuh"
#include "umma.cuh"

namespace gdn {
namespace chunk {

constexpr int C = 64;                    // tokens per chunk
constexpr int LDA = 68;                  // fp32 row stride of the solve matrices
constexpr uint32_t kTileTP = 16384;      // [T ; P'] f16, K-major 128 x 64
// Gate record of a chunk (fp32): beta e^gamma, beta, e^{gamma_C - gamma},
// scale e^gamma (64 each), then e^{gamma_C}.
constexpr uint32_t kGateBytes = 4 * 256 + 16;
constexpr int GR_BEG = 0, GR_BETA = 64, GR_FK = 128, GR_FQ = 192, GR_DECAY = 256;
constexpr uint32_t kSlotBytes = kTileTP + kGateBytes;
constexpr uint32_t kTileKQ = 32768;      // [K ; Q] f16, K-major 128 x 128

// Workspace: (floor(T/64) + N) chunk slots; per slot HV (chunk, v-head)
// records of kSlotBytes, then per slot H [K ; Q] tiles of kTileKQ.
__host__ __device__ inline long long ws_slots(int N, int T) { return (long long)(T / 64) + N; }
__device__ __forceinline__ unsigned char* ws_kq(const PrefillParams& p, const unsigned char* ws) {
    return const_cast<unsigned char*>(ws) + (size_t)ws_slots(p.N, p.T) * p.HV * kSlotBytes;
}

// Clock budget of one wait for MMA completion (~70 ms at 1.9 GHz; the MMAs of
// a chunk take microseconds).  On expiry the CTA stops, frees its TMEM and
// leaves kDevStatTimeout in the status word.
constexpr long long kWaitBudget = 1ll << 27;

__device__ __forceinline__ void st_f16x8(unsigned char* base, uint32_t off, const float* x) {
    __half2 h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
    *reinterpret_cast<uint4*>(base + off) = *reinterpret_cast<uint4*>(h);
}

__device__ __forceinline__ void unpack_bf16x8(const uint4& raw, float* x) {
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 f = __bfloat1622float2(b[i]);
        x[2 * i] = f.x;
        x[2 * i + 1] = f.y;
    }
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
    // src-size 0 zero-fills the 16 bytes without reading memory
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_n() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ bool wait_mma(uint64_t* bar, uint32_t parity) {
    // every thread waits; the CTA agrees on the outcome
    const bool ok = umma::mbar_wait(bar, parity, kWaitBudget);
    return !__syncthreads_or(!ok);
}

// Every thread waits on its own (the mbarrier orders the MMA's results for
// each waiter); a timeout is remembered in `failed` and acted on at the next
// CTA-wide vote.
__device__ __forceinline__ void wait_local(uint64_t* bar, uint32_t parity, bool& failed) {
    if (!umma::mbar_wait(bar, parity, kWaitBudget)) failed = true;
}

__device__ __forceinline__ void sync_for_mma() {
    umma::fence_proxy_async_smem();
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
}

// ============================================================================
// prep kernel
// ============================================================================
namespace prep {

constexpr int NT = 128;
constexpr uint32_t OFF_KQ = 0;                     // [K ; Q] bf16 K-major 128 x 128   32 KiB
// A and the level scratch X only live after MMA_A has consumed [K ; Q], so
// they share its 32 KiB; three CTAs fit on an SM.
constexpr uint32_t OFF_A = 0;                      // A fp32 [64][LDA]                 17 KiB
constexpr uint32_t OFF_X = OFF_A + 64 * LDA * 4;   // solve scratch, rows 16-63        12.75 KiB
constexpr uint32_t OFF_TP = 32768;                 // [T ; P] f16 K-major 128 x 64     16 KiB
constexpr uint32_t OFF_TB = OFF_TP + kTileTP;      // T as MN-major B (m x j) f16        8 KiB
constexpr uint32_t OFF_T = OFF_TB + 8192;          // T fp32 [64][LDA]                 17 KiB
constexpr uint32_t OFF_G = OFF_T + 64 * LDA * 4;   // gamma[64]
constexpr uint32_t OFF_BETA = OFF_G + 256;         // beta[64]
constexpr uint32_t SMEM_BYTES = OFF_BETA + 256 + 1024;  // + alignment slack
static_assert(OFF_X + 48 * LDA * 4 <= OFF_TP, "A and X fit in the [K ; Q] tile");
constexpr uint32_t TM_COLS = 64;

// Blocked T = (I + A)^-1 for the 64 x 64 strictly lower A in sA (fp32, row
// stride LDA); writes T into sT, whose upper blocks must already be zero.
// sX holds rows 16-63 of the level scratch X.
__device__ __forceinline__ void solve_T(const float* sA, float* sT, float* sX, int tid) {
    const int warp = tid >> 5, lane = tid & 31;
    // diagonal blocks: warp b inverts I + A_bb by right-looking substitution,
    // lane l < 16 owning column l
    if (lane < 16) {
        const int b0 = 16 * warp;
        float x[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) x[r] = (r == lane) ? 1.f : 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const float xj = x[j];
#pragma unroll
            for (int r = j + 1; r < 16; ++r) x[r] -= sA[(b0 + r) * LDA + b0 + j] * xj;
        }
#pragma unroll
        for (int r = 0; r < 16; ++r) sT[(b0 + r) * LDA + b0 + lane] = x[r];
    }
    __syncthreads();
    // off-diagonal blocks, level d = i - j: X_ij = sum_k A_ik T_kj, then
    // T_ij = -T_ii X_ij.  Thread -> (rows r0, r0 + 1; column c) of a block.
    const int c = tid & 15, r0 = (tid >> 4) * 2;
    // outer loops stay rolled: the kernel is large and instruction fetch,
    // not arithmetic, limits it
#pragma unroll 1
    for (int d = 1; d < 4; ++d) {
#pragma unroll 1
        for (int j = 0; j + d < 4; ++j) {
            const int i = j + d;
            float acc0 = 0.f, acc1 = 0.f;
#pragma unroll 1
            for (int k = j; k < i; ++k) {
                const float* a0 = sA + (16 * i + r0) * LDA + 16 * k;
                const float* tk = sT + (16 * k) * LDA + 16 * j + c;
#pragma unroll
                for (int s4 = 0; s4 < 16; s4 += 4) {
                    const float4 x0 = *reinterpret_cast<const float4*>(a0 + s4);
                    const float4 x1 = *reinterpret_cast<const float4*>(a0 + LDA + s4);
                    const float t0 = tk[(s4 + 0) * LDA], t1 = tk[(s4 + 1) * LDA];
                    const float t2 = tk[(s4 + 2) * LDA], t3 = tk[(s4 + 3) * LDA];
                    acc0 += x0.x * t0 + x0.y * t1 + x0.z * t2 + x0.w * t3;
                    acc1 += x1.x * t0 + x1.y * t1 + x1.z * t2 + x1.w * t3;
                }
            }
            sX[(16 * i + r0 - 16) * LDA + 16 * j + c] = acc0;
            sX[(16 * i + r0 - 15) * LDA + 16 * j + c] = acc1;
        }
        __syncthreads();
#pragma unroll 1
        for (int j = 0; j + d < 4; ++j) {
            const int i = j + d;
            const float* t0r = sT + (16 * i + r0) * LDA + 16 * i;
            const float* xc = sX + (16 * i - 16) * LDA + 16 * j + c;
            float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
            for (int s4 = 0; s4 < 16; s4 += 4) {
                const float4 y0 = *reinterpret_cast<const float4*>(t0r + s4);
                const float4 y1 = *reinterpret_cast<const float4*>(t0r + LDA + s4);
                const float x0 = xc[(s4 + 0) * LDA], x1 = xc[(s4 + 1) * LDA];
                const float x2 = xc[(s4 + 2) * LDA], x3 = xc[(s4 + 3) * LDA];
                acc0 += y0.x * x0 + y0.y * x1 + y0.z * x2 + y0.w * x3;
                acc1 += y1.x * x0 + y1.y * x1 + y1.z * x2 + y1.w * x3;
            }
            sT[(16 * i + r0) * LDA + 16 * j + c] = -acc0;
            sT[(16 * i + r0 + 1) * LDA + 16 * j + c] = -acc1;
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(NT, 3) gdn_prefill_chunk_prep_kernel(const PrefillParams p, unsigned char* ws) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t mbar[2];
    __shared__ uint32_t tmem_base_sh;

    const int tid = threadIdx.x, warp = tid >> 5;
    const long long s = blockIdx.x / p.HV;
    const int hv = blockIdx.x % p.HV, hq = hv / p.rep;

    // locate the chunk: the largest n with floor(cu[n] / 64) + n <= s, then j
    int lo = 0, hi = p.N - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        long long a, b;
        seq_bounds(p, mid, a, b);
        if (a / C + mid <= s) lo = mid; else hi = mid - 1;
    }
    const int n = lo;
    long long t0, t1;
    seq_bounds(p, n, t0, t1);
    const long long j = s - (t0 / C + n);
    if (j < 0 || t0 + C * j >= t1) return;  // slot of no chunk
    const long long tc = t0 + C * j;
    const int len = (int)((t1 - tc) < C ? (t1 - tc) : C);

    float* sA = reinterpret_cast<float*>(sm + OFF_A);
    float* sT = reinterpret_cast<float*>(sm + OFF_T);
    float* sX = reinterpret_cast<float*>(sm + OFF_X);
    float* sG = reinterpret_cast<float*>(sm + OFF_G);
    float* sBeta = reinterpret_cast<float*>(sm + OFF_BETA);

    // raw k rows -> [K ; Q] rows 0-63, q rows -> rows 64-127 (bf16, swizzled K-major)
    const uint32_t sKQ = umma::smem_u32(sm + OFF_KQ);
#pragma unroll
    for (int it = 0; it < C * 16 / NT; ++it) {
        const int idx = tid + it * NT, r = idx >> 4, c = idx & 15;
        const bool ok = r < len;
        const size_t row = ok ? ((size_t)(tc + r) * p.H + hq) * kDim + c * 8 : 0;
        cp_async16(sKQ + umma::kmaj_off(r, c * 8, 128), p.k + row, ok);
        cp_async16(sKQ + umma::kmaj_off(64 + r, c * 8, 128), p.q + row, ok);
    }
    cp_async_commit();
    for (int idx = tid; idx < 64 * 64; idx += NT) {  // T's upper blocks are zero
        const int i = idx >> 6, jj = idx & 63;
        if ((jj >> 4) > (i >> 4)) sT[i * LDA + jj] = 0.f;
    }
    // gates and the inclusive scan of log g (warps 0 and 1)
    float lg = 0.f, beta = 0.f;
    if (tid < len) {
        const size_t gi = (size_t)(tc + tid) * p.HV + hv;
        lg = log_gate(p.A_log[hv], bf16_to_f32(p.a[gi]), p.dt_bias[hv]);
        beta = sigmoidf_(bf16_to_f32(p.b[gi]));
    }
    if (warp < 2) {
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, lg, o);
            if ((tid & 31) >= o) lg += y;
        }
        if (warp == 0) sG[tid] = lg;
        sBeta[tid] = beta;
    }
    if (warp == 0) {
        umma::tmem_alloc(&tmem_base_sh, TM_COLS);
        umma::tmem_relinquish();
    }
    if (tid == 0) {
        umma::mbar_init(&mbar[0], 1);
        umma::mbar_init(&mbar[1], 1);
        umma::fence_mbar_init();
    }
    __syncthreads();
    if (warp == 1) sG[tid] = lg + sG[31];
    cp_async_wait_all();
    sync_for_mma();
    const uint32_t tmem = tmem_base_sh;
    const uint32_t lane_base = (uint32_t)(32 * warp) << 16;

    // MMA_A: [K ; Q] K^T in bf16
    if (tid == 0) {
        constexpr uint32_t ID = umma::idesc_f16(128, 64, 1, 1, 0, 0);
#pragma unroll
        for (int k0 = 0; k0 < kDim; k0 += 16)
            umma::mma_f16(tmem, umma::desc_kmaj(sKQ, 128, k0), umma::desc_kmaj(sKQ, 128, k0), ID, k0 > 0);
        umma::mma_commit(&mbar[0]);
    }
    if (!wait_mma(&mbar[0], 0)) goto done;
    umma::fence_after_sync();

    // the first v-head of each q/k head also publishes the chunk's [K ; Q]
    // tile for the chain kernel: the same swizzled layout, converted to f16
    if (hv % p.rep == 0) {
        uint4* dst = reinterpret_cast<uint4*>(ws_kq(p, ws) + ((size_t)s * p.H + hq) * kTileKQ);
#pragma unroll 4
        for (int idx = tid; idx < (int)(kTileKQ / 16); idx += NT) {
            float x[8];
            unpack_bf16x8(reinterpret_cast<const uint4*>(sm + OFF_KQ)[idx], x);
            __half2 h[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) h[e] = __floats2half2_rn(x[2 * e], x[2 * e + 1]);
            dst[idx] = *reinterpret_cast<uint4*>(h);
        }
    }
    __syncthreads();  // [K ; Q] is overwritten by A and X from here on

    // masks: rows 0-63 -> A (fp32), rows 64-127 -> P (f16, rows 64-127 of [T ; P])
    {
        const int i = tid & 63;
        const float gi = sG[i];
        const float bi = sBeta[i];
#pragma unroll 1
        for (int c16 = 0; c16 < C; c16 += 16) {
            float d[16];
            umma::tmem_ld16(tmem + lane_base + c16, d);
            float r[16];
            if (tid < 64) {
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const int jj = c16 + e;
                    r[e] = (jj < i) ? bi * __expf(fminf(gi - sG[jj], 0.f)) * d[e] : 0.f;
                }
#pragma unroll
                for (int e = 0; e < 16; e += 4)
                    *reinterpret_cast<float4*>(sA + i * LDA + c16 + e) = make_float4(r[e], r[e + 1], r[e + 2], r[e + 3]);
            } else {
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const int jj = c16 + e;
                    r[e] = (jj <= i) ? p.scale * __expf(fminf(gi - sG[jj], 0.f)) * d[e] : 0.f;
                }
                st_f16x8(sm + OFF_TP, umma::kmaj_off(64 + i, c16, 128), r);
                st_f16x8(sm + OFF_TP, umma::kmaj_off(64 + i, c16 + 8, 128), r + 8);
            }
        }
    }
    __syncthreads();

    // T = (I + A)^-1; f16 copies: rows 0-63 of [T ; P] and T as MN-major B
    solve_T(sA, sT, sX, tid);
    {
        const int i = tid >> 1, h = (tid & 1) * 32;  // row i, columns h..h+31
        const float* tr = sT + i * LDA + h;
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
            const float4 a = *reinterpret_cast<const float4*>(tr + c);
            const float4 b = *reinterpret_cast<const float4*>(tr + c + 4);
            const float x[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
            st_f16x8(sm + OFF_TP, umma::kmaj_off(i, h + c, 128), x);  // A rows: T[i][j]
            st_f16x8(sm + OFF_TB, umma::mnmaj_off(h + c, i, C), x);   // B: (n = m, k = j) = T[j][m]
        }
    }
    sync_for_mma();

    // MMA_P: [T ; P] T -> rows 64-127 = P' = P T
    if (tid == 0) {
        constexpr uint32_t ID = umma::idesc_f16(128, 64, 0, 0, 0, 1);
        const uint32_t sTP = umma::smem_u32(sm + OFF_TP), sTB = umma::smem_u32(sm + OFF_TB);
#pragma unroll
        for (int k0 = 0; k0 < C; k0 += 16)
            umma::mma_f16(tmem, umma::desc_kmaj(sTP, 128, k0), umma::desc_mnmaj(sTB, C, k0), ID, k0 > 0);
        umma::mma_commit(&mbar[1]);
    }
    if (!wait_mma(&mbar[1], 0)) goto done;
    umma::fence_after_sync();
    if (tid >= 64) {
        const int i = tid - 64;
#pragma unroll
        for (int c16 = 0; c16 < C; c16 += 16) {
            float d[16];
            umma::tmem_ld16(tmem + lane_base + c16, d);
            st_f16x8(sm + OFF_TP, umma::kmaj_off(64 + i, c16, 128), d);
            st_f16x8(sm + OFF_TP, umma::kmaj_off(64 + i, c16 + 8, 128), d + 8);
        }
    }
    __syncthreads();

    // slot <- [T ; P'] tile as laid out in shared memory, gamma, beta
    {
        unsigned char* slot = ws + ((size_t)s * p.HV + hv) * kSlotBytes;
#pragma unroll
        for (int it = 0; it < (int)(kTileTP / 16 / NT); ++it) {
            const int idx = tid + it * NT;
            reinterpret_cast<uint4*>(slot)[idx] = reinterpret_cast<const uint4*>(sm + OFF_TP)[idx];
        }
        float* gr = reinterpret_cast<float*>(slot + kTileTP);
        if (tid < 64) {  // gamma <= 0: every factor is in (0, 1] (times scale)
            const float eg = expf(sG[tid]);
            gr[GR_BEG + tid] = sBeta[tid] * eg;
            gr[GR_BETA + tid] = sBeta[tid];
            gr[GR_FK + tid] = expf(fminf(sG[C - 1] - sG[tid], 0.f));
            gr[GR_FQ + tid] = p.scale * eg;
        }
        if (tid < 4) gr[GR_DECAY + tid] = expf(sG[C - 1]);
    }

done:
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 0) umma::tmem_dealloc(tmem, TM_COLS);
}

}  // namespace prep

// ============================================================================
// chain kernel
// ============================================================================
namespace chain {

constexpr int NT = 256;  // 8 warps: TMEM lane quarter = warp % 4, column half = warp / 4
constexpr int NBUF = 3;  // data of chunk j lives in buffer j % 3
constexpr uint32_t TM_1 = 0, TM_2 = 64, TM_3 = 128, TM_S = 192, TM_COLS = 256;
constexpr int kLowerBarrier = 1;  // named barrier of the four warps on TMEM lanes 0-63

// VT state columns (v) per CTA: 64, or 32 when a 64-wide split would leave
// SMs idle (few sequences x v-heads).  The B operands S, Y and Delta~ have
// N = VT and are MN-major: 128-byte swizzle for 64 columns, 64-byte for 32.
template <int VT>
struct Cfg {
    static constexpr int HALF = VT / 2;                     // columns per thread
    static constexpr uint32_t VROW = VT * 2 + 16;           // raw v row stride (padded)
    static constexpr uint32_t S_BYTES = VT * kDim * 2;      // S f16 tile
    static constexpr uint32_t YD_BYTES = VT * C * 2;        // Y / Delta~ f16 tiles
    static constexpr uint32_t OFF_KQ = 0;                         // [K ; Q] (workspace copy), 3 bufs
    static constexpr uint32_t OFF_TP = OFF_KQ + NBUF * kTileKQ;   // [T ; P'] (workspace copy), 3 bufs
    static constexpr uint32_t OFF_SH = OFF_TP + NBUF * kTileTP;   // S, MN-major (v x k)
    static constexpr uint32_t OFF_Y = OFF_SH + S_BYTES;           // Y, MN-major (v x token)
    static constexpr uint32_t OFF_DL = OFF_Y + YD_BYTES;          // Delta~, MN-major (v x token)
    static constexpr uint32_t OFF_RV = OFF_DL + YD_BYTES;         // v rows bf16 [3][64][VROW]
    static constexpr uint32_t OFF_GB = OFF_RV + NBUF * C * VROW;  // gate records, 3 bufs
    static constexpr uint32_t SMEM_BYTES = OFF_GB + NBUF * kGateBytes + 1024;
    static_assert(SMEM_BYTES <= 232448, "dynamic shared memory limit");
    static_assert(OFF_Y % 1024 == 0 && OFF_DL % 1024 == 0 && OFF_RV % 16 == 0, "tile alignment");

    // byte offset of element (v, k) of an MN-major B tile whose K extent is kext
    static __device__ __forceinline__ uint32_t b_off(uint32_t v, uint32_t k, uint32_t kext) {
        if constexpr (VT == 32) return umma::mnmaj64_off(v, k);
        else return umma::mnmaj_off(v, k, kext);
    }
    static __device__ __forceinline__ uint64_t b_desc(uint32_t tile, uint32_t kext, uint32_t k0) {
        if constexpr (VT == 32) return umma::desc_mnmaj64(tile, k0);
        else return umma::desc_mnmaj(tile, kext, k0);
    }
    static __device__ __forceinline__ void ld(uint32_t taddr, float (&v)[HALF]) {
        if constexpr (HALF == 16) umma::tmem_ld16(taddr, v);
        else umma::tmem_ld32(taddr, v);
    }
    static __device__ __forceinline__ void ld2(uint32_t ta, uint32_t tb, float (&va)[HALF], float (&vb)[HALF]) {
        if constexpr (HALF == 16) umma::tmem_ld16x2(ta, tb, va, vb);
        else umma::tmem_ld32x2(ta, tb, va, vb);
    }
    static __device__ __forceinline__ void st(uint32_t taddr, const float (&v)[HALF]) {
        if constexpr (HALF == 16) umma::tmem_st16(taddr, v);
        else umma::tmem_st32(taddr, v);
    }
};

__device__ __forceinline__ void lower_sync() {
    asm volatile("bar.sync %0, %1;" ::"r"(kLowerBarrier), "r"(128) : "memory");
}

// Copies of chunk [tc, tc + len) (workspace slot `slot`) into buffer `buf`:
// the loader warp starts three bulk copies of the [K ; Q] and [T ; P'] tiles
// and the gates, completing on `bar`; every thread copies its share of the v
// rows with cp.async (rows past len zero-filled) as one commit group.
template <int VT>
__device__ __forceinline__ void issue_loads(const PrefillParams& p, const unsigned char* ws, unsigned char* sm,
                                            uint64_t* bar, int buf, long long tc, int len, long long slot,
                                            int hq, int hv, int v0, int tid, bool loader) {
    if (loader) {
        const int lane = tid & 31;
        using G = Cfg<VT>;
        if (lane == 0) umma::mbar_arrive_expect_tx(bar, kTileKQ + kTileTP + kGateBytes);
        __syncwarp();
        const unsigned char* rec = ws + ((size_t)slot * p.HV + hv) * kSlotBytes;
        const unsigned char* kq = ws_kq(p, ws) + ((size_t)slot * p.H + hq) * kTileKQ;
        if (lane == 0) umma::bulk_g2s(umma::smem_u32(sm + G::OFF_KQ + buf * kTileKQ), kq, kTileKQ / 2, bar);
        if (lane == 1)
            umma::bulk_g2s(umma::smem_u32(sm + G::OFF_KQ + buf * kTileKQ + kTileKQ / 2), kq + kTileKQ / 2,
                           kTileKQ / 2, bar);
        if (lane == 2) umma::bulk_g2s(umma::smem_u32(sm + G::OFF_TP + buf * kTileTP), rec, kTileTP, bar);
        if (lane == 3)
            umma::bulk_g2s(umma::smem_u32(sm + G::OFF_GB + buf * kGateBytes), rec + kTileTP, kGateBytes, bar);
    }
    constexpr uint32_t VROW = Cfg<VT>::VROW;
    const uint32_t rv = umma::smem_u32(sm + Cfg<VT>::OFF_RV) + buf * (C * VROW);
#pragma unroll
    for (int it = 0; it < C * (VT / 8) / NT; ++it) {
        const int idx = tid + it * NT, r = idx / (VT / 8), c = idx % (VT / 8);
        const bool ok = r < len;
        const size_t off = ok ? ((size_t)(tc + r) * p.HV + hv) * kDim + v0 + c * 8 : 0;
        cp_async16(rv + r * VROW + c * 16, p.v + off, ok);
    }
    cp_async_commit();
}

template <int VT>
__global__ void __launch_bounds__(NT, 1) gdn_prefill_chunk_chain_kernel(const PrefillParams p,
                                                                        const unsigned char* ws) {
    using G = Cfg<VT>;
    constexpr int HALF = G::HALF;
    constexpr uint32_t VROW = G::VROW;
    constexpr uint32_t OFF_KQ = G::OFF_KQ, OFF_TP = G::OFF_TP, OFF_SH = G::OFF_SH, OFF_Y = G::OFF_Y;
    constexpr uint32_t OFF_DL = G::OFF_DL, OFF_RV = G::OFF_RV, OFF_GB = G::OFF_GB;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t mbar[3];   // MMA_1, MMA_2, MMA_3 completion
    __shared__ uint64_t ldbar[NBUF];  // chunk data of buffer 0 / 1 / 2 landed
    __shared__ uint32_t tmem_base_sh;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quarter = warp & 3, half = warp >> 2;
    const bool lower = quarter < 2;       // TMEM lanes 0-63: the K rows (Y, Delta~)
    const int row = 32 * quarter + lane;  // TMEM lane owned by this thread
    const int vt = blockIdx.x % (kDim / VT);
    const long long nh = blockIdx.x / (kDim / VT);
    const int hv = (int)(nh % p.HV), n = (int)(nh / p.HV);
    const int hq = hv / p.rep;
    const int v0 = vt * VT;
    const int cb = HALF * half;  // this thread's first column within the tile
    constexpr int kLoader = 2;   // warp issuing the bulk copies

    long long t0, t1;
    seq_bounds(p, n, t0, t1);
    if (tid < VT) zero_uncovered_outputs(p, n, t0, t1, hv, v0 + tid, true);
    const size_t state_off = ((size_t)nh * kDim + v0) * kDim;  // [n][hv][v0][0]
    if (t1 == t0) {  // empty sequence: the final state stays zero
        for (int idx = tid; idx < VT * kDim / 4; idx += NT)
            reinterpret_cast<float4*>(p.new_state + state_off)[idx] = make_float4(0.f, 0.f, 0.f, 0.f);
        return;
    }
    const long long slot0 = t0 / C + n;
    const long long nchunks = (t1 - t0 + C - 1) / C;
    auto chunk_len = [&](long long j) { const long long r = t1 - t0 - C * j; return (int)(r < C ? r : C); };

    if (warp == 0) {
        umma::tmem_alloc(&tmem_base_sh, TM_COLS);
        umma::tmem_relinquish();
    }
    if (tid == 0) {
#pragma unroll
        for (int b = 0; b < 3; ++b) umma::mbar_init(&mbar[b], 1);
#pragma unroll
        for (int b = 0; b < NBUF; ++b) umma::mbar_init(&ldbar[b], 1);
        umma::fence_mbar_init();
    }
    __syncthreads();
    issue_loads<VT>(p, ws, sm, &ldbar[0], 0, t0, chunk_len(0), slot0, hq, hv, v0, tid, warp == kLoader);
    if (nchunks > 1)
        issue_loads<VT>(p, ws, sm, &ldbar[1], 1, t0 + C, chunk_len(1), slot0 + 1, hq, hv, v0, tid, warp == kLoader);
    umma::fence_after_sync();
    const uint32_t tmem = tmem_base_sh;
    const uint32_t tl = tmem + ((uint32_t)(32 * quarter) << 16);  // this warp's lane quarter

    // initial state: S[k = row][v] for this thread's 32 columns -> TMEM (fp32) and f16 operand
    {
        float sv[HALF];
#pragma unroll
        for (int e = 0; e < HALF; ++e) sv[e] = p.state ? p.state[state_off + (size_t)(cb + e) * kDim + row] : 0.f;
        G::st(tl + TM_S + cb, sv);
#pragma unroll
        for (int c8 = 0; c8 < HALF; c8 += 8) st_f16x8(sm + OFF_SH, G::b_off(cb + c8, row, kDim), sv + c8);
    }
    // chunk 0's v rows (copied by all threads) become visible at the barrier
    if (nchunks > 1) cp_async_wait_n<1>(); else cp_async_wait_n<0>();
    sync_for_mma();
    bool failed = false;

    const uint32_t sKQ0 = umma::smem_u32(sm + OFF_KQ), sTP0 = umma::smem_u32(sm + OFF_TP);
    const uint32_t sSH = umma::smem_u32(sm + OFF_SH), sY = umma::smem_u32(sm + OFF_Y);
    const uint32_t sDL = umma::smem_u32(sm + OFF_DL);
    constexpr uint32_t ID_S = umma::idesc_f16(128, VT, 0, 0, 0, 1);  // [K;Q] x S (MN-major B)
    constexpr uint32_t ID_Y = umma::idesc_f16(128, VT, 0, 0, 0, 1);  // [T;P'] x Y (MN-major B)
    constexpr uint32_t ID_D = umma::idesc_f16(128, VT, 0, 0, 1, 1);  // K^T x Delta~ (both MN-major)

    for (long long j = 0; j < nchunks; ++j) {
        const int b = (int)(j % NBUF);
        const uint32_t par = (uint32_t)(j & 1), lpar = (uint32_t)((j / NBUF) & 1);
        const long long tc = t0 + C * j;
        const int len = chunk_len(j);
        wait_local(&ldbar[b], lpar, failed);
        const float* gr = reinterpret_cast<const float*>(sm + OFF_GB + b * kGateBytes);
        const uint32_t sKQ = sKQ0 + b * kTileKQ;

        // ---- MMA_1: [K ; Q] S ----
        if (tid == 0) {
            umma::fence_after_sync();
#pragma unroll
            for (int k0 = 0; k0 < kDim; k0 += 16)
                umma::mma_f16(tmem + TM_1, umma::desc_kmaj(sKQ, 128, k0), G::b_desc(sSH, kDim, k0), ID_S,
                              k0 > 0);
            umma::mma_commit(&mbar[0]);
        }
        // while MMA_1 runs: stream in chunk j + 2 (its buffer was chunk j - 1's)
        if (j + 2 < nchunks)
            issue_loads<VT>(p, ws, sm, &ldbar[(j + 2) % NBUF], (int)((j + 2) % NBUF), tc + 2 * C, chunk_len(j + 2),
                        slot0 + j + 2, hq, hv, v0, tid, warp == kLoader);
        wait_local(&mbar[0], par, failed);
        umma::fence_after_sync();

        // ---- lower: Y = beta (V - e^gamma KS) -> MMA_2;  upper: keep QS ----
        float qs[HALF];
        {
            float d[HALF];
            G::ld(tl + TM_1 + cb, d);
            if (lower) {
                const int i = row;
                const bool live = i < len;
                const float beg = gr[GR_BEG + i], b_i = gr[GR_BETA + i];
                const unsigned char* vrow = sm + OFF_RV + b * (C * VROW) + i * VROW + cb * 2;
#pragma unroll
                for (int c8 = 0; c8 < HALF; c8 += 8) {
                    float vv[8], y[8];
                    unpack_bf16x8(*reinterpret_cast<const uint4*>(vrow + c8 * 2), vv);
#pragma unroll
                    for (int e = 0; e < 8; ++e) y[e] = live ? fmaf(-beg, d[c8 + e], b_i * vv[e]) : 0.f;
                    st_f16x8(sm + OFF_Y, G::b_off(cb + c8, i, C), y);
                }
                umma::fence_proxy_async_smem();
                umma::fence_before_sync();
                lower_sync();
                if (tid == 0) {
                    umma::fence_after_sync();
                    const uint32_t sTP = sTP0 + b * kTileTP;
#pragma unroll
                    for (int k0 = 0; k0 < C; k0 += 16)
                        umma::mma_f16(tmem + TM_2, umma::desc_kmaj(sTP, 128, k0), G::b_desc(sY, C, k0), ID_Y,
                                      k0 > 0);
                    umma::mma_commit(&mbar[1]);
                }
            } else {
#pragma unroll
                for (int e = 0; e < HALF; ++e) qs[e] = d[e];
            }
        }
        wait_local(&mbar[1], par, failed);
        umma::fence_after_sync();

        // ---- lower: Delta~ = e^{gamma_C - gamma} Delta -> MMA_3;  upper: outputs ----
        {
            float d[HALF];
            G::ld(tl + TM_2 + cb, d);
            if (lower) {
                const float fk = gr[GR_FK + row];
#pragma unroll
                for (int e = 0; e < HALF; ++e) d[e] *= fk;
#pragma unroll
                for (int c8 = 0; c8 < HALF; c8 += 8) st_f16x8(sm + OFF_DL, G::b_off(cb + c8, row, C), d + c8);
                umma::fence_proxy_async_smem();
                umma::fence_before_sync();
                lower_sync();
                if (tid == 0) {
                    // K^T read as MN-major from the [K ; Q] tile: its two 64-wide k
                    // blocks are the tile's 16 KiB slabs
                    umma::fence_after_sync();
#pragma unroll
                    for (int k0 = 0; k0 < C; k0 += 16)
                        umma::mma_f16(tmem + TM_3, umma::desc_sw128(sKQ + (k0 >> 3) * 1024u, 16384u, 1024u),
                                      G::b_desc(sDL, C, k0), ID_D, k0 > 0);
                    umma::mma_commit(&mbar[2]);
                }
            } else {
                const int i = row - 64;
                if (i < len) {
                    const float fq = gr[GR_FQ + i];  // scale e^{gamma_i}
                    __nv_bfloat16* op = p.out + ((size_t)(tc + i) * p.HV + hv) * kDim + v0 + cb;
#pragma unroll
                    for (int c8 = 0; c8 < HALF; c8 += 8) {
                        __nv_bfloat162 o[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            o[e] = __floats2bfloat162_rn(fmaf(fq, qs[c8 + 2 * e], d[c8 + 2 * e]),
                                                         fmaf(fq, qs[c8 + 2 * e + 1], d[c8 + 2 * e + 1]));
                        *reinterpret_cast<uint4*>(op + c8) = *reinterpret_cast<uint4*>(o);
                    }
                }
            }
        }
        wait_local(&mbar[2], par, failed);
        umma::fence_after_sync();

        // ---- S = e^{gamma_C} S + K^T Delta~ (TMEM, fp32) and its f16 operand copy ----
        {
            const float decay = gr[GR_DECAY];
            float sv[HALF], d[HALF];
            G::ld2(tl + TM_S + cb, tl + TM_3 + cb, sv, d);
#pragma unroll
            for (int e = 0; e < HALF; ++e) sv[e] = fmaf(decay, sv[e], d[e]);
            G::st(tl + TM_S + cb, sv);
#pragma unroll
            for (int c8 = 0; c8 < HALF; c8 += 8) st_f16x8(sm + OFF_SH, G::b_off(cb + c8, row, kDim), sv + c8);
            // checkpoint: a full chunk that ends on a multiple of ckpt_every
            if (p.ckpt != nullptr && len == C && (C * (j + 1)) % p.ckpt_every == 0) {
                float* cd = ckpt_dst(p, n, hv, C * (j + 1));
                if (cd != nullptr) {
#pragma unroll
                    for (int e = 0; e < HALF; ++e) __stcs(cd + (size_t)(v0 + cb + e) * kDim + row, sv[e]);
                }
            }
        }
        // the next chunk's v rows (copied by all threads) become visible at this barrier;
        // the CTA stops here if any wait of this chunk timed out
        if (j + 2 < nchunks) cp_async_wait_n<1>(); else cp_async_wait_n<0>();
        umma::fence_proxy_async_smem();
        umma::fence_before_sync();
        if (__syncthreads_or(failed)) goto done;
        umma::fence_after_sync();
    }

    // final state (fp32, k-last): for each v, consecutive threads write consecutive k
    {
        float sv[HALF];
        G::ld(tl + TM_S + cb, sv);
#pragma unroll
        for (int e = 0; e < HALF; ++e) __stcs(p.new_state + state_off + (size_t)(cb + e) * kDim + row, sv[e]);
    }

done:
    cp_async_wait_all();  // no copy may still target shared memory when the CTA exits
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 0) umma::tmem_dealloc(tmem, TM_COLS);
}

}  // namespace chain
}  // namespace chunk

size_t prefill_workspace_bytes(int N, int T, int H, int HV) {
    return (size_t)chunk::ws_slots(N, T) * ((size_t)HV * chunk::kSlotBytes + (size_t)H * chunk::kTileKQ);
}

void launch_prefill_chunk(const PrefillParams& p, void* workspace, cudaStream_t st) {
    static bool attr_set = false;
    static int num_sms = 148;
    if (!attr_set) {
        cudaFuncSetAttribute(chunk::prep::gdn_prefill_chunk_prep_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)chunk::prep::SMEM_BYTES);
        cudaFuncSetAttribute(chunk::chain::gdn_prefill_chunk_chain_kernel<64>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)chunk::chain::Cfg<64>::SMEM_BYTES);
        cudaFuncSetAttribute(chunk::chain::gdn_prefill_chunk_chain_kernel<32>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)chunk::chain::Cfg<32>::SMEM_BYTES);
        int dev = 0, sms = 0;
        if (cudaGetDevice(&dev) == cudaSuccess &&
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && sms > 0)
            num_sms = sms;
        attr_set = true;
    }
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    const long long slots = chunk::ws_slots(p.N, p.T);
    chunk::prep::gdn_prefill_chunk_prep_kernel<<<(unsigned)(slots * p.HV), chunk::prep::NT,
                                                 chunk::prep::SMEM_BYTES, st>>>(p, ws);
    // one chain per (sequence, v-head, V tile): split V into 32-wide tiles when
    // 64-wide ones would not cover the SMs (e.g. a single long sequence)
    const long long chains64 = (long long)p.N * p.HV * (kDim / 64);
    if (chains64 < num_sms) {
        chunk::chain::gdn_prefill_chunk_chain_kernel<32><<<(unsigned)(chains64 * 2), chunk::chain::NT,
                                                           chunk::chain::Cfg<32>::SMEM_BYTES, st>>>(p, ws);
    } else {
        chunk::chain::gdn_prefill_chunk_chain_kernel<64><<<(unsigned)chains64, chunk::chain::NT,
                                                           chunk::chain::Cfg<64>::SMEM_BYTES, st>>>(p, ws);
    }
}

}  // namespace gdn

extern "C" int gdn_device_status(int clear) {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, gdn::g_device_status, sizeof(v)) != cudaSuccess) return -1;
    if (clear && v) {
        const unsigned int z = 0;
        if (cudaMemcpyToSymbol(gdn::g_device_status, &z, sizeof(z)) != cudaSuccess) return -1;
    }
    return (int)v;
}
