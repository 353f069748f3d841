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
// One CTA (128 threads, thread t <-> TMEM lane t) owns one (sequence, v-head,
// 64-wide V tile) and walks its chunks in order.  Per chunk:
//   MMA_A : [K ; Q] (128 x 128) x K^T           -> TMEM cols [0, 64)
//   masks : rows 0-63 -> A (fp32, smem), rows 64-127 -> P (f16, A operand)
//   MMA_1 : [K ; diag(scale e^gamma) Q] x S      -> TMEM cols [64, 128)  (overlaps the solve)
//   solve : T = (I + A)^-1 on the CUDA cores in fp32, blocked by 16:
//           the four diagonal blocks by right-looking substitution (one warp
//           each), then the off-diagonal blocks level by level,
//           T_ij = -T_ii sum_{k=j}^{i-1} A_ik T_kj
//   MMA_P : [T ; P] (128 x 64) x T               -> rows 64-127 = P' = P T
//   Y     : rows 0-63 (f16, smem);  rows 64-127 keep Q~S for the output
//   MMA_2 : [T ; P'] (128 x 64) x Y              -> TMEM cols [128, 192)
//   out   : rows 64-127: O = Q~S + P'Y -> bf16 -> HBM;  rows 0-63: Delta (f16, smem)
//   MMA_3 : K~^T (128 x 64, MN-major) x Delta    -> TMEM cols [192, 256)
//   state : S = e^{gamma_C} S + K~^T Delta (fp32, smem), f16 copy for MMA_1
// Operands are f16 (inputs are bf16 with |q|,|k| <= 1 after L2-normalisation;
// f16 keeps 3 more mantissa bits), accumulation is fp32 in TMEM and the state
// carried between chunks is fp32.
#include "gdn_prefill_common.cuh"
#include "umma.cuh"

namespace gdn {
namespace chunk {

constexpr int C = 64;    // tokens per chunk
constexpr int VT = 64;   // state columns (v) per CTA
constexpr int NT = 128;  // threads per CTA

// Shared-memory map (bytes from a 1024-byte aligned base).
constexpr int LDA = 68;                         // fp32 row stride of the solve matrices
constexpr uint32_t OFF_KQ = 0;                  // [K ; Q] K-major 128 x 128 f16      32 KiB
constexpr uint32_t OFF_TP = OFF_KQ + 32768;     // [T ; P'] K-major 128 x 64 f16      16 KiB
constexpr uint32_t OFF_TB = OFF_TP + 16384;     // T as MN-major B (m x j) f16         8 KiB
constexpr uint32_t OFF_SH = OFF_TB + 8192;      // S^T K-major VT x 128 f16 (B op)    16 KiB
constexpr uint32_t OFF_Y = OFF_SH + 16384;      // Y MN-major (v x 64 tokens) f16      8 KiB
constexpr uint32_t OFF_DL = OFF_Y + 8192;       // Delta MN-major (v x 64 tokens) f16  8 KiB
constexpr uint32_t OFF_KT = OFF_DL + 8192;      // K~ MN-major (k x 64 tokens) f16    16 KiB
constexpr uint32_t OFF_SF = OFF_KT + 16384;     // S fp32 [v][k] (VT x 128)           32 KiB
constexpr uint32_t OFF_A = OFF_SF + 32768;      // A fp32 [64][LDA]                   17 KiB
constexpr uint32_t OFF_T = OFF_A + 64 * LDA * 4;  // T fp32 [64][LDA]                 17 KiB
// solve scratch: rows 16-63 of a [64][LDA] fp32 matrix (12.75 KiB), aliased onto
// the Y / Delta tiles, which are idle while T is being solved
constexpr uint32_t OFF_X = OFF_Y;
constexpr uint32_t OFF_RK = OFF_T + 64 * LDA * 4;  // raw next-chunk k rows bf16 [64][128]  16 KiB
constexpr uint32_t OFF_RQ = OFF_RK + 16384;        // raw next-chunk q rows bf16 [64][128]  16 KiB
constexpr uint32_t OFF_RV = OFF_RQ + 16384;        // raw v rows bf16 [2][64][VT] (swizzled) 16 KiB
constexpr uint32_t OFF_G = OFF_RV + 2 * C * VT * 2;  // gamma[64] fp32
constexpr uint32_t OFF_BETA = OFF_G + 256;      // beta[64] fp32
constexpr uint32_t SMEM_USED = OFF_BETA + 256;
constexpr uint32_t SMEM_BYTES = SMEM_USED + 1024;  // + alignment slack
static_assert(48 * LDA * 4 <= 16384, "solve scratch fits the Y / Delta tiles");
static_assert(SMEM_BYTES <= 232448, "dynamic shared memory limit");

constexpr uint32_t TM_A = 0, TM_1 = 64, TM_2 = 128, TM_3 = 192, TM_COLS = 256;

// Clock budget of one wait for MMA completion (~70 ms at 1.9 GHz; a chunk's
// MMAs take microseconds).  On expiry the CTA stops, frees its TMEM and
// leaves kDevStatTimeout in the status word.
constexpr long long kWaitBudget = 1ll << 27;

__device__ __forceinline__ void st_f16x8(unsigned char* base, uint32_t off, const float* x) {
    __half2 h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
    *reinterpret_cast<uint4*>(base + off) = *reinterpret_cast<uint4*>(h);
}

__device__ __forceinline__ void ld_bf16x8(const __nv_bfloat16* p, float* x) {
    uint4 raw = *reinterpret_cast<const uint4*>(p);
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

// Raw-row buffers of one chunk: q and k rows [64][128] bf16, linear; v rows
// [64][VT] bf16 with 16-byte chunk c of row r stored at c ^ (r & 7).
__device__ __forceinline__ uint32_t rawv_off(int r, int c) { return r * (VT * 2) + ((c ^ (r & 7)) << 4); }

// Issues the asynchronous copies of chunk [tc, tc + len) into the raw buffers
// (rows past len are zero-filled).  Piece idx of q / k is copied by thread
// idx % NT, the same thread that later converts it.
__device__ __forceinline__ void prefetch_chunk(const PrefillParams& p, uint32_t rk, uint32_t rq, uint32_t rv,
                                               long long tc, int len, int hq, int hv, int v0, int tid) {
#pragma unroll
    for (int it = 0; it < C * 16 / NT; ++it) {
        const int idx = tid + it * NT, r = idx >> 4, c = idx & 15;
        const bool ok = r < len;
        const size_t row = ok ? ((size_t)(tc + r) * p.H + hq) * kDim + c * 8 : 0;
        cp_async16(rk + idx * 16, p.k + row, ok);
        cp_async16(rq + idx * 16, p.q + row, ok);
    }
#pragma unroll
    for (int it = 0; it < C * (VT / 8) / NT; ++it) {
        const int idx = tid + it * NT, r = idx / (VT / 8), c = idx % (VT / 8);
        const bool ok = r < len;
        const size_t off = ok ? ((size_t)(tc + r) * p.HV + hv) * kDim + v0 + c * 8 : 0;
        cp_async16(rv + rawv_off(r, c), p.v + off, ok);
    }
    cp_async_commit();
}

// Converts raw bf16 q / k rows into the f16 K-major [K ; Q] operand tile.
__device__ __forceinline__ void convert_qk(unsigned char* sm, int tid) {
#pragma unroll
    for (int it = 0; it < C * 16 / NT; ++it) {
        const int idx = tid + it * NT, r = idx >> 4, c = idx & 15;
        float x[8];
        ld_bf16x8(reinterpret_cast<const __nv_bfloat16*>(sm + OFF_RK + idx * 16), x);
        st_f16x8(sm + OFF_KQ, umma::kmaj_off(r, c * 8, 128), x);
        ld_bf16x8(reinterpret_cast<const __nv_bfloat16*>(sm + OFF_RQ + idx * 16), x);
        st_f16x8(sm + OFF_KQ, umma::kmaj_off(64 + r, c * 8, 128), x);
    }
}

// Blocked T = (I + A)^-1 for the 64 x 64 strictly lower A in sA (fp32,
// row stride LDA); writes T into sT (upper blocks must already be zero).
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
    // off-diagonal blocks, level d = i - j: X_ij = sum_k A_ik T_kj, then T_ij = -T_ii X_ij.
    // Thread -> (rows r0, r0+1; column c) of a 16 x 16 block.
    const int c = tid & 15, r0 = (tid >> 4) * 2;
#pragma unroll
    for (int d = 1; d < 4; ++d) {
#pragma unroll
        for (int j = 0; j + d < 4; ++j) {
            const int i = j + d;
            float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
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
            sX[(16 * i + r0 - 16) * LDA + 16 * j + c] = acc0;  // sX holds rows 16-63
            sX[(16 * i + r0 - 15) * LDA + 16 * j + c] = acc1;
        }
        __syncthreads();
#pragma unroll
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

__global__ void __launch_bounds__(NT, 1) gdn_prefill_chunk_kernel(const PrefillParams p) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t mbar[5];
    __shared__ uint32_t tmem_base_sh;

    const int tid = threadIdx.x, warp = tid >> 5;
    const int vt = blockIdx.x % (kDim / VT);
    const long long nh = blockIdx.x / (kDim / VT);
    const int hv = (int)(nh % p.HV), n = (int)(nh / p.HV);
    const int hq = hv / p.rep;
    const int v0 = vt * VT;

    long long t0, t1;
    seq_bounds(p, n, t0, t1);
    if (tid < VT) zero_uncovered_outputs(p, n, t0, t1, hv, v0 + tid, true);

    float* sSf = reinterpret_cast<float*>(sm + OFF_SF);  // [v][k]
    float* sA = reinterpret_cast<float*>(sm + OFF_A);    // [i][j], stride LDA
    float* sT = reinterpret_cast<float*>(sm + OFF_T);    // [i][j], stride LDA
    float* sX = reinterpret_cast<float*>(sm + OFF_X);
    float* sG = reinterpret_cast<float*>(sm + OFF_G);
    float* sBeta = reinterpret_cast<float*>(sm + OFF_BETA);
    const size_t state_off = ((size_t)nh * kDim + v0) * kDim;  // new_state[n][hv][v0][0]

    if (t1 == t0) {  // empty sequence: the final state stays zero
        for (int idx = tid; idx < VT * kDim / 4; idx += NT)
            reinterpret_cast<float4*>(p.new_state + state_off)[idx] = make_float4(0.f, 0.f, 0.f, 0.f);
        return;
    }

    // initial state: fp32 [v][k] in smem and its f16 K-major copy (B of MMA_1)
    for (int idx = tid; idx < VT * kDim; idx += NT) {
        const int v = idx >> 7, k = idx & 127;
        const float s = p.state ? p.state[state_off + idx] : 0.f;
        sSf[idx] = s;
        *reinterpret_cast<__half*>(sm + OFF_SH + umma::kmaj_off(v, k, VT)) = __float2half_rn(s);
    }
    // T is lower triangular: its upper blocks stay zero for the whole kernel
    for (int idx = tid; idx < 64 * 64; idx += NT) {
        const int i = idx >> 6, j = idx & 63;
        if ((j >> 4) > (i >> 4)) sT[i * LDA + j] = 0.f;
    }

    if (warp == 0) {
        umma::tmem_alloc(&tmem_base_sh, TM_COLS);
        umma::tmem_relinquish();
    }
    if (tid == 0) {
#pragma unroll
        for (int b = 0; b < 5; ++b) umma::mbar_init(&mbar[b], 1);
        umma::fence_mbar_init();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = tmem_base_sh;
    const uint32_t lane_base = (uint32_t)(32 * warp) << 16;

    const uint32_t sKQ = umma::smem_u32(sm + OFF_KQ), sTP = umma::smem_u32(sm + OFF_TP);
    const uint32_t sTB = umma::smem_u32(sm + OFF_TB);
    const uint32_t sSH = umma::smem_u32(sm + OFF_SH), sY = umma::smem_u32(sm + OFF_Y);
    const uint32_t sDL = umma::smem_u32(sm + OFF_DL), sKT = umma::smem_u32(sm + OFF_KT);
    constexpr uint32_t ID_KK = umma::idesc_f16(128, 64, 0, 0, 0, 0);   // [K;Q] x K
    constexpr uint32_t ID_S = umma::idesc_f16(128, VT, 0, 0, 0, 0);    // [K;Q~] x S
    constexpr uint32_t ID_P = umma::idesc_f16(128, 64, 0, 0, 0, 1);    // [T;P] x T (MN-major B)
    constexpr uint32_t ID_Y = umma::idesc_f16(128, VT, 0, 0, 0, 1);    // [T;P'] x Y (MN-major B)
    constexpr uint32_t ID_D = umma::idesc_f16(128, VT, 0, 0, 1, 1);    // K~^T x Delta

    const float A_log = p.A_log[hv], dt_bias = p.dt_bias[hv];
    const float scale = p.scale;
    uint32_t parity = 0;

    // first chunk's rows and gates
    const uint32_t rawK = umma::smem_u32(sm + OFF_RK), rawQ = umma::smem_u32(sm + OFF_RQ);
    const uint32_t rawV = umma::smem_u32(sm + OFF_RV);
    int buf = 0;
    __nv_bfloat16 ga = __float2bfloat16_rn(0.f), gb = ga;
    {
        const int l0 = (int)((t1 - t0) < C ? (t1 - t0) : C);
        prefetch_chunk(p, rawK, rawQ, rawV, t0, l0, hq, hv, v0, tid);
        if (tid < l0) {
            ga = p.a[(size_t)(t0 + tid) * p.HV + hv];
            gb = p.b[(size_t)(t0 + tid) * p.HV + hv];
        }
    }

    for (long long tc = t0; tc < t1; tc += C, parity ^= 1, buf ^= 1) {
        const int len = (int)((t1 - tc) < C ? (t1 - tc) : C);

        // ---- (a) this chunk's rows arrived: convert q / k; gates; prefetch the next chunk ----
        cp_async_wait_all();
        __syncthreads();
        convert_qk(sm, tid);
        float lg = 0.f, beta = 0.f;
        if (tid < len) {
            lg = log_gate(A_log, bf16_to_f32(ga), dt_bias);
            beta = sigmoidf_(bf16_to_f32(gb));
        }
        {
            const long long tn = tc + C;
            if (tn < t1) {
                const int ln = (int)((t1 - tn) < C ? (t1 - tn) : C);
                prefetch_chunk(p, rawK, rawQ, rawV + (uint32_t)(buf ^ 1) * (C * VT * 2), tn, ln, hq, hv, v0, tid);
                if (tid < ln) {
                    ga = p.a[(size_t)(tn + tid) * p.HV + hv];
                    gb = p.b[(size_t)(tn + tid) * p.HV + hv];
                }
            }
        }
        // inclusive scan of log g over the 64 tokens (warps 0 and 1)
        if (warp < 2) {
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                float y = __shfl_up_sync(0xffffffffu, lg, o);
                if ((tid & 31) >= o) lg += y;
            }
            if (warp == 0) sG[tid] = lg;
            sBeta[tid] = beta;
        }
        __syncthreads();
        if (warp == 1) sG[tid] = lg + sG[31];
        umma::fence_proxy_async_smem();
        umma::fence_before_sync();
        __syncthreads();
        umma::fence_after_sync();

        // ---- (b) MMA_A: [K;Q] K^T ----
        if (tid == 0) {
#pragma unroll
            for (int k0 = 0; k0 < kDim; k0 += 16)
                umma::mma_f16(tmem + TM_A, umma::desc_kmaj(sKQ, 128, k0), umma::desc_kmaj(sKQ, 128, k0), ID_KK,
                              k0 > 0);
            umma::mma_commit(&mbar[0]);
        }
        if (__syncthreads_or(!umma::mbar_wait(&mbar[0], parity, kWaitBudget))) goto done;
        umma::fence_after_sync();

        const float gC = sG[C - 1];
        // ---- (c) masks -> A (fp32) and P (f16 operand); Q~ and K~ operands ----
        {
            const int i = tid & 63;
            const float gi = sG[i];
#pragma unroll
            for (int c16 = 0; c16 < C; c16 += 16) {
                float d[16];
                umma::tmem_ld16(tmem + lane_base + TM_A + c16, d);
                float r[16];
                if (tid < 64) {
                    const float bi = sBeta[i];
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const int j = c16 + e;
                        r[e] = (j < i) ? bi * __expf(fminf(gi - sG[j], 0.f)) * d[e] : 0.f;
                    }
#pragma unroll
                    for (int e = 0; e < 16; e += 4)
                        *reinterpret_cast<float4*>(sA + i * LDA + c16 + e) = make_float4(r[e], r[e + 1], r[e + 2], r[e + 3]);
                } else {
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const int j = c16 + e;
                        r[e] = (j <= i) ? scale * __expf(fminf(gi - sG[j], 0.f)) * d[e] : 0.f;
                    }
                    st_f16x8(sm + OFF_TP, umma::kmaj_off(64 + i, c16, 128), r);
                    st_f16x8(sm + OFF_TP, umma::kmaj_off(64 + i, c16 + 8, 128), r + 8);
                }
            }
            if (tid >= 64) {
                // Q~ row i = scale e^{gamma_i} q_i, in place over Q (rows 64-127)
                const float f = scale * expf(gi);
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    const uint32_t off = umma::kmaj_off(64 + i, c * 8, 128);
                    uint4 raw = *reinterpret_cast<uint4*>(sm + OFF_KQ + off);
                    __half2* h = reinterpret_cast<__half2*>(&raw);
                    float x[8];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        float2 f2 = __half22float2(h[e]);
                        x[2 * e] = f2.x * f;
                        x[2 * e + 1] = f2.y * f;
                    }
                    st_f16x8(sm + OFF_KQ, off, x);
                }
            } else {
                // K~ row i = e^{gamma_C - gamma_i} k_i, MN-major (m = k index, K-dim = token)
                const float f = expf(fminf(gC - gi, 0.f));
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    uint4 raw = *reinterpret_cast<uint4*>(sm + OFF_KQ + umma::kmaj_off(i, c * 8, 128));
                    __half2* h = reinterpret_cast<__half2*>(&raw);
                    float x[8];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        float2 f2 = __half22float2(h[e]);
                        x[2 * e] = f2.x * f;
                        x[2 * e + 1] = f2.y * f;
                    }
                    st_f16x8(sm + OFF_KT, umma::mnmaj_off(c * 8, i, C), x);
                }
            }
        }
        umma::fence_proxy_async_smem();
        umma::fence_before_sync();
        __syncthreads();
        umma::fence_after_sync();

        // ---- (d) MMA_1: [K ; Q~] S (runs during the solve) ----
        if (tid == 0) {
#pragma unroll
            for (int k0 = 0; k0 < kDim; k0 += 16)
                umma::mma_f16(tmem + TM_1, umma::desc_kmaj(sKQ, 128, k0), umma::desc_kmaj(sSH, VT, k0), ID_S,
                              k0 > 0);
            umma::mma_commit(&mbar[1]);
        }

        // ---- (e) T = (I + A)^-1; f16 copies: rows 0-63 of [T;P] and T as MN-major B ----
        solve_T(sA, sT, sX, tid);
        {
            const int i = tid >> 1, h = (tid & 1) * 32;  // row i, columns h..h+31
            const float* tr = sT + i * LDA + h;
#pragma unroll
            for (int c = 0; c < 32; c += 8) {
                float x[8];
                const float4 a = *reinterpret_cast<const float4*>(tr + c);
                const float4 b = *reinterpret_cast<const float4*>(tr + c + 4);
                x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
                x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
                st_f16x8(sm + OFF_TP, umma::kmaj_off(i, h + c, 128), x);  // A rows: T[i][j]
                st_f16x8(sm + OFF_TB, umma::mnmaj_off(h + c, i, C), x);   // B: (n = m, k = j) = T[j][m]
            }
        }
        umma::fence_proxy_async_smem();
        umma::fence_before_sync();
        __syncthreads();
        umma::fence_after_sync();

        // ---- (f) MMA_P: [T ; P] T -> rows 64-127 = P' ----
        if (tid == 0) {
#pragma unroll
            for (int k0 = 0; k0 < C; k0 += 16)
                umma::mma_f16(tmem + TM_A, umma::desc_kmaj(sTP, 128, k0), umma::desc_mnmaj(sTB, C, k0), ID_P,
                              k0 > 0);
            umma::mma_commit(&mbar[2]);
        }

        // ---- (g) Y rows (0-63) from MMA_1; keep Q~S rows (64-127) ----
        if (__syncthreads_or(!umma::mbar_wait(&mbar[1], parity, kWaitBudget))) goto done;
        umma::fence_after_sync();
        float qs[VT];
        if (tid < 64) {
            const int i = tid;
            const float eg = expf(sG[i]), b_i = sBeta[i];
#pragma unroll
            for (int c16 = 0; c16 < VT; c16 += 16) {
                float d[16];
                umma::tmem_ld16(tmem + lane_base + TM_1 + c16, d);
                float y[16];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint4 raw = *reinterpret_cast<const uint4*>(
                        sm + OFF_RV + buf * (C * VT * 2) + rawv_off(i, c16 / 8 + h));
                    const __nv_bfloat162* vb = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 vv = __bfloat1622float2(vb[e]);
                        y[8 * h + 2 * e] = b_i * (vv.x - eg * d[8 * h + 2 * e]);
                        y[8 * h + 2 * e + 1] = b_i * (vv.y - eg * d[8 * h + 2 * e + 1]);
                    }
                }
                st_f16x8(sm + OFF_Y, umma::mnmaj_off(c16, i, C), y);
                st_f16x8(sm + OFF_Y, umma::mnmaj_off(c16 + 8, i, C), y + 8);
            }
        } else {
#pragma unroll
            for (int c16 = 0; c16 < VT; c16 += 16) {
                float d[16];
                umma::tmem_ld16(tmem + lane_base + TM_1 + c16, d);
#pragma unroll
                for (int e = 0; e < 16; ++e) qs[c16 + e] = d[e];
            }
        }
        // P' rows (64-127) over P in [T ; P]
        if (__syncthreads_or(!umma::mbar_wait(&mbar[2], parity, kWaitBudget))) goto done;
        umma::fence_after_sync();
        if (tid >= 64) {
            const int i = tid - 64;
#pragma unroll
            for (int c16 = 0; c16 < C; c16 += 16) {
                float d[16];
                umma::tmem_ld16(tmem + lane_base + TM_A + c16, d);
                st_f16x8(sm + OFF_TP, umma::kmaj_off(64 + i, c16, 128), d);
                st_f16x8(sm + OFF_TP, umma::kmaj_off(64 + i, c16 + 8, 128), d + 8);
            }
        }
        umma::fence_proxy_async_smem();
        umma::fence_before_sync();
        __syncthreads();
        umma::fence_after_sync();

        // ---- (h) MMA_2: [T ; P'] Y ----
        if (tid == 0) {
#pragma unroll
            for (int k0 = 0; k0 < C; k0 += 16)
                umma::mma_f16(tmem + TM_2, umma::desc_kmaj(sTP, 128, k0), umma::desc_mnmaj(sY, C, k0), ID_Y,
                              k0 > 0);
            umma::mma_commit(&mbar[3]);
        }
        if (__syncthreads_or(!umma::mbar_wait(&mbar[3], parity, kWaitBudget))) goto done;
        umma::fence_after_sync();

        // ---- (i) Delta rows (0-63) -> smem; output rows (64-127) -> HBM ----
        if (tid < 64) {
            const int i = tid;
#pragma unroll
            for (int c16 = 0; c16 < VT; c16 += 16) {
                float d[16];
                umma::tmem_ld16(tmem + lane_base + TM_2 + c16, d);
                st_f16x8(sm + OFF_DL, umma::mnmaj_off(c16, i, C), d);
                st_f16x8(sm + OFF_DL, umma::mnmaj_off(c16 + 8, i, C), d + 8);
            }
        } else {
            const int i = tid - 64;
            __nv_bfloat16* op = p.out + ((size_t)(tc + i) * p.HV + hv) * kDim + v0;
#pragma unroll
            for (int c16 = 0; c16 < VT; c16 += 16) {
                float d[16];
                umma::tmem_ld16(tmem + lane_base + TM_2 + c16, d);
                if (i < len) {
                    __nv_bfloat162 o[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        o[e] = __floats2bfloat162_rn(qs[c16 + 2 * e] + d[2 * e], qs[c16 + 2 * e + 1] + d[2 * e + 1]);
                    reinterpret_cast<uint4*>(op + c16)[0] = reinterpret_cast<uint4*>(o)[0];
                    reinterpret_cast<uint4*>(op + c16)[1] = reinterpret_cast<uint4*>(o)[1];
                }
            }
        }
        umma::fence_proxy_async_smem();
        umma::fence_before_sync();
        __syncthreads();
        umma::fence_after_sync();

        // ---- (j) MMA_3: K~^T Delta ----
        if (tid == 0) {
#pragma unroll
            for (int k0 = 0; k0 < C; k0 += 16)
                umma::mma_f16(tmem + TM_3, umma::desc_mnmaj(sKT, C, k0), umma::desc_mnmaj(sDL, C, k0), ID_D,
                              k0 > 0);
            umma::mma_commit(&mbar[4]);
        }
        if (__syncthreads_or(!umma::mbar_wait(&mbar[4], parity, kWaitBudget))) goto done;
        umma::fence_after_sync();

        // ---- (k) state update: thread k owns row k of S (all VT columns) ----
        {
            const int k = tid;
            const float decay = expf(gC);
#pragma unroll
            for (int c16 = 0; c16 < VT; c16 += 16) {
                float d[16];
                umma::tmem_ld16(tmem + lane_base + TM_3 + c16, d);
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const int v = c16 + e;
                    const float s = fmaf(decay, sSf[v * kDim + k], d[e]);
                    sSf[v * kDim + k] = s;
                    *reinterpret_cast<__half*>(sm + OFF_SH + umma::kmaj_off(v, k, VT)) = __float2half_rn(s);
                }
            }
        }
        umma::fence_proxy_async_smem();
        umma::fence_before_sync();
        __syncthreads();
        umma::fence_after_sync();
    }

    // final state (fp32, k-last): consecutive threads write consecutive k
    for (int idx = tid; idx < VT * kDim; idx += NT) __stcs(p.new_state + state_off + idx, sSf[idx]);

done:
    cp_async_wait_all();  // no copy may still target shared memory when the CTA exits
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 0) umma::tmem_dealloc(tmem, TM_COLS);
}

}  // namespace chunk

void launch_prefill_chunk(const PrefillParams& p, cudaStream_t st) {
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(chunk::gdn_prefill_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)chunk::SMEM_BYTES);
        attr_set = true;
    }
    const long long blocks = (long long)p.N * p.HV * (kDim / chunk::VT);
    chunk::gdn_prefill_chunk_kernel<<<(unsigned)blocks, chunk::NT, chunk::SMEM_BYTES, st>>>(p);
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
