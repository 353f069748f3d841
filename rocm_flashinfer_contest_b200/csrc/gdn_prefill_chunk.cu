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
//   masks : rows 0-63 -> A (fp32, smem), rows 64-127 -> P (fp32, registers)
//   solve : threads 0-63 forward-substitute the columns of T, threads 64-127
//           back-substitute the rows of P' (fp32, CUDA cores, in parallel)
//   MMA_1 : [K ; diag(scale e^gamma) Q] x S      -> TMEM cols [64, 128)
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
constexpr uint32_t OFF_KQ = 0;                  // [K ; Q] K-major 128 x 128 f16      32 KiB
constexpr uint32_t OFF_TP = OFF_KQ + 32768;     // [T ; P'] K-major 128 x 64 f16      16 KiB
constexpr uint32_t OFF_SH = OFF_TP + 16384;     // S^T K-major VT x 128 f16 (B op)    16 KiB
constexpr uint32_t OFF_Y = OFF_SH + 16384;      // Y MN-major (v x 64 tokens) f16      8 KiB
constexpr uint32_t OFF_DL = OFF_Y + 8192;       // Delta MN-major (v x 64 tokens) f16  8 KiB
constexpr uint32_t OFF_KT = OFF_DL + 8192;      // K~ MN-major (k x 64 tokens) f16    16 KiB
constexpr uint32_t OFF_SF = OFF_KT + 16384;     // S fp32 [v][k] (VT x 128)           32 KiB
constexpr uint32_t OFF_A = OFF_SF + 32768;      // A fp32 [i][j] 64 x 64              16 KiB
constexpr uint32_t OFF_AT = OFF_A + 16384;      // A^T fp32 [j][i] 64 x 64            16 KiB
constexpr uint32_t OFF_G = OFF_AT + 16384;      // gamma[64] fp32
constexpr uint32_t OFF_BETA = OFF_G + 256;      // beta[64] fp32
constexpr uint32_t SMEM_USED = OFF_BETA + 256;
constexpr uint32_t SMEM_BYTES = SMEM_USED + 1024;  // + alignment slack

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

// Load the 64 x 128 bf16 rows of q or k for the chunk's tokens into a
// K-major f16 tile (row r <- token t0 + r; rows past `len` are zero).
__device__ __forceinline__ void stage_qk_rows(unsigned char* tile, uint32_t row0, const __nv_bfloat16* src,
                                              long long t0, int len, int H, int hq, int tid) {
    for (int idx = tid; idx < C * 16; idx += NT) {
        const int r = idx >> 4, c = idx & 15;  // row, 8-element chunk
        float x[8];
        if (r < len) {
            ld_bf16x8(src + ((size_t)(t0 + r) * H + hq) * kDim + c * 8, x);
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) x[e] = 0.f;
        }
        st_f16x8(tile, umma::kmaj_off(row0 + r, c * 8, 128), x);
    }
}

__global__ void __launch_bounds__(NT, 1) gdn_prefill_chunk_kernel(const PrefillParams p) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t mbar;
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

    float* sSf = reinterpret_cast<float*>(sm + OFF_SF);   // [v][k]
    float* sA = reinterpret_cast<float*>(sm + OFF_A);     // [i][j]
    float* sAT = reinterpret_cast<float*>(sm + OFF_AT);   // [j][i]
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

    if (warp == 0) {
        umma::tmem_alloc(&tmem_base_sh, TM_COLS);
        umma::tmem_relinquish();
    }
    if (tid == 0) {
        umma::mbar_init(&mbar, 1);
        umma::fence_mbar_init();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = tmem_base_sh;
    const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
    uint32_t phase = 0;

    const uint32_t sKQ = umma::smem_u32(sm + OFF_KQ), sTP = umma::smem_u32(sm + OFF_TP);
    const uint32_t sSH = umma::smem_u32(sm + OFF_SH), sY = umma::smem_u32(sm + OFF_Y);
    const uint32_t sDL = umma::smem_u32(sm + OFF_DL), sKT = umma::smem_u32(sm + OFF_KT);
    constexpr uint32_t ID_KK = umma::idesc_f16(128, 64, 0, 0, 0, 0);   // K-major x K-major
    constexpr uint32_t ID_S = umma::idesc_f16(128, VT, 0, 0, 0, 0);    // [K;Q~] x S
    constexpr uint32_t ID_Y = umma::idesc_f16(128, VT, 0, 0, 0, 1);    // [T;P'] x Y (MN-major B)
    constexpr uint32_t ID_D = umma::idesc_f16(128, VT, 0, 0, 1, 1);    // K~^T x Delta

    const float A_log = p.A_log[hv], dt_bias = p.dt_bias[hv];
    const float scale = p.scale;

    for (long long tc = t0; tc < t1; tc += C) {
        const int len = (int)((t1 - tc) < C ? (t1 - tc) : C);

        // ---- (a) stage K and Q rows, gates ----
        stage_qk_rows(sm + OFF_KQ, 0, p.k, tc, len, p.H, hq, tid);
        stage_qk_rows(sm + OFF_KQ, 64, p.q, tc, len, p.H, hq, tid);
        float lg = 0.f, beta = 0.f;
        if (tid < C && tid < len) {
            const size_t gi = (size_t)(tc + tid) * p.HV + hv;
            lg = log_gate(A_log, bf16_to_f32(p.a[gi]), dt_bias);
            beta = sigmoidf_(bf16_to_f32(p.b[gi]));
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
            umma::mma_commit(&mbar);
        }
        if (__syncthreads_or(!umma::mbar_wait(&mbar, phase, kWaitBudget))) goto done;
        phase ^= 1;
        umma::fence_after_sync();

        const float gC = sG[C - 1];
        // ---- (c) masks; Q~ and K~ operands ----
        float prow[C];  // threads 64-127: row of P (fp32)
        {
            const int i = tid & 63;
            const float gi = sG[i];
#pragma unroll
            for (int c16 = 0; c16 < C; c16 += 16) {
                float d[16];
                umma::tmem_ld16(tmem + lane_base + TM_A + c16, d);
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const int j = c16 + e;
                    const float dec = expf(fminf(gi - sG[j], 0.f));
                    if (tid < 64) {
                        const float a = (j < i) ? sBeta[i] * dec * d[e] : 0.f;
                        sA[i * C + j] = a;
                        sAT[j * C + i] = a;
                    } else {
                        prow[j] = (j <= i) ? scale * dec * d[e] : 0.f;
                    }
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
        __syncthreads();

        // ---- (d) solves: T = (I + A)^-1 by columns; P' = P T by rows ----
        if (tid < 64) {
            const int m = tid;
            float x[C];
#pragma unroll
            for (int i = 0; i < C; ++i) {
                float acc = (i == m) ? 1.f : 0.f;
                const float4* arow = reinterpret_cast<const float4*>(sA + i * C);
#pragma unroll
                for (int j4 = 0; j4 < i / 4; ++j4) {
                    const float4 a4 = arow[j4];
                    acc -= a4.x * x[4 * j4] + a4.y * x[4 * j4 + 1] + a4.z * x[4 * j4 + 2] + a4.w * x[4 * j4 + 3];
                }
#pragma unroll
                for (int j = (i / 4) * 4; j < i; ++j) acc -= sA[i * C + j] * x[j];
                x[i] = acc;
            }
            // column m of T into rows 0-63 of [T ; P'] (K-major: element (i, m))
#pragma unroll
            for (int i = 0; i < C; ++i)
                *reinterpret_cast<__half*>(sm + OFF_TP + umma::kmaj_off(i, m, 128)) = __float2half_rn(x[i]);
        } else {
            // P'[r][m] = P[r][m] - sum_{j>m} P'[r][j] A[j][m]   (m descending)
            float y[C];
#pragma unroll
            for (int m = C - 1; m >= 0; --m) {
                float acc = prow[m];
                const float* acol = sAT + m * C;  // A[j][m] for j = 0..63
#pragma unroll
                for (int j = m + 1; j < C; ++j) acc -= y[j] * acol[j];
                y[m] = acc;
            }
            const int r = tid - 64;
#pragma unroll
            for (int c = 0; c < C / 8; ++c) st_f16x8(sm + OFF_TP, umma::kmaj_off(64 + r, c * 8, 128), y + 8 * c);
        }
        umma::fence_proxy_async_smem();
        umma::fence_before_sync();
        __syncthreads();
        umma::fence_after_sync();

        // ---- (e) MMA_1: [K ; Q~] S ----
        if (tid == 0) {
#pragma unroll
            for (int k0 = 0; k0 < kDim; k0 += 16)
                umma::mma_f16(tmem + TM_1, umma::desc_kmaj(sKQ, 128, k0), umma::desc_kmaj(sSH, VT, k0), ID_S,
                              k0 > 0);
            umma::mma_commit(&mbar);
        }
        if (__syncthreads_or(!umma::mbar_wait(&mbar, phase, kWaitBudget))) goto done;
        phase ^= 1;
        umma::fence_after_sync();

        // ---- (f) Y rows (0-63); keep Q~S rows (64-127) ----
        float qs[VT];
        if (tid < 64) {
            const int i = tid;
            const float eg = expf(sG[i]), b_i = sBeta[i];
            float vrow[VT];
            if (i < len) {
                const __nv_bfloat16* vp = p.v + ((size_t)(tc + i) * p.HV + hv) * kDim + v0;
#pragma unroll
                for (int c = 0; c < VT / 8; ++c) ld_bf16x8(vp + 8 * c, vrow + 8 * c);
            } else {
#pragma unroll
                for (int e = 0; e < VT; ++e) vrow[e] = 0.f;
            }
#pragma unroll
            for (int c16 = 0; c16 < VT; c16 += 16) {
                float d[16];
                umma::tmem_ld16(tmem + lane_base + TM_1 + c16, d);
                float y[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) y[e] = b_i * (vrow[c16 + e] - eg * d[e]);
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
        umma::fence_proxy_async_smem();
        umma::fence_before_sync();
        __syncthreads();
        umma::fence_after_sync();

        // ---- (g) MMA_2: [T ; P'] Y ----
        if (tid == 0) {
#pragma unroll
            for (int k0 = 0; k0 < C; k0 += 16)
                umma::mma_f16(tmem + TM_2, umma::desc_kmaj(sTP, 128, k0), umma::desc_mnmaj(sY, C, k0), ID_Y,
                              k0 > 0);
            umma::mma_commit(&mbar);
        }
        if (__syncthreads_or(!umma::mbar_wait(&mbar, phase, kWaitBudget))) goto done;
        phase ^= 1;
        umma::fence_after_sync();

        // ---- (h) Delta rows (0-63) -> smem; output rows (64-127) -> HBM ----
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

        // ---- (i) MMA_3: K~^T Delta ----
        if (tid == 0) {
#pragma unroll
            for (int k0 = 0; k0 < C; k0 += 16)
                umma::mma_f16(tmem + TM_3, umma::desc_mnmaj(sKT, C, k0), umma::desc_mnmaj(sDL, C, k0), ID_D,
                              k0 > 0);
            umma::mma_commit(&mbar);
        }
        if (__syncthreads_or(!umma::mbar_wait(&mbar, phase, kWaitBudget))) goto done;
        phase ^= 1;
        umma::fence_after_sync();

        // ---- (j) state update: thread k owns row k of S (all VT columns) ----
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

    // final state (fp32, k-last): thread k writes column k of rows v0..v0+VT
    for (int idx = tid; idx < VT * kDim; idx += NT) __stcs(p.new_state + state_off + idx, sSf[idx]);

done:
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
