// gdn_prefill_scan.cuh — the chunked prefill as a scan over per-chunk state
// transitions (included by gdn_prefill_chunk.cu: its kernels share that
// translation unit's device status word and helpers).
//
// Same chunk maths as the chain kernels of gdn_prefill_chunk.cu (C = 64,
// gamma, A, P, T = (I + A)^-1, P' = P T, K~ = diag(e^{gamma_C - gamma}) K),
// regrouped so that the state enters each chunk through ONE product:
//   S_{j+1} = e^{gamma_C} S_j - Abar S_j + Et V        (state [K] x [V])
//   O_j     = Qt S_j + Pt V
// with, per (chunk, v-head),
//   Et   = K~^T T diag(beta)                       [K x C]
//   Abar = Et diag(e^gamma) K                      [K x K]
//   Pt   = P' diag(beta)                           [C x C]
//   Qt   = diag(scale e^gamma) Q - Pt diag(e^gamma) K   [C x K]
// (expanding Delta = T beta (V - e^gamma K S) in S' = e^{gamma_C} S + K~^T Delta
// and O = scale e^gamma Q S + P' Y).  The state-independent operators are
// built by a prep kernel for all chunks at once; the chain then walks the
// chunks of a (sequence, v-head) with one tensor-core round trip per chunk on
// its critical path: S_j (f16, tensor memory) x Abar_j^T -> the state
// threads add e^{gamma_C} S_j in fp32 -> S_{j+1}.  Et V and the outputs hang
// off that path.  The e^{gamma_C} S_j term stays in fp32 registers, so the
// state loses precision only through f16 operands, as in the other chains.
#pragma once

namespace scan {

// Record of one (chunk, v-head) in the workspace, written by the prep and
// read by the chain with one bulk copy; every tile is in the 128-byte-swizzled
// K-major layout the chain's MMAs read (B operands):
//   -Abar  rows k', columns k       128 x 128  32 KiB
//   Et     rows k, columns token    128 x 64   16 KiB
//   Qt     rows token, columns k     64 x 128  16 KiB
//   Pt     rows token i, columns j   64 x 64    8 KiB
//   e^{gamma_C} (fp32), padding                 16 B
constexpr uint32_t REC_ABAR = 0, REC_E = 32768, REC_QT = 49152, REC_P = 65536, REC_DECAY = 73728;
constexpr uint32_t kRecBytes = 73744;

__host__ __device__ inline size_t workspace_bytes(int N, int T, int HV) {
    return (size_t)ws_slots(N, T) * HV * kRecBytes;
}

// ============================================================================
// prep: one CTA per (chunk, v-head), 128 threads, three CTAs per SM
// ============================================================================
namespace prep {

using ::gdn::chunk::prep::ix;
constexpr int NT = 128;
constexpr uint32_t OFF_KQ = 0;                      // [K ; Q] f16 K-major 128 x 128, whole kernel
constexpr uint32_t OFF_A = kTileKQ;                 // A fp32 [64][LDA] during the solve
constexpr uint32_t OFF_T = OFF_A + 64 * LDA * 4;    // T fp32 [64][LDA] during the solve
// after the solve the two fp32 matrices' 34 KiB hold the f16 operand tiles
constexpr uint32_t OFF_TP = OFF_A;                  // [T diag(beta) ; P] K-major 128 x 64       16 KiB
constexpr uint32_t OFF_T1 = 51200;                  // diag(f_K) T diag(beta), 64 x 64 (MN-major B) 8 KiB
constexpr uint32_t OFF_EP = OFF_A;                  // [Et diag(e^g) ; Pt diag(e^g)] K-major 192 x 64, 24 KiB
constexpr uint32_t OFF_GM = OFF_T + 64 * LDA * 4;   // gamma[64], beta[64]
constexpr uint32_t SMEM_BYTES = OFF_GM + 512 + 1024;  // + alignment slack
static_assert(OFF_A % 1024 == 0 && OFF_T1 % 1024 == 0, "tile alignment");
static_assert(OFF_T1 >= OFF_TP + kTileTP && OFF_T1 + 8192 <= OFF_GM, "T1 after [T ; P], before the gates");
static_assert(OFF_EP + 24576 <= OFF_GM, "[E2 ; P2] inside the solve matrices' space");
static_assert(3 * (SMEM_BYTES + 1024) <= 233472, "three CTAs per SM");
constexpr uint32_t TM_COLS = 128;  // 3 CTAs x 128 columns fit the SM's 512

// MMA_E reads T1 = diag(f_K) T diag(beta) MN-major (k = token i, n = token j):
// a row-major 64 x 64 tile in the K-major layout of 64 rows is that operand.
constexpr bool rows64_are_mn_major() {
    for (uint32_t i = 0; i < 64; ++i)
        for (uint32_t j = 0; j < 64; ++j)
            if (umma::kmaj_off(i, j, 64) != umma::mnmaj_off(j, i, 64)) return false;
    return true;
}
static_assert(rows64_are_mn_major(), "a K-major 64-row tile doubles as the MN-major B operand");

__global__ void __launch_bounds__(NT, 3) gdn_prefill_scan_prep_kernel(const PrefillParams p, unsigned char* ws) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t mbar[4];
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
    float* sG = reinterpret_cast<float*>(sm + OFF_GM);
    float* sBeta = sG + 64;
    unsigned char* rec = ws + ((size_t)s * p.HV + hv) * kRecBytes;

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
        for (int i = 0; i < 4; ++i) umma::mbar_init(&mbar[i], 1);
        umma::fence_mbar_init();
    }
    __syncthreads();
    if (warp == 1) sG[tid] = lg + sG[31];
    cp_async_wait_all();
    __syncthreads();
    // every product here takes [K ; Q] as f16: normalised rows are written as
    // f16, raw bf16 rows are converted (exact for |x| in f16's normal range)
    if (p.qk_l2norm) {
        l2norm_row_to_f16(sm + OFF_KQ, tid, 128);
    } else {
#pragma unroll 4
        for (int idx = tid; idx < (int)(kTileKQ / 16); idx += NT) {
            uint4* cell = reinterpret_cast<uint4*>(sm + OFF_KQ) + idx;
            float x[8];
            unpack_bf16x8(*cell, x);
            st_f16x8(reinterpret_cast<unsigned char*>(cell), 0, x);
        }
    }
    sync_for_mma();
    const uint32_t tmem = tmem_base_sh;
    const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
    const uint64_t dKQ = umma::desc_kmaj(sKQ, 128, 0);
    const uint64_t dKmn = umma::desc_sw128(sKQ, 16384u, 1024u);  // K rows read MN-major (K^T as A, K as B)
    const uint64_t dEP = umma::desc_kmaj(umma::smem_u32(sm + OFF_EP), 192, 0);

    // MMA_G: [K ; Q] K^T -> columns 0-63
    if (tid == 0) {
        constexpr uint32_t ID = umma::idesc_f16(128, 64, 0, 0, 0, 0);
#pragma unroll
        for (int k0 = 0; k0 < kDim; k0 += 16) {
            const uint64_t a = umma::desc_add(dKQ, umma::koff_kmaj(128, k0));
            umma::mma_f16(tmem, a, a, ID, k0 > 0);
        }
        umma::mma_commit(&mbar[0]);
    }
    if (!wait_mma(&mbar[0], 0)) goto done;
    umma::fence_after_sync();

    // A = beta_i e^{gamma_i - gamma_j} k_i.k_j (j < i), rows 0-63 (warps 0, 1)
    if (tid < 64) {
        const int i = tid;
        const float gi = sG[i], bi = sBeta[i];
#pragma unroll 1
        for (int c16 = 0; c16 < C; c16 += 16) {
            float d[16], r[16];
            umma::tmem_ld16(tmem + lane_base + c16, d);
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const int jj = c16 + e;
                r[e] = (jj < i) ? bi * __expf(fminf(gi - sG[jj], 0.f)) * d[e] : 0.f;
            }
#pragma unroll
            for (int e = 0; e < 16; e += 4)
                *reinterpret_cast<float4*>(sA + ix(i, c16 + e)) = make_float4(r[e], r[e + 1], r[e + 2], r[e + 3]);
        }
    }
    __syncthreads();
    ::gdn::chunk::prep::solve_T(sA, sT, tid);

    // f16 copies of T: T diag(beta) -> rows 0-63 of [T ; P] (the B operand of
    // MMA_P, read MN-major from those rows) and diag(f_K) T diag(beta) -> T1
    {
        const int i = tid >> 1, h = (tid & 1) * 32;  // row i, columns h..h+31
        float t[32];
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
            // blocks above the diagonal are zero and are never stored in sT
            if (((h + c) >> 4) <= (i >> 4)) {
                const float4 a = *reinterpret_cast<const float4*>(sT + ix(i, h + c));
                const float4 b = *reinterpret_cast<const float4*>(sT + ix(i, h + c + 4));
                t[c] = a.x; t[c + 1] = a.y; t[c + 2] = a.z; t[c + 3] = a.w;
                t[c + 4] = b.x; t[c + 5] = b.y; t[c + 6] = b.z; t[c + 7] = b.w;
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) t[c + e] = 0.f;
            }
        }
        const float fk = __expf(fminf(sG[C - 1] - sG[i], 0.f));
        __syncthreads();  // T1 overwrites part of sT
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
            float x[8], y[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                x[e] = t[c + e] * sBeta[h + c + e];
                y[e] = fk * x[e];
            }
            st_f16x8(sm + OFF_TP, umma::kmaj_off(i, h + c, 128), x);
            st_f16x8(sm + OFF_T1, umma::kmaj_off(i, h + c, 64), y);
        }
    }
    // P = scale e^{gamma_i - gamma_j} q_i.k_j (j <= i) -> rows 64-127 of [T ; P]
    // (warps 2, 3 read TMEM lanes 64-127 of MMA_G)
    if (tid >= 64) {
        const int i = tid - 64;
        const float gi = sG[i];
#pragma unroll 1
        for (int c16 = 0; c16 < C; c16 += 16) {
            float d[16], r[16];
            umma::tmem_ld16(tmem + lane_base + c16, d);
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const int jj = c16 + e;
                r[e] = (jj <= i) ? p.scale * __expf(fminf(gi - sG[jj], 0.f)) * d[e] : 0.f;
            }
            st_f16x8(sm + OFF_TP, umma::kmaj_off(64 + i, c16, 128), r);
            st_f16x8(sm + OFF_TP, umma::kmaj_off(64 + i, c16 + 8, 128), r + 8);
        }
    }
    sync_for_mma();

    // MMA_P: [T diag(beta) ; P] x T diag(beta) -> columns 0-63, rows 64-127 = Pt
    // MMA_E: K^T x T1 -> columns 64-127 = Et
    if (tid == 0) {
        constexpr uint32_t IDP = umma::idesc_f16(128, 64, 0, 0, 0, 1);
        constexpr uint32_t IDE = umma::idesc_f16(128, 64, 0, 0, 1, 1);
        const uint64_t dTP = umma::desc_kmaj(umma::smem_u32(sm + OFF_TP), 128, 0);
        const uint64_t dTB = umma::desc_mnmaj(umma::smem_u32(sm + OFF_TP), C, 0);
        const uint64_t dT1 = umma::desc_mnmaj(umma::smem_u32(sm + OFF_T1), C, 0);
#pragma unroll
        for (int k0 = 0; k0 < C; k0 += 16)
            umma::mma_f16(tmem, umma::desc_add(dTP, umma::koff_kmaj(128, k0)),
                          umma::desc_add(dTB, umma::koff_mnmaj(k0)), IDP, k0 > 0);
#pragma unroll
        for (int k0 = 0; k0 < C; k0 += 16)
            umma::mma_f16(tmem + 64, umma::desc_add(dKmn, umma::koff_mnmaj(k0)),
                          umma::desc_add(dT1, umma::koff_mnmaj(k0)), IDE, k0 > 0);
        umma::mma_commit(&mbar[1]);
    }
    if (!wait_mma(&mbar[1], 0)) goto done;
    umma::fence_after_sync();

    // Pt (record) and Pt diag(e^gamma) (rows 128-191 of [E2 ; P2]); Et
    // (record) and Et diag(e^gamma) (rows 0-127).  Thread = TMEM lane.
    {
        float eg[16];
        if (tid >= 64) {
            const int i = tid - 64;
#pragma unroll 1
            for (int c16 = 0; c16 < C; c16 += 16) {
                float d[16];
                umma::tmem_ld16(tmem + lane_base + c16, d);
#pragma unroll
                for (int e = 0; e < 16; ++e) eg[e] = __expf(sG[c16 + e]);
                st_f16x8(rec + REC_P, umma::kmaj_off(i, c16, 64), d);
                st_f16x8(rec + REC_P, umma::kmaj_off(i, c16 + 8, 64), d + 8);
#pragma unroll
                for (int e = 0; e < 16; ++e) d[e] *= eg[e];
                st_f16x8(sm + OFF_EP, umma::kmaj_off(128 + i, c16, 192), d);
                st_f16x8(sm + OFF_EP, umma::kmaj_off(128 + i, c16 + 8, 192), d + 8);
            }
        }
#pragma unroll 1
        for (int c16 = 0; c16 < C; c16 += 16) {
            float d[16];
            umma::tmem_ld16(tmem + lane_base + 64 + c16, d);
#pragma unroll
            for (int e = 0; e < 16; ++e) eg[e] = __expf(sG[c16 + e]);
            st_f16x8(rec + REC_E, umma::kmaj_off(tid, c16, 128), d);
            st_f16x8(rec + REC_E, umma::kmaj_off(tid, c16 + 8, 128), d + 8);
#pragma unroll
            for (int e = 0; e < 16; ++e) d[e] *= eg[e];
            st_f16x8(sm + OFF_EP, umma::kmaj_off(tid, c16, 192), d);
            st_f16x8(sm + OFF_EP, umma::kmaj_off(tid, c16 + 8, 192), d + 8);
        }
        if (tid == 0)
            *reinterpret_cast<float4*>(rec + REC_DECAY) = make_float4(__expf(sG[C - 1]), 0.f, 0.f, 0.f);
    }
    sync_for_mma();

    // MMA_A: [E2 ; P2] rows 0-127 x K -> columns 0-127 = Abar
    if (tid == 0) {
        constexpr uint32_t ID = umma::idesc_f16(128, 128, 0, 0, 0, 1);
#pragma unroll
        for (int k0 = 0; k0 < C; k0 += 16)
            umma::mma_f16(tmem, umma::desc_add(dEP, umma::koff_kmaj(192, k0)),
                          umma::desc_add(dKmn, umma::koff_mnmaj(k0)), ID, k0 > 0);
        umma::mma_commit(&mbar[2]);
    }
    if (!wait_mma(&mbar[2], 0)) goto done;
    umma::fence_after_sync();
    // -Abar row k' = tid -> record (two 64-column slabs)
#pragma unroll 1
    for (int c32 = 0; c32 < kDim; c32 += 32) {
        float d[32];
        umma::tmem_ld32(tmem + lane_base + c32, d);
#pragma unroll
        for (int e = 0; e < 32; ++e) d[e] = -d[e];
#pragma unroll
        for (int e = 0; e < 32; e += 8) st_f16x8(rec + REC_ABAR, umma::kmaj_off(tid, c32 + e, 128), d + e);
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();

    // MMA_Q: [E2 ; P2] rows 64-191 x K -> columns 0-127; rows 64-127 = Pt diag(e^gamma) K
    if (tid == 0) {
        constexpr uint32_t ID = umma::idesc_f16(128, 128, 0, 0, 0, 1);
        const uint64_t a0 = umma::desc_add(dEP, 64 * 128);
#pragma unroll
        for (int k0 = 0; k0 < C; k0 += 16)
            umma::mma_f16(tmem, umma::desc_add(a0, umma::koff_kmaj(192, k0)),
                          umma::desc_add(dKmn, umma::koff_mnmaj(k0)), ID, k0 > 0);
        umma::mma_commit(&mbar[3]);
    }
    if (!wait_mma(&mbar[3], 0)) goto done;
    umma::fence_after_sync();
    // Qt row i = scale e^{gamma_i} q_i - (Pt diag(e^gamma) K)_i -> record
    if (tid >= 64) {
        const int i = tid - 64;
        const float fq = p.scale * __expf(sG[i]);
#pragma unroll 1
        for (int c32 = 0; c32 < kDim; c32 += 32) {
            float d[32];
            umma::tmem_ld32(tmem + lane_base + c32, d);
#pragma unroll
            for (int e = 0; e < 32; e += 8) {
                const __half2* qh =
                    reinterpret_cast<const __half2*>(sm + OFF_KQ + umma::kmaj_off(64 + i, c32 + e, 128));
                float x[8];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float2 q2 = __half22float2(qh[u]);
                    x[2 * u] = fmaf(fq, q2.x, -d[e + 2 * u]);
                    x[2 * u + 1] = fmaf(fq, q2.y, -d[e + 2 * u + 1]);
                }
                st_f16x8(rec + REC_QT, umma::kmaj_off(i, c32 + e, 64), x);
            }
        }
    }

done:
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 0) umma::tmem_dealloc(tmem, TM_COLS);
}

}  // namespace prep

// ============================================================================
// chain: one CTA per (sequence, v-head), state transposed (state row v =
// TMEM lane v, as the k-last storage S^T[v][k])
// ============================================================================
// Per chunk j, with the state's f16 copy SA_j = S_j^T and the v rows' f16
// copy VA_j = V_j^T as A operands in tensor memory and the record's tiles as
// B operands in shared memory:
//   X2(j): X  = VA_j Et_j^T                 (issued as soon as VA_j is ready)
//   X1(j): X += SA_j (-Abar_j)^T            (the one product on the critical path)
//   O(j) : O  = SA_j Qt_j^T + VA_j Pt_j^T   (the chunk's outputs, [v][token])
// and the state threads form S_{j+1}^T = e^{gamma_C} S_j^T + X in fp32
// registers and its f16 copy for X1(j+1).
//
// Warp roles (TMEM lane quarter = warp % 4, thread = state row v = 32 * quarter + lane):
//   warps 0-7    the state: fp32 in registers, 64 columns k per thread
//                (warps 0-3 columns 0-63, warps 4-7 columns 64-127);
//                checkpoints and the final state;
//   warps 8-11   the outputs (64 tokens of row v per thread, bf16 stores,
//                32 consecutive v per warp store) and the f16 A copy of
//                the next chunks' v rows;
//   warp 12      one thread issues every MMA, in one order;
//   warp 13      one thread loads the records (one bulk copy per chunk, two
//                buffers) and the v rows (one TMA tensor copy per chunk,
//                three buffers).
namespace chain {

constexpr int NT = 448;                  // 14 warps
constexpr int kSThreads = 256, kOThreads = 128;
constexpr int kOBase = 256;
constexpr int kIssuer = 384;             // warp 12, lane 0
constexpr int kLoaderWarp = 13;
constexpr int NB = 2;                    // record buffers (chunk i in i % 2)
constexpr int NV = 3;                    // v-row buffers (chunk i in i % 3)
constexpr uint32_t kRecStride = (kRecBytes + 1023) / 1024 * 1024;
constexpr uint32_t kTileV = C * kDim * 2;  // 16 KiB, bf16 [token][v]
constexpr uint32_t OFF_REC = 0;
constexpr uint32_t OFF_V = NB * kRecStride;
constexpr uint32_t SMEM_BYTES = OFF_V + NV * kTileV + 1024;
static_assert(SMEM_BYTES <= 232448, "dynamic shared memory limit");
static_assert(kRecStride % 1024 == 0 && OFF_V % 1024 == 0, "tile alignment");
// no prep CTA fits beside a chain CTA, so the chain's 512 TMEM columns are
// never contended
static_assert(SMEM_BYTES + prep::SMEM_BYTES > 233472, "chain CTA alone on its SM");
constexpr uint32_t TM_X = 0, TM_O = 128, TM_SA = 256, TM_VA = 384, TM_COLS = 512;

constexpr uint32_t ID_N128 = umma::idesc_f16(128, 128, 0, 0, 0, 0);  // A (TMEM) x K-major B, N = 128
constexpr uint32_t ID_N64 = umma::idesc_f16(128, 64, 0, 0, 0, 0);    // N = 64

struct Bars {
    uint64_t ldR[NB];   // record of the chunk in buffer i % 2 landed
    uint64_t ldV[NV];   // v rows of the chunk in buffer i % 3 landed
    uint64_t vr[2];     // VA[i % 2] written (output threads)
    uint64_t sr[2];     // SA[i % 2] written (state threads)
    uint64_t mX;        // X1(i) complete
    uint64_t xr;        // state threads have read X_i
    uint64_t mO[2];     // O(i) complete
    uint64_t od[2];     // output threads have read O[i % 2]
    uint64_t fin;       // drain of the issuer's MMAs
};

__device__ __forceinline__ uint32_t ph(long long use) { return (uint32_t)(use & 1); }
__device__ __forceinline__ void arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(umma::smem_u32(bar)) : "memory");
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

__global__ void __launch_bounds__(NT, 1) gdn_prefill_scan_chain_kernel(const PrefillParams p,
                                                                     const unsigned char* ws,
                                                                     const __grid_constant__ CUtensorMap tmap_v) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ Bars B;
    __shared__ uint32_t tmem_base_sh;
    __shared__ volatile int abort_flag;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quarter = warp & 3;
    const int v = 32 * quarter + lane;  // state row (TMEM lane) of this thread
    const int hv = (int)(blockIdx.x % p.HV), n = (int)(blockIdx.x / p.HV);

    long long t0, t1;
    seq_bounds(p, n, t0, t1);
    if (tid < kDim) zero_uncovered_outputs(p, n, t0, t1, hv, tid, true);
    const size_t state_off = ((size_t)n * p.HV + hv) * kDim * kDim;  // [n][hv][v][k]
    const long long slot0 = t0 / C + n;
    const long long nchunks = (t1 - t0 + C - 1) / C;
    if (nchunks == 0) {  // empty sequence: the final state is zero
        for (int idx = tid; idx < kDim * kDim / 4; idx += NT)
            reinterpret_cast<float4*>(p.new_state + state_off)[idx] = make_float4(0.f, 0.f, 0.f, 0.f);
        return;
    }
    const int ni = (int)nchunks;
    auto chunk_len = [&](long long j) { const long long r = t1 - t0 - C * j; return (int)(r < C ? r : C); };
    auto rec_of = [&](int i) { return sm + OFF_REC + (i % NB) * kRecStride; };

    if (warp == 0) {
        umma::tmem_alloc(&tmem_base_sh, TM_COLS);
        umma::tmem_relinquish();
    }
    if (tid == 0) {
        for (int b = 0; b < NB; ++b) umma::mbar_init(&B.ldR[b], 1);
        for (int b = 0; b < NV; ++b) umma::mbar_init(&B.ldV[b], 1);
        for (int b = 0; b < 2; ++b) {
            umma::mbar_init(&B.vr[b], kOThreads);
            umma::mbar_init(&B.sr[b], kSThreads);
            umma::mbar_init(&B.mO[b], 1);
            umma::mbar_init(&B.od[b], kOThreads);
        }
        umma::mbar_init(&B.mX, 1);
        umma::mbar_init(&B.xr, kSThreads);
        umma::mbar_init(&B.fin, 1);
        umma::fence_mbar_init();
        abort_flag = 0;
    }
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = tmem_base_sh;
    const uint32_t tl = tmem + ((uint32_t)(32 * quarter) << 16);
    bool failed = false;
    // bounded wait; a failure is remembered (and every later wait then fails at once)
    auto wait = [&](uint64_t* bar, uint32_t parity) {
        if (failed || abort_flag) { failed = true; return; }
        if (!umma::mbar_wait(bar, parity, kWaitBudget)) { failed = true; abort_flag = 1; }
    };
    int issuedR = 0, issuedV = 0;  // loads issued by the loader warp (chunks 0 .. issued - 1)

    if (warp == kLoaderWarp) {
        // ---- records (bulk, 2 buffers) and v rows (tensor copy, 3 buffers) ----
        auto loadR = [&](int i) {
            if (lane == 0) {
                umma::mbar_arrive_expect_tx(&B.ldR[i % NB], kRecBytes);
                umma::bulk_g2s(umma::smem_u32(rec_of(i)), ws + ((size_t)(slot0 + i) * p.HV + hv) * kRecBytes,
                               kRecBytes, &B.ldR[i % NB]);
            }
            __syncwarp();
        };
        auto loadV = [&](int i) {
            if (lane == 0) {
                umma::mbar_arrive_expect_tx(&B.ldV[i % NV], kTileV);
                ::gdn::chunk::chain3::tma_load_v(umma::smem_u32(sm + OFF_V + (i % NV) * kTileV), &tmap_v, hv,
                                                 (int)(t0 + C * (long long)i), &B.ldV[i % NV]);
            }
            __syncwarp();
        };
        for (int i = 0; i < NB && i < ni; ++i) loadR(i);
        for (int i = 0; i < NV && i < ni; ++i) loadV(i);
        issuedR = ni < NB ? ni : NB;
        issuedV = ni < NV ? ni : NV;
        for (int i = 0; i < ni && !failed; ++i) {
            if (i + NV < ni) {  // v rows of chunk i copied into VA
                wait(&B.vr[i % 2], ph(i / 2));
                if (failed) break;
                loadV(i + NV);
                issuedV = i + NV + 1;
            }
            if (i + NB < ni) {
                // record buffer of chunk i: every MMA of chunk i done, and the
                // state threads have read its e^{gamma_C} (before S_{i+1})
                wait(&B.mO[i % 2], ph(i / 2));
                wait(&B.sr[(i + 1) % 2], ph((i + 1) / 2));
                if (failed) break;
                loadR(i + NB);
                issuedR = i + NB + 1;
            }
        }
    } else if (tid == kIssuer) {
        // ---- the MMA issuer: descriptors built once, stepped by constant offsets ----
        const uint64_t dR0 = umma::desc_kmaj(umma::smem_u32(sm + OFF_REC), 128, 0);
        const uint64_t dQ0 = umma::desc_kmaj(umma::smem_u32(sm + OFF_REC + REC_QT), 64, 0);
        const uint64_t dP0 = umma::desc_kmaj(umma::smem_u32(sm + OFF_REC + REC_P), 64, 0);
        for (int i = 0; i < ni && !failed; ++i) {
            const uint32_t rb = (uint32_t)(i % NB) * kRecStride;
            const uint32_t sa = tmem + TM_SA + (uint32_t)(i % 2) * 64, va = tmem + TM_VA + (uint32_t)(i % 2) * 32;
            // X2(i): X = VA_i Et_i^T, once the record and VA_i are in and X_{i-1} has been read
            wait(&B.ldR[i % NB], ph(i / NB));
            wait(&B.vr[i % 2], ph(i / 2));
            if (i > 0) wait(&B.xr, ph(i - 1));
            if (failed) break;
            umma::fence_after_sync();
#pragma unroll
            for (int k0 = 0; k0 < C; k0 += 16)
                umma::mma_f16_ts(tmem + TM_X, va + k0 / 2, umma::desc_add(dR0, rb + REC_E + umma::koff_kmaj(128, k0)),
                                 ID_N128, k0 > 0);
            // X1(i): X += SA_i (-Abar_i)^T, once S_i's f16 copy is written
            wait(&B.sr[i % 2], ph(i / 2));
            if (failed) break;
            umma::fence_after_sync();
#pragma unroll
            for (int k0 = 0; k0 < kDim; k0 += 16)
                umma::mma_f16_ts(tmem + TM_X, sa + k0 / 2, umma::desc_add(dR0, rb + umma::koff_kmaj(128, k0)),
                                 ID_N128, true);
            umma::mma_commit(&B.mX);
            // O(i) = SA_i Qt_i^T + VA_i Pt_i^T, once O[i % 2] has been read (chunk i - 2)
            if (i >= 2) wait(&B.od[i % 2], ph((i - 2) / 2));
            if (failed) break;
            umma::fence_after_sync();
            const uint32_t od = tmem + TM_O + (uint32_t)(i % 2) * 64;
#pragma unroll
            for (int k0 = 0; k0 < kDim; k0 += 16)
                umma::mma_f16_ts(od, sa + k0 / 2, umma::desc_add(dQ0, rb + umma::koff_kmaj(64, k0)), ID_N64, k0 > 0);
#pragma unroll
            for (int k0 = 0; k0 < C; k0 += 16)
                umma::mma_f16_ts(od, va + k0 / 2, umma::desc_add(dP0, rb + umma::koff_kmaj(64, k0)), ID_N64, true);
            umma::mma_commit(&B.mO[i % 2]);
        }
        // drain: every MMA issued here completes before the CTA exits
        umma::mma_commit(&B.fin);
        if (!umma::mbar_wait(&B.fin, 0, kWaitBudget)) failed = true;
    } else if (warp < 8) {
        // ---- the state: row v, columns c0 .. c0 + 63, fp32 in registers ----
        const int c0 = 64 * (warp >> 2);
        float s[64];
        {
            const float* srow = p.state ? p.state + state_off + (size_t)v * kDim + c0 : nullptr;
#pragma unroll
            for (int e = 0; e < 64; e += 4) {
                const float4 f = srow ? *reinterpret_cast<const float4*>(srow + e) : make_float4(0.f, 0.f, 0.f, 0.f);
                s[e] = f.x; s[e + 1] = f.y; s[e + 2] = f.z; s[e + 3] = f.w;
            }
            uint32_t h[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) h[e] = pack_f16x2(s[2 * e], s[2 * e + 1]);
            umma::tmem_st32_u32(tl + TM_SA + c0 / 2, h);
            umma::fence_before_sync();
            arrive(&B.sr[0]);
        }
        for (int i = 0; i < ni && !failed; ++i) {
            wait(&B.mX, ph(i));
            wait(&B.ldR[i % NB], ph(i / NB));
            if (failed) break;
            umma::fence_after_sync();
            const float decay = *reinterpret_cast<const float*>(rec_of(i) + REC_DECAY);
#pragma unroll
            for (int hh = 0; hh < 64; hh += 32) {  // two 32-column halves keep fewer registers live
                float x[32];
                umma::tmem_ld32(tl + TM_X + c0 + hh, x);
                if (hh == 32) {
                    umma::fence_before_sync();
                    arrive(&B.xr);
                }
#pragma unroll
                for (int e = 0; e < 32; e += 2) {
                    const float2 r = __ffma2_rn(make_float2(decay, decay), make_float2(s[hh + e], s[hh + e + 1]),
                                                make_float2(x[e], x[e + 1]));
                    s[hh + e] = r.x; s[hh + e + 1] = r.y;
                }
            }
            const long long done_tok = C * (long long)(i + 1);
            if (p.ckpt != nullptr && chunk_len(i) == C && done_tok % p.ckpt_every == 0) {
                float* cd = ckpt_dst(p, n, hv, done_tok);
                if (cd != nullptr) {
#pragma unroll
                    for (int e = 0; e < 64; e += 4)
                        __stcs(reinterpret_cast<float4*>(cd + (size_t)v * kDim + c0 + e),
                               make_float4(s[e], s[e + 1], s[e + 2], s[e + 3]));
                }
            }
            if (i + 1 < ni) {
                uint32_t h[32];
#pragma unroll
                for (int e = 0; e < 32; ++e) h[e] = pack_f16x2(s[2 * e], s[2 * e + 1]);
                umma::tmem_st32_u32(tl + TM_SA + (uint32_t)((i + 1) % 2) * 64 + c0 / 2, h);
                umma::fence_before_sync();
                arrive(&B.sr[(i + 1) % 2]);
            }
        }
        if (!failed) {  // the final state, fp32 k-last
            float* drow = p.new_state + state_off + (size_t)v * kDim + c0;
#pragma unroll
            for (int e = 0; e < 64; e += 4)
                __stcs(reinterpret_cast<float4*>(drow + e), make_float4(s[e], s[e + 1], s[e + 2], s[e + 3]));
        }
    } else if (warp < 12) {
        // ---- outputs and the f16 copies of the v rows ----
        // VA_i[v][t] = v rows of chunk i (f16, pairs of tokens per 32-bit
        // column); tokens past the chunk's end are zero
        auto copy_v = [&](int i) {
            wait(&B.ldV[i % NV], ph(i / NV));
            if (failed) return;
            const int len = chunk_len(i);
            const unsigned short* col = reinterpret_cast<const unsigned short*>(sm + OFF_V + (i % NV) * kTileV) + v;
            uint32_t h[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) {
                const float lo = 2 * e < len ? __uint_as_float((uint32_t)col[(2 * e) * kDim] << 16) : 0.f;
                const float hi = 2 * e + 1 < len ? __uint_as_float((uint32_t)col[(2 * e + 1) * kDim] << 16) : 0.f;
                h[e] = pack_f16x2(lo, hi);
            }
            umma::tmem_st32_u32(tl + TM_VA + (uint32_t)(i % 2) * 32, h);
            umma::fence_before_sync();
            arrive(&B.vr[i % 2]);
        };
        copy_v(0);
        if (ni > 1) copy_v(1);
        for (int i = 0; i < ni && !failed; ++i) {
            const long long tc = t0 + C * (long long)i;
            const int len = chunk_len(i);
            wait(&B.mO[i % 2], ph(i / 2));
            if (failed) break;
            umma::fence_after_sync();
            float o[64];
            {
                float oa[32], ob[32];
                umma::tmem_ld32x2(tl + TM_O + (uint32_t)(i % 2) * 64, tl + TM_O + (uint32_t)(i % 2) * 64 + 32, oa, ob);
#pragma unroll
                for (int e = 0; e < 32; ++e) { o[e] = oa[e]; o[32 + e] = ob[e]; }
            }
            umma::fence_before_sync();
            arrive(&B.od[i % 2]);
            // VA[i % 2] is free (X2(i) and O(i) are done): the v rows of chunk i + 2
            if (i + 2 < ni) copy_v(i + 2);
            // a warp stores 32 consecutive v of one token row per instruction
            __nv_bfloat16* op = p.out + ((size_t)tc * p.HV + hv) * kDim + v;
            const size_t stride = (size_t)p.HV * kDim;
#pragma unroll
            for (int t = 0; t < 64; ++t)
                if (t < len) op[(size_t)t * stride] = __float2bfloat16_rn(o[t]);
        }
    }

    // ---- exit: copies in flight land first ----
    umma::fence_before_sync();
    failed = __syncthreads_or(failed) || abort_flag;
    if (failed && warp == kLoaderWarp) {
        if (lane == 0) atomicOr(&g_device_status, kDevStatTimeout);
        for (int i = (issuedR > NB ? issuedR - NB : 0); i < issuedR; ++i)
            umma::mbar_wait(&B.ldR[i % NB], ph(i / NB), kWaitBudget);
        for (int i = (issuedV > NV ? issuedV - NV : 0); i < issuedV; ++i)
            umma::mbar_wait(&B.ldV[i % NV], ph(i / NV), kWaitBudget);
    }
    __syncthreads();
    if (warp == 0) umma::tmem_dealloc(tmem, TM_COLS);
}

}  // namespace chain
}  // namespace scan
