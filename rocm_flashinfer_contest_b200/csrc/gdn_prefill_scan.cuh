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
// read by the chain; both tiles are in the 128-byte-swizzled K-major layout
// of the chain's B operands, with 192 rows so that one N = 192 product
// yields the state update and the outputs together:
//   [-Abar ; Qt]  rows 0-127: -Abar row k'; rows 128-191: Qt row (token);
//                 columns k (two 64-column slabs of 24 KiB)     48 KiB
//   [Et ; Pt]     rows 0-127: Et row k; rows 128-191: Pt row (token i);
//                 columns token (j)                             24 KiB
//   e^{gamma_C} (fp32), padding to a multiple of 256 bytes         256 B
// (the prep writes the tiles with 32-byte stores: records, and so the
// workspace, are 32-byte aligned)
constexpr uint32_t REC_AQ = 0, REC_EP = 49152, REC_DECAY = 73728;
constexpr uint32_t kRecBytes = 73984;
constexpr uint32_t kRecRows = 192;

// The records, then one ready flag (uint32) per record: the prep sets it
// (release, device scope) once the record is written, the chain acquires it
// before reading the record, so the two kernels may run concurrently.  The
// host zeroes the flags before each launch pair.
__host__ __device__ inline size_t records_bytes(int N, int T, int HV) {
    return (size_t)ws_slots(N, T) * HV * kRecBytes;
}
__host__ __device__ inline size_t flags_bytes(int N, int T, int HV) {
    return ((size_t)ws_slots(N, T) * HV * 4 + 255) / 256 * 256;
}
__host__ __device__ inline size_t workspace_bytes(int N, int T, int HV) {
    return records_bytes(N, T, HV) + flags_bytes(N, T, HV);
}
__device__ __forceinline__ unsigned int* ready_flag(const PrefillParams& p, const unsigned char* ws, long long slot,
                                                    int hv) {
    return reinterpret_cast<unsigned int*>(const_cast<unsigned char*>(ws) + records_bytes(p.N, p.T, p.HV)) +
           (size_t)slot * p.HV + hv;
}
__device__ __forceinline__ unsigned int ld_acquire(const unsigned int* a) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
    return v;
}
// Bounded wait for a record's ready flag (acquire); false after ~kWaitBudget cycles.
__device__ __forceinline__ bool wait_ready(const unsigned int* flag) {
    if (ld_acquire(flag) != 0u) return true;
    const long long t0 = clock64();
    while (ld_acquire(flag) == 0u) {
        if (clock64() - t0 > kWaitBudget) {
            atomicOr(&g_device_status, kDevStatTimeout);
            return false;
        }
        __nanosleep(64);
    }
    return true;
}

// 16 f16 values (columns k0 .. k0 + 15, k0 a multiple of 16) of row `row` of
// a K-major 128-byte-swizzled tile in global memory, as one 32-byte store:
// chunks k0/8 and k0/8 + 1 of a row stay one aligned 32-byte pair under the
// swizzle (XOR with row % 8), in swapped order when the row is odd.  A warp
// of rows then writes whole 32-byte sectors.
__device__ __forceinline__ void st_f16x16_tile(unsigned char* tile, uint32_t row, uint32_t k0, uint32_t rows,
                                               const float* x) {
    uint32_t h[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        __half2 t = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
        h[i] = *reinterpret_cast<uint32_t*>(&t);
    }
    if (row & 1u) {
#pragma unroll
        for (int i = 0; i < 4; ++i) { const uint32_t t = h[i]; h[i] = h[4 + i]; h[4 + i] = t; }
    }
    asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
                 :: "l"(tile + (umma::kmaj_off(row, k0, rows) & ~31u)), "r"(h[0]), "r"(h[1]), "r"(h[2]), "r"(h[3]),
                    "r"(h[4]), "r"(h[5]), "r"(h[6]), "r"(h[7])
                 : "memory");
}

// ============================================================================
// prep: one CTA per chunk and one or two v-heads of a q/k head
// ============================================================================
namespace prep {

using ::gdn::chunk::prep::ix;
// A CTA builds the records of NU v-heads of one chunk that share a q/k head
// (NU = 2 when HV / H is even): one [K ; Q] tile, its f16 conversion and its
// Gram product serve both; each v-head (a group of 128 threads, its own
// shared-memory region and 128 TMEM columns) then takes its masks, solve and
// products.  Per group, the solve matrices' 34 KiB hold the f16 operand
// tiles once the solve is done.
constexpr uint32_t OFF_KQ = 0;                      // [K ; Q] f16 K-major 128 x 128, whole kernel
constexpr uint32_t kGroupBytes = 35840;             // per v-head region (1 KiB multiple)
constexpr uint32_t G_A = 0;                         // A fp32 [64][LDA] during the solve
constexpr uint32_t G_T = 64 * LDA * 4;              // T fp32 [64][LDA] during the solve
constexpr uint32_t G_TP = 0;                        // [T diag(beta) ; P] K-major 128 x 64       16 KiB
constexpr uint32_t G_T1 = 18432;                    // diag(f_K) T diag(beta), 64 x 64 (MN-major B) 8 KiB
constexpr uint32_t G_EP = 0;                        // [Et diag(e^g) ; Pt diag(e^g)] K-major 192 x 64, 24 KiB
constexpr uint32_t G_GM = 2 * 64 * LDA * 4;         // gamma[64], beta[64], e^gamma[64]
static_assert(G_T1 % 1024 == 0 && G_T1 >= G_TP + kTileTP && G_T1 + 8192 <= G_GM, "T1 after [T ; P], before the gates");
static_assert(G_EP + 24576 <= G_GM && G_GM + 768 <= kGroupBytes && kGroupBytes % 1024 == 0, "group region");
template <int NU> constexpr uint32_t smem_bytes() { return kTileKQ + NU * kGroupBytes + 1024; }  // + alignment slack
template <int NU> constexpr int ctas_per_sm() { return NU == 1 ? 3 : 2; }
static_assert(3 * (smem_bytes<1>() + 1024) <= 233472 && 2 * (smem_bytes<2>() + 1024) <= 233472,
              "three one-head or two two-head CTAs per SM");
static_assert(3 * 128 <= 512 && 2 * 256 <= 512, "their TMEM columns fit the SM's 512");

// MMA_E reads T1 = diag(f_K) T diag(beta) MN-major (k = token i, n = token j):
// a row-major 64 x 64 tile in the K-major layout of 64 rows is that operand.
constexpr bool rows64_are_mn_major() {
    for (uint32_t i = 0; i < 64; ++i)
        for (uint32_t j = 0; j < 64; ++j)
            if (umma::kmaj_off(i, j, 64) != umma::mnmaj_off(j, i, 64)) return false;
    return true;
}
static_assert(rows64_are_mn_major(), "a K-major 64-row tile doubles as the MN-major B operand");

template <int NU>
__global__ void __launch_bounds__(128 * NU, ctas_per_sm<NU>()) gdn_prefill_scan_prep_kernel(const PrefillParams p,
                                                                                        unsigned char* ws) {
    constexpr int NT = 128 * NU;
    constexpr uint32_t TM_COLS = 128 * NU;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t mbar[4];
    __shared__ uint32_t tmem_base_sh;

    const int tid = threadIdx.x, warp = tid >> 5;
    const int g = tid >> 7, gt = tid & 127, gwarp = warp & 3;  // v-head group, thread and warp within it
    const int groups = p.HV / NU;
    const long long s = blockIdx.x / groups;
    const int hv0 = (int)(blockIdx.x % groups) * NU;
    const int hv = hv0 + g, hq = hv0 / p.rep;

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

    unsigned char* gm = sm + kTileKQ + g * kGroupBytes;  // this v-head's region
    float* sA = reinterpret_cast<float*>(gm + G_A);
    float* sT = reinterpret_cast<float*>(gm + G_T);
    float* sG = reinterpret_cast<float*>(gm + G_GM);
    float* sBeta = sG + 64;
    float* sEg = sG + 128;  // e^gamma per token: the column factors of the read-outs, one exp each
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
    // gates and the inclusive scan of log g (warps 0 and 1 of each group)
    float lg = 0.f, beta = 0.f;
    if (gt < len) {
        const size_t gi = (size_t)(tc + gt) * p.HV + hv;
        lg = log_gate(p.A_log[hv], bf16_to_f32(p.a[gi]), p.dt_bias[hv]);
        beta = sigmoidf_(bf16_to_f32(p.b[gi]));
    }
    if (gwarp < 2) {
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, lg, o);
            if ((gt & 31) >= o) lg += y;
        }
        if (gwarp == 0) sG[gt] = lg;
        sBeta[gt] = beta;
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
    if (gwarp == 1) sG[gt] = lg + sG[31];
    cp_async_wait_all();
    __syncthreads();
    if (gt < C) sEg[gt] = __expf(sG[gt]);  // read after the masks' and solve's barriers
    // every product here takes [K ; Q] as f16: normalised rows are written as
    // f16, raw bf16 rows are converted (exact for |x| in f16's normal range)
    if (p.qk_l2norm) {
        if (tid < 128) l2norm_row_to_f16(sm + OFF_KQ, tid, 128);
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
    const uint32_t lane_base = (uint32_t)(32 * gwarp) << 16;
    const uint32_t tg = tmem + 128 * g;  // this v-head's 128 TMEM columns
    const uint64_t dKQ = umma::desc_kmaj(sKQ, 128, 0);
    const uint64_t dKmn = umma::desc_sw128(sKQ, 16384u, 1024u);  // K rows read MN-major (K^T as A, K as B)
    bool ok = false;

    // MMA_G: [K ; Q] K^T -> columns 0-63 (read by every v-head's masks)
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

    // Both masks in one pass, each read from its own TMEM lanes:
    //   A = beta_i e^{gamma_i - gamma_j} k_i.k_j (j < i), rows 0-63 (warps 0, 1 of
    //       the group), into the strictly lower part of sA (whole float4
    //       groups below the diagonal, i.e. columns < ceil4(i));
    //   P = scale e^{gamma_i - gamma_j} q_i.k_j (j <= i), rows 64-127 (warps 2, 3),
    //       as f16 into the part of sA the solve never touches: P row i (i + 1
    //       values) in row 63 - i from column ceil4(63 - i) on, which leaves
    //       4 (i + 2) bytes of room (with the padding columns 64-67).
    // P reaches its tile after the solve, once sA is free.
    {
        const int i = gt & 63;
        const bool arow = gt < 64;
        const float gi = sG[i];
        const float coef = arow ? sBeta[i] : p.scale;
        const int lim = arow ? i : i + 1;  // columns jj < lim are kept
        unsigned char* prow = reinterpret_cast<unsigned char*>(sA + ix(63 - i, ((63 - i) + 3) & ~3));
#pragma unroll 1
        for (int c16 = 0; c16 < C; c16 += 16) {
            // the warp's rows are 32 * (warp % 2) .. + 31: blocks of columns
            // past them are zero for all of its threads (a warp-uniform exit,
            // as tcgen05.ld is executed by whole warps)
            if (c16 > 32 * (gwarp & 1) + 31) break;
            float d[16], r[16];
            umma::tmem_ld16(tmem + lane_base + c16, d);
            if (c16 >= lim) continue;
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const int jj = c16 + e;
                r[e] = (jj < lim) ? coef * __expf(fminf(gi - sG[jj], 0.f)) * d[e] : 0.f;
            }
            if (arow) {
#pragma unroll
                for (int e = 0; e < 16; e += 4)
                    if (c16 + e < i)
                        *reinterpret_cast<float4*>(sA + ix(i, c16 + e)) = make_float4(r[e], r[e + 1], r[e + 2], r[e + 3]);
            } else {
                st_f16x8(prow, 2 * c16, r);
                if (c16 + 8 < lim) st_f16x8(prow, 2 * c16 + 16, r + 8);
            }
        }
    }
    // from the masks to the T copies each v-head group works on its own
    // matrices: its own named barrier (1 + g), not the whole CTA
    ::gdn::chunk::prep::group_bar(1 + g);
    ::gdn::chunk::prep::solve_T(sA, sT, gt, 1 + g);

    // f16 copies of T: T diag(beta) -> rows 0-63 of [T ; P] (the B operand of
    // MMA_P, read MN-major from those rows) and diag(f_K) T diag(beta) -> T1;
    // the P rows from their place in sA -> rows 64-127 of [T ; P].  Every
    // thread reads its part first: the tiles overlay sA and sT.
    {
        const int i = gt >> 1, h = (gt & 1) * 32;  // row i, columns h..h+31
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
        // P row pi (threads 64-127 of the group): 8 chunks of 8 f16, chunks past the diagonal zero
        const int pi = gt - 64;
        uint4 pr[8];
        if (gt >= 64) {
            const unsigned char* prow = reinterpret_cast<const unsigned char*>(sA + ix(63 - pi, ((63 - pi) + 3) & ~3));
#pragma unroll
            for (int c = 0; c < 8; ++c)
                pr[c] = 8 * c <= pi ? *reinterpret_cast<const uint4*>(prow + 16 * c) : make_uint4(0u, 0u, 0u, 0u);
        }
        ::gdn::chunk::prep::group_bar(1 + g);  // the tiles below overwrite sA and part of sT
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
            float x[8], y[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                x[e] = t[c + e] * sBeta[h + c + e];
                y[e] = fk * x[e];
            }
            st_f16x8(gm + G_TP, umma::kmaj_off(i, h + c, 128), x);
            st_f16x8(gm + G_T1, umma::kmaj_off(i, h + c, 64), y);
        }
        if (gt >= 64) {
#pragma unroll
            for (int c = 0; c < 8; ++c)
                *reinterpret_cast<uint4*>(gm + G_TP + umma::kmaj_off(64 + pi, 8 * c, 128)) = pr[c];
        }
    }
    sync_for_mma();

    // per v-head u (columns 128u ..): MMA_P: [T diag(beta) ; P] x T diag(beta)
    // -> columns 0-63, rows 64-127 = Pt;  MMA_E: K^T x T1 -> columns 64-127 = Et
    if (tid == 0) {
        constexpr uint32_t IDP = umma::idesc_f16(128, 64, 0, 0, 0, 1);
        constexpr uint32_t IDE = umma::idesc_f16(128, 64, 0, 0, 1, 1);
#pragma unroll
        for (int u = 0; u < NU; ++u) {
            unsigned char* um = sm + kTileKQ + u * kGroupBytes;
            const uint64_t dTP = umma::desc_kmaj(umma::smem_u32(um + G_TP), 128, 0);
            const uint64_t dTB = umma::desc_mnmaj(umma::smem_u32(um + G_TP), C, 0);
            const uint64_t dT1 = umma::desc_mnmaj(umma::smem_u32(um + G_T1), C, 0);
#pragma unroll
            for (int k0 = 0; k0 < C; k0 += 16)
                umma::mma_f16(tmem + 128 * u, umma::desc_add(dTP, umma::koff_kmaj(128, k0)),
                              umma::desc_add(dTB, umma::koff_mnmaj(k0)), IDP, k0 > 0);
#pragma unroll
            for (int k0 = 0; k0 < C; k0 += 16)
                umma::mma_f16(tmem + 128 * u + 64, umma::desc_add(dKmn, umma::koff_mnmaj(k0)),
                              umma::desc_add(dT1, umma::koff_mnmaj(k0)), IDE, k0 > 0);
        }
        umma::mma_commit(&mbar[1]);
    }
    if (!wait_mma(&mbar[1], 0)) goto done;
    umma::fence_after_sync();

    // Pt (record rows 128-191 of [Et ; Pt]) and Pt diag(e^gamma) (rows 128-191
    // of [E2 ; P2]); Et (record rows 0-127) and Et diag(e^gamma) (rows 0-127).
    // Thread = TMEM lane.
    {
        float eg[16];
        if (gt >= 64) {
            const int i = gt - 64;
#pragma unroll 1
            for (int c16 = 0; c16 < C; c16 += 16) {
                float d[16];
                umma::tmem_ld16(tg + lane_base + c16, d);
#pragma unroll
                for (int e = 0; e < 16; ++e) eg[e] = sEg[c16 + e];
                st_f16x16_tile(rec + REC_EP, 128 + i, c16, kRecRows, d);
#pragma unroll
                for (int e = 0; e < 16; ++e) d[e] *= eg[e];
                st_f16x8(gm + G_EP, umma::kmaj_off(128 + i, c16, 192), d);
                st_f16x8(gm + G_EP, umma::kmaj_off(128 + i, c16 + 8, 192), d + 8);
            }
        }
#pragma unroll 1
        for (int c16 = 0; c16 < C; c16 += 16) {
            float d[16];
            umma::tmem_ld16(tg + lane_base + 64 + c16, d);
#pragma unroll
            for (int e = 0; e < 16; ++e) eg[e] = sEg[c16 + e];
            st_f16x16_tile(rec + REC_EP, gt, c16, kRecRows, d);
#pragma unroll
            for (int e = 0; e < 16; ++e) d[e] *= eg[e];
            st_f16x8(gm + G_EP, umma::kmaj_off(gt, c16, 192), d);
            st_f16x8(gm + G_EP, umma::kmaj_off(gt, c16 + 8, 192), d + 8);
        }
        if (gt == 0)
            *reinterpret_cast<float4*>(rec + REC_DECAY) = make_float4(__expf(sG[C - 1]), 0.f, 0.f, 0.f);
    }
    sync_for_mma();

    // MMA_A: [E2 ; P2] rows 0-127 x K -> columns 0-127 = Abar (per v-head)
    if (tid == 0) {
        constexpr uint32_t ID = umma::idesc_f16(128, 128, 0, 0, 0, 1);
#pragma unroll
        for (int u = 0; u < NU; ++u) {
            const uint64_t dEP = umma::desc_kmaj(umma::smem_u32(sm + kTileKQ + u * kGroupBytes + G_EP), 192, 0);
#pragma unroll
            for (int k0 = 0; k0 < C; k0 += 16)
                umma::mma_f16(tmem + 128 * u, umma::desc_add(dEP, umma::koff_kmaj(192, k0)),
                              umma::desc_add(dKmn, umma::koff_mnmaj(k0)), ID, k0 > 0);
        }
        umma::mma_commit(&mbar[2]);
    }
    if (!wait_mma(&mbar[2], 0)) goto done;
    umma::fence_after_sync();
    // -Abar row k' = gt -> record rows 0-127 of [-Abar ; Qt]
#pragma unroll 1
    for (int c32 = 0; c32 < kDim; c32 += 32) {
        float d[32];
        umma::tmem_ld32(tg + lane_base + c32, d);
#pragma unroll
        for (int e = 0; e < 32; ++e) d[e] = -d[e];
#pragma unroll
        for (int e = 0; e < 32; e += 16) st_f16x16_tile(rec + REC_AQ, gt, c32 + e, kRecRows, d + e);
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();

    // MMA_Q: [E2 ; P2] rows 64-191 x K -> columns 0-127; rows 64-127 = Pt diag(e^gamma) K
    if (tid == 0) {
        constexpr uint32_t ID = umma::idesc_f16(128, 128, 0, 0, 0, 1);
#pragma unroll
        for (int u = 0; u < NU; ++u) {
            const uint64_t a0 =
                umma::desc_add(umma::desc_kmaj(umma::smem_u32(sm + kTileKQ + u * kGroupBytes + G_EP), 192, 0), 64 * 128);
#pragma unroll
            for (int k0 = 0; k0 < C; k0 += 16)
                umma::mma_f16(tmem + 128 * u, umma::desc_add(a0, umma::koff_kmaj(192, k0)),
                              umma::desc_add(dKmn, umma::koff_mnmaj(k0)), ID, k0 > 0);
        }
        umma::mma_commit(&mbar[3]);
    }
    if (!wait_mma(&mbar[3], 0)) goto done;
    umma::fence_after_sync();
    // Qt row i = scale e^{gamma_i} q_i - (Pt diag(e^gamma) K)_i -> record rows 128-191 of [-Abar ; Qt]
    if (gt >= 64) {
        const int i = gt - 64;
        const float fq = p.scale * __expf(sG[i]);
#pragma unroll 1
        for (int c32 = 0; c32 < kDim; c32 += 32) {
            float d[32];
            umma::tmem_ld32(tg + lane_base + c32, d);
#pragma unroll
            for (int e = 0; e < 32; e += 16) {
                float x[16];
#pragma unroll
                for (int h8 = 0; h8 < 16; h8 += 8) {
                    const __half2* qh =
                        reinterpret_cast<const __half2*>(sm + OFF_KQ + umma::kmaj_off(64 + i, c32 + e + h8, 128));
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float2 q2 = __half22float2(qh[u]);
                        x[h8 + 2 * u] = fmaf(fq, q2.x, -d[e + h8 + 2 * u]);
                        x[h8 + 2 * u + 1] = fmaf(fq, q2.y, -d[e + h8 + 2 * u + 1]);
                    }
                }
                st_f16x16_tile(rec + REC_AQ, 128 + i, c32 + e, kRecRows, x);
            }
        }
    }
    ok = true;

done:
    umma::fence_before_sync();
    __syncthreads();
    // every thread's record writes, then the records' ready flags (release, device scope)
    if (ok && gt == 0) {
        __threadfence();
        asm volatile("st.release.gpu.global.u32 [%0], %1;" :: "l"(ready_flag(p, ws, s, hv)), "r"(1u) : "memory");
    }
    if (warp == 0) umma::tmem_dealloc(tmem, TM_COLS);
}

}  // namespace prep


// ============================================================================
// chain: one CTA per (sequence, v-head), state transposed (state row v =
// TMEM lane v, as the k-last storage S^T[v][k])
// ============================================================================
// Per chunk j, with the state's f16 copy SA = S_j^T in tensor memory, the v
// rows V_j (f16, MN-major: v contiguous) in shared memory as A operands, and
// the record's two 192-row tiles as B operands, two groups of N = 192
// products fill one accumulator [X | O] (128 + 64 columns):
//   MMA_V(j): [X | O]  = V_j^T [Et ; Pt]^T       (issued as soon as V_j is in)
//   MMA_S(j): [X | O] += SA [-Abar ; Qt]^T       (the critical path)
// X = -Abar S_j + Et V_j (the state update) and O = Qt S_j + Pt V_j (the
// chunk's outputs, [v][token]); the state threads then form S_{j+1}^T =
// e^{gamma_C} S_j^T + X in fp32 registers and its f16 copy for MMA_S(j+1).
// Twelve products and four waits per chunk for the one issuing thread.
//
// Tensor memory: [X | O] twice (chunk j in j % 2, 2 x 192 columns) and SA
// (64 columns: the next copy is written only after MMA_S(j) completes).
//
// Shared memory: the record's two tiles in rings of two ([-Abar ; Qt] 48 KiB,
// [Et ; Pt] 24 KiB, both freed when MMA_S(j) completes; e^{gamma_C} is read
// from global memory by the state threads), the v rows in a
// ring of four (two 64-wide TMA boxes with the 128-byte swizzle per chunk:
// the MN-major operand layout; converted from bf16 to f16 in place, tokens
// past the chunk's end zeroed), and one output tile staged as bf16 rows so
// that the stores are coalesced 16-byte rows (one 2-byte store per token and
// thread measured ~3,700 cycles per chunk: it was the step's bound).
//
// Warp roles (TMEM lane quarter = warp % 4, thread = state row v = 32 * quarter + lane):
//   warps 0-7    the state: fp32 in registers, 64 columns k per thread
//                (warps 0-3 columns 0-63, warps 4-7 columns 64-127);
//                checkpoints and the final state; after each state update,
//                the f16 conversion of the v rows (two chunks ahead);
//   warps 8-11   the outputs: staged as bf16 rows, one TMA tensor store per
//                full chunk (16-byte thread stores for a partial one);
//   warp 12      one thread issues every MMA, in one order;
//   warp 13      one thread loads the two record tiles and the v rows
//                (TMA tensor copies, four chunks ahead).
namespace chain {

constexpr int NT = 448;                  // 14 warps
constexpr int kSThreads = 256, kOThreads = 128;
constexpr int kOBase = 256;
constexpr int kIssuer = 384;             // warp 12, lane 0
constexpr int kLoaderWarp = 13;
constexpr int NA = 2;                    // [-Abar ; Qt] buffers (chunk i in i % 2)
constexpr int NE = 2;                    // [Et ; Pt] buffers (chunk i in i % 2)
constexpr int NV = 4;                    // v-row buffers (chunk i in i % 4)
constexpr uint32_t kTileAQ = REC_EP - REC_AQ;      // 48 KiB
constexpr uint32_t kTileEP = REC_DECAY - REC_EP;   // 24 KiB
constexpr uint32_t kTileV = C * kDim * 2;          // 16 KiB: two MN-major 64-v blocks of 64 tokens
constexpr uint32_t kTileO = C * kDim * 2;          // 16 KiB, bf16 [token][v]
constexpr uint32_t OFF_AQ = 0;
constexpr uint32_t OFF_EP = NA * kTileAQ;
constexpr uint32_t OFF_V = OFF_EP + NE * kTileEP;
constexpr uint32_t OFF_O = OFF_V + NV * kTileV;
constexpr uint32_t SMEM_BYTES = OFF_O + kTileO + 1024;
static_assert(SMEM_BYTES <= 232448 - 512, "dynamic shared memory limit (with the static barriers)");
static_assert(kTileAQ % 1024 == 0 && kTileEP % 1024 == 0 && OFF_EP % 1024 == 0 && OFF_V % 1024 == 0 &&
              OFF_O % 1024 == 0, "tile alignment");
// no prep CTA fits beside a chain CTA, so the chain's TMEM columns are never contended
static_assert(SMEM_BYTES + prep::smem_bytes<1>() > 233472, "chain CTA alone on its SM");
constexpr uint32_t kXO = 192;            // [X | O] columns
constexpr uint32_t TM_XO = 0, TM_SA = 2 * kXO, TM_COLS = 512;
static_assert(TM_SA + 64 <= TM_COLS, "tensor memory budget");
constexpr int kBarO = 1;                 // named barrier of the output warps

constexpr uint32_t ID_S = umma::idesc_f16(128, kXO, 0, 0, 0, 0);  // A (TMEM) x K-major B, N = 192
constexpr uint32_t ID_V = umma::idesc_f16(128, kXO, 0, 0, 1, 0);  // MN-major A (shared) x K-major B

struct Bars {
    uint64_t ldA[NA];   // [-Abar ; Qt] of the chunk in buffer i % 2 landed
    uint64_t ldE[NE];   // [Et ; Pt] of the chunk in buffer i % 2 landed
    uint64_t ldV[NV];   // v rows of the chunk in buffer i % 4 landed
    uint64_t vr[2];     // v rows of chunk i converted to f16 (state threads)
    uint64_t sr;        // SA written (state threads), once per chunk
    uint64_t mXO[2];    // MMA_S(i) complete: [X | O] of chunk i ready, its tiles, v rows and SA read
    uint64_t xo[2];     // state and output threads have read [X | O][i % 2]
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
// TMA load of one chunk's v rows as two 64-wide boxes {64 v, 1 head, 64
// tokens} of the [T, HV, 128] bf16 tensor (128-byte swizzle) at (64h, hv,
// tc) -> half h of the tile: line t = token, the MN-major operand layout.
// Rows at or past T are zero-filled.
__device__ __forceinline__ void tma_load_v_sw(uint32_t dst, const CUtensorMap* map, int hv, int tc, uint64_t* bar) {
#pragma unroll
    for (int h = 0; h < 2; ++h)
        asm volatile(
            "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
            :: "r"(dst + h * (kTileV / 2)), "l"(reinterpret_cast<uint64_t>(map)), "r"(64 * h), "r"(hv), "r"(tc),
               "r"(umma::smem_u32(bar))
            : "memory");
}

// TMA store of one full chunk's output rows (bf16 [token][v], 256-byte rows)
// as the box {128 v, 1 head, 64 tokens} of the [T, HV, 128] output tensor at
// (0, hv, tc), in a bulk group of the issuing thread.
__device__ __forceinline__ void tma_store_o(const CUtensorMap* map, uint32_t src, int hv, int tc) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];"
                 :: "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(hv), "r"(tc), "r"(src) : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__global__ void __launch_bounds__(NT, 1) gdn_prefill_scan_chain_kernel(const PrefillParams p,
                                                                     const unsigned char* ws,
                                                                     const __grid_constant__ CUtensorMap tmap_v,
                                                                     const __grid_constant__ CUtensorMap tmap_o) {
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
    auto rec_g = [&](int i) { return ws + ((size_t)(slot0 + i) * p.HV + hv) * kRecBytes; };

    if (warp == 0) {
        umma::tmem_alloc(&tmem_base_sh, TM_COLS);
        umma::tmem_relinquish();
    }
    if (tid == 0) {
        for (int b = 0; b < NV; ++b) umma::mbar_init(&B.ldV[b], 1);
        for (int b = 0; b < 2; ++b) {
            umma::mbar_init(&B.ldA[b], 1);
            umma::mbar_init(&B.ldE[b], 1);
            umma::mbar_init(&B.vr[b], kSThreads);
            umma::mbar_init(&B.mXO[b], 1);
            umma::mbar_init(&B.xo[b], kSThreads + kOThreads);
        }
        umma::mbar_init(&B.sr, kSThreads);
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
    // loads issued by the loader warp (chunks 0 .. issued - 1)
    int issuedA = 0, issuedE = 0, issuedV = 0;

    if (warp == kLoaderWarp) {
        // ---- the record's two tiles (bulk copies) and the v rows (tensor copies) ----
        auto load = [&](int i) {
            bool ok = true;
            if (lane == 0) {
                const unsigned char* r = rec_g(i);
                // the record is complete (its prep may run beside this kernel);
                // the bulk copies below read it through the async proxy
                ok = wait_ready(ready_flag(p, ws, slot0 + i, hv));
                if (ok) {
                    asm volatile("fence.proxy.async.global;" ::: "memory");
                    umma::mbar_arrive_expect_tx(&B.ldE[i % NE], kTileEP);
                    umma::bulk_g2s(umma::smem_u32(sm + OFF_EP + (i % NE) * kTileEP), r + REC_EP, kTileEP,
                                   &B.ldE[i % NE]);
                    umma::mbar_arrive_expect_tx(&B.ldA[i % NA], kTileAQ);
                    umma::bulk_g2s(umma::smem_u32(sm + OFF_AQ + (i % NA) * kTileAQ), r + REC_AQ, kTileAQ,
                                   &B.ldA[i % NA]);
                }
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (ok) {
                issuedA = issuedE = i + 1;
            } else {
                failed = true;
                abort_flag = 1;
            }
        };
        auto load_v = [&](int i) {  // chunk i's v rows into buffer i % 4
            if (lane == 0) {
                umma::mbar_arrive_expect_tx(&B.ldV[i % NV], kTileV);
                tma_load_v_sw(umma::smem_u32(sm + OFF_V + (i % NV) * kTileV), &tmap_v, hv,
                              (int)(t0 + C * (long long)i), &B.ldV[i % NV]);
            }
            __syncwarp();
            issuedV = i + 1;
        };
        for (int i = 0; i < NV && i < ni; ++i) load_v(i);
        for (int i = 0; i < NA && i < ni && !failed; ++i) load(i);
        for (int i = 0; i + NA < ni && !failed; ++i) {
            // MMA_V(i) and MMA_S(i) have read chunk i's tiles and v rows
            wait(&B.mXO[i % 2], ph(i / 2));
            if (failed) break;
            if (i + NV < ni) load_v(i + NV);
            load(i + NA);
        }
    } else if (tid == kIssuer) {
        // ---- the MMA issuer: descriptors built once, stepped by constant offsets ----
        const uint64_t dA0 = umma::desc_kmaj(umma::smem_u32(sm + OFF_AQ), kRecRows, 0);
        const uint64_t dE0 = umma::desc_kmaj(umma::smem_u32(sm + OFF_EP), kRecRows, 0);
        const uint64_t dV0 = umma::desc_mnmaj(umma::smem_u32(sm + OFF_V), C, 0);
        const uint32_t sa = tmem + TM_SA;
        // MMA_V(i): [X | O][i % 2] = V_i^T [Et ; Pt]_i^T, once the tile and the
        // converted v rows are in and [X | O] of chunk i - 2 has been read
        auto mma_v = [&](int i) {
            wait(&B.ldE[i % NE], ph(i / NE));
            wait(&B.vr[i % 2], ph(i / 2));
            if (i >= 2) wait(&B.xo[i % 2], ph((i - 2) / 2));
            if (failed) return;
            umma::fence_after_sync();
            const uint32_t d = tmem + TM_XO + (uint32_t)(i % 2) * kXO;
            const uint32_t eb = (uint32_t)(i % NE) * kTileEP, vb = (uint32_t)(i % NV) * kTileV;
#pragma unroll
            for (int k0 = 0; k0 < C; k0 += 16)
                umma::mma_f16(d, umma::desc_add(dV0, vb + umma::koff_mnmaj(k0)),
                              umma::desc_add(dE0, eb + umma::koff_kmaj(kRecRows, k0)), ID_V, k0 > 0);
        };
        mma_v(0);
        for (int i = 0; i < ni && !failed; ++i) {
            // MMA_S(i): [X | O][i % 2] += SA [-Abar ; Qt]_i^T, once S_i's f16 copy is written
            wait(&B.ldA[i % NA], ph(i / NA));
            wait(&B.sr, ph(i));
            if (failed) break;
            umma::fence_after_sync();
            const uint32_t d = tmem + TM_XO + (uint32_t)(i % 2) * kXO;
            const uint32_t ab = (uint32_t)(i % NA) * kTileAQ;
#pragma unroll
            for (int k0 = 0; k0 < kDim; k0 += 16)
                umma::mma_f16_ts(d, sa + k0 / 2, umma::desc_add(dA0, ab + umma::koff_kmaj(kRecRows, k0)), ID_S,
                                 true);
            umma::mma_commit(&B.mXO[i % 2]);
            if (i + 1 < ni) mma_v(i + 1);
        }
        // drain: every MMA issued here completes before the CTA exits
        umma::mma_commit(&B.fin);
        if (!umma::mbar_wait(&B.fin, 0, kWaitBudget)) failed = true;
    } else if (warp < 8) {
        // ---- the state: row v, columns c0 .. c0 + 63, fp32 in registers;
        // off the critical path, the f16 conversion of the v rows (two
        // chunks ahead) ----
        const int c0 = 64 * (warp >> 2);
        // chunk i's v rows -> f16 in place; tokens past the chunk's end are
        // zero (line t of each 64-v block is token t)
        auto convert_v = [&](int i) {
            wait(&B.ldV[i % NV], ph(i / NV));
            if (failed) return;
            const int len = chunk_len(i);
            uint4* tile = reinterpret_cast<uint4*>(sm + OFF_V + (i % NV) * kTileV);
#pragma unroll
            for (int it = 0; it < (int)(kTileV / 16 / kSThreads); ++it) {
                const int idx = tid + it * kSThreads;
                const int t = (idx >> 3) & 63;
                float x[8];
                unpack_bf16x8(tile[idx], x);
                if (t >= len) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) x[e] = 0.f;
                }
                st_f16x8(reinterpret_cast<unsigned char*>(tile + idx), 0, x);
            }
            umma::fence_proxy_async_smem();  // generic writes -> the MMA's operand reads
            arrive(&B.vr[i % 2]);
        };
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
            arrive(&B.sr);
        }
        convert_v(0);
        if (ni > 1) convert_v(1);
        // e^{gamma_C} of each chunk straight from the record in global memory
        // (after acquiring its ready flag), one chunk ahead.
        // The state threads wait on no barrier of the record tiles: they are
        // refilled as soon as MMA_S is done, and a thread held up by its
        // checkpoint stores could then see a barrier two phases ahead.
        auto decay_of = [&](int i) {
            if (!wait_ready(ready_flag(p, ws, slot0 + i, hv))) { failed = true; abort_flag = 1; return 0.f; }
            float d;
            asm volatile("ld.relaxed.gpu.global.f32 %0, [%1];" : "=f"(d) : "l"(rec_g(i) + REC_DECAY) : "memory");
            return d;
        };
        float decay_next = decay_of(0);
        for (int i = 0; i < ni && !failed; ++i) {
            const float decay = decay_next;
            if (i + 1 < ni) decay_next = decay_of(i + 1);
            wait(&B.mXO[i % 2], ph(i / 2));
            if (failed) break;
            umma::fence_after_sync();
            const uint32_t x0 = tl + TM_XO + (uint32_t)(i % 2) * kXO + c0;
#pragma unroll
            for (int hh = 0; hh < 64; hh += 32) {  // two 32-column halves keep fewer registers live
                float x[32];
                umma::tmem_ld32(x0 + hh, x);
                if (hh == 32) {
                    umma::fence_before_sync();
                    arrive(&B.xo[i % 2]);
                }
#pragma unroll
                for (int e = 0; e < 32; e += 2) {
                    const float2 r = __ffma2_rn(make_float2(decay, decay), make_float2(s[hh + e], s[hh + e + 1]),
                                                make_float2(x[e], x[e + 1]));
                    s[hh + e] = r.x; s[hh + e + 1] = r.y;
                }
            }
            if (i + 1 < ni) {  // MMA_S(i) has read SA: the next copy replaces it
                uint32_t h[32];
#pragma unroll
                for (int e = 0; e < 32; ++e) h[e] = pack_f16x2(s[2 * e], s[2 * e + 1]);
                umma::tmem_st32_u32(tl + TM_SA + c0 / 2, h);
                umma::fence_before_sync();
                arrive(&B.sr);
            }
            // the v rows of chunk i + 2 for MMA_V(i + 2)
            if (i + 2 < ni) convert_v(i + 2);
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
        }
        if (!failed) {  // the final state, fp32 k-last
            float* drow = p.new_state + state_off + (size_t)v * kDim + c0;
#pragma unroll
            for (int e = 0; e < 64; e += 4)
                __stcs(reinterpret_cast<float4*>(drow + e), make_float4(s[e], s[e + 1], s[e + 2], s[e + 3]));
        }
    } else if (warp < 12) {
        // ---- the outputs ----
        // Every exit from this role's loop is decided together (named barrier
        // with an or of the failures), so no output thread is left at a
        // barrier that the others have abandoned.
        const int o = tid - kOBase;
        const bool olead = o == 0;
        unsigned short* otile = reinterpret_cast<unsigned short*>(sm + OFF_O);
        for (int i = 0; i < ni; ++i) {
            const long long tc = t0 + C * (long long)i;
            const int len = chunk_len(i);
            wait(&B.mXO[i % 2], ph(i / 2));
            if (olead) umma::bulk_wait_read0();  // the previous chunk's TMA store has read the tile
            // orders that (and the previous chunk's thread stores) before the writes below
            if (::gdn::chunk::chain3::group_sync_or(kBarO, kOThreads, failed)) break;
            umma::fence_after_sync();
            {
                const uint32_t o0 = tl + TM_XO + (uint32_t)(i % 2) * kXO + 128;
#pragma unroll
                for (int hh = 0; hh < 64; hh += 32) {
                    float ov[32];
                    umma::tmem_ld32(o0 + hh, ov);
                    if (hh == 32) {
                        umma::fence_before_sync();
                        arrive(&B.xo[i % 2]);
                    }
#pragma unroll
                    for (int e = 0; e < 32; ++e)
                        otile[(hh + e) * kDim + v] = __bfloat16_as_ushort(__float2bfloat16_rn(ov[e]));
                }
            }
            umma::fence_proxy_async_smem();  // the staged rows -> the TMA store
            if (::gdn::chunk::chain3::group_sync_or(kBarO, kOThreads, failed)) break;
            if (len == C) {
                // a full chunk: one tensor store of its 64 rows
                if (olead) tma_store_o(&tmap_o, umma::smem_u32(otile), hv, (int)tc);
            } else {
                // the sequence's last, partial chunk: the rows past its end
                // belong to the next sequence, so only rows < len are stored
#pragma unroll 1
                for (int c = o; c < C * 16; c += kOThreads) {
                    const int r = c >> 4, q = c & 15;
                    if (r < len)
                        __stcs(reinterpret_cast<uint4*>(p.out + ((size_t)(tc + r) * p.HV + hv) * kDim) + q,
                               reinterpret_cast<const uint4*>(otile + r * kDim)[q]);
                }
            }
        }
        if (olead) umma::bulk_wait_read0();  // the tile stays in shared memory until the last store has read it
    }

    // ---- exit: copies in flight land first ----
    umma::fence_before_sync();
    failed = __syncthreads_or(failed) || abort_flag;
    if (failed) {
        if (tid == 0) atomicOr(&g_device_status, kDevStatTimeout);
        if (warp == kLoaderWarp) {
            for (int i = (issuedA > NA ? issuedA - NA : 0); i < issuedA; ++i) {
                umma::mbar_wait(&B.ldA[i % NA], ph(i / NA), kWaitBudget);
                umma::mbar_wait(&B.ldE[i % NE], ph(i / NE), kWaitBudget);
            }
            for (int i = (issuedV > NV ? issuedV - NV : 0); i < issuedV; ++i)
                umma::mbar_wait(&B.ldV[i % NV], ph(i / NV), kWaitBudget);
        }
    }
    __syncthreads();
    if (warp == 0) umma::tmem_dealloc(tmem, TM_COLS);
}

}  // namespace chain
}  // namespace scan
