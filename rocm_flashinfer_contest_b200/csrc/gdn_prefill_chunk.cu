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
#include <mutex>

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
constexpr uint32_t kTileG = 16384;       // G = [K ; Q]_j K_{j-1}^T f16, K-major 128 x 64

// Workspace: (floor(T/64) + N) chunk slots; per slot HV (chunk, v-head)
// records of kSlotBytes, then per slot H [K ; Q] tiles of kTileKQ, then per
// slot H cross-Gram tiles of kTileG.
__host__ __device__ inline long long ws_slots(int N, int T) { return (long long)(T / 64) + N; }
__device__ __forceinline__ unsigned char* ws_kq(const PrefillParams& p, const unsigned char* ws) {
    return const_cast<unsigned char*>(ws) + (size_t)ws_slots(p.N, p.T) * p.HV * kSlotBytes;
}
__device__ __forceinline__ unsigned char* ws_g(const PrefillParams& p, const unsigned char* ws) {
    return ws_kq(p, ws) + (size_t)ws_slots(p.N, p.T) * p.H * kTileKQ;
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

// L2-normalises row `row` of a bf16 K-major tile (`rows` rows, 128 columns)
// in place and stores it as f16: x * rsqrt(sum(x^2) + 1e-6) in fp32 (the
// rule of FLA's l2norm behind AITER's use_qk_l2norm_in_kernel,
// fla/modules/l2norm.py:42).  f16 keeps 3 more mantissa bits of the unit
// vector than bf16; every later use of the tile reads it as f16.
__device__ __forceinline__ void l2norm_row_to_f16(unsigned char* tile, uint32_t row, uint32_t rows) {
    float ss = 0.f;
#pragma unroll 4
    for (uint32_t c = 0; c < kDim; c += 8) {
        float x[8];
        unpack_bf16x8(*reinterpret_cast<const uint4*>(tile + umma::kmaj_off(row, c, rows)), x);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(x[e], x[e], ss);
    }
    const float inv = rsqrtf(ss + 1e-6f);
#pragma unroll 4
    for (uint32_t c = 0; c < kDim; c += 8) {
        const uint32_t off = umma::kmaj_off(row, c, rows);
        float x[8];
        unpack_bf16x8(*reinterpret_cast<const uint4*>(tile + off), x);
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] *= inv;
        st_f16x8(tile, off, x);
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
// A and T only live after MMA_A has consumed [K ; Q], so they take its
// 32 KiB and 2 KiB more; with the [T ; P] tile, the gate record and the gates
// a CTA holds ~52 KiB and four CTAs (and their 4 x 128 TMEM columns) fit on
// an SM.
constexpr uint32_t OFF_A = 0;                      // A fp32 [64][LDA]                 17 KiB
constexpr uint32_t OFF_T = 64 * LDA * 4;           // T fp32 [64][LDA]                 17 KiB
constexpr uint32_t OFF_TP = 2 * 64 * LDA * 4;      // [T ; P] f16 K-major 128 x 64     16 KiB
constexpr uint32_t OFF_GR = OFF_TP + kTileTP;      // gate record (kGateBytes)
constexpr uint32_t OFF_G = OFF_GR + 1056;          // gamma[64]
constexpr uint32_t OFF_BETA = OFF_G + 256;         // beta[64]
constexpr uint32_t SMEM_BYTES = OFF_BETA + 256 + 1024;  // + alignment slack
static_assert(OFF_TP % 1024 == 0 && OFF_TP >= kTileKQ, "[T ; P] tile after [K ; Q], 1 KiB aligned");
static_assert(kGateBytes <= OFF_G - OFF_GR, "gate record fits");
static_assert(4 * (SMEM_BYTES + 1024) <= 233472, "four CTAs per SM");
// The previous chunk's K rows (bf16, K-major 64 x 128) for the cross-Gram
// G_j = [K ; Q]_j K_{j-1}^T borrow the [T ; P] region, which is only written
// after G has been computed.
constexpr uint32_t OFF_KP = OFF_TP;
constexpr uint32_t TM_COLS = 128;  // columns 0-63: [K ; Q] K^T, then P'; 64-127: G

// Element (r, c) of a 64 x 64 fp32 solve matrix: rows padded to LDA floats,
// so eight consecutive rows put one float4 column on all 32 banks (the masks'
// row-per-thread stores), and so do rows r, r + 4, r + 8, r + 12 (the solve's
// four-row float4 loads); offsets stay compile-time immediates.
__device__ __forceinline__ int ix(int r, int c) { return r * LDA + c; }

// Blocked T = (I + A)^-1 for the 64 x 64 strictly lower A in sA; writes the
// diagonal and lower 16 x 16 blocks of T into sT (the upper blocks are never
// read).  Every matrix access goes through ix().
__device__ __forceinline__ void solve_T(const float* sA, float* sT, int tid) {
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
            for (int r = j + 1; r < 16; ++r) x[r] -= sA[ix(b0 + r, b0 + j)] * xj;
        }
#pragma unroll
        for (int r = 0; r < 16; ++r) sT[ix(b0 + r, b0 + lane)] = x[r];
    }
    __syncthreads();
    // Off-diagonal blocks, one column block at a time: for i > j,
    //   X_ij = sum_{k=j}^{i-1} A_ik T_kj,   T_ij = -T_ii X_ij.
    // Column blocks are independent once the diagonal inverses exist, so each
    // warp walks down its own 8 columns of one (warps 0, 3: column block 0)
    // or two (warps 1, 2: column blocks 1 and 2) column blocks; a lane holds
    // 4 rows of one column.  X_ij passes through the T_ij block itself (only
    // this warp touches these columns), so the walk needs no block-wide
    // barrier and no scratch matrix.
    const int half = (warp == 0 || warp == 1) ? 0 : 1;
    const int cc = 8 * half + (lane & 7);  // column within the column block
    const int rq = (lane >> 3) * 4;        // first of this lane's 4 rows
    const int jfirst = (warp == 0 || warp == 3) ? 0 : 1;
    const int jlast = (warp == 0 || warp == 3) ? 0 : 2;
#pragma unroll 1
    for (int j = jfirst; j <= jlast; ++j) {
        const int col = 16 * j + cc;
#pragma unroll 1
        for (int i = j + 1; i < 4; ++i) {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
            for (int k = j; k < i; ++k) {
#pragma unroll
                for (int s4 = 0; s4 < 16; s4 += 4) {
                    const float t0 = sT[ix(16 * k + s4 + 0, col)], t1 = sT[ix(16 * k + s4 + 1, col)];
                    const float t2 = sT[ix(16 * k + s4 + 2, col)], t3 = sT[ix(16 * k + s4 + 3, col)];
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const float4 x = *reinterpret_cast<const float4*>(sA + ix(16 * i + rq + r, 16 * k + s4));
                        acc[r] = fmaf(x.x, t0, fmaf(x.y, t1, fmaf(x.z, t2, fmaf(x.w, t3, acc[r]))));
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < 4; ++r) sT[ix(16 * i + rq + r, col)] = acc[r];
            __syncwarp();
            float xc[16];
#pragma unroll
            for (int s = 0; s < 16; ++s) xc[s] = sT[ix(16 * i + s, col)];
            __syncwarp();  // every lane holds its X column before T_ij replaces it
            float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int s4 = 0; s4 < 16; s4 += 4) {
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const float4 y = *reinterpret_cast<const float4*>(sT + ix(16 * i + rq + r, 16 * i + s4));
                    o[r] = fmaf(y.x, xc[s4], fmaf(y.y, xc[s4 + 1], fmaf(y.z, xc[s4 + 2], fmaf(y.w, xc[s4 + 3], o[r]))));
                }
            }
#pragma unroll
            for (int r = 0; r < 4; ++r) sT[ix(16 * i + rq + r, col)] = -o[r];
            __syncwarp();
        }
    }
    __syncthreads();
}

// MMA_P reads rows 0-63 of the K-major [T ; P] tile as an MN-major operand.
constexpr bool t_rows_are_mn_major() {
    for (uint32_t i = 0; i < 64; ++i)
        for (uint32_t j = 0; j < 64; ++j)
            if (umma::kmaj_off(i, j, 128) != umma::mnmaj_off(j, i, 64)) return false;
    return true;
}
static_assert(t_rows_are_mn_major(), "T rows of the [T ; P] tile double as the MN-major B operand");

__global__ void __launch_bounds__(NT, 4) gdn_prefill_chunk_prep_kernel(const PrefillParams p, unsigned char* ws) {
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
    // the first v-head of a q/k head publishes the chunk's [K ; Q] tile; for
    // every chunk after the first the second v-head (the first when there is
    // only one) publishes the cross-Gram tile G, so the extra work is split
    // (the previous chunk is a full one, so all its rows are valid)
    const bool publish = hv % p.rep == 0;
    const bool gram = (p.rep > 1 ? hv % p.rep == 1 : true) && p.cross_gram && j > 0;
    if (gram) {
        const uint32_t sKP = umma::smem_u32(sm + OFF_KP);
#pragma unroll
        for (int it = 0; it < C * 16 / NT; ++it) {
            const int idx = tid + it * NT, r = idx >> 4, c = idx & 15;
            cp_async16(sKP + umma::kmaj_off(r, c * 8, 64), p.k + ((size_t)(tc - C + r) * p.H + hq) * kDim + c * 8,
                       true);
        }
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
        umma::mbar_init(&mbar[0], 1);
        umma::mbar_init(&mbar[1], 1);
        umma::fence_mbar_init();
    }
    __syncthreads();
    if (warp == 1) sG[tid] = lg + sG[31];
    cp_async_wait_all();
    if (p.qk_l2norm) {
        // thread r normalises row r of [K ; Q] (and of K_{j-1}); rows past
        // the sequence are zero and stay zero
        __syncthreads();
        l2norm_row_to_f16(sm + OFF_KQ, tid, 128);
        if (gram && tid < C) l2norm_row_to_f16(sm + OFF_KP, tid, 64);
    }
    sync_for_mma();
    const uint32_t tmem = tmem_base_sh;
    const uint32_t lane_base = (uint32_t)(32 * warp) << 16;

    // MMA_A: [K ; Q] K^T (bf16, or f16 once normalised); MMA_G: [K ; Q] K_{j-1}^T
    if (tid == 0) {
        const uint32_t ID = p.qk_l2norm ? umma::idesc_f16(128, 64, 0, 0, 0, 0) : umma::idesc_f16(128, 64, 1, 1, 0, 0);
        const uint64_t dKQ = umma::desc_kmaj(sKQ, 128, 0);
#pragma unroll
        for (int k0 = 0; k0 < kDim; k0 += 16) {
            const uint64_t a = umma::desc_add(dKQ, umma::koff_kmaj(128, k0));
            umma::mma_f16(tmem, a, a, ID, k0 > 0);
        }
        if (gram) {
            const uint64_t dKP = umma::desc_kmaj(umma::smem_u32(sm + OFF_KP), 64, 0);
#pragma unroll
            for (int k0 = 0; k0 < kDim; k0 += 16)
                umma::mma_f16(tmem + 64, umma::desc_add(dKQ, umma::koff_kmaj(128, k0)),
                              umma::desc_add(dKP, umma::koff_kmaj(64, k0)), ID, k0 > 0);
        }
        umma::mma_commit(&mbar[0]);
    }
    if (!wait_mma(&mbar[0], 0)) goto done;
    umma::fence_after_sync();

    // G tile (f16, K-major 128 x 64, the layout of the chain's MMA operand):
    // thread = row (TMEM lane), 64 columns
    if (gram) {
        unsigned char* gt = ws_g(p, ws) + ((size_t)s * p.H + hq) * kTileG;
        const int row = tid;
#pragma unroll 1
        for (int c16 = 0; c16 < C; c16 += 16) {
            float d[16];
            umma::tmem_ld16(tmem + lane_base + 64 + c16, d);
            __half2 h[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) h[e] = __floats2half2_rn(d[2 * e], d[2 * e + 1]);
            *reinterpret_cast<uint4*>(gt + umma::kmaj_off(row, c16, 128)) = *reinterpret_cast<uint4*>(h);
            *reinterpret_cast<uint4*>(gt + umma::kmaj_off(row, c16 + 8, 128)) = *reinterpret_cast<uint4*>(h + 4);
        }
    }

    // the first v-head of each q/k head also publishes the chunk's [K ; Q]
    // tile for the chain kernel: the same swizzled layout, converted to f16
    if (publish) {
        uint4* dst = reinterpret_cast<uint4*>(ws_kq(p, ws) + ((size_t)s * p.H + hq) * kTileKQ);
        if (p.qk_l2norm) {  // already f16
#pragma unroll 4
            for (int idx = tid; idx < (int)(kTileKQ / 16); idx += NT)
                dst[idx] = reinterpret_cast<const uint4*>(sm + OFF_KQ)[idx];
        } else
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

    // masks: rows 0-63 -> A (fp32), rows 64-127 -> P (f16, rows 64-127 of [T ; P]).
    // Both use e^{gamma_i - gamma_j}: A = beta_i e^{..} k_i.k_j for j < i,
    // P = scale e^{..} q_i.k_j for j <= i; one code path with a per-thread
    // coefficient and column bound keeps the kernel's instruction footprint
    // small (four CTAs of this kernel run different phases on one SM).
    {
        const int i = tid & 63;
        const bool arow = tid < 64;
        const float gi = sG[i];
        const float coef = arow ? sBeta[i] : p.scale;
        const int lim = arow ? i : i + 1;  // columns jj < lim are kept
#pragma unroll 1
        for (int c16 = 0; c16 < C; c16 += 16) {
            float d[16], r[16];
            umma::tmem_ld16(tmem + lane_base + c16, d);
            // the warp's rows are 32 * (warp % 2) .. + 31: a block of
            // columns past them is all zero (warp-uniform)
            if (c16 > 32 * (warp & 1) + 31) {
#pragma unroll
                for (int e = 0; e < 16; ++e) r[e] = 0.f;
            } else {
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const int jj = c16 + e;
                    r[e] = (jj < lim) ? coef * __expf(fminf(gi - sG[jj], 0.f)) * d[e] : 0.f;
                }
            }
            if (arow) {
#pragma unroll
                for (int e = 0; e < 16; e += 4)
                    *reinterpret_cast<float4*>(sA + ix(i, c16 + e)) = make_float4(r[e], r[e + 1], r[e + 2], r[e + 3]);
            } else {
                st_f16x8(sm + OFF_TP, umma::kmaj_off(64 + i, c16, 128), r);
                st_f16x8(sm + OFF_TP, umma::kmaj_off(64 + i, c16 + 8, 128), r + 8);
            }
        }
    }
    __syncthreads();

    // T = (I + A)^-1; f16 copy: rows 0-63 of [T ; P]
    solve_T(sA, sT, tid);
    {
        const int i = tid >> 1, h = (tid & 1) * 32;  // row i, columns h..h+31
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
            // blocks above the diagonal are zero and are never stored in sT
            float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            if (((h + c) >> 4) <= (i >> 4)) {
                const float4 a = *reinterpret_cast<const float4*>(sT + ix(i, h + c));
                const float4 b = *reinterpret_cast<const float4*>(sT + ix(i, h + c + 4));
                x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
                x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
            }
            st_f16x8(sm + OFF_TP, umma::kmaj_off(i, h + c, 128), x);  // T[i][j]
        }
    }
    sync_for_mma();

    // MMA_P: [T ; P] T -> rows 64-127 = P' = P T.  The B operand is T read
    // MN-major from rows 0-63 of the same tile: for a row i < 64 the K-major
    // byte offset of (i, j) equals the MN-major offset of (mn = j, k = i)
    // with a K extent of 64, so those 8 KiB are T as a (k = i, n = j) operand.
    if (tid == 0) {
        constexpr uint32_t ID = umma::idesc_f16(128, 64, 0, 0, 0, 1);
        const uint64_t dTP = umma::desc_kmaj(umma::smem_u32(sm + OFF_TP), 128, 0);
        const uint64_t dTB = umma::desc_mnmaj(umma::smem_u32(sm + OFF_TP), C, 0);
#pragma unroll
        for (int k0 = 0; k0 < C; k0 += 16)
            umma::mma_f16(tmem, umma::desc_add(dTP, umma::koff_kmaj(128, k0)), umma::desc_add(dTB, umma::koff_mnmaj(k0)),
                          ID, k0 > 0);
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
    } else {
        // meanwhile the chunk's gate record: gamma <= 0, so every factor is
        // in (0, 1] (times scale)
        float* gr = reinterpret_cast<float*>(sm + OFF_GR);
        const float eg = expf(sG[tid]);
        gr[GR_BEG + tid] = sBeta[tid] * eg;
        gr[GR_BETA + tid] = sBeta[tid];
        gr[GR_FK + tid] = expf(fminf(sG[C - 1] - sG[tid], 0.f));
        gr[GR_FQ + tid] = p.scale * eg;
        if (tid < 4) gr[GR_DECAY + tid] = expf(sG[C - 1]);
    }
    umma::fence_proxy_async_smem();  // the tile's rows and the gate record -> the bulk copies below
    __syncthreads();

    // slot <- [T ; P'] tile as laid out in shared memory and the gate record (two bulk copies)
    {
        unsigned char* slot = ws + ((size_t)s * p.HV + hv) * kSlotBytes;
        if (tid == 0) {
            umma::bulk_s2g(slot, umma::smem_u32(sm + OFF_TP), kTileTP);
            umma::bulk_s2g(slot + kTileTP, umma::smem_u32(sm + OFF_GR), kGateBytes);
        }
    }

done:
    if (tid == 0) umma::bulk_wait_read0();  // the tile and gates stay in shared memory until copied out
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
    // byte offset of the K step at k0 from the descriptor b_desc(tile, kext, 0)
    static __host__ __device__ constexpr uint32_t b_koff(uint32_t k0) {
        return VT == 32 ? umma::koff_mnmaj64(k0) : umma::koff_mnmaj(k0);
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
    // operand descriptors, built once; every K step and buffer is a constant offset
    const uint64_t dKQ0 = umma::desc_kmaj(sKQ0, 128, 0), dKT0 = umma::desc_sw128(sKQ0, 16384u, 1024u);
    const uint64_t dTP0 = umma::desc_kmaj(sTP0, 128, 0);
    const uint64_t dSH = G::b_desc(sSH, kDim, 0), dY = G::b_desc(sY, C, 0), dDL = G::b_desc(sDL, C, 0);

    for (long long j = 0; j < nchunks; ++j) {
        const int b = (int)(j % NBUF);
        const uint32_t par = (uint32_t)(j & 1), lpar = (uint32_t)((j / NBUF) & 1);
        const long long tc = t0 + C * j;
        const int len = chunk_len(j);
        wait_local(&ldbar[b], lpar, failed);
        const float* gr = reinterpret_cast<const float*>(sm + OFF_GB + b * kGateBytes);

        // ---- MMA_1: [K ; Q] S ----
        if (tid == 0) {
            umma::fence_after_sync();
#pragma unroll
            for (int k0 = 0; k0 < kDim; k0 += 16)
                umma::mma_f16(tmem + TM_1, umma::desc_add(dKQ0, b * kTileKQ + umma::koff_kmaj(128, k0)),
                              umma::desc_add(dSH, G::b_koff(k0)), ID_S, k0 > 0);
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
#pragma unroll
                    for (int k0 = 0; k0 < C; k0 += 16)
                        umma::mma_f16(tmem + TM_2, umma::desc_add(dTP0, b * kTileTP + umma::koff_kmaj(128, k0)),
                                      umma::desc_add(dY, G::b_koff(k0)), ID_Y, k0 > 0);
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
                        umma::mma_f16(tmem + TM_3, umma::desc_add(dKT0, b * kTileKQ + umma::koff_mnmaj(k0)),
                                      umma::desc_add(dDL, G::b_koff(k0)), ID_D, k0 > 0);
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

// ============================================================================
// chain kernel, split-path form (32-wide V tiles)
// ============================================================================
// The state reaches the next chunk's products only through
//   R_{j+1} = [K;Q]_{j+1} S_{j+1} = [K;Q]_{j+1} (e^{gamma_C,j} S_j) + G_{j+1} Dt_j,
// G_{j+1} = [K;Q]_{j+1} K_j^T (published by the prep), Dt_j = Delta~ of chunk
// j.  The first term needs only S_j, so it is issued a chunk early (MMA_1a)
// and the critical path per chunk is two tensor-core round trips:
//   R_j -> Y_j -> MMA_2 = [T;P']_j Y_j -> Dt_j -> MMA_1b = G_{j+1} Dt_j -> R_{j+1}.
// The state update S_{j+1} = e^{gamma_C} S_j + K_j^T Dt_j (MMA_3 plus an FMA
// per element), the outputs and the loads run beside it.
//
// Warp roles (TMEM lane quarter = warp % 4):
//   warps 0,1,4,5   lanes 0-63, 16 columns each: Y and Dt;
//   warps 2,3,6,7   lanes 64-127, 16 columns each: the outputs;
//   warps 8-11      all lanes, 32 columns each: the state, held in registers
//                   for the whole sequence, and its f16 operand copies;
//                   thread 256 also issues the bulk copies;
//   warp 12         one thread (issuer X) issues MMA_2(j) and MMA_3(j);
//   warp 13         one thread (issuer Y) issues MMA_1a(j+1) and MMA_1b(j+1).
//                   MMAs that feed one accumulator always come from the same
//                   thread, so they reach the tensor pipe in issue order; two
//                   issuers halve the serial issue work on the critical path
//                   (about 60 cycles per M128 N32 MMA plus each wait and commit).
//                   A commit covers only its own thread's MMAs, so every
//                   reader waits on the commit of the issuer that wrote it.
// Producers hand operands to the issuers through mbarriers they arrive on.
// Every wait is bounded; a timeout raises a shared abort flag that every loop
// checks, so no thread is left waiting on a barrier that will not complete.
namespace chain2 {

constexpr int VT = 32, HALF = 16;
constexpr int NT = 448;                  // 14 warps
constexpr int kLoader = 256;             // bulk-copy issuer (state warps)
constexpr int kMma = 384;                // MMA issuer X: MMA_2 and MMA_3 (accumulators TM_2, TM_3)
constexpr int kMmaR = 416;               // MMA issuer Y: MMA_1a and MMA_1b (accumulator R)
constexpr int kSW = 128;                 // state-warp threads
constexpr int NB = 3;                    // chunk m's data in buffer m % 3
constexpr uint32_t TM_R = 0;             // R[2]: columns 0-31 / 32-63
constexpr uint32_t TM_2 = 64;            // MMA_2 results [2]: 64-95 / 96-127
constexpr uint32_t TM_3 = 128, TM_COLS = 256;
constexpr uint32_t VROW = VT * 2 + 16;
constexpr uint32_t SH_BYTES = VT * kDim * 2;
constexpr uint32_t YD_BYTES = VT * C * 2;
constexpr uint32_t OFF_KQ = 0;                          // 3 x [K ; Q]
constexpr uint32_t OFF_TP = OFF_KQ + NB * kTileKQ;      // 3 x [T ; P']
constexpr uint32_t OFF_G = OFF_TP + NB * kTileTP;       // 2 x G
constexpr uint32_t OFF_SH = OFF_G + 2 * kTileG;         // 2 x f16 e^{gamma_C} S (MN-major, 64-byte swizzle)
constexpr uint32_t OFF_Y = OFF_SH + 2 * SH_BYTES;
constexpr uint32_t OFF_DL = OFF_Y + YD_BYTES;
constexpr uint32_t OFF_RV = OFF_DL + YD_BYTES;          // 3 x v rows
constexpr uint32_t OFF_GB = OFF_RV + NB * C * VROW;     // 3 x gate records
constexpr uint32_t SMEM_BYTES = OFF_GB + NB * kGateBytes + 1024;
static_assert(SMEM_BYTES <= 232448, "dynamic shared memory limit");
static_assert(OFF_G % 1024 == 0 && OFF_SH % 1024 == 0 && OFF_Y % 1024 == 0 && OFF_DL % 1024 == 0 &&
              OFF_GB % 16 == 0, "tile alignment");

constexpr uint32_t ID_S = umma::idesc_f16(128, VT, 0, 0, 0, 1);  // K-major A x MN-major B
constexpr uint32_t ID_D = umma::idesc_f16(128, VT, 0, 0, 1, 1);  // K^T (MN-major) x Dt

__device__ __forceinline__ uint32_t b_off(uint32_t v, uint32_t k) { return umma::mnmaj64_off(v, k); }

// A descriptor advanced by `bytes` (a multiple of 16): the start address
// field is bits 0-13 of the descriptor, in 16-byte units, and no shared
// memory address carries out of it.
__device__ __forceinline__ uint64_t dadd(uint64_t d, uint32_t bytes) { return d + (bytes >> 4); }
// K offsets of the three operand forms for the K step at element k0
__host__ __device__ constexpr uint32_t koff_kmaj128(int k0) { return (k0 >> 6) * 128u * 128u + (k0 & 63) * 2u; }
__host__ __device__ constexpr uint32_t koff_mn64(int k0) { return (k0 >> 3) * 512u; }
__host__ __device__ constexpr uint32_t koff_kt(int k0) { return (k0 >> 3) * 1024u; }

__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" :: "r"(umma::smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(umma::smem_u32(bar)) : "memory");
}

struct Bars {
    uint64_t ld[NB];    // chunk data landed: 1 expect_tx arrive + 128 cp.async arrives
    uint64_t ldG[2];    // G_m landed (index (m - 1) % 2)
    uint64_t init;      // state warps: SH[0], SH[1] written (128 arrivals)
    uint64_t yr;        // lower threads: Y_j in shared memory (128 arrivals)
    uint64_t dr;        // lower threads: Dt_j in shared memory (128 arrivals)
    uint64_t od[2];     // output threads: done with R_j, MMA_2(j) (128 arrivals, index j % 2)
    uint64_t mR[2];     // R_j complete (index j % 2)
    uint64_t m1a[2];    // MMA_1a(m) complete (index m % 2)
    uint64_t m2[2];     // MMA_2(j) complete (index j % 2)
    uint64_t m3;        // MMA_3(j) complete
    uint64_t mSd;       // state warps: S_{j+1} formed, SH for MMA_1a(j + 2) written (128 arrivals)
    uint64_t fin[2];    // drain of each issuer's MMAs at exit
};

// Chunk m's [K ; Q], [T ; P'] and gates (bulk copies by the loader) and its
// v rows (cp.async by the 128 state-warp threads) into buffer m % 3.
__device__ __forceinline__ void load_chunk(const PrefillParams& p, const unsigned char* ws, unsigned char* sm,
                                           Bars& B, int buf, long long tc, int len, long long slot, int hq, int hv,
                                           int v0, int sw, bool lead) {
    if (lead) {
        umma::mbar_arrive_expect_tx(&B.ld[buf], kTileKQ + kTileTP + kGateBytes);
        const unsigned char* rec = ws + ((size_t)slot * p.HV + hv) * kSlotBytes;
        const unsigned char* kq = ws_kq(p, ws) + ((size_t)slot * p.H + hq) * kTileKQ;
        umma::bulk_g2s(umma::smem_u32(sm + OFF_KQ + buf * kTileKQ), kq, kTileKQ / 2, &B.ld[buf]);
        umma::bulk_g2s(umma::smem_u32(sm + OFF_KQ + buf * kTileKQ + kTileKQ / 2), kq + kTileKQ / 2, kTileKQ / 2,
                       &B.ld[buf]);
        umma::bulk_g2s(umma::smem_u32(sm + OFF_TP + buf * kTileTP), rec, kTileTP, &B.ld[buf]);
        umma::bulk_g2s(umma::smem_u32(sm + OFF_GB + buf * kGateBytes), rec + kTileTP, kGateBytes, &B.ld[buf]);
    }
    const uint32_t rv = umma::smem_u32(sm + OFF_RV) + buf * (C * VROW);
#pragma unroll
    for (int it = 0; it < C * (VT / 8) / kSW; ++it) {
        const int idx = sw + it * kSW, r = idx / (VT / 8), c = idx % (VT / 8);
        const bool ok = r < len;
        const size_t off = ok ? ((size_t)(tc + r) * p.HV + hv) * kDim + v0 + c * 8 : 0;
        cp_async16(rv + r * VROW + c * 16, p.v + off, ok);
    }
    cp_async_mbar_arrive_noinc(&B.ld[buf]);
}

__device__ __forceinline__ void load_g(const PrefillParams& p, const unsigned char* ws, unsigned char* sm, Bars& B,
                                       int gb, long long slot, int hq) {
    umma::mbar_arrive_expect_tx(&B.ldG[gb], kTileG);
    umma::bulk_g2s(umma::smem_u32(sm + OFF_G + gb * kTileG), ws_g(p, ws) + ((size_t)slot * p.H + hq) * kTileG,
                   kTileG, &B.ldG[gb]);
}

__device__ __forceinline__ bool wait_b(uint64_t* bar, uint32_t parity) {
    return umma::mbar_wait(bar, parity, kWaitBudget);
}
__device__ __forceinline__ uint32_t ph(long long use) { return (uint32_t)(use & 1); }

// f16 copy of scale * s (32 columns of lane `row`) into an SH tile.
__device__ __forceinline__ void store_sh(unsigned char* sm, int which, int row, float scale, const float (&s)[32]) {
#pragma unroll
    for (int c8 = 0; c8 < 32; c8 += 8) {
        float x[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = scale * s[c8 + e];
        st_f16x8(sm + OFF_SH + which * SH_BYTES, b_off(c8, row), x);
    }
}

__global__ void __launch_bounds__(NT, 1) gdn_prefill_chunk_chain2_kernel(const PrefillParams p,
                                                                       const unsigned char* ws) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ Bars B;
    __shared__ uint32_t tmem_base_sh;
    __shared__ volatile int abort_flag;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quarter = warp & 3;
    const int row = 32 * quarter + lane;  // TMEM lane of this thread
    const bool lower = warp < 8 && quarter < 2;
    const bool upper = warp < 8 && quarter >= 2;
    const bool state = warp >= 8 && warp < 12;
    const int sw = tid - 256;                          // state-warp thread index 0..127
    const int cb = warp < 8 ? HALF * (warp >> 2) : 0;  // first column of this thread
    const int vt = blockIdx.x % (kDim / VT);
    const long long nh = blockIdx.x / (kDim / VT);
    const int hv = (int)(nh % p.HV), n = (int)(nh / p.HV);
    const int hq = hv / p.rep;
    const int v0 = vt * VT;

    long long t0, t1;
    seq_bounds(p, n, t0, t1);
    if (tid < VT) zero_uncovered_outputs(p, n, t0, t1, hv, v0 + tid, true);
    const size_t state_off = ((size_t)nh * kDim + v0) * kDim;  // [n][hv][v0][0]
    if (t1 == t0) {
        for (int idx = tid; idx < VT * kDim / 4; idx += NT)
            reinterpret_cast<float4*>(p.new_state + state_off)[idx] = make_float4(0.f, 0.f, 0.f, 0.f);
        return;
    }
    const long long slot0 = t0 / C + n;
    const long long nchunks = (t1 - t0 + C - 1) / C;
    auto chunk_len = [&](long long j) { const long long r = t1 - t0 - C * j; return (int)(r < C ? r : C); };
    auto gates_of = [&](long long m) {
        return reinterpret_cast<const float*>(sm + OFF_GB + (int)(m % NB) * kGateBytes);
    };

    if (warp == 0) {
        umma::tmem_alloc(&tmem_base_sh, TM_COLS);
        umma::tmem_relinquish();
    }
    if (tid == 0) {
        for (int b = 0; b < NB; ++b) umma::mbar_init(&B.ld[b], 1 + kSW);
        for (int b = 0; b < 2; ++b) {
            umma::mbar_init(&B.ldG[b], 1);
            umma::mbar_init(&B.od[b], 128);
            umma::mbar_init(&B.mR[b], 1);
            umma::mbar_init(&B.m1a[b], 1);
            umma::mbar_init(&B.m2[b], 1);
        }
        umma::mbar_init(&B.init, kSW);
        umma::mbar_init(&B.yr, 128);
        umma::mbar_init(&B.dr, 128);
        umma::mbar_init(&B.m3, 1);
        umma::mbar_init(&B.mSd, kSW);
        umma::mbar_init(&B.fin[0], 1);
        umma::mbar_init(&B.fin[1], 1);
        umma::fence_mbar_init();
        abort_flag = 0;
    }
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = tmem_base_sh;
    const uint32_t tl = tmem + ((uint32_t)(32 * quarter) << 16);
    const bool lead = tid == kLoader;
    bool failed = false;
    long long last_ld[NB] = {-1, -1, -1}, last_g[2] = {-1, -1};  // issued loads (loader's record)
    auto fail = [&]() { failed = true; abort_flag = 1; };

    if (tid == kMma || tid == kMmaR) {
        // ---- two MMA issuers, one per accumulator group: descriptors computed
        // once, advanced by constant offsets.  tcgen05.commit covers only the
        // issuing thread's MMAs; every reader waits on the commit of the
        // issuer that wrote what it reads. ----
        const uint64_t dKQ0 = umma::desc_kmaj(umma::smem_u32(sm + OFF_KQ), 128, 0);
        const uint64_t dKT0 = umma::desc_sw128(umma::smem_u32(sm + OFF_KQ), 16384u, 1024u);
        const uint64_t dTP0 = umma::desc_kmaj(umma::smem_u32(sm + OFF_TP), 128, 0);
        const uint64_t dG0 = umma::desc_kmaj(umma::smem_u32(sm + OFF_G), 128, 0);
        const uint64_t dSH0 = umma::desc_mnmaj64(umma::smem_u32(sm + OFF_SH), 0);
        const uint64_t dY = umma::desc_mnmaj64(umma::smem_u32(sm + OFF_Y), 0);
        const uint64_t dDL = umma::desc_mnmaj64(umma::smem_u32(sm + OFF_DL), 0);
        const int me = tid == kMma ? 0 : 1;
        bool ok = true;
        if (me == 1) {
            auto mma_1a = [&](long long m) {  // R_m = [K ; Q]_m SH[m % 2]
                const uint64_t a = dadd(dKQ0, (uint32_t)(m % NB) * kTileKQ), bsh = dadd(dSH0, (uint32_t)(m % 2) * SH_BYTES);
                const uint32_t d = tmem + TM_R + (uint32_t)(m % 2) * VT;
#pragma unroll
                for (int k0 = 0; k0 < kDim; k0 += 16)
                    umma::mma_f16(d, dadd(a, koff_kmaj128(k0)), dadd(bsh, koff_mn64(k0)), ID_S, k0 > 0);
            };
            ok = wait_b(&B.init, 0) && wait_b(&B.ld[0], 0);
            if (ok) {
                umma::fence_after_sync();
                mma_1a(0);
                umma::mma_commit(&B.m1a[0]);
                umma::mma_commit(&B.mR[0]);
            }
            for (long long j = 0; j + 1 < nchunks && ok && !abort_flag; ++j) {
                // MMA_1a(j+1) = [K ; Q]_{j+1} (e^{gamma_C,j} S_j): S_j formed (SH written), chunk j+1
                // landed, R[(j+1) % 2] read (chunk j - 1)
                if (j >= 1) ok = wait_b(&B.mSd, ph(j - 1));
                ok = ok && wait_b(&B.ld[(j + 1) % NB], ph((j + 1) / NB));
                if (ok && j >= 1) ok = wait_b(&B.od[(j + 1) % 2], ph((j - 1) / 2));
                if (!ok) break;
                umma::fence_after_sync();
                mma_1a(j + 1);
                umma::mma_commit(&B.m1a[(j + 1) % 2]);
                // Dt_j ready: MMA_1b(j+1) = G_{j+1} Dt_j onto R_{j+1}
                ok = wait_b(&B.dr, ph(j)) && wait_b(&B.ldG[j % 2], ph(j / 2));
                if (!ok) break;
                umma::fence_after_sync();
                const uint32_t d = tmem + TM_R + (uint32_t)((j + 1) % 2) * VT;
#pragma unroll
                for (int k0 = 0; k0 < C; k0 += 16)
                    umma::mma_f16(d, dadd(dG0, (uint32_t)(j % 2) * kTileG + koff_kmaj128(k0)),
                                  dadd(dDL, koff_mn64(k0)), ID_S, true);
                umma::mma_commit(&B.mR[(j + 1) % 2]);
            }
        } else {
            for (long long j = 0; j < nchunks && ok && !abort_flag; ++j) {
                const int b = (int)(j % NB);
                // MMA_2(j) = [T ; P']_j Y_j, once Y_j is written and TM_2[j % 2] has been read (outputs of j - 2)
                ok = wait_b(&B.yr, ph(j));
                if (ok && j >= 2) ok = wait_b(&B.od[j % 2], ph((j - 2) / 2));
                if (!ok) break;
                umma::fence_after_sync();
                {
                    const uint32_t d2 = tmem + TM_2 + (uint32_t)(j % 2) * VT;
#pragma unroll
                    for (int k0 = 0; k0 < C; k0 += 16)
                        umma::mma_f16(d2, dadd(dTP0, b * kTileTP + koff_kmaj128(k0)), dadd(dY, koff_mn64(k0)), ID_S,
                                      k0 > 0);
                    umma::mma_commit(&B.m2[j % 2]);
                }
                // MMA_3(j) = K_j^T Dt_j, once Dt_j is written and TM_3 has been read (state of chunk j - 1)
                ok = wait_b(&B.dr, ph(j));
                if (ok && j >= 1) ok = wait_b(&B.mSd, ph(j - 1));
                if (!ok) break;
                umma::fence_after_sync();
#pragma unroll
                for (int k0 = 0; k0 < C; k0 += 16)
                    umma::mma_f16(tmem + TM_3, dadd(dKT0, b * kTileKQ + koff_kt(k0)), dadd(dDL, koff_mn64(k0)), ID_D,
                                  k0 > 0);
                umma::mma_commit(&B.m3);
            }
        }
        if (!ok) fail();
        // drain: every MMA issued here completes before the CTA exits
        umma::mma_commit(&B.fin[me]);
        if (!wait_b(&B.fin[me], 0)) fail();
    } else if (state) {
        // ---- state warps: S (fp32, registers) for TMEM lane `row`, 32 columns ----
        for (long long m = 0; m < NB && m < nchunks; ++m) {
            load_chunk(p, ws, sm, B, (int)m, t0 + C * m, chunk_len(m), slot0 + m, hq, hv, v0, sw, lead);
            last_ld[m] = m;
        }
        if (lead) {
            for (long long m = 1; m <= 2 && m < nchunks; ++m) {
                load_g(p, ws, sm, B, (int)((m - 1) % 2), slot0 + m, hq);
                last_g[(m - 1) % 2] = m;
            }
        }
        float sv[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) sv[e] = p.state ? p.state[state_off + (size_t)e * kDim + row] : 0.f;
        if (!wait_b(&B.ld[0], 0)) fail();
        if (!failed) {
            store_sh(sm, 0, row, 1.f, sv);                                         // MMA_1a(0): S_0
            if (nchunks > 1) store_sh(sm, 1, row, gates_of(0)[GR_DECAY], sv);    // MMA_1a(1): e^{gamma_C,0} S_0
        }
        umma::fence_proxy_async_smem();
        mbar_arrive(&B.init);

        for (long long j = 0; j < nchunks && !abort_flag; ++j) {
            const int len = chunk_len(j);
            const float* gr = gates_of(j);
            const bool more = j + 2 < nchunks;  // MMA_1a(j + 2) will read SH[j % 2]
            bool ok = wait_b(&B.ld[j % NB], ph(j / NB)) && wait_b(&B.m3, ph(j));
            if (ok) {
                umma::fence_after_sync();
                float d[32];
                umma::tmem_ld32(tl + TM_3, d);
                const float decay = gr[GR_DECAY];
#pragma unroll
                for (int e = 0; e < 32; ++e) sv[e] = fmaf(decay, sv[e], d[e]);
            }
            if (ok && more) {
                ok = wait_b(&B.m1a[j % 2], ph(j / 2)) && wait_b(&B.ld[(j + 1) % NB], ph((j + 1) / NB));
                if (ok) store_sh(sm, (int)(j % 2), row, gates_of(j + 1)[GR_DECAY], sv);
            }
            // the output threads are done with chunk j's buffer (read before
            // their arrival) before the state may move on and refill it
            ok = ok && wait_b(&B.od[j % 2], ph(j / 2));
            if (!ok) { fail(); break; }
            umma::fence_proxy_async_smem();
            umma::fence_before_sync();
            mbar_arrive(&B.mSd);
            if (p.ckpt != nullptr && len == C && (C * (j + 1)) % p.ckpt_every == 0) {
                float* cd = ckpt_dst(p, n, hv, C * (j + 1));
                if (cd != nullptr) {
#pragma unroll
                    for (int e = 0; e < 32; ++e) __stcs(cd + (size_t)(v0 + e) * kDim + row, sv[e]);
                }
            }
            // chunk j's buffers are free: chunk j + 3's data; G_{j + 3} into the
            // buffer of G_{j + 1}, consumed by MMA_1b(j + 1) before MMA_3(j)
            if (j + NB < nchunks) {
                load_chunk(p, ws, sm, B, (int)(j % NB), t0 + C * (j + NB), chunk_len(j + NB), slot0 + j + NB, hq, hv,
                           v0, sw, lead);
                last_ld[j % NB] = j + NB;
            }
            if (lead && j + 3 < nchunks) {
                // G_{j+1} (same buffer) is read by MMA_1b(j+1), which issuer Y commits to mR
                if (wait_b(&B.mR[(j + 1) % 2], ph((j + 1) / 2))) {
                    load_g(p, ws, sm, B, (int)((j + 2) % 2), slot0 + j + 3, hq);
                    last_g[(j + 2) % 2] = j + 3;
                } else {
                    fail();
                }
            }
            if (j + 1 == nchunks) {  // final state, fp32 k-last
#pragma unroll
                for (int e = 0; e < 32; ++e) __stcs(p.new_state + state_off + (size_t)e * kDim + row, sv[e]);
            }
        }
    } else if (upper) {
        // ---- output warps: O = scale e^gamma QS + P'Y for token row - 64 ----
        for (long long j = 0; j < nchunks && !abort_flag; ++j) {
            const int len = chunk_len(j);
            const long long tc = t0 + C * j;
            const float* gr = gates_of(j);
            if (!(wait_b(&B.ld[j % NB], ph(j / NB)) && wait_b(&B.mR[j % 2], ph(j / 2)) &&
                  wait_b(&B.m2[j % 2], ph(j / 2)))) { fail(); break; }
            umma::fence_after_sync();
            float qs[HALF], d[HALF];
            umma::tmem_ld16x2(tl + TM_R + (uint32_t)(j % 2) * VT + cb, tl + TM_2 + (uint32_t)(j % 2) * VT + cb, qs, d);
            const int i = row - 64;
            const float fq = gr[GR_FQ + i];
            umma::fence_before_sync();
            mbar_arrive(&B.od[j % 2]);
            if (i < len) {
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
    } else if (lower) {
        // ---- lower warps: Y_j, Dt_j ----
        for (long long j = 0; j < nchunks && !abort_flag; ++j) {
            const int b = (int)(j % NB);
            const int len = chunk_len(j);
            const float* gr = gates_of(j);
            if (!(wait_b(&B.ld[b], ph(j / NB)) && wait_b(&B.mR[j % 2], ph(j / 2)))) { fail(); break; }
            umma::fence_after_sync();
            {
                float d[HALF];
                umma::tmem_ld16(tl + TM_R + (uint32_t)(j % 2) * VT + cb, d);
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
                    st_f16x8(sm + OFF_Y, b_off(cb + c8, i), y);
                }
            }
            umma::fence_proxy_async_smem();
            umma::fence_before_sync();
            mbar_arrive(&B.yr);
            if (!wait_b(&B.m2[j % 2], ph(j / 2))) { fail(); break; }
            umma::fence_after_sync();
            {
                float d[HALF];
                umma::tmem_ld16(tl + TM_2 + (uint32_t)(j % 2) * VT + cb, d);
                const float fk = gr[GR_FK + row];
#pragma unroll
                for (int e = 0; e < HALF; ++e) d[e] *= fk;
#pragma unroll
                for (int c8 = 0; c8 < HALF; c8 += 8) st_f16x8(sm + OFF_DL, b_off(cb + c8, row), d + c8);
            }
            umma::fence_proxy_async_smem();
            umma::fence_before_sync();
            mbar_arrive(&B.dr);
        }
    }

    // ---- exit: copies in flight land first ----
    cp_async_wait_all();
    umma::fence_before_sync();
    failed = __syncthreads_or(failed) || abort_flag;
    if (failed && lead) {
        atomicOr(&g_device_status, kDevStatTimeout);
        for (int b = 0; b < NB; ++b)
            if (last_ld[b] >= 0) wait_b(&B.ld[b], ph(last_ld[b] / NB));
        for (int b = 0; b < 2; ++b)
            if (last_g[b] >= 1) wait_b(&B.ldG[b], ph((last_g[b] - 1) / 2));
    }
    __syncthreads();
    if (warp == 0) umma::tmem_dealloc(tmem, TM_COLS);
}

}  // namespace chain2
}  // namespace chunk

size_t prefill_workspace_bytes(int N, int T, int H, int HV) {
    return (size_t)chunk::ws_slots(N, T) *
           ((size_t)HV * chunk::kSlotBytes + (size_t)H * (chunk::kTileKQ + chunk::kTileG));
}

namespace {

// Launch set-up of the chunked kernels, per device: the opt-in to more than
// 48 KiB of dynamic shared memory is a property of the kernel in the context
// of the device that is current when it is set, and the SM count steers the
// choice of chain kernel.  Done once per device, with that device current,
// under std::call_once (host threads may race on the first call).
constexpr int kMaxDevices = 64;
struct ChunkLaunchSetup {
    std::once_flag once;
    cudaError_t status = cudaErrorNotReady;
    int num_sms = 0;
};
ChunkLaunchSetup g_setup[kMaxDevices];

cudaError_t chunk_setup_current_device(int& num_sms) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    ChunkLaunchSetup& s = g_setup[dev];
    std::call_once(s.once, [&]() {
        cudaError_t r = cudaFuncSetAttribute(chunk::prep::gdn_prefill_chunk_prep_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)chunk::prep::SMEM_BYTES);
        if (r == cudaSuccess)
            r = cudaFuncSetAttribute(chunk::chain::gdn_prefill_chunk_chain_kernel<64>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)chunk::chain::Cfg<64>::SMEM_BYTES);
        if (r == cudaSuccess)
            r = cudaFuncSetAttribute(chunk::chain2::gdn_prefill_chunk_chain2_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)chunk::chain2::SMEM_BYTES);
        int sms = 0;
        if (r == cudaSuccess) r = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (r == cudaSuccess && sms <= 0) r = cudaErrorInvalidValue;
        s.num_sms = sms;
        s.status = r;
    });
    num_sms = s.num_sms;
    return s.status;
}

}  // namespace

int launch_prefill_chunk(const PrefillParams& p, void* workspace, cudaStream_t st) {
    int num_sms = 0;
    if (chunk_setup_current_device(num_sms) != cudaSuccess) return GDN_ERR_CUDA;
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    const long long slots = chunk::ws_slots(p.N, p.T);
    // one chain per (sequence, v-head, V tile): 32-wide tiles on the split
    // critical path when 64-wide ones would not cover the SMs (e.g. a single
    // long sequence); that path needs the prep's cross-Gram tiles
    const long long chains64 = (long long)p.N * p.HV * (kDim / 64);
    const bool split = chains64 < num_sms;
    PrefillParams q = p;
    q.cross_gram = split ? 1 : 0;
    chunk::prep::gdn_prefill_chunk_prep_kernel<<<(unsigned)(slots * p.HV), chunk::prep::NT,
                                                 chunk::prep::SMEM_BYTES, st>>>(q, ws);
    if (split) {
        chunk::chain2::gdn_prefill_chunk_chain2_kernel<<<(unsigned)(chains64 * 2), chunk::chain2::NT,
                                                         chunk::chain2::SMEM_BYTES, st>>>(q, ws);
    } else {
        chunk::chain::gdn_prefill_chunk_chain_kernel<64><<<(unsigned)chains64, chunk::chain::NT,
                                                           chunk::chain::Cfg<64>::SMEM_BYTES, st>>>(p, ws);
    }
    return gdn_launch_status();
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
