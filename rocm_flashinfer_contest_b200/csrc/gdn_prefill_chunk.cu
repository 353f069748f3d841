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
// A prep kernel and one of two chain kernels:
//  * prep  (one CTA per (chunk, v-head), all chunks of all sequences at once):
//      the state-independent part — gates, gamma, MMA [K ; Q] K^T (bf16 as
//      given), the decay masks, T = (I + A)^-1 by a blocked solve on the CUDA
//      cores in fp32, and P' = P T on the tensor cores — and writes the f16
//      operand tile [T ; P'] (already in its shared-memory swizzled layout)
//      and the chunk's gate factors into a workspace slot; per q/k head it
//      also publishes the chunk's f16 [K ; Q] tile and the cross-Gram tile
//      G_j = [K ; Q]_j K_{j-1}^T.
//  * a chain walks the chunks of a (sequence, v-head) in order:
//        MMA_1 : [K ; Q] x S     -> KS (rows 0-63: Y = beta (V - e^gamma KS)), QS (rows 64-127)
//        MMA_2 : [T ; P'] x Y    -> Delta (rows 0-63), P'Y (rows 64-127);
//                                   O = scale e^gamma QS + P'Y
//        MMA_3 : K^T x Delta~ with Delta~ = diag(e^{gamma_C - gamma}) Delta,
//                S = e^{gamma_C} S + K^T Delta~  (= K~^T Delta)
//      with MMA_1 of the next chunk split as [K ; Q]_{j+1} (e^{gamma_C} S_j)
//      (issued early) plus G_{j+1} Delta~_j, so two tensor-core round trips
//      remain on the critical path.  The diagonal scalings of Q and K act on
//      rows of the products, so [K ; Q] is a plain f16 copy of the input rows,
//      and its K rows are byte for byte an MN-major K^T tile, which MMA_3
//      reads in place.  chain2 splits a head's V columns over four CTAs
//      (32-wide tiles; for few, long sequences); chain3 keeps a whole head in
//      one CTA, transposed so the state-side operands live in tensor memory
//      (for batches of sequences).
// Operands are f16 except in the prep MMA (bf16 inputs as given); every
// accumulation is fp32 and the state carried between chunks is fp32.
//
// Workspace slot of chunk j of sequence n: floor(cu[n] / 64) + n + j, which is
// below floor(T / 64) + N for every chunk, so the workspace holds
// (floor(T / 64) + N) * HV slots of kSlotBytes.
#include <cuda.h>
#include <stdlib.h>

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

// Row r, columns c .. c+3 of the 16 x 16 x 16 product X Y of two blocks
// (X, Y: their top-left elements in solve matrices, row stride LDA).
__device__ __forceinline__ float4 blk_product_row(const float* X, const float* Y, int r, int c) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k4 = 0; k4 < 16; k4 += 4) {
        const float4 x = *reinterpret_cast<const float4*>(X + ix(r, k4));
        const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const float4 y = *reinterpret_cast<const float4*>(Y + ix(k4 + kk, c));
            acc.x = fmaf(xs[kk], y.x, acc.x);
            acc.y = fmaf(xs[kk], y.y, acc.y);
            acc.z = fmaf(xs[kk], y.z, acc.z);
            acc.w = fmaf(xs[kk], y.w, acc.w);
        }
    }
    return acc;
}
// Lower block (i, j) number n of (1,0) (2,0) (3,0) (2,1) (3,1) (3,2).
__device__ __forceinline__ int blk_pair_i(int n) { return n < 3 ? n + 1 : (n == 3 ? 2 : 3); }
__device__ __forceinline__ int blk_pair_j(int n) { return n < 3 ? 0 : (n == 5 ? 2 : 1); }
__device__ __forceinline__ float4 f4_sub(float4 a, float4 b) {
    return make_float4(a.x - b.x, a.y - b.y, a.z - b.z, a.w - b.w);
}

// Barrier of the 128 threads that work on one solve matrix: the whole CTA
// (id 0) or the named barrier `id` of its thread group, so that the groups of
// a CTA that solve different matrices need not wait for one another.
__device__ __forceinline__ void group_bar(int id) {
    if (id == 0) __syncthreads();
    else asm volatile("bar.sync %0, 128;" ::"r"(id) : "memory");
}

// Blocked T = (I + A)^-1 for the 64 x 64 strictly lower A in sA; writes the
// diagonal and lower 16 x 16 blocks of T into sT (the upper blocks are never
// read) and leaves intermediate blocks in the lower blocks of sA (the upper
// triangle of sA, where the scan prep parks P, is not touched).  Every matrix
// access goes through ix(); tid: 0..127 within the matrix's thread group,
// bar_id: its barrier (group_bar).
__device__ __forceinline__ void solve_T(const float* sA, float* sT, int tid, int bar_id = 0) {
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
    group_bar(bar_id);
    // Off-diagonal blocks by the product form.  With E_i = (I + A_ii)^-1 (the
    // diagonal blocks just written) and M_ij = E_i A_ij (i > j),
    //   I + A = diag(I + A_ii) (I + M),   (I + M)^-1 = I - M + M^2 - M^3
    // (M is strictly block-lower with 4 blocks, so M^4 = 0).  Writing W for
    // (I + M)^-1: W_10 = -M_10, W_21 = -M_21, W_32 = -M_32,
    //   W_20 = M_21 M_10 - M_20,  W_31 = M_32 M_21 - M_31,
    //   W_30 = (M_31 M_10 - M_30) - M_32 W_20,
    // and T_ij = W_ij E_j.  Sixteen 16 x 16 x 16 products in four stages of
    // independent products (6, 3, 1, 6), each spread over all 128 threads
    // (64 per product, four outputs per thread), in place of a substitution
    // whose row blocks wait on one another.  M and W overwrite the lower
    // blocks of A, which nothing reads after the solve.
    float* sAw = const_cast<float*>(sA);
    const int half = tid >> 6, pt = tid & 63;
    const int r = pt >> 2, c = 4 * (pt & 3);  // this thread's row and first column in a product
    // stage 1: M_ij = E_i A_ij for (1,0) (2,0) | (3,0) (2,1) | (3,1) (3,2)
    {
        float4 m[3];
#pragma unroll
        for (int q = 0; q < 3; ++q) {
            const int i = blk_pair_i(2 * q + half), j = blk_pair_j(2 * q + half);
            m[q] = blk_product_row(sT + ix(16 * i, 16 * i), sA + ix(16 * i, 16 * j), r, c);
        }
        group_bar(bar_id);
#pragma unroll
        for (int q = 0; q < 3; ++q) {
            const int i = blk_pair_i(2 * q + half), j = blk_pair_j(2 * q + half);
            *reinterpret_cast<float4*>(sAw + ix(16 * i + r, 16 * j + c)) = m[q];
        }
        group_bar(bar_id);
    }
    // stage 2: W_20 = M_21 M_10 - M_20 and Q_30 = M_31 M_10 - M_30 (half 0),
    // W_31 = M_32 M_21 - M_31 (half 1)
    {
        float4 w0, w1 = make_float4(0.f, 0.f, 0.f, 0.f);
        if (half == 0) {
            w0 = blk_product_row(sA + ix(32, 16), sA + ix(16, 0), r, c);
            w1 = blk_product_row(sA + ix(48, 16), sA + ix(16, 0), r, c);
            w0 = f4_sub(w0, *reinterpret_cast<const float4*>(sA + ix(32 + r, c)));
            w1 = f4_sub(w1, *reinterpret_cast<const float4*>(sA + ix(48 + r, c)));
        } else {
            w0 = blk_product_row(sA + ix(48, 32), sA + ix(32, 16), r, c);
            w0 = f4_sub(w0, *reinterpret_cast<const float4*>(sA + ix(48 + r, 16 + c)));
        }
        group_bar(bar_id);
        if (half == 0) {
            *reinterpret_cast<float4*>(sAw + ix(32 + r, c)) = w0;
            *reinterpret_cast<float4*>(sAw + ix(48 + r, c)) = w1;
        } else {
            *reinterpret_cast<float4*>(sAw + ix(48 + r, 16 + c)) = w0;
        }
        group_bar(bar_id);
    }
    // stage 3: W_30 = Q_30 - M_32 W_20 (half 0)
    {
        float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
        if (half == 0)
            w = f4_sub(*reinterpret_cast<const float4*>(sA + ix(48 + r, c)),
                       blk_product_row(sA + ix(48, 32), sA + ix(32, 0), r, c));
        group_bar(bar_id);
        if (half == 0) *reinterpret_cast<float4*>(sAw + ix(48 + r, c)) = w;
        group_bar(bar_id);
    }
    // stage 4: T_ij = W_ij E_j (W_10, W_21, W_32 are -M): (1,0) (2,0) | (3,0) (2,1) | (3,1) (3,2)
    {
#pragma unroll
        for (int q = 0; q < 3; ++q) {
            const int i = blk_pair_i(2 * q + half), j = blk_pair_j(2 * q + half);
            float4 t = blk_product_row(sA + ix(16 * i, 16 * j), sT + ix(16 * j, 16 * j), r, c);
            if (i == j + 1) t = make_float4(-t.x, -t.y, -t.z, -t.w);
            *reinterpret_cast<float4*>(sT + ix(16 * i + r, 16 * j + c)) = t;
        }
    }
    group_bar(bar_id);
}

// MMA_P reads rows 0-63 of the K-major [T ; P] tile as an MN-major operand.
constexpr bool t_rows_are_mn_major() {
    for (uint32_t i = 0; i < 64; ++i)
        for (uint32_t j = 0; j < 64; ++j)
            if (umma::kmaj_off(i, j, 128) != umma::mnmaj_off(j, i, 64)) return false;
    return true;
}
static_assert(t_rows_are_mn_major(), "T rows of the [T ; P] tile double as the MN-major B operand");

__global__ void __launch_bounds__(NT, 4) gdn_prefill_chunk_prep_kernel(const PrefillParams p, unsigned char* ws,
                                                                      long long slot_base) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t mbar[2];
    __shared__ uint32_t tmem_base_sh;

    const int tid = threadIdx.x, warp = tid >> 5;
    const long long s = slot_base + blockIdx.x / p.HV;
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

// ============================================================================
// chain kernel, transposed form: one CTA per (sequence, v-head), all 128 v
// ============================================================================
// The chain's products are taken transposed, with the state's V index as the
// MMA's M dimension (M = 128 = all of V), so the per-step operands that come
// from the state side live in tensor memory as A operands and the chunk's
// tiles from the prep are B operands with N = 128:
//   MMA_1a(j+1): R^T  = (e^{gamma_C,j} S_j)^T [K;Q]_{j+1}^T   (A = S^T f16 in TMEM)
//   MMA_1b(j+1): R^T += Dt_j^T G_{j+1}^T                      (A = Dt^T f16 in TMEM)
//   MMA_2(j)   : [Delta | P'Y]^T = Y_j^T [T;P']_j^T           (A = Y^T f16 in TMEM)
//   MMA_3(j)   : S^T  += Dt_j^T K_j   (fp32 state accumulated in TMEM; the
//                state threads first scale it by e^{gamma_C,j})
// R^T (lane v, columns t': K S, then Q S), Y^T, Dt^T and the outputs are
// handled one state row v per thread, each token half of a chunk by its own
// warp.  Each chunk tile is read from shared memory once per head (against
// four times with 32-wide V tiles) and the A operands cost no shared-memory
// bandwidth, so one CTA serves a whole head: this is the chain for batches
// of sequences, where (sequence, v-head) pairs fill the SMs.  The critical
// path per chunk is two tensor-core round trips
// (R -> Y -> MMA_2 -> Dt -> MMA_1b -> R).
//
// Warp roles (TMEM lane quarter = warp % 4, thread = state row v = 32 * quarter + lane):
//   warps 0-7    Y_j and Dt_j (tokens 0-31: warps 0-3, 32-63: warps 4-7);
//   warps 8-15   the outputs O = scale e^gamma QS + P'Y of the same token
//                halves, staged in shared memory and stored as coalesced
//                16-byte rows;
//   warps 16-19  the state: scale S by e^{gamma_C} in TMEM, its f16 A copy,
//                checkpoints and the final state;
//   warp 20      one thread issues every MMA, in one order (an accumulator is
//                only ever written by this thread, and its commits cover all
//                earlier MMAs);
//   warp 21      bulk copies of the chunk tiles and gates, a tensor copy of the v rows.
// (Folding the state work into the output warps, 18 warps at 96 registers,
// measured 2-7 % slower: the state path then waits for the outputs.)
namespace chain3 {

constexpr int NT = 704;                  // 22 warps
constexpr int kYThreads = 256, kOThreads = 256, kSThreads = 128;
constexpr int kOBase = 256;
constexpr int kIssuer = 640;             // warp 20, lane 0
constexpr int kLoaderWarp = 21;
constexpr int NA = 3;                    // [K;Q] and gate buffers (chunk i in i % 3)
constexpr int NB = 2;                    // [T;P'], G and v-row buffers (chunk i in i % 2)
constexpr uint32_t TM_R = 0, TM_D2 = 128, TM_S = 256, TM_SA = 384, TM_YA = 448, TM_DA = 480;
constexpr uint32_t TM_COLS = 512;
constexpr uint32_t kVRow = kDim * 2;      // one token's v row, bf16
constexpr uint32_t kTileV = C * kVRow;    // 16 KiB
constexpr uint32_t OFF_KQ = 0;
constexpr uint32_t OFF_TP = OFF_KQ + NA * kTileKQ;
constexpr uint32_t OFF_G = OFF_TP + NB * kTileTP;
constexpr uint32_t OFF_V = OFF_G + NB * kTileG;
constexpr uint32_t OFF_O = OFF_V + NB * kTileV;  // a chunk's output rows, bf16 [t][v]
constexpr uint32_t OFF_GB = OFF_O + kTileV;
constexpr uint32_t SMEM_BYTES = OFF_GB + NA * kGateBytes + 1024;
static_assert(SMEM_BYTES <= 232448, "dynamic shared memory limit");
static_assert(OFF_TP % 1024 == 0 && OFF_G % 1024 == 0 && OFF_V % 1024 == 0 && OFF_O % 16 == 0 && OFF_GB % 16 == 0,
              "tile alignment");
constexpr int kBarO = 1;  // named barrier of the output warps
// one CTA of this kernel and no prep CTA fit on an SM together, so the 512
// TMEM columns are never contended
static_assert(SMEM_BYTES + prep::SMEM_BYTES > 233472, "chain CTA alone on its SM");

constexpr uint32_t ID_K = umma::idesc_f16(128, 128, 0, 0, 0, 0);  // A (TMEM) x K-major B
constexpr uint32_t ID_M = umma::idesc_f16(128, 128, 0, 0, 0, 1);  // A (TMEM) x MN-major B (K_j for MMA_3)

struct Bars {
    uint64_t ldA[NA];    // [K;Q] + gates of the chunk in buffer i % 3 landed
    uint64_t ldB[NB];    // [T;P'] + G (bulk) + v rows (tensor copy) of the chunk in buffer i % 2 landed
    uint64_t freeA[NA];  // Y, output and state threads done with the gates of buffer i % 3
    uint64_t mR[2];      // R_i complete (i % 2)
    uint64_t m2[2];      // MMA_2(i) complete
    uint64_t m3[2];      // MMA_3(i) complete
    uint64_t rc;         // Y and output threads have read R_i
    uint64_t yr;         // Y_i in TMEM
    uint64_t dr;         // Dt_i in TMEM
    uint64_t od;         // output threads have read P'Y_i
    uint64_t sr;         // state scaled and its f16 copy written, phases 0 .. chunks
    uint64_t fin;        // drain of the issuer's MMAs
};

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint64_t dadd(uint64_t d, uint32_t bytes) { return d + (bytes >> 4); }
__device__ __forceinline__ uint32_t ph(long long use) { return (uint32_t)(use & 1); }
__device__ __forceinline__ void arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(umma::smem_u32(bar)) : "memory");
}
__device__ __forceinline__ float bf16_bits_to_f32(unsigned short b) { return __uint_as_float((uint32_t)b << 16); }
// Named barrier of `count` threads that also ors their `pred`s: every
// participant gets the same answer, so a group leaves its loop together.
__device__ __forceinline__ bool group_sync_or(int id, int count, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r) : "r"((uint32_t)pred), "r"(id), "r"(count) : "memory");
    return r != 0;
}

// TMA load of one chunk's v rows: box {128 v, 1 head, 64 tokens} of the
// [T, HV, 128] bf16 tensor at (0, hv, tc) -> shared memory as [t][v]; rows at
// or past T are zero-filled, rows past the sequence are read but carry beta = 0
__device__ __forceinline__ void tma_load_v(uint32_t dst, const CUtensorMap* map, int hv, int tc, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        :: "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(hv), "r"(tc), "r"(umma::smem_u32(bar))
        : "memory");
}

__global__ void __launch_bounds__(NT, 1) gdn_prefill_chunk_chain3_kernel(const PrefillParams p,
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
    const int hq = hv / p.rep;

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
    auto gates_of = [&](int i) { return reinterpret_cast<const float*>(sm + OFF_GB + (i % NA) * kGateBytes); };

    if (warp == 0) {
        umma::tmem_alloc(&tmem_base_sh, TM_COLS);
        umma::tmem_relinquish();
    }
    if (tid == 0) {
        for (int b = 0; b < NA; ++b) {
            umma::mbar_init(&B.ldA[b], 1);
            umma::mbar_init(&B.freeA[b], kYThreads + kOThreads + kSThreads);
        }
        for (int b = 0; b < NB; ++b) umma::mbar_init(&B.ldB[b], 1);
        for (int b = 0; b < 2; ++b) {
            umma::mbar_init(&B.mR[b], 1);
            umma::mbar_init(&B.m2[b], 1);
            umma::mbar_init(&B.m3[b], 1);
        }
        umma::mbar_init(&B.rc, kYThreads + kOThreads);
        umma::mbar_init(&B.yr, kYThreads);
        umma::mbar_init(&B.dr, kYThreads);
        umma::mbar_init(&B.od, kOThreads);
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
    int issuedA = 0, issuedB = 0;  // loads issued by the loader warp (chunks 0 .. issued - 1)

    if (warp == kLoaderWarp) {
        // ---- A = [K;Q] + gates (bulk, 3 buffers); B = [T;P'] + G (bulk) + v rows (tensor copy), 2 buffers ----
        auto loadA = [&](int i) {
            const long long j = i, slot = slot0 + j;
            const int b = i % NA;
            if (lane == 0) {
                umma::mbar_arrive_expect_tx(&B.ldA[b], kTileKQ + kGateBytes);
                const unsigned char* kq = ws_kq(p, ws) + ((size_t)slot * p.H + hq) * kTileKQ;
                const unsigned char* rec = ws + ((size_t)slot * p.HV + hv) * kSlotBytes;
                umma::bulk_g2s(umma::smem_u32(sm + OFF_KQ + b * kTileKQ), kq, kTileKQ / 2, &B.ldA[b]);
                umma::bulk_g2s(umma::smem_u32(sm + OFF_KQ + b * kTileKQ + kTileKQ / 2), kq + kTileKQ / 2,
                               kTileKQ / 2, &B.ldA[b]);
                umma::bulk_g2s(umma::smem_u32(sm + OFF_GB + b * kGateBytes), rec + kTileTP, kGateBytes, &B.ldA[b]);
            }
            __syncwarp();
        };
        auto loadB = [&](int i) {
            const long long j = i, slot = slot0 + j, tc = t0 + C * j;
            const int b = i % NB;
            const bool g = i > 0;  // G_j only feeds MMA_1b(j), which the first chunk of a launch has not
            if (lane == 0) {
                umma::mbar_arrive_expect_tx(&B.ldB[b], kTileTP + (g ? kTileG : 0) + kTileV);
                const unsigned char* rec = ws + ((size_t)slot * p.HV + hv) * kSlotBytes;
                umma::bulk_g2s(umma::smem_u32(sm + OFF_TP + b * kTileTP), rec, kTileTP, &B.ldB[b]);
                if (g)
                    umma::bulk_g2s(umma::smem_u32(sm + OFF_G + b * kTileG),
                                   ws_g(p, ws) + ((size_t)slot * p.H + hq) * kTileG, kTileG, &B.ldB[b]);
                tma_load_v(umma::smem_u32(sm + OFF_V + b * kTileV), &tmap_v, hv, (int)tc, &B.ldB[b]);
            }
            __syncwarp();
        };
        for (int i = 0; i < NA && i < ni; ++i) loadA(i);
        for (int i = 0; i < NB && i < ni; ++i) loadB(i);
        issuedA = ni < NA ? ni : NA;
        issuedB = ni < NB ? ni : NB;
        for (int i = 0; i < ni && !failed; ++i) {
            if (i + NB < ni) {  // buffer of chunk i: MMA_2(i) done (after MMA_1b(i) and the Y threads' reads)
                wait(&B.m2[i % 2], ph(i / 2));
                if (failed) break;
                loadB(i + NB);
                issuedB = i + NB + 1;
            }
            if (i + NA < ni) {  // MMA_3(i) done (after MMA_1a(i)) and every thread done with the gates
                wait(&B.m3[i % 2], ph(i / 2));
                wait(&B.freeA[i % NA], ph(i / NA));
                if (failed) break;
                loadA(i + NA);
                issuedA = i + NA + 1;
            }
        }
    } else if (tid == kIssuer) {
        // ---- the MMA issuer ----
        const uint64_t dKQ0 = umma::desc_kmaj(umma::smem_u32(sm + OFF_KQ), 128, 0);
        const uint64_t dKT0 = umma::desc_sw128(umma::smem_u32(sm + OFF_KQ), 16384u, 1024u);
        const uint64_t dTP0 = umma::desc_kmaj(umma::smem_u32(sm + OFF_TP), 128, 0);
        const uint64_t dG0 = umma::desc_kmaj(umma::smem_u32(sm + OFF_G), 128, 0);
        auto mma_1a = [&](int i) {  // R^T = SA [K;Q]_i^T (overwrites R)
            const uint64_t b0 = dadd(dKQ0, (uint32_t)(i % NA) * kTileKQ);
#pragma unroll
            for (int k0 = 0; k0 < kDim; k0 += 16)
                umma::mma_f16_ts(tmem + TM_R, tmem + TM_SA + k0 / 2, dadd(b0, umma::koff_kmaj(128, k0)), ID_K,
                                 k0 > 0);
        };
        wait(&B.sr, 0);
        wait(&B.ldA[0], 0);
        if (!failed) {
            umma::fence_after_sync();
            mma_1a(0);
            umma::mma_commit(&B.mR[0]);
        }
        for (int i = 0; i < ni && !failed; ++i) {
            // MMA_2(i): [Delta | P'Y]^T = Y^T [T;P']_i^T, once Y_i is in TMEM and P'Y_{i-1} has been read
            wait(&B.yr, ph(i));
            wait(&B.ldB[i % NB], ph(i / NB));
            if (i > 0) wait(&B.od, ph(i - 1));
            if (failed) break;
            umma::fence_after_sync();
            {
                const uint64_t b0 = dadd(dTP0, (uint32_t)(i % NB) * kTileTP);
#pragma unroll
                for (int k0 = 0; k0 < C; k0 += 16)
                    umma::mma_f16_ts(tmem + TM_D2, tmem + TM_YA + k0 / 2, dadd(b0, umma::koff_kmaj(128, k0)), ID_K,
                                     k0 > 0);
                umma::mma_commit(&B.m2[i % 2]);
            }
            if (i + 1 < ni) {
                // MMA_1a(i+1) once R_i has been read and the scaled state's f16 copy is written
                wait(&B.rc, ph(i));
                wait(&B.sr, ph(i + 1));
                wait(&B.ldA[(i + 1) % NA], ph((i + 1) / NA));
                if (failed) break;
                umma::fence_after_sync();
                mma_1a(i + 1);
                // MMA_1b(i+1): R^T += Dt_i^T G_{i+1}^T
                wait(&B.dr, ph(i));
                wait(&B.ldB[(i + 1) % NB], ph((i + 1) / NB));
                if (failed) break;
                umma::fence_after_sync();
                const uint64_t b0 = dadd(dG0, (uint32_t)((i + 1) % NB) * kTileG);
#pragma unroll
                for (int k0 = 0; k0 < C; k0 += 16)
                    umma::mma_f16_ts(tmem + TM_R, tmem + TM_DA + k0 / 2, dadd(b0, umma::koff_kmaj(128, k0)), ID_K,
                                     true);
                umma::mma_commit(&B.mR[(i + 1) % 2]);
            } else {
                wait(&B.dr, ph(i));
                wait(&B.sr, ph(i + 1));
                if (failed) break;
                umma::fence_after_sync();
            }
            // MMA_3(i): S^T += Dt_i^T K_i onto the state the state threads scaled by e^{gamma_C,i}
            const uint64_t b0 = dadd(dKT0, (uint32_t)(i % NA) * kTileKQ);
#pragma unroll
            for (int k0 = 0; k0 < C; k0 += 16)
                umma::mma_f16_ts(tmem + TM_S, tmem + TM_DA + k0 / 2, dadd(b0, umma::koff_mnmaj(k0)), ID_M, true);
            umma::mma_commit(&B.m3[i % 2]);
        }
        // drain: every MMA issued here completes before the CTA exits
        umma::mma_commit(&B.fin);
        if (!umma::mbar_wait(&B.fin, 0, kWaitBudget)) failed = true;
    } else if (warp < 8) {
        // ---- Y_i = beta (V - e^gamma KS) and Dt_i = e^{gamma_C - gamma} Delta, row v, 32 tokens ----
        const int h0 = 32 * (warp >> 2);  // this warp's first token of the chunk
        for (int i = 0; i < ni && !failed; ++i) {
            wait(&B.ldA[i % NA], ph(i / NA));
            wait(&B.ldB[i % NB], ph(i / NB));
            if (failed) break;
            const float* gr = gates_of(i);
            wait(&B.mR[i % 2], ph(i / 2));
            if (failed) break;
            umma::fence_after_sync();
            {
                float ks[32];
                umma::tmem_ld32(tl + TM_R + h0, ks);
                umma::fence_before_sync();
                arrive(&B.rc);
                uint32_t y[16];
#pragma unroll
                for (int e = 0; e < 32; e += 4) {
                    const float4 be = *reinterpret_cast<const float4*>(gr + GR_BEG + h0 + e);
                    const float4 bt = *reinterpret_cast<const float4*>(gr + GR_BETA + h0 + e);
                    const unsigned short* vcol =
                        reinterpret_cast<const unsigned short*>(sm + OFF_V + (i % NB) * kTileV) + (h0 + e) * kDim + v;
                    const float2 bv01 = __fmul2_rn(make_float2(bt.x, bt.y), make_float2(bf16_bits_to_f32(vcol[0]), bf16_bits_to_f32(vcol[kDim])));
                    const float2 bv23 = __fmul2_rn(make_float2(bt.z, bt.w), make_float2(bf16_bits_to_f32(vcol[2 * kDim]), bf16_bits_to_f32(vcol[3 * kDim])));
                    const float2 y01 = __ffma2_rn(make_float2(-be.x, -be.y), make_float2(ks[e], ks[e + 1]), bv01);
                    const float2 y23 = __ffma2_rn(make_float2(-be.z, -be.w), make_float2(ks[e + 2], ks[e + 3]), bv23);
                    y[e / 2] = pack_f16x2(y01.x, y01.y);
                    y[e / 2 + 1] = pack_f16x2(y23.x, y23.y);
                }
                umma::tmem_st16_u32_nowait(tl + TM_YA + h0 / 2, y);
                umma::tmem_wait_st();
                umma::fence_before_sync();
                arrive(&B.yr);
            }
            wait(&B.m2[i % 2], ph(i / 2));
            if (failed) break;
            umma::fence_after_sync();
            {
                float dl[32];
                umma::tmem_ld32(tl + TM_D2 + h0, dl);
                uint32_t d[16];
#pragma unroll
                for (int e = 0; e < 32; e += 4) {
                    const float4 fk = *reinterpret_cast<const float4*>(gr + GR_FK + h0 + e);
                    const float2 d01 = __fmul2_rn(make_float2(fk.x, fk.y), make_float2(dl[e], dl[e + 1]));
                    const float2 d23 = __fmul2_rn(make_float2(fk.z, fk.w), make_float2(dl[e + 2], dl[e + 3]));
                    d[e / 2] = pack_f16x2(d01.x, d01.y);
                    d[e / 2 + 1] = pack_f16x2(d23.x, d23.y);
                }
                umma::tmem_st16_u32_nowait(tl + TM_DA + h0 / 2, d);
                umma::tmem_wait_st();
                umma::fence_before_sync();
                arrive(&B.dr);
                arrive(&B.freeA[i % NA]);
            }
        }
    } else if (warp < 16) {
        // ---- outputs O[t][v] = scale e^{gamma_t} QS + P'Y (32 tokens per warp): staged
        // as bf16 rows in shared memory, then written back as coalesced 16-byte stores ----
        const int h0 = 32 * ((warp - 8) >> 2);
        const int o = tid - kOBase;
        unsigned char* otile = sm + OFF_O;
        for (int i = 0; i < ni; ++i) {
            const long long j = i, tc = t0 + C * j;
            const int len = chunk_len(j);
            wait(&B.ldA[i % NA], ph(i / NA));
            wait(&B.mR[i % 2], ph(i / 2));
            float qs[32];
            if (!failed) {
                umma::fence_after_sync();
                umma::tmem_ld32(tl + TM_R + 64 + h0, qs);
                umma::fence_before_sync();
                arrive(&B.rc);
            }
            wait(&B.m2[i % 2], ph(i / 2));
            // every output thread has copied the previous chunk's rows out of the tile
            if (group_sync_or(kBarO, kOThreads, failed)) break;
            umma::fence_after_sync();
            const float* gr = gates_of(i);
            unsigned short* ocol = reinterpret_cast<unsigned short*>(otile) + h0 * kDim + v;
#pragma unroll
            for (int hh = 0; hh < 32; hh += 16) {
                float py[16];
                umma::tmem_ld16(tl + TM_D2 + 64 + h0 + hh, py);
                if (hh == 16) {
                    umma::fence_before_sync();
                    arrive(&B.od);
                }
#pragma unroll
                for (int e = 0; e < 16; e += 4) {
                    const float4 fq = *reinterpret_cast<const float4*>(gr + GR_FQ + h0 + hh + e);
                    const float2 o01 = __ffma2_rn(make_float2(fq.x, fq.y), make_float2(qs[hh + e], qs[hh + e + 1]),
                                                  make_float2(py[e], py[e + 1]));
                    const float2 o23 = __ffma2_rn(make_float2(fq.z, fq.w), make_float2(qs[hh + e + 2], qs[hh + e + 3]),
                                                  make_float2(py[e + 2], py[e + 3]));
                    ocol[(hh + e) * kDim] = __bfloat16_as_ushort(__float2bfloat16_rn(o01.x));
                    ocol[(hh + e + 1) * kDim] = __bfloat16_as_ushort(__float2bfloat16_rn(o01.y));
                    ocol[(hh + e + 2) * kDim] = __bfloat16_as_ushort(__float2bfloat16_rn(o23.x));
                    ocol[(hh + e + 3) * kDim] = __bfloat16_as_ushort(__float2bfloat16_rn(o23.y));
                }
            }
            arrive(&B.freeA[i % NA]);
            if (group_sync_or(kBarO, kOThreads, failed)) break;  // the tile holds the chunk's rows
            // 16 threads per 256-byte token row: coalesced 16-byte stores
#pragma unroll 1
            for (int c = o; c < C * 16; c += kOThreads) {
                const int r = c >> 4, q = c & 15;
                if (r < len)
                    __stcs(reinterpret_cast<uint4*>(p.out + ((size_t)(tc + r) * p.HV + hv) * kDim) + q,
                           *reinterpret_cast<const uint4*>(otile + r * kVRow + q * 16));
            }
        }
    } else if (warp < 20) {
        // ---- the state (fp32 in TMEM): scale by e^{gamma_C}, f16 A copy, checkpoints, final ----
        const float* srow = p.state ? p.state + state_off + (size_t)v * kDim : nullptr;
        float* drow = p.new_state + state_off + (size_t)v * kDim;
        auto ckpt_store = [&](long long done, int c16, const float* x) {
            float* cd = ckpt_dst(p, n, hv, done);
            if (cd != nullptr) {
#pragma unroll
                for (int e = 0; e < 16; e += 4)
                    __stcs(reinterpret_cast<float4*>(cd + (size_t)v * kDim + c16 + e), make_float4(x[e], x[e + 1], x[e + 2], x[e + 3]));
            }
        };
        wait(&B.ldA[0], 0);
        if (!failed) {
            const float decay = gates_of(0)[GR_DECAY];
            // S_0 -> TMEM (scaled by e^{gamma_C}) and its f16 copy (unscaled, for MMA_1a of the first chunk)
#pragma unroll 1
            for (int c = 0; c < kDim; c += 32) {
                float x[32];
#pragma unroll
                for (int e = 0; e < 32; e += 4) {
                    const float4 f = srow ? *reinterpret_cast<const float4*>(srow + c + e) : make_float4(0.f, 0.f, 0.f, 0.f);
                    x[e] = f.x; x[e + 1] = f.y; x[e + 2] = f.z; x[e + 3] = f.w;
                }
                uint32_t h[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) h[e] = pack_f16x2(x[2 * e], x[2 * e + 1]);
                umma::tmem_st16_u32_nowait(tl + TM_SA + c / 2, h);
#pragma unroll
                for (int e = 0; e < 32; ++e) x[e] *= decay;
                umma::tmem_st32_nowait(tl + TM_S + c, x);
            }
            umma::tmem_wait_st();
            umma::fence_before_sync();
            arrive(&B.sr);                       // phase 0
        }
        wait(&B.mR[0], 0);                       // MMA_1a of the first chunk has read the copy
        if (!failed) {
            umma::fence_after_sync();
#pragma unroll 1
            for (int c = 0; c < kDim; c += 32) {  // f16 copy of e^{gamma_C} S for MMA_1a of the next chunk
                float x[32];
                umma::tmem_ld32(tl + TM_S + c, x);
                uint32_t h[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) h[e] = pack_f16x2(x[2 * e], x[2 * e + 1]);
                umma::tmem_st16_u32_nowait(tl + TM_SA + c / 2, h);
            }
            umma::tmem_wait_st();
            umma::fence_before_sync();
            arrive(&B.sr);                       // phase 1
            arrive(&B.freeA[0]);
        }
        for (int i = 1; i < ni && !failed; ++i) {
            // MMA_3(i - 1) done: TMEM holds S_i; scale it, f16 copy for MMA_1a(i+1)
            wait(&B.m3[(i - 1) % 2], ph((i - 1) / 2));
            wait(&B.ldA[i % NA], ph(i / NA));
            if (failed) break;
            umma::fence_after_sync();
            const long long j = i;
            const bool ck = p.ckpt != nullptr && chunk_len(j - 1) == C && (C * j) % p.ckpt_every == 0;
            const float decay = gates_of(i)[GR_DECAY];
#pragma unroll 1
            for (int c = 0; c < kDim; c += 32) {
                float x[32];
                umma::tmem_ld32(tl + TM_S + c, x);
                if (ck) {
                    ckpt_store(C * j, c, x);
                    ckpt_store(C * j, c + 16, x + 16);
                }
#pragma unroll
                for (int e = 0; e < 32; ++e) x[e] *= decay;
                umma::tmem_st32_nowait(tl + TM_S + c, x);
                uint32_t h[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) h[e] = pack_f16x2(x[2 * e], x[2 * e + 1]);
                umma::tmem_st16_u32_nowait(tl + TM_SA + c / 2, h);
            }
            umma::tmem_wait_st();
            umma::fence_before_sync();
            arrive(&B.sr);                       // phase i + 1
            arrive(&B.freeA[i % NA]);
        }
        // the final state -> new_state, and its checkpoint
        wait(&B.m3[(ni - 1) % 2], ph((ni - 1) / 2));
        if (!failed) {
            umma::fence_after_sync();
            const bool ck = p.ckpt != nullptr && chunk_len(nchunks - 1) == C && (C * nchunks) % p.ckpt_every == 0;
#pragma unroll 1
            for (int c = 0; c < kDim; c += 32) {
                float x[32];
                umma::tmem_ld32(tl + TM_S + c, x);
                if (ck) {
                    ckpt_store(C * nchunks, c, x);
                    ckpt_store(C * nchunks, c + 16, x + 16);
                }
#pragma unroll
                for (int e = 0; e < 32; e += 4)
                    __stcs(reinterpret_cast<float4*>(drow + c + e), make_float4(x[e], x[e + 1], x[e + 2], x[e + 3]));
            }
        }
    }

    // ---- exit: copies in flight land first ----
    umma::fence_before_sync();
    failed = __syncthreads_or(failed) || abort_flag;
    if (failed && warp == kLoaderWarp) {
        if (lane == 0) atomicOr(&g_device_status, kDevStatTimeout);
        for (int i = (issuedA > NA ? issuedA - NA : 0); i < issuedA; ++i)
            umma::mbar_wait(&B.ldA[i % NA], ph(i / NA), kWaitBudget);
        for (int i = (issuedB > NB ? issuedB - NB : 0); i < issuedB; ++i)
            umma::mbar_wait(&B.ldB[i % NB], ph(i / NB), kWaitBudget);
    }
    __syncthreads();
    if (warp == 0) umma::tmem_dealloc(tmem, TM_COLS);
}

}  // namespace chain3

#include "gdn_prefill_scan.cuh"

}  // namespace chunk

size_t prefill_workspace_bytes_split(int N, int T, int H, int HV) {
    return (size_t)chunk::ws_slots(N, T) *
           ((size_t)HV * chunk::kSlotBytes + (size_t)H * (chunk::kTileKQ + chunk::kTileG));
}

size_t prefill_workspace_bytes(int N, int T, int H, int HV) {
    const size_t a = prefill_workspace_bytes_split(N, T, H, HV), b = chunk::scan::workspace_bytes(N, T, HV);
    return a > b ? a : b;
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
            r = cudaFuncSetAttribute(chunk::chain2::gdn_prefill_chunk_chain2_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)chunk::chain2::SMEM_BYTES);
        if (r == cudaSuccess)
            r = cudaFuncSetAttribute(chunk::chain3::gdn_prefill_chunk_chain3_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)chunk::chain3::SMEM_BYTES);
        if (r == cudaSuccess)
            r = cudaFuncSetAttribute(chunk::scan::prep::gdn_prefill_scan_prep_kernel<1>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)chunk::scan::prep::smem_bytes<1>());
        if (r == cudaSuccess)
            r = cudaFuncSetAttribute(chunk::scan::prep::gdn_prefill_scan_prep_kernel<2>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)chunk::scan::prep::smem_bytes<2>());
        if (r == cudaSuccess)
            r = cudaFuncSetAttribute(chunk::scan::chain::gdn_prefill_scan_chain_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)chunk::scan::chain::SMEM_BYTES);
        int sms = 0;
        if (r == cudaSuccess) r = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (r == cudaSuccess && sms <= 0) r = cudaErrorInvalidValue;
        s.num_sms = sms;
        s.status = r;
    });
    num_sms = s.num_sms;
    return s.status;
}

// The scan path's streams, per device: the prep runs on a low-priority
// stream and the chain on a high-priority one, both forked from the caller's
// stream and joined back into it by events; created on first use with that
// device current.  The mutex keeps one call's record / wait / launch sequence
// whole when host threads share a device.
struct ScanStreams {
    std::once_flag once;
    cudaError_t status = cudaErrorNotReady;
    cudaStream_t lo = nullptr, hi = nullptr;
    cudaEvent_t fork = nullptr, join_lo = nullptr, join_hi = nullptr;
    std::mutex mu;
};
ScanStreams g_scan_streams[kMaxDevices];

ScanStreams* scan_streams_current_device() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    ScanStreams& s = g_scan_streams[dev];
    std::call_once(s.once, [&]() {
        int least = 0, greatest = 0;
        cudaError_t r = cudaDeviceGetStreamPriorityRange(&least, &greatest);
        if (r == cudaSuccess) r = cudaStreamCreateWithPriority(&s.lo, cudaStreamNonBlocking, least);
        if (r == cudaSuccess) r = cudaStreamCreateWithPriority(&s.hi, cudaStreamNonBlocking, greatest);
        if (r == cudaSuccess) r = cudaEventCreateWithFlags(&s.fork, cudaEventDisableTiming);
        if (r == cudaSuccess) r = cudaEventCreateWithFlags(&s.join_lo, cudaEventDisableTiming);
        if (r == cudaSuccess) r = cudaEventCreateWithFlags(&s.join_hi, cudaEventDisableTiming);
        s.status = r;
    });
    return s.status == cudaSuccess ? &s : nullptr;
}

// The driver's tensor-map encoder, looked up through the runtime once, so
// the library has no link-time dependency on the driver library (it then
// also loads on machines without a GPU driver, where nothing is launched).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled_fn() {
    static std::once_flag once;
    static EncodeTiledFn fn = nullptr;
    std::call_once(once, []() {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    });
    return fn;
}

// Tensor map of the v input [T, HV, 128] bf16 for the chain's TMA loads:
// dimensions (128, HV, T), box (128, 1, 64).  Encoding is a host-side
// computation (no device call).
bool encode_v_map(const PrefillParams& p, CUtensorMap* map) {
    const EncodeTiledFn encode = encode_tiled_fn();
    if (encode == nullptr) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)kDim, (cuuint64_t)p.HV, (cuuint64_t)p.T};
    const cuuint64_t strides[2] = {(cuuint64_t)kDim * 2, (cuuint64_t)p.HV * kDim * 2};
    const cuuint32_t box[3] = {(cuuint32_t)kDim, 1u, (cuuint32_t)chunk::C};
    const cuuint32_t estr[3] = {1u, 1u, 1u};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<__nv_bfloat16*>(p.v), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The same tensor for the scan chain: box (64, 1, 64) with the 128-byte
// swizzle, so two boxes per chunk land as the MN-major operand layout (line
// t = token, 64 v per line).
bool encode_v_map_sw128(const PrefillParams& p, CUtensorMap* map) {
    const EncodeTiledFn encode = encode_tiled_fn();
    if (encode == nullptr) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)kDim, (cuuint64_t)p.HV, (cuuint64_t)p.T};
    const cuuint64_t strides[2] = {(cuuint64_t)kDim * 2, (cuuint64_t)p.HV * kDim * 2};
    const cuuint32_t box[3] = {64u, 1u, (cuuint32_t)chunk::C};
    const cuuint32_t estr[3] = {1u, 1u, 1u};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<__nv_bfloat16*>(p.v), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The output [T, HV, 128] bf16 for the scan chain's tensor stores of full
// chunks: box (128, 1, 64), no swizzle (the staged tile is [token][v]).
bool encode_o_map(const PrefillParams& p, CUtensorMap* map) {
    const EncodeTiledFn encode = encode_tiled_fn();
    if (encode == nullptr) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)kDim, (cuuint64_t)p.HV, (cuuint64_t)p.T};
    const cuuint64_t strides[2] = {(cuuint64_t)kDim * 2, (cuuint64_t)p.HV * kDim * 2};
    const cuuint32_t box[3] = {(cuuint32_t)kDim, 1u, (cuuint32_t)chunk::C};
    const cuuint32_t estr[3] = {1u, 1u, 1u};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, p.out, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

int launch_prefill_chunk(const PrefillParams& p, void* workspace, size_t workspace_bytes, cudaStream_t st,
                         bool aux_streams) {
    int num_sms = 0;
    if (chunk_setup_current_device(num_sms) != cudaSuccess) return GDN_ERR_CUDA;
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    const long long slots = chunk::ws_slots(p.N, p.T);
    // Chain kernel, by measurement on B200 (ms, CUDA events, L2 flushed):
    //  * one sequence whose chain leaves at least half of the SMs free (2 HV <=
    //    SMs): the scan chain (4), its prep running beside it on the free SMs
    //    (HV = 32: 1,024 tokens 0.062 against 0.060 for the split chain, 4,096
    //    0.156 / 0.169, 8,192 0.279 / 0.312; HV = 16, 8,192 tokens: 0.223 /
    //    0.263; HV = 8: 0.215 / 0.224);
    //  * otherwise the split-path chain (2: four 32-wide V tiles per head, one
    //    CTA per SM) when all its CTAs fit in one wave, i.e. few (sequence,
    //    v-head) pairs: four SMs share each head's per-chunk work;
    //  * otherwise the transposed chain (3), one CTA per (sequence, v-head):
    //    16 sequences of config 3 (8,184 tokens, HV = 32) 0.267 against 0.374
    //    (split) and 0.337 (scan, whose prep finishes a sequence's chunks
    //    only after the earlier sequences' and so cannot run ahead of
    //    every chain at once).
    // GDN_PREFILL_CHAIN = 2, 3 or 4 forces one of them (all compute the same
    // result within the operand rounding; the tests run every chunked case
    // through each); the scan chain needs the larger workspace layout.
    const long long pairs = (long long)p.N * p.HV;
    // the scan path's records are written with 32-byte stores: it needs its
    // layout's size and a 256-byte aligned workspace (torch's allocations are)
    const bool scan_fits = workspace_bytes >= chunk::scan::workspace_bytes(p.N, p.T, p.HV) &&
                           (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0;
    int which = (p.N == 1 && 2 * pairs <= num_sms && scan_fits) ? 4 : 4 * pairs <= num_sms ? 2 : 3;
    const char* sel = getenv("GDN_PREFILL_CHAIN");
    if (sel && sel[0] >= '2' && sel[0] <= '4' && sel[1] == '\0' && (sel[0] != '4' || scan_fits)) which = sel[0] - '0';
    if (which == 4) {
        CUtensorMap tmap_v, tmap_o;
        if (!encode_v_map_sw128(p, &tmap_v) || !encode_o_map(p, &tmap_o)) return GDN_ERR_CUDA;
        if (cudaMemsetAsync(ws + chunk::scan::records_bytes(p.N, p.T, p.HV), 0,
                            chunk::scan::flags_bytes(p.N, p.T, p.HV), st) != cudaSuccess)
            return GDN_ERR_CUDA;
        // the two v-heads of a q/k head share one prep CTA when HV / H is even
        const bool pair = p.rep % 2 == 0;
        auto prep = [&](cudaStream_t s) {
            if (pair)
                chunk::scan::prep::gdn_prefill_scan_prep_kernel<2><<<(unsigned)(slots * p.HV / 2), 256,
                                                                     chunk::scan::prep::smem_bytes<2>(), s>>>(p, ws);
            else
                chunk::scan::prep::gdn_prefill_scan_prep_kernel<1><<<(unsigned)(slots * p.HV), 128,
                                                                     chunk::scan::prep::smem_bytes<1>(), s>>>(p, ws);
        };
        auto chain = [&](cudaStream_t s) {
            chunk::scan::chain::gdn_prefill_scan_chain_kernel<<<(unsigned)pairs, chunk::scan::chain::NT,
                                                                chunk::scan::chain::SMEM_BYTES, s>>>(p, ws, tmap_v,
                                                                                                     tmap_o);
        };
        // The chain waits on each record's ready flag, so the prep may run
        // beside it.  The prep is launched first, on a low-priority stream,
        // and never waits: the results are right whether or not the two
        // kernels overlap (a profiler or CUDA_LAUNCH_BLOCKING runs them one
        // after the other).  The chain follows on a high-priority stream, so
        // its CTAs (one per SM) take the first SMs the prep's CTAs free.
        // This pays when the chain leaves at least half of the SMs to the
        // prep; otherwise, while the caller's stream is being captured into
        // a graph, and for callers that allocate nothing (no library stream
        // or event), both run in order on the caller's stream.
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(st, &cap) != cudaSuccess) return GDN_ERR_CUDA;
        ScanStreams* ss = (aux_streams && cap == cudaStreamCaptureStatusNone && 2 * pairs <= num_sms)
                              ? scan_streams_current_device() : nullptr;
        if (ss != nullptr) {
            std::lock_guard<std::mutex> lock(ss->mu);
            if (cudaEventRecord(ss->fork, st) != cudaSuccess || cudaStreamWaitEvent(ss->lo, ss->fork, 0) != cudaSuccess ||
                cudaStreamWaitEvent(ss->hi, ss->fork, 0) != cudaSuccess)
                return GDN_ERR_CUDA;
            prep(ss->lo);
            chain(ss->hi);
            if (cudaEventRecord(ss->join_lo, ss->lo) != cudaSuccess || cudaEventRecord(ss->join_hi, ss->hi) != cudaSuccess ||
                cudaStreamWaitEvent(st, ss->join_lo, 0) != cudaSuccess || cudaStreamWaitEvent(st, ss->join_hi, 0) != cudaSuccess)
                return GDN_ERR_CUDA;
        } else {
            prep(st);
            chain(st);
        }
        return gdn_launch_status();
    }
    PrefillParams q = p;
    q.cross_gram = 1;  // both chains take the next chunk's R through the cross-Gram tiles
    chunk::prep::gdn_prefill_chunk_prep_kernel<<<(unsigned)(slots * p.HV), chunk::prep::NT,
                                                 chunk::prep::SMEM_BYTES, st>>>(q, ws, 0);
    if (which == 2) {
        chunk::chain2::gdn_prefill_chunk_chain2_kernel<<<(unsigned)(pairs * (kDim / chunk::chain2::VT)),
                                                         chunk::chain2::NT, chunk::chain2::SMEM_BYTES, st>>>(q, ws);
    } else {
        CUtensorMap tmap_v;
        if (!encode_v_map(p, &tmap_v)) return GDN_ERR_CUDA;
        chunk::chain3::gdn_prefill_chunk_chain3_kernel<<<(unsigned)pairs, chunk::chain3::NT,
                                                         chunk::chain3::SMEM_BYTES, st>>>(q, ws, tmap_v);
    }
    return gdn_launch_status();
}

}  // namespace gdn

namespace gdn {
int mtp_stream_status(bool clear);  // gdn_mtp_stream.cu
}

// The status words of the prefill's and of the streaming MTP kernel's
// translation units, or-ed.
extern "C" int gdn_device_status(int clear) {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, gdn::g_device_status, sizeof(v)) != cudaSuccess) return -1;
    if (clear && v) {
        const unsigned int z = 0;
        if (cudaMemcpyToSymbol(gdn::g_device_status, &z, sizeof(z)) != cudaSuccess) return -1;
    }
    const int m = gdn::mtp_stream_status(clear != 0);
    if (m < 0) return -1;
    return (int)(v | (unsigned int)m);
}
