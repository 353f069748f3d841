// gdn_mtp.cu — pool-indexed multi-token gated-delta-rule decode for B200 (sm_100a).
//
// Serves speculative-decoding verification and pool-indexed decode: batch
// entry i advances the state held in pool slot idx[i] over T tokens.  The
// maths is the contest's MTP definition (flashinfer-python 0.6.11.post2,
// flashinfer/trace/templates/gdn.py:378-465, `_gdn_mtp_reference`) and the
// API is flashinfer's `gated_delta_rule_mtp` (flashinfer/gdn_decode.py:557-745):
//   * an index outside [0, pool_size) is padding (the -1 convention of
//     gdn_decode.py:182-193): zero output, no state read or written;
//   * optional per-token state snapshots into inter[slot, t] (gdn.py:457-460),
//     `cache_steps` >= T token slots per pool slot (gdn_decode.py:686-692),
//     or, with snap_entry, into row i * T + t of the buffer for batch entry i
//     (the row flashinfer's CuTe MTP kernel writes, gdn_kernels/
//     gdn_decode_mtp.py:645: batch-scoped, packed with stride T);
//   * optional in-kernel q/k L2 normalisation, x * rsqrt(sum(x^2) + 1e-6)
//     (`use_qk_l2norm`, gdn_decode.py:571);
//   * the pool in fp32 or in bf16 (the bf16-state decode of
//     gdn_decode.py:206-260): a bf16 state is widened on load, advanced in
//     fp32 over all T tokens and rounded to bf16 (nearest-even) once, when the
//     final state is stored;
//   * optional output slots (`output_state_indices`, gdn_decode.py:176-181):
//     the final state of entry i goes to slot out_idx[i] instead of idx[i].
//
// Per token, with the state row S[v, :] held in registers across all T tokens
// (the same row split as the single-token decode kernel: 8 lanes per 512-byte
// row, 16 values per lane):
//   sk = S.k   sq = S.q   kq = k.q
//   delta = beta * (v - g*sk);  o = scale*(g*sq + delta*kq);  S = g*S + delta*k
// The pool row is read once and written once whatever T is; each snapshot
// adds one streaming write.  Kernels here: the pool decode (T = 1), the staged
// token loop and the chunk form (T > 1); the persistent streaming kernel of
// gdn_mtp_stream.cu takes part of the T > 1 calls (see gdn_mtp_fwd).
#include <stdlib.h>
#include <string.h>

#include "gdn_mtp_common.cuh"

namespace gdn {

// ROWS_PER_CTA rows of one (batch entry, v-head) per CTA of 4 warps; the pool
// holds StateT (float or __nv_bfloat16).
// Resident CTAs per SM each instantiation is compiled for (register cap
// 65536 / (128 * n)).  The fp32 32-row kernels stream the pool at B = 64 and
// gain from one more resident CTA (more state bytes in flight): a T > 1 token
// loop 149.5 -> 141.3 us at T = 4 with 96 instead of 123 registers, the
// T = 1 kernel 47.1 -> 46.1 us with 80 instead of 92, both without spills
// of note; the other instantiations keep the occupancy their register
// counts give them (a tighter cap made the bf16 64-row decode spill and
// run slower).
template <int ROWS, typename StateT>
constexpr int mtp_min_blocks() {
    return sizeof(StateT) == 4 ? 5 : (ROWS == 64 ? 3 : ROWS == 32 ? 4 : 5);
}
template <int ROWS, typename StateT>
constexpr int pool_decode_min_blocks() {
    return sizeof(StateT) == 4 ? (ROWS == 32 ? 6 : 8) : (ROWS == 64 ? 5 : 8);
}

// ---------------------------------------------------------------------------
// Chunk form of the multi-token step.  Tokens are taken C at a time (C = 2 or
// 4); a last chunk of n < C tokens is padded with neutral tokens (k = q = v =
// 0, log gate 0, beta 0), whose delta is 0.  For a chunk that starts from the
// state S0 held in registers, with L_t the cumulative log gate of its first
// t + 1 tokens and E_t = exp(L_t), unrolling the per-token recurrence gives
//   g_t S_{t-1} k_t = E_t S0 k_t + sum_{s<t} (E_t/E_s) (k_s.k_t) delta_s
//   delta_t = beta_t (v_t - E_t S0 k_t - sum_{s<t} (E_t/E_s) (k_s.k_t) delta_s)
//   o_t     = scale (E_t S0 q_t + sum_{s<=t} (E_t/E_s) (k_s.q_t) delta_s)
// so the 2C row products S0.k_t, S0.q_t do not depend on one another: they
// are formed in one pass over the row and reduced together by one transposing
// shuffle reduction, and the only dependent work left per row is a C x C
// triangular solve on scalars.  The head-level products k_s.k_t, k_s.q_t and
// the q/k norms are the same for every row: each warp forms them once per
// chunk and turns them into a table of coefficients.  The rows are then
// advanced token by token, S_t = g_t S_{t-1} + delta_t k_t (the definition's
// own update order), which also gives the snapshots.

// A shared-memory float4 load the compiler neither merges with an earlier load
// of the same address nor moves: the key vectors are read again for the state
// update rather than kept in registers from the dot products.
__device__ __forceinline__ float4 lds4_fresh(const float4* p) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"((unsigned)__cvta_generic_to_shared(p)));
    return v;
}


template <int C>
struct MtpChunkDims {
    static constexpr int nKK = C * (C - 1) / 2;  // k_s.k_t, s < t
    static constexpr int nKQ = C * (C + 1) / 2;  // k_s.q_t, s <= t
    // head-level products: [0,C) |k_t|^2, [C,2C) |q_t|^2, then k_s.k_t, then k_s.q_t
    static constexpr int nRaw = 2 * C + nKK + nKQ;
    static constexpr int nRawSlots = nRaw <= 8 ? 8 : nRaw <= 16 ? 16 : 32;
    // coefficient table: [0,C) cA, [C,2C) cB, [2C,2C+nKK) cM, then nKQ cO,
    // then C inverse key norms, then C gates
    static constexpr int offM = 2 * C, offO = offM + nKK, offK = offO + nKQ, offG = offK + C;
    static constexpr int nTab = offG + C;
    static_assert(nRaw <= 32 && nTab <= 32, "one table entry per lane");
};

// Vectors of head-level product i: indices into [k_0 .. k_{C-1}, q_0 .. q_{C-1}],
// -1 for an unused slot.
template <int C>
__host__ __device__ constexpr int mtp_raw_vec(int i, bool second) {
    using D = MtpChunkDims<C>;
    if (i < 2 * C) return i;
    if (i < D::offO) {
        int s = i - D::offM, t = 1;
        while (s >= t) s -= t++;
        return second ? t : s;
    }
    if (i < D::offK) {
        int s = i - D::offO, t = 0;
        while (s > t) s -= ++t;
        return second ? C + t : s;
    }
    return -1;
}

template <int C, int ROWS>
struct MtpChunkShared {
    float4 kq[2 * C][kDim / 4];  // the chunk's keys then queries, widened, not normalised
    float v[C][ROWS];       // v of this CTA's rows
    float L[C], lg[C], beta[C];
    float raw[4][32];       // per warp: head-level products
    float tab[4][32];       // per warp: coefficients
};

// Transposing sum over a group of lanes: N partial values per lane, summed over
// the lanes that differ in lane bits M, M/2, ..., 1.  Each level hands half of
// the values to the partner lane and keeps the other half, so N values cost
// N - 1 shuffles (not N log N) and the lane ends with the full sum of value
// (lane & (2M - 1)) >> log2(2M / N).
template <int N, int M>
__device__ __forceinline__ float xpose_sum(float* r, int lane) {
    if constexpr (M == 0) {
        static_assert(N == 1, "more values than lanes");
        return r[0];
    } else if constexpr (N == 1) {
        r[0] += __shfl_xor_sync(0xffffffffu, r[0], M);
        return xpose_sum<1, M / 2>(r, lane);
    } else {
        constexpr int H = N / 2;
        const bool up = (lane & M) != 0;
#pragma unroll
        for (int i = 0; i < H; ++i) {
            const float give = up ? r[i] : r[i + H];
            const float keep = up ? r[i + H] : r[i];
            r[i] = keep + __shfl_xor_sync(0xffffffffu, give, M);
        }
        return xpose_sum<H, M / 2>(r, lane);
    }
}

// Coefficient j of a chunk's table (one per lane, see MtpChunkDims):
//   cA[t]    = beta_t E_t |k_t|^-1
//   cB[t]    = scale E_t |q_t|^-1
//   cM[t][s] = beta_t (E_t/E_s) k^_s.k^_t          (s < t)
//   cO[t][s] = scale (E_t/E_s) k^_s.q^_t            (s <= t)
//   |k_t|^-1 and g_t = exp(log gate)
// with |x|^-1 = rsqrt(sum x^2 + 1e-6) under in-kernel L2 normalisation, else 1.
template <int C>
__device__ __forceinline__ float mtp_coef(int j, const float* raw, const float* L, const float* lg,
                                          const float* beta, float scale, int l2) {
    using D = MtpChunkDims<C>;
    auto inv = [&](int i) { return l2 ? rsqrtf(raw[i] + 1e-6f) : 1.0f; };
    if (j < C) return beta[j] * expf(L[j]) * inv(j);
    if (j < D::offM) return scale * expf(L[j - C]) * inv(j);
    if (j < D::offO) {
        int s = j - D::offM, t = 1;
        while (s >= t) s -= t++;
        return beta[t] * expf(L[t] - L[s]) * inv(s) * inv(t) * raw[j];
    }
    if (j < D::offK) {
        int s = j - D::offO, t = 0;
        while (s > t) s -= ++t;
        return scale * expf(L[t] - L[s]) * inv(s) * inv(C + t) * raw[j];
    }
    if (j < D::offG) return inv(j - D::offK);
    return expf(lg[j - D::offG]);
}

template <int ROWS_PER_CTA, typename StateT, int C>
__global__ void __launch_bounds__(128, mtp_min_blocks<ROWS_PER_CTA, StateT>())
    gdn_mtp_chunk_kernel(const MtpParams p) {
    using D = MtpChunkDims<C>;
    constexpr int kRowsPerWarp = ROWS_PER_CTA / 4;
    constexpr int kPasses = kRowsPerWarp / 4;
    constexpr int kBlocksPerHead = kDim / ROWS_PER_CTA;
    constexpr int kRowSh = C == 4 ? 0 : 1;                                     // 8 lanes, 2C row values
    constexpr int kRawSh = D::nRawSlots == 32 ? 0 : D::nRawSlots == 16 ? 1 : 2;  // 32 lanes, nRawSlots values
    static_assert(kPasses >= 1 && kRowsPerWarp % 4 == 0, "4 rows per warp pass");
    static_assert(C == 2 || C == 4, "chunk of 2 or 4 tokens");
    __shared__ MtpChunkShared<C, ROWS_PER_CTA> sm;

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int sub = lane & 7;
    const int rsub = lane >> 3;
    const long long head = blockIdx.x / kBlocksPerHead;  // bi * HV + hv
    const int rb = blockIdx.x % kBlocksPerHead;
    const int bi = (int)(head / p.HV), hv = (int)(head % p.HV);
    const int hq = hv / p.rep;
    const int lrow = warp * kRowsPerWarp + rsub;  // this lane's first row within the CTA
    const int row_base = rb * ROWS_PER_CTA + lrow;
    const int T = p.T;

    const long long slot = mtp_index(p.idx, p.idx64, bi);
    if (slot < 0 || slot >= p.pool_size) {  // padding entry (the whole CTA)
        if (sub == 0) {
            for (int t = 0; t < T; ++t) {
                const size_t ob = (((size_t)bi * T + t) * p.HV + hv) * kDim + row_base;
#pragma unroll
                for (int ps = 0; ps < kPasses; ++ps) p.out[ob + ps * 4] = __float2bfloat16_rn(0.0f);
            }
        }
        return;
    }

    const size_t row_off = (size_t)row_base * kDim;
    const size_t sbase = ((size_t)slot * p.HV + hv) * kDim * kDim + row_off;
    const StateT* pin = static_cast<const StateT*>(p.pool_in);
    float4 s[kPasses][4];
#pragma unroll
    for (int ps = 0; ps < kPasses; ++ps) mtp_load_row(pin, sbase + (size_t)ps * 4 * kDim, sub, s[ps]);
    const long long snap_row = mtp_snap_row(p, bi, slot);
    const float A_log = p.A_log[hv], dt_bias = p.dt_bias[hv];
    const float* tab = sm.tab[warp];

    for (int c0 = 0; c0 < T; c0 += C) {
        const int n = min(C, T - c0);
        const size_t bt0 = (size_t)bi * T + c0;
        if (c0 > 0) __syncthreads();  // every warp is done with the previous chunk
        // ---- stage the chunk: q, k widened; v of this CTA's rows; gates
        for (int e = tid; e < 2 * C * 32; e += 128) {
            const int vec = e >> 5, c4 = e & 31;
            const int t = vec < C ? vec : vec - C;
            float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
            if (t < n) {
                const __nv_bfloat16* src = (vec < C ? p.k : p.q) + ((bt0 + t) * p.H + hq) * kDim + 4 * c4;
                x = mtp_widen4(*reinterpret_cast<const uint2*>(src));
            }
            sm.kq[vec][c4] = x;
        }
        for (int e = tid; e < C * ROWS_PER_CTA; e += 128) {
            const int t = e / ROWS_PER_CTA, r = e % ROWS_PER_CTA;
            sm.v[t][r] = t < n ? bf16_to_f32(p.v[((bt0 + t) * p.HV + hv) * kDim + rb * ROWS_PER_CTA + r]) : 0.f;
        }
        if (tid < C) {
            float L = 0.f, lg = 0.f, beta = 0.f;
            for (int u = 0; u <= tid && u < n; ++u) {
                lg = log_gate(A_log, bf16_to_f32(p.a[(bt0 + u) * p.HV + hv]), dt_bias);
                L += lg;
            }
            if (tid < n) beta = sigmoidf_(bf16_to_f32(p.b[(bt0 + tid) * p.HV + hv]));
            else lg = 0.f;
            sm.L[tid] = L;
            sm.lg[tid] = lg;
            sm.beta[tid] = beta;
        }
        __syncthreads();

        // ---- head-level products and the coefficient table (each warp its own copy).
        // Lane l holds elements 4l .. 4l+3 of every vector; products i and
        // i + H are formed together and folded at once by the first level
        // of the transposing sum, so only H partial values are live.
        {
            constexpr int H = D::nRawSlots / 2;
            const bool up = (lane & 16) != 0;
            float r[H];
#pragma unroll
            for (int i = 0; i < H; ++i) {
                float lo = 0.f, hi = 0.f;
                if (mtp_raw_vec<C>(i, false) >= 0)
                    lo = mtp_dot4(sm.kq[mtp_raw_vec<C>(i, false)][lane], sm.kq[mtp_raw_vec<C>(i, true)][lane]);
                if (mtp_raw_vec<C>(i + H, false) >= 0)
                    hi = mtp_dot4(sm.kq[mtp_raw_vec<C>(i + H, false)][lane], sm.kq[mtp_raw_vec<C>(i + H, true)][lane]);
                r[i] = (up ? hi : lo) + __shfl_xor_sync(0xffffffffu, up ? lo : hi, 16);
            }
            const float tot = xpose_sum<H, 8>(r, lane);
            const int rs = lane >> kRawSh;
            if ((lane & ((1 << kRawSh) - 1)) == 0 && rs < D::nRaw) sm.raw[warp][rs] = tot;
            __syncwarp();
            if (lane < D::nTab)
                sm.tab[warp][lane] = mtp_coef<C>(lane, sm.raw[warp], sm.L, sm.lg, sm.beta, p.scale, p.l2norm);
            __syncwarp();
        }

        // ---- the 2C row products against the chunk's starting state (each
        // key / query group read once for all of the lane's rows)
        float2 ak[kPasses][C], aq[kPasses][C];
#pragma unroll
        for (int ps = 0; ps < kPasses; ++ps)
#pragma unroll
            for (int t = 0; t < C; ++t) ak[ps][t] = aq[ps][t] = make_float2(0.f, 0.f);
#pragma unroll
        for (int t = 0; t < C; ++t) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int c4 = mtp_col<StateT>(sub, j) >> 2;
                const float4 kf = sm.kq[t][c4], qf = sm.kq[C + t][c4];
#pragma unroll
                for (int ps = 0; ps < kPasses; ++ps) {
                    ak[ps][t] = dot4_acc2(s[ps][j], kf, ak[ps][t]);
                    aq[ps][t] = dot4_acc2(s[ps][j], qf, aq[ps][t]);
                }
            }
        }

        // ---- per row: reduce, solve for delta, write the outputs
        float dk[kPasses][C];  // delta_t |k_t|^-1: the multiple of the raw key each token adds
        {
#pragma unroll
            for (int ps = 0; ps < kPasses; ++ps) {
                float r[2 * C];
#pragma unroll
                for (int t = 0; t < C; ++t) {
                    r[t] = ak[ps][t].x + ak[ps][t].y;
                    r[C + t] = aq[ps][t].x + aq[ps][t].y;
                }
                const float mine = xpose_sum<2 * C, 4>(r, lane);  // row value (sub >> kRowSh) in full
                const int lr = lrow + 4 * ps;
                float d[C];
#pragma unroll
                for (int t = 0; t < C; ++t) {
                    const float at = __shfl_sync(0xffffffffu, mine, (lane & ~7) | (t << kRowSh));
                    float x = sm.beta[t] * sm.v[t][lr] - tab[t] * at;
#pragma unroll
                    for (int s2 = 0; s2 < t; ++s2) x -= tab[D::offM + t * (t - 1) / 2 + s2] * d[s2];
                    d[t] = x;
                }
                // the lanes holding S0.q_t write o_t, each from its own row of cO
                const int my = (sub >> kRowSh) - C;
                if (my >= 0 && my < n && (sub & ((1 << kRowSh) - 1)) == 0) {
                    const float* co = tab + D::offO + my * (my + 1) / 2;
                    float o = tab[C + my] * mine;
#pragma unroll
                    for (int s2 = 0; s2 < C; ++s2) o += (s2 <= my ? co[s2] : 0.f) * d[s2];
                    stg_bf16(p.out + ((bt0 + my) * p.HV + hv) * kDim + row_base + 4 * ps, o);
                }
#pragma unroll
                for (int t = 0; t < C; ++t) dk[ps][t] = d[t] * tab[D::offK + t];
            }
        }

        // ---- advance the rows token by token (and take the snapshots); a
        // padding token has g = 1 and delta = 0 and leaves the rows as they are
#pragma unroll
        for (int t = 0; t < C; ++t) {
            const float g = tab[D::offG + t];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float4 kf = lds4_fresh(&sm.kq[t][mtp_col<StateT>(sub, j) >> 2]);
#pragma unroll
                for (int ps = 0; ps < kPasses; ++ps) s[ps][j] = gs_plus_dk(g, s[ps][j], dk[ps][t], kf);
            }
            if constexpr (sizeof(StateT) == 4) {  // snapshots exist for fp32 pools only
                if (snap_row >= 0 && t < n) {
                    float* dst = p.inter + (((size_t)snap_row + c0 + t) * p.HV + hv) * kDim * kDim + row_off;
#pragma unroll
                    for (int ps = 0; ps < kPasses; ++ps) mtp_store_row(dst, (size_t)ps * 4 * kDim, sub, s[ps]);
                }
            }
        }
    }

    const long long oslot = p.out_idx != nullptr ? mtp_index(p.out_idx, p.idx64, bi) : slot;
    if (p.pool_out != nullptr && oslot >= 0 && oslot < p.pool_size) {
        StateT* pout = static_cast<StateT*>(p.pool_out);
        const size_t obase = ((size_t)oslot * p.HV + hv) * kDim * kDim + row_off;
#pragma unroll
        for (int ps = 0; ps < kPasses; ++ps) mtp_store_row(pout, obase + (size_t)ps * 4 * kDim, sub, s[ps]);
    }
}

// ---------------------------------------------------------------------------
// Staged token loop (T > 1).  The per-token recurrence above, with
// everything a token contributes that does not depend on the state prepared
// once per CTA before the loop, beside the state load: q and k widened to fp32
// in shared memory (and normalised, under in-kernel L2 normalisation), k.q,
// the gate g and beta per token, and v of the CTA's rows.  The loop then reads
// only shared memory: no global-load round trip per token (under a saturated
// memory system that round trip, not the arithmetic, set the cost of each
// extra token), and no gate or norm arithmetic repeated by every lane.
// Tokens are staged kStage at a time.

constexpr int kStage = 8;

template <int ROWS>
struct MtpStageShared {
    float4 k[kStage][kDim / 4];
    float4 q[kStage][kDim / 4];
    float v[kStage][ROWS];
    float g[kStage], beta[kStage], kq[kStage];
};

template <int ROWS_PER_CTA, typename StateT>
__global__ void __launch_bounds__(128, mtp_min_blocks<ROWS_PER_CTA, StateT>())
    gdn_mtp_staged_kernel(const MtpParams p) {
    constexpr int kRowsPerWarp = ROWS_PER_CTA / 4;
    constexpr int kPasses = kRowsPerWarp / 4;
    constexpr int kBlocksPerHead = kDim / ROWS_PER_CTA;
    static_assert(kPasses >= 1 && kRowsPerWarp % 4 == 0, "4 rows per warp pass");
    __shared__ MtpStageShared<ROWS_PER_CTA> sm;

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int sub = lane & 7;
    const int rsub = lane >> 3;
    const long long head = blockIdx.x / kBlocksPerHead;  // bi * HV + hv
    const int rb = blockIdx.x % kBlocksPerHead;
    const int bi = (int)(head / p.HV), hv = (int)(head % p.HV);
    const int hq = hv / p.rep;
    const int lrow = warp * kRowsPerWarp + rsub;  // this lane's first row within the CTA
    const int row_base = rb * ROWS_PER_CTA + lrow;
    const int T = p.T;

    const long long slot = mtp_index(p.idx, p.idx64, bi);
    if (slot < 0 || slot >= p.pool_size) {  // padding entry (the whole CTA)
        if (sub == 0) {
            for (int t = 0; t < T; ++t) {
                const size_t ob = (((size_t)bi * T + t) * p.HV + hv) * kDim + row_base;
#pragma unroll
                for (int ps = 0; ps < kPasses; ++ps) p.out[ob + ps * 4] = __float2bfloat16_rn(0.0f);
            }
        }
        return;
    }

    const size_t row_off = (size_t)row_base * kDim;
    const size_t sbase = ((size_t)slot * p.HV + hv) * kDim * kDim + row_off;
    const StateT* pin = static_cast<const StateT*>(p.pool_in);
    float4 s[kPasses][4];
#pragma unroll
    for (int ps = 0; ps < kPasses; ++ps) mtp_load_row(pin, sbase + (size_t)ps * 4 * kDim, sub, s[ps]);
    const long long snap_row = mtp_snap_row(p, bi, slot);
    const bool upper = (sub & 4) != 0;

    for (int t0 = 0; t0 < T; t0 += kStage) {
        const int n = min(kStage, T - t0);
        const size_t bt0 = (size_t)bi * T + t0;
        if (t0 > 0) __syncthreads();  // every warp is done with the previous block of tokens
        for (int e = tid; e < 2 * n * 32; e += 128) {
            const int vec = e >> 5, c4 = e & 31;
            const int t = vec >> 1;
            const __nv_bfloat16* src = ((vec & 1) ? p.q : p.k) + ((bt0 + t) * p.H + hq) * kDim + 4 * c4;
            ((vec & 1) ? sm.q : sm.k)[t][c4] = mtp_widen4(*reinterpret_cast<const uint2*>(src));
        }
        for (int e = tid; e < n * ROWS_PER_CTA; e += 128) {
            const int t = e / ROWS_PER_CTA, r = e % ROWS_PER_CTA;
            sm.v[t][r] = bf16_to_f32(p.v[((bt0 + t) * p.HV + hv) * kDim + rb * ROWS_PER_CTA + r]);
        }
        if (tid < n) {
            const size_t vh = (bt0 + tid) * p.HV + hv;
            sm.g[tid] = expf(log_gate(p.A_log[hv], bf16_to_f32(p.a[vh]), p.dt_bias[hv]));
            sm.beta[tid] = sigmoidf_(bf16_to_f32(p.b[vh]));
        }
        __syncthreads();
        // one warp per token: norms, k.q (and the normalised vectors)
        for (int t = warp; t < n; t += 4) {
            float4 kv = sm.k[t][lane], qv = sm.q[t][lane];
            float kk = mtp_dot4(kv, kv), qq = mtp_dot4(qv, qv), kq = mtp_dot4(kv, qv);
#pragma unroll
            for (int m = 16; m >= 1; m >>= 1) {
                kk += __shfl_xor_sync(0xffffffffu, kk, m);
                qq += __shfl_xor_sync(0xffffffffu, qq, m);
                kq += __shfl_xor_sync(0xffffffffu, kq, m);
            }
            if (p.l2norm) {
                const float ik = rsqrtf(kk + 1e-6f), iq = rsqrtf(qq + 1e-6f);
                sm.k[t][lane] = make_float4(kv.x * ik, kv.y * ik, kv.z * ik, kv.w * ik);
                sm.q[t][lane] = make_float4(qv.x * iq, qv.y * iq, qv.z * iq, qv.w * iq);
                kq *= ik * iq;
            }
            if (lane == 0) sm.kq[t] = kq;
        }
        __syncthreads();

        for (int t = 0; t < n; ++t) {
            const float g = sm.g[t], beta = sm.beta[t], kq = sm.kq[t];
            float4 kf[4], qf[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int c4 = mtp_col<StateT>(sub, j) >> 2;
                kf[j] = sm.k[t][c4];
                qf[j] = sm.q[t][c4];
            }
            const size_t ob = ((bt0 + t) * p.HV + hv) * kDim + row_base;
            float* snap_dst = snap_row >= 0
                                  ? p.inter + (((size_t)snap_row + t0 + t) * p.HV + hv) * kDim * kDim + row_off
                                  : nullptr;
#pragma unroll
            for (int ps = 0; ps < kPasses; ++ps) {
                float2 sk2 = make_float2(0.f, 0.f), sq2 = make_float2(0.f, 0.f);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    sk2 = dot4_acc2(s[ps][j], kf[j], sk2);
                    sq2 = dot4_acc2(s[ps][j], qf[j], sq2);
                }
                const float sk = sk2.x + sk2.y, sq = sq2.x + sq2.y;
                float give = upper ? sk : sq;
                float keep = upper ? sq : sk;
                keep += __shfl_xor_sync(0xffffffffu, give, 4);
                keep += __shfl_xor_sync(0xffffffffu, keep, 1);
                keep += __shfl_xor_sync(0xffffffffu, keep, 2);
                // keep == full sk on lanes sub < 4, full sq on lanes sub >= 4
                const float sk_all = __shfl_sync(0xffffffffu, keep, lane & ~4);
                const float delta = beta * (sm.v[t][lrow + 4 * ps] - g * sk_all);
                if (sub == 4) stg_bf16(p.out + ob + ps * 4, p.scale * (g * keep + delta * kq));
#pragma unroll
                for (int j = 0; j < 4; ++j) s[ps][j] = gs_plus_dk(g, s[ps][j], delta, kf[j]);
                if constexpr (sizeof(StateT) == 4) {  // snapshots exist for fp32 pools only
                    if (snap_dst != nullptr) mtp_store_row(snap_dst, (size_t)ps * 4 * kDim, sub, s[ps]);
                }
            }
        }
    }

    const long long oslot = p.out_idx != nullptr ? mtp_index(p.out_idx, p.idx64, bi) : slot;
    if (p.pool_out != nullptr && oslot >= 0 && oslot < p.pool_size) {
        StateT* pout = static_cast<StateT*>(p.pool_out);
        const size_t obase = ((size_t)oslot * p.HV + hv) * kDim * kDim + row_off;
#pragma unroll
        for (int ps = 0; ps < kPasses; ++ps) mtp_store_row(pout, obase + (size_t)ps * 4 * kDim, sub, s[ps]);
    }
}

// ---------------------------------------------------------------------------
// Single-token form (T == 1: pool-indexed decode).  Nothing carries over to a
// next token, so each lane keeps its rows as loaded (packed: bf16 stays two
// bytes per value in registers) and widens one row pass at a time.  That
// keeps the register count near the batch decode kernel's and with it the
// bytes in flight per SM, which is what bounds an HBM stream.

// Everything one token contributes to one lane (q, k still packed bf16).
template <int kPasses>
struct MtpToken {
    uint2 q[4], k[4];
    float v[kPasses];
    float a, b;
};

template <typename StateT, int kPasses>
__device__ __forceinline__ void mtp_load_token(MtpToken<kPasses>& tk, const MtpParams& p, size_t bt,
                                               int hq, int hv, int sub, int row_base) {
    const __nv_bfloat16* qh = p.q + (bt * p.H + hq) * kDim;
    const __nv_bfloat16* kh = p.k + (bt * p.H + hq) * kDim;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        tk.q[j] = *reinterpret_cast<const uint2*>(qh + mtp_col<StateT>(sub, j));
        tk.k[j] = *reinterpret_cast<const uint2*>(kh + mtp_col<StateT>(sub, j));
    }
    const size_t vh = bt * p.HV + hv;
#pragma unroll
    for (int ps = 0; ps < kPasses; ++ps) tk.v[ps] = bf16_to_f32(p.v[vh * kDim + row_base + ps * 4]);
    tk.a = bf16_to_f32(p.a[vh]);
    tk.b = bf16_to_f32(p.b[vh]);
}

template <typename StateT>
struct RowPack;
template <>
struct RowPack<float> {
    float4 w[4];
};
template <>
struct RowPack<__nv_bfloat16> {
    uint4 w[2];
};

__device__ __forceinline__ void pack_load(RowPack<float>& r, const float* base, size_t off, int sub) {
#pragma unroll
    for (int j = 0; j < 4; ++j) r.w[j] = __ldcs(reinterpret_cast<const float4*>(base + off + mtp_col<float>(sub, j)));
}
__device__ __forceinline__ void pack_load(RowPack<__nv_bfloat16>& r, const __nv_bfloat16* base, size_t off, int sub) {
#pragma unroll
    for (int p = 0; p < 2; ++p)
        r.w[p] = __ldcs(reinterpret_cast<const uint4*>(base + off + mtp_col<__nv_bfloat16>(sub, 2 * p)));
}
__device__ __forceinline__ void pack_widen(const RowPack<float>& r, float4 (&x)[4]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = r.w[j];
}
__device__ __forceinline__ void pack_widen(const RowPack<__nv_bfloat16>& r, float4 (&x)[4]) {
#pragma unroll
    for (int p = 0; p < 2; ++p) {
        x[2 * p] = mtp_widen4(make_uint2(r.w[p].x, r.w[p].y));
        x[2 * p + 1] = mtp_widen4(make_uint2(r.w[p].z, r.w[p].w));
    }
}

template <int ROWS_PER_CTA, typename StateT>
__global__ void __launch_bounds__(128, pool_decode_min_blocks<ROWS_PER_CTA, StateT>())
    gdn_pool_decode_kernel(const MtpParams p) {
    constexpr int kRowsPerWarp = ROWS_PER_CTA / 4;
    constexpr int kPasses = kRowsPerWarp / 4;
    constexpr int kBlocksPerHead = kDim / ROWS_PER_CTA;
    static_assert(kPasses >= 1 && kRowsPerWarp % 4 == 0, "4 rows per warp pass");

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sub = lane & 7;
    const int rsub = lane >> 3;
    const long long head = blockIdx.x / kBlocksPerHead;  // bi * HV + hv
    const int rb = blockIdx.x % kBlocksPerHead;
    const int bi = (int)(head / p.HV), hv = (int)(head % p.HV);
    const int hq = hv / p.rep;
    const int row_base = rb * ROWS_PER_CTA + warp * kRowsPerWarp + rsub;
    const size_t ob = (size_t)head * kDim + row_base;  // [B, 1, HV, V]

    const long long slot = mtp_index(p.idx, p.idx64, bi);
    if (slot < 0 || slot >= p.pool_size) {  // padding entry
        if (sub == 0) {
#pragma unroll
            for (int ps = 0; ps < kPasses; ++ps) p.out[ob + ps * 4] = __float2bfloat16_rn(0.0f);
        }
        return;
    }

    const size_t row_off = (size_t)row_base * kDim;
    const size_t sbase = ((size_t)slot * p.HV + hv) * kDim * kDim + row_off;
    const StateT* pin = static_cast<const StateT*>(p.pool_in);
    RowPack<StateT> rows[kPasses];
#pragma unroll
    for (int ps = 0; ps < kPasses; ++ps) pack_load(rows[ps], pin, sbase + (size_t)ps * 4 * kDim, sub);

    MtpToken<kPasses> tk;
    mtp_load_token<StateT>(tk, p, (size_t)bi, hq, hv, sub, row_base);
    float4 qf[4], kf[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        qf[j] = mtp_widen4(tk.q[j]);
        kf[j] = mtp_widen4(tk.k[j]);
    }
    const float g = expf(log_gate(p.A_log[hv], tk.a, p.dt_bias[hv]));
    const float beta = sigmoidf_(tk.b);
    if (p.l2norm) {
        float qq = 0.f, kk = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            qq += mtp_dot4(qf[j], qf[j]);
            kk += mtp_dot4(kf[j], kf[j]);
        }
        const float iq = rsqrtf(row8_sum(qq) + 1e-6f), ik = rsqrtf(row8_sum(kk) + 1e-6f);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            qf[j] = make_float4(qf[j].x * iq, qf[j].y * iq, qf[j].z * iq, qf[j].w * iq);
            kf[j] = make_float4(kf[j].x * ik, kf[j].y * ik, kf[j].z * ik, kf[j].w * ik);
        }
    }
    float kq = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) kq += mtp_dot4(kf[j], qf[j]);
    kq = row8_sum(kq);

    const long long oslot = p.out_idx != nullptr ? mtp_index(p.out_idx, p.idx64, bi) : slot;
    StateT* pout = (p.pool_out != nullptr && oslot >= 0 && oslot < p.pool_size) ? static_cast<StateT*>(p.pool_out)
                                                                                : nullptr;
    const size_t obase = ((size_t)oslot * p.HV + hv) * kDim * kDim + row_off;
    const long long snap_row = mtp_snap_row(p, bi, slot);
    float* snap_dst = snap_row >= 0 ? p.inter + ((size_t)snap_row * p.HV + hv) * kDim * kDim + row_off : nullptr;
    const bool upper = (sub & 4) != 0;
#pragma unroll
    for (int ps = 0; ps < kPasses; ++ps) {
        float4 x[4];
        pack_widen(rows[ps], x);
        float2 sk2 = make_float2(0.f, 0.f), sq2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            sk2 = dot4_acc2(x[j], kf[j], sk2);
            sq2 = dot4_acc2(x[j], qf[j], sq2);
        }
        const float sk = sk2.x + sk2.y, sq = sq2.x + sq2.y;
        float give = upper ? sk : sq;
        float keep = upper ? sq : sk;
        keep += __shfl_xor_sync(0xffffffffu, give, 4);
        keep += __shfl_xor_sync(0xffffffffu, keep, 1);
        keep += __shfl_xor_sync(0xffffffffu, keep, 2);
        const float sk_all = __shfl_sync(0xffffffffu, keep, lane & ~4);
        const float delta = beta * (tk.v[ps] - g * sk_all);
        if (sub == 4) p.out[ob + ps * 4] = __float2bfloat16_rn(p.scale * (g * keep + delta * kq));
#pragma unroll
        for (int j = 0; j < 4; ++j) x[j] = gs_plus_dk(g, x[j], delta, kf[j]);
        if constexpr (sizeof(StateT) == 4) {  // snapshots exist for fp32 pools only
            if (snap_dst != nullptr) mtp_store_row(snap_dst, (size_t)ps * 4 * kDim, sub, x);
        }
        if (pout != nullptr) mtp_store_row(pout, obase + (size_t)ps * 4 * kDim, sub, x);
    }
}

}  // namespace gdn

extern "C" int gdn_mtp_fwd(const void* q, const void* k, const void* v, const void* pool_in,
                           void* pool_out, int state_bf16, const void* indices, const void* out_indices,
                           int indices_int64, const float* A_log, const void* a, const float* dt_bias,
                           const void* b, float scale, int B, int T, int H, int HV, int K, int V,
                           int pool_size, int flags, void* out, float* intermediate, int inter_slots,
                           int cache_steps, void* stream) {
    if (B < 0 || T < 0 || H <= 0 || HV <= 0 || pool_size < 0) return GDN_ERR_INVALID;
    if ((indices_int64 != 0 && indices_int64 != 1) || (flags & ~(GDN_MTP_QK_L2NORM | GDN_MTP_SNAPSHOTS_BY_ENTRY)) ||
        (state_bf16 != 0 && state_bf16 != 1))
        return GDN_ERR_INVALID;
    if (K != gdn::kDim || V != gdn::kDim || HV % H != 0) return GDN_ERR_UNSUPPORTED;
    if (intermediate && (inter_slots < 0 || cache_steps < T || state_bf16)) return GDN_ERR_INVALID;
    const size_t elem = state_bf16 ? 2 : 4;
    const size_t head_bytes = elem * gdn::kDim * gdn::kDim;
    const size_t pool_bytes = (size_t)pool_size * HV * head_bytes;
    const bool copy_pool = pool_out != nullptr && pool_out != pool_in && pool_size > 0;
    if (copy_pool) {
        if (!pool_in) return GDN_ERR_INVALID;
        const char* i0 = static_cast<const char*>(pool_in);
        const char* o0 = static_cast<const char*>(pool_out);
        if (o0 < i0 + pool_bytes && i0 < o0 + pool_bytes) return GDN_ERR_INVALID;  // partial overlap
        if (!gdn_aligned(pool_out, 16) || !gdn_aligned(pool_in, 16)) return GDN_ERR_ALIGN;
    }
    if ((long long)B * T > 0) {
        if (!q || !k || !v || !pool_in || !indices || !A_log || !a || !dt_bias || !b || !out)
            return GDN_ERR_INVALID;
        const uintptr_t ia = indices_int64 ? 8 : 4;
        if (!gdn_aligned(q, 8) || !gdn_aligned(k, 8) || !gdn_aligned(pool_in, 16) ||
            (pool_out && !gdn_aligned(pool_out, 16)) || (intermediate && !gdn_aligned(intermediate, 16)) ||
            !gdn_aligned(v, 2) || !gdn_aligned(out, 2) || !gdn_aligned(a, 2) || !gdn_aligned(b, 2) ||
            !gdn_aligned(A_log, 4) || !gdn_aligned(dt_bias, 4) || !gdn_aligned(indices, ia) ||
            (out_indices && !gdn_aligned(out_indices, ia)))
            return GDN_ERR_ALIGN;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (copy_pool) {
        // slots no batch entry writes keep their value in the new pool
        if (cudaMemcpyAsync(pool_out, pool_in, pool_bytes, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
            return GDN_ERR_CUDA;
    }
    if ((long long)B * T == 0) return GDN_OK;
    if (scale == 0.0f) scale = 1.0f / sqrtf((float)K);

    gdn::MtpParams p;
    p.q = static_cast<const __nv_bfloat16*>(q);
    p.k = static_cast<const __nv_bfloat16*>(k);
    p.v = static_cast<const __nv_bfloat16*>(v);
    p.pool_in = pool_in;
    p.pool_out = pool_out;
    p.idx = indices;
    p.out_idx = out_indices;
    p.idx64 = indices_int64;
    p.A_log = A_log;
    p.a = static_cast<const __nv_bfloat16*>(a);
    p.dt_bias = dt_bias;
    p.b = static_cast<const __nv_bfloat16*>(b);
    p.out = static_cast<__nv_bfloat16*>(out);
    p.inter = intermediate;
    p.scale = scale;
    p.T = T;
    p.H = H;
    p.HV = HV;
    p.rep = HV / H;
    p.pool_size = pool_size;
    p.inter_slots = intermediate ? inter_slots : 0;
    p.cache_steps = cache_steps;
    p.l2norm = (flags & GDN_MTP_QK_L2NORM) != 0;
    p.snap_entry = (flags & GDN_MTP_SNAPSHOTS_BY_ENTRY) != 0;
    const long long heads = (long long)B * HV;
    const bool small = heads * (gdn::kDim / 32) < 4 * 148;
    // Kernel form.  Default, by measurement on B200 (µs at B = 64, HV = 32, L2
    // flushed): T = 1 -> the per-CTA pool decode; T > 1 with snapshots -> the
    // staged loop (the snapshot writes keep it HBM-bound); T > 1 without
    // snapshots -> the streaming kernel for fp32 pools up to T = 4 (T = 2:
    // 59.9 vs 74.8, T = 4: 72.5 vs 89.5) and bf16 pools up to T = 3 (T = 3:
    // 60.1 vs 64.5), the staged loop otherwise (its 20 warps per SM hide the
    // longer token chains better).  GDN_MTP_FORM = "stream", "staged" or
    // "chunk" forces a T > 1 form (stream falls back when the call does not
    // qualify).
    const char* form = getenv("GDN_MTP_FORM");
    const bool forced = form != nullptr && *form != 0;
    const bool stream_default = !small && intermediate == nullptr && (state_bf16 ? T <= 3 : T <= 4);
    if (T > 1 && (forced ? strcmp(form, "stream") == 0 : stream_default)) {
        const int r = gdn::launch_mtp_stream(p, B, state_bf16 != 0, st);
        if (r != 1) return r;
    }
    if (T == 1) {
        // bf16 rows are half as long: twice the rows per CTA for the same bytes in flight
        const int rows = small ? 16 : state_bf16 ? 64 : 32;
        const unsigned grid = (unsigned)(heads * (gdn::kDim / rows));
        if (state_bf16) {
            if (rows == 16) gdn::gdn_pool_decode_kernel<16, __nv_bfloat16><<<grid, 128, 0, st>>>(p);
            else gdn::gdn_pool_decode_kernel<64, __nv_bfloat16><<<grid, 128, 0, st>>>(p);
        } else {
            if (rows == 16) gdn::gdn_pool_decode_kernel<16, float><<<grid, 128, 0, st>>>(p);
            else gdn::gdn_pool_decode_kernel<32, float><<<grid, 128, 0, st>>>(p);
        }
        return gdn_launch_status();
    }
    const bool chunk = forced && strcmp(form, "chunk") == 0;
    if (state_bf16) {
        // half the bytes per row: 64 rows per CTA keep as many bytes in flight
        const bool large = heads * (gdn::kDim / 64) >= 8 * 148;
        const int rows = small ? 16 : large ? 64 : 32;
        const unsigned grid = (unsigned)(heads * (gdn::kDim / rows));
        using BF = __nv_bfloat16;
        if (chunk && T == 2) {
            if (rows == 16) gdn::gdn_mtp_chunk_kernel<16, BF, 2><<<grid, 128, 0, st>>>(p);
            else if (rows == 32) gdn::gdn_mtp_chunk_kernel<32, BF, 2><<<grid, 128, 0, st>>>(p);
            else gdn::gdn_mtp_chunk_kernel<64, BF, 2><<<grid, 128, 0, st>>>(p);
        } else if (chunk) {
            if (rows == 16) gdn::gdn_mtp_chunk_kernel<16, BF, 4><<<grid, 128, 0, st>>>(p);
            else if (rows == 32) gdn::gdn_mtp_chunk_kernel<32, BF, 4><<<grid, 128, 0, st>>>(p);
            else gdn::gdn_mtp_chunk_kernel<64, BF, 4><<<grid, 128, 0, st>>>(p);
        } else {
            if (rows == 16) gdn::gdn_mtp_staged_kernel<16, BF><<<grid, 128, 0, st>>>(p);
            else if (rows == 32) gdn::gdn_mtp_staged_kernel<32, BF><<<grid, 128, 0, st>>>(p);
            else gdn::gdn_mtp_staged_kernel<64, BF><<<grid, 128, 0, st>>>(p);
        }
    } else {
        const unsigned grid = (unsigned)(heads * (gdn::kDim / (small ? 16 : 32)));
        if (chunk && T == 2) {
            if (small) gdn::gdn_mtp_chunk_kernel<16, float, 2><<<grid, 128, 0, st>>>(p);
            else gdn::gdn_mtp_chunk_kernel<32, float, 2><<<grid, 128, 0, st>>>(p);
        } else if (chunk) {
            if (small) gdn::gdn_mtp_chunk_kernel<16, float, 4><<<grid, 128, 0, st>>>(p);
            else gdn::gdn_mtp_chunk_kernel<32, float, 4><<<grid, 128, 0, st>>>(p);
        } else {
            if (small) gdn::gdn_mtp_staged_kernel<16, float><<<grid, 128, 0, st>>>(p);
            else gdn::gdn_mtp_staged_kernel<32, float><<<grid, 128, 0, st>>>(p);
        }
    }
    return gdn_launch_status();
}
