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
// adds one streaming write.  q/k/v/gates of token t+1 are loaded while token t
// computes, so the only exposed latency is the first state load.
#include "gdn_common.cuh"

namespace gdn {

struct MtpParams {
    const __nv_bfloat16* q;  // [B, T, H, 128]
    const __nv_bfloat16* k;
    const __nv_bfloat16* v;  // [B, T, HV, 128]
    const void* pool_in;     // [pool, HV, 128, 128] fp32 or bf16
    void* pool_out;          // nullable: final state not written
    const void* idx;         // [B] int32 or int64
    const void* out_idx;     // nullable: final state to slot idx[i]
    const float* A_log;
    const __nv_bfloat16* a;  // [B, T, HV]
    const float* dt_bias;
    const __nv_bfloat16* b;
    __nv_bfloat16* out;      // [B, T, HV, 128]
    float* inter;            // nullable: [inter_slots, cache_steps, HV, 128, 128]
    float scale;
    int T, H, HV, rep, pool_size, inter_slots, cache_steps, idx64, l2norm;
    int snap_entry;          // snapshots indexed by batch entry (row bi * T + t), not by pool slot
};

__device__ __forceinline__ float mtp_dot4(float4 x, float4 y) {
    return x.x * y.x + x.y * y.y + x.z * y.z + x.w * y.w;
}

// Column layout of a lane's 16 values of a row (4 groups of 4).  fp32 state:
// group j at columns 4*sub + 32*j (one 16-byte access per group).  bf16 state:
// groups 2p, 2p+1 at columns 8*sub + 64*p (+4), so one 16-byte access moves
// two groups and a row needs two accesses per lane.
// First snapshot row (in units of one head's V x K state times HV) of batch
// entry bi reading pool slot `slot`, or -1 when its snapshots do not fit in
// the buffer (an entry is written whole or not at all).
__device__ __forceinline__ long long mtp_snap_row(const MtpParams& p, int bi, long long slot) {
    if (p.inter == nullptr) return -1;
    if (p.snap_entry) {
        const long long r = (long long)bi * p.T;
        return r + p.T <= (long long)p.inter_slots * p.cache_steps ? r : -1;
    }
    return slot < p.inter_slots ? slot * p.cache_steps : -1;
}

template <typename StateT>
__device__ __forceinline__ int mtp_col(int sub, int j) {
    return sizeof(StateT) == 4 ? 4 * sub + 32 * j : 8 * sub + 64 * (j >> 1) + 4 * (j & 1);
}

__device__ __forceinline__ float4 mtp_widen4(uint2 raw);

// One row's 16 values for this lane (row base `off`, in elements), widened.
__device__ __forceinline__ void mtp_load_row(const float* base, size_t off, int sub, float4 (&r)[4]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) r[j] = __ldcs(reinterpret_cast<const float4*>(base + off + mtp_col<float>(sub, j)));
}
__device__ __forceinline__ void mtp_load_row(const __nv_bfloat16* base, size_t off, int sub, float4 (&r)[4]) {
#pragma unroll
    for (int p = 0; p < 2; ++p) {
        uint4 raw = __ldcs(reinterpret_cast<const uint4*>(base + off + mtp_col<__nv_bfloat16>(sub, 2 * p)));
        r[2 * p] = mtp_widen4(make_uint2(raw.x, raw.y));
        r[2 * p + 1] = mtp_widen4(make_uint2(raw.z, raw.w));
    }
}
__device__ __forceinline__ void mtp_store_row(float* base, size_t off, int sub, const float4 (&r)[4]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) __stcs(reinterpret_cast<float4*>(base + off + mtp_col<float>(sub, j)), r[j]);
}
__device__ __forceinline__ uint32_t mtp_pack2(float x, float y) {
    __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ void mtp_store_row(__nv_bfloat16* base, size_t off, int sub, const float4 (&r)[4]) {
#pragma unroll
    for (int p = 0; p < 2; ++p) {
        const float4 a = r[2 * p], b = r[2 * p + 1];
        uint4 raw = make_uint4(mtp_pack2(a.x, a.y), mtp_pack2(a.z, a.w), mtp_pack2(b.x, b.y), mtp_pack2(b.z, b.w));
        __stcs(reinterpret_cast<uint4*>(base + off + mtp_col<__nv_bfloat16>(sub, 2 * p)), raw);
    }
}

__device__ __forceinline__ long long mtp_index(const void* idx, int idx64, int i) {
    return idx64 ? static_cast<const long long*>(idx)[i] : (long long)static_cast<const int*>(idx)[i];
}

__device__ __forceinline__ float row8_sum(float x) {
    x += __shfl_xor_sync(0xffffffffu, x, 1);
    x += __shfl_xor_sync(0xffffffffu, x, 2);
    x += __shfl_xor_sync(0xffffffffu, x, 4);
    return x;
}

// Everything one token contributes to one lane (q, k still packed bf16).
template <int kPasses>
struct MtpToken {
    uint2 q[4], k[4];
    float v[kPasses];
    float a, b;
};

__device__ __forceinline__ float4 mtp_widen4(uint2 raw) {
    __nv_bfloat162 lo = *reinterpret_cast<__nv_bfloat162*>(&raw.x);
    __nv_bfloat162 hi = *reinterpret_cast<__nv_bfloat162*>(&raw.y);
    float2 x = __bfloat1622float2(lo), y = __bfloat1622float2(hi);
    return make_float4(x.x, x.y, y.x, y.y);
}

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

// ROWS_PER_CTA rows of one (batch entry, v-head) per CTA of 4 warps; the pool
// holds StateT (float or __nv_bfloat16).
// Resident CTAs per SM each instantiation is compiled for (register cap
// 65536 / (128 * n)).  The fp32 32-row kernels stream the pool at B = 64 and
// gain from one more resident CTA (more state bytes in flight): the T > 1
// kernel 149.5 -> 141.3 us at T = 4 with 96 instead of 123 registers, the
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

template <int ROWS_PER_CTA, typename StateT>
__global__ void __launch_bounds__(128, mtp_min_blocks<ROWS_PER_CTA, StateT>()) gdn_mtp_kernel(const MtpParams p) {
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
    const int T = p.T;

    const long long slot = mtp_index(p.idx, p.idx64, bi);
    if (slot < 0 || slot >= p.pool_size) {  // padding entry
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
    const bool snap = snap_row >= 0;
    const bool upper = (sub & 4) != 0;
    MtpToken<kPasses> cur, nxt;
    mtp_load_token<StateT>(cur, p, (size_t)bi * T, hq, hv, sub, row_base);

    for (int t = 0; t < T; ++t) {
        const size_t bt = (size_t)bi * T + t;
        mtp_load_token<StateT>(nxt, p, t + 1 < T ? bt + 1 : bt, hq, hv, sub, row_base);

        float4 qf[4], kf[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            qf[j] = mtp_widen4(cur.q[j]);
            kf[j] = mtp_widen4(cur.k[j]);
        }
        const float g = expf(log_gate(p.A_log[hv], cur.a, p.dt_bias[hv]));
        const float beta = sigmoidf_(cur.b);
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

        const size_t ob = (bt * p.HV + hv) * kDim + row_base;
        float* snap_dst = snap ? p.inter + (((size_t)snap_row + t) * p.HV + hv) * kDim * kDim + row_off : nullptr;
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
            const float delta = beta * (cur.v[ps] - g * sk_all);
            if (sub == 4) p.out[ob + ps * 4] = __float2bfloat16_rn(p.scale * (g * keep + delta * kq));
#pragma unroll
            for (int j = 0; j < 4; ++j) s[ps][j] = gs_plus_dk(g, s[ps][j], delta, kf[j]);
            if constexpr (sizeof(StateT) == 4) {  // snapshots exist for fp32 pools only
                if (snap) mtp_store_row(snap_dst, (size_t)ps * 4 * kDim, sub, s[ps]);
            }
        }
        cur = nxt;
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
    if (state_bf16) {
        // half the bytes per row: 64 rows per CTA keep as many bytes in flight
        const bool large = heads * (gdn::kDim / 64) >= 8 * 148;
        const int rows = small ? 16 : large ? 64 : 32;
        const unsigned grid = (unsigned)(heads * (gdn::kDim / rows));
        if (rows == 16) gdn::gdn_mtp_kernel<16, __nv_bfloat16><<<grid, 128, 0, st>>>(p);
        else if (rows == 32) gdn::gdn_mtp_kernel<32, __nv_bfloat16><<<grid, 128, 0, st>>>(p);
        else gdn::gdn_mtp_kernel<64, __nv_bfloat16><<<grid, 128, 0, st>>>(p);
    } else {
        const unsigned grid = (unsigned)(heads * (gdn::kDim / (small ? 16 : 32)));
        if (small) gdn::gdn_mtp_kernel<16, float><<<grid, 128, 0, st>>>(p);
        else gdn::gdn_mtp_kernel<32, float><<<grid, 128, 0, st>>>(p);
    }
    return gdn_launch_status();
}
