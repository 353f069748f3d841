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
//     `cache_steps` >= T token slots per pool slot (gdn_decode.py:686-692);
//   * optional in-kernel q/k L2 normalisation, x * rsqrt(sum(x^2) + 1e-6)
//     (`use_qk_l2norm`, gdn_decode.py:571).
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
    const float* pool_in;    // [pool, HV, 128, 128]
    float* pool_out;         // nullable: final state not written
    const void* idx;         // [B] int32 or int64
    const float* A_log;
    const __nv_bfloat16* a;  // [B, T, HV]
    const float* dt_bias;
    const __nv_bfloat16* b;
    __nv_bfloat16* out;      // [B, T, HV, 128]
    float* inter;            // nullable: [inter_slots, cache_steps, HV, 128, 128]
    float scale;
    int T, H, HV, rep, pool_size, inter_slots, cache_steps, idx64, l2norm;
};

__device__ __forceinline__ float mtp_dot4(float4 x, float4 y) {
    return x.x * y.x + x.y * y.y + x.z * y.z + x.w * y.w;
}

__device__ __forceinline__ float row8_sum(float x) {
    x += __shfl_xor_sync(0xffffffffu, x, 1);
    x += __shfl_xor_sync(0xffffffffu, x, 2);
    x += __shfl_xor_sync(0xffffffffu, x, 4);
    return x;
}

// Everything one token contributes to one lane.
template <int kPasses>
struct MtpToken {
    float4 q[4], k[4];
    float v[kPasses];
    float a, b;
};

template <int kPasses>
__device__ __forceinline__ void mtp_load_token(MtpToken<kPasses>& tk, const MtpParams& p, size_t bt,
                                               int hq, int hv, int sub, int row_base) {
    const __nv_bfloat16* qh = p.q + (bt * p.H + hq) * kDim + 4 * sub;
    const __nv_bfloat16* kh = p.k + (bt * p.H + hq) * kDim + 4 * sub;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        tk.q[j] = load_bf16x4(qh + 32 * j);
        tk.k[j] = load_bf16x4(kh + 32 * j);
    }
    const size_t vh = bt * p.HV + hv;
#pragma unroll
    for (int ps = 0; ps < kPasses; ++ps) tk.v[ps] = bf16_to_f32(p.v[vh * kDim + row_base + ps * 4]);
    tk.a = bf16_to_f32(p.a[vh]);
    tk.b = bf16_to_f32(p.b[vh]);
}

// ROWS_PER_CTA rows of one (batch entry, v-head) per CTA of 4 warps.
template <int ROWS_PER_CTA>
__global__ void __launch_bounds__(128) gdn_mtp_kernel(const MtpParams p) {
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

    const long long slot = p.idx64 ? static_cast<const long long*>(p.idx)[bi]
                                   : (long long)static_cast<const int*>(p.idx)[bi];
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

    const size_t row_off = (size_t)row_base * kDim + 4 * sub;
    const size_t sbase = ((size_t)slot * p.HV + hv) * kDim * kDim + row_off;
    float4 s[kPasses][4];
#pragma unroll
    for (int ps = 0; ps < kPasses; ++ps)
#pragma unroll
        for (int j = 0; j < 4; ++j)
            s[ps][j] = __ldcs(reinterpret_cast<const float4*>(p.pool_in + sbase + (size_t)ps * 4 * kDim + 32 * j));

    const bool snap = p.inter != nullptr && slot < p.inter_slots;
    const bool upper = (sub & 4) != 0;
    MtpToken<kPasses> cur, nxt;
    mtp_load_token(cur, p, (size_t)bi * T, hq, hv, sub, row_base);

    for (int t = 0; t < T; ++t) {
        const size_t bt = (size_t)bi * T + t;
        mtp_load_token(nxt, p, t + 1 < T ? bt + 1 : bt, hq, hv, sub, row_base);

        const float g = expf(log_gate(p.A_log[hv], cur.a, p.dt_bias[hv]));
        const float beta = sigmoidf_(cur.b);
        if (p.l2norm) {
            float qq = 0.f, kk = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                qq += mtp_dot4(cur.q[j], cur.q[j]);
                kk += mtp_dot4(cur.k[j], cur.k[j]);
            }
            const float iq = rsqrtf(row8_sum(qq) + 1e-6f), ik = rsqrtf(row8_sum(kk) + 1e-6f);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                cur.q[j] = make_float4(cur.q[j].x * iq, cur.q[j].y * iq, cur.q[j].z * iq, cur.q[j].w * iq);
                cur.k[j] = make_float4(cur.k[j].x * ik, cur.k[j].y * ik, cur.k[j].z * ik, cur.k[j].w * ik);
            }
        }
        float kq = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) kq += mtp_dot4(cur.k[j], cur.q[j]);
        kq = row8_sum(kq);

        const size_t ob = (bt * p.HV + hv) * kDim + row_base;
        float* snap_dst = snap ? p.inter + (((size_t)slot * p.cache_steps + t) * p.HV + hv) * kDim * kDim + row_off
                               : nullptr;
#pragma unroll
        for (int ps = 0; ps < kPasses; ++ps) {
            float sk = 0.f, sq = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                sk += mtp_dot4(s[ps][j], cur.k[j]);
                sq += mtp_dot4(s[ps][j], cur.q[j]);
            }
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
            for (int j = 0; j < 4; ++j) {
                s[ps][j].x = fmaf(g, s[ps][j].x, delta * cur.k[j].x);
                s[ps][j].y = fmaf(g, s[ps][j].y, delta * cur.k[j].y);
                s[ps][j].z = fmaf(g, s[ps][j].z, delta * cur.k[j].z);
                s[ps][j].w = fmaf(g, s[ps][j].w, delta * cur.k[j].w);
            }
            if (snap) {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    __stcs(reinterpret_cast<float4*>(snap_dst + (size_t)ps * 4 * kDim + 32 * j), s[ps][j]);
            }
        }
        cur = nxt;
    }

    if (p.pool_out != nullptr) {
#pragma unroll
        for (int ps = 0; ps < kPasses; ++ps)
#pragma unroll
            for (int j = 0; j < 4; ++j)
                __stcs(reinterpret_cast<float4*>(p.pool_out + sbase + (size_t)ps * 4 * kDim + 32 * j), s[ps][j]);
    }
}

}  // namespace gdn

extern "C" int gdn_mtp_fwd(const void* q, const void* k, const void* v, const float* pool_in,
                           float* pool_out, const void* indices, int indices_int64,
                           const float* A_log, const void* a, const float* dt_bias, const void* b,
                           float scale, int B, int T, int H, int HV, int K, int V, int pool_size,
                           int qk_l2norm, void* out, float* intermediate, int inter_slots,
                           int cache_steps, void* stream) {
    if (B < 0 || T < 0 || H <= 0 || HV <= 0 || pool_size < 0) return GDN_ERR_INVALID;
    if ((indices_int64 != 0 && indices_int64 != 1) || (qk_l2norm != 0 && qk_l2norm != 1))
        return GDN_ERR_INVALID;
    if (K != gdn::kDim || V != gdn::kDim || HV % H != 0) return GDN_ERR_UNSUPPORTED;
    if (intermediate && (inter_slots < 0 || cache_steps < T)) return GDN_ERR_INVALID;
    const size_t head_bytes = sizeof(float) * gdn::kDim * gdn::kDim;
    const size_t pool_bytes = (size_t)pool_size * HV * head_bytes;
    const bool copy_pool = pool_out != nullptr && pool_out != pool_in && pool_size > 0;
    if (copy_pool) {
        if (!pool_in) return GDN_ERR_INVALID;
        const char* i0 = reinterpret_cast<const char*>(pool_in);
        const char* o0 = reinterpret_cast<const char*>(pool_out);
        if (o0 < i0 + pool_bytes && i0 < o0 + pool_bytes) return GDN_ERR_INVALID;  // partial overlap
        if (!gdn_aligned(pool_out, 16) || !gdn_aligned(pool_in, 16)) return GDN_ERR_ALIGN;
    }
    if ((long long)B * T > 0) {
        if (!q || !k || !v || !pool_in || !indices || !A_log || !a || !dt_bias || !b || !out)
            return GDN_ERR_INVALID;
        if (!gdn_aligned(q, 8) || !gdn_aligned(k, 8) || !gdn_aligned(pool_in, 16) ||
            (pool_out && !gdn_aligned(pool_out, 16)) || (intermediate && !gdn_aligned(intermediate, 16)) ||
            !gdn_aligned(v, 2) || !gdn_aligned(out, 2) || !gdn_aligned(a, 2) || !gdn_aligned(b, 2) ||
            !gdn_aligned(A_log, 4) || !gdn_aligned(dt_bias, 4) ||
            !gdn_aligned(indices, indices_int64 ? 8 : 4))
            return GDN_ERR_ALIGN;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (copy_pool) {
        // slots no batch entry names keep their value in the new pool
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
    p.l2norm = qk_l2norm;
    const long long heads = (long long)B * HV;
    if (heads * (gdn::kDim / 32) < 4 * 148) {
        gdn::gdn_mtp_kernel<16><<<(unsigned)(heads * (gdn::kDim / 16)), 128, 0, st>>>(p);
    } else {
        gdn::gdn_mtp_kernel<32><<<(unsigned)(heads * (gdn::kDim / 32)), 128, 0, st>>>(p);
    }
    return gdn_launch_status();
}
