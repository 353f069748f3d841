// gdn_prefill_recurrent.cu — token-serial varlen prefill for B200 (sm_100a).
//
// The short-sequence path of the prefill (the role AITER's
// fused_recurrent_gated_delta_rule plays in solutions/gdn_prefill/main.py:76-80),
// following the contest definition token by token
// (flashinfer/trace/templates/gdn.py:230-271).  The state rows of one
// (sequence, v-head) live in registers for the whole sequence: a CTA of four
// warps owns 16 rows (4 per warp, 8 lanes per 512-byte row, as in the decode
// kernel), so a head is split over 8 CTAs and nothing but the inputs and the
// outputs moves through memory.  The next token's q/k/v/gates are loaded
// while the current token is processed.  With checkpoints enabled the rows
// are also stored after every `ckpt_every` tokens.  With qk_l2norm the q and
// k head vectors are normalised in registers, in fp32, before they are used.
#include "gdn_common.cuh"
#include "gdn_prefill_common.cuh"

namespace gdn {

__device__ __forceinline__ float dot4r(float4 x, float4 y) {
    return x.x * y.x + x.y * y.y + x.z * y.z + x.w * y.w;
}

struct TokenRaw {
    uint2 q[4], k[4];
    __nv_bfloat16 v, a, b;
};

__device__ __forceinline__ void load_token(const PrefillParams& p, long long t, int hq, int hv,
                                           int row, int sub, TokenRaw& r) {
    const __nv_bfloat16* qh = p.q + ((size_t)t * p.H + hq) * kDim + 4 * sub;
    const __nv_bfloat16* kh = p.k + ((size_t)t * p.H + hq) * kDim + 4 * sub;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        r.q[j] = *reinterpret_cast<const uint2*>(qh + 32 * j);
        r.k[j] = *reinterpret_cast<const uint2*>(kh + 32 * j);
    }
    r.v = p.v[((size_t)t * p.HV + hv) * kDim + row];
    r.a = p.a[(size_t)t * p.HV + hv];
    r.b = p.b[(size_t)t * p.HV + hv];
}

__device__ __forceinline__ float4 widen(uint2 raw) {
    __nv_bfloat162 lo = *reinterpret_cast<__nv_bfloat162*>(&raw.x);
    __nv_bfloat162 hi = *reinterpret_cast<__nv_bfloat162*>(&raw.y);
    float2 x = __bfloat1622float2(lo), y = __bfloat1622float2(hi);
    return make_float4(x.x, x.y, y.x, y.y);
}

__global__ void __launch_bounds__(128) gdn_prefill_recurrent_kernel(const PrefillParams p) {
    constexpr int kRowsPerCta = 16;
    constexpr int kBlocksPerHead = kDim / kRowsPerCta;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sub = lane & 7, rsub = lane >> 3;
    const int rb = blockIdx.x % kBlocksPerHead;
    const long long nh = blockIdx.x / kBlocksPerHead;
    const int hv = (int)(nh % p.HV), n = (int)(nh / p.HV);
    const int hq = hv / p.rep;
    const int row = rb * kRowsPerCta + warp * 4 + rsub;

    long long t0, t1;
    seq_bounds(p, n, t0, t1);
    zero_uncovered_outputs(p, n, t0, t1, hv, row, sub == 4);

    float* ns = p.new_state + ((size_t)nh * kDim + row) * kDim + 4 * sub;
    float4 s[4];
    if (t1 == t0) {  // empty sequence: the final state stays zero
#pragma unroll
        for (int j = 0; j < 4; ++j) reinterpret_cast<float4*>(ns)[8 * j] = make_float4(0.f, 0.f, 0.f, 0.f);
        return;
    }
    if (p.state != nullptr) {
        const float* is = p.state + ((size_t)nh * kDim + row) * kDim + 4 * sub;
#pragma unroll
        for (int j = 0; j < 4; ++j) s[j] = __ldcs(reinterpret_cast<const float4*>(is + 32 * j));
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) s[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const float A_log = p.A_log[hv], dt_bias = p.dt_bias[hv];
    const bool upper = (sub & 4) != 0;

    TokenRaw nxt;
    load_token(p, t0, hq, hv, row, sub, nxt);
    int until_ckpt = p.ckpt_every;  // tokens left before the next checkpoint
    for (long long t = t0; t < t1; ++t) {
        TokenRaw cur = nxt;
        if (t + 1 < t1) load_token(p, t + 1, hq, hv, row, sub, nxt);
        float4 qf[4], kf[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            qf[j] = widen(cur.q[j]);
            kf[j] = widen(cur.k[j]);
        }
        const float g = expf(log_gate(A_log, bf16_to_f32(cur.a), dt_bias));
        const float beta = sigmoidf_(bf16_to_f32(cur.b));
        if (p.qk_l2norm) {
            // the 8 lanes of a row hold a whole q and k head vector
            float qq = 0.f, kk = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                qq += dot4r(qf[j], qf[j]);
                kk += dot4r(kf[j], kf[j]);
            }
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) {
                qq += __shfl_xor_sync(0xffffffffu, qq, o);
                kk += __shfl_xor_sync(0xffffffffu, kk, o);
            }
            const float iq = rsqrtf(qq + 1e-6f), ik = rsqrtf(kk + 1e-6f);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                qf[j] = make_float4(qf[j].x * iq, qf[j].y * iq, qf[j].z * iq, qf[j].w * iq);
                kf[j] = make_float4(kf[j].x * ik, kf[j].y * ik, kf[j].z * ik, kf[j].w * ik);
            }
        }
        float kq = dot4r(kf[0], qf[0]) + dot4r(kf[1], qf[1]) + dot4r(kf[2], qf[2]) + dot4r(kf[3], qf[3]);
        float2 sk2 = make_float2(0.f, 0.f), sq2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            sk2 = dot4_acc2(s[j], kf[j], sk2);
            sq2 = dot4_acc2(s[j], qf[j], sq2);
        }
        const float sk = sk2.x + sk2.y, sq = sq2.x + sq2.y;
        kq += __shfl_xor_sync(0xffffffffu, kq, 1);
        kq += __shfl_xor_sync(0xffffffffu, kq, 2);
        kq += __shfl_xor_sync(0xffffffffu, kq, 4);
        float give = upper ? sk : sq;
        float keep = upper ? sq : sk;
        keep += __shfl_xor_sync(0xffffffffu, give, 4);
        keep += __shfl_xor_sync(0xffffffffu, keep, 1);
        keep += __shfl_xor_sync(0xffffffffu, keep, 2);
        const float sk_all = __shfl_sync(0xffffffffu, keep, lane & ~4);
        const float delta = beta * (bf16_to_f32(cur.v) - g * sk_all);
        if (sub == 4)
            p.out[((size_t)t * p.HV + hv) * kDim + row] = __float2bfloat16_rn(p.scale * (g * keep + delta * kq));
#pragma unroll
        for (int j = 0; j < 4; ++j) s[j] = gs_plus_dk(g, s[j], delta, kf[j]);
        if (p.ckpt != nullptr && --until_ckpt == 0) {
            until_ckpt = p.ckpt_every;
            float* cd = ckpt_dst(p, n, hv, t - t0 + 1);
            if (cd != nullptr) {
                float* dst = cd + (size_t)row * kDim + 4 * sub;
#pragma unroll
                for (int j = 0; j < 4; ++j) __stcs(reinterpret_cast<float4*>(dst + 32 * j), s[j]);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) __stcs(reinterpret_cast<float4*>(ns + 32 * j), s[j]);
}

void launch_prefill_recurrent(const PrefillParams& p, cudaStream_t st) {
    const long long blocks = (long long)p.N * p.HV * (kDim / 16);
    gdn_prefill_recurrent_kernel<<<(unsigned)blocks, 128, 0, st>>>(p);
}

}  // namespace gdn
