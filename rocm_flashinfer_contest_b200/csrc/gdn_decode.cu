// gdn_decode.cu — single-token gated-delta-rule decode for B200 (sm_100a).
//
// Replaces the reference solution's fused Triton kernel `_klast_decode_kernel`
// and its launcher `_run_klast` (solutions/gdn_decode/main.py:38-114).  The
// maths is the contest definition (flashinfer/trace/templates/gdn.py:72-93):
// per v-head, with the k-last state row S[v, :] (128 contiguous fp32)
//
//   sk     = S[v,:] . k            sq = S[v,:] . q          kq = k . q
//   delta  = beta * (v[v] - g * sk)         (= new_v - old_v of gdn.py:84-85)
//   S'[v,:]= g * S[v,:] + delta * k        (= old - k(x)old_v + k(x)new_v)
//   o[v]   = scale * (g * sq + delta * kq)  (= scale * q^T S')
//
// Every state row is independent, so the kernel is one streaming pass over
// the state: each row is read once (16-byte, coalesced, evict-first loads)
// and written once (streaming stores).  Nothing else of size touches HBM, so
// the kernel is bound by HBM bandwidth: 8 bytes of state traffic per element.
//
// Thread layout: 8 lanes share one 512-byte row, each lane holding 16 values
// as four float4 at columns 4*(lane%8) + 32*j, so one warp-wide vector load
// covers four whole rows (2 KiB contiguous).  The two 128-long dot products of
// a row are reduced over its 8 lanes with one exchange-halves step plus two
// butterfly steps (3 shuffles for both sums) and one broadcast.
#include "gdn_common.cuh"

namespace gdn {

struct DecodeParams {
    const __nv_bfloat16* q;
    const __nv_bfloat16* k;
    const __nv_bfloat16* v;
    const float* state;  // nullable: zero initial state
    const float* A_log;
    const __nv_bfloat16* a;
    const float* dt_bias;
    const __nv_bfloat16* b;
    __nv_bfloat16* out;
    float* new_state;
    float scale;
    int HV, rep;  // rep = HV / H
    int H;
};

__device__ __forceinline__ float dot4(float4 x, float4 y) {
    return x.x * y.x + x.y * y.y + x.z * y.z + x.w * y.w;
}

// ROWS_PER_CTA rows of one v-head per CTA of 4 warps; 4 rows per warp pass.
template <int ROWS_PER_CTA>
__global__ void __launch_bounds__(128) gdn_decode_kernel(const DecodeParams p) {
    constexpr int kRowsPerWarp = ROWS_PER_CTA / 4;
    constexpr int kPasses = kRowsPerWarp / 4;
    constexpr int kBlocksPerHead = kDim / ROWS_PER_CTA;
    static_assert(kPasses >= 1 && kRowsPerWarp % 4 == 0, "4 rows per warp pass");

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sub = lane & 7;   // lane within the row's 8
    const int rsub = lane >> 3; // row within the warp's 4
    const long long head = blockIdx.x / kBlocksPerHead;  // b * HV + hv
    const int rb = blockIdx.x % kBlocksPerHead;
    const int bi = (int)(head / p.HV), hv = (int)(head % p.HV);
    const int hq = hv / p.rep;
    const int row_base = rb * ROWS_PER_CTA + warp * kRowsPerWarp + rsub;

    const size_t sbase = (size_t)head * kDim * kDim + (size_t)row_base * kDim + 4 * sub;

    // Issue the state loads first: they are the only long-latency traffic.
    float4 s[kPasses][4];
    if (p.state != nullptr) {
#pragma unroll
        for (int ps = 0; ps < kPasses; ++ps)
#pragma unroll
            for (int j = 0; j < 4; ++j)
                s[ps][j] = __ldcs(reinterpret_cast<const float4*>(p.state + sbase + (size_t)ps * 4 * kDim + 32 * j));
    } else {
#pragma unroll
        for (int ps = 0; ps < kPasses; ++ps)
#pragma unroll
            for (int j = 0; j < 4; ++j) s[ps][j] = make_float4(0.f, 0.f, 0.f, 0.f);
    }

    const __nv_bfloat16* qh = p.q + ((size_t)bi * p.H + hq) * kDim + 4 * sub;
    const __nv_bfloat16* kh = p.k + ((size_t)bi * p.H + hq) * kDim + 4 * sub;
    float4 qf[4], kf[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        qf[j] = load_bf16x4(qh + 32 * j);
        kf[j] = load_bf16x4(kh + 32 * j);
    }
    float vv[kPasses];
#pragma unroll
    for (int ps = 0; ps < kPasses; ++ps)
        vv[ps] = bf16_to_f32(p.v[(size_t)head * kDim + row_base + ps * 4]);

    const float g = expf(log_gate(p.A_log[hv], bf16_to_f32(p.a[head]), p.dt_bias[hv]));
    const float beta = sigmoidf_(bf16_to_f32(p.b[head]));

    float kq = dot4(kf[0], qf[0]) + dot4(kf[1], qf[1]) + dot4(kf[2], qf[2]) + dot4(kf[3], qf[3]);
    kq += __shfl_xor_sync(0xffffffffu, kq, 1);
    kq += __shfl_xor_sync(0xffffffffu, kq, 2);
    kq += __shfl_xor_sync(0xffffffffu, kq, 4);

    const bool upper = (sub & 4) != 0;  // after the exchange: lower half owns sk, upper owns sq
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
        // keep == full sk on lanes sub<4, full sq on lanes sub>=4
        const float sk_all = __shfl_sync(0xffffffffu, keep, lane & ~4);
        const float delta = beta * (vv[ps] - g * sk_all);
        if (sub == 4) {
            const float o = p.scale * (g * keep + delta * kq);
            p.out[(size_t)head * kDim + row_base + ps * 4] = __float2bfloat16_rn(o);
        }
        float* dst = p.new_state + sbase + (size_t)ps * 4 * kDim;
#pragma unroll
        for (int j = 0; j < 4; ++j) __stcs(reinterpret_cast<float4*>(dst + 32 * j), gs_plus_dk(g, s[ps][j], delta, kf[j]));
    }
}

}  // namespace gdn

extern "C" int gdn_decode_fwd(const void* q, const void* k, const void* v, const float* state,
                              const float* A_log, const void* a, const float* dt_bias,
                              const void* b, float scale, int B, int H, int HV, int K, int V,
                              void* out, float* new_state, void* stream) {
    if (B < 0 || H <= 0 || HV <= 0) return GDN_ERR_INVALID;
    if (K != gdn::kDim || V != gdn::kDim || HV % H != 0) return GDN_ERR_UNSUPPORTED;
    if (B == 0) return GDN_OK;
    if (!q || !k || !v || !A_log || !a || !dt_bias || !b || !out || !new_state)
        return GDN_ERR_INVALID;
    if (!gdn_aligned(q, 8) || !gdn_aligned(k, 8) || !gdn_aligned(new_state, 16) ||
        (state && !gdn_aligned(state, 16)) || !gdn_aligned(v, 2) || !gdn_aligned(out, 2) ||
        !gdn_aligned(a, 2) || !gdn_aligned(b, 2) || !gdn_aligned(A_log, 4) ||
        !gdn_aligned(dt_bias, 4))
        return GDN_ERR_ALIGN;
    if (scale == 0.0f) scale = 1.0f / sqrtf((float)K);

    gdn::DecodeParams p;
    p.q = static_cast<const __nv_bfloat16*>(q);
    p.k = static_cast<const __nv_bfloat16*>(k);
    p.v = static_cast<const __nv_bfloat16*>(v);
    p.state = state;
    p.A_log = A_log;
    p.a = static_cast<const __nv_bfloat16*>(a);
    p.dt_bias = dt_bias;
    p.b = static_cast<const __nv_bfloat16*>(b);
    p.out = static_cast<__nv_bfloat16*>(out);
    p.new_state = new_state;
    p.scale = scale;
    p.HV = HV;
    p.H = H;
    p.rep = HV / H;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const long long heads = (long long)B * HV;
    // Small batches: halve the rows per CTA so the grid still covers 148 SMs.
    if (heads * (gdn::kDim / 32) < 4 * 148) {
        gdn::gdn_decode_kernel<16><<<(unsigned)(heads * (gdn::kDim / 16)), 128, 0, st>>>(p);
    } else {
        gdn::gdn_decode_kernel<32><<<(unsigned)(heads * (gdn::kDim / 32)), 128, 0, st>>>(p);
    }
    return gdn_launch_status();
}
