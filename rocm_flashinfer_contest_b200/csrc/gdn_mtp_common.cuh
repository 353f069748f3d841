// gdn_mtp_common.cuh — parameters and row helpers shared by the multi-token
// (pool-indexed) decode kernels: the per-CTA kernels of gdn_mtp.cu and the
// persistent streaming kernel of gdn_mtp_stream.cu.
#pragma once

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

// Column layout of a lane's 16 values of a row (4 groups of 4).  fp32 state:
// group j at columns 4*sub + 32*j (one 16-byte access per group).  bf16 state:
// groups 2p, 2p+1 at columns 8*sub + 64*p (+4), so one 16-byte access moves
// two groups and a row needs two accesses per lane.
template <typename StateT>
__device__ __forceinline__ int mtp_col(int sub, int j) {
    return sizeof(StateT) == 4 ? 4 * sub + 32 * j : 8 * sub + 64 * (j >> 1) + 4 * (j & 1);
}

__device__ __forceinline__ float4 mtp_widen4(uint2 raw) {
    __nv_bfloat162 lo = *reinterpret_cast<__nv_bfloat162*>(&raw.x);
    __nv_bfloat162 hi = *reinterpret_cast<__nv_bfloat162*>(&raw.y);
    float2 x = __bfloat1622float2(lo), y = __bfloat1622float2(hi);
    return make_float4(x.x, x.y, y.x, y.y);
}

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

// One bf16 output value, stored through the global state space (a store the
// compiler knows cannot touch shared memory).
__device__ __forceinline__ void stg_bf16(__nv_bfloat16* p, float x) {
    const __nv_bfloat16 h = __float2bfloat16_rn(x);
    asm volatile("st.global.b16 [%0], %1;" ::"l"(p), "h"(*reinterpret_cast<const unsigned short*>(&h)) : "memory");
}

// Persistent streaming form (gdn_mtp_stream.cu).  Launches it and returns
// GDN_OK when the call is one it serves (1 <= T <= kStreamMaxT, HV even and at
// most 256, q / k / v 16-byte and a / b 4-byte aligned), else returns 1 and
// launches nothing.  B: batch entries.
constexpr int kStreamMaxT = 8;
int launch_mtp_stream(const MtpParams& p, int B, bool state_bf16, cudaStream_t st);
// Device status word of the streaming kernel's translation unit (bounded
// waits that ran out); cleared when `clear`.
int mtp_stream_status(bool clear);

}  // namespace gdn
