// Parameters and sequence bookkeeping shared by the prefill kernels.
#pragma once

#include "gdn_common.cuh"

namespace gdn {

struct PrefillParams {
    const __nv_bfloat16* q;  // [T, H, K]
    const __nv_bfloat16* k;  // [T, H, K]
    const __nv_bfloat16* v;  // [T, HV, V]
    const float* state;      // [N, HV, V, K] or null
    const float* A_log;      // [HV]
    const __nv_bfloat16* a;  // [T, HV]
    const float* dt_bias;    // [HV]
    const __nv_bfloat16* b;  // [T, HV]
    const void* cu_seqlens;  // [N + 1], int32 or int64
    __nv_bfloat16* out;      // [T, HV, V]
    float* new_state;        // [N, HV, V, K]
    float scale;
    int cu_is_int64;
    int N, T, H, HV, rep;    // rep = HV / H
    // optional state checkpoints (flashinfer's chunk_gated_delta_rule,
    // flashinfer/gdn_prefill.py:113-115,161-174): the state after tokens
    // every, 2*every, ... of sequence n goes to ckpt[ckpt_cu[n] + i]
    float* ckpt;               // [ckpt_total, HV, V, K] or null
    const long long* ckpt_cu;  // [N + 1]
    long long ckpt_total;
    int ckpt_every;            // > 0, a multiple of 64, when ckpt is set
    int cross_gram;            // chunked path: the prep also publishes G tiles
    int qk_l2norm;             // normalise q and k rows in the kernel: x * rsqrt(sum(x^2) + 1e-6)
};

// Destination of the checkpoint after `done` tokens of sequence n (done a
// multiple of ckpt_every), or null when the index falls outside the
// sequence's range or the buffer (a malformed ckpt_cu cannot send a store
// out of bounds).
__device__ __forceinline__ float* ckpt_dst(const PrefillParams& p, int n, int hv, long long done) {
    const long long first = p.ckpt_cu[n], end = p.ckpt_cu[n + 1];
    const long long i = first + done / p.ckpt_every - 1;
    if (i < first || i >= end || i < 0 || i >= p.ckpt_total) return nullptr;
    return p.ckpt + ((size_t)i * p.HV + hv) * kDim * kDim;
}

__device__ __forceinline__ long long load_cu(const PrefillParams& p, int i) {
    return p.cu_is_int64 ? static_cast<const long long*>(p.cu_seqlens)[i]
                         : (long long)static_cast<const int*>(p.cu_seqlens)[i];
}

// Token range [t0, t1) of sequence n, clamped into [0, T] and made monotone so
// a malformed cu_seqlens cannot send any access out of bounds.
__device__ __forceinline__ void seq_bounds(const PrefillParams& p, int n, long long& t0, long long& t1) {
    long long a = load_cu(p, n), b = load_cu(p, n + 1);
    a = a < 0 ? 0 : (a > p.T ? p.T : a);
    b = b < a ? a : (b > p.T ? p.T : b);
    t0 = a;
    t1 = b;
}

// Tokens before cu_seqlens[0] or from cu_seqlens[N] on belong to no sequence;
// the reference leaves their output at zero (gdn.py:221-223).  The CTAs of the
// first / last sequence write those zeros for their own (head, row).
__device__ __forceinline__ void zero_uncovered_outputs(const PrefillParams& p, int n, long long t0,
                                                       long long t1, int hv, int row, bool writer) {
    if (!writer) return;
    const __nv_bfloat16 z = __float2bfloat16_rn(0.0f);
    if (n == 0)
        for (long long t = 0; t < t0; ++t) p.out[((size_t)t * p.HV + hv) * kDim + row] = z;
    if (n == p.N - 1)
        for (long long t = t1; t < p.T; ++t) p.out[((size_t)t * p.HV + hv) * kDim + row] = z;
}

// Argument checks shared by the prefill entry points (sizes, null pointers,
// alignment; no CUDA call): GDN_OK or the status to return.
int prefill_check_args(const void* q, const void* k, const void* v, const float* state, const float* A_log,
                       const void* a, const float* dt_bias, const void* b, const void* cu_seqlens,
                       int cu_seqlens_is_int64, int N, int T, int H, int HV, int K, int V, const void* out,
                       const float* new_state);
void launch_prefill_recurrent(const PrefillParams& p, cudaStream_t st);
// Launches the chunked kernels (prep, then a chain kernel); returns a GDN_*
// status (GDN_ERR_CUDA when the per-device launch set-up or a launch fails).
// `workspace_bytes` steers the choice of chain: the scan chain needs the
// larger of the two workspace layouts.  With `aux_streams` the scan chain's
// prep may run on library streams beside it (created on first use);
// without, everything runs in order on `st`.
int launch_prefill_chunk(const PrefillParams& p, void* workspace, size_t workspace_bytes, cudaStream_t st,
                         bool aux_streams);
// gdn_prefill_fwd restricted to the caller's stream (no library stream or
// event is created): the entry point for callers that allocate nothing.
int prefill_fwd_one_stream(const void* q, const void* k, const void* v, const float* state, const float* A_log,
                           const void* a, const float* dt_bias, const void* b, const void* cu_seqlens,
                           int cu_seqlens_is_int64, int N, int T, float scale, int H, int HV, int K, int V,
                           void* out, float* new_state, void* workspace, size_t workspace_bytes, void* stream);
// Workspace of the chunked path: enough for every chain (the scan chain's
// layout is the larger one), and the split-path layout alone (the least a
// chunked call can run in).
size_t prefill_workspace_bytes(int N, int T, int H, int HV);
size_t prefill_workspace_bytes_split(int N, int T, int H, int HV);

}  // namespace gdn
