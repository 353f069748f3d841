// gdn_prefill_host.cu — varlen prefill with every operand in host memory.
//
// For a caller whose tokens and states live in host memory the prefill is
// PCIe-bound: q, k, v go up and the output comes back (8192 tokens at
// H = 16, HV = 32: 135 MB up, 67 MB down) while the kernels take a fraction
// of that.  The tokens are cut into segments (64-token aligned, so chunk
// boundaries stay where one call would put them; the last ones shrink, see
// segment_starts) and pipelined over three
// streams: segment s + 1 is copied up (library stream `up`) while segment s
// is prefilled (the caller's stream) and segment s - 1's output is copied
// back (library stream `down`).  The running state of every sequence stays
// in the device workspace: each segment's prefill starts from it and writes
// it back in place, so a sequence cut by a segment boundary continues exactly
// as a second prefill call from the first call's final state would (the
// recurrence is a left fold over tokens).
#include <algorithm>
#include <mutex>
#include <vector>

#include "gdn_common.cuh"
#include "gdn_prefill_common.cuh"

namespace {

constexpr int kDefaultSegment = 2048;

struct HostLayout {
    size_t state, A_log, dt_bias, cu_full, ring, ring_stride, q, k, v, a, b, out, cu, pws, total;
};

inline size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

HostLayout host_layout(int N, int H, int HV, int seg) {
    const size_t d = gdn::kDim;
    HostLayout L;
    size_t off = 0;
    L.state = off;   off += up256(size_t(N) * HV * d * d * 4);
    L.A_log = off;   off += up256(size_t(HV) * 4);
    L.dt_bias = off; off += up256(size_t(HV) * 4);
    L.cu_full = off; off += up256(size_t(N + 1) * 8);
    // one ring slot: a segment's inputs, output and cu_seqlens
    size_t r = 0;
    L.q = r;   r += up256(size_t(seg) * H * d * 2);
    L.k = r;   r += up256(size_t(seg) * H * d * 2);
    L.v = r;   r += up256(size_t(seg) * HV * d * 2);
    L.a = r;   r += up256(size_t(seg) * HV * 2);
    L.b = r;   r += up256(size_t(seg) * HV * 2);
    L.out = r; r += up256(size_t(seg) * HV * d * 2);
    L.cu = r;  r += up256(size_t(N + 1) * 8);
    L.ring_stride = r;
    L.ring = off;    off += 2 * r;
    L.pws = off;     off += up256(gdn::prefill_workspace_bytes(N, seg, H, HV));
    L.total = off;
    return L;
}

// cu_seg[i] = clamp(cu[n0 + i], s0, s1) - s0 for i = 0 .. count - 1
__global__ void segment_cu_kernel(const long long* cu, int n0, int count, long long s0, long long s1,
                                  long long* cu_seg) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) {
        long long c = cu[n0 + i];
        c = c < s0 ? s0 : (c > s1 ? s1 : c);
        cu_seg[i] = c - s0;
    }
}

// widen an int32 cu_seqlens to int64 (the segment kernel reads int64)
__global__ void widen_cu_kernel(const int* cu32, int count, long long* cu64) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) cu64[i] = cu32[i];
}

struct HostPipe {
    bool ready = false;
    cudaStream_t up = nullptr, down = nullptr;
    cudaEvent_t h2d[2] = {}, comp[2] = {}, d2h[2] = {}, all_done = nullptr;
};
constexpr int kMaxDevices = 64;
std::mutex g_pipe_mu;
HostPipe g_pipe[kMaxDevices];

bool init_pipe(HostPipe& pp) {
    if (pp.ready) return true;
    if (cudaStreamCreateWithFlags(&pp.up, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&pp.down, cudaStreamNonBlocking) != cudaSuccess)
        return false;
    cudaEvent_t* evs[] = {&pp.h2d[0], &pp.h2d[1], &pp.comp[0], &pp.comp[1], &pp.d2h[0], &pp.d2h[1], &pp.all_done};
    for (cudaEvent_t* e : evs)
        if (cudaEventCreateWithFlags(e, cudaEventDisableTiming) != cudaSuccess) return false;
    // recorded once so the first call's waits on them are satisfied at once
    for (int i = 0; i < 2; ++i)
        if (cudaEventRecord(pp.comp[i], pp.down) != cudaSuccess || cudaEventRecord(pp.d2h[i], pp.down) != cudaSuccess)
            return false;
    if (cudaEventRecord(pp.all_done, pp.down) != cudaSuccess) return false;
    pp.ready = true;
    return true;
}

int effective_segment(int segment_tokens) {
    const int s = segment_tokens > 0 ? segment_tokens : kDefaultSegment;
    return std::max(64, (s + 63) / 64 * 64);
}

}  // namespace

// Segment starts (and T at the end): segments of `seg` tokens, except that
// the last `seg` or fewer tokens are cut in halves down to kTailTokens
// (2048 -> 1024, 512, 256, 256), all 64-aligned.  Once the last upload has
// landed only the last segment's prefill and copy back are left, so a short
// last segment keeps that tail short while the long ones keep the per-copy
// overheads low.
constexpr long long kTailTokens = 256;
std::vector<long long> segment_starts(long long T, long long seg) {
    std::vector<long long> s;
    long long s0 = 0;
    while (T - s0 > seg) {
        s.push_back(s0);
        s0 += seg;
    }
    while (T - s0 > kTailTokens) {
        s.push_back(s0);
        s0 += ((T - s0) / 2 + 63) / 64 * 64;
    }
    if (T > s0) s.push_back(s0);
    s.push_back(T);
    return s;
}

extern "C" size_t gdn_prefill_host_workspace_bytes(int N, int T, int H, int HV, int segment_tokens) {
    if (N < 0 || T < 0 || H <= 0 || HV <= 0 || segment_tokens < 0 || (N == 0 && T == 0)) return 0;
    const int seg = T > 0 ? std::min(effective_segment(segment_tokens), (T + 63) / 64 * 64) : 64;
    return host_layout(std::max(N, 1), H, HV, seg).total;
}

extern "C" int gdn_prefill_fwd_host(const void* q, const void* k, const void* v, const float* state,
                                    const float* A_log, const void* a, const float* dt_bias, const void* b,
                                    const void* cu_seqlens, int cu_seqlens_is_int64, int N, int T, float scale,
                                    int H, int HV, int K, int V, void* out, float* new_state, void* workspace,
                                    size_t workspace_bytes, int segment_tokens, void* stream) {
    if (N < 0 || T < 0 || H <= 0 || HV <= 0 || segment_tokens < 0) return GDN_ERR_INVALID;
    if (cu_seqlens_is_int64 != 0 && cu_seqlens_is_int64 != 1) return GDN_ERR_INVALID;
    if (K != gdn::kDim || V != gdn::kDim || HV % H != 0) return GDN_ERR_UNSUPPORTED;
    if (N == 0 && T == 0) return GDN_OK;
    if (!cu_seqlens || !A_log || !dt_bias || !workspace) return GDN_ERR_INVALID;
    if (N > 0 && !new_state) return GDN_ERR_INVALID;
    if (T > 0 && (!q || !k || !v || !a || !b || !out)) return GDN_ERR_INVALID;
    // cu_seqlens is in host memory here, so it is checked on the host
    std::vector<long long> cu(N + 1);
    for (int n = 0; n <= N; ++n)
        cu[n] = cu_seqlens_is_int64 ? static_cast<const long long*>(cu_seqlens)[n]
                                    : (long long)static_cast<const int*>(cu_seqlens)[n];
    if (cu[0] < 0 || cu[N] > T) return GDN_ERR_INVALID;
    for (int n = 0; n < N; ++n)
        if (cu[n + 1] < cu[n]) return GDN_ERR_INVALID;
    const int seg = T > 0 ? std::min(effective_segment(segment_tokens), (T + 63) / 64 * 64) : 64;
    const HostLayout L = host_layout(std::max(N, 1), H, HV, seg);
    if (workspace_bytes < L.total) return GDN_ERR_INVALID;
    if (!gdn_aligned(workspace, 256)) return GDN_ERR_ALIGN;
    if (scale == 0.0f) scale = 1.0f / sqrtf((float)K);

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return GDN_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_pipe_mu);
    HostPipe& pp = g_pipe[dev];
    if (!init_pipe(pp)) return GDN_ERR_CUDA;

    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    char* ws = static_cast<char*>(workspace);
    float* d_state = reinterpret_cast<float*>(ws + L.state);
    long long* d_cu = reinterpret_cast<long long*>(ws + L.cu_full);
    const size_t head_state = (size_t)HV * K * V * 4;
    const cudaMemcpyKind h2d = cudaMemcpyHostToDevice, d2h = cudaMemcpyDeviceToHost;
    int status = GDN_OK;
    auto ok = [&](cudaError_t e) {
        if (e != cudaSuccess && status == GDN_OK) status = GDN_ERR_CUDA;
        return status == GDN_OK;
    };

    // the previous call's copies back read the workspace until all_done
    ok(cudaStreamWaitEvent(cs, pp.all_done, 0));
    ok(cudaStreamWaitEvent(pp.up, pp.all_done, 0));
    // state, gates' per-head constants and cu_seqlens: on the caller's stream
    if (N > 0) {
        if (state) ok(cudaMemcpyAsync(d_state, state, (size_t)N * head_state, h2d, cs));
        else ok(cudaMemsetAsync(d_state, 0, (size_t)N * head_state, cs));
    }
    ok(cudaMemcpyAsync(ws + L.A_log, A_log, (size_t)HV * 4, h2d, cs));
    ok(cudaMemcpyAsync(ws + L.dt_bias, dt_bias, (size_t)HV * 4, h2d, cs));
    if (cu_seqlens_is_int64) {
        ok(cudaMemcpyAsync(d_cu, cu_seqlens, (size_t)(N + 1) * 8, h2d, cs));
    } else {
        // int32 copy into ring slot 0's cu area, widened on the device; that area
        // is next written by segment 0's cu kernel, later on this same stream
        int* tmp32 = reinterpret_cast<int*>(ws + L.ring + L.cu);
        ok(cudaMemcpyAsync(tmp32, cu_seqlens, (size_t)(N + 1) * 4, h2d, cs));
        if (status == GDN_OK) {
            widen_cu_kernel<<<(N + 1 + 255) / 256, 256, 0, cs>>>(tmp32, N + 1, d_cu);
            ok(cudaGetLastError());
        }
    }
    // the first uploads wait for the set-up above (it reuses ring slot 0's cu area)
    ok(cudaEventRecord(pp.h2d[1], cs));
    ok(cudaStreamWaitEvent(pp.up, pp.h2d[1], 0));

    const std::vector<long long> starts = segment_starts(T, seg);
    const int nseg = (int)starts.size() - 1;
    for (int si = 0; si < nseg && status == GDN_OK; ++si) {
        const int r = si & 1;
        char* slot = ws + L.ring + (size_t)r * L.ring_stride;
        const long long s0 = starts[si], s1 = starts[si + 1];
        const long long nt = s1 - s0;
        // 1. upload the segment (after the prefill of segment si - 2 is done with this slot)
        ok(cudaStreamWaitEvent(pp.up, pp.comp[r], 0));
        ok(cudaMemcpyAsync(slot + L.q, static_cast<const char*>(q) + s0 * H * K * 2, nt * H * K * 2, h2d, pp.up));
        ok(cudaMemcpyAsync(slot + L.k, static_cast<const char*>(k) + s0 * H * K * 2, nt * H * K * 2, h2d, pp.up));
        ok(cudaMemcpyAsync(slot + L.v, static_cast<const char*>(v) + s0 * HV * V * 2, nt * HV * V * 2, h2d, pp.up));
        ok(cudaMemcpyAsync(slot + L.a, static_cast<const char*>(a) + s0 * HV * 2, nt * HV * 2, h2d, pp.up));
        ok(cudaMemcpyAsync(slot + L.b, static_cast<const char*>(b) + s0 * HV * 2, nt * HV * 2, h2d, pp.up));
        ok(cudaEventRecord(pp.h2d[r], pp.up));
        // 2. prefill the sequences that have tokens in [s0, s1), in place on their running states,
        //    once the upload has landed and segment si - 2's output has been copied back
        ok(cudaStreamWaitEvent(cs, pp.h2d[r], 0));
        ok(cudaStreamWaitEvent(cs, pp.d2h[r], 0));
        int n0 = 0;
        while (n0 < N && cu[n0 + 1] <= s0) ++n0;  // first sequence ending after s0
        int n1 = n0;
        while (n1 < N && cu[n1] < s1) ++n1;       // one past the last sequence starting before s1
        // skip sequences with no token in the segment at either end (empty ones are zeroed below)
        while (n0 < n1 && cu[n0 + 1] <= s0) ++n0;
        while (n1 > n0 && cu[n1 - 1] >= s1) --n1;
        long long* cu_seg = reinterpret_cast<long long*>(slot + L.cu);
        if (status != GDN_OK) break;
        if (n1 > n0) {
            const int cnt = n1 - n0 + 1;
            segment_cu_kernel<<<(cnt + 255) / 256, 256, 0, cs>>>(d_cu, n0, cnt, s0, s1, cu_seg);
            if (!ok(cudaGetLastError())) break;
            float* st = d_state + (size_t)n0 * HV * K * V;
            const int rc = gdn_prefill_fwd(slot + L.q, slot + L.k, slot + L.v, st,
                                           reinterpret_cast<const float*>(ws + L.A_log), slot + L.a,
                                           reinterpret_cast<const float*>(ws + L.dt_bias), slot + L.b, cu_seg, 1,
                                           n1 - n0, (int)nt, scale, H, HV, K, V, slot + L.out, st, ws + L.pws,
                                           workspace_bytes - L.pws, cs);
            if (rc != GDN_OK) {
                status = rc;
                break;
            }
        } else {
            // no sequence covers these tokens: their output is zero
            if (!ok(cudaMemsetAsync(slot + L.out, 0, nt * HV * V * 2, cs))) break;
        }
        ok(cudaEventRecord(pp.comp[r], cs));
        // 3. copy the segment's output back
        ok(cudaStreamWaitEvent(pp.down, pp.comp[r], 0));
        ok(cudaMemcpyAsync(static_cast<char*>(out) + s0 * HV * V * 2, slot + L.out, nt * HV * V * 2, d2h, pp.down));
        ok(cudaEventRecord(pp.d2h[r], pp.down));
    }
    if (status == GDN_OK && N > 0) {
        // zero-length sequences end with an all-zero state, like the single call
        for (int n = 0; n < N && status == GDN_OK;) {
            if (cu[n + 1] != cu[n]) {
                ++n;
                continue;
            }
            int e = n;
            while (e < N && cu[e + 1] == cu[e]) ++e;
            ok(cudaMemsetAsync(d_state + (size_t)n * HV * K * V, 0, (size_t)(e - n) * head_state, cs));
            n = e;
        }
        ok(cudaEventRecord(pp.comp[0], cs));
        ok(cudaStreamWaitEvent(pp.down, pp.comp[0], 0));
        ok(cudaMemcpyAsync(new_state, d_state, (size_t)N * head_state, d2h, pp.down));
    }
    // join: the caller's stream continues after the last copy back, even on an error
    const bool joined = cudaEventRecord(pp.comp[0], cs) == cudaSuccess &&
                        cudaStreamWaitEvent(pp.down, pp.comp[0], 0) == cudaSuccess &&
                        cudaEventRecord(pp.all_done, pp.down) == cudaSuccess &&
                        cudaStreamWaitEvent(cs, pp.all_done, 0) == cudaSuccess &&
                        cudaStreamWaitEvent(pp.up, pp.all_done, 0) == cudaSuccess;
    if (!joined && status == GDN_OK) status = GDN_ERR_CUDA;
    return status;
}
