// gdn_prefill_noalloc.cu — the varlen prefill for callers that cannot allocate
// device memory.
//
// gdn_prefill_fwd needs a device workspace for its chunked kernels, which a
// caller normally gets from its own allocator.  Some callers have none to use
// at this point: a host that binds the C ABI directly (cgo, JNI, a plain C
// serving loop) without a caching allocator, where cudaMalloc would be slow
// and may synchronise the device in the middle of a latency-critical step,
// or a runtime whose memory is carved up once at start-up and forbids later
// allocations.  gdn_prefill_fwd_noalloc serves them from a fixed scratch
// array that this library defines at file scope: it exists on every device
// that loads the library and stays there until the process exits.
#include <mutex>

#include "gdn_prefill_common.cuh"

namespace {

constexpr size_t kScratchBytes = (size_t)16 << 20;  // 16 MiB
constexpr int kMaxDevices = 64;

// The workspace of gdn_prefill_fwd_noalloc.  Host code must not use this name
// as a device address (on the host it names a stand-in object); it asks the
// runtime for the device address once per device instead.
static __device__ __align__(256) unsigned char g_prefill_scratch[kScratchBytes];

std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_prefill_scratch on the current device, looked up on the
// first call made with that device current and cached afterwards.  A
// cudaDeviceReset() tears down the context that holds the array, so the
// cached address is stale afterwards: the header says so.
int scratch_on_current_device(void** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return GDN_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_scratch_addr[dev] == nullptr) {
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_prefill_scratch) != cudaSuccess || ptr == nullptr)
            return GDN_ERR_CUDA;
        g_scratch_addr[dev] = ptr;
    }
    *out = g_scratch_addr[dev];
    return GDN_OK;
}

}  // namespace

extern "C" int gdn_prefill_fwd_noalloc(const void* q, const void* k, const void* v, const float* state,
                                       const float* A_log, const void* a, const float* dt_bias,
                                       const void* b, const void* cu_seqlens, int cu_seqlens_is_int64,
                                       int N, int T, float scale, int H, int HV, int K, int V, void* out,
                                       float* new_state, void* stream) {
    // argument errors rank before the size check, as for every other prefill
    // entry point; neither makes a CUDA call
    const int chk = gdn::prefill_check_args(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, cu_seqlens_is_int64,
                                            N, T, H, HV, K, V, out, new_state);
    if (chk != GDN_OK) return chk;
    if (gdn::prefill_workspace_bytes_split(N, T, H, HV) > kScratchBytes) return GDN_ERR_TOO_LARGE;
    if (N == 0 && T == 0) return GDN_OK;
    void* scratch = nullptr;
    const int st = scratch_on_current_device(&scratch);
    if (st != GDN_OK) return st;
    return gdn::prefill_fwd_one_stream(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, cu_seqlens_is_int64, N, T,
                                       scale, H, HV, K, V, out, new_state, scratch, kScratchBytes, stream);
}
