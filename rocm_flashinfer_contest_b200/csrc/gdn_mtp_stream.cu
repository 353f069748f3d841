// gdn_mtp_stream.cu — persistent streaming form of the pool-indexed
// multi-token gated-delta-rule decode (T = 1 .. 8) for B200 (sm_100a).
//
// Same maths, API and semantics as the per-CTA kernels of gdn_mtp.cu (the
// contest's MTP definition, flashinfer/trace/templates/gdn.py:378-465, and
// flashinfer's gated_delta_rule_mtp, flashinfer/gdn_decode.py:557-745).  What
// changes is how the pool rows reach the SM.  A per-CTA kernel holds its block
// of state rows in registers from load to store, so while it computes it has
// no bytes in flight, and the more tokens an entry has, the fewer bytes an SM
// keeps in flight.  Here each CTA walks a contiguous range of work items (one
// item = ROWS state rows of one (entry, v-head)) through a ring of NS
// shared-memory stages:
//   * one producer warp fills stage i % NS with everything item i reads, up
//     to NS items ahead of the consumers: the state rows by one bulk copy
//     (cp.async.bulk on the TMA engine, no multicast, evict-first in L2;
//     completion counted in bytes on the stage's mbarrier) and the item's q / k
//     / v rows and gates by per-lane asynchronous copies (cp.async, 16 and 4
//     bytes; each lane's completion arrives on the same mbarrier), so the
//     producer never waits on a load;
//   * four consumer warps take the items in order: rows from the stage into
//     registers, the per-token quantities (q / k widened, norms, k.q, g, beta,
//     v) into a double-buffered token area, release of the stage (the producer
//     refills it at once), then the token loop: per token and row
//       sk = S.k, sq = S.q, delta = beta (v - g sk),
//       o = scale (g sq + delta k.q), S = g S + delta k
//     with the snapshots and the final rows stored straight from registers.
// So the state stream keeps running while the consumers compute.  Every
// mbarrier wait is bounded; a wait that runs out sets the translation unit's
// status word (read by gdn_device_status) and the CTA winds down: no further
// copies are issued and the producer waits (bounded) for those in flight
// before it exits.
#include <mutex>

#include "gdn_mtp_common.cuh"
#include "umma.cuh"

namespace gdn {
namespace mtp_stream {

constexpr int kConsumers = 128;            // four warps
constexpr int kThreads = kConsumers + 32;  // and one producer warp
constexpr int kMaxStages = 4;
constexpr long long kWaitBudget = 1ll << 27;  // SM clock cycles per wait (~70 ms)
constexpr int kMaxHV = 256;                   // A_log / dt_bias held in shared memory

// Byte offsets inside one stage; they depend on T, so they are computed on
// the host and passed in: the state rows (ROWS x 512 or 256 B, the bulk
// copy), then q and k rows (256 B per token), the item's v rows (T x ROWS x
// 2 B) and, per token, the aligned 4-byte words holding the bf16 gates a and b
// of the item's v-head (the half hv & 1 of each word).
struct StageLayout {
    uint32_t q, k, v, a, b, tx, bytes;  // tx: bytes of the bulk copy; bytes: stage stride
    int ns;                             // stages in the ring
};

inline StageLayout stage_layout(int rows, int elem, int T) {
    StageLayout L;
    L.tx = (uint32_t)rows * kDim * elem;
    L.q = L.tx;
    L.k = L.q + 256u * T;
    L.v = L.k + 256u * T;
    L.a = L.v + 2u * T * rows;
    L.b = L.a + 4u * kStreamMaxT;
    L.bytes = (L.b + 4u * kStreamMaxT + 127u) & ~127u;
    L.ns = kMaxStages;
    return L;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
// One arrival on the mbarrier once every cp.async this thread issued so far has
// landed (counted among the barrier's expected arrivals).
__device__ __forceinline__ void cp_async_arrive(uint64_t* mbar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(umma::smem_u32(mbar)) : "memory");
}

// This lane's share of item w's q / k / v rows and gates, copied into the stage
// at `st` (shared address): 16-byte words lane, lane + 32, ... of the q and k
// rows (vector 2t + (0 for q, 1 for k), 16 words each) and of the v rows, and
// for lane l < 2T the gate word of a_l (l < T) or b_{l-T}.
template <int TM, int ROWS>
__device__ __forceinline__ void copy_tokens(const MtpParams& p, int w, uint32_t st, const StageLayout& L, int lane) {
    constexpr int kBlocksPerHead = kDim / ROWS;
    constexpr int kVWords = (TM * ROWS / 8 + 31) / 32;
    const int T = p.T;
    const long long head = w / kBlocksPerHead;
    const int rb = w % kBlocksPerHead;
    const int bi = (int)(head / p.HV), hv = (int)(head % p.HV);
    const int hq = hv / p.rep;
    const size_t bt0 = (size_t)bi * T;
#pragma unroll
    for (int u = 0; u < TM; ++u) {
        const int wi = lane + 32 * u, vec = wi >> 4, t = vec >> 1;
        if (t < T)
            cp_async16(st + ((vec & 1) ? L.k : L.q) + 256 * t + 16 * (wi & 15),
                       ((vec & 1) ? p.k : p.q) + ((bt0 + t) * p.H + hq) * kDim + 8 * (wi & 15));
    }
#pragma unroll
    for (int u = 0; u < kVWords; ++u) {
        const int wi = lane + 32 * u, t = wi / (ROWS / 8);
        if (t < T)
            cp_async16(st + L.v + 16 * wi,
                       p.v + ((bt0 + t) * p.HV + hv) * kDim + (size_t)rb * ROWS + 8 * (wi % (ROWS / 8)));
    }
    if (lane < 2 * T) {
        const int t = lane < T ? lane : lane - T;
        const __nv_bfloat16* g = (lane < T ? p.a : p.b) + (((bt0 + t) * p.HV + hv) & ~(size_t)1);
        cp_async4(st + (lane < T ? L.a : L.b) + 4 * t, g);
    }
}

__device__ __forceinline__ float4 lds_f4(const unsigned char* p) { return *reinterpret_cast<const float4*>(p); }

// One lane's 16 values of state row `r` of the stage, widened.
__device__ __forceinline__ void stage_row(const unsigned char* st, int r, int sub, float4 (&x)[4], float) {
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = lds_f4(st + (size_t)r * kDim * 4 + 4 * mtp_col<float>(sub, j));
}
__device__ __forceinline__ void stage_row(const unsigned char* st, int r, int sub, float4 (&x)[4], __nv_bfloat16) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint4 raw = *reinterpret_cast<const uint4*>(st + (size_t)r * kDim * 2 + 2 * mtp_col<__nv_bfloat16>(sub, 2 * h));
        x[2 * h] = mtp_widen4(make_uint2(raw.x, raw.y));
        x[2 * h + 1] = mtp_widen4(make_uint2(raw.z, raw.w));
    }
}

template <int ROWS, typename StateT, int TM>
__global__ void __launch_bounds__(kThreads, 3)
    gdn_mtp_stream_kernel(const MtpParams p, const StageLayout L, int per_cta, int n_items) {
    constexpr int kRowsPerWarp = ROWS / 4;
    constexpr int kPasses = kRowsPerWarp / 4;
    constexpr int kBlocksPerHead = kDim / ROWS;
    static_assert(kPasses >= 1 && kRowsPerWarp % 4 == 0, "4 rows per warp pass");
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint64_t full[kMaxStages], empty[kMaxStages];
    __shared__ long long slot_of[kMaxStages];
    __shared__ volatile int abort_flag;
    __shared__ float s_alog[kMaxHV], s_dtb[kMaxHV];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int first = blockIdx.x * per_cta;
    const int count = min(n_items, first + per_cta) - first;
    const int T = p.T;
    const int NS = L.ns;

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            umma::mbar_init(&full[s], 33);  // the bulk copy's expect_tx arrive + one per producer lane
            umma::mbar_init(&empty[s], 4);  // one arrive per consumer warp
        }
        abort_flag = 0;
        umma::fence_mbar_init();
    }
    for (int h = tid; h < p.HV; h += kThreads) {
        s_alog[h] = p.A_log[h];
        s_dtb[h] = p.dt_bias[h];
    }
    __syncthreads();
    if (count <= 0) return;

    if (warp == 4) {
        // ---------------- producer ----------------
        long long cur_bi = -1, cur_slot = -1;
        const uint64_t read_once = umma::l2_evict_first_policy();
        // everything item j reads, into stage j % NS (free: fresh, or released)
        auto issue = [&](int j) {
            const int s = j % NS;
            const int w = first + j;
            const long long head = w / kBlocksPerHead;
            const int rb = w % kBlocksPerHead;
            const int bi = (int)(head / p.HV), hv = (int)(head % p.HV);
            if (bi != cur_bi) {
                cur_bi = bi;
                cur_slot = mtp_index(p.idx, p.idx64, bi);
            }
            const bool valid = cur_slot >= 0 && cur_slot < p.pool_size;
            const uint32_t st = umma::smem_u32(smem + (size_t)s * L.bytes);
            if (lane == 0) {
                slot_of[s] = cur_slot;  // published by the arrive (release) below
                umma::mbar_arrive_expect_tx(&full[s], valid ? L.tx : 0u);
                if (valid)
                    umma::bulk_g2s_hint(st,
                                        static_cast<const StateT*>(p.pool_in) +
                                            (((size_t)cur_slot * p.HV + hv) * kDim + (size_t)rb * ROWS) * kDim,
                                        L.tx, &full[s], read_once);
            }
            if (valid) copy_tokens<TM, ROWS>(p, w, st, L, lane);
            cp_async_arrive(&full[s]);
        };
        int issued = 0;
        for (; issued < min(NS, count); ++issued) issue(issued);
        for (int i = 0; issued < count; ++i) {
            // item i + NS goes into item i's stage once the consumers release it
            if (!umma::mbar_wait(&empty[i % NS], (i / NS) & 1, kWaitBudget) || abort_flag) {
                abort_flag = 1;
                break;
            }
            issue(issued++);
        }
        // no copy may still be landing in shared memory when the CTA exits
        asm volatile("cp.async.wait_all;" ::: "memory");
        if (lane == 0) {
            for (int j = max(0, issued - NS); j < issued; ++j)
                umma::mbar_wait(&full[j % NS], (j / NS) & 1, kWaitBudget);
        }
        return;
    }

    // ---------------- consumers ----------------
    // Each warp works through the items on its own: it reads its rows, the q /
    // k / v rows and the gates from the stage, forms the per-token scalars
    // itself (8-lane sums, as every row group of the warp holds whole q and k
    // vectors) and releases the stage with its own arrive once it is done with
    // it.  No barrier joins the warps.
    const int sub = lane & 7, rsub = lane >> 3;
    const int lrow = warp * kRowsPerWarp + rsub;  // this lane's first row within the item
    const bool upper = (sub & 4) != 0;
    for (int i = 0; i < count; ++i) {
        const int s = i % NS;
        if (!umma::mbar_wait(&full[s], (i / NS) & 1, kWaitBudget)) {
            abort_flag = 1;
            break;
        }
        const unsigned char* st = smem + (size_t)s * L.bytes;
        const long long slot = slot_of[s];
        const int w = first + i;
        const long long head = w / kBlocksPerHead;
        const int rb = w % kBlocksPerHead;
        const int bi = (int)(head / p.HV), hv = (int)(head % p.HV);
        const int row_base = rb * ROWS + lrow;
        const size_t bt0 = (size_t)bi * T;
        if (!(slot >= 0 && slot < p.pool_size)) {  // padding entry: zero output, no state read or written
            __syncwarp();
            if (lane == 0) umma::mbar_arrive_expect_tx(&empty[s], 0u);
            if (sub == 0) {
                for (int t = 0; t < T; ++t) {
                    const size_t ob = ((bt0 + t) * p.HV + hv) * kDim + row_base;
#pragma unroll
                    for (int ps = 0; ps < kPasses; ++ps) p.out[ob + ps * 4] = __float2bfloat16_rn(0.0f);
                }
            }
            continue;
        }
        float4 x[kPasses][4];
#pragma unroll
        for (int ps = 0; ps < kPasses; ++ps) stage_row(st, lrow + 4 * ps, sub, x[ps], StateT());
        const size_t row_off = (size_t)row_base * kDim;
        const long long snap_row = mtp_snap_row(p, bi, slot);
        const long long oslot = p.out_idx != nullptr ? mtp_index(p.out_idx, p.idx64, bi) : slot;
        // lane t < T forms token t's gate and beta once; the token loop takes
        // them by shuffle instead of every lane recomputing them per token
        float g_lane = 1.f, beta_lane = 0.f;
        if (lane < T) {
            const float ga = bf16_to_f32(reinterpret_cast<const __nv_bfloat16*>(st + L.a + 4 * lane)[hv & 1]);
            const float gb = bf16_to_f32(reinterpret_cast<const __nv_bfloat16*>(st + L.b + 4 * lane)[hv & 1]);
            g_lane = expf(log_gate(s_alog[hv], ga, s_dtb[hv]));
            beta_lane = sigmoidf_(gb);
        }
        for (int t = 0; t < T; ++t) {
            float4 kf[4], qf[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int c = mtp_col<StateT>(sub, j);
                kf[j] = mtp_widen4(*reinterpret_cast<const uint2*>(st + L.k + 256 * t + 2 * c));
                qf[j] = mtp_widen4(*reinterpret_cast<const uint2*>(st + L.q + 256 * t + 2 * c));
            }
            const float g = __shfl_sync(0xffffffffu, g_lane, t);
            const float beta = __shfl_sync(0xffffffffu, beta_lane, t);
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
            const __nv_bfloat16* sv = reinterpret_cast<const __nv_bfloat16*>(st + L.v) + ROWS * t;
            const size_t ob = ((bt0 + t) * p.HV + hv) * kDim + row_base;
            float* snap_dst =
                snap_row >= 0 ? p.inter + (((size_t)snap_row + t) * p.HV + hv) * kDim * kDim + row_off : nullptr;
#pragma unroll
            for (int ps = 0; ps < kPasses; ++ps) {
                float2 sk2 = make_float2(0.f, 0.f), sq2 = make_float2(0.f, 0.f);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    sk2 = dot4_acc2(x[ps][j], kf[j], sk2);
                    sq2 = dot4_acc2(x[ps][j], qf[j], sq2);
                }
                const float sk = sk2.x + sk2.y, sq = sq2.x + sq2.y;
                float give = upper ? sk : sq;
                float keep = upper ? sq : sk;
                keep += __shfl_xor_sync(0xffffffffu, give, 4);
                keep += __shfl_xor_sync(0xffffffffu, keep, 1);
                keep += __shfl_xor_sync(0xffffffffu, keep, 2);
                // keep == full sk on lanes sub < 4, full sq on lanes sub >= 4
                const float sk_all = __shfl_sync(0xffffffffu, keep, lane & ~4);
                const float delta = beta * (bf16_to_f32(sv[lrow + 4 * ps]) - g * sk_all);
                if (sub == 4) stg_bf16(p.out + ob + ps * 4, p.scale * (g * keep + delta * kq));
#pragma unroll
                for (int j = 0; j < 4; ++j) x[ps][j] = gs_plus_dk(g, x[ps][j], delta, kf[j]);
                if constexpr (sizeof(StateT) == 4) {  // snapshots exist for fp32 pools only
                    if (snap_dst != nullptr) mtp_store_row(snap_dst, (size_t)ps * 4 * kDim, sub, x[ps]);
                }
            }
        }
        __syncwarp();  // every lane is done with the stage
        if (lane == 0) umma::mbar_arrive_expect_tx(&empty[s], 0u);
        if (p.pool_out != nullptr && oslot >= 0 && oslot < p.pool_size) {
            StateT* pout = static_cast<StateT*>(p.pool_out);
            const size_t obase = ((size_t)oslot * p.HV + hv) * kDim * kDim + row_off;
#pragma unroll
            for (int ps = 0; ps < kPasses; ++ps) mtp_store_row(pout, obase + (size_t)ps * 4 * kDim, sub, x[ps]);
        }
    }
}

// Launch geometry of one instantiation on the current device: CTAs per SM
// for a given dynamic shared-memory size, from the kernel's registers and the
// device's shared memory (queried once per instantiation and device).
struct KernelInfo {
    int regs = 0, static_smem = 0, sms = 0, smem_sm = 0, smem_optin = 0;
    bool ok = false;
    // the driver's resident-CTA count per dynamic shared-memory size seen
    size_t occ_smem[8] = {};
    int occ_ctas[8] = {};
};

template <int ROWS, typename StateT, int TM>
static std::mutex& kernel_info_mutex() {
    static std::mutex mu;
    return mu;
}

template <int ROWS, typename StateT, int TM>
static const KernelInfo& kernel_info() {
    std::mutex& mu = kernel_info_mutex<ROWS, StateT, TM>();
    static KernelInfo info[16];
    static bool done[16] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 16) {
        static KernelInfo none;
        return none;
    }
    std::lock_guard<std::mutex> lk(mu);
    if (!done[dev]) {  // set once the queries succeed (a failed attempt is retried on the next call)
        KernelInfo& k = info[dev];
        cudaFuncAttributes fa;
        auto fn = gdn_mtp_stream_kernel<ROWS, StateT, TM>;
        if (cudaFuncGetAttributes(&fa, fn) == cudaSuccess &&
            cudaDeviceGetAttribute(&k.sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
            cudaDeviceGetAttribute(&k.smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) == cudaSuccess &&
            cudaDeviceGetAttribute(&k.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) == cudaSuccess) {
            k.regs = fa.numRegs;
            k.static_smem = (int)fa.sharedSizeBytes;
            // all of the unified L1 / shared memory as shared memory, so that as
            // many rings fit on an SM as the registers allow
            k.ok = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        k.smem_optin - k.static_smem) == cudaSuccess &&
                   cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                                        (int)cudaSharedmemCarveoutMaxShared) == cudaSuccess;
        }
        cudaGetLastError();
        done[dev] = k.ok;
    }
    return info[dev];
}

template <int ROWS, typename StateT, int TM>
static int launch(const MtpParams& p, int B, cudaStream_t st) {
    const KernelInfo& k = kernel_info<ROWS, StateT, TM>();
    if (!k.ok) return 1;
    StageLayout L = stage_layout(ROWS, (int)sizeof(StateT), p.T);
    const int by_regs = 65536 / (kThreads * ((k.regs + 7) & ~7));
    // the deepest ring (3 or 4 stages) at the most CTAs per SM: more consumer
    // warps per SM first, then more stages
    int per_sm = 0;
    size_t smem = 0;
    for (int ns = kMaxStages; ns >= 3; --ns) {
        const size_t b = (size_t)ns * L.bytes;
        if ((int)b + k.static_smem > k.smem_optin) continue;
        const int n = min(by_regs, k.smem_sm / ((int)b + k.static_smem + 1024));  // 1 KiB reserved per CTA
        if (n > per_sm) {
            per_sm = n;
            smem = b;
            L.ns = ns;
        }
    }
    if (per_sm < 1) return 1;
    // the driver's count for the chosen size, which the grid must not exceed
    // (asked once per size and cached: no runtime query on later calls, which
    // may be inside a graph capture)
    int resident = 0;
    {
        std::lock_guard<std::mutex> lk(kernel_info_mutex<ROWS, StateT, TM>());
        KernelInfo& km = const_cast<KernelInfo&>(k);
        int slot = -1;
        for (int e = 0; e < 8; ++e) {
            if (km.occ_smem[e] == smem) {
                resident = km.occ_ctas[e];
                break;
            }
            if (km.occ_smem[e] == 0 && slot < 0) slot = e;
        }
        if (resident == 0) {
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, gdn_mtp_stream_kernel<ROWS, StateT, TM>,
                                                              kThreads, smem) != cudaSuccess) {
                cudaGetLastError();
                return 1;
            }
            if (slot >= 0) {
                km.occ_smem[slot] = smem;
                km.occ_ctas[slot] = resident;
            }
        }
    }
    per_sm = min(per_sm, resident);
    if (per_sm < 1) return 1;
    const long long n_items = (long long)B * p.HV * (kDim / ROWS);
    const long long slots = (long long)k.sms * per_sm;
    const int per_cta = (int)((n_items + slots - 1) / slots);
    const unsigned grid = (unsigned)((n_items + per_cta - 1) / per_cta);
    gdn_mtp_stream_kernel<ROWS, StateT, TM><<<grid, kThreads, smem, st>>>(p, L, per_cta, (int)n_items);
    return gdn_launch_status();
}

}  // namespace mtp_stream

int launch_mtp_stream(const MtpParams& p, int B, bool state_bf16, cudaStream_t st) {
    // HV even: a gate word (two bf16 of one v-head pair) never reaches past the array
    if (p.T < 1 || p.T > kStreamMaxT || p.HV > mtp_stream::kMaxHV || p.HV % 2 != 0) return 1;
    if (!gdn_aligned(p.q, 16) || !gdn_aligned(p.k, 16) || !gdn_aligned(p.v, 16) || !gdn_aligned(p.a, 4) ||
        !gdn_aligned(p.b, 4))
        return 1;
    if ((long long)B * p.HV * (kDim / 32) >= (1ll << 31)) return 1;
    if (state_bf16) {
        return p.T == 1   ? mtp_stream::launch<32, __nv_bfloat16, 1>(p, B, st)
               : p.T <= 4 ? mtp_stream::launch<32, __nv_bfloat16, 4>(p, B, st)
                          : mtp_stream::launch<32, __nv_bfloat16, kStreamMaxT>(p, B, st);
    }
    return p.T == 1   ? mtp_stream::launch<32, float, 1>(p, B, st)
           : p.T <= 4 ? mtp_stream::launch<32, float, 4>(p, B, st)
                      : mtp_stream::launch<32, float, kStreamMaxT>(p, B, st);
}

int mtp_stream_status(bool clear) {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_status, sizeof(v)) != cudaSuccess) return -1;
    if (clear && v) {
        const unsigned int z = 0;
        if (cudaMemcpyToSymbol(g_device_status, &z, sizeof(z)) != cudaSuccess) return -1;
    }
    return (int)v;
}

}  // namespace gdn
