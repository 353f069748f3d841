/*
 * CPU oracle for the gated-delta-rule (GDN) decode and prefill paths.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the CUDA kernels are
 * compared against, and the CPU baseline that bench.py times beside them.  No
 * product code path may call it.
 *
 * It restates, in plain C with fp32 arithmetic, the contest's pure-torch
 * reference that the reference repository is scored against
 * (jhinpan/rocm-flashinfer-contest: tools/local_verify.py:94,108 builds and runs
 * it; the definitions live in the third-party package flashinfer-python
 * 0.6.11.post2, flashinfer/trace/templates/gdn.py).  Per step and per v-head:
 *
 *   x     = a + dt_bias                              gdn.py:51 / :214
 *   g     = exp(-exp(A_log) * softplus(x))           gdn.py:52 / :215
 *           softplus(x) = x if x > 20 else log1p(exp(x))   (torch default,
 *           threshold 20; also solutions/gdn_decode/main.py:82-84)
 *   beta  = sigmoid(b)                               gdn.py:53 / :216
 *   GVA   : v-head h reads q/k head h / (HV / H)     gdn.py:66-67 / :218-219
 *   with S the state as [K][V] (stored k-last, [V][K]):
 *     old    = g * S                                 gdn.py:83 / :256
 *     old_v  = k^T old          (per v)              gdn.py:84 / :258
 *     new_v  = beta*v + (1-beta)*old_v               gdn.py:85 / :259
 *     S      = old - k (x) old_v + k (x) new_v       gdn.py:86-88 / :260-266
 *     o      = scale * q^T S    -> bf16               gdn.py:90,93 / :268-269
 *   prefill: sequences delimited by cu_seqlens; a zero-length sequence keeps
 *   an all-zero final state even when an initial state is given (gdn.py:234-235);
 *   the output is rounded to bf16 per token (gdn.py:269).
 *
 * Parity of this restatement is pinned by tests/golden/ (fixtures generated
 * from the flashinfer reference by tests/golden/make_golden.py).
 *
 * Layouts are the contest's, all contiguous:
 *   decode : q,k [B,H,K]; v [B,HV,V]; state/new_state [B,HV,V,K]; a,b [B,HV];
 *            out [B,HV,V]
 *   prefill: q,k [T,H,K]; v [T,HV,V]; a,b [T,HV]; cu_seqlens [N+1] (int64);
 *            state/new_state [N,HV,V,K]; out [T,HV,V]
 * bf16 inputs are passed widened to fp32 (exact); the output is returned as
 * bf16 bit patterns (round to nearest even, as torch's .to(bfloat16)).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static uint16_t f32_to_bf16_rne(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) {
        return (uint16_t)((u >> 16) | 0x0040u); /* quiet NaN */
    }
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

static float softplus_t20(float x) {
    /* torch.nn.functional.softplus(x, beta=1, threshold=20) */
    return x > 20.0f ? x : log1pf(expf(x));
}

static void gates(float A_log, float a, float dt_bias, float b, float *g, float *beta) {
    float x = a + dt_bias;
    *g = expf(-expf(A_log) * softplus_t20(x));
    *beta = 1.0f / (1.0f + expf(-b));
}

/* One token of the recurrence for one v-head, updating the k-last [V][K] state
 * S in place.  Writes scale * q^T S_new (fp32, V values) into o. */
static void step_head(float *S, const float *q, const float *k, const float *v,
                      float g, float beta, float scale, int K, int V, float *o) {
    for (int vi = 0; vi < V; ++vi) {
        float *row = S + (size_t)vi * K;
        float old_v = 0.0f;
        for (int ki = 0; ki < K; ++ki) {
            row[ki] *= g; /* old = g * S */
            old_v += k[ki] * row[ki];
        }
        float new_v = beta * v[vi] + (1.0f - beta) * old_v;
        float acc = 0.0f;
        for (int ki = 0; ki < K; ++ki) {
            row[ki] = row[ki] - k[ki] * old_v + k[ki] * new_v;
            acc += q[ki] * row[ki];
        }
        o[vi] = scale * acc;
    }
}

static int resolve_threads(int nthreads) {
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
    return nthreads;
#else
    (void)nthreads;
    return 1;
#endif
}

int gdn_oracle_decode(const float *q, const float *k, const float *v, const float *state,
                      const float *A_log, const float *a, const float *dt_bias,
                      const float *b, float scale, int B, int H, int HV, int K, int V,
                      uint16_t *out_bf16, float *out_f32, float *new_state, int nthreads) {
    if (B < 0 || H <= 0 || HV <= 0 || K <= 0 || V <= 0 || HV % H) return 1;
    if (scale == 0.0f) scale = 1.0f / sqrtf((float)K);
    const int rep = HV / H;
    const long long heads = (long long)B * HV;
    nthreads = resolve_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads)
    for (long long bh = 0; bh < heads; ++bh) {
        int bi = (int)(bh / HV), h = (int)(bh % HV), hq = h / rep;
        float *S = new_state + (size_t)bh * V * K;
        if (state) memcpy(S, state + (size_t)bh * V * K, sizeof(float) * (size_t)V * K);
        else memset(S, 0, sizeof(float) * (size_t)V * K);
        float g, beta;
        gates(A_log[h], a[bh], dt_bias[h], b[bh], &g, &beta);
        float *o = (float *)malloc(sizeof(float) * V);
        step_head(S, q + ((size_t)bi * H + hq) * K, k + ((size_t)bi * H + hq) * K,
                  v + (size_t)bh * V, g, beta, scale, K, V, o);
        for (int vi = 0; vi < V; ++vi) {
            out_bf16[(size_t)bh * V + vi] = f32_to_bf16_rne(o[vi]);
            if (out_f32) out_f32[(size_t)bh * V + vi] = o[vi];
        }
        free(o);
    }
    return 0;
}

/* q/k L2 normalisation, x / sqrt(sum(x^2) + 1e-6) (on == 0: a plain copy). */
static void l2norm_copy(float *dst, const float *src, int K, int on) {
    float ss = 0.0f;
    for (int i = 0; i < K; ++i) ss += src[i] * src[i];
    float inv = on ? 1.0f / sqrtf(ss + 1e-6f) : 1.0f;
    for (int i = 0; i < K; ++i) dst[i] = src[i] * inv;
}

/* ckpt (optional): the state after tokens every, 2*every, ... of sequence n
 * is copied to ckpt[ckpt_cu[n] + i] (flashinfer's chunk_gated_delta_rule
 * checkpoints, flashinfer/gdn_prefill.py:161-174).  qk_l2norm != 0 first
 * normalises each q and k head vector (l2norm_copy): the option
 * use_qk_l2norm_in_kernel of the AITER kernels the reference calls
 * (solutions/gdn_prefill/main.py:72,79, there False), whose rule is FLA's
 * l2norm, 1 / sqrt(sum(x^2) + eps) with eps = 1e-6 (fla/modules/l2norm.py:42,140). */
int gdn_oracle_prefill(const float *q, const float *k, const float *v, const float *state,
                       const float *A_log, const float *a, const float *dt_bias,
                       const float *b, const int64_t *cu_seqlens, int N, int T, float scale,
                       int H, int HV, int K, int V, uint16_t *out_bf16, float *new_state,
                       float *ckpt, const int64_t *ckpt_cu, int every, int qk_l2norm,
                       int nthreads) {
    if (ckpt && (every <= 0 || !ckpt_cu)) return 1;
    if (N < 0 || T < 0 || H <= 0 || HV <= 0 || K <= 0 || V <= 0 || HV % H) return 1;
    if (N > 0 && (cu_seqlens[0] < 0 || cu_seqlens[N] > T)) return 1;
    for (int n = 0; n < N; ++n)
        if (cu_seqlens[n + 1] < cu_seqlens[n]) return 1;
    if (scale == 0.0f) scale = 1.0f / sqrtf((float)K);
    const int rep = HV / H;
    /* tokens outside every sequence keep a zero output, as the reference's
     * torch.zeros output buffer does (gdn.py:221-223) */
    memset(out_bf16, 0, sizeof(uint16_t) * (size_t)T * HV * V);
    nthreads = resolve_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads)
    for (long long nh = 0; nh < (long long)N * HV; ++nh) {
        int n = (int)(nh / HV), h = (int)(nh % HV), hq = h / rep;
        float *S = new_state + (size_t)nh * V * K;
        int64_t t0 = cu_seqlens[n], t1 = cu_seqlens[n + 1];
        if (t1 - t0 <= 0) { /* gdn.py:234-235: state stays zero */
            memset(S, 0, sizeof(float) * (size_t)V * K);
            continue;
        }
        if (state) memcpy(S, state + (size_t)nh * V * K, sizeof(float) * (size_t)V * K);
        else memset(S, 0, sizeof(float) * (size_t)V * K);
        float *o = (float *)malloc(sizeof(float) * V);
        float *qn = (float *)malloc(sizeof(float) * K), *kn = (float *)malloc(sizeof(float) * K);
        for (int64_t t = t0; t < t1; ++t) {
            float g, beta;
            gates(A_log[h], a[(size_t)t * HV + h], dt_bias[h], b[(size_t)t * HV + h], &g, &beta);
            l2norm_copy(qn, q + ((size_t)t * H + hq) * K, K, qk_l2norm);
            l2norm_copy(kn, k + ((size_t)t * H + hq) * K, K, qk_l2norm);
            step_head(S, qn, kn, v + ((size_t)t * HV + h) * V, g, beta, scale, K, V, o);
            for (int vi = 0; vi < V; ++vi)
                out_bf16[((size_t)t * HV + h) * V + vi] = f32_to_bf16_rne(o[vi]);
            if (ckpt && (t - t0 + 1) % every == 0) {
                int64_t ci = ckpt_cu[n] + (t - t0 + 1) / every - 1;
                memcpy(ckpt + ((size_t)ci * HV + h) * V * K, S, sizeof(float) * (size_t)V * K);
            }
        }
        free(o);
        free(qn);
        free(kn);
    }
    return 0;
}

/* Multi-token decode over a state pool: the contest's MTP definition
 * (flashinfer/trace/templates/gdn.py:378-460, _gdn_mtp_reference).  pool_out
 * starts as a copy of pool_in (gdn.py:425); batch entry i advances the state
 * pool_in[idx[i]] over its T tokens (gdn.py:427-455), writing the bf16 output
 * of every token and, when `inter` is given, the state after every token to
 * inter[idx[i], t] (gdn.py:457-460); the final state goes to pool_out[idx[i]]
 * (gdn.py:463).  An index outside [0, pool_size) marks a padding entry: its
 * output is zero and no state is touched (the serving kernels' -1 padding
 * convention; the torch template would wrap negative indices instead).
 * `inter` has `cache_steps` (>= T) token slots per pool slot.
 * qk_l2norm != 0 first normalises each q and k head vector as
 * x / sqrt(sum(x^2) + 1e-6), the in-kernel option `use_qk_l2norm` of
 * flashinfer's gated_delta_rule_mtp (flashinfer/gdn_decode.py:571; the
 * kernel's rsqrt(sum + 1e-6), gdn_kernels/gdn_decode_mtp.py:359-360).
 * out_idx (NULL: idx) names the slot each entry's final state is written to
 * (`output_state_indices`, flashinfer/gdn_decode.py:176-181); an out-of-range
 * output slot skips the write.  round_bf16 != 0 is the bf16-state form
 * (gdn_decode.py:206-260): pool_in holds bf16 values (widened), the state is
 * advanced in fp32 and rounded to bf16 (nearest even) once, when stored. */
static float round_bf16(float f) {
    uint32_t u = (uint32_t)f32_to_bf16_rne(f) << 16;
    float r;
    memcpy(&r, &u, 4);
    return r;
}

int gdn_oracle_mtp(const float *q, const float *k, const float *v, const float *pool_in,
                   float *pool_out, const int64_t *idx, const int64_t *out_idx, const float *A_log,
                   const float *a, const float *dt_bias, const float *b, float scale, int B, int T,
                   int H, int HV, int K, int V, int pool_size, int round_bf16_state, int qk_l2norm,
                   uint16_t *out_bf16, float *inter, int cache_steps, long long inter_rows,
                   int snap_by_entry, int nthreads) {
    if (B < 0 || T < 0 || H <= 0 || HV <= 0 || K <= 0 || V <= 0 || HV % H || pool_size < 0) return 1;
    if (inter && (cache_steps < T || inter_rows < 0)) return 1;
    if (scale == 0.0f) scale = 1.0f / sqrtf((float)K);
    const int rep = HV / H;
    const size_t head = (size_t)V * K;
    if (pool_out != pool_in) memcpy(pool_out, pool_in, sizeof(float) * (size_t)pool_size * HV * head);
    memset(out_bf16, 0, sizeof(uint16_t) * (size_t)B * T * HV * V);
    nthreads = resolve_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads)
    for (long long bh = 0; bh < (long long)B * HV; ++bh) {
        int bi = (int)(bh / HV), h = (int)(bh % HV), hq = h / rep;
        int64_t slot = idx[bi];
        if (slot < 0 || slot >= pool_size) continue;
        /* first snapshot row of this entry, or -1: an entry's T rows are
         * written whole or not at all (by pool slot: inter[slot, t]; by entry:
         * row bi * T + t, flashinfer's CuTe kernel, gdn_decode_mtp.py:645) */
        long long row0 = -1;
        if (inter) {
            long long r = snap_by_entry ? (long long)bi * T : (long long)slot * cache_steps;
            long long need = snap_by_entry ? (long long)T : (long long)cache_steps;
            if (r + need <= inter_rows) row0 = r;
        }
        float *S = (float *)malloc(sizeof(float) * head);
        memcpy(S, pool_in + ((size_t)slot * HV + h) * head, sizeof(float) * head);
        float *o = (float *)malloc(sizeof(float) * (V + 2 * K));
        float *qn = o + V, *kn = o + V + K;
        for (int t = 0; t < T; ++t) {
            size_t bt = (size_t)bi * T + t;
            float g, beta;
            gates(A_log[h], a[bt * HV + h], dt_bias[h], b[bt * HV + h], &g, &beta);
            l2norm_copy(qn, q + (bt * H + hq) * K, K, qk_l2norm);
            l2norm_copy(kn, k + (bt * H + hq) * K, K, qk_l2norm);
            step_head(S, qn, kn, v + (bt * HV + h) * V, g, beta, scale, K, V, o);
            for (int vi = 0; vi < V; ++vi) out_bf16[(bt * HV + h) * V + vi] = f32_to_bf16_rne(o[vi]);
            if (row0 >= 0)
                memcpy(inter + (((size_t)row0 + t) * HV + h) * head, S, sizeof(float) * head);
        }
        int64_t oslot = out_idx ? out_idx[bi] : slot;
        if (oslot >= 0 && oslot < pool_size) {
            float *dst = pool_out + ((size_t)oslot * HV + h) * head;
            for (size_t e = 0; e < head; ++e) dst[e] = round_bf16_state ? round_bf16(S[e]) : S[e];
        }
        free(o);
        free(S);
    }
    return 0;
}
