/*
 * gdn_b200.h — C ABI of the B200 (sm_100a) gated-delta-rule (GDN) kernels.
 *
 * These entry points are the drop-in boundary under the contest solutions'
 * Python `run(...)` functions.  They take plain device pointers, sizes and a
 * CUDA stream (passed as void*), allocate nothing (the prefill's scratch is a
 * caller-provided workspace), never synchronise the host, and return a
 * status code (GDN_OK == 0); argument errors are reported before anything is
 * launched.
 *
 * Layouts (all contiguous, k-last state as in the contest definitions
 * gdn_decode_*_k_last / gdn_prefill_*_k_last):
 *   decode : q,k [B,1,H,K] bf16; v [B,1,HV,V] bf16; a,b [B,1,HV] bf16;
 *            A_log,dt_bias [HV] fp32; state/new_state [B,HV,V,K] fp32;
 *            out [B,1,HV,V] bf16
 *   prefill: q,k [T,H,K] bf16; v [T,HV,V] bf16; a,b [T,HV] bf16;
 *            cu_seqlens [N+1] int32 or int64; state/new_state [N,HV,V,K] fp32;
 *            out [T,HV,V] bf16
 *   mtp    : q,k [B,T,H,K] bf16; v [B,T,HV,V] bf16; a,b [B,T,HV] bf16;
 *            pool [pool_size,HV,V,K] fp32 or bf16; indices [B] int32 or int64;
 *            intermediate [inter_slots,cache_steps,HV,V,K] fp32; out [B,T,HV,V] bf16
 * Supported sizes: K == V == 128, H >= 1, HV % H == 0 (v-head h reads q/k head
 * h / (HV/H)).  `state` may be NULL (zero initial state).  `scale` == 0 means
 * 1/sqrt(K).  Decode: pointers to q and k must be 8-byte aligned; prefill:
 * q, k, v and out 16-byte aligned; state pointers 16-byte aligned always.
 */
#ifndef GDN_B200_H_
#define GDN_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GDN_OK 0
#define GDN_ERR_INVALID 1     /* null pointer, negative size, bad flag        */
#define GDN_ERR_UNSUPPORTED 2 /* K != 128, V != 128, HV % H != 0              */
#define GDN_ERR_ALIGN 3       /* a pointer violates the alignment above       */
#define GDN_ERR_CUDA 4        /* the launch failed (cudaGetLastError)         */
#define GDN_ERR_DEVICE 5      /* a kernel reported an error (bounded wait timed out) */
#define GDN_ERR_TOO_LARGE 6   /* needs more than gdn_prefill_fwd_noalloc's fixed scratch */

/* flags of gdn_mtp_fwd */
#define GDN_MTP_QK_L2NORM 1          /* normalise q and k in the kernel */
#define GDN_MTP_SNAPSHOTS_BY_ENTRY 2 /* intermediate states indexed by batch entry, not pool slot */

/* flags of gdn_prefill_fwd_ex */
#define GDN_PREFILL_QK_L2NORM 1 /* normalise q and k in the kernel: x * rsqrt(sum(x^2) + 1e-6) */

/* Version of this ABI (bumped on any signature change or addition; 3 adds
 * gdn_mtp_fwd and gdn_prefill_fwd_checkpointed, 4 gdn_decode_fwd_host,
 * gdn_prefill_fwd_host, gdn_prefill_fwd_ex and gdn_mtp_fwd's flags word). */
int gdn_abi_version(void);

/* Human-readable text for a status code. */
const char *gdn_strerror(int status);

/* Error bits recorded by the prefill kernels and the streaming multi-token
 * decode kernel since the last clear (1 = a bounded wait on an mbarrier timed
 * out); synchronises the device.  clear != 0 resets the word.  Returns -1 if
 * it cannot be read. */
int gdn_device_status(int clear);

/*
 * One decode step (one token per sequence) for B sequences.
 *
 * Replaces the reference solution's kernel launch `_run_klast`
 * (solutions/gdn_decode/main.py:97-114) behind `run` (main.py:117-135); the
 * maths is the contest definition gdn_decode_*_k_last
 * (flashinfer/trace/templates/gdn.py:27-94).
 *
 * new_state may equal state (in-place update); any other overlap between
 * inputs and outputs is not allowed.
 */
int gdn_decode_fwd(const void *q, const void *k, const void *v, const float *state,
                   const float *A_log, const void *a, const float *dt_bias, const void *b,
                   float scale, int B, int H, int HV, int K, int V, void *out,
                   float *new_state, void *stream);

/*
 * gdn_decode_fwd with every operand in HOST memory (q .. b, state, out and
 * new_state host pointers; pinned memory for the copies to overlap): for a
 * caller that keeps the recurrent states off the device between steps.  No
 * counterpart in the reference, whose `run` takes device tensors
 * (solutions/gdn_decode/main.py:117-135); the results are bit-identical to
 * gdn_decode_fwd on device copies of the same inputs.
 *
 * The batch is cut into `chunks` slices (0: about 16 MiB of state each, at
 * most 16).  Slice c is copied up and advanced on `stream` while slice c - 1
 * is copied back on a stream this library creates per device (with two
 * events, on the first call); `stream` is made to wait for the last copy
 * back, so work queued on it afterwards (or a synchronisation of it) sees
 * the results in `out` and `new_state`.  The state is advanced in place in
 * `workspace` (device memory, 256-byte aligned, at least
 * gdn_decode_host_workspace_bytes(B, H, HV) bytes; contents on entry do not
 * matter), and each call first waits for the previous call's copies back on
 * this device, so calls may reuse one workspace from any stream.  new_state
 * may equal state.  Host enqueue is serialised per process by a mutex.  Not
 * for use inside a stream capture.
 */
int gdn_decode_fwd_host(const void *q, const void *k, const void *v, const float *state,
                        const float *A_log, const void *a, const float *dt_bias, const void *b,
                        float scale, int B, int H, int HV, int K, int V, void *out,
                        float *new_state, void *workspace, size_t workspace_bytes, int chunks,
                        void *stream);

/* Device workspace bytes gdn_decode_fwd_host needs for (B, H, HV) with
 * K == V == 128: one copy of the state plus the step's inputs and outputs. */
size_t gdn_decode_host_workspace_bytes(int B, int H, int HV);

/*
 * Variable-length prefill over N sequences packed into T tokens.
 *
 * Replaces the body of the reference solution's `run`
 * (solutions/gdn_prefill/main.py:31-84: host gates, state transposes and the
 * AITER chunk / recurrent kernels); the maths is the contest definition
 * gdn_prefill_*_k_last (flashinfer/trace/templates/gdn.py:189-273).
 *
 * cu_seqlens is read on the device only.  A zero-length sequence gets an
 * all-zero new_state (gdn.py:234-235); tokens outside [cu_seqlens[0],
 * cu_seqlens[N]) get a zero output.  Entries are clamped to [0, T] so a
 * malformed cu_seqlens cannot make the kernel read or write out of bounds.
 * new_state may equal state (in-place update).
 *
 * T >= GDN_PREFILL_CHUNK_MIN (environment, default 128) runs the chunked
 * tensor-core kernels, which need a device workspace (16-byte aligned; its
 * contents on entry do not matter) of gdn_prefill_workspace_bytes(N, T, H, HV)
 * bytes; a smaller one of at least (floor(T/64) + N) * (17,424 * HV + 49,152 * H)
 * bytes restricts the call to the kernels whose layout fits it.  Shorter
 * batches run the token-serial kernel and need none (workspace may then be
 * NULL).  For one sequence the call may run part of its work on two library
 * streams forked from `stream` and joined back into it by events (created on
 * the first such call on a device); the caller sees only `stream`.
 */
int gdn_prefill_fwd(const void *q, const void *k, const void *v, const float *state,
                    const float *A_log, const void *a, const float *dt_bias, const void *b,
                    const void *cu_seqlens, int cu_seqlens_is_int64, int N, int T,
                    float scale, int H, int HV, int K, int V, void *out, float *new_state,
                    void *workspace, size_t workspace_bytes, void *stream);

/*
 * gdn_prefill_fwd that also stores state checkpoints: the state of sequence n
 * after its first every, 2*every, ... tokens (every = checkpoint_every_n_tokens,
 * a positive multiple of 64) goes to
 * state_checkpoints[checkpoint_cu_starts[n] + i] ([num_checkpoints, HV, V, K]
 * fp32, k-last, 16-byte aligned), i = 0 .. len_n / every - 1, so
 * checkpoint_cu_starts ([N + 1] int64, device) must give sequence n
 * len_n / every slots.  These are the arguments and the layout of flashinfer's
 * chunk_gated_delta_rule (flashinfer/gdn_prefill.py:113-115,161-174), whose
 * Blackwell kernel stores the same states.  An index outside a sequence's
 * range or the buffer skips the store.  Workspace as gdn_prefill_fwd.
 */
int gdn_prefill_fwd_checkpointed(const void *q, const void *k, const void *v, const float *state,
                                 const float *A_log, const void *a, const float *dt_bias, const void *b,
                                 const void *cu_seqlens, int cu_seqlens_is_int64, int N, int T,
                                 float scale, int H, int HV, int K, int V, void *out, float *new_state,
                                 float *state_checkpoints, const int64_t *checkpoint_cu_starts,
                                 long long num_checkpoints, int checkpoint_every_n_tokens,
                                 void *workspace, size_t workspace_bytes, void *stream);

/*
 * gdn_prefill_fwd with every option: checkpoints as in
 * gdn_prefill_fwd_checkpointed when state_checkpoints is not NULL (then
 * checkpoint_every_n_tokens > 0; NULL needs 0, as flashinfer requires,
 * flashinfer/gdn_prefill.py:187-206), and `flags`:
 *   GDN_PREFILL_QK_L2NORM  q and k head vectors are L2-normalised in the
 *                          kernel, x * rsqrt(sum(x^2) + 1e-6): the option
 *                          use_qk_l2norm_in_kernel of the AITER kernels the
 *                          reference calls (solutions/gdn_prefill/main.py:72,79),
 *                          FLA's rule (fla/modules/l2norm.py:42).  The chunked
 *                          kernels keep the unit vectors in f16, the
 *                          token-serial kernel in fp32.
 * Unknown flag bits return GDN_ERR_INVALID.  Workspace as gdn_prefill_fwd.
 */
int gdn_prefill_fwd_ex(const void *q, const void *k, const void *v, const float *state,
                       const float *A_log, const void *a, const float *dt_bias, const void *b,
                       const void *cu_seqlens, int cu_seqlens_is_int64, int N, int T,
                       float scale, int H, int HV, int K, int V, void *out, float *new_state,
                       float *state_checkpoints, const int64_t *checkpoint_cu_starts,
                       long long num_checkpoints, int checkpoint_every_n_tokens, int flags,
                       void *workspace, size_t workspace_bytes, void *stream);

/*
 * gdn_prefill_fwd with every operand in HOST memory (q .. b, state, the
 * [N + 1] cu_seqlens, out and new_state host pointers; pinned memory for the
 * copies to overlap): for a caller that keeps tokens and states off the
 * device.  No counterpart in the reference, whose `run` takes device tensors
 * (solutions/gdn_prefill/main.py:31-84).
 *
 * The tokens are cut into segments of `segment_tokens` (0: 2048; rounded up
 * to a multiple of 64), the last `segment_tokens` or fewer halved down to
 * 256-token pieces (2048 -> 1024, 512, 256, 256) so that little work is left
 * once the last upload has landed.  Segment s + 1 is copied up on a stream this library
 * creates per device while segment s is prefilled on `stream` and segment
 * s - 1's output is copied back on a second library stream; every sequence's
 * running state stays in `workspace` between segments, so a sequence cut by a
 * segment boundary continues from its state (the results equal one
 * gdn_prefill_fwd call to rounding: a cut moves the boundary between two of
 * its tensor-core chunks only when the sequence does not start on a multiple
 * of 64 tokens).  cu_seqlens is read and validated on the host (non-decreasing,
 * within [0, T]: else GDN_ERR_INVALID).  `stream` waits for the last copy
 * back; each call first waits for the previous call's on this device, so one
 * workspace (device memory, 256-byte aligned, at least
 * gdn_prefill_host_workspace_bytes(N, T, H, HV, segment_tokens) bytes) may be
 * reused from any stream.  Not for use inside a stream capture.
 */
int gdn_prefill_fwd_host(const void *q, const void *k, const void *v, const float *state,
                         const float *A_log, const void *a, const float *dt_bias, const void *b,
                         const void *cu_seqlens, int cu_seqlens_is_int64, int N, int T, float scale,
                         int H, int HV, int K, int V, void *out, float *new_state, void *workspace,
                         size_t workspace_bytes, int segment_tokens, void *stream);

/* Device workspace bytes gdn_prefill_fwd_host needs: every sequence's state,
 * two segments of inputs and outputs, and one segment's chunk workspace. */
size_t gdn_prefill_host_workspace_bytes(int N, int T, int H, int HV, int segment_tokens);

/*
 * Workspace bytes gdn_prefill_fwd needs for (N, T, H, HV): 0 when the call
 * will take the token-serial kernel.  For each of floor(T/64) + N chunk slots
 * the chunked kernels keep either, per v-head, the chunk's [T ; P'] operand
 * tile and gates (17,424 bytes) and, per q/k head, its f16 [K ; Q] operand
 * tile (32,768 bytes) and its cross-Gram tile [K ; Q] K_prev^T (16,384 bytes);
 * or (the scan kernels) per v-head the chunk's state-transition record
 * (73,984 bytes) and a 4-byte ready flag (the flags rounded up to 256 bytes).
 * The value is the larger of the two layouts.  No counterpart in the
 * reference, whose AITER kernels allocate their intermediates with torch.
 */
size_t gdn_prefill_workspace_bytes(int N, int T, int H, int HV);

/*
 * gdn_prefill_fwd for callers that cannot allocate device memory.  No
 * counterpart in the reference, whose Python solution allocates through
 * torch.
 *
 * Callers that bind this library directly (cgo, JNI, a C serving loop) have
 * no caching allocator to hand a workspace from; cudaMalloc there is slow and
 * can synchronise the device in the middle of a latency-critical step, and
 * some runtimes carve up device memory once at start-up and allow no
 * allocation afterwards.  This entry point takes the same arguments as
 * gdn_prefill_fwd minus the workspace, which it takes from a scratch array of
 * 16 MiB defined inside the library: every device that loads the library
 * holds those 16 MiB until the process exits.  It calls no cudaMalloc,
 * cudaFree or other allocating routine.
 *
 * Limit: (floor(T/64) + N) * (17,424 * HV + 49,152 * H) must not exceed
 * 16 MiB (16,777,216 bytes) when the chunked kernels run (for example T < 768
 * at N = 1, H = 16, HV = 32, or T < 2,944 at N = 4, H = 4, HV = 8); larger
 * problems return GDN_ERR_TOO_LARGE before anything is launched.  Problems
 * below the chunk threshold need no scratch at all.  Every launch goes to
 * `stream` (no library stream or event is created).
 *
 * The first call on a device looks up the scratch array's device address
 * with that device current (the device of `stream` must be the current
 * device, as for every entry point here); make that first call before any
 * stream capture.  The address is kept for the life of the process: after a
 * cudaDeviceReset() on a device, whose context held the array, this entry
 * point must not be called on that device again.  Argument errors
 * (GDN_ERR_INVALID, GDN_ERR_UNSUPPORTED) are reported before
 * GDN_ERR_TOO_LARGE.  All calls share the one array and its contents carry over
 * from the previous call; the kernels overwrite every byte they read, so
 * nothing needs clearing, but calls whose work overlaps on the GPU (on
 * different streams, or different host threads) race on it and must be
 * serialised by the caller.
 */
int gdn_prefill_fwd_noalloc(const void *q, const void *k, const void *v, const float *state,
                            const float *A_log, const void *a, const float *dt_bias, const void *b,
                            const void *cu_seqlens, int cu_seqlens_is_int64, int N, int T,
                            float scale, int H, int HV, int K, int V, void *out, float *new_state,
                            void *stream);

/*
 * Pool-indexed multi-token decode (speculative-decoding verification; T == 1
 * is pool-indexed single-token decode): batch entry i advances the state in
 * pool slot indices[i] over its T tokens.
 *
 * Replaces flashinfer's `gated_delta_rule_mtp` (flashinfer/gdn_decode.py:557-745)
 * and the pool / bf16-state forms of `gated_delta_rule_decode_pretranspose`
 * (gdn_decode.py:118-330), whose CuTe DSL kernels need sm_90; the maths is the
 * contest's MTP definition (flashinfer/trace/templates/gdn.py:378-465).
 *
 *   pool_out == pool_in : final states written in place (disable_state_update
 *                         = False in flashinfer's API);
 *   pool_out == NULL    : no final state written (disable_state_update = True);
 *   other pool_out      : a new pool (the definition's `final_state`): the whole
 *                         pool is copied first (cudaMemcpyAsync on `stream`),
 *                         then the written slots are overwritten.  It must not
 *                         overlap pool_in.
 * state_bf16 == 0: the pools hold fp32; 1: they hold bf16 — the state is
 * widened on load, advanced in fp32 over all T tokens and rounded to bf16
 * (nearest-even) once, when stored.  out_indices (NULL: same as indices, same
 * integer type) names the slot each entry's final state is written to
 * (`output_state_indices`); an out-of-range output slot skips the write.
 * An index outside [0, pool_size) in `indices` marks padding (flashinfer's
 * -1): its output rows are written as zeros and no state is read or written.
 * No slot may be written by one entry and read or written by another.  When
 * `intermediate` ([inter_slots, cache_steps, HV, V, K] fp32, cache_steps >=
 * T; fp32 pools only) is not NULL, the state after token t of batch entry i
 * (read from slot s) is written
 *   - without GDN_MTP_SNAPSHOTS_BY_ENTRY: to intermediate[s, t], for
 *     s < inter_slots (the contest definition, gdn.py:457-460);
 *   - with it: to state row i * T + t of the buffer seen as
 *     [inter_slots * cache_steps] rows, if entry i's T rows fit (the rows
 *     flashinfer's gated_delta_rule_mtp kernel writes,
 *     gdn_kernels/gdn_decode_mtp.py:645; = intermediate[i, t] when
 *     cache_steps == T).
 * Padding entries write no snapshot.  `flags`:
 *   GDN_MTP_QK_L2NORM           normalise every q and k head vector in the
 *                               kernel as x * rsqrt(sum(x^2) + 1e-6)
 *                               (`use_qk_l2norm`); without it they are taken
 *                               as given (the contest definition);
 *   GDN_MTP_SNAPSHOTS_BY_ENTRY  snapshot rows by batch entry, as above.
 * Unknown flag bits return GDN_ERR_INVALID.  Alignment as decode: q, k 8
 * bytes; pools and intermediate 16 bytes; indices their own size.  B == 0 or
 * T == 0 launches no kernel (only the pool copy).
 */
int gdn_mtp_fwd(const void *q, const void *k, const void *v, const void *pool_in,
                void *pool_out, int state_bf16, const void *indices, const void *out_indices,
                int indices_int64, const float *A_log, const void *a, const float *dt_bias,
                const void *b, float scale, int B, int T, int H, int HV, int K, int V,
                int pool_size, int flags, void *out, float *intermediate, int inter_slots,
                int cache_steps, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_H_ */
