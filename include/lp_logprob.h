/*
 * lp_logprob.h — C ABI of the B200 (sm_100a) token-logprob library (liblp_b200.so).
 *
 * The library computes, for a tied LM head W[V, d] and hidden states H[T, d] (bf16):
 *     z[t, v]  = softcap(H[t] . W[v])            softcap(x) = c * tanh(x / c), or x
 *     logp[t]  = z[t, y_t] - log sum_v exp(z[t, v])
 * and the vector-Jacobian product of logp with respect to H and W, without ever writing
 * the [T, V] logits to memory. It replaces the reference's logprob backends
 * (yixiaoer/gemma4-posttrain-jax):
 *     gemma4_posttrain_jax/losses.py:72-147   _single_partition_logps   (forward)
 *     gemma4_posttrain_jax/losses.py:172-260  _vocab_parallel_logps_and_normalization
 *     gemma4_posttrain_jax/losses.py:307-343  per_token_logps (backend switch)
 *     gemma4_posttrain_jax/pallas/lm_head_logprob_tpuv4.py:41-94,97-152,216-297
 *                                               custom_vjp fwd / bwd and the dW kernel
 * Vocabulary parallelism: each caller process holds one shard W[v_off : v_off + Vs] and
 * calls lp_fwd on it; the per-shard (max, sum, owned target logit) triples are exchanged
 * by the caller's collective (NCCL all-gather) and merged by lp_combine, or exchanged over
 * NVLink inside the forward by lp_fwd_sum where the GPUs share an NVSwitch multicast.
 *
 * Conventions
 *   - All pointers are device pointers unless stated. `stream` is a cudaStream_t (NULL =
 *     legacy default stream). Calls only enqueue work; nothing synchronises the host.
 *   - Every entry point returns LP_OK (0) or a negative LP_E* code; lp_last_error()
 *     returns a message for the calling thread. No C++ exception crosses this boundary.
 *   - Buffers are owned by the caller. Scratch memory is a caller-provided `workspace`
 *     of at least the size the matching *_workspace_bytes() function returns.
 *   - Requirements checked on every call: bf16 H and W, d % 8 == 0, ldh % 8 == 0,
 *     16-byte aligned base pointers, an sm_100 device.
 *   - Kernels never spin without a time limit: a broken pipeline makes the kernel exit
 *     and record a device error code, read (and cleared) by lp_device_error().
 */
#ifndef LP_LOGPROB_H_
#define LP_LOGPROB_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LP_API __attribute__((visibility("default")))
#else
#define LP_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define LP_OK 0
#define LP_EINVAL (-1)        /* bad argument: shape, alignment, null pointer        */
#define LP_ECUDA (-2)         /* CUDA runtime / driver error                          */
#define LP_EWORKSPACE (-3)    /* workspace smaller than *_workspace_bytes() asks for  */
#define LP_EDEVICE (-4)       /* a kernel recorded a device-side error (timeout)      */
#define LP_EUNSUPPORTED (-5)  /* not an sm_100 device                                 */

/* lp_bwd flags */
#define LP_BWD_DH_F32 1  /* dH written as f32 (default: bf16)                   */
#define LP_BWD_DW_BF16 2 /* dW written as bf16 (default: f32)                   */
#define LP_BWD_NO_DW 4   /* frozen head: skip dW (fwd + dH only)               */
#define LP_BWD_NO_DH 8   /* skip dH                                            */

/* Library version (major * 10000 + minor * 100 + patch). */
LP_API int lp_version(void);

/* Message describing the last error returned on this thread ("" if none). */
LP_API const char* lp_last_error(void);

/* Number of kernels this library has launched in this process (all devices). */
LP_API long long lp_launch_count(void);

/* Tensor-core CTA group of the GEMMs: 0 (default) lets each GEMM use the group measured
 * faster for it (CTA pairs on two SMs, 256x256 tiles, for the forward, the dZ recompute, dH
 * and dW; single CTAs, 128x256 tiles, for the sampler head and for the dW GEMM of a token
 * chunk of at most 1024 rows); 1 or 2 forces one group for every GEMM (also
 * LP_B200_CTA_GROUP=1|2). Results agree to f32 rounding; lp_get_cta_group() returns the
 * forced group or 0. */
LP_API int lp_set_cta_group(int cg);
LP_API int lp_get_cta_group(void);

/* Tuning aid: per-GEMM pipeline counters (cycles the TMA, MMA and epilogue warps wait on
 * each barrier, summed over CTAs). lp_debug_enable(1) allocates and zeroes the counters of
 * the current device; lp_debug_read fills out[5][8] (forward, dZ, dH, dW, other x
 * {producer wait, MMA wait on loads, MMA wait on accumulator, epilogue wait, MMA-thread
 * cycles, K blocks, epilogue busy, tiles}). */
LP_API int lp_debug_enable(int on);
LP_API int lp_debug_read(unsigned long long* out);

/* CTA pairs of the pair GEMMs that can be resident on the current device (-1 on error). */
LP_API int lp_device_pairs(void);

/* Per-kernel timing (for benchmarks): while enabled, every kernel launch of this library
 * is bracketed by CUDA events on its stream. Enabling (or disabling) clears the record. */
LP_API int lp_profile_enable(int on);

/* Sums the recorded launches per kernel name (synchronises on the events):
 * names: max_tags * 32 chars (NUL-terminated names), total_ms / launches: max_tags each. */
LP_API int lp_profile_read(int max_tags, char* names, double* total_ms, long long* launches, int* n_tags);

/* Reads and clears the device-side error code recorded by kernels on `device`
 * (0 = none; 1..4 = a bounded wait inside a GEMM gave up; 5 = a wait for another rank of a
 * vocabulary mesh gave up). Synchronises that device. */
LP_API int lp_device_error(int device, int* code);

/* The same code without any CUDA call or synchronisation: kernels also write it to mapped
 * host memory, so a caller that has already waited for its stream (for instance to read a
 * count back) can check the kernels it waited for at no cost. Returns 0 while nothing has
 * been recorded on `device` since the last lp_device_error(device, ...) (which clears it),
 * and 0 before the library has run anything on that device. */
LP_API int lp_device_error_poll(int device);

/* Scratch bytes lp_fwd needs for T tokens against a shard of Vs rows. */
LP_API size_t lp_fwd_workspace_bytes(int64_t T, int64_t Vs);

/*
 * Forward over one vocabulary shard (replaces losses.py:98-147 and the per-shard body of
 * losses.py:199-248).
 *   H        bf16 [T, ldh] (first d columns used)          W  bf16 [Vs, d]
 *   y        int32 [T] global target ids; ids outside [v_off, v_off + Vs) are not owned
 *   softcap  c > 0 applies c * tanh(x / c); c <= 0 disables it (reference: None)
 *   stats    f32 [3, T]: shard max, shard sum exp(z - max), owned target logit (0 if not owned)
 *   logp     f32 [T] or NULL: stats[2] - (stats[0] + log stats[1]); only meaningful when
 *            the shard is the whole vocabulary (v_off == 0, Vs == V)
 */
LP_API int lp_fwd(void* stream, const void* H, int64_t T, int64_t d, int64_t ldh, const void* W, int64_t Vs, int64_t v_off,
           const int32_t* y, float softcap, float* stats, float* logp, void* workspace, size_t workspace_bytes);

/* Size of the fixed device scratch lp_fwd_noalloc uses. The library's device code is one
 * module, so every GPU on which the library has run any kernel holds this array until the
 * process exits, whether or not it ever calls lp_fwd_noalloc. */
#define LP_NOALLOC_SCRATCH_BYTES (8u << 20)

/*
 * Allocation-free forward. No counterpart in the reference: it exists for callers that
 * cannot allocate device memory where they call the logprob forward, e.g. an FFI custom
 * call that its framework hands only input and output buffers, or a long-running host loop
 * that must not grow device memory after start-up. It computes exactly what lp_fwd
 * computes, with the same arguments, except that there is no workspace: the scratch is one
 * fixed LP_NOALLOC_SCRATCH_BYTES device array inside the library.
 *   - Nothing is allocated: no cudaMalloc / cudaFree, no allocating library call.
 *   - The first call on a device looks up that device's scratch address (the device must
 *     be current); make that first call before any stream capture.
 *   - All calls share the one array, so calls that overlap on the GPU (different streams,
 *     or different host threads) race and corrupt each other's results: serialise them.
 *     The array keeps the last call's contents; every scratch value a call reads is
 *     written earlier in that same call, so nothing needs clearing between calls.
 *   - The scratch holds 16 bytes per token for each vocabulary group of the tile plan
 *     (a running max and sum for each half of a group's columns) plus a 4-byte target
 *     logit per token. Where lp_fwd's plan would need more, the groups are widened (fewer
 *     groups of more 256-row vocabulary tiles; the results are the same); with a single
 *     group the limit is 419,424 tokens (8 MiB / 20 B, less 256-byte alignment). More tokens
 *     return LP_EINVAL.
 *     Wider groups make fewer, longer work units (ceil(T / 128) x groups): above about
 *     233k tokens there is one group, so each unit streams the whole shard for 128 rows.
 */
LP_API int lp_fwd_noalloc(void* stream, const void* H, int64_t T, int64_t d, int64_t ldh, const void* W, int64_t Vs,
                          int64_t v_off, const int32_t* y, float softcap, float* stats, float* logp);

/*
 * Merge P per-shard triples (replaces the pmax / psum combine of losses.py:219,243-245).
 *   shard_stats f32 [P, 3, T] (lp_fwd's `stats` of every shard, in shard order)
 *   logp        f32 [T]       global target log-probability
 *   norm        f32 [2, T] or NULL: global max and global sum exp(z - max), the
 *               reference's `normalization` output (losses.py:246-247)
 */
LP_API int lp_combine(void* stream, const float* shard_stats, int P, int64_t T, float* logp, float* norm);

/*
 * lp_fwd on one rank of a vocabulary mesh with the exchange of the per-shard triples done
 * over NVLink inside the forward's finalize kernel: the pmax / psum combine of
 * losses.py:219,243-245 without a separate collective (it replaces lp_fwd + an all-gather
 * + lp_combine, with the same floats as that sequence). Each rank stores its rows'
 * (max, sum, owned target logit) into its slot of every rank's copy of a symmetric
 * exchange buffer (NVLS multicast store), counts itself once on an exchange counter in
 * every copy, waits until all `world` ranks have done so and merges the slots locally.
 *   exchange / exchange_multicast  this rank's address and the multicast address of an f32x4
 *                     [world, ld_exchange] buffer bound on every rank (16-byte aligned)
 *   counter / counter_multicast    one u32 in the same kind of memory, zero when the buffer
 *                     was set up; never reset: call number `epoch` (1, 2, ...) of this
 *                     (exchange, counter) pair waits for epoch * world
 *   arrivals          one u32 in this GPU's memory, zero before the first call (each call
 *                     leaves it zero)
 *   logp / norm       f32 [T] global target logp / f32 [2, T] global (max, sum), as lp_combine
 *   timeout_ms        bound of the wait for the other ranks (device error on expiry)
 * Every rank makes the same calls in the same order, stream-ordered on each rank, and
 * consecutive calls alternate between two (exchange, counter) pairs: a rank overwrites a
 * slot only after the call with the other pair has seen every rank finish reading it.
 * The workspace is lp_fwd_workspace_bytes(T, Vs).
 */
LP_API int lp_fwd_sum(void* stream, const void* H, int64_t T, int64_t d, int64_t ldh, const void* W, int64_t Vs,
                      int64_t v_off, const int32_t* y, float softcap, void* exchange, void* exchange_multicast,
                      int64_t ld_exchange, unsigned* counter, unsigned* counter_multicast, unsigned* arrivals,
                      unsigned epoch, int rank, int world, int timeout_ms, float* logp, float* norm, void* workspace,
                      size_t workspace_bytes);

/* Scratch bytes lp_bwd needs; token_chunk <= 0 selects the default chunk. */
LP_API size_t lp_bwd_workspace_bytes(int64_t T, int64_t d, int64_t Vs, int64_t token_chunk, int flags);

/*
 * Backward over one vocabulary shard (replaces the AD of losses.py:98-147 / :199-248 and
 * pallas/lm_head_logprob_tpuv4.py:88-152,216-297). For every token chunk the logits tile
 * is recomputed, dZ = g * (onehot(y) - softmax(z)) * (1 - tanh^2) formed in registers and
 * fed to two tensor-core GEMMs:
 *   dH[T, d]  = dZ . W       (partial over this shard: the caller sums over shards)
 *   dW[Vs, d] = dZ^T . H     (complete for this shard: no communication)
 *   norm  f32 [2, T]  global max / sum from lp_combine (or lp_fwd when P == 1)
 *   g     f32 [T]     upstream d loss / d logp
 *   dH    bf16 or f32 [T, ld_dh] (LP_BWD_DH_F32), may be NULL with LP_BWD_NO_DH
 *   dW    f32 or bf16 [Vs, d] (LP_BWD_DW_BF16), may be NULL with LP_BWD_NO_DW
 */
LP_API int lp_bwd(void* stream, const void* H, int64_t T, int64_t d, int64_t ldh, const void* W, int64_t Vs, int64_t v_off,
           const int32_t* y, float softcap, const float* norm, const float* g, void* dH, int64_t ld_dh, void* dW,
           int flags, int64_t token_chunk, void* workspace, size_t workspace_bytes);

/*
 * lp_bwd on one rank of a vocabulary mesh, with the sum of the dH partials over the mesh's
 * shards (the psum of the bf16 hidden cotangent, the transpose of losses.py:253-259) done
 * inside the dH GEMM over NVLink: each rank stores its bf16 partial tiles into its own copy
 * of a symmetric buffer and counts them on per-row-block counters in every rank's copy
 * (multimem.red); reduce items of the same persistent launch then sum rank r's share of each
 * finished row block across all copies through the NVSwitch (multimem.ld_reduce, f32
 * accumulation) and store the result to every copy (multimem.st). On return (stream order)
 * every rank's dH copy holds the sum once all ranks have passed the next lp_peer_barrier.
 *   dH / dH_multicast   this rank's address and the multicast address of a bf16 [T, ld_dh]
 *                       buffer bound on every rank (NVLS multicast object); 16-B aligned
 *   counters / counters_multicast  u32 [lp_bwd_sum_counters(T)] in the same kind of memory,
 *                       zero on every rank when the call starts: zero them once when the
 *                       buffer is set up (before any rank's first call), and after each call
 *                       on this rank's stream, before the lp_peer_barrier that follows it
 *                       (every rank reduces a share of every row block, so its counters have
 *                       reached their final counts when its call's dH GEMM ends)
 *   rank, world         this rank's position in the mesh and the mesh size
 *   timeout_ms          bound of every wait for the other ranks' tiles (device error on expiry)
 * Other arguments as lp_bwd (dH is always bf16; LP_BWD_DH_F32 / LP_BWD_NO_DH are rejected).
 * The workspace is lp_bwd_workspace_bytes(T, d, Vs, token_chunk, flags).
 */
LP_API size_t lp_bwd_sum_counters(int64_t T);
LP_API int lp_bwd_sum(void* stream, const void* H, int64_t T, int64_t d, int64_t ldh, const void* W, int64_t Vs,
                      int64_t v_off, const int32_t* y, float softcap, const float* norm, const float* g, void* dH,
                      void* dH_multicast, int64_t ld_dh, unsigned* counters, unsigned* counters_multicast, int rank,
                      int world, int timeout_ms, void* dW, int flags, int64_t token_chunk, void* workspace,
                      size_t workspace_bytes);

/* lp_head flags */
#define LP_HEAD_LOGPROBS 1 /* the logits buffer receives log-probabilities z - logsumexp(z) */

/* Scratch bytes lp_head needs for B rows against V vocabulary rows. */
LP_API size_t lp_head_workspace_bytes(int64_t B, int64_t V);

/*
 * Sampler LM head (replaces forward_lm_head, model.py:676-680, and the full-vocabulary
 * log-softmax and greedy pick of _sample_token, sampler.py:145-161,184): one tensor-core
 * GEMM over the whole vocabulary for B decode rows, with the softcap, a running
 * log-sum-exp and the row argmax in its epilogue.
 *   H        bf16 [B, ldh]                W  bf16 [V, d] (the whole vocabulary)
 *   logits   f32 [B, ld_logits] (ld_logits >= V, % 4 == 0, 16-byte aligned) or NULL: the
 *            softcapped logits z, or with LP_HEAD_LOGPROBS the log-probabilities
 *            z - (max + log sum); NULL skips the [B, V] store (greedy decoding needs none)
 *   norm     f32 [2, B] or NULL: row max of z and sum exp(z - max) (needed with LOGPROBS)
 *   argmax   int32 [B] or NULL: first column of the row maximum (greedy token)
 *   argmax_logp  f32 [B] or NULL: log-probability of that column
 * The workspace is lp_head_workspace_bytes(B, V).
 */
LP_API int lp_head(void* stream, const void* H, int64_t B, int64_t d, int64_t ldh, const void* W, int64_t V,
                   float softcap, float* logits, int64_t ld_logits, int flags, float* norm, int32_t* argmax,
                   float* argmax_logp, void* workspace, size_t workspace_bytes);

/* Scratch bytes lp_compact needs for B * N response slots. */
LP_API size_t lp_compact_workspace_bytes(int64_t B, int64_t N);

/*
 * Response-token compaction (replaces the slice + where of losses.py:667-669,682, which
 * computes every padded slot): slot s = b * N + j is valid when mask[s] != 0.
 *   idx    int32 [B * N]  compact row -> slot, valid rows first, slot order preserved
 *   pos    int32 [B * N]  slot -> compact row, or -1 for invalid slots
 *   count  int32 [1]      number of valid slots
 * When `hidden` is non-NULL the valid rows are also gathered:
 *   H_out[i]  = hidden[b * hidden_bstride + (j + row_offset) * hidden_rstride, 0:d]  (bf16)
 *   y_out[i]  = ids[slot]
 * (row_offset = prompt_width - 1 reproduces hidden[:, P-1 : P+N-1].)
 */
LP_API int lp_compact(void* stream, const uint8_t* mask, int64_t B, int64_t N, const void* hidden, int64_t hidden_bstride,
               int64_t hidden_rstride, int64_t row_offset, int64_t d, const int32_t* ids, void* H_out, int32_t* y_out,
               int32_t* idx, int32_t* pos, int32_t* count, void* workspace, size_t workspace_bytes);

/*
 * Scatter compact rows back to the slot layout, zero-filling invalid slots:
 *   row(s)[0:width] = pos[s] >= 0 ? src[pos[s], 0:width] : 0     for s in [0, slots)
 *   row(s) = out + (s / rows_per_group) * group_stride + (s % rows_per_group) * out_stride
 * so a strided [B, N, width] view (rows_per_group = N) such as the response slice of a
 * [B, S, d] gradient is written in place. With pos = a list of source rows it is a row
 * gather. elem_bytes is 2 (bf16) or 4 (f32) for src; out_elem_bytes equals it, or is 2
 * with f32 src (rows converted to bf16 on the way). Strides are in elements.
 */
LP_API int lp_scatter_rows(void* stream, const void* src, int64_t src_stride, const int32_t* pos, int64_t slots,
                    int64_t width, int elem_bytes, void* out, int64_t out_stride, int64_t rows_per_group,
                    int64_t group_stride, int out_elem_bytes);

/*
 * Device-side barrier of the `world` ranks of a vocabulary mesh, on `stream` (one small
 * kernel). It follows every lp_bwd_sum: when it passes, every rank's multicast stores have
 * landed and every rank has zeroed its counters for the next call. No barrier is needed
 * before lp_bwd_sum: another rank's sums reach this rank's copy only after this rank's own
 * dH GEMM of the same call has started, i.e. after it has consumed its previous dH.
 *   signal_pads  device array [world] of u64: this process's address of each rank's
 *                signal pad (peer-mapped memory, u32 slots, zero-initialised)
 *   channel      slot row used: slots [channel * world, (channel + 1) * world) of each pad
 *   timeout_ms   bound of every wait; on expiry the kernel records a device error
 *                (lp_device_error) and returns instead of hanging
 */
LP_API int lp_peer_barrier(void* stream, const unsigned long long* signal_pads, int rank, int world, int channel,
                           int timeout_ms);

/*
 * Test hook of the tensor-core core (no reference counterpart): D[M, N] = A . B^T in f32,
 * bf16 operands. a_mn = 0: A is [M, K] row-major (lda >= K); a_mn = 1: A is stored
 * transposed, [K, M] row-major (lda >= M). Likewise b_mn for B ([N, K] or [K, N]).
 */
LP_API int lp_gemm_bf16(void* stream, const void* A, int64_t M, int64_t K, int64_t lda, int a_mn, const void* B, int64_t N,
                 int64_t ldb, int b_mn, float* D, int64_t ldd);

#ifdef __cplusplus
}
#endif

#endif /* LP_LOGPROB_H_ */
