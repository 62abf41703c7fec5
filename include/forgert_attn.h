/*
 * forgert_attn.h - C ABI of the B200 (sm_100a) flash-decode attention engine.
 *
 * Drop-in replacement for the attention launchers of ForgeRT
 * (kernels/attention.cuh).  Plain C types only: device pointers are `void*`
 * to fp16 (IEEE binary16) data, `stream` is a `cudaStream_t` passed as
 * `void*` (NULL = the legacy default stream, as in the reference), and every
 * entry point returns an `int` status instead of the reference's `void`.
 *
 * Layouts follow the reference runtime:
 *   q, out            [num_heads, head_dim]                      (one token)
 *   k_cache, v_cache  [>= kv_len, num_kv_heads, head_dim]        (one layer's view
 *                     of the cache [layers x 2 x max_seq_len x num_kv_heads x head_dim],
 *                     runtime/kv_cache.cpp:29-37)
 *   query head h reads kv head h / (num_heads / num_kv_heads).
 *
 * Pointers are caller-owned device memory.  k/v bases must be 16-byte aligned
 * (tiles are moved with TMA tensor copies); q/out 4-byte aligned.
 *
 * Workspace: calls that split the KV range (decode; prefill of short or
 * few-head prompts) keep per-split (m, l, acc) partial states in a
 * library-owned per-device buffer that grows on demand with cudaMalloc.  Growth cannot happen inside CUDA-graph capture, so size it with
 * fr_reserve_workspace() before capturing; a capture that would need more
 * returns FR_ERR_WORKSPACE.  The buffer is shared by all calls on a device:
 * calls on different streams of one device must not overlap in time.
 */
#ifndef FORGERT_ATTN_H
#define FORGERT_ATTN_H

#include <stddef.h>

#if defined(__GNUC__)
#define FR_API __attribute__((visibility("default")))
#else
#define FR_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define FR_OK 0
#define FR_ERR_INVALID_ARG 1   /* null pointer, non-positive size, H % Hkv != 0 */
#define FR_ERR_UNSUPPORTED 2   /* head_dim not in {64, 128} */
#define FR_ERR_MISALIGNED 3    /* k/v not 16-byte aligned, q/out not 4-byte aligned */
#define FR_ERR_CUDA 4          /* a CUDA runtime call failed: see fr_last_cuda_error() */
#define FR_ERR_TIMEOUT 5       /* a bounded in-kernel wait ran out (fr_get_device_error) */
#define FR_ERR_WORKSPACE 6     /* workspace too small while a stream is capturing */
#define FR_ERR_SCRATCH_LIMIT 7 /* fr_decode_attn_noalloc: partials exceed its static scratch */

/* Size of the static device scratch used by fr_decode_attn_noalloc (1 MiB). */
#define FR_NOALLOC_SCRATCH_BYTES (1u << 20)

/* Single-token decode attention over kv_len cached positions.
 * Replaces decode_attn_v4_flash (kernels/attention.cuh:65-71; definition
 * kernels/attention_decode.cu:535-556).  Output: out[h] = softmax(q[h].K^T /
 * sqrt(D)) . V in fp16, fp32 accumulation.  kv_len must be >= 1. */
FR_API int fr_decode_attn(const void* q, const void* k_cache, const void* v_cache, void* out,
                   int num_heads, int num_kv_heads, int head_dim, int kv_len, void* stream);

/* fr_decode_attn without any device allocation, for callers that cannot
 * call cudaMalloc: code running under another framework's allocator or
 * memory pool, plugins whose host owns every device allocation, processes
 * that must not grow their device footprint after start-up.  No counterpart
 * in the reference (its launchers need no scratch: one CTA per head, no KV
 * split).  Same arguments and results as fr_decode_attn.  It splits the KV
 * range with fr_decode_attn's base split count (one CTA per SM, without the
 * thread-block clusters or the fused merge), so its split boundaries can
 * differ from fr_decode_attn's; the partials go to a static 1 MiB device
 * array (FR_NOALLOC_SCRATCH_BYTES) and in-kernel errors to a static error
 * word, both held by every GPU that loads the library until exit.  A call
 * whose partials need more returns FR_ERR_SCRATCH_LIMIT before launching
 * anything: the need is num_heads * splits * (head_dim + 2) * 4 bytes with
 * splits ~ SMs / num_kv_heads, e.g. on a 148-SM B200 0.40 MB for 12 heads /
 * 2 kv heads at kv_len 16384 and 0.54 MB for 28 / 4 at kv_len 131072, while
 * 16 heads over one kv head at kv_len 16384 (128 splits, 1.06 MB) is refused.
 * The first call on a device does a one-time set-up (looks up the arrays'
 * device addresses, sets kernel attributes): make that first call before any
 * stream capture.  All calls on a device share the one array, so calls that
 * overlap on the GPU (different streams, no ordering) race; serialise them.
 * A bounded in-kernel wait that runs out is recorded in the static error
 * word (read with fr_get_device_error, which allocates nothing); the CTA
 * concerned contributes an empty partial, so the output is wrong but no
 * earlier call's scratch is folded in. */
FR_API int fr_decode_attn_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                  void* out, int num_heads, int num_kv_heads, int head_dim,
                                  int kv_len, void* stream);

/* Batched, ragged decode over a KV pool: sequence b's cache rows are pool
 * rows [row_offsets[b], row_offsets[b] + kv_lens[b]) of
 *   k_pool, v_pool  [pool_rows, num_kv_heads, head_dim] fp16 (16-byte aligned)
 * (the reference's per-layer cache layout, with all sequences' rows in one
 * allocation, as a paged/ragged serving cache keeps them).
 *   q, out         [batch, num_heads, head_dim]
 *   row_offsets    device int64 array (length batch)
 *   kv_lens        device int32 array (length batch); 0 is allowed and yields zeros
 *   max_kv_len     host upper bound of kv_lens (sizes the launch)
 * Rows of the pool past a sequence's end are never used, whatever they hold.
 * No reference counterpart (the reference decodes one sequence per call,
 * attention.cuh:30); it generalises decode_attn_v4_flash to a batch. */
FR_API int fr_decode_attn_batched(const void* q, const void* k_pool, const void* v_pool,
                                  const long long* row_offsets, const int* kv_lens, void* out,
                                  int batch, int num_heads, int num_kv_heads, int head_dim,
                                  long long pool_rows, int max_kv_len, void* stream);

/* Batched decode over a paged KV cache (block table).
 *   k_pages, v_pages  [num_pages, page_size, num_kv_heads, head_dim] fp16
 *                     (16-byte aligned): each page holds page_size cache rows
 *                     in the reference's row layout
 *   block_table       device int32 [batch, max_blocks_per_seq]: position t of
 *                     sequence b lives in page block_table[b][t / page_size],
 *                     row t % page_size
 *   kv_lens           device int32 [batch]; 0 is allowed and yields zeros
 *   q, out            [batch, num_heads, head_dim]
 *   page_size         a multiple of 16 rows
 *   max_kv_len        host upper bound of kv_lens, <= max_blocks_per_seq * page_size
 * Only the first ceil(kv_lens[b] / page_size) entries of a row are read; page
 * ids outside [0, num_pages) read as zero rows, and rows of the last page
 * past kv_lens[b] are never used, whatever they hold.  No reference
 * counterpart: the reference keeps one contiguous cache per layer
 * (runtime/kv_cache.cpp:14-37) and lists paging as future work (README.md:31). */
FR_API int fr_decode_attn_paged(const void* q, const void* k_pages, const void* v_pages,
                                const int* block_table, const int* kv_lens, void* out,
                                int batch, int num_heads, int num_kv_heads, int head_dim,
                                int page_size, int num_pages, int max_blocks_per_seq,
                                int max_kv_len, void* stream);

/* Partial attention over positions [0, kv_len) of the given cache view:
 * writes one log-sum-exp state per query head instead of an output, for
 * KV ranges that are split across GPUs.  No reference counterpart.
 *   state_ml  [num_heads, 2] fp32: (m, l), m = running max of score*log2(e)/sqrt(D)
 *   state_acc [num_heads, head_dim] fp32: sum_t 2^(s_t - m) v_t
 * kv_len == 0 yields the empty state (m = -inf, l = 0, acc = 0). */
FR_API int fr_decode_attn_partial(const void* q, const void* k_cache, const void* v_cache,
                           int kv_len, float* state_ml, float* state_acc, int num_heads,
                           int num_kv_heads, int head_dim, void* stream);

/* Log-sum-exp merge of num_states partial states per head (as written by
 * fr_decode_attn_partial, stacked state-major: state s of head h at
 * states_ml[(s*num_heads + h)*2] and states_acc[(s*num_heads + h)*head_dim]).
 * out[h] = fp16( sum_s acc_s 2^(m_s - m*) / sum_s l_s 2^(m_s - m*) ).
 * No reference counterpart (the reference never splits the KV range). */
FR_API int fr_lse_merge(const float* states_ml, const float* states_acc, int num_states, void* out,
                 int num_heads, int head_dim, void* stream);

/* fr_lse_merge with explicit distances (in floats) between consecutive
 * states of one head, for states gathered into one buffer per rank:
 * state s of head h at states_ml[s*ml_state_stride + 2h] and
 * states_acc[s*acc_state_stride + h*head_dim].  ml_state_stride must be even.
 * No reference counterpart. */
FR_API int fr_lse_merge_strided(const float* states_ml, const float* states_acc, int num_states,
                                void* out, int num_heads, int head_dim,
                                long long ml_state_stride, long long acc_state_stride,
                                void* stream);

/* ---- Cross-GPU long-context decode (KV range split across GPUs) ----------
 * One sequence's cache rows are split in contiguous ranges, one per GPU (one
 * process per GPU).  fr_decode_attn_exchange computes this GPU's split-KV
 * state and, in the same kernel, stores its (m, l, acc) slices into every
 * GPU's exchange buffer over NVLink/NVSwitch (plain peer stores), waits
 * (bounded) until all GPUs' states of a head group have arrived in its own
 * buffer and merges them into out: the all-gather + log-sum-exp merge of a
 * KV-range split, without a collective library call.  Every GPU gets the
 * full result.  No reference counterpart (the reference runs on one GPU).
 *
 * Set-up, once per process group: every rank calls fr_exchange_alloc (one
 * buffer of fr_exchange_bytes bytes, zeroed, on the current device) and
 * sends its 64-byte IPC handle to the others (e.g. an all-gather of bytes),
 * then opens each peer's handle with fr_exchange_open.  bufs[j] is rank j's
 * buffer as seen from this process (bufs[rank] = the local one).
 * All ranks must make the same sequence of calls with the same num_heads,
 * num_kv_heads and head_dim (local_kv_len may differ); a call returns once
 * launched.  Each state word is stored with the call's sequence number in
 * one 8-byte access, so a receiver needs no fence or flag: it waits until the
 * words it reads carry its own call number.  If a peer does not take part,
 * the wait ends after about a second (FORGERT_EXCHANGE_WAIT_MS, 1 to 5000,
 * read once per process; fr_exchange_wait_limit_ms() returns the value in
 * force) with FR_ERR_TIMEOUT from fr_get_device_error; the exchange state is
 * then inconsistent and every rank must fr_exchange_reset its buffer (stream
 * ordered) before the next call.
 *   q, out     [num_heads, head_dim] fp16 (the same q on every rank)
 *   k_local, v_local  this GPU's rows [local_kv_len, num_kv_heads, head_dim] */
FR_API size_t fr_exchange_bytes(int num_heads, int head_dim, int world);
FR_API int fr_exchange_alloc(size_t bytes, void** buf, void* ipc_handle /* 64 bytes out */);
FR_API int fr_exchange_open(const void* ipc_handle, void** peer_buf);
FR_API int fr_exchange_close(void* peer_buf);
FR_API int fr_exchange_free(void* buf);
FR_API int fr_exchange_reset(void* buf, size_t bytes, void* stream);
FR_API int fr_decode_attn_exchange(const void* q, const void* k_local, const void* v_local,
                                   int local_kv_len, void* out, int num_heads, int num_kv_heads,
                                   int head_dim, void* const* bufs, int rank, int world,
                                   void* stream);
FR_API int fr_exchange_wait_limit_ms(void);

/* RoPE cos/sin tables [max_seq_len, head_dim/2] fp32 into caller-allocated
 * device buffers: theta(pos, f) = pos / (base^(2f/head_dim) * scale), evaluated
 * in fp64 on the host and rounded once.  Synchronous, like the reference.
 * Replaces rope_precompute_tables (kernels/rope.cuh:227-231, rope.cu:28-56),
 * minus its allocation. */
FR_API int fr_rope_tables(float* cos_tab, float* sin_tab, int max_seq_len, int head_dim, float base,
                   float scale);

/* RoPE cos/sin tables [max_seq_len, head_dim/2] fp32 computed on the device,
 * stream-ordered, with the reference's own single-precision arithmetic: the
 * same values as rope_precompute_tables (kernels/rope.cu:28-56, built with
 * --use_fast_math, whose fast sine and cosine drift from the exact values as
 * theta = pos / base^(2f/D) grows - up to ~16000 rad at max_seq_len 16384).
 * Use it where results must match the reference engine bit for bit;
 * fr_rope_tables gives the exactly rounded tables.  Caller-allocated
 * buffers; replaces rope_precompute_tables minus its allocation. */
FR_API int fr_rope_tables_device(float* cos_tab, float* sin_tab, int max_seq_len, int head_dim,
                                 float base, float scale, void* stream);

/* Fused decode prologue: NeoX (half-split) RoPE on q and k in place for
 * tokens t < seq_len at position pos_offset + t, then appends the rotated k
 * and v rows to the layer cache at row pos_offset + t.  Replaces the
 * sequence rope_v2_fused (kernels/rope.cu:193-207) + the two KV-append
 * cudaMemcpyAsync calls of runtime/executor.cpp:140-152.
 *   q [seq_len, num_heads, head_dim], k, v [seq_len, num_kv_heads, head_dim] */
FR_API int fr_rope_append(void* q, void* k, const void* v, void* k_cache, void* v_cache,
                   const float* cos_tab, const float* sin_tab, int seq_len, int num_heads,
                   int num_kv_heads, int head_dim, int pos_offset, void* stream);

/* The same prologue with the projection biases folded in: q += q_bias,
 * k += k_bias, v += v_bias (one fp16 round-to-nearest addition per element,
 * as bias_add_broadcast, kernels/elementwise.cu:81-98), then RoPE on q and k
 * and the KV append, in one launch.  Replaces the six launches of
 * runtime/executor.cpp:135-152 (three bias adds, rope_v2_fused, two copies).
 * Any bias may be NULL (no add); q_bias [num_heads*head_dim], k_bias and
 * v_bias [num_kv_heads*head_dim] fp16, v_bias 16-byte aligned.  q and k are
 * left rotated and v biased in place, as the reference sequence leaves them. */
FR_API int fr_qkv_bias_rope_append(void* q, void* k, void* v, const void* q_bias,
                                   const void* k_bias, const void* v_bias, void* k_cache,
                                   void* v_cache, const float* cos_tab, const float* sin_tab,
                                   int seq_len, int num_heads, int num_kv_heads, int head_dim,
                                   int pos_offset, void* stream);

/* Causal prefill attention: query position s attends to positions 0..s.
 * Replaces prefill_attn_causal (kernels/attention.cuh:76-82; definition
 * kernels/attention_decode.cu:563-619): a flash-attention kernel on the
 * tcgen05 tensor cores, one CTA per (128 query positions, query head)
 * (FORGERT_PREFILL_KERNEL=mma selects the mma.sync form, 64 positions per CTA).
 *   q, out [seq_len, num_heads, head_dim]; k, v [seq_len, num_kv_heads, head_dim]
 * q, k, v 16-byte aligned (tensor-memory-access copies), out 4-byte aligned. */
FR_API int fr_prefill_attn(const void* q, const void* k, const void* v, void* out, int seq_len,
                    int num_heads, int num_kv_heads, int head_dim, void* stream);

/* Grows the current device's workspace to at least `bytes` (call before
 * CUDA-graph capture).  fr_decode_workspace_size() gives the bytes one call
 * of fr_decode_attn_batched with these sizes needs (fr_decode_attn: batch 1). */
FR_API int fr_reserve_workspace(size_t bytes);
FR_API size_t fr_decode_workspace_size(int batch, int num_heads, int num_kv_heads, int head_dim,
                                int max_kv_len);
/* Workspace bytes fr_prefill_attn uses for seq_len positions and num_heads
 * query heads (0 when the call needs none).  Prefill splits the K/V range
 * of long query tiles over several CTAs when the grid would otherwise leave
 * SMs idle; inside a CUDA-graph capture whose workspace is too small it runs
 * unsplit (same result, fewer CTAs), so reserve this much with
 * fr_reserve_workspace() before capturing a prefill. */
FR_API size_t fr_prefill_workspace_size(int seq_len, int num_heads, int head_dim);

/* Reads (and optionally clears) the current device's in-kernel error words
 * (the regular entry points' and fr_decode_attn_noalloc's): 0 = none,
 * otherwise a bounded wait ran out (FR_ERR_TIMEOUT is returned by the
 * status).  Synchronises the device; creates no state and allocates
 * nothing. */
FR_API int fr_get_device_error(int clear, int* device_code);

/* Device memory the library has allocated with cudaMalloc on the current
 * device (its error word and workspace; exchange buffers are the caller's),
 * 0 when none.  Creates no state and allocates nothing.  Diagnostics; no
 * reference counterpart. */
FR_API size_t fr_allocated_bytes(void);

/* Last CUDA error code (cudaError_t as int) seen by this thread's calls. */
FR_API int fr_last_cuda_error(void);
FR_API const char* fr_status_string(int status);
FR_API int fr_version(void);

/* Launch overlap for fr_decode_attn on a non-default stream: when enabled,
 * K/V rows [0, kv_len - 1) may be read before the kernel's grid-dependency
 * wait, i.e. while the preceding kernel in the stream is still running
 * (programmatic dependent launch).  Enable it only when those rows are never
 * written by the kernels immediately preceding the call - true for the
 * reference's decode step, where only row kv_len - 1 is new.  q, the newest
 * row and every output always wait.  Process-wide, default off; returns the
 * previous setting.  No reference counterpart. */
FR_API int fr_set_launch_overlap(int enable);

/* Stream-ordered copy of `bytes` from src to dst by a kernel.  Each pointer
 * may be device memory or page-locked host memory (cudaHostAlloc,
 * cudaMallocHost, cudaHostRegister), which the kernel reaches through its
 * device mapping; pageable host memory gives FR_ERR_INVALID_ARG.  For the
 * small per-step transfers of a decode step (a layer's q, token ids, an
 * argmax result; the reference's runtime/executor.cpp:288-311 uses
 * cudaMemcpy for these): it avoids the copy engine's fixed cost (~10 us per
 * copy on B200), is graph-capturable and takes part in programmatic
 * dependent launch like the attention calls.  16-byte aligned pointers copy
 * by 16-byte vectors.  No reference counterpart. */
FR_API int fr_copy_async(void* dst, const void* src, size_t bytes, void* stream);

/* Number of kernels this library has launched (or recorded into a CUDA graph
 * under capture) in this process.  Diagnostics only; no reference
 * counterpart. */
FR_API unsigned long long fr_launch_count(void);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* FORGERT_ATTN_H */
