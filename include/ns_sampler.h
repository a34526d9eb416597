/*
 * ns_sampler.h -- C ABI of the B200-native token sampler.
 *
 * Drop-in for the sampling step of apollo722/nano-inference:
 *   Sampler.select_batch   src/nano_inference/sampling/sampler.py:36-91
 *   Sampler.select         src/nano_inference/sampling/sampler.py:11-34
 *   SamplerBase            src/nano_inference/sampling/base.py:10-25
 * The reference is pure Python over torch; its "FFI" for this path is the
 * Python call above.  A host binding (ctypes) passes device pointers taken from
 * torch tensors plus the current CUDA stream; nothing here uses torch types.
 *
 * Conventions
 *   - All pointers are DEVICE pointers unless stated otherwise.
 *   - Every call is asynchronous on `stream` and returns an ns_status (0 = ok)
 *     for argument / launch errors.  Errors found on the device (bad token id,
 *     NaN/inf probabilities, capacity overflow) are written per row into the
 *     output: out_ids[b] < 0 is the (negative) ns_status of row b.
 *   - The sampler never writes the logits (the reference mutates them in place
 *     at sampler.py:52; no caller depends on it).
 *   - ns_sample and ns_vp_local take a caller-allocated device workspace of
 *     ns_sampler_workspace_bytes bytes (256-byte aligned; 0 bytes, and NULL
 *     allowed, when max_history <= 1024).  It holds the history rank arrays
 *     of blocks that meet more distinct history ids than their shared memory
 *     keeps, so shared memory does not grow with the history length.  A call
 *     needs no particular contents on entry and leaves nothing the next call
 *     reads, but two calls that overlap on the device must not share one.
 */
#ifndef NS_SAMPLER_H
#define NS_SAMPLER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t (struct CUstream_st*). */
typedef struct CUstream_st* ns_stream_t;

typedef enum ns_status {
    NS_OK = 0,
    NS_ERR_INVALID_ARGUMENT = -1,
    NS_ERR_WORKSPACE_TOO_SMALL = -2,
    NS_ERR_UNSUPPORTED_DTYPE = -3,
    NS_ERR_CUDA = -4,
    NS_ERR_DEVICE_TIMEOUT = -5,        /* a bounded device-side wait gave up */
    NS_ERR_TOKEN_ID_OUT_OF_RANGE = -6, /* reference: IndexError at sampler.py:104 */
    NS_ERR_INVALID_DISTRIBUTION = -7,  /* NaN / +inf / all -inf in a sampled row;
                                          reference: torch.multinomial raises */
    NS_ERR_HISTORY_TOO_LONG = -8,      /* more distinct history ids than the
                                          per-block table holds */
    NS_ERR_CANDIDATE_OVERFLOW = -9,    /* ties at a top-k threshold exceed the
                                          candidate buffers */
    NS_ERR_UNSUPPORTED = -10
} ns_status;

typedef enum ns_dtype {
    NS_DTYPE_F32 = 0,
    NS_DTYPE_BF16 = 1,   /* widened to fp32 exactly, as the engine's .float() */
    NS_DTYPE_F16 = 2
} ns_dtype;

/* Human-readable text for an ns_status.  Never NULL. */
const char* ns_status_string(int status);

/* ABI version (major * 100 + minor). */
int ns_version(void);

/*
 * Workspace bytes ns_sample / ns_vp_local need for this problem size
 * (vocab: the columns the call reads).  0 when max_history <= 1024 (a
 * block's distinct history ids fit its shared memory); otherwise 12 B per
 * block per min(max_history, columns of a block): batch x (1-8 blocks per
 * row, by batch, vocab and the current device's SM count) blocks; 100.7 MB at
 * batch 256, vocab 151936, max_history 32768 on a 148-SM device.  Without a
 * device the widest clusters the vocabulary allows are assumed (an upper
 * bound).
 * Replaces: nothing (the reference allocates per call inside torch ops).
 */
int ns_sampler_workspace_bytes(int64_t batch, int64_t vocab, int64_t max_history,
                               size_t* out_bytes);

/*
 * Dynamic shared memory per block that ns_sample uses for this problem on a
 * device with sm_count SMs (a row with a history; no device needed): the
 * launch's own geometry and layout arithmetic.  It does not grow with
 * max_history -- a block keeps at most 1024 distinct history ids in shared
 * memory and the rest go to the workspace -- so two blocks fit an SM at any
 * history length (about 111 KB at vocab 151936, batch 256, 148 SMs).
 * Replaces: nothing (a sizing query).
 */
int ns_sampler_smem_bytes(int dtype, int64_t batch, int64_t vocab, int64_t max_history, int sm_count,
                          size_t* out_bytes);

/*
 * Sample one token per row.
 * Replaces: Sampler.select_batch (sampler.py:36-91), including
 *   _apply_repetition_penalty (sampler.py:93-108), greedy argmax (:60-70),
 *   temperature (:73-76), _apply_top_k_top_p (:110-133) and the
 *   softmax + multinomial draw (:86-89), which becomes an inverse-CDF draw.
 *
 * logits        [batch, row_stride] of `dtype`; only the first `vocab`
 *               columns of each row are read.  Element-aligned; 16-byte
 *               aligned rows are the fast path.
 * hist_ids      int32 token ids, CSR by row (prompt + outputs, duplicates
 *               allowed; context_builder.py:208-213).  May be NULL.
 * hist_offsets  int64 [batch + 1] row offsets into hist_ids.  May be NULL.
 * max_history   host-side upper bound on any row's history length.
 * temperature   fp32 [batch]; 0 => greedy.  (SamplingParams.temperature)
 * top_k         int32 [batch]; active iff 0 < k < vocab.
 * top_p         fp32 [batch]; active iff 0 < p < 1.
 * repetition_penalty, presence_penalty, frequency_penalty
 *               fp32 [batch] each, or NULL for 1.0 / 0.0 / 0.0.
 * uniforms      fp32 [batch] in [0,1), one draw per row; if NULL the kernel
 *               draws Philox4x32-10(counter = (row, philox_offset),
 *               key = philox_seed).
 * out_ids       int64 [batch]: sampled token id, or a negative ns_status.
 * workspace     device scratch of at least ns_sampler_workspace_bytes(batch,
 *               vocab, max_history) bytes, 256-byte aligned; otherwise the
 *               call returns NS_ERR_WORKSPACE_TOO_SMALL.
 */
int ns_sample(const void* logits, int dtype, int64_t batch, int64_t vocab, int64_t row_stride,
              const int32_t* hist_ids, const int64_t* hist_offsets, int64_t max_history,
              const float* temperature, const int32_t* top_k, const float* top_p,
              const float* repetition_penalty, const float* presence_penalty,
              const float* frequency_penalty,
              const float* uniforms, uint64_t philox_seed, uint64_t philox_offset,
              int64_t* out_ids, void* workspace, size_t workspace_bytes, ns_stream_t stream);

/*
 * Device-resident token histories for a decode loop: append each row's
 * sampled id to its history without a host round trip.
 * Replaces: the host-side history rebuild of the reference -- prompt +
 *   outputs lists built per step (engine/context_builder.py:208-213), the new
 *   id appended to the outputs (driver/output_processor.py:46) -- which
 *   select_batch then re-uploads.
 * Input: the CSR history (hist_ids int32, hist_offsets int64 [batch + 1]; both
 * NULL for empty histories) and new_ids int64 [batch] (ns_sample's out_ids).
 * Output (other buffers than the input): the same rows each followed by its
 * new id: out_hist_offsets[b] = hist_offsets[b] + b, out_hist_ids of
 * hist_offsets[batch] + batch elements.  out_capacity: elements out_hist_ids
 * holds; the caller sizes it (nothing past it is written).  A negative new id
 * (a failed row) is stored as -1, which the next ns_sample reports as
 * NS_ERR_TOKEN_ID_OUT_OF_RANGE for that row.
 */
int ns_hist_append(const int32_t* hist_ids, const int64_t* hist_offsets, int64_t batch, const int64_t* new_ids,
                   int32_t* out_hist_ids, int64_t* out_hist_offsets, int64_t out_capacity, ns_stream_t stream);

/*
 * ns_sample for callers that cannot allocate device memory.  No counterpart
 * in the reference: it is an addition of this library.
 *
 * Some callers may not call cudaMalloc (or any allocating routine) around a
 * sampling step: an engine whose device memory is carved up once at start-up
 * by its own pool, a plug-in living inside a host runtime that owns all
 * allocation, or code that must not allocate between steps.  This call takes
 * the same arguments as ns_sample except the workspace, and uses a scratch
 * array of NS_NOALLOC_SCRATCH_BYTES that is part of the library itself (a
 * fixed device array that every GPU which loads the library holds until the
 * process exits).
 *
 *   - A call whose ns_sampler_workspace_bytes(batch, vocab, max_history) is
 *     larger than NS_NOALLOC_SCRATCH_BYTES is refused with
 *     NS_ERR_WORKSPACE_TOO_SMALL before anything is launched.  Up to
 *     max_history 1024 no scratch is needed at all; at vocab 151936 and one
 *     block per row the limit allows about batch x max_history <= 1.39 M
 *     (for example batch 256 with histories of up to 5461 ids).
 *   - The first call on a device looks up that device's address of the
 *     array (no allocation); make that first call before any stream capture.
 *   - Every call on a device uses the same array.  The kernel clears what
 *     it needs before it reads it, so no call depends on what an earlier one
 *     left there, but two calls that overlap on the GPU (different streams
 *     without ordering) race on it: serialise them.
 *   - It calls no cudaMalloc, cudaFree or other allocating routine.
 */
#define NS_NOALLOC_SCRATCH_BYTES ((size_t)16 << 20)

int ns_sample_noalloc(const void* logits, int dtype, int64_t batch, int64_t vocab, int64_t row_stride,
                      const int32_t* hist_ids, const int64_t* hist_offsets, int64_t max_history,
                      const float* temperature, const int32_t* top_k, const float* top_p,
                      const float* repetition_penalty, const float* presence_penalty,
                      const float* frequency_penalty,
                      const float* uniforms, uint64_t philox_seed, uint64_t philox_offset,
                      int64_t* out_ids, ns_stream_t stream);

/*
 * Debug readback: the penalised logits of whole rows, fp32, for bit-exact
 * comparison with a reference.  out[b * out_stride + j] = logits[b][j] widened
 * to fp32, then for every distinct id of row b's history the value the
 * sampling kernels use: repetition (x * rep if x < 0 else x / rep), then
 * x - frequency * count, then x - presence, each rounded to fp32.  No
 * temperature.  row_status int32 [batch]: NS_OK or
 * NS_ERR_TOKEN_ID_OUT_OF_RANGE (that row of out holds only the widened
 * logits).  O(history^2) per row: a checking tool, not a hot path.
 * Replaces: Sampler._apply_repetition_penalty (sampler.py:93-108) as a
 *   standalone step (the reference applies it in place at sampler.py:52-57).
 */
int ns_penalize_debug(const void* logits, int dtype, int64_t batch, int64_t vocab, int64_t row_stride,
                      const int32_t* hist_ids, const int64_t* hist_offsets, const float* repetition_penalty,
                      const float* presence_penalty, const float* frequency_penalty, float* out,
                      int64_t out_stride, int32_t* row_status, ns_stream_t stream);

/*
 * Vocab-parallel sampling (tensor-parallel lm_head output: each device holds
 * a contiguous column slice of every row).  No reference counterpart: the
 * reference samples whole rows only (sampler.py:36-91); these calls split that
 * same computation into a local step, an all-gather of small per-row records
 * (done by the caller, e.g. NCCL), and a merge that every rank runs on the
 * same gathered bytes, so all ranks produce the same ids -- the ids ns_sample
 * would produce on the whole rows.
 *
 * Record layout (int64): [batch] survivor counts (or negative ns_status),
 * then [batch][cap] keys.  ns_vp_record_int64s gives its length.
 */
int ns_vp_record_int64s(int64_t batch, int cap, int64_t* out_count);

/*
 * Local step on this device's slice: columns [vocab_offset, vocab_offset +
 * vocab_local) of a vocab_total-wide row.  History ids are global ids; each
 * slice penalises the ones it holds.  Writes per row the top-k survivors
 * (ties at the k-th value kept) as keys, or for greedy rows (T == 0) one key.
 * Rows with top-k off or k > 240 report NS_ERR_UNSUPPORTED; more than `cap`
 * survivors report NS_ERR_CANDIDATE_OVERFLOW.  cap in [1, 1024].  workspace:
 * ns_sampler_workspace_bytes(batch, vocab_local, max_history) bytes, as in
 * ns_sample.
 */
int ns_vp_local(const void* logits, int dtype, int64_t batch, int64_t vocab_local, int64_t row_stride,
                int64_t vocab_offset, int64_t vocab_total,
                const int32_t* hist_ids, const int64_t* hist_offsets, int64_t max_history,
                const float* temperature, const int32_t* top_k, const float* top_p,
                const float* repetition_penalty, const float* presence_penalty,
                const float* frequency_penalty, int cap, int64_t* record,
                void* workspace, size_t workspace_bytes, ns_stream_t stream);

/*
 * Merge the all-gathered records (n_ranks consecutive records, rank order)
 * into one id per row: global top-k with ties, top-p, inverse CDF with the
 * row's uniform (or Philox as in ns_sample; the row index is the counter).
 * out_ids as in ns_sample.  n_ranks in [1, 64].
 */
int ns_vp_merge(const int64_t* gathered, int n_ranks, int64_t batch, int cap, int64_t vocab_total,
                const float* temperature, const int32_t* top_k, const float* top_p,
                const float* uniforms, uint64_t philox_seed, uint64_t philox_offset,
                int64_t* out_ids, ns_stream_t stream);

/*
 * Peer-memory exchange for the vocab-parallel merge (no reference
 * counterpart).  Instead of an all-gather, every rank keeps its record in its
 * own device memory and the merge kernel reads all ranks' records in place
 * over NVLink (peer loads), after a bounded wait on flags the ranks set.
 * Per step (two record buffers used on alternate steps, so a rank never
 * overwrites a record a peer may still read; `epoch` is this rank's step
 * counter in device memory, zero at first):
 *   ns_vp_local(... record = my_records[step % 2] ...)
 *   ns_vp_signal(rank_flags, n, me, epoch)   -- ++*epoch; every rank's flags[me] = *epoch
 *   ns_vp_merge_peers(records[r] = rank r's my_records[step % 2], ..., my_flags, epoch)
 * The merge waits until my_flags[r] >= *epoch for every r; a rank whose
 * flags do not get there within 200 ms gets NS_ERR_DEVICE_TIMEOUT in its
 * out_ids.  The counter lives on the device, so a captured CUDA graph of an
 * even number of steps can be replayed.  n_ranks in [1, 8].
 */
#define NS_IPC_HANDLE_BYTES 64

int ns_vp_signal(int64_t* const* rank_flags, int n_ranks, int my_rank, int64_t* epoch, ns_stream_t stream);

int ns_vp_merge_peers(const int64_t* const* rank_records, int n_ranks, const int64_t* my_flags,
                      const int64_t* epoch, int64_t batch, int cap, int64_t vocab_total, const float* temperature,
                      const int32_t* top_k, const float* top_p, const float* uniforms, uint64_t philox_seed,
                      uint64_t philox_offset, int64_t* out_ids, ns_stream_t stream);

/* Device buffer for records and flags (zero-filled), and its release. */
int ns_vp_peer_alloc(size_t bytes, void** out_ptr);
int ns_vp_peer_free(void* ptr);

/* CUDA IPC: a buffer's handle (NS_IPC_HANDLE_BYTES bytes, host memory) and
 * its mapping in another process on the same node (peer access enabled). */
int ns_ipc_handle(const void* ptr, void* out_handle);
int ns_ipc_open(const void* handle, void** out_ptr);
int ns_ipc_close(void* ptr);

#ifdef __cplusplus
}
#endif

#endif /* NS_SAMPLER_H */
