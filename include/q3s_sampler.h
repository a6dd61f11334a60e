/*
 * q3s_sampler.h — C ABI of the B200 token sampler for the Qwen3-TTS talker and
 * code predictor (qwen3tts-rs 0.2.0, src/talker/sampling.rs).
 *
 * The reference sampler downloads every logit row to the host and samples it on
 * one CPU thread.  This library samples rows where they already live (device
 * memory) and returns only the token id and a status byte per row.  Every entry
 * point below names the reference interface it replaces.
 *
 * Conventions
 *   - Functions return Q3S_OK (0) or a negative Q3S_E_* code; the text of the
 *     last failure on the calling thread is in q3s_last_error().
 *   - Per-row sampling outcomes are Q3S_STATUS_* bytes (>= 0).  Their messages
 *     (q3s_status_message) are the reference's error strings.
 *   - "stream" is a cudaStream_t passed as void*; NULL is the legacy default
 *     stream.  Batch calls are asynchronous on that stream.
 *   - No torch types: plain pointers and sizes.
 */
#ifndef Q3S_SAMPLER_H
#define Q3S_SAMPLER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define Q3S_ABI_VERSION 2 /* 2: q3s_batch.history_ends appended */

/* ---- return codes of API calls ------------------------------------------ */
#define Q3S_OK 0
#define Q3S_E_INVALID_ARGUMENT (-1)
#define Q3S_E_CUDA (-2)
#define Q3S_E_NO_DEVICE (-3)
#define Q3S_E_OUT_OF_MEMORY (-4)
#define Q3S_E_SAMPLING (-5) /* a single-row call whose row status is not OK */

/* ---- per-row outcome (status byte) --------------------------------------
 * Values and messages follow src/talker/sampling.rs:
 *   INVALID_REPETITION_PENALTY  :281-285
 *   INVALID_TEMPERATURE         :286-291
 *   INVALID_TOP_P               :292-296
 *   SUPPRESSION_NO_CANDIDATE    :642-647 (sampled) and :58-59 (greedy_select)
 *   NO_CANDIDATE                :588-590 (greedy), :648-650, :705-708
 *   INVALID_DENOMINATOR         :675-678, :715-718
 * A row counts one Philox draw (its subsequence advances by one) exactly when
 * do_sample is set and the status is OK (sampling.rs:298-305, 330-332).     */
#define Q3S_STATUS_OK 0
#define Q3S_STATUS_INVALID_REPETITION_PENALTY 1
#define Q3S_STATUS_INVALID_TEMPERATURE 2
#define Q3S_STATUS_INVALID_TOP_P 3
#define Q3S_STATUS_SUPPRESSION_NO_CANDIDATE 4
#define Q3S_STATUS_NO_CANDIDATE 5
#define Q3S_STATUS_INVALID_DENOMINATOR 6
#define Q3S_STATUS_UNSUPPORTED 7 /* vocabulary larger than Q3S_MAX_VOCAB */
#define Q3S_STATUS_INVALID_CODE 8 /* q3s_embed_sum: a code outside its codebook (row zeroed) */
#define Q3S_STATUS_HISTORY_FULL 9 /* q3s_commit_rows: no room to append the sampled c0 id */
#define Q3S_STATUS_NOT_RUN 255   /* row was never reached (internal error) */

/* Largest vocabulary one row may have (the codec vocabularies are 3072 and 2048). */
#define Q3S_MAX_VOCAB 4096

/* ---- element types of logits -------------------------------------------- */
#define Q3S_DTYPE_F32 0
#define Q3S_DTYPE_BF16 1 /* upcast exactly to f32 before any arithmetic */

/* "None" for suppress_from / allow_suppressed_token. */
#define Q3S_NONE (-1)

/* Mirrors SamplingOptions (sampling.rs:19-25).  The f64 fields keep the
 * reference's f64 validation and comparisons (rp != 1.0, top_p < 1.0); the
 * kernel casts to f32 where the reference does (`as f32`). */
typedef struct q3s_sampling_options {
  double temperature;
  uint64_t top_k; /* 0 = off */
  double top_p;
  double repetition_penalty;
} q3s_sampling_options;

/* Per-row parameters of a batched call (device memory, 48 bytes).
 * suppress_from / allow_token: Q3S_NONE for None; values beyond the row's
 * vocabulary are legal and behave as in the reference. */
typedef struct q3s_row_params {
  double temperature;
  double top_p;
  double repetition_penalty;
  uint32_t top_k;        /* 0 = off; values >= vocabulary keep every candidate */
  uint32_t do_sample;    /* 0 = greedy argmax over raw logits (sampling.rs:576-591) */
  int32_t suppress_from; /* Q3S_NONE or index */
  int32_t allow_token;   /* Q3S_NONE or index */
  uint32_t ctr_lo;       /* Philox counter word 0; the reference's Sampler keeps it 0 */
  uint32_t reserved;
} q3s_row_params;

/* One batched sampling launch.  All pointers are device pointers unless noted.
 *
 * Row r's logits start at element row_offsets[r] (or r*row_stride when
 * row_offsets is NULL) and hold row_vocab[r] (or vocab) elements.  Its
 * parameters are params[r*params_stride] (params_stride 0 broadcasts one
 * struct).  Its history is history[history_offsets[r] .. history_offsets[r+1])
 * (no history when history_offsets is NULL), or
 * history[history_offsets[r] .. history_ends[r]) when history_ends is set
 * (per-row ranges that need not abut: fixed-capacity per-session slots).
 * Its Philox key/counter are seeds[r] / subseqs[r]. */
typedef struct q3s_batch {
  const void* logits;
  int32_t dtype;
  int32_t vocab;
  int64_t num_rows;
  int64_t row_stride;
  const int64_t* row_offsets;     /* [num_rows] or NULL */
  const int32_t* row_vocab;       /* [num_rows] or NULL */
  const q3s_row_params* params;   /* [num_rows] or [1] */
  int64_t params_stride;          /* 0 or 1 */
  const uint64_t* seeds;          /* [num_rows] */
  const uint64_t* subseqs;        /* [num_rows] */
  const uint16_t* history;        /* concatenated c0 history ids */
  const int64_t* history_offsets; /* [num_rows + 1] or NULL */
  uint32_t* tokens;               /* out [num_rows] */
  uint8_t* status;                /* out [num_rows] */
  /* Optional, for testing and debugging (NULL in production):            */
  const float* uniform_override;  /* [num_rows]: use this draw instead of Philox */
  float* probs;                   /* out [num_rows * probs_stride]: final softmax over survivors */
  uint8_t* masks;                 /* out [num_rows * probs_stride]: bit0 candidate, bit1 top-k, bit2 top-p */
  int64_t probs_stride;
  const int64_t* history_ends;    /* [num_rows] or NULL (see above) */
} q3s_batch;

/* Codebook embedding sum after sampling (talker.rs:568-580): for each row,
 * out = ((T0[c0] + T1[c1]) + ... + T(G-1)[c(G-1)]) + text, every addition
 * rounded to the element type, in that order.  T0 is the talker's codec
 * embedding (codebook 0), T1.. the code predictor's codebook embeddings;
 * text is the trailing text hidden state or tts_pad. */
#define Q3S_MAX_CODE_GROUPS 32

typedef struct q3s_embed_batch {
  int32_t dtype;              /* Q3S_DTYPE_F32 or Q3S_DTYPE_BF16 (tables, text and out) */
  int32_t groups;             /* G, 1..Q3S_MAX_CODE_GROUPS (16 for the 12 Hz models) */
  int32_t hidden;             /* H, elements per embedding row */
  int32_t reserved;
  int64_t num_rows;           /* R */
  const uint32_t* codes;      /* [R, G], row-major */
  const void* const* tables;  /* HOST array of G device pointers; table g is [vocab[g], H] */
  const int32_t* vocab;       /* HOST array [G] */
  const void* text;           /* [R, H] (or one row), added last; NULL for none */
  int64_t text_stride;        /* elements between text rows; 0 broadcasts one row */
  void* out;                  /* [R, H] */
  uint8_t* status;            /* [R]: Q3S_STATUS_OK, or Q3S_STATUS_INVALID_CODE */
} q3s_embed_batch;

/* ---- library / context --------------------------------------------------- */
typedef struct q3s_context q3s_context;

int q3s_abi_version(void);
const char* q3s_last_error(void);
const char* q3s_status_message(int status);

/* One context per (device, host thread).  Holds the launch configuration and
 * small staging buffers for single-row calls. */
int q3s_context_create(int device, q3s_context** out);
void q3s_context_destroy(q3s_context* ctx);

/* Batched sampling: the fused penalty / mask / temperature / top-k / top-p /
 * Philox-draw kernel over many rows.  Replaces, per row, one call of
 * Sampler::sample_with_mode_and_transfer_observer (sampling.rs:247-334) minus
 * its host download (sampling.rs:273).  Does not advance any counter: the
 * caller advances subseq for rows whose status is OK and do_sample is set. */
int q3s_sample_batch(q3s_context* ctx, const q3s_batch* batch, void* stream);

/* Testing hook, no counterpart in the reference.  Every wait of the sampling
 * kernel is bounded: a row whose staged logits do not arrive in time ends
 * with Q3S_STATUS_NOT_RUN (the rows after it in its block too) and the call
 * returns, so a stuck copy never hangs the device.  This sets, for the
 * batched launches of `ctx`, the per-row wait limit (stage_wait_ns; 0 keeps
 * the default of one second) and, with hold_refill != 0, stops the kernel
 * from refilling a ring stage after its first row, so that every later row's
 * wait runs out without any copy in flight.  Tests use it to exercise the
 * give-up path; production code never calls it. */
int q3s_context_set_test_hooks(q3s_context* ctx, uint64_t stage_wait_ns, int32_t hold_refill);

/* Diagnostics, no counterpart in the reference: which path of the sampling
 * kernel each row took.  The reference runs one algorithm on the host; the
 * kernel decides most rows from a short candidate list and sends the rest to
 * slower, equally exact paths, and these counts show how often.           */
#define Q3S_PATH_INVALID 0          /* status set before sampling (validation, vocabulary) */
#define Q3S_PATH_GREEDY 1           /* do_sample = 0 */
#define Q3S_PATH_TOPK 2             /* candidate list, top-k finisher */
#define Q3S_PATH_TOPK_TOPP 3        /* candidate list, top-k then top-p finisher */
#define Q3S_PATH_FRONT_DONE 4       /* decided by the scan (no candidate, +inf after temperature) */
#define Q3S_PATH_NUCLEUS 5          /* top-p without top-k from the staged row */
#define Q3S_PATH_GENERAL_RULES 6    /* general: top_k 0, > 256 or >= vocab; 1/T 0 or inf; bf16 */
#define Q3S_PATH_GENERAL_INF 7      /* general: +inf raw logit */
#define Q3S_PATH_GENERAL_TAU 8      /* general: no threshold on the vector maxima */
#define Q3S_PATH_GENERAL_OVERFLOW 9 /* general: more candidates than the list holds */
#define Q3S_PATH_GENERAL_WIDE 10    /* general: more than 256 top-k survivors under top-p */
#define Q3S_PATH_GENERAL_NUCLEUS 11 /* general: the nucleus outgrew its candidates */
#define Q3S_PATH_COUNT 12

/* stats: NULL (off) or a device array of 2 * Q3S_PATH_COUNT u64.  While set,
 * every batched launch of `ctx` adds to stats[p] the rows that took path p
 * and to stats[Q3S_PATH_COUNT + p] the SM clock cycles their warps spent on
 * them (from taking the row to storing its result).  Nothing is cleared.
 * Such launches run the kernel's debug build (same results, slower). */
int q3s_context_set_path_stats(q3s_context* ctx, uint64_t* stats);

/* Bytes of the file-scope device workspace of q3s_sample_batch_static, held on
 * every device that loads the library until the process exits. */
#define Q3S_STATIC_SCRATCH_BYTES (32u * 1024u * 1024u)

/* q3s_sample_batch without any device allocation, for callers that must not
 * call cudaMalloc: an engine whose device memory belongs to its own pool
 * allocator (a stray allocation can exceed that pool's budget), or a
 * per-step generation loop that cannot take the device-wide synchronisation
 * cudaMalloc / cudaFree may cause.  The same kernel runs, with its
 * general-path workspace in a file-scope device array of
 * Q3S_STATIC_SCRATCH_BYTES instead of a context allocation.  No counterpart
 * in the reference, which samples on the host (src/talker/sampling.rs) and
 * keeps no device workspace.  Same arguments and results as
 * q3s_sample_batch; in addition it rejects vocab > Q3S_MAX_VOCAB with
 * Q3S_E_INVALID_ARGUMENT, and it launches only as many blocks as the array
 * holds workspace for (about 14 bytes per vocabulary entry per warp, up to
 * 16 warps a block: 73 blocks at vocab 2048, 48 at 3072, 45 at 4096).  Every
 * call looks up the array's address on its device (cudaGetSymbolAddress,
 * which allocates nothing); the first call on a device may load the module,
 * so make it before any stream capture.  Calls share the array and
 * nothing in it has to start at zero; calls whose kernels overlap on the GPU
 * race on it, so order them on one stream or with events. */
int q3s_sample_batch_static(q3s_context* ctx, const q3s_batch* batch, void* stream);

/* The embedding sum of many rows (streams) in one launch, on the device that
 * holds the sampled codes.  Replaces, per row, the embedding_lookup and
 * tensor additions of talker.rs:568-580 (embedding_lookup:
 * src/talker/primitives.rs:17-25).  A row with a code at or beyond its
 * codebook's vocabulary gets status Q3S_STATUS_INVALID_CODE and zeros
 * (the reference's index_select fails there). */
int q3s_embed_sum(q3s_context* ctx, const q3s_embed_batch* batch, void* stream);

/* Greedy argmax with the talker reserved-token mask, many rows, on device.
 * mode Q3S_GREEDY_SELECT follows greedy_select (sampling.rs:40-60): first
 * index of the IEEE maximum over finite allowed entries; status
 * SUPPRESSION_NO_CANDIDATE when none.  mode Q3S_GREEDY_ON_DEVICE follows
 * greedy_select_on_device (sampling.rs:72-117): the token is vocab (the
 * sentinel) when no finite candidate remains, status stays OK; ties resolve to
 * the lowest index (the contract stated at sampling.rs:70-71). */
#define Q3S_GREEDY_SELECT 0
#define Q3S_GREEDY_ON_DEVICE 1
int q3s_greedy_batch(q3s_context* ctx, const void* logits, int32_t dtype, int64_t num_rows,
                     int64_t row_stride, int32_t vocab, int64_t suppress_from,
                     int64_t allow_token, int32_t mode, uint32_t* tokens, uint8_t* status,
                     void* stream);

/* ---- producer fusion: head projection + sampling --------------------------
 * The logits of a decode step come from a head projection without bias,
 * logits = hidden · weightᵀ: the talker's codec_head (talker.rs:87-89, used
 * at :501) and the code predictor's lm_heads[g] (code_predictor.rs:402),
 * via primitives.rs:32-42.  q3s_head_sample computes that projection and
 * samples its rows in one launch, for the small batches of the decode loop
 * (at most Q3S_HEAD_MAX_ROWS rows): every block computes a slice of the
 * logits (f32 products and sums of the bf16 weights and the hidden values,
 * in a fixed order, so every launch gives the same logits), writes it to
 * `logits`, and the last block to finish samples every row with the
 * sampler of q3s_sample_batch.  The logits stay in L2 between the two; the
 * caller gets them too.  The reference computes the projection with its
 * matmul (bf16 with f32 accumulation in an order of the library's choosing),
 * so logits agree with it within rounding, and the sampled ids are exactly
 * those q3s_sample_batch gives for the returned logits.
 *
 * sample: the rows' sampling arguments as for q3s_sample_batch (vocab,
 * num_rows, params, seeds, subseqs, history, tokens, status, ...); its
 * logits, dtype, row_stride, row_offsets, row_vocab, probs and masks are not
 * used (probs / masks must be NULL).  Path statistics are not collected. */
#define Q3S_HEAD_MAX_ROWS 16
typedef struct q3s_head_batch {
  const void* hidden;            /* [num_rows, hidden_size], row stride hidden_stride elements */
  int32_t hidden_dtype;          /* Q3S_DTYPE_F32 or Q3S_DTYPE_BF16 */
  int32_t hidden_size;           /* H, a positive multiple of 8 */
  int64_t hidden_stride;         /* >= H */
  const uint16_t* weight;        /* bf16 [sample.vocab, H], row-major, 16-byte aligned */
  float* logits;                 /* out [num_rows, sample.vocab] f32 */
  q3s_batch sample;
} q3s_head_batch;

int q3s_head_sample(q3s_context* ctx, const q3s_head_batch* batch, void* stream);

/* ---- device-resident decode frame ---------------------------------------
 * The host work that follows every Sampler call of the talker and
 * code-predictor loops, done on the device: the sampled id becomes the next
 * step's input (Tensor::new(&[next_val]) at code_predictor.rs:365, 414 and
 * talker.rs:530; the codes of a frame, code_predictor.rs:421), the counter
 * advances on a draw (sampling.rs:330-332) and the c0 id joins the talker's
 * history (talker.rs:562-566).  With it, the 16 sampling launches of a frame
 * (1 talker + 15 code-predictor groups) run back to back with no host round
 * trip; the caller reads frame_status (and the codes) once per frame.
 *
 * For each row r of a finished batched launch, in stream order after it:
 *   codes[r * codes_stride + group] = tokens[r]            (codes non-NULL)
 *   if frame_status is NULL or frame_status[r] is OK:
 *     subseqs[r] += 1 when status[r] is OK and the row sampled (do_sample)
 *     with history: on OK, history[history_ends[r]++] = tokens[r] if
 *       history_ends[r] < history_limits[r], else status Q3S_STATUS_HISTORY_FULL
 *     frame_status[r] = that status                       (frame_status non-NULL)
 * so a stream's counter and history stop at its first failed call, where the
 * reference's frame stops with an error.  All pointers are device pointers;
 * NULL skips that part. */
typedef struct q3s_commit {
  int64_t num_rows;
  const q3s_row_params* params; /* the launch's params (for do_sample) */
  int64_t params_stride;        /* 0 or 1 */
  const uint32_t* tokens;       /* the launch's outputs */
  const uint8_t* status;
  uint64_t* subseqs;            /* in/out, usually the launch's own subseqs array */
  uint32_t* codes;              /* [num_rows, codes_stride] frame codes (u32, q3s_embed_sum's input) */
  int64_t codes_stride;
  int32_t group;                /* column of this launch's ids */
  int32_t reserved;
  uint8_t* frame_status;        /* in/out: first non-OK status of the frame, per row */
  uint16_t* history;            /* append target (the c0 history of each row) */
  int64_t* history_ends;        /* in/out: one past each row's last id */
  const int64_t* history_limits;/* capacity end of each row's history range */
} q3s_commit;

int q3s_commit_rows(q3s_context* ctx, const q3s_commit* commit, void* stream);

/* q3s_sample_batch followed by q3s_commit_rows, in one launch: each row's
 * warp commits the row right after storing its result.  `commit`'s
 * num_rows, params, params_stride, tokens and status are not read (the
 * batch's are used); its other fields are as for q3s_commit_rows.  Rows are
 * the batch's rows, so `subseqs` is usually the batch's own subseqs array
 * and the history fields the batch's history, history_ends and a limits
 * array.  The batch's probs and masks must be NULL, and the context's path
 * statistics are not collected for these launches. */
int q3s_sample_commit(q3s_context* ctx, const q3s_batch* batch, const q3s_commit* commit,
                      void* stream);

/* ---- continuous batching of sessions ------------------------------------
 * The scheduler the reference plans for many concurrent synthesis sessions
 * (tasks/P12-c-abi-and-continuous-batching.md:11-16: P12-T03 per-session
 * scheduler state, P12-T04 bounded talker / predictor batching; the
 * SessionScheduler contract add / tick / cancel of
 * templates/rust-contracts/session.rs), for the sampling side of a frame.
 * Each session keeps what its own Sampler and talker loop keep in the
 * reference: seed and subsequence counter (sampling.rs:144-179), talker and
 * code-predictor options, the talker suppression, and its c0 history
 * (talker.rs:500-566), all on the device.  One frame (the contract's tick)
 * is begin_frame, one step per code group (group 0: the talker row of every
 * active session, with its history; groups 1..G-1: code-predictor rows),
 * then end_frame; each step is one sampling launch over all active
 * sessions plus the device-side commit (q3s_commit_rows), so a session's
 * ids, counter and history are those it would get alone.
 *
 * Sessions join (add) and leave (cancel) between frames: both take effect
 * at the next begin_frame, which also retires every session whose frame
 * ended with a non-OK status (the reference's session step returns its
 * error).  begin_frame reports the active sessions in row order: row r of
 * every step's logits belongs to ids[r].  All calls of one scheduler go on
 * one stream, from one host thread. */
typedef struct q3s_scheduler q3s_scheduler;

typedef struct q3s_session_config {
  uint64_t id;                    /* unique among the scheduler's sessions */
  uint64_t seed;                  /* Sampler::new(seed), sampling.rs:158-170 */
  uint64_t subseq;                /* starting subsequence counter (0 for a new request) */
  q3s_sampling_options talker;    /* talker options (plan-resolved, talker.rs:452-461) */
  q3s_sampling_options predictor; /* code-predictor options (code_predictor.rs:357-364) */
  int32_t talker_do_sample;
  int32_t predictor_do_sample;
  int32_t suppress_from;          /* talker row suppression (Q3S_NONE: none) */
  int32_t allow_token;            /* the token it still allows (EOS), or Q3S_NONE */
  const uint16_t* history;        /* HOST: initial c0 history, copied by q3s_scheduler_add */
  int64_t history_len;
} q3s_session_config;

/* max_sessions slots; `groups` code groups per frame (16 for the 12 Hz
 * models: 1 talker + 15 code-predictor); history_capacity c0 ids per session
 * (a session whose history is full stops with Q3S_STATUS_HISTORY_FULL). */
int q3s_scheduler_create(q3s_context* ctx, int32_t max_sessions, int32_t groups,
                         int64_t history_capacity, q3s_scheduler** out);
void q3s_scheduler_destroy(q3s_scheduler* sched);
/* Joins at the next begin_frame.  Rejects a duplicate id, a history longer
 * than the capacity, and an add that would exceed max_sessions. */
int q3s_scheduler_add(q3s_scheduler* sched, const q3s_session_config* config);
/* Leaves at the next begin_frame (a pending add is simply dropped). */
int q3s_scheduler_cancel(q3s_scheduler* sched, uint64_t id);
/* Applies joins and leaves, writes the active session ids in row order to
 * ids[0 .. min(n, cap)) (HOST) and their number to *n. */
int q3s_scheduler_begin_frame(q3s_scheduler* sched, uint64_t* ids, int32_t cap, int32_t* n,
                              void* stream);
/* Step `group` (0, 1, .. in order): logits row r (device, dtype, `vocab`
 * entries, row_stride elements apart) belongs to session ids[r]. */
int q3s_scheduler_step(q3s_scheduler* sched, int32_t group, const void* logits, int32_t dtype,
                       int32_t vocab, int64_t row_stride, void* stream);
/* After the last group: one device-to-host copy of the frame's codes
 * (HOST [n * groups], row-major) and statuses (HOST [n]); synchronises. */
int q3s_scheduler_end_frame(q3s_scheduler* sched, uint32_t* codes, uint8_t* status,
                            void* stream);
/* The frame's codes on the device ([n, groups] u32, the input of
 * q3s_embed_sum), valid until the next begin_frame. */
const uint32_t* q3s_scheduler_codes(const q3s_scheduler* sched);
/* An active session's counter and c0 history (HOST copies; synchronous). */
int q3s_scheduler_session_state(q3s_scheduler* sched, uint64_t id, uint64_t* subseq,
                                int64_t* history_len, uint16_t* history, int64_t cap);

/* ---- stateful sampler: the drop-in for `Sampler` ------------------------ */
/* Mirrors Sampler (sampling.rs:144-335): one Philox stream (seed, subsequence
 * counter) shared by the talker and code-predictor calls of one request. */
typedef struct q3s_sampler q3s_sampler;

typedef struct q3s_sampler_diagnostics { /* SamplerDiagnostics, sampling.rs:27-37 */
  uint32_t call_count;
  uint32_t sampled_calls;
  uint32_t greedy_calls;
  uint32_t history_nonempty_calls;
  uint8_t history_nonempty_sequence[64];
  uint8_t sequence[64];
  uint64_t sequence_len;
} q3s_sampler_diagnostics;

/* Transfer observer (TransferObserver, src/alignment_stage_dump.rs:40-51).
 * The device sampler moves one token per call instead of the full logit
 * vector; the event reports what crossed the device boundary. */
#define Q3S_TRANSFER_SAMPLED_TOKEN 0 /* 1 element device->host per call */
typedef void (*q3s_transfer_callback)(void* user_data, int32_t direction, int32_t event,
                                      uint64_t elements);

/* Sampler::new (sampling.rs:158-170). */
int q3s_sampler_create(q3s_context* ctx, uint64_t seed, q3s_sampler** out);
void q3s_sampler_destroy(q3s_sampler* s);
/* Sampler::subsequence_counter (sampling.rs:174); the setter supports resume
 * from a saved (seed, subsequence) pair. */
uint64_t q3s_sampler_subsequence_counter(const q3s_sampler* s);
void q3s_sampler_set_subsequence_counter(q3s_sampler* s, uint64_t subseq);
/* Sampler::diagnostics (sampling.rs:179). */
int q3s_sampler_get_diagnostics(const q3s_sampler* s, q3s_sampler_diagnostics* out);

/* Sampler::sample_with_mode_and_transfer_observer (sampling.rs:247-334).
 * logits: device pointer to n elements of dtype.  history: HOST pointer to
 * hist_len u16 ids (the c0 history).  suppress_from / allow_token: Q3S_NONE
 * for None.  Returns Q3S_OK with *token set, Q3S_E_SAMPLING with *row_status
 * set to the reference error, or another negative code.  Synchronises the
 * stream to read the token (4 bytes + 1 status byte). */
int q3s_sampler_sample_with_mode(q3s_sampler* s, const void* logits, int32_t dtype, int64_t n,
                                 const q3s_sampling_options* options, int32_t do_sample,
                                 int64_t suppress_from, int64_t allow_token,
                                 const uint16_t* history, int64_t hist_len,
                                 q3s_transfer_callback observer, void* observer_user_data,
                                 uint32_t* token, int32_t* row_status, void* stream);
/* Sampler::sample / sample_with_transfer_observer (sampling.rs:183-221):
 * do_sample = temperature > 0. */
int q3s_sampler_sample(q3s_sampler* s, const void* logits, int32_t dtype, int64_t n,
                       const q3s_sampling_options* options, int64_t suppress_from,
                       int64_t allow_token, const uint16_t* history, int64_t hist_len,
                       uint32_t* token, int32_t* row_status, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* Q3S_SAMPLER_H */
