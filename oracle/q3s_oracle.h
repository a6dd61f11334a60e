/*
 * ORACLE — test infrastructure only.  A CPU restatement of the reference
 * sampler (qwen3tts-rs 0.2.0, src/talker/sampling.rs).  Only tests/, the smoke
 * check of __graft_entry__.py and bench.py's CPU-baseline leg use it; the
 * product library never links or calls it.
 *
 * Parity is pinned against the reference's own fixtures
 * (fixtures/alignment/p02_*.json) and the literal cases of its unit tests
 * (src/talker/sampling.rs:789-1147), converted to tests/golden/ by
 * tests/golden/make_golden.py.
 */
#ifndef Q3S_ORACLE_H
#define Q3S_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status values: identical numbers to include/q3s_sampler.h. */
enum {
  Q3O_OK = 0,
  Q3O_INVALID_REPETITION_PENALTY = 1,
  Q3O_INVALID_TEMPERATURE = 2,
  Q3O_INVALID_TOP_P = 3,
  Q3O_SUPPRESSION_NO_CANDIDATE = 4,
  Q3O_NO_CANDIDATE = 5,
  Q3O_INVALID_DENOMINATOR = 6,
};

/* exp used for every f32 exponential of the sampler.
 *   Q3O_EXP_CR   correctly rounded binary32 exp, evaluated in binary64 with a
 *                Cody-Waite reduction and a degree-13 Taylor polynomial; the
 *                product kernel evaluates the same operation sequence.
 *   Q3O_EXP_LIBM the platform expf (glibc here), which is what Rust's f32::exp
 *                calls on Linux. */
enum { Q3O_EXP_CR = 0, Q3O_EXP_LIBM = 1 };

typedef struct q3o_options { /* SamplingOptions, sampling.rs:19-25 */
  double temperature;
  uint64_t top_k;
  double top_p;
  double repetition_penalty;
} q3o_options;

/* Optional intermediate results of one sampled call (any pointer may be NULL;
 * arrays have n entries). */
typedef struct q3o_trace {
  float* after_penalty;   /* row after apply_repetition_penalty (sampling.rs:592-606) */
  float* after_temperature; /* after mask + temperature (sampling.rs:608-631) */
  float* final_probs;     /* exp(x - max) / sum over the survivors, 0 elsewhere */
  uint8_t* masks;         /* bit0 finite candidate, bit1 kept by top-k, bit2 kept by top-p */
  float topk_threshold;   /* -inf when top-k did not mask */
  float draw_threshold;   /* (r as f32) * sum */
  float draw_sum;         /* the sequential f32 softmax sum */
  double boundary_gap;    /* min |cum_j - threshold| / sum over the crossing neighbours */
  double topp_gap;        /* min over the nucleus decisions (positions >= 1) of
                             |cumulative before the position - top_p|; +inf without top-p */
} q3o_trace;

typedef struct q3o_sampler { /* Sampler state, sampling.rs:144-155 */
  uint64_t seed;
  uint64_t subseq_counter;
  uint32_t ctr_lo;
  uint32_t call_count, sampled_calls, greedy_calls, history_nonempty_calls;
  uint8_t history_nonempty_sequence[64];
  uint8_t sequence[64];
  uint64_t sequence_len;
} q3o_sampler;

float q3o_expf(float x, int exp_mode);
float q3o_cr_expf(float x);

/* philox4x32_10 (sampling.rs:350-361) and next_uniform (:363-375). */
void q3o_philox4x32_10(const uint32_t ctr[4], uint32_t seed_lo, uint32_t seed_hi, uint32_t out[4]);
float q3o_next_uniform(uint64_t seed, uint64_t subsequence, uint32_t ctr_lo);

/* apply_repetition_penalty (sampling.rs:732-773), in place on n values. */
void q3o_apply_repetition_penalty(float* logits, size_t n, const uint16_t* history, size_t hist_len,
                                  double penalty);

/* sample_logits_with_scratch (sampling.rs:561-730).  suppress_from /
 * allow_token < 0 mean None.  `uniform` is the value rand01() would return
 * (as f32); *drew reports whether rand01 was called. */
int q3o_sample_logits(const float* logits, size_t n, q3o_options opt, int64_t suppress_from,
                      int64_t allow_token, const uint16_t* history, size_t hist_len, float uniform,
                      int exp_mode, uint32_t* token, int* drew, q3o_trace* trace);

/* greedy_select (sampling.rs:40-60). */
int q3o_greedy_select(const float* logits, size_t n, int64_t suppress_from, int64_t allow_token,
                      uint32_t* token);
/* greedy_select_on_device (sampling.rs:72-117): returns n when nothing is finite. */
uint32_t q3o_greedy_select_on_device(const float* logits, size_t n, int64_t suppress_from,
                                     int64_t allow_token);

/* Sampler (sampling.rs:158-334). */
void q3o_sampler_init(q3o_sampler* s, uint64_t seed);
int q3o_sampler_sample_with_mode(q3o_sampler* s, const float* logits, size_t n, q3o_options opt,
                                 int do_sample, int64_t suppress_from, int64_t allow_token,
                                 const uint16_t* history, size_t hist_len, int exp_mode,
                                 uint32_t* token, q3o_trace* trace);

/* One batched call with the same row layout as q3s_batch (host memory).
 * Row r: logits + offsets[r], vocab[r] elements; parameters params[r] as the
 * q3s_row_params layout (48 bytes); history ids hist[hoff[r]..hoff[r+1]).
 * nthreads > 1 splits rows across POSIX threads. */
typedef struct q3o_row_params { /* same layout as q3s_row_params */
  double temperature;
  double top_p;
  double repetition_penalty;
  uint32_t top_k;
  uint32_t do_sample;
  int32_t suppress_from;
  int32_t allow_token;
  uint32_t ctr_lo;
  uint32_t reserved;
} q3o_row_params;

int q3o_sample_rows(const float* logits, int64_t num_rows, const int64_t* offsets,
                    const int32_t* vocab, const q3o_row_params* params, int64_t params_stride,
                    const uint64_t* seeds, const uint64_t* subseqs, const uint16_t* hist,
                    const int64_t* hoff, const float* uniform_override, int exp_mode,
                    uint32_t* tokens, uint8_t* status, float* probs, uint8_t* masks,
                    int64_t probs_stride, double* boundary_gap, int nthreads);

/* q3o_sample_rows plus the per-row top-p decision gap (q3o_trace.topp_gap);
 * topp_gap may be NULL. */
int q3o_sample_rows_ex(const float* logits, int64_t num_rows, const int64_t* offsets,
                       const int32_t* vocab, const q3o_row_params* params, int64_t params_stride,
                       const uint64_t* seeds, const uint64_t* subseqs, const uint16_t* hist,
                       const int64_t* hoff, const float* uniform_override, int exp_mode,
                       uint32_t* tokens, uint8_t* status, float* probs, uint8_t* masks,
                       int64_t probs_stride, double* boundary_gap, double* topp_gap,
                       int nthreads);

#ifdef __cplusplus
}
#endif
#endif
