// ORACLE — test infrastructure only.
//
// A CPU restatement of the reference sampler of qwen3tts-rs 0.2.0
// (src/talker/sampling.rs).  Each function cites the lines it follows.  Only
// tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load this
// library; the product library never links or calls it.
//
// Build: oracle/Makefile (g++ -O3 -ffp-contract=off; binary32 arithmetic in
// SSE registers, so every f32 operation rounds exactly once as in Rust).
//
// Parity pin: tests/test_oracle_golden.py replays the reference's fixtures
// (fixtures/alignment/p02_*.json) and the literal cases of its unit tests.

#include "q3s_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>

namespace {

inline bool is_finite(float v) { return fabsf(v) <= 3.40282347e38f; }

inline uint32_t f2u(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

inline uint64_t d2u(double d) {
  uint64_t u;
  memcpy(&u, &d, 8);
  return u;
}

inline double u2d(uint64_t u) {
  double d;
  memcpy(&d, &u, 8);
  return d;
}

// f32::total_cmp key (sampling.rs:587, :690): flips negative patterns so that
// integer order equals the IEEE total order.
inline int32_t total_key(float f) {
  int32_t i = (int32_t)f2u(f);
  return i ^ (int32_t)(((uint32_t)(i >> 31)) >> 1);
}

// Random123 / cuRAND Philox constants (sampling.rs:12-17).
const uint32_t PHILOX_M0 = 0xD2511F53u;
const uint32_t PHILOX_M1 = 0xCD9E8D57u;
const uint32_t PHILOX_W0 = 0x9E3779B9u;
const uint32_t PHILOX_W1 = 0xBB67AE85u;
const float CURAND_2POW32_INV = 2.3283064365386963e-10f;

}  // namespace

// ---------------------------------------------------------------------------
// exp.  Correctly rounded binary32 exp from binary64 arithmetic:
//   k = round(x / ln2), r = x - k*ln2 (two-constant Cody-Waite split, fused),
//   exp(r) by its Taylor series to degree 13 in Horner form (|r| <= 0.347, so
//   the truncation error is below 2^-57), scaled by 2^k and rounded once to
//   binary32.  The kernel evaluates the identical operation sequence.  An
//   exhaustive check over every binary32 input in [-104, 0] against long
//   double expl agrees bit for bit (tests/test_oracle_golden.py samples it).
// ---------------------------------------------------------------------------
extern "C" float q3o_cr_expf(float xf) {
  if (xf != xf) return xf + xf;
  if (xf < -104.0f) return 0.0f;  // exp(-104) < 2^-150: rounds to +0
  if (xf > 89.0f) return INFINITY;  // exp(89) > FLT_MAX
  const double INV_LN2 = 0x1.71547652b82fep+0;  // 1/ln2 rounded to binary64
  const double LN2_HI = 0x1.62e42fefa39efp-1;   // ln2 rounded to binary64
  const double LN2_LO = 0x1.abc9e3b39803fp-56;  // ln2 - LN2_HI rounded
  double x = (double)xf;
  double kd = nearbyint(x * INV_LN2);
  double r = fma(-kd, LN2_HI, x);
  r = fma(-kd, LN2_LO, r);
  // Taylor coefficients 1/n!, each the binary64 nearest to the exact value.
  double p = 0x1.6124613a86d09p-33;        // 1/13!
  p = fma(p, r, 0x1.1eed8eff8d898p-29);    // 1/12!
  p = fma(p, r, 0x1.ae64567f544e4p-26);    // 1/11!
  p = fma(p, r, 0x1.27e4fb7789f5cp-22);    // 1/10!
  p = fma(p, r, 0x1.71de3a556c734p-19);    // 1/9!
  p = fma(p, r, 0x1.a01a01a01a01ap-16);    // 1/8!
  p = fma(p, r, 0x1.a01a01a01a01ap-13);    // 1/7!
  p = fma(p, r, 0x1.6c16c16c16c17p-10);    // 1/6!
  p = fma(p, r, 0x1.1111111111111p-7);     // 1/5!
  p = fma(p, r, 0x1.5555555555555p-5);     // 1/4!
  p = fma(p, r, 0x1.5555555555555p-3);     // 1/3!
  p = fma(p, r, 0.5);                      // 1/2!
  p = fma(p, r, 1.0);
  p = fma(p, r, 1.0);
  int64_t k = (int64_t)kd;  // in [-151, 129]
  double scale = u2d((uint64_t)(k + 1023) << 52);
  return (float)(p * scale);
}

extern "C" float q3o_expf(float x, int exp_mode) {
  return exp_mode == Q3O_EXP_LIBM ? expf(x) : q3o_cr_expf(x);
}

// ---------------------------------------------------------------------------
// Philox4x32-10: mulhilo32 (sampling.rs:337-341), philox_round (:343-348),
// philox4x32_10 (:350-361), next_uniform (:363-375).
// ---------------------------------------------------------------------------
extern "C" void q3o_philox4x32_10(const uint32_t ctr[4], uint32_t seed_lo, uint32_t seed_hi,
                                  uint32_t out[4]) {
  uint32_t s0 = ctr[0], s1 = ctr[1], s2 = ctr[2], s3 = ctr[3];
  uint32_t k0 = seed_lo, k1 = seed_hi;
  for (int round = 0; round < 10; ++round) {
    if (round > 0) {
      k0 += PHILOX_W0;
      k1 += PHILOX_W1;
    }
    uint64_t p0 = (uint64_t)PHILOX_M0 * s0;
    uint64_t p1 = (uint64_t)PHILOX_M1 * s2;
    uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    uint32_t n0 = hi1 ^ s1 ^ k0;
    uint32_t n2 = hi0 ^ s3 ^ k1;
    s0 = n0;
    s1 = lo1;
    s2 = n2;
    s3 = lo0;
  }
  out[0] = s0;
  out[1] = s1;
  out[2] = s2;
  out[3] = s3;
}

extern "C" float q3o_next_uniform(uint64_t seed, uint64_t subsequence, uint32_t ctr_lo) {
  uint32_t ctr[4] = {ctr_lo, 0u, (uint32_t)(subsequence & 0xFFFFFFFFu),
                     (uint32_t)(subsequence >> 32)};
  uint32_t w[4];
  q3o_philox4x32_10(ctr, (uint32_t)(seed & 0xFFFFFFFFu), (uint32_t)(seed >> 32), w);
  return ((float)w[0] + 0.5f) * CURAND_2POW32_INV;
}

// ---------------------------------------------------------------------------
// apply_repetition_penalty (sampling.rs:732-773): every distinct id < n in the
// history, once: x < 0 ? x * p : x / p, with p = penalty as f32.
// ---------------------------------------------------------------------------
extern "C" void q3o_apply_repetition_penalty(float* logits, size_t n, const uint16_t* history,
                                             size_t hist_len, double penalty) {
  if (penalty == 1.0 || hist_len == 0) return;
  std::vector<uint8_t> seen(n, 0);
  const float p = (float)penalty;
  for (size_t h = 0; h < hist_len; ++h) {
    size_t idx = history[h];
    if (idx >= n) continue;
    if (seen[idx]) continue;
    seen[idx] = 1;
    float score = logits[idx];
    logits[idx] = score < 0.0f ? score * p : score / p;
  }
}

namespace {

inline bool index_allowed(size_t idx, int64_t suppress_from, int64_t allow_token) {
  // suppress_from.map(|start| idx < start || Some(idx) == allow).unwrap_or(true)
  if (suppress_from < 0) return true;
  return (int64_t)idx < suppress_from || (allow_token >= 0 && (int64_t)idx == allow_token);
}

struct Cand {
  uint32_t idx;
  float v;
};

}  // namespace

// ---------------------------------------------------------------------------
// sample_logits_with_scratch (sampling.rs:561-730), statement by statement.
// ---------------------------------------------------------------------------
extern "C" int q3o_sample_logits(const float* logits, size_t n, q3o_options opt,
                                 int64_t suppress_from, int64_t allow_token,
                                 const uint16_t* history, size_t hist_len, float uniform,
                                 int exp_mode, uint32_t* token, int* drew, q3o_trace* trace) {
  *drew = 0;
  // Greedy branch (:574-591): argmax over raw logits, total_cmp, lowest index.
  if (opt.temperature <= 0.0) {
    int64_t best = -1;
    int32_t best_key = 0;
    for (size_t i = 0; i < n; ++i) {
      float v = logits[i];
      if (!is_finite(v) || !index_allowed(i, suppress_from, allow_token)) continue;
      int32_t key = total_key(v);
      if (best < 0 || key > best_key) {  // ties keep the lower index
        best = (int64_t)i;
        best_key = key;
      }
    }
    if (best < 0) return Q3O_NO_CANDIDATE;
    *token = (uint32_t)best;
    return Q3O_OK;
  }
  // :592-596 copy.
  std::vector<float> pen(logits, logits + n);
  // :598-606 repetition penalty.
  if (opt.repetition_penalty != 1.0) {
    q3o_apply_repetition_penalty(pen.data(), n, history, hist_len, opt.repetition_penalty);
  }
  if (trace && trace->after_penalty) memcpy(trace->after_penalty, pen.data(), n * sizeof(float));
  // :608-616 non-finite and suppression mask.
  for (size_t i = 0; i < n; ++i) {
    float v = pen[i];
    bool suppressed = suppress_from >= 0 && (int64_t)i >= suppress_from &&
                      !(allow_token >= 0 && (int64_t)i == allow_token);
    if (!is_finite(v) || suppressed) pen[i] = -INFINITY;
  }
  // :628-631 temperature as a reciprocal multiply.
  const float inv_temp = 1.0f / (float)opt.temperature;
  for (size_t i = 0; i < n; ++i) pen[i] = pen[i] * inv_temp;
  if (trace && trace->after_temperature)
    memcpy(trace->after_temperature, pen.data(), n * sizeof(float));
  // :633-652 candidates, sorted by (value desc, index asc).
  std::vector<Cand> cand;
  cand.reserve(n);
  for (size_t i = 0; i < n; ++i)
    if (is_finite(pen[i])) cand.push_back(Cand{(uint32_t)i, pen[i]});
  if (trace && trace->masks)
    for (size_t i = 0; i < n; ++i) trace->masks[i] = is_finite(pen[i]) ? 1 : 0;
  if (trace) trace->topk_threshold = -INFINITY;
  if (cand.empty()) {
    return suppress_from >= 0 ? Q3O_SUPPRESSION_NO_CANDIDATE : Q3O_NO_CANDIDATE;
  }
  std::sort(cand.begin(), cand.end(), [](const Cand& a, const Cand& b) {
    if (a.v > b.v) return true;  // cmp_logit_desc (:775-779); +0 and -0 compare equal
    if (a.v < b.v) return false;
    return a.idx < b.idx;
  });
  // :654-663 top-k keeps every value >= the k-th largest.
  if (opt.top_k > 0 && cand.size() > opt.top_k) {
    const float threshold = cand[opt.top_k - 1].v;
    for (size_t i = 0; i < n; ++i)
      if (pen[i] < threshold) pen[i] = -INFINITY;
    if (trace) trace->topk_threshold = threshold;
  }
  if (trace && trace->masks)
    for (size_t i = 0; i < n; ++i)
      if ((trace->masks[i] & 1) && is_finite(pen[i])) trace->masks[i] |= 2;
  // :665-698 top-p over the full-vocabulary softmax.
  if (opt.top_p < 1.0) {
    float max_logit = -INFINITY;
    for (size_t i = 0; i < n; ++i)
      if (is_finite(pen[i])) max_logit = std::max(max_logit, pen[i]);
    float total = 0.0f;
    for (size_t i = 0; i < n; ++i) total = total + q3o_expf(pen[i] - max_logit, exp_mode);
    if (!is_finite(total) || total <= 0.0f) return Q3O_INVALID_DENOMINATOR;
    const float cutoff = max_logit - 16.0f;
    const float inv_total = 1.0f / total;
    std::vector<Cand> probs;
    for (size_t i = 0; i < n; ++i) {
      float v = pen[i];
      if (is_finite(v) && v >= cutoff) {
        probs.push_back(Cand{(uint32_t)i, q3o_expf(v - max_logit, exp_mode) * inv_total});
      } else {
        pen[i] = -INFINITY;
      }
    }
    std::sort(probs.begin(), probs.end(), [](const Cand& a, const Cand& b) {
      int32_t ka = total_key(a.v), kb = total_key(b.v);
      if (ka != kb) return ka > kb;
      return a.idx < b.idx;
    });
    float cumulative = 0.0f;
    const float top_p = (float)opt.top_p;
    double gap = INFINITY;
    for (size_t pos = 0; pos < probs.size(); ++pos) {
      if (pos > 0) gap = std::min(gap, fabs((double)cumulative - (double)top_p));
      if (pos > 0 && cumulative >= top_p) pen[probs[pos].idx] = -INFINITY;
      cumulative = cumulative + probs[pos].v;
    }
    if (trace) trace->topp_gap = gap;
  }
  if (trace && trace->masks)
    for (size_t i = 0; i < n; ++i)
      if ((trace->masks[i] & 2) && is_finite(pen[i])) trace->masks[i] |= 4;
  // :700-729 final softmax over the survivors and the vocabulary-order draw.
  float max_logit = -INFINITY;
  for (size_t i = 0; i < n; ++i)
    if (is_finite(pen[i])) max_logit = std::max(max_logit, pen[i]);
  if (!is_finite(max_logit)) return Q3O_NO_CANDIDATE;
  float sum = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    pen[i] = q3o_expf(pen[i] - max_logit, exp_mode);
    sum = sum + pen[i];
  }
  if (!is_finite(sum) || sum <= 0.0f) return Q3O_INVALID_DENOMINATOR;
  *drew = 1;
  const float threshold = uniform * sum;
  float cumulative = 0.0f;
  size_t chosen = n - 1;
  float before = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    before = cumulative;
    cumulative = cumulative + pen[i];
    if (cumulative >= threshold) {
      chosen = i;
      break;
    }
  }
  *token = (uint32_t)chosen;
  if (trace) {
    trace->draw_threshold = threshold;
    trace->draw_sum = sum;
    double g1 = (double)cumulative - (double)threshold;
    double g0 = (double)threshold - (double)before;
    trace->boundary_gap = std::min(g0, g1) / (double)sum;
    if (trace->final_probs)
      for (size_t i = 0; i < n; ++i) trace->final_probs[i] = (float)((double)pen[i] / (double)sum);
  }
  return Q3O_OK;
}

// ---------------------------------------------------------------------------
// greedy_select (sampling.rs:40-60): first index of the IEEE maximum.
// ---------------------------------------------------------------------------
extern "C" int q3o_greedy_select(const float* logits, size_t n, int64_t suppress_from,
                                 int64_t allow_token, uint32_t* token) {
  int64_t best = -1;
  float score = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    float v = logits[i];
    if (!is_finite(v) || !index_allowed(i, suppress_from, allow_token)) continue;
    if (best < 0 || v > score) {
      best = (int64_t)i;
      score = v;
    }
  }
  if (best < 0) return Q3O_SUPPRESSION_NO_CANDIDATE;
  *token = (uint32_t)best;
  return Q3O_OK;
}

// greedy_select_on_device (sampling.rs:72-117): invalid entries become -inf, a
// f32::MIN sentinel is appended at index n, and the lowest index of the IEEE
// maximum is returned (the documented contract of :70-71).
extern "C" uint32_t q3o_greedy_select_on_device(const float* logits, size_t n,
                                                int64_t suppress_from, int64_t allow_token) {
  float best_v = -3.40282347e38f;  // the sentinel
  size_t best = n;
  bool suppress = suppress_from >= 0 && (uint64_t)suppress_from < n;
  for (size_t i = 0; i < n; ++i) {
    bool allowed = !suppress || (int64_t)i < suppress_from ||
                   (allow_token >= 0 && (uint64_t)allow_token < n && (int64_t)i == allow_token);
    float v = (allowed && is_finite(logits[i])) ? logits[i] : -INFINITY;
    if (v > best_v || (v == best_v && i < best)) {
      best_v = v;
      best = i;
    }
  }
  return (uint32_t)best;
}

// ---------------------------------------------------------------------------
// Sampler (sampling.rs:158-334).
// ---------------------------------------------------------------------------
extern "C" void q3o_sampler_init(q3o_sampler* s, uint64_t seed) {
  memset(s, 0, sizeof(*s));
  s->seed = seed;
}

static inline uint32_t sat_inc(uint32_t v) { return v == 0xFFFFFFFFu ? v : v + 1; }

extern "C" int q3o_sampler_sample_with_mode(q3o_sampler* s, const float* logits, size_t n,
                                            q3o_options opt, int do_sample, int64_t suppress_from,
                                            int64_t allow_token, const uint16_t* history,
                                            size_t hist_len, int exp_mode, uint32_t* token,
                                            q3o_trace* trace) {
  // :257-272 diagnostics.
  s->call_count = sat_inc(s->call_count);
  if (do_sample)
    s->sampled_calls = sat_inc(s->sampled_calls);
  else
    s->greedy_calls = sat_inc(s->greedy_calls);
  if (hist_len > 0) s->history_nonempty_calls = sat_inc(s->history_nonempty_calls);
  if (s->sequence_len < 64) {
    s->sequence[s->sequence_len] = do_sample ? 1 : 0;
    s->history_nonempty_sequence[s->sequence_len] = hist_len > 0 ? 1 : 0;
    s->sequence_len += 1;
  }
  // :281-296 validation.
  if (!isfinite(opt.repetition_penalty) || opt.repetition_penalty <= 0.0)
    return Q3O_INVALID_REPETITION_PENALTY;
  if (do_sample && (!isfinite(opt.temperature) || opt.temperature <= 0.0))
    return Q3O_INVALID_TEMPERATURE;
  if (!isfinite(opt.top_p) || opt.top_p <= 0.0 || opt.top_p > 1.0) return Q3O_INVALID_TOP_P;
  // :298-328: greedy runs with temperature -1 and no penalty.
  q3o_options eff = opt;
  if (!do_sample) {
    eff.temperature = -1.0;
    eff.repetition_penalty = 1.0;
  }
  float u = q3o_next_uniform(s->seed, s->subseq_counter, s->ctr_lo);
  int drew = 0;
  int st = q3o_sample_logits(logits, n, eff, suppress_from, allow_token, history, hist_len, u,
                             exp_mode, token, &drew, trace);
  // :330-332 the counter moves only for a sampled call that drew.
  if (do_sample && drew) s->subseq_counter += 1;
  return st;
}

// ---------------------------------------------------------------------------
// Batched driver in the layout of q3s_batch (one independent call per row).
// ---------------------------------------------------------------------------
namespace {

struct RowsJob {
  const float* logits;
  const int64_t* offsets;
  const int32_t* vocab;
  const q3o_row_params* params;
  int64_t params_stride;
  const uint64_t* seeds;
  const uint64_t* subseqs;
  const uint16_t* hist;
  const int64_t* hoff;
  const float* uniform_override;
  int exp_mode;
  uint32_t* tokens;
  uint8_t* status;
  float* probs;
  uint8_t* masks;
  int64_t probs_stride;
  double* boundary_gap;
  double* topp_gap;
  int64_t begin, end;
};

void run_rows(const RowsJob* j) {
  for (int64_t r = j->begin; r < j->end; ++r) {
    const q3o_row_params* p = &j->params[r * j->params_stride];
    const float* row = j->logits + j->offsets[r];
    size_t n = (size_t)j->vocab[r];
    const uint16_t* h = j->hoff ? j->hist + j->hoff[r] : nullptr;
    size_t hl = j->hoff ? (size_t)(j->hoff[r + 1] - j->hoff[r]) : 0;
    q3o_trace tr;
    memset(&tr, 0, sizeof(tr));
    tr.final_probs = j->probs ? j->probs + r * j->probs_stride : nullptr;
    tr.masks = j->masks ? j->masks + r * j->probs_stride : nullptr;
    if (tr.final_probs) memset(tr.final_probs, 0, n * sizeof(float));
    if (tr.masks) memset(tr.masks, 0, n);
    tr.boundary_gap = INFINITY;
    tr.topp_gap = INFINITY;
    uint32_t tok = 0;
    int st;
    if (!isfinite(p->repetition_penalty) || p->repetition_penalty <= 0.0) {
      st = Q3O_INVALID_REPETITION_PENALTY;
    } else if (p->do_sample && (!isfinite(p->temperature) || p->temperature <= 0.0)) {
      st = Q3O_INVALID_TEMPERATURE;
    } else if (!isfinite(p->top_p) || p->top_p <= 0.0 || p->top_p > 1.0) {
      st = Q3O_INVALID_TOP_P;
    } else {
      q3o_options o;
      o.temperature = p->do_sample ? p->temperature : -1.0;
      o.top_k = p->top_k;
      o.top_p = p->top_p;
      o.repetition_penalty = p->do_sample ? p->repetition_penalty : 1.0;
      float u = j->uniform_override ? j->uniform_override[r]
                                    : q3o_next_uniform(j->seeds[r], j->subseqs[r], p->ctr_lo);
      int drew = 0;
      st = q3o_sample_logits(row, n, o, p->suppress_from, p->allow_token, h, hl, u, j->exp_mode,
                             &tok, &drew, &tr);
    }
    j->tokens[r] = st == Q3O_OK ? tok : 0u;
    j->status[r] = (uint8_t)st;
    if (j->boundary_gap) j->boundary_gap[r] = tr.boundary_gap;
    if (j->topp_gap) j->topp_gap[r] = tr.topp_gap;
  }
}

void* rows_thread(void* arg) {
  run_rows((const RowsJob*)arg);
  return nullptr;
}

}  // namespace

extern "C" int q3o_sample_rows_ex(const float* logits, int64_t num_rows, const int64_t* offsets,
                                  const int32_t* vocab, const q3o_row_params* params,
                                  int64_t params_stride, const uint64_t* seeds,
                                  const uint64_t* subseqs, const uint16_t* hist,
                                  const int64_t* hoff, const float* uniform_override, int exp_mode,
                                  uint32_t* tokens, uint8_t* status, float* probs, uint8_t* masks,
                                  int64_t probs_stride, double* boundary_gap, double* topp_gap,
                                  int nthreads) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > num_rows) nthreads = (int)(num_rows > 0 ? num_rows : 1);
  std::vector<RowsJob> jobs(nthreads);
  std::vector<pthread_t> tids(nthreads);
  for (int t = 0; t < nthreads; ++t) {
    RowsJob& j = jobs[t];
    j.logits = logits;
    j.offsets = offsets;
    j.vocab = vocab;
    j.params = params;
    j.params_stride = params_stride;
    j.seeds = seeds;
    j.subseqs = subseqs;
    j.hist = hist;
    j.hoff = hoff;
    j.uniform_override = uniform_override;
    j.exp_mode = exp_mode;
    j.tokens = tokens;
    j.status = status;
    j.probs = probs;
    j.masks = masks;
    j.probs_stride = probs_stride;
    j.boundary_gap = boundary_gap;
    j.topp_gap = topp_gap;
    j.begin = num_rows * t / nthreads;
    j.end = num_rows * (t + 1) / nthreads;
  }
  if (nthreads == 1) {
    run_rows(&jobs[0]);
    return 0;
  }
  for (int t = 0; t < nthreads; ++t) pthread_create(&tids[t], nullptr, rows_thread, &jobs[t]);
  for (int t = 0; t < nthreads; ++t) pthread_join(tids[t], nullptr);
  return 0;
}

extern "C" int q3o_sample_rows(const float* logits, int64_t num_rows, const int64_t* offsets,
                               const int32_t* vocab, const q3o_row_params* params,
                               int64_t params_stride, const uint64_t* seeds,
                               const uint64_t* subseqs, const uint16_t* hist, const int64_t* hoff,
                               const float* uniform_override, int exp_mode, uint32_t* tokens,
                               uint8_t* status, float* probs, uint8_t* masks,
                               int64_t probs_stride, double* boundary_gap, int nthreads) {
  return q3o_sample_rows_ex(logits, num_rows, offsets, vocab, params, params_stride, seeds,
                            subseqs, hist, hoff, uniform_override, exp_mode, tokens, status,
                            probs, masks, probs_stride, boundary_gap, nullptr, nthreads);
}
