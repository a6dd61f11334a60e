// C ABI of the B200 sampler (include/q3s_sampler.h): contexts, the batched
// launch, the greedy launch and the stateful `Sampler` mirror of
// src/talker/sampling.rs:144-335.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/q3s_sampler.h"
#include "q3s_internal.h"
#include "q3s_kernels.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  std::string m = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  return fail(e == cudaErrorMemoryAllocation ? Q3S_E_OUT_OF_MEMORY : Q3S_E_CUDA, m);
}

// Makes `device` current for the scope and restores the caller's device.
struct DeviceGuard {
  int prev = -1;
  cudaError_t err = cudaSuccess;
  explicit DeviceGuard(int device) {
    err = cudaGetDevice(&prev);
    if (err == cudaSuccess && prev != device) err = cudaSetDevice(device);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

// Host staging of one single-row call: parameters, Philox key/counter and the
// history offsets, copied to the device in one transfer.
struct SingleRow {
  q3s_row_params params;
  unsigned long long seed;
  unsigned long long subseq;
  long long hist_len;
};

int launch_batch(q3s_context* ctx, const q3s_batch* b, const SingleRow* row, void* stream,
                 const q3s_commit* commit = nullptr);
int validate_batch(const q3s_batch* b);
int stream_workspace(q3s_context* ctx, void* stream, size_t need, bool with_counter,
                     unsigned char** scratch, unsigned** counter);

}  // namespace

struct q3s_context {
  int device = 0;
  int sm_count = 0;
  size_t smem_optin = 0;
  std::mutex mu;
  // Single-row staging (stateful sampler calls).  The row's parameters go
  // in the kernel arguments.  d_hist holds the last history uploaded, and
  // h_hist (pinned) a copy of its first hist_dev ids, so a call whose
  // history extends that one uploads only the new ids (the talker's c0
  // history grows by one id per frame).  The token and status byte are
  // written by the kernel straight into h_out (mapped pinned memory; d_out
  // is its device address), so no copy is issued for them.
  uint16_t* h_hist = nullptr;  // pinned
  uint16_t* d_hist = nullptr;
  size_t hist_cap = 0;
  size_t hist_dev = 0;
  unsigned* h_out = nullptr;  // mapped pinned: token, status byte in the next word
  unsigned* d_out = nullptr;
  // General-path workspaces of the sampling kernel, one per stream that has
  // launched through this context (grown on demand), so launches on
  // different streams never share one.
  struct Workspace {
    cudaStream_t stream;
    unsigned char* ptr;
    size_t bytes;
    unsigned* counter;  // q3s_head_sample's completion counter (zeroed once)
  };
  std::mutex ws_mu;
  std::vector<Workspace> ws;
  // Testing hooks (q3s_context_set_test_hooks).
  uint64_t test_wait_ns = 0;
  int test_hold_refill = 0;
  // Diagnostics (q3s_context_set_path_stats).
  unsigned long long* path_stats = nullptr;
};

struct q3s_sampler {
  q3s_context* ctx;
  uint64_t seed;
  uint64_t subseq;
  uint32_t ctr_lo;
  q3s_sampler_diagnostics diag;
};

namespace q3s {

ContextInfo context_info(const q3s_context* ctx) {
  return ContextInfo{ctx->device, ctx->sm_count, ctx->smem_optin};
}

int record_error(int code, const std::string& msg) { return fail(code, msg); }

int record_cuda_error(cudaError_t e, const char* what) { return cuda_fail(e, what); }

}  // namespace q3s

extern "C" {

int q3s_abi_version(void) { return Q3S_ABI_VERSION; }

const char* q3s_last_error(void) { return g_last_error.c_str(); }

const char* q3s_status_message(int status) {
  switch (status) {
    case Q3S_STATUS_OK:
      return "ok";
    case Q3S_STATUS_INVALID_REPETITION_PENALTY:
      return "invalid repetition_penalty: expected finite value > 0.0";
    case Q3S_STATUS_INVALID_TEMPERATURE:
      return "invalid temperature: expected finite value > 0.0 when sampling is enabled";
    case Q3S_STATUS_INVALID_TOP_P:
      return "invalid top_p: expected finite value in (0.0, 1.0]";
    case Q3S_STATUS_SUPPRESSION_NO_CANDIDATE:
      return "suppression left no finite candidate";
    case Q3S_STATUS_NO_CANDIDATE:
      return "no finite sampling candidate";
    case Q3S_STATUS_INVALID_DENOMINATOR:
      return "invalid softmax denominator";
    case Q3S_STATUS_UNSUPPORTED:
      return "vocabulary larger than the sampler supports";
    case Q3S_STATUS_INVALID_CODE:
      return "embedding code outside its codebook";
    case Q3S_STATUS_HISTORY_FULL:
      return "c0 history capacity exhausted";
    default:
      return "row not processed";
  }
}

int q3s_context_create(int device, q3s_context** out) {
  if (!out) return fail(Q3S_E_INVALID_ARGUMENT, "q3s_context_create: out is NULL");
  *out = nullptr;
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0) return fail(Q3S_E_NO_DEVICE, "no CUDA device available");
  if (device < 0 || device >= count)
    return fail(Q3S_E_INVALID_ARGUMENT, "q3s_context_create: device index out of range");
  DeviceGuard g(device);
  if (g.err != cudaSuccess) return cuda_fail(g.err, "cudaSetDevice");
  q3s_context* c = new q3s_context();
  c->device = device;
  int v = 0;
  if ((e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess) {
    delete c;
    return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
  }
  c->sm_count = v;
  if ((e = cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, device)) !=
      cudaSuccess) {
    delete c;
    return cuda_fail(e, "cudaDeviceGetAttribute(shared memory)");
  }
  c->smem_optin = (size_t)v;
  *out = c;
  return Q3S_OK;
}

void q3s_context_destroy(q3s_context* c) {
  if (!c) return;
  {
    DeviceGuard g(c->device);
    if (c->h_hist) cudaFreeHost(c->h_hist);
    if (c->d_hist) cudaFree(c->d_hist);
    if (c->h_out) cudaFreeHost(c->h_out);
    for (auto& w : c->ws) {
      if (w.ptr) cudaFree(w.ptr);
      if (w.counter) cudaFree(w.counter);
    }
  }
  delete c;
}

int q3s_sample_batch(q3s_context* ctx, const q3s_batch* b, void* stream) {
  if (!ctx || !b) return fail(Q3S_E_INVALID_ARGUMENT, "q3s_sample_batch: NULL context or batch");
  if (b->num_rows < 0) return fail(Q3S_E_INVALID_ARGUMENT, "num_rows must be >= 0");
  if (b->num_rows == 0) return Q3S_OK;
  const int rc = validate_batch(b);
  if (rc != Q3S_OK) return rc;
  return launch_batch(ctx, b, nullptr, stream);
}

int q3s_sample_commit(q3s_context* ctx, const q3s_batch* b, const q3s_commit* c, void* stream) {
  if (!ctx || !b || !c)
    return fail(Q3S_E_INVALID_ARGUMENT, "q3s_sample_commit: NULL context, batch or commit");
  if (b->num_rows < 0) return fail(Q3S_E_INVALID_ARGUMENT, "num_rows must be >= 0");
  if (b->num_rows == 0) return Q3S_OK;
  int rc = validate_batch(b);
  if (rc != Q3S_OK) return rc;
  if (b->probs || b->masks)
    return fail(Q3S_E_INVALID_ARGUMENT, "q3s_sample_commit: no debug outputs (probs, masks)");
  if (c->codes && (c->group < 0 || c->codes_stride <= c->group))
    return fail(Q3S_E_INVALID_ARGUMENT, "q3s_sample_commit: group outside codes_stride");
  if (c->history && (!c->history_ends || !c->history_limits))
    return fail(Q3S_E_INVALID_ARGUMENT,
                "q3s_sample_commit: history needs history_ends and history_limits");
  return launch_batch(ctx, b, nullptr, stream, c);
}

}  // extern "C"

namespace {

int validate_batch(const q3s_batch* b) {
  if (b->dtype != Q3S_DTYPE_F32 && b->dtype != Q3S_DTYPE_BF16)
    return fail(Q3S_E_INVALID_ARGUMENT, "dtype must be Q3S_DTYPE_F32 or Q3S_DTYPE_BF16");
  if (b->vocab < 0) return fail(Q3S_E_INVALID_ARGUMENT, "vocab must be >= 0");
  if (!b->logits || !b->params || !b->tokens || !b->status)
    return fail(Q3S_E_INVALID_ARGUMENT, "logits, params, tokens and status are required");
  if (!b->uniform_override && (!b->seeds || !b->subseqs))
    return fail(Q3S_E_INVALID_ARGUMENT, "seeds and subseqs are required");
  if (b->params_stride != 0 && b->params_stride != 1)
    return fail(Q3S_E_INVALID_ARGUMENT, "params_stride must be 0 or 1");
  if (!b->row_offsets && b->row_stride < 0)
    return fail(Q3S_E_INVALID_ARGUMENT, "row_stride must be >= 0");
  if (b->history_offsets && !b->history)
    return fail(Q3S_E_INVALID_ARGUMENT, "history_offsets without history");
  if ((b->probs || b->masks) && b->probs_stride < b->vocab)
    return fail(Q3S_E_INVALID_ARGUMENT, "probs_stride must be >= vocab");
  return Q3S_OK;
}

// The stream's own workspace of at least `need` bytes (grown on demand) and,
// with `with_counter`, its zeroed completion counter: launches on one stream
// are ordered, so they may share them; another stream gets others.
int stream_workspace(q3s_context* ctx, void* stream, size_t need, bool with_counter,
                     unsigned char** scratch, unsigned** counter) {
  std::lock_guard<std::mutex> lock(ctx->ws_mu);
  const cudaStream_t key = (cudaStream_t)stream;
  q3s_context::Workspace* w = nullptr;
  for (auto& x : ctx->ws)
    if (x.stream == key) w = &x;
  if (!w) {
    ctx->ws.push_back(q3s_context::Workspace{key, nullptr, 0, nullptr});
    w = &ctx->ws.back();
  }
  cudaError_t e;
  if (need > w->bytes) {
    // cudaFree waits for the device, so no launch still uses the old one.
    if (w->ptr) cudaFree(w->ptr);
    w->ptr = nullptr;
    w->bytes = 0;
    if ((e = cudaMalloc((void**)&w->ptr, need)) != cudaSuccess)
      return cuda_fail(e, "cudaMalloc(sampler workspace)");
    w->bytes = need;
  }
  if (with_counter && !w->counter) {
    if ((e = cudaMalloc((void**)&w->counter, 256)) != cudaSuccess)
      return cuda_fail(e, "cudaMalloc(completion counter)");
    if ((e = cudaMemsetAsync(w->counter, 0, 256, key)) != cudaSuccess)
      return cuda_fail(e, "cudaMemsetAsync(completion counter)");
  }
  *scratch = w->ptr;
  if (counter) *counter = w->counter;
  return Q3S_OK;
}

// The launch of a validated batch.  `row` (single-row calls of the stateful
// sampler): the row's parameters, Philox key and counter and history length
// travel in the kernel arguments instead of b->params / seeds / subseqs /
// history_offsets.
int launch_batch(q3s_context* ctx, const q3s_batch* b, const SingleRow* row, void* stream,
                 const q3s_commit* commit) {
  DeviceGuard g(ctx->device);
  if (g.err != cudaSuccess) return cuda_fail(g.err, "cudaSetDevice");
  q3s::KernelArgs a;
  a.logits = b->logits;
  a.dtype = b->dtype;
  a.vocab = b->vocab;
  a.num_rows = b->num_rows;
  a.row_stride = b->row_stride;
  a.row_offsets = reinterpret_cast<const long long*>(b->row_offsets);
  a.row_vocab = b->row_vocab;
  a.params = b->params;
  a.params_stride = b->params_stride;
  a.seeds = reinterpret_cast<const unsigned long long*>(b->seeds);
  a.subseqs = reinterpret_cast<const unsigned long long*>(b->subseqs);
  a.history = b->history;
  a.history_offsets = reinterpret_cast<const long long*>(b->history_offsets);
  a.history_ends = b->history_offsets ? reinterpret_cast<const long long*>(b->history_ends)
                                      : nullptr;
  a.tokens = b->tokens;
  a.status = b->status;
  a.uniform_override = b->uniform_override;
  a.probs = b->probs;
  a.masks = b->masks;
  a.probs_stride = b->probs_stride;
  if (ctx->test_wait_ns) a.wait_ns = ctx->test_wait_ns;
  a.hold_refill = ctx->test_hold_refill;
  a.path_stats = ctx->path_stats;
  if (commit) {
    a.commit = 1;
    a.c_codes = commit->codes;
    a.c_codes_stride = commit->codes_stride;
    a.c_group = commit->group;
    a.c_frame_status = commit->frame_status;
    a.c_subseqs = reinterpret_cast<unsigned long long*>(commit->subseqs);
    a.c_history = commit->history;
    a.c_history_ends = reinterpret_cast<long long*>(commit->history_ends);
    a.c_history_limits = reinterpret_cast<const long long*>(commit->history_limits);
  }
  if (row) {
    a.inline_row = 1;
    a.row_params = row->params;
    a.row_seed = row->seed;
    a.row_subseq = row->subseq;
    a.row_hist_len = row->hist_len;
  }
  int cap = b->vocab < Q3S_MAX_VOCAB ? b->vocab : Q3S_MAX_VOCAB;
  a.vcap = ((cap > 0 ? cap : 1) + 31) / 32 * 32;
  int warps = q3s::sample_max_warps(a.vcap, b->dtype, ctx->smem_optin);
  if (warps < 1) return fail(Q3S_E_INVALID_ARGUMENT, "vocabulary does not fit shared memory");
  // A batch that does not fill every SM with full blocks spreads its rows
  // over all SMs with fewer warps per block: rows run in parallel rather
  // than queueing on a few SMs.
  if (b->num_rows < (long long)warps * ctx->sm_count)
    warps = (int)((b->num_rows + ctx->sm_count - 1) / ctx->sm_count);
  long long blocks = (b->num_rows + warps - 1) / warps;
  if (blocks > ctx->sm_count) blocks = ctx->sm_count;
  const size_t need = (size_t)blocks * warps * q3s::sample_scratch_per_warp(a.vcap);
  int rc = stream_workspace(ctx, stream, need, false, &a.scratch, nullptr);
  if (rc != Q3S_OK) return rc;
  cudaError_t e = q3s::launch_sample(a, (int)blocks, warps, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "sample kernel launch");
  return Q3S_OK;
}

}  // namespace

extern "C" {

int q3s_context_set_test_hooks(q3s_context* ctx, uint64_t stage_wait_ns, int32_t hold_refill) {
  if (!ctx) return fail(Q3S_E_INVALID_ARGUMENT, "q3s_context_set_test_hooks: NULL context");
  ctx->test_wait_ns = stage_wait_ns;
  ctx->test_hold_refill = hold_refill ? 1 : 0;
  return Q3S_OK;
}

int q3s_head_sample(q3s_context* ctx, const q3s_head_batch* hb, void* stream) {
  if (!ctx || !hb) return fail(Q3S_E_INVALID_ARGUMENT, "q3s_head_sample: NULL context or batch");
  const q3s_batch* b = &hb->sample;
  if (b->num_rows < 0 || b->num_rows > Q3S_HEAD_MAX_ROWS)
    return fail(Q3S_E_INVALID_ARGUMENT,
                "q3s_head_sample: num_rows must be in [0, " + std::to_string(Q3S_HEAD_MAX_ROWS) + "]");
  if (b->num_rows == 0) return Q3S_OK;
  if (b->vocab < 1 || b->vocab > Q3S_MAX_VOCAB)
    return fail(Q3S_E_INVALID_ARGUMENT, "q3s_head_sample: vocab must be in [1, 4096]");
  if (!hb->hidden || !hb->weight || !hb->logits || !b->params || !b->tokens || !b->status)
    return fail(Q3S_E_INVALID_ARGUMENT,
                "q3s_head_sample: hidden, weight, logits, params, tokens and status are required");
  if (hb->hidden_dtype != Q3S_DTYPE_F32 && hb->hidden_dtype != Q3S_DTYPE_BF16)
    return fail(Q3S_E_INVALID_ARGUMENT, "hidden_dtype must be Q3S_DTYPE_F32 or Q3S_DTYPE_BF16");
  if (hb->hidden_size < 8 || hb->hidden_size % 8 != 0 || hb->hidden_stride < hb->hidden_size)
    return fail(Q3S_E_INVALID_ARGUMENT,
                "q3s_head_sample: hidden_size must be a positive multiple of 8 and "
                "hidden_stride >= hidden_size");
  if (reinterpret_cast<uintptr_t>(hb->weight) % 16 != 0)
    return fail(Q3S_E_INVALID_ARGUMENT, "q3s_head_sample: weight must be 16-byte aligned");
  if (!b->uniform_override && (!b->seeds || !b->subseqs))
    return fail(Q3S_E_INVALID_ARGUMENT, "seeds and subseqs are required");
  if (b->params_stride != 0 && b->params_stride != 1)
    return fail(Q3S_E_INVALID_ARGUMENT, "params_stride must be 0 or 1");
  if (b->history_offsets && !b->history)
    return fail(Q3S_E_INVALID_ARGUMENT, "history_offsets without history");
  if (b->probs || b->masks)
    return fail(Q3S_E_INVALID_ARGUMENT, "q3s_head_sample: no debug outputs (probs, masks)");
  const int vcap = (b->vocab + 31) / 32 * 32;
  if ((size_t)b->num_rows * hb->hidden_size * 4 > q3s::head_smem(vcap))
    return fail(Q3S_E_INVALID_ARGUMENT, "q3s_head_sample: hidden rows do not fit shared memory");
  if (q3s::head_smem(vcap) > ctx->smem_optin)
    return fail(Q3S_E_INVALID_ARGUMENT, "vocabulary does not fit shared memory");
  DeviceGuard g(ctx->device);
  if (g.err != cudaSuccess) return cuda_fail(g.err, "cudaSetDevice");
  q3s::KernelArgs a;
  a.logits = hb->logits;
  a.dtype = Q3S_DTYPE_F32;
  a.vocab = b->vocab;
  a.num_rows = b->num_rows;
  a.row_stride = b->vocab;
  a.row_offsets = nullptr;
  a.row_vocab = nullptr;
  a.params = b->params;
  a.params_stride = b->params_stride;
  a.seeds = reinterpret_cast<const unsigned long long*>(b->seeds);
  a.subseqs = reinterpret_cast<const unsigned long long*>(b->subseqs);
  a.history = b->history;
  a.history_offsets = reinterpret_cast<const long long*>(b->history_offsets);
  a.history_ends = b->history_offsets ? reinterpret_cast<const long long*>(b->history_ends)
                                      : nullptr;
  a.tokens = b->tokens;
  a.status = b->status;
  a.uniform_override = b->uniform_override;
  a.probs = nullptr;
  a.masks = nullptr;
  a.probs_stride = 0;
  if (ctx->test_wait_ns) a.wait_ns = ctx->test_wait_ns;
  a.vcap = vcap;
  q3s::HeadArgs h;
  h.hidden = hb->hidden;
  h.hidden_dtype = hb->hidden_dtype;
  h.hidden_size = hb->hidden_size;
  h.hidden_stride = hb->hidden_stride;
  h.weight = hb->weight;
  h.vocab = b->vocab;
  h.logits = hb->logits;
  long long grid = (b->vocab + 15) / 16;
  if (grid > ctx->sm_count) grid = ctx->sm_count;
  int rc = stream_workspace(ctx, stream, (size_t)16 * q3s::sample_scratch_per_warp(vcap), true,
                            &a.scratch, &h.counter);
  if (rc != Q3S_OK) return rc;
  const cudaError_t e = q3s::launch_head_sample(h, a, (int)grid, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "head sample kernel launch");
  return Q3S_OK;
}

int q3s_context_set_path_stats(q3s_context* ctx, uint64_t* stats) {
  if (!ctx) return fail(Q3S_E_INVALID_ARGUMENT, "q3s_context_set_path_stats: NULL context");
  ctx->path_stats = reinterpret_cast<unsigned long long*>(stats);
  return Q3S_OK;
}

int q3s_greedy_batch(q3s_context* ctx, const void* logits, int32_t dtype, int64_t num_rows,
                     int64_t row_stride, int32_t vocab, int64_t suppress_from, int64_t allow_token,
                     int32_t mode, uint32_t* tokens, uint8_t* status, void* stream) {
  if (!ctx || !logits || !tokens || !status)
    return fail(Q3S_E_INVALID_ARGUMENT, "q3s_greedy_batch: NULL argument");
  if (num_rows < 0 || vocab < 0 || row_stride < 0)
    return fail(Q3S_E_INVALID_ARGUMENT, "q3s_greedy_batch: negative size");
  if (dtype != Q3S_DTYPE_F32 && dtype != Q3S_DTYPE_BF16)
    return fail(Q3S_E_INVALID_ARGUMENT, "dtype must be Q3S_DTYPE_F32 or Q3S_DTYPE_BF16");
  if (mode != Q3S_GREEDY_SELECT && mode != Q3S_GREEDY_ON_DEVICE)
    return fail(Q3S_E_INVALID_ARGUMENT, "unknown greedy mode");
  if (num_rows == 0) return Q3S_OK;
  DeviceGuard g(ctx->device);
  if (g.err != cudaSuccess) return cuda_fail(g.err, "cudaSetDevice");
  long long blocks = (num_rows + 7) / 8;
  const long long cap = (long long)ctx->sm_count * 8;
  if (blocks > cap) blocks = cap;
  cudaError_t e = q3s::launch_greedy(logits, dtype, num_rows, row_stride, vocab, suppress_from,
                                     allow_token, mode, tokens, status, (int)blocks,
                                     (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "greedy kernel launch");
  return Q3S_OK;
}

// ---------------------------------------------------------------------------
// Stateful sampler.
// ---------------------------------------------------------------------------
int q3s_sampler_create(q3s_context* ctx, uint64_t seed, q3s_sampler** out) {
  if (!ctx || !out) return fail(Q3S_E_INVALID_ARGUMENT, "q3s_sampler_create: NULL argument");
  q3s_sampler* s = new q3s_sampler();
  s->ctx = ctx;
  s->seed = seed;
  s->subseq = 0;
  s->ctr_lo = 0;
  std::memset(&s->diag, 0, sizeof(s->diag));
  *out = s;
  return Q3S_OK;
}

void q3s_sampler_destroy(q3s_sampler* s) { delete s; }

uint64_t q3s_sampler_subsequence_counter(const q3s_sampler* s) { return s ? s->subseq : 0; }

void q3s_sampler_set_subsequence_counter(q3s_sampler* s, uint64_t subseq) {
  if (s) s->subseq = subseq;
}

int q3s_sampler_get_diagnostics(const q3s_sampler* s, q3s_sampler_diagnostics* out) {
  if (!s || !out) return fail(Q3S_E_INVALID_ARGUMENT, "q3s_sampler_get_diagnostics: NULL argument");
  *out = s->diag;
  return Q3S_OK;
}

static uint32_t sat_inc(uint32_t v) { return v == 0xFFFFFFFFu ? v : v + 1; }

static int ensure_single_row(q3s_context* c, int64_t hist_len) {
  cudaError_t e;
  if (!c->h_out) {
    if ((e = cudaHostAlloc((void**)&c->h_out, 16, cudaHostAllocMapped)) != cudaSuccess)
      return cuda_fail(e, "cudaHostAlloc(mapped)");
    if ((e = cudaHostGetDevicePointer((void**)&c->d_out, c->h_out, 0)) != cudaSuccess) {
      cudaFreeHost(c->h_out);
      c->h_out = nullptr;
      return cuda_fail(e, "cudaHostGetDevicePointer");
    }
  }
  if ((size_t)hist_len > c->hist_cap) {
    size_t cap = c->hist_cap ? c->hist_cap : 1024;
    while (cap < (size_t)hist_len) cap *= 2;
    if (c->h_hist) cudaFreeHost(c->h_hist);
    if (c->d_hist) cudaFree(c->d_hist);
    c->h_hist = nullptr;
    c->d_hist = nullptr;
    c->hist_cap = 0;
    c->hist_dev = 0;
    if ((e = cudaMallocHost((void**)&c->h_hist, cap * sizeof(uint16_t))) != cudaSuccess)
      return cuda_fail(e, "cudaMallocHost");
    if ((e = cudaMalloc((void**)&c->d_hist, cap * sizeof(uint16_t))) != cudaSuccess)
      return cuda_fail(e, "cudaMalloc");
    c->hist_cap = cap;
  }
  return Q3S_OK;
}

int q3s_sampler_sample_with_mode(q3s_sampler* s, const void* logits, int32_t dtype, int64_t n,
                                 const q3s_sampling_options* o, int32_t do_sample,
                                 int64_t suppress_from, int64_t allow_token,
                                 const uint16_t* history, int64_t hist_len,
                                 q3s_transfer_callback observer, void* observer_user_data,
                                 uint32_t* token, int32_t* row_status, void* stream) {
  if (!s || !o || !token || (hist_len > 0 && !history) || hist_len < 0 || n < 0)
    return fail(Q3S_E_INVALID_ARGUMENT, "q3s_sampler_sample_with_mode: bad argument");
  if (n > 0 && !logits) return fail(Q3S_E_INVALID_ARGUMENT, "logits is NULL");
  if (dtype != Q3S_DTYPE_F32 && dtype != Q3S_DTYPE_BF16)
    return fail(Q3S_E_INVALID_ARGUMENT, "dtype must be Q3S_DTYPE_F32 or Q3S_DTYPE_BF16");
  if (n > Q3S_MAX_VOCAB) {
    if (row_status) *row_status = Q3S_STATUS_UNSUPPORTED;
    return fail(Q3S_E_SAMPLING, q3s_status_message(Q3S_STATUS_UNSUPPORTED));
  }
  // Diagnostics (sampling.rs:257-272).
  q3s_sampler_diagnostics& d = s->diag;
  d.call_count = sat_inc(d.call_count);
  if (do_sample)
    d.sampled_calls = sat_inc(d.sampled_calls);
  else
    d.greedy_calls = sat_inc(d.greedy_calls);
  if (hist_len > 0) d.history_nonempty_calls = sat_inc(d.history_nonempty_calls);
  if (d.sequence_len < 64) {
    d.sequence[d.sequence_len] = do_sample ? 1 : 0;
    d.history_nonempty_sequence[d.sequence_len] = hist_len > 0 ? 1 : 0;
    d.sequence_len += 1;
  }
  // Validation (sampling.rs:281-296).
  int st = Q3S_STATUS_OK;
  if (!std::isfinite(o->repetition_penalty) || o->repetition_penalty <= 0.0)
    st = Q3S_STATUS_INVALID_REPETITION_PENALTY;
  else if (do_sample && (!std::isfinite(o->temperature) || o->temperature <= 0.0))
    st = Q3S_STATUS_INVALID_TEMPERATURE;
  else if (!std::isfinite(o->top_p) || o->top_p <= 0.0 || o->top_p > 1.0)
    st = Q3S_STATUS_INVALID_TOP_P;
  if (st != Q3S_STATUS_OK) {
    if (row_status) *row_status = st;
    return fail(Q3S_E_SAMPLING, q3s_status_message(st));
  }
  q3s_context* c = s->ctx;
  std::lock_guard<std::mutex> lock(c->mu);
  DeviceGuard g(c->device);
  if (g.err != cudaSuccess) return cuda_fail(g.err, "cudaSetDevice");
  const bool need_hist = do_sample && o->repetition_penalty != 1.0 && hist_len > 0;
  int rc = ensure_single_row(c, need_hist ? hist_len : 0);
  if (rc != Q3S_OK) return rc;
  cudaStream_t st_ = (cudaStream_t)stream;
  SingleRow r;
  std::memset(&r, 0, sizeof(r));
  r.params.temperature = o->temperature;
  r.params.top_p = o->top_p;
  r.params.repetition_penalty = o->repetition_penalty;
  r.params.top_k = o->top_k > 0xFFFFFFFFull ? 0xFFFFFFFFu : (uint32_t)o->top_k;
  r.params.do_sample = do_sample ? 1u : 0u;
  r.params.suppress_from = suppress_from < 0 ? Q3S_NONE
                           : suppress_from > 0x7FFFFFFF ? 0x7FFFFFFF
                                                        : (int32_t)suppress_from;
  r.params.allow_token =
      (allow_token < 0 || allow_token > 0x7FFFFFFF) ? Q3S_NONE : (int32_t)allow_token;
  r.params.ctr_lo = s->ctr_lo;
  r.seed = s->seed;
  r.subseq = s->subseq;
  r.hist_len = need_hist ? hist_len : 0;
  cudaError_t e;
  if (need_hist) {
    // Upload only what the device copy lacks: everything after the ids it
    // already holds, when this history starts with them.
    const size_t len = (size_t)hist_len;
    size_t keep = c->hist_dev <= len &&
                          std::memcmp(c->h_hist, history, c->hist_dev * sizeof(uint16_t)) == 0
                      ? c->hist_dev
                      : 0;
    if (keep < len) {
      std::memcpy(c->h_hist + keep, history + keep, (len - keep) * sizeof(uint16_t));
      if ((e = cudaMemcpyAsync(c->d_hist + keep, c->h_hist + keep,
                               (len - keep) * sizeof(uint16_t), cudaMemcpyHostToDevice, st_)) !=
          cudaSuccess) {
        c->hist_dev = 0;
        return cuda_fail(e, "history upload");
      }
    }
    c->hist_dev = len;
  }
  q3s_batch b;
  std::memset(&b, 0, sizeof(b));
  b.logits = logits ? logits : c->d_out;  // n == 0 reads nothing
  b.dtype = dtype;
  b.vocab = (int32_t)n;
  b.num_rows = 1;
  b.row_stride = 0;
  b.history = need_hist ? c->d_hist : nullptr;
  b.tokens = c->d_out;
  b.status = reinterpret_cast<uint8_t*>(c->d_out + 1);
  rc = launch_batch(c, &b, &r, stream);
  if (rc != Q3S_OK) return rc;
  if ((e = cudaStreamSynchronize(st_)) != cudaSuccess) return cuda_fail(e, "stream synchronize");
  if (observer) observer(observer_user_data, 0, Q3S_TRANSFER_SAMPLED_TOKEN, 1);
  const volatile unsigned* out = c->h_out;
  const int rs = (int)(out[1] & 0xFFu);
  if (row_status) *row_status = rs;
  if (rs != Q3S_STATUS_OK) return fail(Q3S_E_SAMPLING, q3s_status_message(rs));
  *token = out[0];
  // The counter moves only for a sampled call that drew (sampling.rs:330-332).
  if (do_sample) s->subseq += 1;
  return Q3S_OK;
}

int q3s_sampler_sample(q3s_sampler* s, const void* logits, int32_t dtype, int64_t n,
                       const q3s_sampling_options* o, int64_t suppress_from, int64_t allow_token,
                       const uint16_t* history, int64_t hist_len, uint32_t* token,
                       int32_t* row_status, void* stream) {
  if (!o) return fail(Q3S_E_INVALID_ARGUMENT, "options is NULL");
  return q3s_sampler_sample_with_mode(s, logits, dtype, n, o, o->temperature > 0.0 ? 1 : 0,
                                      suppress_from, allow_token, history, hist_len, nullptr,
                                      nullptr, token, row_status, stream);
}

}  // extern "C"
