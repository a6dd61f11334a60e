// Continuous batching of synthesis sessions over the sampler: the
// scheduler the reference plans in tasks/P12-c-abi-and-continuous-batching.md
// (P12-T03 per-session scheduler state, P12-T04 bounded multi-lane
// talker / code-predictor batching) behind the SessionScheduler contract of
// templates/rust-contracts/session.rs (add, tick, cancel), reduced to what
// the sampler owns.  Every session keeps what its own Sampler and talker
// loop keep in the reference (sampling.rs:144-179, talker.rs:500-566): a
// Philox seed and subsequence counter, its talker and code-predictor
// options, the talker suppression and its c0 history.  One frame samples
// every active session's talker row and then its 15 code-predictor groups,
// one launch per step over all sessions, so a session's ids are the ones it
// would get alone (its rows use only its own state).
//
// Device layout: M slots, sessions compacted into slots [0, n) at every
// frame boundary (a leaving session's slot takes the last session's state:
// swap-remove, so the moves never chain).  Per slot: seed, subsequence,
// talker and predictor row parameters, a history range of `history_capacity`
// ids at slot * capacity, its end, and the frame's codes row and status.
// Each step is one launch that samples and commits (q3s_sample_commit); the
// talker step's commit appends the c0 ids, so the history never leaves the
// device.
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/q3s_sampler.h"
#include "q3s_internal.h"

namespace q3s {
namespace sched {

// A new session's state as staged for install_kernel.
struct SlotInit {
  uint64_t seed;
  uint64_t subseq;
  q3s_row_params talker;
  q3s_row_params predictor;
  int64_t hist_off;  // offset of its initial history in the staged ids
  int64_t hist_len;
  int slot;
  int pad;
};

struct SlotMove {
  int src, dst;
};

struct SlotArrays {
  uint64_t* seeds;
  uint64_t* subseqs;
  q3s_row_params* talker;
  q3s_row_params* predictor;
  uint16_t* hist;
  int64_t* hend;
  int64_t hcap;
};

// One block per new session: its scalars, then its history ids.
__global__ void install_kernel(SlotArrays s, const SlotInit* init, const uint16_t* ids) {
  const SlotInit in = init[blockIdx.x];
  const long long base = (long long)in.slot * s.hcap;
  for (long long i = threadIdx.x; i < in.hist_len; i += blockDim.x)
    s.hist[base + i] = ids[in.hist_off + i];
  if (threadIdx.x == 0) {
    s.seeds[in.slot] = in.seed;
    s.subseqs[in.slot] = in.subseq;
    s.talker[in.slot] = in.talker;
    s.predictor[in.slot] = in.predictor;
    s.hend[in.slot] = base + in.hist_len;
  }
}

// One block per move: slot src's state into slot dst (src > dst, and no
// slot is both a source and a destination of one launch).
__global__ void move_kernel(SlotArrays s, const SlotMove* moves) {
  const SlotMove m = moves[blockIdx.x];
  const long long sb = (long long)m.src * s.hcap, db = (long long)m.dst * s.hcap;
  const long long len = s.hend[m.src] - sb;
  for (long long i = threadIdx.x; i < len; i += blockDim.x) s.hist[db + i] = s.hist[sb + i];
  __syncthreads();
  if (threadIdx.x == 0) {
    s.seeds[m.dst] = s.seeds[m.src];
    s.subseqs[m.dst] = s.subseqs[m.src];
    s.talker[m.dst] = s.talker[m.src];
    s.predictor[m.dst] = s.predictor[m.src];
    s.hend[m.dst] = db + len;
  }
}

struct PendingAdd {
  q3s_session_config cfg;
  std::vector<uint16_t> history;
};

q3s_row_params row_params(const q3s_sampling_options& o, int do_sample, int32_t sf,
                          int32_t allow) {
  q3s_row_params p;
  std::memset(&p, 0, sizeof(p));
  p.temperature = o.temperature;
  p.top_p = o.top_p;
  p.repetition_penalty = o.repetition_penalty;
  p.top_k = o.top_k > 0xFFFFFFFFull ? 0xFFFFFFFFu : (uint32_t)o.top_k;
  p.do_sample = do_sample ? 1u : 0u;
  p.suppress_from = sf;
  p.allow_token = allow;
  return p;
}

}  // namespace sched
}  // namespace q3s

struct q3s_scheduler {
  q3s_context* ctx = nullptr;
  int device = 0;
  int M = 0;   // slots
  int G = 0;   // code groups per frame (1 talker + G-1 predictor)
  long long hcap = 0;
  // Device state.
  q3s::sched::SlotArrays s{};
  int64_t* hstart = nullptr;  // slot * hcap
  int64_t* hlim = nullptr;    // (slot + 1) * hcap
  uint32_t* codes = nullptr;    // [M, G]
  uint8_t* fstat = nullptr;     // [M]
  uint32_t* tokens = nullptr;   // [M]
  uint8_t* status = nullptr;    // [M]
  q3s::sched::SlotInit* d_init = nullptr;
  q3s::sched::SlotMove* d_moves = nullptr;
  uint16_t* d_ids = nullptr;    // staged initial histories, M * hcap
  // Host state.
  std::vector<uint64_t> ids;    // session of each active slot, [n]
  std::vector<uint8_t> failed;  // slot stopped in the last frame
  std::vector<q3s::sched::PendingAdd> adds;
  std::vector<uint64_t> cancels;
  q3s::sched::SlotInit* h_init = nullptr;  // pinned
  q3s::sched::SlotMove* h_moves = nullptr; // pinned
  uint16_t* h_ids = nullptr;        // pinned, M * hcap
  uint32_t* h_codes = nullptr;      // pinned, [M, G]
  uint8_t* h_status = nullptr;      // pinned, [M]
  bool in_frame = false;
  int next_group = 0;
  int frame_rows = 0;
};

namespace {

int sched_fail(int code, const std::string& msg) { return q3s::record_error(code, msg); }

struct OnDevice {
  int prev = -1;
  cudaError_t err = cudaSuccess;
  explicit OnDevice(int d) {
    err = cudaGetDevice(&prev);
    if (err == cudaSuccess && prev != d) err = cudaSetDevice(d);
  }
  ~OnDevice() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

void release(q3s_scheduler* q) {
  void* dev[] = {q->s.seeds, q->s.subseqs, q->s.talker, q->s.predictor, q->s.hist, q->s.hend,
                 q->hstart, q->hlim, q->codes, q->fstat, q->tokens, q->status, q->d_init,
                 q->d_moves, q->d_ids};
  for (void* p : dev)
    if (p) cudaFree(p);
  void* host[] = {q->h_init, q->h_moves, q->h_ids, q->h_codes, q->h_status};
  for (void* p : host)
    if (p) cudaFreeHost(p);
}

bool live(const q3s_scheduler* q, uint64_t id) {
  for (uint64_t x : q->ids)
    if (x == id) return true;
  for (const auto& a : q->adds)
    if (a.cfg.id == id) return true;
  return false;
}

}  // namespace

extern "C" {

int q3s_scheduler_create(q3s_context* ctx, int32_t max_sessions, int32_t groups,
                         int64_t history_capacity, q3s_scheduler** out) {
  if (!ctx || !out) return sched_fail(Q3S_E_INVALID_ARGUMENT, "q3s_scheduler_create: NULL argument");
  *out = nullptr;
  if (max_sessions < 1 || groups < 1 || groups > Q3S_MAX_CODE_GROUPS || history_capacity < 1)
    return sched_fail(Q3S_E_INVALID_ARGUMENT,
                      "q3s_scheduler_create: need max_sessions >= 1, 1 <= groups <= 32, "
                      "history_capacity >= 1");
  const q3s::ContextInfo ci = q3s::context_info(ctx);
  OnDevice g(ci.device);
  if (g.err != cudaSuccess) return q3s::record_cuda_error(g.err, "cudaSetDevice");
  q3s_scheduler* q = new q3s_scheduler();
  q->ctx = ctx;
  q->device = ci.device;
  q->M = max_sessions;
  q->G = groups;
  q->hcap = history_capacity;
  q->s.hcap = history_capacity;
  const size_t M = (size_t)max_sessions, H = (size_t)history_capacity;
  cudaError_t e = cudaSuccess;
  auto dm = [&](void** p, size_t bytes) {
    if (e == cudaSuccess) e = cudaMalloc(p, bytes);
  };
  auto hm = [&](void** p, size_t bytes) {
    if (e == cudaSuccess) e = cudaMallocHost(p, bytes);
  };
  dm((void**)&q->s.seeds, M * 8);
  dm((void**)&q->s.subseqs, M * 8);
  dm((void**)&q->s.talker, M * sizeof(q3s_row_params));
  dm((void**)&q->s.predictor, M * sizeof(q3s_row_params));
  dm((void**)&q->s.hist, M * H * 2);
  dm((void**)&q->s.hend, M * 8);
  dm((void**)&q->hstart, M * 8);
  dm((void**)&q->hlim, M * 8);
  dm((void**)&q->codes, M * groups * 4);
  dm((void**)&q->fstat, M);
  dm((void**)&q->tokens, M * 4);
  dm((void**)&q->status, M);
  dm((void**)&q->d_init, M * sizeof(q3s::sched::SlotInit));
  dm((void**)&q->d_moves, M * sizeof(q3s::sched::SlotMove));
  dm((void**)&q->d_ids, M * H * 2);
  hm((void**)&q->h_init, M * sizeof(q3s::sched::SlotInit));
  hm((void**)&q->h_moves, M * sizeof(q3s::sched::SlotMove));
  hm((void**)&q->h_ids, M * H * 2);
  hm((void**)&q->h_codes, M * groups * 4);
  hm((void**)&q->h_status, M);
  if (e == cudaSuccess) {
    std::vector<int64_t> a(M), b(M);
    for (size_t i = 0; i < M; ++i) {
      a[i] = (int64_t)(i * H);
      b[i] = (int64_t)((i + 1) * H);
    }
    e = cudaMemcpy(q->hstart, a.data(), M * 8, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(q->hlim, b.data(), M * 8, cudaMemcpyHostToDevice);
  }
  if (e != cudaSuccess) {
    release(q);
    delete q;
    return q3s::record_cuda_error(e, "q3s_scheduler_create");
  }
  *out = q;
  return Q3S_OK;
}

void q3s_scheduler_destroy(q3s_scheduler* q) {
  if (!q) return;
  {
    OnDevice g(q->device);
    release(q);
  }
  delete q;
}

int q3s_scheduler_add(q3s_scheduler* q, const q3s_session_config* c) {
  if (!q || !c) return sched_fail(Q3S_E_INVALID_ARGUMENT, "q3s_scheduler_add: NULL argument");
  if (c->history_len < 0 || (c->history_len > 0 && !c->history))
    return sched_fail(Q3S_E_INVALID_ARGUMENT, "q3s_scheduler_add: bad history");
  if (c->history_len > q->hcap)
    return sched_fail(Q3S_E_INVALID_ARGUMENT,
                      "q3s_scheduler_add: history longer than the scheduler's capacity of " +
                          std::to_string(q->hcap) + " ids");
  if (live(q, c->id))
    return sched_fail(Q3S_E_INVALID_ARGUMENT,
                      "q3s_scheduler_add: session " + std::to_string(c->id) + " already added");
  // Sessions leaving at the next frame boundary: cancelled or failed (a slot
  // that is both counts once).
  long long leaving = 0;
  for (size_t i = 0; i < q->ids.size(); ++i) {
    bool out = i < q->failed.size() && q->failed[i];
    for (uint64_t id : q->cancels)
      if (q->ids[i] == id) out = true;
    leaving += out ? 1 : 0;
  }
  if ((long long)q->ids.size() - leaving + (long long)q->adds.size() + 1 > q->M)
    return sched_fail(Q3S_E_INVALID_ARGUMENT,
                      "q3s_scheduler_add: all " + std::to_string(q->M) + " sessions are in use");
  q3s::sched::PendingAdd a;
  a.cfg = *c;
  a.history.assign(c->history, c->history + c->history_len);
  a.cfg.history = nullptr;
  q->adds.push_back(std::move(a));
  return Q3S_OK;
}

int q3s_scheduler_cancel(q3s_scheduler* q, uint64_t id) {
  if (!q) return sched_fail(Q3S_E_INVALID_ARGUMENT, "q3s_scheduler_cancel: NULL scheduler");
  for (size_t i = 0; i < q->adds.size(); ++i)
    if (q->adds[i].cfg.id == id) {
      q->adds.erase(q->adds.begin() + (long)i);
      return Q3S_OK;
    }
  for (uint64_t x : q->ids)
    if (x == id) {
      for (uint64_t y : q->cancels)
        if (y == id) return Q3S_OK;
      q->cancels.push_back(id);
      return Q3S_OK;
    }
  return sched_fail(Q3S_E_INVALID_ARGUMENT,
                    "q3s_scheduler_cancel: no session " + std::to_string(id));
}

int q3s_scheduler_begin_frame(q3s_scheduler* q, uint64_t* ids, int32_t cap, int32_t* n_out,
                              void* stream) {
  if (!q || !n_out) return sched_fail(Q3S_E_INVALID_ARGUMENT, "q3s_scheduler_begin_frame: NULL argument");
  if (q->in_frame)
    return sched_fail(Q3S_E_INVALID_ARGUMENT,
                      "q3s_scheduler_begin_frame: the previous frame has not ended");
  OnDevice g(q->device);
  if (g.err != cudaSuccess) return q3s::record_cuda_error(g.err, "cudaSetDevice");
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e;
  // Leaving sessions: cancelled, or stopped by a failed call last frame.
  const int n0 = (int)q->ids.size();
  std::vector<uint8_t> leave(n0, 0);
  for (int i = 0; i < n0; ++i) {
    if (i < (int)q->failed.size() && q->failed[i]) leave[i] = 1;
    for (uint64_t id : q->cancels)
      if (q->ids[i] == id) leave[i] = 1;
  }
  q->cancels.clear();
  q->failed.clear();
  // Swap-remove: the last staying session fills the first free slot.
  int last = n0 - 1, nm = 0;
  auto drop = [&]() {
    while (last >= 0 && leave[last]) --last;
  };
  drop();
  for (int i = 0; i < last; ++i) {
    if (!leave[i]) continue;
    q->h_moves[nm++] = q3s::sched::SlotMove{last, i};
    q->ids[i] = q->ids[last];
    leave[i] = 0;
    leave[last] = 1;
    --last;
    drop();
  }
  q->ids.resize((size_t)(last + 1));
  if (nm > 0) {
    if ((e = cudaMemcpyAsync(q->d_moves, q->h_moves, nm * sizeof(q3s::sched::SlotMove),
                             cudaMemcpyHostToDevice, st)) != cudaSuccess)
      return q3s::record_cuda_error(e, "scheduler move upload");
    q3s::sched::move_kernel<<<nm, 256, 0, st>>>(q->s, q->d_moves);
    if ((e = cudaGetLastError()) != cudaSuccess) return q3s::record_cuda_error(e, "move kernel");
  }
  // Joining sessions take the slots after the staying ones (add() keeps
  // their number within the slots; checked again before any slot is written).
  const int na = (int)q->adds.size();
  if ((long long)q->ids.size() + na > q->M)
    return sched_fail(Q3S_E_INVALID_ARGUMENT, "q3s_scheduler_begin_frame: more sessions than slots");
  if (na > 0) {
    long long off = 0;
    for (int k = 0; k < na; ++k) {
      const q3s_session_config& c = q->adds[k].cfg;
      const int slot = (int)q->ids.size();
      q3s::sched::SlotInit& in = q->h_init[k];
      std::memset(&in, 0, sizeof(in));
      in.seed = c.seed;
      in.subseq = c.subseq;
      in.talker = q3s::sched::row_params(c.talker, c.talker_do_sample, c.suppress_from, c.allow_token);
      in.predictor = q3s::sched::row_params(c.predictor, c.predictor_do_sample, Q3S_NONE, Q3S_NONE);
      in.hist_off = off;
      in.hist_len = (long long)q->adds[k].history.size();
      in.slot = slot;
      if (in.hist_len)
        std::memcpy(q->h_ids + off, q->adds[k].history.data(), (size_t)in.hist_len * 2);
      off += in.hist_len;
      q->ids.push_back(c.id);
    }
    if ((e = cudaMemcpyAsync(q->d_init, q->h_init, na * sizeof(q3s::sched::SlotInit),
                             cudaMemcpyHostToDevice, st)) != cudaSuccess ||
        (off > 0 && (e = cudaMemcpyAsync(q->d_ids, q->h_ids, (size_t)off * 2,
                                          cudaMemcpyHostToDevice, st)) != cudaSuccess))
      return q3s::record_cuda_error(e, "scheduler install upload");
    q3s::sched::install_kernel<<<na, 256, 0, st>>>(q->s, q->d_init, q->d_ids);
    if ((e = cudaGetLastError()) != cudaSuccess) return q3s::record_cuda_error(e, "install kernel");
    // The staging buffers are reused by the next frame boundary, after
    // end_frame has synchronised this stream.
    q->adds.clear();
  }
  const int n = (int)q->ids.size();
  if (n > 0 && (e = cudaMemsetAsync(q->fstat, 0, (size_t)n, st)) != cudaSuccess)
    return q3s::record_cuda_error(e, "scheduler frame status reset");
  for (int i = 0; i < n && i < cap; ++i)
    if (ids) ids[i] = q->ids[i];
  *n_out = n;
  q->frame_rows = n;
  q->next_group = 0;
  q->in_frame = true;
  return Q3S_OK;
}

int q3s_scheduler_step(q3s_scheduler* q, int32_t group, const void* logits, int32_t dtype,
                       int32_t vocab, int64_t row_stride, void* stream) {
  if (!q) return sched_fail(Q3S_E_INVALID_ARGUMENT, "q3s_scheduler_step: NULL scheduler");
  if (!q->in_frame) return sched_fail(Q3S_E_INVALID_ARGUMENT, "q3s_scheduler_step: no frame begun");
  if (group != q->next_group)
    return sched_fail(Q3S_E_INVALID_ARGUMENT,
                      "q3s_scheduler_step: expected group " + std::to_string(q->next_group));
  const int n = q->frame_rows;
  q->next_group = group + 1;
  if (n == 0) return Q3S_OK;
  q3s_batch b;
  std::memset(&b, 0, sizeof(b));
  b.logits = logits;
  b.dtype = dtype;
  b.vocab = vocab;
  b.num_rows = n;
  b.row_stride = row_stride;
  b.params = group == 0 ? q->s.talker : q->s.predictor;
  b.params_stride = 1;
  b.seeds = q->s.seeds;
  b.subseqs = q->s.subseqs;
  if (group == 0) {
    b.history = q->s.hist;
    b.history_offsets = q->hstart;
    b.history_ends = q->s.hend;
  }
  b.tokens = q->tokens;
  b.status = q->status;
  q3s_commit c;
  std::memset(&c, 0, sizeof(c));
  c.num_rows = n;
  c.params = b.params;
  c.params_stride = 1;
  c.tokens = q->tokens;
  c.status = q->status;
  c.subseqs = q->s.subseqs;
  c.codes = q->codes;
  c.codes_stride = q->G;
  c.group = group;
  c.frame_status = q->fstat;
  if (group == 0) {
    c.history = q->s.hist;
    c.history_ends = q->s.hend;
    c.history_limits = q->hlim;
  }
  return q3s_sample_commit(q->ctx, &b, &c, stream);
}

int q3s_scheduler_end_frame(q3s_scheduler* q, uint32_t* codes, uint8_t* status, void* stream) {
  if (!q) return sched_fail(Q3S_E_INVALID_ARGUMENT, "q3s_scheduler_end_frame: NULL scheduler");
  if (!q->in_frame) return sched_fail(Q3S_E_INVALID_ARGUMENT, "q3s_scheduler_end_frame: no frame begun");
  if (q->next_group != q->G)
    return sched_fail(Q3S_E_INVALID_ARGUMENT,
                      "q3s_scheduler_end_frame: " + std::to_string(q->G - q->next_group) +
                          " groups not stepped");
  OnDevice g(q->device);
  if (g.err != cudaSuccess) return q3s::record_cuda_error(g.err, "cudaSetDevice");
  const int n = q->frame_rows;
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = cudaSuccess;
  if (n > 0) {
    if ((e = cudaMemcpyAsync(q->h_codes, q->codes, (size_t)n * q->G * 4, cudaMemcpyDeviceToHost,
                             st)) != cudaSuccess ||
        (e = cudaMemcpyAsync(q->h_status, q->fstat, (size_t)n, cudaMemcpyDeviceToHost, st)) !=
            cudaSuccess)
      return q3s::record_cuda_error(e, "scheduler frame download");
  }
  if ((e = cudaStreamSynchronize(st)) != cudaSuccess)
    return q3s::record_cuda_error(e, "scheduler frame synchronize");
  q->failed.assign((size_t)n, 0);
  for (int i = 0; i < n; ++i) q->failed[i] = q->h_status[i] != Q3S_STATUS_OK ? 1 : 0;
  if (codes && n > 0) std::memcpy(codes, q->h_codes, (size_t)n * q->G * 4);
  if (status && n > 0) std::memcpy(status, q->h_status, (size_t)n);
  q->in_frame = false;
  return Q3S_OK;
}

const uint32_t* q3s_scheduler_codes(const q3s_scheduler* q) { return q ? q->codes : nullptr; }

int q3s_scheduler_session_state(q3s_scheduler* q, uint64_t id, uint64_t* subseq,
                                int64_t* history_len, uint16_t* history, int64_t cap) {
  if (!q) return sched_fail(Q3S_E_INVALID_ARGUMENT, "q3s_scheduler_session_state: NULL scheduler");
  int slot = -1;
  for (size_t i = 0; i < q->ids.size(); ++i)
    if (q->ids[i] == id) slot = (int)i;
  if (slot < 0)
    return sched_fail(Q3S_E_INVALID_ARGUMENT,
                      "q3s_scheduler_session_state: no active session " + std::to_string(id));
  OnDevice g(q->device);
  if (g.err != cudaSuccess) return q3s::record_cuda_error(g.err, "cudaSetDevice");
  uint64_t sub = 0;
  int64_t end = 0;
  cudaError_t e;
  if ((e = cudaMemcpy(&sub, q->s.subseqs + slot, 8, cudaMemcpyDeviceToHost)) != cudaSuccess ||
      (e = cudaMemcpy(&end, q->s.hend + slot, 8, cudaMemcpyDeviceToHost)) != cudaSuccess)
    return q3s::record_cuda_error(e, "q3s_scheduler_session_state");
  const long long len = end - (long long)slot * q->hcap;
  if (subseq) *subseq = sub;
  if (history_len) *history_len = len;
  if (history && cap > 0) {
    const long long k = len < cap ? len : cap;
    if (k > 0 && (e = cudaMemcpy(history, q->s.hist + (long long)slot * q->hcap, (size_t)k * 2,
                                 cudaMemcpyDeviceToHost)) != cudaSuccess)
      return q3s::record_cuda_error(e, "q3s_scheduler_session_state history");
  }
  return Q3S_OK;
}

}  // extern "C"
