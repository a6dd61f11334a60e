// Fused per-step sampling kernel for the Qwen3-TTS talker / code predictor.
//
// Per row: repetition penalty over the row's history (sampling.rs:592-606,
// 732-773), suppression / non-finite mask (:608-616), temperature as a
// reciprocal multiply (:628-631), top-k keeping every tie of the k-th value
// (:633-663), top-p over the full-vocabulary softmax (:665-698) and the
// vocabulary-order multinomial draw with Philox4x32-10 (:700-729, :337-375).
// Greedy rows take the total_cmp argmax of the raw logits (:574-591).
//
// Exactness: every f32 operation of the reference is performed with the same
// rounding, and every f32 running sum the reference accumulates sequentially
// (the top-p denominator, the nucleus cumulative, the final softmax sum and
// the draw's cumulative) is accumulated sequentially here too, over the same
// non-zero terms in the same order.  Terms the reference adds that are exact
// zeros (exp(-inf)) are skipped, which leaves an f32 sum unchanged.  The
// order-free parts (maxima, counts, selection, sorting) are parallel.
//
// Data movement and work split.  A persistent grid of warps strides over the
// rows.  Each warp owns one shared-memory stage; its next row arrives by a
// bulk copy (TMA, cp.async.bulk, no multicast) completing on the warp's
// mbarrier while the warp works on the current row.  Common rows take the
// fast path:
//   1. the warp scans the stage once, keeping each 16-byte vector's maximum
//      in registers, and reduces the row maximum;
//   2. it picks a threshold tau on the vector maxima such that at least k
//      vectors (hence at least k elements) reach it, so the candidates
//      {x >= tau} contain the whole top-k set, ties included;
//   3. it re-reads only the vectors whose maximum reaches tau and gathers
//      their candidates (a few dozen to a few hundred per row) into a short
//      list, then releases the stage to the next row's copy;
//   4. the list is finished warp-cooperatively with register bitonic sorts
//      of 32-bit keys (32, 128 or 512 of them): one sort gives the exact
//      k-th largest, a second puts the survivors in vocabulary order, top-p
//      sorts by (p desc, index asc) and back; each sequential f32 chain runs
//      on one lane over a shared-memory array in that order.
// Rows outside the fast path (top_k off or above 256, a temperature whose
// reciprocal is 0 or infinite, too many candidates, +inf logits) run the
// same algorithm warp-cooperatively on full-row lists kept in a per-warp
// global workspace ("general path").

#include <atomic>
#include <cstdint>

#include "../../include/q3s_sampler.h"
#include "q3s_device.cuh"
#include "q3s_kernels.h"

namespace q3s {
namespace {

constexpr int MAX_WARPS = 16;
constexpr int RING = 8;  // row stages per block, shared by its warps
constexpr int ROW_CAP = 512;      // candidates one fast row may hold
constexpr int FAST_MAX_K = 256;
constexpr uint64_t WAIT_LIMIT_NS = 1000000000ull;  // bounded wait for a stage: 1 s

template <int DT>
struct Elem;
template <>
struct Elem<Q3S_DTYPE_F32> {
  static constexpr int BYTES = 4, EPV = 4;
};
template <>
struct Elem<Q3S_DTYPE_BF16> {
  static constexpr int BYTES = 2, EPV = 8;
};

__host__ __device__ inline size_t align16(size_t b) { return (b + 15) & ~size_t(15); }

// 16-byte vectors per lane chunk of the fast-path scan for a row capacity:
// ceil(vcap * es / 512) rounded up to a multiple of 8.
__host__ __device__ constexpr int chunk_vectors(int vcap, int es) {
  return (((vcap * es + 511) / 512) + 7) & ~7;
}

// The stage holds a row with up to 15 bytes of leading misalignment, and at
// least the 32 lane chunks the fast-path scan reads.
__host__ __device__ inline size_t stage_bytes(int vcap, int es) {
  const size_t row = align16((size_t)vcap * es + 16);
  const size_t chunks = (size_t)512 * chunk_vectors(vcap, es);
  return row > chunks ? row : chunks;
}

// Per-warp shared memory (6.8 KB for a 3072-entry row; with the 8 shared
// row stages, 16 warps fit an SM).  Kb is one 2 KB area whose users never
// overlap in time: the flagged-vector list of the collection, the
// k-th-value gather and softmax terms of the top-k finisher, the sort keys
// (aliasing the softmax terms) of the top-p finisher, and the general
// path's sort keys.
constexpr int KB_BYTES = 2048 + 32;  // 512 softmax terms + zero padding to a multiple of 8
// [0]: top-k threshold t; [16, 80): k-th-value bucket counts; [80, 144) and
// [144, 208): the largest and smallest order key per bucket.
constexpr int HIST_WORDS = 208;

struct FastSpace {
  unsigned char* stage;     // the current row's ring stage (TMA destination)
  uint2* list;              // [ROW_CAP] candidates (x bits, index); general-path histogram
  unsigned long long* Kb;   // KB_BYTES, see above
  uint32_t* bm;             // [vcap/32] history bitmap
  uint32_t* hist;           // [HIST_WORDS]
};

// Shared memory of a block: the ring control block, RING stages, then one
// area per warp.  Rows go to warps by ticket (in order); ticket t uses stage
// t % RING, generation t / RING.  A stage's generation g+1 is issued by the
// warp of generation g once it has read the stage, and `issued` lets a warp
// wait for its own generation before testing the barrier's phase parity
// (parity alone cannot tell generation g+1 from g-1).
struct RingCtl {
  uint64_t full[RING];      // stage barriers (one arrival + the copy's bytes)
  uint32_t issued[RING];    // generations issued per stage
  uint32_t consumed[RING];  // generations waited for per stage
  uint32_t ticket;          // next ticket
  uint32_t abort;           // set when a wait gave up: no more copies, rows NOT_RUN
};
constexpr size_t CTL_BYTES = 256;
static_assert(sizeof(RingCtl) <= CTL_BYTES, "ring control block");
// The plan ring (PLAN_SLOTS x 32 bytes) follows the control block.
constexpr size_t HEAD_BYTES = CTL_BYTES + 96 * 32;

__host__ __device__ inline size_t warp_bytes(int vcap) {
  return 8u * ROW_CAP + KB_BYTES + 4u * HIST_WORDS + align16(4u * (vcap / 32));
}

__host__ __device__ inline size_t block_smem(int vcap, int es, int warps) {
  return HEAD_BYTES + RING * stage_bytes(vcap, es) + (size_t)warps * warp_bytes(vcap);
}

__device__ inline FastSpace carve_warp(unsigned char* base, int vcap) {
  FastSpace f;
  size_t o = 0;
  f.stage = nullptr;
  f.list = reinterpret_cast<uint2*>(base + o);
  o += 8u * ROW_CAP;
  f.Kb = reinterpret_cast<unsigned long long*>(base + o);
  o += KB_BYTES;
  f.hist = reinterpret_cast<uint32_t*>(base + o);
  o += 4u * HIST_WORDS;
  f.bm = reinterpret_cast<uint32_t*>(base + o);
  return f;
}

// Per-warp global workspace of the general path.
struct GenSpace {
  float* A;      // [vcap] the row, then x
  float* B;      // [vcap] list values
  float* BX;     // [vcap] list x
  uint16_t* BI;  // [vcap] list indices
};

__host__ __device__ inline size_t gen_bytes(int vcap) {
  return align16(4u * vcap) * 3 + align16(2u * vcap);
}

__device__ inline GenSpace carve_gen(unsigned char* base, int vcap) {
  GenSpace g;
  g.A = reinterpret_cast<float*>(base);
  g.B = reinterpret_cast<float*>(base + align16(4u * vcap));
  g.BX = reinterpret_cast<float*>(base + 2 * align16(4u * vcap));
  g.BI = reinterpret_cast<uint16_t*>(base + 3 * align16(4u * vcap));
  return g;
}

struct RowOut {
  int status;
  uint32_t token;
};

// Where a row's elements sit in the stage: element i at byte (mis + i) * es.
struct StageView {
  int n;    // elements
  int mis;  // leading misalignment in elements
  int Q;    // 16-byte vectors covering the row
  const void* p0;     // the row in global memory (element 0)
  const uint4* g16;   // global 16-byte vector q of the stage layout is g16[q]
};

// Row geometry shared by the copy issuer and the consumer.
struct RowGeom {
  const unsigned char* p0;  // first byte of the row
  uint32_t bytes;           // row bytes
  uint32_t mis_bytes;       // p0 & 15
  uint32_t head_end;        // bytes [0, head_end) of the row come from plain loads
  uint32_t tail_begin;      // bytes [tail_begin, bytes) too
};

__device__ __forceinline__ RowGeom row_geom(const KernelArgs& a, long long row, int n, int es) {
  RowGeom g;
  const long long off = a.row_offsets ? a.row_offsets[row] : row * a.row_stride;
  g.p0 = static_cast<const unsigned char*>(a.logits) + off * es;
  g.bytes = (uint32_t)n * es;
  const uintptr_t s = reinterpret_cast<uintptr_t>(g.p0);
  g.mis_bytes = (uint32_t)(s & 15u);
  const uintptr_t a0 = (s + 15u) & ~(uintptr_t)15u;
  const uintptr_t a1 = (s + g.bytes) & ~(uintptr_t)15u;
  if (a1 > a0) {
    g.head_end = (uint32_t)(a0 - s);
    g.tail_begin = (uint32_t)(a1 - s);
  } else {
    g.head_end = g.bytes;
    g.tail_begin = g.bytes;
  }
  return g;
}

__device__ __forceinline__ int row_vocab(const KernelArgs& a, long long row) {
  return a.row_vocab ? a.row_vocab[row] : a.vocab;
}

__device__ __forceinline__ bool row_fits(const KernelArgs& a, int n) {
  return n >= 0 && n <= a.vocab && n <= a.vcap;
}

// Lane 0: arms the stage barrier and starts the interior bulk copy of `row`.
// Rows that do not fit the stage arm the barrier with no bytes.
template <int DT>
__device__ void issue_row(const KernelArgs& a, long long row, unsigned char* stage, uint64_t* bar) {
  constexpr int es = Elem<DT>::BYTES;
  const int n = row_vocab(a, row);
  uint32_t bytes = 0;
  RowGeom g;
  if (row_fits(a, n)) {
    g = row_geom(a, row, n, es);
    bytes = g.tail_begin - g.head_end;
  }
  mbar_arrive_expect_tx(bar, bytes);
  if (bytes > 0) bulk_copy_g2s(stage + g.mis_bytes + g.head_end, g.p0 + g.head_end, bytes, bar);
}

// After the barrier completes: the lanes copy the unaligned head and tail.
template <int DT>
__device__ StageView complete_stage(const KernelArgs& a, long long row, int n, unsigned char* stage) {
  constexpr int es = Elem<DT>::BYTES;
  const RowGeom g = row_geom(a, row, n, es);
  const unsigned lane = lane_id();
  const int hn = (int)(g.head_end / es);
  const int t0 = (int)(g.tail_begin / es);
  for (int i = lane; i < hn; i += 32) {
    if (es == 4)
      reinterpret_cast<float*>(stage + g.mis_bytes)[i] = __ldg(reinterpret_cast<const float*>(g.p0) + i);
    else
      reinterpret_cast<unsigned short*>(stage + g.mis_bytes)[i] =
          __ldg(reinterpret_cast<const unsigned short*>(g.p0) + i);
  }
  for (int i = t0 + lane; i < n; i += 32) {
    if (es == 4)
      reinterpret_cast<float*>(stage + g.mis_bytes)[i] = __ldg(reinterpret_cast<const float*>(g.p0) + i);
    else
      reinterpret_cast<unsigned short*>(stage + g.mis_bytes)[i] =
          __ldg(reinterpret_cast<const unsigned short*>(g.p0) + i);
  }
  __syncwarp();
  StageView v;
  v.n = n;
  v.mis = (int)(g.mis_bytes / es);
  v.Q = (int)((g.mis_bytes + g.bytes + 15u) / 16u);
  v.p0 = g.p0;
  v.g16 = reinterpret_cast<const uint4*>(g.p0 - g.mis_bytes);
  return v;
}

template <int DT>
__device__ __forceinline__ void unpack_vec(const uint4& v, float (&e)[Elem<DT>::EPV]) {
  if (DT == Q3S_DTYPE_F32) {
    e[0] = __uint_as_float(v.x);
    e[1] = __uint_as_float(v.y);
    e[2] = __uint_as_float(v.z);
    e[3] = __uint_as_float(v.w);
  } else {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      e[2 * t] = __uint_as_float(w[t] << 16);
      e[2 * t + 1] = __uint_as_float(w[t] & 0xFFFF0000u);
    }
  }
}

template <int DT>
__device__ __forceinline__ void unpack(const unsigned char* stage, int q, float (&e)[Elem<DT>::EPV]) {
  unpack_vec<DT>(*reinterpret_cast<const uint4*>(stage + 16 * q), e);
}

// Option validation of sampling.rs:281-296 (f64 comparisons).
__device__ inline int validate(const q3s_row_params& p) {
  if (!isfinite(p.repetition_penalty) || p.repetition_penalty <= 0.0)
    return Q3S_STATUS_INVALID_REPETITION_PENALTY;
  if (p.do_sample && (!isfinite(p.temperature) || p.temperature <= 0.0))
    return Q3S_STATUS_INVALID_TEMPERATURE;
  if (!isfinite(p.top_p) || p.top_p <= 0.0 || p.top_p > 1.0) return Q3S_STATUS_INVALID_TOP_P;
  return Q3S_STATUS_OK;
}

__device__ __forceinline__ bool idx_allowed(int i, int sf, int allow) {
  return sf < 0 || i < sf || (allow >= 0 && i == allow);
}

// A row's parameters as the kernel uses them (32 bytes), computed ahead for
// 32 rows at a time, one lane per row: the draw, the f32 casts, the
// validation status and the flags.  suppress_from / allow_token are clamped
// to [-1, n], which keeps every comparison with an index below n.
struct RowPlan {
  float u;       // the draw: Philox word 0 of (seed, subseq, ctr_lo), or the override
  float inv;     // 1 / (temperature as f32)
  float pf;      // repetition penalty as f32
  float top_p;   // top_p as f32
  uint32_t k;    // top_k
  uint32_t nf;   // row vocabulary (low 16 bits) | flags (high 16 bits)
  uint32_t sa;   // suppress_from (low 16, signed) | allow_token (high 16, signed)
  uint32_t tag;  // the ticket this plan belongs to
};
static_assert(sizeof(RowPlan) == 32, "plan record");
constexpr uint32_t PF_STATUS = 7u;  // Q3S_STATUS_* of the row (validation, vocabulary)
constexpr uint32_t PF_DO_SAMPLE = 1u << 3;
constexpr uint32_t PF_USE_PEN = 1u << 4;  // sampled, penalty != 1 and a non-empty history
constexpr uint32_t PF_TOP_P = 1u << 5;    // top_p < 1
constexpr uint32_t NO_TAG = 0xFFFFFFFFu;
constexpr int PLAN_SLOTS = 96;  // three batches of 32 tickets

__device__ __forceinline__ uint32_t clamp16(long long v, int n) {
  const int c = v < 0 ? -1 : (v > n ? n : (int)v);
  return (uint32_t)(uint16_t)(int16_t)c;
}

// The history range of `row`: [history_begin, history_end).
__device__ __forceinline__ long long history_begin(const KernelArgs& a, long long row) {
  return a.inline_row ? 0 : a.history_offsets[row];
}

__device__ __forceinline__ long long history_end(const KernelArgs& a, long long row) {
  if (a.inline_row) return a.row_hist_len;
  return a.history_ends ? a.history_ends[row] : a.history_offsets[row + 1];
}

__device__ RowPlan compute_plan(const KernelArgs& a, long long row, uint32_t ticket) {
  const q3s_row_params P = a.inline_row ? a.row_params : a.params[row * a.params_stride];
  int n = row_vocab(a, row);
  const int st = row_fits(a, n) ? validate(P) : Q3S_STATUS_UNSUPPORTED;
  n = n < 0 ? 0 : (n > 65535 ? 65535 : n);
  uint32_t flags = (uint32_t)st;
  if (P.do_sample) flags |= PF_DO_SAMPLE;
  if (P.top_p < 1.0) flags |= PF_TOP_P;
  if (P.do_sample && P.repetition_penalty != 1.0 && (a.inline_row ? a.history != nullptr
                                                                  : a.history_offsets != nullptr) &&
      history_end(a, row) > history_begin(a, row))
    flags |= PF_USE_PEN;
  RowPlan p;
  p.u = a.uniform_override ? a.uniform_override[row]
          : a.inline_row ? philox_uniform(a.row_seed, a.row_subseq, P.ctr_lo)
                         : philox_uniform(a.seeds[row], a.subseqs[row], P.ctr_lo);
  p.inv = __fdiv_rn(1.0f, (float)P.temperature);
  p.pf = (float)P.repetition_penalty;
  p.top_p = (float)P.top_p;
  p.k = P.top_k;
  p.nf = (uint32_t)n | (flags << 16);
  p.sa = clamp16(P.suppress_from, n) | (clamp16(P.allow_token, n) << 16);
  p.tag = ticket;
  return p;
}

// Publishes a plan: the tag is invalidated first and written last, so a
// reader that sees the same matching tag before and after reading the data
// read a consistent record.
__device__ __forceinline__ void store_plan(RowPlan* slot, const RowPlan& p) {
  volatile uint32_t* w = reinterpret_cast<volatile uint32_t*>(slot);
  w[7] = NO_TAG;
  __threadfence_block();
  w[0] = __float_as_uint(p.u);
  w[1] = __float_as_uint(p.inv);
  w[2] = __float_as_uint(p.pf);
  w[3] = __float_as_uint(p.top_p);
  w[4] = p.k;
  w[5] = p.nf;
  w[6] = p.sa;
  __threadfence_block();
  w[7] = p.tag;
}

__device__ __forceinline__ bool load_plan(const RowPlan* slot, uint32_t ticket, RowPlan& p) {
  const volatile uint32_t* w = reinterpret_cast<const volatile uint32_t*>(slot);
  if (w[7] != ticket) return false;
  __threadfence_block();
  p.u = __uint_as_float(w[0]);
  p.inv = __uint_as_float(w[1]);
  p.pf = __uint_as_float(w[2]);
  p.top_p = __uint_as_float(w[3]);
  p.k = w[4];
  p.nf = w[5];
  p.sa = w[6];
  p.tag = ticket;
  __threadfence_block();
  return w[7] == ticket;
}

// The history bitmap of a row (sampling.rs:732-773: every id < n of the
// history marks its entry once): bm[0 .. ceil(n/32)) = one bit per id.  The
// ids are read as 16-byte vectors of 8, four vectors per lane in flight (1024
// ids per round trip of the warp), plus the unaligned head and tail one id
// per lane; vector slots past the end read as 0xFFFF, which no row's
// vocabulary reaches.  Lanes whose ids share a bitmap word would serialise on
// an atomic OR, so histories longer than 64 ids are marked with plain byte
// stores into a byte map `bytes` (32 * ceil(n/32) bytes, 16-byte aligned; an
// id listed twice stores the same 1), which is then packed into bm, four
// bytes of 0/1 at a time by one multiply: bytes b0..b3 of x land on bits
// 24..27 of x * 0x01020408 (each byte lands on distinct bits, so nothing
// carries).
__device__ __forceinline__ void mark_id(uint32_t* bm, uint32_t id, int n) {
  if ((int)id < n) atomicOr(&bm[id >> 5], 1u << (id & 31));
}

__device__ __forceinline__ void mark_byte(unsigned char* bytes, uint32_t id, int n) {
  if ((int)id < n) bytes[id] = 1;
}

__device__ __forceinline__ uint32_t pack_bytes4(uint32_t x) { return (x * 0x01020408u) >> 24; }

template <bool BYTES>
__device__ __forceinline__ void mark_ids(const unsigned short* h, long long cnt, int n,
                                         uint32_t* bm, unsigned char* bytes) {
  const int lane = (int)lane_id();
  auto mark = [&](uint32_t id) {
    if (BYTES)
      mark_byte(bytes, id, n);
    else
      mark_id(bm, id, n);
  };
  long long head = (long long)(((16u - (uint32_t)(reinterpret_cast<uintptr_t>(h) & 15u)) & 15u) >> 1);
  if (head > cnt) head = cnt;
  if (lane < head) mark(__ldg(h + lane));
  const uint4* v = reinterpret_cast<const uint4*>(h + head);
  const long long nv = (cnt - head) >> 3;
  for (long long q0 = 0; q0 < nv; q0 += 128) {
    uint4 w[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const long long q = q0 + r * 32 + lane;
      w[r] = q < nv ? __ldg(v + q) : make_uint4(~0u, ~0u, ~0u, ~0u);
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const uint32_t ws[4] = {w[r].x, w[r].y, w[r].z, w[r].w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        mark(ws[t] & 0xFFFFu);
        mark(ws[t] >> 16);
      }
    }
  }
  for (long long t = head + nv * 8 + lane; t < cnt; t += 32) mark(__ldg(h + t));
}

__device__ __noinline__ void fill_history(const unsigned short* h, long long cnt, int n,
                                          uint32_t* bm, unsigned char* bytes) {
  const int lane = (int)lane_id();
  const int W = (n + 31) >> 5;
  if (cnt <= 64) {
    for (int w = lane; w < W; w += 32) bm[w] = 0u;
    __syncwarp();
    mark_ids<false>(h, cnt, n, bm, bytes);
    __syncwarp();
    return;
  }
  uint4* B4 = reinterpret_cast<uint4*>(bytes);
  for (int q = lane; q < 2 * W; q += 32) B4[q] = make_uint4(0u, 0u, 0u, 0u);
  __syncwarp();
  mark_ids<true>(h, cnt, n, bm, bytes);
  __syncwarp();
  for (int w = lane; w < W; w += 32) {
    const uint4 a = B4[2 * w], b = B4[2 * w + 1];
    bm[w] = pack_bytes4(a.x) | (pack_bytes4(a.y) << 4) | (pack_bytes4(a.z) << 8) |
            (pack_bytes4(a.w) << 12) | (pack_bytes4(b.x) << 16) | (pack_bytes4(b.y) << 20) |
            (pack_bytes4(b.z) << 24) | (pack_bytes4(b.w) << 28);
  }
  __syncwarp();
}

// Per-row transform inputs.
struct RowCtx {
  int n, mis, Q;
  int nj;  // vectors per lane chunk of the fast-path scan (runtime-chunk kernels)
  const uint4* g16;  // the row's 16-byte vectors in global memory (stage layout)
  float inv;      // 1 / (temperature as f32)
  float pf;       // repetition penalty as f32
  bool use_pen;
  int sf, allow;
  const uint32_t* bm;
};

// x of element i from its raw value v.  XF: penalty, mask and temperature of
// sampling.rs:598-631.  Without XF the raw value is returned (rows with no
// penalty and no suppression select on raw values and scale afterwards).
template <bool XF, bool EDGE>
__device__ __forceinline__ float xform(float v, int i, const RowCtx& r) {
  if (EDGE && (unsigned)i >= (unsigned)r.n) return neg_inf();
  if (!XF) return v;
  if (r.use_pen && ((r.bm[i >> 5] >> (i & 31)) & 1u))
    v = v < 0.0f ? __fmul_rn(v, r.pf) : __fdiv_rn(v, r.pf);
  const bool sup = r.sf >= 0 && i >= r.sf && i != r.allow;
  if (!is_finite(v) || sup) v = neg_inf();
  return __fmul_rn(v, r.inv);
}

// Debug outputs of one row (probs and masks), NULL when not requested.
struct DebugRow {
  unsigned char* masks;
  float* probs;
};

// ===========================================================================
// General path (warp-cooperative over full-row lists).
// ===========================================================================

// k-th smallest (1-based) key among the valid elements, MSB-first radix
// selection with 8-bit digits from bit `top_shift + 8` down.  Requires at
// least k valid elements whose keys are below 2^(top_shift + 8).
template <typename K, class KeyFn>
__device__ K warp_select(int n, uint32_t k, KeyFn keyfn, uint32_t* hist, int top_shift) {
  const unsigned lane = lane_id();
  K prefix = 0, mask = 0;
  uint32_t kk = k;
#pragma unroll 1
  for (int shift = top_shift; shift >= 0; shift -= 8) {
    for (int b = lane; b < 256; b += 32) hist[b] = 0u;
    __syncwarp();
    for (int i = lane; i < n; i += 32) {
      K key;
      if (keyfn(i, key) && (key & mask) == prefix)
        atomicAdd(&hist[(uint32_t)(key >> shift) & 255u], 1u);
    }
    __syncwarp();
    uint32_t c[8];
    uint32_t s = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      c[q] = hist[8 * lane + q];
      s += c[q];
    }
    const uint32_t incl = warp_inclusive_scan(s);
    const unsigned ball = __ballot_sync(FULL, incl >= kk);
    const int src = ball ? __ffs(ball) - 1 : 31;
    uint32_t digit = 255, before = 0;
    if ((int)lane == src) {
      uint32_t acc = incl - s;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (acc + c[q] >= kk) {
          digit = 8 * lane + q;
          before = acc;
          break;
        }
        acc += c[q];
      }
    }
    digit = __shfl_sync(FULL, digit, src);
    before = __shfl_sync(FULL, before, src);
    kk -= before;
    prefix |= (K)digit << shift;
    mask |= (K)0xFFu << shift;
    __syncwarp();
  }
  return prefix;
}

template <int R, typename T>
__device__ __forceinline__ void bitonic(T (&v)[R]);

// Ascending bitonic sort of 256 keys held 8 per lane (element lane*8 + r).
__device__ inline void bitonic_sort_256(unsigned long long (&v)[8]) { bitonic<8>(v); }

// Sequential f32 sum of B[0..count) (global workspace, 16-byte aligned) by
// lane 0, in order, staged through the warp's shared area S (STAGE_TERMS
// floats, 16-byte aligned): the warp copies STAGE_TERMS terms at a time into
// S (zero-padded to a multiple of 8), lane 0 adds them eight per step with its
// shared loads one step ahead, and with `prefix` the running sums go back to
// B.  Result broadcast to every lane.  The same additions in the same order
// as a plain loop, without a global-memory round trip per step.
constexpr int STAGE_TERMS = 1024;

__device__ __forceinline__ float4 lds4(uint32_t a);
__device__ __forceinline__ void sts4(uint32_t a, const float4& v);

__device__ float chain_staged(float* B, int count, bool prefix, float* S) {
  const int lane = (int)lane_id();
  float c = 0.0f;
  for (int base = 0; base < count; base += STAGE_TERMS) {
    const int m = min(STAGE_TERMS, count - base);
    const int m8 = (m + 7) & ~7;
    const float4* B4 = reinterpret_cast<const float4*>(B + base);
    float4* S4 = reinterpret_cast<float4*>(S);
    for (int q = lane; q < (m >> 2); q += 32) S4[q] = B4[q];
    for (int j = (m & ~3) + lane; j < m8; j += 32) S[j] = j < m ? B[base + j] : 0.0f;
    __syncwarp();
    if (lane == 0) {
      const uint32_t s0 = smem_u32(S);
      const int n8 = m8 >> 3;
      float4 na = lds4(s0), nb = lds4(s0 + 16u);
      for (int q = 0; q < n8; ++q) {
        float4 va = na, vb = nb;
        const uint32_t a = s0 + 32u * (uint32_t)q;
        if (q + 1 < n8) {
          na = lds4(a + 32u);
          nb = lds4(a + 48u);
        }
        c = __fadd_rn(c, va.x);
        va.x = c;
        c = __fadd_rn(c, va.y);
        va.y = c;
        c = __fadd_rn(c, va.z);
        va.z = c;
        c = __fadd_rn(c, va.w);
        va.w = c;
        c = __fadd_rn(c, vb.x);
        vb.x = c;
        c = __fadd_rn(c, vb.y);
        vb.y = c;
        c = __fadd_rn(c, vb.z);
        vb.z = c;
        c = __fadd_rn(c, vb.w);
        vb.w = c;
        if (prefix) {
          sts4(a, va);
          sts4(a + 16u, vb);
        }
      }
    }
    __syncwarp();
    if (prefix) {
      float4* W4 = reinterpret_cast<float4*>(B + base);
      for (int q = lane; q < (m >> 2); q += 32) W4[q] = S4[q];
      for (int j = (m & ~3) + lane; j < m; j += 32) B[base + j] = S[j];
    }
    __syncwarp();
    c = __shfl_sync(FULL, c, 0);
  }
  return c;
}

__device__ __forceinline__ unsigned long long nucleus_key(float p, uint16_t idx) {
  return ((unsigned long long)(~__float_as_uint(p)) << 32) | idx;
}

__device__ __forceinline__ unsigned long long pack_top_p(int status, int ns, float m2) {
  return ((unsigned long long)(unsigned)status << 56) | ((unsigned long long)(unsigned)ns << 32) |
         __float_as_uint(m2);
}

template <int R, typename T>
__device__ __forceinline__ void bitonic(T (&v)[R]);

// Status of top_p_from_candidates when the candidates cannot decide the
// nucleus (the caller then walks the whole list).
constexpr int TOPP_UNDECIDED = 0x7F;
constexpr int TOPP_CANDS = 256;  // candidates one warp sorts in registers (8 per lane)

// The nucleus from the list's largest entries (sampling.rs:665-698).  The
// reference sorts every entry within 16 of the maximum by (p desc, index
// asc) and keeps the positions before the first position > 0 whose
// preceding cumulative reaches top_p.  Here:
//   * a 64-bucket histogram of x over [m1 - 16, m1] (count and, for sizing
//     only, the mass of exp(x - m1) per bucket; the map is monotone in x)
//     picks the fewest top buckets whose mass reaches top_p with a margin;
//   * their entries (at most TOPP_CANDS) are sorted by (p desc, index asc)
//     with the reference's p = exp(x - m1) * inv_total, and one lane walks
//     the sequential f32 cumulative in that order;
//   * the walk decides the nucleus exactly when it closes inside the
//     candidates and its last member's p is strictly above the largest p of
//     any entry outside them (which is then ordered after it), or when the
//     candidates are every entry within 16 of the maximum.
// Otherwise one more bucket is tried, then TOPP_UNDECIDED is returned.  On
// success the list is compacted to the nucleus as apply_top_p leaves it.
// hist: 128 words; keys: TOPP_CANDS entries.
__device__ unsigned long long top_p_from_candidates(float* B, float* BX, uint16_t* BI, int ns,
                                                    float m1, float total, float top_p,
                                                    unsigned long long* keys, uint32_t* hist) {
  const int lane = (int)lane_id();
  const uint32_t lt = lanemask_lt();
  const float inv_total = __fdiv_rn(1.0f, total);
  const float cutoff = __fsub_rn(m1, 16.0f);
  uint32_t* cnt = hist;
  float* mass = reinterpret_cast<float*>(hist + 64);
  auto bucket = [&](float x) {
    const int b = (int)__fmul_rn(__fsub_rn(m1, x), 4.0f);
    return b > 63 ? 63 : b;
  };
  cnt[lane] = 0u;
  cnt[lane + 32] = 0u;
  mass[lane] = 0.0f;
  mass[lane + 32] = 0.0f;
  __syncwarp();
  for (int j = lane; j < ns; j += 32) {
    const float x = BX[j];
    if (x >= cutoff) {
      const int b = bucket(x);
      atomicAdd(&cnt[b], 1u);
      atomicAdd(&mass[b], B[j]);
    }
  }
  __syncwarp();
  // Lane l holds buckets 2l and 2l + 1; inclusive prefix counts and masses.
  const uint32_t c0 = cnt[2 * lane], c1 = cnt[2 * lane + 1];
  const float w0 = mass[2 * lane], w1 = mass[2 * lane + 1];
  uint32_t cs = c0 + c1;
  float ws = w0 + w1;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t a = __shfl_up_sync(FULL, cs, o);
    const float b = __shfl_up_sync(FULL, ws, o);
    if (lane >= o) {
      cs += a;
      ws += b;
    }
  }
  const uint32_t eligible = __shfl_sync(FULL, cs, 31);
  // Smallest bucket whose cumulative mass reaches top_p * total, with a
  // margin for the sizing sums' rounding.
  const float target = __fmul_rn(__fmul_rn(top_p, total), 1.001f);
  const bool r0 = ws - w1 >= target, r1 = ws >= target;
  const unsigned b0 = __ballot_sync(FULL, r0), b1 = __ballot_sync(FULL, r1);
  int first = 63;
  if (b0 | b1) {
    const int l0 = b0 ? __ffs(b0) - 1 : 32, l1 = b1 ? __ffs(b1) - 1 : 32;
    first = l0 <= l1 ? 2 * l0 : 2 * l1 + 1;
  }
  __syncwarp();
#pragma unroll 1
  for (int bsel = first; bsel <= first + 1 && bsel <= 63; ++bsel) {
    // Candidates: entries within 16 of the maximum in buckets <= bsel.
    const uint32_t ncand = __shfl_sync(FULL, (bsel & 1) ? cs : cs - c1, bsel >> 1);
    if (ncand > (uint32_t)TOPP_CANDS) break;
    const bool complete = ncand == eligible;
    float xout = neg_inf();  // largest x of an entry within 16 outside the candidates
    int cnt_c = 0;
    for (int j0 = 0; j0 < ns; j0 += 32) {
      const int j = j0 + lane;
      bool in = false;
      float x = neg_inf();
      if (j < ns) {
        x = BX[j];
        if (x >= cutoff) {
          if (bucket(x) <= bsel)
            in = true;
          else
            xout = fmaxf(xout, x);
        }
      }
      const unsigned bb = __ballot_sync(FULL, in);
      if (in) {
        const float p = __fmul_rn(B[j], inv_total);
        keys[cnt_c + __popc(bb & lt)] =
            ((unsigned long long)(~__float_as_uint(p)) << 32) |
            ((uint32_t)BI[j] << 16) | (uint32_t)j;
      }
      cnt_c += __popc(bb);
    }
    xout = warp_max(xout);
    __syncwarp();
    unsigned long long v[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int e = lane * 8 + r;
      v[r] = e < cnt_c ? keys[e] : ~0ull;
    }
    __syncwarp();
    bitonic<8>(v);
#pragma unroll
    for (int r = 0; r < 8; ++r) keys[lane * 8 + r] = v[r];
    __syncwarp();
    // The walk (sampling.rs:690-697) over the sorted candidates.
    int J = 0;
    bool closed = false;
    float plast = 0.0f;
    if (lane == 0) {
      float cum = 0.0f;
      for (int q = 0; q < cnt_c; ++q) {
        if (q > 0 && cum >= top_p) {
          closed = true;
          break;
        }
        const float p = __uint_as_float(~(uint32_t)(keys[q] >> 32));
        cum = __fadd_rn(cum, p);
        plast = p;
        J = q + 1;
      }
      if (!closed && J == cnt_c && cum >= top_p) closed = true;  // the next entry is masked
    }
    J = __shfl_sync(FULL, J, 0);
    closed = __shfl_sync(FULL, closed ? 1 : 0, 0) != 0;
    plast = __shfl_sync(FULL, plast, 0);
    bool ok = complete || closed;
    if (ok && !complete && xout > neg_inf()) {
      // Every entry outside the candidates has p <= pout: it sorts after
      // the last nucleus member when that member's p is larger.
      const float pout = __fmul_rn(cr_expf(__fsub_rn(xout, m1)), inv_total);
      ok = plast > pout;
    }
    if (!ok) continue;
    // The nucleus: positions [0, J).  Mark its list positions, take their
    // maximum x, then compact the list in place with exp(x - m2).
    uint32_t* marks = hist;  // 128 words: one bit per list position (ns <= 4096)
    for (int w = lane; w < 128; w += 32) marks[w] = 0u;
    __syncwarp();
    float m2 = neg_inf();
    for (int q = lane; q < J; q += 32) {
      const uint32_t j = (uint32_t)keys[q] & 0xFFFFu;
      atomicOr(&marks[j >> 5], 1u << (j & 31));
      m2 = fmaxf(m2, BX[j]);
    }
    m2 = warp_max(m2);
    __syncwarp();
    if (!(m2 > neg_inf())) return pack_top_p(Q3S_STATUS_NO_CANDIDATE, 0, 0.0f);
    int ns2 = 0;
    for (int j0 = 0; j0 < ns; j0 += 32) {
      const int j = j0 + lane;
      const bool p = j < ns && ((marks[j >> 5] >> (j & 31)) & 1u);
      const int i = p ? BI[j] : 0;
      const float x = p ? BX[j] : 0.0f;
      __syncwarp();
      const unsigned b = __ballot_sync(FULL, p);
      if (p) {
        const int d = ns2 + __popc(b & lt);
        BI[d] = (uint16_t)i;
        BX[d] = x;
        B[d] = cr_expf(__fsub_rn(x, m2));
      }
      ns2 += __popc(b);
      __syncwarp();
    }
    return pack_top_p(Q3S_STATUS_OK, ns2, m2);
  }
  return pack_top_p(TOPP_UNDECIDED, 0, 0.0f);
}

// Top-p over a survivor list in vocabulary order (sampling.rs:665-698) given
// its full-vocabulary softmax denominator `total`: the max - 16 cutoff and
// the nucleus walked in (p desc, index asc) order, 256 at a time.  On return
// the list holds the nucleus (vocabulary order, B = exp(x - m2)).  Returns
// status, nucleus length and m2 packed by pack_top_p.
__device__ unsigned long long apply_top_p(float* B, float* BX, uint16_t* BI, int ns, float m1,
                                          float total, float top_p, unsigned long long* keys,
                                          uint32_t* hist) {
  const unsigned lane = lane_id();
  const float inv_total = __fdiv_rn(1.0f, total);
  const float cutoff = __fsub_rn(m1, 16.0f);
  int np = 0;
  for (int j = lane; j < ns; j += 32) {
    const float p = BX[j] >= cutoff ? __fmul_rn(B[j], inv_total) : 0.0f;
    B[j] = p;
    np += p > 0.0f ? 1 : 0;
  }
  np = __reduce_add_sync(FULL, np);
  __syncwarp();
  // The first position > 0 whose preceding cumulative reaches top_p starts
  // the masked tail.
  float cum = 0.0f;
  int pos = 0;
  unsigned long long cut = ~0ull, last = 0ull;
  int remaining = np;
  auto pkey = [&](int j, unsigned long long& k) {
    const float p = B[j];
    k = nucleus_key(p, BI[j]);
    return p > 0.0f && k > last;
  };
#pragma unroll 1
  while (remaining > 0) {
    const int m = remaining < 256 ? remaining : 256;
    unsigned long long hi = ~0ull;
    if (remaining > 256) hi = warp_select<unsigned long long>(ns, 256u, pkey, hist, 56);
    int cnt = 0;
    for (int j0 = 0; j0 < ns; j0 += 32) {
      const int j = j0 + lane;
      unsigned long long k = 0;
      const bool p = j < ns && pkey(j, k) && k <= hi;
      const unsigned b = __ballot_sync(FULL, p);
      if (p) {
        const int d = cnt + __popc(b & lanemask_lt());
        if (d < 256) keys[d] = k;
      }
      cnt += __popc(b);
    }
    if (cnt > 256) cnt = 256;
    __syncwarp();
    unsigned long long v[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int e = lane * 8 + r;
      v[r] = e < cnt ? keys[e] : ~0ull;
    }
    __syncwarp();
    bitonic_sort_256(v);
#pragma unroll
    for (int r = 0; r < 8; ++r) keys[lane * 8 + r] = v[r];
    __syncwarp();
    if (lane == 0) {
      for (int q = 0; q < cnt; ++q) {
        const unsigned long long k = keys[q];
        const float p = __uint_as_float(~(uint32_t)(k >> 32));
        if (pos > 0 && cum >= top_p) {
          cut = k;
          break;
        }
        cum = __fadd_rn(cum, p);
        ++pos;
      }
    }
    cut = __shfl_sync(FULL, cut, 0);
    cum = __shfl_sync(FULL, cum, 0);
    pos = __shfl_sync(FULL, pos, 0);
    __syncwarp();
    if (cut != ~0ull) break;
    last = hi;
    remaining -= m;
  }
  // Final survivors: nucleus members before the cut.
  float m2 = neg_inf();
  for (int j = lane; j < ns; j += 32) {
    const float p = B[j];
    if (p > 0.0f && nucleus_key(p, BI[j]) >= cut) B[j] = 0.0f;
    if (B[j] > 0.0f) m2 = fmaxf(m2, BX[j]);
  }
  m2 = warp_max(m2);
  __syncwarp();
  if (!(m2 > neg_inf())) return pack_top_p(Q3S_STATUS_NO_CANDIDATE, 0, 0.0f);
  // Compact the survivors in place with the final softmax numerators.
  int ns2 = 0;
  for (int j0 = 0; j0 < ns; j0 += 32) {
    const int j = j0 + lane;
    const bool p = j < ns && B[j] > 0.0f;
    const int i = p ? BI[j] : 0;
    const float x = p ? BX[j] : 0.0f;
    __syncwarp();
    const unsigned b = __ballot_sync(FULL, p);
    if (p) {
      const int d = ns2 + __popc(b & lanemask_lt());
      BI[d] = (uint16_t)i;
      BX[d] = x;
      B[d] = cr_expf(__fsub_rn(x, m2));
    }
    ns2 += __popc(b);
    __syncwarp();
  }
  return pack_top_p(Q3S_STATUS_OK, ns2, m2);
}

// General path: mask, temperature, top-k, top-p and the draw over the full row
// held as f32 in A (global workspace).  Kept out of line with scalar and
// pointer arguments only, so the fast path's state stays in registers.
// hist: 1024 words (radix histograms, chain staging); hist2: 128 words.
__device__ __noinline__ unsigned long long general_compute(
    float* A, float* GB, float* GBX, uint16_t* GBI, const uint32_t* bm, uint32_t* hist,
    uint32_t* hist2, unsigned long long* keys, int n, float inv, float pf, int use_pen, int sf,
    int allow,
    unsigned top_k, int use_top_p, float top_p, float u, unsigned char* masks, float* probs) {
  const unsigned lane = lane_id();
  RowCtx rc;
  rc.n = n;
  rc.mis = 0;
  rc.Q = 0;
  rc.nj = 0;
  rc.g16 = nullptr;
  rc.inv = inv;
  rc.pf = pf;
  rc.use_pen = use_pen != 0;
  rc.sf = sf;
  rc.allow = allow;
  rc.bm = bm;
  RowOut out{Q3S_STATUS_OK, 0u};
  // Mask and temperature (sampling.rs:608-631).
  float mx = neg_inf();
  int nfin = 0;
  bool nan_seen = false;
  for (int i = lane; i < n; i += 32) {
    const float x = xform<true, false>(A[i], i, rc);
    A[i] = x;
    mx = fmaxf(mx, x);
    nfin += is_finite(x) ? 1 : 0;
    nan_seen |= (x != x);
    if (masks && is_finite(x)) masks[i] = 1;
  }
  mx = warp_max(mx);
  nfin = __reduce_add_sync(FULL, nfin);
  nan_seen = __any_sync(FULL, nan_seen);
  __syncwarp();
  if (nfin == 0) {
    out = {sf >= 0 ? Q3S_STATUS_SUPPRESSION_NO_CANDIDATE : Q3S_STATUS_NO_CANDIDATE, 0u};
  } else if (nan_seen || mx == __int_as_float(0x7f800000)) {
    // A NaN or +inf after the temperature survives top-k and top-p and makes
    // the softmax denominator non-finite (sampling.rs:675-678, 715-718).
    out = {Q3S_STATUS_INVALID_DENOMINATOR, 0u};
  } else {
    // Top-k threshold: the k-th largest finite value (sampling.rs:654-663).
    float t = neg_inf();
    if (top_k > 0u && (uint32_t)nfin > top_k) {
      const uint32_t key = warp_select<uint32_t>(
          n, top_k,
          [&](int i, uint32_t& k) {
            const float x = A[i];
            k = ~total_key(x);
            return x > neg_inf();
          },
          hist, 24);
      t = from_total_key(~key);
    }
    // Survivor list in vocabulary order.
    int ns = 0;
    for (int i0 = 0; i0 < n; i0 += 32) {
      const int i = i0 + lane;
      const float x = i < n ? A[i] : neg_inf();
      const bool p = x >= t && x > neg_inf();
      const unsigned b = __ballot_sync(FULL, p);
      if (p) {
        const int j = ns + __popc(b & lanemask_lt());
        GBI[j] = (uint16_t)i;
        GBX[j] = x;
        GB[j] = cr_expf(__fsub_rn(x, mx));
        if (masks) masks[i] |= 2;
      }
      ns += __popc(b);
    }
    __syncwarp();
    float m2 = mx;
    float* S = reinterpret_cast<float*>(hist);  // chain staging (STAGE_TERMS floats)
    if (use_top_p) {
      // Denominator: sequential f32 sum in vocabulary order (sampling.rs:666-679).
      const float total = chain_staged(GB, ns, false, S);
      unsigned long long r;
      if (!is_finite(total) || total <= 0.0f) {
        r = pack_top_p(Q3S_STATUS_INVALID_DENOMINATOR, 0, 0.0f);
      } else {
        r = top_p_from_candidates(GB, GBX, GBI, ns, mx, total, top_p, keys, hist2);
        if ((int)(r >> 56) == TOPP_UNDECIDED)
          r = apply_top_p(GB, GBX, GBI, ns, mx, total, top_p, keys, hist);
      }
      const int st = (int)(r >> 56);
      if (st != Q3S_STATUS_OK) {
        out = {st, 0u};
        ns = -1;
      } else {
        ns = (int)((r >> 32) & 0xFFFFFFu);
        m2 = __uint_as_float((uint32_t)r);
      }
    }
    if (ns >= 0) {
      // Final softmax sum and the draw (sampling.rs:700-729).
      const float sum = chain_staged(GB, ns, true, S);
      if (!is_finite(sum) || sum <= 0.0f) {
        out = {Q3S_STATUS_INVALID_DENOMINATOR, 0u};
      } else {
        const float thr = __fmul_rn(u, sum);
        int first = ns;
        for (int j = lane; j < ns; j += 32) {
          if (GB[j] >= thr) {
            first = j;
            break;
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) first = min(first, __shfl_xor_sync(FULL, first, o));
        out = {Q3S_STATUS_OK, first < ns ? (uint32_t)GBI[first] : (uint32_t)(n - 1)};
        if (masks || probs) {
          for (int j = lane; j < ns; j += 32) {
            const int i = GBI[j];
            if (masks) masks[i] |= 4;
            if (probs) {
              const float e = cr_expf(__fsub_rn(GBX[j], m2));
              probs[i] = __double2float_rn((double)e / (double)sum);
            }
          }
        }
      }
    }
  }
  __syncwarp();
  return ((unsigned long long)(unsigned)out.status << 32) | out.token;
}

// ===========================================================================
// Fast path: warp scan and candidate collection.
// ===========================================================================

// A row's stage is released exactly once, as soon as the row no longer
// reads it: lane 0 issues the stage's next generation (ticket + RING) and
// publishes it in `issued`.
struct Releaser {
  const KernelArgs* a;
  RingCtl* ctl;
  unsigned char* stage;
  int slot;
  long long next;  // row of the stage's next generation
  uint32_t gen;    // that generation
  bool done;
};

template <int DT>
__device__ __forceinline__ void release(Releaser& r) {
  if (r.done) return;
  r.done = true;
  __syncwarp();
  if (lane_id() == 0 && r.next < r.a->num_rows && !r.a->hold_refill &&
      *reinterpret_cast<volatile uint32_t*>(&r.ctl->abort) == 0u) {
    fence_proxy_async_smem();
    issue_row<DT>(*r.a, r.next, r.stage, &r.ctl->full[r.slot]);
    __threadfence_block();
    *reinterpret_cast<volatile uint32_t*>(&r.ctl->issued[r.slot]) = r.gen + 1u;
  }
}

// Waits for generation `gen` of stage `slot`: first until it has been issued
// (a later generation's parity must not be tested against an earlier
// phase), then for its bytes.  False when a wait gave up (after limit_ns) or
// the block aborts.
__device__ bool wait_stage(RingCtl* ctl, int slot, uint32_t gen, uint64_t limit_ns) {
  if (*reinterpret_cast<volatile uint32_t*>(&ctl->abort) != 0u) return false;
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  while (*reinterpret_cast<volatile uint32_t*>(&ctl->issued[slot]) <= gen) {
    if (*reinterpret_cast<volatile uint32_t*>(&ctl->abort) != 0u) return false;
    __nanosleep(128);
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > limit_ns) return false;
  }
  __threadfence_block();
  return mbar_wait_bounded(&ctl->full[slot], gen & 1u, limit_ns);
}

// Vector maxima of the stage (registers) and the row maximum.  Lane l owns
// the contiguous chunk of NJ 16-byte vectors [l*NJ, (l+1)*NJ), so chunks
// follow vocabulary order.  Step j reads chunk vector j ^ (l & 7): the 8
// lanes of each shared-memory phase then hit 8 distinct bank groups (NJ is a
// multiple of 8, so the XOR permutes the chunk), and every address is one of
// 8 per-lane bases plus an immediate offset.  vm[j] is the maximum of that
// vector.  Vectors past the row hold stale bytes; EDGE rows mask them by
// index.  RT (runtime chunk): a row that exactly fills 32 chunks of r.nj
// vectors (r.nj <= NJ, a multiple of 8) scans those without EDGE; its
// vectors j >= r.nj have maximum -inf.
template <int DT, int NJ, bool XF, bool EDGE, bool RT>
__device__ __forceinline__ float scan_stage(const FastSpace& f, const RowCtx& r, float (&vm)[NJ]) {
  constexpr int EPV = Elem<DT>::EPV;
  const int lane = (int)lane_id();
  const int sw = lane & 7;
  const int nj = (RT && !EDGE) ? r.nj : NJ;
  const uint4* chunk = reinterpret_cast<const uint4*>(f.stage) + lane * nj;
  float mx = neg_inf();
  // Groups of 8 vectors; a runtime chunk ends at a group boundary (one
  // uniform test per group after the first).
#pragma unroll
  for (int g = 0; g < NJ / 8; ++g) {
    if (RT && !EDGE && g > 0 && 8 * g >= nj) {
#pragma unroll
      for (int j = 8 * g; j < NJ; ++j) vm[j] = neg_inf();
      break;
    }
#pragma unroll
    for (int j = 8 * g; j < 8 * g + 8; ++j) {
      const int v = (j & ~7) | ((j & 7) ^ sw);
      const uint4 w = chunk[v];
      float e[EPV];
      unpack_vec<DT>(w, e);
      float m = neg_inf();
#pragma unroll
      for (int c = 0; c < EPV; ++c)
        m = fmaxf(m, xform<XF, EDGE>(e[c], (lane * nj + v) * EPV + c - r.mis, r));
      vm[j] = m;
      mx = fmaxf(mx, m);
    }
  }
  return warp_max(mx);
}

// Penalty, suppression and temperature (sampling.rs:592-631) applied in place
// to an f32 row in its stage: the penalty on the history ids, then each lane
// masks and scales its own scan chunk in a rolled loop, so the scan that
// follows is the plain one and its unrolled body stays small.  The values
// written are xform's, so they equal what the collection recomputes from the
// row in global memory.  With EDGE, entries outside
// [0, n) become -inf (the scan masks them by index as well).
// The repetition penalty (sampling.rs:732-773) on the raw f32 row in its
// stage, element i at row[i]: one update per set bit of the history bitmap,
// so each distinct id < n is penalised once; the lanes take the bitmap words
// in turn.
__device__ __forceinline__ void penalize_stage(float* row, int n, const uint32_t* bm, float pf) {
  const int lane = (int)lane_id();
  for (int w = lane; w < ((n + 31) >> 5); w += 32) {
    uint32_t bits = bm[w];
    while (bits) {
      const int i = (w << 5) + __ffs(bits) - 1;
      bits &= bits - 1;
      const float v = row[i];
      row[i] = v < 0.0f ? __fmul_rn(v, pf) : __fdiv_rn(v, pf);
    }
  }
  __syncwarp();
}

template <int NJ, bool EDGE, bool RT>
__device__ __forceinline__ void xform_stage_f32(const FastSpace& f, const RowCtx& rp) {
  // The penalty on the history ids first, then mask and temperature.
  RowCtx r = rp;
  if (r.use_pen) {
    penalize_stage(reinterpret_cast<float*>(f.stage) + r.mis, r.n, r.bm, r.pf);
    r.use_pen = false;
  }
  const int lane = (int)lane_id();
  const int sw = lane & 7;
  const int nj = (RT && !EDGE) ? r.nj : NJ;
  uint4* chunk = reinterpret_cast<uint4*>(f.stage) + lane * nj;
#pragma unroll 1
  for (int j = 0; j < nj; ++j) {
    const int v = (j & ~7) | ((j & 7) ^ sw);
    uint4 w = chunk[v];
    const int i0 = (lane * nj + v) * 4 - r.mis;
    w.x = __float_as_uint(xform<true, EDGE>(__uint_as_float(w.x), i0, r));
    w.y = __float_as_uint(xform<true, EDGE>(__uint_as_float(w.y), i0 + 1, r));
    w.z = __float_as_uint(xform<true, EDGE>(__uint_as_float(w.z), i0 + 2, r));
    w.w = __float_as_uint(xform<true, EDGE>(__uint_as_float(w.w), i0 + 3, r));
    chunk[v] = w;
  }
}

// Bit v set when chunk vector v of this lane has its maximum >= tau.
template <int NJ>
__device__ __forceinline__ uint32_t chunk_flags(const float (&vm)[NJ], float tau) {
  uint32_t F = 0;
#pragma unroll
  for (int j = 0; j < NJ; ++j) F |= (vm[j] >= tau ? 1u : 0u) << j;
  // Bit j stands for chunk vector j ^ sw: permute bit positions by XOR.
  const int sw = (int)lane_id() & 7;
  if (sw & 1) F = ((F & 0x55555555u) << 1) | ((F >> 1) & 0x55555555u);
  if (sw & 2) F = ((F & 0x33333333u) << 2) | ((F >> 2) & 0x33333333u);
  if (sw & 4) F = ((F & 0x0F0F0F0Fu) << 4) | ((F >> 4) & 0x0F0F0F0Fu);
  return F;
}

template <int NJ>
__device__ __forceinline__ int count_ge(const float (&vm)[NJ], float tau) {
  int c = 0;
#pragma unroll
  for (int j = 0; j < NJ; ++j) c += vm[j] >= tau ? 1 : 0;
  return (int)__reduce_add_sync(FULL, (unsigned)c);
}

// A threshold tau such that between k and hi vectors have their maximum at
// or above it, searched as a distance d below the row maximum.  The first
// probe is the warp's previous threshold `prev` (an absolute value: it
// tracks rows of similar distribution far better than a distance from a row
// maximum that fluctuates), nudged toward the middle of the window after
// each acceptance.  False when no finite threshold reaches k vectors.
template <int NJ>
__device__ bool find_tau(const float (&vm)[NJ], float mx, int k, int hi, float& prev,
                         float& tau) {
  float lo = 0.0f, dhi = -1.0f, best = -1.0f;
  float d = __fsub_rn(mx, prev);
  if (!(d > 0.0f && d < __int_as_float(0x7f800000))) d = 1.0f;  // no (usable) previous
#pragma unroll 1
  for (int it = 0; it < 48; ++it) {
    const float t = __fsub_rn(mx, d);
    if (!(t > neg_inf())) break;
    const int c = count_ge(vm, t);
    if (c >= k) best = best < 0.0f ? d : fminf(best, d);
    if (c < k) {
      lo = d;
      d = dhi < 0.0f ? __fmul_rn(d, 2.0f) : 0.5f * (lo + dhi);
    } else if (c > hi) {
      dhi = d;
      d = 0.5f * (lo + dhi);
    } else {
      prev = __fsub_rn(mx, 2 * c < k + hi ? __fmul_rn(d, 1.03125f) : __fmul_rn(d, 0.96875f));
      tau = t;
      return true;
    }
    if (dhi >= 0.0f && !(dhi - lo > 0.0f)) break;
    if (!(d < __int_as_float(0x7f800000))) break;
  }
  if (best < 0.0f) return false;
  tau = __fsub_rn(mx, best);
  prev = tau;
  return tau > neg_inf();
}

// Bucket of x in [lo, lo + 64/scale) for the k-th-value histogram: a
// monotone map of x (equal values share a bucket), clamped to [0, 63].
// Bucket of x in an interval [a, b] with rs = 1 / (b - a): 63 - floor(64 z^4)
// for z = (b - x) * rs, clamped to [0, 63].  Every step is a monotone f32
// operation, so the map is monotone in x (equal values share a bucket); z^4
// makes the buckets narrow near a, where the candidates of a top-k tail
// crowd.  NaN (0 * inf at x = b) goes to the top bucket, as x = b does.
__device__ __forceinline__ int kbucket(float x, float b, float rs) {
  const float z = __fmul_rn(__fsub_rn(b, x), rs);
  const float z2 = __fmul_rn(z, z);
  const float m = __fmul_rn(64.0f, __fmul_rn(z2, z2));
  return m >= 63.0f ? 0 : (m > 0.0f ? 63 - (int)m : 63);
}

// Zeroes a level of the k-th-value histogram (counts, largest and smallest
// order key per bucket).
__device__ __forceinline__ void hist_clear(uint32_t* h) {
  const int lane = (int)lane_id();
  h[lane] = 0u;
  h[lane + 32] = 0u;
  h[64 + lane] = 0u;
  h[96 + lane] = 0u;
  h[128 + lane] = 0xFFFFFFFFu;
  h[160 + lane] = 0xFFFFFFFFu;
}

__device__ __forceinline__ void hist_add(uint32_t* h, int b, float x) {
  const uint32_t key = total_key(x);
  atomicAdd(&h[b], 1u);
  atomicMax(&h[64 + b], key);
  atomicMin(&h[128 + b], key);
}

// The candidates {x >= tau} of the flagged vectors, in vocabulary order, as
// (x after the temperature, index) into L.  The flagged vectors are first
// listed warp-wide (lane-major = vocabulary order) in Qs, then read back
// and processed 32 at a time, one per lane, with ballot prefix counts
// placing each lane's candidates.  STAGED: the vectors come from the stage,
// which already holds x (f32 rows transformed in place); otherwise from
// global memory (L2: the row was staged moments ago), transformed again
// when XF.  Returns the number of candidates, or -1 when there are more
// than ROW_CAP.
template <int DT, int NJ, bool XF, bool EDGE, bool RT, bool STAGED>
__device__ __forceinline__ int collect_cands(const RowCtx& r, uint32_t flags, float tau,
                                             uint16_t* Qs, uint2* L, const uint4* stage) {
  constexpr int EPV = Elem<DT>::EPV;
  const int lane = (int)lane_id();
  const int nf = __popc(flags);
  const int incl = (int)warp_inclusive_scan((uint32_t)nf);
  const int NF = __shfl_sync(FULL, incl, 31);
  {
    const int nj = (RT && !EDGE) ? r.nj : NJ;
    int p = incl - nf;
    uint32_t fl = flags;
    while (fl) {
      Qs[p++] = (uint16_t)(lane * nj + __ffs(fl) - 1);
      fl &= fl - 1;
    }
  }
  __syncwarp();
  const uint32_t lt = lanemask_lt();
  int base = 0;
  // Each lane's next vector is loaded one iteration ahead.
  auto load = [&](int q) { return STAGED ? stage[q] : __ldg(r.g16 + q); };
  int qn = lane < NF ? (int)Qs[lane] : -1;
  uint4 wn = qn >= 0 ? load(qn) : make_uint4(0u, 0u, 0u, 0u);
  for (int i0 = 0; i0 < NF; i0 += 32) {
    const int q = qn;
    const uint4 w = wn;
    const int inext = i0 + 32 + lane;
    qn = inext < NF ? (int)Qs[inext] : -1;
    if (qn >= 0) wn = load(qn);
    float x[EPV];
    uint32_t bits = 0;
    if (q >= 0) {
      float e[EPV];
      unpack_vec<DT>(w, e);
#pragma unroll
      for (int c = 0; c < EPV; ++c) {
        x[c] = STAGED ? e[c] : xform<XF, EDGE>(e[c], q * EPV + c - r.mis, r);
        bits |= (x[c] >= tau ? 1u : 0u) << c;
      }
    }
    const int cnt = __popc(bits);
    int pre = 0, tot = 0;
#pragma unroll
    for (int d = 0; (1 << d) <= EPV; ++d) {
      const uint32_t b = __ballot_sync(FULL, (cnt >> d) & 1);
      pre += __popc(b & lt) << d;
      tot += __popc(b) << d;
    }
    if (base + tot > ROW_CAP) return -1;
    int o = base + pre;
#pragma unroll
    for (int c = 0; c < EPV; ++c)
      if (bits & (1u << c))
        L[o++] = make_uint2(__float_as_uint((XF || STAGED) ? x[c] : __fmul_rn(x[c], r.inv)),
                            (uint32_t)(q * EPV + c - r.mis));
    base += tot;
  }
  __syncwarp();
  return base;
}

// ===========================================================================
// Fast path: warp-cooperative finish of a row from its candidate list.
// ===========================================================================

__device__ __forceinline__ float ex(const uint2& e) { return __uint_as_float(e.x); }

// Ascending bitonic sort of 32*R keys held R per lane (element lane*R + r);
// R is a power of two.  The merge sizes and the cross-lane strides (>= R) are
// loops: only the R register operations of one step are unrolled, plus the
// log2(R) in-lane steps whose register pairs must be static.  The sorts run
// on rows that reach the finishers; straight-line code for all 36 steps of a
// 256-key sort would evict the hot path from the instruction cache.
template <int R, typename T>
__device__ __forceinline__ void bitonic(T (&v)[R]) {
  const int lane = (int)lane_id();
#pragma unroll 1
  for (int size = 2; size <= 32 * R; size <<= 1) {
#pragma unroll 1
    for (int stride = size >> 1; stride >= R; stride >>= 1) {
      const int ls = stride / R;
      const bool lower = (lane & ls) == 0;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const bool up = ((lane * R + r) & size) == 0;
        const T o = __shfl_xor_sync(FULL, v[r], ls);
        v[r] = (lower == up) ? (o < v[r] ? o : v[r]) : (o > v[r] ? o : v[r]);
      }
    }
#pragma unroll
    for (int stride = R >> 1; stride > 0; stride >>= 1) {
      if (stride < size) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
          if ((r & stride) == 0) {
            const bool up = ((lane * R + r) & size) == 0;
            const T a = v[r], b = v[r + stride];
            if ((a > b) == up) {
              v[r] = b;
              v[r + stride] = a;
            }
          }
        }
      }
    }
  }
}

__device__ __forceinline__ unsigned long long pack_out(int status, uint32_t token) {
  return ((unsigned long long)(unsigned)status << 32) | token;
}

// exp(x) for x <= 0 (finite or -inf): cr_expf without the NaN and overflow
// branches, which such arguments never take; same operations otherwise.  The
// underflow case (x < -104, exp(x) rounds to 0) is a select after the
// arithmetic, not a branch around it, so that the independent calls of a
// lane (the nucleus path's four per 16-byte vector) interleave.
__device__ __forceinline__ float cr_expf_nonpos(float xf) {
  const double x = (double)xf;
  // rint(x / ln2) by the 1.5 * 2^52 addition (round to nearest even, exact
  // for |x / ln2| < 2^51); k is the low word of the sum.
  const double big = __dadd_rn(__dmul_rn(x, 0x1.71547652b82fep+0), 0x1.8p52);
  const double kd = __dsub_rn(big, 0x1.8p52);
  double r = __fma_rn(-kd, 0x1.62e42fefa39efp-1, x);
  r = __fma_rn(-kd, 0x1.abc9e3b39803fp-56, r);
  double p = 0x1.6124613a86d09p-33;
  p = __fma_rn(p, r, 0x1.1eed8eff8d898p-29);
  p = __fma_rn(p, r, 0x1.ae64567f544e4p-26);
  p = __fma_rn(p, r, 0x1.27e4fb7789f5cp-22);
  p = __fma_rn(p, r, 0x1.71de3a556c734p-19);
  p = __fma_rn(p, r, 0x1.a01a01a01a01ap-16);
  p = __fma_rn(p, r, 0x1.a01a01a01a01ap-13);
  p = __fma_rn(p, r, 0x1.6c16c16c16c17p-10);
  p = __fma_rn(p, r, 0x1.1111111111111p-7);
  p = __fma_rn(p, r, 0x1.5555555555555p-5);
  p = __fma_rn(p, r, 0x1.5555555555555p-3);
  p = __fma_rn(p, r, 0.5);
  p = __fma_rn(p, r, 1.0);
  p = __fma_rn(p, r, 1.0);
  const int k = __double2loint(big);
  const double scale = __hiloint2double((k + 1023) << 20, 0);
  const float e = __double2float_rn(__dmul_rn(p, scale));
  return xf < -104.0f ? 0.0f : e;
}

// Shared-memory vector load and store through the shared window (32-bit
// addresses), whatever address space the compiler could infer for a pointer.
__device__ __forceinline__ float4 lds4(uint32_t a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(a)
               : "memory");
  return v;
}

__device__ __forceinline__ void sts4(uint32_t a, const float4& v) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

// Sequential f32 sum of B[0..count) by lane 0 (B in shared memory, 16-byte
// aligned and zero-padded to a multiple of 8), with the running sums written
// back in place when PREFIX is set; returns the total to every lane.  Eight
// terms per step, loads one step ahead of the additions.
template <bool PREFIX>
__device__ __forceinline__ float chain_smem(float* B, int count) {
  float c = 0.0f;
  if (lane_id() == 0) {
    const uint32_t base = smem_u32(B);
    const int n8 = (count + 7) >> 3;
    float4 na = make_float4(0.f, 0.f, 0.f, 0.f), nb = na;
    if (n8 > 0) {
      na = lds4(base);
      nb = lds4(base + 16u);
    }
    for (int q = 0; q < n8; ++q) {
      float4 va = na, vb = nb;
      const uint32_t a = base + 32u * (uint32_t)q;
      if (q + 1 < n8) {
        na = lds4(a + 32u);
        nb = lds4(a + 48u);
      }
      c = __fadd_rn(c, va.x);
      va.x = c;
      c = __fadd_rn(c, va.y);
      va.y = c;
      c = __fadd_rn(c, va.z);
      va.z = c;
      c = __fadd_rn(c, va.w);
      va.w = c;
      c = __fadd_rn(c, vb.x);
      vb.x = c;
      c = __fadd_rn(c, vb.y);
      vb.y = c;
      c = __fadd_rn(c, vb.z);
      vb.z = c;
      c = __fadd_rn(c, vb.w);
      vb.w = c;
      if (PREFIX) {
        sts4(a, va);
        sts4(a + 16u, vb);
      }
    }
  }
  __syncwarp();
  return __shfl_sync(FULL, c, 0);
}

// Final softmax over the survivors L[0..ns) (vocabulary order, every x <= m2,
// their maximum) and the vocabulary-order draw (sampling.rs:700-729):
// exp(x - m2) in Bb (zero-padded to a multiple of 8), one lane's sequential
// f32 prefix sums, and the first survivor whose running sum reaches u * sum
// (the last index of the row when none does).  Bb: ns + 8 floats.
__device__ __forceinline__ unsigned long long draw_tail(const uint2* L, int ns, int n, float m2,
                                                        float u, float* Bb, unsigned char* masks,
                                                        float* probs) {
  const int lane = (int)lane_id();
  for (int j = lane; j < ns; j += 32) Bb[j] = cr_expf_nonpos(__fsub_rn(ex(L[j]), m2));
  if (lane < ((8 - (ns & 7)) & 7)) Bb[ns + lane] = 0.0f;  // zero-pad to a multiple of 8
  __syncwarp();
  const float sum = chain_smem<true>(Bb, ns);
  if (!is_finite(sum) || sum <= 0.0f) return pack_out(Q3S_STATUS_INVALID_DENOMINATOR, 0u);
  const float thr = __fmul_rn(u, sum);
  uint32_t token = (uint32_t)(n - 1);
  for (int j0 = 0; j0 < ns; j0 += 32) {
    const int j = j0 + lane;
    const unsigned bb = __ballot_sync(FULL, j < ns && Bb[j] >= thr);
    if (bb) {
      token = L[j0 + __ffs(bb) - 1].y;
      break;
    }
  }
  if (masks || probs) {
    for (int j = lane; j < ns; j += 32) {
      const uint2 en = L[j];
      if (masks) masks[en.y] |= 4;
      if (probs)
        probs[en.y] = __double2float_rn((double)cr_expf(__fsub_rn(ex(en), m2)) / (double)sum);
    }
  }
  __syncwarp();
  return pack_out(Q3S_STATUS_OK, token);
}

// t, the k-th largest x of the candidates L[0..c) (x after the temperature,
// index), k <= c <= ROW_CAP, ties kept (sampling.rs:654-663): a 64-bucket
// histogram (count, largest and smallest order key per bucket) of the
// candidates in a value interval [a, b] (first [lo, Mx]) locates the bucket
// holding the k-th largest.  When t is the bucket's largest or smallest value
// it is read off directly; a bucket of at most 32 values is ranked exactly; a
// fuller one becomes the next interval (its own smallest and largest value,
// which land in different buckets, so every level shrinks it).  The bucket
// map is monotone, so a bucket's members are exactly the candidates between
// its smallest and largest value.  h: the histogram (HIST_WORDS - 16 words);
// Bb: 32 floats of gather space.
__device__ __forceinline__ float kth_largest(const uint2* L, int c, int k, float Mx, float lo,
                                             float* Bb, uint32_t* h) {
  const int lane = (int)lane_id();
  const uint32_t lt = lanemask_lt();
  float t = Mx;
  if (k > 1) {
    float a = lo, b = Mx;
    uint32_t need = (uint32_t)k;  // rank of t among the candidates in [a, b], from the top
#pragma unroll 1
    while (true) {
      if (!(a < b)) {
        t = b;
        break;
      }
      const float d = __fsub_rn(b, a);
      const float rs = __frcp_rn(d < __int_as_float(0x7f800000) ? d : 3.40282347e38f);
      hist_clear(h);
      __syncwarp();
      for (int j = lane; j < c; j += 32) {
        const float x = ex(L[j]);
        if (a <= x && x <= b) hist_add(h, kbucket(x, b, rs), x);
      }
      __syncwarp();
      // Suffix counts from the top bucket down: suf = members in buckets
      // >= 2 * lane (lane 0: all members, >= need).
      const uint32_t h0 = h[2 * lane], h1 = h[2 * lane + 1];
      uint32_t suf = h0 + h1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t w = __shfl_down_sync(FULL, suf, o);
        if (lane + o < 32) suf += w;
      }
      const unsigned ball = __ballot_sync(FULL, suf >= need);
      const int Lh = 31 - __clz(ball);
      const uint32_t sL = __shfl_sync(FULL, suf, Lh);
      const uint32_t a0 = __shfl_sync(FULL, h0, Lh), a1 = __shfl_sync(FULL, h1, Lh);
      int B;
      uint32_t nB;
      if (sL - a0 >= need) {
        B = 2 * Lh + 1;
        need -= sL - a0 - a1;
        nB = a1;
      } else {
        B = 2 * Lh;
        need -= sL - a0;
        nB = a0;
      }
      // 1 <= need <= nB.
      if (need == 1u) {
        t = from_total_key(h[64 + B]);
        break;
      }
      if (need == nB) {
        t = from_total_key(h[128 + B]);
        break;
      }
      if (nB <= 32u) {
        // Gather bucket B and rank its values exactly.
        uint32_t base = 0;
        for (int j0 = 0; j0 < c; j0 += 32) {
          const int j = j0 + lane;
          float x = 0.0f;
          bool in = false;
          if (j < c) {
            x = ex(L[j]);
            in = a <= x && x <= b && kbucket(x, b, rs) == B;
          }
          const unsigned bb = __ballot_sync(FULL, in);
          if (in) Bb[base + __popc(bb & lt)] = x;
          base += __popc(bb);
        }
        __syncwarp();
        const float g = lane < (int)nB ? Bb[lane] : 0.0f;
        uint32_t gt = 0, ge = 0;
        for (int i = 0; i < (int)nB; ++i) {
          const float w = __shfl_sync(FULL, g, i);
          gt += w > g ? 1u : 0u;
          ge += w >= g ? 1u : 0u;
        }
        const unsigned hit = __ballot_sync(FULL, lane < (int)nB && gt < need && need <= ge);
        t = __shfl_sync(FULL, g, __ffs(hit) - 1);
        __syncwarp();
        break;
      }
      // Next interval: bucket B's own extent.
      a = from_total_key(h[128 + B]);
      b = from_total_key(h[64 + B]);
      __syncwarp();
    }
  }
  return t;
}

// Keeps the candidates x >= t, compacted in place in vocabulary order (d <= j,
// and every read of an iteration precedes its writes); returns their number.
__device__ __forceinline__ int compact_ge(uint2* L, int c, float t) {
  const int lane = (int)lane_id();
  const uint32_t lt = lanemask_lt();
  int ns = 0;
  for (int j0 = 0; j0 < c; j0 += 32) {
    const int j = j0 + lane;
    uint2 en = make_uint2(0u, 0u);
    bool sv = false;
    if (j < c) {
      en = L[j];
      sv = ex(en) >= t;
    }
    const unsigned bb = __ballot_sync(FULL, sv);
    if (sv) L[ns + __popc(bb & lt)] = en;
    ns += __popc(bb);
  }
  __syncwarp();
  return ns;
}

// Finishes a row without top-p from its candidates L[0..c) in vocabulary
// order, k <= c <= ROW_CAP: the statements of sampling.rs:654-663 and
// 700-729 on the candidate set, which holds every element >= the k-th
// largest x (all others are masked by top-k).  The survivors x >= t are
// compacted in place, still in vocabulary order, with exp(x - Mx) in Bb
// (masked entries are exact zeros of the reference's sums and are skipped);
// one lane accumulates the sequential f32 prefix sums, and the draw is the
// first survivor whose running sum reaches u * sum.  Bb: ROW_CAP + 8 floats.
// Writes t to tsm[0].
__device__ __forceinline__ unsigned long long finish_topk_hist(
    uint2* L, int c, int k, int n, float Mx, float lo, float u, float* Bb, uint32_t* h,
    float* tsm, unsigned char* masks, float* probs) {
  const int lane = (int)lane_id();
  const float t = kth_largest(L, c, k, Mx, lo, Bb, h);
  if (lane == 0) tsm[0] = t;
  const int ns = compact_ge(L, c, t);
  return draw_tail(L, ns, n, Mx, u, Bb, masks, probs);
}

// Status of finish_topp_hist when the survivors outnumber its sort (the row
// then takes the general path).
constexpr int WIDE_GENERAL = 0x7E;

// The nucleus walk of sampling.rs:680-697 over the survivors L[0..ns) in
// vocabulary order, ns <= 32 R (one instantiation, R = 8: a second one
// costs more in instruction-cache misses than its shorter sort saves): each survivor within 16 of the maximum has
// p = Bb[j] * inv_total (Bb[j] = exp(x - Mx)); the reference visits them by
// (p desc, index asc) and keeps the positions before the first position > 0
// whose preceding cumulative reaches top_p.  Here the p values alone are
// sorted (32-bit keys ~bits(p): ascending key = descending p; ties keep equal
// p, which is all the cumulative needs), one lane chains their prefix sums
// into P (32 R floats), and the first position q >= 1 with P[q - 1] >= top_p
// is found in parallel.  Returns J, the nucleus size; kJ is the key of its
// last member and gt the number of survivors with a smaller key (larger p):
// the nucleus is every survivor with key < kJ plus the J - gt survivors of
// key kJ with the smallest indices.
template <int R>
__device__ __forceinline__ int topp_walk(const uint2* L, const float* Bb, int ns, float cutoff,
                                         float inv_total, float top_p, float* P, uint32_t& kJ,
                                         int& gt) {
  const int lane = (int)lane_id();
  uint32_t v[R];
  int cnt = 0;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int j = lane * R + r;
    v[r] = 0xFFFFFFFFu;
    if (j < ns && ex(L[j]) >= cutoff) {
      v[r] = ~__float_as_uint(__fmul_rn(Bb[j], inv_total));
      ++cnt;
    }
  }
  const int m = (int)__reduce_add_sync(FULL, (unsigned)cnt);
  bitonic<R>(v);
#pragma unroll
  for (int r = 0; r < R; ++r) P[lane * R + r] = v[r] != 0xFFFFFFFFu ? __uint_as_float(~v[r]) : 0.0f;
  __syncwarp();
  chain_smem<true>(P, m);
  int first = m;
  for (int q = 1 + lane; q < m; q += 32) {
    if (P[q - 1] >= top_p) {
      first = q;
      break;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) first = min(first, __shfl_xor_sync(FULL, first, o));
  const int J = first;  // >= 1: the row maximum is always within 16 of itself
  uint32_t mine = 0u;
#pragma unroll
  for (int r = 0; r < R; ++r)
    if (lane * R + r == J - 1) mine = v[r];
  kJ = __shfl_sync(FULL, mine, (J - 1) / R);
  int g = 0;
#pragma unroll
  for (int r = 0; r < R; ++r) g += v[r] < kJ ? 1 : 0;
  gt = (int)__reduce_add_sync(FULL, (unsigned)g);
  __syncwarp();
  return J;
}

// Finishes a top-p row from its candidates L[0..c) in vocabulary order,
// k <= c <= ROW_CAP (sampling.rs:654-729): the exact k-th largest t and the
// survivors x >= t as in finish_topk_hist; the top-p denominator, the
// sequential f32 sum of exp(x - Mx) over the survivors in vocabulary order
// (every other entry is masked, an exact zero of the reference's sum); the
// nucleus by topp_walk, compacted in place (vocabulary order) and drawn by
// draw_tail with its own maximum.  More than 256 survivors: WIDE_GENERAL.
// Bb: the exp terms in [0, 256 + 8), the walk's prefix sums in [256, 512).
__device__ __forceinline__ unsigned long long finish_topp_hist(
    uint2* L, int c, int k, int n, float Mx, float lo, float u, float top_p, float* Bb,
    uint32_t* h, float* tsm, unsigned char* masks, float* probs) {
  const int lane = (int)lane_id();
  const uint32_t lt = lanemask_lt();
  const float t = kth_largest(L, c, k, Mx, lo, Bb, h);
  if (lane == 0) tsm[0] = t;
  const int ns = compact_ge(L, c, t);
  if (ns > 256) return pack_out(WIDE_GENERAL, 0u);
  // Denominator (sampling.rs:666-679).
  for (int j = lane; j < ns; j += 32) Bb[j] = cr_expf_nonpos(__fsub_rn(ex(L[j]), Mx));
  if (lane < ((8 - (ns & 7)) & 7)) Bb[ns + lane] = 0.0f;  // zero-pad to a multiple of 8
  __syncwarp();
  const float total = chain_smem<false>(Bb, ns);
  if (!is_finite(total) || total <= 0.0f) return pack_out(Q3S_STATUS_INVALID_DENOMINATOR, 0u);
  const float inv_total = __fdiv_rn(1.0f, total);
  const float cutoff = __fsub_rn(Mx, 16.0f);
  uint32_t kJ;
  int gt;
  const int J = topp_walk<8>(L, Bb, ns, cutoff, inv_total, top_p, Bb + 256, kJ, gt);
  const int need = J - gt;  // members of key kJ, by index
  // Compact the nucleus in place (vocabulary order kept) and take its maximum.
  int n2 = 0, ties = 0;
  float m2 = neg_inf();
  for (int j0 = 0; j0 < ns; j0 += 32) {
    const int j = j0 + lane;
    uint2 en = make_uint2(0u, 0u);
    uint32_t key = 0xFFFFFFFFu;
    if (j < ns) {
      en = L[j];
      if (ex(en) >= cutoff) key = ~__float_as_uint(__fmul_rn(Bb[j], inv_total));
    }
    const unsigned tb = __ballot_sync(FULL, key == kJ);
    const bool keep = key < kJ || (key == kJ && ties + __popc(tb & lt) < need);
    ties += __popc(tb);
    if (keep) m2 = fmaxf(m2, ex(en));
    const unsigned bb = __ballot_sync(FULL, keep);
    if (keep) L[n2 + __popc(bb & lt)] = en;
    n2 += __popc(bb);
  }
  __syncwarp();
  m2 = warp_max(m2);
  if (!(m2 > neg_inf())) return pack_out(Q3S_STATUS_NO_CANDIDATE, 0u);
  return draw_tail(L, n2, n, m2, u, Bb, masks, probs);
}

// Debug pass over the stage: bit0 finite x, bit1 x >= t (OR-ed in).
template <int DT, bool XF>
__device__ void debug_masks(const void* p0, const RowCtx& r, float t, unsigned char* masks) {
  const unsigned lane = lane_id();
  for (int i = lane; i < r.n; i += 32) {
    float x = xform<XF, false>(load_elem<DT>(p0, i), i, r);
    if (!XF) x = is_finite(x) ? __fmul_rn(x, r.inv) : neg_inf();
    unsigned char m = 0;
    if (is_finite(x)) m = 1;
    if (is_finite(x) && x >= t) m |= 2;
    masks[i] |= m;
  }
  __syncwarp();
}

// Outcomes of the templated front of the fast path.  The FRONT_GEN_*
// outcomes send the row to the general path, each for its own reason.
enum {
  FRONT_DONE = 1,
  FRONT_LIST = 2,
  FRONT_GEN_INF = 3,       // a raw +inf logit (rows selecting on raw values)
  FRONT_GEN_TAU = 4,       // no usable threshold on the vector maxima
  FRONT_GEN_OVERFLOW = 5,  // more than ROW_CAP candidates
};

// Fast path, up to the candidate list: scan, release of the stage, tau and
// the collection.  FRONT_LIST leaves c candidates in f.list with the row
// maximum Mx and the lower bound lo of their values (after the temperature);
// FRONT_DONE sets `out`; FRONT_GEN_* sends the row to the general path
// (which reads the row from global memory).
template <int DT, int NJ, bool XF, bool EDGE, bool RT>
__device__ int fast_front(const FastSpace& f, int k, bool use_top_p, const RowCtx& rc,
                          Releaser& rel, float& delta, RowOut& out, int& c_out, float& Mx_out,
                          float& lo_out) {
  // f32 rows with a transform hold x in their stage after the in-place
  // transform: their candidates are collected from it, and the stage is
  // released after the collection instead of after the scan.
  constexpr bool STAGED = XF && DT == Q3S_DTYPE_F32;
  float vm[NJ];
  float mx;
  if (STAGED) {
    // f32 rows are transformed in the stage first; the scan is then plain.
    xform_stage_f32<NJ, EDGE, RT>(f, rc);
    mx = scan_stage<DT, NJ, false, EDGE, RT>(f, rc, vm);
  } else {
    mx = scan_stage<DT, NJ, XF, EDGE, RT>(f, rc, vm);
  }
  if (!STAGED) release<DT>(rel);  // everything below reads the row from global memory
  if (!XF && mx == __int_as_float(0x7f800000)) return FRONT_GEN_INF;  // raw +inf
  if (mx == neg_inf() || mx != mx) {
    out = {rc.sf >= 0 ? Q3S_STATUS_SUPPRESSION_NO_CANDIDATE : Q3S_STATUS_NO_CANDIDATE, 0u};
    return FRONT_DONE;
  }
  const float Mx = XF ? mx : __fmul_rn(mx, rc.inv);
  if (Mx == __int_as_float(0x7f800000)) {
    out = {Q3S_STATUS_INVALID_DENOMINATOR, 0u};
    return FRONT_DONE;
  }
  const int hi = k <= 128 ? max(2 * k, 64) : k + 96;
  float tau = mx;  // k == 1: the maximum and its ties
  if (k > 1 && !find_tau(vm, mx, k, hi, delta, tau)) return FRONT_GEN_TAU;
  // Raw-domain selection: lower tau until its image lies strictly below the
  // image of tau, so no element below the new tau can tie the k-th largest
  // x after the multiply.
  if (!XF && rc.inv != 1.0f) {
    const float img = __fmul_rn(tau, rc.inv);
    float t2 = tau;
    bool ok = false;
#pragma unroll 1
    for (int it = 0; it < 8 && !ok; ++it) {
      t2 = __fsub_rn(t2, fmaxf(fabsf(t2) * 3.814697265625e-06f, 1.1754944e-38f));
      ok = __fmul_rn(t2, rc.inv) < img;
    }
    if (!ok) return FRONT_GEN_TAU;
    tau = t2;
  }
  const uint32_t flags = chunk_flags(vm, tau);
  const int c = collect_cands<DT, NJ, XF, EDGE, RT, STAGED>(
      rc, flags, tau, reinterpret_cast<uint16_t*>(f.Kb), f.list,
      reinterpret_cast<const uint4*>(f.stage));
  if (STAGED) release<DT>(rel);
  if (c < k) return FRONT_GEN_OVERFLOW;  // more than ROW_CAP candidates (or none: impossible)
  c_out = c;
  Mx_out = Mx;
  lo_out = XF ? tau : __fmul_rn(tau, rc.inv);  // every candidate lies in [lo, Mx]
  return FRONT_LIST;
}

// Greedy row (sampling.rs:574-591) straight from the stage.
template <int DT>
__device__ RowOut greedy_stage(const FastSpace& f, const StageView& s, int sf, int allow) {
  constexpr int EPV = Elem<DT>::EPV;
  const unsigned lane = lane_id();
  unsigned long long best = 0ull;
  for (int q = lane; q < s.Q; q += 32) {
    float e[EPV];
    unpack<DT>(f.stage, q, e);
#pragma unroll
    for (int c = 0; c < EPV; ++c) {
      const int i = q * EPV + c - s.mis;
      if ((unsigned)i < (unsigned)s.n && is_finite(e[c]) && idx_allowed(i, sf, allow)) {
        const unsigned long long k =
            ((unsigned long long)total_key(e[c]) << 32) | (0xFFFFFFFFu - (uint32_t)i);
        best = k > best ? k : best;
      }
    }
  }
  best = warp_max_u64(best);
  if (best == 0ull) return {Q3S_STATUS_NO_CANDIDATE, 0u};
  return {Q3S_STATUS_OK, 0xFFFFFFFFu - (uint32_t)best};
}

// Top-p without top-k (top_k 0, or at least the vocabulary) on an f32 row
// held in its stage (sampling.rs:592-729).  The reference takes the softmax
// denominator over the whole row and walks every entry within 16 of the
// maximum in (p desc, index asc) order; the nucleus it keeps is, in practice,
// a small set of the largest entries.  Here, all in the stage:
//   * the penalty goes to the history ids only (one per set bit of the
//     history bitmap), then one pass masks, scales by the temperature and
//     takes the maximum Mx: the stage holds x;
//   * a histogram of the entries within 16 of the maximum by 0.5-wide
//     bands of Mx - x gives the deepest band B whose cumulative count is at
//     most 256; the entries of bands <= B are the candidates (x and index,
//     in any order), and the largest x of the other entries within 16 of the
//     maximum, xout, is kept;
//   * the same pass turns the stage into e = exp(x - Mx) (masked entries
//     and entries outside the row are exact zeros), and one lane adds the
//     stage in vocabulary order up to the suppressed range, then the allowed
//     token inside it: every skipped entry is an exact zero of the
//     reference's sequential f32 denominator;
//   * nucleus_finish sorts the candidates by (p desc, index asc) with
//     p = e * inv_total and walks them with one lane.  The walk decides the
//     nucleus exactly when it closed and its last member's p is above
//     pout = p(xout), the largest p outside the candidates (every other entry
//     then sorts after it), or when no entry outside them is within 16 of
//     the maximum.  The nucleus, sorted back into vocabulary order, is drawn
//     by draw_tail with its own maximum.
// Two out-of-line halves with scalar and pointer arguments only, so that the
// fast path's row state stays in registers: nucleus_front (everything that
// reads the stage; the caller then releases it) and nucleus_finish.  Both
// return WIDE_GENERAL (the row takes the general path) when the candidates
// cannot decide the nucleus.
//
// nucleus_front's results besides the packed (status, candidate count):
// hist[1] Mx, hist[2] xout (-inf: none), hist[3] the denominator (f32
// bits); hist[16 .. 48) holds its histogram.  The candidates are list[0..c).
__device__ __forceinline__ int xband(float x, float Mx) {
  const int b = (int)__fmul_rn(__fsub_rn(Mx, x), 2.0f);
  return b > 31 ? 31 : b;
}

template <int NJ>
__device__ __noinline__ unsigned long long nucleus_front(
    unsigned char* stage, uint2* list, uint32_t* hist, const uint32_t* bm, int n, int mis,
    float inv, float pf, int use_pen, int sf, int allow, int edge, int nj) {
  const int lane = (int)lane_id();
  const uint32_t lt = lanemask_lt();
  float* row = reinterpret_cast<float*>(stage) + mis;  // element i at row[i]
  if (use_pen) penalize_stage(row, n, bm, pf);
  RowCtx rc;
  rc.n = n;
  rc.mis = mis;
  rc.Q = 0;
  rc.nj = nj;
  rc.g16 = nullptr;
  rc.inv = inv;
  rc.pf = pf;
  rc.use_pen = false;
  rc.sf = sf;
  rc.allow = allow;
  rc.bm = bm;
  const int sw = lane & 7;
  float4* chunk = reinterpret_cast<float4*>(stage) + lane * nj;
  // Mask and temperature in place (sampling.rs:608-631), and the maximum.
  float mx = neg_inf();
#pragma unroll 1
  for (int j = 0; j < nj; ++j) {
    const int v = (j & ~7) | ((j & 7) ^ sw);
    float4 w = chunk[v];
    const int i0 = (lane * nj + v) * 4 - mis;
    if (edge) {
      w.x = xform<true, true>(w.x, i0, rc);
      w.y = xform<true, true>(w.y, i0 + 1, rc);
      w.z = xform<true, true>(w.z, i0 + 2, rc);
      w.w = xform<true, true>(w.w, i0 + 3, rc);
    } else {
      w.x = xform<true, false>(w.x, i0, rc);
      w.y = xform<true, false>(w.y, i0 + 1, rc);
      w.z = xform<true, false>(w.z, i0 + 2, rc);
      w.w = xform<true, false>(w.w, i0 + 3, rc);
    }
    mx = fmaxf(mx, fmaxf(fmaxf(w.x, w.y), fmaxf(w.z, w.w)));
    chunk[v] = w;
  }
  mx = warp_max(mx);
  if (mx == neg_inf())
    return pack_out(sf >= 0 ? Q3S_STATUS_SUPPRESSION_NO_CANDIDATE : Q3S_STATUS_NO_CANDIDATE, 0u);
  if (!(mx < __int_as_float(0x7f800000)))  // +inf after the temperature
    return pack_out(Q3S_STATUS_INVALID_DENOMINATOR, 0u);
  const float Mx = mx;
  const float cutoff = __fsub_rn(Mx, 16.0f);
  // Histogram of the entries within 16 of the maximum by band.
  uint32_t* cnt = hist + 16;
  cnt[lane] = 0u;
  __syncwarp();
#pragma unroll 1
  for (int j = 0; j < nj; ++j) {
    const int v = (j & ~7) | ((j & 7) ^ sw);
    const float4 w = chunk[v];
    if (w.x >= cutoff) atomicAdd(&cnt[xband(w.x, Mx)], 1u);
    if (w.y >= cutoff) atomicAdd(&cnt[xband(w.y, Mx)], 1u);
    if (w.z >= cutoff) atomicAdd(&cnt[xband(w.z, Mx)], 1u);
    if (w.w >= cutoff) atomicAdd(&cnt[xband(w.w, Mx)], 1u);
  }
  __syncwarp();
  // The deepest band whose cumulative count still fits 256.
  uint32_t cs = cnt[lane];
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t a = __shfl_up_sync(FULL, cs, o);
    if (lane >= o) cs += a;
  }
  const unsigned fit = __ballot_sync(FULL, cs <= 256u);  // a prefix of the bands
  if (!(fit & 1u)) return pack_out(WIDE_GENERAL, 0u);   // the top band alone is too full
  const int B = 31 - __clz(fit);
  // Candidates (bands <= B) and xout; e = exp(x - Mx) in place.
  float xout = neg_inf();
  int c = 0;
#pragma unroll 1
  for (int j = 0; j < nj; ++j) {
    const int v = (j & ~7) | ((j & 7) ^ sw);
    const float4 w = chunk[v];
    const float x[4] = {w.x, w.y, w.z, w.w};
    const int i0 = (lane * nj + v) * 4 - mis;
    float e[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const bool elig = x[t] >= cutoff;
      const bool cand = elig && xband(x[t], Mx) <= B;
      if (elig && !cand) xout = fmaxf(xout, x[t]);
      const unsigned bb = __ballot_sync(FULL, cand);
      if (cand) list[c + __popc(bb & lt)] = make_uint2(__float_as_uint(x[t]), (uint32_t)(i0 + t));
      c += __popc(bb);
      e[t] = cr_expf_nonpos(__fsub_rn(x[t], Mx));
    }
    chunk[v] = make_float4(e[0], e[1], e[2], e[3]);
  }
  xout = warp_max(xout);
  __syncwarp();
  // Denominator (sampling.rs:666-679): vocabulary order up to the suppressed
  // range, then the allowed token inside it; everything else is zero.
  // The chain covers stage positions [0, span): entries below `lim` and the
  // zeros around them (span is padded to a multiple of 8, so an allowed
  // token inside the padding is already added in its place).
  const int lim = (sf >= 0 && sf < n) ? sf : n;
  const int span = (mis + lim + 7) & ~7;
  float total = chain_smem<false>(reinterpret_cast<float*>(stage), span);
  if (lim < n && allow >= span - mis && allow < n) total = __fadd_rn(total, row[allow]);
  if (lane == 0) {
    hist[1] = __float_as_uint(Mx);
    hist[2] = __float_as_uint(xout);
    hist[3] = __float_as_uint(total);
  }
  __syncwarp();
  return pack_out(Q3S_STATUS_OK, (uint32_t)c);
}

// The nucleus from nucleus_front's candidates list[0..c) (any order) and the
// draw.  The stage still holds e = exp(x - Mx) at every element (row[i]),
// and the row maximum Mx always belongs to the nucleus (it leads the
// (p desc, index asc) order), so the final softmax terms exp(x - m2) of the
// reference are the stage's e values: nothing is recomputed.
//   * topp_walk sorts the candidates' p = e * inv_total as 32-bit keys, one
//     lane chains the cumulative and a parallel search finds the nucleus size
//     J; the candidates decide the nucleus when the walk closed and its last
//     p is above pout, the largest p of an entry outside them, or when no
//     entry outside them is within 16 of the maximum (else WIDE_GENERAL);
//   * members (key below the last member's key kJ, and the J - gt entries of
//     key kJ with the smallest indices) are marked in a bitmap over the
//     vocabulary, so that one ordered pass over its words lists the nucleus in
//     vocabulary order with its e values: one lane's sequential f32 prefix
//     sums and a parallel search for the first running sum >= u * sum.
// More than 32 candidates tied at the cut (equal p) also return
// WIDE_GENERAL.  hist: hist[1..3] from nucleus_front, hist[64..192) the
// member bitmap (n <= 4096); Kb: the e values and prefix sums (512 floats);
// list[256..512): tied indices, then the nucleus indices (u16).
__device__ __noinline__ unsigned long long nucleus_finish(uint2* list, unsigned long long* Kb,
                                                          uint32_t* hist, const float* row, int c,
                                                          int n, float top_p, float u,
                                                          unsigned char* masks, float* probs) {
  const int lane = (int)lane_id();
  const uint32_t lt = lanemask_lt();
  const float Mx = __uint_as_float(hist[1]);
  const float xout = __uint_as_float(hist[2]);
  const float total = __uint_as_float(hist[3]);
  if (!is_finite(total) || total <= 0.0f) return pack_out(Q3S_STATUS_INVALID_DENOMINATOR, 0u);
  const float inv_total = __fdiv_rn(1.0f, total);
  float* Bb = reinterpret_cast<float*>(Kb);
  for (int j = lane; j < c; j += 32) Bb[j] = row[list[j].y];
  __syncwarp();
  uint32_t kJ;
  int gt;
  const int J = topp_walk<8>(list, Bb, c, neg_inf(), inv_total, top_p, Bb + 256, kJ, gt);
  const bool closed = J < c || Bb[256 + c - 1] >= top_p;
  if (xout > neg_inf()) {  // an entry outside the candidates is within 16 of the maximum
    const float pout = __fmul_rn(cr_expf_nonpos(__fsub_rn(xout, Mx)), inv_total);
    if (!closed || !(__uint_as_float(~kJ) > pout)) return pack_out(WIDE_GENERAL, 0u);
  }
  // Members into the bitmap; candidates tied at the cut listed aside.
  const int need = J - gt;
  uint32_t* bm = hist + 64;
  const int W = (n + 31) >> 5;
  for (int w = lane; w < W; w += 32) bm[w] = 0u;
  __syncwarp();
  uint16_t* tie = reinterpret_cast<uint16_t*>(list + 256);
  int T = 0;
  for (int j0 = 0; j0 < c; j0 += 32) {
    const int j = j0 + lane;
    uint32_t key = 0xFFFFFFFFu, idx = 0u;
    if (j < c) {
      idx = list[j].y;
      key = ~__float_as_uint(__fmul_rn(Bb[j], inv_total));
    }
    if (key < kJ) atomicOr(&bm[idx >> 5], 1u << (idx & 31));
    const unsigned tb = __ballot_sync(FULL, key == kJ);
    if (key == kJ && T + __popc(tb & lt) < 32) tie[T + __popc(tb & lt)] = (uint16_t)idx;
    T += __popc(tb);
  }
  __syncwarp();
  if (T > 32) return pack_out(WIDE_GENERAL, 0u);
  {
    const uint32_t mine = lane < T ? tie[lane] : 0xFFFFu;
    int rank = 0;
    for (int t = 0; t < T; ++t) rank += __shfl_sync(FULL, mine, t) < mine ? 1 : 0;
    if (lane < T && rank < need) atomicOr(&bm[mine >> 5], 1u << (mine & 31));
  }
  __syncwarp();
  // The nucleus in vocabulary order: lane l takes words [l * wpl, (l+1) * wpl).
  const int wpl = (W + 31) >> 5;
  int cnt = 0;
  for (int k = 0; k < wpl; ++k) {
    const int w = lane * wpl + k;
    if (w < W) cnt += __popc(bm[w]);
  }
  const int incl = (int)warp_inclusive_scan((uint32_t)cnt);
  const int J2 = __shfl_sync(FULL, incl, 31);
  uint16_t* nidx = reinterpret_cast<uint16_t*>(list + 256);
  int pos = incl - cnt;
  for (int k = 0; k < wpl; ++k) {
    const int w = lane * wpl + k;
    uint32_t bits = w < W ? bm[w] : 0u;
    while (bits) {
      const int i = (w << 5) + __ffs(bits) - 1;
      bits &= bits - 1;
      Bb[pos] = row[i];
      nidx[pos] = (uint16_t)i;
      ++pos;
    }
  }
  if (lane < ((8 - (J2 & 7)) & 7)) Bb[J2 + lane] = 0.0f;  // zero-pad to a multiple of 8
  __syncwarp();
  // Final softmax sum and the draw (sampling.rs:700-729) over e = exp(x - Mx).
  float* E = Bb;
  // The debug outputs keep the terms: the chain overwrites them with running
  // sums.  J2 = J <= 256 members, at most 8 per lane.
  float ev[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) ev[r] = (masks || probs) && lane + 32 * r < J2 ? E[lane + 32 * r] : 0.0f;
  const float sum = chain_smem<true>(E, J2);
  if (!is_finite(sum) || sum <= 0.0f) return pack_out(Q3S_STATUS_INVALID_DENOMINATOR, 0u);
  const float thr = __fmul_rn(u, sum);
  uint32_t token = (uint32_t)(n - 1);
  for (int q0 = 0; q0 < J2; q0 += 32) {
    const int q = q0 + lane;
    const unsigned bb = __ballot_sync(FULL, q < J2 && E[q] >= thr);
    if (bb) {
      token = nidx[q0 + __ffs(bb) - 1];
      break;
    }
  }
  if (masks || probs) {
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int q = lane + 32 * r;
      if (q >= J2) continue;
      const int i = nidx[q];
      if (masks) masks[i] |= 4;
      if (probs) probs[i] = __double2float_rn((double)ev[r] / (double)sum);
    }
  }
  __syncwarp();
  return pack_out(Q3S_STATUS_OK, token);
}

// A sampled row: fast path when it applies, else the general path.
// DBG: the launch fills the debug outputs (probs, masks).  Production
// launches compile without that code, which would otherwise weigh on the
// register allocation of the hot path.
// `path` receives the Q3S_PATH_* the row took (read by debug launches only).
// RT: the launch's rows may be shorter than the kernel's chunk (mixed
// vocabularies), see the dispatch below.
template <int DT, int NJ, bool DBG, bool RT>
__device__ RowOut sampled_row(const KernelArgs& a, const FastSpace& f, const GenSpace& g,
                              const RowPlan& pl, int sf, int allow, const StageView& s,
                              Releaser& rel, float& delta, const DebugRow& dbg_in, int& path) {
  const DebugRow dbg{DBG ? dbg_in.masks : nullptr, DBG ? dbg_in.probs : nullptr};
  const uint32_t flags = pl.nf >> 16;
  const bool use_top_p = (flags & PF_TOP_P) != 0u;
  RowCtx rc;
  rc.n = s.n;
  rc.mis = s.mis;
  rc.Q = s.Q;
  rc.g16 = s.g16;
  rc.inv = pl.inv;
  rc.pf = pl.pf;
  rc.sf = sf;
  rc.allow = allow;
  rc.bm = f.bm;
  rc.use_pen = (flags & PF_USE_PEN) != 0u;
  const float u = pl.u;
  const bool inv_ok = rc.inv > 0.0f && rc.inv < __int_as_float(0x7f800000);
  const bool fast = inv_ok && pl.k >= 1u && pl.k <= (uint32_t)FAST_MAX_K &&
                    pl.k < (uint32_t)s.n && s.Q <= 32 * NJ;
  path = Q3S_PATH_GENERAL_RULES;
  // A row is scanned without per-element index masks when it fills exactly
  // 32 lane chunks: of NJ vectors, or, in a runtime-chunk launch (RT), of
  // any multiple of 8 vectors below NJ (the 2048-entry code-predictor rows
  // beside 3072-entry talker rows).  Both kinds then run one code path,
  // which keeps the instruction cache to one copy of the scan.  Every other
  // row is EDGE.
  const bool aligned = s.mis == 0 && (s.n % Elem<DT>::EPV) == 0;
  const bool exact = aligned && (RT ? ((s.Q & 255) == 0 && s.Q <= 32 * NJ) : s.Q == 32 * NJ);
  rc.nj = exact ? (s.Q >> 5) : NJ;
  if (fast) {
    const bool xf = rc.use_pen || rc.sf >= 0;
    const bool edge = !exact;
    const int k = (int)pl.k;
    RowOut out;
    int c = 0;
    float Mx = 0.0f, lo = 0.0f;
    int fr;
    if (xf)
      fr = edge ? fast_front<DT, NJ, true, true, RT>(f, k, use_top_p, rc, rel, delta, out, c, Mx, lo)
                : fast_front<DT, NJ, true, false, RT>(f, k, use_top_p, rc, rel, delta, out, c, Mx,
                                                      lo);
    else
      fr = edge ? fast_front<DT, NJ, false, true, RT>(f, k, use_top_p, rc, rel, delta, out, c, Mx,
                                                      lo)
                : fast_front<DT, NJ, false, false, RT>(f, k, use_top_p, rc, rel, delta, out, c, Mx,
                                                       lo);
    if (fr == FRONT_DONE) {
      path = Q3S_PATH_FRONT_DONE;
      return out;
    }
    path = fr == FRONT_GEN_INF ? Q3S_PATH_GENERAL_INF
           : fr == FRONT_GEN_TAU ? Q3S_PATH_GENERAL_TAU
                                 : Q3S_PATH_GENERAL_OVERFLOW;
    if (fr == FRONT_LIST) {
      float* tsm = reinterpret_cast<float*>(f.hist);
      float* Bb = reinterpret_cast<float*>(f.Kb);
      unsigned long long r;
      if (!use_top_p) {
        r = finish_topk_hist(f.list, c, k, s.n, Mx, lo, u, Bb, f.hist + 16, tsm, dbg.masks,
                             dbg.probs);
      } else {
        r = finish_topp_hist(f.list, c, k, s.n, Mx, lo, u, pl.top_p, Bb, f.hist + 16, tsm,
                             dbg.masks, dbg.probs);
      }
      out = {(int)(r >> 32), (uint32_t)r};
      path = use_top_p ? Q3S_PATH_TOPK_TOPP : Q3S_PATH_TOPK;
      if (out.status == WIDE_GENERAL) {
        path = Q3S_PATH_GENERAL_WIDE;
        goto general;
      }
      if (dbg.masks) {
        __syncwarp();
        if (xf)
          debug_masks<DT, true>(s.p0, rc, tsm[0], dbg.masks);
        else
          debug_masks<DT, false>(s.p0, rc, tsm[0], dbg.masks);
      }
      return out;
    }
  }
general:
  if constexpr (DT == Q3S_DTYPE_F32) {
    // Top-p without top-k: the nucleus from the stage-resident row.
    if (use_top_p && inv_ok && (pl.k == 0u || pl.k >= (uint32_t)s.n) && s.Q <= 32 * NJ) {
      unsigned long long r =
          nucleus_front<NJ>(f.stage, f.list, f.hist, f.bm, s.n, s.mis, rc.inv, rc.pf,
                            rc.use_pen ? 1 : 0, rc.sf, rc.allow, exact ? 0 : 1, rc.nj);
      if ((int)(r >> 32) == Q3S_STATUS_OK) {
        r = nucleus_finish(f.list, f.Kb, f.hist, reinterpret_cast<const float*>(f.stage) + s.mis,
                           (int)(uint32_t)r, s.n, pl.top_p, u, dbg.masks, dbg.probs);
      }
      release<DT>(rel);
      const RowOut out{(int)(r >> 32), (uint32_t)r};
      path = out.status == WIDE_GENERAL ? Q3S_PATH_GENERAL_NUCLEUS : Q3S_PATH_NUCLEUS;
      if (out.status != WIDE_GENERAL) {
        if (dbg.masks && out.status == Q3S_STATUS_OK) {
          __syncwarp();
          debug_masks<DT, true>(s.p0, rc, neg_inf(), dbg.masks);
        }
        return out;
      }
    }
  }
  const unsigned lane = lane_id();
  release<DT>(rel);
  for (int i = lane; i < s.n; i += 32) g.A[i] = load_elem<DT>(s.p0, i);
  __syncwarp();
  const unsigned long long r = general_compute(
      g.A, g.B, g.BX, g.BI, f.bm, reinterpret_cast<uint32_t*>(f.list), f.hist, f.Kb, s.n, rc.inv,
      rc.pf,
      rc.use_pen ? 1 : 0, rc.sf, rc.allow, pl.k, use_top_p ? 1 : 0, pl.top_p, u, dbg.masks,
      dbg.probs);
  return {(int)(r >> 32), (uint32_t)r};
}

// The commit of one row (the per-row statements of q3s_commit_rows): the id
// into the frame's code column; unless the row's frame already failed, the
// subsequence advanced on a draw, the id appended to the row's history range
// (HISTORY_FULL when it has no room) and the first failure kept.
// Inlined: an out-of-line function taking the kernel arguments by reference
// makes the compiler copy them to local memory for every thread.
__device__ __forceinline__ void commit_row(const KernelArgs& a, long long row, RowOut out,
                                           bool do_sample) {
  if (a.c_codes) a.c_codes[row * a.c_codes_stride + a.c_group] = out.token;
  if (a.c_frame_status && a.c_frame_status[row] != Q3S_STATUS_OK) return;
  int st = out.status;
  if (st == Q3S_STATUS_OK && a.c_subseqs && do_sample) a.c_subseqs[row] += 1;
  if (st == Q3S_STATUS_OK && a.c_history) {
    const long long e = a.c_history_ends[row];
    if (e < a.c_history_limits[row]) {
      a.c_history[e] = (unsigned short)out.token;
      a.c_history_ends[row] = e + 1;
    } else {
      st = Q3S_STATUS_HISTORY_FULL;
    }
  }
  if (a.c_frame_status) a.c_frame_status[row] = (unsigned char)st;
}

// The body of a sampling block: block `bid` of `G` blocks that stride over
// the rows, in the dynamic shared memory `smem` (block_smem bytes).  The
// sampling kernel runs it with its own block index; the fused head kernel's
// last block runs it as the one block of a one-block grid.
// CM: the launch commits each row (q3s_sample_commit); other launches
// carry no commit code.
template <int DT, int NJ, bool DBG, bool RT, bool CM = false>
__device__ __forceinline__ void sample_block(const KernelArgs& a, unsigned char* smem,
                                             const long long bid, const long long G) {
  constexpr int es = Elem<DT>::BYTES;
  const int warp = threadIdx.x >> 5;
  const int warps = blockDim.x >> 5;
  const unsigned lane = lane_id();
  RingCtl* ctl = reinterpret_cast<RingCtl*>(smem);
  RowPlan* plans = reinterpret_cast<RowPlan*>(smem + CTL_BYTES);
  const size_t sbytes = stage_bytes(a.vcap, es);
  unsigned char* ring = smem + HEAD_BYTES;
  FastSpace f = carve_warp(ring + RING * sbytes + (size_t)warp * warp_bytes(a.vcap), a.vcap);
  const long long gw = bid * warps + warp;
  const GenSpace g = carve_gen(a.scratch + (size_t)gw * gen_bytes(a.vcap), a.vcap);
  if (threadIdx.x == 0) {
    for (int s = 0; s < RING; ++s) {
      mbar_init(&ctl->full[s], 1);
      ctl->issued[s] = 0u;
      ctl->consumed[s] = 0u;
    }
    ctl->ticket = 0u;
    ctl->abort = 0u;
    fence_mbarrier_init();
    fence_proxy_async_smem();
    for (int s = 0; s < RING; ++s) {
      const long long row = bid + (long long)s * G;
      if (row < a.num_rows) {
        issue_row<DT>(a, row, ring + s * sbytes, &ctl->full[s]);
        ctl->issued[s] = 1u;
      }
    }
  }
  // Plans of the first two batches of tickets, one thread per ticket.
  for (int i = threadIdx.x; i < PLAN_SLOTS; i += blockDim.x)
    reinterpret_cast<volatile uint32_t*>(&plans[i])[7] = NO_TAG;
  if (threadIdx.x < 64) {
    const long long row = bid + (long long)threadIdx.x * G;
    if (row < a.num_rows) store_plan(&plans[threadIdx.x], compute_plan(a, row, threadIdx.x));
  }
  __syncthreads();
  float delta = __int_as_float(0x7fc00000);  // previous tau of this warp (none yet)
#pragma unroll 1
  while (true) {
    uint32_t t = 0;
    if (lane == 0) t = atomicAdd(&ctl->ticket, 1u);
    t = __shfl_sync(FULL, t, 0);
    const long long row = bid + (long long)t * G;
    if (row >= a.num_rows) break;
    const long long clk0 = DBG ? clock64() : 0;
    const int slot = (int)(t % RING);
    const uint32_t gen = t / RING;
    f.stage = ring + slot * sbytes;
    Releaser rel{&a, ctl, f.stage, slot, bid + (long long)(t + RING) * G, gen + 1u, false};
    // The warp that opens a batch of 32 tickets plans the batch after it,
    // one lane per ticket.
    if ((t & 31u) == 0u && t >= 32u) {
      const uint32_t tp = t + 32u + lane;
      const long long prow = bid + (long long)tp * G;
      if (prow < a.num_rows) store_plan(&plans[tp % PLAN_SLOTS], compute_plan(a, prow, tp));
    }
    RowPlan pl;
    if (!__all_sync(FULL, load_plan(&plans[t % PLAN_SLOTS], t, pl))) pl = compute_plan(a, row, t);
    const int n = (int)(pl.nf & 0xFFFFu);
    const uint32_t pflags = pl.nf >> 16;
    const int st = (int)(pflags & PF_STATUS);
    const int sf = (int)(int16_t)(pl.sa & 0xFFFFu);
    const int allow = (int)(int16_t)(pl.sa >> 16);
    DebugRow dbg{nullptr, nullptr};
    if (DBG && a.masks && st == Q3S_STATUS_OK) dbg.masks = a.masks + row * a.probs_stride;
    if (DBG && a.probs && st == Q3S_STATUS_OK) dbg.probs = a.probs + row * a.probs_stride;
    if (dbg.masks)
      for (int i = lane; i < n; i += 32) dbg.masks[i] = 0;
    if (dbg.probs)
      for (int i = lane; i < n; i += 32) dbg.probs[i] = 0.0f;
    // History bitmap of a sampled row with a penalty (filled while the
    // stage copy may still be in flight).
    if (st == Q3S_STATUS_OK && (pflags & PF_USE_PEN)) {
      const long long h0 = history_begin(a, row), h1 = history_end(a, row);
      fill_history(a.history + h0, h1 - h0, n, f.bm, reinterpret_cast<unsigned char*>(f.list));
    }
    const bool ready = wait_stage(ctl, slot, gen, a.wait_ns);
    if (!__all_sync(FULL, ready)) {
      // A wait gave up (or the block aborts): this row is not run, no copy
      // is issued any more, and later tickets fail fast.
      if (lane == 0) {
        atomicExch(&ctl->abort, 1u);
        a.tokens[row] = 0u;
        a.status[row] = (unsigned char)Q3S_STATUS_NOT_RUN;
      }
      __syncwarp();
      continue;
    }
    if (lane == 0) ctl->consumed[slot] = gen + 1u;
    RowOut out{st, 0u};
    int path = Q3S_PATH_INVALID;
    if (st == Q3S_STATUS_OK) {
      const StageView s = complete_stage<DT>(a, row, n, f.stage);
      if (!(pflags & PF_DO_SAMPLE)) {
        out = greedy_stage<DT>(f, s, sf, allow);
        path = Q3S_PATH_GREEDY;
      } else {
        out = sampled_row<DT, NJ, DBG, RT>(a, f, g, pl, sf, allow, s, rel, delta, dbg, path);
      }
    }
    release<DT>(rel);
    if (lane == 0) {
      a.tokens[row] = out.token;
      a.status[row] = (unsigned char)out.status;
      if constexpr (CM) commit_row(a, row, out, (pflags & PF_DO_SAMPLE) != 0u);
      if (DBG && a.path_stats) {
        atomicAdd(&a.path_stats[path], 1ull);
        atomicAdd(&a.path_stats[Q3S_PATH_COUNT + path], (unsigned long long)(clock64() - clk0));
      }
    }
    __syncwarp();
  }
  // After an abort, copies may still be in flight into the ring: wait (with
  // a limit) for each before the block's shared memory goes away.
  __syncthreads();
  if (threadIdx.x == 0 && ctl->abort != 0u)
    for (int s = 0; s < RING; ++s)
      if (ctl->issued[s] > ctl->consumed[s])
        mbar_wait_bounded(&ctl->full[s], ctl->consumed[s] & 1u, WAIT_LIMIT_NS);
}

template <int DT, int NJ, bool DBG, bool RT, bool CM>
__global__ void __launch_bounds__(MAX_WARPS * 32, 1) sample_kernel(const KernelArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  sample_block<DT, NJ, DBG, RT, CM>(a, smem, blockIdx.x, gridDim.x);
}

// Producer fusion: the head projection logits = hidden · Wᵀ of the talker's
// codec_head (talker.rs:87-89) or a code-predictor lm_head
// (code_predictor.rs:402), then the sampling of its rows, in one launch.
// Every block stages the (at most MAX_WARPS) hidden rows as f32 in shared
// memory and computes a slice of the outputs, one warp per output: each lane
// reads 16-byte vectors of the weight row, multiplies by the hidden values
// (bf16 x f32, each product and sum rounded separately) and the lanes' partial
// sums are combined by a fixed butterfly, so every launch computes the same
// f32 logits.  The logits go to the caller's buffer, where they stay in L2.
// The last block to finish its slice (a device-scope counter, reset by that
// block) runs the sampling block over all rows, one warp per row.
template <int NJ>
__global__ void __launch_bounds__(MAX_WARPS * 32, 1)
    head_sample_kernel(const HeadArgs h, const KernelArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ int last_block;
  const int R = (int)a.num_rows;
  const int H = h.hidden_size;
  float* hs = reinterpret_cast<float*>(smem);  // [R, H]
  // Staged with 16-byte loads, four per thread in flight, when every row
  // starts on a 16-byte boundary; element by element otherwise.
  const int hes = h.hidden_dtype == Q3S_DTYPE_F32 ? 4 : 2;
  if (((reinterpret_cast<uintptr_t>(h.hidden) | (uintptr_t)(h.hidden_stride * hes)) & 15u) == 0u) {
    const int per_row = H * hes / 16;  // 16-byte vectors per row
    const int total = R * per_row;
    for (int i0 = threadIdx.x; i0 < total; i0 += 4 * blockDim.x) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * (int)blockDim.x;
        if (i < total) {
          const int r = i / per_row, c = i - r * per_row;
          v[u] = __ldg(reinterpret_cast<const uint4*>(static_cast<const unsigned char*>(h.hidden) +
                                                      (long long)r * h.hidden_stride * hes) + c);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * (int)blockDim.x;
        if (i < total) {
          const int r = i / per_row, c = i - r * per_row;
          if (hes == 4) {
            *reinterpret_cast<uint4*>(hs + r * H + 4 * c) = v[u];
          } else {
            const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
            float4* d = reinterpret_cast<float4*>(hs + r * H + 8 * c);
            d[0] = make_float4(__uint_as_float(w[0] << 16), __uint_as_float(w[0] & 0xFFFF0000u),
                               __uint_as_float(w[1] << 16), __uint_as_float(w[1] & 0xFFFF0000u));
            d[1] = make_float4(__uint_as_float(w[2] << 16), __uint_as_float(w[2] & 0xFFFF0000u),
                               __uint_as_float(w[3] << 16), __uint_as_float(w[3] & 0xFFFF0000u));
          }
        }
      }
    }
  } else {
    for (int i = threadIdx.x; i < R * H; i += blockDim.x) {
      const int r = i / H, k = i - r * H;
      const long long off = (long long)r * h.hidden_stride + k;
      hs[i] = h.hidden_dtype == Q3S_DTYPE_F32
                  ? static_cast<const float*>(h.hidden)[off]
                  : __uint_as_float((uint32_t)static_cast<const uint16_t*>(h.hidden)[off] << 16);
    }
  }
  __syncthreads();
  const int lane = (int)lane_id();
  const int warps = blockDim.x >> 5;
  const long long nw = (long long)gridDim.x * warps;
  const int Q = H >> 3;  // 16-byte weight vectors per row
  for (long long v = (long long)blockIdx.x * warps + (threadIdx.x >> 5); v < h.vocab; v += nw) {
    const uint4* wrow = reinterpret_cast<const uint4*>(h.weight + v * H);
    float acc[MAX_WARPS];
#pragma unroll
    for (int r = 0; r < MAX_WARPS; ++r) acc[r] = 0.0f;
    // Four weight vectors per lane in flight, then their products in order.
    for (int q0 = lane; q0 < Q; q0 += 128) {
      uint4 w4[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        w4[u] = q0 + 32 * u < Q ? __ldg(wrow + q0 + 32 * u) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int q = q0 + 32 * u;
        if (q >= Q) break;
        const uint32_t ww[4] = {w4[u].x, w4[u].y, w4[u].z, w4[u].w};
        float wv[8];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          wv[2 * t] = __uint_as_float(ww[t] << 16);
          wv[2 * t + 1] = __uint_as_float(ww[t] & 0xFFFF0000u);
        }
#pragma unroll
        for (int r = 0; r < MAX_WARPS; ++r) {
          if (r < R) {
            const float4 h0 = *reinterpret_cast<const float4*>(hs + r * H + 8 * q);
            const float4 h1 = *reinterpret_cast<const float4*>(hs + r * H + 8 * q + 4);
            float s2 = acc[r];
            s2 = __fadd_rn(s2, __fmul_rn(wv[0], h0.x));
            s2 = __fadd_rn(s2, __fmul_rn(wv[1], h0.y));
            s2 = __fadd_rn(s2, __fmul_rn(wv[2], h0.z));
            s2 = __fadd_rn(s2, __fmul_rn(wv[3], h0.w));
            s2 = __fadd_rn(s2, __fmul_rn(wv[4], h1.x));
            s2 = __fadd_rn(s2, __fmul_rn(wv[5], h1.y));
            s2 = __fadd_rn(s2, __fmul_rn(wv[6], h1.z));
            s2 = __fadd_rn(s2, __fmul_rn(wv[7], h1.w));
            acc[r] = s2;
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < MAX_WARPS; ++r) {
      if (r < R) {
        float x = acc[r];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) x = __fadd_rn(x, __shfl_xor_sync(FULL, x, o));
        if (lane == r) h.logits[(long long)r * h.vocab + v] = x;
      }
    }
  }
  // Completion: every block publishes its slice, the last one samples.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(h.counter, 1u);
    last_block = prev == gridDim.x - 1u;
    if (last_block) {
      __threadfence();       // the other blocks' logits are visible from here on
      *h.counter = 0u;       // ready for the next launch on this stream
    }
  }
  __syncthreads();
  if (!last_block) return;
  // The sampling block reads the logits with bulk copies (the async proxy).
  asm volatile("fence.proxy.async.global;" ::: "memory");
  __syncthreads();
  sample_block<Q3S_DTYPE_F32, NJ, false, false>(a, smem, 0, 1);
}

// Greedy argmax rows (sampling.rs:40-60 and :72-117), one warp per row.
template <int DT>
__global__ void greedy_kernel(const void* logits, long long num_rows, long long row_stride,
                              int n, long long sf, long long allow, int mode, uint32_t* tokens,
                              uint8_t* status) {
  const unsigned lane = lane_id();
  const long long warps = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long row = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < num_rows;
       row += warps) {
    const void* base = logits;
    const long long off = row * row_stride;
    // Keys: IEEE order with -0 == +0 in the high word, lowest index wins ties.
    unsigned long long best = 0ull;
    if (mode == Q3S_GREEDY_ON_DEVICE)
      best = ((unsigned long long)total_key(-3.40282347e38f) << 32) | (0xFFFFFFFFu - (uint32_t)n);
    const bool suppress = sf >= 0 && (mode == Q3S_GREEDY_SELECT || sf < n);
    for (int i = lane; i < n; i += 32) {
      float v = load_elem<DT>(base, off + i);
      bool ok = is_finite(v) &&
                (!suppress || i < sf ||
                 (allow >= 0 && i == allow && (mode == Q3S_GREEDY_SELECT || allow < n)));
      if (mode == Q3S_GREEDY_ON_DEVICE) {
        if (!ok) v = neg_inf();
        ok = true;
      }
      if (ok) {
        if (v == 0.0f) v = 0.0f;
        const unsigned long long c =
            ((unsigned long long)total_key(v) << 32) | (0xFFFFFFFFu - (uint32_t)i);
        best = c > best ? c : best;
      }
    }
    best = warp_max_u64(best);
    if (lane == 0) {
      if (best == 0ull) {
        tokens[row] = 0u;
        status[row] = Q3S_STATUS_SUPPRESSION_NO_CANDIDATE;
      } else {
        tokens[row] = 0xFFFFFFFFu - (uint32_t)best;
        status[row] = Q3S_STATUS_OK;
      }
    }
  }
}

constexpr int MAX_DEVICES = 64;

// Raises a kernel's dynamic shared-memory limit on the current device to at
// least `smem`, once per (kernel, device, size): the attribute call is not
// repeated on every launch.
template <typename K>
cudaError_t ensure_smem(K kernel, std::atomic<int>* set, size_t smem) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::atomic<int>* slot = (dev >= 0 && dev < MAX_DEVICES) ? &set[dev] : nullptr;
  if (slot && slot->load(std::memory_order_relaxed) >= (int)smem) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess && slot) {
    int cur = slot->load(std::memory_order_relaxed);
    while (cur < (int)smem && !slot->compare_exchange_weak(cur, (int)smem)) {
    }
  }
  return e;
}

template <int DT, int NJ, bool DBG, bool RT, bool CM = false>
cudaError_t launch_dbg(const KernelArgs& a, int grid, int warps, cudaStream_t stream) {
  static std::atomic<int> smem_set[MAX_DEVICES];
  const size_t smem = block_smem(a.vcap, Elem<DT>::BYTES, warps);
  cudaError_t e = ensure_smem(sample_kernel<DT, NJ, DBG, RT, CM>, smem_set, smem);
  if (e != cudaSuccess) return e;
  sample_kernel<DT, NJ, DBG, RT, CM><<<grid, warps * 32, smem, stream>>>(a);
  return cudaGetLastError();
}

// Launches with per-row vocabularies run the runtime-chunk kernel when the
// kernel's chunk holds two or more groups of 8 vectors (a shorter exact row
// is then possible); all other launches keep the fixed-chunk code.
// Committing launches (q3s_sample_commit) run their own instantiation,
// without debug outputs, fixed chunk or runtime chunk as for the others.
template <int DT, int NJ>
cudaError_t launch_t(const KernelArgs& a, int grid, int warps, cudaStream_t stream) {
  if (a.commit) {
    if constexpr (NJ >= 16) {
      if (a.row_vocab) return launch_dbg<DT, NJ, false, true, true>(a, grid, warps, stream);
    }
    return launch_dbg<DT, NJ, false, false, true>(a, grid, warps, stream);
  }
  const bool dbg = a.probs || a.masks || a.path_stats;
  if constexpr (NJ >= 16) {
    if (a.row_vocab)
      return dbg ? launch_dbg<DT, NJ, true, true>(a, grid, warps, stream)
                 : launch_dbg<DT, NJ, false, true>(a, grid, warps, stream);
  }
  return dbg ? launch_dbg<DT, NJ, true, false>(a, grid, warps, stream)
             : launch_dbg<DT, NJ, false, false>(a, grid, warps, stream);
}

}  // namespace

size_t sample_smem_per_warp(int vcap, int dtype) {
  (void)dtype;
  return warp_bytes(vcap);
}

size_t sample_scratch_per_warp(int vcap) { return gen_bytes(vcap); }

int sample_max_warps(int vcap, int dtype, size_t smem_limit) {
  const size_t fixed = block_smem(vcap, dtype == Q3S_DTYPE_F32 ? 4 : 2, 0);
  if (smem_limit <= fixed) return 0;
  int w = (int)((smem_limit - fixed) / warp_bytes(vcap));
  return w > MAX_WARPS ? MAX_WARPS : w;
}

cudaError_t launch_sample(const KernelArgs& a, int grid, int warps, cudaStream_t stream) {
  // NJ: the lane chunk of the fast-path scan for the row capacity.
  if (a.dtype == Q3S_DTYPE_F32) {
    switch (chunk_vectors(a.vcap, 4)) {
      case 8: return launch_t<Q3S_DTYPE_F32, 8>(a, grid, warps, stream);
      case 16: return launch_t<Q3S_DTYPE_F32, 16>(a, grid, warps, stream);
      case 24: return launch_t<Q3S_DTYPE_F32, 24>(a, grid, warps, stream);
      default: return launch_t<Q3S_DTYPE_F32, 32>(a, grid, warps, stream);
    }
  }
  if (chunk_vectors(a.vcap, 2) == 8) return launch_t<Q3S_DTYPE_BF16, 8>(a, grid, warps, stream);
  return launch_t<Q3S_DTYPE_BF16, 16>(a, grid, warps, stream);
}

size_t head_smem(int vcap) { return block_smem(vcap, 4, MAX_WARPS); }

cudaError_t launch_head_sample(const HeadArgs& h, const KernelArgs& a, int grid,
                               cudaStream_t stream) {
  const size_t smem = block_smem(a.vcap, 4, MAX_WARPS);
  static std::atomic<int> smem_set[4][MAX_DEVICES];
  cudaError_t e;
  switch (chunk_vectors(a.vcap, 4)) {
    case 8:
      if ((e = ensure_smem(head_sample_kernel<8>, smem_set[0], smem)) != cudaSuccess) return e;
      head_sample_kernel<8><<<grid, MAX_WARPS * 32, smem, stream>>>(h, a);
      break;
    case 16:
      if ((e = ensure_smem(head_sample_kernel<16>, smem_set[1], smem)) != cudaSuccess) return e;
      head_sample_kernel<16><<<grid, MAX_WARPS * 32, smem, stream>>>(h, a);
      break;
    case 24:
      if ((e = ensure_smem(head_sample_kernel<24>, smem_set[2], smem)) != cudaSuccess) return e;
      head_sample_kernel<24><<<grid, MAX_WARPS * 32, smem, stream>>>(h, a);
      break;
    default:
      if ((e = ensure_smem(head_sample_kernel<32>, smem_set[3], smem)) != cudaSuccess) return e;
      head_sample_kernel<32><<<grid, MAX_WARPS * 32, smem, stream>>>(h, a);
      break;
  }
  return cudaGetLastError();
}

cudaError_t launch_greedy(const void* logits, int dtype, long long num_rows, long long row_stride,
                          int n, long long sf, long long allow, int mode, uint32_t* tokens,
                          uint8_t* status, int grid, cudaStream_t stream) {
  if (dtype == Q3S_DTYPE_F32)
    greedy_kernel<Q3S_DTYPE_F32>
        <<<grid, 256, 0, stream>>>(logits, num_rows, row_stride, n, sf, allow, mode, tokens, status);
  else
    greedy_kernel<Q3S_DTYPE_BF16>
        <<<grid, 256, 0, stream>>>(logits, num_rows, row_stride, n, sf, allow, mode, tokens, status);
  return cudaGetLastError();
}

}  // namespace q3s
