// Fused per-step sampling kernel for the Qwen3-TTS talker / code predictor.
//
// One warp samples one row: repetition penalty over the row's history
// (sampling.rs:592-606, 732-773), suppression / non-finite mask (:608-616),
// temperature as a reciprocal multiply (:628-631), top-k keeping every tie of
// the k-th value (:633-663), top-p over the full-vocabulary softmax (:665-698)
// and the vocabulary-order multinomial draw with Philox4x32-10 (:700-729,
// :337-375).  Greedy rows take the total_cmp argmax of the raw logits
// (:574-591).
//
// Exactness: every f32 operation of the reference is performed with the same
// rounding, and every f32 running sum the reference accumulates sequentially
// (the top-p denominator, the nucleus cumulative, the final softmax sum and
// the draw's cumulative) is accumulated sequentially here too, over the same
// non-zero terms in the same order.  Terms the reference adds that are exact
// zeros (exp(-inf)) are skipped, which leaves an f32 sum unchanged.  The
// parallel parts (max, counts, selection, sorting) are order-free.
//
// Data movement: a persistent grid of warps strides over rows.  Each warp
// owns one shared-memory stage; its next row is fetched by a bulk copy (TMA,
// cp.async.bulk, no multicast) that completes on the warp's mbarrier while the
// warp finishes the current row.  The row is read from the stage once in the
// common case (the "fast path"):
//   1. one scan of the stage computes every 16-byte vector's maximum (kept in
//      registers) and the row maximum;
//   2. a threshold tau is chosen on the vector maxima so that at least k
//      vectors (hence at least k elements) reach it: the candidates
//      {x >= tau} then contain the whole top-k set, ties included;
//   3. only the vectors whose maximum reaches tau are re-read to collect the
//      candidates (a few hundred of the row's thousands of elements); the
//      stage is then released to the next row's copy;
//   4. the exact k-th largest candidate is found by radix selection, the
//      survivors are put in vocabulary order through a bitmap, and the
//      softmax / top-p / draw run on that short list.
// Rows outside the fast path (top_k off or above 256, a temperature whose
// reciprocal is 0 or infinite, a candidate overflow) run the same algorithm
// on full-row lists kept in a per-warp global workspace ("general path").

#include <cstdint>

#include "../../include/q3s_sampler.h"
#include "q3s_device.cuh"
#include "q3s_kernels.h"

namespace q3s {
namespace {

constexpr int MAX_WARPS = 10;
constexpr int SEG = 24;         // candidate slots per lane (interleaved: slot t of lane l at t*32+l)
constexpr int CAP = 32 * SEG;   // fast-path candidate capacity per warp
constexpr int LCAP = 512;       // fast-path survivor-list capacity per warp
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

__host__ __device__ inline size_t stage_bytes(int vcap, int es) {
  return align16((size_t)vcap * es + 16);
}

// Per-warp shared memory of the fast path.
struct FastSpace {
  unsigned char* stage;        // raw row, TMA destination
  uint2* cand;                 // [CAP] (x bits, index); the nucleus sort aliases it
  float* B;                    // [LCAP] softmax numerators of the survivor list
  float* BX;                   // [LCAP] x of the survivor list
  uint16_t* BI;                // [LCAP] vocabulary index of the survivor list
  uint32_t* bm;                // [vcap/32] history bitmap, then survivor bitmap
  uint16_t* wpre;              // [vcap/32] survivors before each bitmap word
  uint32_t* hist;              // [256]
  uint64_t* mbar;              // stage barrier
  uint32_t* counter;           // candidate slot counter
};

__host__ __device__ inline size_t fast_bytes(int vcap, int es) {
  return stage_bytes(vcap, es) + 8u * CAP + 4u * LCAP * 2 + align16(2u * LCAP) +
         align16(4u * (vcap / 32)) + align16(2u * (vcap / 32)) + 4u * 256 + 16u;
}

__device__ inline FastSpace carve_fast(unsigned char* base, int vcap, int es) {
  FastSpace f;
  size_t o = 0;
  f.stage = base;
  o += stage_bytes(vcap, es);
  f.cand = reinterpret_cast<uint2*>(base + o);
  o += 8u * CAP;
  f.B = reinterpret_cast<float*>(base + o);
  o += 4u * LCAP;
  f.BX = reinterpret_cast<float*>(base + o);
  o += 4u * LCAP;
  f.BI = reinterpret_cast<uint16_t*>(base + o);
  o += align16(2u * LCAP);
  f.bm = reinterpret_cast<uint32_t*>(base + o);
  o += align16(4u * (vcap / 32));
  f.wpre = reinterpret_cast<uint16_t*>(base + o);
  o += align16(2u * (vcap / 32));
  f.hist = reinterpret_cast<uint32_t*>(base + o);
  o += 4u * 256;
  f.mbar = reinterpret_cast<uint64_t*>(base + o);
  f.counter = reinterpret_cast<uint32_t*>(base + o + 8);
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

// Where row r's elements sit in the stage: element i at byte mis*es + i*es.
struct StageView {
  int n;    // elements
  int mis;  // leading misalignment in elements
  int Q;    // 16-byte vectors covering the row
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
__device__ void issue_row(const KernelArgs& a, long long row, const FastSpace& f) {
  constexpr int es = Elem<DT>::BYTES;
  const int n = row_vocab(a, row);
  uint32_t bytes = 0;
  RowGeom g;
  if (row_fits(a, n)) {
    g = row_geom(a, row, n, es);
    bytes = g.tail_begin - g.head_end;
  }
  mbar_arrive_expect_tx(f.mbar, bytes);
  if (bytes > 0) bulk_copy_g2s(f.stage + g.mis_bytes + g.head_end, g.p0 + g.head_end, bytes, f.mbar);
}

// After the barrier completes: the lanes copy the unaligned head and tail.
template <int DT>
__device__ StageView complete_stage(const KernelArgs& a, long long row, int n, const FastSpace& f) {
  constexpr int es = Elem<DT>::BYTES;
  const RowGeom g = row_geom(a, row, n, es);
  const unsigned lane = lane_id();
  const int hn = (int)(g.head_end / es);
  const int t0 = (int)(g.tail_begin / es);
  for (int i = lane; i < hn; i += 32) {
    if (es == 4)
      reinterpret_cast<float*>(f.stage + g.mis_bytes)[i] = __ldg(reinterpret_cast<const float*>(g.p0) + i);
    else
      reinterpret_cast<unsigned short*>(f.stage + g.mis_bytes)[i] =
          __ldg(reinterpret_cast<const unsigned short*>(g.p0) + i);
  }
  for (int i = t0 + lane; i < n; i += 32) {
    if (es == 4)
      reinterpret_cast<float*>(f.stage + g.mis_bytes)[i] = __ldg(reinterpret_cast<const float*>(g.p0) + i);
    else
      reinterpret_cast<unsigned short*>(f.stage + g.mis_bytes)[i] =
          __ldg(reinterpret_cast<const unsigned short*>(g.p0) + i);
  }
  __syncwarp();
  StageView v;
  v.n = n;
  v.mis = (int)(g.mis_bytes / es);
  v.Q = (int)((g.mis_bytes + g.bytes + 15u) / 16u);
  return v;
}

template <int DT>
__device__ __forceinline__ void unpack(const unsigned char* stage, int q, float (&e)[Elem<DT>::EPV]) {
  const uint4 v = *reinterpret_cast<const uint4*>(stage + 16 * q);
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
__device__ __forceinline__ float stage_elem(const unsigned char* stage, int mis, int i) {
  if (DT == Q3S_DTYPE_F32) return reinterpret_cast<const float*>(stage)[mis + i];
  return __uint_as_float(((uint32_t) reinterpret_cast<const unsigned short*>(stage)[mis + i]) << 16);
}

// Everything the kernel reads about a row besides its logits.
struct RowMeta {
  q3s_row_params P;
  int n;
  long long h0, h1;  // history range
  unsigned long long seed, subseq;
  float uo;  // uniform override
};

__device__ __forceinline__ RowMeta load_meta(const KernelArgs& a, long long row) {
  RowMeta m;
  m.n = row_vocab(a, row);
  m.P = a.params[row * a.params_stride];
  m.h0 = m.h1 = 0;
  if (a.history_offsets) {
    m.h0 = a.history_offsets[row];
    m.h1 = a.history_offsets[row + 1];
  }
  m.seed = a.seeds ? a.seeds[row] : 0ull;
  m.subseq = a.subseqs ? a.subseqs[row] : 0ull;
  m.uo = a.uniform_override ? a.uniform_override[row] : 0.0f;
  return m;
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

// Per-row transform inputs.
struct RowCtx {
  int n, mis, Q;
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

// Ascending bitonic sort of 256 keys held 8 per lane (element lane*8 + r).
__device__ inline void bitonic_sort_256(unsigned long long (&v)[8]) {
  const unsigned lane = lane_id();
#pragma unroll
  for (int size = 2; size <= 256; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (stride >= 8) {
        const int ls = stride >> 3;
        const bool lower = (lane & ls) == 0;
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const bool up = (((int)lane * 8 + r) & size) == 0;
          const unsigned long long o = __shfl_xor_sync(FULL, v[r], ls);
          const bool keep_min = (lower == up);
          v[r] = keep_min ? (o < v[r] ? o : v[r]) : (o > v[r] ? o : v[r]);
        }
      } else {
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          if ((r & stride) == 0) {
            const bool up = (((int)lane * 8 + r) & size) == 0;
            const unsigned long long a = v[r], b = v[r + stride];
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

// Sequential f32 sum of B[0..count) by lane 0, in order; when `prefix` is set
// B[j] is replaced by the running sum.  Result broadcast to every lane.
// B is 16-byte aligned; four terms are loaded at a time, added in order.
__device__ inline float chain_sum(float* B, int count, bool prefix) {
  float c = 0.0f;
  if (lane_id() == 0) {
    float4* B4 = reinterpret_cast<float4*>(B);
    const int n4 = count >> 2;
    if (prefix) {
      for (int q = 0; q < n4; ++q) {
        float4 v = B4[q];
        c = __fadd_rn(c, v.x);
        v.x = c;
        c = __fadd_rn(c, v.y);
        v.y = c;
        c = __fadd_rn(c, v.z);
        v.z = c;
        c = __fadd_rn(c, v.w);
        v.w = c;
        B4[q] = v;
      }
      for (int j = n4 << 2; j < count; ++j) {
        c = __fadd_rn(c, B[j]);
        B[j] = c;
      }
    } else {
      for (int q = 0; q < n4; ++q) {
        const float4 v = B4[q];
        c = __fadd_rn(c, v.x);
        c = __fadd_rn(c, v.y);
        c = __fadd_rn(c, v.z);
        c = __fadd_rn(c, v.w);
      }
      for (int j = n4 << 2; j < count; ++j) c = __fadd_rn(c, B[j]);
    }
  }
  __syncwarp();
  return __shfl_sync(FULL, c, 0);
}

__device__ __forceinline__ unsigned long long nucleus_key(float p, uint16_t idx) {
  return ((unsigned long long)(~__float_as_uint(p)) << 32) | idx;
}

// Debug outputs of one row (probs and masks), NULL when not requested.
struct DebugRow {
  unsigned char* masks;
  float* probs;
};

// Top-p over a survivor list in vocabulary order (sampling.rs:665-698): the
// full-vocabulary softmax denominator, the max - 16 cutoff and the nucleus
// walked in (p desc, index asc) order.  On return the list holds the nucleus
// (in vocabulary order, B = exp(x - m2)), *ns_io its length, *m2_out its max.
// Kept out of line: only rows with top_p < 1 execute it.
__device__ __noinline__ int apply_top_p(float* B, float* BX, uint16_t* BI, int* ns_io, float m1,
                                        double top_p_d, unsigned long long* keys, uint32_t* hist,
                                        float* m2_out) {
  const unsigned lane = lane_id();
  const int ns = *ns_io;
  // Denominator: sequential f32 sum in vocabulary order.
  const float total = chain_sum(B, ns, false);
  if (!is_finite(total) || total <= 0.0f) return Q3S_STATUS_INVALID_DENOMINATOR;
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
  // Walk the probabilities in (p desc, index asc) order, 256 at a time; the
  // first position > 0 whose preceding cumulative reaches top_p starts the
  // masked tail.
  const float top_p = (float)top_p_d;
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
  if (!(m2 > neg_inf())) return Q3S_STATUS_NO_CANDIDATE;
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
  *ns_io = ns2;
  *m2_out = m2;
  return Q3S_STATUS_OK;
}

// Top-p, final softmax and draw over a survivor list in vocabulary order:
// B[j] = exp(x_j - m1), BX[j] = x_j, BI[j] = index, m1 = max x (sampling.rs:665-729).
__device__ RowOut finish_list(float* B, float* BX, uint16_t* BI, int ns, float m1,
                              const q3s_row_params& P, unsigned long long* keys, uint32_t* hist,
                              float u, int n, const DebugRow& dbg) {
  const unsigned lane = lane_id();
  float m2 = m1;
  if (P.top_p < 1.0) {
    const int st = apply_top_p(B, BX, BI, &ns, m1, P.top_p, keys, hist, &m2);
    if (st != Q3S_STATUS_OK) return {st, 0u};
  }

  // Final softmax sum and the draw (sampling.rs:700-729).
  const float sum = chain_sum(B, ns, true);
  if (!is_finite(sum) || sum <= 0.0f) return {Q3S_STATUS_INVALID_DENOMINATOR, 0u};
  const float thr = __fmul_rn(u, sum);
  int first = ns;
  for (int j = lane; j < ns; j += 32) {
    if (B[j] >= thr) {
      first = j;
      break;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) first = min(first, __shfl_xor_sync(FULL, first, o));
  const uint32_t token = first < ns ? (uint32_t)BI[first] : (uint32_t)(n - 1);
  if (dbg.masks || dbg.probs) {
    for (int j = lane; j < ns; j += 32) {
      const int i = BI[j];
      if (dbg.masks) dbg.masks[i] |= 4;
      if (dbg.probs) {
        const float e = cr_expf(__fsub_rn(BX[j], m2));
        dbg.probs[i] = __double2float_rn((double)e / (double)sum);
      }
    }
  }
  __syncwarp();
  return {Q3S_STATUS_OK, token};
}

// ---------------------------------------------------------------------------
// Row handlers.  Each releases the stage (`release`) exactly once, as soon as
// it no longer reads it.
// ---------------------------------------------------------------------------
struct Releaser {
  const KernelArgs* a;
  const FastSpace* f;
  long long next;
  bool done;
};

template <int DT>
__device__ __forceinline__ void release(Releaser& r) {
  if (r.done) return;
  r.done = true;
  __syncwarp();
  if (lane_id() == 0) {
    fence_proxy_async_smem();
    if (r.next < r.a->num_rows) issue_row<DT>(*r.a, r.next, *r.f);
  }
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

// General path: the full row as f32 in the global workspace, then full-row
// passes (any top_k, any temperature).
template <int DT>
__device__ __noinline__ RowOut general_row(const FastSpace& f, const GenSpace& g, const StageView& s,
                              const q3s_row_params& P, const RowCtx& rc, float u, Releaser& rel,
                              const DebugRow& dbg) {
  const unsigned lane = lane_id();
  const int n = s.n;
  float* A = g.A;
  for (int i = lane; i < n; i += 32) A[i] = stage_elem<DT>(f.stage, s.mis, i);
  __syncwarp();
  release<DT>(rel);
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
    if (dbg.masks && is_finite(x)) dbg.masks[i] = 1;
  }
  mx = warp_max(mx);
  nfin = __reduce_add_sync(FULL, nfin);
  nan_seen = __any_sync(FULL, nan_seen);
  __syncwarp();
  if (nfin == 0)
    return {rc.sf >= 0 ? Q3S_STATUS_SUPPRESSION_NO_CANDIDATE : Q3S_STATUS_NO_CANDIDATE, 0u};
  // A NaN or +inf after the temperature survives top-k and top-p and makes
  // the softmax denominator non-finite (sampling.rs:675-678, 715-718).
  if (nan_seen || mx == __int_as_float(0x7f800000)) return {Q3S_STATUS_INVALID_DENOMINATOR, 0u};
  // Top-k threshold: the k-th largest finite value (sampling.rs:654-663).
  float t = neg_inf();
  if (P.top_k > 0u && (uint32_t)nfin > P.top_k) {
    const uint32_t key = warp_select<uint32_t>(
        n, P.top_k,
        [&](int i, uint32_t& k) {
          const float x = A[i];
          k = ~total_key(x);
          return x > neg_inf();
        },
        f.hist, 24);
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
      g.BI[j] = (uint16_t)i;
      g.BX[j] = x;
      g.B[j] = cr_expf(__fsub_rn(x, mx));
      if (dbg.masks) dbg.masks[i] |= 2;
    }
    ns += __popc(b);
  }
  __syncwarp();
  return finish_list(g.B, g.BX, g.BI, ns, mx, P, reinterpret_cast<unsigned long long*>(f.cand),
                     f.hist, u, n, dbg);
}

// Vector maxima of the stage (registers) and the row maximum.
template <int DT, int NJ, bool XF, bool EDGE>
__device__ __forceinline__ float scan_stage(const FastSpace& f, const RowCtx& r, float (&vm)[NJ]) {
  constexpr int EPV = Elem<DT>::EPV;
  const int lane = (int)lane_id();
  float mx = neg_inf();
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const int q = lane + 32 * j;
    float m = neg_inf();
    if (q < r.Q) {
      float e[EPV];
      unpack<DT>(f.stage, q, e);
#pragma unroll
      for (int c = 0; c < EPV; ++c) m = fmaxf(m, xform<XF, EDGE>(e[c], q * EPV + c - r.mis, r));
    }
    vm[j] = m;
    mx = fmaxf(mx, m);
  }
  return warp_max(mx);
}

template <int NJ>
__device__ __forceinline__ int count_ge(const float (&vm)[NJ], float tau) {
  int c = 0;
#pragma unroll
  for (int j = 0; j < NJ; ++j) c += vm[j] >= tau ? 1 : 0;
  return (int)__reduce_add_sync(FULL, (unsigned)c);
}

// Candidates {x >= tau} of the flagged vectors, each lane into its own slots
// of f.cand (slot t of lane l at t*32 + l: conflict-free), as (x after the
// temperature, index).  Returns this lane's count (above SEG: overflow).
template <int DT, int NJ, bool XF, bool EDGE>
__device__ int collect(const FastSpace& f, const RowCtx& r, const float (&vm)[NJ], float tau) {
  constexpr int EPV = Elem<DT>::EPV;
  const int lane = (int)lane_id();
  uint64_t flags = 0;
#pragma unroll
  for (int j = 0; j < NJ; ++j) flags |= (vm[j] >= tau ? 1ull : 0ull) << j;
  int cnt = 0;
  while (flags) {
    const int j = __ffsll((long long)flags) - 1;
    flags &= flags - 1;
    const int q = lane + 32 * j;
    float e[EPV];
    unpack<DT>(f.stage, q, e);
#pragma unroll
    for (int c = 0; c < EPV; ++c) {
      const float x = xform<XF, EDGE>(e[c], q * EPV + c - r.mis, r);
      if (x >= tau) {
        if (cnt < SEG) {
          const float xv = XF ? x : __fmul_rn(x, r.inv);
          f.cand[cnt * 32 + lane] = make_uint2(__float_as_uint(xv), (uint32_t)(q * EPV + c - r.mis));
        }
        ++cnt;
      }
    }
  }
  __syncwarp();
  return cnt;
}

// Exact k-th largest x among the candidates (each lane holds `mine` of
// them).  Bins of equal width over the current value range, counted from the
// top; the range narrows to the bin that holds the k-th value until that bin
// holds one value (or one distinct value).  The bin function
// floor((x - lo) * scale) is monotone in x, so the bins partition the
// candidates in value order.
__device__ float select_kth_candidate(const FastSpace& f, int mine, int k) {
  const unsigned lane = lane_id();
  float lo = __int_as_float(0x7f800000), hi = neg_inf();
  for (int t = 0; t < mine; ++t) {
    const float x = __uint_as_float(f.cand[t * 32 + lane].x);
    lo = fminf(lo, x);
    hi = fmaxf(hi, x);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = fminf(lo, __shfl_xor_sync(FULL, lo, o));
    hi = fmaxf(hi, __shfl_xor_sync(FULL, hi, o));
  }
  uint32_t kk = (uint32_t)k;
#pragma unroll 1
  for (int pass = 0; pass < 8; ++pass) {
    if (!(hi > lo)) return hi;  // one distinct value left
    const float width = __fsub_rn(hi, lo);
    if (!(width < __int_as_float(0x7f800000))) break;  // range too wide: key radix below
    const float scale = __fdiv_rn(63.5f, width);
    // 64 bins, counted in f.hist.
    f.hist[lane] = 0u;
    f.hist[lane + 32] = 0u;
    __syncwarp();
    for (int t = 0; t < mine; ++t) {
      const float x = __uint_as_float(f.cand[t * 32 + lane].x);
      if (x >= lo && x <= hi) {
        const int b = min(63, (int)__fmul_rn(__fsub_rn(x, lo), scale));
        atomicAdd(&f.hist[b], 1u);
      }
    }
    __syncwarp();
    // Lane l owns bins 63-2l and 62-2l (counted from the top).
    const uint32_t c0 = f.hist[63 - 2 * lane], c1 = f.hist[62 - 2 * lane];
    const uint32_t s = c0 + c1;
    const uint32_t incl = warp_inclusive_scan(s);
    const unsigned ball = __ballot_sync(FULL, incl >= kk);
    const int src = ball ? __ffs(ball) - 1 : 31;
    int bin = 0;
    uint32_t before = 0, inbin = 0;
    if ((int)lane == src) {
      const uint32_t acc = incl - s;
      if (acc + c0 >= kk) {
        bin = 63 - 2 * lane;
        before = acc;
        inbin = c0;
      } else {
        bin = 62 - 2 * lane;
        before = acc + c0;
        inbin = c1;
      }
    }
    bin = __shfl_sync(FULL, bin, src);
    before = __shfl_sync(FULL, before, src);
    inbin = __shfl_sync(FULL, inbin, src);
    kk -= before;
    // Value range of the chosen bin.
    float nlo = __int_as_float(0x7f800000), nhi = neg_inf();
    for (int t = 0; t < mine; ++t) {
      const float x = __uint_as_float(f.cand[t * 32 + lane].x);
      if (x >= lo && x <= hi && min(63, (int)__fmul_rn(__fsub_rn(x, lo), scale)) == bin) {
        nlo = fminf(nlo, x);
        nhi = fmaxf(nhi, x);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      nlo = fminf(nlo, __shfl_xor_sync(FULL, nlo, o));
      nhi = fmaxf(nhi, __shfl_xor_sync(FULL, nhi, o));
    }
    lo = nlo;
    hi = nhi;
    if (inbin == 1u) return hi;
    __syncwarp();
  }
  // Fallback: radix selection on total-order keys below the current range.
  const uint32_t kmax = total_key(hi);
  const uint32_t kspan = kmax - total_key(lo);
  const int bits = 32 - __clz(kspan | 1u);
  const int top = ((bits + 7) / 8) * 8 - 8;
  const float flo = lo, fhi = hi;
  // warp_select visits slot j = t*32 + lane from lane `lane`: its own slots.
  const uint32_t rel_k = warp_select<uint32_t>(
      32 * SEG, kk,
      [&](int j, uint32_t& key) {
        const float x = __uint_as_float(f.cand[j].x);
        key = kmax - total_key(x);
        return (j >> 5) < mine && x >= flo && x <= fhi;
      },
      f.hist, top);
  return from_total_key(kmax - rel_k);
}

// Debug pass over the stage: bit0 finite x, bit1 x >= t.
template <int DT, bool XF>
__device__ void debug_masks(const FastSpace& f, const RowCtx& r, float t, unsigned char* masks) {
  const unsigned lane = lane_id();
  for (int i = lane; i < r.n; i += 32) {
    float x = xform<XF, false>(stage_elem<DT>(f.stage, r.mis, i), i, r);
    if (!XF) x = is_finite(x) ? __fmul_rn(x, r.inv) : neg_inf();
    unsigned char m = 0;
    if (is_finite(x)) m = 1;
    if (is_finite(x) && x >= t) m |= 2;
    masks[i] = m;
  }
  __syncwarp();
}

// Fast path; returns false (before releasing the stage) when the row must
// take the general path instead.
template <int DT, int NJ, bool XF, bool EDGE>
__device__ bool fast_row(const FastSpace& f, const StageView& s, const q3s_row_params& P,
                         const RowCtx& rc, float u, Releaser& rel, const DebugRow& dbg,
                         float& delta, RowOut& out) {
  const unsigned lane = lane_id();
  const int n = s.n;
  float vm[NJ];
  const float mx = scan_stage<DT, NJ, XF, EDGE>(f, rc, vm);
  // Row maximum in the x domain.
  if (!XF && mx == __int_as_float(0x7f800000)) return false;  // raw +inf: general path
  if (mx == neg_inf() || mx != mx) {
    release<DT>(rel);
    out = {rc.sf >= 0 ? Q3S_STATUS_SUPPRESSION_NO_CANDIDATE : Q3S_STATUS_NO_CANDIDATE, 0u};
    return true;
  }
  const float Mx = XF ? mx : __fmul_rn(mx, rc.inv);
  if (Mx == __int_as_float(0x7f800000)) {
    release<DT>(rel);
    out = {Q3S_STATUS_INVALID_DENOMINATOR, 0u};
    return true;
  }
  // Threshold on the vector maxima: count in [k, hi].
  const int k = (int)P.top_k;
  const int hi = k <= 128 ? max(2 * k, 64) : k + 96;
  float vmin = __int_as_float(0x7f800000);
#pragma unroll
  for (int j = 0; j < NJ; ++j)
    if (vm[j] > neg_inf()) vmin = fminf(vmin, vm[j]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) vmin = fminf(vmin, __shfl_xor_sync(FULL, vmin, o));
  const float span = __fsub_rn(mx, vmin);
  if (!(span < __int_as_float(0x7f800000))) return false;
  if (count_ge(vm, vmin) < k) return false;  // fewer than k finite vectors
  float lo = 0.0f, hiD = span;
  bool hi_known = false;
  float d = (delta > 0.0f && delta <= span) ? delta : span * 0.25f;
  float best = span;  // smallest distance seen whose count reaches k
  bool accepted = false;
#pragma unroll 1
  for (int it = 0; it < 24; ++it) {
    const int c = count_ge(vm, __fsub_rn(mx, d));
    if (c >= k) best = fminf(best, d);
    if (c < k) {
      lo = d;
      d = hi_known ? 0.5f * (lo + hiD) : fminf(span, d > 0.0f ? 2.0f * d : span * 0.0625f);
    } else if (c > hi) {
      hiD = d;
      hi_known = true;
      d = 0.5f * (lo + hiD);
    } else {
      accepted = true;
      break;
    }
    if (hiD - lo <= 0.0f) break;
  }
  if (!accepted) d = best;
  float tau = __fsub_rn(mx, d);
  // Raw-domain selection: lower tau until its image lies strictly below the
  // image of every value that reaches the chosen count, so no element with
  // v < tau can tie the k-th largest x after the multiply.
  if (!XF && rc.inv != 1.0f) {
    const float img = __fmul_rn(tau, rc.inv);
    float t2 = tau;
    bool ok = false;
#pragma unroll 1
    for (int it = 0; it < 8 && !ok; ++it) {
      t2 = __fsub_rn(t2, fmaxf(fabsf(t2) * 3.814697265625e-06f, 1.1754944e-38f));
      ok = __fmul_rn(t2, rc.inv) < img;
    }
    if (!ok) return false;
    tau = t2;
  }
  const int mine = collect<DT, NJ, XF, EDGE>(f, rc, vm, tau);
  const bool overflow = __any_sync(FULL, mine > SEG);
  const int c = (int)__reduce_add_sync(FULL, (unsigned)mine);
  // The survivors (at most c) must fit the list; decided before release.
  if (overflow || c < k || c > LCAP) return false;
  delta = d;
  if (!dbg.masks) release<DT>(rel);

  // Exact k-th largest candidate.
  const float t = select_kth_candidate(f, mine, k);
  // The debug masks recompute x with the history bitmap, which the survivor
  // bitmap below overwrites.
  if (dbg.masks) debug_masks<DT, XF>(f, rc, t, dbg.masks);
  // Survivors x >= t, in vocabulary order through a bitmap.
  const int words = (n + 31) >> 5;
  for (int w = lane; w < words; w += 32) f.bm[w] = 0u;
  __syncwarp();
  for (int s = 0; s < mine; ++s) {
    const uint2 e = f.cand[s * 32 + lane];
    if (__uint_as_float(e.x) >= t) atomicOr(&f.bm[e.y >> 5], 1u << (e.y & 31));
  }
  __syncwarp();
  const int per = (words + 31) >> 5;
  const int w0 = min(words, (int)lane * per), w1 = min(words, w0 + per);
  int own = 0;
  for (int w = w0; w < w1; ++w) own += __popc(f.bm[w]);
  const int incl = (int)warp_inclusive_scan((uint32_t)own);
  int run = incl - own;
  for (int w = w0; w < w1; ++w) {
    f.wpre[w] = (uint16_t)run;
    run += __popc(f.bm[w]);
  }
  const int ns = __shfl_sync(FULL, incl, 31);
  __syncwarp();
  for (int s = 0; s < mine; ++s) {
    const uint2 e = f.cand[s * 32 + lane];
    const float x = __uint_as_float(e.x);
    if (x >= t) {
      const uint32_t w = e.y >> 5, b = e.y & 31;
      const int p = f.wpre[w] + __popc(f.bm[w] & ((1u << b) - 1u));
      f.BI[p] = (uint16_t)e.y;
      f.BX[p] = x;
      f.B[p] = cr_expf(__fsub_rn(x, Mx));
    }
  }
  __syncwarp();
  out = finish_list(f.B, f.BX, f.BI, ns, Mx, P, reinterpret_cast<unsigned long long*>(f.cand),
                    f.hist, u, n, dbg);
  release<DT>(rel);
  return true;
}

template <int DT, int NJ>
__device__ RowOut sampled_row(const KernelArgs& a, const FastSpace& f, const GenSpace& g,
                              const RowMeta& m, const StageView& s, Releaser& rel, float& delta,
                              const DebugRow& dbg) {
  const q3s_row_params& P = m.P;
  RowCtx rc;
  rc.n = s.n;
  rc.mis = s.mis;
  rc.Q = s.Q;
  rc.inv = __fdiv_rn(1.0f, (float)P.temperature);
  rc.pf = (float)P.repetition_penalty;
  rc.sf = P.suppress_from;
  rc.allow = P.allow_token;
  rc.bm = f.bm;
  rc.use_pen = P.repetition_penalty != 1.0 && m.h1 > m.h0;
  const float u = a.uniform_override ? m.uo : philox_uniform(m.seed, m.subseq, P.ctr_lo);
  const bool inv_ok = rc.inv > 0.0f && rc.inv < __int_as_float(0x7f800000);
  const bool fast = inv_ok && P.top_k >= 1u && P.top_k <= (uint32_t)FAST_MAX_K &&
                    P.top_k < (uint32_t)s.n;
  if (fast) {
    const bool xf = rc.use_pen || rc.sf >= 0;
    const bool edge = s.mis != 0 || (s.n % Elem<DT>::EPV) != 0;
    RowOut out;
    bool done;
    if (xf)
      done = edge ? fast_row<DT, NJ, true, true>(f, s, P, rc, u, rel, dbg, delta, out)
                  : fast_row<DT, NJ, true, false>(f, s, P, rc, u, rel, dbg, delta, out);
    else
      done = edge ? fast_row<DT, NJ, false, true>(f, s, P, rc, u, rel, dbg, delta, out)
                  : fast_row<DT, NJ, false, false>(f, s, P, rc, u, rel, dbg, delta, out);
    if (done) return out;
  }
  return general_row<DT>(f, g, s, P, rc, u, rel, dbg);
}

template <int DT, int NJ>
__global__ void __launch_bounds__(MAX_WARPS * 32, 1) sample_kernel(const KernelArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int es = Elem<DT>::BYTES;
  const int warp = threadIdx.x >> 5;
  const int warps = blockDim.x >> 5;
  const unsigned lane = lane_id();
  const FastSpace f = carve_fast(smem + (size_t)warp * fast_bytes(a.vcap, es), a.vcap, es);
  const long long gw = (long long)blockIdx.x * warps + warp;
  const GenSpace g = carve_gen(a.scratch + (size_t)gw * gen_bytes(a.vcap), a.vcap);
  if (lane == 0) {
    mbar_init(f.mbar, 1);
    fence_mbarrier_init();
    fence_proxy_async_smem();
  }
  __syncwarp();
  const long long stride = (long long)gridDim.x * warps;
  long long row = gw;
  if (row < a.num_rows && lane == 0) issue_row<DT>(a, row, f);
  uint32_t phase = 0;
  float delta = 0.0f;
  // Per-row metadata is loaded one row ahead so its latency overlaps a row.
  RowMeta cur;
  if (row < a.num_rows) cur = load_meta(a, row);
  for (; row < a.num_rows; row += stride) {
    Releaser rel{&a, &f, row + stride, false};
    RowMeta nxt;
    if (row + stride < a.num_rows) nxt = load_meta(a, row + stride);
    const int n = cur.n;
    const q3s_row_params& P = cur.P;
    int st = row_fits(a, n) ? validate(P) : Q3S_STATUS_UNSUPPORTED;
    DebugRow dbg{nullptr, nullptr};
    if (a.masks && st == Q3S_STATUS_OK) dbg.masks = a.masks + row * a.probs_stride;
    if (a.probs && st == Q3S_STATUS_OK) dbg.probs = a.probs + row * a.probs_stride;
    if (dbg.masks)
      for (int i = lane; i < n; i += 32) dbg.masks[i] = 0;
    if (dbg.probs)
      for (int i = lane; i < n; i += 32) dbg.probs[i] = 0.0f;
    // History bitmap of a sampled row with a penalty (filled while the
    // stage copy is in flight).
    if (st == Q3S_STATUS_OK && P.do_sample && P.repetition_penalty != 1.0) {
      const long long h0 = cur.h0, h1 = cur.h1;
      if (h1 > h0) {
        const int words = (n + 31) >> 5;
        for (int w = lane; w < words; w += 32) f.bm[w] = 0u;
        __syncwarp();
        for (long long h = h0 + lane; h < h1; h += 32) {
          const int id = a.history[h];
          if (id < n) atomicOr(&f.bm[id >> 5], 1u << (id & 31));
        }
        __syncwarp();
      }
    }
    const bool ready = mbar_wait_bounded(f.mbar, phase, WAIT_LIMIT_NS);
    phase ^= 1u;
    if (!ready) {
      // The stage never arrived: mark this warp's remaining rows and stop
      // after giving the copy in flight another bounded wait.
      mbar_wait_bounded(f.mbar, phase ^ 1u, WAIT_LIMIT_NS);
      for (long long r = row; r < a.num_rows; r += stride)
        if (lane == 0) {
          a.tokens[r] = 0u;
          a.status[r] = (unsigned char)Q3S_STATUS_NOT_RUN;
        }
      return;
    }
    RowOut out{st, 0u};
    if (st == Q3S_STATUS_OK) {
      const StageView s = complete_stage<DT>(a, row, n, f);
      if (!P.do_sample) {
        out = greedy_stage<DT>(f, s, P.suppress_from, P.allow_token);
        release<DT>(rel);
      } else {
        out = sampled_row<DT, NJ>(a, f, g, cur, s, rel, delta, dbg);
      }
    }
    release<DT>(rel);
    if (lane == 0) {
      a.tokens[row] = out.token;
      a.status[row] = (unsigned char)out.status;
    }
    __syncwarp();
    cur = nxt;
  }
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

template <int DT, int NJ>
cudaError_t launch_t(const KernelArgs& a, int grid, int warps, cudaStream_t stream) {
  const size_t smem = fast_bytes(a.vcap, Elem<DT>::BYTES) * (size_t)warps;
  cudaError_t e = cudaFuncSetAttribute(sample_kernel<DT, NJ>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  sample_kernel<DT, NJ><<<grid, warps * 32, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace

size_t sample_smem_per_warp(int vcap, int dtype) {
  return fast_bytes(vcap, dtype == Q3S_DTYPE_F32 ? 4 : 2);
}

size_t sample_scratch_per_warp(int vcap) { return gen_bytes(vcap); }

int sample_max_warps(int vcap, int dtype, size_t smem_limit) {
  const size_t per = sample_smem_per_warp(vcap, dtype);
  int w = (int)(smem_limit / per);
  return w > MAX_WARPS ? MAX_WARPS : w;
}

cudaError_t launch_sample(const KernelArgs& a, int grid, int warps, cudaStream_t stream) {
  // NJ: 16-byte vectors per lane for the largest row (plus one for a
  // misaligned start).
  if (a.dtype == Q3S_DTYPE_F32) {
    const int q = (a.vcap * 4 + 15) / 16 + 1;
    if (q <= 32 * 8) return launch_t<Q3S_DTYPE_F32, 8>(a, grid, warps, stream);
    if (q <= 32 * 17) return launch_t<Q3S_DTYPE_F32, 17>(a, grid, warps, stream);
    if (q <= 32 * 25) return launch_t<Q3S_DTYPE_F32, 25>(a, grid, warps, stream);
    return launch_t<Q3S_DTYPE_F32, 33>(a, grid, warps, stream);
  }
  const int q = (a.vcap * 2 + 15) / 16 + 1;
  if (q <= 32 * 9) return launch_t<Q3S_DTYPE_BF16, 9>(a, grid, warps, stream);
  return launch_t<Q3S_DTYPE_BF16, 17>(a, grid, warps, stream);
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
