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
// parallel parts (max, counts, radix selection, sorting) are order-free.
//
// Layout: a persistent grid of warps strides over rows.  Each warp owns a
// shared-memory workspace: the row as f32 (A), a compacted list of surviving
// candidates in vocabulary order (B values, BI indices), a bitmap, a 256-bin
// histogram and a 256-key sort buffer.

#include <cstdint>

#include "../../include/q3s_sampler.h"
#include "q3s_device.cuh"
#include "q3s_kernels.h"

namespace q3s {
namespace {

constexpr int MAX_WARPS = 8;

struct WarpSpace {
  float* A;                 // [vcap] the row: raw logits, then transformed values x
  float* B;                 // [vcap] values of the candidate list
  uint16_t* BI;             // [vcap] vocabulary indices of the candidate list
  uint32_t* bm;             // [vcap/32] history bitmap
  uint32_t* hist;           // [256]
  unsigned long long* keys; // [256]
};

__host__ __device__ inline size_t align16(size_t b) { return (b + 15) & ~size_t(15); }

__host__ __device__ inline size_t warp_space_bytes(int vcap) {
  return align16(4u * vcap) * 2 + align16(2u * vcap) + align16(4u * (vcap / 32)) + 4u * 256 +
         8u * 256;
}

__device__ inline WarpSpace carve(unsigned char* base, int vcap) {
  WarpSpace w;
  size_t o = 0;
  w.A = reinterpret_cast<float*>(base + o);
  o += align16(4u * vcap);
  w.B = reinterpret_cast<float*>(base + o);
  o += align16(4u * vcap);
  w.BI = reinterpret_cast<uint16_t*>(base + o);
  o += align16(2u * vcap);
  w.bm = reinterpret_cast<uint32_t*>(base + o);
  o += align16(4u * (vcap / 32));
  w.hist = reinterpret_cast<uint32_t*>(base + o);
  o += 4u * 256;
  w.keys = reinterpret_cast<unsigned long long*>(base + o);
  return w;
}

// Copies n logits of the row into A as f32 (16-byte vector loads when the row
// start is aligned).
template <int DT>
__device__ void load_row(float* A, const void* base, long long off, int n) {
  const unsigned lane = lane_id();
  if (DT == Q3S_DTYPE_F32) {
    const float* src = static_cast<const float*>(base) + off;
    int done = 0;
    if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
      const int n4 = n >> 2;
      const float4* s4 = reinterpret_cast<const float4*>(src);
      float4* a4 = reinterpret_cast<float4*>(A);
      for (int q = lane; q < n4; q += 32) a4[q] = __ldg(s4 + q);
      done = n4 << 2;
    }
    for (int i = done + lane; i < n; i += 32) A[i] = __ldg(src + i);
  } else {
    const unsigned short* src = static_cast<const unsigned short*>(base) + off;
    int done = 0;
    if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
      const int n8 = n >> 3;
      const uint4* s8 = reinterpret_cast<const uint4*>(src);
      float4* a4 = reinterpret_cast<float4*>(A);
      for (int q = lane; q < n8; q += 32) {
        const uint4 v = __ldg(s8 + q);
        a4[2 * q] = make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u),
                                __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xFFFF0000u));
        a4[2 * q + 1] =
            make_float4(__uint_as_float(v.z << 16), __uint_as_float(v.z & 0xFFFF0000u),
                        __uint_as_float(v.w << 16), __uint_as_float(v.w & 0xFFFF0000u));
      }
      done = n8 << 3;
    }
    for (int i = done + lane; i < n; i += 32) A[i] = load_elem<Q3S_DTYPE_BF16>(src, i);
  }
  __syncwarp();
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

// k-th smallest (1-based) key among the valid elements, MSB-first radix
// selection with 8-bit digits.  Requires at least k valid elements.
template <typename K, class KeyFn>
__device__ K warp_select(int n, uint32_t k, KeyFn keyfn, uint32_t* hist) {
  constexpr int BITS = 8 * sizeof(K);
  const unsigned lane = lane_id();
  K prefix = 0, mask = 0;
  uint32_t kk = k;
#pragma unroll 1
  for (int shift = BITS - 8; shift >= 0; shift -= 8) {
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
    const int src = __ffs(ball) - 1;
    uint32_t digit = 0, before = 0;
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
__device__ inline float chain_sum(float* B, int count, bool prefix) {
  float c = 0.0f;
  if (lane_id() == 0) {
    if (prefix) {
      for (int j = 0; j < count; ++j) {
        c = __fadd_rn(c, B[j]);
        B[j] = c;
      }
    } else {
      for (int j = 0; j < count; ++j) c = __fadd_rn(c, B[j]);
    }
  }
  __syncwarp();
  return __shfl_sync(FULL, c, 0);
}

__device__ __forceinline__ unsigned long long nucleus_key(float p, uint16_t idx) {
  return ((unsigned long long)(~__float_as_uint(p)) << 32) | idx;
}

struct RowOut {
  int status;
  uint32_t token;
};

template <int DT>
__device__ RowOut sample_row(const KernelArgs& a, const WarpSpace& w, long long row, int n,
                             const q3s_row_params& P) {
  const unsigned lane = lane_id();
  const long long off = a.row_offsets ? a.row_offsets[row] : row * a.row_stride;
  float* A = w.A;
  float* B = w.B;
  uint16_t* BI = w.BI;
  const int sf = P.suppress_from, allow = P.allow_token;
  const bool dbg = a.masks != nullptr;
  unsigned char* mrow = dbg ? a.masks + row * a.probs_stride : nullptr;
  float* prow = a.probs ? a.probs + row * a.probs_stride : nullptr;
  if (dbg)
    for (int i = lane; i < n; i += 32) mrow[i] = 0;
  if (prow)
    for (int i = lane; i < n; i += 32) prow[i] = 0.0f;

  load_row<DT>(A, a.logits, off, n);

  // Greedy (sampling.rs:574-591): total_cmp maximum of the raw finite,
  // allowed logits; ties to the lowest index; no penalty, no draw.
  if (!P.do_sample) {
    unsigned long long best = 0ull;
    for (int i = lane; i < n; i += 32) {
      const float v = A[i];
      if (is_finite(v) && idx_allowed(i, sf, allow)) {
        const unsigned long long c =
            ((unsigned long long)total_key(v) << 32) | (0xFFFFFFFFu - (uint32_t)i);
        best = c > best ? c : best;
      }
    }
    best = warp_max_u64(best);
    if (best == 0ull) return {Q3S_STATUS_NO_CANDIDATE, 0u};
    return {Q3S_STATUS_OK, 0xFFFFFFFFu - (uint32_t)best};
  }

  // Repetition penalty (sampling.rs:598-606, 732-773): every distinct history
  // id < n once, marked in a bitmap.
  long long h0 = 0, h1 = 0;
  if (a.history_offsets) {
    h0 = a.history_offsets[row];
    h1 = a.history_offsets[row + 1];
  }
  const bool use_pen = P.repetition_penalty != 1.0 && h1 > h0;
  const float pf = (float)P.repetition_penalty;
  if (use_pen) {
    const int words = (n + 31) >> 5;
    for (int q = lane; q < words; q += 32) w.bm[q] = 0u;
    __syncwarp();
    for (long long h = h0 + lane; h < h1; h += 32) {
      const int id = a.history[h];
      if (id < n) atomicOr(&w.bm[id >> 5], 1u << (id & 31));
    }
    __syncwarp();
  }

  // Mask and temperature (sampling.rs:608-631).
  const float inv_temp = __fdiv_rn(1.0f, (float)P.temperature);
  float mx = neg_inf();
  int nfin = 0;
  bool nan_seen = false;
  for (int i = lane; i < n; i += 32) {
    float v = A[i];
    if (use_pen && ((w.bm[i >> 5] >> (i & 31)) & 1u))
      v = v < 0.0f ? __fmul_rn(v, pf) : __fdiv_rn(v, pf);
    const bool suppressed = sf >= 0 && i >= sf && !(allow >= 0 && i == allow);
    if (!is_finite(v) || suppressed) v = neg_inf();
    const float x = __fmul_rn(v, inv_temp);
    A[i] = x;
    mx = fmaxf(mx, x);
    nfin += is_finite(x) ? 1 : 0;
    nan_seen |= (x != x);
    if (dbg && is_finite(x)) mrow[i] = 1;
  }
  mx = warp_max(mx);
  nfin = __reduce_add_sync(FULL, nfin);
  nan_seen = __any_sync(FULL, nan_seen);
  __syncwarp();
  // No finite candidate (sampling.rs:642-651).
  if (nfin == 0)
    return {sf >= 0 ? Q3S_STATUS_SUPPRESSION_NO_CANDIDATE : Q3S_STATUS_NO_CANDIDATE, 0u};
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
        w.hist);
    t = from_total_key(~key);
  }
  auto survives = [&](float x) { return x >= t && x > neg_inf(); };
  if (dbg) {
    for (int i = lane; i < n; i += 32)
      if (survives(A[i])) mrow[i] |= 2;
  }

  // Candidate list in vocabulary order.  With top-p the values are
  // exp(x - max) of the denominator; otherwise those of the final softmax.
  const float m1 = mx;
  int ns = 0;
  for (int i0 = 0; i0 < n; i0 += 32) {
    const int i = i0 + lane;
    const bool p = i < n && survives(A[i]);
    const unsigned b = __ballot_sync(FULL, p);
    if (p) {
      const int j = ns + __popc(b & lanemask_lt());
      BI[j] = (uint16_t)i;
      B[j] = cr_expf(__fsub_rn(A[i], m1));
    }
    ns += __popc(b);
  }
  __syncwarp();

  float m2 = m1;
  if (P.top_p < 1.0) {
    // Top-p (sampling.rs:665-698).  Denominator: sequential f32 sum in
    // vocabulary order; max_logit is m1 because the maximum survives top-k.
    const float total = chain_sum(B, ns, false);
    if (!is_finite(total) || total <= 0.0f) return {Q3S_STATUS_INVALID_DENOMINATOR, 0u};
    const float inv_total = __fdiv_rn(1.0f, total);
    const float cutoff = __fsub_rn(m1, 16.0f);
    int np = 0;
    for (int j = lane; j < ns; j += 32) {
      const float p = A[BI[j]] >= cutoff ? __fmul_rn(B[j], inv_total) : 0.0f;
      B[j] = p;
      np += p > 0.0f ? 1 : 0;
    }
    np = __reduce_add_sync(FULL, np);
    __syncwarp();
    // Walk the probabilities in (p desc, index asc) order, 256 at a time; the
    // first position > 0 whose preceding cumulative reaches top_p starts the
    // masked tail.
    const float top_p = (float)P.top_p;
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
      if (remaining > 256) hi = warp_select<unsigned long long>(ns, 256u, pkey, w.hist);
      int cnt = 0;
      for (int j0 = 0; j0 < ns; j0 += 32) {
        const int j = j0 + lane;
        unsigned long long k = 0;
        const bool p = j < ns && pkey(j, k) && k <= hi;
        const unsigned b = __ballot_sync(FULL, p);
        if (p) w.keys[cnt + __popc(b & lanemask_lt())] = k;
        cnt += __popc(b);
      }
      __syncwarp();
      unsigned long long v[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const int e = lane * 8 + r;
        v[r] = e < cnt ? w.keys[e] : ~0ull;
      }
      __syncwarp();
      bitonic_sort_256(v);
#pragma unroll
      for (int r = 0; r < 8; ++r) w.keys[lane * 8 + r] = v[r];
      __syncwarp();
      if (lane == 0) {
        for (int q = 0; q < cnt; ++q) {
          const unsigned long long k = w.keys[q];
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
      if (cut != ~0ull) break;
      last = hi;
      remaining -= m;
    }
    // Final survivors: nucleus members before the cut.
    m2 = neg_inf();
    for (int j = lane; j < ns; j += 32) {
      const float p = B[j];
      if (p > 0.0f && nucleus_key(p, BI[j]) >= cut) B[j] = 0.0f;
      if (B[j] > 0.0f) m2 = fmaxf(m2, A[BI[j]]);
    }
    m2 = warp_max(m2);
    __syncwarp();
    if (!(m2 > neg_inf())) return {Q3S_STATUS_NO_CANDIDATE, 0u};
    // Compact the survivors in place with the final softmax numerators.
    int ns2 = 0;
    for (int j0 = 0; j0 < ns; j0 += 32) {
      const int j = j0 + lane;
      const bool p = j < ns && B[j] > 0.0f;
      const int i = p ? BI[j] : 0;
      __syncwarp();
      const unsigned b = __ballot_sync(FULL, p);
      if (p) {
        const int d = ns2 + __popc(b & lanemask_lt());
        BI[d] = (uint16_t)i;
        B[d] = cr_expf(__fsub_rn(A[i], m2));
      }
      ns2 += __popc(b);
      __syncwarp();
    }
    ns = ns2;
  }

  // Final softmax sum and the draw (sampling.rs:700-729).
  const float sum = chain_sum(B, ns, true);
  if (!is_finite(sum) || sum <= 0.0f) return {Q3S_STATUS_INVALID_DENOMINATOR, 0u};
  const float u = a.uniform_override ? a.uniform_override[row]
                                     : philox_uniform(a.seeds[row], a.subseqs[row], P.ctr_lo);
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
  if (dbg || prow) {
    for (int j = lane; j < ns; j += 32) {
      const int i = BI[j];
      if (dbg) mrow[i] |= 4;
      if (prow) {
        const float e = cr_expf(__fsub_rn(A[i], m2));
        prow[i] = __double2float_rn((double)e / (double)sum);
      }
    }
  }
  return {Q3S_STATUS_OK, token};
}

template <int DT>
__global__ void __launch_bounds__(MAX_WARPS * 32, 1) sample_kernel(const KernelArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int warp = threadIdx.x >> 5;
  const int warps = blockDim.x >> 5;
  const WarpSpace w = carve(smem + (size_t)warp * warp_space_bytes(a.vcap), a.vcap);
  const long long stride = (long long)gridDim.x * warps;
  for (long long row = (long long)blockIdx.x * warps + warp; row < a.num_rows; row += stride) {
    const int n = a.row_vocab ? a.row_vocab[row] : a.vocab;
    const q3s_row_params P = a.params[row * a.params_stride];
    RowOut out{Q3S_STATUS_UNSUPPORTED, 0u};
    if (n >= 0 && n <= a.vocab && n <= a.vcap) {
      out.status = validate(P);
      if (out.status == Q3S_STATUS_OK) out = sample_row<DT>(a, w, row, n, P);
    }
    if (lane_id() == 0) {
      a.tokens[row] = out.token;
      a.status[row] = (unsigned char)out.status;
    }
    __syncwarp();
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

}  // namespace

size_t sample_smem_per_warp(int vcap) { return warp_space_bytes(vcap); }

int sample_max_warps(int vcap, size_t smem_limit) {
  const size_t per = warp_space_bytes(vcap);
  int w = (int)(smem_limit / per);
  return w > MAX_WARPS ? MAX_WARPS : w;
}

cudaError_t launch_sample(const KernelArgs& a, int grid, int warps, cudaStream_t stream) {
  const size_t smem = warp_space_bytes(a.vcap) * (size_t)warps;
  cudaError_t e;
  if (a.dtype == Q3S_DTYPE_F32) {
    e = cudaFuncSetAttribute(sample_kernel<Q3S_DTYPE_F32>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    sample_kernel<Q3S_DTYPE_F32><<<grid, warps * 32, smem, stream>>>(a);
  } else {
    e = cudaFuncSetAttribute(sample_kernel<Q3S_DTYPE_BF16>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    sample_kernel<Q3S_DTYPE_BF16><<<grid, warps * 32, smem, stream>>>(a);
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
