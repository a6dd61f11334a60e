// Codebook embedding sum after sampling (talker.rs:568-580): per row,
// out = ((T0[c0] + T1[c1]) + ... + T(G-1)[c(G-1)]) + text, each addition
// rounded to the element type in that order, as the reference's sequential
// tensor additions do (candle binary add, patches/candle-kernels/src/
// binary.cu:5).  For bf16 the sum of two bf16 values is formed in f32 and
// rounded once to bf16: the f32 sum is exact unless the exponents differ by
// more than 16, and then both roundings return the larger term, so this is
// the correctly rounded bf16 sum.
//
// HBM-bound gather: a row reads G rows of H elements from the tables (and
// one text row) and writes H.  One block of 128 threads per row, each thread
// 8 consecutive elements (16-byte bf16 or 32-byte f32 vectors); all G
// vectors are loaded before the sequential additions.
#include <cstdint>
#include <string>

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../../include/q3s_sampler.h"
#include "q3s_internal.h"

namespace q3s {
namespace {

constexpr int EMBED_THREADS = 128;
constexpr int EMBED_VEC = 8;

struct EmbedArgs {
  const void* tables[Q3S_MAX_CODE_GROUPS];
  int vocab[Q3S_MAX_CODE_GROUPS];
  const uint32_t* codes;
  const void* text;
  long long text_stride;
  void* out;
  uint8_t* status;
  long long rows;
  int groups;
  int hidden;
};

__device__ __forceinline__ float bf(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }
__device__ __forceinline__ uint16_t to_bf(float v) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

// Eight elements of a row as f32 (bf16 upcasts exactly).
template <int DT>
__device__ __forceinline__ void load8(const void* base, long long off, float (&v)[EMBED_VEC]) {
  if (DT == Q3S_DTYPE_F32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + off);
    const float4 a = __ldg(p), b = __ldg(p + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 w = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + off));
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      v[2 * t] = bf((uint16_t)(u[t] & 0xFFFFu));
      v[2 * t + 1] = bf((uint16_t)(u[t] >> 16));
    }
  }
}

template <int DT>
__device__ __forceinline__ float load1(const void* base, long long off) {
  if (DT == Q3S_DTYPE_F32) return static_cast<const float*>(base)[off];
  return bf(static_cast<const uint16_t*>(base)[off]);
}

// acc + x rounded to the element type (acc already is of that type).
template <int DT>
__device__ __forceinline__ float add_t(float acc, float x) {
  const float s = __fadd_rn(acc, x);
  return DT == Q3S_DTYPE_F32 ? s : bf(to_bf(s));
}

template <int DT>
__device__ __forceinline__ void store8(void* base, long long off, const float (&v)[EMBED_VEC]) {
  if (DT == Q3S_DTYPE_F32) {
    float4* p = reinterpret_cast<float4*>(static_cast<float*>(base) + off);
    p[0] = make_float4(v[0], v[1], v[2], v[3]);
    p[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint4 w;
    w.x = (uint32_t)to_bf(v[0]) | ((uint32_t)to_bf(v[1]) << 16);
    w.y = (uint32_t)to_bf(v[2]) | ((uint32_t)to_bf(v[3]) << 16);
    w.z = (uint32_t)to_bf(v[4]) | ((uint32_t)to_bf(v[5]) << 16);
    w.w = (uint32_t)to_bf(v[6]) | ((uint32_t)to_bf(v[7]) << 16);
    *reinterpret_cast<uint4*>(static_cast<uint16_t*>(base) + off) = w;
  }
}

template <int DT>
__device__ __forceinline__ void store1(void* base, long long off, float v) {
  if (DT == Q3S_DTYPE_F32)
    static_cast<float*>(base)[off] = v;
  else
    static_cast<uint16_t*>(base)[off] = to_bf(v);
}

// Raw 16-byte vectors of one group's 8 elements (two for f32, one for bf16).
template <int DT>
struct Raw {
  static constexpr int N = DT == Q3S_DTYPE_F32 ? 2 : 1;
  uint4 w[N];
};

template <int DT>
__device__ __forceinline__ void load_raw(const void* base, long long off, Raw<DT>& r) {
  const uint4* p = reinterpret_cast<const uint4*>(static_cast<const unsigned char*>(base) +
                                                  off * (DT == Q3S_DTYPE_F32 ? 4 : 2));
#pragma unroll
  for (int i = 0; i < Raw<DT>::N; ++i) r.w[i] = __ldg(p + i);
}

// acc[e] + element e of r, rounded to the element type, e = 0..7 in order.
template <int DT>
__device__ __forceinline__ void add_raw(float (&acc)[EMBED_VEC], const Raw<DT>& r) {
  float v[EMBED_VEC];
  if (DT == Q3S_DTYPE_F32) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      v[4 * i] = __uint_as_float(r.w[i].x);
      v[4 * i + 1] = __uint_as_float(r.w[i].y);
      v[4 * i + 2] = __uint_as_float(r.w[i].z);
      v[4 * i + 3] = __uint_as_float(r.w[i].w);
    }
  } else {
    const uint32_t u[4] = {r.w[0].x, r.w[0].y, r.w[0].z, r.w[0].w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      v[2 * t] = bf((uint16_t)(u[t] & 0xFFFFu));
      v[2 * t + 1] = bf((uint16_t)(u[t] >> 16));
    }
  }
#pragma unroll
  for (int e = 0; e < EMBED_VEC; ++e) acc[e] = add_t<DT>(acc[e], v[e]);
}

// VEC_OK: every table, the text and the output start 16-byte aligned and H
// is a multiple of 8, so whole 8-element vectors are aligned.
template <int DT, bool VEC_OK>
__global__ void __launch_bounds__(EMBED_THREADS) embed_sum_kernel(const EmbedArgs a) {
  __shared__ long long rowoff[Q3S_MAX_CODE_GROUPS];
  __shared__ int bad;
  const int G = a.groups, H = a.hidden;
  for (long long r = blockIdx.x; r < a.rows; r += gridDim.x) {
    __syncthreads();  // the previous row's offsets are no longer read
    if (threadIdx.x == 0) bad = 0;
    __syncthreads();
    if ((int)threadIdx.x < G) {
      const uint32_t c = a.codes[r * G + threadIdx.x];
      if (c >= (uint32_t)a.vocab[threadIdx.x]) bad = 1;
      rowoff[threadIdx.x] = (long long)c * H;
    }
    __syncthreads();
    const bool ok = bad == 0;
    const long long orow = r * H;
    const long long trow = r * a.text_stride;
    if (VEC_OK) {
      for (int h = threadIdx.x * EMBED_VEC; h < H; h += EMBED_THREADS * EMBED_VEC) {
        float acc[EMBED_VEC];
        if (ok) {
          load8<DT>(a.tables[0], rowoff[0] + h, acc);
          // The next NB groups' vectors are all loaded before their adds, so
          // NB gathers are in flight per thread; the adds keep group order.
          constexpr int NB = 8 / Raw<DT>::N;
#pragma unroll 1
          for (int g0 = 1; g0 < G; g0 += NB) {
            Raw<DT> r[NB];
#pragma unroll
            for (int j = 0; j < NB; ++j)
              if (g0 + j < G) load_raw<DT>(a.tables[g0 + j], rowoff[g0 + j] + h, r[j]);
#pragma unroll
            for (int j = 0; j < NB; ++j)
              if (g0 + j < G) add_raw<DT>(acc, r[j]);
          }
          if (a.text) {
            float v[EMBED_VEC];
            load8<DT>(a.text, trow + h, v);
#pragma unroll
            for (int e = 0; e < EMBED_VEC; ++e) acc[e] = add_t<DT>(acc[e], v[e]);
          }
        } else {
#pragma unroll
          for (int e = 0; e < EMBED_VEC; ++e) acc[e] = 0.0f;
        }
        store8<DT>(a.out, orow + h, acc);
      }
    } else {
      for (int h = threadIdx.x; h < H; h += EMBED_THREADS) {
        float acc = 0.0f;
        if (ok) {
          acc = load1<DT>(a.tables[0], rowoff[0] + h);
          for (int g = 1; g < G; ++g) acc = add_t<DT>(acc, load1<DT>(a.tables[g], rowoff[g] + h));
          if (a.text) acc = add_t<DT>(acc, load1<DT>(a.text, trow + h));
        }
        store1<DT>(a.out, orow + h, acc);
      }
    }
    if (threadIdx.x == 0) a.status[r] = ok ? (uint8_t)Q3S_STATUS_OK : (uint8_t)Q3S_STATUS_INVALID_CODE;
  }
}

template <int DT>
cudaError_t launch_embed(const EmbedArgs& a, bool vec_ok, int grid, cudaStream_t stream) {
  if (vec_ok)
    embed_sum_kernel<DT, true><<<grid, EMBED_THREADS, 0, stream>>>(a);
  else
    embed_sum_kernel<DT, false><<<grid, EMBED_THREADS, 0, stream>>>(a);
  return cudaGetLastError();
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Makes `device` current for the scope and restores the caller's device.
struct EmbedDevice {
  int prev = -1;
  cudaError_t err = cudaSuccess;
  explicit EmbedDevice(int device) {
    err = cudaGetDevice(&prev);
    if (err == cudaSuccess && prev != device) err = cudaSetDevice(device);
  }
  ~EmbedDevice() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace
}  // namespace q3s

extern "C" int q3s_embed_sum(q3s_context* ctx, const q3s_embed_batch* b, void* stream) {
  using q3s::record_error;
  if (!ctx || !b) return record_error(Q3S_E_INVALID_ARGUMENT, "q3s_embed_sum: NULL context or batch");
  if (b->num_rows < 0) return record_error(Q3S_E_INVALID_ARGUMENT, "num_rows must be >= 0");
  if (b->dtype != Q3S_DTYPE_F32 && b->dtype != Q3S_DTYPE_BF16)
    return record_error(Q3S_E_INVALID_ARGUMENT, "dtype must be Q3S_DTYPE_F32 or Q3S_DTYPE_BF16");
  if (b->groups < 1 || b->groups > Q3S_MAX_CODE_GROUPS)
    return record_error(Q3S_E_INVALID_ARGUMENT,
                        "groups must be in 1.." + std::to_string(Q3S_MAX_CODE_GROUPS));
  if (b->hidden < 1) return record_error(Q3S_E_INVALID_ARGUMENT, "hidden must be >= 1");
  if (b->num_rows == 0) return Q3S_OK;
  if (!b->codes || !b->tables || !b->vocab || !b->out || !b->status)
    return record_error(Q3S_E_INVALID_ARGUMENT, "codes, tables, vocab, out and status are required");
  if (b->text && b->text_stride < 0)
    return record_error(Q3S_E_INVALID_ARGUMENT, "text_stride must be >= 0");
  q3s::EmbedArgs a;
  bool vec_ok = b->hidden % 8 == 0 && q3s::aligned16(b->out) &&
                (!b->text || (q3s::aligned16(b->text) && b->text_stride % 8 == 0));
  for (int g = 0; g < b->groups; ++g) {
    if (!b->tables[g]) return record_error(Q3S_E_INVALID_ARGUMENT, "a codebook table is NULL");
    if (b->vocab[g] < 1) return record_error(Q3S_E_INVALID_ARGUMENT, "a codebook vocabulary is < 1");
    a.tables[g] = b->tables[g];
    a.vocab[g] = b->vocab[g];
    vec_ok = vec_ok && q3s::aligned16(b->tables[g]);
  }
  for (int g = b->groups; g < Q3S_MAX_CODE_GROUPS; ++g) {
    a.tables[g] = nullptr;
    a.vocab[g] = 0;
  }
  a.codes = b->codes;
  a.text = b->text;
  a.text_stride = b->text_stride;
  a.out = b->out;
  a.status = b->status;
  a.rows = b->num_rows;
  a.groups = b->groups;
  a.hidden = b->hidden;
  const q3s::ContextInfo ci = q3s::context_info(ctx);
  q3s::EmbedDevice dg(ci.device);
  if (dg.err != cudaSuccess) return q3s::record_cuda_error(dg.err, "cudaSetDevice");
  long long grid = b->num_rows;
  const long long cap = (long long)ci.sm_count * 16;
  if (grid > cap) grid = cap;
  const cudaError_t e =
      b->dtype == Q3S_DTYPE_F32
          ? q3s::launch_embed<Q3S_DTYPE_F32>(a, vec_ok, (int)grid, (cudaStream_t)stream)
          : q3s::launch_embed<Q3S_DTYPE_BF16>(a, vec_ok, (int)grid, (cudaStream_t)stream);
  if (e != cudaSuccess) return q3s::record_cuda_error(e, "embed kernel launch");
  return Q3S_OK;
}
