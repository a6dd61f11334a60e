// q3s_sample_batch_static: the batched sampling launch of q3s_sample_batch
// with its general-path workspace in a file-scope device array, so that a
// call allocates nothing (no cudaMalloc, cudaFree or allocating library
// routine).  It serves callers that must not allocate device memory while
// they generate: engines whose device memory is owned by their own pool
// allocator, and per-step loops that cannot take the synchronisation an
// allocation may cause.  The kernel and its results are those of
// q3s_sample_batch.
//
// The array is Q3S_STATIC_SCRATCH_BYTES (32 MiB) on every device that loads
// the library, held until the process exits.  Every call looks its address
// up with the call's device current (cudaGetSymbolAddress allocates nothing),
// so the address stays right after a device reset re-creates the context and
// reloads the module.  The first call on a device may load the module: make
// that first call before any stream capture.  Every call on a device shares the array; the
// kernel writes every workspace word of a row before reading it, so nothing
// has to start at zero and nothing is cleared.  Calls whose kernels overlap
// on the GPU (other streams, other host threads, other contexts of the same
// device) race on the array: order them on one stream or with events.
#include <string>

#include <cuda_runtime.h>

#include "../../include/q3s_sampler.h"
#include "q3s_internal.h"
#include "q3s_kernels.h"

namespace {

__device__ __align__(256) unsigned char g_static_scratch[Q3S_STATIC_SCRATCH_BYTES];

// Device address of g_static_scratch on the current device.  Host code only
// holds a stand-in for the array, never its device address, so the address
// is asked of the runtime for the current device on every call.
cudaError_t static_scratch(unsigned char** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
  if (e != cudaSuccess) return e;
  *out = static_cast<unsigned char*>(p);
  return cudaSuccess;
}

// Makes `device` current for the scope and restores the caller's device.
struct CurrentDevice {
  int prev = -1;
  cudaError_t err = cudaSuccess;
  explicit CurrentDevice(int device) {
    err = cudaGetDevice(&prev);
    if (err == cudaSuccess && prev != device) err = cudaSetDevice(device);
  }
  ~CurrentDevice() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace

extern "C" int q3s_sample_batch_static(q3s_context* ctx, const q3s_batch* b, void* stream) {
  using q3s::record_error;
  if (!ctx || !b)
    return record_error(Q3S_E_INVALID_ARGUMENT, "q3s_sample_batch_static: NULL context or batch");
  if (b->num_rows < 0) return record_error(Q3S_E_INVALID_ARGUMENT, "num_rows must be >= 0");
  if (b->vocab < 0) return record_error(Q3S_E_INVALID_ARGUMENT, "vocab must be >= 0");
  if (b->vocab > Q3S_MAX_VOCAB)
    return record_error(Q3S_E_INVALID_ARGUMENT,
                        "q3s_sample_batch_static: vocab " + std::to_string(b->vocab) +
                            " exceeds the static-workspace maximum of " +
                            std::to_string(Q3S_MAX_VOCAB));
  if (b->num_rows == 0) return Q3S_OK;
  if (b->dtype != Q3S_DTYPE_F32 && b->dtype != Q3S_DTYPE_BF16)
    return record_error(Q3S_E_INVALID_ARGUMENT, "dtype must be Q3S_DTYPE_F32 or Q3S_DTYPE_BF16");
  if (!b->logits || !b->params || !b->tokens || !b->status)
    return record_error(Q3S_E_INVALID_ARGUMENT, "logits, params, tokens and status are required");
  if (!b->uniform_override && (!b->seeds || !b->subseqs))
    return record_error(Q3S_E_INVALID_ARGUMENT, "seeds and subseqs are required");
  if (b->params_stride != 0 && b->params_stride != 1)
    return record_error(Q3S_E_INVALID_ARGUMENT, "params_stride must be 0 or 1");
  if (!b->row_offsets && b->row_stride < 0)
    return record_error(Q3S_E_INVALID_ARGUMENT, "row_stride must be >= 0");
  if (b->history_offsets && !b->history)
    return record_error(Q3S_E_INVALID_ARGUMENT, "history_offsets without history");
  if ((b->probs || b->masks) && b->probs_stride < b->vocab)
    return record_error(Q3S_E_INVALID_ARGUMENT, "probs_stride must be >= vocab");
  const q3s::ContextInfo ci = q3s::context_info(ctx);
  CurrentDevice g(ci.device);
  if (g.err != cudaSuccess) return q3s::record_cuda_error(g.err, "cudaSetDevice");
  unsigned char* scratch = nullptr;
  cudaError_t e = static_scratch(&scratch);
  if (e != cudaSuccess) return q3s::record_cuda_error(e, "cudaGetSymbolAddress(static workspace)");
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
  a.vcap = ((b->vocab > 0 ? b->vocab : 1) + 31) / 32 * 32;
  const int warps = q3s::sample_max_warps(a.vcap, b->dtype, ci.smem_optin);
  if (warps < 1) return record_error(Q3S_E_INVALID_ARGUMENT, "vocabulary does not fit shared memory");
  // As many blocks as the static workspace holds, at most one per SM.
  const size_t per_block = (size_t)warps * q3s::sample_scratch_per_warp(a.vcap);
  long long blocks = (b->num_rows + warps - 1) / warps;
  if (blocks > ci.sm_count) blocks = ci.sm_count;
  const long long fit = (long long)(Q3S_STATIC_SCRATCH_BYTES / per_block);
  if (fit < 1)
    return record_error(Q3S_E_INVALID_ARGUMENT,
                        "q3s_sample_batch_static: one block needs " + std::to_string(per_block) +
                            " workspace bytes, more than the static " +
                            std::to_string((size_t)Q3S_STATIC_SCRATCH_BYTES));
  if (blocks > fit) blocks = fit;
  a.scratch = scratch;
  e = q3s::launch_sample(a, (int)blocks, warps, (cudaStream_t)stream);
  if (e != cudaSuccess) return q3s::record_cuda_error(e, "sample kernel launch");
  return Q3S_OK;
}
