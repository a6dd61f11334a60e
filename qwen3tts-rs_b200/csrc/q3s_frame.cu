// Device-resident decode frame: the per-row commit that follows each
// batched sampling launch of a frame (1 talker row + 15 code-predictor
// groups per stream), so that a frame's launches run back to back with no
// host round trip.  The reference does this work on the host after every
// Sampler call: the sampled id is uploaded again as the next step's input
// (Tensor::new(&[next_val]), code_predictor.rs:365, 414; talker.rs:530) and
// collected into the frame's codes (code_predictor.rs:421), the Philox
// subsequence advances on a draw (sampling.rs:330-332), and the c0 id joins
// the talker's repetition history (talker.rs:562-566).  A failed call ends
// the reference's frame with an error; here the row's first failure is kept
// in frame_status and freezes its counter and history.
//
// One thread per row, grid-stride: a few bytes per row, launch-bound.
#include <cstdint>

#include <cuda_runtime.h>

#include "../../include/q3s_sampler.h"
#include "q3s_internal.h"

namespace q3s {
namespace {

__global__ void commit_kernel(q3s_commit c) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x; r < c.num_rows;
       r += stride) {
    const uint32_t token = c.tokens[r];
    int st = c.status[r];
    if (c.codes) c.codes[r * c.codes_stride + c.group] = token;
    if (c.frame_status && c.frame_status[r] != Q3S_STATUS_OK) continue;
    if (st == Q3S_STATUS_OK && c.subseqs && c.params[r * c.params_stride].do_sample)
      c.subseqs[r] += 1;
    if (st == Q3S_STATUS_OK && c.history) {
      const long long e = c.history_ends[r];
      if (e < c.history_limits[r]) {
        c.history[e] = (uint16_t)token;
        c.history_ends[r] = e + 1;
      } else {
        st = Q3S_STATUS_HISTORY_FULL;
      }
    }
    if (c.frame_status) c.frame_status[r] = (uint8_t)st;
  }
}

}  // namespace
}  // namespace q3s

extern "C" int q3s_commit_rows(q3s_context* ctx, const q3s_commit* c, void* stream) {
  using q3s::record_error;
  if (!ctx || !c) return record_error(Q3S_E_INVALID_ARGUMENT, "q3s_commit_rows: NULL argument");
  if (c->num_rows < 0) return record_error(Q3S_E_INVALID_ARGUMENT, "num_rows must be >= 0");
  if (c->num_rows == 0) return Q3S_OK;
  if (!c->tokens || !c->status)
    return record_error(Q3S_E_INVALID_ARGUMENT, "q3s_commit_rows: tokens and status are required");
  if (c->subseqs && !c->params)
    return record_error(Q3S_E_INVALID_ARGUMENT, "q3s_commit_rows: subseqs need params");
  if (c->params_stride != 0 && c->params_stride != 1)
    return record_error(Q3S_E_INVALID_ARGUMENT, "params_stride must be 0 or 1");
  if (c->codes && (c->group < 0 || c->codes_stride <= c->group))
    return record_error(Q3S_E_INVALID_ARGUMENT, "q3s_commit_rows: group outside codes_stride");
  if (c->history && (!c->history_ends || !c->history_limits))
    return record_error(Q3S_E_INVALID_ARGUMENT,
                        "q3s_commit_rows: history needs history_ends and history_limits");
  const q3s::ContextInfo ci = q3s::context_info(ctx);
  int prev = -1;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return q3s::record_cuda_error(e, "cudaGetDevice");
  if (prev != ci.device && (e = cudaSetDevice(ci.device)) != cudaSuccess)
    return q3s::record_cuda_error(e, "cudaSetDevice");
  long long blocks = (c->num_rows + 255) / 256;
  if (blocks > 4LL * ci.sm_count) blocks = 4LL * ci.sm_count;
  q3s::commit_kernel<<<(int)blocks, 256, 0, (cudaStream_t)stream>>>(*c);
  e = cudaGetLastError();
  if (prev != ci.device) cudaSetDevice(prev);
  if (e != cudaSuccess) return q3s::record_cuda_error(e, "commit kernel launch");
  return Q3S_OK;
}
