// Internal interface between the C ABI (q3s_capi.cpp) and the kernels
// (q3s_sample.cu).  Not installed; callers use include/q3s_sampler.h.
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

#include "../../include/q3s_sampler.h"

namespace q3s {

struct KernelArgs {
  const void* logits;
  int dtype;
  int vocab;  // every row's vocabulary, or an upper bound when row_vocab is set
  long long num_rows;
  long long row_stride;
  const long long* row_offsets;
  const int* row_vocab;
  const q3s_row_params* params;
  long long params_stride;
  const unsigned long long* seeds;
  const unsigned long long* subseqs;
  const unsigned short* history;
  const long long* history_offsets;
  const long long* history_ends;  // NULL: row r ends at history_offsets[r + 1]
  unsigned* tokens;
  unsigned char* status;
  const float* uniform_override;
  float* probs;
  unsigned char* masks;
  long long probs_stride;
  int vcap;  // per-warp row capacity in elements (multiple of 32)
  unsigned char* scratch;  // general-path workspace: sample_scratch_per_warp(vcap) per warp
  // Limit of each per-row stage wait (the end-of-block drain keeps its own
  // one-second limit).  Testing hook: hold_refill stops the ring refills, so
  // every row after a stage's first one waits for a generation nothing issues.
  unsigned long long wait_ns = 1000000000ull;
  int hold_refill = 0;
  // Diagnostics (q3s_context_set_path_stats): per Q3S_PATH_* row counts and
  // warp cycles, accumulated by the debug instantiation; NULL in production.
  unsigned long long* path_stats = nullptr;
  // A single-row launch (the stateful sampler) passes its row by value:
  // parameters, Philox key and counter, and the length of its history at
  // `history` (no history_offsets), so nothing but the history is uploaded.
  int inline_row = 0;
  q3s_row_params row_params{};
  unsigned long long row_seed = 0, row_subseq = 0;
  long long row_hist_len = 0;
  // In-kernel commit (q3s_sample_commit): after storing a row's result, its
  // warp does what q3s_commit_rows does for the row.  subseqs / history /
  // history_ends are the launch's own arrays, written for this row only.
  int commit = 0;
  unsigned* c_codes = nullptr;
  long long c_codes_stride = 0;
  int c_group = 0;
  unsigned char* c_frame_status = nullptr;
  unsigned long long* c_subseqs = nullptr;
  unsigned short* c_history = nullptr;
  long long* c_history_ends = nullptr;
  const long long* c_history_limits = nullptr;
};

// The head projection of q3s_head_sample (logits = hidden · weightᵀ).
struct HeadArgs {
  const void* hidden;      // [rows, hidden_size], row stride hidden_stride elements
  int hidden_dtype;        // Q3S_DTYPE_F32 or Q3S_DTYPE_BF16
  int hidden_size;         // a multiple of 8
  long long hidden_stride;
  const unsigned short* weight;  // bf16 [vocab, hidden_size], 16-byte aligned
  int vocab;
  float* logits;           // out [rows, vocab]
  unsigned* counter;       // blocks done; 0 before the launch, 0 again after it
};

size_t sample_smem_per_warp(int vcap, int dtype);
size_t head_smem(int vcap);
cudaError_t launch_head_sample(const HeadArgs& h, const KernelArgs& a, int grid,
                               cudaStream_t stream);
size_t sample_scratch_per_warp(int vcap);
int sample_max_warps(int vcap, int dtype, size_t smem_limit);
cudaError_t launch_sample(const KernelArgs& a, int grid, int warps, cudaStream_t stream);
cudaError_t launch_greedy(const void* logits, int dtype, long long num_rows, long long row_stride,
                          int n, long long sf, long long allow, int mode, uint32_t* tokens,
                          uint8_t* status, int grid, cudaStream_t stream);

}  // namespace q3s
