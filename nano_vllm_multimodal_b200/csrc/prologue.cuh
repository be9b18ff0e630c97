// Shared declarations of the two attention-prologue kernels.
#pragma once

#include "nib_common.cuh"

namespace nib {

constexpr int kPipeMaxWarps = 8;
constexpr int kPipeStages = 3;
constexpr uint32_t kPipeSmemBudget = 220 * 1024;  // dynamic shared memory per CTA
constexpr int64_t kPipeMinTokens = 2048;          // below this the register kernel is used

struct PipeLayout {
  int warps;             // warps per CTA, each with its own stage ring
  int stages;            // stages per warp (tokens in flight = stages - 1)
  uint32_t row_bytes;    // bytes of one token's [q|k|v] row
  uint32_t stage_bytes;  // row + table row, rounded up to 128
  uint32_t smem_bytes;   // dynamic shared memory per CTA
};

// true when q/k/v are consecutive head ranges of one 16-byte aligned row
bool prologue_pipe_eligible(const nib_qk_prologue_args& a);
int launch_prologue_pipe(const nib_qk_prologue_args& a, cudaStream_t st);

}  // namespace nib
