// Shared declarations of the two attention-prologue kernels.
#pragma once

#include "nib_common.cuh"

namespace nib {

// CTA shape of the pipelined kernel (one CTA per SM). With 16-bit norm
// weights (or no norm) the kernel takes about 155 registers, so 12 warps with a
// 2-stage ring (one token in flight per warp) fit; float32 weights need more
// registers and use 8 warps x 3 stages. A warp spends microseconds per token,
// far longer than one row's load takes, so a deeper ring does not help; the
// time follows the bytes moved (skipping all of the arithmetic saves 5%).
// Which warp count wins depends on the clock a box holds: at 262,144 tokens
// 12 x 2 was 4% faster than 8 x 2 near 1,700 MHz and 4-7% slower at 1,870-1,950
// MHz; a 16-warp layout measured within +-3% of 12 x 2. Launches of at most
// kPipeFewTokens tokens use 8 x 2: at 32,768 tokens (a rank's share of the
// 262,144-token step at 8 GPUs, where the SMs run at their 1,965 MHz maximum)
// that took 0.1086 ms against 0.1173 ms for 12 x 2 (chunked M-RoPE, whose fp32
// rotation needs the warps, keeps 12).
template <typename W>
constexpr int pipe_max_warps() { return sizeof(W) == 4 ? 8 : 12; }
constexpr int pipe_max_warps(bool fp32_weights) { return fp32_weights ? 8 : 12; }
constexpr int pipe_max_stages(bool fp32_weights) { return fp32_weights ? 3 : 2; }
constexpr int kPipeFewTokenWarps = 8;
constexpr int64_t kPipeFewTokens = 65536;
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

// rotary alone (no norm, no store): the warp-per-token kernel of rope_rows.cu
bool rope_rows_eligible(const nib_qk_prologue_args& a);
int launch_rope_rows(const nib_qk_prologue_args& a, cudaStream_t st);

}  // namespace nib
