// Self-test of the bounded bulk-copy wait (nib_selftest_bounded_wait).
//
// The pipelined prologue (prologue_pipe.cu) waits on an mbarrier for each
// token's bulk copy. If the bytes never arrive, the wait gives up after its
// limit, the warp flags kDevTimeout, waits (again bounded) for its other copies
// in flight and returns. This kernel runs that same sequence on purpose, with
// a caller-chosen short limit: stage 0 is armed for more bytes than its copy
// brings, so its phase never completes; stage 1 is an ordinary copy that the
// drain waits for. No spin is unbounded and no copy is left in flight, so the
// kernel returns and the context stays usable.
#include "bulk_copy.cuh"

namespace nib {

__global__ void bounded_wait_selftest_kernel(const unsigned char* __restrict__ src,
                                             unsigned long long limit_ns, unsigned int* status,
                                             int* drained) {
  __shared__ __align__(16) unsigned char buf[2][16];
  __shared__ __align__(8) uint64_t bars[2];
  const int lane = threadIdx.x & 31;
  pdl_enter();
  if (lane == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (lane == 0) {
    fence_proxy_async();
    mbar_arrive_expect_tx(&bars[0], 32);  // 16 of these 32 bytes will never come
    bulk_load(buf[0], src, 16, &bars[0]);
    mbar_arrive_expect_tx(&bars[1], 16);
    bulk_load(buf[1], src + 16, 16, &bars[1]);
  }
  const bool ok = mbar_wait(&bars[0], 0, limit_ns);
  if (!__all_sync(0xffffffffu, ok)) {
    if (lane == 0) flag(status, kDevTimeout);
    // the same drain as the prologue: let the warp's other copy land, bounded
    const bool landed = mbar_wait(&bars[1], 0, limit_ns);
    if (lane == 0) *drained = landed && buf[1][0] == src[16] ? 1 : 0;
    return;
  }
  if (lane == 0) *drained = -1;  // the incomplete phase completed: must not happen
}

}  // namespace nib

using namespace nib;

extern "C" int nib_selftest_bounded_wait(const void* src, int64_t limit_ns, unsigned int* status,
                                         int* drained, void* stream) {
  NIB_REQUIRE(src && status && drained, "selftest_bounded_wait: null pointer");
  NIB_REQUIRE(reinterpret_cast<uintptr_t>(src) % 16 == 0, "selftest_bounded_wait: src must be 16-byte aligned");
  NIB_REQUIRE(limit_ns >= 1000 && limit_ns <= static_cast<int64_t>(kWaitLimitNs),
              "selftest_bounded_wait: limit_ns must be within [1 us, 2 s]");
  ::nib::launch_k(bounded_wait_selftest_kernel, 1, 32, 0, as_stream(stream),
      static_cast<const unsigned char*>(src), static_cast<unsigned long long>(limit_ns), status,
      drained);
  return launch_status("selftest_bounded_wait");
}
