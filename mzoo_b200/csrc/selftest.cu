// Self-test of the bounded device waits every kernel of this library relies on.
//
// Every mbarrier wait in the kernels (tc::mbar_wait / tc::mbar_wait_cl) gives up after a
// time limit, records a site code in the caller's error word and lets the kernel drain
// and return, so that a bug shows up as an error status instead of a hung GPU.  This
// entry point exercises exactly that path on purpose: one thread waits on an mbarrier that
// nothing ever arrives on, with a short limit; the wait must run out, write its code
// (901 for the CTA-scope wait, 902 for the cluster-scope one) and the kernel must exit
// normally, leaving the context usable.  No fault, trap or endless loop is involved.
#include "tc.cuh"

namespace mzb {
namespace selftest {

constexpr int CODE_CTA = 901, CODE_CLUSTER = 902;

__global__ void bounded_wait_kernel(long long limit_ns, int scope, int* err) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (scope == 0)
      tc::mbar_wait(&bar, 0, err, CODE_CTA, uint64_t(limit_ns));
    else
      tc::mbar_wait_cl(&bar, 0, err, CODE_CLUSTER, uint64_t(limit_ns));
  }
}

}  // namespace selftest
}  // namespace mzb

extern "C" int mzb_selftest_bounded_wait(int64_t limit_ns, int scope, int* err, void* stream) {
  MZB_REQUIRE(limit_ns > 0 && limit_ns <= 2000000000LL, MZB_ERR_SHAPE,
              "selftest_bounded_wait: limit_ns=%lld must be in (0, 2e9]", (long long)limit_ns);
  MZB_REQUIRE(scope == 0 || scope == 1, MZB_ERR_SHAPE, "selftest_bounded_wait: scope must be 0 (cta) or 1 (cluster)");
  MZB_REQUIRE(err != nullptr, MZB_ERR_SHAPE, "selftest_bounded_wait: needs an error word");
  mzb::selftest::bounded_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns, scope, err);
  return mzb::launch_status("selftest_bounded_wait");
}
