// diag.cuh -- small self-checks of device building blocks the hot kernels rely on, run
// through the C ABI by the GPU tests:
//   k_diag_wait_timeout  the abort path of a bounded mbarrier wait: a wait on a barrier
//                        that nothing completes gives up after the host-given limit,
//                        records the fault (beacon_device_status), lets the bulk copy the
//                        kernel has in flight land, frees its TMEM and returns;
//   k_diag_exp2_poly     the FMA-pipe exponential of the attention softmax (exp2_poly2)
//                        evaluated on host-given arguments, to be checked against 2^x.
#pragma once

#include "attention.cuh"
#include "sm100.cuh"

namespace beacon {

enum : unsigned int {
  kSiteDiagWait = 0x501,   // the wait that is meant to run out
  kSiteDiagDrain = 0x502,  // the wait for the kernel's own copy in flight
};

__device__ __align__(16) uint32_t g_diag_src[4] = {1u, 2u, 3u, 4u};

// One warp.  out[0] = 1 if the wait gave up (it must), out[1] = the first word of the
// copy that landed (1), out[2] = 1 once TMEM was released.
__global__ void __launch_bounds__(32, 1) k_diag_wait_timeout(uint64_t limit_ns, uint32_t* out) {
  __shared__ __align__(16) uint32_t buf[4];
  __shared__ uint64_t bar_copy, bar_never;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar_copy, 1);
    mbar_init(&bar_never, 1);  // nothing ever arrives on it
    abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncwarp();
  tmem_alloc(&tmem_slot, 32);
  tmem_relinquish();
  tc_fence_before();
  __syncwarp();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&bar_copy, 16);
    bulk_load(buf, g_diag_src, 16, &bar_copy);
  }
  __syncwarp();
  const bool got = __all_sync(0xffffffffu, mbar_wait_for(&bar_never, 0, &abort_flag, kSiteDiagWait, limit_ns));
  // abort path: the copy this kernel issued must land before it may exit (its own wait is
  // bounded as well, by the same limit)
  volatile int no_abort = 0;
  const bool landed = __all_sync(0xffffffffu, mbar_wait_for(&bar_copy, 0, &no_abort, kSiteDiagDrain, limit_ns));
  tc_fence_before();
  __syncwarp();
  tc_fence_after();
  tmem_dealloc(tmem, 32);
  if (threadIdx.x == 0) {
    out[0] = got ? 0u : 1u;
    out[1] = landed ? buf[0] : 0u;
    out[2] = 1u;
  }
}

// out[i] = exp2_poly2(in[i]); n even.
__global__ void k_diag_exp2_poly(float* __restrict__ out, const float* __restrict__ in, long long n) {
  for (long long i = 2 * ((long long)blockIdx.x * blockDim.x + threadIdx.x); i + 1 < n;
       i += 2LL * gridDim.x * blockDim.x) {
    float r0, r1;
    exp2_poly2(r0, r1, in[i], in[i + 1]);
    out[i] = r0;
    out[i + 1] = r1;
  }
}

}  // namespace beacon
