// rt_selftest_bounded_wait: exercises the failure path every kernel of the
// library shares, without a fault.
//
// One block of four warps allocates tensor memory as the attention kernels
// do, then warp 1 waits on an mbarrier that nothing ever arrives at, through
// the same bounded wait (mbar_wait_limit) the kernels use, with a short
// limit. When it runs out the wait raises the block's abort flag and the
// sticky RT_ERR_TIMEOUT device status; warps 2 and 3, parked on a second
// barrier that nothing completes either, must then leave at once through the
// abort flag (not through their own, much longer, limit); the block frees its
// tensor memory and exits. The host reads the status with rt_device_status()
// and the context stays usable.

namespace rt {
namespace selftest {

__global__ void __launch_bounds__(128, 1) bounded_wait_kernel(long long limit_cycles, int32_t* report) {
  __shared__ __align__(8) uint64_t never[2];
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_flag;
  __shared__ long long waited[4];
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&never[0], 1);
    mbar_init(&never[1], 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base_s, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const long long t0 = clock64();
  bool ok = true;
  if (warp == 1) {
    ok = __all_sync(0xFFFFFFFFu, mbar_wait_limit(&never[0], 0, &abort_flag, limit_cycles));
  } else if (warp >= 2) {
    // ten times the limit: these waits may only end through the abort flag
    ok = __all_sync(0xFFFFFFFFu, mbar_wait_limit(&never[1], 0, &abort_flag, 10 * limit_cycles));
  }
  if ((threadIdx.x & 31) == 0) waited[warp] = ok ? -1 : clock64() - t0;
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base_s, 32);
  }
  if (threadIdx.x == 0) {
    // report: [0] abort flag, [1] waits that gave up (of 3), [2] SM clocks the
    // running-out wait took (millions), [3] the longest of the others' (millions)
    report[0] = abort_flag;
    report[1] = (waited[1] >= 0) + (waited[2] >= 0) + (waited[3] >= 0);
    report[2] = (int32_t)(waited[1] / 1000000);
    report[3] = (int32_t)(max(waited[2], waited[3]) / 1000000);
  }
}

}  // namespace selftest
}  // namespace rt

extern "C" int rt_selftest_bounded_wait(int64_t limit_cycles, int32_t* report, void* stream) {
  using namespace rt;
  if (!report || limit_cycles <= 0 || limit_cycles > RT_WAIT_CYCLES) return RT_ERR_INVALID_ARGUMENT;
  DeviceGuard guard(report);
  if (guard.status() != RT_OK) return guard.status();
  selftest::bounded_wait_kernel<<<1, 128, 0, static_cast<cudaStream_t>(stream)>>>(limit_cycles, report);
  return check_launch("bounded_wait_kernel launch");
}
