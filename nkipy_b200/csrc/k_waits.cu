// The budget of the kernels' waits on counters that other ranks or other
// CTAs advance, and a probe of that bounded wait.
//
// A kernel that waits for another rank (the fused GEMM + all-reduce waiting
// for row-block arrival counts, the in-switch all-reduce's barrier) polls the
// counter for at most wait_limit_cycles(); when the budget runs out it raises
// its device error flag, leaves the wait and returns, so a rank that died or
// never launched turns into an error status (nkb_device_error) instead of a
// hung GPU.  nkb_wait_probe runs the same bounded wait on a caller-supplied
// counter, so the expiry path can be exercised on one GPU with a counter that
// nothing advances.
#include <algorithm>
#include <atomic>

#include "common.cuh"

namespace nkb {
namespace waits {

__device__ int g_error = 0;
std::atomic<unsigned long long> g_limit_us{1000000};  // 1 s

__global__ void probe_kernel(const uint32_t *counter, uint32_t target, long long limit) {
  if (threadIdx.x == 0 && !wait_counter_geq(counter, target, limit, nullptr, 1000)) atomicExch(&g_error, 1);
}

}  // namespace waits

long long wait_limit_cycles() {
  int dev = 0, khz = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, dev) != cudaSuccess ||
      khz <= 0)
    khz = 1965000;  // B200 maximum SM clock
  // cycles at the maximum clock: at a lower clock the wait lasts longer, never shorter
  const unsigned long long us = waits::g_limit_us.load();
  const long double cyc = (long double)us * (long double)khz / 1000.0L;
  return cyc > 9.0e18L ? (long long)9000000000000000000LL : std::max<long long>(1, (long long)cyc);
}

int wait_probe_launch(const uint32_t *counter, uint32_t target, cudaStream_t stream) {
  if (!counter) return fail(NKB_ERR_INVALID, "counter is NULL");
  if (reinterpret_cast<uintptr_t>(counter) & 3) return fail(NKB_ERR_INVALID, "counter not 4-byte aligned");
  waits::probe_kernel<<<1, 32, 0, stream>>>(counter, target, wait_limit_cycles());
  return launch_status("probe_kernel");
}

int waits_read_and_clear_error(int *flag) {
  int zero = 0;
  NKB_CUDA_TRY(cudaMemcpyFromSymbol(flag, waits::g_error, sizeof(int)));
  if (*flag) NKB_CUDA_TRY(cudaMemcpyToSymbol(waits::g_error, &zero, sizeof(int)));
  return NKB_OK;
}

}  // namespace nkb

extern "C" int nkb_set_wait_limit_us(uint64_t us) {
  if (us == 0) return nkb::fail(NKB_ERR_INVALID, "wait limit must be positive");
  nkb::waits::g_limit_us.store(us);
  return NKB_OK;
}

extern "C" int nkb_get_wait_limit_us(uint64_t *us) {
  if (!us) return nkb::fail(NKB_ERR_INVALID, "us is NULL");
  *us = nkb::waits::g_limit_us.load();
  return NKB_OK;
}

