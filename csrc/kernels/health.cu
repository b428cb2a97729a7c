// Device-side health probe for failure detection.
//
// `wait_flag_probe` waits for *flag >= expected (system-scope acquire loads) for at most
// `timeout_ns` of global time, exactly as the fused-collective kernels wait for peers. On a
// timeout it records (code 3, site 99) in the device error word and returns, so the context
// stays usable and the host sees the failure on its next check. It is what the failure-
// detection tests drive with a flag nothing sets, and what a runtime can launch to ask whether
// a peer signalled within a deadline. No trap, no unbounded loop.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace hrm {
namespace {

__device__ __forceinline__ int ld_acquire_sys_i32(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void wait_flag_probe_kernel(const int* flag, int expected, unsigned long long timeout_ns, int* status,
                                       int* err) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const unsigned long long t0 = globaltimer_ns();
  while (ld_acquire_sys_i32(flag) < expected) {
    if (globaltimer_ns() - t0 > timeout_ns) {
      *status = 1;
      report_error(err, kErrPeerWaitTimeout, 99);
      return;
    }
    __nanosleep(1000);
  }
  *status = 0;
}

}  // namespace

at::Tensor device_error_word();

// Returns a device int32 status (0 = flag seen, 1 = timed out); never blocks the host.
at::Tensor wait_flag_probe(const at::Tensor& flag, int64_t expected, double timeout_s) {
  TORCH_CHECK(flag.is_cuda() && flag.scalar_type() == at::kInt && flag.numel() >= 1, "flag: CUDA int32 tensor");
  TORCH_CHECK(timeout_s > 0 && timeout_s <= 5.0, "probe timeout must be in (0, 5] seconds");
  c10::cuda::CUDAGuard guard(flag.device());
  auto status = at::full({1}, -1, flag.options());
  wait_flag_probe_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      flag.data_ptr<int>(), (int)expected, (unsigned long long)(timeout_s * 1e9), status.data_ptr<int>(),
      device_error_word().data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return status;
}

}  // namespace hrm
