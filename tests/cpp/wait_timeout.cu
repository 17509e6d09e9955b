// Test harness (not part of the library): runs the library's own bounded
// mbarrier wait (vb::mbar_wait_bounded, verbo_b200/csrc/device.cuh) on a
// barrier that nothing ever arrives on, so the wait must give up after its
// limit and report it, leaving the CUDA context usable.  No fault, no trap:
// the kernel simply returns with a flag set.
#include <cuda_runtime.h>

#include "device.cuh"

namespace {

__global__ void never_arrives(unsigned* gave_up, unsigned long long* waited_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) vb::mbar_init(&bar, 1);  // one arrival expected, none made
  __syncthreads();
  const unsigned long long t0 = vb::gtimer();
  const bool done = vb::mbar_wait_bounded(&bar, 0);
  if (threadIdx.x == 0) {
    *gave_up = done ? 0u : 1u;
    *waited_ns = vb::gtimer() - t0;
  }
}

}  // namespace

// Returns a cudaError_t value; *gave_up is 1 when the wait ran out.
extern "C" int run_wait_timeout(unsigned* gave_up, unsigned long long* waited_ns, unsigned long long* limit_ns) {
  unsigned* d_flag = nullptr;
  unsigned long long* d_ns = nullptr;
  cudaError_t e = cudaMalloc(&d_flag, sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMalloc(&d_ns, sizeof(unsigned long long));
  if (e == cudaSuccess) {
    never_arrives<<<1, 32>>>(d_flag, d_ns);
    e = cudaDeviceSynchronize();
  }
  if (e == cudaSuccess) e = cudaMemcpy(gave_up, d_flag, sizeof(unsigned), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemcpy(waited_ns, d_ns, sizeof(unsigned long long), cudaMemcpyDeviceToHost);
  *limit_ns = vb::kWaitLimitNs;
  cudaFree(d_flag);
  cudaFree(d_ns);
  return static_cast<int>(e);
}
