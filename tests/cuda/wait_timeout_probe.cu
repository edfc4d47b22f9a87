// Test-only probe of the kernels' failure path: an mbarrier wait on a phase
// that never completes must give up after the bounded wait, record its site
// code in the device status word and return, leaving the context usable.
#include "../../teenyformers_b200/csrc/sm100.cuh"

__global__ void wait_timeout_kernel(int* result) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    tfb::mbar_init(tfb::smem_u32(&bar), 1);  // nothing ever arrives
    abort_flag = 0;
    tfb::fence_mbar_init();
  }
  __syncthreads();
  const bool ok = tfb::mbar_wait(tfb::smem_u32(&bar), 0, &abort_flag, 77);
  if (threadIdx.x == 0) {
    result[0] = ok ? 1 : 0;
    result[1] = abort_flag;
    result[2] = tfb::g_device_status;
  }
}

__global__ void add_one_kernel(int* x) { x[3] += 1; }

extern "C" int wait_timeout_probe(int* result) {
  wait_timeout_kernel<<<1, 32>>>(result);
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  add_one_kernel<<<1, 1>>>(result);  // the context still runs work afterwards
  return cudaDeviceSynchronize() == cudaSuccess ? 0 : -2;
}
