// Self-test of the bounded mbarrier wait that every pipelined kernel of this library uses.
//
// The probe kernel waits on an mbarrier that nothing ever arrives on. The wait must give up
// after its cycle limit, record TLLM_DEV_WAIT_TIMEOUT + kSelftestSite in this file's device
// status word and return, leaving the CUDA context usable. No fault, trap or unbounded loop
// is involved.
#include "common.h"
#include "ptx.cuh"

namespace tllm {

__device__ int g_selftest_status = 0;

int selftest_read_status(int *out) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_selftest_status, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "cudaMemcpyFromSymbol(selftest status)");
  const int zero = 0;
  e = cudaMemcpyToSymbol(g_selftest_status, &zero, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "cudaMemcpyToSymbol(selftest status)");
  *out = v;
  return TLLM_OK;
}

namespace {

constexpr int kSelftestSite = 0x7F;

__global__ void bounded_wait_probe(long long limit_cycles) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // Phase 0 of `bar` never completes: this wait can only end by running out.
    mbar_wait_limit(smem_u32(&bar), 0, &abort_flag, &g_selftest_status,
                    TLLM_DEV_WAIT_TIMEOUT + kSelftestSite, limit_cycles);
  }
}

}  // namespace
}  // namespace tllm

extern "C" int tllm_selftest_bounded_wait(void *stream) {
  tllm::clear_error();
  // About 10 ms at B200 clocks: long enough to be unambiguous, short for a test.
  tllm::bounded_wait_probe<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(20000000LL);
  return tllm::cuda_status(cudaGetLastError(), "bounded_wait_probe launch");
}
