// Host-side plumbing shared by every entry point of libtllm_sm100a.so: status strings,
// per-device attribute cache, and TMA tensor-map encoding through the driver entry point
// (so the library does not link libcuda directly).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstddef>

#include "../../include/tllm_sm100.h"

namespace tllm {

// Records a formatted message as the calling thread's last error and returns `code`.
int fail(int code, const char *fmt, ...);
// Clears the calling thread's last error.
void clear_error();
// Maps a CUDA runtime status to TLLM_ERR_CUDA with context; TLLM_OK when err == success.
int cuda_status(cudaError_t err, const char *what);

// Number of SMs of the current device (cached per device, thread-safe).
int sm_count();
// Current device ordinal (or -1 with the last error set).
int current_device();

// cuTensorMapEncodeTiled resolved once through cudaGetDriverEntryPoint.
int encode_tiled(CUtensorMap *map, CUtensorMapDataType dtype, uint32_t rank, void *base,
                 const uint64_t *dims, const uint64_t *strides_bytes, const uint32_t *box,
                 CUtensorMapSwizzle swizzle);

// Launch attributes of one kernel on the current device: its register count and how many of
// its CTAs (cluster_x == 1) or clusters (cluster_x > 1) can be resident at once.
struct KernelLaunchInfo {
  int num_regs;
  int resident;
};
// Once per (kernel, device, dynamic shared memory, threads, cluster width): raises the kernel's
// dynamic shared memory limit to smem_bytes and reads its launch attributes; later calls return
// the cached values without driver calls (the per-call host cost of small launches).
int prepare_kernel(const void *kern, int smem_bytes, int threads, int cluster_x,
                   KernelLaunchInfo *out);

// Device error word (one per device image): kernels that give up on a bounded wait
// record a TLLM_DEV_* code here instead of hanging.
int read_and_clear_device_status(int *out);

}  // namespace tllm

#define TLLM_CHECK_ARG(cond, ...)                          \
  do {                                                     \
    if (!(cond)) return ::tllm::fail(TLLM_ERR_INVALID, __VA_ARGS__); \
  } while (0)

#define TLLM_CUDA_TRY(expr)                                        \
  do {                                                             \
    cudaError_t e__ = (expr);                                      \
    if (e__ != cudaSuccess) return ::tllm::cuda_status(e__, #expr); \
  } while (0)
