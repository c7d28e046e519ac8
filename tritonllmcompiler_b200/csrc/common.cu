// Status plumbing, device attribute cache and TMA descriptor encoding for libtllm_sm100a.so.
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.h"

namespace tllm {

namespace {
thread_local char t_last_error[512] = {0};

std::mutex g_attr_mutex;
int g_sm_count[64] = {0};

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
cudaError_t g_encode_status = cudaSuccess;
}  // namespace

int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { t_last_error[0] = 0; }

int cuda_status(cudaError_t err, const char *what) {
  if (err == cudaSuccess) return TLLM_OK;
  return fail(TLLM_ERR_CUDA, "%s failed: %s (%s)", what, cudaGetErrorName(err),
              cudaGetErrorString(err));
}

int current_device() {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cuda_status(e, "cudaGetDevice");
    return -1;
  }
  return dev;
}

int sm_count() {
  int dev = current_device();
  if (dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lock(g_attr_mutex);
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

namespace {
struct PreparedKernel {
  const void *kern;
  int dev, smem, threads, cluster_x;
  KernelLaunchInfo info;
};
std::mutex g_prepared_mutex;
std::vector<PreparedKernel> g_prepared;

// Everything a tensor map encodes; equal keys give identical maps (a map is a pure function of
// these), so a cached map is reused whatever memory the address belongs to now.
struct TmapKey {
  uint64_t base;
  uint64_t dims[5];
  uint64_t strides[4];
  uint32_t box[5];
  uint32_t dtype, rank, swizzle, pad;
};
struct TmapEntry {
  bool valid;
  TmapKey key;
  CUtensorMap map;
};
constexpr int kTmapCacheEntries = 32;
}  // namespace

int encode_tiled_uncached(CUtensorMap *map, CUtensorMapDataType dtype, uint32_t rank, void *base,
                          const uint64_t *dims, const uint64_t *strides_bytes, const uint32_t *box,
                          CUtensorMapSwizzle swizzle);

int prepare_kernel(const void *kern, int smem_bytes, int threads, int cluster_x,
                   KernelLaunchInfo *out) {
  const int dev = current_device();
  if (dev < 0) return TLLM_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_prepared_mutex);
  for (const PreparedKernel &p : g_prepared) {
    if (p.kern == kern && p.dev == dev && p.smem == smem_bytes && p.threads == threads &&
        p.cluster_x == cluster_x) {
      *out = p.info;
      return TLLM_OK;
    }
  }
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(dynamic shared memory)");
  cudaFuncAttributes fa;
  e = cudaFuncGetAttributes(&fa, kern);
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncGetAttributes");
  KernelLaunchInfo info{fa.numRegs, 0};
  if (cluster_x > 1) {
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_status(e, "cudaDeviceGetAttribute(SM count)");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(sms / cluster_x * cluster_x));
    cfg.blockDim = dim3(static_cast<unsigned>(threads));
    cfg.dynamicSmemBytes = static_cast<size_t>(smem_bytes);
    e = cudaOccupancyMaxActiveClusters(&info.resident, kern, &cfg);
    if (e != cudaSuccess) return cuda_status(e, "cudaOccupancyMaxActiveClusters");
  } else {
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&info.resident, kern, threads, smem_bytes);
    if (e != cudaSuccess) return cuda_status(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  }
  g_prepared.push_back(PreparedKernel{kern, dev, smem_bytes, threads, cluster_x, info});
  *out = info;
  return TLLM_OK;
}

int encode_tiled(CUtensorMap *map, CUtensorMapDataType dtype, uint32_t rank, void *base,
                 const uint64_t *dims, const uint64_t *strides_bytes, const uint32_t *box,
                 CUtensorMapSwizzle swizzle) {
  // Per-thread cache of recent maps: repeated calls on the same buffers (a decode loop, a
  // benchmark) skip the driver call.
  thread_local TmapEntry cache[kTmapCacheEntries] = {};
  thread_local int next_slot = 0;
  TmapKey key;
  memset(&key, 0, sizeof(key));
  key.base = reinterpret_cast<uint64_t>(base);
  for (uint32_t i = 0; i < rank && i < 5; ++i) {
    key.dims[i] = dims[i];
    key.box[i] = box[i];
    if (i + 1 < rank) key.strides[i] = strides_bytes[i];
  }
  key.dtype = static_cast<uint32_t>(dtype);
  key.rank = rank;
  key.swizzle = static_cast<uint32_t>(swizzle);
  for (int i = 0; i < kTmapCacheEntries; ++i) {
    if (cache[i].valid && memcmp(&cache[i].key, &key, sizeof(key)) == 0) {
      *map = cache[i].map;
      return TLLM_OK;
    }
  }
  const int rc = encode_tiled_uncached(map, dtype, rank, base, dims, strides_bytes, box, swizzle);
  if (rc) return rc;
  TmapEntry &slot = cache[next_slot];
  next_slot = (next_slot + 1) % kTmapCacheEntries;
  slot.valid = true;
  slot.key = key;
  slot.map = *map;
  return TLLM_OK;
}

int encode_tiled_uncached(CUtensorMap *map, CUtensorMapDataType dtype, uint32_t rank, void *base,
                          const uint64_t *dims, const uint64_t *strides_bytes, const uint32_t *box,
                          CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, [] {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    g_encode_status = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (g_encode_status == cudaSuccess && q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) {
    if (g_encode_status != cudaSuccess)
      return cuda_status(g_encode_status, "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
    return fail(TLLM_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  }
  // The driver call needs the device's context current on this thread; a thread that has
  // not made a runtime call yet (for example torch's autograd worker) may not have it, and
  // cudaSetDevice binds the primary context.
  {
    thread_local int bound_dev = -1;
    int dev = -1;
    if (cudaGetDevice(&dev) == cudaSuccess && dev != bound_dev) {
      cudaError_t e = cudaSetDevice(dev);
      if (e != cudaSuccess) return cuda_status(e, "cudaSetDevice");
      bound_dev = dev;
    }
  }
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult r = g_encode(map, dtype, rank, base, reinterpret_cast<const cuuint64_t *>(dims),
                        reinterpret_cast<const cuuint64_t *>(strides_bytes),
                        reinterpret_cast<const cuuint32_t *>(box), elem_strides,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(TLLM_ERR_INVALID, "cuTensorMapEncodeTiled failed (CUresult %d, rank %u)",
                static_cast<int>(r), rank);
  return TLLM_OK;
}

// Per-translation-unit device status readers (defined next to each kernel family).
int flash_read_status(int *out);
int swiglu_read_status(int *out);
int selftest_read_status(int *out);
int pkv_read_status(int *out);
int ppf_read_status(int *out);
int fbwd_read_status(int *out);
int swiglu8_read_status(int *out);
int qkv_read_status(int *out);
namespace paged {
int read_status(int *out);
}

int read_and_clear_device_status(int *out) {
  int (*readers[])(int *) = {flash_read_status, swiglu_read_status, paged::read_status,
                             selftest_read_status, pkv_read_status, ppf_read_status,
                             fbwd_read_status, swiglu8_read_status, qkv_read_status};
  int first = 0;
  for (auto rd : readers) {
    int v = 0;
    int rc = rd(&v);
    if (rc) return rc;
    if (!first) first = v;
  }
  *out = first;
  return TLLM_OK;
}

}  // namespace tllm

extern "C" {

const char *tllm_version(void) { return "0.2.0"; }

const char *tllm_last_error(void) { return tllm::t_last_error; }

int tllm_debug_status(int *out) {
  if (!out) return tllm::fail(TLLM_ERR_INVALID, "tllm_debug_status: out is null");
  tllm::clear_error();
  return tllm::read_and_clear_device_status(out);
}

// ---- CUDA IPC plumbing for peer output buffers (set-up, not the hot path) ----

int tllm_ipc_get_handle(const void *ptr, void *handle_out, uint64_t *offset_out) {
  tllm::clear_error();
  if (!ptr || !handle_out || !offset_out)
    return tllm::fail(TLLM_ERR_INVALID, "tllm_ipc_get_handle: null argument");
  static PFN_cuMemGetAddressRange_v3020 range_fn = nullptr;
  if (!range_fn) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
      return tllm::fail(TLLM_ERR_CUDA, "cuMemGetAddressRange is not available from the driver");
    range_fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range_fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return tllm::fail(TLLM_ERR_INVALID, "tllm_ipc_get_handle: pointer is not device memory");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
  if (e != cudaSuccess) return tllm::cuda_status(e, "cudaIpcGetMemHandle");
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = reinterpret_cast<uint64_t>(ptr) - static_cast<uint64_t>(base);
  return TLLM_OK;
}

int tllm_ipc_open(const void *handle, uint64_t offset, void **ptr_out, void **base_out) {
  tllm::clear_error();
  if (!handle || !ptr_out || !base_out)
    return tllm::fail(TLLM_ERR_INVALID, "tllm_ipc_open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void *base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return tllm::cuda_status(e, "cudaIpcOpenMemHandle");
  *base_out = base;
  *ptr_out = static_cast<char *>(base) + offset;
  return TLLM_OK;
}

int tllm_ipc_close(void *base) {
  tllm::clear_error();
  return tllm::cuda_status(cudaIpcCloseMemHandle(base), "cudaIpcCloseMemHandle");
}

int tllm_copy2d_async(void *dst, size_t dpitch, const void *src, size_t spitch, size_t width,
                      size_t height, void *stream) {
  tllm::clear_error();
  if (width == 0 || height == 0) return TLLM_OK;
  if (!dst || !src) return tllm::fail(TLLM_ERR_INVALID, "tllm_copy2d_async: null pointer");
  if (dpitch < width || spitch < width)
    return tllm::fail(TLLM_ERR_INVALID, "tllm_copy2d_async: pitch below the row width");
  return tllm::cuda_status(cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, height,
                                             cudaMemcpyDefault, static_cast<cudaStream_t>(stream)),
                           "cudaMemcpy2DAsync");
}

}  // extern "C"
