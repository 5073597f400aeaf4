// Allocation-free entry point for the dead-column mask + compaction (K1).
//
// gw_mask_compact needs a small zero-initialised scratch buffer from the caller.
// Some callers cannot provide one: code that runs where device allocation is
// not allowed or not safe -- an inference server that plans all device memory
// up front and treats any later cudaMalloc as a fault, a plugin loaded into a
// host process that owns every allocation itself, or a callback that runs
// while a caching allocator holds its lock. gw_mask_compact_static serves them:
// its scratch lives in a file-scope __device__ array below, which every GPU
// that loads this library holds (GW_MASK_STATIC_MAX_COLS / 8 bytes, ~128 KiB)
// until the process exits. No cudaMalloc / cudaFree or allocating library call
// is made on this path.
//
// The array's name in host code is only a host-side stand-in, not a device
// address, so the host fetches the real address with cudaGetSymbolAddress once
// per device (with that device current) and passes it to the kernel.
#include <mutex>

#include "gw_common.cuh"
#include "gw_internal.h"

namespace {

constexpr int64_t kMaxCols = GW_MASK_STATIC_MAX_COLS;
// Same layout as the caller-provided workspace: 16-byte ticket header, then one
// bit per column, rounded up to 256 bytes.
constexpr size_t kScratchBytes = ((16 + (kMaxCols + 31) / 32 * 4) + 255) / 256 * 256;

static __device__ __align__(256) uint32_t g_mask_static_scratch[kScratchBytes / sizeof(uint32_t)];

constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
void* g_static_addr[kMaxDevices] = {};

// Device address of the scratch array on `device` (which must be current).
cudaError_t static_scratch(int device, void** out) {
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (!g_static_addr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_mask_static_scratch);
    if (e != cudaSuccess) return e;
    g_static_addr[device] = p;
  }
  *out = g_static_addr[device];
  return cudaSuccess;
}

}  // namespace

extern "C" int gw_mask_compact_static(const void* x, int dtype, int64_t rows, int64_t cols,
                                      int64_t ld, double threshold, int32_t* mask,
                                      int64_t* alive_idx, int32_t* alive_count, void* stream) {
  if (dtype != GW_DTYPE_F16 && dtype != GW_DTYPE_BF16 && dtype != GW_DTYPE_F32) return GW_ERR_DTYPE;
  if (rows < 0 || cols < 0 || ld < 0 || (rows > 1 && ld < cols)) return GW_ERR_SHAPE;
  // Sizes beyond the static scratch are rejected before anything is launched.
  if (cols > kMaxCols) return GW_ERR_WORKSPACE;
  // Errors take the same route as gw_mask_compact's: gw::current_device and
  // gw::cuda_fail record the CUDA error text for gw_last_cuda_error and clear
  // the runtime's pending error.
  const gw::DeviceInfo* d = nullptr;
  int dev = -1;
  int st = gw::current_device(&d, &dev);
  if (st != GW_OK) return st;
  if (dev >= kMaxDevices) return GW_ERR_DEVICE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (cols == 0) {
    if (alive_count) {
      e = cudaMemsetAsync(alive_count, 0, sizeof(int32_t), s);
      if (e != cudaSuccess) return gw::cuda_fail(e);
    }
    return GW_OK;
  }
  if (rows > 0 && !x) return GW_ERR_NULL;
  void* scratch = nullptr;
  e = static_scratch(dev, &scratch);
  if (e != cudaSuccess) return gw::cuda_fail(e);
  // The array keeps whatever the previous call left; the kernel needs the
  // ticket and flag words it uses to start at zero.
  const size_t used = gw::mask_workspace_bytes(cols);
  e = cudaMemsetAsync(scratch, 0, used, s);
  if (e != cudaSuccess) return gw::cuda_fail(e);
  e = gw::launch_mask_compact(x, dtype, rows, cols, ld, static_cast<float>(threshold), mask,
                              alive_idx, alive_count, scratch, d->sm_count, s);
  return e == cudaSuccess ? GW_OK : gw::cuda_fail(e);
}
