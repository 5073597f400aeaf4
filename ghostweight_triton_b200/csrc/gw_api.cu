// C-ABI layer: argument validation, per-device set-up and kernel dispatch.
// Declarations (with the reference interface each entry point replaces) are in
// include/ghostweight_b200.h.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "gw_common.cuh"
#include "gw_internal.h"

// Module-wide device error word (GW_DEVICE_ERR_* bits). Kernels receive its
// device address, fetched once per device with cudaGetSymbolAddress.
__device__ unsigned int g_gw_device_error = 0;
// A counter no code ever increments: the wait of gw_selftest_wait_timeout.
__device__ unsigned int g_gw_never_set = 0;

namespace gw {
namespace {
// gw_selftest_wait_timeout: both waits can only end by running out of time.
__global__ void selftest_wait_kernel(unsigned long long limit_ns, unsigned int* err) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  const uint32_t b = smem_u32(&bar);
  mbar_init(b, 1);               // one arrival expected, none ever made
  mbar_init_fence();
  mbar_wait(b, 0u, nullptr, err, limit_ns);
  wait_counter_geq(&g_gw_never_set, 1u, nullptr, err, limit_ns);
}
}  // namespace
}  // namespace gw

namespace gw {

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
DeviceInfo g_info[kMaxDevices];
bool g_ready[kMaxDevices] = {};
}  // namespace

thread_local char g_cuda_msg[256] = "no error";

const DeviceInfo* device_info(int device) {
  if (device < 0 || device >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_ready[device]) return &g_info[device];
  DeviceInfo d;
  if (cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    return nullptr;
  if (cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess)
    return nullptr;
  if (cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess)
    return nullptr;
  if (d.cc_major == 10) {
    void* p = nullptr;
    // `device` is the current device here (callers pass cudaGetDevice()).
    if (cudaGetSymbolAddress(&p, g_gw_device_error) != cudaSuccess) return nullptr;
    d.err_word = static_cast<unsigned int*>(p);
  }
  g_info[device] = d;
  g_ready[device] = true;
  return &g_info[device];
}

void* tensor_map_encoder() {
  static void* fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = f;
  });
  return fn;
}

bool make_tmap_kmajor(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld,
                      int box_cols, int box_rows) {
  // A few recently encoded maps per host thread: the packed weight and the
  // reused workspace recur from call to call, and encoding is a driver call.
  struct Entry {
    const void* base;
    int64_t rows, cols, ld;
    int box_cols, box_rows;
    CUtensorMap map;
  };
  constexpr int kCache = 8;
  thread_local Entry cache[kCache];
  thread_local int filled = 0, next = 0;
  for (int i = 0; i < filled; ++i) {
    const Entry& e = cache[i];
    if (e.base == base && e.rows == rows && e.cols == cols && e.ld == ld &&
        e.box_cols == box_cols && e.box_rows == box_rows) {
      *map = e.map;
      return true;
    }
  }
  using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                     const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                     const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                     CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  auto encode = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!encode) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2u};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  if (encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides,
             box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  Entry& e = cache[next];
  e = Entry{base, rows, cols, ld, box_cols, box_rows, *map};
  next = (next + 1) % kCache;
  if (filled < kCache) ++filled;
  return true;
}

}  // namespace gw

namespace gw {

int cuda_fail(cudaError_t e) {
  // Clear the error the runtime keeps for this thread, so the next call of
  // this library does not see it again.
  cudaGetLastError();
  std::snprintf(g_cuda_msg, sizeof(g_cuda_msg), "%s: %s", cudaGetErrorName(e),
                cudaGetErrorString(e));
  return GW_ERR_CUDA;
}

int current_device(const DeviceInfo** out, int* device) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e);
  const DeviceInfo* d = device_info(dev);
  if (!d) {
    e = cudaGetLastError();
    return cuda_fail(e != cudaSuccess ? e : cudaErrorInvalidDevice);
  }
  if (d->cc_major != 10 || !d->err_word) return GW_ERR_DEVICE;
  *out = d;
  if (device) *device = dev;
  return GW_OK;
}

}  // namespace gw

namespace {

using gw::cuda_fail;
using gw::current_device;

bool valid_dtype(int dt) { return dt == GW_DTYPE_F16 || dt == GW_DTYPE_BF16 || dt == GW_DTYPE_F32; }
bool valid_epi(int e) { return e == GW_EPI_NONE || e == GW_EPI_GELU_ERF || e == GW_EPI_GELU_TANH; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
// A [rows, cols] matrix with leading dimension ld is well-formed.
bool matrix_ok(int64_t rows, int64_t cols, int64_t ld) {
  return rows >= 0 && cols >= 0 && ld >= 0 && (rows <= 1 || ld >= cols);
}

}  // namespace

extern "C" {

const char* gw_status_string(int status) {
  switch (status) {
    case GW_OK: return "ok";
    case GW_ERR_SHAPE: return "invalid shape or leading dimension";
    case GW_ERR_DTYPE: return "unsupported dtype";
    case GW_ERR_ALIGN: return "pointer or leading dimension not aligned as required";
    case GW_ERR_NULL: return "required pointer is NULL";
    case GW_ERR_WORKSPACE: return "workspace missing or too small";
    case GW_ERR_CUDA: return "CUDA error";
    case GW_ERR_DEVICE: return "current device is not an sm_100 (B200) GPU";
    case GW_ERR_UNSUPPORTED: return "unsupported configuration";
    default: return "unknown status";
  }
}

const char* gw_last_cuda_error(void) { return gw::g_cuda_msg; }

const char* gw_version(void) { return "0.1.0"; }

int gw_device_supported(int device) {
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return major == 10 ? 1 : 0;
}

int gw_get_device_error(int reset, unsigned int* out) {
  if (!out) return GW_ERR_NULL;
  const gw::DeviceInfo* d = nullptr;
  int st = current_device(&d);
  if (st != GW_OK) return st;
  cudaError_t e = cudaMemcpyFromSymbol(out, g_gw_device_error, sizeof(unsigned int));
  if (e != cudaSuccess) return cuda_fail(e);
  if (reset) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_gw_device_error, &zero, sizeof(unsigned int));
    if (e != cudaSuccess) return cuda_fail(e);
  }
  return GW_OK;
}

size_t gw_mask_workspace_bytes(int64_t cols) {
  return gw::mask_workspace_bytes(cols < 0 ? 0 : cols);
}

int gw_mask_compact(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld,
                    double threshold, int32_t* mask, int64_t* alive_idx, int32_t* alive_count,
                    void* workspace, size_t workspace_bytes, void* stream) {
  if (!valid_dtype(dtype)) return GW_ERR_DTYPE;
  if (!matrix_ok(rows, cols, ld) || cols > 0x7FFFFFFFll) return GW_ERR_SHAPE;
  const gw::DeviceInfo* d = nullptr;
  int st = current_device(&d);
  if (st != GW_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cols == 0) {
    if (alive_count) {
      cudaError_t e = cudaMemsetAsync(alive_count, 0, sizeof(int32_t), s);
      if (e != cudaSuccess) return cuda_fail(e);
    }
    return GW_OK;
  }
  if (rows > 0 && !x) return GW_ERR_NULL;
  if (!workspace) return GW_ERR_NULL;
  if (workspace_bytes < gw::mask_workspace_bytes(cols)) return GW_ERR_WORKSPACE;
  if (!aligned16(workspace)) return GW_ERR_ALIGN;
  // The reference passes the threshold as an fp32 kernel scalar (mask.py:100).
  const float thr = static_cast<float>(threshold);
  cudaError_t e = gw::launch_mask_compact(x, dtype, rows, cols, ld, thr, mask, alive_idx,
                                          alive_count, workspace, d->sm_count, s);
  return e == cudaSuccess ? GW_OK : cuda_fail(e);
}

int gw_gather_columns(const void* src, int dtype, int64_t rows, int64_t cols, int64_t ld_src,
                      const int64_t* idx, int64_t n_idx, void* dst, int64_t ld_dst,
                      int64_t pad_to, void* stream) {
  if (!valid_dtype(dtype)) return GW_ERR_DTYPE;
  if (!matrix_ok(rows, cols, ld_src) || n_idx < 0 || pad_to < n_idx ||
      !matrix_ok(rows, pad_to, ld_dst))
    return GW_ERR_SHAPE;
  const gw::DeviceInfo* d = nullptr;
  int st = current_device(&d);
  if (st != GW_OK) return st;
  if (rows == 0 || pad_to == 0) return GW_OK;
  if (!dst || (n_idx > 0 && (!src || !idx))) return GW_ERR_NULL;
  cudaError_t e = gw::launch_gather_columns(src, dtype, rows, ld_src, cols, idx, n_idx, dst,
                                            ld_dst, pad_to, d->err_word, d->sm_count,
                                            static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? GW_OK : cuda_fail(e);
}

int gw_gather_columns_dev(const void* src, int dtype, int64_t rows, int64_t cols, int64_t ld_src,
                          const int64_t* idx, int64_t n_idx_max, const int32_t* n_idx_dev,
                          void* dst, int64_t ld_dst, int64_t pad_to, void* stream) {
  if (!valid_dtype(dtype)) return GW_ERR_DTYPE;
  if (!matrix_ok(rows, cols, ld_src) || n_idx_max < 0 || n_idx_max > 0x7FFFFFFFll ||
      pad_to < n_idx_max || !matrix_ok(rows, pad_to, ld_dst))
    return GW_ERR_SHAPE;
  const gw::DeviceInfo* d = nullptr;
  int st = current_device(&d);
  if (st != GW_OK) return st;
  if (rows == 0 || pad_to == 0) return GW_OK;
  if (!dst || !n_idx_dev || (n_idx_max > 0 && (!src || !idx))) return GW_ERR_NULL;
  cudaError_t e = gw::launch_gather_columns(src, dtype, rows, ld_src, cols, idx, n_idx_max, dst,
                                            ld_dst, pad_to, d->err_word, d->sm_count,
                                            static_cast<cudaStream_t>(stream), false, n_idx_dev);
  return e == cudaSuccess ? GW_OK : cuda_fail(e);
}

int gw_gather_rows(const void* src, int dtype, int64_t rows, int64_t cols, int64_t ld_src,
                   const int64_t* idx, int64_t n_idx, void* dst, int64_t ld_dst, void* stream) {
  if (!valid_dtype(dtype)) return GW_ERR_DTYPE;
  if (!matrix_ok(rows, cols, ld_src) || n_idx < 0 || !matrix_ok(n_idx, cols, ld_dst))
    return GW_ERR_SHAPE;
  const gw::DeviceInfo* d = nullptr;
  int st = current_device(&d);
  if (st != GW_OK) return st;
  if (n_idx == 0 || cols == 0) return GW_OK;
  if (!src || !idx || !dst) return GW_ERR_NULL;
  cudaError_t e = gw::launch_gather_rows(src, dtype, rows, cols, ld_src, idx, n_idx, dst, ld_dst,
                                         d->err_word, d->sm_count,
                                         static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? GW_OK : cuda_fail(e);
}

int gw_gather_rows_t(const void* src, int dtype, int64_t rows, int64_t cols, int64_t ld_src,
                     const int64_t* idx, int64_t n_idx, void* dst, int64_t ld_dst,
                     int64_t pad_to, void* stream) {
  if (!valid_dtype(dtype)) return GW_ERR_DTYPE;
  if (!matrix_ok(rows, cols, ld_src) || n_idx < 0 || pad_to < n_idx ||
      !matrix_ok(cols, pad_to, ld_dst))
    return GW_ERR_SHAPE;
  const gw::DeviceInfo* d = nullptr;
  int st = current_device(&d);
  if (st != GW_OK) return st;
  if (cols == 0 || pad_to == 0) return GW_OK;
  if (!dst || (n_idx > 0 && (!src || !idx))) return GW_ERR_NULL;
  cudaError_t e = gw::launch_gather_rows_t(src, dtype, rows, cols, ld_src, idx, n_idx, dst,
                                           ld_dst, pad_to, d->err_word,
                                           static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? GW_OK : cuda_fail(e);
}

namespace {
// GEMM workspace layout: [header: the in-kernel gather's epoch, claim counters
// and unit flags, 256-aligned][x' = M x ldp, 16-bit]. Its contents on entry
// do not matter (the overlap strategy tags its flags with a call number).
int64_t gemm_ld_pad(int64_t n_alive) { return (n_alive + 63) / 64 * 64; }
size_t gemm_ws_header(int64_t M, int64_t n_alive) { return gw::tc2_gather_header_bytes(M, n_alive); }
}  // namespace

int gw_gather_rows_t_dev(const void* src, int dtype, int64_t rows, int64_t cols, int64_t ld_src,
                         const int64_t* idx, int64_t n_idx_max, const int32_t* n_idx_dev,
                         void* dst, int64_t ld_dst, int64_t pad_to, void* stream) {
  if (!valid_dtype(dtype)) return GW_ERR_DTYPE;
  if (!matrix_ok(rows, cols, ld_src) || n_idx_max < 0 || n_idx_max > 0x7FFFFFFFll ||
      pad_to < n_idx_max || !matrix_ok(cols, pad_to, ld_dst))
    return GW_ERR_SHAPE;
  const gw::DeviceInfo* d = nullptr;
  int st = current_device(&d);
  if (st != GW_OK) return st;
  if (cols == 0 || pad_to == 0) return GW_OK;
  if (!dst || !n_idx_dev || (n_idx_max > 0 && (!src || !idx))) return GW_ERR_NULL;
  cudaError_t e = gw::launch_gather_rows_t(src, dtype, rows, cols, ld_src, idx, n_idx_max, dst,
                                           ld_dst, pad_to, d->err_word,
                                           static_cast<cudaStream_t>(stream), n_idx_dev);
  return e == cudaSuccess ? GW_OK : cuda_fail(e);
}

namespace {
// GW_DECODE_GEMM=0 turns the decode-shaped kernel off (A/B measurements).
bool decode_gemm_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("GW_DECODE_GEMM");
    return !(v && v[0] == '0');
  }();
  return on;
}

// Dense-A GEMM y = act(a @ w^T + bias) on the kernel that suits the shape:
// the CTA-pair kernel when there are enough 256 x 256 tiles for every SM
// pair; for at most 32 rows the decode kernel (features on the MMA's M side,
// split-K in a cluster); cluster split-K when the output has too few tiles to
// occupy half of the SMs; else the single-CTA persistent kernel.
// With peers, the output is also written into each peer buffer: by the pair
// kernel's epilogue, tile by tile, or by a copy kernel after the other kernels.
// With a_cols, a is x [M, a_width] and K the count of alive columns, which form
// 64-column runs starting at a_cols[64 j] (GW_GEMM_RUNS).
struct GemmChoice {
  int kernel = GW_KERNEL_SINGLE;
  gw::DecodePlan dp;
  gw::SplitKPlan sk;
};

GemmChoice choose_gemm(int64_t M, int64_t N, int64_t K, const gw::DeviceInfo* d) {
  GemmChoice c;
  if (gw::use_pair_gemm(M, N, d->sm_count)) {
    c.kernel = GW_KERNEL_PAIR;
    return c;
  }
  if (decode_gemm_enabled()) c.dp = gw::plan_decode(M, N, K, d->sm_count);
  if (c.dp.split >= 2) {
    c.kernel = GW_KERNEL_DECODE;
    return c;
  }
  c.sk = gw::plan_splitk(M, N, K, d->sm_count);
  if (c.sk.split >= 2) c.kernel = GW_KERNEL_SPLITK;
  return c;
}

cudaError_t launch_dense_gemm(const void* a, int dtype, int64_t M, int64_t K, int64_t lda,
                              const void* w, int64_t N, int64_t ldw, const void* bias, int epilogue,
                              void* y, int64_t ldy, const gw::DeviceInfo* d, cudaStream_t s,
                              void* const* peers = nullptr, int n_peers = 0,
                              const int64_t* a_cols = nullptr, int64_t a_width = 0) {
  const GemmChoice c = choose_gemm(M, N, K, d);
  if (c.kernel == GW_KERNEL_PAIR)
    return gw::launch_gemm_tc2(a, dtype, M, K, lda, w, N, ldw, bias, epilogue, y, ldy,
                               d->err_word, d->sm_count, s, peers, n_peers, a_cols, a_width);
  cudaError_t e;
  if (c.kernel == GW_KERNEL_DECODE)
    e = gw::launch_gemm_decode(c.dp, a, dtype, M, K, lda, w, N, ldw, bias, epilogue, y, ldy,
                               d->err_word, s, a_cols, a_width);
  else if (c.kernel == GW_KERNEL_SPLITK)
    e = gw::launch_gemm_splitk(c.sk, a, dtype, M, K, lda, w, N, ldw, bias, epilogue, y, ldy,
                               d->err_word, s, a_cols, a_width);
  else
    e = gw::launch_gemm_tc(0, a, dtype, M, a_cols ? a_width : K, lda, w, N, ldw, nullptr, K, bias,
                           epilogue, y, ldy, d->err_word, d->sm_count, s, a_cols);
  if (e != cudaSuccess || n_peers == 0) return e;
  return gw::launch_copy_to_peers(y, M, N, ldy, peers, n_peers, d->sm_count, s);
}
}  // namespace

size_t gw_gather_gemm_workspace_bytes(int64_t M, int64_t n_alive, int dtype) {
  if (M <= 0 || n_alive <= 0 || dtype == GW_DTYPE_F32) return 0;
  return gemm_ws_header(M, n_alive) +
         static_cast<size_t>((M * gemm_ld_pad(n_alive) * 2 + 255) / 256 * 256);
}

int gw_gather_gemm(const void* x, int dtype, int64_t M, int64_t K, int64_t ldx,
                   const void* w_packed, int64_t N, int64_t ldw, const int64_t* idx,
                   int64_t n_alive, const void* bias, int epilogue, void* y, int64_t ldy,
                   int strategy, void* workspace, size_t workspace_bytes, void* stream) {
  if (!valid_dtype(dtype)) return GW_ERR_DTYPE;
  if (!valid_epi(epilogue)) return GW_ERR_UNSUPPORTED;
  if (strategy != GW_GEMM_AUTO && strategy != GW_GEMM_FUSED && strategy != GW_GEMM_PREGATHER &&
      strategy != GW_GEMM_OVERLAP && strategy != GW_GEMM_RUNS)
    return GW_ERR_UNSUPPORTED;
  if (!matrix_ok(M, K, ldx) || n_alive < 0 || !matrix_ok(N, n_alive, ldw) ||
      !matrix_ok(M, N, ldy))
    return GW_ERR_SHAPE;
  const gw::DeviceInfo* d = nullptr;
  int st = current_device(&d);
  if (st != GW_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (M == 0 || N == 0) return GW_OK;
  if (!y) return GW_ERR_NULL;
  cudaError_t e;
  if (n_alive == 0) {
    e = gw::launch_fill_bias(y, dtype, M, N, ldy, bias, epilogue, s);
    return e == cudaSuccess ? GW_OK : cuda_fail(e);
  }
  if (!x || !w_packed || !idx) return GW_ERR_NULL;
  if (dtype == GW_DTYPE_F32) {
    e = gw::launch_gemm_f32(static_cast<const float*>(x), M, K, ldx,
                            static_cast<const float*>(w_packed), N, ldw, idx, n_alive,
                            static_cast<const float*>(bias), epilogue, static_cast<float*>(y),
                            ldy, d->err_word, s);
    return e == cudaSuccess ? GW_OK : cuda_fail(e);
  }
  if (!aligned16(w_packed) || (ldw % 8) != 0) return GW_ERR_ALIGN;
  if (n_alive > 0x7FFFFFFFll - 64) return GW_ERR_SHAPE;
  if (strategy == GW_GEMM_RUNS) {
    if ((n_alive % 64) != 0) return GW_ERR_UNSUPPORTED;
    if (!aligned16(x) || (ldx % 8) != 0) return GW_ERR_ALIGN;
    e = launch_dense_gemm(x, dtype, M, n_alive, ldx, w_packed, N, ldw, bias, epilogue, y, ldy, d,
                          s, nullptr, 0, idx, K);
    return e == cudaSuccess ? GW_OK : cuda_fail(e);
  }
  if ((strategy == GW_GEMM_AUTO || strategy == GW_GEMM_FUSED) && M <= 4 && decode_gemm_enabled()) {
    // At most 4 rows (single-sequence decoding): the decode kernel gathers
    // x[:, idx] itself, one launch instead of two. With more rows its
    // per-element gather loads cost more than the separate gather launch.
    const gw::DecodePlan dp = gw::plan_decode(M, N, n_alive, d->sm_count);
    if (dp.split >= 2) {
      e = gw::launch_gemm_decode_gather(dp, x, dtype, M, K, ldx, idx, n_alive, w_packed, N, ldw,
                                        bias, epilogue, y, ldy, d->err_word, s);
      return e == cudaSuccess ? GW_OK : cuda_fail(e);
    }
  }
  const size_t need = gw_gather_gemm_workspace_bytes(M, n_alive, dtype);
  const bool ws_ok = workspace != nullptr && workspace_bytes >= need;
  int strat = strategy;
  if (strat == GW_GEMM_AUTO) strat = ws_ok ? GW_GEMM_PREGATHER : GW_GEMM_FUSED;
  if (strat == GW_GEMM_FUSED) {
    e = gw::launch_gemm_tc(1, x, dtype, M, K, ldx, w_packed, N, ldw, idx, n_alive, bias,
                           epilogue, y, ldy, d->err_word, d->sm_count, s);
    return e == cudaSuccess ? GW_OK : cuda_fail(e);
  }
  if (!workspace) return GW_ERR_NULL;
  if (!ws_ok) return GW_ERR_WORKSPACE;
  if (!aligned16(workspace)) return GW_ERR_ALIGN;
  const int64_t ldp = gemm_ld_pad(n_alive);
  void* xg = static_cast<char*>(workspace) + gemm_ws_header(M, n_alive);
  if (strat == GW_GEMM_OVERLAP && gw::use_pair_gemm(M, N, d->sm_count) &&
      gw::tc2_gather_supported(M, n_alive)) {
    // One launch: the pair kernel gathers x' into the workspace while its MMAs
    // consume the finished units.
    gw::Tc2Gather g;
    g.x = x;
    g.ldx = ldx;
    g.K = K;
    g.idx = idx;
    g.xg = xg;
    g.ldp = ldp;
    g.header = workspace;
    e = gw::launch_gemm_tc2(xg, dtype, M, n_alive, ldp, w_packed, N, ldw, bias, epilogue, y, ldy,
                            d->err_word, d->sm_count, s, nullptr, 0, nullptr, 0, nullptr, &g);
    return e == cudaSuccess ? GW_OK : cuda_fail(e);
  }
  // Pregather (also the overlap strategy's shapes that do not run on CTA pairs).
  e = gw::launch_gather_columns(x, dtype, M, ldx, K, idx, n_alive, xg, ldp, n_alive,
                                d->err_word, d->sm_count, s, true);
  if (e != cudaSuccess) return cuda_fail(e);
  e = launch_dense_gemm(xg, dtype, M, n_alive, ldp, w_packed, N, ldw, bias, epilogue, y, ldy, d, s);
  return e == cudaSuccess ? GW_OK : cuda_fail(e);
}

int gw_gather_gemm_dev(const void* x, int dtype, int64_t M, int64_t K, int64_t ldx,
                       const void* w_packed, int64_t N, int64_t ldw, const int64_t* idx,
                       int64_t n_alive_max, const int32_t* n_alive_dev, const void* bias,
                       int epilogue, void* y, int64_t ldy, void* workspace, size_t workspace_bytes,
                       void* stream) {
  if (!valid_dtype(dtype)) return GW_ERR_DTYPE;
  if (!valid_epi(epilogue)) return GW_ERR_UNSUPPORTED;
  if (!matrix_ok(M, K, ldx) || n_alive_max < 0 || n_alive_max > K ||
      !matrix_ok(N, n_alive_max, ldw) || !matrix_ok(M, N, ldy))
    return GW_ERR_SHAPE;
  const gw::DeviceInfo* d = nullptr;
  int st = current_device(&d);
  if (st != GW_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (M == 0 || N == 0) return GW_OK;
  if (!y) return GW_ERR_NULL;
  cudaError_t e;
  if (n_alive_max == 0) {
    e = gw::launch_fill_bias(y, dtype, M, N, ldy, bias, epilogue, s);
    return e == cudaSuccess ? GW_OK : cuda_fail(e);
  }
  if (!x || !w_packed || !idx || !n_alive_dev) return GW_ERR_NULL;
  if (dtype == GW_DTYPE_F32) {
    e = gw::launch_gemm_f32(static_cast<const float*>(x), M, K, ldx,
                            static_cast<const float*>(w_packed), N, ldw, idx, n_alive_max,
                            static_cast<const float*>(bias), epilogue, static_cast<float*>(y),
                            ldy, d->err_word, s, n_alive_dev);
    return e == cudaSuccess ? GW_OK : cuda_fail(e);
  }
  const int64_t ldp = gemm_ld_pad(n_alive_max);
  if (!aligned16(w_packed) || (ldw % 8) != 0) return GW_ERR_ALIGN;
  if (ldw < ldp) return GW_ERR_SHAPE;           // W' is zero up to the 64-column boundary
  if (n_alive_max > 0x7FFFFFFFll - 64) return GW_ERR_SHAPE;
  if (!workspace) return GW_ERR_NULL;
  if (workspace_bytes < gw_gather_gemm_workspace_bytes(M, n_alive_max, dtype)) return GW_ERR_WORKSPACE;
  if (!aligned16(workspace)) return GW_ERR_ALIGN;
  void* xg = static_cast<char*>(workspace) + gemm_ws_header(M, n_alive_max);
  e = gw::launch_gather_columns(x, dtype, M, ldx, K, idx, n_alive_max, xg, ldp, ldp, d->err_word,
                                d->sm_count, s, true, n_alive_dev);
  if (e != cudaSuccess) return cuda_fail(e);
  // The count is known only on the device: the persistent kernels, whose
  // launch does not depend on it, read it (decode and split-K plans do).
  if (gw::use_pair_gemm(M, N, d->sm_count))
    e = gw::launch_gemm_tc2(xg, dtype, M, ldp, ldp, w_packed, N, ldw, bias, epilogue, y, ldy,
                            d->err_word, d->sm_count, s, nullptr, 0, nullptr, 0, n_alive_dev);
  else
    e = gw::launch_gemm_tc(0, xg, dtype, M, ldp, ldp, w_packed, N, ldw, nullptr, ldp, bias,
                           epilogue, y, ldy, d->err_word, d->sm_count, s, nullptr, n_alive_dev);
  return e == cudaSuccess ? GW_OK : cuda_fail(e);
}

int gw_gather_gemm_peers(const void* x, int dtype, int64_t M, int64_t K, int64_t ldx,
                         const void* w_packed, int64_t N, int64_t ldw, const int64_t* idx,
                         int64_t n_alive, const void* bias, int epilogue, void* y, int64_t ldy,
                         void* const* peer_y, int n_peers, int strategy, void* workspace,
                         size_t workspace_bytes, void* stream) {
  if (dtype != GW_DTYPE_F16 && dtype != GW_DTYPE_BF16) return GW_ERR_DTYPE;
  if (!valid_epi(epilogue)) return GW_ERR_UNSUPPORTED;
  if (n_peers < 0 || n_peers > GW_MAX_PEERS) return GW_ERR_UNSUPPORTED;
  if (strategy != GW_GEMM_AUTO && strategy != GW_GEMM_PREGATHER && strategy != GW_GEMM_RUNS)
    return GW_ERR_UNSUPPORTED;
  if (!matrix_ok(M, K, ldx) || n_alive < 0 || !matrix_ok(N, n_alive, ldw) ||
      !matrix_ok(M, N, ldy))
    return GW_ERR_SHAPE;
  const gw::DeviceInfo* d = nullptr;
  int st = current_device(&d);
  if (st != GW_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (M == 0 || N == 0) return GW_OK;
  if (!y || (n_peers > 0 && !peer_y)) return GW_ERR_NULL;
  for (int i = 0; i < n_peers; ++i) {
    if (!peer_y[i]) return GW_ERR_NULL;
    if (!aligned16(peer_y[i])) return GW_ERR_ALIGN;
  }
  if (!aligned16(y) || (ldy % 8) != 0) return GW_ERR_ALIGN;
  cudaError_t e;
  if (n_alive == 0) {
    e = gw::launch_fill_bias(y, dtype, M, N, ldy, bias, epilogue, s);
    if (e == cudaSuccess) e = gw::launch_copy_to_peers(y, M, N, ldy, peer_y, n_peers, d->sm_count, s);
    return e == cudaSuccess ? GW_OK : cuda_fail(e);
  }
  if (!x || !w_packed || !idx) return GW_ERR_NULL;
  if (!aligned16(w_packed) || (ldw % 8) != 0) return GW_ERR_ALIGN;
  if (n_alive > 0x7FFFFFFFll - 64) return GW_ERR_SHAPE;
  if (strategy == GW_GEMM_RUNS) {
    if ((n_alive % 64) != 0) return GW_ERR_UNSUPPORTED;
    if (!aligned16(x) || (ldx % 8) != 0) return GW_ERR_ALIGN;
    e = launch_dense_gemm(x, dtype, M, n_alive, ldx, w_packed, N, ldw, bias, epilogue, y, ldy, d,
                          s, peer_y, n_peers, idx, K);
    return e == cudaSuccess ? GW_OK : cuda_fail(e);
  }
  if (!workspace) return GW_ERR_NULL;
  if (workspace_bytes < gw_gather_gemm_workspace_bytes(M, n_alive, dtype)) return GW_ERR_WORKSPACE;
  if (!aligned16(workspace)) return GW_ERR_ALIGN;
  const int64_t ldp = gemm_ld_pad(n_alive);
  void* xg = static_cast<char*>(workspace) + gemm_ws_header(M, n_alive);
  e = gw::launch_gather_columns(x, dtype, M, ldx, K, idx, n_alive, xg, ldp, n_alive,
                                d->err_word, d->sm_count, s, true);
  if (e != cudaSuccess) return cuda_fail(e);
  e = launch_dense_gemm(xg, dtype, M, n_alive, ldp, w_packed, N, ldw, bias, epilogue, y, ldy, d, s,
                        peer_y, n_peers);
  return e == cudaSuccess ? GW_OK : cuda_fail(e);
}

int gw_dynamic_linear(const void* x, int dtype, int64_t M, int64_t K, int64_t ldx,
                      const void* w, int64_t N, int64_t ldw, double threshold, const void* bias,
                      int epilogue, void* y, int64_t ldy, int32_t* alive_count, int32_t* mask,
                      void* stream) {
  if (dtype != GW_DTYPE_F16 && dtype != GW_DTYPE_BF16) return GW_ERR_DTYPE;
  if (!valid_epi(epilogue)) return GW_ERR_UNSUPPORTED;
  if (!matrix_ok(M, K, ldx) || !matrix_ok(N, K, ldw) || !matrix_ok(M, N, ldy)) return GW_ERR_SHAPE;
  if (!gw::dyn_linear_supported(M, K) || N > int64_t{65535} * 128) return GW_ERR_UNSUPPORTED;
  if (!aligned16(x) || !aligned16(w) || (ldx % 8) != 0 || (ldw % 8) != 0) return GW_ERR_UNSUPPORTED;
  const gw::DeviceInfo* d = nullptr;
  int st = current_device(&d);
  if (st != GW_OK) return st;
  if (N == 0) {
    if (alive_count) {
      cudaError_t e = cudaMemsetAsync(alive_count, 0, sizeof(int32_t), static_cast<cudaStream_t>(stream));
      if (e != cudaSuccess) return cuda_fail(e);
    }
    return GW_OK;
  }
  if (!x || !w || !y) return GW_ERR_NULL;
  // The reference passes the threshold as an fp32 kernel scalar (mask.py:100).
  cudaError_t e = gw::launch_dyn_linear(x, dtype, M, K, ldx, w, N, ldw, static_cast<float>(threshold),
                                        bias, epilogue, y, ldy, alive_count, mask, d->err_word,
                                        static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? GW_OK : cuda_fail(e);
}

int gw_packed_gemm(const void* a, int dtype, int64_t M, int64_t K, int64_t lda,
                   const void* w_packed, int64_t N, int64_t ldw, const void* bias, int epilogue,
                   void* y, int64_t ldy, void* stream) {
  if (dtype != GW_DTYPE_F16 && dtype != GW_DTYPE_BF16) return GW_ERR_DTYPE;
  if (!valid_epi(epilogue)) return GW_ERR_UNSUPPORTED;
  if (!matrix_ok(M, K, lda) || !matrix_ok(N, K, ldw) || !matrix_ok(M, N, ldy))
    return GW_ERR_SHAPE;
  const gw::DeviceInfo* d = nullptr;
  int st = current_device(&d);
  if (st != GW_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (M == 0 || N == 0) return GW_OK;
  if (!y) return GW_ERR_NULL;
  cudaError_t e;
  if (K == 0) {
    e = gw::launch_fill_bias(y, dtype, M, N, ldy, bias, epilogue, s);
    return e == cudaSuccess ? GW_OK : cuda_fail(e);
  }
  if (!a || !w_packed) return GW_ERR_NULL;
  if (!aligned16(a) || !aligned16(w_packed) || (lda % 8) != 0 || (ldw % 8) != 0)
    return GW_ERR_ALIGN;
  e = launch_dense_gemm(a, dtype, M, K, lda, w_packed, N, ldw, bias, epilogue, y, ldy, d, s);
  return e == cudaSuccess ? GW_OK : cuda_fail(e);
}

int gw_gemm_plan(int64_t M, int64_t N, int64_t K, int* kernel, int* tile_n, int* split) {
  if (M < 0 || N < 0 || K < 0) return GW_ERR_SHAPE;
  if (!kernel) return GW_ERR_NULL;
  const gw::DeviceInfo* d = nullptr;
  int st = current_device(&d);
  if (st != GW_OK) return st;
  const GemmChoice c = choose_gemm(M, N, K, d);
  int tn = 0, sp = 0;
  if (c.kernel == GW_KERNEL_PAIR) {
    tn = gw::pair_gemm_tile_width(M, N, d->sm_count);
  } else if (c.kernel == GW_KERNEL_DECODE) {
    sp = c.dp.split;
  } else if (c.kernel == GW_KERNEL_SPLITK) {
    tn = c.sk.bn;
    sp = c.sk.split;
  }
  *kernel = c.kernel;
  if (tile_n) *tile_n = tn;
  if (split) *split = sp;
  return GW_OK;
}

int gw_selftest_wait_timeout(int64_t limit_ns, void* stream) {
  const gw::DeviceInfo* d = nullptr;
  int st = current_device(&d);
  if (st != GW_OK) return st;
  const int64_t lim = limit_ns < 100000 ? 100000 : (limit_ns > 1000000000 ? 1000000000 : limit_ns);
  gw::selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<unsigned long long>(lim), d->err_word);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? GW_OK : cuda_fail(e);
}

int gw_validate_indices(const int64_t* idx, int64_t n, int64_t K, int32_t* bad_count,
                        void* stream) {
  if (n < 0 || K < 0) return GW_ERR_SHAPE;
  if (!bad_count || (n > 0 && !idx)) return GW_ERR_NULL;
  const gw::DeviceInfo* d = nullptr;
  int st = current_device(&d);
  if (st != GW_OK) return st;
  cudaError_t e = gw::launch_validate_indices(idx, n, K, bad_count,
                                              static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? GW_OK : cuda_fail(e);
}

int gw_index_runs(const int64_t* idx, int64_t n, int64_t K, int32_t* bad_count, void* stream) {
  if (n < 0 || K < 0) return GW_ERR_SHAPE;
  if (!bad_count || (n > 0 && !idx)) return GW_ERR_NULL;
  const gw::DeviceInfo* d = nullptr;
  int st = current_device(&d);
  if (st != GW_OK) return st;
  cudaError_t e = gw::launch_index_runs(idx, n, K, bad_count, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? GW_OK : cuda_fail(e);
}

}  // extern "C"
