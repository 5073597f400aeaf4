// K2: gathers and the one-time weight compaction (HBM-bound copies).
//
//   gather_columns : dst[r, j] = src[r, idx[j]]      (A side of gather_compact,
//                    ghostweight_triton/kernels/gather.py:19-55, and the packing
//                    of nn.Linear.weight [N, K] into the K'-major GEMM operand)
//   gather_rows    : dst[j, :] = src[idx[j], :]      (W side, gather.py:58-94)
//   gather_rows_t  : dst[n, j] = src[idx[j], n]      (packs a [K, N] weight, the
//                    orientation ghostweight_matmul takes, into [N, K'])
//
// The column gather maps lanes to consecutive OUTPUT columns, so one warp
// instruction reads 32 consecutive alive indices of one row (for sorted lists
// that is a narrow window of the row: few sectors per request) and writes 32
// consecutive outputs (fully coalesced stores). Column indices are loaded once
// per CTA and reused for every row the CTA handles.
#include <algorithm>

#include "gw_common.cuh"
#include "gw_internal.h"

namespace gw {

namespace {

constexpr int kGThreads = 256;
constexpr int kGWarps = kGThreads / 32;
constexpr int kColsPerLane = 8;                    // outputs per lane per row
constexpr int kColChunk = 32 * kColsPerLane;       // 256 output columns per CTA

// Column index codes held in registers: >= 0 source column, -1 write zero.
template <typename raw>
__global__ void __launch_bounds__(kGThreads)
gather_columns_kernel(const raw* __restrict__ src, int64_t rows, int64_t ld_src, int64_t cols_src,
                      const int64_t* __restrict__ idx, int64_t n_idx, raw* __restrict__ dst,
                      int64_t ld_dst, int64_t pad_to, unsigned int* err, int early_dependents,
                      const int32_t* __restrict__ n_dev, int vec_rows) {
  // Launched as a programmatic dependent of the previous kernel of the stream
  // (which may have produced src or idx): wait for it to complete. When dst is
  // the x' of the GEMM launched next (early_dependents), let that GEMM start
  // its prologue early; it waits for this grid to finish before reading x'.
  // Otherwise (a packed weight, a caller's buffer) the next kernel starts
  // only when this grid has finished: a GEMM may read its weight operand
  // before its own wait.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (early_dependents) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * kColChunk;
  if (n_dev) {
    // The count lives on the device (written by the mask kernel): n_idx and
    // pad_to are upper bounds. Columns [n, round_up(max(n, 1), 64)) are zero,
    // the ones past that are left alone (a GEMM reading this count never
    // reaches them).
    const int64_t n = min(static_cast<int64_t>(max(*n_dev, 0)), n_idx);
    n_idx = n;
    pad_to = min(pad_to, (max(n, int64_t{1}) + 63) / 64 * 64);
    if (c0 >= pad_to) return;
  }

  int64_t scol[kColsPerLane];
  bool live[kColsPerLane];
  bool bad = false;
#pragma unroll
  for (int e = 0; e < kColsPerLane; ++e) {
    const int64_t j = c0 + lane + 32 * e;
    live[e] = j < pad_to;
    int64_t c = -1;
    if (j < n_idx) {
      c = __ldg(idx + j);
      if (c < 0 || c >= cols_src) { bad = true; c = -1; }
    }
    scol[e] = c;
  }
  if (bad && blockIdx.y == 0 && warp == 0) raise_error(err, GW_DERR_BAD_INDEX);

  // Runs: lanes 8k .. 8k+7 hold the 8 consecutive outputs c0 + 32 e + 8k ..
  // + 7. When, in every such group, they come from 8 consecutive source
  // columns starting at a multiple of 8 (a mask that kills whole column
  // blocks), lane l instead moves outputs c0 + 8 l .. + 7 as one 16-byte
  // vector per row. The test uses the indices already loaded (shuffles, no
  // further loads), and every warp reaches the same answer from the same
  // chunk, so the choice needs no barrier. Scattered, invalid or unaligned
  // indices, a chunk past the alive count, unaligned rows and 4-byte elements
  // keep the per-element loop below.
  if (sizeof(raw) == 2 && vec_rows && c0 + kColChunk <= n_idx) {
    // The first group decides most lists (a scattered list fails it at
    // once); only a list that passes it has the other seven checked.
    const int64_t base0 = __shfl_sync(0xFFFFFFFFu, scol[0], lane & ~7);
    bool run = base0 >= 0 && (base0 & 7) == 0 && scol[0] == base0 + (lane & 7);
    if (__all_sync(0xFFFFFFFFu, run)) {
#pragma unroll
      for (int e = 1; e < kColsPerLane; ++e) {
        const int64_t base = __shfl_sync(0xFFFFFFFFu, scol[e], lane & ~7);
        run = run && base >= 0 && (base & 7) == 0 && scol[e] == base + (lane & 7);
      }
    }
    if (__all_sync(0xFFFFFFFFu, run)) {
      const int64_t j0 = c0 + 8 * lane;
      const int64_t v0 = __ldg(idx + j0);
      for (int64_t r = static_cast<int64_t>(blockIdx.y) * kGWarps + warp; r < rows;
           r += static_cast<int64_t>(gridDim.y) * kGWarps) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(src + r * ld_src + v0));
        *reinterpret_cast<uint4*>(dst + r * ld_dst + j0) = v;
      }
      return;
    }
  }

  for (int64_t r = static_cast<int64_t>(blockIdx.y) * kGWarps + warp; r < rows;
       r += static_cast<int64_t>(gridDim.y) * kGWarps) {
    const raw* srow = src + r * ld_src;
    raw* drow = dst + r * ld_dst;
    raw vals[kColsPerLane];
#pragma unroll
    for (int e = 0; e < kColsPerLane; ++e) vals[e] = (scol[e] >= 0) ? __ldg(srow + scol[e]) : raw(0);
#pragma unroll
    for (int e = 0; e < kColsPerLane; ++e)
      if (live[e]) drow[c0 + lane + 32 * e] = vals[e];
  }
}

// One CTA row-slab copies whole rows; 16-byte vectors when everything is aligned.
template <typename raw, bool VEC>
__global__ void __launch_bounds__(kGThreads)
gather_rows_kernel(const raw* __restrict__ src, int64_t rows_src, int64_t cols, int64_t ld_src,
                   const int64_t* __restrict__ idx, int64_t n_idx, raw* __restrict__ dst,
                   int64_t ld_dst, unsigned int* err) {
  constexpr int VPT = VEC ? static_cast<int>(16 / sizeof(raw)) : 1;
  const int64_t nvec = cols / VPT;
  for (int64_t j = blockIdx.y; j < n_idx; j += gridDim.y) {
    int64_t r = __ldg(idx + j);
    const bool ok = (r >= 0 && r < rows_src);
    if (!ok && threadIdx.x == 0 && blockIdx.x == 0) raise_error(err, GW_DERR_BAD_INDEX);
    for (int64_t v = static_cast<int64_t>(blockIdx.x) * kGThreads + threadIdx.x; v < nvec;
         v += static_cast<int64_t>(gridDim.x) * kGThreads) {
      if constexpr (VEC) {
        uint4 q = make_uint4(0, 0, 0, 0);
        if (ok) q = __ldg(reinterpret_cast<const uint4*>(src + r * ld_src) + v);
        reinterpret_cast<uint4*>(dst + j * ld_dst)[v] = q;
      } else {
        dst[j * ld_dst + v] = ok ? __ldg(src + r * ld_src + v) : raw(0);
      }
    }
  }
}

// dst[n, j] = src[idx[j], n] through a 64x64 shared-memory tile.
constexpr int kTTile = 64;
template <typename raw>
__global__ void __launch_bounds__(kGThreads)
gather_rows_t_kernel(const raw* __restrict__ src, int64_t rows_src, int64_t cols, int64_t ld_src,
                     const int64_t* __restrict__ idx, int64_t n_idx, raw* __restrict__ dst,
                     int64_t ld_dst, int64_t pad_to, unsigned int* err,
                     const int32_t* __restrict__ n_dev) {
  __shared__ raw tile[kTTile][kTTile + 1];
  const int tx = threadIdx.x & 63;   // 0..63
  const int ty = threadIdx.x >> 6;   // 0..3
  const int64_t j0 = static_cast<int64_t>(blockIdx.x) * kTTile;   // output column block (alive)
  const int64_t n0 = static_cast<int64_t>(blockIdx.y) * kTTile;   // output row block (features)
  if (n_dev) {
    // Count on the device: as in gather_columns_kernel (whole CTAs past the
    // zero-filled range return before the barrier).
    const int64_t n = min(static_cast<int64_t>(max(*n_dev, 0)), n_idx);
    n_idx = n;
    pad_to = min(pad_to, (max(n, int64_t{1}) + 63) / 64 * 64);
    if (j0 >= pad_to) return;
  }
  bool bad = false;
#pragma unroll 4
  for (int i = 0; i < kTTile / 4; ++i) {
    const int jj = ty + 4 * i;
    const int64_t j = j0 + jj;
    const int64_t n = n0 + tx;
    raw v = raw(0);
    if (j < n_idx && n < cols) {
      const int64_t r = __ldg(idx + j);
      if (r >= 0 && r < rows_src) v = __ldg(src + r * ld_src + n);
      else bad = true;
    }
    tile[jj][tx] = v;
  }
  if (bad) raise_error(err, GW_DERR_BAD_INDEX);
  __syncthreads();
#pragma unroll 4
  for (int i = 0; i < kTTile / 4; ++i) {
    const int nn = ty + 4 * i;
    const int64_t n = n0 + nn;
    const int64_t j = j0 + tx;
    if (n < cols && j < pad_to) dst[n * ld_dst + j] = tile[tx][nn];
  }
}

template <int DT>
__global__ void fill_bias_kernel(typename Elem<DT>::raw* __restrict__ y, int64_t M, int64_t N,
                                 int64_t ldy, const typename Elem<DT>::raw* __restrict__ bias,
                                 int epi) {
  const int64_t total = M * N;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = t / N, n = t - m * N;
    float v = bias ? Elem<DT>::to_f(bias[n]) : 0.0f;
    v = apply_epilogue(v, epi);
    y[m * ldy + n] = Elem<DT>::from_f(v);
  }
}

__global__ void validate_indices_kernel(const int64_t* __restrict__ idx, int64_t n, int64_t K,
                                        int32_t* bad) {
  int local = 0;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < n;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = idx[t];
    local += (c < 0 || c >= K) ? 1 : 0;
  }
  local = __reduce_add_sync(0xFFFFFFFFu, local);
  if ((threadIdx.x & 31) == 0 && local) atomicAdd(bad, local);
}

// Entries that break the 64-column-run structure: idx[64 j + r] must equal
// idx[64 j] + r, idx[64 j] must be a multiple of 8, every entry must lie in
// [0, K) and the list must end on a whole run.
__global__ void index_runs_kernel(const int64_t* __restrict__ idx, int64_t n, int64_t K,
                                  int32_t* bad) {
  int local = 0;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < n;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = t & 63;
    const int64_t start = idx[t - r];
    const int64_t c = idx[t];
    local += (c < 0 || c >= K || c != start + r || (start & 7) != 0 || t - r + 64 > n) ? 1 : 0;
  }
  local = __reduce_add_sync(0xFFFFFFFFu, local);
  if ((threadIdx.x & 31) == 0 && local) atomicAdd(bad, local);
}

inline unsigned clamp_grid(int64_t v, int64_t hi) {
  if (v < 1) v = 1;
  if (v > hi) v = hi;
  return static_cast<unsigned>(v);
}

}  // namespace

cudaError_t launch_gather_columns(const void* src, int dtype, int64_t rows, int64_t ld_src,
                                  int64_t cols_src, const int64_t* idx, int64_t n_idx, void* dst,
                                  int64_t ld_dst, int64_t pad_to, unsigned int* err,
                                  int sm_count, cudaStream_t stream, bool early_dependents,
                                  const int32_t* n_dev) {
  if (rows == 0 || pad_to == 0) return cudaSuccess;
  const int64_t col_blocks = (pad_to + kColChunk - 1) / kColChunk;
  const int64_t target = static_cast<int64_t>(sm_count > 0 ? sm_count : 148) * 8;
  const unsigned gy = clamp_grid(std::min<int64_t>((rows + kGWarps - 1) / kGWarps,
                                                   (target + col_blocks - 1) / col_blocks),
                                 65535);
  dim3 grid(static_cast<unsigned>(col_blocks), gy);
  // Whole 16-byte vectors of 16-bit rows can move at once (source and
  // destination rows 16-byte aligned).
  const int vec_rows = (dtype != GW_DTYPE_F32 &&
                        ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u) == 0 &&
                        ld_src % 8 == 0 && ld_dst % 8 == 0) ? 1 : 0;
  if (dtype == GW_DTYPE_F32) {
    return launch_pdl(gather_columns_kernel<uint32_t>, grid, dim3(kGThreads), stream,
                      static_cast<const uint32_t*>(src), rows, ld_src, cols_src, idx, n_idx,
                      static_cast<uint32_t*>(dst), ld_dst, pad_to, err, early_dependents ? 1 : 0,
                      n_dev, 0);
  }
  return launch_pdl(gather_columns_kernel<uint16_t>, grid, dim3(kGThreads), stream,
                    static_cast<const uint16_t*>(src), rows, ld_src, cols_src, idx, n_idx,
                    static_cast<uint16_t*>(dst), ld_dst, pad_to, err, early_dependents ? 1 : 0,
                    n_dev, vec_rows);
}

namespace {
// y [rows, cols] -> each peer buffer at the same offsets, 16 bytes per thread
// and step (rows are 16-byte aligned; a ragged row end is copied per element).
struct PeerList {
  uint16_t* p[kMaxPeers];
};

__global__ void __launch_bounds__(kGThreads)
copy_to_peers_kernel(const uint16_t* __restrict__ y, int64_t rows, int64_t cols, int64_t ld,
                     PeerList peers, int n_peers) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t vec_per_row = (cols + 7) / 8;
  const int64_t total = rows * vec_per_row;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * kGThreads + threadIdx.x; v < total;
       v += static_cast<int64_t>(gridDim.x) * kGThreads) {
    const int64_t r = v / vec_per_row;
    const int64_t c = (v - r * vec_per_row) * 8;
    const uint16_t* src = y + r * ld + c;
    if (c + 8 <= cols) {
      const uint4 q = __ldg(reinterpret_cast<const uint4*>(src));
      for (int i = 0; i < n_peers; ++i) *reinterpret_cast<uint4*>(peers.p[i] + r * ld + c) = q;
    } else {
      for (int i = 0; i < n_peers; ++i)
        for (int64_t j = c; j < cols; ++j) peers.p[i][r * ld + j] = y[r * ld + j];
    }
  }
  __threadfence_system();
}
}  // namespace

cudaError_t launch_copy_to_peers(const void* y, int64_t rows, int64_t cols, int64_t ld,
                                 void* const* peers, int n_peers, int sm_count, cudaStream_t stream) {
  if (rows == 0 || cols == 0 || n_peers == 0) return cudaSuccess;
  if (n_peers < 0 || n_peers > kMaxPeers) return cudaErrorInvalidValue;
  PeerList list{};
  for (int i = 0; i < n_peers; ++i) list.p[i] = static_cast<uint16_t*>(peers[i]);
  const int64_t total = rows * ((cols + 7) / 8);
  const unsigned grid = clamp_grid(std::min<int64_t>((total + kGThreads - 1) / kGThreads,
                                                     static_cast<int64_t>(sm_count > 0 ? sm_count : 148) * 8),
                                   1 << 20);
  return launch_pdl(copy_to_peers_kernel, dim3(grid), dim3(kGThreads), stream,
                    static_cast<const uint16_t*>(y), rows, cols, ld, list, n_peers);
}

cudaError_t launch_gather_rows(const void* src, int dtype, int64_t rows_src, int64_t cols,
                               int64_t ld_src, const int64_t* idx, int64_t n_idx, void* dst,
                               int64_t ld_dst, unsigned int* err, int sm_count,
                               cudaStream_t stream) {
  if (n_idx == 0 || cols == 0) return cudaSuccess;
  const int esize = dtype == GW_DTYPE_F32 ? 4 : 2;
  const int vpt = 16 / esize;
  const bool vec = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u) == 0 &&
                   ld_src % vpt == 0 && ld_dst % vpt == 0 && cols % vpt == 0;
  const int64_t nvec = vec ? cols / vpt : cols;
  const unsigned gx = clamp_grid((nvec + kGThreads - 1) / kGThreads, 1 << 20);
  const int64_t target = static_cast<int64_t>(sm_count > 0 ? sm_count : 148) * 8;
  const unsigned gy = clamp_grid(std::min<int64_t>(n_idx, (target + gx - 1) / gx), 65535);
  dim3 grid(gx, gy);
#define GW_ROWS_LAUNCH(T, V)                                                                 \
  gather_rows_kernel<T, V><<<grid, kGThreads, 0, stream>>>(static_cast<const T*>(src),       \
                                                            rows_src, cols, ld_src, idx,     \
                                                            n_idx, static_cast<T*>(dst),     \
                                                            ld_dst, err)
  if (esize == 4) {
    if (vec) GW_ROWS_LAUNCH(uint32_t, true); else GW_ROWS_LAUNCH(uint32_t, false);
  } else {
    if (vec) GW_ROWS_LAUNCH(uint16_t, true); else GW_ROWS_LAUNCH(uint16_t, false);
  }
#undef GW_ROWS_LAUNCH
  return cudaGetLastError();
}

cudaError_t launch_gather_rows_t(const void* src, int dtype, int64_t rows_src, int64_t cols,
                                 int64_t ld_src, const int64_t* idx, int64_t n_idx, void* dst,
                                 int64_t ld_dst, int64_t pad_to, unsigned int* err,
                                 cudaStream_t stream, const int32_t* n_dev) {
  if (cols == 0 || pad_to == 0) return cudaSuccess;
  const int64_t gx = (pad_to + kTTile - 1) / kTTile;
  const int64_t gy = (cols + kTTile - 1) / kTTile;
  if (gx > 0x7FFFFFFFll || gy > 65535) return cudaErrorInvalidValue;
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy));
  if (dtype == GW_DTYPE_F32) {
    gather_rows_t_kernel<uint32_t><<<grid, kGThreads, 0, stream>>>(
        static_cast<const uint32_t*>(src), rows_src, cols, ld_src, idx, n_idx,
        static_cast<uint32_t*>(dst), ld_dst, pad_to, err, n_dev);
  } else {
    gather_rows_t_kernel<uint16_t><<<grid, kGThreads, 0, stream>>>(
        static_cast<const uint16_t*>(src), rows_src, cols, ld_src, idx, n_idx,
        static_cast<uint16_t*>(dst), ld_dst, pad_to, err, n_dev);
  }
  return cudaGetLastError();
}

cudaError_t launch_fill_bias(void* y, int dtype, int64_t M, int64_t N, int64_t ldy,
                             const void* bias, int epilogue, cudaStream_t stream) {
  if (M == 0 || N == 0) return cudaSuccess;
  const unsigned grid = clamp_grid((M * N + 255) / 256, 148 * 32);
  switch (dtype) {
    case GW_DTYPE_F16:
      fill_bias_kernel<GW_DTYPE_F16><<<grid, 256, 0, stream>>>(
          static_cast<uint16_t*>(y), M, N, ldy, static_cast<const uint16_t*>(bias), epilogue);
      break;
    case GW_DTYPE_BF16:
      fill_bias_kernel<GW_DTYPE_BF16><<<grid, 256, 0, stream>>>(
          static_cast<uint16_t*>(y), M, N, ldy, static_cast<const uint16_t*>(bias), epilogue);
      break;
    default:
      fill_bias_kernel<GW_DTYPE_F32><<<grid, 256, 0, stream>>>(
          static_cast<uint32_t*>(y), M, N, ldy, static_cast<const uint32_t*>(bias), epilogue);
      break;
  }
  return cudaGetLastError();
}

cudaError_t launch_validate_indices(const int64_t* idx, int64_t n, int64_t K, int32_t* bad,
                                    cudaStream_t stream) {
  cudaError_t e = cudaMemsetAsync(bad, 0, sizeof(int32_t), stream);
  if (e != cudaSuccess || n == 0) return e;
  const unsigned grid = clamp_grid((n + 255) / 256, 1024);
  validate_indices_kernel<<<grid, 256, 0, stream>>>(idx, n, K, bad);
  return cudaGetLastError();
}

cudaError_t launch_index_runs(const int64_t* idx, int64_t n, int64_t K, int32_t* bad,
                              cudaStream_t stream) {
  cudaError_t e = cudaMemsetAsync(bad, 0, sizeof(int32_t), stream);
  if (e != cudaSuccess || n == 0) return e;
  const unsigned grid = clamp_grid((n + 255) / 256, 1024);
  index_runs_kernel<<<grid, 256, 0, stream>>>(idx, n, K, bad);
  return cudaGetLastError();
}

}  // namespace gw
