// K1: dead-column mask fused with stream compaction (one launch).
//
// Semantics follow the reference Triton kernel ghostweight_triton/kernels/
// mask.py:21-59 bit for bit: per column the running max starts at 0.0 (mask.py:46),
// NaN entries never win the max (tl.maximum ignores NaN), values are compared in
// fp32 after conversion (mask.py:53) and a column is alive iff max > fp32(threshold)
// (mask.py:58). Since max starts at 0, that is exactly
//     alive[k] = (0 > thr) || any_r( fp32(|x[r,k]|) > thr )
// (a NaN compares false), which needs one bit per column instead of a float, so
// the cross-CTA combine is an OR of 32-bit words.
//
// Layout/parallelism (HBM-bound, row-major [rows, cols] input):
//   * a warp covers 32 consecutive 16-byte vectors of one row (512 contiguous
//     bytes, fully coalesced); 8 warps of a CTA walk different rows; each CTA
//     owns a 32-vector column strip and a contiguous chunk of rows;
//   * 4 rows are loaded per batch per thread (streaming, no L1 allocation),
//     the last batch of a chunk included (clamped rows, masked results);
//   * a warp whose columns are all alive stops reading (warp-uniform exit);
//   * per-CTA alive bits are OR-ed into a 32-bit word array in the workspace,
//     then the CTA takes a ticket with one acquire-release atomic;
//   * the last CTA to finish (ticket counter) performs the compaction: a
//     block-wide prefix sum of popcounts places every alive column's index in
//     shared memory, from where mask[], the ascending alive index list (the
//     torch.nonzero of module.py:104) and the count are written with coalesced
//     stores; it also resets the workspace to zero for the next call. (One
//     thread per flag word writing its own indices scatters 8-byte stores over
//     the index list, about one L2 transaction each, which took the last CTA
//     about 1 us longer at 4096 columns.)
#include "gw_common.cuh"
#include "gw_internal.h"

namespace gw {

namespace {

constexpr int kMaskThreads = 256;
constexpr int kMaskWarps = kMaskThreads / 32;
constexpr int kMaskUnroll = 4;

// Workspace: [0] ticket counter, [4..16) padding, then ceil(cols/32) flag words.
constexpr size_t kFlagsOffset = 16;

__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t atom_add_acq_rel(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Columns the last CTA compacts per pass: one flag word per thread.
constexpr int kPassCols = kMaskThreads * 32;

// Alive bits (bit e for element e) of one 16-byte vector.
template <int DT>
__device__ __forceinline__ uint32_t vec_bits(const uint4 v, float thr) {
  uint32_t b = 0;
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  if constexpr (DT == GW_DTYPE_F32) {
#pragma unroll
    for (int e = 0; e < 4; ++e) b |= (fabsf(__uint_as_float(w[e])) > thr ? 1u : 0u) << e;
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float lo = Elem<DT>::to_f(static_cast<uint16_t>(w[e] & 0xFFFFu));
      const float hi = Elem<DT>::to_f(static_cast<uint16_t>(w[e] >> 16));
      b |= (fabsf(lo) > thr ? 1u : 0u) << (2 * e);
      b |= (fabsf(hi) > thr ? 1u : 0u) << (2 * e + 1);
    }
  }
  return b;
}

// VEC = true: each thread owns one 16-byte vector (8 x 16-bit or 4 x fp32
// columns); requires 16-byte aligned base, ld and cols multiples of the vector.
// VEC = false: each thread owns one column (scalar loads).
template <int DT, bool VEC>
__global__ void __launch_bounds__(kMaskThreads, 8)
mask_compact_kernel(const void* __restrict__ x, int64_t rows, int64_t cols, int64_t ld,
                    float thr, int64_t rows_per_cta, uint32_t* __restrict__ ws,
                    int32_t* __restrict__ mask, int64_t* __restrict__ idx,
                    int32_t* __restrict__ count) {
  using raw = typename Elem<DT>::raw;
  constexpr int VPT = VEC ? static_cast<int>(16 / sizeof(raw)) : 1;   // columns per thread
  constexpr uint32_t kFull = (VPT == 32) ? 0xFFFFFFFFu : ((1u << VPT) - 1u);

  // Launched as a programmatic dependent: x may come from the previous kernel
  // of the stream, which may let this grid start early, so wait for it before
  // any access. Then let the next kernel begin its launch; whatever it reads
  // of this grid's results (mask, indices, count) it reads after its own
  // griddepcontrol.wait, which waits for this whole grid.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  uint32_t* ticket = ws;
  uint32_t* flags = ws + kFlagsOffset / sizeof(uint32_t);

  __shared__ uint32_t s_bits[kMaskWarps][32];
  __shared__ int s_last;
  __shared__ int s_scan[kMaskWarps];
  __shared__ uint32_t s_word[kMaskThreads];
  __shared__ uint16_t s_pos[kPassCols];   // alive columns of one pass, relative to its start

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const bool all_alive = (0.0f > thr);   // max starts at 0: every column alive

  const int64_t nvec = VEC ? cols / VPT : cols;
  const int64_t v = static_cast<int64_t>(blockIdx.x) * 32 + lane;
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * rows_per_cta;
  const int64_t r1 = min(rows, r0 + rows_per_cta);

  uint32_t bits = 0;
  const bool have = (v < nvec);
  if (!all_alive) {
    const raw* col = static_cast<const raw*>(x) + (have ? v * VPT : 0);
    // 4 rows in flight per thread in every batch, the last one included: rows
    // past the chunk load the chunk's last row again (a valid address) and are
    // masked out, so no row is read on its own. A warp whose columns are all
    // alive leaves the loop and reads nothing more.
    for (int64_t r = r0 + warp; r < r1; r += kMaskUnroll * kMaskWarps) {
      if (__all_sync(0xFFFFFFFFu, !have || bits == kFull)) break;
      if (have) {
        if constexpr (VEC) {
          uint4 q[kMaskUnroll];
#pragma unroll
          for (int u = 0; u < kMaskUnroll; ++u)
            q[u] = ld_stream_v4(col + min(r + u * kMaskWarps, r1 - 1) * ld);
#pragma unroll
          for (int u = 0; u < kMaskUnroll; ++u)
            bits |= (r + u * kMaskWarps < r1) ? vec_bits<DT>(q[u], thr) : 0u;
        } else {
          raw q[kMaskUnroll];
#pragma unroll
          for (int u = 0; u < kMaskUnroll; ++u) q[u] = __ldg(col + min(r + u * kMaskWarps, r1 - 1) * ld);
#pragma unroll
          for (int u = 0; u < kMaskUnroll; ++u)
            bits |= (r + u * kMaskWarps < r1 && fabsf(Elem<DT>::to_f(q[u])) > thr) ? 1u : 0u;
        }
      }
    }
  }
  s_bits[warp][lane] = bits;
  __syncthreads();

  if (warp == 0) {
    uint32_t b = 0;
#pragma unroll
    for (int w = 0; w < kMaskWarps; ++w) b |= s_bits[w][lane];
    // Pack lane bits into 32-column words: G lanes share one word.
    constexpr int G = 32 / VPT;
    uint32_t word = b << ((lane % G) * VPT);
#pragma unroll
    for (int off = G / 2; off > 0; off >>= 1) word |= __shfl_xor_sync(0xFFFFFFFFu, word, off);
    if ((lane % G) == 0 && word != 0u) {
      const int64_t w_idx = (static_cast<int64_t>(blockIdx.x) * 32 * VPT + lane * VPT) / 32;
      atomicOr(flags + w_idx, word);
    }
    // __syncwarp orders the other lanes' flag updates before lane 0's
    // release; the acquire half makes every CTA's flags visible to the last
    // one, whose other threads read them after the barrier below.
    __syncwarp();
    if (lane == 0) {
      const uint32_t total = gridDim.x * gridDim.y;
      const uint32_t prev = atom_add_acq_rel(ticket, 1u);
      s_last = (prev == total - 1u) ? 1 : 0;
    }
  }
  __syncthreads();
  if (!s_last) return;

  // ---- Last CTA: stream compaction over the alive words --------------------
  const int64_t nwords = (cols + 31) / 32;
  const bool mask_vec = (reinterpret_cast<uintptr_t>(mask) & 15u) == 0;
  int64_t base = 0;
  for (int64_t w0 = 0; w0 < nwords; w0 += kMaskThreads) {
    const int64_t w = w0 + threadIdx.x;
    uint32_t word = 0;
    if (w < nwords) {
      word = ld_relaxed_gpu(flags + w);
      flags[w] = 0u;
      if (all_alive) word = 0xFFFFFFFFu;
      const int64_t rem = cols - w * 32;
      if (rem < 32) word &= (1u << rem) - 1u;
    }
    // Block-wide exclusive scan of popcounts.
    const int c = __popc(word);
    int incl = c;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int t = __shfl_up_sync(0xFFFFFFFFu, incl, off);
      if (lane >= off) incl += t;
    }
    if (lane == 31) s_scan[warp] = incl;
    s_word[threadIdx.x] = word;
    __syncthreads();
    int warp_base = 0, pass_total = 0;
#pragma unroll
    for (int i = 0; i < kMaskWarps; ++i) {
      if (i < warp) warp_base += s_scan[i];
      pass_total += s_scan[i];
    }
    if (idx) {
      int p = warp_base + (incl - c);
      uint32_t rest = word;
      while (rest) {
        const int e = __ffs(rest) - 1;
        s_pos[p++] = static_cast<uint16_t>(threadIdx.x * 32 + e);
        rest &= rest - 1u;
      }
    }
    __syncthreads();
    const int64_t c0 = w0 * 32;
    const int pcols = static_cast<int>(min(static_cast<int64_t>(kPassCols), cols - c0));
    if (mask) {
      int done = 0;
      if (mask_vec) {
        int4* m4 = reinterpret_cast<int4*>(mask + c0);
        for (int q = threadIdx.x; q < pcols / 4; q += kMaskThreads) {
          const uint32_t b = s_word[q >> 3] >> ((q & 7) * 4);
          m4[q] = make_int4(b & 1u, (b >> 1) & 1u, (b >> 2) & 1u, (b >> 3) & 1u);
        }
        done = pcols & ~3;
      }
      for (int q = done + threadIdx.x; q < pcols; q += kMaskThreads)
        mask[c0 + q] = (s_word[q >> 5] >> (q & 31)) & 1u;
    }
    if (idx)
      for (int j = threadIdx.x; j < pass_total; j += kMaskThreads) idx[base + j] = c0 + s_pos[j];
    base += pass_total;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    if (count) *count = static_cast<int32_t>(base);
    *ticket = 0u;
  }
}

}  // namespace

size_t mask_workspace_bytes(int64_t cols) {
  const size_t words = static_cast<size_t>((cols + 31) / 32);
  const size_t bytes = kFlagsOffset + words * sizeof(uint32_t);
  return (bytes + 255) & ~static_cast<size_t>(255);
}

cudaError_t launch_mask_compact(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld,
                                float thr, int32_t* mask, int64_t* idx, int32_t* count,
                                void* workspace, int sm_count, cudaStream_t stream) {
  const int esize = (dtype == GW_DTYPE_F32) ? 4 : 2;
  const int vpt = 16 / esize;
  const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) && (ld % vpt == 0) &&
                   (cols % vpt == 0);
  const int64_t nvec = vec ? cols / vpt : cols;
  const int64_t col_tiles = (nvec + 31) / 32;
  // Enough CTAs for ~8 resident per SM; at least 32 rows per CTA.
  const int64_t target = static_cast<int64_t>(sm_count > 0 ? sm_count : 148) * 8;
  int64_t row_tiles = (target + col_tiles - 1) / col_tiles;
  const int64_t max_row_tiles = (rows + 31) / 32;
  if (row_tiles > max_row_tiles) row_tiles = max_row_tiles;
  if (row_tiles < 1) row_tiles = 1;
  if (row_tiles > 65535) row_tiles = 65535;
  int64_t rows_per_cta = (rows + row_tiles - 1) / row_tiles;
  if (rows_per_cta > 0) row_tiles = (rows + rows_per_cta - 1) / rows_per_cta;
  if (row_tiles < 1) row_tiles = 1;
  if (col_tiles > 0x7FFFFFFFll) return cudaErrorInvalidValue;

  dim3 grid(static_cast<unsigned>(col_tiles), static_cast<unsigned>(row_tiles));
  uint32_t* ws = static_cast<uint32_t*>(workspace);
#define GW_MASK_LAUNCH(DT, V)                                                               \
  launch_pdl(mask_compact_kernel<DT, V>, grid, dim3(kMaskThreads), stream, x, rows, cols, ld,  \
             thr, rows_per_cta, ws, mask, idx, count)
  switch (dtype) {
    case GW_DTYPE_F16:
      return vec ? GW_MASK_LAUNCH(GW_DTYPE_F16, true) : GW_MASK_LAUNCH(GW_DTYPE_F16, false);
    case GW_DTYPE_BF16:
      return vec ? GW_MASK_LAUNCH(GW_DTYPE_BF16, true) : GW_MASK_LAUNCH(GW_DTYPE_BF16, false);
    case GW_DTYPE_F32:
      return vec ? GW_MASK_LAUNCH(GW_DTYPE_F32, true) : GW_MASK_LAUNCH(GW_DTYPE_F32, false);
    default:
      return cudaErrorInvalidValue;
  }
#undef GW_MASK_LAUNCH
}

}  // namespace gw
