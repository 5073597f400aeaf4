// K1 + K2 + K3 in one launch for small batches with a per-forward activation
// mask (GhostLinear's default dynamic mode at decode sizes, M <= 32 rows):
//
//   alive[k] = (max_m fp32(|x[m, k]|) > thr)          (mask.py:21-59 semantics)
//   y[m, n]  = act( sum_{k alive} x[m, k] * W[n, k] + bias[n] )
//
// The reference runs dead_neuron_mask, torch.nonzero and ghostweight_matmul
// (module.py:103-114): three launches and a host synchronisation; the
// device-count path of this library runs mask, weight packing, gather and
// GEMM as four launches, and its packing reads all of W and writes W' once
// more. Here one clustered kernel does everything, reading x and W once:
//
//   * the k split is over the ORIGINAL columns: CTA s of a cluster of S owns
//     columns [s KS, (s + 1) KS) (KS <= 512, a multiple of 64), so it needs
//     only the alive columns of its own range, and no prefix sum over the
//     whole row is needed: each CTA reads x[:, range] (16-byte loads), ORs
//     the alive bits of its columns over the rows, and numbers its alive
//     columns 0 .. K'_s - 1 with a warp scan over 64 eight-column vectors;
//   * it then writes the alive values of x into the 128-byte-swizzled x' tile
//     (MP = 16 or 32 rows) and gathers W[n0 : n0 + 128, range] with 16-byte
//     loads into the W' tile (vectors without an alive column are not read),
//     keeping only alive columns; both tiles are zero past K'_s up to the next
//     multiple of 64;
//   * one thread issues tcgen05 MMAs D[n, m] = W'[n, :] . x'[m, :] (M = 128
//     output features, N = MP rows of x, K = K'_s) into TMEM; four warps drain
//     the accumulator into shared memory;
//   * after a cluster barrier CTA s sums feature slice s (128 / S features)
//     over the S ranks' partials in rank order (DSMEM loads; the result does
//     not depend on timing), adds the bias, applies the activation, rounds
//     once and stores y; a second cluster barrier keeps every CTA's partials
//     alive until all have been read;
//   * rank 0 of feature block 0 also writes the alive count (the sum of the
//     ranks' K'_s) and, if asked, the int32 mask of all K columns.
//
// Exactly the reference's mask semantics: the running max starts at 0 (so a
// negative threshold keeps every column), NaN never wins it, and the compare
// is a strict fp32 greater-than. Requires x and W rows 16-byte aligned (K, ldx
// and ldw multiples of 8) and K <= 16 * 512. The only wait is the MMA
// completion (bounded, gw_common.cuh); the cluster barriers are reached by
// every thread of every CTA on every path. No TMA, no multicast.
#include <algorithm>
#include <mutex>

#include <cuda.h>

#include "gw_common.cuh"
#include "gw_internal.h"

namespace gw {

namespace {

constexpr int kDyN = 128;                   // output features per block (MMA M)
constexpr int kDyKS = 512;                  // original columns per CTA, at most
constexpr int kDyVec = kDyKS / 8;           // 16-byte vectors per row of a range (64)
constexpr int kDyAtoms = kDyKS / 64;        // k atoms of 64 columns, at most
constexpr int kDyThreads = 256;
constexpr int kDyMaxRows = 32;

template <int MP>
struct DyCfg {
  static constexpr int kWAtomBytes = kDyN * 128;            // 128 rows x 64 columns x 2 B
  static constexpr int kXAtomBytes = MP * 128;
  static constexpr int kWBytes = kDyAtoms * kWAtomBytes;    // 128 KB
  static constexpr int kXBytes = kDyAtoms * kXAtomBytes;    // 16 or 32 KB
  static constexpr int kPartStride = MP + 4;                // floats per feature row (16-byte rows)
  static constexpr int kPartBytes = kDyN * kPartStride * 4;
  static constexpr int kTmemCols = 32;
  // Per warp, two rows of W's range staged densely (kStageRows x 1 KB).
  static constexpr int kStageRows = 4;
  static constexpr int kStageBytes = 8 * kStageRows * kDyKS * 2;   // 32 KB
  static constexpr int kMiscBytes = 2048;                          // bits, positions, alive list, barriers
  static constexpr int kSmemBytes = 1024 + kWBytes + kXBytes + kStageBytes + kMiscBytes;
  static_assert(kPartBytes <= kWBytes, "partials live in the W' tile after the MMAs");
  static_assert(kSmemBytes <= 232448, "shared memory budget per CTA");
};

struct DyParams {
  const uint16_t* x;
  int64_t ldx;
  int64_t M;
  int64_t K;
  const uint16_t* w;         // W [N, K] (nn.Linear weight), row stride ldw
  int64_t ldw;
  int64_t N;
  float thr;
  const uint16_t* bias;
  int epi;
  uint16_t* y;
  int64_t ldy;
  int y_vec_ok;
  int ks;                    // columns per rank (multiple of 64, <= kDyKS)
  int split;                 // cluster size S
  int32_t* count;            // alive count (rank 0 of block 0), may be null
  int32_t* mask;             // int32 [K] mask (ranks of block 0), may be null
  unsigned int* err;
};

// Not volatile: used only after the cluster barrier that publishes the data
// (an asm volatile with a memory clobber, which nothing moves across), so the
// compiler may issue many of these loads before using any.
__device__ __forceinline__ float ld_dsmem_f32(uint32_t cluster_addr) {
  float v;
  asm("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr));
  return v;
}
__device__ __forceinline__ int32_t ld_dsmem_s32(uint32_t cluster_addr) {
  int32_t v;
  asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(cluster_addr) : "memory");
  return v;
}

// Byte offset of element (row r, column c) of a K-major tile of 64-column
// atoms (atom_bytes apart), each row 128 bytes with 16-byte chunk j stored at
// chunk position j ^ (r % 8) (the 128-byte swizzle the MMA descriptors read).
__device__ __forceinline__ uint32_t tile_off(int r, int c, int atom_bytes) {
  const int a = c >> 6;
  const int cc = c & 63;
  return static_cast<uint32_t>(a * atom_bytes + r * 128 + ((((cc >> 3) ^ r) & 7) << 4) + ((cc & 7) << 1));
}

// Alive bits of the eight 16-bit values of a vector: |v| > thr in fp32; NaN
// compares false.
template <int DT>
__device__ __forceinline__ uint32_t alive8(const uint4 q, float thr) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
  uint32_t b = 0;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float lo = Elem<DT>::to_f(static_cast<uint16_t>(w[e] & 0xFFFFu));
    const float hi = Elem<DT>::to_f(static_cast<uint16_t>(w[e] >> 16));
    b |= (fabsf(lo) > thr ? 1u : 0u) << (2 * e);
    b |= (fabsf(hi) > thr ? 1u : 0u) << (2 * e + 1);
  }
  return b;
}

// 16-byte load issued only when `pred` is set (zeros otherwise); inline PTX so
// that a batch of such loads is issued back to back, none behind a branch.
__device__ __forceinline__ uint4 ld_nc_v4_if(const void* p, bool pred) {
  uint4 v;
  asm volatile(
      "{\n\t.reg .pred q;\n\t"
      "setp.ne.u32 q, %5, 0;\n\t"
      "mov.u32 %0, 0;\n\tmov.u32 %1, 0;\n\tmov.u32 %2, 0;\n\tmov.u32 %3, 0;\n\t"
      "@q ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];\n\t}"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p), "r"(pred ? 1u : 0u));
  return v;
}

template <int MP, int DT>
__global__ void __launch_bounds__(kDyThreads, 1) gemm_dyn_kernel(const DyParams p) {
  using C = DyCfg<MP>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_s & 1023u)) & 1023u);
  const uint32_t w_s = smem_u32(smem);              // W' tile (later: the partial sums)
  const uint32_t x_s = w_s + C::kWBytes;            // x' tile
  uint8_t* stage = smem + C::kWBytes + C::kXBytes;  // per-warp dense rows of W's range
  uint8_t* misc = stage + C::kStageBytes;
  uint8_t* vb = misc;                                // [4][kDyVec] alive bits per row group
  int32_t* vpos = reinterpret_cast<int32_t*>(misc + 256);    // [kDyVec] first local position
  uint8_t* vmask = misc + 512;                       // [kDyVec] alive bits of the vector
  int32_t* kcount = reinterpret_cast<int32_t*>(misc + 576);  // this rank's K'_s
  const uint32_t mma_bar = smem_u32(misc + 584);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + 592);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 596);
  int16_t* acol = reinterpret_cast<int16_t*>(misc + 1024);   // [kDyKS] range column of alive p
  float* part = reinterpret_cast<float*>(smem);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int rank = static_cast<int>(cluster_ctarank());    // == blockIdx.x
  const int n_blk = static_cast<int>(blockIdx.y);
  const int S = p.split;
  const int64_t col0 = static_cast<int64_t>(rank) * p.ks;
  const int64_t rem_cols = p.K - col0;
  const int ncols = rem_cols <= 0 ? 0 : static_cast<int>(rem_cols < p.ks ? rem_cols : p.ks);
  const int nvec = ncols >> 3;                       // K is a multiple of 8
  const int64_t n0 = static_cast<int64_t>(n_blk) * kDyN;
  const int rows = static_cast<int>(p.M);

  if (tid == 0) {
    mbar_init(mma_bar, 1);
    *abort_flag = 0;
    mbar_init_fence();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");   // x (and W) may come from the previous kernel

  // ---------------------------------------------------------------- A: x and its alive bits
  // Thread t: vector v = t % 64 of the range, rows g, g + 4, ... (g = t / 64).
  constexpr int RPT = MP / 4;
  const int v = tid & (kDyVec - 1);
  const int g = tid >> 6;
  uint4 xv[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int r = g + 4 * i;
    const bool ok = v < nvec && r < rows;
    xv[i] = ld_nc_v4_if(p.x + (ok ? static_cast<int64_t>(r) * p.ldx + col0 + 8 * v : 0), ok);
  }
  uint32_t bits = 0;
#pragma unroll
  for (int i = 0; i < RPT; ++i)
    if (v < nvec && g + 4 * i < rows) bits |= alive8<DT>(xv[i], p.thr);
  if (0.0f > p.thr && v < nvec) bits = 0xFFu;        // the running max starts at 0
  vb[g * kDyVec + v] = static_cast<uint8_t>(bits);
  __syncthreads();

  // ---------------------------------------------------------------- B: number the alive columns
  if (warp == 0) {
    const uint32_t m0 = vb[lane] | vb[kDyVec + lane] | vb[2 * kDyVec + lane] | vb[3 * kDyVec + lane];
    const int l1 = lane + 32;
    const uint32_t m1 = vb[l1] | vb[kDyVec + l1] | vb[2 * kDyVec + l1] | vb[3 * kDyVec + l1];
    const int c0 = __popc(m0), c1 = __popc(m1);
    int s0 = c0, s1 = c1;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int t0 = __shfl_up_sync(0xFFFFFFFFu, s0, off);
      const int t1 = __shfl_up_sync(0xFFFFFFFFu, s1, off);
      if (lane >= off) { s0 += t0; s1 += t1; }
    }
    const int total0 = __shfl_sync(0xFFFFFFFFu, s0, 31);
    vpos[lane] = s0 - c0;
    vpos[l1] = total0 + s1 - c1;
    vmask[lane] = static_cast<uint8_t>(m0);
    vmask[l1] = static_cast<uint8_t>(m1);
    if (lane == 31) *kcount = total0 + s1;
  }
  __syncthreads();
  const int kp = *kcount;
  const int nkb = (kp + 63) >> 6;
  if (p.mask && n_blk == 0)
    for (int c = tid; c < ncols; c += kDyThreads) p.mask[col0 + c] = (vmask[c >> 3] >> (c & 7)) & 1;

  // ---------------------------------------------------------------- C: x' and W' tiles
  // The last k atom is zero past K'_s (the MMA reads whole 16-column steps and
  // 0 * stale data could be NaN); the alive list acol[p] = range column of the
  // p-th alive column is written at the same time.
  if (kp & 63) {
    const uint32_t wa = w_s + static_cast<uint32_t>((nkb - 1) * C::kWAtomBytes);
    const uint32_t xa = x_s + static_cast<uint32_t>((nkb - 1) * C::kXAtomBytes);
    for (int o = tid * 16; o < C::kWAtomBytes; o += kDyThreads * 16)
      asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" :: "r"(wa + o), "r"(0u) : "memory");
    for (int o = tid * 16; o < C::kXAtomBytes; o += kDyThreads * 16)
      asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" :: "r"(xa + o), "r"(0u) : "memory");
  }
  if (tid < nvec) {
    uint32_t mv = vmask[tid];
    int pv = vpos[tid];
    while (mv) {
      const int e = __ffs(mv) - 1;
      acol[pv++] = static_cast<int16_t>(8 * tid + e);
      mv &= mv - 1u;
    }
  }
  __syncthreads();
  // Lane l produces alive positions p = 32 i + l: its range columns, once.
  constexpr int kMaxI = kDyKS / 32;
  const int ni = (kp + 31) >> 5;
  int cp[kMaxI];
#pragma unroll
  for (int i = 0; i < kMaxI; ++i) {
    const int pp = 32 * i + lane;
    cp[i] = pp < kp ? acol[pp] : 0;
  }
  // x': rows warp, warp + 8, ... of x, 2-byte loads of the alive columns
  // (x is small and was just read, so these come from L2).
  for (int r = warp; r < rows; r += 8) {
    const uint16_t* xr = p.x + static_cast<int64_t>(r) * p.ldx + col0;
    uint16_t xv2[kMaxI];
    // Unconditional loads (an invalid position reads column 0 of the range and
    // is not stored), so that all of a row's loads are in flight at once.
#pragma unroll
    for (int i = 0; i < kMaxI; ++i) xv2[i] = __ldg(xr + cp[i]);
#pragma unroll
    for (int i = 0; i < kMaxI; ++i)
      if (i < ni && 32 * i + lane < kp)
        *reinterpret_cast<uint16_t*>(smem + C::kWBytes + tile_off(r, 32 * i + lane, C::kXAtomBytes)) = xv2[i];
  }
  {
    // W': warp w handles rows 16 w .. 16 w + 15 of the feature block in four
    // batches of four rows. A batch is read densely (16-byte loads; vectors
    // with no alive column and rows past N are not read) into the warp's
    // staging rows, then lane l copies alive positions 32 i + l from there
    // into the swizzled tile. The next batch's loads are issued before the
    // current batch is staged, so they are in flight during the copies.
    uint8_t* st_w = stage + warp * (C::kStageRows * kDyKS * 2);
    const uint32_t st_s = smem_u32(st_w);
    const bool liveA = vmask[lane] != 0, liveB = vmask[lane + 32] != 0;
    auto load_batch = [&](int b, uint4 (&q)[C::kStageRows][2]) {
#pragma unroll
      for (int j = 0; j < C::kStageRows; ++j) {
        const int r = warp * 16 + b * C::kStageRows + j;
        const bool live = n0 + r < p.N;
        const uint16_t* wr = p.w + (live ? (n0 + r) * p.ldw + col0 : 0);
        q[j][0] = ld_nc_v4_if(wr + 8 * lane, live && liveA);
        q[j][1] = ld_nc_v4_if(wr + 8 * (lane + 32), live && liveB);
      }
    };
    uint4 qa[C::kStageRows][2], qb[C::kStageRows][2];
    load_batch(0, qa);
#pragma unroll
    for (int b = 0; b < 16 / C::kStageRows; ++b) {
      uint4 (&cur)[C::kStageRows][2] = (b & 1) ? qb : qa;
      uint4 (&nxt)[C::kStageRows][2] = (b & 1) ? qa : qb;
      if (b + 1 < 16 / C::kStageRows) load_batch(b + 1, nxt);
#pragma unroll
      for (int j = 0; j < C::kStageRows; ++j) {
        reinterpret_cast<uint4*>(st_w + j * kDyKS * 2)[lane] = cur[j][0];
        reinterpret_cast<uint4*>(st_w + j * kDyKS * 2)[lane + 32] = cur[j][1];
      }
      __syncwarp();
      // Plain loads and stores: the compiler issues a row's loads together.
      const uint16_t* st16 = reinterpret_cast<const uint16_t*>(st_w);
#pragma unroll
      for (int j = 0; j < C::kStageRows; ++j) {
        const int r = warp * 16 + b * C::kStageRows + j;
        uint16_t vals[kMaxI];
#pragma unroll
        for (int i = 0; i < kMaxI; ++i) vals[i] = st16[j * kDyKS + cp[i]];
#pragma unroll
        for (int i = 0; i < kMaxI; ++i)
          if (i < ni && 32 * i + lane < kp)
            *reinterpret_cast<uint16_t*>(smem + tile_off(r, 32 * i + lane, C::kWAtomBytes)) = vals[i];
      }
      __syncwarp();                                  // the staging rows are free again
    }
  }
  fence_proxy_async_smem();                          // the tiles are read by the tensor core
  __syncthreads();

  // ---------------------------------------------------------------- D: MMAs into TMEM
  if (tid == 0 && nkb > 0) {
    constexpr uint32_t idesc = idesc_f16(DT == GW_DTYPE_BF16 ? 1u : 0u, kDyN, MP);
    tc_fence_after();
    for (int kb = 0; kb < nkb; ++kb) {
      const uint64_t wd = smem_desc_kmajor_sw128(w_s + static_cast<uint32_t>(kb * C::kWAtomBytes));
      const uint64_t xd = smem_desc_kmajor_sw128(x_s + static_cast<uint32_t>(kb * C::kXAtomBytes));
#pragma unroll
      for (int k = 0; k < 4; ++k)
        tc_mma_f16(tmem_base, wd + 2u * k, xd + 2u * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
    }
    tc_commit(mma_bar);
  }

  // ---------------------------------------------------------------- E: drain to shared memory
  // Warp w < 4 reads TMEM lanes 32 w .. 32 w + 31 (features of the block);
  // column m is row m of x. The partial sums overwrite the W' tile, so they
  // are written only after the MMAs have finished reading it.
  if (warp < 4) {
    uint32_t acc[MP];
#pragma unroll
    for (int c = 0; c < MP; ++c) acc[c] = 0u;
    if (nkb > 0 && mbar_wait(mma_bar, 0u, abort_flag, p.err)) {
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < MP; c += 16)
        tc_ld_32x32b_x16(tmem_base + (static_cast<uint32_t>(warp * 32) << 16) + c, acc + c);
      tc_wait_ld();
    }
    tc_fence_before();
    float4* row = reinterpret_cast<float4*>(part + (warp * 32 + lane) * C::kPartStride);
#pragma unroll
    for (int m = 0; m < MP; m += 4)
      row[m / 4] = make_float4(__uint_as_float(acc[m]), __uint_as_float(acc[m + 1]),
                               __uint_as_float(acc[m + 2]), __uint_as_float(acc[m + 3]));
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }

  // ---------------------------------------------------------------- F: cluster reduction
  cluster_sync();                                    // every rank's partials are in place
  {
    const int f0 = rank * kDyN / S;
    const int f1 = (rank + 1) * kDyN / S;
    const int nf = f1 - f0;
    const uint32_t part_s = w_s;
    // Up to four outputs per thread and pass, all of their S partials loaded
    // before any is added (sums in rank order: the result is reproducible).
    constexpr int kT = 4;
    const int tasks = rows * nf;
    for (int t0 = tid; t0 < tasks; t0 += kT * kDyThreads) {
      float part_q[kT][16];
#pragma unroll
      for (int u = 0; u < kT; ++u) {
        const int t = t0 + u * kDyThreads;
        const int m = t < tasks ? t / nf : 0;
        const int f = t < tasks ? f0 + (t - m * nf) : f0;
        const uint32_t local = part_s + static_cast<uint32_t>((f * C::kPartStride + m) * 4);
#pragma unroll
        for (int q = 0; q < 16; ++q)
          part_q[u][q] = q < S ? ld_dsmem_f32(mapa_shared(local, static_cast<uint32_t>(q))) : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < kT; ++u) {
        const int t = t0 + u * kDyThreads;
        if (t >= tasks) continue;
        const int m = t / nf;
        const int64_t n = n0 + f0 + (t - m * nf);
        if (n >= p.N) continue;
        float s = 0.0f;
#pragma unroll
        for (int q = 0; q < 16; ++q)
          if (q < S) s += part_q[u][q];
        if (p.bias) s += Elem<DT>::to_f(__ldg(p.bias + n));
        s = apply_epilogue16(s, p.epi);
        p.y[static_cast<int64_t>(m) * p.ldy + n] = Elem<DT>::from_f(s);
      }
    }
    if (p.count && n_blk == 0 && rank == 0 && tid == 0) {
      int32_t total = 0;
      const uint32_t kc = smem_u32(kcount);
      for (int q = 0; q < S; ++q) total += ld_dsmem_s32(mapa_shared(kc, static_cast<uint32_t>(q)));
      *p.count = total;
    }
  }
  cluster_sync();                                    // no rank leaves while others read its partials
}

template <int MP, int DT>
cudaError_t launch_dyn(const DyParams& p, int64_t blocks, cudaStream_t stream) {
  auto kern = gemm_dyn_kernel<MP, DT>;
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kern), DyCfg<MP>::kSmemBytes);
  if (e != cudaSuccess) return e;
  if (p.split > 8) {
    // Clusters of 9 to 16 CTAs are a non-portable size.
    static std::once_flag once[64];
    int dev = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if (dev >= 0 && dev < 64)
      std::call_once(once[dev], [&] {
        if (cudaFuncSetAttribute(reinterpret_cast<const void*>(kern),
                                 cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
          (void)cudaGetLastError();
      });
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.split), static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(kDyThreads);
  cfg.dynamicSmemBytes = DyCfg<MP>::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(p.split);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

}  // namespace

bool dyn_linear_supported(int64_t M, int64_t K) {
  return M >= 1 && M <= kDyMaxRows && K >= 8 && (K % 8) == 0 && K <= 16 * kDyKS;
}

cudaError_t launch_dyn_linear(const void* x, int dtype, int64_t M, int64_t K, int64_t ldx,
                              const void* w, int64_t N, int64_t ldw, float thr, const void* bias,
                              int epilogue, void* y, int64_t ldy, int32_t* count, int32_t* mask,
                              unsigned int* err, cudaStream_t stream) {
  if (!dyn_linear_supported(M, K) || N <= 0) return cudaErrorInvalidValue;
  const int64_t blocks = (N + kDyN - 1) / kDyN;
  if (blocks > 65535) return cudaErrorInvalidValue;
  DyParams p{};
  p.x = static_cast<const uint16_t*>(x);
  p.ldx = ldx;
  p.M = M;
  p.K = K;
  p.w = static_cast<const uint16_t*>(w);
  p.ldw = ldw;
  p.N = N;
  p.thr = thr;
  p.bias = static_cast<const uint16_t*>(bias);
  p.epi = epilogue;
  p.y = static_cast<uint16_t*>(y);
  p.ldy = ldy;
  p.split = static_cast<int>((K + kDyKS - 1) / kDyKS);
  p.ks = static_cast<int>(((K + p.split - 1) / p.split + 63) / 64 * 64);
  p.count = count;
  p.mask = mask;
  p.err = err;
  const bool bf = dtype == GW_DTYPE_BF16;
  if (M <= 16) return bf ? launch_dyn<16, GW_DTYPE_BF16>(p, blocks, stream) : launch_dyn<16, GW_DTYPE_F16>(p, blocks, stream);
  return bf ? launch_dyn<32, GW_DTYPE_BF16>(p, blocks, stream) : launch_dyn<32, GW_DTYPE_F16>(p, blocks, stream);
}

}  // namespace gw
