// K3, small-M variant: split-K over a thread-block cluster, reduced in
// distributed shared memory.
//
//   y[m, n] = act( sum_j a[m, j] * w[n, j] + bias[n] )      a = x' (dense, compacted)
//
// When the output has too few 128 x BN tiles to occupy the SMs (a few dozen
// to a few hundred rows: small batches; at most 32 rows usually go to the
// decode kernel, gw_gemm_decode.cu), the persistent kernels
// leave most SMs idle and each busy SM streams a long k range alone. Here a
// cluster of S CTAs (S = 2, 4 or 8) shares one output tile: CTA s of the
// cluster accumulates k-blocks [s * nkb / S, (s + 1) * nkb / S) on its tensor
// cores (tcgen05, TMEM accumulator), so S times as many SMs stream W' and x'.
// The partial tiles never leave the chip:
//   1. each CTA drains its accumulator (valid rows only) into its own shared
//      memory, fp32, row stride BN + 4 words (bank-conflict-free 16-byte rows);
//   2. cluster barrier;
//   3. CTA s reduces column slice [s * BN / S, (s + 1) * BN / S) of the tile,
//      reading the S partial tiles over DSMEM in fixed order s' = 0..S-1 (the
//      result does not depend on timing), adds bias, applies the activation,
//      rounds once and stores y;
//   4. relaxed cluster arrive once every DSMEM read of the CTA has completed,
//      then cluster wait (peers' shared memory stays valid until every read;
//      the stores of y need no ordering with the peers).
// The plan (tile width BN, cluster size S) minimises a cost estimate fitted to
// measured times (plan_splitk below).
// The cluster is gang-scheduled, so its barriers cannot wait on a CTA that is
// not running; every other wait is bounded (gw_common.cuh). No TMA multicast.
//
// Roles (192 threads): warp 0 TMA producer, warp 1 TMEM allocator + MMA
// issuer, warps 2..5 TMEM drain; all six warps share the reduction.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <initializer_list>
#include <mutex>

#include <cuda.h>

#include "gw_common.cuh"
#include "gw_internal.h"

namespace gw {

namespace {

constexpr int kSkBM = 128;
constexpr int kSkBK = 64;
constexpr int kSkThreads = 192;

template <int BN>
struct SkCfg {
  static constexpr int kABytes = kSkBM * kSkBK * 2;
  static constexpr int kBBytes = BN * kSkBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStagesFit = (196 * 1024) / kStageBytes;
  static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
  static constexpr int kRedStride = BN + 4;                       // floats per partial row
  static constexpr int kRedBytes = kSkBM * kRedStride * 4;
  static constexpr int kRingBytes =
      kStages * kStageBytes > kRedBytes ? kStages * kStageBytes : kRedBytes;
  // Up to 128 columns a stage's four MMAs take fewer tensor cycles than one
  // issuing thread needs (about 200 cycles per stage wait, 70-80 per MMA), so
  // two threads issue: even k-blocks into accumulator 0, odd ones into
  // accumulator 1 (BN columns further on), which the drain adds.
  static constexpr bool kDual = BN <= 128;
  static constexpr int kAccCols = kDual ? 2 * BN : BN;
  static constexpr int kTmemCols = kAccCols < 32 ? 32 : kAccCols;  // power of two >= 32
  static constexpr int kSmemBytes = 1024 + kRingBytes + 256;
  static_assert(kSmemBytes <= 232448, "shared memory budget per CTA");
};

struct SkParams {
  int64_t M;
  int64_t N;
  const uint16_t* bias;
  int epi;
  uint16_t* y;
  int64_t ldy;
  int y_vec_ok;              // 8-byte stores of four outputs allowed
  int num_kb;
  int m_tiles;
  int split;                 // cluster size S
  int a_tx_bytes;            // bytes of one x' box (its rows: min(M rounded up to 8, 128))
  unsigned int* err;
  const int64_t* a_cols;     // alive columns in 64-column runs: A is x, k-block kb at a_cols[64 kb]
  int64_t a_width;           // columns of x (with a_cols)
};

__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t cluster_addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(cluster_addr) : "memory");
  return v;
}

// CTA `rank` of the cluster sums column slice [rank * BN / S, (rank + 1) * BN / S)
// of the S partial tiles (row stride BN + 4 floats at `red_local` in every
// CTA) and emits it. Each thread owns one group of four columns of the slice
// and walks the rows rows0, rows0 + step, ... (step = threads / groups), so the
// bias, the column bounds and the output pointer are set up once per thread;
// per row it loads the S partial float4s (16 / S rows per round, all loads
// issued before the first add so their latencies overlap), sums them in rank
// order (the result does not depend on timing), applies the epilogue and
// stores four outputs. (A mapping of one (row, group) task per iteration spent
// about 200 cycles of dependent index arithmetic per task with six warps per SM.)
template <int S, int BN, int DT, int EPI>
__device__ __forceinline__ void reduce_slice(const SkParams& p, uint32_t red_local, int rank,
                                             int m_blk, int n_blk, int rows_valid, bool ok) {
  constexpr int kStride = SkCfg<BN>::kRedStride;
  constexpr int kGroups = BN / 4 / S;              // float4 groups per row in this CTA's slice
  constexpr int kStep = kSkThreads / kGroups;      // rows between two rows of one thread
  constexpr int kRows = 16 / S;                    // rows per round: 16 loads in flight
  static_assert(kSkThreads % kGroups == 0, "every thread owns one column group");
  const int grp = static_cast<int>(threadIdx.x) % kGroups;
  const int row0 = static_cast<int>(threadIdx.x) / kGroups;
  const int col = (rank * kGroups + grp) * 4;      // first column of the group in the tile
  const int64_t n0 = static_cast<int64_t>(n_blk) * BN + col;
  float b[4] = {0.f, 0.f, 0.f, 0.f};
  if (p.bias) add_bias4<DT>(b, p.bias, n0, p.N);
  const bool vec = p.y_vec_ok && n0 + 4 <= p.N;
  const int64_t y_step = static_cast<int64_t>(kStep) * p.ldy;
  uint16_t* yp = p.y + (static_cast<int64_t>(m_blk) * kSkBM + row0) * p.ldy + n0;
  const uint32_t col_addr = red_local + static_cast<uint32_t>(col * 4);
  float sink = 0.f;
  for (int r = row0; r < rows_valid; r += kRows * kStep, yp += kRows * y_step) {
    float4 v[kRows][S];
#pragma unroll
    for (int u = 0; u < kRows; ++u) {
      if (r + u * kStep < rows_valid) {
        const uint32_t addr = col_addr + static_cast<uint32_t>((r + u * kStep) * kStride * 4);
#pragma unroll
        for (int s = 0; s < S; ++s) v[u][s] = ld_dsmem_f4(mapa_shared(addr, s));
      }
    }
    if (!ok) {
      // This CTA's accumulator never arrived (error recorded): no outputs, but
      // the loaded values are consumed, so every read of a peer's shared memory
      // has completed before the caller's relaxed cluster arrive.
#pragma unroll
      for (int u = 0; u < kRows; ++u) {
        if (r + u * kStep < rows_valid) {
#pragma unroll
          for (int s = 0; s < S; ++s) sink += v[u][s].x + v[u][s].y + v[u][s].z + v[u][s].w;
        }
      }
      continue;
    }
#pragma unroll
    for (int u = 0; u < kRows; ++u) {
      if (r + u * kStep >= rows_valid) break;
      float4 acc = v[u][0];
#pragma unroll
      for (int s = 1; s < S; ++s) {
        acc.x += v[u][s].x; acc.y += v[u][s].y; acc.z += v[u][s].z; acc.w += v[u][s].w;
      }
      float f[4] = {acc.x, acc.y, acc.z, acc.w};
      if (p.bias) {
#pragma unroll
        for (int j = 0; j < 4; ++j) f[j] += b[j];
      }
      activate4<EPI>(f);
      uint16_t* yr = yp + u * y_step;
      if (vec) {
        const uint32_t lo = static_cast<uint32_t>(Elem<DT>::from_f(f[0])) |
                            (static_cast<uint32_t>(Elem<DT>::from_f(f[1])) << 16);
        const uint32_t hi = static_cast<uint32_t>(Elem<DT>::from_f(f[2])) |
                            (static_cast<uint32_t>(Elem<DT>::from_f(f[3])) << 16);
        *reinterpret_cast<uint2*>(yr) = make_uint2(lo, hi);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (n0 + j < p.N) yr[j] = Elem<DT>::from_f(f[j]);
      }
    }
  }
  asm volatile("" ::"f"(sink));
}

// Issues the MMAs of k-blocks first, first + step, ... of this CTA's range
// (local indices) into accumulator d, one commit per k-block to its stage's
// empty barrier, then one to tfull (or raises the abort flag) and one to
// drain_bar.
template <int BN, int DT, typename FullF, typename EmptyF>
__device__ __forceinline__ void sk_issue(const SkParams& p, uint32_t sbase, uint32_t d, int nk,
                                         int first, int step, FullF full, EmptyF empty,
                                         uint32_t tfull, uint32_t drain_bar,
                                         volatile int* abort_flag) {
  using C = SkCfg<BN>;
  constexpr uint32_t idesc = idesc_f16(DT == GW_DTYPE_BF16 ? 1u : 0u, kSkBM, BN);
  bool ok = true;
  for (int used = first; used < nk; used += step) {
    const int s = used % C::kStages;
    const uint32_t ph = (used / C::kStages) & 1u;
    if (!mbar_wait(full(s), ph, abort_flag, p.err)) { ok = false; break; }
    tc_fence_after();
    const uint32_t a_s = sbase + s * C::kStageBytes;
    const uint64_t a_desc = smem_desc_kmajor_sw128(a_s);
    const uint64_t b_desc = smem_desc_kmajor_sw128(a_s + C::kABytes);
#pragma unroll
    for (int k = 0; k < kSkBK / 16; ++k)
      tc_mma_f16(d, a_desc + 2u * k, b_desc + 2u * k, idesc, (used > first || k > 0) ? 1u : 0u);
    tc_commit(empty(s));
  }
  if (ok) tc_commit(tfull);
  else *abort_flag = 1;            // the drain warps stop waiting for tfull
  tc_commit(drain_bar);
}

template <int BN, int DT, int EPI>
__global__ void __launch_bounds__(kSkThreads, 1)
gemm_splitk_kernel(const __grid_constant__ CUtensorMap tmap_b,
                   const __grid_constant__ CUtensorMap tmap_a, const SkParams p) {
  using C = SkCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_s & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  uint8_t* bar_region = smem + C::kRingBytes;
  const uint32_t bar0 = smem_u32(bar_region);
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (C::kStages + s); };
  const uint32_t tfull = bar0 + 8u * (2 * C::kStages);
  const uint32_t drain_bar = tfull + 8u;
  static_assert(8 * (2 * 8 + 2) <= 192, "barrier region overflows into the TMEM slot");
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_region + 192);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bar_region + 196);
  volatile int* acc_ok = reinterpret_cast<volatile int*>(bar_region + 200);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = static_cast<int>(cluster_ctarank());   // == blockIdx.x, the k split
  const int tile = static_cast<int>(blockIdx.y);
  const int m_blk = tile % p.m_tiles;
  const int n_blk = tile / p.m_tiles;
  const int kb0 = static_cast<int>(static_cast<int64_t>(rank) * p.num_kb / p.split);
  const int kb1 = static_cast<int>(static_cast<int64_t>(rank + 1) * p.num_kb / p.split);
  const int64_t rows_left = p.M - static_cast<int64_t>(m_blk) * kSkBM;
  const int rows_valid = rows_left >= kSkBM ? kSkBM : static_cast<int>(rows_left);
  const bool dual = C::kDual && kb1 - kb0 >= 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    mbar_init(tfull, dual ? 2 : 1);       // one commit per issuing thread
    mbar_init(drain_bar, dual ? 2 : 1);
    *abort_flag = 0;
    *acc_ok = 0;
    mbar_init_fence();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      asm volatile("griddepcontrol.wait;" ::: "memory");   // x' may come from the previous kernel
      int issued = 0;
      bool ok = true;
      int64_t nxt = p.a_cols ? run_start_load(p.a_cols, kb0) : 0;   // next k-block's run start
      for (int kb = kb0; kb < kb1; ++kb, ++issued) {
        const int s = issued % C::kStages;
        const uint32_t ph = (issued / C::kStages) & 1u;
        const int64_t cur = nxt;
        if (p.a_cols && kb + 1 < kb1) nxt = run_start_load(p.a_cols, kb + 1);
        if (!mbar_wait(empty(s), ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
        const uint32_t a_s = sbase + s * C::kStageBytes;
        mbar_arrive_expect_tx(full(s), C::kBBytes + p.a_tx_bytes);
        tma_load_2d(a_s + C::kABytes, &tmap_b, kb * kSkBK, n_blk * BN, full(s));
        const int ax = p.a_cols ? run_start_check(cur, p.a_width, p.err) : kb * kSkBK;
        tma_load_2d(a_s, &tmap_a, ax, m_blk * kSkBM, full(s));
      }
      if (!ok) {
        // Loads still in flight complete before the ring is reused or the CTA exits.
        const int first = issued > C::kStages ? issued - C::kStages : 0;
        for (int i = first; i < issued; ++i)
          mbar_wait(full(i % C::kStages), (i / C::kStages) & 1u, nullptr, p.err, 100000000ull);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even k-blocks)
    if (lane == 0) {
      sk_issue<BN, DT>(p, sbase, tmem_base, kb1 - kb0, 0, dual ? 2 : 1, full, empty, tfull, drain_bar,
                       abort_flag);
      // Every MMA (of both issuers) has finished reading shared memory and
      // writing TMEM before the ring is reused as the reduction buffer and
      // TMEM is freed.
      mbar_wait(drain_bar, 0u, nullptr, p.err, 100000000ull);
    }
    __syncwarp();
  } else {
    if (dual && warp == 2) {
      // ---------------------------------------------------------- MMA issuer (odd k-blocks)
      if (lane == 0)
        sk_issue<BN, DT>(p, sbase, tmem_base + BN, kb1 - kb0, 1, 2, full, empty, tfull, drain_bar,
                         abort_flag);
      __syncwarp();
    }
    // ------------------------------------------------------------ TMEM drain
    // Warp w reads TMEM lanes 32 (w % 4) .. +31 = rows of the tile.
    const int q = warp & 3;
    const int row = q * 32 + lane;
    if (mbar_wait(tfull, 0u, abort_flag, p.err)) {
      tc_fence_after();
      if (q * 32 < rows_valid) {
        float* red_row = reinterpret_cast<float*>(smem) + row * C::kRedStride;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t acc[32];
          const uint32_t t_chunk = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + c * 32;
          tc_ld_32x32b_x32(t_chunk, acc);
          if (dual) {
            uint32_t odd[32];
            tc_ld_32x32b_x32(t_chunk + BN, odd);
            tc_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j)
              acc[j] = __float_as_uint(__uint_as_float(acc[j]) + __uint_as_float(odd[j]));
          } else {
            tc_wait_ld();
          }
          if (row < rows_valid) {
            float4* dst = reinterpret_cast<float4*>(red_row + c * 32);
#pragma unroll
            for (int v = 0; v < 8; ++v)
              dst[v] = make_float4(__uint_as_float(acc[4 * v]), __uint_as_float(acc[4 * v + 1]),
                                   __uint_as_float(acc[4 * v + 2]), __uint_as_float(acc[4 * v + 3]));
          }
        }
      }
      if (q == 0 && lane == 0) *acc_ok = 1;
    }
    tc_fence_before();
  }

  // The ring must be idle before it is overwritten: the drain above runs only
  // after tfull, which follows the last MMA; on an error path the MMA warp has
  // drained the tensor pipe and the producer its loads before this barrier.
  __syncthreads();
  cluster_sync();                      // every partial tile of the cluster is in shared memory

  // ------------------------------------------------------------ reduce-scatter over DSMEM
  {
    const bool ok = *acc_ok != 0;
    if (p.split == 8) reduce_slice<8, BN, DT, EPI>(p, smem_u32(smem), rank, m_blk, n_blk, rows_valid, ok);
    else if (p.split == 4) reduce_slice<4, BN, DT, EPI>(p, smem_u32(smem), rank, m_blk, n_blk, rows_valid, ok);
    else reduce_slice<2, BN, DT, EPI>(p, smem_u32(smem), rank, m_blk, n_blk, rows_valid, ok);
  }

  // Every DSMEM read of this thread has completed: its values were stored to y
  // or consumed. The outputs need no ordering with the peers, so the arrive is
  // relaxed and does not wait for the stores of y to be acknowledged.
  cluster_arrive_relaxed();
  cluster_wait();                      // peers have finished reading this CTA's partial tile
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

template <int BN, int DT>
cudaError_t launch_sk(const CUtensorMap& tb, const CUtensorMap& ta, const SkParams& p,
                      int64_t tiles, cudaStream_t stream) {
  using C = SkCfg<BN>;
  // One instantiation per activation: the reduction loop is unrolled over
  // 16 / S tasks, and runtime-selected activation code in it ran cold in the
  // instruction cache.
  auto kern = p.epi == GW_EPI_GELU_ERF    ? gemm_splitk_kernel<BN, DT, GW_EPI_GELU_ERF>
              : p.epi == GW_EPI_GELU_TANH ? gemm_splitk_kernel<BN, DT, GW_EPI_GELU_TANH>
                                          : gemm_splitk_kernel<BN, DT, GW_EPI_NONE>;
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kern), C::kSmemBytes);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.split), static_cast<unsigned>(tiles));
  cfg.blockDim = dim3(kSkThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
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
  return cudaLaunchKernelEx(&cfg, kern, tb, ta, p);
}

// Clusters of S CTAs of the BN-wide kernel that fit on the current device at
// once, for BN in {256, 128, 64, 32} x S in {8, 4, 2} (occupancy queries, run
// once per device). Clusters of 8 CTAs that each need most of an SM's shared
// memory do not tile every GPC: on a 148-SM B200 only 15 fit, not 18.
struct ClusterTable {
  int n[4][3];
};

template <int BN>
int query_active_clusters(int s) {
  auto kern = gemm_splitk_kernel<BN, GW_DTYPE_F16, GW_EPI_NONE>;
  constexpr int smem = SkCfg<BN>::kSmemBytes;
  if (ensure_smem_attr(reinterpret_cast<const void*>(kern), smem) != cudaSuccess) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(s), 1);
  cfg.blockDim = dim3(kSkThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(s);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
  return n > 0 ? n : 0;
}

const ClusterTable* cluster_table() {
  static std::mutex mu;
  static ClusterTable tables[64];
  static bool ready[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    (void)cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!ready[dev]) {
    const int ss[3] = {8, 4, 2};
    for (int si = 0; si < 3; ++si) {
      tables[dev].n[0][si] = query_active_clusters<256>(ss[si]);
      tables[dev].n[1][si] = query_active_clusters<128>(ss[si]);
      tables[dev].n[2][si] = query_active_clusters<64>(ss[si]);
      tables[dev].n[3][si] = query_active_clusters<32>(ss[si]);
    }
    (void)cudaGetLastError();
    ready[dev] = true;
  }
  return &tables[dev];
}

}  // namespace

SplitKPlan plan_splitk(int64_t M, int64_t N, int64_t K, int sm_count) {
  SplitKPlan best;
  const int64_t sms = sm_count > 0 ? sm_count : 148;
  const int64_t m_tiles = (M + kSkBM - 1) / kSkBM;
  const int64_t num_kb = (K + kSkBK - 1) / kSkBK;
  if (M <= 0 || N <= 0 || num_kb < 2) return best;
  // The persistent kernels already fill at least half of the SMs.
  if (m_tiles * ((N + 255) / 256) * 2 > sms) return best;
  // Among the plans whose clusters all run in one wave, the one with the
  // least estimated time. The estimate is a least-squares fit to measured
  // times of every feasible plan over 60 shapes (M = 48..512, N = 768..11008,
  // K' = 768..11008; back-to-back calls, operands in L2):
  //   0.19 kb + 0.004 load + r_S red   (microseconds)
  // with kb the k-blocks of one CTA, load the kilobytes of x' and W' it
  // streams, red the kilobytes it reads in the reduction (valid rows x BN
  // fp32 values) and r_S = 0.021 / 0.029 / 0.041 for S = 2 / 4 / 8 (the DSMEM
  // reads of a larger cluster are slower per byte). Its choices came within
  // 0.4% of the measured best plan summed over the shapes; choosing the most
  // CTAs instead was 5% slower, and up to 1.6x on single shapes. 32-wide
  // tiles, never the fastest measured, are used only when no wider tile fits.
  const ClusterTable* table = cluster_table();
  if (!table) return best;
  const int bns[4] = {256, 128, 64, 32};
  const int ss[3] = {8, 4, 2};
  // GW_SPLITK="BN,S" forces a tile width and cluster size where they fit;
  // GW_SPLITK=0 turns the kernel off (tuning and tests).
  static const int forced[2] = {[] {
    const char* v = std::getenv("GW_SPLITK");
    return v ? (v[0] == '0' ? -1 : std::atoi(v)) : 0;
  }(), [] {
    const char* v = std::getenv("GW_SPLITK");
    const char* c = v ? std::strchr(v, ',') : nullptr;
    return c ? std::atoi(c + 1) : 0;
  }()};
  if (forced[0] < 0) return best;
  const int64_t rows = std::min<int64_t>((M + 7) / 8 * 8, kSkBM);   // rows of one x' box
  const int64_t rows_valid = std::min<int64_t>(M, kSkBM);
  auto estimate = [&](int bn, int s) {
    const int64_t kb = (num_kb + s - 1) / s;
    const double load = static_cast<double>(kb) * static_cast<double>(rows + bn) * kSkBK * 2 / 1024.0;
    const double red = static_cast<double>(rows_valid) * bn * 4 / 1024.0;
    const double r = s == 2 ? 0.021 : s == 4 ? 0.029 : 0.041;
    return 0.19 * static_cast<double>(kb) + 0.004 * load + r * red + (bn < 64 ? 1e3 : 0.0);
  };
  bool found = false;
  double best_cost = 0.0;
  for (int bi = 0; bi < 4; ++bi) {
    const int bn = bns[bi];
    const int64_t tiles = m_tiles * ((N + bn - 1) / bn);
    for (int si = 0; si < 3; ++si) {
      const int s = ss[si];
      if (s > num_kb || tiles * s > sms || tiles > table->n[bi][si]) continue;
      if (bn == forced[0] && s == forced[1]) {
        best.bn = bn;
        best.split = s;
        best.tiles = tiles;
        return best;
      }
      const double cost = estimate(bn, s);
      if (!found || cost < best_cost) {
        found = true;
        best_cost = cost;
        best.bn = bn;
        best.split = s;
        best.tiles = tiles;
      }
    }
  }
  return best;
}

cudaError_t launch_gemm_splitk(const SplitKPlan& plan, const void* a, int dtype, int64_t M,
                               int64_t K, int64_t lda, const void* w, int64_t N, int64_t ldw,
                               const void* bias, int epilogue, void* y, int64_t ldy,
                               unsigned int* err, cudaStream_t stream, const int64_t* a_cols,
                               int64_t a_width) {
  if (plan.split < 2 || plan.split > 8 || plan.tiles <= 0 || plan.tiles > 65535)
    return cudaErrorInvalidValue;
  SkParams p{};
  p.M = M;
  p.N = N;
  p.bias = static_cast<const uint16_t*>(bias);
  p.epi = epilogue;
  p.y = static_cast<uint16_t*>(y);
  p.ldy = ldy;
  p.y_vec_ok = ((reinterpret_cast<uintptr_t>(y) & 7u) == 0 && (ldy % 4) == 0) ? 1 : 0;
  p.num_kb = static_cast<int>((K + kSkBK - 1) / kSkBK);
  p.m_tiles = static_cast<int>((M + kSkBM - 1) / kSkBM);
  p.split = plan.split;
  p.err = err;
  p.a_cols = a_cols;
  p.a_width = a_width;
  if (p.num_kb < plan.split) return cudaErrorInvalidValue;
  if (a_cols && (K % kSkBK) != 0) return cudaErrorInvalidValue;
  // With fewer than 128 rows the x' box covers only the rows that exist; the
  // MMA still reads 128 rows of shared memory, and the rows past the box hold
  // stale data that reaches only output rows that are never stored.
  const int a_rows = M >= kSkBM ? kSkBM : static_cast<int>((M + 7) / 8 * 8);
  p.a_tx_bytes = a_rows * kSkBK * 2;

  CUtensorMap ta, tb;
  if (!make_tmap_kmajor(&ta, a, M, a_cols ? a_width : K, lda, kSkBK, a_rows))
    return cudaErrorInvalidValue;
  if (!make_tmap_kmajor(&tb, w, N, K, ldw, kSkBK, plan.bn)) return cudaErrorInvalidValue;
  const bool bf = dtype == GW_DTYPE_BF16;
  switch (plan.bn) {
    case 256: return bf ? launch_sk<256, GW_DTYPE_BF16>(tb, ta, p, plan.tiles, stream)
                        : launch_sk<256, GW_DTYPE_F16>(tb, ta, p, plan.tiles, stream);
    case 128: return bf ? launch_sk<128, GW_DTYPE_BF16>(tb, ta, p, plan.tiles, stream)
                        : launch_sk<128, GW_DTYPE_F16>(tb, ta, p, plan.tiles, stream);
    case 64: return bf ? launch_sk<64, GW_DTYPE_BF16>(tb, ta, p, plan.tiles, stream)
                       : launch_sk<64, GW_DTYPE_F16>(tb, ta, p, plan.tiles, stream);
    case 32: return bf ? launch_sk<32, GW_DTYPE_BF16>(tb, ta, p, plan.tiles, stream)
                       : launch_sk<32, GW_DTYPE_F16>(tb, ta, p, plan.tiles, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace gw
