// K3, decode-shaped variant (at most 32 rows of x'): the operands swap roles
// so that the tensor core's 128-row side runs over output features.
//
//   y[m, n] = act( sum_j a[m, j] * w[n, j] + bias[n] )      a = x' (dense, compacted)
//
// With a handful of rows, a 128 x BN output tile wastes most of the MMA's M
// side and leaves the accumulator's valid rows in one TMEM lane quadrant, so
// one warp drains it. Here one MMA computes D[n, m] = W'[n, :] . a[m, :] for a
// 128-row block of W' (MMA M = 128) and every row of a, padded to MP = 16 or
// 32 (MMA N = MP): all four lane quadrants hold valid features and the
// accumulator is MP columns wide. (With 33..64 rows the larger receive
// buffer and exchange measured slower than the cluster split-K kernel.)
//
// A cluster of S CTAs (S = 2, 4, 8 or 16) shares one 128-feature block; CTA s
// accumulates k-blocks [s * nkb / S, (s + 1) * nkb / S) and owns feature slice
// s (128 / S features). The partial sums are pushed, not pulled: the drain
// warps write the accumulator into the idle operand ring, one row of MP floats
// per feature, and one thread per owner sends that owner's rows in a single
// bulk copy (the TMA engine, DSMEM) into slot s of its receive buffer, counted
// on the owner's mbarrier. The owner waits for that barrier alone, tells each
// sender that its copy has landed (a remote mbarrier arrive, so the sender's
// ring stays valid until then), sums the S slots in rank order (the result
// does not depend on timing), adds the bias, applies the activation, rounds
// once and stores y. The only cluster barrier publishes the initialised
// mbarriers: its arrive is in the prologue, its wait just before the first
// copy. W' is requested before waiting for the previous kernel of the stream
// (weights do not come from it): as many stages as the ring holds into shared
// memory, the rest of the CTA's range into L2, so with programmatic dependent
// launch the latency overlaps that kernel's tail. The
// shared-memory footprint allows two CTAs per SM.
//
// Roles (192 threads): warp 0 TMA producer, warp 1 TMEM allocator + MMA
// issuer, warps 2..5 TMEM drain and send (warp w reads lane quadrant w % 4);
// all six warps share the reduction. In gather mode (x and the alive list
// instead of a compacted x'), warps 2..5 first gather x[:, idx] into the
// stages' a tiles while TMA streams W': one launch per layer, no x' in memory. Every mbarrier wait is bounded
// (gw_common.cuh). No TMA multicast.
#include <cstdlib>
#include <mutex>

#include <cuda.h>

#include "gw_common.cuh"
#include "gw_internal.h"

namespace gw {

namespace {

constexpr int kDcN = 128;                       // W' rows (output features) per block = MMA M
constexpr int kDcK = 64;                        // k-block: one 128-byte swizzle atom
constexpr int kDcThreads = 192;
constexpr int kDcWBytes = kDcN * kDcK * 2;      // 16 KB of W' per stage
constexpr int kDecodeMaxRows = 32;

template <int MP>
struct DcCfg {
  static constexpr int kXBytes = MP * kDcK * 2;                 // 2 or 4 KB of a per stage
  static constexpr int kStageBytes = kDcWBytes + kXBytes;       // multiple of 1024
  static constexpr int kStages = MP == 16 ? 5 : 4;
  static constexpr int kRingBytes = kStages * kStageBytes;
  // Receive buffer: 128 rows (source rank s, feature f of this CTA's slice) of
  // MP partial sums, 16-byte aligned rows. The send staging area (row = feature
  // of the block) has the same shape and lives in the ring.
  static constexpr int kRecvStride = MP + 4;                    // floats per row
  static constexpr int kRecvBytes = kDcN * kRecvStride * 4;
  // Two accumulators of MP columns (even and odd k-blocks, issued by two
  // threads), a power of two >= 32.
  static constexpr int kTmemCols = 2 * MP < 32 ? 32 : 2 * MP;
  static constexpr int kSmemBytes = 1024 + kRingBytes + kRecvBytes + 256;
  // Two CTAs per SM (228 KB of shared memory, 1 KB reserved per CTA).
  static_assert(2 * (kSmemBytes + 1024) <= 233472, "two CTAs per SM");
  static_assert(kStageBytes % 1024 == 0, "stages keep 1024-byte alignment");
  static_assert((kRecvStride * 4) % 16 == 0, "16-byte receive rows");
  static_assert(kRecvBytes <= kRingBytes, "send staging fits in the ring");
};

struct DcParams {
  int64_t M;
  int64_t N;
  const uint16_t* bias;
  int epi;
  uint16_t* y;
  int64_t ldy;
  int y_vec_ok;              // 8-byte stores of four outputs allowed
  int num_kb;
  int split;                 // cluster size S
  int x_tx_bytes;            // bytes of one box of a (its rows: M rounded up to 8)
  unsigned int* err;
  const int64_t* a_cols;     // alive columns in 64-column runs: a is x, k-block kb at a_cols[64 kb]
  int64_t a_width;           // columns of x (with a_cols)
  // Gather mode (gx != null): a = x[:, gidx] is gathered into shared memory by
  // the drain warps (idle until the main loop ends) instead of loaded by TMA.
  const uint16_t* gx;
  int64_t ldx;
  int64_t x_cols;            // K of x: gathered indices outside [0, x_cols) read as zero
  const int64_t* gidx;
  int64_t n_alive;
};

// Gather mode: one warp fills the a tile (MP rows x 64 columns, 128-byte
// swizzled rows) of k-block kb. Lane l takes the alive columns 64 kb + 2 l and
// + 1 (indices loaded once) for every row, so a warp's loads of one row cover
// 64 consecutive alive columns (a few hundred bytes of x) and its 4-byte
// shared-memory stores one whole 128-byte row. Columns past n_alive are zero
// (W' is zero there, and 0 * garbage could be NaN); rows past M are left as
// they are (they reach only accumulator columns that are never stored).
template <int MP>
__device__ __forceinline__ void dc_gather_tile(const DcParams& p, uint32_t xs, int kb, int lane) {
  const int64_t c0 = static_cast<int64_t>(kb) * kDcK + 2 * lane;
  int64_t col[2];
  bool bad = false;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    col[j] = -1;
    if (c0 + j < p.n_alive) {
      const int64_t c = __ldg(p.gidx + c0 + j);
      if (c < 0 || c >= p.x_cols) bad = true;
      else col[j] = c;
    }
  }
  if (bad) raise_error(p.err, GW_DERR_BAD_INDEX);
  const int chunk = lane >> 2;                 // 16-byte chunk of the row
  const uint32_t within = static_cast<uint32_t>((lane & 3) * 4);
  uint32_t v[MP];
#pragma unroll
  for (int r = 0; r < MP; ++r) {
    v[r] = 0u;
    if (r < p.M) {
      const uint16_t* xr = p.gx + static_cast<int64_t>(r) * p.ldx;
      const uint32_t lo = col[0] >= 0 ? static_cast<uint32_t>(__ldg(xr + col[0])) : 0u;
      const uint32_t hi = col[1] >= 0 ? static_cast<uint32_t>(__ldg(xr + col[1])) : 0u;
      v[r] = lo | (hi << 16);
    }
  }
#pragma unroll
  for (int r = 0; r < MP; ++r) {
    if (r < p.M) {
      const uint32_t addr = xs + static_cast<uint32_t>(r * 128 + ((chunk ^ (r & 7)) << 4)) + within;
      asm volatile("st.shared.b32 [%0], %1;" :: "r"(addr), "r"(v[r]) : "memory");
    }
  }
}

// CTA `rank` owns features [rank * F, (rank + 1) * F) of the block, F = 128 / S.
// Once every slot of its receive buffer has landed it sums the S slots in rank
// order and writes the slice out. One task = one row m x four features; rows
// vary fastest across threads (conflict-free reads of the receive rows).
template <int MP, int DT>
__device__ __forceinline__ void dc_finish(const DcParams& p, const float* recv, int rank,
                                          int n_blk, int rows) {
  constexpr int kStride = DcCfg<MP>::kRecvStride;
  const int S = p.split;
  const int F = kDcN / S;
  const int tasks = rows * (F / 4);
  for (int t = threadIdx.x; t < tasks; t += kDcThreads) {
    const int m = t % rows;
    const int g = t / rows;
    float f[4] = {0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < S; ++s) {
      const float* r = recv + (s * F + 4 * g) * kStride + m;
#pragma unroll
      for (int j = 0; j < 4; ++j) f[j] += r[j * kStride];
    }
    const int64_t n0 = static_cast<int64_t>(n_blk) * kDcN + rank * F + 4 * g;
    if (n0 >= p.N) continue;
    if (p.bias) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (n0 + j < p.N) f[j] += Elem<DT>::to_f(__ldg(p.bias + n0 + j));
    }
    if (p.epi != GW_EPI_NONE) {
#pragma unroll
      for (int j = 0; j < 4; ++j) f[j] = apply_epilogue16(f[j], p.epi);
    }
    uint16_t* yp = p.y + static_cast<int64_t>(m) * p.ldy + n0;
    if (p.y_vec_ok && n0 + 4 <= p.N) {
      *reinterpret_cast<uint2*>(yp) = make_uint2(Elem<DT>::pack2(f[0], f[1]), Elem<DT>::pack2(f[2], f[3]));
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (n0 + j < p.N) yp[j] = Elem<DT>::from_f(f[j]);
    }
  }
}

// Issues the MMAs of k-blocks first, first + step, ... of this CTA's range
// (local indices; `used` counts ring slots in order) into accumulator d, with
// one commit per k-block to its stage's empty barrier, then one to tfull (or
// raises the abort flag) and one to drain_bar.
template <int MP, int DT, typename FullF, typename EmptyF>
__device__ __forceinline__ void dc_issue(const DcParams& p, uint32_t sbase, uint32_t d, int nk,
                                         int first, int step, FullF full, EmptyF empty,
                                         uint32_t tfull, uint32_t drain_bar,
                                         volatile int* abort_flag) {
  using C = DcCfg<MP>;
  constexpr uint32_t idesc = idesc_f16(DT == GW_DTYPE_BF16 ? 1u : 0u, kDcN, MP);
  bool ok = true;
  for (int used = first; used < nk; used += step) {
    const int s = used % C::kStages;
    const uint32_t ph = (used / C::kStages) & 1u;
    if (!mbar_wait(full(s), ph, abort_flag, p.err)) { ok = false; break; }
    tc_fence_after();
    const uint32_t w_s = sbase + s * C::kStageBytes;
    const uint64_t w_desc = smem_desc_kmajor_sw128(w_s);
    const uint64_t a_desc = smem_desc_kmajor_sw128(w_s + kDcWBytes);
#pragma unroll
    for (int k = 0; k < kDcK / 16; ++k)
      tc_mma_f16(d, w_desc + 2u * k, a_desc + 2u * k, idesc, (used > first || k > 0) ? 1u : 0u);
    tc_commit(empty(s));
  }
  if (ok) tc_commit(tfull);
  else *abort_flag = 1;            // the drain warps stop waiting for tfull
  tc_commit(drain_bar);
}

template <int MP, int DT>
__global__ void __launch_bounds__(kDcThreads, 2)
gemm_decode_kernel(const __grid_constant__ CUtensorMap tmap_w,
                   const __grid_constant__ CUtensorMap tmap_a, const DcParams p) {
  using C = DcCfg<MP>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_s & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  float* recv = reinterpret_cast<float*>(smem + C::kRingBytes);
  const uint32_t recv_s = sbase + C::kRingBytes;
  uint8_t* bar_region = smem + C::kRingBytes + C::kRecvBytes;
  const uint32_t bar0 = smem_u32(bar_region);
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (C::kStages + s); };
  const uint32_t tfull = bar0 + 8u * (2 * C::kStages);
  const uint32_t drain_bar = tfull + 8u;
  const uint32_t recv_bar = tfull + 16u;   // all S slots of this CTA's slice have landed
  const uint32_t sent_bar = tfull + 24u;   // every owner has received this CTA's copy
  static_assert(8 * (2 * C::kStages + 4) <= 192, "barrier region overflows into the TMEM slot");
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_region + 192);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bar_region + 196);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = static_cast<int>(cluster_ctarank());   // == blockIdx.x, the k split
  const int n_blk = static_cast<int>(blockIdx.y);
  const int kb0 = static_cast<int>(static_cast<int64_t>(rank) * p.num_kb / p.split);
  const int kb1 = static_cast<int>(static_cast<int64_t>(rank + 1) * p.num_kb / p.split);
  const int rows = static_cast<int>(p.M);                 // <= MP
  const int S = p.split;
  const int F = kDcN / S;                                 // features per slice
  const uint32_t slice_bytes = static_cast<uint32_t>(F * C::kRecvStride * 4);
  // One thread issuing waits about 200 cycles per stage and 70-80 per MMA,
  // more than the tensor core needs for a 128 x MP x 64 k-block, so the main
  // loop is issue-bound. With two k-blocks or more (and no gather, whose warps
  // are busy), warp 1 issues the even k-blocks into accumulator 0 and the
  // first drain warp the odd ones into accumulator 1; the drain adds the two.
  const bool dual = !p.gx && kb1 - kb0 >= 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(full(s), p.gx ? 2 : 1);    // gather mode: the producer's and the gathering warp's arrivals
      mbar_init(empty(s), 1);
    }
    mbar_init(tfull, dual ? 2 : 1);       // one commit per issuing thread
    mbar_init(drain_bar, dual ? 2 : 1);
    mbar_init(recv_bar, 1);
    mbar_init(sent_bar, static_cast<uint32_t>(S));
    // Every CTA of the cluster (this one included) sends one slice here.
    mbar_arrive_expect_tx(recv_bar, static_cast<uint32_t>(S) * slice_bytes);
    *abort_flag = 0;
    mbar_init_fence();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_a);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  cluster_arrive();                    // this CTA's mbarriers are initialised
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  uint32_t acc[MP];                    // drain warps: this thread's feature, MP rows
#pragma unroll
  for (int c = 0; c < MP; ++c) acc[c] = 0u;   // zeros are sent if the accumulator never arrives

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const int nk = kb1 - kb0;
      // W' is complete before the previous kernel of the stream starts (the
      // library's weight packs let the next kernel start only when they have
      // finished), so it is requested before waiting for that kernel; a and
      // the run starts may come from it. As many stages as the ring holds are
      // loaded into shared memory now, the rest of this CTA's range into L2.
      const int pre = nk < C::kStages ? nk : C::kStages;
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(full(i), kDcWBytes + p.x_tx_bytes);
        tma_load_2d(sbase + i * C::kStageBytes, &tmap_w, (kb0 + i) * kDcK, n_blk * kDcN, full(i));
      }
      for (int kb = kb0 + pre; kb < kb1; ++kb) tma_prefetch_l2_2d(&tmap_w, kb * kDcK, n_blk * kDcN);
      asm volatile("griddepcontrol.wait;" ::: "memory");
      int issued = 0;
      bool ok = true;
      int64_t nxt = p.a_cols ? run_start_load(p.a_cols, kb0) : 0;   // next k-block's run start
      for (int kb = kb0; kb < kb1; ++kb, ++issued) {
        const int s = issued % C::kStages;
        const uint32_t ph = (issued / C::kStages) & 1u;
        const int64_t cur = nxt;
        if (p.a_cols && kb + 1 < kb1) nxt = run_start_load(p.a_cols, kb + 1);
        const uint32_t w_s = sbase + s * C::kStageBytes;
        if (issued >= pre) {
          if (!mbar_wait(empty(s), ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
          mbar_arrive_expect_tx(full(s), kDcWBytes + p.x_tx_bytes);
          tma_load_2d(w_s, &tmap_w, kb * kDcK, n_blk * kDcN, full(s));
        }
        if (!p.gx) {
          const int ax = p.a_cols ? run_start_check(cur, p.a_width, p.err) : kb * kDcK;
          tma_load_2d(w_s + kDcWBytes, &tmap_a, ax, 0, full(s));
        }
      }
      if (!ok) {
        // Loads still in flight complete before the CTA exits.
        const int first = issued > C::kStages ? issued - C::kStages : 0;
        for (int i = first; i < issued; ++i)
          mbar_wait(full(i % C::kStages), (i / C::kStages) & 1u, nullptr, p.err, 100000000ull);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even k-blocks)
    if (lane == 0) {
      dc_issue<MP, DT>(p, sbase, tmem_base, kb1 - kb0, 0, dual ? 2 : 1, full, empty, tfull,
                       drain_bar, abort_flag);
      // Every MMA (of both issuers) has finished writing TMEM before TMEM is freed.
      mbar_wait(drain_bar, 0u, nullptr, p.err, 100000000ull);
    }
    __syncwarp();
  } else {
    if (dual && warp == 2) {
      // ---------------------------------------------------------- MMA issuer (odd k-blocks)
      if (lane == 0)
        dc_issue<MP, DT>(p, sbase, tmem_base + MP, kb1 - kb0, 1, 2, full, empty, tfull, drain_bar,
                         abort_flag);
      __syncwarp();
    }
    if (p.gx) {
      // ---------------------------------------------------------- gather a
      // Warp w fills the a tiles of stages w - 2, w + 2, ... (x and the alive
      // list may come from the previous kernel of the stream).
      asm volatile("griddepcontrol.wait;" ::: "memory");
      const int nk = kb1 - kb0;
      for (int i = warp - 2; i < nk; i += 4) {
        const int s = i % C::kStages;
        const uint32_t ph = (i / C::kStages) & 1u;
        int ok = 1;
        if (lane == 0) ok = mbar_wait(empty(s), ph ^ 1u, abort_flag, p.err) ? 1 : 0;
        if (!__shfl_sync(0xFFFFFFFFu, ok, 0)) break;
        dc_gather_tile<MP>(p, sbase + s * C::kStageBytes + kDcWBytes, kb0 + i, lane);
        fence_proxy_async_smem();        // the tile is read by the tensor core
        __syncwarp();
        if (lane == 0) mbar_arrive(full(s));
      }
    }
    // ------------------------------------------------------------ TMEM drain
    // Warp w reads TMEM lanes 32 (w % 4) .. +31 = output features of the block;
    // column m of the accumulator is row m of y.
    if (mbar_wait(tfull, 0u, abort_flag, p.err)) {
      tc_fence_after();
      const uint32_t t_lane = tmem_base + (static_cast<uint32_t>((warp & 3) * 32) << 16);
#pragma unroll
      for (int c = 0; c < MP; c += 16) tc_ld_32x32b_x16(t_lane + c, acc + c);
      if (dual) {
        uint32_t odd[MP];
#pragma unroll
        for (int c = 0; c < MP; c += 16) tc_ld_32x32b_x16(t_lane + MP + c, odd + c);
        tc_wait_ld();
#pragma unroll
        for (int c = 0; c < MP; ++c)
          acc[c] = __float_as_uint(__uint_as_float(acc[c]) + __uint_as_float(odd[c]));
      } else {
        tc_wait_ld();
      }
    }
    tc_fence_before();
  }

  // The producer has drained its loads and the MMA thread the tensor pipe (on
  // every path), and the drain's TMEM reads are complete: the ring is idle.
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
  if (warp >= 2) {
    // ------------------------------------------------------------ send
    // Row `feat` of the staging area = this CTA's partial sums of that feature.
    const int feat = (warp & 3) * 32 + lane;
    float4* row = reinterpret_cast<float4*>(smem + feat * C::kRecvStride * 4);
#pragma unroll
    for (int m = 0; m < MP; m += 4)
      row[m / 4] = make_float4(__uint_as_float(acc[m]), __uint_as_float(acc[m + 1]),
                               __uint_as_float(acc[m + 2]), __uint_as_float(acc[m + 3]));
    fence_proxy_async_smem();          // the rows are read by the bulk copies
    named_bar_sync(1, 128);            // the four drain warps
  }
  cluster_wait();                      // every owner's mbarriers are initialised
  if (warp >= 2) {
    const int owner = threadIdx.x - 64;
    if (owner < S)
      bulk_copy_to_cta(mapa_shared(recv_s + static_cast<uint32_t>(rank) * slice_bytes, owner),
                       sbase + static_cast<uint32_t>(owner) * slice_bytes, slice_bytes,
                       mapa_shared(recv_bar, owner));
  }

  // Every slot of this CTA's slice has landed: its own and the S - 1 peers'.
  const bool got = mbar_wait_cluster(recv_bar, 0u, nullptr, p.err);
  // Tell every sender that its copy into this CTA has landed.
  if (threadIdx.x < S) mbar_arrive_cluster(mapa_shared(sent_bar, threadIdx.x));
  if (got) dc_finish<MP, DT>(p, recv, rank, n_blk, rows);
  // This CTA's ring is the source of its copies: it stays valid, and the CTA
  // alive, until every owner has received its slice.
  mbar_wait_cluster(sent_bar, 0u, nullptr, p.err);
}

template <int MP, int DT>
cudaError_t set_decode_attrs() {
  auto kern = gemm_decode_kernel<MP, DT>;
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kern), DcCfg<MP>::kSmemBytes);
  if (e != cudaSuccess) return e;
  // Clusters of 16 CTAs are a non-portable size; the occupancy query in
  // decode_table() decides whether the device runs them.
  static std::once_flag once[64];
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if (dev >= 0 && dev < 64)
    std::call_once(once[dev], [&] {
      if (cudaFuncSetAttribute(reinterpret_cast<const void*>(kern),
                               cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
        (void)cudaGetLastError();
    });
  return cudaSuccess;
}

template <int MP, int DT>
cudaError_t launch_dc(const CUtensorMap& tw, const CUtensorMap& ta, const DcParams& p,
                      int64_t blocks, cudaStream_t stream) {
  auto kern = gemm_decode_kernel<MP, DT>;
  cudaError_t e = set_decode_attrs<MP, DT>();
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.split), static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(kDcThreads);
  cfg.dynamicSmemBytes = DcCfg<MP>::kSmemBytes;
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
  return cudaLaunchKernelEx(&cfg, kern, tw, ta, p);
}

// Clusters of S CTAs of the MP-wide kernel that fit on the device at once, for
// MP in {16, 32} x S in {16, 8, 4, 2} (occupancy queries, once per device).
struct DecodeTable {
  int n[2][4];
};

template <int MP>
int query_decode_clusters(int s) {
  auto kern = gemm_decode_kernel<MP, GW_DTYPE_F16>;
  if (set_decode_attrs<MP, GW_DTYPE_F16>() != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(s), 1);
  cfg.blockDim = dim3(kDcThreads);
  cfg.dynamicSmemBytes = DcCfg<MP>::kSmemBytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(s);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    n = 0;
  }
  return n > 0 ? n : 0;
}

const DecodeTable* decode_table() {
  static std::mutex mu;
  static DecodeTable tables[64];
  static bool ready[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    (void)cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!ready[dev]) {
    const int ss[4] = {16, 8, 4, 2};
    for (int si = 0; si < 4; ++si) {
      tables[dev].n[0][si] = query_decode_clusters<16>(ss[si]);
      tables[dev].n[1][si] = query_decode_clusters<32>(ss[si]);
    }
    ready[dev] = true;
  }
  return &tables[dev];
}

}  // namespace

DecodePlan plan_decode(int64_t M, int64_t N, int64_t K, int sm_count) {
  DecodePlan best;
  if (M <= 0 || M > kDecodeMaxRows || N <= 0 || K <= 0) return best;
  const int mi = M <= 16 ? 0 : 1;
  const int64_t sms = sm_count > 0 ? sm_count : 148;
  const int64_t blocks = (N + kDcN - 1) / kDcN;
  const int64_t num_kb = (K + kDcK - 1) / kDcK;
  if (blocks > 65535) return best;
  const DecodeTable* table = decode_table();
  if (!table) return best;
  static const int forced = [] {
    const char* v = std::getenv("GW_DECODE_SPLIT");
    return v ? std::atoi(v) : 0;
  }();
  // Most CTAs within one wave of clusters (two CTAs per SM), keeping at least
  // two k-blocks per CTA; ties keep the smaller cluster (less reduction).
  const int ss[4] = {16, 8, 4, 2};
  int64_t best_ctas = 0;
  for (int si = 3; si >= 0; --si) {
    const int s = ss[si];
    if (forced && s != forced) continue;
    if (num_kb < 2 * s && !(s == 2 && num_kb >= 2)) continue;
    if (blocks * s > 2 * sms || blocks > table->n[mi][si]) continue;
    if (blocks * s > best_ctas) {
      best_ctas = blocks * s;
      best.split = s;
    }
  }
  if (best.split >= 2) {
    best.mp = mi == 0 ? 16 : 32;
    best.blocks = blocks;
  } else {
    best.split = 1;
  }
  return best;
}

namespace {
cudaError_t launch_decode_params(const DecodePlan& plan, DcParams& p, int dtype, const void* a,
                                 int64_t lda, const void* w, int64_t ldw, int64_t K,
                                 cudaStream_t stream) {
  // The box of a covers only the rows that exist (rounded up to 8); the MMA
  // reads MP rows of shared memory, and the rows past the box hold stale data
  // that reaches only accumulator columns m >= M, which are never stored.
  const int a_rows = static_cast<int>((p.M + 7) / 8 * 8);
  p.x_tx_bytes = p.gx ? 0 : a_rows * kDcK * 2;
  CUtensorMap ta, tw;
  if (!make_tmap_kmajor(&tw, w, p.N, K, ldw, kDcK, kDcN)) return cudaErrorInvalidValue;
  if (p.gx) {
    ta = tw;                          // unused: a is gathered in the kernel
  } else if (!make_tmap_kmajor(&ta, a, p.M, p.a_cols ? p.a_width : K, lda, kDcK, a_rows)) {
    return cudaErrorInvalidValue;
  }
  const bool bf = dtype == GW_DTYPE_BF16;
  switch (plan.mp) {
    case 16: return bf ? launch_dc<16, GW_DTYPE_BF16>(tw, ta, p, plan.blocks, stream)
                       : launch_dc<16, GW_DTYPE_F16>(tw, ta, p, plan.blocks, stream);
    case 32: return bf ? launch_dc<32, GW_DTYPE_BF16>(tw, ta, p, plan.blocks, stream)
                       : launch_dc<32, GW_DTYPE_F16>(tw, ta, p, plan.blocks, stream);
    default: return cudaErrorInvalidValue;
  }
}

DcParams decode_params(const DecodePlan& plan, int64_t M, int64_t K, int64_t N, const void* bias,
                       int epilogue, void* y, int64_t ldy, unsigned int* err) {
  DcParams p{};
  p.M = M;
  p.N = N;
  p.bias = static_cast<const uint16_t*>(bias);
  p.epi = epilogue;
  p.y = static_cast<uint16_t*>(y);
  p.ldy = ldy;
  p.y_vec_ok = ((reinterpret_cast<uintptr_t>(y) & 7u) == 0 && (ldy % 4) == 0) ? 1 : 0;
  p.num_kb = static_cast<int>((K + kDcK - 1) / kDcK);
  p.split = plan.split;
  p.err = err;
  return p;
}
}  // namespace

cudaError_t launch_gemm_decode_gather(const DecodePlan& plan, const void* x, int dtype, int64_t M,
                                      int64_t K, int64_t ldx, const int64_t* idx, int64_t n_alive,
                                      const void* w, int64_t N, int64_t ldw, const void* bias,
                                      int epilogue, void* y, int64_t ldy, unsigned int* err,
                                      cudaStream_t stream) {
  if (plan.split < 2 || plan.split > 16 || plan.blocks <= 0 || plan.blocks > 65535 ||
      M <= 0 || M > plan.mp || n_alive <= 0)
    return cudaErrorInvalidValue;
  DcParams p = decode_params(plan, M, n_alive, N, bias, epilogue, y, ldy, err);
  if (p.num_kb < plan.split) return cudaErrorInvalidValue;
  p.gx = static_cast<const uint16_t*>(x);
  p.ldx = ldx;
  p.x_cols = K;
  p.gidx = idx;
  p.n_alive = n_alive;
  return launch_decode_params(plan, p, dtype, nullptr, 0, w, ldw, n_alive, stream);
}

cudaError_t launch_gemm_decode(const DecodePlan& plan, const void* a, int dtype, int64_t M,
                               int64_t K, int64_t lda, const void* w, int64_t N, int64_t ldw,
                               const void* bias, int epilogue, void* y, int64_t ldy,
                               unsigned int* err, cudaStream_t stream, const int64_t* a_cols,
                               int64_t a_width) {
  if (plan.split < 2 || plan.split > 16 || plan.blocks <= 0 || plan.blocks > 65535 ||
      M <= 0 || M > plan.mp)
    return cudaErrorInvalidValue;
  DcParams p = decode_params(plan, M, K, N, bias, epilogue, y, ldy, err);
  if (p.num_kb < plan.split) return cudaErrorInvalidValue;
  if (a_cols && (K % kDcK) != 0) return cudaErrorInvalidValue;
  p.a_cols = a_cols;
  p.a_width = a_width;
  return launch_decode_params(plan, p, dtype, a, lda, w, ldw, K, stream);
}

}  // namespace gw
