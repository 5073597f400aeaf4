// K3, CTA-pair variant: y[256-row pair tile, 256 cols] on tcgen05 with cta_group::2.
//
// Same product as gemm_tc_kernel's TMA mode (dense A = the gathered x', packed
// W'), but two CTAs of a cluster share one 256 x 256 accumulator tile:
//   * each CTA TMA-loads its own 128 rows of A and its own 128 rows of B
//     (half of the tile's 256 output features) for every 64-wide k-block, so
//     per SM only 32 KB cross L2 per k-block instead of 48 KB for 128 x 256;
//     the loads of both CTAs complete on the leader CTA's barrier;
//   * the leader's MMA thread issues tcgen05.mma.cta_group::2 (M = 256,
//     N = 256, K = 16) reading both CTAs' shared memory and writing both
//     CTAs' TMEM (128 lanes x 256 fp32 columns each, double-buffered);
//   * MMA completion is multicast to both CTAs (tcgen05.commit ... multicast)
//     to free their stages and publish finished accumulators;
//   * each CTA's four epilogue warps drain its own TMEM (bias, GELU, one
//     rounding) into swizzled staging tiles that the TMA unit stores to y,
//     and arrive on the leader's accumulator-empty barrier (remote arrive for
//     the second CTA) as soon as their TMEM reads are done;
//   * launch_dependents right after the prologue lets the next kernel of the
//     stream (the next layer's gather, another GEMM) be scheduled onto SMs as
//     they drain in the last wave; it waits for this grid's completion itself.
// No TMA multicast: each CTA loads only its own halves.
// Every wait is bounded (gw_common.cuh); the kernel never hangs on a lost
// arrival, it records GW_DEVICE_ERR_WAIT_TIMEOUT and unwinds.
//
// In-kernel gather (GATHER = true, gw_gather_gemm's overlap strategy): A is
// x' = x[:, idx] in the workspace, and the kernel builds it itself while the
// MMAs run. x' is cut into units of 128 rows (half a pair tile) x 64 alive
// columns (one k atom). Before their first epilogue, the eight epilogue warps
// of every CTA claim units (two at a time) from a counter in the workspace
// header, gather them with 2-byte loads (lane l: alive columns 2l and 2l+1,
// one 4-byte store per row) and publish each finished unit through its flag.
// The TMA producer waits for a unit's flag before loading it. Units are
// claimed in the order the tiles consume them (groups of as many row blocks
// as one wave of tiles covers, k atom by k atom inside a group) and tiles are
// walked row block by row block, so the first wave of MMAs waits only for the
// first units. Units are claimed, not assigned, so no CTA ever waits for a
// unit that only a CTA which is not resident could produce.
// Flags and counters carry the call's number: the header's 64-bit epoch E is
// read by every CTA after griddepcontrol.wait (so the previous call on the
// stream has finished), the call works with E + 1 (a flag is ready when it
// equals E + 1; the counters hold E + 1 in their upper 40 bits and reset
// themselves when they see an older number), and the last CTA to finish
// stores E + 1 as the new epoch. Nothing needs clearing between calls, the
// workspace's contents on entry do not matter, and every replay of a CUDA
// graph gets a fresh number.
#include <algorithm>
#include <cstdlib>

#include <cuda.h>

#include "gw_common.cuh"
#include "gw_internal.h"

namespace gw {

namespace {

constexpr int kHalfM = 128;            // rows per CTA
constexpr int kPairM = 2 * kHalfM;
constexpr int kBK2 = 64;
constexpr int kThreads2 = 320;         // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue
constexpr int kEpiWarps2 = 8;          // two per TMEM lane quadrant
// A stage holds two 64-wide k atoms (128 of K) of A and of B: the single MMA
// thread waits once and issues 8 MMAs per stage, so its per-stage overhead
// (barrier wait, fence, commit) is paid once per 1024 tensor cycles.
constexpr int kAtoms2 = 2;
constexpr int kStages2 = 3;
constexpr int kAAtomBytes2 = kHalfM * kBK2 * 2;      // one 128-row x 64-col atom of A (16 KB)
constexpr int kABytes2 = kAtoms2 * kAAtomBytes2;
constexpr int kTmemCols2 = 512;         // two accumulators of up to 256 columns
// Epilogue staging for TMA stores: per epilogue warp one 32-row x 64-column
// 16-bit tile (4 KB, 128-byte swizzled rows).
constexpr int kEpiCols = 64;
constexpr int kEpiTileBytes = 32 * kEpiCols * 2;
constexpr int kEpiBytes = kEpiWarps2 * kEpiTileBytes;

// Pair tile width BN (256 or 192): each CTA holds BN / 2 rows of W' per atom;
// the two epilogue warps of a lane quadrant take columns [0, 128) and
// [128, BN) of the tile.
template <int BN>
struct Tc2Cfg {
  static_assert(BN == 256 || BN == 192, "pair tile width");
  static constexpr int kHalfN = BN / 2;
  static constexpr int kBAtomBytes = kHalfN * kBK2 * 2;         // 16 or 12 KB
  static constexpr int kBBytes = kAtoms2 * kBAtomBytes;
  static constexpr int kStageBytes = kABytes2 + kBBytes;
  static constexpr int kSmemBytes = 1024 + kStages2 * kStageBytes + kEpiBytes + 256;
  static_assert(kBAtomBytes % 1024 == 0, "swizzle atoms stay 1024-byte aligned");
  static_assert(kSmemBytes <= 232448, "shared memory budget per CTA");
  static constexpr int kCols0 = 128;                            // first warp of a quadrant
  static constexpr int kCols1 = BN - 128;                       // second warp
};

struct Tc2Params {
  int64_t M;
  int64_t N;
  const uint16_t* bias;
  int epi;
  int y_vec_ok;
  int y_tma;                 // y stored through tmap_y (16-byte aligned rows)
  uint16_t* y;
  int64_t ldy;
  int num_kb;               // 64-wide k atoms of K
  int num_ks;               // stages of kStageK2 per tile
  int m_tiles;
  int n_tiles;
  int num_tiles;
  // Jobs: tiles [0, num_full) whole, then each tile of [num_full, num_tiles)
  // as two jobs of 128 columns (the last, partial round of tiles split in
  // half so that it spreads over the pairs); num_jobs counts both kinds.
  int num_full;
  int num_jobs;
  unsigned int* err;
  // Peer outputs: every finished tile is also stored, at the same place, into
  // these buffers of other GPUs (same ldy; device addresses valid here).
  int n_peers;
  uint16_t* peers[kMaxPeers];
  // Alive columns in 64-column runs: A is x itself and k atom kb starts at
  // column a_cols[64 kb] (null: A is the compacted x', atom kb at 64 kb).
  const int64_t* a_cols;
  int64_t a_width;          // columns of x (with a_cols)
  // K' on the device (num_kb is then an upper bound; see device_num_kb).
  const int32_t* k_dev;
  // In-kernel gather (GATHER): A = x' [M, n_alive] (leading dimension ldp) is
  // built from x [M, gK] (leading dimension ldgx) through the alive list.
  const uint16_t* gx;
  int64_t ldgx;
  int64_t gK;
  const int64_t* gidx;
  int64_t n_alive;
  uint16_t* xg;
  int64_t ldp;
  // Workspace header, 64-bit words: [0] epoch, [1] unit claim counter, [2]
  // finished-CTA counter, [3] unused, then one flag per unit (half-panel hp,
  // k atom kb) at 4 + hp * num_kb + kb.
  unsigned long long* ghdr;
  int g_hp;                 // half-panels (128-row blocks) per claim group
  int h_total;              // half-panels: 2 * m_tiles
  int m_major;              // tiles walked row block by row block (gather order)
};

// Tile t -> (row block, column block): column blocks fastest when m_major
// (the in-kernel gather's order), row blocks fastest otherwise.
__device__ __forceinline__ void tile_coords(int tile, const Tc2Params& p, int& m_blk, int& n_blk) {
  if (p.m_major) {
    m_blk = tile / p.n_tiles;
    n_blk = tile - m_blk * p.n_tiles;
  } else {
    n_blk = tile / p.m_tiles;
    m_blk = tile - n_blk * p.m_tiles;
  }
}

// Job -> (row block, column block, sub): sub = -1 for a whole tile, else
// which 128-column half of the tile the job covers.
__device__ __forceinline__ void job_coords(int job, const Tc2Params& p, int& m_blk, int& n_blk,
                                           int& sub) {
  if (job < p.num_full) {
    tile_coords(job, p, m_blk, n_blk);
    sub = -1;
  } else {
    const int j = job - p.num_full;
    tile_coords(p.num_full + (j >> 1), p, m_blk, n_blk);
    sub = j & 1;
  }
}

__device__ __forceinline__ void st_release_gpu_u64(unsigned long long* p, uint64_t v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" :: "l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_gpu_u64(const unsigned long long* p) {
  uint64_t v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Counters tagged with the call's number: (number << 24) | count. Adds n and
// returns the count before the add; a counter holding another number (an
// earlier call's, or whatever the workspace held) counts as 0. The common case
// is one atomicAdd; only the first claims of a call, which find the old
// number, install the new one with compare-and-swap.
constexpr int kCountBits = 24;
__device__ __forceinline__ uint32_t tagged_add(unsigned long long* ctr, uint64_t call, uint32_t n) {
  constexpr uint64_t kCountMask = (uint64_t{1} << kCountBits) - 1;
  const uint64_t tag = call & ((uint64_t{1} << (64 - kCountBits)) - 1);
  uint64_t old = atomicAdd(ctr, static_cast<unsigned long long>(n));
  if ((old >> kCountBits) == tag) return static_cast<uint32_t>(old & kCountMask);
  uint64_t cur = old + n;                      // the counter as our add left it
  for (;;) {
    const uint64_t prev = atomicCAS(ctr, cur, (tag << kCountBits) | n);
    if (prev == cur) return 0u;                // installed: we own [0, n)
    if ((prev >> kCountBits) == tag) {         // someone else installed it: count on it
      old = atomicAdd(ctr, static_cast<unsigned long long>(n));
      if ((old >> kCountBits) == tag) return static_cast<uint32_t>(old & kCountMask);
      cur = old + n;
    } else {
      cur = prev;                              // still an old number: try again on it
    }
  }
}

__device__ __forceinline__ uint64_t ld_relaxed_gpu_u64(const unsigned long long* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_gpu() {
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
}
__device__ __forceinline__ void st_relaxed_gpu_u64(unsigned long long* p, uint64_t v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" :: "l"(p), "l"(v) : "memory");
}

// Which of the flags f[0, n) (n <= 16) already equal `value`: 16 independent
// relaxed loads (one round trip for all), then one acquire fence if any was
// set, which makes the data published before those flags visible.
__device__ __forceinline__ uint32_t flags_ready(const unsigned long long* f, int n, uint64_t value) {
  uint64_t v[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = i < n ? ld_relaxed_gpu_u64(f + i) : 0;
  uint32_t bits = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) bits |= (i < n && v[i] == value) ? (1u << i) : 0u;
  if (bits) fence_acq_rel_gpu();
  return bits;
}

// Bounded wait until *flag == value (acquire); same contract as wait_counter_geq.
__device__ __forceinline__ bool wait_flag_eq(const unsigned long long* flag, uint64_t value,
                                             volatile int* abort_flag, unsigned int* err) {
  if (ld_acquire_gpu_u64(flag) == value) return true;
  const unsigned long long t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (ld_acquire_gpu_u64(flag) == value) return true;
    if ((i & 63u) == 0u) {
      if (abort_flag && *abort_flag) return false;
      if (global_timer_ns() - t0 > GW_WAIT_LIMIT_NS) {
        if (abort_flag) *abort_flag = 1;
        raise_error(err, GW_DERR_WAIT_TIMEOUT);
        return false;
      }
    }
  }
}

// Unit u of the claim order -> (half-panel, k atom). Groups of g_hp
// half-panels (the last one may be smaller), k atom by k atom inside a group.
__device__ __forceinline__ void unit_coords(int u, const Tc2Params& p, int& hp, int& kb) {
  const int g_units = p.g_hp * p.num_kb;
  const int g = u / g_units;
  const int r = u - g * g_units;
  const int hp0 = g * p.g_hp;
  const int gsz = min(p.g_hp, p.h_total - hp0);
  kb = r / gsz;
  hp = hp0 + (r - kb * gsz);
}

// The epilogue warps' gather of x' (see the file comment). e: 0..7, the
// warp's 16 rows of a unit; call: this call's number (epoch + 1). Returns
// when every unit has been claimed.
template <int DT>
__device__ __forceinline__ void gather_units(const Tc2Params& p, int e, int lane,
                                             volatile int* slot, uint64_t call) {
  // Software-pipelined over batches of two units: the claim of the next batch
  // is issued before this batch's loads, and the next batch's alive indices
  // are loaded while this batch is published, so one iteration costs about
  // one round trip to memory instead of four in series.
  const int units = p.h_total * p.num_kb;
  const bool leader = e == 0 && lane == 0;
  bool bad = false;
  int64_t c[2][2];                       // [unit of the batch][column 2 lane + i]
  auto load_idx = [&](int u0) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int u = u0 + h;
      c[h][0] = c[h][1] = -1;
      if (u < units) {
        int hp, kb;
        unit_coords(u, p, hp, kb);
        const int64_t j0 = static_cast<int64_t>(kb) * kBK2 + 2 * lane;
        if (j0 < p.n_alive) c[h][0] = __ldg(p.gidx + j0);
        if (j0 + 1 < p.n_alive) c[h][1] = __ldg(p.gidx + j0 + 1);
      }
    }
  };
  if (leader) slot[0] = static_cast<int>(tagged_add(p.ghdr + 1, call, 2u));
  named_bar_sync(1, kEpiWarps2 * 32);
  int u0 = slot[0];
  load_idx(u0);
  for (int it = 0; u0 < units; ++it) {
    // Next batch's claim, into the other slot (read after the barrier below).
    if (leader) slot[(it + 1) & 1] = static_cast<int>(tagged_add(p.ghdr + 1, call, 2u));
    uint32_t v[2][16];
    int64_t row0[2];
    int rows_here[2], kbu[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int u = u0 + h;
      int hp = 0, kb = 0;
      if (u < units) unit_coords(u, p, hp, kb);
      kbu[h] = kb;
      row0[h] = static_cast<int64_t>(hp) * kHalfM + e * 16;
      const int64_t rem = p.M - row0[h];
      rows_here[h] = (u >= units || rem <= 0) ? 0 : (rem >= 16 ? 16 : static_cast<int>(rem));
      int64_t c0 = c[h][0], c1 = c[h][1];
      if (c0 >= p.gK || c0 < -1 || c1 >= p.gK || c1 < -1) bad = true;
      if (c0 >= p.gK || c0 < 0) c0 = -1;
      if (c1 >= p.gK || c1 < 0) c1 = -1;
      // Branch-free loads, so that all of the batch's loads are in flight at
      // once: rows past M re-read the last valid row and dead or bad columns
      // read column 0; both are masked to zero.
      const int rlast = max(rows_here[h] - 1, 0);
      const int64_t rbase = rows_here[h] > 0 ? row0[h] * p.ldgx : 0;
      const uint16_t* b0 = p.gx + rbase + (c0 >= 0 ? c0 : 0);
      const uint16_t* b1 = p.gx + rbase + (c1 >= 0 ? c1 : 0);
      const uint32_t m0 = c0 >= 0 ? 0xFFFFu : 0u;
      const uint32_t m1 = c1 >= 0 ? 0xFFFF0000u : 0u;
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        const int64_t off = static_cast<int64_t>(min(r, rlast)) * p.ldgx;
        const uint32_t lo = __ldg(b0 + off);
        const uint32_t hi = __ldg(b1 + off);
        v[h][r] = (lo & m0) | ((hi << 16) & m1);
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (rows_here[h] > 0) {
        uint32_t* dst = reinterpret_cast<uint32_t*>(p.xg + row0[h] * p.ldp +
                                                    static_cast<int64_t>(kbu[h]) * kBK2) + lane;
        const int64_t step = p.ldp / 2;
#pragma unroll
        for (int r = 0; r < 16; ++r)
          if (r < rows_here[h]) dst[r * step] = v[h][r];
      }
    }
    fence_proxy_async_global();        // x' stores -> visible to the TMA (async proxy) loads
    named_bar_sync(1, kEpiWarps2 * 32);  // this batch stored; the next claim is in its slot
    const int u_next = slot[(it + 1) & 1];
    load_idx(u_next);                  // in flight while the batch is published
    if (leader) {
      // One release fence for the batch (it covers every warp's stores, which
      // the barrier ordered before it), then both flags as relaxed stores.
      fence_acq_rel_gpu();
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int u = u0 + h;
        if (u < units) {
          int hp, kb;
          unit_coords(u, p, hp, kb);
          st_relaxed_gpu_u64(p.ghdr + 4 + static_cast<int64_t>(hp) * p.num_kb + kb, call);
        }
      }
    }
    u0 = u_next;
  }
  if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) raise_error(p.err, GW_DERR_BAD_INDEX);
}

template <int BN, int DT, int EPI, bool GATHER>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads2, 1)
gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmap_b,
                const __grid_constant__ CUtensorMap tmap_bh,
                const __grid_constant__ CUtensorMap tmap_a,
                const __grid_constant__ CUtensorMap tmap_y, const Tc2Params p) {
  using C = Tc2Cfg<BN>;
  constexpr int kHalfN = C::kHalfN;
  constexpr int kStageBytes2 = C::kStageBytes;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_s & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  uint8_t* epi_stage = smem + kStages2 * kStageBytes2;     // 1024-byte aligned
  uint8_t* bar_region = epi_stage + kEpiBytes;
  const uint32_t bar0 = smem_u32(bar_region);
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (kStages2 + s); };
  auto tfull = [&](int b) { return bar0 + 8u * (2 * kStages2 + b); };
  auto tempty = [&](int b) { return bar0 + 8u * (2 * kStages2 + 2 + b); };
  const uint32_t drain_bar = bar0 + 8u * (2 * kStages2 + 4);
  static_assert(8 * (2 * kStages2 + 5) <= 192, "barrier region overflows into the TMEM slot");
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_region + 192);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bar_region + 196);
  volatile int* claim_slot = reinterpret_cast<volatile int*>(bar_region + 200);   // GATHER: 2 ints
  uint64_t call = 0;           // GATHER: this call's number (the header's epoch + 1)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();          // 0 = leader of the pair
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int num_pairs = static_cast<int>(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages2; ++s) {
      mbar_init(full(s), 1);      // leader's expect_tx arrival (+ both CTAs' bytes)
      mbar_init(empty(s), 1);     // leader's multicast MMA commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull(b), 1);     // leader's multicast commit
      mbar_init(tempty(b), 2 * kEpiWarps2);   // every epilogue warp of both CTAs (on the leader)
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    mbar_init_fence();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    if (p.num_jobs > p.num_full) tma_prefetch_desc(&tmap_bh);
    if (p.y_tma) tma_prefetch_desc(&tmap_y);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), kTmemCols2);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();          // peers' barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      asm volatile("griddepcontrol.wait;" ::: "memory");   // A may come from the previous kernel
      if constexpr (GATHER) call = *reinterpret_cast<volatile unsigned long long*>(p.ghdr) + 1;
      const int num_kb = p.k_dev ? device_num_kb(p.k_dev, p.num_kb) : p.num_kb;
      const int num_ks = (num_kb + kAtoms2 - 1) / kAtoms2;
      uint32_t it = 0;
      bool ok = true;
      // a_cols: run starts of the stage after the current one, loaded ahead.
      int64_t nxt0 = 0, nxt1 = 0;
      int snap_kb = -16;            // GATHER: first k atom of the last flag snapshot
      uint32_t ready_bits = 0;
      if (p.a_cols) {
        nxt0 = run_start_load(p.a_cols, 0);
        if (num_kb > 1) nxt1 = run_start_load(p.a_cols, 1);
      }
      for (int job = pair; ok && job < p.num_jobs; job += num_pairs) {
        int m_blk, n_blk, sub;
        job_coords(job, p, m_blk, n_blk, sub);
        const int a_row = m_blk * kPairM + static_cast<int>(rank) * kHalfM;
        // A half job's W' rows: 64 per CTA through the 64-row box of tmap_bh,
        // in the first half of each B atom slot.
        const int b_row = sub < 0 ? n_blk * BN + static_cast<int>(rank) * kHalfN
                                  : n_blk * BN + sub * 128 + static_cast<int>(rank) * 64;
        const void* tb = sub < 0 ? static_cast<const void*>(&tmap_b) : static_cast<const void*>(&tmap_bh);
        const uint32_t b_atom_bytes = sub < 0 ? C::kBAtomBytes : 64 * kBK2 * 2;
        for (int ks = 0; ks < num_ks; ++ks, ++it) {
          const int s = it % kStages2;
          const uint32_t ph = (it / kStages2) & 1u;
          const int64_t cur0 = nxt0, cur1 = nxt1;
          if (p.a_cols) {
            const int nk = (ks + 1 == num_ks ? 0 : ks + 1) * kAtoms2;
            nxt0 = run_start_load(p.a_cols, nk);
            if (nk + 1 < num_kb) nxt1 = run_start_load(p.a_cols, nk + 1);
          }
          if (!mbar_wait_cluster(empty(s), ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
          const uint32_t a_s = sbase + s * kStageBytes2;
          const uint32_t b_s = a_s + kABytes2;
          const uint32_t leader_full = mapa_shared(full(s), 0);
          // The last stage of an odd number of atoms carries one atom.
          const int atoms = min(kAtoms2, num_kb - ks * kAtoms2);
          if (rank == 0)
            mbar_arrive_expect_tx(full(s), 2u * atoms * (kAAtomBytes2 + b_atom_bytes));
          if constexpr (GATHER) {
            // W' first (it does not depend on the gather), then each unit of x'
            // once its flag says it is complete; count the flag down.
            for (int a = 0; a < atoms; ++a)
              tma_load_2d_pair(b_s + a * C::kBAtomBytes, tb, (ks * kAtoms2 + a) * kBK2, b_row,
                               leader_full);
            // The flags of this half-panel are read 16 at a time (ready_bits
            // covers k atoms [snap_kb, snap_kb + 16)); only an atom that was not
            // ready in the last snapshot takes a fresh snapshot and, if still
            // not ready, polls its own flag.
            const unsigned long long* hp_flags =
                p.ghdr + 4 + static_cast<int64_t>(2 * m_blk + static_cast<int>(rank)) * p.num_kb;
            if (ks == 0) snap_kb = -16;
            for (int a = 0; a < atoms; ++a) {
              const int kb = ks * kAtoms2 + a;
              bool ready = kb - snap_kb < 16 && ((ready_bits >> (kb - snap_kb)) & 1u);
              if (!ready) {
                snap_kb = kb;
                ready_bits = flags_ready(hp_flags + kb, min(16, num_kb - kb), call);
                if (!(ready_bits & 1u) && !wait_flag_eq(hp_flags + kb, call, abort_flag, p.err)) {
                  ok = false;
                  break;
                }
                // One proxy fence after each acquisition orders everything it
                // made visible (the gatherers' generic stores) before all of our
                // later TMA reads; atoms covered by an earlier snapshot need none.
                fence_proxy_async_global();
              }
              tma_load_2d_pair(a_s + a * kAAtomBytes2, &tmap_a, kb * kBK2, a_row, leader_full);
            }
            if (!ok) break;
          } else {
            for (int a = 0; a < atoms; ++a) {
              const int kx = (ks * kAtoms2 + a) * kBK2;
              const int ax = p.a_cols ? run_start_check(a == 0 ? cur0 : cur1, p.a_width, p.err) : kx;
              tma_load_2d_pair(a_s + a * kAAtomBytes2, &tmap_a, ax, a_row, leader_full);
              tma_load_2d_pair(b_s + a * C::kBAtomBytes, tb, kx, b_row, leader_full);
            }
          }
        }
      }
      if (!ok && rank == 0) {
        const uint32_t first = it > static_cast<uint32_t>(kStages2) ? it - kStages2 : 0u;
        for (uint32_t i = first; i < it; ++i)
          mbar_wait_cluster(full(i % kStages2), (i / kStages2) & 1u, nullptr, p.err, 100000000ull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc_full = idesc_f16(DT == GW_DTYPE_BF16 ? 1u : 0u, kPairM, BN);
      constexpr uint32_t idesc_half = idesc_f16(DT == GW_DTYPE_BF16 ? 1u : 0u, kPairM, 128);
      int num_kb = p.num_kb;
      if (p.k_dev) {                   // K' written by an earlier kernel: read it after the wait
        asm volatile("griddepcontrol.wait;" ::: "memory");
        num_kb = device_num_kb(p.k_dev, p.num_kb);
      }
      const int num_ks = (num_kb + kAtoms2 - 1) / kAtoms2;
      uint32_t it = 0, lt = 0;
      bool ok = true;
      for (int job = pair; ok && job < p.num_jobs; job += num_pairs, ++lt) {
        const uint32_t b = lt & 1u;
        const uint32_t aph = (lt >> 1) & 1u;
        // A half job is a 256 x 128 MMA into the first 128 columns of the
        // accumulator; B holds 64 rows per CTA at the same addresses.
        const uint32_t idesc = job < p.num_full ? idesc_full : idesc_half;
        if (!mbar_wait_cluster(tempty(b), aph ^ 1u, abort_flag, p.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * BN;
        for (int ks = 0; ks < num_ks; ++ks, ++it) {
          const int s = it % kStages2;
          const uint32_t ph = (it / kStages2) & 1u;
          if (!mbar_wait_cluster(full(s), ph, abort_flag, p.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_s = sbase + s * kStageBytes2;
          const uint64_t a_desc = smem_desc_kmajor_sw128(a_s);
          const uint64_t b_desc = smem_desc_kmajor_sw128(a_s + kABytes2);
          const bool two = ks * kAtoms2 + 1 < num_kb;
          // Atom 1 of A and of B starts one atom further on (>> 4 in the
          // descriptor); each 16-wide k step advances 32 bytes inside the atom.
#pragma unroll
          for (int k = 0; k < kBK2 / 16; ++k)
            tc_mma_f16_pair(d_tmem, a_desc + 2u * k, b_desc + 2u * k, idesc,
                            (ks > 0 || k > 0) ? 1u : 0u);
          if (two) {
#pragma unroll
            for (int k = 0; k < kBK2 / 16; ++k)
              tc_mma_f16_pair(d_tmem, a_desc + (kAAtomBytes2 >> 4) + 2u * k,
                              b_desc + (C::kBAtomBytes >> 4) + 2u * k, idesc, 1u);
          }
          tc_commit_pair_mc(empty(s), 0x3);
        }
        if (!ok) break;
        tc_commit_pair_mc(tfull(b), 0x3);
      }
      tc_commit_pair_mc(drain_bar, 0x1);
      mbar_wait(drain_bar, 0u, nullptr, p.err, 100000000ull);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    // Eight warps: warp w drains TMEM lanes 32 (w % 4) .. +31 (rows of this
    // CTA's half tile) and columns [0, 128) (h = (w - 2) / 4 = 0) or
    // [128, BN) (h = 1) of the tile, in 64-column chunks. Each 32-column tcgen05 load is issued before the
    // previous one is converted; bias + activation + one packed rounding per
    // pair of values; then a TMA store from the warp's 128-byte-swizzled
    // staging tile, or direct stores when y's rows are not 16-byte aligned.
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t leader_tempty0 = mapa_shared(tempty(0), 0);
    const uint32_t leader_tempty1 = mapa_shared(tempty(1), 0);
    uint8_t* sb = epi_stage + (warp - 2) * kEpiTileBytes;
    if constexpr (GATHER) {
      // x, the alive list and the workspace may come from the previous kernel.
      asm volatile("griddepcontrol.wait;" ::: "memory");
      call = *reinterpret_cast<volatile unsigned long long*>(p.ghdr) + 1;
      gather_units<DT>(p, warp - 2, lane, claim_slot, call);
    }
    uint32_t lt = 0;
    for (int job = pair; job < p.num_jobs; job += num_pairs, ++lt) {
      int m_blk, n_blk, sub;
      job_coords(job, p, m_blk, n_blk, sub);
      const uint32_t b = lt & 1u;
      const uint32_t aph = (lt >> 1) & 1u;
      if (!mbar_wait_cluster(tfull(b), aph, abort_flag, p.err)) break;
      tc_fence_after();
      const int64_t warp_row0 = static_cast<int64_t>(m_blk) * kPairM + rank * kHalfM + q * 32;
      const int64_t row = warp_row0 + lane;
      const bool row_ok = row < p.M;
      uint16_t* yrow = p.y + (row_ok ? row * p.ldy : 0);
      // Whole tile: columns [0, 128) (half 0) or [128, BN) (half 1). Half
      // job: 64 columns each, [0, 64) and [64, 128) of its 128.
      const int col0 = sub < 0 ? half * C::kCols0 : half * 64;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + b * BN + col0;
      const int64_t n_warp = static_cast<int64_t>(n_blk) * BN + (sub < 0 ? 0 : sub * 128) + col0;
      const int steps = sub < 0 ? (half ? C::kCols1 : C::kCols0) / 32 : 2;   // 32-column loads (even)
      uint32_t acc[32];
      tc_ld_32x32b_x32(t_row, acc);
#pragma unroll 1
      for (int st = 0; st < steps; ++st) {
        tc_wait_ld();
        float f[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(acc[j]);
        if (st + 1 < steps) tc_ld_32x32b_x32(t_row + (st + 1) * 32, acc);
        const int c = st >> 1;                          // 64-column chunk
        const int h = st & 1;                           // its 32-column half
        const int64_t n_chunk = n_warp + c * kEpiCols;
        const int64_t n_base = n_chunk + h * 32;
        if (p.y_tma && h == 0) {
          // The staging tile's previous TMA store must have read it.
          if (lane == 0) bulk_wait_group_read<0>();
          __syncwarp();
        }
        if (p.bias) add_bias32<DT>(f, p.bias, n_base, p.N);
        activate32<EPI>(f);
        uint32_t packed[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) packed[j] = Elem<DT>::pack2(f[2 * j], f[2 * j + 1]);
        if (p.y_tma) {
          // Row `lane` of the staging tile, 128-byte swizzle: 16-byte unit
          // v of the row lives at unit (v ^ (row & 7)).
          uint4* srow = reinterpret_cast<uint4*>(sb + lane * (kEpiCols * 2));
#pragma unroll
          for (int v = 0; v < 4; ++v)
            srow[(h * 4 + v) ^ (lane & 7)] =
                make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
          if (h == 1) {
            fence_proxy_async_smem();    // staging writes -> visible to the TMA unit
            __syncwarp();
            if (lane == 0) {
              if (warp_row0 < p.M && n_chunk < p.N)
                tma_store_2d(&tmap_y, smem_u32(sb), static_cast<int32_t>(n_chunk),
                             static_cast<int32_t>(warp_row0));
              bulk_commit_group();
            }
            if (p.n_peers > 0 && warp_row0 < p.M && n_chunk < p.N) {
              // The same 32 x 64 tile to every peer over NVLink: eight lanes per
              // row write its 128 bytes, four rows per pass.
              const int unit = lane & 7;
              const int64_t col = n_chunk + unit * 8;
#pragma unroll 1
              for (int pass = 0; pass < 8; ++pass) {
                const int r = pass * 4 + (lane >> 3);
                const int64_t grow = warp_row0 + r;
                if (grow >= p.M) break;
                const uint4 v = *reinterpret_cast<const uint4*>(sb + r * (kEpiCols * 2) +
                                                               ((unit ^ (r & 7)) << 4));
                for (int i = 0; i < p.n_peers; ++i) {
                  uint16_t* dst = p.peers[i] + grow * p.ldy + col;
                  if (col + 8 <= p.N) {
                    *reinterpret_cast<uint4*>(dst) = v;
                  } else {
                    const uint16_t* e = reinterpret_cast<const uint16_t*>(&v);
                    for (int j = 0; j < 8 && col + j < p.N; ++j) dst[j] = e[j];
                  }
                }
              }
            }
          }
        } else if (row_ok) {
          if (p.y_vec_ok && n_base + 32 <= p.N) {
            uint4* dst = reinterpret_cast<uint4*>(yrow + n_base);
#pragma unroll
            for (int v = 0; v < 4; ++v)
              dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (n_base + j < p.N) yrow[n_base + j] = Elem<DT>::from_f(f[j]);
          }
        }
      }
      // All TMEM reads of this accumulator are complete: hand it back. After
      // this pair's last job nothing waits for it (the MMA thread waits for an
      // accumulator only before a later job), so no remote arrive is left in
      // flight into the leader when the CTAs finish.
      tc_fence_before();
      __syncwarp();
      if (lane == 0 && job + num_pairs < p.num_jobs) {
        if (rank == 0) mbar_arrive(tempty(b));
        else mbar_arrive_cluster(b ? leader_tempty1 : leader_tempty0);
      }
    }
    // Staging tiles stay valid (and y complete) until every TMA store has finished.
    if (lane == 0) bulk_wait_group_all();
    __syncwarp();
    if (p.n_peers > 0) __threadfence_system();   // peer stores ordered before the kernel ends
  }

  __syncthreads();
  // Both CTAs are done before either frees TMEM or exits. By now the leader's
  // MMAs into this CTA's TMEM and their reads of its shared memory are
  // complete (its epilogue waited for the last accumulator), the peer's TMA
  // loads into the leader's barriers were all consumed, and no remote
  // arrive follows the last job. So the arrive need not order this CTA's
  // earlier memory operations (its y stores are complete, and no peer reads
  // them): a relaxed arrive, about 0.5 us less than a release one.
  cluster_arrive_relaxed();
  cluster_wait();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols2);
  }
  if constexpr (GATHER) {
    // The last CTA to finish moves the epoch on (every CTA has read it by now).
    // Thread 0 is the TMA producer, which read the call number after its wait.
    if (threadIdx.x == 0 && tagged_add(p.ghdr + 2, call, 1u) + 1u == gridDim.x) {
      // Both counters start the next call at zero under its number, so its
      // first claims take the single-atomicAdd path.
      constexpr uint64_t kTagMask = (uint64_t{1} << (64 - kCountBits)) - 1;
      const uint64_t next = ((call + 1) & kTagMask) << kCountBits;
      p.ghdr[1] = next;
      p.ghdr[2] = next;
      st_release_gpu_u64(p.ghdr, call);
    }
  }
}

}  // namespace

namespace {
// Pair tile width for an M x N output: the one that minimises rounds x the
// bytes a CTA loads per k atom (A 16 KB + B BN/2 rows), rounds = waves of
// pair tiles over the SM pairs. Ties keep 256.
int pair_tile_width(int64_t M, int64_t N, int sm_count) {
  const int64_t pairs = std::max<int64_t>(1, (sm_count > 0 ? sm_count : 148) / 2);
  const int64_t m_tiles = (M + kPairM - 1) / kPairM;
  auto cost = [&](int bn) {
    const int64_t tiles = m_tiles * ((N + bn - 1) / bn);
    const int64_t rounds = (tiles + pairs - 1) / pairs;
    return rounds * (16 + bn / 16);
  };
  return cost(192) < cost(256) ? 192 : 256;
}
}  // namespace

int pair_gemm_tile_width(int64_t M, int64_t N, int sm_count) {
  // GW_GEMM_PAIR_BN=256|192 overrides the tile width (tuning, tests).
  static const int forced_bn = [] {
    const char* v = std::getenv("GW_GEMM_PAIR_BN");
    return v ? std::atoi(v) : 0;
  }();
  return (forced_bn == 256 || forced_bn == 192) ? forced_bn : pair_tile_width(M, N, sm_count);
}

namespace {
// GW_GEMM_PAIR_TAIL=0 keeps the last round of tiles whole (tuning, tests).
bool pair_tail_split_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("GW_GEMM_PAIR_TAIL");
    return !(v && std::atoi(v) == 0);
  }();
  return on;
}
}  // namespace

bool use_pair_gemm(int64_t M, int64_t N, int sm_count) {
  // GW_GEMM_PAIR=0 forces the single-CTA kernel, =1 the pair kernel (tuning, tests).
  static const int forced = [] {
    const char* v = std::getenv("GW_GEMM_PAIR");
    return v ? std::atoi(v) : -1;
  }();
  if (forced == 0) return false;
  if (forced == 1) return true;
  if (M <= kHalfM || N <= 128) return false;
  // Pairs pay off once their tiles occupy most SM pairs; below that, 128-row
  // tiles spread the work over more SMs (measured).
  const int64_t pairs = (sm_count > 0 ? sm_count : 148) / 2;
  const int bn = pair_tile_width(M, N, sm_count);
  const int64_t pair_tiles = ((M + kPairM - 1) / kPairM) * ((N + bn - 1) / bn);
  return bn == 256 ? pair_tiles >= pairs : 10 * pair_tiles >= 8 * pairs;
}

template <int BN>
cudaError_t launch_tc2_bn(int dtype, Tc2Params& p, const void* a, int64_t M, int64_t K,
                          int64_t lda, const void* w, int64_t N, int64_t ldw, void* y,
                          int64_t ldy, int sm_count, cudaStream_t stream) {
  using C = Tc2Cfg<BN>;
  const int64_t m_tiles = (M + kPairM - 1) / kPairM;
  const int64_t n_tiles = (N + BN - 1) / BN;
  const int64_t num_tiles = m_tiles * n_tiles;
  if (num_tiles > 0x7FFFFFFFll) return cudaErrorInvalidValue;
  p.m_tiles = static_cast<int>(m_tiles);
  p.n_tiles = static_cast<int>(n_tiles);
  p.num_tiles = static_cast<int>(num_tiles);
  CUtensorMap ta, tb, tbh, ty;
  // With a_cols, A is x [M, a_width] (K = the alive count, a multiple of 64).
  if (p.a_cols && (K % kBK2) != 0) return cudaErrorInvalidValue;
  if (!make_tmap_kmajor(&ta, a, M, p.a_cols ? p.a_width : K, lda, kBK2, kHalfM))
    return cudaErrorInvalidValue;
  if (!make_tmap_kmajor(&tb, w, N, K, ldw, kBK2, C::kHalfN)) return cudaErrorInvalidValue;
  tbh = tb;                  // read only by half jobs (set below)
  // TMA-store epilogue when y's rows are 16-byte aligned (else direct stores).
  p.y_tma = p.y_vec_ok && make_tmap_kmajor(&ty, y, M, N, ldy, kEpiCols, 32) ? 1 : 0;
  if (!p.y_tma) ty = ta;     // not read by the kernel
  if (p.n_peers > 0 && !p.y_tma) return cudaErrorInvalidValue;   // peer stores ride the TMA path

  const int64_t pairs = std::max<int64_t>(1, (sm_count > 0 ? sm_count : 148) / 2);
  // The last, partial round of 256-wide tiles leaves pairs idle for a whole
  // tile time. When at most half the pairs would be busy in it, its tiles run
  // as two 128-column jobs each, so the round takes a half job (which loads
  // three quarters of a tile's bytes) and spreads over twice as many pairs.
  p.num_full = p.num_tiles;
  p.num_jobs = p.num_tiles;
  const int64_t rem = num_tiles % pairs;
  if (BN == 256 && !p.ghdr && pair_tail_split_enabled() && rem > 0 && 2 * rem <= pairs) {
    if (!make_tmap_kmajor(&tbh, w, N, K, ldw, kBK2, 64)) return cudaErrorInvalidValue;
    p.num_full = static_cast<int>(num_tiles - rem);
    p.num_jobs = static_cast<int>(num_tiles + rem);
  }
  const int grid = static_cast<int>(2 * std::min<int64_t>(p.num_jobs, pairs));
  if (p.ghdr) {
    // In-kernel gather: tiles row block by row block; claim groups of as many
    // half-panels as one wave of tiles spans.
    p.m_major = 1;
    p.h_total = static_cast<int>(2 * m_tiles);
    const int64_t wave_rows = (pairs + n_tiles - 1) / n_tiles;      // row blocks per wave
    p.g_hp = static_cast<int>(std::min<int64_t>(2 * m_tiles, 2 * std::max<int64_t>(1, wave_rows)));
  }

  const bool bf = dtype == GW_DTYPE_BF16;
#define GW_TC2_KERN(G)                                                          \
  (p.epi == GW_EPI_GELU_ERF                                                     \
       ? (bf ? gemm_tc2_kernel<BN, GW_DTYPE_BF16, GW_EPI_GELU_ERF, G>           \
             : gemm_tc2_kernel<BN, GW_DTYPE_F16, GW_EPI_GELU_ERF, G>)           \
   : p.epi == GW_EPI_GELU_TANH                                                  \
       ? (bf ? gemm_tc2_kernel<BN, GW_DTYPE_BF16, GW_EPI_GELU_TANH, G>          \
             : gemm_tc2_kernel<BN, GW_DTYPE_F16, GW_EPI_GELU_TANH, G>)          \
       : (bf ? gemm_tc2_kernel<BN, GW_DTYPE_BF16, GW_EPI_NONE, G>               \
             : gemm_tc2_kernel<BN, GW_DTYPE_F16, GW_EPI_NONE, G>))
  auto kern = p.ghdr ? GW_TC2_KERN(true) : GW_TC2_KERN(false);
#undef GW_TC2_KERN
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kern), C::kSmemBytes);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kThreads2);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, tb, tbh, ta, ty, p);
}

cudaError_t launch_gemm_tc2(const void* a, int dtype, int64_t M, int64_t K, int64_t lda,
                            const void* w, int64_t N, int64_t ldw, const void* bias, int epilogue,
                            void* y, int64_t ldy, unsigned int* err, int sm_count,
                            cudaStream_t stream, void* const* peers, int n_peers,
                            const int64_t* a_cols, int64_t a_width, const int32_t* k_dev,
                            const Tc2Gather* gather) {
  Tc2Params p{};
  p.M = M;
  p.N = N;
  p.bias = static_cast<const uint16_t*>(bias);
  p.epi = epilogue;
  p.y = static_cast<uint16_t*>(y);
  p.ldy = ldy;
  p.y_vec_ok = ((reinterpret_cast<uintptr_t>(y) & 15u) == 0 && (ldy % 8) == 0) ? 1 : 0;
  p.num_kb = static_cast<int>((K + kBK2 - 1) / kBK2);
  p.num_ks = (p.num_kb + kAtoms2 - 1) / kAtoms2;
  p.err = err;
  if (n_peers < 0 || n_peers > kMaxPeers || (n_peers > 0 && !peers)) return cudaErrorInvalidValue;
  p.n_peers = n_peers;
  for (int i = 0; i < n_peers; ++i) p.peers[i] = static_cast<uint16_t*>(peers[i]);
  p.a_cols = a_cols;
  p.a_width = a_width;
  p.k_dev = k_dev;
  if (gather) {
    if (a_cols || k_dev || !gather->x || !gather->idx || !gather->xg || !gather->header ||
        (gather->ldp % 8) != 0 || gather->ldp < K)
      return cudaErrorInvalidValue;
    p.gx = static_cast<const uint16_t*>(gather->x);
    p.ldgx = gather->ldx;
    p.gK = gather->K;
    p.gidx = gather->idx;
    p.n_alive = K;
    p.xg = static_cast<uint16_t*>(gather->xg);
    p.ldp = gather->ldp;
    if (!tc2_gather_supported(M, K)) return cudaErrorInvalidValue;
    p.ghdr = static_cast<unsigned long long*>(gather->header);
    a = gather->xg;
    lda = gather->ldp;
  }
  const int bn = pair_gemm_tile_width(M, N, sm_count);
  return bn == 192 ? launch_tc2_bn<192>(dtype, p, a, M, K, lda, w, N, ldw, y, ldy, sm_count, stream)
                   : launch_tc2_bn<256>(dtype, p, a, M, K, lda, w, N, ldw, y, ldy, sm_count, stream);
}

size_t tc2_gather_header_bytes(int64_t M, int64_t n_alive) {
  const int64_t half_panels = 2 * ((M + kPairM - 1) / kPairM);
  const int64_t kb = (n_alive + kBK2 - 1) / kBK2;
  return static_cast<size_t>((8 * (4 + half_panels * kb) + 255) / 256 * 256);
}

bool tc2_gather_supported(int64_t M, int64_t n_alive) {
  const int64_t half_panels = 2 * ((M + kPairM - 1) / kPairM);
  const int64_t kb = (n_alive + kBK2 - 1) / kBK2;
  return half_panels * kb + 2 < (int64_t{1} << kCountBits);
}

}  // namespace gw
