// K3: fused gather-GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
//   y[m, n] = act( sum_j x[m, idx[j]] * w[n, j] + bias[n] )      fp16 / bf16 in, fp32 accumulate
//
// This is the B200 replacement of ghostweight_triton/kernels/matmul.py:27-82
// (which gathers A columns and W rows with pointer loads inside a 64x64x32
// tl.dot loop) plus the bias add of module.py:116-117. Design:
//
//   * persistent kernel, one 448-thread CTA per SM, 128 x BN output tiles
//     (BN = 256 or 128), K' consumed in 64-wide k-blocks (128 B of fp16/bf16,
//     one 128-byte swizzle atom), 4-stage shared-memory ring;
//   * warp 0      : TMA producer for the packed weight tile w[n0:n0+BN, k:k+64]
//                   (and for A too when A is an already compacted matrix);
//   * warp 1      : TMEM allocator and the single-thread tcgen05.mma issuer
//                   (128 x BN x 16 per instruction, 4 per k-block), commits
//                   free smem stages and publish finished accumulators;
//   * warps 2..9  : A-operand gather (SMEM mode): two groups of four warps
//                   take alternate k-blocks; a warp loads 32 rows x 64 alive
//                   columns of x straight from global memory (lane <-> alive
//                   column), waits for the stage to be free and writes the
//                   values into the 128B-swizzled K-major shared-memory layout
//                   tcgen05 reads (no scratch, one launch);
//   * warps 10..13: epilogue -- tcgen05.ld of the fp32 accumulator (one TMEM
//                   lane per output row), bias, optional GELU, one rounding to
//                   the output type, 16-byte stores;
//   * the accumulator is double-buffered in TMEM (2 x BN columns), so the
//     epilogue of tile t overlaps the main loop of tile t+1.
// No TMA multicast is used anywhere (the kernel also runs in multi-GPU jobs).
// Every mbarrier wait is bounded (gw_common.cuh); on a timeout all roles leave
// their loops, in-flight TMA loads and MMAs are drained, TMEM is freed and the
// device error word records the event.
#include <algorithm>
#include <cstdlib>

#include <cuda.h>

#include "gw_common.cuh"
#include "gw_internal.h"

namespace gw {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 448;
constexpr int kMaxStages = 8;
constexpr int kWarpTma = 0;
constexpr int kWarpMma = 1;
constexpr int kWarpGather0 = 2;
constexpr int kGatherWarps = 8;      // two groups of four
constexpr int kWarpEpi0 = 10;        // four epilogue warps (gather modes)
// With a dense A operand the gather warps are free: warps 6..13 drain TMEM,
// two per lane quadrant, each with half of the tile's columns.
constexpr int kWarpEpi0Dense = 6;
template <int AMODE> constexpr int epi_warps() { return AMODE == 0 ? 8 : 4; }

// How the A operand (x[:, alive]) reaches shared memory.
constexpr int kATma = 0;        // dense [M, K'] matrix by TMA (already compacted)
constexpr int kASmemGather = 1; // producer warps gather into shared memory

constexpr int pow2_at_least(int v) { int p = 32; while (p < v) p <<= 1; return p; }

template <int BN>
struct TcCfg {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  // As many stages as fit in ~200 KB of shared memory (4 for BN=256, 5 for 192, 6 for 128).
  static constexpr int kStagesFit = (200 * 1024) / kStageBytes;
  static constexpr int kStages = kStagesFit > kMaxStages ? kMaxStages : kStagesFit;
  static constexpr int kTmemCols = pow2_at_least(2 * BN);   // two accumulator buffers
  static constexpr int kBarBytes = 256;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kBarBytes;
};

struct TcParams {
  const uint16_t* x;
  int64_t ldx;
  int64_t M;
  int64_t K;
  const int64_t* idx;
  int64_t n_alive;
  int64_t N;
  const uint16_t* bias;
  int epi;
  int y_vec_ok;
  uint16_t* y;
  int64_t ldy;
  int num_kb;
  int m_tiles;
  int n_tiles;
  int num_tiles;
  unsigned int* err;
  const int64_t* a_cols;        // kATma: k-block kb of A starts at x column a_cols[64 kb] (or null)
  const int32_t* k_dev;         // kATma: K' on the device (num_kb an upper bound; see device_num_kb)
};

template <int BN, int DT, int AMODE, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_b,
               const __grid_constant__ CUtensorMap tmap_a, const TcParams p) {
  using C = TcCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment (of the shared-window address) for the swizzled tiles.
  const uint32_t raw_s = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_s & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);

  uint8_t* bar_region = smem + C::kStages * C::kStageBytes;
  const uint32_t bar0 = smem_u32(bar_region);
  // barriers: full_a[S] full_b[S] empty[S] tfull[2] tempty[2] drain
  auto full_a = [&](int s) { return bar0 + 8u * s; };
  auto full_b = [&](int s) { return bar0 + 8u * (C::kStages + s); };
  auto empty = [&](int s) { return bar0 + 8u * (2 * C::kStages + s); };
  auto tfull = [&](int b) { return bar0 + 8u * (3 * C::kStages + b); };
  auto tempty = [&](int b) { return bar0 + 8u * (3 * C::kStages + 2 + b); };
  const uint32_t drain_bar = bar0 + 8u * (3 * C::kStages + 4);
  static_assert(8 * (3 * C::kStages + 5) <= 192, "barrier region overflows into the TMEM slot");
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_region + 192);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bar_region + 196);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(full_a(s), kGatherWarps / 2);
      mbar_init(full_b(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull(b), 1);
      mbar_init(tempty(b), epi_warps<AMODE>());
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    mbar_init_fence();
  }
  if (warp == kWarpTma && lane == 0) {
    tma_prefetch_desc(&tmap_b);
    if (AMODE != kASmemGather) tma_prefetch_desc(&tmap_a);
  }
  if (warp == kWarpMma) {
    tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == kWarpTma) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      // A dense A operand may have been written by the previous kernel on the
      // stream (the pregather launch): with programmatic dependent launch this
      // CTA got here early, so wait for that grid before reading it.
      if (AMODE == kATma) asm volatile("griddepcontrol.wait;" ::: "memory");
      const int num_kb = (AMODE == kATma && p.k_dev) ? device_num_kb(p.k_dev, p.num_kb) : p.num_kb;
      uint32_t it = 0;
      bool ok = true;
      const int64_t* a_cols = AMODE == kATma ? p.a_cols : nullptr;
      int64_t nxt = a_cols ? run_start_load(a_cols, 0) : 0;   // next k-block's run start
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        const int m_blk = tile % p.m_tiles;
        const int n_blk = tile / p.m_tiles;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % C::kStages;
          const uint32_t ph = (it / C::kStages) & 1u;
          const int64_t cur = nxt;
          if (a_cols) nxt = run_start_load(a_cols, kb + 1 == num_kb ? 0 : kb + 1);
          if (!mbar_wait(empty(s), ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
          const uint32_t a_s = sbase + s * C::kStageBytes;
          const uint32_t b_s = a_s + C::kABytes;
          if (AMODE == kASmemGather) {
            mbar_arrive_expect_tx(full_b(s), C::kBBytes);
            tma_load_2d(b_s, &tmap_b, kb * kBK, n_blk * BN, full_b(s));
          } else {
            mbar_arrive_expect_tx(full_b(s), C::kBBytes + C::kABytes);
            tma_load_2d(b_s, &tmap_b, kb * kBK, n_blk * BN, full_b(s));
            const int ax = a_cols ? run_start_check(cur, p.K, p.err) : kb * kBK;
            tma_load_2d(a_s, &tmap_a, ax, m_blk * kBM, full_b(s));
          }
        }
      }
      if (!ok) {
        // Drain loads still in flight before the CTA exits (bounded, 100 ms).
        const uint32_t first = it > static_cast<uint32_t>(C::kStages) ? it - C::kStages : 0u;
        for (uint32_t i = first; i < it; ++i)
          mbar_wait(full_b(i % C::kStages), (i / C::kStages) & 1u, nullptr, p.err, 100000000ull);
      }
    }
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(DT == GW_DTYPE_BF16 ? 1u : 0u, kBM, BN);
      int num_kb = p.num_kb;
      if (AMODE == kATma && p.k_dev) {  // K' written by an earlier kernel: read it after the wait
        asm volatile("griddepcontrol.wait;" ::: "memory");
        num_kb = device_num_kb(p.k_dev, p.num_kb);
      }
      uint32_t it = 0, lt = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x, ++lt) {
        const uint32_t b = lt & 1u;
        const uint32_t aph = (lt >> 1) & 1u;
        if (!mbar_wait(tempty(b), aph ^ 1u, abort_flag, p.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * BN;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % C::kStages;
          const uint32_t ph = (it / C::kStages) & 1u;
          if (!mbar_wait(full_b(s), ph, abort_flag, p.err)) { ok = false; break; }
          if (AMODE == kASmemGather && !mbar_wait(full_a(s), ph, abort_flag, p.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_s = sbase + s * C::kStageBytes;
          const uint64_t a_desc = smem_desc_kmajor_sw128(a_s);
          const uint64_t b_desc = smem_desc_kmajor_sw128(a_s + C::kABytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            // +32 bytes per 16-element k step inside the swizzle atom (>> 4 in the descriptor).
            tc_mma_f16(d_tmem, a_desc + 2u * k, b_desc + 2u * k, idesc,
                       (kb > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit(empty(s));
        }
        if (!ok) break;
        tc_commit(tfull(b));
      }
      // All MMAs of this thread complete before TMEM can be released.
      tc_commit(drain_bar);
      mbar_wait(drain_bar, 0u, nullptr, p.err, 100000000ull);
    }
    __syncwarp();
  } else if (warp < (AMODE == kATma ? kWarpEpi0Dense : kWarpEpi0)) {
    // ------------------------------------------------------------ gather producers
    if (AMODE == kASmemGather) {
      const int gw_idx = warp - kWarpGather0;
      const uint32_t grp = static_cast<uint32_t>(gw_idx >> 2);
      const int wrow = (gw_idx & 3) * 32;
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        const int m_blk = tile % p.m_tiles;
        const int64_t row0 = static_cast<int64_t>(m_blk) * kBM + wrow;
        const int64_t rem = p.M - row0;
        const int rows_here = rem <= 0 ? 0 : (rem >= 32 ? 32 : static_cast<int>(rem));
        const uint16_t* xw = p.x + (rows_here > 0 ? row0 * p.ldx : 0);
        for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
          if ((it & 1u) != grp) continue;
          const int s = it % C::kStages;
          const uint32_t ph = (it / C::kStages) & 1u;
          const int64_t k0 = static_cast<int64_t>(kb) * kBK + lane;
          int64_t c0 = -1, c1 = -1;
          bool bad = false;
          if (k0 < p.n_alive) {
            c0 = __ldg(p.idx + k0);
            if (c0 < 0 || c0 >= p.K) { bad = true; c0 = -1; }
          }
          if (k0 + 32 < p.n_alive) {
            c1 = __ldg(p.idx + k0 + 32);
            if (c1 < 0 || c1 >= p.K) { bad = true; c1 = -1; }
          }
          if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) raise_error(p.err, GW_DERR_BAD_INDEX);
          uint16_t v0[32], v1[32];
#pragma unroll
          for (int r = 0; r < 32; ++r) {
            const bool rv = r < rows_here;
            v0[r] = (rv && c0 >= 0) ? __ldg(xw + r * p.ldx + c0) : static_cast<uint16_t>(0);
            v1[r] = (rv && c1 >= 0) ? __ldg(xw + r * p.ldx + c1) : static_cast<uint16_t>(0);
          }
          if (!mbar_wait(empty(s), ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
          uint8_t* a_tile = smem + s * C::kStageBytes;
          const int ch0 = lane >> 3;
          const int byte_in_chunk = (lane & 7) << 1;
#pragma unroll
          for (int r = 0; r < 32; ++r) {
            const int row = wrow + r;
            const int sw = row & 7;
            uint8_t* rowp = a_tile + row * 128 + byte_in_chunk;
            *reinterpret_cast<uint16_t*>(rowp + ((ch0 ^ sw) << 4)) = v0[r];
            *reinterpret_cast<uint16_t*>(rowp + (((ch0 + 4) ^ sw) << 4)) = v1[r];
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(full_a(s));
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Warp w drains TMEM lanes 32 (w % 4) .. +31 (its rows of the tile); with
    // eight epilogue warps each takes half of the BN columns. The next
    // 32-column tcgen05 load is issued before the current one is converted;
    // bias, activation, one packed rounding per pair, 16-byte stores.
    constexpr int kEpiWarps = epi_warps<AMODE>();
    constexpr int kCols = BN / (kEpiWarps / 4);         // columns per warp
    constexpr int kSteps = kCols / 32;
    const int q = warp & 3;                       // TMEM lane quarter this warp may access
    const int part = (warp - (AMODE == kATma ? kWarpEpi0Dense : kWarpEpi0)) >> 2;
    const int row_in_tile = q * 32 + lane;
    uint32_t lt = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++lt) {
      const int m_blk = tile % p.m_tiles;
      const int n_blk = tile / p.m_tiles;
      const uint32_t b = lt & 1u;
      const uint32_t aph = (lt >> 1) & 1u;
      if (!mbar_wait(tfull(b), aph, abort_flag, p.err)) break;
      tc_fence_after();
      const int64_t row = static_cast<int64_t>(m_blk) * kBM + row_in_tile;
      const bool row_ok = row < p.M;
      uint16_t* yrow = p.y + (row_ok ? row * p.ldy : 0);
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + b * BN + part * kCols;
      const int64_t n_warp = static_cast<int64_t>(n_blk) * BN + part * kCols;
      uint32_t acc[32];
      tc_ld_32x32b_x32(t_row, acc);
#pragma unroll 1
      for (int c = 0; c < kSteps; ++c) {
        tc_wait_ld();
        float f[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(acc[j]);
        if (c + 1 < kSteps) tc_ld_32x32b_x32(t_row + (c + 1) * 32, acc);
        const int64_t n_base = n_warp + c * 32;
        if (p.bias) add_bias32<DT>(f, p.bias, n_base, p.N);
        activate32<EPI>(f);
        if (row_ok) {
          if (p.y_vec_ok && n_base + 32 <= p.N) {
            uint32_t packed[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) packed[j] = Elem<DT>::pack2(f[2 * j], f[2 * j + 1]);
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
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty(b));
    }
  }

  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
template <int BN, int DT, int AMODE>
cudaError_t launch_tc(const CUtensorMap& tb, const CUtensorMap& ta, const TcParams& p,
                      int sm_count, cudaStream_t stream) {
  using C = TcCfg<BN>;
  auto kern = p.epi == GW_EPI_GELU_ERF    ? gemm_tc_kernel<BN, DT, AMODE, GW_EPI_GELU_ERF>
              : p.epi == GW_EPI_GELU_TANH ? gemm_tc_kernel<BN, DT, AMODE, GW_EPI_GELU_TANH>
                                          : gemm_tc_kernel<BN, DT, AMODE, GW_EPI_NONE>;
  // Opt in to the large dynamic shared-memory carve-out (idempotent, cheap).
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kern), C::kSmemBytes);
  if (e != cudaSuccess) return e;
  const int grid = std::min(p.num_tiles, sm_count > 0 ? sm_count : 148);
  if (AMODE == kASmemGather) {
    kern<<<grid, kThreads, C::kSmemBytes, stream>>>(tb, ta, p);
    return cudaGetLastError();
  }
  {
    // Programmatic dependent launch: the prologue (barriers, TMEM, descriptor
    // prefetch) overlaps the tail of the previous kernel on the stream; the
    // TMA warp waits for that kernel before it reads the A operand.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, tb, ta, p);
  }
}

}  // namespace

cudaError_t launch_gemm_tc(int a_mode, const void* x, int dtype, int64_t M, int64_t K,
                           int64_t ldx, const void* w, int64_t N, int64_t ldw,
                           const int64_t* idx, int64_t n_alive, const void* bias, int epilogue,
                           void* y, int64_t ldy, unsigned int* err, int sm_count,
                           cudaStream_t stream, const int64_t* a_cols, const int32_t* k_dev) {
  // Tile width 256 (measured best on B200 where there are several waves:
  // wider tiles reuse A more per byte moved), 128 for narrow N. When 256-wide
  // tiles leave SMs idle in a single wave and 192-wide ones still fit in one
  // (N = 768: 3 -> 4 column tiles), 192 (measured faster for such layers).
  // GW_GEMM_BN=128|192|256 overrides the choice (tuning and tests).
  const int64_t m_tiles = (M + kBM - 1) / kBM;
  const int64_t sms = sm_count > 0 ? sm_count : 148;
  int BN = N <= 128 ? 128 : 256;
  if (BN == 256 && m_tiles * ((N + 255) / 256) < sms && m_tiles * ((N + 191) / 192) <= sms &&
      (N + 191) / 192 > (N + 255) / 256)
    BN = 192;
  {
    static const int forced = [] {
      const char* v = std::getenv("GW_GEMM_BN");
      return v ? std::atoi(v) : 0;
    }();
    if (forced == 128 || forced == 192 || forced == 256) BN = forced;
  }
  const int64_t n_tiles = (N + BN - 1) / BN;
  const int64_t num_tiles = m_tiles * n_tiles;
  if (num_tiles > 0x7FFFFFFFll || m_tiles > 0x7FFFFFFFll) return cudaErrorInvalidValue;
  const int64_t num_kb = (n_alive + kBK - 1) / kBK;
  if (a_mode != kATma && a_mode != kASmemGather) return cudaErrorInvalidValue;

  TcParams p{};
  p.x = static_cast<const uint16_t*>(x);
  p.ldx = ldx;
  p.M = M;
  p.K = K;
  p.idx = idx;
  p.n_alive = n_alive;
  p.N = N;
  p.bias = static_cast<const uint16_t*>(bias);
  p.epi = epilogue;
  p.y = static_cast<uint16_t*>(y);
  p.ldy = ldy;
  p.y_vec_ok = ((reinterpret_cast<uintptr_t>(y) & 15u) == 0 && (ldy % 8) == 0) ? 1 : 0;
  p.num_kb = static_cast<int>(num_kb);
  p.m_tiles = static_cast<int>(m_tiles);
  p.n_tiles = static_cast<int>(n_tiles);
  p.num_tiles = static_cast<int>(num_tiles);
  p.err = err;
  p.a_cols = a_mode == kATma ? a_cols : nullptr;
  p.k_dev = a_mode == kATma ? k_dev : nullptr;
  if (p.a_cols && (n_alive % kBK) != 0) return cudaErrorInvalidValue;

  CUtensorMap tb, ta;
  if (!make_tmap_kmajor(&tb, w, N, n_alive, ldw, kBK, BN)) return cudaErrorInvalidValue;
  if (a_mode == kASmemGather) {
    ta = tb;   // unused by the shared-memory gather variant
  } else if (a_mode == kATma) {
    // A is the compacted x' [M, n_alive], or x [M, K] itself with a_cols.
    if (!make_tmap_kmajor(&ta, x, M, a_cols ? K : n_alive, ldx, kBK, kBM)) return cudaErrorInvalidValue;
  }

#define GW_TC_MODES(BNV, DTV)                                                                     \
  switch (a_mode) {                                                                              \
    case kATma: return launch_tc<BNV, DTV, kATma>(tb, ta, p, static_cast<int>(sms), stream);      \
    default:                                                                                     \
      return launch_tc<BNV, DTV, kASmemGather>(tb, ta, p, static_cast<int>(sms), stream);        \
  }
  if (BN == 256) {
    if (dtype == GW_DTYPE_BF16) { GW_TC_MODES(256, GW_DTYPE_BF16) }
    GW_TC_MODES(256, GW_DTYPE_F16)
  } else if (BN == 192) {
    if (dtype == GW_DTYPE_BF16) { GW_TC_MODES(192, GW_DTYPE_BF16) }
    GW_TC_MODES(192, GW_DTYPE_F16)
  } else {
    if (dtype == GW_DTYPE_BF16) { GW_TC_MODES(128, GW_DTYPE_BF16) }
    GW_TC_MODES(128, GW_DTYPE_F16)
  }
#undef GW_TC_MODES
}

}  // namespace gw
