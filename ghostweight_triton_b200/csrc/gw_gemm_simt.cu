// K3-fp32: exact single-precision gather-GEMM on the FP32 pipes (no TF32).
//
// The reference runs fp32 inputs through tl.dot with allow_tf32=False
// (ghostweight_triton/kernels/matmul.py:127-130) so results hold a 1e-4
// tolerance; tcgen05 has no exact-fp32 kind, so fp32 uses FFMA:
//   y[m, n] = act( sum_j x[m, idx[j]] * w[n, j] + bias[n] )
// Tiles of 128 x 128 outputs, k-steps of 8, 256 threads each owning an 8 x 8
// register micro-tile; the A tile is gathered through the index list while it
// is staged into shared memory (k-major), the packed weight tile is read with
// consecutive threads on consecutive k. Double-buffered shared memory, one
// __syncthreads per k-step.
#include "gw_common.cuh"
#include "gw_internal.h"

namespace gw {

namespace {

constexpr int kSBM = 128;
constexpr int kSBN = 128;
constexpr int kSBK = 8;
constexpr int kSThreads = 256;

__global__ void __launch_bounds__(kSThreads)
gemm_f32_kernel(const float* __restrict__ x, int64_t M, int64_t K, int64_t ldx,
                const float* __restrict__ w, int64_t N, int64_t ldw,
                const int64_t* __restrict__ idx, int64_t n_alive,
                const float* __restrict__ bias, int epi, float* __restrict__ y, int64_t ldy,
                unsigned int* err, const int32_t* __restrict__ n_dev) {
  // n_dev: the alive count on the device (n_alive is then an upper bound).
  if (n_dev) n_alive = min(n_alive, static_cast<int64_t>(max(*n_dev, 0)));
  // +4 floats per k-row: conflict-free loader stores, rows stay 16-byte aligned.
  __shared__ __align__(16) float As[2][kSBK][kSBM + 4];
  __shared__ __align__(16) float Bs[2][kSBK][kSBN + 4];

  const int tid = threadIdx.x;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kSBM;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * kSBN;

  // Loader mapping: 128 rows x 8 k per tile = 1024 elements, 4 per thread.
  // Thread t loads k = t % 8 for rows t / 8 + 32 * i (i = 0..3).
  const int lk = tid & 7;
  const int lr = tid >> 3;   // 0..31

  // Compute mapping: 16 x 16 threads, each 8 x 8 outputs (rows ty*4 + {0..3, 64..67}).
  const int tx = tid & 15;
  const int ty = tid >> 4;

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

  const int64_t nk = (n_alive + kSBK - 1) / kSBK;
  bool bad = false;

  auto load_tile = [&](int64_t kt, float (&a_reg)[4], float (&b_reg)[4]) {
    const int64_t kk = kt * kSBK + lk;
    int64_t col = -1;
    if (kk < n_alive) {
      col = __ldg(idx + kk);
      if (col < 0 || col >= K) { bad = true; col = -1; }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t m = m0 + lr + 32 * i;
      a_reg[i] = (m < M && col >= 0) ? __ldg(x + m * ldx + col) : 0.0f;
      const int64_t n = n0 + lr + 32 * i;
      b_reg[i] = (n < N && kk < n_alive) ? __ldg(w + n * ldw + kk) : 0.0f;
    }
  };
  auto store_tile = [&](int buf, const float (&a_reg)[4], const float (&b_reg)[4]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      As[buf][lk][lr + 32 * i] = a_reg[i];
      Bs[buf][lk][lr + 32 * i] = b_reg[i];
    }
  };

  float a_reg[4], b_reg[4];
  if (nk > 0) {
    load_tile(0, a_reg, b_reg);
    store_tile(0, a_reg, b_reg);
  }
  __syncthreads();

  for (int64_t kt = 0; kt < nk; ++kt) {
    const int buf = static_cast<int>(kt & 1);
    const bool more = (kt + 1 < nk);
    if (more) load_tile(kt + 1, a_reg, b_reg);
#pragma unroll
    for (int k = 0; k < kSBK; ++k) {
      float a[8], b[8];
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4 + 64]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * 4 + 64]);
      a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
      a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
      b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
      b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (more) store_tile(buf ^ 1, a_reg, b_reg);
    __syncthreads();
  }
  if (bad) raise_error(err, GW_DERR_BAD_INDEX);

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t m = m0 + ty * 4 + (i & 3) + (i >= 4 ? 64 : 0);
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t n = n0 + tx * 4 + (j & 3) + (j >= 4 ? 64 : 0);
      if (n >= N) continue;
      float v = acc[i][j];
      if (bias) v += __ldg(bias + n);
      y[m * ldy + n] = apply_epilogue(v, epi);
    }
  }
}

}  // namespace

cudaError_t launch_gemm_f32(const float* x, int64_t M, int64_t K, int64_t ldx, const float* w,
                            int64_t N, int64_t ldw, const int64_t* idx, int64_t n_alive,
                            const float* bias, int epilogue, float* y, int64_t ldy,
                            unsigned int* err, cudaStream_t stream, const int32_t* n_dev) {
  if (M == 0 || N == 0) return cudaSuccess;
  const int64_t gx = (N + kSBN - 1) / kSBN;
  const int64_t gy = (M + kSBM - 1) / kSBM;
  if (gx > 0x7FFFFFFFll || gy > 65535) return cudaErrorInvalidValue;
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy));
  gemm_f32_kernel<<<grid, kSThreads, 0, stream>>>(x, M, K, ldx, w, N, ldw, idx, n_alive, bias,
                                                  epilogue, y, ldy, err, n_dev);
  return cudaGetLastError();
}

}  // namespace gw
