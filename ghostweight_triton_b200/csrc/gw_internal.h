// Host-side launchers shared between the kernel translation units and the
// C-ABI layer (gw_api.cu). Not part of the public ABI.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace gw {

// Per-device facts cached by gw_api.cu.
struct DeviceInfo {
  int sm_count = 0;
  int cc_major = 0;
  int cc_minor = 0;
  unsigned int* err_word = nullptr;   // device address of the module error word
};
const DeviceInfo* device_info(int device);   // nullptr on failure
// The current device's info (and, if `device` is not null, its ordinal);
// GW_ERR_DEVICE off sm_100, GW_ERR_CUDA (through cuda_fail) when a runtime
// call fails.
int current_device(const DeviceInfo** out, int* device = nullptr);
// Records `e` as the text gw_last_cuda_error returns, clears the runtime's
// pending error and returns GW_ERR_CUDA.
int cuda_fail(cudaError_t e);

// gw_mask.cu
size_t mask_workspace_bytes(int64_t cols);
cudaError_t launch_mask_compact(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld,
                                float thr, int32_t* mask, int64_t* idx, int32_t* count,
                                void* workspace, int sm_count, cudaStream_t stream);

// gw_gather.cu
// early_dependents: dst is the x' of the GEMM launched right after, which may
// start its prologue before this grid finishes (it waits before reading x').
// Leave it false for anything a later kernel may read before its own wait
// (packed weights, the caller's buffers).
// n_dev (optional): the index count on the device; n_idx and pad_to are then
// upper bounds, and columns [n, round_up(max(n, 1), 64)) are written as zero.
cudaError_t launch_gather_columns(const void* src, int dtype, int64_t rows, int64_t ld_src,
                                  int64_t cols_src, const int64_t* idx, int64_t n_idx, void* dst,
                                  int64_t ld_dst, int64_t pad_to, unsigned int* err,
                                  int sm_count, cudaStream_t stream, bool early_dependents = false,
                                  const int32_t* n_dev = nullptr);
cudaError_t launch_gather_rows(const void* src, int dtype, int64_t rows_src, int64_t cols,
                               int64_t ld_src, const int64_t* idx, int64_t n_idx, void* dst,
                               int64_t ld_dst, unsigned int* err, int sm_count,
                               cudaStream_t stream);
cudaError_t launch_gather_rows_t(const void* src, int dtype, int64_t rows_src, int64_t cols,
                                 int64_t ld_src, const int64_t* idx, int64_t n_idx, void* dst,
                                 int64_t ld_dst, int64_t pad_to, unsigned int* err,
                                 cudaStream_t stream, const int32_t* n_dev = nullptr);
cudaError_t launch_fill_bias(void* y, int dtype, int64_t M, int64_t N, int64_t ldy,
                             const void* bias, int epilogue, cudaStream_t stream);
// Copies y [rows, cols] (leading dimension ld, 16-bit, 16-byte aligned rows)
// into each peer buffer at the same offsets.
cudaError_t launch_copy_to_peers(const void* y, int64_t rows, int64_t cols, int64_t ld,
                                 void* const* peers, int n_peers, int sm_count, cudaStream_t stream);
cudaError_t launch_validate_indices(const int64_t* idx, int64_t n, int64_t K, int32_t* bad,
                                    cudaStream_t stream);
cudaError_t launch_index_runs(const int64_t* idx, int64_t n, int64_t K, int32_t* bad,
                              cudaStream_t stream);

// gw_gemm_tc.cu: tcgen05 gather-GEMM / packed GEMM (fp16, bf16).
// a_mode: 0 -> A is a dense [M, n_alive] matrix loaded by TMA (idx unused)
//         1 -> producer warps gather x[:, idx] into shared memory
// a_mode 0 with a_cols: as launch_gemm_tc2's a_cols (A = x [M, K], k-block kb
// loaded from column a_cols[64 kb], n_alive a multiple of 64). a_mode 0 with
// k_dev: as launch_gemm_tc2's k_dev (n_alive an upper bound).
cudaError_t launch_gemm_tc(int a_mode, const void* x, int dtype, int64_t M, int64_t K,
                           int64_t ldx, const void* w, int64_t N, int64_t ldw,
                           const int64_t* idx, int64_t n_alive, const void* bias, int epilogue,
                           void* y, int64_t ldy, unsigned int* err, int sm_count,
                           cudaStream_t stream, const int64_t* a_cols = nullptr,
                           const int32_t* k_dev = nullptr);

// gw_gemm_tc2.cu: CTA-pair (cta_group::2) tcgen05 GEMM, dense A [M, K] by TMA,
// 256 x 256 tiles per pair. Chained to the previous kernel by programmatic
// dependent launch.
// With n_peers > 0 (at most kMaxPeers; requires y, ldy and every peer buffer
// 16-byte aligned) each finished tile is also stored at the same offset into
// each peer buffer (other GPUs' memory mapped into this process).
constexpr int kMaxPeers = 7;
// With a_cols (alive columns in 64-column runs, each starting at a multiple of
// 8; K = their count, a multiple of 64), A is x [M, a_width] itself and k atom
// kb is loaded from column a_cols[64 kb]: no compacted copy of x is needed.
// With k_dev, K is an upper bound and the kernel reads K' from the device (A
// and W' must be zero in columns [K', round_up(max(K', 1), 64))).
// With gather, the kernel builds A = x[:, idx] itself (K = the alive count):
// its epilogue warps gather x' into gather->xg (leading dimension ldp >= K, a
// multiple of 8) in 128-row x 64-column units published through flags in
// gather->header (tc2_gather_header_bytes(M, K) bytes, 8-byte aligned, any
// contents; see gw_gemm_tc2.cu), while the TMA producer streams finished units.
// Not combined with a_cols or k_dev. tc2_gather_supported says whether the
// unit count fits the header's counters.
struct Tc2Gather {
  const void* x = nullptr;          // [M, K_x], leading dimension ldx
  int64_t ldx = 0;
  int64_t K = 0;                    // columns of x (index bound)
  const int64_t* idx = nullptr;     // alive list, K' entries
  void* xg = nullptr;               // x' [M, ldp]
  int64_t ldp = 0;
  void* header = nullptr;
};
size_t tc2_gather_header_bytes(int64_t M, int64_t n_alive);
bool tc2_gather_supported(int64_t M, int64_t n_alive);
cudaError_t launch_gemm_tc2(const void* a, int dtype, int64_t M, int64_t K, int64_t lda,
                            const void* w, int64_t N, int64_t ldw, const void* bias, int epilogue,
                            void* y, int64_t ldy, unsigned int* err, int sm_count,
                            cudaStream_t stream, void* const* peers = nullptr, int n_peers = 0,
                            const int64_t* a_cols = nullptr, int64_t a_width = 0,
                            const int32_t* k_dev = nullptr, const Tc2Gather* gather = nullptr);
// Whether the CTA-pair kernel serves a dense-A GEMM of this shape.
bool use_pair_gemm(int64_t M, int64_t N, int sm_count);
// Tile width (192 or 256) the pair kernel uses for an M x N output.
int pair_gemm_tile_width(int64_t M, int64_t N, int sm_count);

// gw_gemm_simt.cu: exact-fp32 gather-GEMM.
// n_dev (optional): the alive count on the device, n_alive its upper bound.
cudaError_t launch_gemm_f32(const float* x, int64_t M, int64_t K, int64_t ldx, const float* w,
                            int64_t N, int64_t ldw, const int64_t* idx, int64_t n_alive,
                            const float* bias, int epilogue, float* y, int64_t ldy,
                            unsigned int* err, cudaStream_t stream,
                            const int32_t* n_dev = nullptr);

// gw_gemm_splitk.cu: split-K over a cluster of `split` CTAs reduced in DSMEM,
// for dense-A GEMMs whose output has too few tiles to occupy the SMs.
// a_cols / a_width: as launch_gemm_tc2's.
struct SplitKPlan {
  int bn = 0;            // tile width (32 .. 256)
  int split = 1;         // cluster size; 1 = not worth it (use the persistent kernels)
  int64_t tiles = 0;
};
SplitKPlan plan_splitk(int64_t M, int64_t N, int64_t K, int sm_count);
cudaError_t launch_gemm_splitk(const SplitKPlan& plan, const void* a, int dtype, int64_t M,
                               int64_t K, int64_t lda, const void* w, int64_t N, int64_t ldw,
                               const void* bias, int epilogue, void* y, int64_t ldy,
                               unsigned int* err, cudaStream_t stream,
                               const int64_t* a_cols = nullptr, int64_t a_width = 0);

// gw_gemm_decode.cu: at most 32 rows of A; the MMA runs over 128-feature
// blocks of W' (M = 128) and all rows of A padded to mp (N = 16 or 32),
// split-K over a cluster of `split` CTAs reduced in DSMEM, two CTAs per SM.
struct DecodePlan {
  int mp = 0;            // padded rows of A: 16 or 32
  int split = 1;         // cluster size; 1 = no plan
  int64_t blocks = 0;    // 128-feature blocks of W'
};
DecodePlan plan_decode(int64_t M, int64_t N, int64_t K, int sm_count);
cudaError_t launch_gemm_decode(const DecodePlan& plan, const void* a, int dtype, int64_t M,
                               int64_t K, int64_t lda, const void* w, int64_t N, int64_t ldw,
                               const void* bias, int epilogue, void* y, int64_t ldy,
                               unsigned int* err, cudaStream_t stream,
                               const int64_t* a_cols = nullptr, int64_t a_width = 0);
// Same, with A = x[:, idx] gathered inside the kernel (x [M, K], leading
// dimension ldx; no alignment requirement on x): one launch, no x' in memory.
cudaError_t launch_gemm_decode_gather(const DecodePlan& plan, const void* x, int dtype, int64_t M,
                                      int64_t K, int64_t ldx, const int64_t* idx, int64_t n_alive,
                                      const void* w, int64_t N, int64_t ldw, const void* bias,
                                      int epilogue, void* y, int64_t ldy, unsigned int* err,
                                      cudaStream_t stream);

// gw_gemm_dyn.cu: the per-forward activation mask, its compaction and the
// gather-GEMM in one clustered launch, for at most 32 rows (fp16/bf16; x and
// W rows 16-byte aligned, K a multiple of 8, K <= 8192). count (the alive
// count) and mask (int32 [K]) are optional outputs.
bool dyn_linear_supported(int64_t M, int64_t K);
cudaError_t launch_dyn_linear(const void* x, int dtype, int64_t M, int64_t K, int64_t ldx,
                              const void* w, int64_t N, int64_t ldw, float thr, const void* bias,
                              int epilogue, void* y, int64_t ldy, int32_t* count, int32_t* mask,
                              unsigned int* err, cudaStream_t stream);

// Driver entry point for cuTensorMapEncodeTiled (resolved once, no libcuda link).
void* tensor_map_encoder();
// 2-D tile map over a [rows, cols] 16-bit row-major matrix with row stride ld
// (elements): box = box_cols x box_rows, 128-byte swizzle, zero fill outside.
bool make_tmap_kmajor(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld,
                      int box_cols, int box_rows);

}  // namespace gw
