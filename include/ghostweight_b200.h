/*
 * ghostweight_b200.h -- C ABI of the B200 (sm_100a) column-sparse linear hot path.
 *
 * The library (ghostweight_triton_b200/libghostweight_b200.so) replaces the
 * Triton kernels of ghostweight-triton (ghostweight_triton/kernels/*.py) with
 * hand-written CUDA for sm_100a. Every entry point:
 *   - takes caller-allocated DEVICE pointers, plain sizes and leading
 *     dimensions (in elements), and a cudaStream_t passed as void*;
 *   - never allocates device memory and never synchronises the stream;
 *   - returns a gw_status (0 = success) after validating shapes, dtypes,
 *     alignment and the launch; no torch types cross this boundary.
 * Matrices are row-major: element (r, c) of a matrix with leading dimension
 * ld lives at base[r * ld + c].
 *
 * Index lists ("alive indices") are int64, as the reference passes them
 * (ghostweight_triton/kernels/matmul.py:120, gather.py:128). An index outside
 * [0, K) is read as a zero column (never dereferenced) and raises
 * GW_DEVICE_ERR_BAD_INDEX in the device error word.
 */
#ifndef GHOSTWEIGHT_B200_H
#define GHOSTWEIGHT_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define GW_API __attribute__((visibility("default")))
#else
#define GW_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element types. The reference accepts fp16 and fp32 (tests/conftest.py:101); bf16 is added. */
typedef enum {
  GW_DTYPE_F16 = 0,
  GW_DTYPE_BF16 = 1,
  GW_DTYPE_F32 = 2
} gw_dtype;

/* Fused GEMM epilogue activation (applied after the bias add). */
typedef enum {
  GW_EPI_NONE = 0,
  GW_EPI_GELU_ERF = 1,  /* torch.nn.GELU() / F.gelu(approximate="none") */
  GW_EPI_GELU_TANH = 2  /* F.gelu(approximate="tanh"), GPT-2's gelu_new */
} gw_epilogue;

typedef enum {
  GW_OK = 0,
  GW_ERR_SHAPE = 1,       /* negative / inconsistent sizes or leading dimensions */
  GW_ERR_DTYPE = 2,       /* unsupported dtype for this entry point */
  GW_ERR_ALIGN = 3,       /* pointer or leading dimension misaligned for the kernel */
  GW_ERR_NULL = 4,        /* required pointer is NULL */
  GW_ERR_WORKSPACE = 5,   /* workspace missing or too small */
  GW_ERR_CUDA = 6,        /* a CUDA runtime call or launch failed */
  GW_ERR_DEVICE = 7,      /* current device is not sm_100 (B200) */
  GW_ERR_UNSUPPORTED = 8  /* valid request this build does not implement */
} gw_status;

/* Bits of the device error word (gw_get_device_error). */
#define GW_DEVICE_ERR_WAIT_TIMEOUT 1u
#define GW_DEVICE_ERR_BAD_INDEX 2u

/* Human-readable text for a gw_status value. */
GW_API const char* gw_status_string(int status);

/* Text of the last CUDA error seen by this library on the calling thread. */
GW_API const char* gw_last_cuda_error(void);

/* Library version, e.g. "0.1.0". */
GW_API const char* gw_version(void);

/* 1 if `device` is an sm_100 part this library can launch on, else 0. */
GW_API int gw_device_supported(int device);

/*
 * Reads (and, if reset != 0, clears) the device error word of the current
 * device. Synchronises the device. *out receives GW_DEVICE_ERR_* bits.
 */
GW_API int gw_get_device_error(int reset, unsigned int* out);

/*
 * Dead-column mask fused with stream compaction.
 *
 * Replaces ghostweight_triton/kernels/mask.py:62-104 (dead_neuron_mask,
 * kernel mask.py:21-59) together with the torch.nonzero compaction that
 * follows it at ghostweight_triton/module.py:104 and module.py:129-131.
 *
 * For an [rows, cols] matrix x:
 *   colmax[k]  = max(0, max_r fp32(|x[r, k]|)), NaN entries ignored
 *   mask[k]    = colmax[k] > fp32(threshold) ? 1 : 0           (int32, [cols])
 *   alive_idx  = ascending k with mask[k] == 1                 (int64, [cols] capacity)
 *   *alive_count = number of alive columns                      (int32, device)
 * Applied to an activation [M, K] it is the reference's activation mask; applied
 * to nn.Linear.weight [N, K] it is the per-input-column |W| mask.
 * mask, alive_idx and alive_count may each be NULL if not wanted.
 *
 * workspace: at least gw_mask_workspace_bytes(cols) bytes of device memory that
 * must be all-zero before the first call; every call leaves it all-zero again.
 * Calls sharing one workspace must be ordered on one stream.
 */
GW_API size_t gw_mask_workspace_bytes(int64_t cols);
GW_API int gw_mask_compact(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld,
                           double threshold, int32_t* mask, int64_t* alive_idx,
                           int32_t* alive_count, void* workspace, size_t workspace_bytes,
                           void* stream);

/*
 * Allocation-free variant of gw_mask_compact. It has no counterpart in the
 * reference, which allocates its outputs with torch on every call.
 *
 * For callers that must not allocate device memory after start-up: servers
 * that reserve all device memory in advance and count any later cudaMalloc as
 * a failure, plugins whose host process owns every allocation, and code that
 * runs inside an allocator callback. Same inputs, outputs and semantics as
 * gw_mask_compact, but the scratch lives in a static device array inside the
 * library (about 128 KiB per GPU that loads it, held until the process exits),
 * so no workspace argument is needed and nothing is allocated.
 *
 * Limits and rules:
 *   - cols must be <= GW_MASK_STATIC_MAX_COLS, otherwise GW_ERR_WORKSPACE is
 *     returned and nothing is launched;
 *   - the first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before any stream capture;
 *   - every call on a device shares the one array and clears the part it uses
 *     (cudaMemsetAsync) before launching, so calls that overlap on the GPU
 *     (different streams, no ordering between them) race: order them on one
 *     stream or use gw_mask_compact with separate workspaces.
 */
#define GW_MASK_STATIC_MAX_COLS 1048576
GW_API int gw_mask_compact_static(const void* x, int dtype, int64_t rows, int64_t cols,
                                  int64_t ld, double threshold, int32_t* mask,
                                  int64_t* alive_idx, int32_t* alive_count, void* stream);

/*
 * Column gather: dst[r, j] = src[r, idx[j]] for j < n_idx, and dst[r, j] = 0
 * for n_idx <= j < pad_to (pad_to <= ld_dst; pass pad_to = n_idx for no padding).
 *
 * Replaces the activation side of gather_compact, ghostweight_triton/kernels/
 * gather.py:19-55 (_gather_columns_kernel) and :139-146. With src =
 * nn.Linear.weight [N, K] it is the one-time weight compaction that packs
 * W[:, alive] into the K'-major operand layout of gw_gather_gemm.
 */
GW_API int gw_gather_columns(const void* src, int dtype, int64_t rows, int64_t cols,
                             int64_t ld_src, const int64_t* idx, int64_t n_idx, void* dst,
                             int64_t ld_dst, int64_t pad_to, void* stream);

/*
 * Row gather: dst[j, :] = src[idx[j], :] for j < n_idx.
 *
 * Replaces the weight side of gather_compact, ghostweight_triton/kernels/
 * gather.py:58-94 (_gather_rows_kernel) and :149-156.
 */
GW_API int gw_gather_rows(const void* src, int dtype, int64_t rows, int64_t cols, int64_t ld_src,
                          const int64_t* idx, int64_t n_idx, void* dst, int64_t ld_dst,
                          void* stream);

/*
 * Transposing row gather: dst[n, j] = src[idx[j], n] for n < cols, j < n_idx;
 * dst[n, j] = 0 for n_idx <= j < pad_to.
 *
 * Packs a reference-orientation weight W [K, N] (the `weights` argument of
 * ghostweight_triton/kernels/matmul.py:85-92, i.e. linear.weight.t() from
 * module.py:97, or a transformers Conv1D weight) into the [N, K'] K'-major
 * operand of gw_gather_gemm. It replaces the W-row gather done inside the
 * reference's matmul loop (matmul.py:66-72).
 */
GW_API int gw_gather_rows_t(const void* src, int dtype, int64_t rows, int64_t cols,
                            int64_t ld_src, const int64_t* idx, int64_t n_idx, void* dst,
                            int64_t ld_dst, int64_t pad_to, void* stream);

/*
 * Fused gather-GEMM:
 *   y[m, n] = act( sum_{j < n_alive} x[m, idx[j]] * w_packed[n, j] + bias[n] )
 * x: [M, K] (ldx), w_packed: [N, >= n_alive] K'-major (ldw), bias: [N] or NULL,
 * y: [M, N] (ldy). fp32 accumulation; output rounded once to the input dtype.
 * idx may be in any order and contain repeats. n_alive == 0 gives act(bias)
 * (zeros without bias).
 *
 * Replaces ghostweight_triton/kernels/matmul.py:85-142 (ghostweight_matmul,
 * kernel matmul.py:27-82) plus the separate bias add at module.py:116-117.
 * fp16/bf16 run on tcgen05 tensor cores (requires ldw % 8 == 0 and a 16-byte
 * aligned w_packed); fp32 runs an exact-fp32 FFMA kernel (no TF32), as the
 * reference disables TF32 for fp32 (matmul.py:127-130).
 *
 * strategy (fp16/bf16 only):
 *   GW_GEMM_AUTO      for M <= 4 the decode kernel with the gather inside (one
 *                     launch, no workspace); otherwise GW_GEMM_PREGATHER when a
 *                     large-enough workspace is given, else fused;
 *   GW_GEMM_FUSED     one kernel: warps gather x[:, idx] into shared memory (for
 *                     M <= 4 the decode kernel's gather, as with AUTO);
 *   GW_GEMM_PREGATHER two launches: x[:, idx] -> workspace (dense [M, K'_pad]),
 *                     then the GEMM with both operands loaded by TMA;
 *   GW_GEMM_OVERLAP   one launch where the shape runs on the CTA-pair kernel: its
 *                     epilogue warps gather x[:, idx] into the workspace in
 *                     128-row x 64-column units (before their first epilogue)
 *                     while the TMA/MMA warps already consume the finished
 *                     units; other shapes run GW_GEMM_PREGATHER;
 *   GW_GEMM_RUNS      for alive lists made of 64-column runs (a mask that kills
 *                     whole 64- or 128-column blocks): idx[64 j + r] = idx[64 j] + r
 *                     for r < 64, idx[64 j] a multiple of 8, n_alive a multiple
 *                     of 64. One GEMM launch, no gather and no workspace: each
 *                     64-column block of x is loaded straight from x by TMA.
 *                     Requires x 16-byte aligned and ldx % 8 == 0; n_alive % 64
 *                     != 0 returns GW_ERR_UNSUPPORTED. The kernel checks only the
 *                     run starts (a bad one sets GW_DERR_BAD_INDEX and yields a
 *                     wrong result); gw_index_runs checks the whole list once.
 * workspace: device scratch of at least gw_gather_gemm_workspace_bytes(M, n_alive,
 * dtype) bytes, 16-byte aligned (may be NULL for GW_GEMM_FUSED, GW_GEMM_RUNS and
 * fp32): a header (the overlap strategy's unit flags, tagged with a call number
 * the header also keeps) and x'. Its contents on entry do not matter; calls
 * that use one workspace must be ordered on one stream.
 *
 * Weights are read early: the GEMMs are launched as programmatic dependents
 * of the previous kernel on the stream, and for M <= 64 the kernel requests
 * its first tiles of w_packed before waiting for that kernel. w_packed must
 * therefore not be the output of the immediately preceding GEMM call of this
 * library on the stream (such kernels let their successor start early). Any
 * other producer is safe: this library's packing and gather entry points, and
 * kernels launched without programmatic completion triggers, finish before
 * the GEMM starts.
 */
typedef enum {
  GW_GEMM_AUTO = 0,
  GW_GEMM_FUSED = 1,
  GW_GEMM_PREGATHER = 2,
  GW_GEMM_OVERLAP = 3,
  GW_GEMM_RUNS = 4
} gw_gemm_strategy;

GW_API size_t gw_gather_gemm_workspace_bytes(int64_t M, int64_t n_alive, int dtype);
GW_API int gw_gather_gemm(const void* x, int dtype, int64_t M, int64_t K, int64_t ldx,
                          const void* w_packed, int64_t N, int64_t ldw, const int64_t* idx,
                          int64_t n_alive, const void* bias, int epilogue, void* y, int64_t ldy,
                          int strategy, void* workspace, size_t workspace_bytes, void* stream);

/*
 * gw_gather_gemm (pregather strategy, fp16/bf16) whose output also lands in
 * other GPUs' memory: the M x N block written to y (leading dimension ldy) is
 * written, at the same offsets, into each peer_y[i] -- device addresses valid
 * in this process (e.g. opened CUDA IPC handles of the other ranks' output
 * buffers), same leading dimension. This is the all-gather of a
 * column-parallel layer fused into the GEMM: each rank passes its block of the
 * full [M, N_total] output (y = full + column offset) and the same block of
 * every peer's full output. Where the shape runs on the CTA-pair kernel the
 * peer stores are issued from its epilogue tile by tile (over NVLink, plain
 * stores, no multicast); otherwise a copy kernel follows the GEMM.
 * Requires y, ldy and every peer_y 16-byte aligned and at most GW_MAX_PEERS
 * peers. strategy: GW_GEMM_AUTO or GW_GEMM_PREGATHER (gather into the
 * workspace, sized as for gw_gather_gemm, then the GEMM) or GW_GEMM_RUNS (no
 * gather, no workspace; the conditions of gw_gather_gemm apply); others return
 * GW_ERR_UNSUPPORTED. No synchronisation between GPUs is
 * done here: the caller orders the peers' readers after every rank's call
 * (e.g. a collective on each stream) and must not let a peer overwrite a
 * buffer that is still being read.
 * Replaces the NCCL all-gather after the column-parallel GEMM
 * (ghostweight_triton_b200/sharded.py); no counterpart in the reference.
 */
#define GW_MAX_PEERS 7
GW_API int gw_gather_gemm_peers(const void* x, int dtype, int64_t M, int64_t K, int64_t ldx,
                                const void* w_packed, int64_t N, int64_t ldw, const int64_t* idx,
                                int64_t n_alive, const void* bias, int epilogue, void* y,
                                int64_t ldy, void* const* peer_y, int n_peers, int strategy,
                                void* workspace, size_t workspace_bytes, void* stream);

/*
 * Device-count variants, for the dynamic (per-forward) activation mask without
 * a host synchronisation: the number of valid entries of idx is read from
 * device memory (n_*_dev, an int32, e.g. gw_mask_compact's alive_count), so the
 * mask, the packing, the gather and the GEMM are queued back to back. The
 * reference reads that count on the host (torch.nonzero at
 * ghostweight_triton/module.py:103-108). n_*_max is an upper bound (K); buffers
 * are sized for it.
 *
 * gw_gather_columns_dev / gw_gather_rows_t_dev: as gw_gather_columns /
 * gw_gather_rows_t with n = *n_idx_dev (clamped to [0, n_idx_max]); columns
 * [n, round_up(max(n, 1), 64)) of dst are written as zero, columns past that
 * (up to pad_to) are left as they are.
 *
 * gw_gather_gemm_dev: gw_gather_gemm (fp16/bf16: gather into the workspace,
 * sized by gw_gather_gemm_workspace_bytes(M, n_alive_max, dtype), then the
 * tcgen05 GEMM; fp32: the exact-fp32 kernel) with K' = *n_alive_dev. For
 * fp16/bf16, w_packed must be zero in columns [K', round_up(max(K', 1), 64))
 * (as gw_gather_columns_dev / gw_gather_rows_t_dev with pad_to = ldw leave it)
 * and ldw >= round_up(n_alive_max, 64). K' = 0 gives act(bias).
 */
GW_API int gw_gather_columns_dev(const void* src, int dtype, int64_t rows, int64_t cols,
                                 int64_t ld_src, const int64_t* idx, int64_t n_idx_max,
                                 const int32_t* n_idx_dev, void* dst, int64_t ld_dst,
                                 int64_t pad_to, void* stream);
GW_API int gw_gather_rows_t_dev(const void* src, int dtype, int64_t rows, int64_t cols,
                                int64_t ld_src, const int64_t* idx, int64_t n_idx_max,
                                const int32_t* n_idx_dev, void* dst, int64_t ld_dst,
                                int64_t pad_to, void* stream);
GW_API int gw_gather_gemm_dev(const void* x, int dtype, int64_t M, int64_t K, int64_t ldx,
                              const void* w_packed, int64_t N, int64_t ldw, const int64_t* idx,
                              int64_t n_alive_max, const int32_t* n_alive_dev, const void* bias,
                              int epilogue, void* y, int64_t ldy, void* workspace,
                              size_t workspace_bytes, void* stream);

/*
 * The dynamic-mask layer in one launch, for at most 32 rows (decoding and
 * small batches):
 *   alive[k] = max(0, max_m fp32(|x[m, k]|)) > fp32(threshold)    (NaN ignored)
 *   y[m, n]  = act( sum_{alive k} x[m, k] * w[n, k] + bias[n] )
 * x [M, K] (ldx), w = nn.Linear.weight [N, K] (ldw), bias [N] or NULL, y [M, N]
 * (ldy); fp16 or bf16 with fp32 accumulation and one rounding. alive_count
 * (int32, device) and mask (int32 [K], 1 = alive) are optional outputs.
 *
 * Replaces the dynamic forward of ghostweight_triton/module.py:103-117
 * (dead_neuron_mask, torch.nonzero, ghostweight_matmul and the bias add): one
 * launch that reads x and w once, no index list in memory, no host
 * synchronisation. The k range is split over the original columns across a
 * cluster of CTAs, each of which masks, compacts and multiplies its own
 * columns; partial sums are reduced in distributed shared memory.
 * Requires 1 <= M <= 32, K a multiple of 8 and at most 8192, x and w 16-byte
 * aligned, ldx and ldw multiples of 8; other requests return
 * GW_ERR_UNSUPPORTED (gw_mask_compact with the *_dev entry points covers them).
 */
GW_API int gw_dynamic_linear(const void* x, int dtype, int64_t M, int64_t K, int64_t ldx,
                             const void* w, int64_t N, int64_t ldw, double threshold,
                             const void* bias, int epilogue, void* y, int64_t ldy,
                             int32_t* alive_count, int32_t* mask, void* stream);

/*
 * Dense GEMM over an already-compacted activation (the two-step path of
 * gather.py:1-14: gather_compact followed by a matmul):
 *   y[m, n] = act( sum_{j < K} a[m, j] * w_packed[n, j] + bias[n] )
 * fp16/bf16 only; both operands arrive by TMA (requires 16-byte aligned bases
 * and lda, ldw multiples of 8).
 */
GW_API int gw_packed_gemm(const void* a, int dtype, int64_t M, int64_t K, int64_t lda,
                          const void* w_packed, int64_t N, int64_t ldw, const void* bias,
                          int epilogue, void* y, int64_t ldy, void* stream);

/*
 * Counts indices outside [0, K) into *bad_count (int32, device, overwritten).
 * Debug helper for callers that want the reference's implicit "indices are
 * valid" contract checked (kernels/matmul.py:120 performs no check).
 */
GW_API int gw_validate_indices(const int64_t* idx, int64_t n, int64_t K, int32_t* bad_count,
                               void* stream);

/*
 * Counts the entries of idx[0, n) that break the structure GW_GEMM_RUNS needs
 * into *bad_count (int32, device, overwritten): idx[64 j + r] == idx[64 j] + r,
 * idx[64 j] % 8 == 0, every entry in [0, K), n a multiple of 64 (entries of a
 * trailing partial run count). 0 means gw_gather_gemm may use GW_GEMM_RUNS with
 * this list. No counterpart in the reference, whose gather-GEMM always reads
 * x through idx (kernels/matmul.py:55-63).
 */
GW_API int gw_index_runs(const int64_t* idx, int64_t n, int64_t K, int32_t* bad_count,
                         void* stream);

/*
 * Self-test of the bounded waits every kernel of this library relies on. One
 * thread of one CTA waits on an mbarrier that nothing arrives on, then on a
 * device counter that nothing increments, each with a wall-clock limit of
 * limit_ns (clamped to [1e5, 1e9] ns) instead of the kernels' 2 s. Both waits
 * give up, raise GW_DEVICE_ERR_WAIT_TIMEOUT in the device error word and the
 * kernel returns normally; read the word with gw_get_device_error. For tests of
 * the give-up path (no GPU fault, no hang); the reference has no device waits.
 */
GW_API int gw_selftest_wait_timeout(int64_t limit_ns, void* stream);

/* GEMM kernels (gw_gemm_plan). */
typedef enum {
  GW_KERNEL_PAIR = 1,    /* CTA pairs, 256-row tiles *tile_n columns wide (192 or 256) */
  GW_KERNEL_DECODE = 2,  /* at most 32 rows: output features on the MMA's M side, clusters of *split */
  GW_KERNEL_SPLITK = 3,  /* 128 x *tile_n tiles, k split over clusters of *split CTAs */
  GW_KERNEL_SINGLE = 4   /* persistent single-CTA kernel, 128-row tiles */
} gw_kernel;

/*
 * The kernel gw_packed_gemm runs for an M x N output over K columns on the
 * current device (also gw_gather_gemm's GEMM after its gather, and its runs
 * strategy): *kernel one of gw_kernel, *tile_n the tile width and *split the
 * cluster size where the kernel has them, else 0. tile_n and split may be
 * NULL. For callers that size batches by it and for tests of the dispatch; the
 * reference has one Triton kernel whose launch grid follows from the block
 * sizes (kernels/matmul.py:105-121).
 */
GW_API int gw_gemm_plan(int64_t M, int64_t N, int64_t K, int* kernel, int* tile_n, int* split);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* GHOSTWEIGHT_B200_H */
