/*
 * cutex-b200: MXFP8 block-scaled dense GEMM for NVIDIA B200 (sm_100a).
 *
 * C ABI of libcutex_mxfp8.so. Plain pointers and sizes only; every entry
 * point returns a cutex_status code and never throws. Launches are
 * asynchronous on the caller's stream; the caller allocates and owns every
 * buffer, including the output. The GEMM entry points never allocate device
 * memory and never synchronise.
 *
 * Contract (the reference's fixed Fprop contract, generalised in shape):
 *   D[M,N] (bf16, row-major, row stride ldd elements)
 *     = dequant(A[M,K] e4m3, SFA) . dequant(B[N,K] e4m3, SFB)^T
 *   A and B are K-major (row-major [rows, K]); one E8M0 scale per 1x32
 *   K-block; FP32 accumulation; BF16 output with round-to-nearest-even.
 *
 * Scale-factor layout (SM100 128x4 swizzle): the scale of row r and K-block
 * c (= k/32) of an operand with K columns lives at byte
 *     ((r/128)*(K/128) + c/4)*512 + (r%32)*16 + ((r%128)/32)*4 + c%4
 * so SFA holds ceil(M/128)*128*K/32 bytes and SFB ceil(N/128)*128*K/32.
 * Rows past M (resp. N) in the last 128-row block are padding.
 */
#ifndef CUTEX_MXFP8_H_
#define CUTEX_MXFP8_H_

#include <stdint.h>

#if defined(__GNUC__)
#define CUTEX_API __attribute__((visibility("default")))
#else
#define CUTEX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Opaque stream handle; binary-compatible with cudaStream_t / CUstream. */
typedef struct CUstream_st* cutex_stream_t;

typedef enum cutex_status {
  CUTEX_OK = 0,
  CUTEX_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, bad config field */
  CUTEX_ERR_SHAPE = 2,            /* M, N or K outside the supported range */
  CUTEX_ERR_ALIGN = 3,            /* pointer, stride or K alignment rule violated */
  CUTEX_ERR_UNSUPPORTED_DEVICE = 4, /* current device is not compute capability 10.0 */
  CUTEX_ERR_CUDA = 5,             /* a CUDA runtime/driver call failed */
  CUTEX_ERR_TIMEOUT = 6,          /* a device-side bounded wait expired */
  CUTEX_ERR_WORKSPACE = 7,        /* workspace missing or smaller than required */
  CUTEX_ERR_DEVICE_CHECK = 8      /* a device-side consistency check stopped a kernel */
} cutex_status;

/* Kernel families. */
enum {
  CUTEX_KERNEL_AUTO = 0,
  CUTEX_KERNEL_1CTA = 1,   /* persistent, 128 x tile_n per CTA, cta_group::1 MMA */
  CUTEX_KERNEL_2CTA = 2,   /* persistent, 256 x tile_n per CTA pair, cta_group::2 MMA */
  CUTEX_KERNEL_SKINNY = 3  /* M <= 128: swap-AB, split-K over all SMs (needs workspace) */
};

/*
 * Tunables searched by the autotuner. Zero in any field selects the built-in
 * heuristic for that field.
 */
typedef struct cutex_gemm_config {
  int32_t kernel;         /* CUTEX_KERNEL_* */
  int32_t tile_n;         /* 128 or 256 output columns per MMA tile */
  int32_t stages;         /* shared-memory ring depth */
  int32_t raster_group;   /* output tiles per rasterisation group (>= 1; 0 = library choice of the
                             group and of raster_along_n) */
  int32_t raster_along_n; /* 0: walk M inside a group, 1: walk N inside a group (used when
                             raster_group is set) */
  int32_t split_k;        /* skinny kernel: 0 = stream-K over all SMs, 1 = whole tiles,
                             2 = stream-K over all SMs, 3 = whole tiles for the full waves +
                             stream-K remainder */
  int32_t max_ctas;       /* cap on persistent CTAs (0 = one per SM) */
  int32_t epi_buffers;    /* epilogue staging buffers per warp (1 or 2) */
  int32_t sf_buffers;     /* rotating scale-factor TMEM buffers (1, 2 or 4) */
  int32_t scheduler;      /* 0: dynamic (one cluster per tile, idle clusters take over pending
                             ones through cluster launch control); 1: static persistent grid */
  int32_t reserved[6];    /* must be zero */
} cutex_gemm_config;

/* What a launch with this configuration would do (filled by cutex_mxfp8_query). */
typedef struct cutex_gemm_info {
  int32_t kernel;
  int32_t tile_m;          /* output rows per tile (per CTA pair for the 2-CTA kernel) */
  int32_t tile_n;
  int32_t tile_k;
  int32_t stages;
  int32_t cluster_size;
  int32_t grid_ctas;
  int32_t smem_bytes;
  int32_t num_tiles;
  int32_t split_k;
  int32_t epi_buffers;
  int32_t raster_group;
  int32_t sf_buffers;
  int32_t scheduler;
  int64_t workspace_bytes; /* device workspace the GEMM call needs (0 for most shapes) */
} cutex_gemm_info;

/*
 * Fused epilogue of cutex_mxfp8_gemm_ex:
 *   D = alpha * (A . B^T) + beta * C + bias[col]
 * then BF16 (out_dtype 0) or E4M3 with one E8M0 scale per 1x32 block along N
 * (out_dtype 1: the next layer's MXFP8 operand, same rule as
 * cutex_mxfp8_quantize, scales in the 128x4 swizzled layout of an
 * [M, K = N] operand, ceil(M/128)*128*N/32 bytes in d_scales).
 */
typedef struct cutex_epilogue {
  float alpha;            /* 1.0f for none */
  float beta;             /* 0.0f for none (C is then not read) */
  const void* c;          /* bf16 [M, N], row stride ldc elements, 16-byte aligned; may equal d */
  int64_t ldc;            /* ldc >= N, ldc % 8 == 0 */
  const void* bias;       /* bf16 [N], 16-byte aligned, or NULL */
  int32_t out_dtype;      /* 0 = bf16 D, 1 = e4m3 D (ldd in bytes, ldd % 16 == 0) + d_scales; N % 128 == 0 */
  int32_t reserved0;      /* must be 0 */
  void* d_scales;         /* out_dtype 1: 16-byte aligned */
  int64_t reserved[4];    /* must be 0 */
} cutex_epilogue;

/*
 * MXFP8 GEMM, general shape.
 * Replaces the reference's `@cute.jit dense_gemm_vN(a_ptr, b_ptr, sfa_ptr,
 * sfb_ptr, c_ptr[, max_active_clusters], stream)` launch
 * (cutex/kernels/dense_gemm_v13.py:947-956, dense_gemm_v1.py:89-97) with the
 * shape, output stride and tile configuration as runtime arguments.
 *   a, b, d: 16-byte aligned. sfa, sfb: 16-byte aligned.
 *   K % 128 == 0, K >= 128; N % 16 == 0; ldd >= N and ldd % 8 == 0; M >= 1.
 *   workspace: only the M <= 128 (skinny) kernel uses one, for split-K partial
 *   sums and per-tile arrival counters: at least
 *   cutex_mxfp8_query(...)->workspace_bytes, 256-byte aligned, zero-filled once
 *   before its first use (cudaMemsetAsync); every completed call leaves it
 *   ready for the next one, whatever the next call's shape (the layout is fixed
 *   per device and B tiles per CTA tile: 2 * SMs * tiles * 64 KiB of partial
 *   sums, then 4 bytes per CTA tile of N of arrival counters; tile_n 256 on the
 *   skinny kernel is two 128-row tiles). Calls that may overlap on the GPU need separate
 *   workspaces. With the AUTO kernel and no (or a too small) workspace, M <= 128
 *   runs without the split (whole 128-row tiles per CTA); an explicit
 *   CUTEX_KERNEL_SKINNY config without the workspace returns CUTEX_ERR_WORKSPACE.
 */
CUTEX_API int cutex_mxfp8_gemm(const void* a, const void* b, const void* sfa, const void* sfb, void* d,
                     int64_t M, int64_t N, int64_t K, int64_t ldd,
                     const cutex_gemm_config* cfg, void* workspace, int64_t workspace_bytes,
                     cutex_stream_t stream);

/*
 * cutex_mxfp8_gemm with a fused epilogue (epi may be NULL: plain GEMM). The
 * fused builds are the default CTA-pair (N % 256 == 0) and single-CTA kernels;
 * any M (rows beyond M are not written), no skinny kernel. A cfg that names a
 * tile configuration without a fused build returns CUTEX_ERR_INVALID_ARGUMENT.
 * With out_dtype 1, d is e4m3 [M, N] with row stride ldd bytes.
 * No counterpart in the reference (its epilogue is a plain BF16 store,
 * cutex/kernels/dense_gemm_v13.py:811-914; the C-source metadata it carries is
 * unused, dense_gemm_v13.py:1133-1142).
 */
CUTEX_API int cutex_mxfp8_gemm_ex(const void* a, const void* b, const void* sfa, const void* sfb, void* d,
                                  int64_t M, int64_t N, int64_t K, int64_t ldd, const cutex_gemm_config* cfg,
                                  const cutex_epilogue* epi, void* workspace, int64_t workspace_bytes,
                                  cutex_stream_t stream);

/*
 * CUDA IPC for the fused all-gather's peer buffers (one process per GPU).
 * cutex_ipc_export: the 64-byte handle of the device allocation that holds
 * dev_ptr and dev_ptr's byte offset in it. cutex_ipc_import (another process,
 * another GPU of the node): maps that allocation, returns the address of the
 * same byte in *dev_ptr and the mapping to pass to cutex_ipc_close.
 */
CUTEX_API int cutex_ipc_export(const void* dev_ptr, void* handle, int64_t* offset);
CUTEX_API int cutex_ipc_import(const void* handle, int64_t offset, void** dev_ptr, void** mapping);
CUTEX_API int cutex_ipc_close(void* mapping);

/*
 * TMA store descriptors of the peers' copies of D for cutex_mxfp8_gemm_allgather:
 * peer_d[p] = the first element of this rank's region [M, N] (row stride ldd)
 * inside peer p's full D, mapped with cutex_ipc_import (16-byte aligned;
 * num_peers <= 7). Written into map_buffer (device memory, >= 128 * num_peers
 * bytes, 64-byte aligned) on `stream` by a copy from host memory, which waits
 * for the stream: call it once, when the peers are mapped, not per GEMM. The
 * peer stores of later GEMMs stay inside the regions described here.
 */
CUTEX_API int cutex_mxfp8_allgather_maps(const void* const* peer_d, int32_t num_peers, int64_t M, int64_t N,
                                         int64_t ldd, void* map_buffer, int64_t map_buffer_bytes,
                                         cutex_stream_t stream);

/*
 * N-sharded GEMM with the all-gather of D fused into the epilogue: computes
 * this rank's D[:, n0:n0+N] (d points at its first element inside this
 * rank's full D, row stride ldd) and stores every finished 32 x 64 chunk, by
 * TMA from the same shared-memory staging buffer, also into each peer's copy
 * through the num_peers descriptors that cutex_mxfp8_allgather_maps placed in
 * map_buffer, so the gather overlaps the GEMM tile by tile over NVLink. The
 * peers' copies are complete when every rank's call has completed: order
 * readers after a cross-rank barrier on the stream (e.g. a one-element NCCL
 * all-reduce). Kernel choice as cutex_mxfp8_gemm_ex (no skinny kernel).
 * Replaces the GEMM + ncclAllGather + re-layout sequence (one NCCL
 * collective after the kernel, then a permute).
 */
CUTEX_API int cutex_mxfp8_gemm_allgather(const void* a, const void* b, const void* sfa, const void* sfb, void* d,
                                         int64_t M, int64_t N, int64_t K, int64_t ldd, const void* map_buffer,
                                         int32_t num_peers, const cutex_gemm_config* cfg, cutex_stream_t stream);

/*
 * Self-test of the device error path. No counterpart in the reference, whose
 * only protection against a stuck kernel is a host-side timeout.
 * Runs the GEMM D[M,N] (row stride N) on a build of the single-CTA, static
 * kernel whose bounded waits give up after 1 ms (2 s in every other build)
 * and whose TMA producer issues no copies for each CTA's K-stage number
 * withhold_stage (0 <= withhold_stage < K/128; its first tile). The MMA issuer
 * then waits for data that never arrives while nothing is in flight for that
 * stage; every role times out in turn, lets its in-flight copies land, frees
 * TMEM and exits. Afterwards cutex_last_device_status(stream) must return
 * CUTEX_ERR_TIMEOUT (and clears the word); D is left unwritten, and the device
 * stays usable for later launches.
 */
CUTEX_API int cutex_mxfp8_selftest_wait_timeout(const void* a, const void* b, const void* sfa, const void* sfb,
                                                void* d, int64_t M, int64_t N, int64_t K, int32_t withhold_stage,
                                                cutex_stream_t stream);

/*
 * Resolve a configuration for a shape without launching anything.
 * Replaces the host-side resource accounting of dense_gemm_v13
 * (cutex/kernels/dense_gemm_v13.py:1095-1239: SMEM layouts, tma_bytes, grid).
 */
CUTEX_API int cutex_mxfp8_query(const cutex_gemm_config* cfg, int64_t M, int64_t N, int64_t K,
                      cutex_gemm_info* info);

/*
 * Diagnostics: the same GEMM on an instrumented build of the kernel that
 * records per-role %globaltimer events of the first CTA (pair) into `trace`
 * (caller-allocated, 8-byte aligned, 6 * (trace_cap + 1) * 2 + 4 * grid_ctas
 * uint64 values, grid_ctas from cutex_mxfp8_query: regions [cta_rank * 3 +
 * role], role 0 = TMA producer, 1 = MMA issuer, 2 = epilogue warp 0; record 0
 * of a region = event count, record i = {time_ns, event << 56 | tile << 24 |
 * k_block}; then {start_ns, end_ns} of every CTA, then {start, end} of every
 * CTA's SM cycle counter). Only configurations with an
 * instrumented twin are accepted (CUTEX_ERR_INVALID_ARGUMENT otherwise).
 * Replaces the reference's IKET in-kernel ranges (cutex/trace.py:96-175,
 * cutex/kernels/dense_gemm_v9.py:116-125); benchmark builds carry no tracing.
 */
CUTEX_API int cutex_mxfp8_gemm_trace(const void* a, const void* b, const void* sfa, const void* sfb,
                                     void* d, int64_t M, int64_t N, int64_t K, int64_t ldd,
                                     const cutex_gemm_config* cfg, unsigned long long* trace,
                                     int32_t trace_cap, cutex_stream_t stream);

/*
 * The reference's fixed-shape entry: M = N = K = 16384, D row stride 16384,
 * 2-CTA persistent kernel with at most `max_active_clusters` CTA pairs
 * (<= 0: as many as fit). Mirrors `dense_gemm_v13(a_ptr, b_ptr, sfa_ptr,
 * sfb_ptr, c_ptr, max_active_clusters, stream)`
 * (cutex/kernels/dense_gemm_v13.py:947-956).
 */
CUTEX_API int cutex_dense_gemm_v13(const void* a, const void* b, const void* sfa, const void* sfb, void* c,
                         int32_t max_active_clusters, cutex_stream_t stream);

/*
 * MXFP8 quantiser (OCP MX, E4M3 elements, E8M0 scales): for each 1x32 block
 * of x[rows, K] (row stride ldx elements) the scale exponent is
 * floor(log2(amax)) - 8 clamped to [-127, 127] (all-zero block -> 0x00),
 * elements are x / 2^e rounded to nearest-even and saturated to +-448.
 * Writes q[rows, K] (row stride K bytes) and scales in the 128x4 swizzled
 * layout (ceil(rows/128)*128*K/32 bytes; padding rows are written as 0x00).
 * x_dtype: 0 = float32, 1 = bfloat16. K % 128 == 0.
 * Replaces Transformer Engine's MXFP8Quantizer(rowwise=True,
 * optimize_for_gemm=True) call in the reference runner
 * (modal_dense_gemm.py:358-373).
 */
CUTEX_API int cutex_mxfp8_quantize(const void* x, int32_t x_dtype, int64_t rows, int64_t K, int64_t ldx,
                         void* q, void* sf, cutex_stream_t stream);

/*
 * Columnwise MXFP8 quantiser: for x[rows, cols] (row stride ldx elements)
 * writes qt[cols, rows] = quantise(x^T) (row stride rows bytes) with the same
 * per-block rule as cutex_mxfp8_quantize, the 1x32 blocks running down the
 * columns of x, and the scales in the 128x4 swizzled layout of a [cols, K =
 * rows] operand (ceil(cols/128)*128*rows/32 bytes; padding rows 0x00). qt is
 * the K-major operand of a GEMM that reduces over the rows of x: weight
 * gradients (dW = dY^T X from columnwise dY and X) and input gradients
 * (dX = dY W from rowwise dY and columnwise W). x_dtype: 0 = float32,
 * 1 = bfloat16. rows % 128 == 0, ldx % 8 == 0, ldx >= cols.
 * Replaces Transformer Engine's MXFP8Quantizer(columnwise=True) data for the
 * Dgrad/Wgrad layouts (no GEMM in the reference consumes them; its contract is
 * rowwise Fprop only, cutex/kernels/dense_gemm_contract.py:16-22).
 */
CUTEX_API int cutex_mxfp8_quantize_columnwise(const void* x, int32_t x_dtype, int64_t rows, int64_t cols,
                                              int64_t ldx, void* qt, void* sft, cutex_stream_t stream);

/*
 * MXFP8 GEMM for M <= 128 that allocates nothing and takes no workspace.
 * No counterpart in the reference. For callers that cannot call cudaMalloc at
 * launch time (memory-capped pools, allocators that forbid out-of-band
 * allocations, plugins handed only their operand and output buffers): the
 * split-K skinny kernel runs with its scratch in a fixed device array owned by
 * the library (20 MiB of partial sums + 64 KiB of counters, held on every GPU
 * where the library is loaded until the process exits). Same operands, layout
 * rules and result as cutex_mxfp8_gemm with the split-K skinny kernel.
 *   M <= 128 (else CUTEX_ERR_SHAPE); N <= 2,097,152 and at most 160 SMs (else
 *   CUTEX_ERR_WORKSPACE). The first call on a device performs one-time set-up
 *   (it looks up the scratch array's device address); make that first call
 *   before any stream capture. The set-up is repeated, by the next call, when
 *   the device's CUDA context has changed since (a device reset). Every call
 *   shares the one scratch array: calls that may overlap on the GPU (different
 *   streams, or different host threads) race and must be serialised by the
 *   caller.
 */
CUTEX_API int cutex_mxfp8_gemm_skinny_static(const void* a, const void* b, const void* sfa,
                                             const void* sfb, void* d, int64_t M, int64_t N,
                                             int64_t K, int64_t ldd, cutex_stream_t stream);

/*
 * The GEMM from host buffers to a host buffer: copies the operands to the
 * caller's device buffers, runs the GEMM and copies D back, overlapped. The
 * output is cut into up to blocks x blocks rectangles (rows and columns
 * multiples of 256). The operand row panels are copied in a growing-square
 * order (A panel s and B panel s, then every block whose larger index is s), so
 * each block's GEMM starts as soon as its two panels have landed. Each finished
 * block's D2H copy overlaps the remaining host-to-device copies.
 *
 * Host buffers: a_host [M, K] e4m3, b_host [N, K], sfa_host / sfb_host in the
 * swizzled 128x4 layout (ceil(rows/128)*128*K/32 bytes), d_host [M, N] bf16
 * (row pitch N). Use pinned (page-locked) host memory for the copies to
 * overlap. Device buffers: the same sizes, 16-byte aligned, contents
 * overwritten. `workspace` is passed to every block GEMM (only blocks with
 * M <= 128 can use one). Ordering: starts after prior work on `stream`; work
 * enqueued on `stream` afterwards runs after D has reached d_host. The copies
 * and block GEMMs run on library-owned streams of the current device. Calls
 * that share those streams are serialised.
 * No reference counterpart: the reference always starts from device-resident
 * TE tensors (cutex/kernels/modal_dense_gemm.py:375-406).
 */
CUTEX_API int cutex_mxfp8_gemm_host(const void* a_host, const void* b_host, const void* sfa_host,
                                    const void* sfb_host, void* d_host, void* a_dev, void* b_dev,
                                    void* sfa_dev, void* sfb_dev, void* d_dev, int64_t M, int64_t N,
                                    int64_t K, const cutex_gemm_config* cfg, int32_t blocks,
                                    void* workspace, int64_t workspace_bytes, cutex_stream_t stream);

/* Human-readable text for a cutex_status value (static storage). */
CUTEX_API const char* cutex_status_string(int status);

/*
 * Synchronise `stream`, return the first device-side error recorded by a
 * kernel of this library on the current device since the last call
 * (CUTEX_OK, CUTEX_ERR_TIMEOUT or CUTEX_ERR_DEVICE_CHECK), and clear it.
 */
CUTEX_API int cutex_last_device_status(cutex_stream_t stream);

/*
 * Checked builds (libcutex_mxfp8_checked.so, compiled with -DCUTEX_CHECKED):
 * every kernel also checks the indices it derives before it uses them (GEMM
 * tile coordinates, TMEM column ranges, store origins inside D's padded extent,
 * scale and code offsets, the skinny kernel's segments and workspace slots, the
 * columnwise quantiser's tiles). A failed check faults nothing: the access is
 * skipped, the kernel's roles leave their loops (the others stop at their
 * bounded waits), and the status word reads CUTEX_ERR_DEVICE_CHECK. It stands
 * in for an external memory checker such as compute-sanitizer's memcheck. The
 * reference has no counterpart.
 *
 * cutex_build_checked: 1 for a checked build, 0 otherwise.
 * cutex_device_check_record: synchronise `stream`, then read and clear the site
 *   code (0x211-0x21F; 0 when no check failed) and the offending value of the
 *   check that set the status word. The status word itself is read and cleared
 *   by cutex_last_device_status.
 * cutex_selftest_device_check: checked builds only (else
 *   CUTEX_ERR_INVALID_ARGUMENT): launch one warp in which lane 7 fails a check
 *   with value 0x5EED07 (site 0x21F), touching no memory but the status word and
 *   the record.
 */
CUTEX_API int cutex_build_checked(void);
CUTEX_API int cutex_device_check_record(cutex_stream_t stream, int32_t* site, int64_t* value);
CUTEX_API int cutex_selftest_device_check(cutex_stream_t stream);

/* Number of SMs and the library's build identifier (for autotune cache keys). */
CUTEX_API int cutex_device_sm_count(int32_t* sm_count);
CUTEX_API const char* cutex_version(void);

#ifdef __cplusplus
}
#endif

#endif /* CUTEX_MXFP8_H_ */
