/*
 * sc_b200.h — C ABI of the B200-native enumerate + sparse-coarsen SpMM/SpMV library.
 *
 * Every entry point returns an int status (SC_OK == 0) and never throws or exits;
 * on failure sc_last_error_string() holds a one-line reason (thread-local).
 * Handles are opaque.  No CUDA or torch types appear in the signatures: device
 * buffers are plain pointers, streams are passed as void* (a cudaStream_t).
 *
 * Reference interfaces each group replaces (paths relative to the
 * hosseinal/sparse-computation tree):
 *   .mtx reading          utils/Sparse_io.cpp:48-82 (readCSRMatrixFromMTX) and
 *                         aggregation/utils/sparse_io.cpp:278-402 (sym_lib)
 *   .cfmtx reading        utils/Sparse_io.cpp:84-181 (readCFMTXFile),
 *                         utils/Sparse_io.cpp:186-196 (loadCfmtxMatrices)
 *   companion path        utils/Sparse_io.cpp:28-46 (companionMtxPathFromCFMTX)
 *   enumerate + coarsen   code_gen/ss_format/format_generator.py:36-129
 *   .cfmtx writing        code_gen/ss_format/format_generator.py:132-160
 *   pattern dictionary    code_gen/pattern_utiles/pattern_dictionary.py:29-60
 *   device upload         example_cuda/spmm_demo_gpu_utils.h:38-67,207-245
 *   large-B SpMM launch   example_cuda/spmm_demo_gpu_utils.h:1357-1712
 *   small-B SpMM launch   example_cuda/spmm_small_b_col_demo_gpu_utils.h:1061-2986,4911-5064
 *   SpMV launch           example_cuda/spmv_demo_gpu_utils.h:632-952
 */
#ifndef SC_B200_H
#define SC_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SC_OK 0
#define SC_ERR_ARG 1         /* bad argument (null pointer, size out of range) */
#define SC_ERR_IO 2          /* file cannot be opened / read / written */
#define SC_ERR_FORMAT 3      /* malformed .mtx / .cfmtx / dictionary content */
#define SC_ERR_CUDA 4        /* a CUDA runtime call failed */
#define SC_ERR_UNSUPPORTED 5 /* valid input outside what this build handles */
#define SC_ERR_NOMEM 6       /* host allocation failed */
#define SC_ERR_DEVICE 7      /* a bounded wait inside a kernel expired: that
                                product's C is incomplete (see sc_plan_status) */

typedef struct sc_csr sc_csr;   /* CSR matrix, int32 indices, float64 values */
typedef struct sc_cf sc_cf;     /* pattern-compressed ("CF") matrix, one block per pattern */
typedef struct sc_plan sc_plan; /* device-resident CF matrix + schedule for one B width */

/* Library version (major*10000 + minor*100 + patch). */
int sc_version(void);
/* Reason for the last failed call on this thread ("" when none). */
const char *sc_last_error_string(void);

/* ---------------------------------------------------------------- CSR ---- */

/* Reads a Matrix-Market coordinate file (real | integer | pattern,
 * general | symmetric) into CSR with columns ascending inside each row.
 * Replaces readCSRMatrixFromMTX (utils/Sparse_io.cpp:48-82). */
int sc_mtx_load_csr(const char *mtx_path, sc_csr **out);
/* Copies caller CSR arrays (rowptr has m+1 entries) into a new handle. */
int sc_csr_create(int32_t m, int32_t n, int64_t nnz, const int32_t *rowptr,
                  const int32_t *colind, const double *vals, sc_csr **out);
int sc_csr_dims(const sc_csr *a, int32_t *m, int32_t *n, int64_t *nnz);
/* Borrowed pointers, valid until sc_csr_free. */
int sc_csr_arrays(const sc_csr *a, const int32_t **rowptr, const int32_t **colind,
                  const double **vals);
void sc_csr_free(sc_csr *a);

/* ----------------------------------------------------------------- CF ---- */

/* Parses a .cfmtx file. Values are parsed to float32 exactly as
 * readCFMTXFile does (utils/Sparse_io.cpp:144-150); vector_length 0 in the
 * header is reported as 1 (utils/Sparse_io.cpp:152-154). */
int sc_cf_load(const char *cfmtx_path, sc_cf **out);
/* Pattern enumeration + coarsening on the host, bit-exact with
 * csr_to_compressed_format_converter / transform_row_panel
 * (code_gen/ss_format/format_generator.py:36-129).  dict_path NULL (or
 * "false") selects the default dictionary build_patterns_map(kernel_m, 1)
 * (pattern_dictionary.py:29-37); otherwise it is read like
 * read_pattern_dictionary (pattern_dictionary.py:49-60).  kernel_n == 0 means
 * a column pack of 32 / popcount per pattern (format_generator.py:44-45).
 * nthreads <= 0 uses every host core (row panels are independent). */
int sc_cf_from_csr(const sc_csr *a, int32_t kernel_m, int32_t kernel_n,
                   const char *dict_path, int32_t nthreads, sc_cf **out);
/* Writes the text .cfmtx byte-identically to format_writer
 * (format_generator.py:132-160) for a CF built by sc_cf_from_csr; a CF read
 * by sc_cf_load is written back token for token. */
int sc_cf_write(const sc_cf *cf, const char *path);
/* Binary sidecar of a CF (".cfbin"): the same arrays as raw little-endian
 * data on 16-byte boundaries, for large matrices whose text .cfmtx takes
 * seconds to parse.  No reference counterpart (the reference reads only the
 * text format, utils/Sparse_io.cpp:84-181); a CF loaded from a .cfbin writes
 * back to the same .cfmtx text. */
int sc_cf_write_binary(const sc_cf *cf, const char *path);
int sc_cf_load_binary(const char *path, sc_cf **out);
int sc_cf_dims(const sc_cf *cf, int32_t *num_rows, int32_t *num_cols,
               int32_t *kernel_m, int32_t *num_patterns, int32_t *vector_length);
/* Header line i (0-based, file order): mask string (NUL-terminated, written
 * into mask_out of capacity mask_cap) and pattern id. */
int sc_cf_header_line(const sc_cf *cf, int32_t line, char *mask_out, int32_t mask_cap,
                      int32_t *pattern_id);
/* Sizes of the block of pattern `pattern_id` (body order): popcount of its
 * mask, RPP length, CB length and value count. */
int sc_cf_pattern_sizes(const sc_cf *cf, int32_t pattern_id, int32_t *popcount,
                        int64_t *n_rpp, int64_t *n_cb, int64_t *n_vals);
/* Borrowed pointers to the block (RPP, CB, float32 values). */
int sc_cf_pattern_arrays(const sc_cf *cf, int32_t pattern_id, const int32_t **rpp,
                         const int32_t **cb, const float **vals);
/* Number of real (non-padding) nonzeros stored in the CF. */
int sc_cf_real_nnz(const sc_cf *cf, int64_t *nnz);
void sc_cf_free(sc_cf *cf);
/* "<stem>-<m>-<n>.cfmtx" -> "<stem>.mtx" (utils/Sparse_io.cpp:28-46). */
int sc_companion_mtx_path(const char *cfmtx_path, char *out, int32_t cap);

/* --------------------------------------------------------------- plan ---- */

/* Uploads the CF matrix to `device` and builds the schedule for products with
 * a dense operand of n_cols_b columns (B is K x n_cols_b row-major).  Replaces
 * allocateAndCopyMixedFormat (spmm_demo_gpu_utils.h:207-245) and the
 * generated launch configuration.  kernel_m must be 1..6. */
int sc_plan_create(const sc_cf *cf, int32_t n_cols_b, int32_t device, sc_plan **out);
/* Same, restricted to row panels [panel_begin, panel_end): C rows
 * [panel_begin*kernel_m, min(M, panel_end*kernel_m)) are produced, and the dC
 * pointer given to sc_spmm addresses the first of them.  Used to row-partition
 * one matrix across GPUs. */
int sc_plan_create_panels(const sc_cf *cf, int32_t n_cols_b, int32_t device,
                          int64_t panel_begin, int64_t panel_end, sc_plan **out);

/* sc_plan_create with options.  panel_begin = panel_end = -1 plans the whole
 * matrix, otherwise as sc_plan_create_panels.  flags (OR of):
 *   SC_PLAN_DENSE_OFF   never use the dense-tile tensor-core kernel;
 *   SC_PLAN_DENSE_ON    use it whenever N is a multiple of 128, whatever the
 *                       density (default: density >= 15 %);
 *   SC_PLAN_DENSE_BF16  dense tiles in bf16 instead of 3xTF32: A and B are
 *                       rounded to bf16 (8-bit mantissa), products accumulate
 *                       in fp32; |C - A*B| <= 2^-7 * (|A|*|B|) elementwise
 *                       instead of the fp32 bound.  Opt-in only; the
 *                       reference computes in fp32.
 *   SC_PLAN_VALUES_F16  small-B / SpMV plans (n_cols_b 1, 2, 4; K <= 65536):
 *   SC_PLAN_VALUES_BF16 A's values stored as fp16 (resp. bf16) with 16-bit
 *                       column indices -- half the record bytes; products
 *                       and sums in fp32.  Bound: the fp32 one plus the value
 *                       rounding, 2^-11 (fp16; absolute 2^-25 below 2^-14)
 *                       resp. 2^-8 (bf16) relative per value.  Mirrors the
 *                       reference's half-precision small-B kernels
 *                       (example_cuda/spmm_small_b_col_demo_gpu_utils.h:2987-5168).
 *                       fp16 rejects values beyond +-65504.
 * The flags override the SC_DENSE environment variable. */
#define SC_PLAN_DENSE_OFF 1u
#define SC_PLAN_DENSE_ON 2u
#define SC_PLAN_DENSE_BF16 4u
#define SC_PLAN_VALUES_F16 8u
#define SC_PLAN_VALUES_BF16 16u
/* Test hook for the error path, not for production: in a dense-tile plan's
 * kernel the producer issues no copies, so the MMA issuer's bounded wait
 * expires with nothing in flight; every product of the plan then leaves C
 * unwritten and sets status 2/3 (sc_plan_status, SC_ERR_DEVICE).  In a
 * small-B plan whose B is staged in shared memory (SpMV of a large
 * matrix) the record copies are not issued: the bounded waits expire,
 * C is left unwritten and the status is 7. */
#define SC_PLAN_TEST_STARVE (1u << 30)
int sc_plan_create_ex(const sc_cf *cf, int32_t n_cols_b, int32_t device, int64_t panel_begin,
                      int64_t panel_end, uint32_t flags, sc_plan **out);

typedef struct sc_plan_info {
  int64_t rows;          /* C rows this plan produces */
  int64_t cols;          /* K (rows of B) */
  int64_t n_cols_b;      /* N */
  int64_t panels;        /* row panels in this plan */
  int64_t kernel_m;
  int64_t nnz;           /* real nonzeros (padding excluded) */
  int64_t entries;       /* (panel, column) entries after dropping padding */
  int64_t items;         /* scheduled work items */
  int64_t device_bytes;  /* device memory held by the plan */
  int32_t kernel;        /* 1 = small-B (N<=4) kernel, 2 = large-B kernel,
                            3 = dense-tile tensor-core (tcgen05 3xTF32) kernel */
  int32_t warps_per_panel;
  int32_t dense_bf16;    /* 1: the dense-tile kernel runs on bf16 tiles */
  int32_t value_type;    /* A's stored values: 0 fp32, 1 fp16, 2 bf16 */
} sc_plan_info;
int sc_plan_get_info(const sc_plan *p, sc_plan_info *info);

/* C = A*B (accumulate == 0) or C += A*B (accumulate != 0), fp32, on `stream`
 * (NULL = legacy default stream).  dB: K x N row-major with leading dimension
 * ldb; dC: rows x N row-major with leading dimension ldc.  Asynchronous; only
 * kernel launches, so it may be captured into a CUDA graph.  Replaces the
 * reference kernels' C += A*B with atomics (which needed a zeroed C). */
int sc_spmm(sc_plan *p, const float *dB, int64_t ldb, float *dC, int64_t ldc,
            int32_t accumulate, void *stream);
/* sc_spmm that also stores every C tile into `npeers` (<= 7) peer buffers:
 * other GPUs' copies of C mapped into this process (CUDA IPC / symmetric
 * memory), same layout and ldc, each pointer addressing the same first row as
 * dC.  With A row-partitioned over GPUs (sc_plan_create_panels) and each
 * rank passing its peers' full-C buffers offset to its own rows, the kernel
 * itself performs the all-gather of the C row blocks over NVLink, overlapped
 * with the computation; the caller then runs one cross-GPU barrier on the
 * stream before reading C.  Wide-B plans only.  The reference has no
 * multi-GPU path; this replaces "SpMM then NCCL all-gather". */
int sc_spmm_peers(sc_plan *p, const float *dB, int64_t ldb, float *dC, int64_t ldc, float *const *peer_C,
                  int32_t npeers, int *const *flag_dst, int32_t nflags, int32_t epoch, int32_t accumulate,
                  void *stream);
/* Completion signal of sc_spmm_peers (nflags > 0): right after the product
 * kernel, a one-warp kernel on the same stream stores `epoch` (release,
 * system scope) into flag_dst[0..nflags) -- this rank's slot in each GPU's
 * int flag array (peer-mapped), own GPU included.
 * sc_wait_flags then waits on the stream (one warp, acquire, bounded; on
 * expiry it writes 5 to *status) until flags[0..n) of this GPU have all
 * reached `epoch` (wrap-safe): every rank's C tiles have landed here.  Use a
 * new epoch per product.  Replaces a separate cross-GPU barrier after the
 * product.  No counterpart in the reference (no multi-GPU code there). */
int sc_wait_flags(const int *flags, int32_t n, int32_t epoch, int *status, void *stream);
/* y = A*x or y += A*x (plan built with n_cols_b == 1). */
int sc_spmv(sc_plan *p, const float *dx, float *dy, int32_t accumulate, void *stream);
/* End-to-end product from HOST buffers: copies hB (K x N, dense row-major)
 * to the device, runs sc_spmm, copies C back to hC (rows x N), and
 * synchronizes `stream`.  Staging buffers are allocated on the first call and
 * kept by the plan.  When hC is page-locked host memory the device can
 * address (cudaHostAlloc / cudaMallocHost, or registered and mapped), the
 * kernel writes C into it directly while it computes; otherwise C is staged
 * on the device and copied back in row chunks that overlap the remaining
 * kernels. */
int sc_spmm_host(sc_plan *p, const float *hB, float *hC, void *stream);
/* Device-side error status of a plan's kernels since the last call: waits
 * for all work on the plan's device (cudaDeviceSynchronize), copies the
 * plan's status word to *status and clears it.  0 = no error; 1, 2, 3 = a
 * bounded mbarrier wait of the dense-tile kernel expired (producer, MMA
 * issuer, epilogue) and that CTA skipped its C stores.  Only dense-tile
 * plans (sc_plan_info.kernel == 3) wait inside their kernel; other plans
 * always report 0.  sc_spmm_host checks it itself and returns SC_ERR_DEVICE.
 * The reference checks no kernel status (example_cuda/spmm_demo_gpu_utils.h:16-23
 * checks launch errors only). */
int sc_plan_status(sc_plan *p, int32_t *status);
void sc_plan_free(sc_plan *p);

/* ------------------------------------------------------ allocation-free -- */

/* C = A*B (or C += A*B) for a DENSE row-major fp32 A (m x k, leading
 * dimension lda) on the dense-tile tensor-core kernel, without a plan and
 * without allocating: for callers that cannot call cudaMalloc on their hot
 * path (a process that gives all device memory to its own pool or budget at
 * start-up, or a framework that forbids device allocation there).  No
 * counterpart in the reference.  All scratch (TF32 head/tail tile images of A
 * and B, task list, status word) sits in one 16 MiB array held by every GPU
 * that loads the library until exit; inputs beyond it -- A padded to 128-row
 * blocks plus B, at 8 bytes per element -- are rejected with SC_ERR_ARG.
 * n must be a multiple of 128; C rows 16-byte aligned.  The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress), so make
 * that first call before any stream capture; the address is kept for the
 * life of the process, so a cudaDeviceReset while the library is loaded is
 * not supported.  Calls share the array: calls that overlap on the GPU
 * (different streams at once) race. */
int sc_spmm_dense_noalloc(const float *dA, int64_t lda, int64_t m, int64_t k, const float *dB, int64_t ldb,
                          int64_t n, float *dC, int64_t ldc, int32_t accumulate, void *stream);
/* Status word of sc_spmm_dense_noalloc on the current device (same codes as
 * sc_plan_status): waits for the device, copies the word (it lives in the
 * shared scratch array, so it reports the last call that ran) and clears it.
 * Allocates nothing. */
int sc_noalloc_status(int32_t *status);

/* ------------------------------------------------------------- batches ---- */

typedef struct sc_batch sc_batch; /* several plans executed by one kernel launch */

/* Groups plans that share device, kernel_m and n_cols_b (wide-B widths, i.e.
 * n_cols_b not in {1,2,4}) so that all their row panels run in ONE launch,
 * heaviest panels first -- e.g. the 96 weight matrices of a transformer layer
 * stack.  Replaces one reference launch per matrix
 * (example_cuda/spmm_demo_gpu_utils.h:1705-1712).  The plans must outlive
 * the batch. */
int sc_batch_create(sc_plan *const *plans, int32_t count, sc_batch **out);
/* Binds the operands of every plan (arrays of `count` device pointers and
 * leading dimensions, same meaning as for sc_spmm).  Synchronous upload;
 * re-bind whenever a buffer changes. */
int sc_batch_bind(sc_batch *b, const float *const *dB, const int64_t *ldb, float *const *dC,
                  const int64_t *ldc);
/* C_i = A_i*B_i (or +=) for all plans of the batch, one kernel launch. */
int sc_batch_spmm(sc_batch *b, int32_t accumulate, void *stream);
/* sc_plan_status for the dense-tile launch of a batch (its own status word). */
int sc_batch_status(sc_batch *b, int32_t *status);
void sc_batch_free(sc_batch *b);

/* ---------------------------------------------------------------- graphs -- */

typedef struct sc_graph sc_graph; /* captured CUDA graph of products with fixed operands */

/* Captures `repeat` back-to-back products (sc_spmm of a plan with these
 * operands, or sc_batch_spmm of a bound batch) into one CUDA graph, so that
 * a whole pattern-group schedule -- or many tiny 512-wide layers -- costs one
 * launch.  Replaces the reference's per-trial launches
 * (example_cuda/spmm_demo_gpu_utils.h:1700-1712); the reference has no
 * graphs. */
int sc_graph_capture_plan(sc_plan *p, const float *dB, int64_t ldb, float *dC, int64_t ldc, int32_t accumulate,
                          int32_t repeat, sc_graph **out);
int sc_graph_capture_batch(sc_batch *b, int32_t accumulate, int32_t repeat, sc_graph **out);
int sc_graph_launch(sc_graph *g, void *stream);
void sc_graph_free(sc_graph *g);

#ifdef __cplusplus
}
#endif
#endif /* SC_B200_H */
