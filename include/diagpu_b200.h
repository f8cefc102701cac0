/*
 * diagpu_b200.h -- C ABI of the B200 (sm_100a) DIA sparse linear-algebra
 * library (libdiagpu_b200.so).
 *
 * Conventions
 *   - Every entry point returns an int status: DIA_OK (0) or one of the
 *     DIA_ERR_* codes; dia_last_error() gives the calling thread's message.
 *     Nothing calls exit() (the reference's CUDA_CHECK did).
 *   - Pointers named d_* are device memory owned by the caller; h_* are host
 *     memory.  Kernels are enqueued on the given stream and the call returns
 *     without synchronising unless its comment says otherwise.
 *   - Values are fp32; summation follows the reference CPU routine's order
 *     with separately rounded multiply and add, so results equal the CPU
 *     oracle bit for bit (dense-band tensor-core mode excepted: TF32).
 *   - Row-indexed padded layout ("rows layout"): vals[k*stride + (i - vrow0)]
 *     holds A[i, i + off[k]] for global row i; stride is a multiple of 32
 *     floats (128 bytes) for aligned vector loads; out-of-range entries and
 *     the stride padding are zero.  A contiguous row block of a partitioned
 *     matrix is the same layout with vrow0 = the block's first row.
 *   - HM layout (the reference's SpMSpM layout): diagonal d stored from
 *     position min(row, col) = row + min(d, 0), length n - |d|.
 */
#ifndef DIAGPU_B200_H
#define DIAGPU_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    DIA_OK = 0,
    DIA_ERR_INVALID = 1,     /* bad argument (sizes, null pointers, layout) */
    DIA_ERR_CUDA = 2,        /* a CUDA runtime call or launch failed */
    DIA_ERR_UNSUPPORTED = 3, /* valid input outside what this build handles */
    DIA_ERR_CAPACITY = 4,    /* caller buffer too small (two-call pattern) */
    DIA_ERR_TIMEOUT = 5      /* a peer did not complete in time; communicator aborted */
};

/* Message for the last failing call on this host thread ("" if none). */
const char* dia_last_error(void);
/* Library version, major*10000 + minor*100 + patch. */
int dia_version(void);

/* ----------------------------------------------------------------- SpMV */

/* y[r] = sum_k values[k*cols + r + d_k] * x[r + d_k] for r in [0, rows),
 * terms with r + d_k outside [0, min(cols, x_size)) dropped, k in storage
 * order; y fully overwritten.  d_diag_offsets/d_values form the reference's
 * ReconView (column-indexed Recon, offsets sorted descending by build_recon).
 * Replaces launch_tc_spmv_regdirect (spmv/src/dia_reconstruct.cuh:139-144,
 * spmv/src/tc_spmv_regdirect_kernel.cu:135-147) and computes in FP32 instead
 * of TF32. */
int dia_spmv_recon(int rows, int cols, int num_diags, const int* d_diag_offsets,
                   const float* d_values, const float* d_x, int x_size,
                   float* d_y, cudaStream_t stream);

/* SpMV on the rows layout, for global rows [row_lo, row_hi):
 * y[i - vrow0] = sum_k vals[k*stride + i - vrow0] * x[i + d_k - x_lo],
 * terms with i + d_k outside [0, n_cols) or outside [x_lo, x_hi) dropped.
 * x holds global columns [x_lo, x_hi) (a row block's own columns plus its
 * halo).  Same math as the reference's CPU CSR loop
 * (spmv/bench/bench_cusparse.cu:119-126) when offsets ascend. */
int dia_spmv_rows(int64_t n_rows, int64_t n_cols, int num_diags,
                  const int* d_offsets, const float* d_vals, int64_t stride,
                  int64_t vrow0, int64_t row_lo, int64_t row_hi,
                  const float* d_x, int64_t x_lo, int64_t x_hi, float* d_y,
                  cudaStream_t stream);

/* ----------------------------------------------------- SpMSpM symbolic */

/* Host-side symbolic phase of C = A*B (n x n).  C offsets are the ascending
 * set {da + db : -n < da + db < n} (make_c_structure,
 * spmspm/bench_spmspm.cu:109-131; compute_c_hm_structure,
 * spmspm/paper_hm.cuh:87-117; build_c_layout's k-set,
 * gemm_diag/gemm_diag.cu:387-423), lengths n - |d|, HM starts the prefix
 * sums.  Pairs feeding each C diagonal are listed in A storage order (the
 * order cpu_dia_spgemm, spmspm/bench_spmspm.cu:392-403, sums them).
 * Two-call pattern: pass NULL outputs to get *n_c and *n_pairs, then call
 * again with buffers of those sizes (pair_ptr has *n_c + 1 entries).
 * Repeated offsets in A or B are rejected (DIA_ERR_INVALID). */
int dia_spmspm_symbolic(int n, const int* h_A_off, int nA, const int* h_B_off,
                        int nB, int* n_c, int* h_C_off, int* h_C_len,
                        int64_t* h_C_start, int64_t* n_pairs, int* h_pair_ptr,
                        int* h_pair_a, int* h_pair_b);

/* ------------------------------------------------------ SpMSpM numeric */

/* C = A*B over HM arrays with the argument set of the reference's
 * gather_spgemm_kernel / gather_meta_kernel (spmspm/spmspm.cu:196-211,
 * 257-272): signed offsets, size_t starts, lengths, B_lookup[2n-1] (B index
 * of offset db at db + n - 1, or -1).  Every C position is overwritten.
 * Pairs are resolved on the device in A order; no host synchronisation.
 * Uses stream-ordered scratch (cudaMallocAsync) of C_ndiag * A_ndiag * 24
 * bytes, released on the same stream. */
int dia_spmspm_hm(const float* d_A_values, const size_t* d_A_starts,
                  const int* d_A_off, const int* d_A_len, int A_ndiag,
                  const float* d_B_values, const size_t* d_B_starts,
                  const int* d_B_len, const int* d_B_lookup,
                  float* d_C_values, const size_t* d_C_starts,
                  const int* d_C_off, const int* d_C_len, int C_ndiag, int n,
                  cudaStream_t stream);

/* dia_spmspm_hm without any device allocation.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory while
 * they run (an allocator that reserved all device memory up front, a fixed
 * memory budget, code that must not enter the driver's allocator).  The pair
 * plan lives in a library-owned 8 MiB device array, held on every GPU that
 * loads the library until the process exits, so C_ndiag * A_ndiag * 24 +
 * C_ndiag * 32 must not exceed 8 MiB (DIA_ERR_CAPACITY otherwise).  The
 * first call on a device looks up that array's device address, so make it
 * before any stream capture.  All calls share the one array: calls whose
 * work overlaps on the GPU (other streams, other host threads) race; order
 * them on one stream.  Results equal dia_spmspm_hm bit for bit. */
int dia_spmspm_hm_noalloc(const float* d_A_values, const size_t* d_A_starts,
                          const int* d_A_off, const int* d_A_len, int A_ndiag,
                          const float* d_B_values, const size_t* d_B_starts,
                          const int* d_B_len, const int* d_B_lookup,
                          float* d_C_values, const size_t* d_C_starts,
                          const int* d_C_off, const int* d_C_len, int C_ndiag, int n,
                          cudaStream_t stream);

/* C = A*B on the rows layout (A and C share vrow0 and the output rows
 * [row_lo, row_hi); B holds global rows [b_lo, b_hi) at B_vals[k*B_stride +
 * r - b_vrow0], i.e. a row block plus its halo).  C rows in [row_lo, row_hi)
 * are overwritten, zero outside each diagonal's valid range.  Output offsets
 * d_C_off come from dia_spmspm_symbolic; pairs are resolved on the device.
 * Stream-ordered scratch of nC * nA * 24 bytes. */
int dia_spmspm_rows(int64_t n, const float* d_A_vals, int64_t A_stride,
                    const int* d_A_off, int nA, const float* d_B_vals,
                    int64_t B_stride, int64_t b_vrow0, int64_t b_lo,
                    int64_t b_hi, const int* d_B_off, int nB, float* d_C_vals,
                    int64_t C_stride, const int* d_C_off, int nC,
                    int64_t vrow0, int64_t row_lo, int64_t row_hi,
                    cudaStream_t stream);

/* Planned C = A*B on the rows layout (the analogue of the reference's
 * host Schedule, spmspm/bench_spmspm.cu:137-243, built once and reused).
 * The plan fixes the offsets and the buffer geometry: A and C hold rows
 * [vrow0, vrow0 + nrows) with strides A_stride / C_stride, B holds global
 * rows [b_lo, b_hi) at B_vals[k*B_stride + r - b_vrow0].  It runs the
 * symbolic phase, uploads its tables (cudaMalloc, owned by the plan) and,
 * when A's offsets cluster tightly enough for the operands of a row tile to
 * fit in shared memory, enables the tiled kernel for the interior rows.
 * C offsets come back through dia_spmspm_plan_info. */
typedef struct DiaSpmspmPlan DiaSpmspmPlan;
int dia_spmspm_plan_create(int64_t n, const int* h_A_off, int nA, const int* h_B_off,
                           int nB, int64_t A_stride, int64_t B_stride, int64_t C_stride,
                           int64_t vrow0, int64_t nrows, int64_t b_vrow0, int64_t b_lo,
                           int64_t b_hi, DiaSpmspmPlan** plan);
/* Output structure (any pointer may be NULL), the interior kernel's tile
 * rows (0: generic kernel only; > 0: shared-memory-tiled kernel; < 0: the
 * register-blocked run-pair kernel, for offsets made of equal-length runs
 * of consecutive values) and the row range it covers. */
int dia_spmspm_plan_info(const DiaSpmspmPlan* plan, int* n_c, int* h_C_off, int* h_C_len,
                         int64_t* h_C_start, int* tile_rows, int64_t* tiled_lo,
                         int64_t* tiled_hi);
/* C rows [row_lo, row_hi) of the plan's block (overwritten); use_tiles 0
 * forces the generic kernel.  Results are identical either way.  No
 * allocation, no synchronisation. */
int dia_spmspm_plan_execute(const DiaSpmspmPlan* plan, const float* d_A_vals,
                            const float* d_B_vals, float* d_C_vals, int64_t row_lo,
                            int64_t row_hi, int use_tiles, cudaStream_t stream);
int dia_spmspm_plan_destroy(DiaSpmspmPlan* plan);

/* Lanczos on a symmetric DIA operator (whole matrix, rows layout, stride
 * >= n), m steps without host synchronisation: d_alpha[0..m) and
 * d_beta[0..max(m,1)) (fp64, device) receive the tridiagonal T_m whose
 * extreme eigenvalues approach A's; d_basis (optional, m*n floats) receives
 * v_0 .. v_{m-1}.  Per step: w = fl(A v_j) - fl(beta_{j-1} v_{j-1}),
 * alpha_j = w.v_j and beta_j = ||w - fl(alpha_j v_j)|| in fp64 (exact
 * products, fixed-order sums), v_{j+1} = fl(w * fl(1/beta_j)), scalars used
 * as fp32 in the vector updates; v_0 = x * fl(1/||x||).  d_work holds
 * dia_lanczos_workspace(n) bytes.  The reference has no eigensolver; this
 * serves the ground-state energies of the operators it stores. */
int64_t dia_lanczos_workspace(int64_t n);
int dia_lanczos(int64_t n, int num_diags, const int* d_offsets, const float* d_vals,
                int64_t stride, int m, const float* d_x, double* d_alpha, double* d_beta,
                float* d_basis, void* d_work, int64_t work_bytes, cudaStream_t stream);

/* Complex64 (interleaved fp32 re, im) DIA on the rows layout, whole matrix
 * (vrow0 = 0, stride in complex elements >= n_rows): y = A x with
 * per-term rounding re += fl(fl(ar*xr) - fl(ai*xi)), im += fl(fl(ar*xi) +
 * fl(ai*xr)) in offset storage order (with zero imaginary parts this is the
 * real SpMV bit for bit).  dia_expm_taylor_c64 is the Schroedinger-type
 * evolution y = exp(-i t A) x by the truncated Taylor series v_0 = x,
 * v_j = (-i fl(t/j)) (A v_{j-1}), y = sum v_j, one fused launch per term;
 * d_work holds 2n complex values.  The reference is real-only; these serve
 * the complex Hamiltonians its DIA format targets. */
int dia_spmv_rows_c64(int64_t n_rows, int64_t n_cols, int num_diags, const int* d_offsets,
                      const void* d_vals, int64_t stride, const void* d_x, void* d_y,
                      cudaStream_t stream);
int dia_expm_taylor_c64(int64_t n, int num_diags, const int* d_offsets, const void* d_vals,
                        int64_t stride, float t, int m, const void* d_x, void* d_y,
                        void* d_work, cudaStream_t stream);

/* Matrix Market ingestion (host only, no GPU needed): a coordinate file
 * (real / double / integer / pattern; general / symmetric / skew-symmetric)
 * such as spmv/tools/gen_banded_mtx.cpp writes, laid out as the rows layout:
 * offsets j - i ascending, h_vals[k*stride + i] = A[i, i + off[k]], zero
 * elsewhere (duplicates summed in double in file order, one rounding to
 * fp32).  Two calls: with h_offsets = h_vals = NULL it parses and returns
 * the shape and *num_diags; then with buffers (*num_diags = their capacity,
 * stride >= n_rows) it fills them.  DIA_ERR_UNSUPPORTED for array files,
 * and for complex files (read those with dia_mtx_read_c64). */
int dia_mtx_read(const char* path, int64_t* n_rows, int64_t* n_cols, int* num_diags,
                 int* h_offsets, float* h_vals, int64_t stride);
/* The same into interleaved complex64 rows (h_vals[2*(k*stride + i)] = re,
 * [.. + 1] = im) for the c64 paths: complex files (general, symmetric,
 * skew-symmetric, or hermitian -- mirrored entries conjugated) and every
 * real field (imaginary parts zero).  *is_complex (may be NULL) = 1 when the
 * file's field is complex. */
int dia_mtx_read_c64(const char* path, int64_t* n_rows, int64_t* n_cols, int* num_diags,
                     int* h_offsets, float* h_vals, int64_t stride, int* is_complex);
/* The inverse (host): the rows-layout matrix as a coordinate real general
 * file, rows in order and offsets ascending within a row (the order of
 * spmv/tools/gen_banded_mtx.cpp), 9 significant digits so every fp32 value
 * reads back exactly; stored zeros inside the matrix are written too. */
int dia_mtx_write(const char* path, int64_t n_rows, int64_t n_cols, int num_diags,
                  const int* h_offsets, const float* h_vals, int64_t stride);

/* Pauli-string Hamiltonians (the operators of HamLib's spin, QUBO and
 * molecular sets) into the rows layout (host only, no GPU): H = sum_t c_t
 * P_t on nq qubits (n = 2^nq rows), P_t in symplectic form -- x_mask = the
 * qubits carrying X or Y, z_mask = those carrying Z or Y -- with qubit k on
 * bit k of the basis index, so an X or Y on qubit k moves the column by
 * +-2^k.  Writes the distinct offsets ascending and complex64 values
 * (interleaved re, im; h_vals[2*(k*stride + r)]), summed in double
 * complex in term order and rounded once; *is_real = 1 when every
 * imaginary part is zero.  Two calls, as dia_mtx_read; coef_im may be
 * NULL.  The reference reads HamLib files with tools outside its
 * repository; the DIA mapping follows its talk's appendix
 * (slides/transcript.md:97-116). */
int dia_pauli_to_dia(int nq, int nterms, const uint64_t* h_x_mask, const uint64_t* h_z_mask,
                     const double* h_coef_re, const double* h_coef_im, int* num_diags,
                     int* h_offsets, float* h_vals, int64_t stride, int* is_real);

/* Truncated Taylor series of exp(tA) x for a whole square matrix A on the
 * rows layout (stride >= n): v_0 = x, v_j = (t/j) * A v_{j-1}, y = sum of
 * v_0 .. v_m.  One fused kernel per term (SpMV, scale, running sum); d_work
 * holds 2n floats.  Per element: the SpMV sum in offset storage order, then
 * fl(fl(t/j) * s), then fl(y + v_j), the order of the CPU oracle.  The
 * reference has no such driver (its SpMV is a single product); this chains
 * its SpMV into the time evolution its Hamiltonians are built for. */
int dia_expm_taylor(int64_t n, int num_diags, const int* d_offsets, const float* d_vals,
                    int64_t stride, float t, int m, const float* d_x, float* d_y,
                    float* d_work, cudaStream_t stream);

/* Device-side steps for matrix-power chains (P_{k+1} = P_k * H with H
 * narrow).  The reference resolves a chain step's pairs on the device but
 * takes its output offsets from a host symbolic phase
 * (spmspm/gather_flat.cuh:110-117); these calls keep the whole step on the
 * device, so a chain runs without any host synchronisation:
 *   - A's offsets and count live in device memory (d_A_off, d_nA; nA_cap is
 *     their capacity), as the previous step left them; B's count nB is a
 *     host value (H does not change);
 *   - the output offsets are written ascending to d_C_off and their number
 *     to d_nC -- the sumset of A's and B's offsets inside (-n, n), equal to
 *     dia_spmspm_symbolic's C_off bit for bit.  If the number exceeds nC_cap
 *     only the first nC_cap offsets are written and *d_nC still holds the
 *     full number: the caller checks *d_nC <= nC_cap before using C;
 *   - d_work is caller device memory of dia_spmspm_device_workspace() bytes
 *     (a bitmap of the 2n-1 offsets, scan scratch and the term lists).
 * dia_spmspm_rows_device also computes C = A*B on the rows layout with all
 * n rows present (vrow0 = 0, strides >= n); values equal dia_spmspm_rows'
 * bit for bit (same pair order: A storage order). */
int64_t dia_spmspm_device_workspace(int64_t n, int nA_cap, int nB, int nC_cap);
int dia_spmspm_symbolic_device(int64_t n, const int* d_A_off, const int* d_nA, int nA_cap,
                               const int* d_B_off, int nB, int* d_C_off, int* d_nC,
                               int nC_cap, void* d_work, int64_t work_bytes,
                               cudaStream_t stream);
int dia_spmspm_rows_device(int64_t n, const int* d_A_off, const int* d_nA, int nA_cap,
                           const float* d_A_vals, int64_t A_stride, const int* d_B_off,
                           int nB, const float* d_B_vals, int64_t B_stride, int* d_C_off,
                           int* d_nC, int nC_cap, float* d_C_vals, int64_t C_stride,
                           void* d_work, int64_t work_bytes, cudaStream_t stream);

/* ----------------------------------------------------------- gemm_diag */

/* C += A*B with gemm_diag_kernel's argument set (gemm_diag/gemm_diag.cu:
 * 121-131): row-packed DA[ri*n + row] (P x n), DB (Q x n), offsets off_A /
 * off_B, HM-packed C with int value starts C_offsets, C_lens and
 * k_to_idx[2n-1] from build_c_layout.  Accumulates into C like the
 * reference (which expects C zeroed), without atomics and deterministically.
 * Reads the P + Q offsets back to the host to plan the product (one
 * synchronisation of `stream` per call). */
int dia_gemm_diag(const float* d_DA, const float* d_DB, const int* d_off_A,
                  const int* d_off_B, int P, int Q, int n, float* d_C_data,
                  const int* d_C_offsets, const int* d_C_lens,
                  const int* d_k_to_idx, cudaStream_t stream);

enum {
    DIA_GEMM_AUTO = 0,   /* tensor cores for a contiguous dense band */
    DIA_GEMM_SIMT = 1,   /* exact fp32 diagonal-pair kernel */
    DIA_GEMM_TCGEN05 = 2 /* tcgen05 TF32 dense-band kernel */
};

/* dia_gemm_diag with options: beta 0 overwrites C (no read of C), beta 1
 * accumulates; mode picks the kernel (DIA_GEMM_*).  h_off_A / h_off_B may
 * be host copies of the offsets (skips the read-back) or NULL. */
int dia_gemm_diag_ex(const float* d_DA, const float* d_DB, const int* d_off_A,
                     const int* d_off_B, const int* h_off_A,
                     const int* h_off_B, int P, int Q, int n, float* d_C_data,
                     const int* d_C_offsets, const int* d_C_lens,
                     const int* d_k_to_idx, int beta, int mode,
                     cudaStream_t stream);

/* ------------------------------------------------- row-partitioned (NCCL) */

/* Native halo exchange for row-block partitioned products over 1..N GPUs,
 * one process per GPU.  No counterpart in the reference (single-GPU only);
 * this is the partitioned form of its products.  dia_nccl_unique_id fills
 * an ncclUniqueId (128 bytes) on one rank; the caller distributes it; every
 * rank then calls dia_dist_create (collective, blocking), which creates the
 * NCCL communicator and a private stream. */
typedef struct DiaDist DiaDist;
int dia_nccl_unique_id(void* h_id, int nbytes);
int dia_dist_create(int rank, int world, const void* h_id, DiaDist** dist);
/* dia_dist_create with a deadline.  The communicator is non-blocking: its
 * init and every later call that NCCL completes in the background are
 * polled until timeout_ms; a rank that never joins (or stops answering
 * during set-up) makes the call abort the communicator and return
 * DIA_ERR_TIMEOUT instead of blocking forever.  dia_dist_create uses 120 s.
 * Transfers already running on the GPU are not covered: ranks must learn of
 * a departed peer on the host before their next step. */
int dia_dist_create_timeout(int rank, int world, const void* h_id, int64_t timeout_ms,
                            DiaDist** dist);
/* Abort the communicator (ncclCommAbort); later calls on it fail with
 * DIA_ERR_INVALID.  dia_dist_destroy still frees the handle. */
int dia_dist_abort(DiaDist* dist);
/* Exchange halo columns of a [K rows x pitch] buffer whose column j holds
 * global column ext_lo + j.  h_ranges (8 x int64, global columns): receive
 * from rank-1 [0,1), send to rank-1 [2,3), receive from rank+1 [4,5), send
 * to rank+1 [6,7); empty ranges are skipped.  halo_start orders the
 * exchange after the work already on `stream`; halo_wait makes `stream`
 * wait for it. */
int dia_dist_halo_start(DiaDist* dist, float* d_ext, int64_t ext_lo, int64_t pitch, int K,
                        const int64_t* h_ranges, cudaStream_t stream);
int dia_dist_halo_wait(DiaDist* dist, cudaStream_t stream);
/* One partitioned SpMV step with a single host call (arguments as
 * dia_spmv_rows).  overlap == 2 (fastest measured): the halo is received on
 * the library's high-priority stream, the boundary rows [r0, int_lo) and
 * [int_hi, r1) run there right after it while the interior rows
 * [int_lo, int_hi) run on `stream`; `stream` then waits for both.
 * overlap == 1: interior during the transfer, boundary strips after it, all
 * on `stream`.  overlap == 0: exchange, then one launch over [r0, r1). */
int dia_dist_spmv_step(DiaDist* dist, int64_t n_rows, int64_t n_cols, int num_diags,
                       const int* d_offsets, const float* d_vals, int64_t stride,
                       int64_t vrow0, float* d_x_ext, int64_t x_lo, int64_t x_hi, float* d_y,
                       const int64_t* h_ranges, int64_t r0, int64_t r1, int64_t int_lo,
                       int64_t int_hi, int overlap, cudaStream_t stream);
/* NCCL's asynchronous error state of the communicator (DIA_OK if none). */
int dia_dist_async_error(DiaDist* dist);
int dia_dist_destroy(DiaDist* dist);

/* ---- peer-memory halo: one fused kernel per partitioned SpMV step ----
 *
 * No counterpart in the reference (single-GPU only).  The step kernel
 * itself copies this rank's edge columns of x into its neighbours' receive
 * buffers over NVLink (peer stores through CUDA IPC mappings), publishes the
 * step number in the neighbour's flag word, and computes the block's rows;
 * the boundary tiles, dispatched a quarter of the way through the grid,
 * wait on the flag with a time limit.  Receive buffers alternate by step parity.
 * Bit-identical to the single-GPU SpMV of the whole matrix. */
enum { DIA_DIST_TIMEOUT = 2 };   /* a flag wait ran out of time */

typedef struct DiaPeerHalo {
    float* halo_lo[2];              /* this rank's receive buffers, columns [x_lo, r0), by step parity */
    float* halo_hi[2];              /* columns [r1, x_hi) */
    unsigned long long* flag_lo;    /* last step whose columns the left neighbour delivered */
    unsigned long long* flag_hi;    /* ... the right neighbour delivered */
    unsigned long long* push_count; /* 2 counters (left, right): pushing CTAs finished */
    unsigned int* status;           /* DIA_DIST_* bits set by the kernel */
    float* peer_left_halo_hi[2];    /* the left neighbour's halo_hi buffers (peer memory) */
    unsigned long long* peer_left_flag_hi;
    float* peer_right_halo_lo[2];   /* the right neighbour's halo_lo buffers */
    unsigned long long* peer_right_flag_lo;
    int64_t send_left_hi;           /* columns [r0, send_left_hi) go to the left neighbour */
    int64_t send_right_lo;          /* columns [send_right_lo, r1) go to the right one */
    int has_left, has_right;
    int64_t timeout_ns;             /* limit of one flag wait */
} DiaPeerHalo;

/* The fused step kernel with every buffer given explicitly (the buffers may
 * all be local, e.g. to check the kernel on one GPU with the flags already
 * set).  step counts from 1 and grows by one per call; push_count must have
 * been zeroed before step 1.  d_x_own holds columns [r0, r1); y row i is
 * written at d_y[i - vrow0].  dmin/dmax: smallest and largest offset.
 * At most 128 diagonals; the block needs at least 8 tiles of 1024 rows. */
int dia_spmv_rows_peer(const DiaPeerHalo* halo, uint64_t step, int64_t n_rows, int64_t n_cols,
                       int num_diags, const int* d_offsets, const float* d_vals, int64_t stride,
                       int64_t vrow0, int64_t r0, int64_t r1, int64_t x_lo, int64_t x_hi,
                       int dmin, int dmax, const float* d_x_own, float* d_y,
                       cudaStream_t stream);
/* Collective over the communicator: allocate this rank's receive window
 * (flags, counters, status, double-buffered halo buffers for [x_lo, r0) and
 * [r1, x_hi)), exchange CUDA IPC handles with NCCL, map both neighbours'
 * windows.  h_ranges as for dia_dist_halo_start. */
int dia_dist_peer_setup(DiaDist* dist, int64_t r0, int64_t r1, int64_t x_lo, int64_t x_hi,
                        const int64_t* h_ranges);
/* One partitioned SpMV step through the peer window (after peer_setup). */
int dia_dist_spmv_fused(DiaDist* dist, int64_t n_rows, int64_t n_cols, int num_diags,
                        const int* d_offsets, const float* d_vals, int64_t stride,
                        int64_t vrow0, int dmin, int dmax, const float* d_x_own, float* d_y,
                        cudaStream_t stream);
/* Limit of one flag wait (default 2 s). */
int dia_dist_set_timeout(DiaDist* dist, int64_t ns);
/* Read (synchronously) the DIA_DIST_* bits of the peer window; clear != 0
 * resets them. */
int dia_dist_status(DiaDist* dist, unsigned int* flags, int clear);

/* Device status word shared by the library's kernels.  Kernels that wait on
 * the hardware (the tcgen05 dense-band kernel's mbarrier waits) never spin
 * without bound: on giving up they set a bit here and return early.  Reads
 * the word into *flags (synchronous); clear != 0 resets it.  No counterpart
 * in the reference, whose kernels have no waits. */
enum { DIA_TC_TIMEOUT = 1 };
int dia_device_status(unsigned int* flags, int clear);
/* Test hook of the tcgen05 dense-band kernel (current device): wait_ns sets
 * the limit of each of its waits (0: the default of 2 s); withhold != 0
 * makes one warp of its first CTA skip one arrival, so a wait is certain to
 * run out and the kernel's abort path (stop, drain issued copies and MMAs,
 * free tensor memory, set DIA_TC_TIMEOUT) runs.  Both persist until the
 * next call; reset with (0, 0).  Not for production use. */
int dia_test_tc_wait(uint64_t wait_ns, int withhold);

/* ------------------------------------------------ synthetic test inputs */

/* Fill rows [row0, row0+nrows) of a rows-layout matrix (K diagonals, stride)
 * with the library's counter-based generator: value(seed, d, i) depends only
 * on the offset and the global row, so any row block can be generated on its
 * own.  kind 0: base[k] + lo + (hi-lo)*u, u in [0,1) (24-bit); kind 1:
 * base[k] + hi * (Irwin-Hall-12 normal approximation).  d_base may be NULL.
 * Out-of-range entries and padding are zero. */
int dia_synth_rows(uint64_t seed, int64_t n_rows, int64_t n_cols, int K,
                   const int* d_offsets, const float* d_base, int kind,
                   float lo, float hi, int64_t row0, int64_t nrows,
                   int64_t stride, float* d_vals, cudaStream_t stream);

/* out[j] = lo + (hi-lo)*u(seed, i0 + j) for j in [0, len). */
int dia_synth_vector(uint64_t seed, int64_t i0, int64_t len, float lo, float hi,
                     float* d_out, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* DIAGPU_B200_H */
