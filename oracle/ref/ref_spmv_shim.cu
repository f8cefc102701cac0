/*
 * ref_spmv_shim.cu -- TEST INFRASTRUCTURE: exposes the reference's own SpMV
 * routines through a C ABI so the oracle restatement can be pinned against
 * them.  Compiled from the reference sources where they lie (never copied);
 * the output goes to oracle/_ref/, which is not committed.
 *
 *   spmv/test/test_tc_spmv.cu:39-79  dense_to_dia, spmv_from_recon
 *   spmv/src/dia_reconstruct.cuh:77-107  build_recon
 *   spmv/src/tc_spmv_regdirect_kernel.cu:135-147  launch_tc_spmv_regdirect
 */
#include <algorithm>
#include <cstring>
#include <vector>
#define main ref_main_test_tc_spmv
#include "spmv/test/test_tc_spmv.cu"
#undef main

extern "C" {

/* dense (rows x cols, row-major) -> DIA via the reference's dense_to_dia.
 * Returns K; fills offsets/starts/lengths (capacity rows+cols-1) and values
 * (capacity rows*cols). */
int ref_dense_to_dia(const float* H, int rows, int cols, int* offsets,
                     int* starts, int* lengths, float* values, int* nvals)
{
    DiaMatrix D = dense_to_dia(H, rows, cols);
    const int K = (int)D.offsets.size();
    for (int k = 0; k < K; ++k) {
        offsets[k] = D.offsets[k];
        starts[k] = D.diag_starts[k];
        lengths[k] = D.diag_lengths[k];
    }
    std::memcpy(values, D.values.data(), D.values.size() * sizeof(float));
    *nvals = (int)D.values.size();
    return K;
}

/* DIA -> Recon via the reference's build_recon. */
void ref_build_recon(int rows, int cols, int K, const int* offsets,
                     const int* starts, const int* lengths, const float* values,
                     int nvals, int* out_offsets, float* out_values)
{
    DiaMatrix D;
    D.rows = rows; D.cols = cols;
    D.offsets.assign(offsets, offsets + K);
    D.diag_starts.assign(starts, starts + K);
    D.diag_lengths.assign(lengths, lengths + K);
    D.values.assign(values, values + nvals);
    ReconMatrix R = build_recon(D);
    std::memcpy(out_offsets, R.diag_offsets.data(), K * sizeof(int));
    std::memcpy(out_values, R.values.data(), R.values.size() * sizeof(float));
}

/* Recon SpMV via the reference's spmv_from_recon (serial). */
void ref_spmv_from_recon(int rows, int cols, int K, const int* offsets,
                         const float* recon, const float* x, float* y)
{
    ReconMatrix R;
    R.rows = rows; R.cols = cols; R.num_diags = K;
    R.diag_offsets.assign(offsets, offsets + K);
    R.values.assign(recon, recon + (size_t)K * cols);
    std::vector<float> xv(x, x + cols);
    std::vector<float> yv = spmv_from_recon(R, xv);
    std::memcpy(y, yv.data(), rows * sizeof(float));
}

/* The reference's TF32 tensor-core SpMV launcher on device buffers (the
 * kernel the B200 library is measured against on the GPU box). */
int ref_launch_tc_spmv(int rows, int cols, int K, const int* d_offsets,
                       const float* d_values, const float* d_x, int x_size,
                       float* d_y, void* stream)
{
    ReconView RV{rows, cols, K, d_offsets, d_values};
    launch_tc_spmv_regdirect(RV, d_x, x_size, d_y, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

}  // extern "C"

#include <chrono>
#include <thread>

extern "C" {

/* The reference's spmv_from_recon run on `threads` host threads, each on a
 * contiguous row slice re-expressed as its own (smaller) ReconMatrix so the
 * reference routine itself does the arithmetic.  Slices are built before the
 * clock starts; `reps` passes are timed and the mean milliseconds returned.
 * Returns -1 on bad input. */
double ref_spmv_from_recon_threads(int rows, int cols, int K, const int* offsets,
                                   const float* recon, const float* x, float* y, int threads,
                                   int reps)
{
    if (rows <= 0 || K <= 0 || threads <= 0 || reps <= 0) return -1.0;
    int dmin = offsets[0], dmax = offsets[0];
    for (int k = 0; k < K; ++k) {
        dmin = std::min(dmin, offsets[k]);
        dmax = std::max(dmax, offsets[k]);
    }
    struct Slice { int r0, r1; ReconMatrix R; std::vector<float> xs; };
    std::vector<Slice> sl(threads);
    const int per = (rows + threads - 1) / threads;
    for (int t = 0; t < threads; ++t) {
        Slice& s = sl[t];
        s.r0 = std::min(rows, t * per);
        s.r1 = std::min(rows, s.r0 + per);
        const int nr = s.r1 - s.r0;
        const int c0 = s.r0 + dmin;               /* first global column */
        const int nc = nr + (dmax - dmin);
        s.R.rows = nr; s.R.cols = nc; s.R.num_diags = K;
        for (int k = 0; k < K; ++k) s.R.diag_offsets.push_back(offsets[k] - dmin);
        s.R.values.assign((size_t)K * nc, 0.0f);
        s.xs.assign(nc, 0.0f);
        for (int c = 0; c < nc; ++c) {
            const long g = (long)c0 + c;
            if (g < 0 || g >= cols) continue;
            s.xs[c] = x[g];
            for (int k = 0; k < K; ++k) s.R.values[(size_t)k * nc + c] = recon[(size_t)k * cols + g];
        }
    }
    auto t0 = std::chrono::steady_clock::now();
    for (int rep = 0; rep < reps; ++rep) {
        std::vector<std::thread> pool;
        for (int t = 0; t < threads; ++t)
            pool.emplace_back([&, t] {
                Slice& s = sl[t];
                if (s.r1 <= s.r0) return;
                std::vector<float> ys = spmv_from_recon(s.R, s.xs);
                std::memcpy(y + s.r0, ys.data(), ys.size() * sizeof(float));
            });
        for (auto& th : pool) th.join();
    }
    auto t1 = std::chrono::steady_clock::now();
    return std::chrono::duration<double, std::milli>(t1 - t0).count() / reps;
}

}  // extern "C"
