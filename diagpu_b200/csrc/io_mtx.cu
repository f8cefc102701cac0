/*
 * io_mtx.cu -- Matrix Market ingestion into the DIA rows layout (host code).
 *
 * Reads a coordinate-format Matrix Market file (field real, double, integer
 * or pattern; symmetry general, symmetric or skew-symmetric), e.g. the files
 * the reference's spmv/tools/gen_banded_mtx.cpp writes for external
 * baselines, and lays it out as the library stores matrices: the distinct
 * offsets j - i ascending, and vals[k*stride + i] = A[i, i + off[k]] with
 * zeros elsewhere.  Symmetric files mirror every off-diagonal entry,
 * skew-symmetric ones mirror it negated; duplicate coordinates are summed in
 * double precision in file order; pattern entries are 1.  Values are parsed
 * as double and rounded once to fp32.  Array (dense) files are reported as
 * unsupported.  Complex files (symmetry general, symmetric, skew-symmetric or
 * hermitian; Hermitian mirrors the conjugate) are read by dia_mtx_read_c64
 * into interleaved complex64 rows, which also accepts every real field
 * (imaginary parts zero); dia_mtx_read refuses them rather than drop the
 * imaginary parts.
 *
 * Two calls, like dia_spmspm_symbolic: the first (null outputs) parses the
 * file and returns the shape and the number of diagonals; the second fills
 * the caller's offset and value buffers.  The parsed entries are kept in a
 * per-thread cache between the two calls so a large file is read once.
 */
#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <map>
#include <string>
#include <vector>

#include "../../include/diagpu_b200.h"
#include "dia_core.cuh"

namespace {

struct MtxEntries {
    std::string path;
    int64_t rows = 0, cols = 0;
    std::vector<int64_t> r, c;   /* 0-based, mirrored entries included */
    std::vector<double> v, vi;   /* vi only for complex files */
    bool complex = false;
};

thread_local MtxEntries g_cache;

bool lower_eq(const char* a, const char* b)
{
    for (; *a && *b; ++a, ++b)
        if (tolower((unsigned char)*a) != tolower((unsigned char)*b)) return false;
    return *a == *b;
}

int parse(const char* path, MtxEntries& e)
{
    FILE* f = std::fopen(path, "rb");
    if (!f) return dia::fail(DIA_ERR_INVALID, std::string("dia_mtx_read: cannot open ") + path);
    std::string all;
    {
        char buf[1 << 16];
        size_t got;
        while ((got = std::fread(buf, 1, sizeof(buf), f)) > 0) all.append(buf, got);
        std::fclose(f);
    }
    const char* p = all.c_str();
    const char* end = p + all.size();
    auto next_line = [&](const char*& q) {
        while (q < end && *q != '\n') ++q;
        if (q < end) ++q;
    };
    /* banner */
    char w[5][64] = {};
    if (std::sscanf(p, "%63s %63s %63s %63s %63s", w[0], w[1], w[2], w[3], w[4]) != 5 ||
        !lower_eq(w[0], "%%MatrixMarket") || !lower_eq(w[1], "matrix"))
        return dia::fail(DIA_ERR_INVALID, "dia_mtx_read: missing %%MatrixMarket matrix banner");
    if (!lower_eq(w[2], "coordinate"))
        return dia::fail(DIA_ERR_UNSUPPORTED, "dia_mtx_read: only coordinate files are supported");
    const bool pattern = lower_eq(w[3], "pattern");
    const bool cplx = lower_eq(w[3], "complex");
    if (!pattern && !cplx && !lower_eq(w[3], "real") && !lower_eq(w[3], "double") &&
        !lower_eq(w[3], "integer"))
        return dia::fail(DIA_ERR_UNSUPPORTED,
                         std::string("dia_mtx_read: field '") + w[3] + "' is not supported");
    int sym = 0;   /* 0 general, 1 symmetric, -1 skew-symmetric, 2 hermitian */
    if (lower_eq(w[4], "symmetric"))
        sym = 1;
    else if (lower_eq(w[4], "skew-symmetric"))
        sym = -1;
    else if (cplx && lower_eq(w[4], "hermitian"))
        sym = 2;
    else if (!lower_eq(w[4], "general"))
        return dia::fail(DIA_ERR_UNSUPPORTED,
                         std::string("dia_mtx_read: symmetry '") + w[4] + "' is not supported");
    next_line(p);
    while (p < end && (*p == '%' || *p == '\n' || *p == '\r')) next_line(p);
    char* q;
    errno = 0;
    const long long M = std::strtoll(p, &q, 10);
    const long long N = std::strtoll(q, &q, 10);
    const long long L = std::strtoll(q, &q, 10);
    if (errno || q == p || M <= 0 || N <= 0 || L < 0 || M >= (1LL << 31) || N >= (1LL << 31))
        return dia::fail(DIA_ERR_INVALID, "dia_mtx_read: bad size line");
    p = q;
    next_line(p);
    e = MtxEntries{};
    e.path = path;
    e.rows = M;
    e.cols = N;
    e.complex = cplx;
    if (cplx) e.vi.reserve((size_t)L * (sym ? 2 : 1));
    e.r.reserve((size_t)L * (sym ? 2 : 1));
    e.c.reserve((size_t)L * (sym ? 2 : 1));
    e.v.reserve((size_t)L * (sym ? 2 : 1));
    for (long long t = 0; t < L; ++t) {
        while (p < end && (*p == '%' || *p == '\n' || *p == '\r')) next_line(p);
        if (p >= end) return dia::fail(DIA_ERR_INVALID, "dia_mtx_read: fewer entries than declared");
        const long long i = std::strtoll(p, &q, 10);
        const long long j = std::strtoll(q, &q, 10);
        double v = 1.0, vi = 0.0;
        if (!pattern) {
            const char* vs = q;
            v = std::strtod(vs, &q);
            if (q == vs) return dia::fail(DIA_ERR_INVALID, "dia_mtx_read: entry without a value");
        }
        if (cplx) {
            const char* vs = q;
            vi = std::strtod(vs, &q);
            if (q == vs)
                return dia::fail(DIA_ERR_INVALID, "dia_mtx_read: complex entry without an "
                                                  "imaginary part");
        }
        if (i < 1 || i > M || j < 1 || j > N)
            return dia::fail(DIA_ERR_INVALID, "dia_mtx_read: entry outside the matrix");
        e.r.push_back(i - 1);
        e.c.push_back(j - 1);
        e.v.push_back(v);
        if (cplx) e.vi.push_back(vi);
        if (sym && i != j) {
            e.r.push_back(j - 1);
            e.c.push_back(i - 1);
            e.v.push_back(sym > 0 ? v : -v);
            if (cplx) e.vi.push_back(sym == 1 ? vi : -vi);
        }
        p = q;
        next_line(p);
    }
    return DIA_OK;
}

}  // namespace

using namespace dia;

namespace {

/* Shared body of the two readers; ncomp = 1 (fp32) or 2 (interleaved c64). */
int read_into(const char* who, const char* path, int64_t* n_rows, int64_t* n_cols, int* num_diags,
              int* h_offsets, float* h_vals, int64_t stride, int ncomp, int* is_complex)
{
    if (!path || !n_rows || !n_cols || !num_diags)
        return fail(DIA_ERR_INVALID, std::string(who) + ": null pointer");
    MtxEntries& e = g_cache;
    if (e.path != path || (!h_offsets && !h_vals)) {
        const int rc = parse(path, e);
        if (rc) {
            g_cache = MtxEntries{};
            return rc;
        }
    }
    if (e.complex && ncomp == 1) {
        g_cache = MtxEntries{};
        return fail(DIA_ERR_UNSUPPORTED, std::string(who) + ": complex file; read it with "
                                                            "dia_mtx_read_c64");
    }
    if (is_complex) *is_complex = e.complex ? 1 : 0;
    std::map<int64_t, int> diag;
    for (size_t t = 0; t < e.r.size(); ++t) diag.emplace(e.c[t] - e.r[t], 0);
    *n_rows = e.rows;
    *n_cols = e.cols;
    if (diag.size() > (size_t)INT32_MAX)
        return fail(DIA_ERR_UNSUPPORTED, std::string(who) + ": too many diagonals");
    const int K = (int)diag.size();
    if (!h_offsets && !h_vals) {
        *num_diags = K;
        return DIA_OK;
    }
    if (*num_diags < K) {
        *num_diags = K;
        return fail(DIA_ERR_CAPACITY, std::string(who) + ": offset buffer smaller than the "
                                                         "diagonal count");
    }
    if (h_vals && stride < e.rows)
        return fail(DIA_ERR_INVALID, std::string(who) + ": stride smaller than the row count");
    int k = 0;
    for (auto& kv : diag) {
        kv.second = k;
        if (h_offsets) h_offsets[k] = (int)kv.first;
        ++k;
    }
    *num_diags = K;
    if (h_vals) {
        const size_t rowlen = (size_t)ncomp * (size_t)stride;
        std::memset(h_vals, 0, (size_t)K * rowlen * sizeof(float));
        /* entries ordered by (diagonal, row), file order within a cell
         * (stable sort); a cell's duplicates are summed in double in that
         * order and rounded once */
        std::vector<size_t> idx(e.r.size());
        std::vector<int> kd(e.r.size());
        for (size_t t = 0; t < idx.size(); ++t) {
            idx[t] = t;
            kd[t] = diag[e.c[t] - e.r[t]];
        }
        std::stable_sort(idx.begin(), idx.end(), [&](size_t a, size_t b) {
            return kd[a] != kd[b] ? kd[a] < kd[b] : e.r[a] < e.r[b];
        });
        for (size_t t = 0; t < idx.size();) {
            const size_t a = idx[t];
            double s = 0.0, si = 0.0;
            size_t u = t;
            for (; u < idx.size() && kd[idx[u]] == kd[a] && e.r[idx[u]] == e.r[a]; ++u) {
                s += e.v[idx[u]];
                if (e.complex) si += e.vi[idx[u]];
            }
            float* cell = h_vals + (size_t)kd[a] * rowlen + (size_t)ncomp * (size_t)e.r[a];
            cell[0] = (float)s;
            if (ncomp == 2) cell[1] = (float)si;
            t = u;
        }
    }
    g_cache = MtxEntries{};
    return DIA_OK;
}

}  // namespace

extern "C" int dia_mtx_read(const char* path, int64_t* n_rows, int64_t* n_cols, int* num_diags,
                            int* h_offsets, float* h_vals, int64_t stride)
{
    return read_into("dia_mtx_read", path, n_rows, n_cols, num_diags, h_offsets, h_vals, stride,
                     1, nullptr);
}

extern "C" int dia_mtx_read_c64(const char* path, int64_t* n_rows, int64_t* n_cols, int* num_diags,
                                int* h_offsets, float* h_vals, int64_t stride, int* is_complex)
{
    return read_into("dia_mtx_read_c64", path, n_rows, n_cols, num_diags, h_offsets, h_vals,
                     stride, 2, is_complex);
}

/* The inverse: a rows-layout matrix (host buffers) written as a coordinate
 * real general file, entries row by row with offsets ascending -- the order
 * spmv/tools/gen_banded_mtx.cpp writes -- values with 9 significant digits
 * (enough to read every fp32 value back exactly).  Entries outside the
 * matrix are skipped; stored zeros are kept, so the file's structure is the
 * DIA structure. */
extern "C" int dia_mtx_write(const char* path, int64_t n_rows, int64_t n_cols, int num_diags,
                             const int* h_offsets, const float* h_vals, int64_t stride)
{
    if (!path || n_rows < 0 || n_cols < 0 || num_diags < 0 || stride < n_rows ||
        (num_diags > 0 && (!h_offsets || !h_vals)))
        return fail(DIA_ERR_INVALID, "dia_mtx_write: bad arguments");
    std::vector<int> order(num_diags);
    for (int k = 0; k < num_diags; ++k) order[k] = k;
    std::sort(order.begin(), order.end(),
              [&](int a, int b) { return h_offsets[a] < h_offsets[b]; });
    long long nnz = 0;
    for (int k = 0; k < num_diags; ++k) {
        const long long d = h_offsets[k];
        const long long lo = std::max(0LL, -d), hi = std::min((long long)n_rows, n_cols - d);
        if (hi > lo) nnz += hi - lo;
    }
    FILE* f = std::fopen(path, "w");
    if (!f) return fail(DIA_ERR_INVALID, std::string("dia_mtx_write: cannot open ") + path);
    std::fprintf(f, "%%%%MatrixMarket matrix coordinate real general\n");
    std::fprintf(f, "%% written by diagpu_b200 from %d stored diagonals\n", num_diags);
    std::fprintf(f, "%lld %lld %lld\n", (long long)n_rows, (long long)n_cols, nnz);
    for (int64_t i = 0; i < n_rows; ++i)
        for (int k : order) {
            const int64_t c = i + h_offsets[k];
            if (c < 0 || c >= n_cols) continue;
            std::fprintf(f, "%lld %lld %.9g\n", (long long)(i + 1), (long long)(c + 1),
                         (double)h_vals[(size_t)k * (size_t)stride + (size_t)i]);
        }
    const bool ok = std::ferror(f) == 0;
    std::fclose(f);
    return ok ? DIA_OK : fail(DIA_ERR_INVALID, "dia_mtx_write: write error");
}
