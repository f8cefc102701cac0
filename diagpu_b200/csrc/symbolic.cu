/*
 * symbolic.cu -- host-side symbolic phase of C = A*B (integer work, exact).
 *
 * Output offsets: the ascending set {da + db : -n < da + db < n}, the same
 * set make_c_structure (spmspm/bench_spmspm.cu:109-131),
 * compute_c_hm_structure (spmspm/paper_hm.cuh:87-117) and build_c_layout
 * (gemm_diag/gemm_diag.cu:387-423) produce, with lengths n - |d| and 64-bit
 * HM starts (the reference's int starts overflow beyond 2^31 values).
 * Instead of the reference's 2n-1 presence array (537 MB at n = 67M) the set
 * is formed by sorting the nA*nB sums, so the cost is independent of n.
 * Pairs per output diagonal are listed in A storage order, the order
 * cpu_dia_spgemm (spmspm/bench_spmspm.cu:392-403) accumulates them.
 */
#include <algorithm>
#include <cstdint>
#include <vector>

#include "../../include/diagpu_b200.h"
#include "dia_core.cuh"

using namespace dia;

namespace {
bool has_repeats(const int* off, int k)
{
    std::vector<int> v(off, off + k);
    std::sort(v.begin(), v.end());
    return std::adjacent_find(v.begin(), v.end()) != v.end();
}
}  // namespace

extern "C" int dia_spmspm_symbolic(int n, const int* h_A_off, int nA, const int* h_B_off, int nB,
                                   int* n_c, int* h_C_off, int* h_C_len, int64_t* h_C_start,
                                   int64_t* n_pairs, int* h_pair_ptr, int* h_pair_a,
                                   int* h_pair_b)
{
    if (n < 0 || nA < 0 || nB < 0) return fail(DIA_ERR_INVALID, "dia_spmspm_symbolic: negative size");
    if (!n_c || !n_pairs) return fail(DIA_ERR_INVALID, "dia_spmspm_symbolic: null count pointer");
    if ((nA > 0 && !h_A_off) || (nB > 0 && !h_B_off))
        return fail(DIA_ERR_INVALID, "dia_spmspm_symbolic: null offsets");
    if (has_repeats(h_A_off, nA) || has_repeats(h_B_off, nB))
        return fail(DIA_ERR_INVALID, "dia_spmspm_symbolic: repeated diagonal offset");

    struct Trip { long long dc; int a, b; };
    std::vector<Trip> t;
    t.reserve((size_t)nA * nB);
    for (int a = 0; a < nA; ++a)
        for (int b = 0; b < nB; ++b) {
            const long long dc = (long long)h_A_off[a] + h_B_off[b];
            if (dc > -(long long)n && dc < (long long)n) t.push_back({dc, a, b});
        }
    /* stable: within one output diagonal, pairs keep ascending a */
    std::stable_sort(t.begin(), t.end(), [](const Trip& x, const Trip& y) { return x.dc < y.dc; });

    int nc = 0;
    for (size_t i = 0; i < t.size(); ++i)
        if (i == 0 || t[i].dc != t[i - 1].dc) ++nc;
    const int cap_c = *n_c;
    const int64_t cap_p = *n_pairs;
    *n_c = nc;
    *n_pairs = (int64_t)t.size();
    const bool want_c = h_C_off || h_C_len || h_C_start || h_pair_ptr;
    const bool want_p = h_pair_a || h_pair_b;
    if (!want_c && !want_p) return DIA_OK;
    if (want_c && cap_c < nc)
        return fail(DIA_ERR_CAPACITY, "dia_spmspm_symbolic: C arrays smaller than *n_c");
    if (want_p && cap_p < (int64_t)t.size())
        return fail(DIA_ERR_CAPACITY, "dia_spmspm_symbolic: pair arrays smaller than *n_pairs");

    int c = -1;
    int64_t start = 0;
    for (size_t i = 0; i < t.size(); ++i) {
        if (i == 0 || t[i].dc != t[i - 1].dc) {
            ++c;
            const int d = (int)t[i].dc;
            const int len = n - (d < 0 ? -d : d);
            if (h_C_off) h_C_off[c] = d;
            if (h_C_len) h_C_len[c] = len;
            if (h_C_start) h_C_start[c] = start;
            if (h_pair_ptr) h_pair_ptr[c] = (int)i;
            start += len;
        }
        if (h_pair_a) h_pair_a[i] = t[i].a;
        if (h_pair_b) h_pair_b[i] = t[i].b;
    }
    if (h_pair_ptr) h_pair_ptr[nc] = (int)t.size();
    return DIA_OK;
}
