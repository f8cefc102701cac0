/*
 * io_pauli.cu -- Pauli-string Hamiltonians into the DIA rows layout (host).
 *
 * The operators the reference's DIA format is built for (HamLib spin,
 * QUBO and molecular Hamiltonians) are sums H = sum_t c_t P_t of Pauli
 * strings on q qubits, n = 2^q.  In the symplectic form a string is two bit
 * masks: x (qubits carrying X or Y) and z (qubits carrying Z or Y); with
 * qubit k on bit k of the basis index (the convention of the reference's
 * talk: an X or Y on qubit k moves the column by +-2^k),
 *     P |c> = i^popcount(x & z) * (-1)^popcount(c & z) |c XOR x>,
 * so row r of P has its single entry in column c = r XOR x, on diagonal
 * d = c - r, and a string spans the 2^popcount(x) diagonals
 * sum_k (+-2^k) over the bits k of x.  This file enumerates those
 * offsets, then accumulates every term's entries row by row -- in double
 * complex, terms in input order, one rounding to complex64 at the end --
 * into vals[k*stride + r] (interleaved re, im).  is_real reports whether
 * every imaginary part is exactly zero, so real operators can take the
 * fp32 paths.  Two calls: sizes first (no value buffers), then the fill.
 */
#include <algorithm>
#include <complex>
#include <cstdint>
#include <cstring>
#include <unordered_map>
#include <vector>

#include "../../include/diagpu_b200.h"
#include "dia_core.cuh"

namespace {

constexpr size_t kMaxDiags = (size_t)1 << 16;
/* pattern-to-diagonal tables of all distinct X masks together */
constexpr size_t kMaxPatterns = (size_t)1 << 26;

/* every offset sum_k s_k 2^k over the bits k of x, s_k = +1 or -1, in
 * ascending order (x has at most 16 bits here, so at most 65536 offsets) */
void string_offsets(uint64_t x, std::vector<int64_t>& out)
{
    out.assign(1, 0);
    for (int k = 0; k < 64; ++k) {
        if (!((x >> k) & 1)) continue;
        const int64_t w = (int64_t)1 << k;
        const size_t m = out.size();
        out.resize(2 * m);
        for (size_t i = 0; i < m; ++i) {
            out[m + i] = out[i] + w;
            out[i] -= w;
        }
    }
    std::sort(out.begin(), out.end());
}

int pauli_to_dia(int nq, int nterms, const uint64_t* h_x_mask, const uint64_t* h_z_mask,
                 const double* h_coef_re, const double* h_coef_im, int* num_diags,
                 int* h_offsets, float* h_vals, int64_t stride, int* is_real);

}  // namespace

using namespace dia;

/* Host memory use is bounded before anything large is built: a string with
 * more than 16 X/Y factors alone spans more than 65536 diagonals and is
 * rejected at once, the offset set is merged term by term and the call
 * stops as soon as it passes 65536, and the per-mask pattern tables are
 * shared by terms with the same X mask and capped in total.  An allocation
 * failure anyway becomes DIA_ERR_UNSUPPORTED instead of an exception
 * leaving the C interface. */
extern "C" int dia_pauli_to_dia(int nq, int nterms, const uint64_t* h_x_mask,
                                const uint64_t* h_z_mask, const double* h_coef_re,
                                const double* h_coef_im, int* num_diags, int* h_offsets,
                                float* h_vals, int64_t stride, int* is_real)
{
    try {
        return pauli_to_dia(nq, nterms, h_x_mask, h_z_mask, h_coef_re, h_coef_im, num_diags,
                            h_offsets, h_vals, stride, is_real);
    } catch (const std::bad_alloc&) {
        return fail(DIA_ERR_UNSUPPORTED, "dia_pauli_to_dia: out of host memory");
    }
}

namespace {

int pauli_to_dia(int nq, int nterms, const uint64_t* h_x_mask,
                                const uint64_t* h_z_mask, const double* h_coef_re,
                                const double* h_coef_im, int* num_diags, int* h_offsets,
                                float* h_vals, int64_t stride, int* is_real)
{
    if (nq < 1 || nq > 30 || nterms < 0 || !num_diags)
        return fail(DIA_ERR_INVALID, "dia_pauli_to_dia: need 1 <= nq <= 30 and num_diags");
    if (nterms > 0 && (!h_x_mask || !h_z_mask || !h_coef_re))
        return fail(DIA_ERR_INVALID, "dia_pauli_to_dia: null term arrays");
    const int64_t n = (int64_t)1 << nq;
    const uint64_t all = (uint64_t)n - 1;
    for (int t = 0; t < nterms; ++t)
        if ((h_x_mask[t] | h_z_mask[t]) & ~all)
            return fail(DIA_ERR_INVALID, "dia_pauli_to_dia: a string acts on a qubit >= nq");
    static const char* kTooMany =
        "dia_pauli_to_dia: more than 65536 diagonals (strings with many X/Y are not banded; "
        "DIA does not suit them)";
    for (int t = 0; t < nterms; ++t)
        if (__builtin_popcountll(h_x_mask[t]) > 16) return fail(DIA_ERR_UNSUPPORTED, kTooMany);
    /* distinct X masks: terms sharing one share its offsets and tables */
    std::vector<uint64_t> masks(h_x_mask, h_x_mask + nterms);
    std::sort(masks.begin(), masks.end());
    masks.erase(std::unique(masks.begin(), masks.end()), masks.end());
    size_t patterns = 0;
    for (uint64_t x : masks) {
        patterns += (size_t)1 << __builtin_popcountll(x);
        if (patterns > kMaxPatterns)
            return fail(DIA_ERR_UNSUPPORTED, "dia_pauli_to_dia: too many distinct X/Y patterns "
                                             "(more than 2^26 pattern-table entries)");
    }
    std::vector<int64_t> offs, one, merged;
    for (uint64_t x : masks) {
        string_offsets(x, one);
        merged.resize(offs.size() + one.size());
        merged.erase(std::set_union(offs.begin(), offs.end(), one.begin(), one.end(),
                                    merged.begin()),
                     merged.end());
        offs.swap(merged);
        if (offs.size() > kMaxDiags) return fail(DIA_ERR_UNSUPPORTED, kTooMany);
    }
    const int K = (int)offs.size();
    if (!h_offsets && !h_vals) {
        *num_diags = K;
        return DIA_OK;
    }
    if (*num_diags < K) {
        *num_diags = K;
        return fail(DIA_ERR_CAPACITY, "dia_pauli_to_dia: offset buffer smaller than the count");
    }
    *num_diags = K;
    if (h_offsets)
        for (int k = 0; k < K; ++k) h_offsets[k] = (int)offs[k];
    if (!h_vals) return DIA_OK;
    if (stride < n) return fail(DIA_ERR_INVALID, "dia_pauli_to_dia: stride smaller than 2^nq");
    std::unordered_map<int64_t, int> idx;
    for (int k = 0; k < K; ++k) idx[offs[k]] = k;
    static const std::complex<double> ipow[4] = {{1, 0}, {0, 1}, {-1, 0}, {0, -1}};
    std::vector<std::complex<double>> coef((size_t)nterms);
    for (int t = 0; t < nterms; ++t)
        coef[t] = std::complex<double>(h_coef_re[t], h_coef_im ? h_coef_im[t] : 0.0) *
                  ipow[__builtin_popcountll(h_x_mask[t] & h_z_mask[t]) & 3];
    for (int k = 0; k < K; ++k)
        std::memset(h_vals + 2 * (size_t)k * (size_t)stride, 0,
                    2 * (size_t)stride * sizeof(float));
    /* Per term: the diagonal of row r depends only on the bits of r under x.
     * Those bits, compressed to a pattern p (bit j of p = j-th set bit of
     * x), come from four byte tables; kof[p] is the pattern's diagonal
     * index.  No hashing per row. */
    std::vector<uint32_t> byte_tab(masks.size() * 4 * 256);
    std::vector<std::vector<int>> kof(masks.size());
    std::vector<int> mask_of((size_t)nterms);
    for (int t = 0; t < nterms; ++t)
        mask_of[(size_t)t] = (int)(std::lower_bound(masks.begin(), masks.end(), h_x_mask[t]) -
                                   masks.begin());
    for (size_t t = 0; t < masks.size(); ++t) {
        const uint64_t x = masks[t];
        int bits[64], nb = 0;
        for (int k = 0; k < 64; ++k)
            if ((x >> k) & 1) bits[nb++] = k;
        for (int byte = 0; byte < 4; ++byte)
            for (int v = 0; v < 256; ++v) {
                uint32_t pat = 0;
                for (int j = 0; j < nb; ++j) {
                    const int b = bits[j] - 8 * byte;
                    if (b >= 0 && b < 8 && ((v >> b) & 1)) pat |= 1u << j;
                }
                byte_tab[((size_t)t * 4 + byte) * 256 + v] = pat;
            }
        kof[t].resize((size_t)1 << nb);
        for (uint32_t pat = 0; pat < (1u << nb); ++pat) {
            int64_t d = 0;   /* bit set in the row: column = row - 2^k, else + 2^k */
            for (int j = 0; j < nb; ++j)
                d += ((pat >> j) & 1) ? -((int64_t)1 << bits[j]) : ((int64_t)1 << bits[j]);
            kof[t][pat] = idx[d];
        }
    }
    /* rows in chunks, so the double accumulator (K x chunk) stays near 16 MB
     * and in cache: a power of two between 256 rows and 2^16 */
    int64_t chunk = 256;
    while (chunk < ((int64_t)1 << 16) && (chunk * 2) * K * 16 <= ((int64_t)16 << 20)) chunk *= 2;
    chunk = std::min<int64_t>(n, chunk);
    std::vector<std::complex<double>> acc((size_t)K * (size_t)chunk);
    bool real = true;
    for (int64_t r0 = 0; r0 < n; r0 += chunk) {
        std::fill(acc.begin(), acc.end(), std::complex<double>(0.0, 0.0));
        for (int t = 0; t < nterms; ++t) {
            const uint64_t x = h_x_mask[t], z = h_z_mask[t];
            const int m = mask_of[(size_t)t];
            const uint32_t* tab = &byte_tab[(size_t)m * 4 * 256];
            const int* kt = kof[(size_t)m].data();
            const std::complex<double> c = coef[t], mc = -coef[t];
            for (int64_t r = r0; r < r0 + chunk; ++r) {
                const uint64_t col = (uint64_t)r ^ x;
                const uint32_t ur = (uint32_t)r;
                const uint32_t pat = tab[ur & 255] | tab[256 + ((ur >> 8) & 255)] |
                                     tab[512 + ((ur >> 16) & 255)] | tab[768 + (ur >> 24)];
                acc[(size_t)kt[pat] * chunk + (size_t)(r - r0)] +=
                    __builtin_parityll(col & z) ? mc : c;
            }
        }
        for (int k = 0; k < K; ++k) {
            float* row = h_vals + 2 * (size_t)k * (size_t)stride;
            for (int64_t r = r0; r < r0 + chunk; ++r) {
                const std::complex<double> v = acc[(size_t)k * chunk + (size_t)(r - r0)];
                row[2 * r] = (float)v.real();
                row[2 * r + 1] = (float)v.imag();
                real = real && row[2 * r + 1] == 0.0f;
            }
        }
    }
    if (is_real) *is_real = real ? 1 : 0;
    return DIA_OK;
}

}  // namespace
