// xspmm/io/matrix_market.hpp -- Matrix Market (coordinate) reader into a host CSR, header-only.
//
// Same acceptance rules and result as the reference's utils/matrix_io.hpp:27-98
// (matrix_utils::io::read_mtx), so that code following its examples/04 flow
//   auto h = read_mtx<float>(path);  CSRMatrix<float, int32_t> A(exec, h.num_rows, ...);
//   A.copy_from_host(h.row_ptr.data(), h.col_ind.data(), h.values.data());
// gets the same matrix:
//   * lines that are empty or start with '%' are skipped; the first other line holds
//     "rows cols nnz" (std::runtime_error if it does not parse);
//   * an entry line is "row col [value]" (1-based); the fields are read one after another like
//     istream extractions (skip blanks, longest numeric prefix); a line without two integers is
//     skipped, a missing or unreadable value is 1.0, entries outside the matrix are dropped;
//   * values are read as float (correctly rounded, as strtof) and converted to T;
//   * entries sorted by (row, col), int32 indices; duplicates keep their file order (stable
//     sort; the reference's std::sort leaves that order unspecified).
// The names are also provided in namespace matrix_utils::io for code written against the
// reference's utility header.
#pragma once

#include <algorithm>
#include <cctype>
#include <cerrno>
#include <cstdint>
#include <cstdlib>
#include <fstream>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

namespace xspmm {
namespace io {

template <typename T>
struct HostCSRMatrix {
    int num_rows = 0;
    int num_cols = 0;
    std::vector<int> row_ptr;
    std::vector<int> col_ind;
    std::vector<T> values;
};

namespace detail {

inline const char* skip_blank(const char* p) {
    while (*p && std::isspace(static_cast<unsigned char>(*p))) ++p;
    return p;
}

// istream >> int: optional sign then decimal digits; false (and p unchanged) if none or if the
// value does not fit an int.
inline bool read_int(const char*& p, int& out) {
    const char* q = skip_blank(p);
    const char* d = q + ((*q == '+' || *q == '-') ? 1 : 0);
    if (!std::isdigit(static_cast<unsigned char>(*d))) return false;
    errno = 0;
    char* end = nullptr;
    const long v = std::strtol(q, &end, 10);
    if (errno == ERANGE || v < INT32_MIN || v > INT32_MAX) return false;
    out = static_cast<int>(v);
    p = end;
    return true;
}

// istream >> float for plain decimal text: [+-](digits[.digits] | .digits)[e[+-]digits]; false
// if there is no number or the exponent has no digits.
inline bool read_float(const char* p, float& out) {
    const char* q = skip_blank(p);
    const char* s = q;
    if (*s == '+' || *s == '-') ++s;
    const char* m = s;
    while (std::isdigit(static_cast<unsigned char>(*m))) ++m;
    bool digits = m > s;
    if (*m == '.') {
        ++m;
        const char* f = m;
        while (std::isdigit(static_cast<unsigned char>(*m))) ++m;
        digits = digits || m > f;
    }
    if (!digits) return false;
    if (*m == 'e' || *m == 'E') {
        // an exponent marker is taken into the number by the stream; without digits after it
        // the extraction fails
        const char* e = m + 1;
        if (*e == '+' || *e == '-') ++e;
        if (!std::isdigit(static_cast<unsigned char>(*e))) return false;
        while (std::isdigit(static_cast<unsigned char>(*e))) ++e;
        m = e;
    }
    const std::string tok(q, m);
    out = std::strtof(tok.c_str(), nullptr);
    return true;
}

}  // namespace detail

template <typename T>
HostCSRMatrix<T> read_mtx(const std::string& filename) {
    std::ifstream file(filename);
    if (!file.is_open()) throw std::runtime_error("Could not open MTX file: " + filename);
    std::string line;
    int rows = 0, cols = 0, nnz_hint = 0;
    bool have_dims = false;
    while (std::getline(file, line)) {
        if (line.empty() || line[0] == '%') continue;
        const char* p = line.c_str();
        if (!detail::read_int(p, rows) || !detail::read_int(p, cols) ||
            !detail::read_int(p, nnz_hint))
            throw std::runtime_error("Failed to parse MTX dimensions.");
        have_dims = true;
        break;
    }
    if (!have_dims) throw std::runtime_error("Failed to parse MTX dimensions.");

    struct Entry {
        int r, c;
        float v;
    };
    std::vector<Entry> e;
    if (nnz_hint > 0) e.reserve(static_cast<size_t>(nnz_hint));
    while (std::getline(file, line)) {
        if (line.empty() || line[0] == '%') continue;
        const char* p = line.c_str();
        int r = 0, c = 0;
        if (!detail::read_int(p, r) || !detail::read_int(p, c)) continue;
        float v = 1.0f;
        if (!detail::read_float(p, v)) v = 1.0f;
        if (r < 1 || r > rows || c < 1 || c > cols) continue;
        e.push_back({r - 1, c - 1, v});
    }
    std::stable_sort(e.begin(), e.end(), [](const Entry& a, const Entry& b) {
        return a.r != b.r ? a.r < b.r : a.c < b.c;
    });

    HostCSRMatrix<T> csr;
    csr.num_rows = rows;
    csr.num_cols = cols;
    csr.row_ptr.assign(static_cast<size_t>(rows) + 1, 0);
    csr.col_ind.reserve(e.size());
    csr.values.reserve(e.size());
    for (const Entry& x : e) {
        csr.col_ind.push_back(x.c);
        csr.values.push_back(static_cast<T>(x.v));
        ++csr.row_ptr[static_cast<size_t>(x.r) + 1];
    }
    for (int i = 0; i < rows; ++i) csr.row_ptr[i + 1] += csr.row_ptr[i];
    return csr;
}

}  // namespace io
}  // namespace xspmm

namespace matrix_utils {
namespace io {
using xspmm::io::HostCSRMatrix;
using xspmm::io::read_mtx;
}  // namespace io
}  // namespace matrix_utils
