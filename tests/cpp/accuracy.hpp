// Accuracy comparison for the C++ parity tests (test infrastructure).
//
// Same pass rule as the reference harness's accuracy::CompareArrays
// (include/harness/accuracy.hpp:62-125): element i fails only when BOTH its absolute error
// exceeds abs_tol AND its relative error (to |expected|, or to |actual| when expected is ~0)
// exceeds rel_tol.  In addition to the failing-element maxima the reference reports, the report
// carries the maximum absolute and relative error over ALL elements, which the parity tests
// print beside every result.
#pragma once

#include <cmath>
#include <cstddef>
#include <sstream>
#include <string>
#include <vector>

namespace harness {
namespace accuracy {

struct Tolerance {
    double abs_tol;
    double rel_tol;
};

struct AccuracyReport {
    bool passed = true;
    size_t num_elements = 0;
    size_t mismatch_count = 0;
    double max_abs_error = 0.0;  // over failing elements (reference semantics)
    double max_rel_error = 0.0;
    size_t first_mismatch = 0;
    double global_max_abs = 0.0;  // over all elements
    double global_max_rel = 0.0;

    std::string ToString() const {
        std::ostringstream s;
        s << "AccuracyReport{passed=" << (passed ? "true" : "false") << ", elements=" << num_elements
          << ", mismatches=" << mismatch_count << ", max_abs_err=" << max_abs_error << ", max_rel_err=" << max_rel_error;
        if (mismatch_count) s << ", first_mismatch=" << first_mismatch;
        s << ", all_max_abs=" << global_max_abs << ", all_max_rel=" << global_max_rel << "}";
        return s.str();
    }
};

template <class T>
AccuracyReport CompareArrays(const T* expected, const T* actual, size_t n, Tolerance tol) {
    AccuracyReport r;
    r.num_elements = n;
    for (size_t i = 0; i < n; ++i) {
        const double e = static_cast<double>(expected[i]);
        const double a = static_cast<double>(actual[i]);
        const double abs_err = std::fabs(e - a);
        double rel_err = 0.0;
        if (std::fabs(e) > 1e-12)
            rel_err = abs_err / std::fabs(e);
        else if (std::fabs(a) > 1e-12)
            rel_err = abs_err / std::fabs(a);
        const bool nan_mismatch = std::isnan(e) != std::isnan(a);
        if (abs_err > r.global_max_abs) r.global_max_abs = abs_err;
        if (rel_err > r.global_max_rel) r.global_max_rel = rel_err;
        if (nan_mismatch || (abs_err > tol.abs_tol && rel_err > tol.rel_tol)) {
            if (r.mismatch_count == 0) r.first_mismatch = i;
            ++r.mismatch_count;
            if (abs_err > r.max_abs_error) r.max_abs_error = abs_err;
            if (rel_err > r.max_rel_error) r.max_rel_error = rel_err;
        }
    }
    r.passed = r.mismatch_count == 0;
    return r;
}

template <class T>
AccuracyReport CompareArrays(const std::vector<T>& expected, const std::vector<T>& actual, Tolerance tol) {
    if (expected.size() != actual.size()) {
        AccuracyReport r;
        r.passed = false;
        r.mismatch_count = 1;
        r.max_abs_error = INFINITY;
        return r;
    }
    return CompareArrays(expected.data(), actual.data(), expected.size(), tol);
}

}  // namespace accuracy
}  // namespace harness
