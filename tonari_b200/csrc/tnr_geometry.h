// Host-side periodic metadata for the B200 provider.
//
// Restates tonari csrc/core/geometry.cpp:146-241 (build_periodic_metadata):
// per structure, the pseudo-inverse of the active cell rows ("duals", stored
// duals[9b + 3*cartesian + axis], zero on inactive axes), the image repeat
// count ceil(cutoff * |dual column|) per active axis and the 2^24 image limit.
// The duals must be bit-identical to the reference's because atom wraps are
// floor(position . dual_T); the one-sided Jacobi steps are therefore the same
// (see tnr_geometry.cpp).  Unlike the reference, the image shifts are not
// materialised per structure here: the device enumerates them from the
// repeats (x-major, then y, then z, the reference's order).
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace tnr {

// InputError -> TNR_INPUT_ERROR (Python ValueError); SearchError ->
// TNR_SEARCH_ERROR (Python RuntimeError).  Mirrors tonari csrc/core/errors.h.
struct InputError : std::runtime_error {
    using std::runtime_error::runtime_error;
};
struct SearchError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

inline void require_input(bool condition, const char* message) {
    if (!condition) throw InputError(message);
}
inline void require_search(bool condition, const char* message) {
    if (!condition) throw SearchError(message);
}

struct PeriodicGeometry {
    std::vector<double> duals;         // (B,3,3) [b][cartesian][axis]
    std::vector<int32_t> repeats;      // (B,3)
    std::vector<int64_t> image_begin;  // (B+1) prefix of per-structure image counts
};

// cells (B,3,3) float64, pbc (B,3) bytes, atom_counts (B).
PeriodicGeometry build_geometry(const double* cells, const uint8_t* pbc,
                                const int64_t* atom_counts, int64_t batch, double cutoff);

}  // namespace tnr
