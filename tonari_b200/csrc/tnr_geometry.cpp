// Periodic metadata on the host.  See tnr_geometry.h.
//
// The dual of the active rows is computed with the same one-sided Jacobi
// rotation sequence, convergence test and long-double arithmetic as tonari
// csrc/core/geometry.cpp:37-141, because the wraps floor(position . dual)
// and the image ranges must come out bit-identical to the reference's.
// Structures are independent, so large batches are split over host threads.
#include "tnr_geometry.h"
#include "tnr_pool.h"

#include <algorithm>
#include <cmath>
#include <string>
#include <limits>
#include <mutex>

namespace tnr {
namespace {

constexpr int64_t kImageLimit = int64_t{1} << 24;

// Returns false when the active rows are linearly dependent.
bool dual_of_active_rows(const double* cell, const int* axes, int count,
                         long double (&dual)[3][3]) {
    long double basis[3][3] = {};   // basis[cartesian][column]
    long double rotation[3][3] = {};  // accumulated right rotations
    for (int column = 0; column < count; ++column) {
        rotation[column][column] = 1.0L;
        for (int c = 0; c < 3; ++c) {
            basis[c][column] = static_cast<long double>(cell[3 * axes[column] + c]);
        }
    }
    const long double eps = std::numeric_limits<double>::epsilon();
    for (int sweep = 0; sweep < 64; ++sweep) {
        bool rotated = false;
        for (int p = 0; p < count; ++p) {
            for (int q = p + 1; q < count; ++q) {
                long double npp = 0.0L, nqq = 0.0L, npq = 0.0L;
                for (int c = 0; c < 3; ++c) {
                    npp += basis[c][p] * basis[c][p];
                    nqq += basis[c][q] * basis[c][q];
                    npq += basis[c][p] * basis[c][q];
                }
                if (std::abs(npq) <= 8 * eps * std::sqrt(npp * nqq)) continue;
                rotated = true;
                const long double tau = (nqq - npp) / (2 * npq);
                const long double t = tau == 0.0L
                    ? 1.0L
                    : std::copysign(1.0L, tau) / (std::abs(tau) + std::hypot(1.0L, tau));
                const long double cs = 1.0L / std::hypot(1.0L, t);
                const long double sn = cs * t;
                for (int c = 0; c < 3; ++c) {
                    const long double a = basis[c][p], b = basis[c][q];
                    basis[c][p] = cs * a - sn * b;
                    basis[c][q] = sn * a + cs * b;
                }
                for (int r = 0; r < count; ++r) {
                    const long double a = rotation[r][p], b = rotation[r][q];
                    rotation[r][p] = cs * a - sn * b;
                    rotation[r][q] = sn * a + cs * b;
                }
            }
        }
        if (!rotated) break;
    }
    long double sigma[3] = {};
    long double largest = 0.0L;
    long double smallest = std::numeric_limits<long double>::infinity();
    for (int column = 0; column < count; ++column) {
        long double n2 = 0.0L;
        for (int c = 0; c < 3; ++c) n2 += basis[c][column] * basis[c][column];
        sigma[column] = std::sqrt(n2);
        largest = std::max(largest, sigma[column]);
        smallest = std::min(smallest, sigma[column]);
    }
    if (!(smallest > eps * 3 * std::max(largest, 1.0L))) return false;
    for (int c = 0; c < 3; ++c) {
        for (int axis = 0; axis < count; ++axis) {
            long double value = 0.0L;
            for (int k = 0; k < count; ++k) {
                value += basis[c][k] * rotation[axis][k] / (sigma[k] * sigma[k]);
            }
            dual[c][axis] = value;
        }
    }
    return true;
}

// Fills duals and repeats of one structure; returns the image count.
int64_t structure_geometry(const double* cell, const uint8_t* pbc, int64_t atoms,
                           double cutoff, double* duals, int32_t* repeats) {
    for (int k = 0; k < 9; ++k) {
        require_input(std::isfinite(cell[k]), "cell must contain only finite values");
    }
    for (int k = 0; k < 9; ++k) duals[k] = 0.0;
    repeats[0] = repeats[1] = repeats[2] = 0;
    if (atoms == 0) return 0;
    int axes[3];
    int active = 0;
    for (int axis = 0; axis < 3; ++axis) {
        if (pbc[axis] != 0) axes[active++] = axis;
    }
    if (active > 0) {
        long double dual[3][3] = {};
        require_input(dual_of_active_rows(cell, axes, active, dual),
                      "active periodic cell vectors must be linearly independent");
        for (int column = 0; column < active; ++column) {
            long double norm2 = 0.0L;
            for (int c = 0; c < 3; ++c) {
                const long double v = dual[c][column];
                require_input(std::isfinite(v) && std::abs(v) <= std::numeric_limits<double>::max(),
                              "active periodic cell dual is outside the float64 range");
                duals[3 * c + axes[column]] = static_cast<double>(v);
                norm2 += v * v;
            }
            const long double repeat = std::ceil(cutoff * std::sqrt(norm2));
            require_input(repeat <= std::numeric_limits<int32_t>::max(),
                          "periodic image range exceeds int32 cell shifts");
            repeats[axes[column]] = static_cast<int32_t>(repeat);
        }
    }
    int64_t images = 1;
    for (int axis = 0; axis < 3; ++axis) {
        const int64_t factor = 2 * static_cast<int64_t>(repeats[axis]) + 1;
        require_input(images <= kImageLimit / factor,
                      "periodic image count exceeds the 2^24 resource limit");
        images *= factor;
    }
    return images;
}

}  // namespace

PeriodicGeometry build_geometry(const double* cells, const uint8_t* pbc,
                                const int64_t* atom_counts, int64_t batch, double cutoff) {
    PeriodicGeometry geometry;
    geometry.duals.assign(static_cast<size_t>(9 * batch), 0.0);
    geometry.repeats.assign(static_cast<size_t>(3 * batch), 0);
    std::vector<int64_t> images(static_cast<size_t>(batch), 0);

    // Per-structure work runs on host threads for large batches; errors are
    // reported in batch order, as the reference's sequential loop does, by
    // keeping the lowest failing structure and interleaving the batched image
    // limit check at its position.
    int64_t failed_at = batch;
    std::string failure;
    std::mutex guard;
    auto run = [&](int64_t begin, int64_t end) {
        for (int64_t b = begin; b < end; ++b) {
            try {
                images[b] = structure_geometry(cells + 9 * b, pbc + 3 * b, atom_counts[b],
                                               cutoff, geometry.duals.data() + 9 * b,
                                               geometry.repeats.data() + 3 * b);
            } catch (const InputError& error) {
                std::lock_guard<std::mutex> lock(guard);
                if (b < failed_at) {
                    failed_at = b;
                    failure = error.what();
                }
                return;
            }
        }
    };
    HostPool::instance().parallel_for(batch, 16, run);
    geometry.image_begin.assign(static_cast<size_t>(batch + 1), 0);
    for (int64_t b = 0; b < batch; ++b) {
        if (b == failed_at) throw InputError(failure);
        require_input(geometry.image_begin[b] <= kImageLimit - images[b],
                      "batched periodic image count exceeds the 2^24 resource limit");
        geometry.image_begin[b + 1] = geometry.image_begin[b] + images[b];
    }
    return geometry;
}

}  // namespace tnr
