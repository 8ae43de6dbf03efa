// TEST INFRASTRUCTURE ONLY. A C-ABI shim over the reference's own CPU search
// core (tonari csrc/core/neighbors_cpu.cpp:976-1030, geometry.cpp:146-242),
// compiled together with those unmodified sources by oracle/Makefile into
// oracle/_ref/libtonari_ref.so.  It is the bit-exact pair-set oracle and the
// timed CPU baseline ("kind": "reference"); the product never links it.
//
// The shim mirrors what the reference's Torch-CPU binding does
// (csrc/torch/bindings_cpu.cpp:17-70): convert pbc to bytes, call
// neighbor_list_cpu<T>, then copy_pair_buffers into caller-owned arrays.
// Because the pair count is only known after the search, the result is held
// in an opaque handle until the caller has allocated the output arrays.

#include "neighbors_cpu.h"
#include "errors.h"

#include <cstdint>
#include <cstring>
#include <exception>
#include <new>
#include <span>
#include <string>
#include <vector>

namespace {

struct RefResult {
    neighbor_search::PairBuffers pairs;
    int64_t threads = 1;
};

void set_error(char* buffer, size_t length, const char* message) {
    if (buffer == nullptr || length == 0) {
        return;
    }
    std::strncpy(buffer, message, length - 1);
    buffer[length - 1] = '\0';
}

}  // namespace

extern "C" {

// Status: 0 ok, 1 InputError (Python ValueError), 2 SearchError
// (RuntimeError), 3 other failure.
int tnr_ref_neighbor_list(
    int dtype_is_f64,
    const void* positions,
    int64_t n_atoms,
    const int64_t* batch_ptr,
    int64_t n_structures,
    const void* cell,
    const uint8_t* pbc,
    double cutoff,
    int half_list,
    int include_self,
    int algorithm,
    int64_t num_threads,
    void** handle,
    int64_t* n_pairs,
    char* error,
    size_t error_length) {
    *handle = nullptr;
    *n_pairs = 0;
    try {
        auto* result = new RefResult();
        result->threads = num_threads;
        const auto mode = neighbor_search::pair_mode(half_list != 0, include_self != 0);
        const auto parsed = algorithm == 1
            ? neighbor_search::Algorithm::BruteForce
            : (algorithm == 2 ? neighbor_search::Algorithm::CellList
                              : neighbor_search::Algorithm::Auto);
        std::span<const int64_t> ptr(batch_ptr, static_cast<size_t>(n_structures + 1));
        std::span<const uint8_t> flags(pbc, static_cast<size_t>(3 * n_structures));
        try {
            if (dtype_is_f64) {
                result->pairs = neighbor_search::neighbor_list_cpu<double>(
                    std::span(static_cast<const double*>(positions), static_cast<size_t>(3 * n_atoms)),
                    ptr,
                    std::span(static_cast<const double*>(cell), static_cast<size_t>(9 * n_structures)),
                    flags, cutoff, mode, parsed, num_threads);
            } else {
                result->pairs = neighbor_search::neighbor_list_cpu<float>(
                    std::span(static_cast<const float*>(positions), static_cast<size_t>(3 * n_atoms)),
                    ptr,
                    std::span(static_cast<const float*>(cell), static_cast<size_t>(9 * n_structures)),
                    flags, cutoff, mode, parsed, num_threads);
            }
        } catch (...) {
            delete result;
            throw;
        }
        *handle = result;
        *n_pairs = static_cast<int64_t>(result->pairs.pair_count);
        return 0;
    } catch (const neighbor_search::InputError& e) {
        set_error(error, error_length, e.what());
        return 1;
    } catch (const neighbor_search::SearchError& e) {
        set_error(error, error_length, e.what());
        return 2;
    } catch (const std::exception& e) {
        set_error(error, error_length, e.what());
        return 3;
    }
}

// Copies the held result into pairs (n_pairs, 2) int64 and shifts
// (n_pairs, 3) int32 and releases the handle.
int tnr_ref_take(void* handle, int64_t* pairs, int32_t* shifts, char* error, size_t error_length) {
    auto* result = static_cast<RefResult*>(handle);
    try {
        const size_t count = result->pairs.pair_count;
        neighbor_search::copy_pair_buffers(
            result->pairs,
            std::span(pairs, 2 * count),
            std::span(shifts, 3 * count),
            result->threads);
        delete result;
        return 0;
    } catch (const std::exception& e) {
        delete result;
        set_error(error, error_length, e.what());
        return 3;
    }
}

void tnr_ref_release(void* handle) {
    delete static_cast<RefResult*>(handle);
}

}  // extern "C"
