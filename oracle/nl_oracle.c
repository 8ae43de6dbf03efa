/*
 * TEST INFRASTRUCTURE ONLY -- a CPU restatement of tonari's neighbor-list
 * semantics, used as the checker in tests/, in __graft_entry__.smoke() and as
 * the "port" CPU baseline in bench.py.  The product (tonari_b200) never links,
 * loads or calls this file.
 *
 * Parity is pinned: tests/test_oracle.py checks this restatement against the
 * reference's own CPU core (oracle/_ref, compiled from the reference sources)
 * and against the committed golden fixtures in tests/golden/.
 *
 * What is restated (reference file:line):
 *   - periodic metadata: active-row pseudo-inverse by one-sided Jacobi in
 *     long double, dual layout duals[9b + 3*cart + axis], repeats
 *     ceil(cutoff*|dual column|), image count limit 2^24 and x-major image
 *     enumeration                       csrc/core/geometry.cpp:37-241
 *   - representative wraps floor(sum_c pos_c * dual_T[c][a]) in long double
 *                                        csrc/core/neighbors_cpu.cpp:92-133
 *   - candidate evaluation: output shift = image - wrap_t + wrap_s, pair
 *     identity policy, public displacement formula evaluated in T without
 *     contraction, strict d^2 < (T)(cutoff*cutoff), int32 output check
 *                                        csrc/core/neighbors_cpu.cpp:222-273
 *                                        csrc/core/pair_policy.h:42-79
 *   - brute-force loop order source -> target -> image
 *                                        csrc/core/neighbors_cpu.cpp:330-361
 *   - input checks and their messages    csrc/core/neighbors_cpu.cpp:986-1013
 *
 * The restatement always uses the brute-force enumeration: the reference's
 * cell list is a candidate filter whose final decision is the same public
 * formula, so the pair set is the same.  Build with -ffp-contract=off.
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_OK 0
#define ORACLE_INPUT_ERROR 1
#define ORACLE_SEARCH_ERROR 2
#define ORACLE_ALLOC_ERROR 3

static const int64_t kMaximumImageShifts = (int64_t)1 << 24;

typedef struct {
    char* message;
    size_t length;
} error_sink;

static int fail(error_sink* sink, int status, const char* message) {
    if (sink->message && sink->length) {
        strncpy(sink->message, message, sink->length - 1);
        sink->message[sink->length - 1] = '\0';
    }
    return status;
}

/* geometry.cpp:37-141.  Returns 0 on success, -1 if the active rows are
 * linearly dependent. */
static int active_pseudoinverse(const double* cell, const int* axes, int count,
                                long double dual[3][3]) {
    long double columns[3][3] = {{0}};
    long double right[3][3] = {{0}};
    for (int column = 0; column < count; ++column) {
        right[column][column] = 1.0L;
        for (int c = 0; c < 3; ++c) {
            columns[c][column] = (long double)cell[3 * axes[column] + c];
        }
    }
    for (int sweep = 0; sweep < 64; ++sweep) {
        int converged = 1;
        for (int first = 0; first < count; ++first) {
            for (int second = first + 1; second < count; ++second) {
                long double nf = 0.0L, ns = 0.0L, inner = 0.0L;
                for (int c = 0; c < 3; ++c) {
                    nf += columns[c][first] * columns[c][first];
                    ns += columns[c][second] * columns[c][second];
                    inner += columns[c][first] * columns[c][second];
                }
                const long double scale = sqrtl(nf * ns);
                if (fabsl(inner) <= 8 * DBL_EPSILON * scale) {
                    continue;
                }
                converged = 0;
                const long double tau = (ns - nf) / (2 * inner);
                const long double tangent = tau == 0.0L
                    ? 1.0L
                    : copysignl(1.0L, tau) / (fabsl(tau) + hypotl(1.0L, tau));
                const long double cosine = 1.0L / hypotl(1.0L, tangent);
                const long double sine = cosine * tangent;
                for (int c = 0; c < 3; ++c) {
                    const long double a = columns[c][first];
                    const long double b = columns[c][second];
                    columns[c][first] = cosine * a - sine * b;
                    columns[c][second] = sine * a + cosine * b;
                }
                for (int row = 0; row < count; ++row) {
                    const long double a = right[row][first];
                    const long double b = right[row][second];
                    right[row][first] = cosine * a - sine * b;
                    right[row][second] = sine * a + cosine * b;
                }
            }
        }
        if (converged) {
            break;
        }
    }
    long double singular[3] = {0};
    long double largest = 0.0L;
    long double smallest = INFINITY;
    for (int column = 0; column < count; ++column) {
        long double norm = 0.0L;
        for (int c = 0; c < 3; ++c) {
            norm += columns[c][column] * columns[c][column];
        }
        singular[column] = sqrtl(norm);
        if (singular[column] > largest) largest = singular[column];
        if (singular[column] < smallest) smallest = singular[column];
    }
    const long double tolerance = DBL_EPSILON * 3 * (largest > 1.0L ? largest : 1.0L);
    if (!(smallest > tolerance)) {
        return -1;
    }
    for (int c = 0; c < 3; ++c) {
        for (int axis = 0; axis < count; ++axis) {
            long double value = 0.0L;
            for (int k = 0; k < count; ++k) {
                value += columns[c][k] * right[axis][k] / (singular[k] * singular[k]);
            }
            dual[c][axis] = value;
        }
    }
    return 0;
}

/* geometry.cpp:146-241: duals (B,3,3) f64, repeats (B,3). */
static int periodic_metadata(const double* cells, const uint8_t* pbc, const int64_t* counts,
                             int64_t batch, double cutoff, double* duals, int64_t* repeats,
                             error_sink* sink) {
    int64_t total_images = 0;
    memset(duals, 0, sizeof(double) * 9 * (size_t)batch);
    memset(repeats, 0, sizeof(int64_t) * 3 * (size_t)batch);
    for (int64_t b = 0; b < batch; ++b) {
        const double* cell = cells + 9 * b;
        for (int k = 0; k < 9; ++k) {
            if (!isfinite(cell[k])) {
                return fail(sink, ORACLE_INPUT_ERROR, "cell must contain only finite values");
            }
        }
        if (counts[b] == 0) {
            continue;
        }
        int axes[3];
        int active = 0;
        for (int a = 0; a < 3; ++a) {
            if (pbc[3 * b + a]) axes[active++] = a;
        }
        int64_t* rep = repeats + 3 * b;
        if (active > 0) {
            long double dual[3][3] = {{0}};
            if (active_pseudoinverse(cell, axes, active, dual) != 0) {
                return fail(sink, ORACLE_INPUT_ERROR,
                            "active periodic cell vectors must be linearly independent");
            }
            for (int column = 0; column < active; ++column) {
                long double norm = 0.0L;
                for (int c = 0; c < 3; ++c) {
                    const long double v = dual[c][column];
                    if (!(isfinite(v) && fabsl(v) <= DBL_MAX)) {
                        return fail(sink, ORACLE_INPUT_ERROR,
                                    "active periodic cell dual is outside the float64 range");
                    }
                    duals[9 * b + 3 * c + axes[column]] = (double)v;
                    norm += v * v;
                }
                const long double repeat = ceill(cutoff * sqrtl(norm));
                if (!(repeat <= 2147483647.0L)) {
                    return fail(sink, ORACLE_INPUT_ERROR,
                                "periodic image range exceeds int32 cell shifts");
                }
                rep[axes[column]] = (int64_t)repeat;
            }
        }
        int64_t images = 1;
        for (int a = 0; a < 3; ++a) {
            const int64_t factor = 2 * rep[a] + 1;
            if (images > kMaximumImageShifts / factor) {
                return fail(sink, ORACLE_INPUT_ERROR,
                            "periodic image count exceeds the 2^24 resource limit");
            }
            images *= factor;
        }
        if (total_images > kMaximumImageShifts - images) {
            return fail(sink, ORACLE_INPUT_ERROR,
                        "batched periodic image count exceeds the 2^24 resource limit");
        }
        total_images += images;
    }
    return ORACLE_OK;
}

/* Growable pair buffer. */
typedef struct {
    int64_t* pairs;
    int32_t* shifts;
    int64_t count;
    int64_t capacity;
} pair_buffer;

static int push_pair(pair_buffer* out, int64_t s, int64_t t, const int64_t* shift) {
    if (out->count == out->capacity) {
        int64_t capacity = out->capacity ? 2 * out->capacity : 1024;
        int64_t* pairs = realloc(out->pairs, sizeof(int64_t) * 2 * (size_t)capacity);
        if (!pairs) return -1;
        out->pairs = pairs;
        int32_t* shifts = realloc(out->shifts, sizeof(int32_t) * 3 * (size_t)capacity);
        if (!shifts) return -1;
        out->shifts = shifts;
        out->capacity = capacity;
    }
    out->pairs[2 * out->count] = s;
    out->pairs[2 * out->count + 1] = t;
    for (int a = 0; a < 3; ++a) out->shifts[3 * out->count + a] = (int32_t)shift[a];
    out->count += 1;
    return 0;
}

/* pair_policy.h:42-79 */
static int keep_identity(int64_t s, int64_t t, const int64_t* shift, int half, int self) {
    const int zero_self = s == t && shift[0] == 0 && shift[1] == 0 && shift[2] == 0;
    if (zero_self) return self;
    if (!half) return 1;
    if (s != t) return s < t;
    for (int a = 0; a < 3; ++a) {
        if (shift[a] != 0) return shift[a] < 0;
    }
    return 1;
}

#define DEFINE_SEARCH(T, NAME)                                                                  \
static int NAME(const T* positions, const int64_t* batch_ptr, int64_t batch, const T* cells,    \
                const double* duals, const int64_t* repeats, double cutoff, int half, int self, \
                pair_buffer* out, error_sink* sink) {                                           \
    const T cutoff_squared = (T)(cutoff * cutoff);                                              \
    const T wrap_bound = (T)2147483648.0;                                                       \
    for (int64_t b = 0; b < batch; ++b) {                                                       \
        const int64_t begin = batch_ptr[b], n = batch_ptr[b + 1] - begin;                       \
        if (n == 0) continue;                                                                   \
        const T* cell = cells + 9 * b;                                                          \
        T dual[9];                                                                              \
        for (int k = 0; k < 9; ++k) dual[k] = (T)duals[9 * b + k];                              \
        int32_t* wraps = malloc(sizeof(int32_t) * 3 * (size_t)n);                               \
        if (!wraps) return fail(sink, ORACLE_ALLOC_ERROR, "out of memory");                     \
        for (int64_t atom = 0; atom < n; ++atom) {                                              \
            const T* p = positions + 3 * (begin + atom);                                        \
            for (int c = 0; c < 3; ++c) {                                                       \
                if (!isfinite(p[c])) {                                                          \
                    free(wraps);                                                                \
                    return fail(sink, ORACLE_SEARCH_ERROR,                                      \
                                "positions must contain only finite values");                   \
                }                                                                               \
            }                                                                                   \
            for (int a = 0; a < 3; ++a) {                                                       \
                long double f = 0.0L;                                                           \
                for (int c = 0; c < 3; ++c) f += (long double)p[c] * (long double)dual[3 * c + a]; \
                if (!(isfinite(f) && f >= -(long double)wrap_bound && f < (long double)wrap_bound)) { \
                    free(wraps);                                                                \
                    return fail(sink, ORACLE_SEARCH_ERROR,                                      \
                        "atom representatives require periodic wraps outside the int32 range"); \
                }                                                                               \
                wraps[3 * atom + a] = (int32_t)floorl(f);                                       \
            }                                                                                   \
        }                                                                                       \
        const int64_t* rep = repeats + 3 * b;                                                   \
        for (int64_t s = 0; s < n; ++s) {                                                       \
            for (int64_t t = 0; t < n; ++t) {                                                   \
                for (int64_t x = -rep[0]; x <= rep[0]; ++x)                                     \
                for (int64_t y = -rep[1]; y <= rep[1]; ++y)                                     \
                for (int64_t z = -rep[2]; z <= rep[2]; ++z) {                                   \
                    const int64_t image[3] = {x, y, z};                                         \
                    int64_t shift[3];                                                           \
                    for (int a = 0; a < 3; ++a)                                                 \
                        shift[a] = image[a] - (int64_t)wraps[3 * t + a] + (int64_t)wraps[3 * s + a]; \
                    if (!keep_identity(s, t, shift, half, self)) continue;                      \
                    const int zero_self = s == t && !shift[0] && !shift[1] && !shift[2];        \
                    if (!zero_self) {                                                           \
                        T d2 = (T)0;                                                            \
                        for (int c = 0; c < 3; ++c) {                                           \
                            T comp = positions[3 * (begin + t) + c] - positions[3 * (begin + s) + c]; \
                            for (int a = 0; a < 3; ++a) comp += (T)shift[a] * cell[3 * a + c];  \
                            d2 += comp * comp;                                                  \
                        }                                                                       \
                        if (d2 >= cutoff_squared) continue;                                     \
                    }                                                                           \
                    for (int a = 0; a < 3; ++a) {                                               \
                        if (shift[a] < INT32_MIN || shift[a] > INT32_MAX) {                     \
                            free(wraps);                                                        \
                            return fail(sink, ORACLE_SEARCH_ERROR,                              \
                                "a cell shift required by the cutoff pairs exceeds the int32 output range"); \
                        }                                                                       \
                    }                                                                           \
                    if (push_pair(out, begin + s, begin + t, shift) != 0) {                     \
                        free(wraps);                                                            \
                        return fail(sink, ORACLE_ALLOC_ERROR, "out of memory");                 \
                    }                                                                           \
                }                                                                               \
            }                                                                                   \
        }                                                                                       \
        free(wraps);                                                                            \
    }                                                                                           \
    return ORACLE_OK;                                                                           \
}

DEFINE_SEARCH(float, search_f32)
DEFINE_SEARCH(double, search_f64)

/* Entry point.  On success *pairs_out / *shifts_out are malloc'd arrays of
 * (n,2) int64 and (n,3) int32 that the caller releases with
 * oracle_free_pairs.  Pairs are source-major. */
int oracle_neighbor_list(int dtype_is_f64, const void* positions, int64_t n_atoms,
                         const int64_t* batch_ptr, int64_t batch, const void* cell,
                         const uint8_t* pbc, double cutoff, int half, int self,
                         int64_t** pairs_out, int32_t** shifts_out, int64_t* n_pairs,
                         char* error, size_t error_length) {
    error_sink sink = {error, error_length};
    *pairs_out = NULL;
    *shifts_out = NULL;
    *n_pairs = 0;
    if (!(isfinite(cutoff) && cutoff > 0)) {
        return fail(&sink, ORACLE_INPUT_ERROR, "cutoff must be finite and positive");
    }
    if (batch_ptr[0] != 0) return fail(&sink, ORACLE_INPUT_ERROR, "batch_ptr must start at zero");
    if (batch_ptr[batch] != n_atoms) {
        return fail(&sink, ORACLE_INPUT_ERROR, "batch_ptr must end at N_total");
    }
    if (n_atoms >= INT32_MAX) {
        return fail(&sink, ORACLE_INPUT_ERROR,
                    "the current implementation supports fewer than 2^31 atoms");
    }
    int64_t* counts = malloc(sizeof(int64_t) * (size_t)(batch + 1));
    double* cells64 = malloc(sizeof(double) * 9 * (size_t)(batch + 1));
    double* duals = malloc(sizeof(double) * 9 * (size_t)(batch + 1));
    int64_t* repeats = malloc(sizeof(int64_t) * 3 * (size_t)(batch + 1));
    int status = ORACLE_OK;
    if (!counts || !cells64 || !duals || !repeats) {
        status = fail(&sink, ORACLE_ALLOC_ERROR, "out of memory");
        goto done;
    }
    for (int64_t b = 0; b < batch; ++b) {
        if (batch_ptr[b + 1] < batch_ptr[b]) {
            status = fail(&sink, ORACLE_INPUT_ERROR, "batch_ptr must be nondecreasing");
            goto done;
        }
        counts[b] = batch_ptr[b + 1] - batch_ptr[b];
    }
    for (int64_t k = 0; k < 9 * batch; ++k) {
        cells64[k] = dtype_is_f64 ? ((const double*)cell)[k] : (double)((const float*)cell)[k];
    }
    status = periodic_metadata(cells64, pbc, counts, batch, cutoff, duals, repeats, &sink);
    if (status != ORACLE_OK) goto done;
    pair_buffer out = {0};
    if (dtype_is_f64) {
        status = search_f64(positions, batch_ptr, batch, cell, duals, repeats, cutoff, half,
                            self, &out, &sink);
    } else {
        status = search_f32(positions, batch_ptr, batch, cell, duals, repeats, cutoff, half,
                            self, &out, &sink);
    }
    if (status != ORACLE_OK) {
        free(out.pairs);
        free(out.shifts);
        goto done;
    }
    *pairs_out = out.pairs;
    *shifts_out = out.shifts;
    *n_pairs = out.count;
done:
    free(counts);
    free(cells64);
    free(duals);
    free(repeats);
    return status;
}

/* Periodic metadata alone (for checking the product's host geometry):
 * duals (B,3,3) f64 and repeats (B,3) int64. */
int oracle_periodic_metadata(const double* cells, const uint8_t* pbc, const int64_t* counts,
                             int64_t batch, double cutoff, double* duals, int64_t* repeats,
                             char* error, size_t error_length) {
    error_sink sink = {error, error_length};
    return periodic_metadata(cells, pbc, counts, batch, cutoff, duals, repeats, &sink);
}

void oracle_free_pairs(int64_t* pairs, int32_t* shifts) {
    free(pairs);
    free(shifts);
}
