/*
 * tonari_b200 -- C ABI of the B200 (sm_100a) neighbor-list provider.
 *
 * One entry point replaces the reference's Torch-CUDA provider
 *   tonari csrc/torch/bindings_cuda.cpp:59-228   neighbor_list(...) -> [P, S]
 * together with the kernels it dispatches to
 *   tonari csrc/torch/neighbors_cuda.cu:443-556       (brute force)
 *   tonari csrc/torch/neighbors_cell_cuda.cu:558-814  (cell list)
 * and, optionally, the d/D/i/j assembly the Python frontend does afterwards
 *   tonari src/tonari/_torch_frontend.py:78-105.
 *
 * The signature uses plain pointers and sizes only.  Device inputs are
 * borrowed for the duration of the call; every device buffer the call needs
 * (workspace and the exact-size outputs) is obtained through the caller's
 * allocator callback on the caller's stream, so a framework allocator (the
 * PyTorch caching allocator in tonari_b200's custom op) owns the outputs.
 *
 * Error behaviour mirrors the reference: TNR_INPUT_ERROR is the reference's
 * InputError (Python ValueError), TNR_SEARCH_ERROR its SearchError / failed
 * TORCH_CHECK (Python RuntimeError); the message is the reference's message.
 */
#ifndef TONARI_B200_H
#define TONARI_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* tnr_stream;

enum tnr_status {
    TNR_OK = 0,
    TNR_INPUT_ERROR = 1,  /* reference InputError  -> ValueError   */
    TNR_SEARCH_ERROR = 2, /* reference SearchError -> RuntimeError */
    TNR_CUDA_ERROR = 3,
    TNR_ALLOC_ERROR = 4
};

enum tnr_dtype { TNR_FLOAT32 = 0, TNR_FLOAT64 = 1 };

/* Same values as tonari csrc/core/algorithm.h:10-29 parse order. */
enum tnr_algorithm { TNR_AUTO = 0, TNR_BRUTE_FORCE = 1, TNR_CELL_LIST = 2 };

/* Output selection (the characters of the public `quantities` string). */
enum tnr_quantity {
    TNR_Q_I = 1u << 0, /* (E,)  int64 source            */
    TNR_Q_J = 1u << 1, /* (E,)  int64 target            */
    TNR_Q_P = 1u << 2, /* (E,2) int64 [source, target]  */
    TNR_Q_S = 1u << 3, /* (E,3) int32 cell shift        */
    TNR_Q_d = 1u << 4, /* (E,)  T     distance          */
    TNR_Q_D = 1u << 5, /* (E,3) T     displacement      */
    /* (2,E) int64 graph layout: row 0 sources, row 1 targets, one buffer.
     * No counterpart in the reference's core API, whose adapters transpose P
     * (tonari docs/design.md:61, README.md:97); it cannot be combined with
     * TNR_Q_I or TNR_Q_J and is not offered by tnr_neighbor_list_static. */
    TNR_Q_EDGE = 1u << 6
};

/* Device allocation callback.  Must return device memory aligned to at least
 * 256 bytes that is usable in stream order on `stream`, or NULL on failure.
 * `release` is called for workspace only; output buffers are handed to the
 * caller in tnr_result and released by the caller. */
typedef struct {
    void* context;
    void* (*allocate)(void* context, size_t bytes, tnr_stream stream);
    void (*release)(void* context, void* pointer, tnr_stream stream);
} tnr_allocator;

typedef struct {
    int32_t dtype;            /* tnr_dtype */
    int64_t n_atoms;          /* N_total */
    int64_t n_structures;     /* B */
    const void* positions;    /* device (N,3) T, contiguous */
    const int64_t* batch_ptr; /* device (B+1) int64 */
    const void* cell;         /* device (B,3,3) T, rows are cell vectors */
    const uint8_t* pbc;       /* device (B,3) bool (one byte each) */
    /* Optional host mirrors of batch_ptr / cell / pbc (same layout and dtype).
     * When all three are non-NULL the call performs no device->host copy of
     * the metadata; when any is NULL it is read from the device pointers. */
    const int64_t* batch_ptr_host;
    const void* cell_host;
    const uint8_t* pbc_host;
    double cutoff;            /* strict, finite, positive */
    int32_t half_list;        /* bool */
    int32_t include_self;     /* bool */
    int32_t algorithm;        /* tnr_algorithm */
    uint32_t quantities;      /* OR of tnr_quantity */
    int64_t index_offset;     /* added to every emitted atom index (shards) */
    int32_t sorted;           /* bool: pairs ordered by source index; when false the
                                 order is unspecified (each unordered pair is
                                 searched once, faster) */
} tnr_request;

typedef struct {
    int64_t n_pairs; /* E */
    int64_t* i;      /* NULL unless TNR_Q_I */
    int64_t* j;      /* NULL unless TNR_Q_J */
    int64_t* P;      /* NULL unless TNR_Q_P */
    int32_t* S;      /* NULL unless TNR_Q_S */
    void* d;         /* NULL unless TNR_Q_d */
    void* D;         /* NULL unless TNR_Q_D */
    int64_t* edge_index; /* NULL unless TNR_Q_EDGE: (2,E) */
} tnr_result;

/*
 * Replaces tonari csrc/torch/bindings_cuda.cpp:59 `neighbor_list`
 * (positions, batch_ptr, cell, pbc, cutoff, half_list, include_self,
 * algorithm, sorted).  With request->sorted the pairs of each source are
 * contiguous and sources ascend; without it the order is unspecified, as in
 * the reference: each unordered pair is searched once and written where it
 * was found, in its canonical orientation (half lists) or in both (full
 * lists), which is faster.
 * Work is enqueued on `stream`; the call returns after the pair count is
 * known and the write pass has been enqueued (outputs are ready in stream
 * order).  On error `message` receives the reference's error text.
 */
int tnr_neighbor_list(const tnr_request* request, const tnr_allocator* allocator,
                      tnr_stream stream, tnr_result* result, char* message,
                      size_t message_length);

/*
 * No counterpart in the reference: an added entry point for callers that
 * cannot allocate device memory when they need a neighbor list -- a framework
 * that forbids allocation on its hot path, or a process whose GPU memory is
 * owned entirely by another allocator's pool, where a cudaMalloc would fail.
 * It allocates nothing: intermediates live in one fixed 8 MiB device array
 * per GPU that this library holds until the process exits, and the caller
 * passes the outputs.  Fill `result` with device pointers for every quantity
 * in request->quantities (a missing one is TNR_INPUT_ERROR), each with room
 * for `pair_capacity` pairs; on return result->n_pairs is the pair count
 * (also when it exceeded the capacity, which returns TNR_ALLOC_ERROR and
 * writes nothing).  At most 65536 atoms and 4096 structures per call (larger
 * requests: TNR_INPUT_ERROR); every candidate is enumerated, so it suits
 * small systems, and request->algorithm is ignored.  All copies and kernels
 * go on `stream`, and the call waits for `stream` to read the pair count.
 * The first call on a device looks up the array's address with that device
 * current -- make it before any stream capture.  All calls share the array:
 * calls that overlap on the GPU race, so serialise them.
 */
int tnr_neighbor_list_static(const tnr_request* request, tnr_stream stream,
                             int64_t pair_capacity, tnr_result* result, char* message,
                             size_t message_length);

/* Candidate pairs for tnr_filter_pairs (device arrays, M rows). */
typedef struct {
    const int64_t* pairs;  /* (M,2) int64 [source, target], indices include index_offset */
    const int32_t* shifts; /* (M,3) int32 cell shifts */
    int64_t n_candidates;  /* M */
} tnr_candidates;

/*
 * No counterpart in the reference, which lists Verlet-skin reuse as future
 * work (tonari docs/design.md:127).  Keeps the candidate pairs (built by
 * tnr_neighbor_list with cutoff + skin) whose public displacement at the
 * current positions, pos[j] - pos[i] + S . cell[b(i)], evaluated exactly as
 * tnr_neighbor_list's decisive test, is strictly shorter than
 * request->cutoff; the kept pairs keep their candidate order.  Uses
 * request->dtype, n_atoms, n_structures, positions, batch_ptr, cell, cutoff,
 * quantities and index_offset; the other request fields are ignored.
 * Outputs are allocated like tnr_neighbor_list's.
 */
int tnr_filter_pairs(const tnr_request* request, const tnr_candidates* candidates,
                     const tnr_allocator* allocator, tnr_stream stream, tnr_result* result,
                     char* message, size_t message_length);

/* Library version string ("major.minor.patch"). */
const char* tnr_version(void);

/* Number of kernels the last successful tnr_neighbor_list call on this host
 * thread launched (instrumentation for benchmarks and tests). */
int64_t tnr_last_launch_count(void);

/* Per-phase device times (ms) of the last call on this host thread when the
 * environment variable TONARI_B200_PHASE_TIMERS=1 is set, else zeros, from
 * CUDA events on the call's stream.  Order: prepare, bin, count kernels,
 * count scan, pair-total readback + output allocation, write kernels.
 * Returns the number written (at most 6). */
int tnr_last_phase_times(float* times_ms, int capacity);

/* Host wall-clock marks (ms since the call began) of the last call on this
 * host thread when TONARI_B200_PHASE_TIMERS=1 is set, else zeros: metadata
 * read, geometry built, prepare launched, extents read back, plans uploaded,
 * ghost totals read back, count pass launched, pair total read back, write
 * pass launched, then (marks 9-11, between marks 3 and 4) device geometry
 * taken over, plans built, bins laid out.  Returns the number written (at
 * most 12). */
int tnr_last_host_times(double* times_ms, int capacity);

#ifdef __cplusplus
}
#endif

#endif /* TONARI_B200_H */
