// Kernel launch interface used by the host scheduler (tnr_api.cpp).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "tnr_plan.h"

namespace tnr {

template <typename T>
struct PrepareArgs {
    const T* positions;
    int64_t n_atoms;
    const int64_t* batch_ptr;
    int64_t batch;
    const PrepareStructure<T>* structures;
    int32_t* atom_struct;
    int32_t* wraps;
    void* wrapped;  // vec4_t<T> [N]
    Reduction<T>* reductions;
    uint32_t* status;
};

template <typename T>
struct BinArgs {
    const StructurePlan<T>* plans;
    const int64_t* cell_prefix;  // [n_cell + 1] atom prefix over cell-mode structures
    const int32_t* cell_structs; // [n_cell]
    int32_t n_cell;
    int64_t n_cell_atoms;
    int32_t max_images;          // largest image count of a cell-list structure
    const int32_t* wraps;
    const void* wrapped;         // vec4_t<T>
    unsigned long long* bin_counts;  // histogram target / scatter cursors
    int32_t pair_once;           // keep only copies a pair-once search can test
    int64_t ghost_capacity;      // ghost slots allocated (scatter only)
    // Ghost arrays: zero images at [0, n_cell_atoms) in source-slot order,
    // other image copies from n_cell_atoms on.
    void* ghost_pos;             // vec4_t<T> [G]   (scatter only)
    int4* ghost_meta;            // [G]             (scatter only)
    void* ghost_orig;            // vec4_t<T> [G]   (scatter only)
    const T* positions;
    int32_t* source_list;        // [sources]       (scatter only)
    int32_t* source_bin;         // [sources]       (scatter only) bin of each listed source
    uint32_t* status;
    const int4* image_shift;        // [images] (x, y, z, 0), x-major per structure
    const void* image_translation;  // vec4_t<T> [images], shift . cell in T
};

template <typename T>
struct SearchArgs {
    const T* positions;
    const int32_t* atom_struct;
    const int32_t* wraps;
    const void* wrapped;  // vec4_t<T>
    const StructurePlan<T>* plans;
    // cell mode
    const unsigned long long* bin_start;
    const void* ghost_pos;  // vec4_t<T>
    const int4* ghost_meta;
    int32_t* source_list;               // cell order (source slot -> atom)
    const int32_t* source_bin;          // [sources] bin of each source, cell order
    int64_t n_sources;
    const int32_t* bin_struct;          // [bins] structure of each bin
    const void* ghost_orig;             // vec4_t<T> [G] original target position, target
    int32_t source_order;               // 0: outputs by atom index; 1: cell order
    int32_t pair_once;                  // each unordered pair tested from one side (cell order only)
    int32_t paired_rows;                // full pair-once lists: both orientations in adjacent rows
    const int64_t* cell_bin_prefix;     // [n_cell + 1] first bin of each cell-list structure
    const int32_t* cell_structs;        // [n_cell]
    int32_t n_cell;
    int64_t n_bins;
    const unsigned long long* bin_word_start;  // [bins + 1] scan of per-bin mask words
    uint32_t* mask_words;               // count pass ballots, read by the write pass
    const int4* image_shift;            // [images]
    // brute mode
    const int64_t* brute_prefix;  // [n_brute + 1]
    const int32_t* brute_structs; // [n_brute]
    int32_t n_brute;
    int64_t n_brute_atoms;
    // Shared-memory bytes one brute-force structure needs staged (positions,
    // wraps, image shifts) when every brute structure fits a CTA; 0 selects
    // the kernel that reads them from global memory.
    int32_t brute_tile_bytes;
    // passes
    uint32_t* counts;           // count pass output
    const int64_t* pair_start;  // write pass input
    int64_t* out_i;
    int64_t* out_j;
    int64_t* out_P;
    int32_t* out_S;
    T* out_d;
    T* out_D;
    int64_t index_offset;
    uint32_t* status;
    int32_t half_list;
    int32_t include_self;
};

// Speculative periodic geometry on the device (one thread per structure):
// the reference's one-sided Jacobi pseudo-inverse evaluated in double instead
// of long double.  Writes the prepare records (cell, dual cast to T), the
// double duals, repeats and image counts; sets `flags` to nonzero when any
// structure needs the host's exact treatment (non-finite cell, near-singular
// active rows, out-of-range duals or repeats, more than 2^24 images).  The
// host checks the image ranges against its long-double geometry, and the
// device checks every atom's wraps against the exact duals
// (launch_verify_wraps), before the call's output is trusted.
struct DeviceGeometry {
    double dual[9];      // [cartesian][axis]
    int32_t repeats[3];
    int32_t images;      // 0 for an empty structure
};

template <typename T>
void launch_geometry(const T* cell, const uint8_t* pbc, const int64_t* batch_ptr, int64_t batch,
                     double cutoff, PrepareStructure<T>* prepare, DeviceGeometry* geometry,
                     uint32_t* flags, Reduction<T>* reductions, cudaStream_t stream);

// Candidate-pair filter (Verlet-skin reuse): one bit per candidate, set when
// its exact public-formula distance is below the cutoff.
template <typename T>
struct FilterArgs {
    const T* positions;
    const int64_t* batch_ptr;
    int64_t batch;
    const T* cell;              // (B,3,3)
    const int64_t* pairs;       // (M,2), with index_offset
    const int32_t* shifts;      // (M,3)
    int64_t n_candidates;
    int64_t index_offset;
    T cutoff_squared;
    uint32_t* keep_words;       // [ceil(M / 32)]
    uint32_t* block_counts;     // [ceil(M / kFilterThreads)]
    const int64_t* block_start; // scan of block_counts
    int64_t* out_i;
    int64_t* out_j;
    int64_t* out_P;
    int32_t* out_S;
    T* out_d;
    T* out_D;
};

constexpr int kFilterThreads = 256;

template <typename T>
void launch_filter(const FilterArgs<T>& args, bool write, cudaStream_t stream);

// Sets *flag when any atom's wraps, recomputed with `duals` ([B][9] in T,
// [cartesian][axis]), differ from `wraps`.
template <typename T>
void launch_verify_wraps(const T* positions, int64_t n_atoms, const int32_t* atom_struct,
                         const T* duals, const int32_t* wraps, uint32_t* flag, cudaStream_t stream);

template <typename T>
void launch_prepare(const PrepareArgs<T>& args, cudaStream_t stream);

template <typename T>
void launch_bin(const BinArgs<T>& args, bool scatter, cudaStream_t stream);

// Fills the per-structure image tables (shift, translation) on the device.
template <typename T>
void launch_image_table(const StructurePlan<T>* plans, int64_t batch, int4* shifts,
                        void* translations, cudaStream_t stream);

// Writes the structure index of every cell-list bin.
template <typename T>
void launch_bin_struct(const int64_t* cell_bin_prefix, const int32_t* cell_structs,
                       int32_t n_cell, int32_t* bin_struct, cudaStream_t stream);

template <typename T>
void launch_stencil_words(const SearchArgs<T>& args, unsigned long long* bin_words,
                          cudaStream_t stream);

// Sets the capacity status bit when *total exceeds capacity (one thread).
void launch_capacity_check(const unsigned long long* total, unsigned long long capacity,
                           uint32_t* status, cudaStream_t stream);

template <typename T>
void launch_cell_search(const SearchArgs<T>& args, bool write, cudaStream_t stream);

template <typename T>
void launch_brute_search(const SearchArgs<T>& args, bool write, cudaStream_t stream);

// Running count of kernels this host thread has launched through this file.
int64_t launched_kernels();

// Exclusive scans (n+1 outputs), three launches each.  `workspace` holds
// scan_workspace_bytes(n) bytes of per-tile sums.  `status` is unused: no
// CTA of the scan waits on another.
size_t scan_workspace_bytes(int64_t n);
void launch_scan_u64(const unsigned long long* in, int64_t n, unsigned long long* out,
                     unsigned long long* out2, void* workspace, uint32_t* status,
                     cudaStream_t stream);
void launch_scan_counts(const uint32_t* in, int64_t n, int64_t* out, void* workspace,
                        uint32_t* status, cudaStream_t stream);

}  // namespace tnr
