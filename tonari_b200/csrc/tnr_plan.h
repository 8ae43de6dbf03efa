// Per-call plan shared by the host scheduler (tnr_api.cpp) and the kernels
// (tnr_kernels.cu).  Plain structs only, so both g++ and nvcc see the same
// layout.
//
// HBM layout of one call (N atoms, B structures, G ghosts, E pairs):
//   atom_struct  int32 [N]          structure of each atom
//   wraps        int32 [N][3]       floor(position . dual_T)  (reference wraps)
//   wrapped      T4    [N]          position - wraps . cell, w unused
//   bin_start    u64   [bins+1]     exclusive scan of (sources << 32 | image copies)
//   ghost_pos    T4    [G]          image copies (x, y, z, order key): the zero
//                                   images at [0, S) by source slot, then the
//                                   other copies cell-sorted from S on
//   ghost_meta   int4  [G]          (image - wrap_target) xyz, target
//   source_list  int32 [S]          atoms of cell-list structures, cell-sorted
//   pair_count   int32 [N]          pairs per source   -> pair_start int64 [N+1]
// Outputs are written source-major at pair_start[source].
#pragma once

#include <cstdint>

namespace tnr {

enum StructureMode : int32_t {
    kModeEmpty = 0,
    kModeBrute = 1,  // every (target, image) candidate, exact predicate
    kModeCell = 2    // ghost copies binned on a Cartesian grid, 27-bin stencil
};

// Status bits written by kernels (atomicOr) and read back with the counts.
enum StatusBit : uint32_t {
    kStatusNonFinite = 1u << 0,     // "positions must contain only finite values"
    kStatusWrapRange = 1u << 1,     // wraps outside int32
    kStatusShiftRange = 1u << 2,    // accepted pair's shift outside int32
    kStatusReserved3 = 1u << 3,     // unused (no kernel waits on another)
    kStatusCapacity = 1u << 4,      // an internal capacity was exceeded
    kStatusCountRange = 1u << 5     // a per-source count overflowed int32
};

// Minimal per-structure data needed by the prepare kernel.
template <typename T>
struct PrepareStructure {
    int64_t atom_begin;
    int64_t atom_end;
    T cell[9];  // rows are cell vectors: cell[3*a + c]
    T dual[9];  // dual[3*c + a], the reference layout cast to T
};

// Per-structure reductions written by the prepare kernel, as order-preserving
// integer keys so that plain atomicMin / atomicMax can combine them.
template <typename T>
struct Reduction;

template <>
struct Reduction<float> {
    int32_t wrapped_min[3];
    int32_t wrapped_max[3];
    int32_t position_abs_max[3];
    int32_t wrap_abs_max[3];
};

template <>
struct Reduction<double> {
    long long wrapped_min[3];
    long long wrapped_max[3];
    long long position_abs_max[3];
    int32_t wrap_abs_max[3];
    int32_t pad;
};

// Full per-structure plan used by the binning and search kernels.
template <typename T>
struct StructurePlan {
    int64_t atom_begin;
    int32_t n_atoms;
    int32_t mode;          // StructureMode
    int64_t image_begin;   // first image of this structure (global image index)
    int32_t n_images;
    int32_t repeats[3];
    int64_t bin_begin;     // first bin of this structure (cell mode)
    int32_t dims[3];       // bins per axis (cell mode)
    int32_t self_images;   // a nonzero lattice translation may be shorter than the search radius
    T cell[9];
    T origin[3];           // lower corner of the bin grid
    T inv_edge;            // 1 / bin edge
    T lower[3];            // culling box for ghosts
    T upper[3];
    T cutoff_squared;      // (T)(cutoff * cutoff) -- the decisive threshold
    T search_squared;      // padded broad-phase threshold
    T inner_squared;       // broad-phase distances below this are accepted
};

}  // namespace tnr
