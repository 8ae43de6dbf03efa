// Neighbor-list kernels for B200 (sm_100a).
//
// Pipeline of one call (host side in tnr_api.cpp):
//   prepare   per atom: structure id, representative wrap, wrapped position,
//             per-structure extents reduced through order-preserving atomics
//   bin       per cell-list atom x image: cull the image copy against the
//             structure's box, histogram it into a Cartesian bin (pass 1) or
//             scatter it into cell-sorted order (pass 2)
//   scan      three-launch exclusive scans (tnr_scan.cuh)
//   search    one warp per source atom: walk the 3x3 rows of the 27-bin
//             stencil as one flattened candidate range (cell list) or every
//             (target, image) candidate (brute force); count pass, then write
//             pass with ballot/popc compaction into the source's output span.
//
// The decisive test is the reference's public formula, evaluated in T without
// contraction (tnr_kernels.cuh exact_component); the cell list's broad phase
// uses a padded radius and accepts without the exact test only inside an inner
// radius, the reference's own scheme (tonari csrc/core/neighbors_cpu.cpp:156-
// 219, 276-327).  Pair sets therefore match the reference CPU path exactly.
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cstdint>
#include <type_traits>

#include "tnr_kernels.cuh"
#include "tnr_launch.h"
#include "tnr_scan.cuh"

namespace tnr {
namespace {

constexpr int kPrepareThreads = 512;
constexpr int kBinThreads = 256;
constexpr int kSearchThreads = 256;
constexpr int kSearchWarps = kSearchThreads / 32;
// Bin kernels: six resident blocks per SM (40 registers) keep more of the
// scatter's returned atomics in flight than four blocks at 56 registers.
#ifndef TNR_BIN_MIN_BLOCKS
#define TNR_BIN_MIN_BLOCKS 6
#endif

// ---------------------------------------------------------------------------
// geometry (speculative, double precision)
// ---------------------------------------------------------------------------

// The reference's active pseudo-inverse (tonari csrc/core/geometry.cpp:15-118)
// and image ranges (:123-219) in double: same rotation sequence, convergence
// test, singular-value tolerance and ceil(cutoff * |dual column|).  The host
// compares the T-cast duals and the repeats with its long-double result.
template <typename T>
__global__ void geometry_kernel(const T* __restrict__ cell, const uint8_t* __restrict__ pbc,
                                const int64_t* __restrict__ batch_ptr, int64_t batch, double cutoff,
                                PrepareStructure<T>* __restrict__ prepare,
                                DeviceGeometry* __restrict__ out, uint32_t* flags,
                                Reduction<T>* __restrict__ reductions) {
    const int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (b >= batch) return;
    {
        // The prepare kernel's extents start from the neutral element.
        Reduction<T> neutral{};
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            neutral.wrapped_min[c] = order_key(static_cast<T>(INFINITY));
            neutral.wrapped_max[c] = order_key(static_cast<T>(-INFINITY));
            neutral.position_abs_max[c] = order_key(T(0));
            neutral.wrap_abs_max[c] = 0;
        }
        reductions[b] = neutral;
    }
    const double eps = 2.220446049250313e-16;  // double epsilon
    double c[9];
    bool bad = false;
#pragma unroll
    for (int k = 0; k < 9; ++k) {
        c[k] = static_cast<double>(cell[9 * b + k]);
        bad = bad || !isfinite(c[k]);
    }
    const int64_t atoms = batch_ptr[b + 1] - batch_ptr[b];
    DeviceGeometry g;
#pragma unroll
    for (int k = 0; k < 9; ++k) g.dual[k] = 0.0;
    g.repeats[0] = g.repeats[1] = g.repeats[2] = 0;
    g.images = 0;
    if (!bad && atoms > 0) {
        int axes[3];
        int active = 0;
        for (int a = 0; a < 3; ++a) {
            if (pbc[3 * b + a] != 0) axes[active++] = a;
        }
        if (active > 0) {
            double columns[3][3] = {};
            double right[3][3] = {};
            for (int col = 0; col < active; ++col) {
                right[col][col] = 1.0;
                for (int x = 0; x < 3; ++x) columns[x][col] = c[3 * axes[col] + x];
            }
            for (int sweep = 0; sweep < 64; ++sweep) {
                bool converged = true;
                for (int p = 0; p < active; ++p) {
                    for (int q = p + 1; q < active; ++q) {
                        double npp = 0.0, nqq = 0.0, npq = 0.0;
                        for (int x = 0; x < 3; ++x) {
                            npp = __dadd_rn(npp, __dmul_rn(columns[x][p], columns[x][p]));
                            nqq = __dadd_rn(nqq, __dmul_rn(columns[x][q], columns[x][q]));
                            npq = __dadd_rn(npq, __dmul_rn(columns[x][p], columns[x][q]));
                        }
                        if (fabs(npq) <= 8 * eps * sqrt(npp * nqq)) continue;
                        converged = false;
                        const double tau = (nqq - npp) / (2 * npq);
                        const double t = tau == 0.0 ? 1.0 : copysign(1.0, tau) / (fabs(tau) + hypot(1.0, tau));
                        const double cs = 1.0 / hypot(1.0, t);
                        const double sn = cs * t;
                        for (int x = 0; x < 3; ++x) {
                            const double u = columns[x][p], v = columns[x][q];
                            columns[x][p] = __dsub_rn(__dmul_rn(cs, u), __dmul_rn(sn, v));
                            columns[x][q] = __dadd_rn(__dmul_rn(sn, u), __dmul_rn(cs, v));
                        }
                        for (int r = 0; r < active; ++r) {
                            const double u = right[r][p], v = right[r][q];
                            right[r][p] = __dsub_rn(__dmul_rn(cs, u), __dmul_rn(sn, v));
                            right[r][q] = __dadd_rn(__dmul_rn(sn, u), __dmul_rn(cs, v));
                        }
                    }
                }
                if (converged) break;
            }
            double sigma[3] = {};
            double largest = 0.0, smallest = INFINITY;
            for (int col = 0; col < active; ++col) {
                double n2 = 0.0;
                for (int x = 0; x < 3; ++x) n2 = __dadd_rn(n2, __dmul_rn(columns[x][col], columns[x][col]));
                sigma[col] = sqrt(n2);
                largest = fmax(largest, sigma[col]);
                smallest = fmin(smallest, sigma[col]);
            }
            // The host tolerance is eps * 3 * max(largest, 1); a margin keeps
            // borderline cells on the exact host path.
            if (!(smallest > eps * 3 * fmax(largest, 1.0) * 4)) bad = true;
            int64_t images = 1;
            for (int col = 0; col < active && !bad; ++col) {
                double n2 = 0.0;
                for (int x = 0; x < 3; ++x) {
                    double value = 0.0;
                    for (int s = 0; s < active; ++s) {
                        value = __dadd_rn(value, __ddiv_rn(__dmul_rn(columns[x][s], right[col][s]),
                                                           __dmul_rn(sigma[s], sigma[s])));
                    }
                    bad = bad || !isfinite(value);
                    g.dual[3 * x + axes[col]] = value;
                    n2 = __dadd_rn(n2, __dmul_rn(value, value));
                }
                const double repeat = ceil(cutoff * sqrt(n2));
                if (!(repeat <= 1048576.0)) {
                    bad = true;
                } else {
                    g.repeats[axes[col]] = static_cast<int32_t>(repeat);
                }
            }
            for (int a = 0; a < 3 && !bad; ++a) {
                images *= 2 * static_cast<int64_t>(g.repeats[a]) + 1;
                if (images > (int64_t{1} << 24)) bad = true;
            }
            g.images = bad ? 0 : static_cast<int32_t>(images);
        } else {
            g.images = 1;
        }
    }
    PrepareStructure<T> st;
    st.atom_begin = batch_ptr[b];
    st.atom_end = batch_ptr[b + 1];
#pragma unroll
    for (int k = 0; k < 9; ++k) {
        st.cell[k] = cell[9 * b + k];
        st.dual[k] = static_cast<T>(g.dual[k]);
    }
    prepare[b] = st;
    out[b] = g;
    if (bad) atomicOr(flags, 1u);
}

// ---------------------------------------------------------------------------
// prepare
// ---------------------------------------------------------------------------

// floor(p . dual_column) from an error-free double-double sum, so the result
// is the floor of the (nearly) exact dot product.  The reference evaluates it
// in x87 long double (tonari csrc/core/neighbors_cpu.cpp:110-122); the two
// agree except when the dot product lies within 2^-100 relative of an integer.
__device__ __forceinline__ double two_prod(double a, double b, double& error) {
    const double p = __dmul_rn(a, b);
    error = fma(a, b, -p);
    return p;
}
__device__ __forceinline__ double two_sum(double a, double b, double& error) {
    const double s = __dadd_rn(a, b);
    const double bb = __dsub_rn(s, a);
    error = __dadd_rn(__dsub_rn(a, __dsub_rn(s, bb)), __dsub_rn(b, bb));
    return s;
}

struct DotFloor {
    double approx;
    double floor_value;
};

__device__ __forceinline__ DotFloor dot_floor(double p0, double p1, double p2, double d0,
                                              double d1, double d2) {
    double l0, l1, l2, e1, e2;
    const double h0 = two_prod(p0, d0, l0);
    const double h1 = two_prod(p1, d1, l1);
    const double h2 = two_prod(p2, d2, l2);
    const double s1 = two_sum(h0, h1, e1);
    const double s2 = two_sum(s1, h2, e2);
    const double low = l0 + l1 + l2 + e1 + e2;
    double f = floor(s2);
    if (f == s2 && low < 0.0) f -= 1.0;
    return {s2, f};
}

template <typename K>
struct Extents {
    K lo[3];
    K hi[3];
    K abs_position[3];
    int32_t abs_wrap[3];
};

template <typename K>
__device__ __forceinline__ void combine(Extents<K>& a, const Extents<K>& b) {
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        a.lo[c] = min(a.lo[c], b.lo[c]);
        a.hi[c] = max(a.hi[c], b.hi[c]);
        a.abs_position[c] = max(a.abs_position[c], b.abs_position[c]);
        a.abs_wrap[c] = max(a.abs_wrap[c], b.abs_wrap[c]);
    }
}

template <typename K>
__device__ __forceinline__ Extents<K> shfl_down(const Extents<K>& v, int offset) {
    Extents<K> out;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        out.lo[c] = __shfl_down_sync(kFullMask, v.lo[c], offset);
        out.hi[c] = __shfl_down_sync(kFullMask, v.hi[c], offset);
        out.abs_position[c] = __shfl_down_sync(kFullMask, v.abs_position[c], offset);
        out.abs_wrap[c] = __shfl_down_sync(kFullMask, v.abs_wrap[c], offset);
    }
    return out;
}

template <typename K, typename R>
__device__ __forceinline__ void publish(R* reduction, const Extents<K>& v) {
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        atomicMin(&reduction->wrapped_min[c], v.lo[c]);
        atomicMax(&reduction->wrapped_max[c], v.hi[c]);
        atomicMax(&reduction->position_abs_max[c], v.abs_position[c]);
        atomicMax(&reduction->wrap_abs_max[c], v.abs_wrap[c]);
    }
}

template <typename T>
__global__ void __launch_bounds__(kPrepareThreads) prepare_kernel(PrepareArgs<T> args) {
    using K = decltype(order_key(T(0)));
    using V = vec4_t<T>;
    __shared__ int32_t block_first_last[2];
    __shared__ Extents<K> warp_partial[kPrepareThreads / 32];

    // The host may check batch_ptr only after this kernel was queued: the
    // block searches below stay in bounds for any batch_ptr that starts at
    // zero; for one that does not, nothing is done and the host reports it.
    if (args.batch_ptr[0] != 0) return;
    const int64_t block_base = static_cast<int64_t>(blockIdx.x) * kPrepareThreads;
    const int64_t atom = block_base + threadIdx.x;
    const bool valid = atom < args.n_atoms;
    if (threadIdx.x < 32) {  // warp 0: 32-way searches, a few dependent loads
        const int64_t last = min(args.n_atoms - 1, block_base + kPrepareThreads - 1);
        const int64_t first = warp_last_le(args.batch_ptr, 0, args.batch, block_base);
        const int64_t closing = warp_last_le(args.batch_ptr, first, args.batch, last);
        if (threadIdx.x == 0) {
            block_first_last[0] = static_cast<int32_t>(first);
            block_first_last[1] = static_cast<int32_t>(closing);
        }
    }
    __syncthreads();

    Extents<K> ext;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        ext.lo[c] = order_key(static_cast<T>(INFINITY));
        ext.hi[c] = order_key(static_cast<T>(-INFINITY));
        ext.abs_position[c] = order_key(T(0));
        ext.abs_wrap[c] = 0;
    }
    int32_t sid = -1;
    if (valid) {
        sid = structure_of(args.batch_ptr, args.batch, atom, block_first_last[0],
                           block_first_last[1] + 1);
        args.atom_struct[atom] = sid;
        const PrepareStructure<T>& st = args.structures[sid];
        const T p[3] = {args.positions[3 * atom], args.positions[3 * atom + 1],
                        args.positions[3 * atom + 2]};
        bool finite = isfinite(p[0]) && isfinite(p[1]) && isfinite(p[2]);
        int32_t w[3] = {0, 0, 0};
        if (!finite) {
            atomicOr(args.status, static_cast<uint32_t>(kStatusNonFinite));
        } else {
#pragma unroll
            for (int a = 0; a < 3; ++a) {
                const DotFloor f = dot_floor(p[0], p[1], p[2], st.dual[a], st.dual[3 + a],
                                             st.dual[6 + a]);
                if (!(isfinite(f.approx) && f.approx >= -2147483648.0 &&
                      f.approx < 2147483648.0)) {
                    atomicOr(args.status, static_cast<uint32_t>(kStatusWrapRange));
                    finite = false;
                } else {
                    w[a] = static_cast<int32_t>(f.floor_value);
                }
            }
        }
        T q[3];
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            T value = p[c];
#pragma unroll
            for (int a = 0; a < 3; ++a) {
                value = sub_rn(value, mul_rn(static_cast<T>(w[a]), st.cell[3 * a + c]));
            }
            q[c] = value;
        }
#pragma unroll
        for (int a = 0; a < 3; ++a) args.wraps[3 * atom + a] = w[a];
        V packed;
        packed.x = q[0];
        packed.y = q[1];
        packed.z = q[2];
        packed.w = T(0);
        reinterpret_cast<V*>(args.wrapped)[atom] = packed;
        if (finite) {
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                ext.lo[c] = order_key(q[c]);
                ext.hi[c] = order_key(q[c]);
                ext.abs_position[c] = order_key(static_cast<T>(fabs(p[c])));
                const long long aw = w[c] < 0 ? -static_cast<long long>(w[c]) : w[c];
                ext.abs_wrap[c] = static_cast<int32_t>(min(aw, static_cast<long long>(INT_MAX)));
            }
        }
    }

    // Segmented warp reduction: atoms are sorted by structure, so equal ids
    // form contiguous runs; min/max are idempotent, so overlapping windows of
    // the doubling shuffle are harmless.
    const int lane = threadIdx.x & 31;
    // A warp of one structure (the common case) reduces each 32-bit key with
    // one redux instruction; warps that straddle structures, and 64-bit keys,
    // take the segmented shuffle.
    const int32_t lane0_sid = __shfl_sync(kFullMask, sid, 0);
    const bool one_structure = __all_sync(kFullMask, sid >= 0 && sid == lane0_sid);
    auto segmented = [&]() {
#pragma unroll
        for (int offset = 1; offset < 32; offset <<= 1) {
            const int32_t other_sid = __shfl_down_sync(kFullMask, sid, offset);
            const Extents<K> other = shfl_down(ext, offset);
            if (lane + offset < 32 && other_sid == sid) combine(ext, other);
        }
    };
    if constexpr (std::is_same<K, int32_t>::value) {
        if (one_structure) {
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                ext.lo[c] = __reduce_min_sync(kFullMask, ext.lo[c]);
                ext.hi[c] = __reduce_max_sync(kFullMask, ext.hi[c]);
                ext.abs_position[c] = __reduce_max_sync(kFullMask, ext.abs_position[c]);
                ext.abs_wrap[c] = __reduce_max_sync(kFullMask, ext.abs_wrap[c]);
            }
        } else {
            segmented();
        }
    } else {
        segmented();
    }
    const int32_t previous_sid = __shfl_up_sync(kFullMask, sid, 1);
    const bool head = sid >= 0 && (lane == 0 || previous_sid != sid);
    __syncthreads();
    const bool uniform = block_first_last[0] == block_first_last[1];
    if (!uniform) {
        if (head) publish(&args.reductions[sid], ext);
        return;
    }
    if (lane == 0) warp_partial[threadIdx.x >> 5] = ext;
    __syncthreads();
    if (threadIdx.x == 0) {
        Extents<K> total = warp_partial[0];
        for (int w = 1; w < kPrepareThreads / 32; ++w) {
            if (block_base + w * 32 < args.n_atoms) combine(total, warp_partial[w]);
        }
        publish(&args.reductions[block_first_last[0]], total);
    }
}


// Check of a speculative geometry: the wraps of every atom recomputed with
// the exact (host, long-double) duals cast to T must equal the wraps the
// call used; any difference sets *flag and the call is repeated on the host
// path.  Equal wraps (with equal image ranges, checked on the host) make
// every later step identical to the host-geometry call.
template <typename T>
__global__ void __launch_bounds__(kPrepareThreads) verify_wraps_kernel(
    const T* __restrict__ positions, int64_t n_atoms, const int32_t* __restrict__ atom_struct,
    const T* __restrict__ duals, const int32_t* __restrict__ wraps, uint32_t* flag) {
    const int64_t atom = static_cast<int64_t>(blockIdx.x) * kPrepareThreads + threadIdx.x;
    if (atom >= n_atoms) return;
    const T* dual = duals + 9 * static_cast<int64_t>(atom_struct[atom]);
    const double p0 = positions[3 * atom], p1 = positions[3 * atom + 1], p2 = positions[3 * atom + 2];
    bool same = true;
#pragma unroll
    for (int a = 0; a < 3; ++a) {
        const DotFloor f = dot_floor(p0, p1, p2, dual[a], dual[3 + a], dual[6 + a]);
        same = same && isfinite(f.approx) && f.approx >= -2147483648.0 && f.approx < 2147483648.0 &&
               static_cast<int32_t>(f.floor_value) == wraps[3 * atom + a];
    }
    if (!same) atomicOr(flag, 1u);
}

// ---------------------------------------------------------------------------
// bin: histogram (pass 1) and scatter (pass 2) of culled image copies
// ---------------------------------------------------------------------------

// One thread per atom of a cell-list structure, looping over the structure's
// images.  An image copy is kept when it lies inside the structure's culling
// box (extent of the wrapped atoms padded by the search radius), the
// reference's rule (tonari csrc/core/neighbors_cpu.cpp:479-495).  Ghost
// records live in two regions of one array: the zero images (the sources)
// at [0, S) in source-slot order and the other image copies at [S, S + I).
// Each bin counter packs (sources << 32 | image copies), so one 64-bit
// atomic hands out the slot in either region.  The zero image is placed
// first so that the atom's other copies carry its source slot.  When the
// atoms alone cannot fill the GPU, gridDim.y > 1 threads share an atom's
// images (thread y takes images y, y + gridDim.y, ...; y = 0 also places the
// zero image); copies then depend on the atom only, not on its slot.
//
// Pair-once calls (args.pair_once) test every unordered pair from one side
// only.  The pair (s, t) through image I of t's wrapped position is the pair
// (t, s) through image -I of s's, so an image copy is kept only when its
// image precedes the zero image in the x-major enumeration (its first nonzero
// component is negative, the canonical shift rule), and every kept copy is
// tested from every source near it.  Zero images (I = 0) are tested from the
// source with the lower source slot.
// Order key of a pair-once image copy: above every source's key(s) + 1
// (2 slot + 2 < 2^31), so the key test accepts it for every source.
constexpr uint32_t kImageCopyKey = 0x7ffffff0u;

template <typename T, bool Scatter>
__global__ void __launch_bounds__(kBinThreads, TNR_BIN_MIN_BLOCKS) bin_kernel(BinArgs<T> args) {
    using V = vec4_t<T>;
    __shared__ int32_t block_first_last[2];
    const int64_t block_base = static_cast<int64_t>(blockIdx.x) * kBinThreads;
    const int64_t index = block_base + threadIdx.x;
    if (threadIdx.x < 32) {  // warp 0: 32-way searches, a few dependent loads
        const int64_t last = min(args.n_cell_atoms - 1, block_base + kBinThreads - 1);
        const int64_t first = warp_last_le(args.cell_prefix, 0, args.n_cell, block_base);
        const int64_t closing = warp_last_le(args.cell_prefix, first, args.n_cell, last);
        if (threadIdx.x == 0) {
            block_first_last[0] = static_cast<int32_t>(first);
            block_first_last[1] = static_cast<int32_t>(closing);
        }
    }
    __syncthreads();
    if (index >= args.n_cell_atoms) return;
    const int32_t c = segment_of(args.cell_prefix, args.n_cell, index, block_first_last[0],
                                 block_first_last[1] + 1);
    const StructurePlan<T>& plan = args.plans[args.cell_structs[c]];
    const int64_t atom = plan.atom_begin + (index - args.cell_prefix[c]);
    const V q = reinterpret_cast<const V*>(args.wrapped)[atom];
    const int32_t wrap[3] = {args.wraps[3 * atom], args.wraps[3 * atom + 1],
                             args.wraps[3 * atom + 2]};
    // The plan's fields live in registers for the image loop (the loop's
    // atomics and stores would otherwise make the compiler reload them).
    const int32_t n_images = plan.n_images;
    const int32_t center = (n_images - 1) / 2;
    const int64_t image_begin = plan.image_begin;
    const int64_t bin_begin = plan.bin_begin;
    const int32_t dims[3] = {plan.dims[0], plan.dims[1], plan.dims[2]};
    const T lower[3] = {plan.lower[0], plan.lower[1], plan.lower[2]};
    const T upper[3] = {plan.upper[0], plan.upper[1], plan.upper[2]};
    const T origin[3] = {plan.origin[0], plan.origin[1], plan.origin[2]};
    const T inv_edge = plan.inv_edge;
    const V* translations = reinterpret_cast<const V*>(args.image_translation) + image_begin;
    auto bin_of = [&](const T (&g)[3]) -> int64_t {
        const int32_t bx = bin_axis(g[0], origin[0], inv_edge, dims[0]);
        const int32_t by = bin_axis(g[1], origin[1], inv_edge, dims[1]);
        const int32_t bz = bin_axis(g[2], origin[2], inv_edge, dims[2]);
        return bin_begin + (static_cast<int64_t>(bx) * dims[1] + by) * dims[2] + bz;
    };
    auto store = [&](uint32_t slot, const T (&g)[3], int32_t k, uint32_t key) {
        V record;
        record.x = g[0];
        record.y = g[1];
        record.z = g[2];
        record.w = index_to_lane(static_cast<int32_t>(key), T(0));
        reinterpret_cast<V*>(args.ghost_pos)[slot] = record;
        if (args.ghost_orig) {  // only the d / D outputs read it
            V original;
            original.x = args.positions[3 * atom];
            original.y = args.positions[3 * atom + 1];
            original.z = args.positions[3 * atom + 2];
            original.w = index_to_lane(static_cast<int32_t>(atom), T(0));
            reinterpret_cast<V*>(args.ghost_orig)[slot] = original;
        }
        const int4 image = args.image_shift[image_begin + k];
        args.ghost_meta[slot] = make_int4(image.x - wrap[0], image.y - wrap[1], image.z - wrap[2],
                                          static_cast<int32_t>(atom));
    };
    // Zero image: the source.
    uint32_t key_base = 2u * static_cast<uint32_t>(atom);  // 2 * (source slot or atom)
    if (blockIdx.y == 0) {
        const V tr = translations[center];
        const T g[3] = {add_rn(q.x, tr.x), add_rn(q.y, tr.y), add_rn(q.z, tr.z)};
        const int64_t home = bin_of(g);
        const unsigned long long old = atomicAdd(&args.bin_counts[home], 1ull << 32);
        const uint32_t source_slot = static_cast<uint32_t>(old >> 32);
        key_base = 2u * (args.pair_once ? source_slot : static_cast<uint32_t>(atom));
        if constexpr (Scatter) {
            // Order key of the copy: 2a + 1 for the zero image, 2a + 2 for
            // the others (a = source slot or atom; read by the search).
            store(source_slot, g, center, key_base + 1u);
            args.source_list[source_slot] = static_cast<int32_t>(atom);
            args.source_bin[source_slot] = static_cast<int32_t>(home);
        }
    }
    // Pair-once: images after the zero image are the reverses of kept ones.
    const int32_t last_image = args.pair_once ? center : n_images;
    const uint32_t image_key = args.pair_once ? kImageCopyKey : key_base + 2u;
    for (int32_t k = blockIdx.y; k < last_image; k += gridDim.y) {
        if (k == center) continue;
        const V tr = translations[k];
        const T g[3] = {add_rn(q.x, tr.x), add_rn(q.y, tr.y), add_rn(q.z, tr.z)};
        const bool inside = g[0] >= lower[0] && g[0] <= upper[0] &&
                            g[1] >= lower[1] && g[1] <= upper[1] &&
                            g[2] >= lower[2] && g[2] <= upper[2];
        if (!inside) continue;
        const int64_t bin = bin_of(g);
        const unsigned long long old = atomicAdd(&args.bin_counts[bin], 1ull);
        if constexpr (Scatter) {
            const int64_t slot = args.n_cell_atoms + static_cast<int64_t>(old & 0xffffffffull);
            if (slot >= args.ghost_capacity) {  // never, for a correct bound
                atomicOr(args.status, static_cast<uint32_t>(kStatusCapacity));
                continue;
            }
            store(static_cast<uint32_t>(slot), g, k, image_key);
        }
    }
}


// ---------------------------------------------------------------------------
// search: count pass and write pass
// ---------------------------------------------------------------------------

// Writes one accepted pair at output row `o`.
template <typename T>
__device__ __forceinline__ void emit_pair(const SearchArgs<T>& a, int64_t o, int64_t source,
                                          int64_t target, const long long (&shift)[3],
                                          const T (&displacement)[3]) {
    const int64_t s = source + a.index_offset;
    const int64_t t = target + a.index_offset;
    if (a.out_i) a.out_i[o] = s;
    if (a.out_j) a.out_j[o] = t;
    if (a.out_P) reinterpret_cast<longlong2*>(a.out_P)[o] = make_longlong2(s, t);
    if (a.out_S) {
        a.out_S[3 * o] = static_cast<int32_t>(shift[0]);
        a.out_S[3 * o + 1] = static_cast<int32_t>(shift[1]);
        a.out_S[3 * o + 2] = static_cast<int32_t>(shift[2]);
    }
    if (a.out_D) {
        a.out_D[3 * o] = displacement[0];
        a.out_D[3 * o + 1] = displacement[1];
        a.out_D[3 * o + 2] = displacement[2];
    }
    if (a.out_d) {
        a.out_d[o] = sqrt(exact_norm2(displacement[0], displacement[1], displacement[2]));
    }
}

template <typename T>
__device__ __forceinline__ void exact_displacement(const T* __restrict__ positions, int64_t source,
                                                   int64_t target, const long long (&shift)[3],
                                                   const T* cell, T (&out)[3]) {
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        out[c] = exact_component(positions[3 * target + c], positions[3 * source + c], shift,
                                 cell, c);
    }
}


// ---- cell list -------------------------------------------------------------
//
// One warp per bin: the bin's 27-bin stencil is loaded once and the warp then
// serves every source atom of the bin in turn.  Each of the nine z-rows of
// the stencil is two contiguous slot ranges, one in the zero-image region
// (the sources of those bins) and one in the image-copy region, so a stencil
// is a list of ranges that the search walks as one flattened candidate
// sequence, 32 candidates per tile.  Candidate k of a source is lane k % 32
// of tile k / 32 in both passes, so the count pass hands its per-tile
// ballots to the write pass as a bitmask at a deterministic offset:
//   bin_word_start[bin] + (source rank in bin) * ceil(candidates / 32).
//
// Pair-once stencils (PairOnce = true) drop the zero-image ranges that can
// hold no tested candidate: rows before the source's own row lie in lower
// bins (lower source slots), and the source's own row starts at its bin.

template <bool PairOnce>
struct StencilShape {
    static constexpr int kZeroRanges = PairOnce ? 5 : 9;
    static constexpr int kRanges = kZeroRanges + 9;
    static constexpr int kTable = PairOnce ? 16 : 32;  // power of two > kRanges
};

template <bool PairOnce>
struct StencilRows {
    int32_t prefix[StencilShape<PairOnce>::kTable];  // candidate index where range r
                                                     // starts; [kRanges] = total, then INT_MAX
    int32_t delta[StencilShape<PairOnce>::kRanges];  // slot = candidate index + delta[range]
};

template <typename T>
__device__ __forceinline__ void bin_coordinates(const StructurePlan<T>& plan, int64_t bin,
                                                int32_t& bx, int32_t& by, int32_t& bz) {
    // A structure has fewer than 2^26 bins: 32-bit division suffices.
    const uint32_t local = static_cast<uint32_t>(bin - plan.bin_begin);
    const uint32_t column = local / static_cast<uint32_t>(plan.dims[2]);
    bz = static_cast<int32_t>(local - column * static_cast<uint32_t>(plan.dims[2]));
    const uint32_t plane = column / static_cast<uint32_t>(plan.dims[1]);
    by = static_cast<int32_t>(column - plane * static_cast<uint32_t>(plan.dims[1]));
    bx = static_cast<int32_t>(plane);
}

// Range r of the stencil of bin (bx, by, bz): first ghost slot and length.
// Ranges [0, kZeroRanges) are zero-image ranges of rows (PairOnce: 4..8,
// else 0..8), the rest the image-copy ranges of rows 0..8; row = 3 dx + dy.
template <bool PairOnce, typename T>
__device__ __forceinline__ void stencil_range(const StructurePlan<T>& plan,
                                              const unsigned long long* __restrict__ bin_start,
                                              int64_t n_sources, int32_t bx, int32_t by,
                                              int32_t bz, int r, int32_t& begin, int32_t& length) {
    constexpr int kZero = StencilShape<PairOnce>::kZeroRanges;
    const bool zero = r < kZero;
    const int row = zero ? (PairOnce ? r + 4 : r) : r - kZero;
    begin = 0;
    length = 0;
    const int32_t x = bx + row / 3 - 1;
    const int32_t y = by + row % 3 - 1;
    if (x >= 0 && x < plan.dims[0] && y >= 0 && y < plan.dims[1]) {
        const int32_t z0 = (PairOnce && zero && row == 4) ? bz : max(bz - 1, 0);
        const int32_t z1 = min(bz + 1, plan.dims[2] - 1);
        const int64_t line = plan.bin_begin + (static_cast<int64_t>(x) * plan.dims[1] + y) * plan.dims[2];
        const unsigned long long lo = bin_start[line + z0];
        const unsigned long long hi = bin_start[line + z1 + 1];
        if (zero) {
            begin = static_cast<int32_t>(lo >> 32);
            length = static_cast<int32_t>(hi >> 32) - begin;
        } else {
            begin = static_cast<int32_t>(n_sources) + static_cast<int32_t>(lo & 0xffffffffull);
            length = static_cast<int32_t>(hi & 0xffffffffull) - static_cast<int32_t>(lo & 0xffffffffull);
        }
    }
}

// Lanes fetch one stencil range each and the warp builds the prefix table
// (into `rows` when non-null); returns the total candidate count
// (warp-uniform).
template <bool PairOnce, typename T>
__device__ __forceinline__ int32_t load_stencil(const StructurePlan<T>& plan,
                                                const unsigned long long* __restrict__ bin_start,
                                                int64_t n_sources, int32_t bx, int32_t by,
                                                int32_t bz, StencilRows<PairOnce>* rows, int lane) {
    constexpr int kRanges = StencilShape<PairOnce>::kRanges;
    constexpr int kTable = StencilShape<PairOnce>::kTable;
    int32_t begin = 0, length = 0;
    if (lane < kRanges) stencil_range<PairOnce>(plan, bin_start, n_sources, bx, by, bz, lane, begin, length);
    int32_t inclusive = length;
#pragma unroll
    for (int offset = 1; offset < 32; offset <<= 1) {
        const int32_t other = __shfl_up_sync(kFullMask, inclusive, offset);
        if (lane >= offset) inclusive += other;
    }
    const int32_t total = __shfl_sync(kFullMask, inclusive, kRanges - 1);
    if (rows) {
        if (lane < kRanges) {
            rows->prefix[lane] = inclusive - length;
            rows->delta[lane] = begin - (inclusive - length);
        } else if (lane == kRanges) {
            rows->prefix[lane] = total;
        } else if (lane < kTable) {
            rows->prefix[lane] = INT_MAX;
        }
    }
    __syncwarp();
    return total;
}

// The same table built by one thread; returns the total.
template <bool PairOnce, typename T>
__device__ __forceinline__ int32_t build_stencil(const StructurePlan<T>& plan,
                                                 const unsigned long long* __restrict__ bin_start,
                                                 int64_t n_sources, int32_t bx, int32_t by,
                                                 int32_t bz, StencilRows<PairOnce>& rows) {
    constexpr int kRanges = StencilShape<PairOnce>::kRanges;
    int32_t prefix = 0;
#pragma unroll
    for (int r = 0; r < kRanges; ++r) {
        int32_t begin, length;
        stencil_range<PairOnce>(plan, bin_start, n_sources, bx, by, bz, r, begin, length);
        rows.prefix[r] = prefix;
        rows.delta[r] = begin - prefix;
        prefix += length;
    }
    rows.prefix[kRanges] = prefix;
#pragma unroll
    for (int r = kRanges + 1; r < StencilShape<PairOnce>::kTable; ++r) rows.prefix[r] = INT_MAX;
    return prefix;
}

// Position of the (n+1)-th set bit of w (0 <= n < popc(w)), by halving.
__device__ __forceinline__ int32_t nth_set_bit(uint32_t w, int32_t n) {
    int32_t position = 0;
#pragma unroll
    for (int width = 16; width > 0; width >>= 1) {
        const uint32_t low = w & ((1u << width) - 1u);
        const int32_t c = __popc(low);
        if (n >= c) {
            n -= c;
            w >>= width;
            position += width;
        } else {
            w = low;
        }
    }
    return position;
}

// Slot of candidate index k (0 <= k < total): the last range whose prefix is
// <= k, found by halving the power-of-two table.
template <bool PairOnce>
__device__ __forceinline__ int32_t slot_of(const StencilRows<PairOnce>& rows, int32_t k) {
    int32_t r = 0;
#pragma unroll
    for (int step = StencilShape<PairOnce>::kTable / 2; step > 0; step >>= 1) {
        r += (rows.prefix[r + step] <= k) ? step : 0;
    }
    return k + rows.delta[r];
}


// slot_of with the lane's current range cached: a new range is looked up only
// when k passes range_end (0 forces a lookup).
template <bool PairOnce>
__device__ __forceinline__ int32_t cached_slot(const StencilRows<PairOnce>& rows, int32_t k,
                                               int32_t& range_end, int32_t& range_delta) {
    if (k >= range_end) {
        int32_t r = 0;
#pragma unroll
        for (int step = StencilShape<PairOnce>::kTable / 2; step > 0; step >>= 1) {
            r += (rows.prefix[r + step] <= k) ? step : 0;
        }
        range_end = rows.prefix[r + 1];
        range_delta = rows.delta[r];
    }
    return k + range_delta;
}

// Per bin: bitmask words of all its sources (sources * ceil(candidates / 32)).
// One thread per bin; its row-bound loads are independent.
template <bool PairOnce, typename T>
__global__ void __launch_bounds__(kBinThreads) stencil_words_kernel(SearchArgs<T> args,
                                                                    int64_t n_bins,
                                                                    unsigned long long* bin_words) {
    const int64_t bin = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (bin >= n_bins) return;
    const unsigned long long sources = (args.bin_start[bin + 1] >> 32) - (args.bin_start[bin] >> 32);
    if (sources == 0) {
        bin_words[bin] = 0;
        return;
    }
    const StructurePlan<T>& plan = args.plans[args.bin_struct[bin]];
    int32_t bx, by, bz;
    bin_coordinates(plan, bin, bx, by, bz);
    int64_t total = 0;
#pragma unroll
    for (int r = 0; r < StencilShape<PairOnce>::kRanges; ++r) {
        int32_t begin, length;
        stencil_range<PairOnce>(plan, args.bin_start, args.n_sources, bx, by, bz, r, begin, length);
        total += length;
    }
    bin_words[bin] = sources * static_cast<unsigned long long>((total + 31) >> 5);
}

// Packed pairs of floats (sm_100 f32x2 arithmetic): two source-candidate
// screening tests per instruction in the count pass.
__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void unpack2(unsigned long long v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
// Squared distances of one point (packed as (c, c) per axis) to two sources;
// per element exactly screen_distance2 below.
__device__ __forceinline__ unsigned long long distance2_pair(
    unsigned long long cx, unsigned long long cy, unsigned long long cz,
    unsigned long long sx, unsigned long long sy, unsigned long long sz) {
    unsigned long long dx, dy, dz, d2;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(dx) : "l"(cx), "l"(sx));
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(dy) : "l"(cy), "l"(sy));
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(dz) : "l"(cz), "l"(sz));
    asm("mul.rn.f32x2 %0, %1, %1;" : "=l"(d2) : "l"(dx));
    asm("fma.rn.f32x2 %0, %1, %1, %0;" : "+l"(d2) : "l"(dy));
    asm("fma.rn.f32x2 %0, %1, %1, %0;" : "+l"(d2) : "l"(dz));
    return d2;
}

// The screening distance in scalar form (double sources in the count pass).
__device__ __forceinline__ double screen_distance2(double cx, double cy, double cz, double sx,
                                                   double sy, double sz) {
    const double dx = __dsub_rn(cx, sx), dy = __dsub_rn(cy, sy), dz = __dsub_rn(cz, sz);
    return __fma_rn(dz, dz, __fma_rn(dy, dy, __dmul_rn(dx, dx)));
}

// 32 x 32 bit-matrix transpose across a warp: on entry bit r of lane c's x
// is element (c, r); on return bit c of lane r's value is that element.
// Five butterfly stages exchange the off-diagonal blocks of width j.
__device__ __forceinline__ uint32_t transpose_bits32(uint32_t x, int lane) {
    const uint32_t low_masks[5] = {0x0000ffffu, 0x00ff00ffu, 0x0f0f0f0fu, 0x33333333u, 0x55555555u};
#pragma unroll
    for (int stage = 0; stage < 5; ++stage) {
        const int j = 16 >> stage;
        const uint32_t m = low_masks[stage];
        const uint32_t y = __shfl_xor_sync(kFullMask, x, j);
        x = (lane & j) ? ((x & ~m) | ((y & ~m) >> j)) : ((x & m) | ((y & m) << j));
    }
    return x;
}

// Count pass, lanes = candidates: the warp serves one bin.  Each lane holds
// one candidate of the bin's stencil (32 per tile) in registers; the bin's
// sources are staged once in shared memory (up to 32 at a time, structure of
// arrays) and read back as broadcasts, four per vector load.  Each lane tests
// its candidate against every source -- for float two sources per packed
// f32x2 instruction -- and shifts the sign bits of d2 - inner2 and
// d2 - search2 into two words (one funnel shift per test); a 32 x 32 bit
// transpose across the warp then gives every source its mask word for the
// tile.  The lanes stay busy whatever the bin's source count.
//
// Half lists and pair-once calls compare order keys.  The ghost record's
// fourth lane carries key 2a + 1 for the zero image of a and 2a + 2 for its
// other images (written by the scatter), a = the atom, or for pair-once
// calls the atom's source slot; a source's key is 2a + 1.
// Key(c) > key(s) + 1 means a(c) > a(s) (accepted by distance alone),
// tested as the sign of (key(s) + 1) - key(c); key(c) == key(s) + 1 is a
// periodic image of the source itself (decided by its shift in the rare
// path); key(c) == key(s) is the zero-shift self pair, which the test neither
// accepts nor flags and which is set afterwards per include_self.
// Full lists accept the self pair by distance (d = 0) and fix it the same
// way.  Pair-once calls leave it out of the bitmask and count it per
// include_self; a pair-once half list emits each accepted pair once in its
// canonical orientation, a full list emits it in both.  Candidates in the band shell are flagged per lane and the flagged
// lanes decide them exactly.
// Accepted-candidate bits are stored transposed -- word w of source rank r at
// base + w * S + r, S the bin's source count -- one coalesced store per tile.

// Appends the sign bit of `value` to `bits` (bits = bits << 1 | sign).
__device__ __forceinline__ uint32_t push_sign(uint32_t bits, float value) {
    return __funnelshift_l(static_cast<uint32_t>(__float_as_int(value)), bits, 1);
}
__device__ __forceinline__ uint32_t push_sign(uint32_t bits, double value) {
    return __funnelshift_l(static_cast<uint32_t>(__double2hiint(value)), bits, 1);
}
__device__ __forceinline__ unsigned long long sub2(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint32_t push_signs2(uint32_t bits, unsigned long long pair) {
    float lo, hi;
    unpack2(pair, lo, hi);
    return push_sign(push_sign(bits, lo), hi);
}

// Appends bit [key(s) + 1 < key(c)] to `bits`.  Keys of one structure differ
// by less than 2^31 (fewer than 2^30 atoms), so the signed difference is exact.
__device__ __forceinline__ uint32_t push_key(uint32_t bits, uint32_t source_key_plus_one,
                                             uint32_t candidate_key) {
    return __funnelshift_l(source_key_plus_one - candidate_key, bits, 1);
}

template <typename T, bool Half, bool PairOnce>
__global__ void __launch_bounds__(kSearchThreads) cell_count_kernel(SearchArgs<T> args) {
    using V = vec4_t<T>;
    constexpr bool Keyed = Half || PairOnce;
    __shared__ StencilRows<PairOnce> stencil[kSearchWarps];
    // Sources of the current block, structure of arrays (16-byte aligned
    // rows so four consecutive sources load as one vector).
    __shared__ __align__(16) T source_x[kSearchWarps][32];
    __shared__ __align__(16) T source_y[kSearchWarps][32];
    __shared__ __align__(16) T source_z[kSearchWarps][32];
    __shared__ __align__(16) uint32_t source_key[kSearchWarps][32];
    __shared__ int32_t source_atom[kSearchWarps][32];
    // A bitmask sized from a bound that the scanned total exceeds (never,
    // for a correct bound) is flagged before this pass: nothing is written.
    if (*args.status & kStatusCapacity) return;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // Warp w serves bins w, w + stride, w + 2 stride, ...; it probes the
    // next 32 of them at once (lane l reads bin base + l * stride) and
    // visits only those with sources (halo bins hold ghosts but no sources),
    // so an empty bin costs no load round trip of its own.
    const int64_t stride = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    for (int64_t base = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
         base < args.n_bins; base += 32 * stride) {
      const int64_t my_bin = base + lane * stride;
      uint32_t my_first = 0, my_count = 0;
      if (my_bin < args.n_bins) {
          my_first = static_cast<uint32_t>(args.bin_start[my_bin] >> 32);
          my_count = static_cast<uint32_t>(args.bin_start[my_bin + 1] >> 32) - my_first;
      }
      unsigned pending = __ballot_sync(kFullMask, my_count != 0u);
      while (pending != 0u) {
        const int chosen = __ffs(pending) - 1;
        pending &= pending - 1u;
        const int64_t bin = base + chosen * stride;
        const uint32_t first_source = __shfl_sync(kFullMask, my_first, chosen);
        const uint32_t n_sources = __shfl_sync(kFullMask, my_count, chosen);
        const StructurePlan<T>& plan = args.plans[args.bin_struct[bin]];
        int32_t bx, by, bz;
        bin_coordinates(plan, bin, bx, by, bz);
        StencilRows<PairOnce>& rows = stencil[warp];
        const int32_t total = load_stencil<PairOnce>(plan, args.bin_start, args.n_sources, bx, by, bz,
                                                     &rows, lane);
        const int32_t words = (total + 31) >> 5;
        uint32_t* mask = args.mask_words + args.bin_word_start[bin];
        const T search2 = plan.search_squared;
        const T inner2 = plan.inner_squared;
        const bool self_images = plan.self_images != 0;
        unsigned long long inner_pair = 0, search_pair = 0;
        if constexpr (std::is_same<T, float>::value) {
            inner_pair = pack2(inner2, inner2);
            search_pair = pack2(search2, search2);
        }

        for (uint32_t base = 0; base < n_sources; base += 32) {
            const int block = static_cast<int>(min(32u, n_sources - base));
            // Sources are padded to a multiple of four with NaN positions;
            // their bits are masked off below.
            const int padded = (block + 3) & ~3;
            const uint32_t valid_mask = block == 32 ? kFullMask : (1u << block) - 1u;
            int32_t my_source = -1;
            int32_t self_k = -1;  // candidate index of my source's zero image
            __syncwarp();
            if (lane < block) {
                my_source = args.source_list[first_source + base + lane];
                const V q = reinterpret_cast<const V*>(args.wrapped)[my_source];
                source_x[warp][lane] = q.x;
                source_y[warp][lane] = q.y;
                source_z[warp][lane] = q.z;
                source_atom[warp][lane] = my_source;
                // key(s) + 1 (keyed searches); the slot is the zero image's.
                const uint32_t slot = first_source + base + lane;
                source_key[warp][lane] = PairOnce ? 2u * slot + 2u
                                                  : 2u * static_cast<uint32_t>(my_source) + 2u;
                if constexpr (!PairOnce) {
#pragma unroll
                    for (int r = 0; r < StencilShape<false>::kZeroRanges; ++r) {
                        const int32_t begin_r = rows.prefix[r] + rows.delta[r];
                        const int32_t length_r = rows.prefix[r + 1] - rows.prefix[r];
                        if (static_cast<int32_t>(slot) >= begin_r &&
                            static_cast<int32_t>(slot) < begin_r + length_r) {
                            self_k = rows.prefix[r] + (static_cast<int32_t>(slot) - begin_r);
                        }
                    }
                }
            } else if (lane < padded) {
                source_x[warp][lane] = source_y[warp][lane] = source_z[warp][lane] =
                    static_cast<T>(NAN);
                source_key[warp][lane] = 0u;
            }
            __syncwarp();
            // Range of the block's key(s) + 1 values.
            uint32_t block_key_lo = 0u, block_key_hi = 0u;
            if constexpr (Keyed) {
                const uint32_t mine = lane < block ? source_key[warp][lane] : 0u;
                block_key_lo = __reduce_min_sync(kFullMask, lane < block ? mine : 0xffffffffu);
                block_key_hi = __reduce_max_sync(kFullMask, mine);
            }
            uint32_t count = 0;
            // This lane's candidate of tile w, loaded one tile ahead.  The
            // lane walks the stencil rows forward (k grows by 32 per tile):
            // `row` is the row holding k, row_end its end.
            int32_t row = 0;
            int32_t row_end = rows.prefix[1];
            auto load_candidate = [&](int32_t w, V& record, int32_t& slot) {
                const int32_t k = 32 * w + lane;
                if (k < total) {
                    while (k >= row_end) row_end = rows.prefix[++row + 1];
                    slot = k + rows.delta[row];
                    record = reinterpret_cast<const V*>(args.ghost_pos)[slot];
                } else {
                    slot = -1;
                    record.x = static_cast<T>(INFINITY);
                    record.y = T(0);
                    record.z = T(0);
                    record.w = index_to_lane(0, T(0));
                }
            };
            V next;
            int32_t next_slot;
            load_candidate(0, next, next_slot);
            uint32_t* mask_out = mask + base + lane;  // word w of my source at w * n_sources
            for (int32_t w = 0; w < words; ++w) {
                const V cand = next;
                const int32_t slot = next_slot;
                if (w + 1 < words) load_candidate(w + 1, next, next_slot);
                const uint32_t key = static_cast<uint32_t>(lane_to_index(cand.w));
                uint32_t key_signs = 0;  // keyed: bit r = key(s_r) + 1 < key(c)
                uint32_t inner_signs = 0, search_signs = 0;
                // A tile whose candidates' keys all lie above or below the
                // block's key(s) + 1 values needs no per-test key bit (a key
                // equal to one of them is a periodic image of that source,
                // which the keyed path flags).
                bool keyed_tile = false;
                uint32_t uniform_keys = 0u;
                if constexpr (Keyed) {
                    keyed_tile = __any_sync(kFullMask, key >= block_key_lo && key <= block_key_hi);
                    uniform_keys = key > block_key_hi ? valid_mask : 0u;
                }
                auto tests = [&](auto with_keys) {
                  constexpr bool KeyBits = decltype(with_keys)::value;
                  if constexpr (std::is_same<T, float>::value) {
                    const unsigned long long cx = pack2(cand.x, cand.x);
                    const unsigned long long cy = pack2(cand.y, cand.y);
                    const unsigned long long cz = pack2(cand.z, cand.z);
                    for (int r0 = 0; r0 < padded; r0 += 4) {
                        const ulonglong2 sx = *reinterpret_cast<const ulonglong2*>(&source_x[warp][r0]);
                        const ulonglong2 sy = *reinterpret_cast<const ulonglong2*>(&source_y[warp][r0]);
                        const ulonglong2 sz = *reinterpret_cast<const ulonglong2*>(&source_z[warp][r0]);
                        const unsigned long long d01 = distance2_pair(cx, cy, cz, sx.x, sy.x, sz.x);
                        const unsigned long long d23 = distance2_pair(cx, cy, cz, sx.y, sy.y, sz.y);
                        inner_signs = push_signs2(push_signs2(inner_signs, sub2(d01, inner_pair)),
                                                  sub2(d23, inner_pair));
                        search_signs = push_signs2(push_signs2(search_signs, sub2(d01, search_pair)),
                                                   sub2(d23, search_pair));
                        if constexpr (KeyBits) {
                            const uint4 k = *reinterpret_cast<const uint4*>(&source_key[warp][r0]);
                            key_signs = push_key(push_key(push_key(push_key(key_signs, k.x, key), k.y, key),
                                                          k.z, key), k.w, key);
                        }
                    }
                  } else {
                    for (int r = 0; r < padded; ++r) {
                        const T d2 = screen_distance2(cand.x, cand.y, cand.z, source_x[warp][r],
                                                      source_y[warp][r], source_z[warp][r]);
                        inner_signs = push_sign(inner_signs, d2 - inner2);
                        search_signs = push_sign(search_signs, d2 - search2);
                        if constexpr (KeyBits) key_signs = push_key(key_signs, source_key[warp][r], key);
                    }
                  }
                };
                if (keyed_tile) tests(std::true_type{}); else tests(std::false_type{});
                // Bit r: d2 to source r below the inner / search radius.
                const uint32_t inside = __brev(inner_signs) >> (32 - padded);
                const uint32_t near = __brev(search_signs) >> (32 - padded);
                uint32_t keep_keys = valid_mask, band_keys = valid_mask;
                if constexpr (Keyed) {
                    keep_keys = band_keys = keyed_tile
                        ? (__brev(key_signs) >> (32 - padded)) & valid_mask : uniform_keys;
                    // key(c) == key(s) + 1: an image of source s itself, only
                    // possible where a lattice translation is shorter than the
                    // search radius; its shift decides it in the rare path.
                    if (keyed_tile && self_images && (key & 1u) == 0u && key != 0u) {
                        for (int r = 0; r < block; ++r) {
                            if (source_key[warp][r] == key) band_keys |= 1u << r;
                        }
                    }
                }
                uint32_t keep_bits = inside & keep_keys;
                uint32_t rare = near & band_keys & ~keep_bits;
                if (__any_sync(kFullMask, rare != 0u) && rare != 0u) {
                    // Rare: band shell, or a half-list periodic image of the
                    // source itself; decided exactly by the candidate's lane.
                    const int4 meta = args.ghost_meta[slot];  // .w: the candidate's atom
                    do {
                        const int r = __ffs(rare) - 1;
                        rare &= rare - 1u;
                        const int32_t source = source_atom[warp][r];
                        const long long shift[3] = {
                            meta.x + static_cast<long long>(args.wraps[3 * source]),
                            meta.y + static_cast<long long>(args.wraps[3 * source + 1]),
                            meta.z + static_cast<long long>(args.wraps[3 * source + 2])};
                        bool keep = true;
                        if (Keyed && meta.w == source) keep = canonical_shift(shift);
                        if (keep && !((inside >> r) & 1u)) {
                            const T* pt = args.positions + 3 * static_cast<int64_t>(meta.w);
                            const T vx = exact_component(pt[0], args.positions[3 * source], shift, plan.cell, 0);
                            const T vy = exact_component(pt[1], args.positions[3 * source + 1], shift, plan.cell, 1);
                            const T vz = exact_component(pt[2], args.positions[3 * source + 2], shift, plan.cell, 2);
                            keep = exact_norm2(vx, vy, vz) < plan.cutoff_squared;
                        }
                        if (keep) keep_bits |= 1u << r;
                    } while (rare != 0u);
                }
                // Transpose the warp's 32 x 32 bit matrix: afterwards lane r
                // holds source r's word (bit c = candidate lane c accepted).
                const uint32_t my_word_bits = transpose_bits32(keep_bits, lane);
                if (lane < block) {
                    uint32_t my_word = my_word_bits;
                    if (!PairOnce && (self_k >> 5) == w) {
                        const uint32_t bit = 1u << (self_k & 31);
                        my_word = args.include_self ? (my_word | bit) : (my_word & ~bit);
                    }
                    *mask_out = my_word;
                    count += __popc(my_word);
                }
                mask_out += n_sources;
            }
            if (PairOnce) count = (Half ? count : 2u * count) + (args.include_self ? 1u : 0u);
            if (lane < block) {
                args.counts[args.source_order ? static_cast<int64_t>(first_source + base + lane)
                                              : my_source] = count;
                if (count > static_cast<uint32_t>(INT_MAX)) {
                    atomicOr(args.status, static_cast<uint32_t>(kStatusCountRange));
                }
            }
        }
      }
    }
}

// Write pass.  The warp replays the count pass's ballots for the sources of
// its bin (32 at a time; each lane first loads one source's data into shared
// memory) and queues accepted (candidate, source) entries.  Every 32 entries
// the whole warp emits 32 consecutive output rows: each lane loads its
// candidate's records (the ghost's shift and the target's original position
// are stored with the ghost, so no dependent gather follows), evaluates the
// public displacement, and the 12-byte S / D rows are staged in shared memory
// so that every global store instruction is a contiguous 128-byte run.
// Unsorted calls write pairs in cell order, so one bin is one contiguous
// output range and the queue streams across its sources; sorted calls write
// each source's pairs at its own offset and flush at source boundaries.
// Distance of an emitted pair from its displacement.  float: d2 * rsqrt(d2)
// (relative error ~2^-22, far inside the 1e-5 contract); double: sqrt.
__device__ __forceinline__ float pair_distance(float x, float y, float z) {
    const float d2 = exact_norm2(x, y, z);
    return d2 > 0.0f ? d2 * rsqrtf(d2) : 0.0f;
}
__device__ __forceinline__ double pair_distance(double x, double y, double z) {
    return sqrt(exact_norm2(x, y, z));
}

template <typename T>
struct WriteShared {
    int32_t queue_k[64];
    uint8_t queue_r[64];
    vec4_t<T> source_pos[32];  // original source position, w = source index
    int4 source_wrap[32];
    int32_t stage_S[96];
    T stage_D[96];
};

// Output sets the write kernels are specialised for (tnr_quantity bits);
// any other set uses the run-time checked variant (Q = 0).
constexpr int kQ_I = 1, kQ_J = 2, kQ_P = 4, kQ_S = 8, kQ_d = 16, kQ_D = 32;

template <int Q>
__device__ __forceinline__ bool wants(const void* pointer, int bit) {
    if constexpr (Q == 0) return pointer != nullptr;
    return (Q & bit) != 0;
}

template <typename T, int Q>
__device__ __forceinline__ void flush_queue(const SearchArgs<T>& args, const StructurePlan<T>& plan,
                                            WriteShared<T>& sh,
                                            int32_t n, int64_t out_row, int lane,
                                            bool need_shift, bool need_vector) {
    using V = vec4_t<T>;
    __syncwarp();
    int32_t shift[3] = {0, 0, 0};
    T vec[3] = {T(0), T(0), T(0)};
    int64_t source = 0, target = 0;
    if (lane < n) {
        const int32_t slot = sh.queue_k[lane];
        const int r = sh.queue_r[lane];
        const V ps = sh.source_pos[r];
        source = lane_to_index(ps.w);
        if (need_shift || need_vector) {
            const int4 meta = args.ghost_meta[slot];
            const int4 ws = sh.source_wrap[r];
            target = meta.w;
            // Cell-list shifts fit int32 by construction of the plan.
            shift[0] = meta.x + ws.x;
            shift[1] = meta.y + ws.y;
            shift[2] = meta.z + ws.z;
            if (need_vector) {
                const V pt = reinterpret_cast<const V*>(args.ghost_orig)[slot];
                const T s0 = static_cast<T>(shift[0]);
                const T s1 = static_cast<T>(shift[1]);
                const T s2 = static_cast<T>(shift[2]);
                const T* cell = plan.cell;
                vec[0] = add_rn(add_rn(add_rn(sub_rn(pt.x, ps.x), mul_rn(s0, cell[0])),
                                       mul_rn(s1, cell[3])), mul_rn(s2, cell[6]));
                vec[1] = add_rn(add_rn(add_rn(sub_rn(pt.y, ps.y), mul_rn(s0, cell[1])),
                                       mul_rn(s1, cell[4])), mul_rn(s2, cell[7]));
                vec[2] = add_rn(add_rn(add_rn(sub_rn(pt.z, ps.z), mul_rn(s0, cell[2])),
                                       mul_rn(s1, cell[5])), mul_rn(s2, cell[8]));
            }
        } else {
            const uint32_t key =
                static_cast<uint32_t>(lane_to_index(reinterpret_cast<const V*>(args.ghost_pos)[slot].w));
            target = static_cast<int32_t>((key - 1u) >> 1);
        }
        const int64_t s = source + args.index_offset;
        const int64_t t = target + args.index_offset;
        if (wants<Q>(args.out_i, kQ_I)) (args.out_i + out_row)[lane] = s;
        if (wants<Q>(args.out_j, kQ_J)) (args.out_j + out_row)[lane] = t;
        if (wants<Q>(args.out_P, kQ_P)) (reinterpret_cast<longlong2*>(args.out_P) + out_row)[lane] = make_longlong2(s, t);
        if (wants<Q>(args.out_d, kQ_d)) (args.out_d + out_row)[lane] = pair_distance(vec[0], vec[1], vec[2]);
        if (wants<Q>(args.out_S, kQ_S)) {
            sh.stage_S[3 * lane] = shift[0];
            sh.stage_S[3 * lane + 1] = shift[1];
            sh.stage_S[3 * lane + 2] = shift[2];
        }
        if (wants<Q>(args.out_D, kQ_D)) {
            sh.stage_D[3 * lane] = vec[0];
            sh.stage_D[3 * lane + 1] = vec[1];
            sh.stage_D[3 * lane + 2] = vec[2];
        }
    }
    __syncwarp();
    const int32_t words = 3 * n;
    if (wants<Q>(args.out_S, kQ_S)) {
        int32_t* out = args.out_S + 3 * out_row;
#pragma unroll
        for (int m = 0; m < 3; ++m) {
            const int32_t e = lane + 32 * m;
            if (e < words) out[e] = sh.stage_S[e];
        }
    }
    if (wants<Q>(args.out_D, kQ_D)) {
        T* out = args.out_D + 3 * out_row;
#pragma unroll
        for (int m = 0; m < 3; ++m) {
            const int32_t e = lane + 32 * m;
            if (e < words) out[e] = sh.stage_D[e];
        }
    }
    __syncwarp();
}

template <typename T, int Q>
__global__ void __launch_bounds__(kSearchThreads) cell_write_kernel(SearchArgs<T> args) {
    using V = vec4_t<T>;
    __shared__ StencilRows<false> stencil[kSearchWarps];
    __shared__ WriteShared<T> shared[kSearchWarps];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const bool need_vector = wants<Q>(args.out_d, kQ_d) || wants<Q>(args.out_D, kQ_D);
    const bool need_shift = wants<Q>(args.out_S, kQ_S);
    const bool by_atom = args.source_order == 0;
    WriteShared<T>& sh = shared[warp];
    const int64_t stride = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    // Bins probed 32 at a time, as in the count pass.
    for (int64_t base = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
         base < args.n_bins; base += 32 * stride) {
      const int64_t my_bin = base + lane * stride;
      uint32_t my_first = 0, my_count = 0;
      if (my_bin < args.n_bins) {
          my_first = static_cast<uint32_t>(args.bin_start[my_bin] >> 32);
          my_count = static_cast<uint32_t>(args.bin_start[my_bin + 1] >> 32) - my_first;
      }
      unsigned pending = __ballot_sync(kFullMask, my_count != 0u);
      while (pending != 0u) {
        const int chosen = __ffs(pending) - 1;
        pending &= pending - 1u;
        const int64_t bin = base + chosen * stride;
        const uint32_t first_source = __shfl_sync(kFullMask, my_first, chosen);
        const uint32_t n_bin_sources = __shfl_sync(kFullMask, my_count, chosen);
        const StructurePlan<T>& plan = args.plans[args.bin_struct[bin]];
        int32_t bx, by, bz;
        bin_coordinates(plan, bin, bx, by, bz);
        StencilRows<false>& rows = stencil[warp];
        const int32_t total = load_stencil<false>(plan, args.bin_start, args.n_sources, bx, by, bz,
                                                  &rows, lane);
        const int32_t words = (total + 31) >> 5;
        const uint32_t* bin_mask = args.mask_words + args.bin_word_start[bin];
        int64_t out_row = by_atom ? 0 : args.pair_start[first_source];

        for (uint32_t base = 0; base < n_bin_sources; base += 32) {
            const uint32_t mine = base + lane;
            int64_t my_start = 0;
            __syncwarp();
            if (mine < n_bin_sources) {
                const int32_t source = args.source_list[first_source + mine];
                if (by_atom) my_start = args.pair_start[source];
                V ps;
                ps.x = args.positions[3 * source];
                ps.y = args.positions[3 * source + 1];
                ps.z = args.positions[3 * source + 2];
                ps.w = index_to_lane(source, T(0));
                sh.source_pos[lane] = ps;
                sh.source_wrap[lane] = make_int4(args.wraps[3 * source], args.wraps[3 * source + 1],
                                                 args.wraps[3 * source + 2], 0);
            }
            __syncwarp();
            const int32_t group = static_cast<int32_t>(min(32u, n_bin_sources - base));
            // Items are (source, word) pairs.  Unsorted: all items of the
            // group form one flat sequence and their pairs are consecutive
            // rows.  Sorted: one source at a time, rows from its own start.
            const int32_t passes = by_atom ? group : 1;
            const int32_t n_items = by_atom ? words : group * words;
            for (int32_t pass = 0; pass < passes; ++pass) {
                if (by_atom) out_row = __shfl_sync(kFullMask, my_start, pass);
                for (int32_t item0 = 0; item0 < n_items; item0 += 32) {
                    const int32_t item = item0 + lane;
                    int32_t r = pass, w = item;
                    if (!by_atom) {
                        r = item / words;
                        w = item - r * words;
                    }
                    const uint32_t word = item < n_items
                        ? bin_mask[static_cast<int64_t>(w) * n_bin_sources + base + r] : 0u;
                    const int32_t count = __popc(word);
                    const int32_t inclusive = warp_inclusive_sum(count);
                    const int32_t exclusive = inclusive - count;
                    const int32_t produced = __shfl_sync(kFullMask, inclusive, 31);
                    for (int32_t i = 0; i < produced; i += 32) {
                        const int32_t g = i + lane;
                        // Lane holding the item of pair g: the last lane
                        // whose exclusive offset is <= g.
                        int32_t at = 0;
#pragma unroll
                        for (int step = 16; step > 0; step >>= 1) {
                            const int32_t probe = __shfl_sync(kFullMask, exclusive, at + step);
                            if (probe <= g) at += step;
                        }
                        const uint32_t item_word = __shfl_sync(kFullMask, word, at);
                        const int32_t item_start = __shfl_sync(kFullMask, exclusive, at);
                        const int32_t item_r = __shfl_sync(kFullMask, r, at);
                        const int32_t item_w = __shfl_sync(kFullMask, w, at);
                        const int32_t n = min(32, produced - i);
                        if (g < produced) {
                            const int32_t bit = nth_set_bit(item_word, g - item_start);
                            sh.queue_k[lane] = slot_of(rows, 32 * item_w + bit);
                            sh.queue_r[lane] = static_cast<uint8_t>(item_r);
                        }
                        flush_queue<T, Q>(args, plan, sh, n, out_row + i, lane, need_shift,
                                    need_vector);
                    }
                    out_row += produced;
                }
            }
        }
      }
    }
}

// Write pass for unsorted calls.  In cell order any 32 consecutive sources
// own one contiguous output range, whatever bins they belong to, so one warp
// takes 32 consecutive sources and may write their pairs in any order inside
// that range.  The sources' stencil-row tables, positions, wraps and cells
// are staged in shared memory.  Work is handed out per bitmask word: the warp
// loads word w of all 32 sources at once (one coalesced load; the next batch
// is already in flight), and a lane whose word is used up takes the next
// nonzero word of the batch, so every lane stays busy however unequal the
// sources' pair counts are (half lists make them very unequal).  In each
// round every busy lane takes one accepted candidate of its word, the ghost
// records of that pair are loaded a round ahead, and the round's rows are
// assigned by a ballot prefix so that each store covers one contiguous run.
//
// Unsorted calls are pair-once: every accepted candidate gives one row in its canonical
// orientation (half lists: the lower atom first, shifts and displacement
// evaluated for that orientation) or two rows (full lists: both
// orientations, in adjacent rows or, when the outputs are not aligned for
// that, in the two halves of each chunk); the group's self pairs
// (include_self) come last.
// Every displacement is the reference's public formula for the row's own
// orientation, so a reversed row equals what the reference computes for it.
#ifndef TNR_EMIT_PER_LANE
#define TNR_EMIT_PER_LANE 6
#endif
constexpr int kEmitPerLane = TNR_EMIT_PER_LANE;
constexpr int kEmitQueue = 32 * kEmitPerLane;

template <typename T>
struct EmitShared {
    StencilRows<true> rows[32];
    // Per-source values as separate 4/8-byte arrays: lanes reading different
    // sources hit different banks.
    T pos[3][32];        // original source position
    int32_t wrap[3][32]; // source wraps
    int32_t atom[32];    // source atom
    T cell[9][32];       // source's cell (read only when the group's sources
                         // span several structures)
    int2 mailbox[32];
    int2 queue[2][kEmitQueue];  // (ghost slot, source lane), double buffered
};

constexpr int kEmitThreads = 128;

// Public displacement of one output row: (to - from) + S . cell in the
// reference's operation order.
template <typename T>
__device__ __forceinline__ void row_vector(const T (&to)[3], const T (&from)[3],
                                           const int32_t (&shift)[3], const T (&cell)[9],
                                           T (&vec)[3]) {
    const T s0 = static_cast<T>(shift[0]);
    const T s1 = static_cast<T>(shift[1]);
    const T s2 = static_cast<T>(shift[2]);
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        vec[c] = add_rn(add_rn(add_rn(sub_rn(to[c], from[c]), mul_rn(s0, cell[c])),
                               mul_rn(s1, cell[3 + c])), mul_rn(s2, cell[6 + c]));
    }
}

template <typename T, int Q>
__device__ __forceinline__ void store_row(const SearchArgs<T>& args, int64_t o, int64_t s,
                                          int64_t t, const int32_t (&shift)[3],
                                          const T (&vec)[3]) {
    if (wants<Q>(args.out_i, kQ_I)) args.out_i[o] = s;
    if (wants<Q>(args.out_j, kQ_J)) args.out_j[o] = t;
    if (wants<Q>(args.out_P, kQ_P)) {
        reinterpret_cast<longlong2*>(args.out_P)[o] = make_longlong2(s, t);
    }
    if (wants<Q>(args.out_S, kQ_S)) {
        int32_t* row = args.out_S + 3 * o;
        row[0] = shift[0];
        row[1] = shift[1];
        row[2] = shift[2];
    }
    if (wants<Q>(args.out_d, kQ_d)) args.out_d[o] = pair_distance(vec[0], vec[1], vec[2]);
    if (wants<Q>(args.out_D, kQ_D)) {
        T* row = args.out_D + 3 * o;
        row[0] = vec[0];
        row[1] = vec[1];
        row[2] = vec[2];
    }
}

// Both orientations of one full-list pair as adjacent rows o (even) and o + 1:
// 16-byte index stores and 8- or 16-byte S, d and D stores (the host checks
// the outputs' alignment; rows of a full list start at even offsets).
template <typename T> struct Pair2;
template <> struct Pair2<float> { using type = float2; };
template <> struct Pair2<double> { using type = double2; };

template <typename T, int Q>
__device__ __forceinline__ void store_row_pair(const SearchArgs<T>& args, int64_t o, int64_t s,
                                               int64_t t, const int32_t (&shift)[3],
                                               const T (&vec)[3], const T (&back)[3]) {
    using T2 = typename Pair2<T>::type;
    if (wants<Q>(args.out_i, kQ_I)) *reinterpret_cast<longlong2*>(args.out_i + o) = make_longlong2(s, t);
    if (wants<Q>(args.out_j, kQ_J)) *reinterpret_cast<longlong2*>(args.out_j + o) = make_longlong2(t, s);
    if (wants<Q>(args.out_P, kQ_P)) {
        longlong2* row = reinterpret_cast<longlong2*>(args.out_P) + o;
        row[0] = make_longlong2(s, t);
        row[1] = make_longlong2(t, s);
    }
    if (wants<Q>(args.out_S, kQ_S)) {
        int2* row = reinterpret_cast<int2*>(args.out_S + 3 * o);
        row[0] = make_int2(shift[0], shift[1]);
        row[1] = make_int2(shift[2], -shift[0]);
        row[2] = make_int2(-shift[1], -shift[2]);
    }
    if (wants<Q>(args.out_d, kQ_d)) {
        // The reversed displacement has the same magnitudes component by
        // component (round-to-nearest is sign-symmetric), so the same d.
        const T d = pair_distance(vec[0], vec[1], vec[2]);
        *reinterpret_cast<T2*>(args.out_d + o) = T2{d, d};
    }
    if (wants<Q>(args.out_D, kQ_D)) {
        T2* row = reinterpret_cast<T2*>(args.out_D + 3 * o);
        row[0] = T2{vec[0], vec[1]};
        row[1] = T2{vec[2], back[0]};
        row[2] = T2{back[1], back[2]};
    }
}

template <typename T, int Q, bool Half>
__global__ void __launch_bounds__(kEmitThreads) cell_emit_kernel(SearchArgs<T> args) {
    using V = vec4_t<T>;
    constexpr int PerLane = kEmitPerLane;
    __shared__ EmitShared<T> shared[kEmitThreads / 32];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const unsigned below = (1u << lane) - 1u;
    const bool need_vector = wants<Q>(args.out_d, kQ_d) || wants<Q>(args.out_D, kQ_D);
    const bool need_shift = wants<Q>(args.out_S, kQ_S) || need_vector;
    EmitShared<T>& sh = shared[warp];
    const int64_t n_groups = (args.n_sources + 31) / 32;
    const int64_t stride = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    for (int64_t group = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
         group < n_groups; group += stride) {
        const int64_t k = group * 32 + lane;
        const bool valid = k < args.n_sources;
        int32_t words = 0;
        const uint32_t* mask = nullptr;
        int64_t mask_stride = 0;
        __syncwarp();  // the previous group's shared data is no longer read
        if (valid) {
            const int32_t source = args.source_list[k];
            const int32_t bin = args.source_bin[k];
            const uint32_t first = static_cast<uint32_t>(args.bin_start[bin] >> 32);
            const uint32_t n_bin_sources = static_cast<uint32_t>(args.bin_start[bin + 1] >> 32) - first;
            const StructurePlan<T>& plan = args.plans[args.bin_struct[bin]];
            int32_t bx, by, bz;
            bin_coordinates(plan, bin, bx, by, bz);
            const int32_t total = build_stencil<true>(plan, args.bin_start, args.n_sources, bx, by,
                                                      bz, sh.rows[lane]);
            words = (total + 31) >> 5;
            mask = args.mask_words + args.bin_word_start[bin] + (k - first);
            mask_stride = n_bin_sources;
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                sh.pos[c][lane] = args.positions[3 * source + c];
                sh.wrap[c][lane] = args.wraps[3 * source + c];
            }
            sh.atom[lane] = source;
            if (need_vector) {
#pragma unroll
                for (int c = 0; c < 9; ++c) sh.cell[c][lane] = plan.cell[c];
            }
        }
        // Usually all 32 sources belong to one structure: its cell then
        // lives in registers instead of being read per pair.
        const int32_t my_struct = valid ? args.bin_struct[args.source_bin[k]] : -1;
        const int32_t first_struct = __shfl_sync(kFullMask, my_struct, 0);
        const bool uniform_cell = __all_sync(kFullMask, !valid || my_struct == first_struct);
        T group_cell[9];
        if (need_vector && uniform_cell) {
#pragma unroll
            for (int c = 0; c < 9; ++c) group_cell[c] = args.plans[first_struct].cell[c];
        }
        const int32_t batches = static_cast<int32_t>(__reduce_max_sync(kFullMask, static_cast<unsigned>(words)));
        __syncwarp();
        int64_t out_row = args.pair_start[group * 32];

        // Word batches: lane l holds word `batch` of source l; the next batch
        // is loaded one batch ahead.  `avail`: nonzero words not yet taken.
        int32_t batch = 0;
        uint32_t stage = words > 0 ? mask[0] : 0u;
        uint32_t stage_next = words > 1 ? mask[mask_stride] : 0u;
        unsigned avail = __ballot_sync(kFullMask, stage != 0u);
        uint32_t bits = 0;  // this lane's current word (untaken candidates)
        int32_t my_r = 0, my_w = 0;
        // Stencil range of the lane's last candidate: candidates below
        // range_end map to slot k + range_delta (bits are taken in order).
        int32_t range_end = 0, range_delta = 0;
        auto refill = [&]() {
            while (true) {
                const unsigned need = __ballot_sync(kFullMask, bits == 0u);
                if (need == 0u) return;
                if (avail == 0u) {
                    if (batch + 1 >= batches) return;
                    ++batch;
                    stage = stage_next;
                    stage_next = batch + 1 < words ? mask[(batch + 1) * mask_stride] : 0u;
                    avail = __ballot_sync(kFullMask, stage != 0u);
                    continue;
                }
                // Hand the batch's untaken nonzero words to the lanes in
                // need, in rank order, through a shared mailbox.
                const int32_t n_avail = __popc(avail);
                const bool offering = (avail >> lane) & 1u;
                const int32_t offer_rank = __popc(avail & below);
                if (offering) sh.mailbox[offer_rank] = make_int2(static_cast<int32_t>(stage), lane);
                __syncwarp();
                const int32_t rank = __popc(need & below);
                if (bits == 0u && rank < n_avail) {
                    const int2 handed = sh.mailbox[rank];
                    bits = static_cast<uint32_t>(handed.x);
                    my_r = handed.y;
                    my_w = batch;
                    range_end = 0;
                }
                avail = __ballot_sync(kFullMask, offering && offer_rank >= __popc(need));
                __syncwarp();
            }
        };
        // Selection rounds fill a queue of (slot, source) entries and need no
        // global loads but the staged mask words.  The queue is double
        // buffered: the ghost records of chunk c (up to PerLane per
        // lane) are requested, the next chunk is selected while they are in
        // flight, and only then is chunk c computed and stored.
        auto fill = [&](int2* queue) -> int32_t {
            int32_t queued = 0;
            while (queued <= 32 * PerLane - 32) {
                refill();
                const bool has = bits != 0u;
                const unsigned ballot = __ballot_sync(kFullMask, has);
                if (ballot == 0u) break;
                if (has) {
                    const int32_t bit = __ffs(bits) - 1;
                    bits &= bits - 1u;
                    queue[queued + __popc(ballot & below)] =
                        make_int2(cached_slot(sh.rows[my_r], 32 * my_w + bit, range_end, range_delta), my_r);
                }
                queued += __popc(ballot);
            }
            __syncwarp();
            return queued;
        };
        int32_t current = 0;
        int32_t queued = fill(sh.queue[0]);
        while (queued > 0) {
            const int2* queue = sh.queue[current];
            int4 meta[PerLane];
            V pt[PerLane];
            int32_t source_r[PerLane];
#pragma unroll
            for (int m = 0; m < PerLane; ++m) {
                const int32_t e = lane + 32 * m;
                source_r[m] = 0;
                if (e < queued) {
                    const int2 entry = queue[e];
                    source_r[m] = entry.y;
                    meta[m] = args.ghost_meta[entry.x];
                    if (need_vector) pt[m] = reinterpret_cast<const V*>(args.ghost_orig)[entry.x];
                }
            }
            const int32_t next_queued = fill(sh.queue[current ^ 1]);
#pragma unroll
            for (int m = 0; m < PerLane; ++m) {
                const int32_t e = lane + 32 * m;
                if (e < queued) {
                    const int32_t r = source_r[m];
                    int64_t a = sh.atom[r];
                    int64_t b = meta[m].w;
                    int32_t shift[3] = {0, 0, 0};
                    if (need_shift) {
                        // Cell-list shifts fit int32 by construction of the plan.
                        shift[0] = meta[m].x + sh.wrap[0][r];
                        shift[1] = meta[m].y + sh.wrap[1][r];
                        shift[2] = meta[m].z + sh.wrap[2][r];
                    }
                    T pa[3] = {T(0), T(0), T(0)}, pb[3] = {T(0), T(0), T(0)};
                    T cell[9];
                    if (need_vector) {
                        pa[0] = sh.pos[0][r];
                        pa[1] = sh.pos[1][r];
                        pa[2] = sh.pos[2][r];
                        pb[0] = pt[m].x;
                        pb[1] = pt[m].y;
                        pb[2] = pt[m].z;
#pragma unroll
                        for (int c = 0; c < 9; ++c) cell[c] = uniform_cell ? group_cell[c] : sh.cell[c][r];
                    }
                    // Half lists: canonical orientation, the lower atom first
                    // (a == b is a periodic self image tested with its
                    // canonical shift).
                    if (Half && b < a) {
                        const int64_t x = a;
                        a = b;
                        b = x;
#pragma unroll
                        for (int c = 0; c < 3; ++c) {
                            shift[c] = -shift[c];
                            const T y = pa[c];
                            pa[c] = pb[c];
                            pb[c] = y;
                        }
                    }
                    T vec[3] = {T(0), T(0), T(0)};
                    if (need_vector) row_vector(pb, pa, shift, cell, vec);
                    if constexpr (Half) {
                        store_row<T, Q>(args, out_row + e, a + args.index_offset,
                                        b + args.index_offset, shift, vec);
                    } else {
                        const int32_t back_shift[3] = {-shift[0], -shift[1], -shift[2]};
                        T back[3] = {T(0), T(0), T(0)};
                        if (need_vector) row_vector(pa, pb, back_shift, cell, back);
                        if (args.paired_rows) {
                            store_row_pair<T, Q>(args, out_row + 2 * e, a + args.index_offset,
                                                 b + args.index_offset, shift, vec, back);
                        } else {
                            store_row<T, Q>(args, out_row + e, a + args.index_offset,
                                            b + args.index_offset, shift, vec);
                            store_row<T, Q>(args, out_row + queued + e, b + args.index_offset,
                                            a + args.index_offset, back_shift, back);
                        }
                    }
                }
            }
            out_row += Half ? queued : 2 * queued;
            queued = next_queued;
            current ^= 1;
        }
        if (args.include_self) {
            // Zero-shift self pairs, after the group's other rows (so those
            // start at the group's first row, which is even for full lists):
            // (p - p) + 0 . cell is +0 in every component.
            if (valid) {
                const int64_t a = static_cast<int64_t>(sh.atom[lane]) + args.index_offset;
                const int32_t zero_shift[3] = {0, 0, 0};
                const T zero_vec[3] = {T(0), T(0), T(0)};
                store_row<T, Q>(args, out_row + lane, a, a, zero_shift, zero_vec);
            }
        }
        __syncwarp();
    }
}


// Brute force: one warp per source atom of a brute-force structure (grid-
// stride over those atoms); lanes stride over the N x I (target, image)
// candidates, target fastest so that consecutive lanes read consecutive
// atoms, with (target, image) cursors advanced incrementally.  Every
// candidate takes the exact predicate (tonari csrc/core/neighbors_cpu.cpp:
// 222-273).  The write pass queues accepted candidates in shared memory and
// emits them 32 at a time into consecutive output rows.
template <typename T>
struct BruteCandidate {
    bool accept;
    long long shift[3];
    T vec[3];
};

template <typename T>
__device__ __forceinline__ BruteCandidate<T> brute_evaluate(const SearchArgs<T>& args,
                                                            const StructurePlan<T>& plan,
                                                            int64_t source, int64_t target,
                                                            int32_t image_index, const T (&ps)[3],
                                                            const long long (&ws)[3]) {
    BruteCandidate<T> out;
    const int4 image = args.image_shift[plan.image_begin + image_index];
    out.shift[0] = static_cast<long long>(image.x) - args.wraps[3 * target] + ws[0];
    out.shift[1] = static_cast<long long>(image.y) - args.wraps[3 * target + 1] + ws[1];
    out.shift[2] = static_cast<long long>(image.z) - args.wraps[3 * target + 2] + ws[2];
    out.vec[0] = out.vec[1] = out.vec[2] = T(0);
    out.accept = false;
    if (!keep_identity(source, target, out.shift, args.half_list != 0, args.include_self != 0)) {
        return out;
    }
    const bool zero_self =
        source == target && out.shift[0] == 0 && out.shift[1] == 0 && out.shift[2] == 0;
    if (zero_self) {
        out.accept = true;
        return out;
    }
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        out.vec[c] = exact_component(args.positions[3 * target + c], ps[c], out.shift, plan.cell, c);
    }
    out.accept = exact_norm2(out.vec[0], out.vec[1], out.vec[2]) < plan.cutoff_squared;
    return out;
}

template <typename T, bool Write>
__global__ void __launch_bounds__(kSearchThreads) brute_search_kernel(SearchArgs<T> args) {
    __shared__ int2 queue[kSearchWarps][64];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const unsigned below = (1u << lane) - 1u;
    const int64_t stride = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    for (int64_t work = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
         work < args.n_brute_atoms; work += stride) {
        const int32_t c = segment_of(args.brute_prefix, args.n_brute, work);
        const StructurePlan<T>& plan = args.plans[args.brute_structs[c]];
        const int64_t source = plan.atom_begin + (work - args.brute_prefix[c]);
        const int64_t order = args.source_order ? args.n_sources + work : source;
            if constexpr (Write) {
                if (args.counts[order] == 0) continue;
        }
        const T ps[3] = {args.positions[3 * source], args.positions[3 * source + 1],
                         args.positions[3 * source + 2]};
        const long long ws[3] = {args.wraps[3 * source], args.wraps[3 * source + 1],
                                 args.wraps[3 * source + 2]};
        const int32_t n = plan.n_atoms;
        const int32_t images = plan.n_images;
        const int32_t step_images = 32 / n;
        const int32_t step_atoms = 32 % n;
        int32_t t = lane % n;
        int32_t image = lane / n;
        uint32_t count = 0;
        int64_t out_row = 0;
        int32_t queued = 0;
        if constexpr (Write) out_row = args.pair_start[order];
        // Warp-uniform trip count: ceil(n * images / 32) iterations.
        const int64_t trips = (static_cast<int64_t>(n) * images + 31) / 32;
        for (int64_t trip = 0; trip < trips; ++trip) {
            bool accept = false;
            if (image < images) {
                const BruteCandidate<T> cand =
                    brute_evaluate(args, plan, source, plan.atom_begin + t, image, ps, ws);
                accept = cand.accept;
                if (!Write && accept) {
                    if (cand.shift[0] < INT_MIN || cand.shift[0] > INT_MAX ||
                        cand.shift[1] < INT_MIN || cand.shift[1] > INT_MAX ||
                        cand.shift[2] < INT_MIN || cand.shift[2] > INT_MAX) {
                        atomicOr(args.status, static_cast<uint32_t>(kStatusShiftRange));
                    }
                }
            }
            const unsigned ballot = __ballot_sync(kFullMask, accept);
            if constexpr (Write) {
                if (ballot) {
                    int2* q = queue[warp];
                    if (accept) q[queued + __popc(ballot & below)] = make_int2(t, image);
                    queued += __popc(ballot);
                    if (queued >= 32) {
                        __syncwarp();
                        const int2 item = q[lane];
                        const BruteCandidate<T> cand = brute_evaluate(
                            args, plan, source, plan.atom_begin + item.x, item.y, ps, ws);
                        emit_pair(args, out_row + lane, source, plan.atom_begin + item.x,
                                  cand.shift, cand.vec);
                        __syncwarp();
                        if (lane < queued - 32) q[lane] = q[32 + lane];
                        __syncwarp();
                        queued -= 32;
                        out_row += 32;
                    }
                }
            } else {
                count += __popc(ballot);
            }
            t += step_atoms;
            image += step_images;
            if (t >= n) {
                t -= n;
                ++image;
            }
        }
        if constexpr (Write) {
            __syncwarp();
            if (lane < queued) {
                const int2 item = queue[warp][lane];
                const BruteCandidate<T> cand = brute_evaluate(
                    args, plan, source, plan.atom_begin + item.x, item.y, ps, ws);
                emit_pair(args, out_row + lane, source, plan.atom_begin + item.x, cand.shift,
                          cand.vec);
            }
            __syncwarp();
        } else {
            if (lane == 0) {
                args.counts[order] = count;
                if (count > static_cast<uint32_t>(INT_MAX)) {
                    atomicOr(args.status, static_cast<uint32_t>(kStatusCountRange));
                }
            }
        }
    }
}

// Brute force, tiled: one CTA per brute-force structure (grid-stride over
// them).  The structure's positions, wraps and image shifts are staged once
// in shared memory; each warp then takes sources in turn and its lanes
// stride over the N x I (target, image) candidates, target fastest, reading
// only shared memory.  Every candidate takes the exact predicate (tonari
// csrc/core/neighbors_cpu.cpp:222-273).  The write pass queues accepted
// candidates per warp and emits them 32 at a time into consecutive rows.
constexpr int kBruteTileThreads = 128;
constexpr int kBruteTileWarps = kBruteTileThreads / 32;
constexpr int kBruteTileMaxBytes = 48 * 1024;

template <typename T>
struct BruteTile {
    const T* px;
    const T* py;
    const T* pz;
    const int32_t* wx;
    const int32_t* wy;
    const int32_t* wz;
    const int32_t* ix;
    const int32_t* iy;
    const int32_t* iz;
};

// `plain`: a structure without periodic axes has one image and zero wraps,
// so every shift is zero and the public displacement is p_t - p_s (adding
// the zero translation changes at most the sign of a zero component).
template <typename T>
__device__ __forceinline__ bool brute_tile_evaluate(const BruteTile<T>& tile, const T (&cell)[9],
                                                    T cutoff_squared, int64_t atom_begin,
                                                    int32_t s, int32_t t, int32_t image,
                                                    bool half, bool include_self, bool plain,
                                                    long long (&shift)[3], T (&vec)[3]) {
    if (plain) {
        shift[0] = shift[1] = shift[2] = 0;
        vec[0] = vec[1] = vec[2] = T(0);
        if (s == t) return include_self;
        if (half && s > t) return false;
        vec[0] = sub_rn(tile.px[t], tile.px[s]);
        vec[1] = sub_rn(tile.py[t], tile.py[s]);
        vec[2] = sub_rn(tile.pz[t], tile.pz[s]);
        return exact_norm2(vec[0], vec[1], vec[2]) < cutoff_squared;
    }
    shift[0] = static_cast<long long>(tile.ix[image]) - tile.wx[t] + tile.wx[s];
    shift[1] = static_cast<long long>(tile.iy[image]) - tile.wy[t] + tile.wy[s];
    shift[2] = static_cast<long long>(tile.iz[image]) - tile.wz[t] + tile.wz[s];
    vec[0] = vec[1] = vec[2] = T(0);
    if (!keep_identity(atom_begin + s, atom_begin + t, shift, half, include_self)) return false;
    if (s == t && shift[0] == 0 && shift[1] == 0 && shift[2] == 0) return true;
    vec[0] = exact_component(tile.px[t], tile.px[s], shift, cell, 0);
    vec[1] = exact_component(tile.py[t], tile.py[s], shift, cell, 1);
    vec[2] = exact_component(tile.pz[t], tile.pz[s], shift, cell, 2);
    return exact_norm2(vec[0], vec[1], vec[2]) < cutoff_squared;
}

template <typename T, bool Write>
__global__ void __launch_bounds__(kBruteTileThreads) brute_tile_kernel(SearchArgs<T> args) {
    extern __shared__ __align__(16) unsigned char tile_bytes[];
    __shared__ int2 queue[kBruteTileWarps][64];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const unsigned below = (1u << lane) - 1u;
    for (int32_t c = blockIdx.x; c < args.n_brute; c += gridDim.x) {
        const StructurePlan<T>& plan = args.plans[args.brute_structs[c]];
        const int32_t n = plan.n_atoms;
        const int32_t images = plan.n_images;
        const int64_t atom_begin = plan.atom_begin;
        const int64_t work_begin = args.brute_prefix[c];
        // Layout: px, py, pz (T[n]); wx, wy, wz (int32[n]); ix, iy, iz (int32[images]).
        BruteTile<T> tile;
        T* p = reinterpret_cast<T*>(tile_bytes);
        int32_t* w = reinterpret_cast<int32_t*>(p + 3 * n);
        int32_t* im = w + 3 * n;
        tile.px = p;
        tile.py = p + n;
        tile.pz = p + 2 * n;
        tile.wx = w;
        tile.wy = w + n;
        tile.wz = w + 2 * n;
        tile.ix = im;
        tile.iy = im + images;
        tile.iz = im + 2 * images;
        __syncthreads();  // the previous structure's tile is no longer read
        for (int32_t k = threadIdx.x; k < n; k += blockDim.x) {
            const int64_t atom = atom_begin + k;
            p[k] = args.positions[3 * atom];
            p[n + k] = args.positions[3 * atom + 1];
            p[2 * n + k] = args.positions[3 * atom + 2];
            w[k] = args.wraps[3 * atom];
            w[n + k] = args.wraps[3 * atom + 1];
            w[2 * n + k] = args.wraps[3 * atom + 2];
        }
        for (int32_t k = threadIdx.x; k < images; k += blockDim.x) {
            const int4 shift = args.image_shift[plan.image_begin + k];
            im[k] = shift.x;
            im[images + k] = shift.y;
            im[2 * images + k] = shift.z;
        }
        T cell[9];
#pragma unroll
        for (int k = 0; k < 9; ++k) cell[k] = plan.cell[k];
        const T cutoff_squared = plan.cutoff_squared;
        __syncthreads();
        const bool half = args.half_list != 0;
        const bool include_self = args.include_self != 0;
        const bool plain = images == 1;
        const int32_t step_images = 32 / n;
        const int32_t step_atoms = 32 % n;
        const int64_t trips = (static_cast<int64_t>(n) * images + 31) / 32;
        for (int32_t s = warp; s < n; s += kBruteTileWarps) {
            const int64_t source = atom_begin + s;
            const int64_t order = args.source_order ? args.n_sources + work_begin + s : source;
            int64_t out_row = 0;
            if constexpr (Write) {
                if (args.counts[order] == 0) continue;
                out_row = args.pair_start[order];
            }
            int32_t t = lane % n;
            int32_t image = lane / n;
            uint32_t count = 0;
            int32_t queued = 0;
            for (int64_t trip = 0; trip < trips; ++trip) {
                bool accept = false;
                long long shift[3];
                T vec[3];
                if (image < images) {
                    accept = brute_tile_evaluate(tile, cell, cutoff_squared, atom_begin, s, t, image,
                                                 half, include_self, plain, shift, vec);
                    if (!Write && accept) {
                        if (shift[0] < INT_MIN || shift[0] > INT_MAX || shift[1] < INT_MIN ||
                            shift[1] > INT_MAX || shift[2] < INT_MIN || shift[2] > INT_MAX) {
                            atomicOr(args.status, static_cast<uint32_t>(kStatusShiftRange));
                        }
                    }
                }
                const unsigned ballot = __ballot_sync(kFullMask, accept);
                if constexpr (Write) {
                    if (ballot) {
                        int2* q = queue[warp];
                        if (accept) q[queued + __popc(ballot & below)] = make_int2(t, image);
                        queued += __popc(ballot);
                        if (queued >= 32) {
                            __syncwarp();
                            const int2 item = q[lane];
                            brute_tile_evaluate(tile, cell, cutoff_squared, atom_begin, s, item.x,
                                                item.y, half, include_self, plain, shift, vec);
                            emit_pair(args, out_row + lane, source, atom_begin + item.x, shift, vec);
                            __syncwarp();
                            if (lane < queued - 32) q[lane] = q[32 + lane];
                            __syncwarp();
                            queued -= 32;
                            out_row += 32;
                        }
                    }
                } else {
                    count += __popc(ballot);
                }
                t += step_atoms;
                image += step_images;
                if (t >= n) {
                    t -= n;
                    ++image;
                }
            }
            if constexpr (Write) {
                __syncwarp();
                if (lane < queued) {
                    const int2 item = queue[warp][lane];
                    long long shift[3];
                    T vec[3];
                    brute_tile_evaluate(tile, cell, cutoff_squared, atom_begin, s, item.x, item.y,
                                        half, include_self, plain, shift, vec);
                    emit_pair(args, out_row + lane, source, atom_begin + item.x, shift, vec);
                }
                __syncwarp();
            } else if (lane == 0) {
                args.counts[order] = count;
                if (count > static_cast<uint32_t>(INT_MAX)) {
                    atomicOr(args.status, static_cast<uint32_t>(kStatusCountRange));
                }
            }
        }
    }
}

// Candidate filter for Verlet-skin reuse: thread per candidate pair; the
// decisive test is the one of the search kernels (exact_component in the
// reference's order, exact_norm2 < (T)(cutoff^2)).  Pass 1 stores one ballot
// word per warp and one count per block; pass 2 writes the kept pairs at
// block offset + rank, so they keep their candidate order.
template <typename T>
__device__ __forceinline__ bool filter_candidate(const FilterArgs<T>& a, int64_t k, int64_t& source,
                                                 int64_t& target, long long (&shift)[3], T (&vec)[3]) {
    source = a.pairs[2 * k] - a.index_offset;
    target = a.pairs[2 * k + 1] - a.index_offset;
    shift[0] = a.shifts[3 * k];
    shift[1] = a.shifts[3 * k + 1];
    shift[2] = a.shifts[3 * k + 2];
    const int32_t b = structure_of(a.batch_ptr, a.batch, source);
    T cell[9];
#pragma unroll
    for (int c = 0; c < 9; ++c) cell[c] = a.cell[9 * static_cast<int64_t>(b) + c];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        vec[c] = exact_component(a.positions[3 * target + c], a.positions[3 * source + c], shift, cell, c);
    }
    return exact_norm2(vec[0], vec[1], vec[2]) < a.cutoff_squared;
}

template <typename T, bool Write>
__global__ void __launch_bounds__(kFilterThreads) filter_kernel(FilterArgs<T> a) {
    __shared__ uint32_t warp_counts[kFilterThreads / 32];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t k = static_cast<int64_t>(blockIdx.x) * kFilterThreads + threadIdx.x;
    if constexpr (!Write) {
        int64_t source = 0, target = 0;
        long long shift[3];
        T vec[3];
        const bool keep = k < a.n_candidates && filter_candidate(a, k, source, target, shift, vec);
        const uint32_t word = __ballot_sync(kFullMask, keep);
        if (lane == 0) {
            if ((k >> 5) < (a.n_candidates + 31) / 32) a.keep_words[k >> 5] = word;
            warp_counts[warp] = __popc(word);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            uint32_t total = 0;
            for (int w = 0; w < kFilterThreads / 32; ++w) total += warp_counts[w];
            a.block_counts[blockIdx.x] = total;
        }
    } else {
        const int64_t word_index = k >> 5;  // the same for the whole warp
        const uint32_t word = word_index < (a.n_candidates + 31) / 32 ? a.keep_words[word_index] : 0u;
        if (lane == 0) warp_counts[warp] = __popc(word);
        __syncthreads();
        int64_t row = a.block_start[blockIdx.x];
        for (int w = 0; w < warp; ++w) row += warp_counts[w];
        row += __popc(word & ((1u << lane) - 1u));
        if (k < a.n_candidates && ((word >> lane) & 1u)) {
            int64_t source, target;
            long long shift[3];
            T vec[3];
            filter_candidate(a, k, source, target, shift, vec);
            const int64_t s = source + a.index_offset, t = target + a.index_offset;
            if (a.out_i) a.out_i[row] = s;
            if (a.out_j) a.out_j[row] = t;
            if (a.out_P) reinterpret_cast<longlong2*>(a.out_P)[row] = make_longlong2(s, t);
            if (a.out_S) {
                a.out_S[3 * row] = static_cast<int32_t>(shift[0]);
                a.out_S[3 * row + 1] = static_cast<int32_t>(shift[1]);
                a.out_S[3 * row + 2] = static_cast<int32_t>(shift[2]);
            }
            if (a.out_D) {
                a.out_D[3 * row] = vec[0];
                a.out_D[3 * row + 1] = vec[1];
                a.out_D[3 * row + 2] = vec[2];
            }
            if (a.out_d) a.out_d[row] = pair_distance(vec[0], vec[1], vec[2]);
        }
    }
}

// Image tables of one structure per block: integer shifts enumerated x-major,
// then y, then z (tonari csrc/core/geometry.cpp:229-237), and their Cartesian
// translations in T.  Only the binning passes read the translations, both
// from this table, so they agree bit for bit.
template <typename T>
__global__ void image_table_kernel(const StructurePlan<T>* __restrict__ plans,
                                   int4* __restrict__ shifts, void* translations_out) {
    using V = vec4_t<T>;
    const StructurePlan<T>& plan = plans[blockIdx.x];
    V* translations = reinterpret_cast<V*>(translations_out);
    for (int32_t k = threadIdx.x; k < plan.n_images; k += blockDim.x) {
        int32_t image[3];
        decode_image(k, plan.repeats, image);
        shifts[plan.image_begin + k] = make_int4(image[0], image[1], image[2], 0);
        V t;
        T c[3];
#pragma unroll
        for (int axis = 0; axis < 3; ++axis) {
            T value = T(0);
#pragma unroll
            for (int a = 0; a < 3; ++a) {
                value = add_rn(value, mul_rn(static_cast<T>(image[a]), plan.cell[3 * a + axis]));
            }
            c[axis] = value;
        }
        t.x = c[0];
        t.y = c[1];
        t.z = c[2];
        t.w = T(0);
        translations[plan.image_begin + k] = t;
    }
}

// One block per cell-list structure writes that structure's index into its
// bins' slots of bin_struct.
__global__ void bin_struct_kernel(const int64_t* __restrict__ cell_bin_prefix,
                                  const int32_t* __restrict__ cell_structs,
                                  int32_t* __restrict__ bin_struct) {
    const int32_t c = blockIdx.x;
    const int64_t begin = cell_bin_prefix[c];
    const int64_t end = cell_bin_prefix[c + 1];
    const int32_t value = cell_structs[c];
    for (int64_t bin = begin + threadIdx.x; bin < end; bin += blockDim.x) bin_struct[bin] = value;
}

int64_t blocks_for(int64_t items, int64_t per_block) { return (items + per_block - 1) / per_block; }

// Grid for a grid-stride kernel: enough blocks to fill every SM at the
// kernel's occupancy, never more than the work needs.
template <typename Kernel>
unsigned persistent_blocks_smem(Kernel kernel, int threads, size_t dynamic_bytes, int64_t needed) {
    int device = 0, sms = 148, per_sm = 1;
    cudaGetDevice(&device);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, dynamic_bytes);
    const int64_t full = static_cast<int64_t>(sms) * std::max(per_sm, 1);
    return static_cast<unsigned>(std::max<int64_t>(1, std::min(needed, full)));
}

template <typename Kernel>
unsigned persistent_blocks(Kernel kernel, int threads, int64_t needed) {
    int device = 0, sms = 148, per_sm = 1;
    cudaGetDevice(&device);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0);
    const int64_t full = static_cast<int64_t>(sms) * std::max(per_sm, 1);
    return static_cast<unsigned>(std::max<int64_t>(1, std::min(needed, full)));
}

}  // namespace
}  // namespace tnr

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
namespace tnr {

namespace {
thread_local int64_t g_kernel_launches = 0;
}  // namespace

int64_t launched_kernels() { return g_kernel_launches; }

template <typename T>
void launch_filter(const FilterArgs<T>& args, bool write, cudaStream_t stream) {
    if (args.n_candidates == 0) return;
    const unsigned blocks = static_cast<unsigned>(blocks_for(args.n_candidates, kFilterThreads));
    if (write) {
        filter_kernel<T, true><<<blocks, kFilterThreads, 0, stream>>>(args);
    } else {
        filter_kernel<T, false><<<blocks, kFilterThreads, 0, stream>>>(args);
    }
    ++g_kernel_launches;
}

template <typename T>
void launch_geometry(const T* cell, const uint8_t* pbc, const int64_t* batch_ptr, int64_t batch,
                     double cutoff, PrepareStructure<T>* prepare, DeviceGeometry* geometry,
                     uint32_t* flags, Reduction<T>* reductions, cudaStream_t stream) {
    if (batch == 0) return;
    geometry_kernel<T><<<static_cast<unsigned>(blocks_for(batch, 128)), 128, 0, stream>>>(
        cell, pbc, batch_ptr, batch, cutoff, prepare, geometry, flags, reductions);
    ++g_kernel_launches;
}

template <typename T>
void launch_verify_wraps(const T* positions, int64_t n_atoms, const int32_t* atom_struct,
                         const T* duals, const int32_t* wraps, uint32_t* flag, cudaStream_t stream) {
    if (n_atoms == 0) return;
    verify_wraps_kernel<T><<<static_cast<unsigned>(blocks_for(n_atoms, kPrepareThreads)),
                             kPrepareThreads, 0, stream>>>(positions, n_atoms, atom_struct, duals,
                                                           wraps, flag);
    ++g_kernel_launches;
}

template <typename T>
void launch_prepare(const PrepareArgs<T>& args, cudaStream_t stream) {
    if (args.n_atoms == 0) return;
    prepare_kernel<T><<<static_cast<unsigned>(blocks_for(args.n_atoms, kPrepareThreads)),
                        kPrepareThreads, 0, stream>>>(args);
    ++g_kernel_launches;
}

template <typename T>
void launch_bin(const BinArgs<T>& args, bool scatter, cudaStream_t stream) {
    if (args.n_cell_atoms == 0) return;
    dim3 grid(static_cast<unsigned>(blocks_for(args.n_cell_atoms, kBinThreads)), 1, 1);
    // Threads per atom: enough to reach about two full waves of the GPU when
    // the atoms alone do not (small batches of structures with many images).
    // Image copies depend on the atom only in pair-once calls (and on the
    // atom index otherwise), so any split gives the same copies.
    {
        int device = 0, sms = 148;
        cudaGetDevice(&device);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
        const int64_t target = int64_t{sms} * 2048 * 2;
        const int64_t split = std::min<int64_t>(args.max_images, target / std::max<int64_t>(args.n_cell_atoms, 1));
        grid.y = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(split, 64)));
    }
    if (scatter) {
        bin_kernel<T, true><<<grid, kBinThreads, 0, stream>>>(args);
    } else {
        bin_kernel<T, false><<<grid, kBinThreads, 0, stream>>>(args);
    }
    ++g_kernel_launches;
}

template <typename T>
void launch_image_table(const StructurePlan<T>* plans, int64_t batch, int4* shifts,
                        void* translations, cudaStream_t stream) {
    if (batch == 0) return;
    image_table_kernel<T><<<static_cast<unsigned>(batch), 128, 0, stream>>>(plans, shifts,
                                                                          translations);
    ++g_kernel_launches;
}

template <typename T>
void launch_bin_struct(const int64_t* cell_bin_prefix, const int32_t* cell_structs,
                       int32_t n_cell, int32_t* bin_struct, cudaStream_t stream) {
    if (n_cell == 0) return;
    bin_struct_kernel<<<static_cast<unsigned>(n_cell), 256, 0, stream>>>(cell_bin_prefix,
                                                                        cell_structs, bin_struct);
    ++g_kernel_launches;
}

__global__ void capacity_check_kernel(const unsigned long long* total, unsigned long long capacity,
                                      uint32_t* status) {
    if (*total > capacity) atomicOr(status, static_cast<uint32_t>(kStatusCapacity));
}

void launch_capacity_check(const unsigned long long* total, unsigned long long capacity,
                           uint32_t* status, cudaStream_t stream) {
    capacity_check_kernel<<<1, 1, 0, stream>>>(total, capacity, status);
    ++g_kernel_launches;
}

template <typename T>
void launch_stencil_words(const SearchArgs<T>& args, unsigned long long* bin_words,
                          cudaStream_t stream) {
    if (args.n_bins == 0) return;
    const unsigned blocks = static_cast<unsigned>(blocks_for(args.n_bins, kBinThreads));
    if (args.pair_once) {
        stencil_words_kernel<true, T><<<blocks, kBinThreads, 0, stream>>>(args, args.n_bins, bin_words);
    } else {
        stencil_words_kernel<false, T><<<blocks, kBinThreads, 0, stream>>>(args, args.n_bins, bin_words);
    }
    ++g_kernel_launches;
}

template <typename T>
void launch_cell_search(const SearchArgs<T>& args, bool write, cudaStream_t stream) {
    if (args.n_sources == 0 || args.n_bins == 0) return;
    const int64_t needed = blocks_for(args.n_bins, kSearchWarps);
    if (write) {
        const int q = (args.out_i ? kQ_I : 0) | (args.out_j ? kQ_J : 0) | (args.out_P ? kQ_P : 0) |
                      (args.out_S ? kQ_S : 0) | (args.out_d ? kQ_d : 0) | (args.out_D ? kQ_D : 0);
        const int64_t groups = blocks_for((args.n_sources + 31) / 32, kEmitThreads / 32);
        auto launch = [&](auto kernel, int64_t work, int threads = kSearchThreads) {
            kernel<<<persistent_blocks(kernel, threads, work), threads, 0, stream>>>(args);
            ++g_kernel_launches;
        };
        if (args.source_order == 0 || !args.pair_once) {
            switch (q) {
                case kQ_P | kQ_S: launch(cell_write_kernel<T, kQ_P | kQ_S>, needed); break;
                case kQ_I | kQ_J | kQ_S | kQ_d | kQ_D:
                    launch(cell_write_kernel<T, kQ_I | kQ_J | kQ_S | kQ_d | kQ_D>, needed); break;
                case kQ_P | kQ_S | kQ_D: launch(cell_write_kernel<T, kQ_P | kQ_S | kQ_D>, needed); break;
                case kQ_P | kQ_D: launch(cell_write_kernel<T, kQ_P | kQ_D>, needed); break;
                default: launch(cell_write_kernel<T, 0>, needed); break;
            }
        } else {
            auto emit = [&](auto half) {
                constexpr bool H = decltype(half)::value;
                switch (q) {
                    case kQ_P | kQ_S: launch(cell_emit_kernel<T, kQ_P | kQ_S, H>, groups, kEmitThreads); break;
                    case kQ_I | kQ_J | kQ_S | kQ_d | kQ_D:
                        launch(cell_emit_kernel<T, kQ_I | kQ_J | kQ_S | kQ_d | kQ_D, H>, groups, kEmitThreads); break;
                    case kQ_P | kQ_S | kQ_D: launch(cell_emit_kernel<T, kQ_P | kQ_S | kQ_D, H>, groups, kEmitThreads); break;
                    case kQ_P | kQ_D: launch(cell_emit_kernel<T, kQ_P | kQ_D, H>, groups, kEmitThreads); break;
                    default: launch(cell_emit_kernel<T, 0, H>, groups, kEmitThreads); break;
                }
            };
            if (args.half_list) emit(std::true_type{}); else emit(std::false_type{});
        }
    } else {
        auto count = [&](auto kernel) {
            kernel<<<persistent_blocks(kernel, kSearchThreads, needed), kSearchThreads, 0, stream>>>(args);
            ++g_kernel_launches;
        };
        if (args.pair_once) {
            if (args.half_list) count(cell_count_kernel<T, true, true>);
            else count(cell_count_kernel<T, false, true>);
        } else {
            if (args.half_list) count(cell_count_kernel<T, true, false>);
            else count(cell_count_kernel<T, false, false>);
        }
    }
}

template <typename T>
void launch_brute_search(const SearchArgs<T>& args, bool write, cudaStream_t stream) {
    if (args.n_brute_atoms == 0) return;
    if (args.brute_tile_bytes > 0 && args.brute_tile_bytes <= kBruteTileMaxBytes) {
        const size_t bytes = static_cast<size_t>(args.brute_tile_bytes);
        if (write) {
            brute_tile_kernel<T, true><<<persistent_blocks_smem(brute_tile_kernel<T, true>,
                                                                kBruteTileThreads, bytes, args.n_brute),
                                         kBruteTileThreads, bytes, stream>>>(args);
        } else {
            brute_tile_kernel<T, false><<<persistent_blocks_smem(brute_tile_kernel<T, false>,
                                                                 kBruteTileThreads, bytes, args.n_brute),
                                          kBruteTileThreads, bytes, stream>>>(args);
        }
        ++g_kernel_launches;
        return;
    }
    const int64_t needed = blocks_for(args.n_brute_atoms, kSearchWarps);
    if (write) {
        brute_search_kernel<T, true><<<persistent_blocks(brute_search_kernel<T, true>,
                                                         kSearchThreads, needed),
                                       kSearchThreads, 0, stream>>>(args);
    ++g_kernel_launches;
    } else {
        brute_search_kernel<T, false><<<persistent_blocks(brute_search_kernel<T, false>,
                                                          kSearchThreads, needed),
                                        kSearchThreads, 0, stream>>>(args);
    ++g_kernel_launches;
    }
}

size_t scan_workspace_bytes(int64_t n) {
    const int64_t tiles = std::max<int64_t>(1, (n + kScanTile - 1) / kScanTile);
    return static_cast<size_t>(tiles) * sizeof(int64_t);
}

namespace {
template <typename In, typename Out>
void launch_scan(const In* in, int64_t n, Out* out, Out* out2, void* workspace, cudaStream_t stream) {
    const int64_t tiles = std::max<int64_t>(1, (n + kScanTile - 1) / kScanTile);
    Out* tile_sums = static_cast<Out*>(workspace);
    scan_reduce_kernel<In, Out><<<static_cast<unsigned>(tiles), kScanThreads, 0, stream>>>(
        in, n, tile_sums);
    scan_tiles_kernel<Out><<<1, kScanTilesThreads, 0, stream>>>(tile_sums, tiles);
    scan_apply_kernel<In, Out><<<static_cast<unsigned>(tiles), kScanThreads, 0, stream>>>(
        in, n, tile_sums, out, out2);
    g_kernel_launches += 3;
}
}  // namespace

void launch_scan_u64(const unsigned long long* in, int64_t n, unsigned long long* out,
                     unsigned long long* out2, void* workspace, uint32_t* status,
                     cudaStream_t stream) {
    (void)status;
    launch_scan<unsigned long long, unsigned long long>(in, n, out, out2, workspace, stream);
}

void launch_scan_counts(const uint32_t* in, int64_t n, int64_t* out, void* workspace,
                        uint32_t* status, cudaStream_t stream) {
    (void)status;
    launch_scan<uint32_t, int64_t>(in, n, out, nullptr, workspace, stream);
}

#define TNR_INSTANTIATE(T)                                                                 \
    template void launch_prepare<T>(const PrepareArgs<T>&, cudaStream_t);                  \
    template void launch_filter<T>(const FilterArgs<T>&, bool, cudaStream_t);              \
    template void launch_verify_wraps<T>(const T*, int64_t, const int32_t*, const T*,         \
                                         const int32_t*, uint32_t*, cudaStream_t);            \
    template void launch_geometry<T>(const T*, const uint8_t*, const int64_t*, int64_t, double, \
                                     PrepareStructure<T>*, DeviceGeometry*, uint32_t*,         \
                                     Reduction<T>*,                                            \
                                     cudaStream_t);                                            \
    template void launch_bin<T>(const BinArgs<T>&, bool, cudaStream_t);                     \
    template void launch_image_table<T>(const StructurePlan<T>*, int64_t, int4*, void*,    \
                                        cudaStream_t);                                       \
    template void launch_bin_struct<T>(const int64_t*, const int32_t*, int32_t, int32_t*,    \
                                       cudaStream_t);                                        \
    template void launch_cell_search<T>(const SearchArgs<T>&, bool, cudaStream_t);          \
    template void launch_stencil_words<T>(const SearchArgs<T>&, unsigned long long*,      \
                                          cudaStream_t);                                     \
    template void launch_brute_search<T>(const SearchArgs<T>&, bool, cudaStream_t);
TNR_INSTANTIATE(float)
TNR_INSTANTIATE(double)
#undef TNR_INSTANTIATE

}  // namespace tnr
