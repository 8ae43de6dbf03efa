// Neighbor-list kernels for B200 (sm_100a).
//
// Pipeline of one call (host side in tnr_api.cpp):
//   prepare   per atom: structure id, representative wrap, wrapped position,
//             per-structure extents reduced through order-preserving atomics
//   bin       per cell-list atom x image: cull the image copy against the
//             structure's box, histogram it into a Cartesian bin (pass 1) or
//             scatter it into cell-sorted order (pass 2)
//   scan      decoupled look-back exclusive scans (tnr_scan.cuh)
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

#include "tnr_kernels.cuh"
#include "tnr_launch.h"
#include "tnr_scan.cuh"

namespace tnr {
namespace {

constexpr int kPrepareThreads = 512;
constexpr int kBinThreads = 256;
constexpr int kSearchThreads = 256;
constexpr int kSearchWarps = kSearchThreads / 32;

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

    const int64_t block_base = static_cast<int64_t>(blockIdx.x) * kPrepareThreads;
    const int64_t atom = block_base + threadIdx.x;
    const bool valid = atom < args.n_atoms;
    if (threadIdx.x == 0) {
        const int64_t last = min(args.n_atoms - 1, block_base + kPrepareThreads - 1);
        block_first_last[0] = structure_of(args.batch_ptr, args.batch, block_base);
        block_first_last[1] = structure_of(args.batch_ptr, args.batch, last);
    }

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
        sid = structure_of(args.batch_ptr, args.batch, atom);
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
#pragma unroll
    for (int offset = 1; offset < 32; offset <<= 1) {
        const int32_t other_sid = __shfl_down_sync(kFullMask, sid, offset);
        const Extents<K> other = shfl_down(ext, offset);
        if (lane + offset < 32 && other_sid == sid) combine(ext, other);
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


// ---------------------------------------------------------------------------
// bin: histogram (pass 1) and scatter (pass 2) of culled image copies
// ---------------------------------------------------------------------------

// One thread per atom of a cell-list structure, looping over the structure's
// images.  An image copy is kept when it lies inside the structure's culling
// box (extent of the wrapped atoms padded by the search radius), the
// reference's rule (tonari csrc/core/neighbors_cpu.cpp:479-495).  The zero
// image is always inside.  Each bin counter packs (sources << 32 | ghosts),
// so one 64-bit atomic hands out both the ghost slot and, for the zero image,
// the source slot.
template <typename T, bool Scatter>
__global__ void __launch_bounds__(kBinThreads) bin_kernel(BinArgs<T> args) {
    using V = vec4_t<T>;
    const int64_t index = static_cast<int64_t>(blockIdx.x) * kBinThreads + threadIdx.x;
    if (index >= args.n_cell_atoms) return;
    const int32_t c = segment_of(args.cell_prefix, args.n_cell, index);
    const StructurePlan<T>& plan = args.plans[args.cell_structs[c]];
    const int64_t atom = plan.atom_begin + (index - args.cell_prefix[c]);
    const V q = reinterpret_cast<const V*>(args.wrapped)[atom];
    const int32_t wrap[3] = {args.wraps[3 * atom], args.wraps[3 * atom + 1],
                             args.wraps[3 * atom + 2]};
    const int32_t center = (plan.n_images - 1) / 2;
    for (int32_t k = 0; k < plan.n_images; ++k) {
        int32_t image[3];
        decode_image(k, plan.repeats, image);
        T g[3];
        bool inside = true;
#pragma unroll
        for (int axis = 0; axis < 3; ++axis) {
            T translation = T(0);
#pragma unroll
            for (int a = 0; a < 3; ++a) {
                translation = add_rn(translation,
                                     mul_rn(static_cast<T>(image[a]), plan.cell[3 * a + axis]));
            }
            const T base = axis == 0 ? q.x : (axis == 1 ? q.y : q.z);
            g[axis] = add_rn(base, translation);
            inside = inside && g[axis] >= plan.lower[axis] && g[axis] <= plan.upper[axis];
        }
        if (!inside && k != center) continue;
        const int32_t bx = bin_axis(g[0], plan.origin[0], plan.inv_edge, plan.dims[0]);
        const int32_t by = bin_axis(g[1], plan.origin[1], plan.inv_edge, plan.dims[1]);
        const int32_t bz = bin_axis(g[2], plan.origin[2], plan.inv_edge, plan.dims[2]);
        const int64_t bin = plan.bin_begin +
            (static_cast<int64_t>(bx) * plan.dims[1] + by) * plan.dims[2] + bz;
        const unsigned long long increment =
            k == center ? (1ull << 32) + 1ull : 1ull;
        const unsigned long long old = atomicAdd(&args.bin_counts[bin], increment);
        if constexpr (Scatter) {
            const uint32_t slot = static_cast<uint32_t>(old & 0xffffffffull);
            V record;
            record.x = g[0];
            record.y = g[1];
            record.z = g[2];
            record.w = index_to_lane(static_cast<int32_t>(atom), T(0));
            reinterpret_cast<V*>(args.ghost_pos)[slot] = record;
            args.ghost_meta[slot] = make_int4(image[0] - wrap[0], image[1] - wrap[1],
                                              image[2] - wrap[2], static_cast<int32_t>(atom));
            if (k == center) {
                args.source_list[static_cast<uint32_t>(old >> 32)] = static_cast<int32_t>(atom);
                args.self_slot[atom] = static_cast<int32_t>(slot);
            }
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

__device__ __forceinline__ bool shift_fits_int32(const long long (&shift)[3]) {
    return shift[0] >= INT_MIN && shift[0] <= INT_MAX && shift[1] >= INT_MIN &&
           shift[1] <= INT_MAX && shift[2] >= INT_MIN && shift[2] <= INT_MAX;
}

// Cell list: one warp per source atom (sources in cell-sorted order, so
// neighbouring warps share stencil bins in L1).  The 27-bin stencil is nine
// z-rows, each a contiguous slot range of the cell-sorted ghost array; the
// warp walks their concatenation 32 candidates at a time so lanes stay busy
// across row boundaries.
template <typename T, bool Write>
__global__ void __launch_bounds__(kSearchThreads) cell_search_kernel(SearchArgs<T> args) {
    using V = vec4_t<T>;
    __shared__ int64_t row_begin[kSearchWarps][9];
    __shared__ int64_t row_prefix[kSearchWarps][10];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t work = static_cast<int64_t>(blockIdx.x) * kSearchWarps + warp;
    if (work >= args.n_sources) return;

    const int32_t source = args.source_list[work];
    const StructurePlan<T>& plan = args.plans[args.atom_struct[source]];
    const V qs = reinterpret_cast<const V*>(args.wrapped)[source];
    const int32_t bx = bin_axis(qs.x, plan.origin[0], plan.inv_edge, plan.dims[0]);
    const int32_t by = bin_axis(qs.y, plan.origin[1], plan.inv_edge, plan.dims[1]);
    const int32_t bz = bin_axis(qs.z, plan.origin[2], plan.inv_edge, plan.dims[2]);

    int64_t begin = 0, length = 0;
    if (lane < 9) {
        const int32_t x = bx + lane / 3 - 1;
        const int32_t y = by + lane % 3 - 1;
        if (x >= 0 && x < plan.dims[0] && y >= 0 && y < plan.dims[1]) {
            const int32_t z0 = max(bz - 1, 0);
            const int32_t z1 = min(bz + 1, plan.dims[2] - 1);
            const int64_t row = plan.bin_begin +
                (static_cast<int64_t>(x) * plan.dims[1] + y) * plan.dims[2];
            begin = static_cast<int64_t>(args.bin_start[row + z0] & 0xffffffffull);
            const int64_t end = static_cast<int64_t>(args.bin_start[row + z1 + 1] & 0xffffffffull);
            length = end - begin;
        }
    }
    const int64_t inclusive = warp_inclusive_sum(length);
    if (lane < 9) {
        row_begin[warp][lane] = begin;
        row_prefix[warp][lane + 1] = inclusive;
    }
    if (lane == 0) row_prefix[warp][0] = 0;
    __syncwarp();
    const int64_t total = __shfl_sync(kFullMask, inclusive, 8);

    const int32_t self = args.self_slot[source];
    const long long ws[3] = {args.wraps[3 * source], args.wraps[3 * source + 1],
                             args.wraps[3 * source + 2]};
    const bool half = args.half_list != 0;
    const bool include_self = args.include_self != 0;
    const bool need_vector = args.out_d != nullptr || args.out_D != nullptr;
    int64_t out_base = 0;
    if constexpr (Write) out_base = args.pair_start[source];
    uint32_t count = 0;
    int row = 0;
    for (int64_t base = 0; base < total; base += 32) {
        const int64_t k = base + lane;
        bool accept = false;
        int32_t target = -1;
        long long shift[3] = {0, 0, 0};
        bool shift_known = false;
        T vec[3] = {T(0), T(0), T(0)};
        bool vec_known = false;
        if (k < total) {
            while (k >= row_prefix[warp][row + 1]) ++row;
            const int64_t slot = row_begin[warp][row] + (k - row_prefix[warp][row]);
            const V g = reinterpret_cast<const V*>(args.ghost_pos)[slot];
            const T dx = g.x - qs.x;
            const T dy = g.y - qs.y;
            const T dz = g.z - qs.z;
            const T d2 = dx * dx + dy * dy + dz * dz;
            if (d2 < plan.search_squared) {
                target = lane_to_index(g.w);
                if (slot == self) {
                    accept = include_self;  // the zero-shift self pair
                    shift_known = true;
                    vec_known = true;
                } else {
                    bool identity = true;
                    if (half && target != source) identity = source < target;
                    const bool exact = !(d2 < plan.inner_squared);
                    if ((half && target == source) || exact || (Write && (args.out_S || need_vector))) {
                        const int4 meta = args.ghost_meta[slot];
                        shift[0] = static_cast<long long>(meta.x) + ws[0];
                        shift[1] = static_cast<long long>(meta.y) + ws[1];
                        shift[2] = static_cast<long long>(meta.z) + ws[2];
                        shift_known = true;
                        if (half && target == source) identity = canonical_shift(shift);
                    }
                    if (identity) {
                        if (exact || (Write && need_vector)) {
                            exact_displacement(args.positions, source, target, shift, plan.cell, vec);
                            vec_known = true;
                            accept = !exact ||
                                exact_norm2(vec[0], vec[1], vec[2]) < plan.cutoff_squared;
                        } else {
                            accept = true;
                        }
                    }
                }
            }
        }
        (void)shift_known;
        (void)vec_known;
        const unsigned mask = __ballot_sync(kFullMask, accept);
        if constexpr (Write) {
            if (accept) {
                const int64_t o = out_base + count + __popc(mask & ((1u << lane) - 1u));
                emit_pair(args, o, source, target, shift, vec);
            }
        }
        count += __popc(mask);
    }
    if constexpr (!Write) {
        if (lane == 0) {
            args.counts[source] = count;
            if (count > static_cast<uint32_t>(INT_MAX)) {
                atomicOr(args.status, static_cast<uint32_t>(kStatusCountRange));
            }
        }
    }
}

// Brute force: one warp per source atom of a brute-force structure; lanes
// stride over the N x I (target, image) candidates, target fastest so that
// consecutive lanes read consecutive atoms.  Every candidate takes the exact
// predicate (tonari csrc/core/neighbors_cpu.cpp:222-273).
template <typename T, bool Write>
__global__ void __launch_bounds__(kSearchThreads) brute_search_kernel(SearchArgs<T> args) {
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t work = static_cast<int64_t>(blockIdx.x) * kSearchWarps + warp;
    if (work >= args.n_brute_atoms) return;
    const int32_t c = segment_of(args.brute_prefix, args.n_brute, work);
    const StructurePlan<T>& plan = args.plans[args.brute_structs[c]];
    const int64_t source = plan.atom_begin + (work - args.brute_prefix[c]);
    const long long ws[3] = {args.wraps[3 * source], args.wraps[3 * source + 1],
                             args.wraps[3 * source + 2]};
    const bool half = args.half_list != 0;
    const bool include_self = args.include_self != 0;
    const int64_t n = plan.n_atoms;
    const int64_t total = n * plan.n_images;
    int64_t out_base = 0;
    if constexpr (Write) out_base = args.pair_start[source];
    uint32_t count = 0;
    for (int64_t base = 0; base < total; base += 32) {
        const int64_t k = base + lane;
        bool accept = false;
        int64_t target = 0;
        long long shift[3] = {0, 0, 0};
        T vec[3] = {T(0), T(0), T(0)};
        if (k < total) {
            const int64_t image_index = k / n;
            target = plan.atom_begin + (k - image_index * n);
            int32_t image[3];
            decode_image(static_cast<int32_t>(image_index), plan.repeats, image);
#pragma unroll
            for (int a = 0; a < 3; ++a) {
                shift[a] = static_cast<long long>(image[a]) -
                           static_cast<long long>(args.wraps[3 * target + a]) + ws[a];
            }
            if (keep_identity(source, target, shift, half, include_self)) {
                const bool zero_self =
                    source == target && shift[0] == 0 && shift[1] == 0 && shift[2] == 0;
                if (zero_self) {
                    accept = true;
                } else {
                    exact_displacement(args.positions, source, target, shift, plan.cell, vec);
                    accept = exact_norm2(vec[0], vec[1], vec[2]) < plan.cutoff_squared;
                }
                if (accept && !shift_fits_int32(shift)) {
                    atomicOr(args.status, static_cast<uint32_t>(kStatusShiftRange));
                }
            }
        }
        const unsigned mask = __ballot_sync(kFullMask, accept);
        if constexpr (Write) {
            if (accept) {
                const int64_t o = out_base + count + __popc(mask & ((1u << lane) - 1u));
                emit_pair(args, o, source, target, shift, vec);
            }
        }
        count += __popc(mask);
    }
    if constexpr (!Write) {
        if (lane == 0) {
            args.counts[source] = count;
            if (count > static_cast<uint32_t>(INT_MAX)) {
                atomicOr(args.status, static_cast<uint32_t>(kStatusCountRange));
            }
        }
    }
}

int64_t blocks_for(int64_t items, int64_t per_block) { return (items + per_block - 1) / per_block; }

}  // namespace
}  // namespace tnr

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
namespace tnr {

template <typename T>
void launch_prepare(const PrepareArgs<T>& args, cudaStream_t stream) {
    if (args.n_atoms == 0) return;
    prepare_kernel<T><<<static_cast<unsigned>(blocks_for(args.n_atoms, kPrepareThreads)),
                        kPrepareThreads, 0, stream>>>(args);
}

template <typename T>
void launch_bin(const BinArgs<T>& args, bool scatter, cudaStream_t stream) {
    if (args.n_cell_atoms == 0) return;
    const unsigned blocks = static_cast<unsigned>(blocks_for(args.n_cell_atoms, kBinThreads));
    if (scatter) {
        bin_kernel<T, true><<<blocks, kBinThreads, 0, stream>>>(args);
    } else {
        bin_kernel<T, false><<<blocks, kBinThreads, 0, stream>>>(args);
    }
}

template <typename T>
void launch_cell_search(const SearchArgs<T>& args, bool write, cudaStream_t stream) {
    if (args.n_sources == 0) return;
    const unsigned blocks = static_cast<unsigned>(blocks_for(args.n_sources, kSearchWarps));
    if (write) {
        cell_search_kernel<T, true><<<blocks, kSearchThreads, 0, stream>>>(args);
    } else {
        cell_search_kernel<T, false><<<blocks, kSearchThreads, 0, stream>>>(args);
    }
}

template <typename T>
void launch_brute_search(const SearchArgs<T>& args, bool write, cudaStream_t stream) {
    if (args.n_brute_atoms == 0) return;
    const unsigned blocks = static_cast<unsigned>(blocks_for(args.n_brute_atoms, kSearchWarps));
    if (write) {
        brute_search_kernel<T, true><<<blocks, kSearchThreads, 0, stream>>>(args);
    } else {
        brute_search_kernel<T, false><<<blocks, kSearchThreads, 0, stream>>>(args);
    }
}

size_t scan_workspace_bytes(int64_t n) {
    const int64_t tiles = std::max<int64_t>(1, (n + kScanTile - 1) / kScanTile);
    // counter + flags, then 8-byte aligned aggregate and inclusive arrays.
    const size_t words = static_cast<size_t>(1 + tiles);
    const size_t head = (words * sizeof(uint32_t) + 15) / 16 * 16;
    return head + 2 * static_cast<size_t>(tiles) * sizeof(int64_t);
}

namespace {
template <typename In, typename Out>
void launch_scan(const In* in, int64_t n, Out* out, Out* out2, void* workspace,
                 uint32_t* status, cudaStream_t stream) {
    const int64_t tiles = std::max<int64_t>(1, (n + kScanTile - 1) / kScanTile);
    const size_t words = static_cast<size_t>(1 + tiles);
    const size_t head = (words * sizeof(uint32_t) + 15) / 16 * 16;
    char* bytes = static_cast<char*>(workspace);
    cudaMemsetAsync(bytes, 0, words * sizeof(uint32_t), stream);
    ScanTileState<Out> state;
    state.counter = reinterpret_cast<uint32_t*>(bytes);
    state.flags = state.counter + 1;
    state.aggregate = reinterpret_cast<Out*>(bytes + head);
    state.inclusive = state.aggregate + tiles;
    exclusive_scan_kernel<In, Out><<<static_cast<unsigned>(tiles), kScanThreads, 0, stream>>>(
        in, n, out, out2, state, status);
}
}  // namespace

void launch_scan_u64(const unsigned long long* in, int64_t n, unsigned long long* out,
                     unsigned long long* out2, void* workspace, uint32_t* status,
                     cudaStream_t stream) {
    launch_scan<unsigned long long, unsigned long long>(in, n, out, out2, workspace, status,
                                                        stream);
}

void launch_scan_counts(const uint32_t* in, int64_t n, int64_t* out, void* workspace,
                        uint32_t* status, cudaStream_t stream) {
    launch_scan<uint32_t, int64_t>(in, n, out, nullptr, workspace, status, stream);
}

#define TNR_INSTANTIATE(T)                                                                 \
    template void launch_prepare<T>(const PrepareArgs<T>&, cudaStream_t);                  \
    template void launch_bin<T>(const BinArgs<T>&, bool, cudaStream_t);                     \
    template void launch_cell_search<T>(const SearchArgs<T>&, bool, cudaStream_t);          \
    template void launch_brute_search<T>(const SearchArgs<T>&, bool, cudaStream_t);
TNR_INSTANTIATE(float)
TNR_INSTANTIATE(double)
#undef TNR_INSTANTIATE

}  // namespace tnr
