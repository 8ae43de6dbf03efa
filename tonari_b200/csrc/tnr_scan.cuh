// Exclusive prefix sum in three launches: per-tile sums, a one-block scan of
// the tile sums, and a pass that rescans each tile from its prefix.
//
// Replaces the reference's torch::cumsum calls (tonari
// csrc/torch/neighbors_cell_cuda.cu:641-656 and :775-777), which are a
// library scan followed by a host round trip.  No CTA waits on another, so
// the scan needs no spin loop; the input is read twice (it is small: one
// word per atom or per bin), every load and store is coalesced (lane-
// contiguous within a warp), and a tile of kScanTile items is one CTA.
//
// out has n + 1 entries: out[k] = sum(in[0:k]), out[n] = total.  When out2 is
// non-null the same values are written there as well (used to initialise the
// scatter cursors of the binning pass in the same sweep).
#pragma once

#include <cstdint>

#include "tnr_plan.h"

namespace tnr {

constexpr int kScanThreads = 256;
constexpr int kScanItems = 16;  // per thread
constexpr int kScanTile = kScanThreads * kScanItems;
constexpr int kScanTilesThreads = 1024;

template <typename Out>
__device__ __forceinline__ Out warp_inclusive_sum(Out value) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int offset = 1; offset < 32; offset <<= 1) {
        const Out other = __shfl_up_sync(0xffffffffu, value, offset);
        if (lane >= offset) value += other;
    }
    return value;
}

// Block-wide sum; every thread receives the total.
template <typename Out, int Threads>
__device__ __forceinline__ Out block_sum(Out value, Out* warp_shared) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1) value += __shfl_xor_sync(0xffffffffu, value, offset);
    if (lane == 0) warp_shared[warp] = value;
    __syncthreads();
    Out total = 0;
#pragma unroll
    for (int w = 0; w < Threads / 32; ++w) total += warp_shared[w];
    __syncthreads();
    return total;
}

// Pass 1: tile_sums[t] = sum of tile t.  Thread k of a warp reads items
// warp_base + 32 * i + k, so each load instruction is one contiguous run.
template <typename In, typename Out>
__global__ void __launch_bounds__(kScanThreads)
scan_reduce_kernel(const In* __restrict__ in, int64_t n, Out* __restrict__ tile_sums) {
    __shared__ Out warp_shared[kScanThreads / 32];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile + warp * (32 * kScanItems);
    Out sum = 0;
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
        const int64_t index = base + 32 * i + lane;
        if (index < n) sum += static_cast<Out>(in[index]);
    }
    const Out total = block_sum<Out, kScanThreads>(sum, warp_shared);
    if (threadIdx.x == 0) tile_sums[blockIdx.x] = total;
}

// Pass 2 (one CTA): tile_sums becomes its exclusive scan, in place.
template <typename Out>
__global__ void __launch_bounds__(kScanTilesThreads)
scan_tiles_kernel(Out* __restrict__ tile_sums, int64_t tiles) {
    __shared__ Out warp_shared[kScanTilesThreads / 32];
    __shared__ Out carry_shared;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    Out carry = 0;
    for (int64_t chunk = 0; chunk < tiles; chunk += kScanTilesThreads) {
        const int64_t index = chunk + threadIdx.x;
        const Out value = index < tiles ? tile_sums[index] : Out(0);
        const Out inclusive = warp_inclusive_sum(value);
        if (lane == 31) warp_shared[warp] = inclusive;
        __syncthreads();
        if (warp == 0) {
            const Out w = warp_shared[lane];
            const Out w_inclusive = warp_inclusive_sum(w);
            warp_shared[lane] = w_inclusive - w;  // exclusive per warp
            if (lane == 31) carry_shared = w_inclusive;
        }
        __syncthreads();
        if (index < tiles) tile_sums[index] = carry + warp_shared[warp] + inclusive - value;
        carry += carry_shared;
        __syncthreads();
    }
}

// Pass 3: every tile rescans its items from its prefix and writes out (and
// out2); the tile holding the last item also writes out[n].
template <typename In, typename Out>
__global__ void __launch_bounds__(kScanThreads)
scan_apply_kernel(const In* __restrict__ in, int64_t n, const Out* __restrict__ tile_prefix,
                  Out* __restrict__ out, Out* __restrict__ out2) {
    __shared__ Out warp_shared[kScanThreads / 32];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile + warp * (32 * kScanItems);
    Out values[kScanItems];
    Out sum = 0;
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
        const int64_t index = base + 32 * i + lane;
        values[i] = index < n ? static_cast<Out>(in[index]) : Out(0);
        sum += values[i];
    }
    // This warp's total, then the prefix of the warps before it.
    Out warp_total = sum;
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1) {
        warp_total += __shfl_xor_sync(0xffffffffu, warp_total, offset);
    }
    if (lane == 0) warp_shared[warp] = warp_total;
    __syncthreads();
    Out running = tile_prefix[blockIdx.x];
    for (int w = 0; w < warp; ++w) running += warp_shared[w];
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
        const Out inclusive = warp_inclusive_sum(values[i]);
        const int64_t index = base + 32 * i + lane;
        if (index < n) {
            out[index] = running + inclusive - values[i];
            if (out2) out2[index] = running + inclusive - values[i];
        }
        running += __shfl_sync(0xffffffffu, inclusive, 31);
    }
    const int64_t last_tile = n == 0 ? 0 : (n - 1) / kScanTile;
    if (blockIdx.x == last_tile && threadIdx.x == kScanThreads - 1) {
        // The last warp's running value is the grand total.
        out[n] = running;
        if (out2) out2[n] = running;
    }
}

}  // namespace tnr
