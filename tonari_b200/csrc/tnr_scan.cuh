// Single-pass exclusive prefix sum with decoupled look-back.
//
// Replaces the reference's torch::cumsum calls (tonari
// csrc/torch/neighbors_cell_cuda.cu:641-656 and :775-777), which are a
// library scan followed by a host round trip.  Each CTA claims a tile id in
// launch order (so every predecessor it waits on is already resident), scans
// its tile in registers and shared memory, publishes its aggregate, and then
// one thread walks back over predecessor tiles until it meets an inclusive
// prefix.  Every wait is bounded: after kScanSpinLimit polls the tile gives
// up, raises kStatusScanTimeout in the status word and carries on with the
// partial prefix, so a failure surfaces as a host error instead of a hang.
//
// out has n + 1 entries: out[k] = sum(in[0:k]), out[n] = total.  When out2 is
// non-null the same values are written there as well (used to initialise the
// scatter cursors of the binning pass in the same sweep).
#pragma once

#include <cstdint>

#include "tnr_plan.h"

namespace tnr {

constexpr int kScanThreads = 256;
constexpr int kScanItems = 8;
constexpr int kScanTile = kScanThreads * kScanItems;
constexpr uint32_t kScanSpinLimit = 1u << 22;

template <typename Out>
struct ScanTileState {
    uint32_t* counter;  // 1 word, zeroed before launch
    uint32_t* flags;    // [tiles], zeroed before launch: 0 none, 1 aggregate, 2 inclusive
    Out* aggregate;     // [tiles]
    Out* inclusive;     // [tiles]
};

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

template <typename In, typename Out>
__global__ void __launch_bounds__(kScanThreads)
exclusive_scan_kernel(const In* __restrict__ in, int64_t n, Out* __restrict__ out,
                      Out* __restrict__ out2, ScanTileState<Out> state, uint32_t* status) {
    __shared__ uint32_t tile_shared;
    __shared__ Out warp_totals[kScanThreads / 32];
    __shared__ Out tile_prefix_shared;
    if (threadIdx.x == 0) tile_shared = atomicAdd(state.counter, 1u);
    __syncthreads();
    const uint32_t tile = tile_shared;
    const int64_t base = static_cast<int64_t>(tile) * kScanTile;

    // Blocked load: thread t owns items [t*kScanItems, (t+1)*kScanItems).
    Out items[kScanItems];
    Out thread_sum = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        const int64_t index = base + threadIdx.x * kScanItems + k;
        items[k] = index < n ? static_cast<Out>(in[index]) : Out(0);
        thread_sum += items[k];
    }
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const Out warp_inclusive = warp_inclusive_sum(thread_sum);
    if (lane == 31) warp_totals[warp] = warp_inclusive;
    __syncthreads();
    if (warp == 0) {
        Out total = lane < kScanThreads / 32 ? warp_totals[lane] : Out(0);
        total = warp_inclusive_sum(total);
        if (lane < kScanThreads / 32) warp_totals[lane] = total;  // inclusive per warp
    }
    __syncthreads();
    const Out tile_total = warp_totals[kScanThreads / 32 - 1];

    if (threadIdx.x == 0) {
        Out prefix = 0;
        volatile uint32_t* flags = state.flags;
        if (tile == 0) {
            state.inclusive[0] = tile_total;
            __threadfence();
            flags[0] = 2u;
        } else {
            state.aggregate[tile] = tile_total;
            __threadfence();
            flags[tile] = 1u;
            int64_t predecessor = static_cast<int64_t>(tile) - 1;
            uint32_t spins = 0;
            while (predecessor >= 0) {
                const uint32_t flag = flags[predecessor];
                if (flag == 0u) {
                    if (++spins > kScanSpinLimit) {
                        atomicOr(status, static_cast<uint32_t>(kStatusScanTimeout));
                        break;
                    }
                    __nanosleep(32);
                    continue;
                }
                __threadfence();
                if (flag == 2u) {
                    prefix += *reinterpret_cast<volatile Out*>(&state.inclusive[predecessor]);
                    break;
                }
                prefix += *reinterpret_cast<volatile Out*>(&state.aggregate[predecessor]);
                --predecessor;
            }
            state.inclusive[tile] = prefix + tile_total;
            __threadfence();
            flags[tile] = 2u;
        }
        tile_prefix_shared = prefix;
    }
    __syncthreads();
    Out running = tile_prefix_shared + (warp > 0 ? warp_totals[warp - 1] : Out(0)) +
                  (warp_inclusive - thread_sum);
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        const int64_t index = base + threadIdx.x * kScanItems + k;
        if (index < n) {
            out[index] = running;
            if (out2) out2[index] = running;
        }
        running += items[k];
    }
    // The tile holding the last element also writes the grand total.
    const int64_t last = n - 1;
    if (n == 0) {
        if (tile == 0 && threadIdx.x == 0) {
            out[0] = 0;
            if (out2) out2[0] = 0;
        }
    } else if (last >= base + threadIdx.x * kScanItems &&
               last < base + (threadIdx.x + 1) * kScanItems) {
        out[n] = running;
        if (out2) out2[n] = running;
    }
}

}  // namespace tnr
