// Host scheduler behind the C ABI (include/tonari_b200.h).
//
// Replaces tonari csrc/torch/bindings_cuda.cpp:59-228 and the host drivers
// neighbor_list_cuda_brute_force (csrc/torch/neighbors_cuda.cu:443-556) and
// neighbor_list_cuda_cell (csrc/torch/neighbors_cell_cuda.cu:558-814).
//
// Differences in design (same results):
//   * algorithm selection is per structure (brute force for small candidate
//     counts, cell list otherwise) instead of one choice for the whole batch;
//   * the cell list bins image copies into a CSR layout by histogram -> scan
//     -> scatter instead of per-bin linked lists, and never falls back to an
//     O(N^2) pass because a wrap is nonzero: its final test is the public
//     displacement formula, like the reference CPU cell list;
//   * sorted calls write each source's pairs at its own offset (no argsort);
//     unsorted calls test each unordered pair once and write in cell order;
//   * host round trips: at most four small device->host reads (input
//     metadata, per-structure extents, ghost total, pair total), each a
//     pinned-memory copy.
#include "tonari_b200.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>

#include <cstring>
#include <limits>
#include <string>
#include <vector>

#include "tnr_geometry.h"
#include "tnr_pool.h"
#include "tnr_launch.h"
#include "tnr_plan.h"

namespace tnr {
namespace {

// Auto rule: a structure whose per-source candidate count (atoms x images)
// is at most this takes the brute-force kernel; TONARI_B200_BRUTE_CANDIDATES
// overrides it (a tuning knob; results do not depend on it).
constexpr int64_t kBruteCandidatesPerSource = 256;

int64_t brute_candidates_per_source() {
    static const int64_t value = [] {
        const char* text = std::getenv("TONARI_B200_BRUTE_CANDIDATES");
        return text ? std::max<int64_t>(0, std::atoll(text)) : kBruteCandidatesPerSource;
    }();
    return value;
}
// The reference's bin-layout safety limits (tonari csrc/core/neighbors_cpu.cpp:23-24).
constexpr int64_t kMaximumDenseBins = int64_t{1} << 26;
constexpr int64_t kMaximumBinsPerImage = 64;
// Total bins of one call (memory guard across a batch).
constexpr int64_t kMaximumTotalBins = int64_t{1} << 28;
constexpr int kRoundoffFactor = 64;
// Calls whose ghost and bitmask bounds fit this much workspace size those
// buffers from the bounds instead of reading the exact totals back (one
// host round trip less).  A 1,024-structure shard of a cfg5-like batch
// bounds at about 2.7 GB; the caching allocator reuses the blocks across
// calls, so only the device memory held grows, not the time.
constexpr int64_t kBoundedWorkspaceBytes = int64_t{4} << 30;
// Calls of at least this many atoms run the speculative wrap check on a side
// stream beside the search.
constexpr int64_t kSideStreamAtoms = 500000;

thread_local int64_t g_launches = 0;
thread_local float g_phase_ms[6] = {0, 0, 0, 0, 0, 0};
constexpr int kHostMarks = 12;
thread_local double g_host_ms[kHostMarks] = {};

struct CudaError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

void check_cuda(cudaError_t error, const char* what) {
    if (error != cudaSuccess) {
        throw CudaError(std::string(what) + ": " + cudaGetErrorString(error));
    }
}

void check_launch(const char* what) { check_cuda(cudaGetLastError(), what); }

// ---- allocation ------------------------------------------------------------

void* default_allocate(void*, size_t bytes, tnr_stream stream) {
    void* pointer = nullptr;
    if (cudaMallocAsync(&pointer, bytes, reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return pointer;
}

void default_release(void*, void* pointer, tnr_stream stream) {
    cudaFreeAsync(pointer, reinterpret_cast<cudaStream_t>(stream));
}

// Workspace buffers of one call, released in stream order when it returns.
class Workspace {
public:
    Workspace(const tnr_allocator& allocator, cudaStream_t stream)
        : allocator_(allocator), stream_(stream) {}
    ~Workspace() {
        for (void* pointer : buffers_) {
            allocator_.release(allocator_.context, pointer,
                               reinterpret_cast<tnr_stream>(stream_));
        }
    }
    Workspace(const Workspace&) = delete;
    Workspace& operator=(const Workspace&) = delete;

    template <typename U>
    U* get(size_t count) {
        void* pointer = raw(std::max<size_t>(count * sizeof(U), 16));
        return static_cast<U*>(pointer);
    }
    // Buffers up to kCarveLimit bytes are carved (256-byte aligned) out of
    // kChunkBytes chunks, so a call makes a few allocator round trips
    // instead of one per small buffer; larger ones are allocated directly.
    // Every chunk and buffer is released in stream order when the call ends.
    void* raw(size_t bytes) {
        bytes = (bytes + 255) / 256 * 256;
        if (bytes <= kCarveLimit) {
            if (chunk_ == nullptr || chunk_used_ + bytes > kChunkBytes) {
                chunk_ = static_cast<char*>(allocate(kChunkBytes));
                chunk_used_ = 0;
            }
            void* pointer = chunk_ + chunk_used_;
            chunk_used_ += bytes;
            return pointer;
        }
        return allocate(bytes);
    }
    // Output buffers are not released by the workspace.
    template <typename U>
    U* output(size_t count) {
        void* pointer = allocator_.allocate(allocator_.context,
                                            std::max<size_t>(count * sizeof(U), 16),
                                            reinterpret_cast<tnr_stream>(stream_));
        if (pointer == nullptr) throw std::bad_alloc();
        outputs_.push_back(pointer);
        return static_cast<U*>(pointer);
    }
    void release_outputs() {
        for (void* pointer : outputs_) {
            allocator_.release(allocator_.context, pointer,
                               reinterpret_cast<tnr_stream>(stream_));
        }
        outputs_.clear();
    }
    void keep_outputs() { outputs_.clear(); }

private:
    static constexpr size_t kCarveLimit = size_t{256} << 10;
    static constexpr size_t kChunkBytes = size_t{4} << 20;
    void* allocate(size_t bytes) {
        void* pointer = allocator_.allocate(allocator_.context, bytes,
                                            reinterpret_cast<tnr_stream>(stream_));
        if (pointer == nullptr) throw std::bad_alloc();
        buffers_.push_back(pointer);
        return pointer;
    }
    tnr_allocator allocator_;
    cudaStream_t stream_;
    std::vector<void*> buffers_;
    std::vector<void*> outputs_;
    char* chunk_ = nullptr;
    size_t chunk_used_ = 0;
};

// Pinned host staging, one growable buffer per host thread.  Every call
// synchronises its stream before returning, so a later call never overwrites
// bytes an earlier copy is still reading.
class Pinned {
public:
    ~Pinned() {
        if (data_) cudaFreeHost(data_);
    }
    char* reserve(size_t bytes) {
        if (bytes > size_) {
            if (data_) cudaFreeHost(data_);
            data_ = nullptr;
            size_ = 0;
            const size_t grown = std::max<size_t>(bytes, 1 << 16);
            check_cuda(cudaHostAlloc(reinterpret_cast<void**>(&data_), grown,
                                     cudaHostAllocPortable), "cudaHostAlloc");
            size_ = grown;
        }
        return data_;
    }

private:
    char* data_ = nullptr;
    size_t size_ = 0;
};

thread_local Pinned g_pinned;

// A second stream (per host thread and device) for work that can overlap the
// call's main stream, with the two events that fork and join it.  Like every
// launch of this library it assumes the current device is the stream's.
struct SideStream {
    cudaStream_t stream = nullptr;
    cudaEvent_t fork = nullptr;
    cudaEvent_t join = nullptr;
    cudaEvent_t metadata = nullptr;  // the call's metadata copy has landed
};

SideStream& side_stream() {
    thread_local SideStream streams[64];
    int device = 0;
    check_cuda(cudaGetDevice(&device), "cudaGetDevice");
    SideStream& side = streams[device & 63];
    if (side.stream == nullptr) {
        check_cuda(cudaStreamCreateWithFlags(&side.stream, cudaStreamNonBlocking), "side stream");
        check_cuda(cudaEventCreateWithFlags(&side.fork, cudaEventDisableTiming), "fork event");
        check_cuda(cudaEventCreateWithFlags(&side.join, cudaEventDisableTiming), "join event");
        check_cuda(cudaEventCreateWithFlags(&side.metadata, cudaEventDisableTiming), "metadata event");
    }
    return side;
}

// Packs several host arrays into a caller-provided pinned region (256-byte
// aligned offsets) and uploads them with a single copy.
class Upload {
public:
    explicit Upload(char* pinned, size_t capacity) : pinned_(pinned), capacity_(capacity) {}
    template <typename U>
    size_t add(const U* data, size_t count) {
        const size_t offset = (size_ + 255) / 256 * 256;
        const size_t bytes = count * sizeof(U);
        if (offset + std::max<size_t>(bytes, 1) > capacity_) {
            throw std::runtime_error("internal error: upload staging overflow");
        }
        if (bytes) std::memcpy(pinned_ + offset, data, bytes);
        size_ = offset + std::max<size_t>(bytes, 1);
        return offset;
    }
    // Reserves room for `count` items to be written in place (no copy).
    template <typename U>
    U* place(size_t count, size_t& offset) {
        offset = add<U>(nullptr, 0);
        const size_t bytes = count * sizeof(U);
        if (offset + std::max<size_t>(bytes, 1) > capacity_) {
            throw std::runtime_error("internal error: upload staging overflow");
        }
        size_ = offset + std::max<size_t>(bytes, 1);
        return reinterpret_cast<U*>(pinned_ + offset);
    }
    char* commit(Workspace& workspace, cudaStream_t stream) {
        char* device = static_cast<char*>(workspace.raw(std::max<size_t>(size_, 16)));
        check_cuda(cudaMemcpyAsync(device, pinned_, size_, cudaMemcpyHostToDevice, stream),
                   "upload");
        return device;
    }

private:
    char* pinned_;
    size_t capacity_;
    size_t size_ = 0;
};

struct PhaseTimer {
    bool enabled = false;
    cudaStream_t stream = nullptr;
    cudaEvent_t events[7] = {};
    int recorded = 0;
    std::chrono::steady_clock::time_point start;
    // Host wall time (ms since the call began) at host mark `index`.
    void host(int index) {
        if (enabled && index < kHostMarks) {
            g_host_ms[index] = std::chrono::duration<double, std::milli>(
                std::chrono::steady_clock::now() - start).count();
        }
    }
    explicit PhaseTimer(cudaStream_t s) : stream(s) {
        const char* flag = std::getenv("TONARI_B200_PHASE_TIMERS");
        enabled = flag && flag[0] == '1';
        for (float& value : g_phase_ms) value = 0.0f;
        for (double& value : g_host_ms) value = 0.0;
        start = std::chrono::steady_clock::now();
        if (enabled) {
            for (auto& event : events) cudaEventCreate(&event);
        }
    }
    ~PhaseTimer() {
        if (enabled) {
            for (auto& event : events) cudaEventDestroy(event);
        }
    }
    void mark(int index) {
        if (enabled && index < 7) {
            cudaEventRecord(events[index], stream);
            recorded = std::max(recorded, index + 1);
        }
    }
    void finish() {
        if (!enabled || recorded < 2) return;
        cudaEventSynchronize(events[recorded - 1]);
        for (int k = 0; k + 1 < recorded && k < 6; ++k) {
            cudaEventElapsedTime(&g_phase_ms[k], events[k], events[k + 1]);
        }
    }
};

}  // namespace
}  // namespace tnr

namespace tnr {
namespace {

// Host mirror of the device order keys (tnr_kernels.cuh order_key).
int32_t host_key(float v) {
    int32_t bits;
    std::memcpy(&bits, &v, 4);
    return bits >= 0 ? bits : bits ^ 0x7fffffff;
}
long long host_key(double v) {
    long long bits;
    std::memcpy(&bits, &v, 8);
    return bits >= 0 ? bits : bits ^ 0x7fffffffffffffffLL;
}
float host_value(int32_t key, float) {
    const int32_t bits = key >= 0 ? key : key ^ 0x7fffffff;
    float v;
    std::memcpy(&v, &bits, 4);
    return v;
}
double host_value(long long key, double) {
    const long long bits = key >= 0 ? key : key ^ 0x7fffffffffffffffLL;
    double v;
    std::memcpy(&v, &bits, 8);
    return v;
}

template <typename T>
Reduction<T> neutral_reduction() {
    Reduction<T> r{};
    for (int c = 0; c < 3; ++c) {
        r.wrapped_min[c] = host_key(std::numeric_limits<T>::infinity());
        r.wrapped_max[c] = host_key(-std::numeric_limits<T>::infinity());
        r.position_abs_max[c] = host_key(T(0));
        r.wrap_abs_max[c] = 0;
    }
    return r;
}

const char* kCannotSafely =
    "cell_list cannot safely process this structure; use algorithm='auto' or 'brute_force'";

enum class CellPlan { kReady, kUnsafe, kPreferBrute };

// Cell-list plan of one structure from its reduced extents, following the
// reference's safety rules (tonari csrc/core/neighbors_cpu.cpp:156-219 for the
// padded search radius, :379-430 for the bin layout).  kUnsafe is the
// reference's "cannot safely process" outcome; kPreferBrute marks inputs this
// implementation routes to the brute-force kernel for its own reasons (output
// shifts that could leave int32), with the same pair set.
template <typename T>
CellPlan plan_cell(StructurePlan<T>& plan, const Reduction<T>& reduction, const T* cell,
               const double* dual, double cutoff) {
    // Half-list order keys of one structure are compared as signed 32-bit
    // differences, exact below 2^30 atoms.
    if (plan.n_atoms >= (int32_t{1} << 30) - 2) return CellPlan::kPreferBrute;
    const T scalar_cutoff = static_cast<T>(cutoff);
    T lo[3], hi[3];
    long double scale = 0.0L;
    for (int c = 0; c < 3; ++c) {
        lo[c] = host_value(reduction.wrapped_min[c], T(0));
        hi[c] = host_value(reduction.wrapped_max[c], T(0));
        if (!std::isfinite(lo[c]) || !std::isfinite(hi[c])) return CellPlan::kUnsafe;
        long double component =
            2.0L * static_cast<long double>(host_value(reduction.position_abs_max[c], T(0)));
        for (int a = 0; a < 3; ++a) {
            const int64_t output_shift =
                static_cast<int64_t>(plan.repeats[a]) + 2 * static_cast<int64_t>(reduction.wrap_abs_max[a]);
            component += static_cast<long double>(output_shift) *
                         std::abs(static_cast<long double>(cell[3 * a + c]));
        }
        scale = std::max(scale, component);
    }
    // Output shifts of cell-list pairs are image - wrap_t + wrap_s; keep them
    // inside int32 so the search kernel needs no range test.
    for (int a = 0; a < 3; ++a) {
        const int64_t bound = static_cast<int64_t>(plan.repeats[a]) +
                              2 * static_cast<int64_t>(reduction.wrap_abs_max[a]);
        if (bound >= std::numeric_limits<int32_t>::max()) return CellPlan::kPreferBrute;
    }
    const long double padding = kRoundoffFactor * std::numeric_limits<T>::epsilon() * scale;
    const long double padded = static_cast<long double>(scalar_cutoff) + padding;
    if (!std::isfinite(static_cast<double>(padded)) || padded > 2 * static_cast<long double>(scalar_cutoff) ||
        padded > std::numeric_limits<T>::max()) {
        return CellPlan::kUnsafe;
    }
    const T search = std::nextafter(static_cast<T>(padded), std::numeric_limits<T>::infinity());
    if (!std::isfinite(search)) return CellPlan::kUnsafe;
    const T inner = std::max(T(0), 2 * scalar_cutoff - search);

    // Reference bin layout test with bin edge = search radius.
    int64_t count = 1;
    int64_t dims0[3];
    for (int c = 0; c < 3; ++c) {
        const T span = hi[c] - lo[c] + 2 * search;
        const T dimension = span / search;
        if (!std::isfinite(dimension) || dimension > kMaximumDenseBins) return CellPlan::kUnsafe;
        dims0[c] = std::max<int64_t>(1, static_cast<int64_t>(std::ceil(dimension)));
        if (count > kMaximumDenseBins / dims0[c]) return CellPlan::kUnsafe;
        count *= dims0[c];
    }
    const int64_t possible_images = static_cast<int64_t>(plan.n_atoms) * plan.n_images;
    if ((count + kMaximumBinsPerImage - 1) / kMaximumBinsPerImage > possible_images) return CellPlan::kUnsafe;

    // Actual grid: the edge is widened by a few ulps of the largest bin
    // coordinate so that two points closer than the search radius can never
    // land two bins apart after rounding.
    const int64_t largest = std::max({dims0[0], dims0[1], dims0[2]}) + 2;
    const double widen = 1.0 + 8.0 * std::numeric_limits<T>::epsilon() * static_cast<double>(largest);
    const T edge = static_cast<T>(static_cast<double>(search) * widen);
    plan.inv_edge = T(1) / edge;
    for (int c = 0; c < 3; ++c) {
        plan.origin[c] = lo[c] - search;
        plan.lower[c] = lo[c] - search;
        plan.upper[c] = hi[c] + search;
        const T span = hi[c] - lo[c] + 2 * search;
        int64_t dim = std::max<int64_t>(1, static_cast<int64_t>(std::ceil(span / edge)));
        dim = std::min(dim, dims0[c]);
        plan.dims[c] = static_cast<int32_t>(dim);
    }
    plan.search_squared = search * search;
    // Every nonzero lattice translation is at least as long as the smallest
    // perpendicular width 1 / |dual column|; only below the search radius
    // can an atom's own image be its candidate.
    plan.self_images = 0;
    for (int a = 0; a < 3; ++a) {
        const double norm = std::sqrt(dual[a] * dual[a] + dual[3 + a] * dual[3 + a] + dual[6 + a] * dual[6 + a]);
        if (static_cast<double>(search) * norm * (1.0 + 1e-6) >= 1.0) plan.self_images = 1;
    }
    plan.inner_squared = inner * inner;
    return CellPlan::kReady;
}

// Raised when the device's speculative geometry cannot be used; the call is
// then repeated with the host's exact geometry.
struct SpeculationFailed {};

// Batches of at least this many float32 structures compute their periodic
// geometry on the device first and verify it on the host while the search
// runs (the host's long-double geometry takes about 1 us per structure).
constexpr int64_t kSpeculativeGeometryBatch = 64;

template <typename T>
bool speculate_geometry(const tnr_request& request) {
    if (!std::is_same<T, float>::value) return false;
    if (request.n_structures < kSpeculativeGeometryBatch || request.n_atoms == 0) return false;
    const char* flag = std::getenv("TONARI_B200_HOST_GEOMETRY");
    return !(flag && flag[0] == '1');
}

// Host arrays of one call, kept per host thread and per element type so that
// consecutive calls reuse their memory: freshly allocated arrays of a large
// batch cost a page fault per 4 KB on first touch (about 0.1 ms for 8,192
// structures).  run() binds each to a local reference, which the host pool's
// lambdas capture, so worker threads read the calling thread's arrays.
template <typename T>
struct HostArrays {
    std::vector<int64_t> batch_ptr;
    std::vector<T> cell;
    std::vector<uint8_t> pbc;
    std::vector<int64_t> counts;
    std::vector<double> cell64;
    std::vector<int32_t> mode;
    std::vector<CellPlan> outcomes;
    std::vector<int32_t> cell_structs, brute_structs;
    std::vector<int64_t> cell_prefix, brute_prefix, cell_bin_prefix;
    PeriodicGeometry geometry;
};

template <typename T>
HostArrays<T>& host_arrays() {
    thread_local HostArrays<T> arrays;
    return arrays;
}

template <typename T>
void run(const tnr_request& request, Workspace& workspace, cudaStream_t stream,
         tnr_result& result, bool speculate) {
    using V4 = typename std::conditional<std::is_same<T, float>::value, float4, double4>::type;
    const int64_t n_atoms = request.n_atoms;
    const int64_t batch = request.n_structures;
    PhaseTimer timer(stream);

    // One pinned block for every later upload and readback of this call.
    const size_t prepare_bytes = static_cast<size_t>(batch) *
        (sizeof(PrepareStructure<T>) + sizeof(Reduction<T>)) + 1024;
    const size_t plan_bytes = static_cast<size_t>(batch) *
        (sizeof(StructurePlan<T>) + 3 * sizeof(int64_t) + 2 * sizeof(int32_t)) +
        8192;
    const size_t read_bytes =
        static_cast<size_t>(batch) * (sizeof(Reduction<T>) + sizeof(DeviceGeometry)) + 2048;
    const size_t block_bytes = prepare_bytes + plan_bytes + read_bytes;

    // Device work of the first phase: wraps, wrapped positions and extents
    // (prepare kernel), after the speculative geometry kernel when the
    // geometry is speculated.  Host path: prepare records and neutral
    // extents are uploaded from the pinned block first.
    PrepareStructure<T>* d_prepare = nullptr;
    Reduction<T>* d_reductions = nullptr;
    int32_t* d_atom_struct = nullptr;
    int32_t* d_wraps = nullptr;
    V4* d_wrapped = nullptr;
    uint32_t* d_status = nullptr;
    DeviceGeometry* d_geometry = nullptr;
    SideStream* side = nullptr;
    int64_t* d_batch_ptr = const_cast<int64_t*>(request.batch_ptr);
    bool launched = false;
    auto launch_first_phase = [&]() {
        if (d_batch_ptr == nullptr) {
            throw InputError("batch_ptr device pointer is required");
        }
        if (speculate) {
            d_prepare = workspace.get<PrepareStructure<T>>(static_cast<size_t>(batch));
            d_reductions = workspace.get<Reduction<T>>(static_cast<size_t>(batch));
        }
        d_atom_struct = workspace.get<int32_t>(n_atoms);
        d_wraps = workspace.get<int32_t>(3 * n_atoms);
        d_wrapped = workspace.get<V4>(n_atoms);
        d_status = workspace.get<uint32_t>(4);
        check_cuda(cudaMemsetAsync(d_status, 0, 4 * sizeof(uint32_t), stream), "memset status");
        if (speculate) {
            d_geometry = workspace.get<DeviceGeometry>(batch);
            launch_geometry<T>(static_cast<const T*>(request.cell), request.pbc, d_batch_ptr, batch,
                               request.cutoff, d_prepare, d_geometry, d_status + 1, d_reductions, stream);
            check_launch("geometry kernel");
        }
        PrepareArgs<T> prepare_args{static_cast<const T*>(request.positions), n_atoms, d_batch_ptr,
                                    batch, d_prepare, d_atom_struct, d_wraps, d_wrapped,
                                    d_reductions, d_status};
        launch_prepare(prepare_args, stream);
        check_launch("prepare kernel");
        // The wrap check (speculative geometry) forks here: it needs only the
        // prepare kernel's wraps and runs beside the search on a side stream.
        // Small calls keep it on the main stream, where it costs less than the
        // fork and join.
        side = speculate && n_atoms >= kSideStreamAtoms ? &side_stream() : nullptr;
        if (side) check_cuda(cudaEventRecord(side->fork, stream), "fork record");
        launched = true;
    };

    // ---- host metadata (tonari csrc/torch/bindings_cuda.cpp:96-131) -------
    // Speculative geometry needs no host metadata to start: its kernels read
    // batch_ptr, cell and pbc on the device, so they are queued right behind
    // the metadata copy and run while the host waits for it and plans.  The
    // host checks batch_ptr afterwards, with the reference's messages and
    // order; the kernels stay within bounds for any batch_ptr that starts at
    // zero, and the prepare kernel does nothing for one that does not.
    HostArrays<T>& arrays = host_arrays<T>();
    std::vector<int64_t>& batch_ptr = arrays.batch_ptr;
    std::vector<T>& cell_t = arrays.cell;
    std::vector<uint8_t>& pbc = arrays.pbc;
    batch_ptr.resize(static_cast<size_t>(batch + 1));
    cell_t.resize(static_cast<size_t>(9 * batch));
    pbc.resize(static_cast<size_t>(3 * batch));
    char* pinned = nullptr;
    if (request.batch_ptr_host && request.cell_host && request.pbc_host) {
        std::memcpy(batch_ptr.data(), request.batch_ptr_host, batch_ptr.size() * sizeof(int64_t));
        std::memcpy(cell_t.data(), request.cell_host, cell_t.size() * sizeof(T));
        std::memcpy(pbc.data(), request.pbc_host, pbc.size());
    } else {
        const size_t b0 = batch_ptr.size() * sizeof(int64_t);
        const size_t b1 = (cell_t.size() * sizeof(T) + 15) / 16 * 16;
        const size_t staging_bytes = b0 + b1 + pbc.size() + 64;
        const bool early = speculate && n_atoms > 0;
        // Early launch: the staging area follows the call's block, which is
        // then reserved once, before any copy into it is queued.
        char* staging = early ? (pinned = g_pinned.reserve(block_bytes + staging_bytes)) + block_bytes
                              : g_pinned.reserve(staging_bytes);
        check_cuda(cudaMemcpyAsync(staging, request.batch_ptr, b0, cudaMemcpyDeviceToHost, stream), "read batch_ptr");
        if (batch) {
            check_cuda(cudaMemcpyAsync(staging + b0, request.cell, cell_t.size() * sizeof(T),
                                       cudaMemcpyDeviceToHost, stream), "read cell");
            check_cuda(cudaMemcpyAsync(staging + b0 + b1, request.pbc, pbc.size(),
                                       cudaMemcpyDeviceToHost, stream), "read pbc");
        }
        if (early) {
            SideStream& events = side_stream();
            check_cuda(cudaEventRecord(events.metadata, stream), "metadata record");
            timer.mark(0);
            launch_first_phase();
            check_cuda(cudaEventSynchronize(events.metadata), "metadata read");
        } else {
            check_cuda(cudaStreamSynchronize(stream), "metadata read");
        }
        std::memcpy(batch_ptr.data(), staging, b0);
        std::memcpy(cell_t.data(), staging + b0, cell_t.size() * sizeof(T));
        std::memcpy(pbc.data(), staging + b0 + b1, pbc.size());
    }
    require_input(batch_ptr[0] == 0, "batch_ptr must start at zero");
    require_input(batch_ptr[batch] == n_atoms, "batch_ptr must end at N_total");
    timer.host(0);  // metadata on the host
    std::vector<int64_t>& counts = arrays.counts;
    counts.resize(static_cast<size_t>(batch));
    for (int64_t b = 0; b < batch; ++b) {
        require_input(batch_ptr[b + 1] >= batch_ptr[b], "batch_ptr must be nondecreasing");
        counts[b] = batch_ptr[b + 1] - batch_ptr[b];
    }
    for (uint8_t& flag : pbc) flag = flag ? 1 : 0;
    // The host geometry works on float64 cells.  Under speculation it runs
    // only for the check beside the count pass, so the widening (about
    // 0.1 ms for 8,192 cells) waits until then.
    std::vector<double>& cell64 = arrays.cell64;
    PeriodicGeometry& geometry = arrays.geometry;
    if (!speculate) {
        cell64.assign(cell_t.begin(), cell_t.end());
        geometry = build_geometry(cell64.data(), pbc.data(), counts.data(), batch, request.cutoff);
    }
    timer.host(1);  // periodic geometry (host path)

    result.n_pairs = 0;
    if (n_atoms == 0) return;
    if (!launched) {
        timer.mark(0);
        // Reserved after the metadata copy above has completed.
        pinned = g_pinned.reserve(block_bytes);
    }
    char* pinned_prepare = pinned;
    char* pinned_plan = pinned + prepare_bytes;
    char* pinned_read = pinned + prepare_bytes + plan_bytes;

    if (!launched) {
        if (!speculate) {
            Upload first(pinned_prepare, prepare_bytes);
            size_t off_prepare = 0, off_reduction = 0;
            PrepareStructure<T>* prepare = first.place<PrepareStructure<T>>(static_cast<size_t>(batch), off_prepare);
            Reduction<T>* neutral = first.place<Reduction<T>>(static_cast<size_t>(batch), off_reduction);
            const Reduction<T> neutral_value = neutral_reduction<T>();
            HostPool::instance().parallel_for(batch, 1024, [&](int64_t begin, int64_t end) {
                for (int64_t b = begin; b < end; ++b) {
                    neutral[b] = neutral_value;
                    PrepareStructure<T>& st = prepare[b];
                    st.atom_begin = batch_ptr[b];
                    st.atom_end = batch_ptr[b + 1];
                    for (int k = 0; k < 9; ++k) {
                        st.cell[k] = cell_t[9 * b + k];
                        st.dual[k] = static_cast<T>(geometry.duals[9 * b + k]);
                    }
                }
            });
            char* first_device = first.commit(workspace, stream);
            d_prepare = reinterpret_cast<PrepareStructure<T>*>(first_device + off_prepare);
            d_reductions = reinterpret_cast<Reduction<T>*>(first_device + off_reduction);
        }
        launch_first_phase();
    }
    timer.host(2);  // prepare launched
    timer.mark(1);

    auto check_status = [&](uint32_t status) {
        require_search(!(status & kStatusNonFinite), "positions must contain only finite values");
        require_search(!(status & kStatusWrapRange),
                       "atom representatives require periodic wraps outside the int32 range");
        require_search(!(status & kStatusShiftRange),
                       "a cell shift required by the cutoff pairs exceeds the int32 output range");
        require_search(!(status & kStatusCapacity), "an internal capacity was exceeded");
        require_search(!(status & kStatusCountRange),
                       "a per-source pair count exceeds the int32 range");
    };

    // Speculative geometry: read back the device's geometry with the extents
    // (one synchronisation) and use it for the plans.  Any flagged structure,
    // an error status or an image total beyond the limit sends the call to
    // the exact host path, which decides results and errors.
    const size_t reduction_bytes = static_cast<size_t>(batch) * sizeof(Reduction<T>);
    const Reduction<T>* reductions = nullptr;
    const DeviceGeometry* speculated = nullptr;  // device geometry records (speculation)
    auto dual_of = [&](int64_t b) -> const double* {
        return speculated ? speculated[b].dual : geometry.duals.data() + 9 * b;
    };
    auto repeats_of = [&](int64_t b, int a) -> int64_t {
        return speculated ? speculated[b].repeats[a] : geometry.repeats[3 * b + a];
    };
    if (speculate) {
        // Pinned read-back block: extents, two status words, then geometry.
        const size_t geometry_offset = (reduction_bytes + 2 * sizeof(uint32_t) + 255) / 256 * 256;
        const DeviceGeometry* device_geometry =
            reinterpret_cast<const DeviceGeometry*>(pinned_read + geometry_offset);
        check_cuda(cudaMemcpyAsync(pinned_read, d_reductions, reduction_bytes,
                                   cudaMemcpyDeviceToHost, stream), "read extents");
        check_cuda(cudaMemcpyAsync(pinned_read + reduction_bytes, d_status, 2 * sizeof(uint32_t),
                                   cudaMemcpyDeviceToHost, stream), "read status");
        check_cuda(cudaMemcpyAsync(pinned_read + geometry_offset, d_geometry,
                                   static_cast<size_t>(batch) * sizeof(DeviceGeometry),
                                   cudaMemcpyDeviceToHost, stream), "read geometry");
        HostPool::instance().prewake();  // the plans are built right after the wait
        check_cuda(cudaStreamSynchronize(stream), "extents");
        reductions = reinterpret_cast<const Reduction<T>*>(pinned_read);
        uint32_t status[2] = {0, 0};
        std::memcpy(status, pinned_read + reduction_bytes, sizeof(status));
        timer.host(3);  // extents and geometry read back
        if (status[0] != 0 || status[1] != 0) throw SpeculationFailed{};
        // The plans read duals and repeats straight from the read-back
        // records; only the image prefix is built here.
        speculated = device_geometry;
        geometry.image_begin.assign(static_cast<size_t>(batch + 1), 0);
        for (int64_t b = 0; b < batch; ++b) {
            geometry.image_begin[b + 1] = geometry.image_begin[b] + device_geometry[b].images;
            if (geometry.image_begin[b + 1] > (int64_t{1} << 24)) throw SpeculationFailed{};
        }
        timer.host(9);  // device geometry taken over
    }

    // ---- per-structure algorithm and plans ---------------------------------
    // Plans are built in place in the pinned upload block by the host pool;
    // without speculation this overlaps the prepare kernel, and the cell
    // plans, which need the extents, follow the read-back.
    std::vector<int32_t>& mode = arrays.mode;
    std::vector<CellPlan>& outcomes = arrays.outcomes;
    mode.assign(static_cast<size_t>(batch), kModeEmpty);
    outcomes.assign(static_cast<size_t>(batch), CellPlan::kUnsafe);
    Upload second(pinned_plan, plan_bytes);
    size_t off_plans = 0;
    StructurePlan<T>* plans = second.place<StructurePlan<T>>(static_cast<size_t>(batch), off_plans);
    auto build_plan = [&](int64_t b) {
        if (counts[b] != 0) {
            const int64_t images = geometry.image_begin[b + 1] - geometry.image_begin[b];
            bool cell = false;
            if (request.algorithm == TNR_CELL_LIST) {
                cell = true;
            } else if (request.algorithm == TNR_AUTO) {
                cell = counts[b] > brute_candidates_per_source() / std::max<int64_t>(images, 1);
            }
            mode[b] = cell ? kModeCell : kModeBrute;
        }
        StructurePlan<T>& plan = plans[b];
        std::memset(&plan, 0, sizeof(plan));
        plan.atom_begin = batch_ptr[b];
        plan.n_atoms = static_cast<int32_t>(counts[b]);
        plan.mode = mode[b];
        plan.image_begin = geometry.image_begin[b];
        plan.n_images = static_cast<int32_t>(geometry.image_begin[b + 1] - geometry.image_begin[b]);
        for (int a = 0; a < 3; ++a) plan.repeats[a] = static_cast<int32_t>(repeats_of(b, a));
        for (int k = 0; k < 9; ++k) plan.cell[k] = cell_t[9 * b + k];
        plan.cutoff_squared = static_cast<T>(request.cutoff * request.cutoff);
        plan.dims[0] = plan.dims[1] = plan.dims[2] = 1;
    };
    auto plan_cells = [&](int64_t b) {
        if (mode[b] == kModeCell) {
            outcomes[b] = plan_cell(plans[b], reductions[b], cell_t.data() + 9 * b,
                                    dual_of(b), request.cutoff);
        }
    };
    HostPool::instance().parallel_for(batch, 256, [&](int64_t begin, int64_t end) {
        for (int64_t b = begin; b < end; ++b) {
            build_plan(b);
            if (speculate) plan_cells(b);
        }
    });
    const bool any_cell = std::any_of(mode.begin(), mode.end(), [](int32_t m) { return m == kModeCell; });
    timer.host(10);  // plans built

    int64_t total_bins = 0;
    if (any_cell) {
        if (!speculate) {
            check_cuda(cudaMemcpyAsync(pinned_read, d_reductions, reduction_bytes,
                                       cudaMemcpyDeviceToHost, stream), "read extents");
            check_cuda(cudaMemcpyAsync(pinned_read + reduction_bytes, d_status,
                                       sizeof(uint32_t), cudaMemcpyDeviceToHost, stream), "read status");
            check_cuda(cudaStreamSynchronize(stream), "extents");
            reductions = reinterpret_cast<const Reduction<T>*>(pinned_read);
            uint32_t status = 0;
            std::memcpy(&status, pinned_read + reduction_bytes, sizeof(status));
            timer.host(3);  // extents read back
            check_status(status);
            HostPool::instance().parallel_for(batch, 256, [&](int64_t begin, int64_t end) {
                for (int64_t b = begin; b < end; ++b) plan_cells(b);
            });
        }
        for (int64_t b = 0; b < batch; ++b) {
            if (mode[b] != kModeCell) continue;
            StructurePlan<T>& plan = plans[b];
            const CellPlan outcome = outcomes[b];
            const int64_t bins = outcome == CellPlan::kReady
                ? int64_t{plan.dims[0]} * plan.dims[1] * plan.dims[2] : 0;
            if (outcome != CellPlan::kReady || total_bins + bins > kMaximumTotalBins) {
                require_search(request.algorithm != TNR_CELL_LIST || outcome == CellPlan::kPreferBrute,
                               kCannotSafely);
                plan.mode = mode[b] = kModeBrute;
                plan.dims[0] = plan.dims[1] = plan.dims[2] = 1;
                continue;
            }
            plan.bin_begin = total_bins;
            total_bins += bins;
        }
    }

    timer.host(11);  // bins laid out
    // ---- work lists -------------------------------------------------------
    std::vector<int32_t>& cell_structs = arrays.cell_structs;
    std::vector<int32_t>& brute_structs = arrays.brute_structs;
    std::vector<int64_t>& cell_prefix = arrays.cell_prefix;
    std::vector<int64_t>& brute_prefix = arrays.brute_prefix;
    cell_structs.clear();
    brute_structs.clear();
    cell_prefix.assign(1, 0);
    brute_prefix.assign(1, 0);
    for (int64_t b = 0; b < batch; ++b) {
        if (mode[b] == kModeCell) {
            cell_structs.push_back(static_cast<int32_t>(b));
            cell_prefix.push_back(cell_prefix.back() + counts[b]);
        } else if (mode[b] == kModeBrute) {
            brute_structs.push_back(static_cast<int32_t>(b));
            brute_prefix.push_back(brute_prefix.back() + counts[b]);
        }
    }
    const int64_t n_cell_atoms = cell_prefix.back();
    const int64_t n_brute_atoms = brute_prefix.back();
    std::vector<int64_t>& cell_bin_prefix = arrays.cell_bin_prefix;
    cell_bin_prefix.clear();
    for (int32_t b : cell_structs) cell_bin_prefix.push_back(plans[b].bin_begin);
    cell_bin_prefix.push_back(total_bins);
    const size_t off_cell_prefix = second.add(cell_prefix.data(), cell_prefix.size());
    const size_t off_cell_structs = second.add(cell_structs.data(), cell_structs.size());
    const size_t off_brute_prefix = second.add(brute_prefix.data(), brute_prefix.size());
    const size_t off_brute_structs = second.add(brute_structs.data(), brute_structs.size());
    const size_t off_cell_bins = second.add(cell_bin_prefix.data(), cell_bin_prefix.size());
    char* second_device = second.commit(workspace, stream);
    timer.host(4);  // plans uploaded
    auto* d_plans = reinterpret_cast<StructurePlan<T>*>(second_device + off_plans);

    // ---- cell list binning: histogram -> scan -> scatter ------------------
    unsigned long long* d_bin_start = nullptr;
    V4* d_ghost_pos = nullptr;
    int4* d_ghost_meta = nullptr;
    int32_t* d_source_list = nullptr;
    int32_t* d_source_bin = nullptr;
    uint32_t* d_mask_words = nullptr;
    unsigned long long* d_bin_word_start = nullptr;
    const int64_t scan_items = std::max<int64_t>(n_atoms, total_bins);
    void* d_scan_workspace = workspace.raw(scan_workspace_bytes(scan_items));
    BinArgs<T> bin_args{};
    bin_args.plans = d_plans;
    bin_args.cell_prefix = reinterpret_cast<const int64_t*>(second_device + off_cell_prefix);
    bin_args.cell_structs = reinterpret_cast<const int32_t*>(second_device + off_cell_structs);
    bin_args.n_cell = static_cast<int32_t>(cell_structs.size());
    bin_args.n_cell_atoms = n_cell_atoms;
    for (int32_t b : cell_structs) bin_args.max_images = std::max(bin_args.max_images, plans[b].n_images);
    bin_args.wraps = d_wraps;
    bin_args.wrapped = d_wrapped;
    bin_args.status = d_status;
    // Unsorted calls test each unordered pair once (cell-order output);
    // sorted calls search every source's full stencil.  Pair-once order keys
    // are 2 * source slot + 2 < 2^31.
    const bool pair_once = !request.sorted && n_cell_atoms < (int64_t{1} << 30) - 16;
    bin_args.pair_once = pair_once ? 1 : 0;
    const int64_t total_images = geometry.image_begin[batch];
    auto* d_image_shift = workspace.get<int4>(std::max<int64_t>(total_images, 1));
    auto* d_image_translation = workspace.get<V4>(std::max<int64_t>(total_images, 1));
    launch_image_table<T>(d_plans, batch, d_image_shift, d_image_translation, stream);
    check_launch("image table kernel");
    bin_args.image_shift = d_image_shift;
    bin_args.image_translation = d_image_translation;
    int32_t* d_bin_struct = nullptr;
    V4* d_ghost_orig = nullptr;
    if (n_cell_atoms > 0) {
        d_bin_struct = workspace.get<int32_t>(total_bins);
        launch_bin_struct<T>(reinterpret_cast<const int64_t*>(second_device + off_cell_bins),
                             bin_args.cell_structs, bin_args.n_cell, d_bin_struct, stream);
        check_launch("bin structure kernel");
        auto* d_bin_counts = workspace.get<unsigned long long>(total_bins);
        d_bin_start = workspace.get<unsigned long long>(total_bins + 1);
        auto* d_cursor = workspace.get<unsigned long long>(total_bins + 1);
        check_cuda(cudaMemsetAsync(d_bin_counts, 0, total_bins * sizeof(unsigned long long), stream),
                   "memset bins");
        bin_args.bin_counts = d_bin_counts;
        launch_bin(bin_args, false, stream);
        check_launch("bin histogram kernel");
        launch_scan_u64(d_bin_counts, total_bins, d_bin_start, d_cursor, d_scan_workspace, d_status,
                        stream);
        check_launch("bin scan kernel");
        // Bitmask words for the count pass -> write pass hand-off: per-bin
        // word counts, scanned into per-bin offsets.
        SearchArgs<T> words_args{};
        words_args.plans = d_plans;
        words_args.bin_start = d_bin_start;
        words_args.cell_bin_prefix = reinterpret_cast<const int64_t*>(second_device + off_cell_bins);
        words_args.cell_structs = bin_args.cell_structs;
        words_args.n_cell = bin_args.n_cell;
        words_args.n_bins = total_bins;
        words_args.bin_struct = d_bin_struct;
        words_args.n_sources = n_cell_atoms;
        words_args.pair_once = bin_args.pair_once;
        auto* d_bin_words = workspace.get<unsigned long long>(total_bins);
        d_bin_word_start = workspace.get<unsigned long long>(total_bins + 1);
        launch_stencil_words(words_args, d_bin_words, stream);
        check_launch("stencil words kernel");
        launch_scan_u64(d_bin_words, total_bins, d_bin_word_start, nullptr, d_scan_workspace,
                        d_status, stream);
        check_launch("mask scan kernel");
        // Ghost and bitmask sizes.  Bounds from the plans: a structure of n
        // atoms and I images places at most n (1 + (I - 1) / 2) copies
        // (pair-once; n I otherwise), and a source's stencil holds at most
        // its structure's copies.  Small calls allocate to those bounds and
        // skip the read-back; the kernels check the capacities.
        int64_t ghost_bound = 0, mask_bound = 0;
        for (int32_t b : cell_structs) {
            const int64_t images = plans[b].n_images;
            const int64_t copies = counts[b] * (pair_once ? 1 + (images - 1) / 2 : images);
            ghost_bound += copies;
            mask_bound += counts[b] * ((copies + 31) / 32);
        }
        const int64_t ghost_record_bytes = static_cast<int64_t>(sizeof(V4) + sizeof(int4)) +
            ((request.quantities & (TNR_Q_d | TNR_Q_D)) ? static_cast<int64_t>(sizeof(V4)) : 0);
        const bool bounded = ghost_bound < std::numeric_limits<int32_t>::max() &&
                             ghost_bound * ghost_record_bytes + mask_bound * 4 <= kBoundedWorkspaceBytes;
        int64_t ghosts = ghost_bound;
        unsigned long long mask_words = static_cast<unsigned long long>(mask_bound);
        if (!bounded) {
            unsigned long long packed_total = 0;
            check_cuda(cudaMemcpyAsync(pinned_read, d_bin_start + total_bins, sizeof(packed_total),
                                       cudaMemcpyDeviceToHost, stream), "read ghost total");
            check_cuda(cudaMemcpyAsync(pinned_read + 8, d_bin_word_start + total_bins, sizeof(mask_words),
                                       cudaMemcpyDeviceToHost, stream), "read mask words");
            check_cuda(cudaStreamSynchronize(stream), "ghost total");
            std::memcpy(&packed_total, pinned_read, sizeof(packed_total));
            std::memcpy(&mask_words, pinned_read + 8, sizeof(mask_words));
            timer.host(5);  // ghost and mask totals read back
            require_search(mask_words < (1ull << 32), "cell-list candidate bitmask exceeds uint32 indexing");
            // Ghost slots: the sources' zero images, then the other copies.
            const int64_t sources = static_cast<int64_t>(packed_total >> 32);
            ghosts = sources + static_cast<int64_t>(packed_total & 0xffffffffull);
            require_search(sources == n_cell_atoms && ghosts < std::numeric_limits<int32_t>::max(),
                           "cell-list image copies exceed int32 indexing");
        }
        d_mask_words = workspace.get<uint32_t>(std::max<unsigned long long>(mask_words, 1));
        if (bounded) {
            launch_capacity_check(d_bin_word_start + total_bins, mask_words, d_status, stream);
            check_launch("capacity check kernel");
        }
        d_ghost_pos = workspace.get<V4>(ghosts);
        d_ghost_meta = workspace.get<int4>(ghosts);
        if (request.quantities & (TNR_Q_d | TNR_Q_D)) d_ghost_orig = workspace.get<V4>(ghosts);
        bin_args.ghost_capacity = ghosts;
        d_source_list = workspace.get<int32_t>(n_cell_atoms);
        d_source_bin = workspace.get<int32_t>(n_cell_atoms);
        bin_args.bin_counts = d_cursor;
        bin_args.ghost_pos = d_ghost_pos;
        bin_args.ghost_meta = d_ghost_meta;
        bin_args.ghost_orig = d_ghost_orig;
        bin_args.positions = static_cast<const T*>(request.positions);
        bin_args.source_list = d_source_list;
        bin_args.source_bin = d_source_bin;
        launch_bin(bin_args, true, stream);
        check_launch("bin scatter kernel");
    }
    timer.mark(2);

    // ---- count pass -> scan -> exact E -------------------------------------
    auto* d_counts = workspace.get<uint32_t>(n_atoms);
    auto* d_pair_start = workspace.get<int64_t>(n_atoms + 1);
    check_cuda(cudaMemsetAsync(d_counts, 0, n_atoms * sizeof(uint32_t), stream), "memset counts");
    SearchArgs<T> search{};
    search.positions = static_cast<const T*>(request.positions);
    search.atom_struct = d_atom_struct;
    search.wraps = d_wraps;
    search.wrapped = d_wrapped;
    search.plans = d_plans;
    search.bin_start = d_bin_start;
    search.ghost_pos = d_ghost_pos;
    search.ghost_meta = d_ghost_meta;
    search.source_list = d_source_list;
    search.source_bin = d_source_bin;
    search.n_sources = n_cell_atoms;
    search.image_shift = bin_args.image_shift;
    search.mask_words = d_mask_words;
    search.bin_word_start = d_bin_word_start;
    search.cell_bin_prefix = reinterpret_cast<const int64_t*>(second_device + off_cell_bins);
    search.cell_structs = reinterpret_cast<const int32_t*>(second_device + off_cell_structs);
    search.n_cell = static_cast<int32_t>(cell_structs.size());
    search.n_bins = total_bins;
    search.bin_struct = d_bin_struct;
    search.ghost_orig = d_ghost_orig;
    search.source_order = request.sorted ? 0 : 1;
    search.pair_once = bin_args.pair_once;
    search.brute_prefix = reinterpret_cast<const int64_t*>(second_device + off_brute_prefix);
    search.brute_structs = reinterpret_cast<const int32_t*>(second_device + off_brute_structs);
    search.n_brute = static_cast<int32_t>(brute_structs.size());
    search.n_brute_atoms = n_brute_atoms;
    // Brute-force structures are staged whole in shared memory when every one
    // of them fits (always under 'auto', whose brute structures have at most
    // 256 candidates per source).
    {
        int64_t largest = 0;
        for (int32_t b : brute_structs) {
            const int64_t images = geometry.image_begin[b + 1] - geometry.image_begin[b];
            largest = std::max<int64_t>(largest, counts[b] * (3 * static_cast<int64_t>(sizeof(T)) + 12) +
                                                     images * 12);
        }
        search.brute_tile_bytes = largest <= 48 * 1024 ? static_cast<int32_t>((largest + 15) / 16 * 16) : 0;
    }
    search.counts = d_counts;
    search.pair_start = d_pair_start;
    search.index_offset = request.index_offset;
    search.status = d_status;
    search.half_list = request.half_list ? 1 : 0;
    search.include_self = request.include_self ? 1 : 0;
    if (n_cell_atoms) {
        launch_cell_search(search, false, stream);
        check_launch("cell count kernel");
    }
    if (n_brute_atoms) {
        launch_brute_search(search, false, stream);
        check_launch("brute count kernel");
    }
    timer.mark(3);
    // The pair-count scan is queued before the host's geometry check so
    // that the device does not wait for it.
    launch_scan_counts(d_counts, n_atoms, d_pair_start, d_scan_workspace, d_status, stream);
    check_launch("pair scan kernel");
    timer.mark(4);
    timer.host(6);  // count pass and scan launched
    if (speculate) {
        // While the search runs: the exact geometry (the reference's long-
        // double arithmetic) must give the same T duals and image ranges as
        // the device, else the call is repeated on the host path.  Its input
        // errors are raised by that repeat, in the reference's order.
        cell64.assign(cell_t.begin(), cell_t.end());
        const PeriodicGeometry exact =
            build_geometry(cell64.data(), pbc.data(), counts.data(), batch, request.cutoff);
        for (int64_t b = 0; b < batch; ++b) {
            for (int a = 0; a < 3; ++a) {
                if (exact.repeats[3 * b + a] != repeats_of(b, a)) throw SpeculationFailed{};
            }
            if (exact.image_begin[b + 1] != geometry.image_begin[b + 1]) throw SpeculationFailed{};
        }
        // The duals may differ in their last bits (the device rounds in
        // double); what the search used of them is the wraps, which the
        // device now recomputes with the exact duals (status word 2).
        T* exact_duals = reinterpret_cast<T*>(pinned_prepare);
        for (int64_t k = 0; k < 9 * batch; ++k) exact_duals[k] = static_cast<T>(exact.duals[k]);
        T* d_exact_duals = workspace.get<T>(9 * batch);
        const cudaStream_t check_stream = side ? side->stream : stream;
        if (side) check_cuda(cudaStreamWaitEvent(side->stream, side->fork, 0), "fork wait");
        check_cuda(cudaMemcpyAsync(d_exact_duals, exact_duals, 9 * batch * sizeof(T),
                                   cudaMemcpyHostToDevice, check_stream), "upload exact duals");
        launch_verify_wraps<T>(static_cast<const T*>(request.positions), n_atoms, d_atom_struct,
                               d_exact_duals, d_wraps, d_status + 2, check_stream);
        check_launch("wrap check kernel");
        if (side) {
            // Join before the status read-back (and before the workspace, the
            // exact duals included, is released on the main stream).
            check_cuda(cudaEventRecord(side->join, side->stream), "join record");
            check_cuda(cudaStreamWaitEvent(stream, side->join, 0), "join wait");
        }
    }
    check_cuda(cudaMemcpyAsync(pinned_read, d_pair_start + n_atoms, sizeof(int64_t),
                               cudaMemcpyDeviceToHost, stream), "read pair total");
    check_cuda(cudaMemcpyAsync(pinned_read + sizeof(int64_t), d_status, 3 * sizeof(uint32_t),
                               cudaMemcpyDeviceToHost, stream), "read status");
    check_cuda(cudaStreamSynchronize(stream), "pair total");
    int64_t n_pairs = 0;
    uint32_t status = 0, wraps_differ = 0;
    std::memcpy(&n_pairs, pinned_read, sizeof(n_pairs));
    std::memcpy(&status, pinned_read + sizeof(int64_t), sizeof(status));
    std::memcpy(&wraps_differ, pinned_read + sizeof(int64_t) + 2 * sizeof(uint32_t), sizeof(wraps_differ));
    if (speculate && wraps_differ) throw SpeculationFailed{};
    timer.host(7);  // pair total read back
    check_status(status);
    require_search(n_pairs >= 0, "neighbor-list output exceeds the int64 range");

    // ---- exact-size outputs and the write pass -----------------------------
    result.n_pairs = n_pairs;
    if (n_pairs == 0) return;
    const uint32_t q = request.quantities;
    const size_t e = static_cast<size_t>(n_pairs);
    if (q & TNR_Q_I) result.i = workspace.output<int64_t>(e);
    if (q & TNR_Q_J) result.j = workspace.output<int64_t>(e);
    if (q & TNR_Q_P) result.P = workspace.output<int64_t>(2 * e);
    if (q & TNR_Q_S) result.S = workspace.output<int32_t>(3 * e);
    if (q & TNR_Q_d) result.d = workspace.output<T>(e);
    if (q & TNR_Q_D) result.D = workspace.output<T>(3 * e);
    if (q & TNR_Q_EDGE) result.edge_index = workspace.output<int64_t>(2 * e);
    search.out_i = result.edge_index ? result.edge_index : result.i;
    search.out_j = result.edge_index ? result.edge_index + e : result.j;
    search.out_P = result.P;
    search.out_S = result.S;
    search.out_d = static_cast<T*>(result.d);
    search.out_D = static_cast<T*>(result.D);
    {
        // Full pair-once lists write both orientations of a pair as adjacent
        // rows with 8- and 16-byte stores when every output is aligned for
        // them (each source's row count is even, and include_self adds one
        // row to each of the 32 sources of a write group, so every group
        // starts at an even row).
        auto aligned = [](const void* p, uintptr_t a) {
            return reinterpret_cast<uintptr_t>(p) % a == 0;
        };
        search.paired_rows = (pair_once && !request.half_list && aligned(search.out_i, 16) &&
                              aligned(search.out_j, 16) && aligned(search.out_P, 16) &&
                              aligned(search.out_S, 8) && aligned(search.out_d, 2 * sizeof(T)) &&
                              aligned(search.out_D, 2 * sizeof(T))) ? 1 : 0;
    }
    timer.mark(5);
    if (q != 0) {
        if (n_cell_atoms) {
            launch_cell_search(search, true, stream);
            check_launch("cell write kernel");
        }
        if (n_brute_atoms) {
            launch_brute_search(search, true, stream);
            check_launch("brute write kernel");
        }
    }
    timer.mark(6);
    timer.host(8);  // write pass launched
    timer.finish();
}

// Verlet-skin filter: count pass (ballot words, per-block counts), scan of
// the block counts, exact-size outputs, write pass.
template <typename T>
void run_filter(const tnr_request& request, const tnr_candidates& candidates,
                Workspace& workspace, cudaStream_t stream, tnr_result& result) {
    const int64_t m = candidates.n_candidates;
    result.n_pairs = 0;
    if (m == 0) return;
    require_input(candidates.pairs != nullptr && candidates.shifts != nullptr,
                  "candidate pairs and shifts are required");
    FilterArgs<T> args{};
    args.positions = static_cast<const T*>(request.positions);
    args.batch_ptr = request.batch_ptr;
    args.batch = request.n_structures;
    args.cell = static_cast<const T*>(request.cell);
    args.pairs = candidates.pairs;
    args.shifts = candidates.shifts;
    args.n_candidates = m;
    args.index_offset = request.index_offset;
    args.cutoff_squared = static_cast<T>(request.cutoff * request.cutoff);
    const int64_t blocks = (m + kFilterThreads - 1) / kFilterThreads;
    args.keep_words = workspace.get<uint32_t>((m + 31) / 32);
    args.block_counts = workspace.get<uint32_t>(blocks);
    auto* block_start = workspace.get<int64_t>(blocks + 1);
    void* scan_workspace = workspace.raw(scan_workspace_bytes(blocks));
    launch_filter(args, false, stream);
    check_launch("filter count kernel");
    launch_scan_counts(args.block_counts, blocks, block_start, scan_workspace, nullptr, stream);
    check_launch("filter scan kernel");
    int64_t* total = reinterpret_cast<int64_t*>(g_pinned.reserve(64));
    check_cuda(cudaMemcpyAsync(total, block_start + blocks, sizeof(int64_t), cudaMemcpyDeviceToHost,
                               stream), "read filter total");
    check_cuda(cudaStreamSynchronize(stream), "filter total");
    const int64_t n_pairs = *total;
    result.n_pairs = n_pairs;
    if (n_pairs == 0) return;
    const uint32_t q = request.quantities;
    const size_t e = static_cast<size_t>(n_pairs);
    if (q & TNR_Q_I) result.i = workspace.output<int64_t>(e);
    if (q & TNR_Q_J) result.j = workspace.output<int64_t>(e);
    if (q & TNR_Q_P) result.P = workspace.output<int64_t>(2 * e);
    if (q & TNR_Q_S) result.S = workspace.output<int32_t>(3 * e);
    if (q & TNR_Q_d) result.d = workspace.output<T>(e);
    if (q & TNR_Q_D) result.D = workspace.output<T>(3 * e);
    if (q & TNR_Q_EDGE) result.edge_index = workspace.output<int64_t>(2 * e);
    args.block_start = block_start;
    args.out_i = result.edge_index ? result.edge_index : result.i;
    args.out_j = result.edge_index ? result.edge_index + e : result.j;
    args.out_P = result.P;
    args.out_S = result.S;
    args.out_d = static_cast<T*>(result.d);
    args.out_D = static_cast<T*>(result.D);
    launch_filter(args, true, stream);
    check_launch("filter write kernel");
}

// Runs the call, speculating on the device geometry where that pays off.  A
// failed speculation (or any input or search error raised under it) repeats
// the call on the host path, whose results and errors are the reference's.
template <typename T>
void run_call(const tnr_request& request, Workspace& workspace, cudaStream_t stream,
              tnr_result& result) {
    if (speculate_geometry<T>(request)) {
        try {
            run<T>(request, workspace, stream, result, true);
            return;
        } catch (const SpeculationFailed&) {
        } catch (const InputError&) {
        } catch (const SearchError&) {
        }
        check_cuda(cudaStreamSynchronize(stream), "speculative geometry");
        workspace.release_outputs();
        result = tnr_result{};
    }
    run<T>(request, workspace, stream, result, false);
}

void set_message(char* message, size_t length, const char* text) {
    if (message == nullptr || length == 0) return;
    std::strncpy(message, text, length - 1);
    message[length - 1] = '\0';
}

}  // namespace
}  // namespace tnr

extern "C" {

int tnr_neighbor_list(const tnr_request* request, const tnr_allocator* allocator,
                      tnr_stream stream_handle, tnr_result* result, char* message,
                      size_t message_length) {
    using namespace tnr;
    if (request == nullptr || result == nullptr) {
        set_message(message, message_length, "request and result must not be null");
        return TNR_INPUT_ERROR;
    }
    *result = tnr_result{};
    g_launches = 0;
    const int64_t launches_before = launched_kernels();
    tnr_allocator chosen{nullptr, default_allocate, default_release};
    if (allocator && allocator->allocate && allocator->release) chosen = *allocator;
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_handle);
    Workspace workspace(chosen, stream);
    try {
        require_input(std::isfinite(request->cutoff) && request->cutoff > 0,
                      "cutoff must be finite and positive");
        require_input(request->n_atoms >= 0 && request->n_structures >= 0,
                      "batch_ptr must have shape (B + 1,)");
        require_input(request->n_atoms < (int64_t{1} << 31),
                      "the current implementation supports fewer than 2^31 atoms");
        require_input(request->algorithm >= TNR_AUTO && request->algorithm <= TNR_CELL_LIST,
                      "algorithm must be 'auto', 'brute_force', or 'cell_list'");
        require_input(request->dtype == TNR_FLOAT32 || request->dtype == TNR_FLOAT64,
                      "positions must have dtype float32 or float64");
        require_input(!(request->quantities & TNR_Q_EDGE) ||
                          !(request->quantities & (TNR_Q_I | TNR_Q_J)),
                      "edge_index cannot be combined with i or j");
        tnr_result local{};
        if (request->dtype == TNR_FLOAT32) {
            run_call<float>(*request, workspace, stream, local);
        } else {
            run_call<double>(*request, workspace, stream, local);
        }
        workspace.keep_outputs();
        *result = local;
        g_launches = launched_kernels() - launches_before;
        return TNR_OK;
    } catch (const InputError& error) {
        workspace.release_outputs();
        set_message(message, message_length, error.what());
        return TNR_INPUT_ERROR;
    } catch (const SearchError& error) {
        workspace.release_outputs();
        set_message(message, message_length, error.what());
        return TNR_SEARCH_ERROR;
    } catch (const std::bad_alloc&) {
        workspace.release_outputs();
        set_message(message, message_length, "device allocation failed");
        return TNR_ALLOC_ERROR;
    } catch (const std::exception& error) {
        workspace.release_outputs();
        set_message(message, message_length, error.what());
        return TNR_CUDA_ERROR;
    }
}

const char* tnr_version(void) { return "0.1.0"; }

int64_t tnr_last_launch_count(void) { return tnr::g_launches; }

int tnr_filter_pairs(const tnr_request* request, const tnr_candidates* candidates,
                     const tnr_allocator* allocator, tnr_stream stream_handle, tnr_result* result,
                     char* message, size_t message_length) {
    using namespace tnr;
    if (request == nullptr || candidates == nullptr || result == nullptr) {
        set_message(message, message_length, "request, candidates and result must not be null");
        return TNR_INPUT_ERROR;
    }
    *result = tnr_result{};
    g_launches = 0;
    const int64_t launches_before = launched_kernels();
    tnr_allocator chosen{nullptr, default_allocate, default_release};
    if (allocator && allocator->allocate && allocator->release) chosen = *allocator;
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_handle);
    Workspace workspace(chosen, stream);
    try {
        require_input(std::isfinite(request->cutoff) && request->cutoff > 0,
                      "cutoff must be finite and positive");
        require_input(request->n_structures >= 1 && request->batch_ptr != nullptr,
                      "batch_ptr must have shape (B + 1,)");
        require_input(candidates->n_candidates >= 0, "the candidate count must not be negative");
        require_input(request->dtype == TNR_FLOAT32 || request->dtype == TNR_FLOAT64,
                      "positions must have dtype float32 or float64");
        require_input(!(request->quantities & TNR_Q_EDGE) ||
                          !(request->quantities & (TNR_Q_I | TNR_Q_J)),
                      "edge_index cannot be combined with i or j");
        tnr_result local{};
        if (request->dtype == TNR_FLOAT32) {
            run_filter<float>(*request, *candidates, workspace, stream, local);
        } else {
            run_filter<double>(*request, *candidates, workspace, stream, local);
        }
        workspace.keep_outputs();
        *result = local;
        g_launches = launched_kernels() - launches_before;
        return TNR_OK;
    } catch (const InputError& error) {
        workspace.release_outputs();
        set_message(message, message_length, error.what());
        return TNR_INPUT_ERROR;
    } catch (const std::bad_alloc&) {
        workspace.release_outputs();
        set_message(message, message_length, "device allocation failed");
        return TNR_ALLOC_ERROR;
    } catch (const std::exception& error) {
        workspace.release_outputs();
        set_message(message, message_length, error.what());
        return TNR_CUDA_ERROR;
    }
}

int tnr_last_host_times(double* times_ms, int capacity) {
    const int count = std::min(capacity, tnr::kHostMarks);
    for (int k = 0; k < count; ++k) times_ms[k] = tnr::g_host_ms[k];
    return count;
}

int tnr_last_phase_times(float* times_ms, int capacity) {
    const int count = std::min(capacity, 6);
    for (int k = 0; k < count; ++k) times_ms[k] = tnr::g_phase_ms[k];
    return count;
}

}  // extern "C"
