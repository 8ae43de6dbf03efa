// tnr_neighbor_list_static: a variant of the brute-force search that never
// allocates device memory.
//
// Who needs it: callers that cannot call cudaMalloc at the moment they want a
// neighbor list -- a framework that forbids allocation on its hot path, or an
// embedding whose device memory is owned entirely by another allocator (a
// memory pool that has reserved the GPU), where a cudaMalloc would fail or
// fragment that pool.  They pass their input and output buffers; every
// intermediate array lives in one fixed-size device array owned by this
// library (kStaticScratchBytes, below), which each GPU that loads the library
// keeps until the process exits.
//
// Limits and rules:
//   * at most kStaticMaxAtoms atoms and kStaticMaxStructures structures per
//     call; larger requests are rejected with TNR_INPUT_ERROR;
//   * every candidate pair is enumerated (brute force), so this is meant for
//     small systems; `algorithm` in the request is ignored;
//   * the first call on a device looks up the scratch array's device address
//     (cudaGetSymbolAddress) with that device current; make that first call
//     before any stream capture;
//   * the call waits for `stream` (it reads the pair count back) and issues
//     all its copies and kernels on `stream`;
//   * all calls share the one array and it keeps the previous call's
//     contents, so calls that overlap on the GPU (different streams or host
//     threads at the same time) race; serialise them.
#include "tonari_b200.h"

#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "tnr_geometry.h"
#include "tnr_launch.h"
#include "tnr_plan.h"

namespace tnr {
namespace {

constexpr int64_t kStaticMaxAtoms = int64_t{1} << 16;
constexpr int64_t kStaticMaxStructures = 4096;
constexpr size_t kStaticScratchBytes = size_t{8} << 20;  // 8 MiB per device
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_address[kMaxDevices] = {};

// Device address of the scratch array for the current device.
void* scratch_address(int device) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (g_scratch_address[device] == nullptr) {
        void* pointer = nullptr;
        const cudaError_t error =
            cudaGetSymbolAddress(&pointer, g_static_scratch);
        if (error != cudaSuccess) {
            throw SearchError(std::string("static scratch set-up failed: ") +
                              cudaGetErrorString(error));
        }
        g_scratch_address[device] = pointer;
    }
    return g_scratch_address[device];
}

// Bump carving of the scratch array; throws when a request does not fit.
class Carver {
public:
    explicit Carver(void* base) : base_(static_cast<char*>(base)) {}
    template <typename U>
    U* take(size_t count) {
        const size_t offset = (used_ + 255) / 256 * 256;
        const size_t bytes = std::max<size_t>(count * sizeof(U), 16);
        if (offset + bytes > kStaticScratchBytes) {
            throw InputError("the request does not fit the static scratch space of "
                             "tnr_neighbor_list_static (8 MiB per device)");
        }
        used_ = offset + bytes;
        return reinterpret_cast<U*>(base_ + offset);
    }

private:
    char* base_;
    size_t used_ = 0;
};

void check(cudaError_t error, const char* what) {
    if (error != cudaSuccess) throw SearchError(std::string(what) + ": " + cudaGetErrorString(error));
}

template <typename T>
Reduction<T> neutral() {
    Reduction<T> r;
    std::memset(&r, 0, sizeof(r));
    return r;  // extents are unused by the brute-force path
}

template <typename T>
void run_static(const tnr_request& request, cudaStream_t stream, int64_t capacity,
                tnr_result& result) {
    using V4 = typename std::conditional<std::is_same<T, float>::value, float4, double4>::type;
    const int64_t n_atoms = request.n_atoms;
    const int64_t batch = request.n_structures;
    require_input(n_atoms <= kStaticMaxAtoms && batch <= kStaticMaxStructures,
                  "tnr_neighbor_list_static accepts at most 65536 atoms and 4096 structures");

    // Host metadata: caller's host mirrors, else reads on `stream` into
    // ordinary host memory, complete once the stream has been synchronised.
    std::vector<int64_t> batch_ptr(static_cast<size_t>(batch + 1));
    std::vector<T> cell(static_cast<size_t>(9 * batch));
    std::vector<uint8_t> pbc(static_cast<size_t>(3 * batch));
    if (request.batch_ptr_host && request.cell_host && request.pbc_host) {
        std::memcpy(batch_ptr.data(), request.batch_ptr_host, batch_ptr.size() * sizeof(int64_t));
        std::memcpy(cell.data(), request.cell_host, cell.size() * sizeof(T));
        std::memcpy(pbc.data(), request.pbc_host, pbc.size());
    } else {
        check(cudaMemcpyAsync(batch_ptr.data(), request.batch_ptr,
                              batch_ptr.size() * sizeof(int64_t), cudaMemcpyDeviceToHost, stream),
              "read batch_ptr");
        if (batch) {
            check(cudaMemcpyAsync(cell.data(), request.cell, cell.size() * sizeof(T),
                                  cudaMemcpyDeviceToHost, stream), "read cell");
            check(cudaMemcpyAsync(pbc.data(), request.pbc, pbc.size(), cudaMemcpyDeviceToHost,
                                  stream), "read pbc");
        }
        check(cudaStreamSynchronize(stream), "read metadata");
    }
    require_input(batch_ptr[0] == 0, "batch_ptr must start at zero");
    require_input(batch_ptr[batch] == n_atoms, "batch_ptr must end at N_total");
    std::vector<int64_t> counts(static_cast<size_t>(batch));
    for (int64_t b = 0; b < batch; ++b) {
        require_input(batch_ptr[b + 1] >= batch_ptr[b], "batch_ptr must be nondecreasing");
        counts[b] = batch_ptr[b + 1] - batch_ptr[b];
    }
    for (uint8_t& flag : pbc) flag = flag ? 1 : 0;
    std::vector<double> cell64(cell.begin(), cell.end());
    const PeriodicGeometry geometry =
        build_geometry(cell64.data(), pbc.data(), counts.data(), batch, request.cutoff);
    result.n_pairs = 0;
    if (n_atoms == 0) return;

    int device = 0;
    check(cudaGetDevice(&device), "cudaGetDevice");
    require_search(device >= 0 && device < kMaxDevices, "device index out of range");
    Carver carve(scratch_address(device));

    // Host-side tables, uploaded into the scratch array.
    std::vector<PrepareStructure<T>> prepare(static_cast<size_t>(batch));
    std::vector<StructurePlan<T>> plans(static_cast<size_t>(batch));
    std::vector<int32_t> brute_structs;
    std::vector<int64_t> brute_prefix{0};
    for (int64_t b = 0; b < batch; ++b) {
        prepare[b].atom_begin = batch_ptr[b];
        prepare[b].atom_end = batch_ptr[b + 1];
        StructurePlan<T>& plan = plans[b];
        std::memset(&plan, 0, sizeof(plan));
        plan.atom_begin = batch_ptr[b];
        plan.n_atoms = static_cast<int32_t>(counts[b]);
        plan.mode = counts[b] ? kModeBrute : kModeEmpty;
        plan.image_begin = geometry.image_begin[b];
        plan.n_images = static_cast<int32_t>(geometry.image_begin[b + 1] - geometry.image_begin[b]);
        for (int a = 0; a < 3; ++a) plan.repeats[a] = geometry.repeats[3 * b + a];
        for (int k = 0; k < 9; ++k) {
            prepare[b].cell[k] = cell[9 * b + k];
            prepare[b].dual[k] = static_cast<T>(geometry.duals[9 * b + k]);
            plan.cell[k] = cell[9 * b + k];
        }
        plan.cutoff_squared = static_cast<T>(request.cutoff * request.cutoff);
        plan.dims[0] = plan.dims[1] = plan.dims[2] = 1;
        if (counts[b]) {
            brute_structs.push_back(static_cast<int32_t>(b));
            brute_prefix.push_back(brute_prefix.back() + counts[b]);
        }
    }
    std::vector<Reduction<T>> reductions(static_cast<size_t>(batch), neutral<T>());
    std::vector<int4> image_shift(static_cast<size_t>(std::max<int64_t>(geometry.image_begin[batch], 1)));
    for (int64_t b = 0; b < batch; ++b) {
        const int32_t* r = geometry.repeats.data() + 3 * b;
        int64_t k = geometry.image_begin[b];
        if (geometry.image_begin[b + 1] == k) continue;
        for (int32_t x = -r[0]; x <= r[0]; ++x)
            for (int32_t y = -r[1]; y <= r[1]; ++y)
                for (int32_t z = -r[2]; z <= r[2]; ++z) image_shift[k++] = make_int4(x, y, z, 0);
    }

    auto* d_prepare = carve.take<PrepareStructure<T>>(prepare.size());
    auto* d_plans = carve.take<StructurePlan<T>>(plans.size());
    auto* d_reductions = carve.take<Reduction<T>>(reductions.size());
    auto* d_brute_structs = carve.take<int32_t>(brute_structs.size());
    auto* d_brute_prefix = carve.take<int64_t>(brute_prefix.size());
    auto* d_image_shift = carve.take<int4>(image_shift.size());
    auto* d_atom_struct = carve.take<int32_t>(n_atoms);
    auto* d_wraps = carve.take<int32_t>(3 * n_atoms);
    auto* d_wrapped = carve.take<V4>(n_atoms);
    auto* d_counts = carve.take<uint32_t>(n_atoms);
    auto* d_pair_start = carve.take<int64_t>(n_atoms + 1);
    auto* d_status = carve.take<uint32_t>(4);
    void* d_scan = carve.take<unsigned char>(scan_workspace_bytes(n_atoms));

    // Uploads are ordered on `stream` before the kernels that read them.  The
    // host vectors stay alive until the stream is synchronised for the pair
    // total below, after the last upload has completed.
    auto upload = [stream](void* destination, const void* source, size_t bytes) {
        if (bytes == 0) return;
        check(cudaMemcpyAsync(destination, source, bytes, cudaMemcpyHostToDevice, stream),
              "upload");
    };
    upload(d_prepare, prepare.data(), prepare.size() * sizeof(prepare[0]));
    upload(d_plans, plans.data(), plans.size() * sizeof(plans[0]));
    upload(d_reductions, reductions.data(), reductions.size() * sizeof(reductions[0]));
    upload(d_brute_structs, brute_structs.data(), brute_structs.size() * sizeof(int32_t));
    upload(d_brute_prefix, brute_prefix.data(), brute_prefix.size() * sizeof(int64_t));
    upload(d_image_shift, image_shift.data(), image_shift.size() * sizeof(int4));
    // Scratch keeps the previous call's bytes: clear what must start at zero.
    check(cudaMemsetAsync(d_status, 0, 4 * sizeof(uint32_t), stream), "clear status");
    check(cudaMemsetAsync(d_counts, 0, n_atoms * sizeof(uint32_t), stream), "clear counts");

    PrepareArgs<T> prepare_args{static_cast<const T*>(request.positions), n_atoms,
                                request.batch_ptr, batch, d_prepare, d_atom_struct, d_wraps,
                                d_wrapped, d_reductions, d_status};
    launch_prepare(prepare_args, stream);
    check(cudaGetLastError(), "prepare kernel");

    SearchArgs<T> search{};
    search.positions = static_cast<const T*>(request.positions);
    search.atom_struct = d_atom_struct;
    search.wraps = d_wraps;
    search.wrapped = d_wrapped;
    search.plans = d_plans;
    search.brute_prefix = d_brute_prefix;
    search.image_shift = d_image_shift;
    search.brute_structs = d_brute_structs;
    search.n_brute = static_cast<int32_t>(brute_structs.size());
    search.n_brute_atoms = brute_prefix.back();
    search.counts = d_counts;
    search.pair_start = d_pair_start;
    search.index_offset = request.index_offset;
    search.status = d_status;
    search.half_list = request.half_list ? 1 : 0;
    search.include_self = request.include_self ? 1 : 0;
    launch_brute_search(search, false, stream);
    check(cudaGetLastError(), "count kernel");
    launch_scan_counts(d_counts, n_atoms, d_pair_start, d_scan, d_status, stream);
    check(cudaGetLastError(), "scan kernel");

    int64_t n_pairs = 0;
    uint32_t status = 0;
    check(cudaMemcpyAsync(&n_pairs, d_pair_start + n_atoms, sizeof(n_pairs), cudaMemcpyDeviceToHost,
                          stream), "read pair total");
    check(cudaMemcpyAsync(&status, d_status, sizeof(status), cudaMemcpyDeviceToHost, stream),
          "read status");
    check(cudaStreamSynchronize(stream), "pair total");
    require_search(!(status & kStatusNonFinite), "positions must contain only finite values");
    require_search(!(status & kStatusWrapRange),
                   "atom representatives require periodic wraps outside the int32 range");
    require_search(!(status & kStatusShiftRange),
                   "a cell shift required by the cutoff pairs exceeds the int32 output range");
    require_search(!(status & (kStatusCapacity | kStatusCountRange)),
                   "the static neighbor-list search failed an internal check");
    result.n_pairs = n_pairs;
    if (n_pairs > capacity) {
        throw std::length_error("the output buffers hold fewer pairs than the neighbor list has; "
                                "n_pairs reports the size needed");
    }
    if (n_pairs == 0) return;
    const uint32_t q = request.quantities;
    search.out_i = (q & TNR_Q_I) ? result.i : nullptr;
    search.out_j = (q & TNR_Q_J) ? result.j : nullptr;
    search.out_P = (q & TNR_Q_P) ? result.P : nullptr;
    search.out_S = (q & TNR_Q_S) ? result.S : nullptr;
    search.out_d = (q & TNR_Q_d) ? static_cast<T*>(result.d) : nullptr;
    search.out_D = (q & TNR_Q_D) ? static_cast<T*>(result.D) : nullptr;
    launch_brute_search(search, true, stream);
    check(cudaGetLastError(), "write kernel");
}

void copy_message(char* message, size_t length, const char* text) {
    if (message == nullptr || length == 0) return;
    std::strncpy(message, text, length - 1);
    message[length - 1] = '\0';
}

}  // namespace
}  // namespace tnr

extern "C" int tnr_neighbor_list_static(const tnr_request* request, tnr_stream stream_handle,
                                        int64_t pair_capacity, tnr_result* result,
                                        char* message, size_t message_length) {
    using namespace tnr;
    if (request == nullptr || result == nullptr) {
        copy_message(message, message_length, "request and result must not be null");
        return TNR_INPUT_ERROR;
    }
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_handle);
    try {
        require_input(std::isfinite(request->cutoff) && request->cutoff > 0,
                      "cutoff must be finite and positive");
        require_input(request->n_atoms >= 0 && request->n_structures >= 0,
                      "batch_ptr must have shape (B + 1,)");
        require_input(request->dtype == TNR_FLOAT32 || request->dtype == TNR_FLOAT64,
                      "positions must have dtype float32 or float64");
        require_input(!(request->quantities & TNR_Q_EDGE),
                      "edge_index is not offered by the allocation-free entry point");
        require_input(pair_capacity >= 0, "pair_capacity must be nonnegative");
        const uint32_t q = request->quantities;
        require_input(!(q & TNR_Q_I) || result->i, "result->i must be set when i is requested");
        require_input(!(q & TNR_Q_J) || result->j, "result->j must be set when j is requested");
        require_input(!(q & TNR_Q_P) || result->P, "result->P must be set when P is requested");
        require_input(!(q & TNR_Q_S) || result->S, "result->S must be set when S is requested");
        require_input(!(q & TNR_Q_d) || result->d, "result->d must be set when d is requested");
        require_input(!(q & TNR_Q_D) || result->D, "result->D must be set when D is requested");
        if (request->dtype == TNR_FLOAT32) {
            run_static<float>(*request, stream, pair_capacity, *result);
        } else {
            run_static<double>(*request, stream, pair_capacity, *result);
        }
        return TNR_OK;
    } catch (const InputError& error) {
        copy_message(message, message_length, error.what());
        return TNR_INPUT_ERROR;
    } catch (const SearchError& error) {
        copy_message(message, message_length, error.what());
        return TNR_SEARCH_ERROR;
    } catch (const std::length_error& error) {
        copy_message(message, message_length, error.what());
        return TNR_ALLOC_ERROR;
    } catch (const std::exception& error) {
        copy_message(message, message_length, error.what());
        return TNR_CUDA_ERROR;
    }
}
