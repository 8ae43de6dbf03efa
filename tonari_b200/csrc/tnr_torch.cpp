// PyTorch custom op `torch.ops.tonari_b200.neighbor_list` over the C ABI.
//
// Schema mirrors the reference provider entry point
// (tonari csrc/torch/bindings_cuda.cpp:59-68) plus the fused-output selection:
//   neighbor_list(positions, batch_ptr, cell, pbc, cutoff, half_list,
//                 include_self, algorithm, sorted, quantities, index_offset)
//     -> [i, j, P, S, d, D]   (tensors not selected by `quantities` are empty)
// Input checks follow bindings_cuda.cpp:69-92.  Device buffers come from the
// PyTorch caching allocator on the current stream through the C ABI's
// allocator callback, so outputs are ordinary tensors owned by PyTorch.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>
#include <torch/torch.h>

#include <string>
#include <unordered_map>
#include <vector>

#include "tonari_b200.h"

namespace {

struct TorchAllocator {
    at::Device device;
    std::unordered_map<void*, at::Tensor> live;
};

void* torch_allocate(void* context, size_t bytes, tnr_stream) {
    auto* self = static_cast<TorchAllocator*>(context);
    try {
        at::Tensor buffer = at::empty({static_cast<int64_t>(bytes)},
                                      at::TensorOptions().dtype(at::kByte).device(self->device));
        void* pointer = buffer.data_ptr();
        self->live.emplace(pointer, std::move(buffer));
        return pointer;
    } catch (...) {
        return nullptr;
    }
}

void torch_release(void* context, void* pointer, tnr_stream) {
    static_cast<TorchAllocator*>(context)->live.erase(pointer);
}

int32_t parse_algorithm(const std::string& name) {
    if (name == "auto") return TNR_AUTO;
    if (name == "brute_force") return TNR_BRUTE_FORCE;
    if (name == "cell_list") return TNR_CELL_LIST;
    TORCH_CHECK_VALUE(false, "algorithm must be 'auto', 'brute_force', or 'cell_list'");
}

uint32_t parse_quantities(const std::string& quantities) {
    uint32_t mask = 0;
    for (char q : quantities) {
        switch (q) {
            case 'i': mask |= TNR_Q_I; break;
            case 'j': mask |= TNR_Q_J; break;
            case 'P': mask |= TNR_Q_P; break;
            case 'S': mask |= TNR_Q_S; break;
            case 'd': mask |= TNR_Q_d; break;
            case 'D': mask |= TNR_Q_D; break;
            case 'E': mask |= TNR_Q_EDGE; break;  // (2,E) graph layout
            default: TORCH_CHECK_VALUE(false, "unsupported quantities: '", std::string(1, q), "'");
        }
    }
    return mask;
}

at::Tensor take(TorchAllocator& allocator, void* pointer, at::ScalarType dtype,
                std::vector<int64_t> shape, const at::TensorOptions& options) {
    if (pointer == nullptr) {
        return at::empty(shape, options.dtype(dtype));
    }
    auto found = allocator.live.find(pointer);
    TORCH_CHECK(found != allocator.live.end(), "tonari_b200: unknown output buffer");
    at::Tensor bytes = std::move(found->second);
    allocator.live.erase(found);
    int64_t elements = 1;
    for (int64_t s : shape) elements *= s;
    const int64_t size = elements * static_cast<int64_t>(c10::elementSize(dtype));
    return bytes.narrow(0, 0, size).view(dtype).view(shape);
}

std::vector<at::Tensor> neighbor_list_cuda(const at::Tensor& positions, const at::Tensor& batch_ptr,
                                           const at::Tensor& cell, const at::Tensor& pbc,
                                           double cutoff, bool half_list, bool include_self,
                                           std::string algorithm, bool sorted,
                                           std::string quantities, int64_t index_offset) {
    TORCH_CHECK(positions.is_cuda(), "positions must be a CUDA tensor");
    TORCH_CHECK(batch_ptr.is_cuda() && cell.is_cuda() && pbc.is_cuda(),
                "all inputs must be CUDA tensors");
    TORCH_CHECK(positions.is_contiguous() && batch_ptr.is_contiguous() && cell.is_contiguous() &&
                    pbc.is_contiguous(),
                "all inputs must be contiguous");
    TORCH_CHECK(positions.dim() == 2 && positions.size(1) == 3,
                "positions must have shape (N_total, 3)");
    TORCH_CHECK(batch_ptr.dim() == 1 && batch_ptr.numel() > 0,
                "batch_ptr must be int64 with shape (B + 1,)");
    TORCH_CHECK(cell.sizes() == at::IntArrayRef({batch_ptr.numel() - 1, 3, 3}),
                "cell must have shape (B, 3, 3)");
    TORCH_CHECK(pbc.sizes() == at::IntArrayRef({batch_ptr.numel() - 1, 3}),
                "pbc must have shape (B, 3)");
    TORCH_CHECK(positions.scalar_type() == cell.scalar_type(),
                "cell and positions must have the same dtype");
    TORCH_CHECK(positions.scalar_type() == at::kFloat || positions.scalar_type() == at::kDouble,
                "positions must have dtype float32 or float64");
    TORCH_CHECK(batch_ptr.scalar_type() == at::kLong, "batch_ptr must have dtype int64");
    TORCH_CHECK(pbc.scalar_type() == at::kBool, "pbc must have dtype bool");
    TORCH_CHECK(batch_ptr.device() == positions.device() && cell.device() == positions.device() &&
                    pbc.device() == positions.device(),
                "positions, cell, pbc, and batch_ptr must be on the same device");

    const c10::cuda::CUDAGuard guard(positions.device());
    const cudaStream_t stream = at::cuda::getCurrentCUDAStream(positions.get_device()).stream();

    tnr_request request{};
    request.dtype = positions.scalar_type() == at::kDouble ? TNR_FLOAT64 : TNR_FLOAT32;
    request.n_atoms = positions.size(0);
    request.n_structures = batch_ptr.numel() - 1;
    request.positions = positions.data_ptr();
    request.batch_ptr = batch_ptr.data_ptr<int64_t>();
    request.cell = cell.data_ptr();
    request.pbc = reinterpret_cast<const uint8_t*>(pbc.data_ptr<bool>());
    request.cutoff = cutoff;
    request.half_list = half_list;
    request.include_self = include_self;
    request.algorithm = parse_algorithm(algorithm);
    request.quantities = parse_quantities(quantities);
    request.index_offset = index_offset;
    request.sorted = sorted;

    TorchAllocator context{positions.device(), {}};
    tnr_allocator allocator{&context, torch_allocate, torch_release};
    tnr_result result{};
    char message[512] = {0};
    const int status = tnr_neighbor_list(&request, &allocator, reinterpret_cast<tnr_stream>(stream),
                                         &result, message, sizeof(message));
    TORCH_CHECK_VALUE(status != TNR_INPUT_ERROR, message);
    TORCH_CHECK(status == TNR_OK, message);

    const int64_t e = result.n_pairs;
    const auto options = positions.options();
    const auto real = positions.scalar_type();
    std::vector<at::Tensor> outputs;
    outputs.push_back(take(context, result.i, at::kLong, {result.i ? e : 0}, options));
    outputs.push_back(take(context, result.j, at::kLong, {result.j ? e : 0}, options));
    outputs.push_back(take(context, result.P, at::kLong, {result.P ? e : 0, 2}, options));
    outputs.push_back(take(context, result.S, at::kInt, {result.S ? e : 0, 3}, options));
    outputs.push_back(take(context, result.d, real, {result.d ? e : 0}, options));
    outputs.push_back(take(context, result.D, real, {result.D ? e : 0, 3}, options));
    outputs.push_back(take(context, result.edge_index, at::kLong, {2, result.edge_index ? e : 0}, options));
    return outputs;
}

std::vector<at::Tensor> collect(TorchAllocator& context, const tnr_result& result,
                                const at::TensorOptions& options, at::ScalarType real) {
    const int64_t e = result.n_pairs;
    std::vector<at::Tensor> outputs;
    outputs.push_back(take(context, result.i, at::kLong, {result.i ? e : 0}, options));
    outputs.push_back(take(context, result.j, at::kLong, {result.j ? e : 0}, options));
    outputs.push_back(take(context, result.P, at::kLong, {result.P ? e : 0, 2}, options));
    outputs.push_back(take(context, result.S, at::kInt, {result.S ? e : 0, 3}, options));
    outputs.push_back(take(context, result.d, real, {result.d ? e : 0}, options));
    outputs.push_back(take(context, result.D, real, {result.D ? e : 0, 3}, options));
    outputs.push_back(take(context, result.edge_index, at::kLong, {2, result.edge_index ? e : 0}, options));
    return outputs;
}

// Verlet-skin reuse: the candidate pairs (from a list built with cutoff +
// skin) whose exact distance at the current positions is below `cutoff`.
std::vector<at::Tensor> filter_pairs_cuda(const at::Tensor& positions, const at::Tensor& batch_ptr,
                                          const at::Tensor& cell, const at::Tensor& pairs,
                                          const at::Tensor& shifts, double cutoff,
                                          std::string quantities, int64_t index_offset) {
    TORCH_CHECK(positions.is_cuda() && batch_ptr.is_cuda() && cell.is_cuda() && pairs.is_cuda() &&
                    shifts.is_cuda(),
                "all inputs must be CUDA tensors");
    TORCH_CHECK(positions.is_contiguous() && batch_ptr.is_contiguous() && cell.is_contiguous() &&
                    pairs.is_contiguous() && shifts.is_contiguous(),
                "all inputs must be contiguous");
    TORCH_CHECK(positions.dim() == 2 && positions.size(1) == 3, "positions must have shape (N_total, 3)");
    TORCH_CHECK(batch_ptr.dim() == 1 && batch_ptr.numel() > 1 && batch_ptr.scalar_type() == at::kLong,
                "batch_ptr must be int64 with shape (B + 1,)");
    TORCH_CHECK(cell.sizes() == at::IntArrayRef({batch_ptr.numel() - 1, 3, 3}) &&
                    cell.scalar_type() == positions.scalar_type(),
                "cell must have shape (B, 3, 3) and the dtype of positions");
    TORCH_CHECK(pairs.dim() == 2 && pairs.size(1) == 2 && pairs.scalar_type() == at::kLong,
                "pairs must be int64 with shape (M, 2)");
    TORCH_CHECK(shifts.dim() == 2 && shifts.size(1) == 3 && shifts.size(0) == pairs.size(0) &&
                    shifts.scalar_type() == at::kInt,
                "shifts must be int32 with shape (M, 3)");
    TORCH_CHECK(positions.scalar_type() == at::kFloat || positions.scalar_type() == at::kDouble,
                "positions must have dtype float32 or float64");
    const c10::cuda::CUDAGuard guard(positions.device());
    const cudaStream_t stream = at::cuda::getCurrentCUDAStream(positions.get_device()).stream();
    tnr_request request{};
    request.dtype = positions.scalar_type() == at::kDouble ? TNR_FLOAT64 : TNR_FLOAT32;
    request.n_atoms = positions.size(0);
    request.n_structures = batch_ptr.numel() - 1;
    request.positions = positions.data_ptr();
    request.batch_ptr = batch_ptr.data_ptr<int64_t>();
    request.cell = cell.data_ptr();
    request.cutoff = cutoff;
    request.quantities = parse_quantities(quantities);
    request.index_offset = index_offset;
    tnr_candidates candidates{pairs.data_ptr<int64_t>(), shifts.data_ptr<int32_t>(), pairs.size(0)};
    TorchAllocator context{positions.device(), {}};
    tnr_allocator allocator{&context, torch_allocate, torch_release};
    tnr_result result{};
    char message[512] = {0};
    const int status = tnr_filter_pairs(&request, &candidates, &allocator,
                                        reinterpret_cast<tnr_stream>(stream), &result, message,
                                        sizeof(message));
    TORCH_CHECK_VALUE(status != TNR_INPUT_ERROR, message);
    TORCH_CHECK(status == TNR_OK, message);
    return collect(context, result, positions.options(), positions.scalar_type());
}

}  // namespace

TORCH_LIBRARY(tonari_b200, m) {
    m.def(
        "filter_pairs(Tensor positions, Tensor batch_ptr, Tensor cell, Tensor pairs, "
        "Tensor shifts, float cutoff, str quantities, int index_offset) -> Tensor[]");
    m.def(
        "neighbor_list(Tensor positions, Tensor batch_ptr, Tensor cell, Tensor pbc, float cutoff, "
        "bool half_list, bool include_self, str algorithm, bool sorted, str quantities, "
        "int index_offset) -> Tensor[]");
}

TORCH_LIBRARY_IMPL(tonari_b200, CUDA, m) {
    m.impl("neighbor_list", &neighbor_list_cuda);
    m.impl("filter_pairs", &filter_pairs_cuda);
}
