#include "executor.hpp"

#include <algorithm>
#include <functional>
#include <climits>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <set>

namespace nvcr_sm100 {

// ---------------------------------------------------------------- internals

struct Executor::IntegerConv {
    int weight_limbs{1}, activation_limbs{1}, activation_bits{8};
    int channels{0}, c_pad{0};   // source channels; K channels per tap padded to a multiple of 16
    int k_real{0}, k_padded{0};  // K = k_taps * c_pad, and rounded up to 128-byte blocks
    // Few source channels: a prepass stages each output position's whole
    // receptive field (channels * taps values in the node's k order), and the
    // fused kernel runs a 1x1 conv over that grid, `window` being 1x1 then.
    bool fields{false};
    int k_taps{1};
    kernels::Window window{1, 1, 1, 1, 0, 0};
    int n_tile{0}, n_tiles{0};
    int out_channels{0};  // logical output channels of the step (halved by chunk-add)
    bool chunk_add{false};
    float* scales{nullptr};
    float* bias{nullptr};
    long long* row_terms{nullptr};
    void* allocation{nullptr};
    long long column_high_factor{0}, column_low_factor{0};
    // K order and weight matrices per source type ([0] FP32, [1] FP16): the
    // channels per halo load make 128-byte records where the padding allows.
    struct Layout {
        int group{0}, groups{0};
        std::int8_t* b_high{nullptr};
        std::int8_t* b_low{nullptr};
        CUtensorMap b_high_map{};
        CUtensorMap b_low_map{};
    };
    Layout layouts[2];
    // Shared-memory ring depths fixed at create time, and the bytes one halo
    // buffer may take.
    int taps{1};
    int a_stages{2}, b_stages{4};
    bool b_resident{false};  // one N tile whose K blocks all stay in shared memory
    int halo_budget{0};
    int producer_sets{1};    // 2: eight producer warps on alternate tiles, four epilogue warps
    // Direct path (w8a8, stride-1 windows up to 3x3, or receptive fields): the
    // activations are quantised per pixel into int8 [pixels][c8] and loaded by
    // TMA; K is tap-major, k = tap * c8 + c, in k_block-byte stages. A
    // multi-tap window falls back to the quantise-on-load path above when its
    // pixels' exponents differ.
    bool direct{false};
    int c8{0};
    int k_block{0}, c_blocks{0}, direct_k_blocks{0};
    int direct_a_stages{0}, direct_b_stages{0}, direct_group{1};
    bool direct_b_resident{false};
    // Every scale and bias finite (the direct conv's vector stores need no NaN
    // handling), and every accumulator below 2^22 in magnitude (127 times the
    // largest row sum of |q|: exact float conversion by integer addition).
    bool finite_columns{true};
    bool small_accumulators{false};
    // Window exponents e for which y * 2^e is exact for every y = RN(x * scale)
    // of the conv (|x| < 2^31, no overflow, nothing subnormal), so that
    // RN(RN(y * 2^e) + bias) is one fused multiply-add; empty when lo > hi.
    int fma_lo{1}, fma_hi{0};
    // Ring depths for tiles of two patches sharing each weight block (deep-K
    // convs with k_block 128 and at most 256 columns); 0 when not prepared.
    int pair_a_stages{0}, pair_b_stages{0}, pair_group{1};
    bool pair_b_resident{false};
    // Row halos (multi-column windows with 128-byte K blocks): patches of one
    // output row of 128 positions whose A stages are single halo rows; ring
    // depths for one patch and for pairs per tile (0 when not prepared).
    int row_bytes{0};
    int row_a_stages{0}, row_b_stages{0};
    bool row_b_resident{false};
    int row_pair_a_stages{0}, row_pair_b_stages{0};
    bool row_pair_b_resident{false};
    void* direct_allocation{nullptr};
    CUtensorMap direct_b_map{};
};

enum class StepKind { generic, integer_conv, chunk_add };

struct Executor::Step {
    StepKind kind{StepKind::generic};
    std::size_t node{0};
    std::vector<std::size_t> reads;
    std::size_t output{0};
    // integer conv
    int conv{-1};
    std::size_t source{0};
    bool fused_im2col{false};
    kernels::Window window{1, 1, 1, 1, 0, 0};
    bool wsilu{false};
    float wsilu_scale{0.0f};
    bool chunk_add{false};
    std::optional<std::size_t> residual;
    int d2s_block{0};  // the output goes through depth_to_space(d2s_block)
};

struct PlannedConv {
    bool source_half{false};       // the conv reads an FP16 program input directly
    bool source_staged{false};     // the source tensor is stored channel-innermost already
    std::size_t staged{0};         // arena offset of the channel-innermost copy of the source
    std::size_t pixel_max{0};      // arena offset of the per-input-pixel maxima
    int positions{0};
    int patch_h{0}, patch_w{0}, tiles_y{0}, tiles_x{0};
    int halo_rows{0}, halo_box_w{0}, halo_bytes{0};
    int halo_buffers{2};  // halo ring depth: what the conv's halo region holds, up to 8
    CUtensorMap halo_map{};
    const void* halo_base{nullptr};  // staged address halo_map was encoded for
    // Direct path: the int8 per-pixel copy, the fallback word (multi-tap
    // windows), the patch shape of the direct conv and its activation map.
    std::size_t quantised{0};
    std::size_t fallback{0};
    int d_patch_h{0}, d_patch_w{0}, d_tiles_y{0}, d_tiles_x{0};
    int m_tiles{1};  // patches per tile sharing each weight block
    bool row_halo{false};  // one-row patches of 128 positions with row-halo A stages
    CUtensorMap a_map{};
    const void* a_base{nullptr};
};

struct Executor::Plan {
    Boundary boundary{Boundary::host};
    std::vector<Extent> extents;
    std::vector<std::size_t> offsets;  // per tensor id, npos when not materialised
    std::vector<PlannedConv> convs;    // per step
    std::size_t arena_bytes{0};
};

namespace {

constexpr std::size_t npos = std::numeric_limits<std::size_t>::max();
constexpr std::size_t alignment = 1024;

std::size_t align_up(std::size_t value, std::size_t to) { return (value + to - 1) / to * to; }

// A conv with few channels (channels * taps <= 64, more than one tap) stages
// each output position's whole receptive field and runs as a 1x1 conv over it.
bool receptive_field_staging(const kernels::Window& window, int in_channels) {
    return window.kernel_h * window.kernel_w > 1 && in_channels <= 64;
}
int round_up(int value, int to) { return (value + to - 1) / to * to; }

Error cuda_error(const char* what, cudaError_t status) {
    return fail(Code::backend_error, std::string(what) + ": " + cudaGetErrorString(status));
}

// First-fit allocator over one arena: offsets only, no device memory.
class OffsetAllocator {
public:
    std::size_t allocate(std::size_t bytes) {
        bytes = align_up(std::max<std::size_t>(bytes, 1), alignment);
        for (auto it = free_.begin(); it != free_.end(); ++it) {
            if (it->second >= bytes) {
                const std::size_t offset = it->first;
                const std::size_t remaining = it->second - bytes;
                free_.erase(it);
                if (remaining > 0) free_.insert({offset + bytes, remaining});
                sizes_[offset] = bytes;
                return offset;
            }
        }
        const std::size_t offset = top_;
        top_ += bytes;
        sizes_[offset] = bytes;
        return offset;
    }
    void release(std::size_t offset) {
        auto found = sizes_.find(offset);
        if (found == sizes_.end()) return;
        std::size_t start = offset;
        std::size_t size = found->second;
        sizes_.erase(found);
        // Coalesce with free neighbours.
        auto next = free_.lower_bound({start, 0});
        if (next != free_.end() && next->first == start + size) {
            size += next->second;
            next = free_.erase(next);
        }
        if (next != free_.begin()) {
            auto previous = std::prev(next);
            if (previous->first + previous->second == start) {
                start = previous->first;
                size += previous->second;
                free_.erase(previous);
            }
        }
        if (start + size == top_) {
            top_ = start;
        } else {
            free_.insert({start, size});
        }
    }
    std::size_t peak() const { return peak_ = std::max(peak_, top_), peak_; }
    void note_peak() { peak_ = std::max(peak_, top_); }

private:
    std::set<std::pair<std::size_t, std::size_t>> free_;
    std::map<std::size_t, std::size_t> sizes_;
    std::size_t top_{0};
    mutable std::size_t peak_{0};
};

const TensorView* find_view(const std::vector<TensorView>& views, const std::string& name) {
    for (const auto& view : views) {
        if (view.name == name) return &view;
    }
    return nullptr;
}

// Halo of a patch of output pixels: input rows and the TMA box width in
// elements (a multiple of `align`, wide enough for a start rounded down to it).
const char* op_name(Op op) {
    switch (op) {
    case Op::conv: return "conv";
    case Op::mul: return "mul";
    case Op::add: return "add";
    case Op::mul_scalar: return "mul_scalar";
    case Op::sigmoid: return "sigmoid";
    case Op::slice_channels: return "slice_channels";
    case Op::depth_to_space: return "depth_to_space";
    case Op::scale_channels: return "scale_channels";
    case Op::clamp: return "clamp";
    case Op::concat: return "concat";
    case Op::crop: return "crop";
    case Op::space_to_depth: return "space_to_depth";
    case Op::im2col: return "im2col";
    }
    return "?";
}

}  // namespace

// ---------------------------------------------------------------- creation

Result<std::unique_ptr<Executor>> Executor::create(Program program, cudaStream_t stream) {
    std::unique_ptr<Executor> executor(new Executor());
    executor->program_ = std::move(program);
    int device = 0;
    cudaError_t status = cudaGetDevice(&device);
    int major = 0;
    int minor = 0;
    if (status == cudaSuccess) status = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    if (status == cudaSuccess) status = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
    if (status == cudaSuccess) {
        status = cudaDeviceGetAttribute(&executor->sm_count_, cudaDevAttrMultiProcessorCount, device);
    }
    if (status != cudaSuccess) return cuda_error("cudaDeviceGetAttribute", status);
    executor->device_ = device;
    if (major != 10 || minor != 0) {
        return fail(Code::incompatible_target,
                    std::string(intconv_profile) + " on this provider needs an sm_100 (B200-class) GPU");
    }
    if (stream != nullptr) {
        executor->stream_ = stream;
    } else {
        status = cudaStreamCreateWithFlags(&executor->stream_, cudaStreamNonBlocking);
        if (status != cudaSuccess) return cuda_error("cudaStreamCreate", status);
        executor->owns_stream_ = true;
    }
    auto prepared = executor->prepare();
    if (!prepared) return prepared.error();
    return executor;
}

Executor::~Executor() {
    if (stream_ != nullptr) cudaStreamSynchronize(stream_);
    clear_graphs();
    for (auto& conv : convs_) {
        cudaFree(conv.allocation);
        cudaFree(conv.direct_allocation);
    }
    for (auto event : events_) cudaEventDestroy(event);
    cudaFree(arena_);
    cudaFree(weights_);
    cudaFree(status_);
    if (fallback_stream_ != nullptr) cudaStreamDestroy(fallback_stream_);
    if (owns_stream_ && stream_ != nullptr) cudaStreamDestroy(stream_);
}

Status Executor::prepare() {
    const std::size_t bytes = std::max<std::size_t>(program_.weights.size(), 1) * sizeof(float);
    cudaError_t status = cudaMalloc(reinterpret_cast<void**>(&weights_), bytes);
    if (status != cudaSuccess) return cuda_error("cudaMalloc weights", status);
    status = cudaMemcpy(weights_, program_.weights.data(), program_.weights.size() * sizeof(float),
                        cudaMemcpyHostToDevice);
    if (status != cudaSuccess) return cuda_error("cudaMemcpy weights", status);
    status = cudaMalloc(reinterpret_cast<void**>(&status_), sizeof(unsigned int));
    if (status != cudaSuccess) return cuda_error("cudaMalloc status", status);
    status = cudaMemset(status_, 0, sizeof(unsigned int));
    if (status != cudaSuccess) return cuda_error("cudaMemset status", status);
    plan_fusions();
    for (std::size_t index = 0; index < steps_.size(); ++index) {
        if (steps_[index].kind != StepKind::integer_conv) continue;
        auto prepared = prepare_integer_conv(index);
        if (!prepared) return prepared;
    }
    // Which program inputs and outputs device runs may leave in the caller's buffers.
    const std::size_t tensor_count = program_.tensor_names.size();
    std::vector<std::vector<std::size_t>> readers(tensor_count);
    for (std::size_t s = 0; s < steps_.size(); ++s) {
        for (const auto id : steps_[s].reads) readers[id].push_back(s);
    }
    std::vector<int> output_uses(tensor_count, 0);
    for (const auto id : program_.outputs) ++output_uses[id];
    input_conv_only_.assign(program_.inputs.size(), false);
    for (std::size_t slot = 0; slot < program_.inputs.size(); ++slot) {
        const auto id = program_.inputs[slot];
        bool only = output_uses[id] == 0;
        for (const auto s : readers[id]) {
            const Step& step = steps_[s];
            only = only && step.kind == StepKind::integer_conv && step.source == id &&
                !(step.residual && *step.residual == id);
        }
        input_conv_only_[slot] = only;
    }
    // Staged tensors, stored channel-innermost ([H][W][c_pad] FP32, then the
    // per-pixel maxima) instead of NCHW. A tensor qualifies when it is no program
    // input or output and its producer is an integer conv (without a
    // depth_to_space fold) or a channel-innermost depthwise 3x3 whose input is
    // staged, and every reader is an integer conv reading it as a multi-tap or
    // pointwise source (not a receptive-field source) or as the residual, or a
    // channel-innermost depthwise 3x3 whose output is staged. The largest such
    // set: start from every candidate and drop violators until none is left.
    auto staged_depthwise = [&](const Step& st) {
        if (st.kind != StepKind::generic) return false;
        const Node& n = program_.nodes[st.node];
        const int c_pad = round_up(n.out_channels, 16);
        return n.op == Op::conv && n.depthwise && n.kernel[0] == 3 && n.kernel[1] == 3 && n.stride[0] == 1 &&
            n.stride[1] == 1 && n.pads[0] == 1 && n.pads[1] == 1 && n.pads[2] == 1 && n.pads[3] == 1 &&
            n.in_channels == n.out_channels && (c_pad == 128 || c_pad == 256);
    };
    std::vector<std::ptrdiff_t> produced_by(tensor_count, -1);
    for (std::size_t s = 0; s < steps_.size(); ++s) produced_by[steps_[s].output] = static_cast<std::ptrdiff_t>(s);
    staged_tensor_.assign(tensor_count, false);
    for (std::size_t id = 0; id < tensor_count; ++id) {
        const auto s = produced_by[id];
        if (s < 0 || output_uses[id] != 0 || readers[id].empty()) continue;
        if (std::find(program_.inputs.begin(), program_.inputs.end(), id) != program_.inputs.end()) continue;
        const Step& producer = steps_[static_cast<std::size_t>(s)];
        staged_tensor_[id] = (producer.kind == StepKind::integer_conv && producer.d2s_block == 0) ||
            staged_depthwise(producer);
    }
    for (bool changed = true; changed;) {
        changed = false;
        for (std::size_t id = 0; id < tensor_count; ++id) {
            if (!staged_tensor_[id]) continue;
            const Step& producer = steps_[static_cast<std::size_t>(produced_by[id])];
            bool ok = producer.kind == StepKind::integer_conv || staged_tensor_[producer.reads[0]];
            for (const auto r : readers[id]) {
                const Step& reader = steps_[r];
                if (reader.kind == StepKind::integer_conv) {
                    if (reader.source == id &&
                        receptive_field_staging(reader.window, program_.nodes[reader.node].in_channels)) {
                        ok = false;
                    }
                } else if (!(staged_depthwise(reader) && staged_tensor_[reader.output])) {
                    ok = false;
                }
            }
            if (!ok) {
                staged_tensor_[id] = false;
                changed = true;
            }
        }
    }
    output_step_.assign(program_.outputs.size(), -1);
    for (std::size_t slot = 0; slot < program_.outputs.size(); ++slot) {
        const auto id = program_.outputs[slot];
        if (output_uses[id] != 1 || !readers[id].empty()) continue;
        for (std::size_t s = 0; s < steps_.size(); ++s) {
            if (steps_[s].kind == StepKind::integer_conv && steps_[s].output == id) {
                output_step_[slot] = static_cast<std::ptrdiff_t>(s);
            }
        }
    }
    return Ok{};
}

// Folds node patterns into single steps. Only tensors that no other node reads
// and that are not program outputs are folded away, so every observable tensor
// keeps its bits; the arithmetic per element is unchanged by folding.
void Executor::plan_fusions() {
    const auto& nodes = program_.nodes;
    const std::size_t tensor_count = program_.tensor_names.size();
    std::vector<int> readers(tensor_count, 0);
    std::vector<std::ptrdiff_t> producer(tensor_count, -1);
    std::vector<bool> is_output(tensor_count, false);
    for (std::size_t i = 0; i < nodes.size(); ++i) {
        for (std::size_t slot = 0; slot < nodes[i].input_count; ++slot) ++readers[nodes[i].inputs[slot]];
        producer[nodes[i].output] = static_cast<std::ptrdiff_t>(i);
    }
    for (const auto id : program_.outputs) is_output[id] = true;
    auto private_tensor = [&](std::size_t id, int expected) { return readers[id] == expected && !is_output[id]; };
    auto same_pair = [](const Node& node, std::size_t a, std::size_t b) {
        return (node.inputs[0] == a && node.inputs[1] == b) || (node.inputs[0] == b && node.inputs[1] == a);
    };
    // nodes[at..at+2] = slice(source, 0, C/2), slice(source, C/2, C), add of the two.
    auto chunk_add_at = [&](std::size_t at, std::size_t source) {
        if (at + 2 >= nodes.size()) return false;
        const auto& first = nodes[at];
        const auto& second = nodes[at + 1];
        const auto& sum = nodes[at + 2];
        const auto channels = program_.tensor_channels[source];
        return channels % 2 == 0 && first.op == Op::slice_channels && first.inputs[0] == source &&
            second.op == Op::slice_channels && second.inputs[0] == source && first.begin == 0 &&
            first.end == channels / 2 && second.begin == channels / 2 && second.end == channels &&
            sum.op == Op::add && sum.input_count == 2 && same_pair(sum, first.output, second.output) &&
            first.output != second.output && private_tensor(first.output, 1) && private_tensor(second.output, 1);
    };

    std::vector<bool> absorbed(nodes.size(), false);
    std::vector<std::ptrdiff_t> im2col_of(nodes.size(), -1);
    for (std::size_t i = 0; i < nodes.size(); ++i) {
        if (!is_integer_pointwise(nodes[i])) continue;
        const auto input = nodes[i].inputs[0];
        const auto j = producer[input];
        if (j >= 0 && nodes[static_cast<std::size_t>(j)].op == Op::im2col && private_tensor(input, 1)) {
            im2col_of[i] = j;
            absorbed[static_cast<std::size_t>(j)] = true;
        }
    }

    steps_.clear();
    for (std::size_t i = 0; i < nodes.size(); ++i) {
        if (absorbed[i]) continue;
        const auto& node = nodes[i];
        Step step;
        step.node = i;
        if (is_integer_pointwise(node)) {
            step.kind = StepKind::integer_conv;
            step.source = node.inputs[0];
            if (im2col_of[i] >= 0) {
                const auto& cols = nodes[static_cast<std::size_t>(im2col_of[i])];
                step.fused_im2col = true;
                step.source = cols.inputs[0];
                step.window = kernels::Window{cols.kernel[0], cols.kernel[1], cols.stride[0], cols.stride[1],
                                              cols.pads[0], cols.pads[1]};
            }
            std::size_t out = node.output;
            std::size_t last = i;
            if (i + 3 < nodes.size()) {
                const auto& scale = nodes[i + 1];
                const auto& gate = nodes[i + 2];
                const auto& product = nodes[i + 3];
                if (scale.op == Op::mul_scalar && scale.inputs[0] == out && gate.op == Op::sigmoid &&
                    gate.inputs[0] == scale.output && product.op == Op::mul && product.input_count == 2 &&
                    same_pair(product, gate.output, out) && gate.output != out && private_tensor(out, 2) &&
                    private_tensor(scale.output, 1) && private_tensor(gate.output, 1)) {
                    step.wsilu = true;
                    step.wsilu_scale = scale.scalar;
                    out = product.output;
                    last = i + 3;
                }
            }
            if (last + 3 < nodes.size() && private_tensor(out, 2) && chunk_add_at(last + 1, out)) {
                step.chunk_add = true;
                out = nodes[last + 3].output;
                last += 3;
            }
            if (last + 1 < nodes.size() && nodes[last + 1].op == Op::add && nodes[last + 1].input_count == 2 &&
                private_tensor(out, 1)) {
                const auto& sum = nodes[last + 1];
                const std::size_t other = sum.inputs[0] == out ? sum.inputs[1]
                    : (sum.inputs[1] == out ? sum.inputs[0] : out);
                if (other != out && producer[other] < static_cast<std::ptrdiff_t>(i)) {
                    step.residual = other;
                    out = sum.output;
                    last += 1;
                }
            }
            if (last + 1 < nodes.size() && nodes[last + 1].op == Op::depth_to_space &&
                nodes[last + 1].inputs[0] == out && nodes[last + 1].block >= 1 && private_tensor(out, 1)) {
                step.d2s_block = nodes[last + 1].block;
                out = nodes[last + 1].output;
                last += 1;
            }
            for (std::size_t folded = i + 1; folded <= last; ++folded) absorbed[folded] = true;
            step.output = out;
            step.reads.push_back(step.source);
            if (step.residual) step.reads.push_back(*step.residual);
        } else if (node.op == Op::slice_channels && chunk_add_at(i, node.inputs[0])) {
            step.kind = StepKind::chunk_add;
            step.source = node.inputs[0];
            step.output = nodes[i + 2].output;
            step.reads.push_back(step.source);
            absorbed[i + 1] = true;
            absorbed[i + 2] = true;
        } else {
            step.kind = StepKind::generic;
            step.output = node.output;
            for (std::size_t slot = 0; slot < node.input_count; ++slot) step.reads.push_back(node.inputs[slot]);
        }
        steps_.push_back(std::move(step));
    }
}

// Quantises one integer conv's weights into int8 limb matrices
// [n_tiles * n_tile][k_padded] (K contiguous, zero padded) with per-row scale,
// bias and exact row term, and encodes their TMA maps.
Status Executor::prepare_integer_conv(std::size_t step_index) {
    Step& step = steps_[step_index];
    const Node& node = program_.nodes[step.node];
    IntegerConv conv;
    conv.weight_limbs = node.weight_bits == 16 ? 2 : 1;
    conv.activation_limbs = node.activation_bits == 16 ? 2 : 1;
    conv.activation_bits = node.activation_bits;
    const int taps = step.window.kernel_h * step.window.kernel_w;
    if (taps <= 0 || node.in_channels % taps != 0) return fail(Code::internal_error, "integer conv window mismatch");
    conv.taps = taps;
    conv.channels = node.in_channels / taps;
    conv.fields = receptive_field_staging(step.window, node.in_channels);
    conv.k_taps = conv.fields ? 1 : taps;
    conv.window = conv.fields ? kernels::Window{1, 1, 1, 1, 0, 0} : step.window;
    conv.c_pad = round_up(conv.fields ? conv.channels * taps : conv.channels, 16);
    conv.k_real = conv.k_taps * conv.c_pad;
    if (conv.k_real > 65536) {
        return fail(Code::invalid_argument, "integer conv reduction length above 65536 is not supported");
    }
    conv.k_padded = round_up(conv.k_real, 128);
    conv.chunk_add = step.chunk_add;
    const int rows = node.out_channels;
    const int accumulators = 1 + ((conv.weight_limbs == 2 || conv.activation_limbs == 2) ? 1 : 0) +
        ((conv.weight_limbs == 2 && conv.activation_limbs == 2) ? 1 : 0);
    const int max_tile = accumulators == 3 ? 128 : 256;
    if (conv.chunk_add) {
        const int pairs = rows / 2;
        conv.n_tiles = (2 * pairs + max_tile - 1) / max_tile;
        conv.n_tile = round_up((pairs + conv.n_tiles - 1) / conv.n_tiles, 16) * 2;
        conv.out_channels = pairs;
    } else {
        conv.n_tiles = (rows + max_tile - 1) / max_tile;
        conv.n_tile = round_up((rows + conv.n_tiles - 1) / conv.n_tiles, 16);
        conv.out_channels = rows;
    }
    const int n_padded = conv.n_tiles * conv.n_tile;
    // Channels per halo load: 128-byte records (64 FP16 or 32 FP32 channels)
    // when they divide the padded channels, else the largest power of two that does.
    for (int half = 0; half < 2; ++half) {
        int group = half ? 64 : 32;
        while (conv.c_pad % group != 0) group /= 2;
        conv.layouts[half].group = group;
    }
    // Smallest halo buffer over the patch shapes for a channel group.
    auto smallest_halo = [&](int group, int element) {
        int best = INT_MAX;
        for (const int patch_w : {32, 16, 64, 8, 128}) {
            const int patch_h = 128 / patch_w;
            const int halo_rows = (patch_h - 1) * conv.window.stride_y + conv.window.kernel_h;
            const int halo_box_w = (patch_w - 1) * conv.window.stride_x + conv.window.kernel_w;
            if (halo_box_w > 256 || halo_rows > 256) continue;
            best = std::min(best, round_up(halo_rows * halo_box_w * group * element, 1024));
        }
        return best;
    };
    // Shared memory: two to four A stages (filled by the producers), two to
    // four B stages (TMA), the per-column parameters, and a halo region of what
    // is left; the deepest rings whose leftover holds two halos of both source
    // types, with smaller channel groups when none does. The region takes as
    // many halo buffers (2..8) as fit once the patch shape is known.
    for (;;) {
        const int need = std::max(smallest_halo(conv.layouts[0].group, 4), smallest_halo(conv.layouts[1].group, 2));
        bool fits = false;
        // Resident weights when one N tile's K blocks fit (no weight ring at all),
        // else deeper rings first: each A or B stage in flight hides one producer
        // -> MMA -> commit round trip.
        const int k_blocks = conv.k_padded / 128;
        const bool can_reside = conv.n_tiles == 1 && k_blocks <= 8;
        constexpr int depths[][3] = {{4, 0, 1}, {3, 0, 1}, {2, 0, 1}, {4, 4, 0}, {3, 4, 0}, {4, 3, 0},
                                     {3, 3, 0}, {2, 4, 0}, {2, 3, 0}, {2, 2, 0}};
        for (const auto& depth : depths) {
            if (depth[2] && !can_reside) continue;
            conv.b_resident = depth[2] != 0;
            conv.a_stages = depth[0];
            conv.b_stages = conv.b_resident ? k_blocks : depth[1];
            const int fixed = kernels::fused_conv_shared_bytes(conv.weight_limbs, conv.activation_limbs, conv.n_tile,
                                                               conv.n_tiles, conv.a_stages, conv.b_stages, 0);
            conv.halo_budget = ((kernels::fused_conv_max_shared - fixed) / 2) / 1024 * 1024;
            if (conv.halo_budget >= need) {
                fits = true;
                break;
            }
        }
        if (fits) break;
        auto& wider = conv.layouts[0].group * 4 >= conv.layouts[1].group * 2 ? conv.layouts[0] : conv.layouts[1];
        if (wider.group <= 16) {
            return fail(Code::invalid_argument, "integer conv window or output channels too large for shared memory");
        }
        wider.group /= 2;
    }
    for (auto& layout : conv.layouts) layout.groups = conv.c_pad / layout.group;
    // Producer time per tile grows with the 16-byte chunks each position
    // quantises (plus a fixed per-tile cost), epilogue time with the output
    // columns: a second producer set (and four epilogue warps instead of eight)
    // when the producers have about twice the epilogue's work and a tile has at
    // most 128 accumulator columns. Measured on the 1920x1088 sweep: the 3x3
    // 64->64 conv gains 21 % with two sets, the 3x3 256->256 convs lose 7 %.
    // NVCR_SM100_PRODUCER_SETS=1|2 overrides (for tuning).
    {
        const int producer_work = conv.k_real / 16 + 12;
        const int epilogue_work = conv.n_tile * accumulators / 4;
        conv.producer_sets = producer_work >= 2 * epilogue_work && conv.n_tile * accumulators <= 128 ? 2 : 1;
        if (const char* forced = std::getenv("NVCR_SM100_PRODUCER_SETS")) {
            if (forced[0] == '1' && forced[1] == 0) conv.producer_sets = 1;
            if (forced[0] == '2' && forced[1] == 0) conv.producer_sets = 2;
        }
        // Each set takes half of the A stages.
        if (conv.a_stages % 2 != 0) conv.producer_sets = 1;
    }
    // Physical weight row -> node row (-1: zero padding). A chunk-add conv puts
    // pair (c, c + C/2) in columns j and j + n_tile/2 of one tile.
    auto source_row = [&](int physical) -> int {
        if (!conv.chunk_add) return physical < rows ? physical : -1;
        const int tile = physical / conv.n_tile;
        const int local = physical % conv.n_tile;
        const int half = conv.n_tile / 2;
        const int pair = tile * half + (local % half);
        if (pair >= rows / 2) return -1;
        return local < half ? pair : rows / 2 + pair;
    };

    const auto quantized = quantize_weights(program_, node);
    // q of (row, K channel c, K tap) from the node's order k = c * taps + tap;
    // padding holds q = 0. A fields conv has one K tap whose channel is k itself.
    auto weight_q = [&](int row, int c, int tap) -> int {
        const std::size_t at = static_cast<std::size_t>(row) * node.in_channels;
        if (conv.fields) return c < node.in_channels ? quantized.values[at + static_cast<std::size_t>(c)] : 0;
        if (c >= conv.channels) return 0;
        return quantized.values[at + static_cast<std::size_t>(c) * taps + tap];
    };
    // Limbs of q: (q >> 8, (q & 255) - 128) for 16-bit weights, q for 8-bit.
    const bool two = conv.weight_limbs == 2;
    auto high_limb = [&](int q) { return two ? q >> 8 : q; };  // arithmetic shift: floor(q / 256)
    auto low_limb = [&](int q) { return two ? (q & 255) - 128 : 0; };

    std::vector<float> scales(n_padded, 0.0f);
    std::vector<float> bias(n_padded, 0.0f);
    std::vector<long long> row_terms(n_padded, 0);
    const long long aw = two ? 256 : 1;
    const long long cw = two ? 128 : 0;
    const long long cx = conv.activation_limbs == 2 ? 128 : 0;
    for (int physical = 0; physical < n_padded; ++physical) {
        const int row = source_row(physical);
        if (row < 0) continue;
        scales[physical] = quantized.scales[static_cast<std::size_t>(row)];
        bias[physical] = program_.weights[node.bias_offset + static_cast<std::size_t>(row)];
        if (!std::isfinite(scales[physical]) || !std::isfinite(bias[physical])) conv.finite_columns = false;
        long long high_sum = 0;
        long long low_sum = 0;
        for (int c = 0; c < conv.c_pad; ++c) {
            for (int tap = 0; tap < conv.k_taps; ++tap) {
                const int q = weight_q(row, c, tap);
                high_sum += high_limb(q);
                low_sum += low_limb(q);
            }
        }
        // cx (aw sum Wh + sum Wl') + K cw cx, over all K = k_taps * c_pad entries.
        row_terms[physical] = cx * (aw * high_sum + low_sum) + static_cast<long long>(conv.k_real) * cw * cx;
    }
    {
        float smallest = std::numeric_limits<float>::infinity();
        float largest = 0.0f;
        for (int physical = 0; physical < n_padded; ++physical) {
            const float magnitude = std::fabs(scales[physical]);
            if (source_row(physical) < 0 || magnitude == 0.0f) continue;
            smallest = std::min(smallest, magnitude);
            largest = std::max(largest, magnitude);
        }
        if (!conv.finite_columns) {
            conv.fma_lo = 1;
            conv.fma_hi = 0;
        } else if (largest == 0.0f) {
            conv.fma_lo = -126;
            conv.fma_hi = 127;
        } else if (smallest >= std::numeric_limits<float>::min()) {
            conv.fma_lo = std::max(-126, -126 - std::ilogb(smallest));
            conv.fma_hi = std::min(127, 94 - std::ilogb(largest));
        }
    }
    // column term factors: cw (ax sum Xh + sum Xl')
    const long long ax = conv.activation_limbs == 2 ? 256 : 1;
    conv.column_high_factor = cw * ax;
    conv.column_low_factor = conv.activation_limbs == 2 ? cw : 0;

    // Weight matrices [n_padded][k_padded] in a layout's K order:
    // k = g * (k_taps * group) + tap * group + (c - g * group); zero bytes past K.
    const std::size_t matrix = static_cast<std::size_t>(n_padded) * conv.k_padded;
    auto build = [&](int group, std::vector<std::int8_t>& high, std::vector<std::int8_t>& low) {
        high.assign(matrix, 0);
        low.assign(two ? matrix : 0, 0);
        for (int physical = 0; physical < n_padded; ++physical) {
            const int row = source_row(physical);
            if (row < 0) continue;
            for (int c = 0; c < conv.c_pad; ++c) {
                const int g = c / group;
                for (int tap = 0; tap < conv.k_taps; ++tap) {
                    const int q = weight_q(row, c, tap);
                    const std::size_t at = static_cast<std::size_t>(physical) * conv.k_padded +
                        static_cast<std::size_t>(g) * conv.k_taps * group + static_cast<std::size_t>(tap) * group +
                        (c - g * group);
                    high[at] = static_cast<std::int8_t>(high_limb(q));
                    if (two) low[at] = static_cast<std::int8_t>(low_limb(q));
                }
            }
        }
    };
    const bool shared_layout = conv.layouts[0].group == conv.layouts[1].group;
    std::vector<std::int8_t> high[2], low[2];
    build(conv.layouts[0].group, high[0], low[0]);
    if (!shared_layout) build(conv.layouts[1].group, high[1], low[1]);

    // One allocation: [scales][bias][row_terms][high 0][low 0][high 1][low 1], each 1024-aligned.
    const std::size_t scales_at = 0;
    const std::size_t bias_at = align_up(scales_at + n_padded * sizeof(float), alignment);
    const std::size_t terms_at = align_up(bias_at + n_padded * sizeof(float), alignment);
    std::size_t matrices_at[2][2] = {{0, 0}, {0, 0}};
    std::size_t total = align_up(terms_at + n_padded * sizeof(long long), alignment);
    for (int layout = 0; layout < (shared_layout ? 1 : 2); ++layout) {
        for (int limb = 0; limb < conv.weight_limbs; ++limb) {
            matrices_at[layout][limb] = total;
            total = align_up(total + matrix, alignment);
        }
    }
    cudaError_t status = cudaMalloc(&conv.allocation, total);
    if (status != cudaSuccess) return cuda_error("cudaMalloc integer weights", status);
    auto* base = static_cast<std::uint8_t*>(conv.allocation);
    conv.scales = reinterpret_cast<float*>(base + scales_at);
    conv.bias = reinterpret_cast<float*>(base + bias_at);
    conv.row_terms = reinterpret_cast<long long*>(base + terms_at);
    struct Upload {
        void* to;
        const void* from;
        std::size_t bytes;
    };
    std::vector<Upload> uploads = {{conv.scales, scales.data(), scales.size() * sizeof(float)},
                                   {conv.bias, bias.data(), bias.size() * sizeof(float)},
                                   {conv.row_terms, row_terms.data(), row_terms.size() * sizeof(long long)}};
    for (int layout = 0; layout < 2; ++layout) {
        const int from = shared_layout ? 0 : layout;
        auto& target = conv.layouts[layout];
        target.b_high = reinterpret_cast<std::int8_t*>(base + matrices_at[from][0]);
        target.b_low = two ? reinterpret_cast<std::int8_t*>(base + matrices_at[from][1]) : target.b_high;
        if (from == layout) {
            uploads.push_back({target.b_high, high[from].data(), matrix});
            if (two) uploads.push_back({target.b_low, low[from].data(), matrix});
        }
    }
    for (const auto& upload : uploads) {
        if (upload.bytes == 0) continue;
        status = cudaMemcpy(upload.to, upload.from, upload.bytes, cudaMemcpyHostToDevice);
        if (status != cudaSuccess) {
            cudaFree(conv.allocation);
            return cuda_error("cudaMemcpy integer weights", status);
        }
    }
    for (auto& layout : conv.layouts) {
        status = kernels::encode_int8_map(&layout.b_high_map, layout.b_high, n_padded, conv.k_padded, conv.n_tile);
        if (status == cudaSuccess) {
            status = kernels::encode_int8_map(&layout.b_low_map, layout.b_low, n_padded, conv.k_padded, conv.n_tile);
        }
        if (status != cudaSuccess) {
            cudaFree(conv.allocation);
            return cuda_error("cuTensorMapEncodeTiled weights", status);
        }
    }
    auto direct = prepare_direct(conv, step, node, quantized);
    if (!direct) {
        cudaFree(conv.allocation);
        return direct;
    }
    step.conv = static_cast<int>(convs_.size());
    convs_.push_back(conv);
    return Ok{};
}

// The direct path of a w8a8 conv when its window allows it: the tap-major int8
// weight matrix [n_tiles * n_tile][taps * c8] (zero rows and channels as
// padding), its TMA map, and the ring depths that fit in shared memory.
Status Executor::prepare_direct(IntegerConv& conv, const Step& step, const Node& node,
                                const IntegerWeights& quantized) {
    if (conv.weight_limbs != 1 || conv.activation_limbs != 1) return Ok{};
    if (const char* forced = std::getenv("NVCR_SM100_DIRECT"); forced != nullptr && forced[0] == '0') return Ok{};
    const kernels::Window& w = step.window;
    const int taps = conv.k_taps;
    if (conv.fields) {
        conv.c8 = round_up(conv.channels * conv.taps, 32);
        if (conv.c8 > 64) return Ok{};
    } else {
        const bool window_ok = w.kernel_h <= 3 && w.kernel_w <= 3 && w.stride_y == 1 && w.stride_x == 1;
        // The plane prepass keeps all channels of 64 pixels in shared memory.
        if (!window_ok || conv.channels > 780) return Ok{};
        conv.c8 = round_up(conv.channels, 32);
    }
    conv.k_block = conv.c8 % 128 == 0 ? 128 : (conv.c8 % 64 == 0 ? 64 : 32);
    conv.c_blocks = conv.c8 / conv.k_block;
    conv.direct_k_blocks = taps * conv.c_blocks;
    const int n_padded = conv.n_tiles * conv.n_tile;
    // K blocks per pipeline stage: each stage costs the MMA thread a wait and a
    // commit (a few hundred cycles), so stages whose MMAs are short (an MMA
    // issues in about max(60, n_tile / 2) cycles) take several K blocks.
    const int block_cycles = (conv.k_block / 32) * std::max(60, conv.n_tile / 2);
    conv.direct_group = 1;
    for (const int group : {1, 2, 3, 4}) {
        if (conv.direct_k_blocks % group != 0) continue;
        conv.direct_group = group;
        if (group * block_cycles >= 500) break;
    }
    bool fits = false;
    // Ring depths: resident weights when one N tile's K blocks fit, else the
    // deepest rings that fit.
    if (!fits && conv.n_tiles == 1 && conv.direct_k_blocks <= 16) {
        for (const int a_stages : {16, 12, 8, 6, 4, 3, 2}) {
            if (a_stages * conv.direct_group > 32) continue;  // one issuing lane per copy of a stage
            if (kernels::direct_conv_shared_bytes(conv.k_block, conv.n_tile, conv.n_tiles, a_stages,
                                                  conv.direct_k_blocks, conv.direct_group, true, 1) <=
                kernels::direct_conv_max_shared) {
                conv.direct_a_stages = a_stages;
                conv.direct_b_stages = conv.direct_k_blocks;
                conv.direct_b_resident = true;
                fits = true;
                break;
            }
        }
    }
    if (!fits) {
        constexpr int depths[][2] = {{16, 16}, {12, 12}, {8, 8}, {6, 6}, {4, 6}, {6, 4},
                                     {4, 4}, {4, 3}, {3, 3}, {3, 2}, {2, 2}};
        for (const int group : {conv.direct_group, 1}) {
            if (fits) break;
            for (const auto& depth : depths) {
                if ((depth[0] > depth[1] ? depth[0] : depth[1]) * group > 32) continue;
                if (kernels::direct_conv_shared_bytes(conv.k_block, conv.n_tile, conv.n_tiles, depth[0], depth[1],
                                                      group, false, 1) <= kernels::direct_conv_max_shared) {
                    conv.direct_a_stages = depth[0];
                    conv.direct_b_stages = depth[1];
                    conv.direct_group = group;
                    fits = true;
                    break;
                }
            }
        }
    }
    if (!fits) return Ok{};
    // Pairs of patches per tile share each weight block between two
    // accumulators: half the weight rows the TMA moves per MAC (deep-K convs
    // with up to 256 columns), and half the MMA thread's waits, commits and tile
    // hand-offs per position (narrow convs). The planner decides per plan.
    const bool narrow = 2 * conv.n_tile <= 256;
    if (narrow || (conv.k_block == 128 && 2 * conv.n_tile <= 512 && conv.direct_k_blocks >= 8)) {
        constexpr int depths[][2] = {{8, 8}, {6, 6}, {4, 4}, {4, 3}, {3, 3}, {3, 2}, {2, 2}};
        const bool resident = conv.n_tiles == 1 && conv.direct_k_blocks <= 16;
        for (const int group : {conv.direct_group == 3 ? 3 : 1, 1}) {  // paired kernels take groups of 1 or 3
            if (conv.pair_a_stages > 0) break;
            for (const auto& depth : depths) {
                const int b_stages = resident ? conv.direct_k_blocks : depth[1];
                if (depth[0] * group * 2 > 32 || (!resident && depth[1] * group > 32)) continue;
                if (kernels::direct_conv_shared_bytes(conv.k_block, conv.n_tile, conv.n_tiles, depth[0], b_stages,
                                                      group, resident, 2) <= kernels::direct_conv_max_shared) {
                    conv.pair_a_stages = depth[0];
                    conv.pair_b_stages = b_stages;
                    conv.pair_group = group;
                    conv.pair_b_resident = resident;
                    break;
                }
            }
        }
    }
    // Row halos: an A stage per (window row, channel block) moves patch_w +
    // kernel_w - 1 rows instead of kernel_w * patch_w, leaving the weights most
    // of the copies; they stream one K block per stage. 128-byte K blocks only:
    // with 64-byte ones (N 64 there) the MMAs on the shifted rows issued at
    // less than half the rate of per-tap boxes' and the conv ran slower.
    if (!conv.fields && w.kernel_w >= 2 && conv.k_block == 128) {
        conv.row_bytes = kernels::direct_row_bytes(128, w.kernel_w, conv.k_block);
        const bool resident = conv.n_tiles == 1 && conv.direct_k_blocks <= 16;
        for (const int m_tiles : {1, 2}) {
            if (m_tiles == 2 && 2 * conv.n_tile > 512) continue;
            constexpr int depths[][2] = {{8, 8}, {6, 8}, {6, 6}, {4, 8}, {4, 6}, {4, 4}, {3, 8}, {3, 6},
                                         {3, 4}, {2, 8}, {2, 6}, {2, 5}, {2, 4}, {2, 3}};
            for (const auto& depth : depths) {
                const int b_stages = resident ? conv.direct_k_blocks : depth[1];
                if (depth[0] * m_tiles > 32 || b_stages > 16) continue;
                if (kernels::direct_conv_row_shared_bytes(conv.k_block, conv.n_tile, conv.n_tiles, depth[0], b_stages,
                                                          resident, m_tiles, conv.row_bytes) >
                    kernels::direct_conv_max_shared) {
                    continue;
                }
                (m_tiles == 1 ? conv.row_a_stages : conv.row_pair_a_stages) = depth[0];
                (m_tiles == 1 ? conv.row_b_stages : conv.row_pair_b_stages) = b_stages;
                (m_tiles == 1 ? conv.row_b_resident : conv.row_pair_b_resident) = resident;
                break;
            }
        }
    }
    const std::size_t row_bytes = static_cast<std::size_t>(taps) * conv.c8;
    std::vector<std::int8_t> matrix(static_cast<std::size_t>(n_padded) * row_bytes, 0);
    const int rows = node.out_channels;
    long long largest_row_sum = 0;
    for (int physical = 0; physical < n_padded; ++physical) {
        int row = physical < rows ? physical : -1;
        if (conv.chunk_add) {
            const int tile = physical / conv.n_tile;
            const int local = physical % conv.n_tile;
            const int half = conv.n_tile / 2;
            const int pair = tile * half + (local % half);
            row = pair >= rows / 2 ? -1 : (local < half ? pair : rows / 2 + pair);
        }
        if (row < 0) continue;
        const std::size_t at = static_cast<std::size_t>(row) * node.in_channels;
        long long row_sum = 0;
        for (int tap = 0; tap < taps; ++tap) {
            for (int c = 0; c < conv.c8; ++c) {
                int q = 0;
                if (conv.fields) {
                    q = c < node.in_channels ? quantized.values[at + static_cast<std::size_t>(c)] : 0;
                } else if (c < conv.channels) {
                    q = quantized.values[at + static_cast<std::size_t>(c) * conv.taps + tap];
                }
                matrix[static_cast<std::size_t>(physical) * row_bytes + static_cast<std::size_t>(tap) * conv.c8 + c] =
                    static_cast<std::int8_t>(q);
                row_sum += q < 0 ? -q : q;
            }
        }
        largest_row_sum = std::max(largest_row_sum, row_sum);
    }
    conv.small_accumulators = largest_row_sum * 127 < (1LL << 22);
    cudaError_t status = cudaMalloc(&conv.direct_allocation, matrix.size());
    if (status != cudaSuccess) return cuda_error("cudaMalloc direct weights", status);
    status = cudaMemcpy(conv.direct_allocation, matrix.data(), matrix.size(), cudaMemcpyHostToDevice);
    if (status == cudaSuccess) {
        status = kernels::encode_weight_map(&conv.direct_b_map, conv.direct_allocation, n_padded, row_bytes,
                                            conv.k_block, conv.n_tile);
    }
    if (status != cudaSuccess) {
        cudaFree(conv.direct_allocation);
        conv.direct_allocation = nullptr;
        return cuda_error("direct weights", status);
    }
    conv.direct = true;
    return Ok{};
}

// ---------------------------------------------------------------- planning

// Arena bytes of a tensor: NCHW FP32, or a staged tensor's records followed by its maxima.
std::size_t Executor::tensor_bytes(const Extent& extent, std::size_t id) const {
    if (!staged_tensor_[id]) return extent.count() * sizeof(float);
    return staged_max_offset(extent, id) + static_cast<std::size_t>(extent.height) * extent.width * sizeof(float);
}

std::size_t Executor::staged_max_offset(const Extent& extent, std::size_t id) const {
    const std::size_t pixels = static_cast<std::size_t>(extent.height) * extent.width;
    return align_up(pixels * static_cast<std::size_t>(round_up(extent.channels, 16)) * sizeof(float), alignment);
}

Result<Executor::Plan*> Executor::plan_for(const std::vector<Extent>& input_extents, Boundary boundary) {
    std::vector<std::int32_t> key{static_cast<std::int32_t>(boundary)};
    for (const auto& e : input_extents) {
        key.push_back(e.channels);
        key.push_back(e.height);
        key.push_back(e.width);
    }
    if (auto found = plans_.find(key); found != plans_.end()) return found->second.get();

    auto plan = std::make_unique<Plan>();
    plan->boundary = boundary;
    const std::size_t tensor_count = program_.tensor_names.size();
    plan->extents.assign(tensor_count, Extent{});
    plan->offsets.assign(tensor_count, npos);
    plan->convs.assign(steps_.size(), PlannedConv{});
    // Extents of every tensor, validated exactly as the reference validates them.
    for (std::size_t slot = 0; slot < program_.inputs.size(); ++slot) {
        plan->extents[program_.inputs[slot]] = input_extents[slot];
    }
    for (const auto& node : program_.nodes) {
        Extent in[2] = {plan->extents[node.inputs[0]], plan->extents[node.inputs[1]]};
        auto extent = output_extent(program_, node, in, node.input_count);
        if (!extent) return extent.error();
        plan->extents[node.output] = extent.value();
    }
    for (const auto& step : steps_) {
        if (step.kind == StepKind::chunk_add) {
            const Extent source = plan->extents[step.source];
            plan->extents[step.output] = Extent{source.channels / 2, source.height, source.width};
        }
    }

    // Lifetimes in steps: a tensor is freed after the last step that reads it.
    const std::size_t step_count = steps_.size();
    std::vector<std::ptrdiff_t> last_read(tensor_count, -1);
    for (std::size_t s = 0; s < step_count; ++s) {
        for (const auto id : steps_[s].reads) last_read[id] = static_cast<std::ptrdiff_t>(s);
    }
    std::vector<bool> pinned(tensor_count, false);
    for (const auto id : program_.outputs) pinned[id] = true;
    for (const auto id : program_.inputs) pinned[id] = pinned[id] || last_read[id] < 0;

    OffsetAllocator allocator;
    auto tensor_bytes = [&](std::size_t id) { return this->tensor_bytes(plan->extents[id], id); };
    for (const auto id : program_.inputs) {
        if (plan->offsets[id] == npos) plan->offsets[id] = allocator.allocate(tensor_bytes(id));
    }
    allocator.note_peak();
    for (std::size_t s = 0; s < step_count; ++s) {
        const Step& step = steps_[s];
        plan->offsets[step.output] = allocator.allocate(tensor_bytes(step.output));
        std::vector<std::size_t> scratch;
        if (step.kind == StepKind::integer_conv) {
            const IntegerConv& conv = convs_[static_cast<std::size_t>(step.conv)];
            const Node& node = program_.nodes[step.node];
            const Extent source = plan->extents[step.source];
            const Extent out = plan->extents[node.output];
            PlannedConv& pc = plan->convs[s];
            pc.positions = out.height * out.width;
            const bool program_input = std::find(program_.inputs.begin(), program_.inputs.end(), step.source) !=
                program_.inputs.end();
            pc.source_half = boundary == Boundary::half && program_input;
            const int element = pc.source_half ? 2 : 4;
            const int record_bytes = conv.layouts[pc.source_half ? 1 : 0].group * element;
            // Patch shape: least padding waste, then the smallest halo that fits.
            int best_waste = INT_MAX;
            int best_bytes = INT_MAX;
            for (const int patch_w : {32, 16, 64, 8, 128}) {
                const int patch_h = 128 / patch_w;
                const int tiles_y = (out.height + patch_h - 1) / patch_h;
                const int tiles_x = (out.width + patch_w - 1) / patch_w;
                const int halo_rows = (patch_h - 1) * conv.window.stride_y + conv.window.kernel_h;
                const int halo_box_w = (patch_w - 1) * conv.window.stride_x + conv.window.kernel_w;
                const int bytes = round_up(halo_rows * halo_box_w * record_bytes, 1024);
                if (bytes > conv.halo_budget || halo_box_w > 256 || halo_rows > 256) continue;
                const long long covered = static_cast<long long>(tiles_y) * tiles_x * 128;
                const int waste = static_cast<int>((covered - pc.positions) * 1000 / std::max(pc.positions, 1));
                if (waste < best_waste - 30 || (waste <= best_waste + 30 && bytes < best_bytes)) {
                    if (waste < best_waste) best_waste = waste;
                    best_bytes = bytes;
                    pc.patch_h = patch_h;
                    pc.patch_w = patch_w;
                    pc.tiles_y = tiles_y;
                    pc.tiles_x = tiles_x;
                    pc.halo_rows = halo_rows;
                    pc.halo_box_w = halo_box_w;
                    pc.halo_bytes = bytes;
                }
            }
            if (pc.patch_w == 0) return fail(Code::invalid_argument, "integer conv window is too large for the halo");
            pc.halo_buffers = std::min(8, 2 * conv.halo_budget / pc.halo_bytes);
            // Staged grid: the source pixels, or the output positions of a fields conv;
            // a staged source tensor is read in place.
            pc.source_staged = staged_tensor_[step.source];
            const bool multi_tap = !conv.fields && conv.k_taps > 1;
            const std::size_t grid_pixels = conv.fields ? static_cast<std::size_t>(pc.positions)
                                                        : static_cast<std::size_t>(source.height) * source.width;
            if (!pc.source_staged) {
                // The quantise-on-load copy: the conv itself, or a direct conv's fallback.
                if (!conv.direct || multi_tap) {
                    pc.staged = allocator.allocate(grid_pixels * conv.c_pad * element);
                    scratch.push_back(pc.staged);
                }
                pc.pixel_max = allocator.allocate(grid_pixels * sizeof(float));
                scratch.push_back(pc.pixel_max);
            }
            if (conv.direct) {
                pc.quantised = allocator.allocate(grid_pixels * conv.c8);
                scratch.push_back(pc.quantised);
                if (multi_tap) {
                    pc.fallback = allocator.allocate(sizeof(unsigned int));
                    scratch.push_back(pc.fallback);
                }
                // Patch shape of the direct conv: least padding waste.
                int least = INT_MAX;
                for (const int patch_w : {32, 16, 64, 8, 128}) {
                    const int patch_h = 128 / patch_w;
                    const int tiles_y = (out.height + patch_h - 1) / patch_h;
                    const int tiles_x = (out.width + patch_w - 1) / patch_w;
                    const long long covered = static_cast<long long>(tiles_y) * tiles_x * 128;
                    const int waste = static_cast<int>((covered - pc.positions) * 1000 / std::max(pc.positions, 1));
                    if (waste < least) {
                        least = waste;
                        pc.d_patch_h = patch_h;
                        pc.d_patch_w = patch_w;
                        pc.d_tiles_y = tiles_y;
                        pc.d_tiles_x = tiles_x;
                    }
                }
                // Row halos when one-row patches of 128 waste at most 1/8 of the
                // positions.
                pc.row_halo = false;
                if (conv.row_a_stages > 0) {
                    const int row_tiles_x = (out.width + 127) / 128;
                    if (static_cast<long long>(row_tiles_x) * 128 * 8 <= static_cast<long long>(out.width) * 9) {
                        pc.row_halo = true;
                        pc.d_patch_h = 1;
                        pc.d_patch_w = 128;
                        pc.d_tiles_y = out.height;
                        pc.d_tiles_x = row_tiles_x;
                    }
                }
                // Tiles of two patches (plain or depth_to_space outputs only) when
                // two accumulators still leave TMEM two buffers, or when the conv
                // has about two tiles per SM or fewer (then one tile per SM needs
                // no second buffer).
                const long long tiles = static_cast<long long>(pc.d_tiles_y) * pc.d_tiles_x * conv.n_tiles;
                const bool pair_ready = pc.row_halo ? conv.row_pair_a_stages > 0 : conv.pair_a_stages > 0;
                if (pair_ready && !step.wsilu && !step.chunk_add && !step.residual &&
                    !staged_tensor_[step.output] && (4 * conv.n_tile <= 512 || tiles <= 2LL * sm_count_)) {
                    pc.m_tiles = 2;
                }
            }
        }
        allocator.note_peak();
        for (const auto offset : scratch) allocator.release(offset);
        // Release what this step read for the last time, and a dead output.
        std::set<std::size_t> done(step.reads.begin(), step.reads.end());
        done.insert(step.output);
        for (const auto id : done) {
            if (!pinned[id] && last_read[id] <= static_cast<std::ptrdiff_t>(s) && plan->offsets[id] != npos) {
                allocator.release(plan->offsets[id]);
            }
        }
    }
    plan->arena_bytes = std::max<std::size_t>(allocator.peak(), alignment);
    auto* raw = plan.get();
    plans_.emplace(std::move(key), std::move(plan));
    return raw;
}

Status Executor::ensure_arena(std::size_t bytes) {
    if (bytes <= arena_bytes_ && arena_ != nullptr) return Ok{};
    if (arena_ != nullptr) {
        // In-flight work may still use the old arena; graphs captured on it go.
        const cudaError_t synced = cudaStreamSynchronize(stream_);
        if (synced != cudaSuccess) return cuda_error("cudaStreamSynchronize", synced);
        clear_graphs();
        cudaFree(arena_);
        arena_ = nullptr;
        arena_bytes_ = 0;
    }
    const cudaError_t status = cudaMalloc(&arena_, bytes);
    if (status != cudaSuccess) {
        return fail(Code::resource_exhausted, std::string("cudaMalloc workspace: ") + cudaGetErrorString(status));
    }
    arena_bytes_ = bytes;
    ++arena_generation_;
    return Ok{};
}

// ---------------------------------------------------------------- execution

Status Executor::launch_step(const Step& step, Plan& plan, std::size_t index) {
    auto* base = run_base_;
    auto tensor = [&](std::size_t id) { return reinterpret_cast<float*>(base + plan.offsets[id]); };
    const Node& node = program_.nodes[step.node];
    const Extent out_extent = plan.extents[step.output];
    const std::size_t count = out_extent.count();
    cudaError_t status = cudaSuccess;
    int launched = 1;
    switch (step.kind) {
    case StepKind::integer_conv: {
        const IntegerConv& conv = convs_[static_cast<std::size_t>(step.conv)];
        const Extent source = plan.extents[step.source];
        const Extent conv_out = plan.extents[node.output];
        PlannedConv& pc = plan.convs[index];
        const IntegerConv::Layout& layout = conv.layouts[pc.source_half ? 1 : 0];
        const int element = pc.source_half ? 2 : 4;
        float* pixel_max = reinterpret_cast<float*>(base + pc.pixel_max);
        void* staged = base + pc.staged;
        if (pc.source_staged) {
            staged = base + plan.offsets[step.source];
            pixel_max = reinterpret_cast<float*>(base + plan.offsets[step.source] +
                                                 staged_max_offset(plan.extents[step.source], step.source));
        }
        const Direct& direct_in = run_inputs_[step.source];
        const void* from = direct_in.data != nullptr ? direct_in.data : tensor(step.source);
        if (direct_in.data != nullptr && direct_in.half != pc.source_half) {
            return fail(Code::internal_error, "integer conv source type does not match its plan");
        }
        // The grid the conv kernels read: source pixels, or output positions
        // whose records are receptive fields.
        const int grid_h = conv.fields ? conv_out.height : source.height;
        const int grid_w = conv.fields ? conv_out.width : source.width;
        const int pixels = grid_h * grid_w;
        const std::string label = program_.tensor_names[step.output];
        const double positions = static_cast<double>(pc.positions);
        const Direct& direct_out = run_outputs_[index];
        void* out = direct_out.data != nullptr ? direct_out.data : tensor(step.output);
        const int out_half = direct_out.data != nullptr && direct_out.half ? 1 : 0;
        float* out_max = nullptr;
        int out_c_pad = 0;
        const double ops = 2.0 * conv.channels * conv.taps * static_cast<double>(node.out_channels) * positions;
        const double out_bytes = static_cast<double>(out_extent.count()) * (out_half ? 2.0 : 4.0) +
            (step.residual ? static_cast<double>(out_extent.count()) * 4.0 : 0.0);
        const float* residual = step.residual ? tensor(*step.residual) : nullptr;
        const int residual_c_pad = step.residual && staged_tensor_[*step.residual]
            ? round_up(plan.extents[*step.residual].channels, 16) : 0;
        if (staged_tensor_[step.output]) {
            const Extent staged_out = plan.extents[step.output];
            out_c_pad = round_up(staged_out.channels, 16);
            out_max = reinterpret_cast<float*>(base + plan.offsets[step.output] +
                                               staged_max_offset(staged_out, step.output));
        }
        auto zero_out_max = [&]() -> Status {
            if (out_max == nullptr) return Ok{};
            const Extent staged_out = plan.extents[step.output];
            const cudaError_t zeroed =
                kernels::zero_floats(out_max, static_cast<std::size_t>(staged_out.height) * staged_out.width, stream_);
            if (zeroed != cudaSuccess) return cuda_error("zeroing staged maxima", zeroed);
            ++launches_;
            return Ok{};
        };
        // The quantise-on-load conv: the conv itself, or (gate not null) a direct
        // conv's fallback that runs only when that conv found a mixed window.
        auto launch_fused = [&](const unsigned int* gate, cudaStream_t on) -> Status {
            cudaError_t launched_status = cudaSuccess;
            if (!pc.source_staged) {
                if (conv.fields) {
                    launched_status = kernels::stage_receptive_fields(
                        from, pc.source_half ? 1 : 0, source.channels, source.height, source.width, step.window,
                        conv_out.height, conv_out.width, conv.c_pad, staged, pixel_max, on);
                } else {
                    launched_status = kernels::stage_source(from, pc.source_half ? 1 : 0, source.channels, conv.c_pad,
                                                            pixels, staged, pixel_max, on, gate);
                }
                if (launched_status != cudaSuccess) return cuda_error("source staging launch", launched_status);
                ++launches_;
                auto marked = mark((gate ? "fallback_stage:" : "stage_source:") + label,
                                   gate ? "fallback" : "stage_source", 0.0,
                                   static_cast<double>(source.count()) * element +
                                       static_cast<double>(pixels) * (conv.c_pad * element + 4.0));
                if (!marked) return marked;
            }
            if (pc.halo_base != staged) {
                launched_status = kernels::encode_halo_map(&pc.halo_map, staged, pc.source_half ? 1 : 0, conv.c_pad,
                                                           grid_h, grid_w, layout.group, pc.halo_box_w, pc.halo_rows);
                if (launched_status != cudaSuccess) return cuda_error("cuTensorMapEncodeTiled halo", launched_status);
                pc.halo_base = staged;
            }
            kernels::FusedConvArgs f{};
            f.source_half = pc.source_half ? 1 : 0;
            f.pixel_max = pixel_max;
            f.channels = conv.fields ? conv.channels * conv.taps : conv.channels;
            f.c_pad = conv.c_pad;
            f.in_h = grid_h;
            f.in_w = grid_w;
            f.out_h = conv_out.height;
            f.out_w = conv_out.width;
            f.window = conv.window;
            f.k_real = conv.k_real;
            f.k_blocks = conv.k_padded / 128;
            f.positions = pc.positions;
            f.patch_h = pc.patch_h;
            f.patch_w = pc.patch_w;
            f.tiles_y = pc.tiles_y;
            f.tiles_x = pc.tiles_x;
            f.p_tiles = pc.tiles_y * pc.tiles_x;
            f.group = layout.group;
            f.groups = layout.groups;
            f.record_bytes = layout.group * element;
            f.halo_rows = pc.halo_rows;
            f.halo_box_w = pc.halo_box_w;
            f.halo_bytes = pc.halo_bytes;
            f.halo_buffers = pc.halo_buffers;
            f.producer_sets = conv.producer_sets;
            f.a_stages = conv.a_stages;
            f.b_stages = conv.b_stages;
            f.b_resident = conv.b_resident ? 1 : 0;
            f.n_tile = conv.n_tile;
            f.n_tiles = conv.n_tiles;
            f.column_high_factor = conv.weight_limbs == 2 ? conv.column_high_factor : 0;
            f.column_low_factor = conv.weight_limbs == 2 ? conv.column_low_factor : 0;
            f.scales = conv.scales;
            f.bias = conv.bias;
            f.row_terms = conv.activation_limbs == 2 ? conv.row_terms : nullptr;
            f.wsilu = step.wsilu ? 1 : 0;
            f.wsilu_scale = step.wsilu_scale;
            f.chunk_add = step.chunk_add ? 1 : 0;
            f.residual = residual;
            f.residual_c_pad = residual_c_pad;
            f.out = out;
            f.out_half = out_half;
            f.out_max = out_max;
            f.out_c_pad = out_c_pad;
            f.out_channels = conv.out_channels;
            f.d2s_block = step.d2s_block;
            f.status = status_;
            f.gate = gate;
            launched_status = kernels::fused_conv(layout.b_high_map, layout.b_low_map, pc.halo_map, conv.weight_limbs,
                                                  conv.activation_limbs, f, on);
            if (launched_status != cudaSuccess) return cuda_error("integer conv launch", launched_status);
            ++launches_;
            if (gate != nullptr) return mark("fallback_conv:" + label, "fallback", 0.0, 0.0);
            return mark("integer_conv:" + label, "integer_conv", ops,
                        static_cast<double>(pixels) * (conv.c_pad * element + 4.0) +
                            static_cast<double>(node.out_channels) * conv.k_real * conv.weight_limbs + out_bytes);
        };
        if (!conv.direct) {
            auto zeroed = zero_out_max();
            if (!zeroed) return zeroed;
            return launch_fused(nullptr, stream_);
        }

        // ---- direct path: per-pixel int8 activations, TMA-fed GEMM
        const bool multi_tap = !conv.fields && conv.k_taps > 1;
        auto* quantised = reinterpret_cast<std::int8_t*>(base + pc.quantised);
        auto* fallback = multi_tap ? reinterpret_cast<unsigned int*>(base + pc.fallback) : nullptr;
        if (conv.fields) {
            status = kernels::quantise_fields(from, pc.source_half ? 1 : 0, source.channels, source.height,
                                              source.width, step.window, conv_out.height, conv_out.width, conv.c8,
                                              quantised, pixel_max, stream_);
        } else if (pc.source_staged) {
            status = kernels::quantise_pixels(staged, kernels::PixelSource::staged_f32, conv.channels,
                                              round_up(source.channels, 16), conv.c8, pixels, quantised, pixel_max,
                                              fallback, stream_);
        } else {
            status = kernels::quantise_pixels(from, pc.source_half ? kernels::PixelSource::planes_f16
                                                                   : kernels::PixelSource::planes_f32,
                                              conv.channels, 0, conv.c8, pixels, quantised, pixel_max, fallback,
                                              stream_);
        }
        if (status != cudaSuccess) return cuda_error("activation quantisation launch", status);
        ++launches_;
        {
            const double read = conv.fields ? static_cast<double>(source.count()) * element
                : (pc.source_staged ? static_cast<double>(pixels) * (round_up(source.channels, 16) * 4.0 + 4.0)
                                    : static_cast<double>(source.count()) * element);
            auto marked = mark("quantise:" + label, "quantise", 0.0,
                               read + static_cast<double>(pixels) * (conv.c8 + (pc.source_staged ? 0.0 : 4.0)));
            if (!marked) return marked;
        }
        if (pc.a_base != quantised) {
            status = kernels::encode_activation_map(
                &pc.a_map, quantised, conv.c8, grid_h, grid_w, conv.k_block,
                pc.row_halo ? static_cast<std::uint32_t>(pc.d_patch_w + conv.window.kernel_w - 1) : pc.d_patch_w,
                pc.row_halo ? 1u : static_cast<std::uint32_t>(pc.d_patch_h));
            if (status != cudaSuccess) return cuda_error("cuTensorMapEncodeTiled activations", status);
            pc.a_base = quantised;
        }
        auto zeroed = zero_out_max();
        if (!zeroed) return zeroed;
        kernels::DirectConvArgs d{};
        d.pixel_max = pixel_max;
        d.in_h = grid_h;
        d.in_w = grid_w;
        d.out_h = conv_out.height;
        d.out_w = conv_out.width;
        d.window = conv.window;
        d.k_block = conv.k_block;
        d.c_blocks = conv.c_blocks;
        d.k_blocks = conv.direct_k_blocks;
        d.positions = pc.positions;
        d.patch_h = pc.d_patch_h;
        d.patch_w = pc.d_patch_w;
        d.tiles_y = pc.d_tiles_y;
        d.tiles_x = pc.d_tiles_x;
        d.p_tiles = pc.d_tiles_y * pc.d_tiles_x;
        d.m_tiles = pc.m_tiles;
        if (pc.row_halo) {
            d.row_halo = 1;
            d.a_row_bytes = conv.row_bytes;
            d.group = conv.window.kernel_w;
            d.a_stages = pc.m_tiles == 2 ? conv.row_pair_a_stages : conv.row_a_stages;
            d.b_stages = pc.m_tiles == 2 ? conv.row_pair_b_stages : conv.row_b_stages;
            d.b_resident = (pc.m_tiles == 2 ? conv.row_pair_b_resident : conv.row_b_resident) ? 1 : 0;
        } else {
            d.group = pc.m_tiles == 2 ? conv.pair_group : conv.direct_group;
            d.a_stages = pc.m_tiles == 2 ? conv.pair_a_stages : conv.direct_a_stages;
            d.b_stages = pc.m_tiles == 2 ? conv.pair_b_stages : conv.direct_b_stages;
            d.b_resident = (pc.m_tiles == 2 ? conv.pair_b_resident : conv.direct_b_resident) ? 1 : 0;
        }
        d.n_tile = conv.n_tile;
        d.n_tiles = conv.n_tiles;
        d.scales = conv.scales;
        d.bias = conv.bias;
        d.wsilu = step.wsilu ? 1 : 0;
        d.wsilu_scale = step.wsilu_scale;
        d.chunk_add = step.chunk_add ? 1 : 0;
        d.residual = residual;
        d.residual_c_pad = residual_c_pad;
        d.out = out;
        d.out_half = out_half;
        d.out_max = out_max;
        d.out_c_pad = out_c_pad;
        d.out_channels = conv.out_channels;
        d.d2s_block = step.d2s_block;
        d.vector_store = out_half && step.d2s_block == 0 && !step.wsilu && !step.chunk_add && residual == nullptr &&
                out_max == nullptr && conv.finite_columns && pc.d_patch_w % 8 == 0 && conv_out.width % 8 == 0 &&
                conv.out_channels % 8 == 0 && (reinterpret_cast<std::uintptr_t>(out) & 15u) == 0
            ? 1
            : 0;
        d.small_accumulators = conv.small_accumulators ? 1 : 0;
        d.fma_lo = conv.fma_lo;
        d.fma_hi = conv.fma_hi;
        d.fallback = fallback;
        d.status = status_;
        // In a captured run the fallback becomes a conditional node: the conv
        // sets its condition when it meets a mixed window, and a replay of a run
        // without one launches nothing more.
        cudaGraph_t captured = nullptr;
        if (multi_tap && capturing_) {
            cudaStreamCaptureStatus capture_status = cudaStreamCaptureStatusNone;
            status = cudaStreamGetCaptureInfo_v3(stream_, &capture_status, nullptr, &captured);
            if (status != cudaSuccess || capture_status != cudaStreamCaptureStatusActive || captured == nullptr) {
                return cuda_error("cudaStreamGetCaptureInfo", status == cudaSuccess ? cudaErrorStreamCaptureInvalidated
                                                                                    : status);
            }
            cudaGraphConditionalHandle condition = 0;
            status = cudaGraphConditionalHandleCreate(&condition, captured, 0u, cudaGraphCondAssignDefault);
            if (status != cudaSuccess) return cuda_error("cudaGraphConditionalHandleCreate", status);
            d.condition = condition;
        }
        status = kernels::direct_conv(pc.a_map, conv.direct_b_map, d, stream_);
        if (status != cudaSuccess) return cuda_error("direct integer conv launch", status);
        ++launches_;
        if (d.condition != 0) {
            cudaStreamCaptureStatus capture_status = cudaStreamCaptureStatusNone;
            const cudaGraphNode_t* after_conv = nullptr;
            std::size_t count_after = 0;
            status = cudaStreamGetCaptureInfo_v3(stream_, &capture_status, nullptr, &captured, &after_conv, nullptr,
                                                 &count_after);
            if (status != cudaSuccess) return cuda_error("cudaStreamGetCaptureInfo", status);
            cudaGraphNodeParams params{};
            params.type = cudaGraphNodeTypeConditional;
            params.conditional.handle = d.condition;
            params.conditional.type = cudaGraphCondTypeIf;
            params.conditional.size = 1;
            cudaGraphNode_t node = nullptr;
            status = cudaGraphAddNode(&node, captured, after_conv, count_after, &params);
            if (status != cudaSuccess) return cuda_error("cudaGraphAddNode conditional", status);
            if (fallback_stream_ == nullptr) {
                status = cudaStreamCreateWithFlags(&fallback_stream_, cudaStreamNonBlocking);
                if (status != cudaSuccess) return cuda_error("cudaStreamCreateWithFlags", status);
            }
            status = cudaStreamBeginCaptureToGraph(fallback_stream_, params.conditional.phGraph_out[0], nullptr, nullptr,
                                                   0, cudaStreamCaptureModeThreadLocal);
            if (status != cudaSuccess) return cuda_error("cudaStreamBeginCaptureToGraph", status);
            const int launched_before = launches_;  // the body's kernels run only after a mixed window
            Status body = launch_fused(nullptr, fallback_stream_);
            launches_ = launched_before;
            cudaGraph_t ended = nullptr;
            const cudaError_t end_status = cudaStreamEndCapture(fallback_stream_, &ended);
            if (!body) return body;
            if (end_status != cudaSuccess) return cuda_error("cudaStreamEndCapture fallback", end_status);
            status = cudaStreamUpdateCaptureDependencies(stream_, &node, 1, cudaStreamSetCaptureDependencies);
            if (status != cudaSuccess) return cuda_error("cudaStreamUpdateCaptureDependencies", status);
            return mark("integer_conv:" + label, "integer_conv", ops, 0.0);
        }
        auto marked = mark("integer_conv:" + label, "integer_conv", ops,
                           static_cast<double>(pixels) * (conv.c8 + 4.0) +
                               static_cast<double>(node.out_channels) * conv.k_taps * conv.c8 + out_bytes);
        if (!marked) return marked;
        if (multi_tap) return launch_fused(fallback, stream_);
        return Ok{};
    }
    case StepKind::chunk_add:
        status = kernels::chunk_add(tensor(step.source), tensor(step.output), count, stream_);
        break;
    case StepKind::generic: {
        const float* a = tensor(node.inputs[0]);
        const Extent in = plan.extents[node.inputs[0]];
        float* out = tensor(step.output);
        switch (node.op) {
        case Op::conv: {
            if (staged_tensor_[step.output]) {
                // Channel-innermost depthwise 3x3: the planner stages its input too.
                const float* staged_in = tensor(node.inputs[0]);
                float* staged_max = reinterpret_cast<float*>(base + plan.offsets[step.output] +
                                                             staged_max_offset(out_extent, step.output));
                status = kernels::depthwise3x3_staged(weights_ + node.weight_offset, weights_ + node.bias_offset,
                                                      node.out_channels, round_up(node.out_channels, 16), staged_in,
                                                      out, staged_max, out_extent.height, out_extent.width, stream_);
                launched = 2;  // zeroing of the maxima, then the depthwise
                break;
            }
            kernels::ConvShape shape{node.in_channels, node.out_channels, node.depthwise ? 1 : 0, in.height, in.width,
                                     out_extent.height, out_extent.width,
                                     kernels::Window{node.kernel[0], node.kernel[1], node.stride[0], node.stride[1],
                                                     node.pads[0], node.pads[1]}};
            status = kernels::conv_fp32(weights_ + node.weight_offset, weights_ + node.bias_offset, a, out, shape,
                                        stream_);
            break;
        }
        case Op::mul:
        case Op::add:
            status = kernels::binary(node.op == Op::mul ? kernels::Binary::mul : kernels::Binary::add, a,
                                     tensor(node.inputs[1]), out, count, stream_);
            break;
        case Op::mul_scalar:
            status = kernels::mul_scalar(a, node.scalar, out, count, stream_);
            break;
        case Op::sigmoid:
            status = kernels::sigmoid(a, out, count, stream_);
            break;
        case Op::slice_channels:
            status = kernels::copy(a + static_cast<std::size_t>(node.begin) * in.height * in.width, out, count,
                                   stream_);
            launched = 0;
            break;
        case Op::depth_to_space:
            status = kernels::depth_to_space(a, out, out_extent.channels, out_extent.height, out_extent.width,
                                             in.height, in.width, node.block, stream_);
            break;
        case Op::space_to_depth:
            status = kernels::space_to_depth(a, out, out_extent.channels, out_extent.height, out_extent.width,
                                             in.height, in.width, node.block, stream_);
            break;
        case Op::scale_channels:
            status = kernels::scale_channels(a, tensor(node.inputs[1]), out, count,
                                             static_cast<std::size_t>(in.height) * in.width, stream_);
            break;
        case Op::clamp:
            status = kernels::clamp(a, node.minimum, node.maximum, out, count, stream_);
            break;
        case Op::crop:
            status = kernels::crop(a, out, out_extent.channels, out_extent.height, out_extent.width, in.height,
                                   in.width, stream_);
            break;
        case Op::concat: {
            const std::size_t head = in.count();
            status = kernels::copy(a, out, head, stream_);
            if (status == cudaSuccess) status = kernels::copy(tensor(node.inputs[1]), out + head, count - head, stream_);
            launched = 0;
            break;
        }
        case Op::im2col:
            status = kernels::im2col(a, out, out_extent.channels, out_extent.height, out_extent.width, in.height,
                                     in.width,
                                     kernels::Window{node.kernel[0], node.kernel[1], node.stride[0], node.stride[1],
                                                     node.pads[0], node.pads[1]},
                                     stream_);
            break;
        }
        break;
    }
    }
    if (status != cudaSuccess) return cuda_error(op_name(node.op), status);
    launches_ += launched;
    double bytes = static_cast<double>(count) * 4.0;
    for (const auto id : step.reads) bytes += static_cast<double>(plan.extents[id].count()) * 4.0;
    return mark(std::string(step.kind == StepKind::chunk_add ? "chunk_add" : op_name(node.op)) + ":" +
                    program_.tensor_names[step.output],
                step.kind == StepKind::chunk_add ? "chunk_add" : op_name(node.op), 0.0, bytes);
}

Status Executor::execute(const std::vector<TensorView>& inputs, const std::vector<TensorView>& outputs,
                         Boundary boundary, void* workspace, std::size_t workspace_bytes) {
    std::vector<Extent> extents;
    std::vector<const TensorView*> input_views;
    for (const auto id : program_.inputs) {
        const auto& name = program_.tensor_names[id];
        const TensorView* view = find_view(inputs, name);
        if (view == nullptr || view->data == nullptr || view->extent.channels != program_.tensor_channels[id] ||
            view->extent.height <= 0 || view->extent.width <= 0) {
            return fail(Code::invalid_argument, program_.name + ": missing or misshapen input " + name);
        }
        extents.push_back(view->extent);
        input_views.push_back(view);
    }
    auto planned = plan_for(extents, boundary);
    if (!planned) return planned.error();
    Plan& plan = *planned.value();
    std::vector<const TensorView*> output_views;
    for (const auto id : program_.outputs) {
        const auto& name = program_.tensor_names[id];
        const TensorView* view = find_view(outputs, name);
        if (view == nullptr || view->data == nullptr || !(view->extent == plan.extents[id])) {
            return fail(Code::invalid_argument, program_.name + ": missing or misshapen output " + name);
        }
        output_views.push_back(view);
    }
    if (workspace == nullptr) {
        auto arena = ensure_arena(plan.arena_bytes);
        if (!arena) return arena;
        run_base_ = static_cast<std::uint8_t*>(arena_);
    } else {
        if (plan.arena_bytes > workspace_bytes) {
            return fail(Code::invalid_argument, program_.name + ": this run needs " + std::to_string(plan.arena_bytes) +
                                                    " bytes of workspace, more than the " +
                                                    std::to_string(workspace_bytes) + " bytes provided");
        }
        run_base_ = static_cast<std::uint8_t*>(workspace);
    }

    // The launch sequence of this run; replayed from a CUDA graph when the same
    // plan, workspace and tensors come again on a device boundary.
    auto enqueue = [&]() -> Status {
        launches_ = 0;
        run_started_ = false;
        auto* base = run_base_;
        // Device runs: integer convs stage their program inputs straight from the
        // caller's buffers and store outputs that nothing reads straight into them.
        const bool device = boundary != Boundary::host;
        run_inputs_.assign(program_.tensor_names.size(), Direct{});
        run_outputs_.assign(steps_.size(), Direct{});
        if (device) {
            for (std::size_t slot = 0; slot < program_.inputs.size(); ++slot) {
                run_inputs_[program_.inputs[slot]] = Direct{input_views[slot]->data, boundary == Boundary::half};
            }
            for (std::size_t slot = 0; slot < program_.outputs.size(); ++slot) {
                if (output_step_[slot] < 0) continue;
                run_outputs_[static_cast<std::size_t>(output_step_[slot])] =
                    Direct{output_views[slot]->data, boundary == Boundary::half};
            }
        }
        auto started = mark("", "", 0.0, 0.0);
        if (!started) return started;
        double input_bytes = 0.0;
        for (std::size_t slot = 0; slot < program_.inputs.size(); ++slot) {
            const auto id = program_.inputs[slot];
            if (device && input_conv_only_[slot]) continue;
            float* target = reinterpret_cast<float*>(base + plan.offsets[id]);
            const std::size_t count = plan.extents[id].count();
            input_bytes += static_cast<double>(count) * 6.0;
            cudaError_t status;
            if (boundary == Boundary::half) {
                status = kernels::half_to_float(static_cast<const std::uint16_t*>(input_views[slot]->data), target, count,
                                                stream_);
                ++launches_;
            } else {
                status = cudaMemcpyAsync(target, input_views[slot]->data, count * sizeof(float),
                                         boundary == Boundary::host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice,
                                         stream_);
            }
            if (status != cudaSuccess) return cuda_error("input conversion", status);
        }
        // Segments only for conversions that ran (staged inputs and direct outputs have none).
        if (input_bytes > 0.0) {
            auto marked = mark("inputs", boundary == Boundary::half ? "half_to_float" : "copy", 0.0, input_bytes);
            if (!marked) return marked;
        }
        for (std::size_t s = 0; s < steps_.size(); ++s) {
            auto launched = launch_step(steps_[s], plan, s);
            if (!launched) return launched;
        }
        double output_bytes = 0.0;
        for (std::size_t slot = 0; slot < program_.outputs.size(); ++slot) {
            const auto id = program_.outputs[slot];
            if (device && output_step_[slot] >= 0) continue;
            const float* source = reinterpret_cast<const float*>(base + plan.offsets[id]);
            const std::size_t count = plan.extents[id].count();
            output_bytes += static_cast<double>(count) * 6.0;
            cudaError_t status;
            if (boundary == Boundary::half) {
                status = kernels::float_to_half(source, static_cast<std::uint16_t*>(output_views[slot]->data), count,
                                                stream_);
                ++launches_;
            } else {
                status = cudaMemcpyAsync(output_views[slot]->data, source, count * sizeof(float),
                                         boundary == Boundary::host ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice,
                                         stream_);
            }
            if (status != cudaSuccess) return cuda_error("output conversion", status);
        }
        if (output_bytes > 0.0) {
            auto marked = mark("outputs", boundary == Boundary::half ? "float_to_half" : "copy", 0.0, output_bytes);
            if (!marked) return marked;
        }
        return Ok{};
    };
    // Runs in a caller's workspace are never captured: instantiating a graph
    // may allocate device memory, which those callers cannot allow.
    if (boundary != Boundary::host && !profiling_ && workspace == nullptr) {
        GraphKey key{&plan, run_base_, static_cast<int>(boundary), {}};
        for (const auto* view : input_views) key.tensors.push_back(view->data);
        for (const auto* view : output_views) key.tensors.push_back(view->data);
        auto replayed = run_graph(key, enqueue);
        if (replayed) return Ok{};
        if (replayed.error().code != Code::try_again) return replayed.error();
    }
    auto enqueued = enqueue();
    if (!enqueued) return enqueued;
    if (boundary == Boundary::host) return synchronize();
    return Ok{};
}

// Runs `enqueue` through a cached CUDA graph for `key`: the first sighting of a
// key runs normally (all lazy set-up happens there) and returns try_again; the
// second is captured (thread-local mode) and replayed; later ones replay. A
// stream the caller is itself capturing is left alone (try_again).
Status Executor::run_graph(const GraphKey& key, const std::function<Status()>& enqueue) {
    cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream_, &capturing) != cudaSuccess || capturing != cudaStreamCaptureStatusNone) {
        cudaGetLastError();
        return fail(Code::try_again, "stream is capturing");
    }
    auto found = graphs_.find(key);
    if (found == graphs_.end()) {
        if (graphs_.size() >= 32) clear_graphs();
        graphs_.emplace(key, CachedGraph{});
        return fail(Code::try_again, "first run of this plan and tensors");
    }
    CachedGraph& cached = found->second;
    if (cached.exec == nullptr) {
        cudaError_t status = cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal);
        if (status != cudaSuccess) return cuda_error("cudaStreamBeginCapture", status);
        capturing_ = true;
        Status enqueued = enqueue();
        capturing_ = false;
        cudaGraph_t graph = nullptr;
        status = cudaStreamEndCapture(stream_, &graph);
        if (!enqueued) {
            if (graph != nullptr) cudaGraphDestroy(graph);
            return enqueued;
        }
        if (status != cudaSuccess || graph == nullptr) {
            if (graph != nullptr) cudaGraphDestroy(graph);
            return cuda_error("cudaStreamEndCapture", status);
        }
        status = cudaGraphInstantiate(&cached.exec, graph, 0);
        cudaGraphDestroy(graph);
        if (status != cudaSuccess) {
            cached.exec = nullptr;
            return cuda_error("cudaGraphInstantiate", status);
        }
        cached.launches = launches_;
    }
    const cudaError_t status = cudaGraphLaunch(cached.exec, stream_);
    if (status != cudaSuccess) return cuda_error("cudaGraphLaunch", status);
    launches_ = cached.launches;
    return Ok{};
}

void Executor::clear_graphs() {
    for (auto& [key, cached] : graphs_) {
        if (cached.exec != nullptr) cudaGraphExecDestroy(cached.exec);
    }
    graphs_.clear();
}

// Records an event on the stream when profiling; the segment since the
// previous event is attributed to `label` (the first call only starts).
// Segments accumulate over runs until profile() collects them, so profiled
// runs need no synchronisation.
Status Executor::mark(const std::string& label, const std::string& kernel, double ops, double bytes) {
    if (!profiling_) return Ok{};
    if (marks_ >= events_.size()) {
        cudaEvent_t event;
        const cudaError_t created = cudaEventCreate(&event);
        if (created != cudaSuccess) return cuda_error("cudaEventCreate", created);
        events_.push_back(event);
    }
    const cudaError_t recorded = cudaEventRecord(events_[marks_], stream_);
    if (recorded != cudaSuccess) return cuda_error("cudaEventRecord", recorded);
    if (run_started_) {
        timings_.push_back(StepTiming{label, kernel, 0.0, ops, bytes});
        segment_starts_.push_back(marks_ - 1);
    }
    run_started_ = true;
    ++marks_;
    return Ok{};
}

Status Executor::run_half(const std::vector<TensorView>& inputs, const std::vector<TensorView>& outputs) {
    return execute(inputs, outputs, Boundary::half);
}

Status Executor::run_half_in_workspace(const std::vector<TensorView>& inputs, const std::vector<TensorView>& outputs,
                                       void* workspace, std::size_t bytes) {
    if (workspace == nullptr) return fail(Code::invalid_argument, "null workspace");
    return execute(inputs, outputs, Boundary::half, workspace, bytes);
}

Status Executor::run_float(const std::vector<TensorView>& inputs, const std::vector<TensorView>& outputs) {
    return execute(inputs, outputs, Boundary::float32);
}

Status Executor::run_host(const std::vector<TensorView>& inputs, const std::vector<TensorView>& outputs) {
    return execute(inputs, outputs, Boundary::host);
}

Status Executor::test_wait_timeout(unsigned int limit_ms) {
    if (limit_ms == 0 || limit_ms > 4000) return fail(Code::invalid_argument, "wait limit must be 1..4000 ms");
    const cudaError_t status =
        kernels::wait_timeout(static_cast<unsigned long long>(limit_ms) * 1000000ull, status_, stream_);
    if (status != cudaSuccess) return cuda_error("wait timeout launch", status);
    return Ok{};
}

Status Executor::synchronize() {
    cudaError_t status = cudaStreamSynchronize(stream_);
    if (status != cudaSuccess) return cuda_error("cudaStreamSynchronize", status);
    unsigned int word = 0;
    status = cudaMemcpy(&word, status_, sizeof(word), cudaMemcpyDeviceToHost);
    if (status != cudaSuccess) return cuda_error("cudaMemcpy status", status);
    if (word != 0) {
        cudaMemset(status_, 0, sizeof(unsigned int));
        return fail(Code::backend_error, "a device-side wait gave up (status word " + std::to_string(word) + ")");
    }
    return Ok{};
}

Result<std::vector<StepTiming>> Executor::profile() {
    auto synced = synchronize();
    if (!synced) return synced.error();
    for (std::size_t i = 0; i < timings_.size(); ++i) {
        float ms = 0.0f;
        const std::size_t first = segment_starts_[i];
        const cudaError_t status = cudaEventElapsedTime(&ms, events_[first], events_[first + 1]);
        if (status != cudaSuccess) return cuda_error("cudaEventElapsedTime", status);
        timings_[i].milliseconds = ms;
    }
    std::vector<StepTiming> collected;
    collected.swap(timings_);
    segment_starts_.clear();
    marks_ = 0;
    return collected;
}

}  // namespace nvcr_sm100
