// Internal C++ interfaces of the B200 montlok runtime. Consumers use the C ABI
// in include/montlok/montlok.h; this header joins the loader, the tree
// compiler and the CUDA layer (csrc/cuda/mlk_cuda.h) behind it.
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <string_view>
#include <vector>

#include "json.hpp"

namespace mlk {

// The values of montlok_status (include/montlok/montlok.h).
enum class Status : int {
    Ok = 0,
    InvalidArgument = 1,
    Io = 2,
    Format = 3,
    Unsupported = 4,
    Shape = 5,
    State = 6,
    Internal = 7,
};

class Error : public std::runtime_error {
public:
    Error(Status status, const std::string& message) : std::runtime_error(message), status_(status) {}
    Status status() const noexcept { return status_; }

private:
    Status status_;
};

[[noreturn]] inline void fail(Status status, const std::string& message) { throw Error(status, message); }

const char* version() noexcept;

// ---------------------------------------------------------------------------
// Model files: safetensors with the spec in __metadata__["montlok"]
// (reference src/core/archive.cpp).
// ---------------------------------------------------------------------------

enum class DType : uint8_t { F64 = 1, F32 = 2, I64 = 3, I32 = 4, U8 = 5, Bool = 6 };

struct Tensor {
    std::string name;
    DType dtype;
    std::vector<int64_t> shape;
    const uint8_t* data;
    size_t nbytes;
    size_t numel() const noexcept;
    std::string describe() const;
};

class Archive {
public:
    static std::shared_ptr<const Archive> from_file(const std::string& path);
    static std::shared_ptr<const Archive> from_bytes(const void* data, size_t size);

    const json::Value& spec() const noexcept { return spec_; }
    const std::string& spec_text() const noexcept { return spec_text_; }
    const Tensor* find(std::string_view name) const noexcept;

    // Typed copies of a tensor whose shape matches `shape` (-1: any extent).
    // f64 accepts F64/F32, i32 accepts I32/I64 (range-checked), u8 U8/BOOL.
    std::vector<double> f64(std::string_view name, const std::vector<int64_t>& shape) const;
    std::vector<int32_t> i32(std::string_view name, const std::vector<int64_t>& shape) const;
    std::vector<uint8_t> u8(std::string_view name, const std::vector<int64_t>& shape) const;

private:
    void parse();
    const Tensor& checked(std::string_view name, const std::vector<int64_t>& shape) const;

    std::vector<uint8_t> bytes_;
    std::vector<Tensor> tensors_;
    json::Value spec_;
    std::string spec_text_;
};

size_t json_size(const json::Value& object, std::string_view key, size_t fallback);
double json_double(const json::Value& object, std::string_view key, double fallback);
std::string json_string(const json::Value& object, std::string_view key, const std::string& fallback);

// ---------------------------------------------------------------------------
// The tree_ensemble family compiled for the GPU.
// ---------------------------------------------------------------------------

enum class Link : int32_t { Identity = 0, Sigmoid = 1, Softmax = 2, Exp = 3 };

// Where a split reads its feature: the variant of the prepared row that
// encodes the split's missing-value rule (see forest.cpp).
enum Variant : int { kNanRight = 0, kNanLeft = 1, kZeroRight = 2, kZeroLeft = 3, kVariants = 4 };

struct ForestImage {
    // Shape and semantics.
    int32_t features = 0, outputs = 0, trees = 0, nodes = 0;
    bool decision_le = true, cast_f32 = false, mean = false;
    Link link = Link::Identity;
    double sigmoid_scale = 1.0;
    std::vector<double> base;      // [outputs]
    std::vector<int32_t> counts;   // [outputs] trees adding to each output

    // Prepared-row slots: slot_of[f * 4 + variant] = slot, or -1 when no split
    // reads that variant of feature f. Slot `pad_slot` always reads "left".
    int32_t slots = 0, pad_slot = 0;
    std::vector<int32_t> slot_of;

    // Nodes in file order, each four words: the key threshold T (go right when
    // key(value) > T), the slot, the left and the right child; a leaf loops
    // to itself and reads the pad slot.
    std::vector<int32_t> node_words;  // [nodes * 4]
    std::vector<double> leaf_value;   // [nodes], 0 for splits
    std::vector<int32_t> roots, depth, tree_output;  // [trees]

    // The exact rule of each split, read when a float64 model's float32 key of
    // the value equals the threshold's key.
    std::vector<double> threshold;    // [nodes]
    std::vector<int32_t> feature;     // [nodes], -1 for leaves
    std::vector<uint8_t> flags;       // [nodes]

    // Complete-tree view: every tree as a complete binary tree of
    // `complete_depth` levels in heap order (children of i at 2i+1, 2i+2),
    // shallower leaves padded with splits that always go left. Built for
    // single-output models of depth <= 8; complete_depth is 0 otherwise.
    int32_t complete_depth = 0;
    std::vector<int32_t> heap_words;    // [trees * (2^d - 1) * 2]: T, slot
    std::vector<int32_t> heap_node_id;  // [trees * (2^d - 1)]: file node, -1 for padding
    std::vector<double> heap_leaf;      // [trees * 2^d]
    std::vector<int32_t> heap_leaf_id;  // [trees * 2^d]: file node of each leaf
    bool heap_leaf_f32 = false;         // every leaf value is exactly a float
};

// Builds the image from a validated spec/archive; throws Error like the
// reference constructor (src/core/trees.cpp:70-156).
std::unique_ptr<ForestImage> build_forest(const Archive& archive, const json::Value& spec, const json::Value& config,
                                          size_t features, size_t sequence);

// ---------------------------------------------------------------------------
// Models
// ---------------------------------------------------------------------------

enum class InputType : uint8_t { F32 = 1, F64 = 2 };

struct Preprocess {
    bool standardize = false, clip = false;
    std::vector<double> mean, scale;
    double lo = 0, hi = 0;
};

class DeviceSet;

class Model {
public:
    static std::shared_ptr<const Model> open(const std::string& path);
    static std::shared_ptr<const Model> from_bytes(const void* data, size_t size);
    ~Model();

    size_t features() const noexcept { return features_; }
    size_t sequence() const noexcept { return sequence_; }
    size_t outputs() const noexcept { return outputs_; }
    bool has_preprocess() const noexcept { return pre_.standardize || pre_.clip; }
    const std::string& family() const noexcept { return family_; }
    const std::string& spec_text() const noexcept { return archive_->spec_text(); }
    const ForestImage& forest() const noexcept { return *forest_; }
    const Preprocess& preprocess() const noexcept { return pre_; }

    // Host buffers (the reference contract); rows are sharded over the
    // devices selected with set_devices().
    void predict(InputType type, const void* x, size_t batch, double* out) const;
    // Device buffers on the current device, work queued on `stream`.
    void predict_device(InputType type, const void* x, size_t batch, double* out, void* stream) const;
    // predict_device with no allocation at all (static scratch; the model
    // must already be resident on the current device).
    void predict_device_noalloc(InputType type, const void* x, size_t batch, double* out, void* stream) const;
    // Leaf node index of every (row, tree); host or device buffers.
    void predict_leaves(InputType type, const void* x, size_t batch, int32_t* leaves, bool device,
                        void* stream) const;
    // Throws Error(Internal) when a device-buffer call on the current device
    // gave up a bounded wait since the last check, and clears that record.
    void check_device_status() const;
    // The kernel a predict of `batch` rows runs on the current device
    // (uploads the model there first).
    const char* kernel_name(size_t batch) const;

private:
    explicit Model(std::shared_ptr<const Archive> archive);
    static std::shared_ptr<const Model> build(std::shared_ptr<const Archive> archive);
    void check_call(InputType type, const void* x, const void* out) const;

    std::shared_ptr<const Archive> archive_;
    std::string family_;
    size_t features_ = 0, sequence_ = 0, outputs_ = 0;
    Preprocess pre_;
    std::unique_ptr<ForestImage> forest_;
    std::unique_ptr<DeviceSet> devices_;
};

// Library-wide settings.
void set_threads(int threads) noexcept;
int threads() noexcept;
void set_latency_threads(int threads);
int latency_threads() noexcept;
// GPUs a host-buffer predict spreads its rows over: 0 = the current device
// only (the default), n = devices 0..n-1 (capped at the devices present).
void set_devices(int count);
int devices() noexcept;

}  // namespace mlk
