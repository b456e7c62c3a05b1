// Model: spec validation and preprocess (reference src/core/runtime.cpp:443-530),
// the tree_ensemble family, and the predict drivers that hand rows to the
// CUDA layer. There is no CPU evaluation path: without a usable GPU every
// predict returns MONTLOK_ERROR_INTERNAL with the CUDA error.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <functional>
#include <thread>

#include "../cuda/mlk_cuda.h"
#include "runtime.hpp"

namespace mlk {

const char* version() noexcept { return "0.2.0"; }

namespace {

constexpr size_t kMaxExtent = size_t(1) << 24;
constexpr size_t kErr = 512;

std::atomic<int> g_threads{0};
std::atomic<int> g_latency_threads{0};
std::atomic<int> g_devices{0};

const json::Value& empty_object() {
    static const json::Value value = json::Value::parse("{}");
    return value;
}

void check_cuda(int status, const char* err) {
    if (status != 0) fail(static_cast<Status>(status), err);
}

// One long-lived host thread per GPU for host-buffer predicts split over
// devices (set_devices): each keeps its own CUDA workspace (streams, device
// buffers, pinned staging) from call to call, so a sharded call allocates
// nothing once every worker has served one call of its size. Calls from
// several threads queue per device.
class DeviceWorkers {
public:
    static DeviceWorkers& get() {
        static DeviceWorkers* workers = new DeviceWorkers();  // never destroyed: workers may be busy at exit
        return *workers;
    }

    // Runs jobs[d] on device d's worker for every d, and returns when all ran.
    void run(std::vector<std::function<void()>>& jobs) {
        struct Pending {
            std::mutex mu;
            std::condition_variable cv;
            size_t left;
        } pending;
        pending.left = jobs.size();
        for (size_t d = 0; d < jobs.size(); ++d) {
            Worker& w = worker(static_cast<int>(d));
            std::lock_guard<std::mutex> lock(w.mu);
            w.queue.push_back([&pending, &jobs, d] {
                jobs[d]();
                std::lock_guard<std::mutex> done(pending.mu);
                if (--pending.left == 0) pending.cv.notify_all();
            });
            w.cv.notify_one();
        }
        std::unique_lock<std::mutex> lock(pending.mu);
        pending.cv.wait(lock, [&] { return pending.left == 0; });
    }

private:
    struct Worker {
        std::mutex mu;
        std::condition_variable cv;
        std::deque<std::function<void()>> queue;
    };

    Worker& worker(int device) {
        std::lock_guard<std::mutex> lock(mu_);
        while (static_cast<int>(workers_.size()) <= device) {
            workers_.push_back(std::make_unique<Worker>());
            Worker* w = workers_.back().get();
            std::thread([w] {
                for (;;) {
                    std::function<void()> job;
                    {
                        std::unique_lock<std::mutex> lock(w->mu);
                        w->cv.wait(lock, [&] { return !w->queue.empty(); });
                        job = std::move(w->queue.front());
                        w->queue.pop_front();
                    }
                    job();
                }
            }).detach();
        }
        return *workers_[static_cast<size_t>(device)];
    }

    std::mutex mu_;
    std::vector<std::unique_ptr<Worker>> workers_;
};

}  // namespace

void set_threads(int threads) noexcept {
    g_threads.store(std::max(threads, 0));
    const int n = threads > 0 ? threads : static_cast<int>(std::thread::hardware_concurrency());
    mlk_cuda_set_copy_threads(std::clamp(n, 1, 256));
}

int threads() noexcept {
    const int n = g_threads.load();
    return std::clamp(n > 0 ? n : static_cast<int>(std::thread::hardware_concurrency()), 1, 256);
}

void set_latency_threads(int threads) {
    if (threads < 0 || threads > 256) fail(Status::InvalidArgument, "latency threads must be in [0, 256]");
    g_latency_threads.store(threads);
    mlk_cuda_set_latency_engine(threads > 0 ? 1 : 0);
}

int latency_threads() noexcept { return g_latency_threads.load(); }

void set_devices(int count) {
    if (count < 0 || count > 1024) fail(Status::InvalidArgument, "device count must be in [0, 1024]");
    g_devices.store(count);
}

int devices() noexcept { return g_devices.load(); }

// The forest's replicas, uploaded to each device on first use.
class DeviceSet {
public:
    DeviceSet(const ForestImage& img, const Preprocess& pre) : img_(img), pre_(pre) {
        v_ = mlk_forest_view{};
        v_.features = img.features;
        v_.outputs = img.outputs;
        v_.trees = img.trees;
        v_.nodes = img.nodes;
        v_.slots = img.slots;
        v_.pad_slot = img.pad_slot;
        v_.decision_le = img.decision_le;
        v_.cast_f32 = img.cast_f32;
        v_.mean = img.mean;
        v_.link = static_cast<int32_t>(img.link);
        v_.sigmoid_scale = img.sigmoid_scale;
        v_.base = img.base.data();
        v_.counts = img.counts.data();
        v_.slot_of = img.slot_of.data();
        v_.node_words = img.node_words.data();
        v_.leaf_value = img.leaf_value.data();
        v_.roots = img.roots.data();
        v_.depth = img.depth.data();
        v_.tree_output = img.tree_output.data();
        v_.threshold = img.threshold.data();
        v_.feature = img.feature.data();
        v_.flags = img.flags.data();
        v_.standardize = pre.standardize;
        v_.clip = pre.clip;
        v_.pre_mean = pre.standardize ? pre.mean.data() : nullptr;
        v_.pre_scale = pre.standardize ? pre.scale.data() : nullptr;
        v_.clip_lo = pre.lo;
        v_.clip_hi = pre.hi;
        v_.complete_depth = img.complete_depth;
        v_.heap_leaf_f32 = img.heap_leaf_f32;
        v_.heap_words = img.heap_words.empty() ? nullptr : img.heap_words.data();
        v_.heap_node_id = img.heap_node_id.empty() ? nullptr : img.heap_node_id.data();
        v_.heap_leaf = img.heap_leaf.empty() ? nullptr : img.heap_leaf.data();
        v_.heap_leaf_id = img.heap_leaf_id.empty() ? nullptr : img.heap_leaf_id.data();
    }

    ~DeviceSet() {
        for (mlk_dev_forest* f : replicas_) mlk_cuda_forest_release(f);
    }

    const mlk_dev_forest* on(int device) {
        std::lock_guard<std::mutex> lock(mu_);
        if (device < 0) fail(Status::Internal, "invalid CUDA device");
        if (static_cast<size_t>(device) >= replicas_.size()) replicas_.resize(static_cast<size_t>(device) + 1, nullptr);
        if (!replicas_[device]) {
            char err[kErr] = {0};
            mlk_dev_forest* f = nullptr;
            check_cuda(mlk_cuda_forest_upload(device, &v_, &f, err, sizeof err), err);
            replicas_[device] = f;
        }
        return replicas_[device];
    }

    // The replica on `device` if one was uploaded; never uploads (allocates).
    const mlk_dev_forest* find(int device) {
        std::lock_guard<std::mutex> lock(mu_);
        if (device < 0 || static_cast<size_t>(device) >= replicas_.size()) return nullptr;
        return replicas_[device];
    }

private:
    const ForestImage& img_;
    const Preprocess& pre_;
    mlk_forest_view v_;
    std::mutex mu_;
    std::vector<mlk_dev_forest*> replicas_;
};

Model::Model(std::shared_ptr<const Archive> archive) : archive_(std::move(archive)) {
    const json::Value& spec = archive_->spec();
    family_ = json_string(spec, "family", "");
    if (family_.empty()) fail(Status::Format, "model spec has no \"family\"");
    const json::Value* inputs = spec.find("inputs");
    const json::Value* outputs = spec.find("outputs");
    if (!inputs || !inputs->is_object()) fail(Status::Format, "model spec has no \"inputs\" object");
    if (!outputs || !outputs->is_object()) fail(Status::Format, "model spec has no \"outputs\" object");
    const size_t features = json_size(*inputs, "features", 0);
    const size_t sequence = json_size(*inputs, "sequence", 0);
    const size_t output_size = json_size(*outputs, "size", 0);
    if (features == 0 || features > kMaxExtent) fail(Status::Format, "inputs.features must be in [1, 2^24]");
    if (sequence > kMaxExtent || features * std::max<size_t>(sequence, 1) > (size_t(1) << 28)) {
        fail(Status::Format, "inputs.sequence is too large");
    }
    if (output_size == 0 || output_size > kMaxExtent) fail(Status::Format, "outputs.size must be in [1, 2^24]");
    if (const json::Value* names = inputs->find("names");
        names && !names->is_null() && (!names->is_array() || names->as_array().size() != features)) {
        fail(Status::Format, "inputs.names must list one name per feature");
    }

    if (const json::Value* pre = spec.find("preprocess"); pre && !pre->is_null()) {
        if (!pre->is_object()) fail(Status::Format, "\"preprocess\" must be an object");
        const json::Value* mean = pre->find("mean");
        const json::Value* scale = pre->find("scale");
        const bool has_mean = mean && !mean->is_null();
        const bool has_scale = scale && !scale->is_null();
        if (has_mean != has_scale) fail(Status::Format, "preprocess needs both \"mean\" and \"scale\"");
        if (has_mean) {
            if (!mean->is_string() || !scale->is_string()) fail(Status::Format, "preprocess mean/scale name tensors in the file");
            const auto f = static_cast<int64_t>(features);
            pre_.mean = archive_->f64(mean->as_string(), {f});
            pre_.scale = archive_->f64(scale->as_string(), {f});
            for (size_t i = 0; i < features; ++i) {
                if (!std::isfinite(pre_.mean[i]) || !std::isfinite(pre_.scale[i]) || !(pre_.scale[i] > 0)) {
                    fail(Status::Format, "preprocess mean must be finite and scale finite and positive");
                }
            }
            pre_.standardize = true;
        }
        if (const json::Value* clip = pre->find("clip"); clip && !clip->is_null()) {
            if (!clip->is_array() || clip->as_array().size() != 2 || !clip->as_array()[0].is_number() ||
                !clip->as_array()[1].is_number()) {
                fail(Status::Format, "preprocess.clip must be [low, high]");
            }
            pre_.lo = clip->as_array()[0].as_number();
            pre_.hi = clip->as_array()[1].as_number();
            if (!(pre_.lo < pre_.hi)) fail(Status::Format, "preprocess.clip needs low < high");
            pre_.clip = true;
        }
    }

    if (family_ != "tree_ensemble") {
        fail(Status::Unsupported, "unknown model family \"" + family_ +
                                      "\" (registered: tree_ensemble; this build runs tree ensembles on the GPU)");
    }
    const json::Value* config = spec.find("config");
    if (config && !config->is_null() && !config->is_object()) fail(Status::Format, "\"config\" must be an object");
    forest_ = build_forest(*archive_, spec, config && config->is_object() ? *config : empty_object(), features, sequence);
    features_ = features;
    sequence_ = sequence;
    outputs_ = output_size;
    devices_ = std::make_unique<DeviceSet>(*forest_, pre_);
}

Model::~Model() = default;

std::shared_ptr<const Model> Model::build(std::shared_ptr<const Archive> archive) {
    return std::shared_ptr<const Model>(new Model(std::move(archive)));
}

std::shared_ptr<const Model> Model::open(const std::string& path) { return build(Archive::from_file(path)); }

std::shared_ptr<const Model> Model::from_bytes(const void* data, size_t size) {
    return build(Archive::from_bytes(data, size));
}

void Model::check_call(InputType type, const void* x, const void* out) const {
    if (!x || !out) fail(Status::InvalidArgument, "null input or output buffer");
    if (type != InputType::F32 && type != InputType::F64) fail(Status::InvalidArgument, "unknown input dtype");
}

void Model::predict(InputType type, const void* x, size_t batch, double* out) const {
    if (batch == 0) return;
    check_call(type, x, out);
    char err[kErr] = {0};
    int count = 0;
    check_cuda(mlk_cuda_device_count(&count, err, sizeof err), err);
    int current = 0;
    check_cuda(mlk_cuda_current_device(&current, err, sizeof err), err);
    const int dtype = static_cast<int>(type);
    const size_t row_bytes = features_ * (type == InputType::F32 ? 4 : 8);
    int use = devices();
    use = use <= 0 ? 1 : std::min(use, count);
    // Rows in contiguous slices, one per device; each device writes its own
    // slice of `out`, so no gather step is needed.
    const size_t per = (batch + static_cast<size_t>(use) - 1) / static_cast<size_t>(use);
    if (use == 1 || per == 0) {
        const mlk_dev_forest* f = devices_->on(use == 1 && devices() <= 0 ? current : 0);
        check_cuda(mlk_cuda_predict_host(f, dtype, x, batch, out, err, sizeof err), err);
        return;
    }
    std::vector<const mlk_dev_forest*> replicas(static_cast<size_t>(use));
    for (int d = 0; d < use; ++d) replicas[d] = devices_->on(d);
    std::vector<int> status(static_cast<size_t>(use), 0);
    std::vector<std::string> message(static_cast<size_t>(use));
    const char* inject = std::getenv("MONTLOK_FAULT_INJECT");
    const bool fail_shard = inject && std::strcmp(inject, "shard") == 0;
    std::vector<std::function<void()>> jobs(static_cast<size_t>(use));
    for (int d = 0; d < use; ++d) {
        const size_t lo = std::min(batch, static_cast<size_t>(d) * per), hi = std::min(batch, lo + per);
        jobs[d] = [&, d, lo, hi] {
            if (lo >= hi) return;
            char e[kErr] = {0};
            if (fail_shard && d == use - 1) {
                status[d] = static_cast<int>(Status::Internal);
                message[d] = "injected shard failure (MONTLOK_FAULT_INJECT=shard)";
                return;
            }
            status[d] = mlk_cuda_predict_host(replicas[d], dtype, static_cast<const char*>(x) + lo * row_bytes, hi - lo,
                                              out + lo * outputs_, e, sizeof e);
            message[d] = e;
        };
    }
    DeviceWorkers::get().run(jobs);
    for (int d = 0; d < use; ++d) {
        if (status[d] != 0) fail(static_cast<Status>(status[d]), "device " + std::to_string(d) + ": " + message[d]);
    }
}

void Model::predict_device(InputType type, const void* x, size_t batch, double* out, void* stream) const {
    if (batch == 0) return;
    check_call(type, x, out);
    char err[kErr] = {0};
    int count = 0, current = 0;
    check_cuda(mlk_cuda_device_count(&count, err, sizeof err), err);
    check_cuda(mlk_cuda_current_device(&current, err, sizeof err), err);
    check_cuda(mlk_cuda_predict_device(devices_->on(current), static_cast<int>(type), x, batch, out, stream, err,
                                       sizeof err),
               err);
}

void Model::predict_device_noalloc(InputType type, const void* x, size_t batch, double* out, void* stream) const {
    if (batch == 0) return;
    check_call(type, x, out);
    char err[kErr] = {0};
    int current = 0;
    check_cuda(mlk_cuda_current_device(&current, err, sizeof err), err);
    const mlk_dev_forest* f = devices_->find(current);
    if (!f) {
        fail(Status::State, "the model is not resident on CUDA device " + std::to_string(current) +
                                " yet: one montlok_model_predict or montlok_model_predict_device call there uploads it "
                                "(those calls allocate), after which the no-allocation entry point can run");
    }
    check_cuda(mlk_cuda_predict_device_noalloc(f, static_cast<int>(type), x, batch, out, stream, err, sizeof err), err);
}

void Model::check_device_status() const {
    char err[kErr] = {0};
    int current = 0;
    check_cuda(mlk_cuda_current_device(&current, err, sizeof err), err);
    const mlk_dev_forest* f = devices_->find(current);
    if (f && mlk_cuda_forest_status(f, 1) != 0) {
        fail(Status::Internal, "a device-buffer predict on CUDA device " + std::to_string(current) +
                                   " gave up waiting for its tree data (bounded wait ran out); its rows were not "
                                   "written");
    }
}

const char* Model::kernel_name(size_t batch) const {
    char err[kErr] = {0};
    int count = 0, current = 0;
    check_cuda(mlk_cuda_device_count(&count, err, sizeof err), err);
    check_cuda(mlk_cuda_current_device(&current, err, sizeof err), err);
    return mlk_cuda_kernel_name(devices_->on(current), batch);
}

void Model::predict_leaves(InputType type, const void* x, size_t batch, int32_t* leaves, bool device,
                           void* stream) const {
    if (batch == 0) return;
    check_call(type, x, leaves);
    char err[kErr] = {0};
    int count = 0, current = 0;
    check_cuda(mlk_cuda_device_count(&count, err, sizeof err), err);
    check_cuda(mlk_cuda_current_device(&current, err, sizeof err), err);
    const mlk_dev_forest* f = devices_->on(current);
    if (device) {
        check_cuda(mlk_cuda_leaves_device(f, static_cast<int>(type), x, batch, leaves, stream, err, sizeof err), err);
    } else {
        check_cuda(mlk_cuda_leaves_host(f, static_cast<int>(type), x, batch, leaves, err, sizeof err), err);
    }
}

}  // namespace mlk
