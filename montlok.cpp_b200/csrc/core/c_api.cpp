// extern "C" implementation of include/montlok/montlok.h. Each entry point
// maps exceptions to a status and the calling thread's last error, as the
// reference's guard() does (src/core/c_api.cpp:33-51).
#include <chrono>
#include <new>
#include <string>
#include <vector>

#include "../cuda/mlk_cuda.h"
#include "montlok/montlok.h"
#include "runtime.hpp"

struct montlok_model {
    std::shared_ptr<const mlk::Model> impl;
};

struct montlok_stream {
    std::shared_ptr<const mlk::Model> model;
    size_t batch;
};

namespace {

using mlk::Error;
using mlk::Status;

thread_local std::string t_error;

void set_error(const char* message) noexcept {
    try {
        t_error = message;
    } catch (...) {
    }
}

template <typename F>
int guard(F&& f) noexcept {
    try {
        f();
        return MONTLOK_OK;
    } catch (const Error& e) {
        set_error(e.what());
        return static_cast<int>(e.status());
    } catch (const std::bad_alloc&) {
        set_error("out of memory");
        return MONTLOK_ERROR_INTERNAL;
    } catch (const std::exception& e) {
        set_error(e.what());
        return MONTLOK_ERROR_INTERNAL;
    } catch (...) {
        set_error("unknown error");
        return MONTLOK_ERROR_INTERNAL;
    }
}

mlk::InputType input_type(montlok_dtype dtype) {
    if (dtype == MONTLOK_FLOAT32) return mlk::InputType::F32;
    if (dtype == MONTLOK_FLOAT64) return mlk::InputType::F64;
    throw Error(Status::InvalidArgument, "dtype must be MONTLOK_FLOAT32 or MONTLOK_FLOAT64");
}

void require(bool ok, const char* what) {
    if (!ok) throw Error(Status::InvalidArgument, what);
}

}  // namespace

extern "C" {

uint32_t montlok_abi_version(void) { return MONTLOK_ABI_VERSION; }

const char* montlok_version(void) { return mlk::version(); }

const char* montlok_last_error(void) { return t_error.c_str(); }

void montlok_set_threads(int threads) { mlk::set_threads(threads); }

int montlok_threads(void) { return mlk::threads(); }

int montlok_set_latency_threads(int threads) {
    return guard([&] { mlk::set_latency_threads(threads); });
}

int montlok_latency_threads(void) { return mlk::latency_threads(); }

const char* montlok_families(void) { return "tree_ensemble"; }

int montlok_model_open(const char* path, montlok_model** model) {
    if (model) *model = nullptr;
    return guard([&] {
        require(path && model, "null argument");
        auto handle = std::make_unique<montlok_model>();
        handle->impl = mlk::Model::open(path);
        *model = handle.release();
    });
}

int montlok_model_open_memory(const void* data, size_t size, montlok_model** model) {
    if (model) *model = nullptr;
    return guard([&] {
        require(model != nullptr && (data != nullptr || size == 0), "null argument");
        auto handle = std::make_unique<montlok_model>();
        handle->impl = mlk::Model::from_bytes(data, size);
        *model = handle.release();
    });
}

void montlok_model_close(montlok_model* model) { delete model; }

int montlok_model_get_info(const montlok_model* model, montlok_model_info* info) {
    return guard([&] {
        require(model && info, "null argument");
        const mlk::Model& m = *model->impl;
        info->features = static_cast<uint32_t>(m.features());
        info->sequence = static_cast<uint32_t>(m.sequence());
        info->outputs = static_cast<uint32_t>(m.outputs());
        info->flags = MONTLOK_MODEL_STREAMABLE | (m.has_preprocess() ? MONTLOK_MODEL_PREPROCESS : 0u);
    });
}

const char* montlok_model_family(const montlok_model* model) { return model ? model->impl->family().c_str() : ""; }

const char* montlok_model_spec(const montlok_model* model) { return model ? model->impl->spec_text().c_str() : ""; }

int montlok_model_predict(const montlok_model* model, montlok_dtype dtype, const void* x, size_t batch, double* out) {
    return guard([&] {
        require(model != nullptr, "null model");
        model->impl->predict(input_type(dtype), x, batch, out);
    });
}

int montlok_stream_open(const montlok_model* model, size_t batch, montlok_stream** stream) {
    if (stream) *stream = nullptr;
    return guard([&] {
        require(model && stream, "null argument");
        if (batch == 0 || batch > (size_t(1) << 24)) throw Error(Status::InvalidArgument, "stream batch must be in [1, 2^24]");
        *stream = new montlok_stream{model->impl, batch};
    });
}

int montlok_stream_step(montlok_stream* stream, montlok_dtype dtype, const void* x, double* out) {
    return guard([&] {
        require(stream != nullptr, "null stream");
        const mlk::InputType type = input_type(dtype);
        if (!x || !out) throw Error(Status::InvalidArgument, "null input or output buffer");
        stream->model->predict(type, x, stream->batch, out);
    });
}

int montlok_stream_reset(montlok_stream* stream) {
    return guard([&] { require(stream != nullptr, "null stream"); });
}

void montlok_stream_close(montlok_stream* stream) { delete stream; }

int montlok_register_family(const montlok_family_v1*) {
    return guard([] { throw Error(Status::Unsupported, "plugin families are not part of the GPU build"); });
}

int montlok_plugin_load(const char*) {
    return guard([] { throw Error(Status::Unsupported, "plugin families are not part of the GPU build"); });
}

int montlok_model_predict_device(const montlok_model* model, montlok_dtype dtype, const void* x, size_t batch,
                                 double* out, void* stream) {
    return guard([&] {
        require(model != nullptr, "null model");
        model->impl->predict_device(input_type(dtype), x, batch, out, stream);
    });
}

int montlok_model_predict_device_noalloc(const montlok_model* model, montlok_dtype dtype, const void* x,
                                         size_t batch, double* out, void* stream) {
    return guard([&] {
        require(model != nullptr, "null model");
        model->impl->predict_device_noalloc(input_type(dtype), x, batch, out, stream);
    });
}

int montlok_model_predict_leaves(const montlok_model* model, montlok_dtype dtype, const void* x, size_t batch,
                                 int32_t* leaves) {
    return guard([&] {
        require(model != nullptr, "null model");
        model->impl->predict_leaves(input_type(dtype), x, batch, leaves, false, nullptr);
    });
}

int montlok_model_predict_leaves_device(const montlok_model* model, montlok_dtype dtype, const void* x, size_t batch,
                                        int32_t* leaves, void* stream) {
    return guard([&] {
        require(model != nullptr, "null model");
        model->impl->predict_leaves(input_type(dtype), x, batch, leaves, true, stream);
    });
}

int montlok_model_device_status(const montlok_model* model) {
    return guard([&] {
        require(model != nullptr, "null model");
        model->impl->check_device_status();
    });
}

int montlok_model_kernel(const montlok_model* model, size_t batch, const char** name) {
    if (name) *name = "";
    return guard([&] {
        require(model && name, "null argument");
        *name = model->impl->kernel_name(batch);
    });
}

int montlok_model_trees(const montlok_model* model, uint32_t* trees) {
    return guard([&] {
        require(model && trees, "null argument");
        *trees = static_cast<uint32_t>(model->impl->forest().trees);
    });
}

int montlok_set_devices(int count) {
    return guard([&] { mlk::set_devices(count); });
}

int montlok_devices(void) { return mlk::devices(); }

int montlok_bench_predict(const montlok_model* model, montlok_dtype dtype, const void* rows, size_t count,
                          size_t batch, size_t iterations, size_t warmup, double* samples_ns, double* mean_ns) {
    return guard([&] {
        require(model && rows && samples_ns && mean_ns && count && batch && iterations, "bad bench arguments");
        const mlk::InputType type = input_type(dtype);
        const mlk::Model& m = *model->impl;
        const size_t width = batch * m.features() * (type == mlk::InputType::F32 ? 4 : 8);
        std::vector<double> out(batch * m.outputs());
        auto call = [&](size_t i) {
            m.predict(type, static_cast<const char*>(rows) + (i % count) * width, batch, out.data());
        };
        using Clock = std::chrono::steady_clock;
        for (size_t i = 0; i < warmup; ++i) call(i);
        for (size_t i = 0; i < iterations; ++i) {
            const auto t0 = Clock::now();
            call(i);
            samples_ns[i] = std::chrono::duration<double, std::nano>(Clock::now() - t0).count();
        }
        const auto t0 = Clock::now();
        for (size_t i = 0; i < iterations; ++i) call(i);
        *mean_ns = std::chrono::duration<double, std::nano>(Clock::now() - t0).count() / static_cast<double>(iterations);
    });
}

int montlok_device_count(void) {
    int count = 0;
    char err[256];
    if (mlk_cuda_device_count(&count, err, sizeof err) != 0) return 0;
    return count;
}

}  // extern "C"
