/*
 * montlok.h - C ABI of the B200 montlok runtime (tree ensembles on the GPU).
 *
 * Drop-in for the model API of montlok.cpp's include/montlok/montlok.h:
 * the same types, status codes, entry points and semantics, so the Python
 * package, C++ clients (montlok.hpp) and FFI bindings written against
 * MONTLOK_ABI_VERSION 1 link unchanged. Models are safetensors files whose
 * __metadata__["montlok"] holds the spec (schema "montlok.model/1"); this
 * build runs the "tree_ensemble" family on NVIDIA B200 GPUs (sm_100a).
 *
 * A loaded model is immutable and may be used from any number of threads at
 * once: every calling thread gets its own CUDA streams and buffers. Every
 * function that can fail returns a montlok_status; montlok_last_error()
 * gives the message of the calling thread's last failure. There is no CPU
 * fallback: on a machine without a usable GPU, predict calls fail with
 * MONTLOK_ERROR_INTERNAL (loading and validation still work).
 *
 * Entry points marked "additive" are not in the reference ABI; they add
 * device-resident buffers, leaf indices and multi-GPU sharding without
 * changing any reference entry point, so ABI version 1 stays valid.
 */
#ifndef MONTLOK_H
#define MONTLOK_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__) || defined(__clang__)
#define MONTLOK_API __attribute__((visibility("default")))
#else
#define MONTLOK_API
#endif

#define MONTLOK_ABI_VERSION 1u

/* Reference: include/montlok/montlok.h:43-52. */
typedef enum montlok_status {
    MONTLOK_OK = 0,
    MONTLOK_ERROR_INVALID_ARGUMENT = 1,
    MONTLOK_ERROR_IO = 2,
    MONTLOK_ERROR_FORMAT = 3,
    MONTLOK_ERROR_UNSUPPORTED = 4,
    MONTLOK_ERROR_SHAPE = 5,
    MONTLOK_ERROR_STATE = 6,
    MONTLOK_ERROR_INTERNAL = 7
} montlok_status;

/* Reference: montlok.h:54-57. */
typedef enum montlok_dtype { MONTLOK_FLOAT32 = 1, MONTLOK_FLOAT64 = 2 } montlok_dtype;

typedef struct montlok_model montlok_model;
typedef struct montlok_stream montlok_stream;

#define MONTLOK_MODEL_STREAMABLE 1u /* stream_* accepted (tree models: stateless) */
#define MONTLOK_MODEL_PREPROCESS 2u /* the model standardizes and clips inputs itself */

/* Reference: montlok.h:68-73. */
typedef struct montlok_model_info {
    uint32_t features;
    uint32_t sequence;
    uint32_t outputs;
    uint32_t flags;
} montlok_model_info;

/* Replaces montlok.h:75-77 (c_api.cpp:67-71). */
MONTLOK_API uint32_t montlok_abi_version(void);
MONTLOK_API const char* montlok_version(void);
MONTLOK_API const char* montlok_last_error(void);

/* Replaces montlok.h:80-81. Host threads used to stage pageable inputs into
 * pinned memory; 0 means one per hardware thread. */
MONTLOK_API void montlok_set_threads(int threads);
MONTLOK_API int montlok_threads(void);

/* Replaces montlok.h:87-88. Accepted for compatibility ([0, 256], otherwise
 * MONTLOK_ERROR_INVALID_ARGUMENT) and reported back; single rows run on the
 * GPU, so no spinning CPU threads are started. */
MONTLOK_API int montlok_set_latency_threads(int threads);
MONTLOK_API int montlok_latency_threads(void);

/* Replaces montlok.h:92: "tree_ensemble". */
MONTLOK_API const char* montlok_families(void);

/* Replaces montlok.h:94-100 (c_api.cpp:96-134). */
MONTLOK_API int montlok_model_open(const char* path, montlok_model** model);
MONTLOK_API int montlok_model_open_memory(const void* data, size_t size, montlok_model** model);
MONTLOK_API void montlok_model_close(montlok_model* model);
MONTLOK_API int montlok_model_get_info(const montlok_model* model, montlok_model_info* info);
MONTLOK_API const char* montlok_model_family(const montlok_model* model);
MONTLOK_API const char* montlok_model_spec(const montlok_model* model);

/* Replaces montlok.h:104-105 (c_api.cpp:136-141; runtime.cpp:554-586;
 * trees.cpp:161-197). x: batch * features values of `dtype`, row-major, in
 * host memory (pageable or pinned; device memory of the current device is
 * also accepted); out: batch * outputs doubles. batch == 0 does nothing. The
 * rows run on the current GPU, or are split over devices 0..n-1 after
 * montlok_set_devices(n). Returns when `out` is written. */
MONTLOK_API int montlok_model_predict(const montlok_model* model, montlok_dtype dtype, const void* x, size_t batch,
                                      double* out);

/* Replaces montlok.h:110-113. A tree model's stream is stateless: each step
 * predicts `batch` rows (reference trees.cpp:199-208). */
MONTLOK_API int montlok_stream_open(const montlok_model* model, size_t batch, montlok_stream** stream);
MONTLOK_API int montlok_stream_step(montlok_stream* stream, montlok_dtype dtype, const void* x, double* out);
MONTLOK_API int montlok_stream_reset(montlok_stream* stream);
MONTLOK_API void montlok_stream_close(montlok_stream* stream);

/* Replaces montlok.h:198-200. Plugin families are host-CPU code and are not
 * part of this build: both return MONTLOK_ERROR_UNSUPPORTED. */
typedef struct montlok_family_v1 montlok_family_v1;
MONTLOK_API int montlok_register_family(const montlok_family_v1* family);
MONTLOK_API int montlok_plugin_load(const char* path);

/* ------------------------------------------------------------------------ */
/* Additive entry points (no reference counterpart)                           */
/* ------------------------------------------------------------------------ */

/* Additive. x and out are device memory of the current CUDA device; the work
 * is queued on `stream` (a cudaStream_t, NULL for the legacy default stream)
 * and the call returns without waiting for it. */
MONTLOK_API int montlok_model_predict_device(const montlok_model* model, montlok_dtype dtype, const void* x,
                                             size_t batch, double* out, void* stream);

/* Additive; no counterpart in the reference. montlok_model_predict_device
 * for callers that cannot allocate GPU memory while they predict: serving
 * loops whose device memory belongs to another allocator (a framework's
 * caching pool that has already reserved the GPU) and latency-critical paths
 * that must not pay for cudaMalloc/cudaFree or the device-wide
 * synchronisation cudaFree implies. It allocates nothing: models the
 * complete-tree, multi-output or deep-tree kernels take keep their key tables
 * in shared memory; for the others the key tables of each 32-row group live
 * in a static 16 MiB device array of this library (present on every GPU that
 * loads it, until the process exits), and the kernel grid is cut to the
 * tables that fit. A model needing more than 16 MiB
 * for one table (more than 131072 feature/missing-rule slots, about 32768
 * features) fails with MONTLOK_ERROR_UNSUPPORTED. The model must already be
 * resident on the current device (after one predict or predict_device call
 * there), else MONTLOK_ERROR_STATE. The first call on a device looks the
 * array's device address up, so make it before any stream capture. Calls
 * share the array: calls whose kernels overlap on the GPU (concurrent
 * streams) race on it and must be serialised by the caller. */
MONTLOK_API int montlok_model_predict_device_noalloc(const montlok_model* model, montlok_dtype dtype, const void* x,
                                                     size_t batch, double* out, void* stream);

/* Additive. The node index (into the file's trees.* tensors) of the leaf each
 * row reaches in each tree: leaves holds batch * trees int32, row-major. The
 * _device form takes device buffers and a stream like predict_device. */
MONTLOK_API int montlok_model_predict_leaves(const montlok_model* model, montlok_dtype dtype, const void* x,
                                             size_t batch, int32_t* leaves);
MONTLOK_API int montlok_model_predict_leaves_device(const montlok_model* model, montlok_dtype dtype, const void* x,
                                                    size_t batch, int32_t* leaves, void* stream);
/* Additive. The device-buffer calls (predict_device, predict_leaves_device,
 * predict_device_noalloc) return before their kernels run, so a kernel that
 * gives up a bounded wait on its tree data (its rows are then not written)
 * cannot fail the call itself. This reports it: MONTLOK_ERROR_INTERNAL when
 * such a kernel on the current device gave up since the last check (the
 * record is then cleared), else MONTLOK_OK. Call it after synchronising the
 * streams of those calls. Host-buffer calls report the same failure from the
 * call itself. */
MONTLOK_API int montlok_model_device_status(const montlok_model* model);
/* Additive. The kernel a predict of `batch` rows runs on the current device
 * (the model is uploaded there first): "complete-tree", "small-batch",
 * "multi-output", "deep-tree", "generic" or "generic-global-keys". The
 * string is static. */
MONTLOK_API int montlok_model_kernel(const montlok_model* model, size_t batch, const char** name);
/* Additive. Trees of a model (the leaves row length). */
MONTLOK_API int montlok_model_trees(const montlok_model* model, uint32_t* trees);

/* Additive. GPUs montlok_model_predict spreads host-buffer rows over: 0 (the
 * default) uses the current device only; n uses devices 0..n-1, each taking a
 * contiguous slice of the rows and writing its own slice of `out`. */
MONTLOK_API int montlok_set_devices(int count);
MONTLOK_API int montlok_devices(void);
/* Additive. CUDA devices visible to the process (0 without a GPU). */
MONTLOK_API int montlok_device_count(void);

/* Additive; the timing loop of the reference's Python bench
 * (src/python/module.cpp:115-150) moved behind the ABI so no binding overhead
 * is timed. rows holds `count` inputs of batch * features values used in
 * turn; `warmup` untimed calls, then `iterations` calls timed one by one into
 * samples_ns, then `iterations` back-to-back calls whose mean is *mean_ns. */
MONTLOK_API int montlok_bench_predict(const montlok_model* model, montlok_dtype dtype, const void* rows, size_t count,
                                      size_t batch, size_t iterations, size_t warmup, double* samples_ns,
                                      double* mean_ns);

#ifdef __cplusplus
}
#endif

#endif /* MONTLOK_H */
