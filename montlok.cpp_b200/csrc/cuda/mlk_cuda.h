/* Internal C interface between the host runtime (csrc/core, built with the
 * host compiler) and the CUDA side (csrc/cuda, built with nvcc for sm_100a).
 * The host side never includes CUDA headers; this layer owns every device
 * buffer, stream and kernel launch.
 *
 * Every function returns 0 on success, or a nonzero montlok_status value with
 * a message written to `err` (capacity `errlen`). */
#ifndef MLK_CUDA_H
#define MLK_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* A compiled tree ensemble as host arrays (see ForestImage in runtime.hpp). */
typedef struct mlk_forest_view {
    int32_t features, outputs, trees, nodes, slots, pad_slot;
    int32_t decision_le, cast_f32, mean, link; /* link: 0 identity, 1 sigmoid, 2 softmax, 3 exp */
    double sigmoid_scale;
    const double* base;          /* [outputs] */
    const int32_t* counts;       /* [outputs] */
    const int32_t* slot_of;      /* [features * 4] */
    const int32_t* node_words;   /* [nodes * 4]: T, slot, left, right */
    const double* leaf_value;    /* [nodes] */
    const int32_t* roots;        /* [trees] */
    const int32_t* depth;        /* [trees] */
    const int32_t* tree_output;  /* [trees] */
    const double* threshold;     /* [nodes] */
    const int32_t* feature;      /* [nodes] */
    const uint8_t* flags;        /* [nodes] */
    /* Preprocess: (x - mean) / scale, then clip to [lo, hi]; NaN stays NaN. */
    int32_t standardize, clip;
    const double* pre_mean;      /* [features] or NULL */
    const double* pre_scale;     /* [features] or NULL */
    double clip_lo, clip_hi;
    /* Complete-tree view (complete_depth > 0): heap-ordered splits and leaves. */
    int32_t complete_depth, heap_leaf_f32;
    const int32_t* heap_words;   /* [trees * (2^d - 1) * 2]: T, slot */
    const int32_t* heap_node_id; /* [trees * (2^d - 1)] */
    const double* heap_leaf;     /* [trees * 2^d] */
    const int32_t* heap_leaf_id; /* [trees * 2^d] */
} mlk_forest_view;

typedef struct mlk_dev_forest mlk_dev_forest;

/* Pointer kinds reported by mlk_cuda_pointer_kind. */
enum { MLK_PTR_PAGEABLE = 0, MLK_PTR_PINNED = 1, MLK_PTR_DEVICE = 2 };

int mlk_cuda_device_count(int* count, char* err, size_t errlen);
/* Host threads that copy pageable inputs into pinned staging. */
void mlk_cuda_set_copy_threads(int threads);
/* Nonzero: host-buffer predicts of at most 8 rows on complete-tree models are
 * answered by a resident kernel of the calling thread (engine_kernels.cu),
 * started on first use; zero: they replay a cached graph, and a thread's
 * engine is released at its next call. */
void mlk_cuda_set_latency_engine(int on);
int mlk_cuda_current_device(int* device, char* err, size_t errlen);
int mlk_cuda_pointer_kind(const void* p, int* kind, int* device);

/* Uploads the forest to `device`. */
int mlk_cuda_forest_upload(int device, const mlk_forest_view* view, mlk_dev_forest** out, char* err, size_t errlen);
void mlk_cuda_forest_release(mlk_dev_forest* forest);
int mlk_cuda_forest_device(const mlk_dev_forest* forest);

/* dtype: 1 float32, 2 float64 (montlok_dtype). x holds batch * features
 * values, out batch * outputs doubles, leaves batch * trees int32 node
 * indices. Device variants take buffers on the forest's device and queue the
 * work on `stream` (a cudaStream_t; NULL is the legacy default stream)
 * without waiting for it. Host variants take host buffers, pipeline the
 * copies and kernels on this thread's own streams and return when `out` is
 * filled. */
int mlk_cuda_predict_device(const mlk_dev_forest* forest, int dtype, const void* x, size_t batch, double* out,
                            void* stream, char* err, size_t errlen);
int mlk_cuda_leaves_device(const mlk_dev_forest* forest, int dtype, const void* x, size_t batch, int32_t* leaves,
                           void* stream, char* err, size_t errlen);
/* predict_device without any allocation: the key tables live in a static
 * device array of this library (forest_kernels.cu), whose size
 * mlk_cuda_noalloc_scratch_bytes() gives. Returns 4
 * (MONTLOK_ERROR_UNSUPPORTED) when one 32-row key table exceeds it. */
size_t mlk_cuda_noalloc_scratch_bytes(void);
int mlk_cuda_predict_device_noalloc(const mlk_dev_forest* forest, int dtype, const void* x, size_t batch,
                                    double* out, void* stream, char* err, size_t errlen);
/* The status word of the forest's device-buffer calls: nonzero when one of
 * their kernels gave up a bounded wait on its tree copies since the word was
 * last cleared (its rows were then not written). `clear` resets it. */
int mlk_cuda_forest_status(const mlk_dev_forest* forest, int clear);
/* The kernel a predict of `batch` rows runs on this forest: "complete-tree",
 * "small-batch", "multi-output", "deep-tree", "generic" or
 * "generic-global-keys". */
const char* mlk_cuda_kernel_name(const mlk_dev_forest* forest, size_t batch);
int mlk_cuda_predict_host(const mlk_dev_forest* forest, int dtype, const void* x, size_t batch, double* out,
                          char* err, size_t errlen);
int mlk_cuda_leaves_host(const mlk_dev_forest* forest, int dtype, const void* x, size_t batch, int32_t* leaves,
                         char* err, size_t errlen);

#ifdef __cplusplus
}
#endif

#endif /* MLK_CUDA_H */
