/* Test infrastructure only: a per-call latency loop around the reference
 * runtime's montlok_model_predict (include/montlok/montlok.h:104-105),
 * linked into oracle/_ref/libmontlok_ref.so so that the CPU baseline of the
 * small-batch configuration is timed without Python between calls. */
#define _POSIX_C_SOURCE 199309L
#include <stddef.h>
#include <time.h>

struct montlok_model;
int montlok_model_predict(const struct montlok_model* model, int dtype, const void* x, size_t batch, double* out);

static double now_ns(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return 1e9 * (double)t.tv_sec + (double)t.tv_nsec;
}

/* Calls predict on `batch` rows at a time, taking the rows of call i from
 * rows + (i % count) * batch * features; `warmup` untimed calls, then
 * `iterations` timed ones whose nanoseconds land in samples_ns. Returns the
 * first nonzero status. */
int ref_time_calls(const struct montlok_model* model, const double* rows, size_t count, size_t batch,
                   size_t features, size_t iterations, size_t warmup, double* out, double* samples_ns) {
    const size_t stride = batch * features;
    for (size_t i = 0; i < warmup; ++i) {
        const int status = montlok_model_predict(model, 2, rows + (i % count) * stride, batch, out);
        if (status) return status;
    }
    for (size_t i = 0; i < iterations; ++i) {
        const double t0 = now_ns();
        const int status = montlok_model_predict(model, 2, rows + (i % count) * stride, batch, out);
        samples_ns[i] = now_ns() - t0;
        if (status) return status;
    }
    return 0;
}
