/* TEST INFRASTRUCTURE ONLY - see tree_oracle.h. Each function cites the
 * reference code it restates (paths relative to the montlok.cpp project). */
#include "tree_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* LightGBM's kZeroThreshold, the float literal 1e-35f (trees.cpp:50-51). */
static const double kZero = (double)1e-35f;
enum { kTreeBlock = 64 }; /* trees per partial sum (trees.cpp:62) */

/* Model::preprocess (runtime.cpp:532-552): widen, (x - mean) / scale, then
 * min(max(v, lo), hi) written as std::max / std::min are, so NaN stays. */
static double raw_value(const oracle_forest* f, int dtype, const void* x, size_t row, int feat) {
    const size_t at = row * (size_t)f->features + (size_t)feat;
    double v = dtype == 1 ? (double)((const float*)x)[at] : ((const double*)x)[at];
    if (f->standardize) v = (v - f->pre_mean[feat]) / f->pre_scale[feat];
    if (f->clip) {
        v = (v < f->clip_lo) ? f->clip_lo : v;
        v = (f->clip_hi < v) ? f->clip_hi : v;
    }
    return v;
}

/* TreeEnsemble::leaf (trees.cpp:411-430), with the float32 narrowing of
 * reference_block (trees.cpp:392-396). Returns the leaf's node index. */
static int32_t leaf_of(const oracle_forest* f, int32_t node, int dtype, const void* x, size_t row) {
    while (f->feature[node] >= 0) {
        double v = raw_value(f, dtype, x, row, f->feature[node]);
        if (f->cast_f32) v = (double)(float)v;
        const unsigned missing = (f->flags[node] >> 1) & 3u;
        const int default_left = f->flags[node] & 1u;
        int go_left;
        if (isnan(v) && missing != 0) {
            go_left = default_left;
        } else {
            if (isnan(v)) v = 0.0;
            if (missing == 2 && v >= -kZero && v <= kZero) {
                go_left = default_left;
            } else {
                const double t = f->threshold[node];
                go_left = f->decision_le ? (v <= t) : (v < t);
            }
        }
        node = go_left ? f->left[node] : f->right[node];
    }
    return node;
}

/* vexp (kernels.hpp:220-253) one lane at a time. */
double oracle_exp(double x) {
    static const double c[13] = {
        1.0 / 6227020800.0, 1.0 / 479001600.0, 1.0 / 39916800.0, 1.0 / 3628800.0, 1.0 / 362880.0,
        1.0 / 40320.0,      1.0 / 5040.0,      1.0 / 720.0,      1.0 / 120.0,     1.0 / 24.0,
        1.0 / 6.0,          0.5,               1.0,
    };
    const double inv_ln2 = 1.4426950408889634074;
    const double ln2_hi = 6.93147180369123816490e-01;
    const double ln2_lo = 1.90821492927058770002e-10;
    const double shifter = 6755399441055744.0;
    x = x < -708.0 ? -708.0 : x;
    x = x > 708.0 ? 708.0 : x;
    volatile double shifted = x * inv_ln2 + shifter; /* kept in memory: rounded as a double */
    const double n = shifted - shifter;
    const double r = (x - n * ln2_hi) - n * ln2_lo;
    double p = c[0];
    for (int i = 1; i < 13; ++i) p = p * r + c[i];
    p = p * r + 1.0;
    uint64_t bits, sbits;
    const double s = shifted;
    memcpy(&bits, &s, 8);
    memcpy(&sbits, &shifter, 8);
    bits = ((bits - sbits) + 1023u) << 52;
    double scale;
    memcpy(&scale, &bits, 8);
    return p * scale;
}

/* apply_link (trees.cpp:432-454). */
static void apply_link(const oracle_forest* f, double* acc) {
    const int K = f->outputs;
    if (f->link == 1) {
        for (int k = 0; k < K; ++k) {
            const double s = acc[k] * f->sigmoid_scale;
            acc[k] = 1.0 / (1.0 + oracle_exp(0.0 - s));
        }
    } else if (f->link == 3) {
        for (int k = 0; k < K; ++k) acc[k] = oracle_exp(acc[k]);
    } else if (f->link == 2) {
        double peak = acc[0];
        for (int k = 1; k < K; ++k) peak = (peak < acc[k]) ? acc[k] : peak;
        for (int k = 0; k < K; ++k) acc[k] -= peak;
        for (int k = 0; k < K; ++k) acc[k] = oracle_exp(acc[k]);
        double total = 0;
        for (int k = 0; k < K; ++k) total += acc[k];
        for (int k = 0; k < K; ++k) acc[k] /= total;
    }
}

/* TreeEnsemble::predict for one row (trees.cpp:161-197 with the association
 * of reference_block, :397-408): the first block of 64 trees adds straight
 * into the base score, each later block sums from 0.0 and is then added to
 * every output; then the mean fix-up and the link. */
static void predict_row(const oracle_forest* f, int dtype, const void* x, size_t row, double* acc, double* part) {
    const int K = f->outputs, T = f->trees;
    for (int k = 0; k < K; ++k) acc[k] = f->mean ? 0.0 : f->base[k];
    const int blocks = (T + kTreeBlock - 1) / kTreeBlock;
    for (int b = 0; b < blocks; ++b) {
        double* sums = b == 0 ? acc : part;
        if (b > 0) {
            for (int k = 0; k < K; ++k) part[k] = 0.0;
        }
        const int t1 = (b + 1) * kTreeBlock < T ? (b + 1) * kTreeBlock : T;
        for (int t = b * kTreeBlock; t < t1; ++t) {
            sums[f->tree_output[t]] += f->value[leaf_of(f, f->roots[t], dtype, x, row)];
        }
        if (b > 0) {
            for (int k = 0; k < K; ++k) acc[k] += part[k];
        }
    }
    if (f->mean) {
        int* counts = calloc((size_t)K, sizeof(int));
        for (int t = 0; t < T; ++t) ++counts[f->tree_output[t]];
        for (int k = 0; k < K; ++k) acc[k] = f->base[k] + (counts[k] ? acc[k] / (double)counts[k] : 0.0);
        free(counts);
    }
    apply_link(f, acc);
}

typedef struct job {
    const oracle_forest* f;
    int dtype;
    const void* x;
    size_t lo, hi;
    double* out;
    int32_t* leaves;
} job;

static void* run(void* arg) {
    const job* j = arg;
    const int K = j->f->outputs, T = j->f->trees;
    if (j->out) {
        double* part = malloc(sizeof(double) * (size_t)(K > 0 ? K : 1));
        for (size_t r = j->lo; r < j->hi; ++r) predict_row(j->f, j->dtype, j->x, r, j->out + r * (size_t)K, part);
        free(part);
    } else {
        for (size_t r = j->lo; r < j->hi; ++r) {
            for (int t = 0; t < T; ++t) {
                j->leaves[r * (size_t)T + (size_t)t] = leaf_of(j->f, j->f->roots[t], j->dtype, j->x, r);
            }
        }
    }
    return NULL;
}

static void split(const oracle_forest* f, int dtype, const void* x, size_t batch, double* out, int32_t* leaves,
                  int threads) {
    if (threads < 1) threads = 1;
    if ((size_t)threads > batch) threads = batch ? (int)batch : 1;
    job* jobs = calloc((size_t)threads, sizeof(job));
    pthread_t* ids = calloc((size_t)threads, sizeof(pthread_t));
    const size_t per = (batch + (size_t)threads - 1) / (size_t)threads;
    for (int i = 0; i < threads; ++i) {
        const size_t lo = (size_t)i * per < batch ? (size_t)i * per : batch;
        const size_t hi = lo + per < batch ? lo + per : batch;
        jobs[i] = (job){f, dtype, x, lo, hi, out, leaves};
        if (i > 0) pthread_create(&ids[i], NULL, run, &jobs[i]);
    }
    run(&jobs[0]);
    for (int i = 1; i < threads; ++i) pthread_join(ids[i], NULL);
    free(ids);
    free(jobs);
}

void oracle_predict(const oracle_forest* f, int dtype, const void* x, size_t batch, double* out, int threads) {
    split(f, dtype, x, batch, out, NULL, threads);
}

void oracle_leaves(const oracle_forest* f, int dtype, const void* x, size_t batch, int32_t* leaves, int threads) {
    split(f, dtype, x, batch, NULL, leaves, threads);
}
