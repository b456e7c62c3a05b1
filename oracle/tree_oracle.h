/* TEST INFRASTRUCTURE ONLY - the CPU checker for the CUDA tree-ensemble path.
 *
 * A plain-C restatement of the reference's tree_ensemble predict
 * (montlok.cpp src/core/trees.cpp, runtime.cpp, kernels.hpp), evaluated the
 * slow, obvious way: the node-by-node walk of leaf() on the file's own node
 * arrays, float64 sums in the reference's block order, the reference's exp.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it;
 * the product library never links or calls it.
 *
 * Parity is pinned by tests/test_oracle.py against the reference's golden
 * fixture (tests/data/gbr.{montlok,io}, copied to tests/golden/), the decision
 * rules of LightGBM and XGBoost, and the reference library itself compiled
 * from its sources (oracle/_ref, when present).
 */
#ifndef MONTLOK_TREE_ORACLE_H
#define MONTLOK_TREE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct oracle_forest {
    int32_t features, outputs, trees, nodes;
    int32_t decision_le, cast_f32, mean, link; /* link: 0 identity, 1 sigmoid, 2 softmax, 3 exp */
    double sigmoid_scale;
    const double* base;          /* [outputs] */
    const int32_t* roots;        /* [trees] */
    const int32_t* tree_output;  /* [trees] */
    const int32_t* feature;      /* [nodes] */
    const double* threshold;     /* [nodes] */
    const int32_t* left;         /* [nodes] */
    const int32_t* right;        /* [nodes] */
    const double* value;         /* [nodes] */
    const uint8_t* flags;        /* [nodes] */
    int32_t standardize, clip;
    const double* pre_mean;      /* [features] */
    const double* pre_scale;     /* [features] */
    double clip_lo, clip_hi;
} oracle_forest;

/* dtype 1: float32 inputs, 2: float64. `threads` > 1 splits rows over pthreads. */
void oracle_predict(const oracle_forest* f, int dtype, const void* x, size_t batch, double* out, int threads);
void oracle_leaves(const oracle_forest* f, int dtype, const void* x, size_t batch, int32_t* leaves, int threads);
/* The reference's exp: clamp, Cody-Waite reduction, degree-13 Taylor series. */
double oracle_exp(double x);

#ifdef __cplusplus
}
#endif

#endif
