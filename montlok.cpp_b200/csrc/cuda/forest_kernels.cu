// Tree-ensemble predict kernels for sm_100a.
//
// One warp owns a group of 32 consecutive rows (lane = row) and keeps them
// on chip for the whole ensemble:
//
//  1. prepare: the group's rows are read coalesced (lane = feature, 32 rows
//     at a time), preprocessed in float64 (clip((x - mean) / scale), NaN kept),
//     cast to float32 when the model asks, transposed through a padded shared
//     tile and written as int32 keys, one column per lane, into the warp's key
//     table [slot][32]. Each slot is a (feature, missing-rule variant) pair;
//     forest.cpp explains the keys and variants. Lane l always reads bank l,
//     so the walk's gathers never conflict.
//  2. walk: each lane walks kIlp trees side by side; a step is one 16-byte
//     node load, one shared key load and one signed compare (go right when
//     key > T). Leaves loop to themselves, so a tree takes exactly its depth
//     in steps and lanes never diverge.
//  3. sum: leaf values are added in float64 in the reference order
//     (src/core/trees.cpp:161-197, 366-388): trees in index order within
//     blocks of 64, the first block on top of the base score, every later
//     block from 0.0 and then added to the total; then the mean fix-up and the
//     link (identity, sigmoid, softmax, exp) with the reference's own exp
//     (src/core/kernels.hpp:220-255), every operation rounded on its own.
//
// A float64 model compares float32 keys of its values first; when a key ties
// with the threshold's key the split is decided on the doubles, re-read from
// the input (exact_right).
#include <algorithm>
#include <climits>
#include <mutex>
#include <vector>

#include "forest.cuh"

namespace mlk::cuda {
namespace {

constexpr int kTreeBlock = 64;  // trees per partial sum
constexpr int kMaxOut = 8;      // outputs held in registers per pass
constexpr int kIlp = 4;         // trees one lane walks side by side
constexpr int kStage = 33;      // padded row length of the transpose tile
constexpr int kStageBytes = 32 * kStage * 8;
constexpr double kZeroThr = static_cast<double>(1e-35f);  // LightGBM kZeroThreshold

__host__ __device__ constexpr int align16(int n) { return (n + 15) & ~15; }
__host__ __device__ constexpr int key_bytes(int slots) { return align16(slots * 32 * 4); }

__device__ __forceinline__ int key32(float v) {
    const unsigned b = __float_as_uint(v);
    const int m = static_cast<int>(b & 0x7fffffffu);
    return (b >> 31) ? -m : m;
}

__device__ __forceinline__ double load_x(const float* p) { return static_cast<double>(__ldg(p)); }
__device__ __forceinline__ double load_x(const double* p) { return __ldg(p); }

// Preprocess and cast of one raw value (reference runtime.cpp:532-552 and the
// cast of trees.cpp:275); std::max/std::min written out so NaN stays NaN.
__device__ __forceinline__ double finish(const ForestArgs& a, double v, double mean, double scale) {
    if (a.standardize) v = __ddiv_rn(__dsub_rn(v, mean), scale);
    if (a.clip) {
        v = (v < a.lo) ? a.lo : v;
        v = (a.hi < v) ? a.hi : v;
    }
    if (a.cast_f32) v = static_cast<double>(__double2float_rn(v));
    return v;
}

__device__ __forceinline__ void put_keys(const ForestArgs& a, int* col, int4 s, double v) {
    const bool nan = v != v;
    const int k = a.cast_f32 ? key32(__double2float_rn(v)) : key32(__double2float_rd(v));
    const bool zero = nan || fabs(v) <= kZeroThr;
    if (s.x >= 0) col[s.x * 32] = nan ? INT_MAX : k;
    if (s.y >= 0) col[s.y * 32] = nan ? INT_MIN : k;
    if (s.z >= 0) col[s.z * 32] = zero ? INT_MAX : k;
    if (s.w >= 0) col[s.w * 32] = zero ? INT_MIN : k;
}

template <typename XT>
__device__ void prepare_group(const ForestArgs& a, const XT* __restrict__ x, long long row0, long long batch,
                              int* keys, double* stage, int lane) {
    for (int f0 = 0; f0 < a.F; f0 += 32) {
        const int feat = f0 + lane;
        const bool live = feat < a.F;
        double mean = 0.0, scale = 1.0;
        if (live && a.standardize) {
            mean = __ldg(a.pre_mean + feat);
            scale = __ldg(a.pre_scale + feat);
        }
#pragma unroll 8
        for (int i = 0; i < 32; ++i) {
            const long long row = row0 + i;
            double v = 0.0;
            if (live && row < batch) v = finish(a, load_x(x + row * a.F + feat), mean, scale);
            stage[i * kStage + lane] = v;
        }
        __syncwarp();
        const int nf = min(32, a.F - f0);
        for (int j = 0; j < nf; ++j) put_keys(a, keys + lane, __ldg(a.slot_of + f0 + j), stage[lane * kStage + j]);
        __syncwarp();
    }
    keys[a.pad_slot * 32 + lane] = INT_MIN;
    __syncwarp();
}

// The split decided on doubles, for a float64 model whose keys tied.
template <typename XT>
__device__ __noinline__ bool exact_right(const ForestArgs& a, const XT* __restrict__ x, long long row,
                                         long long batch, int idx) {
    const int feat = __ldg(a.feature + idx);
    const double t = __ldg(a.threshold + idx);
    double v = 0.0;  // padding rows were prepared as 0.0
    if (row < batch) {
        double mean = 0.0, scale = 1.0;
        if (a.standardize) {
            mean = __ldg(a.pre_mean + feat);
            scale = __ldg(a.pre_scale + feat);
        }
        v = finish(a, load_x(x + row * a.F + feat), mean, scale);
    }
    return a.le ? (v > t) : !(v < t);
}

template <bool TIES, typename XT>
__device__ __forceinline__ int step(const ForestArgs& a, const int* col, int idx, const XT* x, long long row,
                                    long long batch) {
    const int4 n = __ldg(a.nodes + idx);
    const int kv = col[n.y * 32];
    bool right = kv > n.x;
    if (TIES && kv == n.x) right = exact_right(a, x, row, batch, idx);
    return right ? n.w : n.z;
}

// Adds trees [t0, t1) to `sum` in index order (or records their leaves).
template <bool TIES, bool LEAVES, int KC, typename XT>
__device__ __forceinline__ void walk_block(const ForestArgs& a, const int* col, int t0, int t1, int k0,
                                           double (&sum)[KC], const XT* x, long long row, long long batch,
                                           int* leaves) {
    for (int t = t0; t < t1; t += kIlp) {
        int idx[kIlp];
        int steps = 0;
#pragma unroll
        for (int g = 0; g < kIlp; ++g) {
            const int tt = t + g < t1 ? t + g : t;
            idx[g] = __ldg(a.roots + tt);
            steps = max(steps, __ldg(a.depth + tt));
        }
        for (int s = 0; s < steps; ++s) {
#pragma unroll
            for (int g = 0; g < kIlp; ++g) idx[g] = step<TIES>(a, col, idx[g], x, row, batch);
        }
#pragma unroll
        for (int g = 0; g < kIlp; ++g) {
            const int tt = t + g;
            if (tt < t1) {
                if (LEAVES) {
                    if (row < batch) leaves[row * a.T + tt] = idx[g];
                } else {
                    const double v = __ldg(a.leaf_value + idx[g]);
                    if (KC == 1) {
                        sum[0] = __dadd_rn(sum[0], v);
                    } else {
                        const int k = __ldg(a.tree_output + tt) - k0;
#pragma unroll
                        for (int j = 0; j < KC; ++j) {
                            if (j == k) sum[j] = __dadd_rn(sum[j], v);
                        }
                    }
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Link functions: the reference's exp (kernels.hpp:220-253) — clamp to
// [-708, 708], n = round(x / ln 2) through the 1.5 * 2^52 shifter, Cody-Waite
// reduction r = (x - n ln2_hi) - n ln2_lo, exp(r) - 1 by the degree-13 Taylor
// series in Horner form, and 2^n assembled in the exponent bits.
// ---------------------------------------------------------------------------

__device__ __forceinline__ double vexp(double x) {
    constexpr double kInvLn2 = 1.4426950408889634074;
    constexpr double kLn2Hi = 6.93147180369123816490e-01;
    constexpr double kLn2Lo = 1.90821492927058770002e-10;
    constexpr double kShifter = 6755399441055744.0;
    constexpr double c[13] = {
        1.0 / 6227020800.0, 1.0 / 479001600.0, 1.0 / 39916800.0, 1.0 / 3628800.0, 1.0 / 362880.0,
        1.0 / 40320.0,      1.0 / 5040.0,      1.0 / 720.0,      1.0 / 120.0,     1.0 / 24.0,
        1.0 / 6.0,          0.5,               1.0,
    };
    x = (x < -708.0) ? -708.0 : x;
    x = (x > 708.0) ? 708.0 : x;
    const double shifted = __dadd_rn(__dmul_rn(x, kInvLn2), kShifter);
    const double n = __dsub_rn(shifted, kShifter);
    const double r = __dsub_rn(__dsub_rn(x, __dmul_rn(n, kLn2Hi)), __dmul_rn(n, kLn2Lo));
    double p = c[0];
#pragma unroll
    for (int i = 1; i < 13; ++i) p = __dadd_rn(__dmul_rn(p, r), c[i]);
    p = __dadd_rn(__dmul_rn(p, r), 1.0);
    const unsigned long long bits = static_cast<unsigned long long>(__double_as_longlong(shifted)) -
                                    static_cast<unsigned long long>(__double_as_longlong(kShifter));
    return __dmul_rn(p, __longlong_as_double(static_cast<long long>((bits + 1023ull) << 52)));
}

template <int KC>
__device__ __forceinline__ void apply_link(const ForestArgs& a, double (&v)[KC], int kc) {
    if (a.link == 1) {
#pragma unroll
        for (int j = 0; j < KC; ++j) {
            if (j < kc) {
                const double s = __dmul_rn(v[j], a.sigmoid_scale);
                v[j] = __ddiv_rn(1.0, __dadd_rn(1.0, vexp(__dsub_rn(0.0, s))));
            }
        }
    } else if (a.link == 3) {
#pragma unroll
        for (int j = 0; j < KC; ++j) {
            if (j < kc) v[j] = vexp(v[j]);
        }
    } else if (a.link == 2) {
        double peak = v[0];
#pragma unroll
        for (int j = 1; j < KC; ++j) {
            if (j < kc) peak = (peak < v[j]) ? v[j] : peak;
        }
        double total = 0.0;
#pragma unroll
        for (int j = 0; j < KC; ++j) {
            if (j < kc) {
                v[j] = vexp(__dsub_rn(v[j], peak));
                total = __dadd_rn(total, v[j]);
            }
        }
#pragma unroll
        for (int j = 0; j < KC; ++j) {
            if (j < kc) v[j] = __ddiv_rn(v[j], total);
        }
    }
}

template <bool TIES, bool LEAVES, int KC, bool GLOBAL_KEYS, typename XT>
__global__ void __launch_bounds__(64) forest_kernel(const ForestArgs a, const XT* __restrict__ x, long long batch,
                                                     double* __restrict__ out, int* __restrict__ leaves, int k0,
                                                     int kc, int link_here, int* __restrict__ scratch) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    const int warp_bytes = (GLOBAL_KEYS ? 0 : key_bytes(a.slots)) + kStageBytes;
    const long long me = static_cast<long long>(blockIdx.x) * warps + warp;
    int* keys = GLOBAL_KEYS ? scratch + me * a.slots * 32
                            : reinterpret_cast<int*>(smem + warp * warp_bytes);
    double* stage = reinterpret_cast<double*>(smem + warp * warp_bytes + (GLOBAL_KEYS ? 0 : key_bytes(a.slots)));
    const long long groups = (batch + 31) / 32;
    const long long all_warps = static_cast<long long>(gridDim.x) * warps;
    const int blocks = (a.T + kTreeBlock - 1) / kTreeBlock;
    for (long long g = me; g < groups; g += all_warps) {
        const long long row0 = g * 32;
        prepare_group(a, x, row0, batch, keys, stage, lane);
        const long long row = row0 + lane;
        const int* col = keys + lane;
        double acc[KC];
#pragma unroll
        for (int j = 0; j < KC; ++j) acc[j] = (j < kc && !a.mean) ? __ldg(a.base + k0 + j) : 0.0;
        walk_block<TIES, LEAVES, KC>(a, col, 0, min(a.T, kTreeBlock), k0, acc, x, row, batch, leaves);
        for (int b = 1; b < blocks; ++b) {
            double part[KC];
#pragma unroll
            for (int j = 0; j < KC; ++j) part[j] = 0.0;
            walk_block<TIES, LEAVES, KC>(a, col, b * kTreeBlock, min(a.T, (b + 1) * kTreeBlock), k0, part, x, row,
                                         batch, leaves);
#pragma unroll
            for (int j = 0; j < KC; ++j) acc[j] = __dadd_rn(acc[j], part[j]);
        }
        if (!LEAVES && row < batch) {
            if (a.mean) {
#pragma unroll
                for (int j = 0; j < KC; ++j) {
                    if (j < kc) {
                        const int c = __ldg(a.counts + k0 + j);
                        acc[j] = __dadd_rn(__ldg(a.base + k0 + j), c ? __ddiv_rn(acc[j], static_cast<double>(c)) : 0.0);
                    }
                }
            }
            if (link_here) apply_link<KC>(a, acc, kc);
#pragma unroll
            for (int j = 0; j < KC; ++j) {
                if (j < kc) out[row * a.K + k0 + j] = acc[j];
            }
        }
        __syncwarp();
    }
}

// Softmax over rows of more than kMaxOut outputs, after the sums are in `out`
// (reference trees.cpp:443-451).
__global__ void softmax_rows(double* __restrict__ out, long long batch, int K) {
    const long long row = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (row >= batch) return;
    double* v = out + row * K;
    double peak = v[0];
    for (int k = 1; k < K; ++k) peak = (peak < v[k]) ? v[k] : peak;
    double total = 0.0;
    for (int k = 0; k < K; ++k) {
        v[k] = vexp(__dsub_rn(v[k], peak));
        total = __dadd_rn(total, v[k]);
    }
    for (int k = 0; k < K; ++k) v[k] = __ddiv_rn(v[k], total);
}

template <bool TIES, bool LEAVES, int KC, bool GLOBAL_KEYS, typename XT>
void* kernel_of() {
    return reinterpret_cast<void*>(&forest_kernel<TIES, LEAVES, KC, GLOBAL_KEYS, XT>);
}

// The kernel instance for a call.
void* pick(bool ties, bool leaves, int kc, bool global_keys, bool f64) {
#define MLK_PICK(T_, L_, K_, G_)                                       \
    if (ties == T_ && leaves == L_ && kc == K_ && global_keys == G_) { \
        return f64 ? kernel_of<T_, L_, K_, G_, double>()               \
                   : kernel_of<T_, L_, K_, G_, float>();               \
    }
    MLK_PICK(false, false, 1, false)
    MLK_PICK(false, false, 8, false)
    MLK_PICK(true, false, 1, false)
    MLK_PICK(true, false, 8, false)
    MLK_PICK(false, true, 1, false)
    MLK_PICK(true, true, 1, false)
    MLK_PICK(false, false, 1, true)
    MLK_PICK(false, false, 8, true)
    MLK_PICK(true, false, 1, true)
    MLK_PICK(true, false, 8, true)
    MLK_PICK(false, true, 1, true)
    MLK_PICK(true, true, 1, true)
#undef MLK_PICK
    return nullptr;
}

constexpr int kSmemLimit = 227 * 1024;

struct Shape {
    bool global_keys;
    int warps_per_cta;
    int smem;
};

Shape shape_of(const ForestArgs& a) {
    const int per_warp = key_bytes(a.slots) + kStageBytes;
    if (static_cast<long long>(a.slots) * 128 + kStageBytes > kSmemLimit) return {true, 2, 2 * kStageBytes};
    if (2 * per_warp <= kSmemLimit) return {false, 2, 2 * per_warp};
    return {false, 1, per_warp};
}

bool check(cudaError_t e, const char* what, std::string& err) {
    if (e == cudaSuccess) return true;
    err = std::string(what) + ": " + cudaGetErrorString(e);
    return false;
}

}  // namespace

bool prepare_kernels(const DevForest& f, std::string& err) {
    // The limit is a property of the kernel, shared by every model: set it
    // once per device to the most any launch asks for.
    static std::mutex mu;
    static std::vector<int> done;
    std::lock_guard<std::mutex> lock(mu);
    if (std::find(done.begin(), done.end(), f.device) != done.end()) return true;
    for (int ties = 0; ties < 2; ++ties) {
        for (int leaves = 0; leaves < 2; ++leaves) {
            for (int kc : {1, 8}) {
                for (int global_keys = 0; global_keys < 2; ++global_keys) {
                    for (int f64 = 0; f64 < 2; ++f64) {
                        void* k = pick(ties, leaves, kc, global_keys, f64);
                        if (!k) continue;
                        if (!check(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit),
                                   "cudaFuncSetAttribute", err)) {
                            return false;
                        }
                    }
                }
            }
        }
    }
    done.push_back(f.device);
    return true;
}

size_t scratch_bytes(const DevForest& f) {
    const Shape s = shape_of(f.args);
    if (!s.global_keys) return 0;
    return static_cast<size_t>(f.sm_count) * 4 * s.warps_per_cta * f.args.slots * 32 * sizeof(int);
}

bool launch_forest(const DevForest& f, int dtype, const void* x, long long batch, double* out, int* leaves,
                   cudaStream_t stream, std::string& err, int* scratch) {
    if (batch <= 0) return true;
    const ForestArgs& a = f.args;
    const Shape s = shape_of(a);
    const bool ties = !a.cast_f32;
    const bool f64 = dtype == 2;
    const long long groups = (batch + 31) / 32;
    const int per_sm = s.global_keys ? 4 : std::max(1, kSmemLimit / (s.smem + 1024));
    const long long want = (groups + s.warps_per_cta - 1) / s.warps_per_cta;
    const int grid = static_cast<int>(std::min<long long>(want, static_cast<long long>(f.sm_count) * per_sm));
    const int threads = 32 * s.warps_per_cta;
    if (leaves) {
        void* k = pick(ties, true, 1, s.global_keys, f64);
        int k0 = 0, kc = 1, link = 0;
        double* no_out = nullptr;
        void* args[] = {const_cast<ForestArgs*>(&a), const_cast<void**>(&x), &batch, &no_out, &leaves, &k0, &kc, &link,
                        &scratch};
        return check(cudaLaunchKernel(k, grid, threads, args, s.smem, stream), "leaf kernel launch", err);
    }
    const int kc_tmpl = a.K == 1 ? 1 : 8;
    const bool softmax_after = a.link == 2 && a.K > kMaxOut;
    for (int k0 = 0; k0 < a.K; k0 += kMaxOut) {
        int kc = std::min(kMaxOut, a.K - k0);
        int link_here = softmax_after ? 0 : 1;
        int k0v = k0;
        void* k = pick(ties, false, kc_tmpl, s.global_keys, f64);
        int* no_leaves = nullptr;
        void* args[] = {const_cast<ForestArgs*>(&a), const_cast<void**>(&x), &batch, &out, &no_leaves, &k0v, &kc,
                        &link_here, &scratch};
        if (!check(cudaLaunchKernel(k, grid, threads, args, s.smem, stream), "predict kernel launch", err)) return false;
    }
    if (softmax_after) {
        const int tpb = 128;
        const unsigned blocks = static_cast<unsigned>((batch + tpb - 1) / tpb);
        softmax_rows<<<blocks, tpb, 0, stream>>>(out, batch, a.K);
        if (!check(cudaGetLastError(), "softmax kernel launch", err)) return false;
    }
    return true;
}

}  // namespace mlk::cuda
