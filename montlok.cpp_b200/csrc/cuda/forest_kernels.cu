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
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "device_common.cuh"
#include "forest.cuh"
#include "mlk_cuda.h"

namespace mlk::cuda {
namespace {

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

template <bool TIES, bool LEAVES, int KC, bool GLOBAL_KEYS, typename XT>
__global__ void __launch_bounds__(64) forest_kernel(const __grid_constant__ ForestArgs a, const XT* __restrict__ x, long long batch,
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
        prepare_group<32, 32>(a, x, row0, batch, keys, stage, lane);
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

// Global key tables of the generic kernel (models whose 32-row key table
// overflows shared memory), then the small-batch kernel's sums.
size_t key_scratch_bytes(const DevForest& f) {
    const Shape s = shape_of(f.args);
    if (!s.global_keys) return 0;
    return (static_cast<size_t>(f.sm_count) * 4 * s.warps_per_cta * f.args.slots * 32 * sizeof(int) + 255) &
           ~size_t{255};
}

size_t scratch_bytes(const DevForest& f, long long batch) {
    return key_scratch_bytes(f) + (latency_fits(f, batch) ? latency_scratch_bytes(f) : 0);
}

bool launch_forest(const DevForest& f, int dtype, const void* x, long long batch, double* out, int* leaves,
                   cudaStream_t stream, std::string& err, int* scratch, int* counters) {
    if (batch <= 0) return true;
    if (out && !leaves && f.heap.depth > 0) {
        if (scratch && latency_fits(f, batch)) {
            return launch_latency(f, dtype, x, batch, out, stream, err,
                                  reinterpret_cast<unsigned char*>(scratch) + key_scratch_bytes(f), counters);
        }
        return launch_heap(f, dtype, x, batch, out, stream, err);
    }
    if (out && !leaves && f.sparse.teams > 0) return launch_sparse(f, dtype, x, batch, out, stream, err);
    if (out && !leaves && f.deep.records) return launch_deep(f, dtype, x, batch, out, stream, err);
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

// ---------------------------------------------------------------------------
// Predicting without allocating (montlok_model_predict_device_noalloc).
//
// Some callers cannot allocate GPU memory while they predict: serving loops
// whose device memory belongs to another allocator (a framework's caching
// pool that has already reserved the GPU, so a cudaMalloc of ours would fail
// or fragment it), and latency-critical paths that must not pay for
// cudaMalloc/cudaFree or the device-wide synchronisation cudaFree implies.
// For them this path runs the scratch-using variant of the generic kernel
// (per-warp key tables [slot][32] int32 in global memory, normally obtained
// per call) with its scratch in the fixed array below: 16 MiB, present on
// every GPU that loads this library until the process exits. The grid is cut
// to the warps whose tables fit; a model whose single 32-row table exceeds
// the array (more than 131072 feature/missing-rule slots, about 32768
// features) is rejected with MONTLOK_ERROR_UNSUPPORTED.
//
// On the host the array's name is only a stand-in, not a device address: the
// first call on each device, with that device current, looks the real
// address up with cudaGetSymbolAddress and caches it, so that first call
// should come before any stream capture. All calls share the array; every
// table is written in full by the kernel before it is read, so nothing needs
// clearing between calls, but calls whose kernels overlap on the GPU (on
// concurrent streams) race on it and must be serialised by the caller.
// ---------------------------------------------------------------------------

namespace {
constexpr size_t kNoAllocScratchBytes = size_t{16} << 20;
}  // namespace

static __device__ __align__(256) int g_noalloc_scratch[kNoAllocScratchBytes / sizeof(int)];

namespace mlk::cuda {
namespace {

// The device address of g_noalloc_scratch on `device`, looked up once.
bool noalloc_scratch(int device, int** out, std::string& err) {
    static std::mutex mu;
    static std::vector<std::pair<int, int*>> known;
    std::lock_guard<std::mutex> lock(mu);
    for (const auto& k : known) {
        if (k.first == device) {
            *out = k.second;
            return true;
        }
    }
    int previous = -1;
    if (cudaGetDevice(&previous) != cudaSuccess) previous = -1;
    if (previous != device && !check(cudaSetDevice(device), "cudaSetDevice", err)) return false;
    int* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_noalloc_scratch);
    if (previous >= 0 && previous != device) cudaSetDevice(previous);
    if (!check(e, "cudaGetSymbolAddress", err)) return false;
    known.emplace_back(device, p);
    *out = p;
    return true;
}

// 0 on success, else a montlok_status with `err` set.
int launch_forest_noalloc(const DevForest& f, int dtype, const void* x, long long batch, double* out,
                          cudaStream_t stream, std::string& err) {
    if (batch <= 0) return 0;
    // The complete-tree, multi-output and deep-tree kernels keep their key
    // tables in shared memory and need no device scratch at all.
    if (f.heap.depth > 0) return launch_heap(f, dtype, x, batch, out, stream, err) ? 0 : 7;
    if (f.sparse.teams > 0) return launch_sparse(f, dtype, x, batch, out, stream, err) ? 0 : 7;
    if (f.deep.records) return launch_deep(f, dtype, x, batch, out, stream, err) ? 0 : 7;
    const ForestArgs& a = f.args;
    // The generic kernel keeps its key tables in shared memory too when they
    // fit; only wider models use the static array.
    if (!shape_of(a).global_keys) return launch_forest(f, dtype, x, batch, out, nullptr, stream, err, nullptr) ? 0 : 7;
    const size_t table = static_cast<size_t>(a.slots) * 32 * sizeof(int);
    if (table > kNoAllocScratchBytes) {
        err = "the model needs " + std::to_string(table) + " bytes of key table per 32 rows, more than the " +
              std::to_string(kNoAllocScratchBytes) + "-byte scratch of the no-allocation path";
        return 4;
    }
    int* scratch = nullptr;
    if (!noalloc_scratch(f.device, &scratch, err)) return 7;
    const long long fit = static_cast<long long>(kNoAllocScratchBytes / table);  // warps whose tables fit
    const int wpc = fit >= 2 ? 2 : 1;
    const long long groups = (batch + 31) / 32;
    const long long want = std::min({(groups + wpc - 1) / wpc, fit / wpc, static_cast<long long>(f.sm_count) * 4});
    const int grid = static_cast<int>(std::max<long long>(want, 1));
    const int threads = 32 * wpc, smem = wpc * kStageBytes;
    const bool ties = !a.cast_f32, f64 = dtype == 2;
    const int kc_tmpl = a.K == 1 ? 1 : 8;
    const bool softmax_after = a.link == 2 && a.K > kMaxOut;
    for (int k0 = 0; k0 < a.K; k0 += kMaxOut) {
        int kc = std::min(kMaxOut, a.K - k0);
        int link_here = softmax_after ? 0 : 1;
        int k0v = k0;
        int* no_leaves = nullptr;
        void* k = pick(ties, false, kc_tmpl, true, f64);
        void* args[] = {const_cast<ForestArgs*>(&a), const_cast<void**>(&x), &batch, &out, &no_leaves, &k0v, &kc,
                        &link_here, &scratch};
        if (!check(cudaLaunchKernel(k, grid, threads, args, smem, stream), "no-allocation kernel launch", err)) {
            return 7;
        }
    }
    if (softmax_after) {
        const int tpb = 128;
        softmax_rows<<<static_cast<unsigned>((batch + tpb - 1) / tpb), tpb, 0, stream>>>(out, batch, a.K);
        if (!check(cudaGetLastError(), "softmax kernel launch", err)) return 7;
    }
    return 0;
}

}  // namespace
}  // namespace mlk::cuda

extern "C" const char* mlk_cuda_kernel_name(const mlk_dev_forest* forest, size_t batch) {
    using namespace mlk::cuda;
    const DevForest& f = forest->f;
    const long long rows = static_cast<long long>(batch);
    if (f.heap.depth > 0) {
        if (latency_fits(f, rows)) return "small-batch";
        return heap_staged(f, rows) ? "complete-tree-staged" : "complete-tree";
    }
    if (f.sparse.teams > 0) return "multi-output";
    if (f.deep.records) return "deep-tree";
    return shape_of(f.args).global_keys ? "generic-global-keys" : "generic";
}

extern "C" size_t mlk_cuda_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

extern "C" int mlk_cuda_predict_device_noalloc(const mlk_dev_forest* forest, int dtype, const void* x, size_t batch,
                                               double* out, void* stream, char* err, size_t errlen) {
    std::string e;
    const int status = mlk::cuda::launch_forest_noalloc(forest->f, dtype, x, static_cast<long long>(batch), out,
                                                        static_cast<cudaStream_t>(stream), e);
    if (status != 0 && err && errlen) {
        const size_t n = std::min(errlen - 1, e.size());
        std::memcpy(err, e.data(), n);
        err[n] = '\0';
    }
    return status;
}
