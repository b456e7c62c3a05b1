// Deep-tree predict kernel for sm_100a: one output, trees too deep for the
// complete-tree layout (random forests grown to depth 20: c3).
//
// Records. A tree is cut into two-level records, laid out breadth first: a
// split, the split words of its two children and the four exits below them,
// {W top, W left, W right, 0, LL, LR, RL, RR}, 32 bytes that one 256-bit load
// brings in, so a walk pays one dependent L2 round trip per two levels. Split
// words pack the threshold key and the slot as in the complete-tree kernel,
// W = (T & ~mask) | slot; a child that is a leaf gets the pad slot's word
// (its key is INT32_MIN, so it never goes right) and both its exits name the
// leaf. An exit is the index of the next record, or, with the top bit set,
// the number of a leaf value. c3's 200 trees of depth <= 20 are about 80 MB
// of records and 40 MB of float64 leaf values, held in the 126 MB L2; record
// loads carry an evict-last cache policy so the streaming input does not push
// the records out.
//
// Work split. Each warp owns 32 rows (a lane per row) and their key tables
// in shared memory ([slot][32] int32, (k & ~mask) | slot), independent
// of the other warps of its CTA. A lane walks kIlp trees side by side, for
// as many records as the longest walk among them, then loads the leaf values;
// trees whose walk met a tie in the packed compare are walked again with
// those splits decided exactly (exact_right). Leaves are added in tree order
// into 64-tree block partials, block 0 onto the base score, the later blocks
// added in order: the reference's association (trees.cpp:366-388).
#include <algorithm>
#include <cstdint>
#include <mutex>
#include <vector>

#include "device_common.cuh"
#include "forest.cuh"

namespace mlk::cuda {
namespace {

constexpr int kIlp = 8;    // trees a lane walks side by side
constexpr int kWarps = 4;  // warps per CTA, each on its own rows
// Resident CTAs per SM the register budget is cut for (128 registers a
// thread): 16 warps with 8 record loads each in flight ran c3 faster than 12
// warps with 10 or 12, or 20 warps with 6.
constexpr int kMinCtas = 4;
constexpr int kSmemLimit = 227 * 1024;
constexpr uint32_t kLeaf = 0x80000000u;  // exit bit: the rest is a leaf number

__host__ __device__ inline int warp_bytes(int slots) { return slots * 32 * 4; }

__device__ __forceinline__ uint64_t evict_last_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

struct Record {
    uint32_t w[8];
};

// One record in a single 256-bit load (records are 32-byte aligned).
__device__ __forceinline__ Record ldg_record(const uint32_t* p, uint64_t policy) {
    Record r;
    asm volatile("ld.global.nc.L2::cache_hint.v8.u32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8], %9;"
                 : "=r"(r.w[0]), "=r"(r.w[1]), "=r"(r.w[2]), "=r"(r.w[3]), "=r"(r.w[4]), "=r"(r.w[5]),
                   "=r"(r.w[6]), "=r"(r.w[7])
                 : "l"(p), "l"(policy));
    return r;
}

// The key a split word reads and whether the packed compare tied.
__device__ __forceinline__ bool goes_right(const int* col, uint32_t w, uint32_t mask, bool& tie) {
    const int k = col[(w & mask) * 32];  // (key & ~mask) | slot: the word's low bits
    tie |= k == static_cast<int>(w);
    return k > static_cast<int>(w);
}

// One tree walked exactly for one row; returns the exit naming its leaf.
template <typename XT>
__device__ __noinline__ uint32_t walk_exact(const ForestArgs& a, const DeepArgs& d, uint32_t p, int steps,
                                            const int* col, uint32_t mask, const XT* __restrict__ x, long long row,
                                            long long batch) {
    for (int s = 0; s < steps && !(p & kLeaf); ++s) {
        const uint4* r = reinterpret_cast<const uint4*>(d.records + static_cast<size_t>(p) * 8);
        const uint4 lo = __ldg(r), hi = __ldg(r + 1);
        const int* ids = d.node_ids + static_cast<size_t>(p) * 3;
        bool tie = false;
        bool right = goes_right(col, lo.x, mask, tie);
        if (tie) {
            const int node = __ldg(ids);
            if (node >= 0) right = exact_right(a, x, row, batch, node);
        }
        const uint32_t wc = right ? lo.z : lo.y;
        tie = false;
        bool below = goes_right(col, wc, mask, tie);
        if (tie) {
            const int node = __ldg(ids + (right ? 2 : 1));
            if (node >= 0) below = exact_right(a, x, row, batch, node);
        }
        p = right ? (below ? hi.w : hi.z) : (below ? hi.y : hi.x);
    }
    return p;
}

template <bool LEAF32, typename XT>
__global__ void __launch_bounds__(kWarps * 32, kMinCtas) deep_kernel(const __grid_constant__ ForestArgs a, const __grid_constant__ DeepArgs d,
                                                            const XT* __restrict__ x, long long batch,
                                                            double* __restrict__ out) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int* keys = reinterpret_cast<int*>(smem + warp * warp_bytes(a.slots));
    const uint32_t mask = (1u << d.slot_bits) - 1u;
    const uint64_t policy = evict_last_policy();
    const long long groups = (batch + 31) / 32;
    const long long me = static_cast<long long>(blockIdx.x) * kWarps + warp;
    const long long all = static_cast<long long>(gridDim.x) * kWarps;
    const int blocks = (a.T + kTreeBlock - 1) / kTreeBlock;
    const int* col = keys + lane;
    for (long long g = me; g < groups; g += all) {
        const long long row0 = g * 32, row = row0 + lane;
        __syncwarp();  // the previous group's walks are done with the table
        prepare_own_row<32>(a, x, row, batch, keys + lane, 0, a.F, static_cast<int>(mask));
        keys[a.pad_slot * 32 + lane] = INT_MIN;
        __syncwarp();
        double acc = 0.0;
        for (int b = 0; b < blocks; ++b) {
            double part = (b == 0 && !a.mean) ? __ldg(a.base) : 0.0;
            const int end = min(a.T, (b + 1) * kTreeBlock);
            for (int t0 = b * kTreeBlock; t0 < end; t0 += kIlp) {
                const int nt = min(kIlp, end - t0);
                uint32_t p[kIlp];
                bool tie[kIlp];
                int steps = 0;
#pragma unroll
                for (int t = 0; t < kIlp; ++t) {
                    p[t] = t < nt ? __ldg(d.roots + t0 + t) : kLeaf;
                    if (t < nt) steps = max(steps, __ldg(d.steps + t0 + t));
                    tie[t] = false;
                }
                for (int s = 0; s < steps; ++s) {
                    Record r[kIlp];
#pragma unroll
                    for (int t = 0; t < kIlp; ++t) {
                        if (!(p[t] & kLeaf)) r[t] = ldg_record(d.records + static_cast<size_t>(p[t]) * 8, policy);
                    }
#pragma unroll
                    for (int t = 0; t < kIlp; ++t) {
                        if (!(p[t] & kLeaf)) {
                            const bool right = goes_right(col, r[t].w[0], mask, tie[t]);
                            const bool below = goes_right(col, right ? r[t].w[2] : r[t].w[1], mask, tie[t]);
                            p[t] = right ? (below ? r[t].w[7] : r[t].w[6]) : (below ? r[t].w[5] : r[t].w[4]);
                        }
                    }
                }
                bool any = false;
#pragma unroll
                for (int t = 0; t < kIlp; ++t) any |= tie[t];
                if (__any_sync(0xffffffffu, any)) {
#pragma unroll
                    for (int t = 0; t < kIlp; ++t) {
                        if (tie[t]) p[t] = walk_exact(a, d, __ldg(d.roots + t0 + t), steps, col, mask, x, row, batch);
                    }
                }
#pragma unroll
                for (int t = 0; t < kIlp; ++t) {
                    if (t < nt) {
                        const uint32_t leaf = p[t] & ~kLeaf;
                        const double v = LEAF32 ? static_cast<double>(__ldg(static_cast<const float*>(d.leaves) + leaf))
                                                : __ldg(static_cast<const double*>(d.leaves) + leaf);
                        part = __dadd_rn(part, v);
                    }
                }
            }
            acc = b == 0 ? part : __dadd_rn(acc, part);
        }
        if (row < batch) {
            double v[1] = {acc};
            if (a.mean) {
                const int c = __ldg(a.counts);
                v[0] = __dadd_rn(__ldg(a.base), c ? __ddiv_rn(v[0], static_cast<double>(c)) : 0.0);
            }
            apply_link<1>(a, v, 1);
            out[row] = v[0];
        }
        __syncwarp();
    }
}

void* pick_deep(bool leaf32, bool f64) {
    if (leaf32) return f64 ? reinterpret_cast<void*>(&deep_kernel<true, double>)
                           : reinterpret_cast<void*>(&deep_kernel<true, float>);
    return f64 ? reinterpret_cast<void*>(&deep_kernel<false, double>)
               : reinterpret_cast<void*>(&deep_kernel<false, float>);
}

}  // namespace

bool deep_fits(int slots) { return kWarps * warp_bytes(slots) <= kSmemLimit; }

bool launch_deep(const DevForest& f, int dtype, const void* x, long long batch, double* out, cudaStream_t stream,
                 std::string& err) {
    const DeepArgs& d = f.deep;
    void* k = pick_deep(d.leaf32, dtype == 2);
    const int smem = kWarps * warp_bytes(f.args.slots);
    {
        static std::mutex mu;
        static std::vector<std::pair<void*, int>> set;
        std::lock_guard<std::mutex> lock(mu);
        if (std::find(set.begin(), set.end(), std::make_pair(k, f.device)) == set.end()) {
            const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
            if (e != cudaSuccess) {
                err = std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
                return false;
            }
            set.emplace_back(k, f.device);
        }
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kWarps * 32, smem) != cudaSuccess || per_sm < 1) {
        per_sm = 1;
        cudaGetLastError();
    }
    const long long groups = (batch + 31) / 32;
    const long long want = (groups + kWarps - 1) / kWarps;
    const int grid = static_cast<int>(std::min<long long>(want, static_cast<long long>(f.sm_count) * per_sm));
    ForestArgs a = f.args;
    DeepArgs dd = d;
    void* args[] = {&a, &dd, const_cast<void**>(&x), &batch, &out};
    const cudaError_t e = cudaLaunchKernel(k, grid, kWarps * 32, args, smem, stream);
    if (e != cudaSuccess) {
        err = std::string("deep-tree kernel launch: ") + cudaGetErrorString(e);
        return false;
    }
    return true;
}

}  // namespace mlk::cuda
