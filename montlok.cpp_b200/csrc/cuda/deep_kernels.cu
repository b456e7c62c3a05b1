// Deep-tree predict kernel for sm_100a: one output, trees too deep for the
// complete-tree layout (random forests grown to depth 20: c3).
//
// Nodes. Every tree is laid out breadth-first with the two children of a
// split adjacent, 8 bytes a node {W, index of the left child} in one global
// array; a split's word packs the threshold key and the slot as in the
// complete-tree kernel, W = (T & ~mask) | slot, and a leaf is
// {(leaf + 1) << slot_bits | pad slot, own index}: the pad slot's key is
// INT32_MIN, so a leaf never goes right and the walk stays on it, and its
// word names the leaf's value in a separate array. A 20-level forest of 9M
// nodes is 73 MB of nodes plus its leaf values, which stays in the 126 MB L2;
// node loads carry an evict-last cache policy and the rows an evict-first one
// so the streaming input does not push the trees out.
//
// Work split. Each warp owns 32 rows (a lane per row) and their key tables
// in shared memory ([slot][32] int32, k | mask for finite keys), independent
// of the other warps of its CTA. A lane walks kIlp trees side by side, for
// as many steps as the deepest of them plus one load that reads the leaf it
// stands on; trees whose walk met a tie in the packed compare are walked
// again with those splits decided exactly (exact_right). Leaves are added in
// tree order into 64-tree block partials, block 0 onto the base score, the
// later blocks added in order: the reference's association
// (trees.cpp:366-388).
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
constexpr int kSmemLimit = 227 * 1024;

__host__ __device__ inline int warp_bytes(int slots) { return slots * 32 * 4 + kPrepTileBytes; }

__device__ __forceinline__ uint64_t evict_last_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint2 ldg_node(const uint2* p, uint64_t policy) {
    uint2 v;
    asm volatile("ld.global.nc.L2::cache_hint.v2.u32 {%0, %1}, [%2], %3;"
                 : "=r"(v.x), "=r"(v.y)
                 : "l"(p), "l"(policy));
    return v;
}

// One tree walked exactly for one row; returns the leaf's node index.
template <typename XT>
__device__ __noinline__ uint32_t walk_exact(const ForestArgs& a, const DeepArgs& d, uint32_t root, int depth,
                                            const int* col, uint32_t mask, const XT* __restrict__ x, long long row,
                                            long long batch) {
    uint32_t p = root;
    for (int s = 0; s < depth; ++s) {
        const uint2 n = __ldg(d.nodes + p);
        const int k = col[(n.x & mask) * 32];
        bool right = k > static_cast<int>(n.x);
        if (static_cast<uint32_t>(k ^ static_cast<int>(n.x)) <= mask) {
            const int node = __ldg(d.node_ids + p);
            if (node >= 0) right = exact_right(a, x, row, batch, node);
        }
        p = n.y + (right ? 1u : 0u);
    }
    return p;
}

template <bool LEAF32, typename XT>
__global__ void __launch_bounds__(kWarps * 32) deep_kernel(const ForestArgs a, const DeepArgs d,
                                                            const XT* __restrict__ x, long long batch,
                                                            double* __restrict__ out) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int* keys = reinterpret_cast<int*>(smem + warp * warp_bytes(a.slots));
    double* tile = reinterpret_cast<double*>(smem + warp * warp_bytes(a.slots) + a.slots * 32 * 4);
    const uint32_t mask = (1u << d.slot_bits) - 1u;
    const uint64_t policy = evict_last_policy();
    const long long groups = (batch + 31) / 32;
    const long long me = static_cast<long long>(blockIdx.x) * kWarps + warp;
    const long long all = static_cast<long long>(gridDim.x) * kWarps;
    const int blocks = (a.T + kTreeBlock - 1) / kTreeBlock;
    const int* col = keys + lane;
    for (long long g = me; g < groups; g += all) {
        const long long row0 = g * 32, row = row0 + lane;
        prepare_rows<32>(a, x, row0, batch, keys, tile, lane, 0, a.F, static_cast<int>(mask));
        keys[a.pad_slot * 32 + lane] = INT_MIN;
        __syncwarp();
        double acc = 0.0;
        for (int b = 0; b < blocks; ++b) {
            double part = (b == 0 && !a.mean) ? __ldg(a.base) : 0.0;
            const int end = min(a.T, (b + 1) * kTreeBlock);
            for (int t0 = b * kTreeBlock; t0 < end; t0 += kIlp) {
                const int nt = min(kIlp, end - t0);
                uint32_t p[kIlp];
                uint2 n[kIlp];
                bool tie[kIlp];
                int depth = 0;
#pragma unroll
                for (int t = 0; t < kIlp; ++t) {
                    p[t] = t < nt ? static_cast<uint32_t>(__ldg(d.roots + t0 + t)) : 0u;
                    if (t < nt) depth = max(depth, __ldg(a.depth + t0 + t));
                    tie[t] = false;
                }
                for (int s = 0;; ++s) {
#pragma unroll
                    for (int t = 0; t < kIlp; ++t) {
                        if (t < nt) n[t] = ldg_node(d.nodes + p[t], policy);
                    }
                    if (s == depth) break;  // the last load read the leaf each lane stands on
#pragma unroll
                    for (int t = 0; t < kIlp; ++t) {
                        if (t < nt) {
                            const int k = col[(n[t].x & mask) * 32];
                            tie[t] |= static_cast<uint32_t>(k ^ static_cast<int>(n[t].x)) <= mask;
                            p[t] = n[t].y + (k > static_cast<int>(n[t].x) ? 1u : 0u);
                        }
                    }
                }
                bool any = false;
#pragma unroll
                for (int t = 0; t < kIlp; ++t) any |= tie[t];
                if (__any_sync(0xffffffffu, any)) {
#pragma unroll
                    for (int t = 0; t < kIlp; ++t) {
                        if (tie[t]) {
                            const uint32_t leaf = walk_exact(a, d, __ldg(d.roots + t0 + t), depth, col, mask, x, row,
                                                             batch);
                            n[t] = __ldg(d.nodes + leaf);
                        }
                    }
                }
#pragma unroll
                for (int t = 0; t < kIlp; ++t) {
                    if (t < nt) {
                        const uint32_t leaf = (n[t].x >> d.slot_bits) - 1u;
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
