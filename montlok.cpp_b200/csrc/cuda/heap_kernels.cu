// Complete-tree predict kernel for sm_100a (depth <= 8, one output).
//
// Every tree is stored as a complete binary tree of depth D in heap order
// (children of split i at 2i+1 and 2i+2; shallower leaves are padded with
// always-left splits), one 16-byte aligned record per tree: 2^D - 1 splits of
// 8 bytes (threshold key T, slot) followed by 2^D leaf values (float32 when
// every leaf is exactly a float, else float64). Child addresses are implicit,
// so a step is: one 8-byte shared load of the split, one shared load of the
// row's key, one compare, and new offset = 2 * offset + (8 or 16).
//
// A CTA owns R rows (one per thread) for the whole ensemble. Their key
// tables stay in shared memory ([slot][R] int32, lane l reading bank l), and
// the trees stream through two shared buffers of kChunk trees each: thread 0
// issues a 1D bulk async copy (cp.async.bulk, completion on an mbarrier) of
// chunk c+1 while every thread walks the kChunk trees of chunk c side by
// side. Waits on the mbarrier are bounded; on timeout the kernel records an
// error in the forest's status word and stops.
//
// Sums follow the reference order exactly (trees.cpp:366-388): a chunk never
// straddles a block of 64 trees, block 0 adds onto the base score, later
// blocks sum from 0.0 and are added when they end.
#include <algorithm>
#include <cstdint>
#include <mutex>
#include <vector>

#include "device_common.cuh"
#include "forest.cuh"

namespace mlk::cuda {
namespace {

constexpr int kChunk = 8;  // trees per streamed chunk = trees one thread walks side by side
static_assert(kTreeBlock % kChunk == 0, "chunks never straddle a block of 64 trees");
constexpr long long kSpinLimit = 1ll << 26;  // mbarrier polls before giving up

__host__ __device__ constexpr int heap_tree_bytes(int depth, bool leaf32) {
    return (((1 << depth) - 1) * 8 + (1 << depth) * (leaf32 ? 4 : 8) + 15) & ~15;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(bar)) : "memory");
}

// Thread 0: arm the barrier for `bytes` and start the copy global -> shared.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// Waits for phase `parity` of `bar` to complete; false after kSpinLimit polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    for (long long i = 0; i < kSpinLimit; ++i) {
        uint32_t done;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
            : "=r"(done)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

template <int D, int R, bool LEAF32, bool TIES, typename XT>
__global__ void __launch_bounds__(R) heap_kernel(const ForestArgs a, const HeapArgs h, const XT* __restrict__ x,
                                                 long long batch, double* __restrict__ out) {
    constexpr int kSplits = (1 << D) - 1;
    constexpr int kTreeBytes = heap_tree_bytes(D, LEAF32);
    constexpr int kChunkBytes = kChunk * kTreeBytes;
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
    int* keys = reinterpret_cast<int*>(smem + 128);
    const int key_bytes = (a.slots * R * 4 + 127) & ~127;
    double* stage = reinterpret_cast<double*>(smem + 128 + key_bytes);
    const uint32_t tree_off = 128 + key_bytes + (R / 32) * kStageBytes;
    unsigned char* trees = smem + tree_off;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int chunks = (a.T + kChunk - 1) / kChunk;
    const long long groups = (batch + R - 1) / R;
    if (tid == 0) {
        mbar_init(&bar[0]);
        mbar_init(&bar[1]);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    // Thread 0 counts the copies it issued and the ones it saw complete, so a
    // failing CTA can wait out whatever is still in flight before it exits.
    unsigned issued = 0, seen = 0;
    auto issue = [&](int c, unsigned seq) {
        const int n = min(kChunk, a.T - c * kChunk);
        bulk_load(trees + (seq & 1) * kChunkBytes, h.trees + static_cast<size_t>(c) * kChunkBytes,
                  static_cast<uint32_t>(n * kTreeBytes), &bar[seq & 1]);
        ++issued;
    };

    unsigned seq = 0;  // chunks consumed by this CTA so far: buffer seq & 1, phase (seq >> 1) & 1
    const uint32_t col = 128 + tid * 4;  // this thread's key column, as an offset from smem
    for (long long g = blockIdx.x; g < groups; g += gridDim.x) {
        const long long row0 = g * R;
        if (tid == 0) issue(0, seq);
        prepare_group<R>(a, x, row0 + warp * 32, batch, keys + warp * 32, stage + warp * (kStageBytes / 8), lane);
        __syncthreads();
        const long long row = row0 + tid;
        double acc = a.mean ? 0.0 : __ldg(a.base);
        double part = 0.0;
        bool bad = false;  // this thread's wait timed out; decided CTA-wide at the next barrier
        for (int c = 0; c < chunks; ++c, ++seq) {
            if (c > 0 && __syncthreads_or(bad)) break;  // everyone is done with chunk c - 1
            if (tid == 0 && c + 1 < chunks) issue(c + 1, seq + 1);
            if (!mbar_wait(&bar[seq & 1], (seq >> 1) & 1)) {
                bad = true;
                continue;
            }
            if (tid == 0) ++seen;
            // Offsets from `smem`: 32-bit shared addresses. p[t] is tree t's
            // current split; its children sit at base + 2 * (p - base) + 8 / + 16.
            const uint32_t buf = tree_off + (seq & 1) * kChunkBytes;
            const int live = min(kChunk, a.T - c * kChunk);
            uint32_t p[kChunk];
#pragma unroll
            for (int t = 0; t < kChunk; ++t) p[t] = buf + t * kTreeBytes;
#pragma unroll
            for (int d = 0; d < D; ++d) {
#pragma unroll
                for (int t = 0; t < kChunk; ++t) {
                    const uint32_t base = buf + t * kTreeBytes;
                    const int2 n = *reinterpret_cast<const int2*>(smem + p[t]);
                    const int kv = *reinterpret_cast<const int*>(smem + col + n.y * (R * 4));
                    bool right = kv > n.x;
                    if (TIES && kv == n.x && t < live) {
                        const int node =
                            __ldg(h.node_ids + static_cast<size_t>(c * kChunk + t) * kSplits + ((p[t] - base) >> 3));
                        right = exact_right(a, x, row, batch, node);
                    }
                    p[t] = 2 * p[t] - base + (right ? 16u : 8u);
                }
            }
            const bool first_block = c * kChunk < kTreeBlock;
            if (!first_block && (c * kChunk) % kTreeBlock == 0) {
                // A block of 64 trees ended with the previous chunk.
                if (c * kChunk >= 2 * kTreeBlock) acc = __dadd_rn(acc, part);
                part = 0.0;
            }
#pragma unroll
            for (int t = 0; t < kChunk; ++t) {
                if (t < live) {
                    const uint32_t base = buf + t * kTreeBytes;
                    const uint32_t leaf = ((p[t] - base) >> 3) - kSplits;
                    const uint32_t values = base + kSplits * 8;
                    const double v = LEAF32 ? static_cast<double>(*reinterpret_cast<const float*>(smem + values + 4 * leaf))
                                            : *reinterpret_cast<const double*>(smem + values + 8 * leaf);
                    if (first_block) acc = __dadd_rn(acc, v);
                    else part = __dadd_rn(part, v);
                }
            }
        }
        if (__syncthreads_or(bad)) {
            // Leave no bulk copy in flight into shared memory: wait (bounded)
            // for the one issued after the last completed chunk, then stop.
            if (tid == 0) {
                atomicExch(h.status, 1);
                for (unsigned s = seen; s < issued; ++s) mbar_wait(&bar[s & 1], (s >> 1) & 1);
            }
            return;
        }
        if (a.T > kTreeBlock) acc = __dadd_rn(acc, part);
        if (row < batch) {
            double v[1] = {acc};
            if (a.mean) {
                const int n = __ldg(a.counts);
                v[0] = __dadd_rn(__ldg(a.base), n ? __ddiv_rn(v[0], static_cast<double>(n)) : 0.0);
            }
            apply_link<1>(a, v, 1);
            out[row] = v[0];
        }
        __syncthreads();  // keys and buffers are rewritten by the next group
    }
}

template <int D, int R, bool LEAF32, bool TIES, typename XT>
void* heap_of() {
    return reinterpret_cast<void*>(&heap_kernel<D, R, LEAF32, TIES, XT>);
}

template <int D, int R>
void* pick_leaf(bool leaf32, bool ties, bool f64) {
    if (leaf32) {
        if (ties) return f64 ? heap_of<D, R, true, true, double>() : heap_of<D, R, true, true, float>();
        return f64 ? heap_of<D, R, true, false, double>() : heap_of<D, R, true, false, float>();
    }
    if (ties) return f64 ? heap_of<D, R, false, true, double>() : heap_of<D, R, false, true, float>();
    return f64 ? heap_of<D, R, false, false, double>() : heap_of<D, R, false, false, float>();
}

template <int D>
void* pick_rows(int rows, bool leaf32, bool ties, bool f64) {
    switch (rows) {
        case 128: return pick_leaf<D, 128>(leaf32, ties, f64);
        case 64: return pick_leaf<D, 64>(leaf32, ties, f64);
        case 32: return pick_leaf<D, 32>(leaf32, ties, f64);
    }
    return nullptr;
}

void* pick_heap(int depth, int rows, bool leaf32, bool ties, bool f64) {
    switch (depth) {
        case 1: return pick_rows<1>(rows, leaf32, ties, f64);
        case 2: return pick_rows<2>(rows, leaf32, ties, f64);
        case 3: return pick_rows<3>(rows, leaf32, ties, f64);
        case 4: return pick_rows<4>(rows, leaf32, ties, f64);
        case 5: return pick_rows<5>(rows, leaf32, ties, f64);
        case 6: return pick_rows<6>(rows, leaf32, ties, f64);
        case 7: return pick_rows<7>(rows, leaf32, ties, f64);
        case 8: return pick_rows<8>(rows, leaf32, ties, f64);
    }
    return nullptr;
}

constexpr int kHeapSmemLimit = 227 * 1024;

}  // namespace

int heap_smem_bytes(int slots, int depth, bool leaf32, int rows) {
    return 128 + ((slots * rows * 4 + 127) & ~127) + (rows / 32) * kStageBytes +
           2 * kChunk * heap_tree_bytes(depth, leaf32);
}

int heap_record_bytes(int depth, bool leaf32) { return heap_tree_bytes(depth, leaf32); }

int heap_plan_rows(int slots, int depth, bool leaf32) {
    if (depth < 1 || depth > 8) return 0;
    for (int rows : {128, 64, 32}) {
        if (heap_smem_bytes(slots, depth, leaf32, rows) <= kHeapSmemLimit) return rows;
    }
    return 0;
}

bool launch_heap(const DevForest& f, int dtype, const void* x, long long batch, double* out, cudaStream_t stream,
                 std::string& err) {
    const HeapArgs& h = f.heap;
    const bool f64 = dtype == 2;
    void* k = pick_heap(h.depth, h.rows, h.leaf32, !f.args.cast_f32, f64);
    if (!k) {
        err = "no complete-tree kernel for this model";
        return false;
    }
    const int smem = heap_smem_bytes(f.args.slots, h.depth, h.leaf32, h.rows);
    {
        static std::mutex mu;
        static std::vector<std::pair<void*, int>> set;
        std::lock_guard<std::mutex> lock(mu);
        if (std::find(set.begin(), set.end(), std::make_pair(k, f.device)) == set.end()) {
            const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kHeapSmemLimit);
            if (e != cudaSuccess) {
                err = std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
                return false;
            }
            set.emplace_back(k, f.device);
        }
    }
    const long long groups = (batch + h.rows - 1) / h.rows;
    const int per_sm = std::max(1, kHeapSmemLimit / (smem + 1024));
    const int grid = static_cast<int>(std::min<long long>(groups, static_cast<long long>(f.sm_count) * per_sm));
    ForestArgs a = f.args;
    HeapArgs hh = h;
    void* args[] = {&a, &hh, const_cast<void**>(&x), &batch, &out};
    const cudaError_t e = cudaLaunchKernel(k, grid, h.rows, args, smem, stream);
    if (e != cudaSuccess) {
        err = std::string("complete-tree kernel launch: ") + cudaGetErrorString(e);
        return false;
    }
    return true;
}

}  // namespace mlk::cuda
