// Complete-tree predict kernel for sm_100a (depth <= 8, one output).
//
// Every tree is stored as a complete binary tree of depth D in heap order
// (children of split i at 2i+1 and 2i+2; shallower leaves are padded with
// always-left splits), one 16-byte aligned record per tree: 2^D - 1 splits of
// 8 bytes (threshold key T, byte offset of the split's slot in the key table)
// followed by 2^D leaf values (float32 when every leaf is exactly a float,
// else float64). Child addresses are implicit, so a step is: one 8-byte
// shared load of the split, one shared load of the row's key, one compare,
// and new address = 2 * address + (8 or 16) - base.
//
// A CTA owns R rows for the whole ensemble and runs two teams of R threads
// (one thread per row in each). The rows' key tables stay in shared memory
// ([slot][R] int32, lane l always reading bank l). Trees stream through a ring
// of four chunk buffers (kChunk trees each; chunk c of every row group uses
// buffer c % 4) filled by one-dimensional bulk async copies (cp.async.bulk,
// completion counted on one mbarrier per buffer): while team 0 walks chunk
// 2p and team 1 walks chunk 2p + 1, the copies of chunks 2p + 2 and 2p + 3
// are in flight. Team 1 hands the leaf it reached in each tree to team 0
// through a small shared exchange, and team 0 adds every leaf value in tree
// order, so the float64 sums are the reference's (trees.cpp:366-388): a chunk
// never straddles a block of 64 trees, block 0 adds onto the base score,
// later blocks sum from 0.0 and are added when they end.
//
// The device tree array is padded with inert trees to whole chunks, so every
// copy is a full chunk and no walk ever reads an unwritten buffer. Waits on
// the mbarriers are bounded; on timeout the kernel records an error in the
// forest's status word, waits (bounded) for its copies in flight, and stops.
#include <algorithm>
#include <cstdint>
#include <mutex>
#include <vector>

#include "device_common.cuh"
#include "forest.cuh"

namespace mlk::cuda {
namespace {

constexpr int kChunk = 8;    // trees per streamed chunk = trees one thread walks side by side
constexpr int kBuffers = 4;  // chunk buffers: two walked, two in flight
static_assert(kTreeBlock % kChunk == 0, "chunks never straddle a block of 64 trees");
constexpr int kTile = 16;                         // features per transpose tile
constexpr int kTileBytes = 32 * (kTile + 1) * 8;  // one warp's transpose tile
constexpr long long kSpinLimit = 1ll << 26;       // mbarrier polls before giving up
constexpr int kHeapSmemLimit = 227 * 1024;

__host__ __device__ constexpr int heap_tree_bytes(int depth, bool leaf32) {
    return (((1 << depth) - 1) * 8 + (1 << depth) * (leaf32 ? 4 : 8) + 15) & ~15;
}

__host__ __device__ constexpr int align128(int n) { return (n + 127) & ~127; }

// Shared memory layout (byte offsets): barriers at 0 | keys [slots][R] int32
// | exchange [kChunk][R] u8 | ring of four chunk buffers; during the prepare
// phase the ring past buffer 1 holds the transpose tiles.
struct Layout {
    int keys, exchange, ring, total;
};

__host__ __device__ inline Layout layout_of(int slots, int depth, bool leaf32, int rows) {
    Layout l{};
    l.keys = 128;
    l.exchange = l.keys + align128(slots * rows * 4);
    l.ring = l.exchange + align128(kChunk * rows);
    const int chunk = kChunk * heap_tree_bytes(depth, leaf32);
    const int tiles = 2 * (rows / 32) * kTileBytes;  // every warp of both teams prepares
    l.total = l.ring + align128(max(kBuffers * chunk, 2 * chunk + tiles));
    return l;
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

// Shared-memory loads at explicit 32-bit shared addresses.
__device__ __forceinline__ int2 lds_v2(uint32_t a) {
    int2 v;
    asm volatile("ld.shared.v2.s32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ int lds_s32(uint32_t a) {
    int v;
    asm volatile("ld.shared.s32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ double lds_leaf(uint32_t a, bool f32) {
    if (f32) {
        float v;
        asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
        return static_cast<double>(v);
    }
    double v;
    asm volatile("ld.shared.f64 %0, [%1];" : "=d"(v) : "r"(a));
    return v;
}

// Starts pulling [p, p + bytes) into L2 (16-byte aligned interior only).
__device__ __forceinline__ void prefetch_l2(const void* p, size_t bytes) {
    const uintptr_t lo = (reinterpret_cast<uintptr_t>(p) + 15) & ~uintptr_t{15};
    const uintptr_t hi = (reinterpret_cast<uintptr_t>(p) + bytes) & ~uintptr_t{15};
    for (uintptr_t a = lo; a < hi; a += (1u << 20)) {
        const uint32_t n = static_cast<uint32_t>(min(static_cast<uintptr_t>(1u << 20), hi - a));
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(n) : "memory");
    }
}

// Walks the kChunk trees of the chunk at shared address `buf` for one row;
// leaf[t] receives the index (0 .. 2^D - 1) of the leaf reached in tree t.
template <int D, bool TIES, typename XT>
__device__ __forceinline__ void walk_chunk(const ForestArgs& a, const HeapArgs& h, uint32_t buf, uint32_t col,
                                           int chunk, int live, const XT* x, long long row, long long batch,
                                           uint32_t (&leaf)[kChunk], int tree_bytes) {
    constexpr int kSplits = (1 << D) - 1;
    uint32_t p[kChunk], go_left[kChunk], go_right[kChunk];
#pragma unroll
    for (int t = 0; t < kChunk; ++t) {
        p[t] = buf + t * tree_bytes;
        go_left[t] = 8u - p[t];
        go_right[t] = 16u - p[t];
    }
#pragma unroll
    for (int d = 0; d < D; ++d) {
        int2 n[kChunk];
        int kv[kChunk];
#pragma unroll
        for (int t = 0; t < kChunk; ++t) n[t] = lds_v2(p[t]);
#pragma unroll
        for (int t = 0; t < kChunk; ++t) kv[t] = lds_s32(col + n[t].y);
#pragma unroll
        for (int t = 0; t < kChunk; ++t) {
            bool right = kv[t] > n[t].x;
            if (TIES && kv[t] == n[t].x && t < live) {
                const uint32_t base = buf + t * tree_bytes;
                const int node = __ldg(h.node_ids + static_cast<size_t>(chunk * kChunk + t) * kSplits +
                                       ((p[t] - base) >> 3));
                right = exact_right(a, x, row, batch, node);
            }
            p[t] = 2 * p[t] + (right ? go_right[t] : go_left[t]);
        }
    }
#pragma unroll
    for (int t = 0; t < kChunk; ++t) leaf[t] = ((p[t] - (buf + t * tree_bytes)) >> 3) - kSplits;
}

template <int D, int R, bool LEAF32, bool TIES, typename XT>
__global__ void __launch_bounds__(2 * R) heap_kernel(const ForestArgs a, const HeapArgs h, const XT* __restrict__ x,
                                                     long long batch, double* __restrict__ out) {
    constexpr int kSplits = (1 << D) - 1;
    constexpr int kTreeBytes = heap_tree_bytes(D, LEAF32);
    constexpr int kChunkBytes = kChunk * kTreeBytes;
    constexpr int kLeafBytes = LEAF32 ? 4 : 8;
    extern __shared__ __align__(128) unsigned char smem[];
    const Layout L = layout_of(a.slots, D, LEAF32, R);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
    int* keys = reinterpret_cast<int*>(smem + L.keys);
    unsigned char* exchange = smem + L.exchange;
    unsigned char* ring = smem + L.ring;
    const uint32_t ring0 = smem_u32(ring);

    const int tid = threadIdx.x;
    const int team = tid / R, r = tid % R;  // team 0 walks chunk 2p, team 1 chunk 2p + 1
    const int warp = tid >> 5, lane = tid & 31;
    const int chunks = (a.T + kChunk - 1) / kChunk;
    const int pairs = (chunks + 1) / 2;
    const long long groups = (batch + R - 1) / R;
    const size_t row_bytes = static_cast<size_t>(a.F) * sizeof(XT);
    if (tid == 0) {
        for (int b = 0; b < kBuffers; ++b) mbar_init(&bar[b]);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        if (blockIdx.x < groups) {
            const long long r0 = static_cast<long long>(blockIdx.x) * R;
            prefetch_l2(x + r0 * a.F, static_cast<size_t>(min(static_cast<long long>(R), batch - r0)) * row_bytes);
        }
    }
    __syncthreads();

    // Chunk c of the CTA's k-th row group goes to buffer c % 4 and completes
    // that buffer's barrier for the (k * per_buffer(b) + c / 4)-th time, whose
    // parity is what a wait names. Thread 0 remembers the parity of the last
    // copy it issued to each buffer, so a failing CTA can wait out whatever is
    // still in flight before it exits.
    auto parity_of = [&](unsigned k, int c) -> uint32_t {
        const unsigned b = static_cast<unsigned>(c) & 3u;
        const unsigned per_buffer = (static_cast<unsigned>(chunks) + 3u - b) / 4u;
        return (k * per_buffer + static_cast<unsigned>(c >> 2)) & 1u;
    };
    uint32_t issued_mask = 0, issued_parity = 0;
    unsigned k = 0;  // row groups this CTA has started
    auto issue = [&](int c) {
        const unsigned b = static_cast<unsigned>(c) & 3u;
        bulk_load(ring + b * kChunkBytes, h.trees + static_cast<size_t>(c) * kChunkBytes, kChunkBytes, &bar[b]);
        issued_mask |= 1u << b;
        issued_parity = (issued_parity & ~(1u << b)) | (parity_of(k, c) << b);
    };

    const uint32_t col = smem_u32(keys) + r * 4;  // this row's key column
    for (long long g = blockIdx.x; g < groups; g += gridDim.x, ++k) {
        const long long row0 = g * R;
        const long long row = row0 + r;
        if (tid == 0) {
            for (int c = 0; c < min(chunks, 2); ++c) issue(c);
        }
        // Prepare: warp w builds the keys of rows 32 (w % (R / 32)) .. + 31,
        // team 0 for the first half of the features and team 1 for the rest,
        // with its transpose tile in the ring past buffer 1 (free until the
        // copies of chunks 2 and 3 start below).
        {
            const int wr = warp % (R / 32);
            const int half = (a.F + 1) / 2;
            double* tile = reinterpret_cast<double*>(ring + 2 * kChunkBytes + warp * kTileBytes);
            prepare_group<R, kTile>(a, x, row0 + wr * 32, batch, keys + wr * 32, tile, lane, team ? half : 0,
                                    team ? a.F : half, team == 0);
        }
        __syncthreads();
        if (tid == 0) {
            for (int c = 2; c < min(chunks, 4); ++c) issue(c);
            if (g + gridDim.x < groups) {  // the next group's rows into L2 while this one walks
                const long long r1 = row0 + static_cast<long long>(gridDim.x) * R;
                prefetch_l2(x + r1 * a.F, static_cast<size_t>(min(static_cast<long long>(R), batch - r1)) * row_bytes);
            }
        }
        double acc = a.mean ? 0.0 : __ldg(a.base);
        double part = 0.0;
        bool bad = false;  // this thread's wait timed out; decided CTA-wide at the next barrier

        // Adds the leaves of chunk c (indices in leaf[]) in tree order.
        auto add_chunk = [&](int c, const uint32_t (&leaf)[kChunk]) {
            const uint32_t buf = ring0 + (static_cast<unsigned>(c) & 3u) * kChunkBytes;
            const int live = min(kChunk, a.T - c * kChunk);
            const bool first_block = c * kChunk < kTreeBlock;
            if (!first_block && (c * kChunk) % kTreeBlock == 0) {
                // A block of 64 trees ended with the previous chunk.
                if (c * kChunk >= 2 * kTreeBlock) acc = __dadd_rn(acc, part);
                part = 0.0;
            }
#pragma unroll
            for (int t = 0; t < kChunk; ++t) {
                if (t < live) {
                    const double v = lds_leaf(buf + t * kTreeBytes + kSplits * 8 + leaf[t] * kLeafBytes, LEAF32);
                    if (first_block) acc = __dadd_rn(acc, v);
                    else part = __dadd_rn(part, v);
                }
            }
        };

        for (int pr = 0; pr < pairs; ++pr) {
            if (pr > 0) {
                if (__syncthreads_or(bad)) break;  // pair pr - 1 is done: its buffers take pair pr + 1
                if (tid == 0) {
                    for (int c = 2 * pr + 2; c < min(chunks, 2 * pr + 4); ++c) issue(c);
                }
            }
            const int mine = 2 * pr + team;
            uint32_t leaf[kChunk];
            if (mine < chunks) {
                if (!mbar_wait(&bar[mine & 3], parity_of(k, mine))) {
                    bad = true;
                } else {
                    const uint32_t buf = ring0 + (static_cast<unsigned>(mine) & 3u) * kChunkBytes;
                    walk_chunk<D, TIES>(a, h, buf, col, mine, min(kChunk, a.T - mine * kChunk), x, row, batch, leaf,
                                        kTreeBytes);
                    if (team == 0) {
                        add_chunk(mine, leaf);
                    } else {
#pragma unroll
                        for (int t = 0; t < kChunk; ++t) exchange[t * R + r] = static_cast<unsigned char>(leaf[t]);
                    }
                }
            }
            if (__syncthreads_or(bad)) break;  // team 1's leaves are in the exchange
            if (team == 0 && mine + 1 < chunks) {
#pragma unroll
                for (int t = 0; t < kChunk; ++t) leaf[t] = exchange[t * R + r];
                add_chunk(mine + 1, leaf);
            }
        }
        if (__syncthreads_or(bad)) {
            // Leave no bulk copy in flight into shared memory: wait (bounded)
            // for the last copy issued to each buffer, then stop.
            if (tid == 0) {
                atomicExch(h.status, 1);
                for (int b = 0; b < kBuffers; ++b) {
                    if (issued_mask & (1u << b)) mbar_wait(&bar[b], (issued_parity >> b) & 1u);
                }
            }
            return;
        }
        if (team == 0 && row < batch) {
            if (a.T > kTreeBlock) acc = __dadd_rn(acc, part);
            double v[1] = {acc};
            if (a.mean) {
                const int n = __ldg(a.counts);
                v[0] = __dadd_rn(__ldg(a.base), n ? __ddiv_rn(v[0], static_cast<double>(n)) : 0.0);
            }
            apply_link<1>(a, v, 1);
            out[row] = v[0];
        }
        __syncthreads();  // keys, exchange and buffers are rewritten by the next group
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

}  // namespace

int heap_record_bytes(int depth, bool leaf32) { return heap_tree_bytes(depth, leaf32); }

int heap_chunk_trees() { return kChunk; }

// The most rows per CTA (128, 64, 32) whose key tables and ring fit.
bool heap_plan(int slots, int depth, bool leaf32, int& rows, int& buffers) {
    if (depth < 1 || depth > 8) return false;
    for (int r : {128, 64, 32}) {
        if (layout_of(slots, depth, leaf32, r).total <= kHeapSmemLimit) {
            rows = r;
            buffers = kBuffers;
            return true;
        }
    }
    return false;
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
    const int smem = layout_of(f.args.slots, h.depth, h.leaf32, h.rows).total;
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
    const cudaError_t e = cudaLaunchKernel(k, grid, 2 * h.rows, args, smem, stream);
    if (e != cudaSuccess) {
        err = std::string("complete-tree kernel launch: ") + cudaGetErrorString(e);
        return false;
    }
    return true;
}

}  // namespace mlk::cuda
