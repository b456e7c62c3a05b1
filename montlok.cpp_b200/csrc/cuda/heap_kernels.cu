// Complete-tree predict kernel for sm_100a (depth <= 8, one output).
//
// Tree record. Every tree is stored as a complete binary tree of depth D in
// heap order (children of split i at 2i+1 and 2i+2; shallower leaves are
// padded with always-left splits), one 16-byte aligned record per tree:
// 2^D split words of 4 bytes (the last one unused, so the leaves start 8-byte
// aligned) and 2^D leaf values (float32 when every leaf is exactly a float,
// else float64). A split word packs the threshold key and the slot:
//
//     word = (T & ~mask) | slot          mask = 2^slot_bits - 1
//
// and the row's key table holds k' = (k & ~mask) | slot in every slot's row,
// so a key read for a split has the split word's low bits: a step is one
// signed compare, k' > word, exact whenever k and T differ in their high
// bits, and k' == word is exactly the case where they agree (a float32
// within a relative 2^-(23 - slot_bits) of the threshold: rare). The walk
// notes such a tie for the tree (one predicated compare), and after the
// chunk's walk the tied trees are walked again with every tied split
// decided by the reference's own comparison of the prepared double against
// the file threshold. NaN and zero-band keys (INT32_MAX, INT32_MIN with the
// slot in the low bits) never tie with a threshold.
//
// Work split. A CTA owns R rows for the whole ensemble: their key tables
// ([slot][R] int32, lane l always reading bank l) stay in shared memory. Four
// teams of R threads (one thread per row in each) walk disjoint 64-tree
// blocks: team j takes blocks j, j + 4, j + 8, ... Blocks are what the
// reference sums separately (trees.cpp:366-388: block 0 onto the base score,
// every later block from 0.0, then the blocks in order), so a team adds its
// leaves in tree order into its own block partial and never waits for another
// team inside a block. After each round of four blocks the partials meet in
// shared memory (one CTA barrier) and team 0 adds them to the row's sum in
// block order, which reproduces the reference's float64 association exactly.
//
// Streaming. Each team streams its trees through a private pair of chunk
// buffers (4 trees each, one thread walking the 4 side by side), filled by
// one-dimensional bulk async copies (cp.async.bulk) whose completion counts on
// one mbarrier per buffer. No warp waits for its teammates: a warp done with
// a buffer bumps the buffer's counter in shared memory, and the warp whose
// bump completes the team's count refills the buffer two chunks ahead. The
// device tree array is padded with inert trees to whole chunks, so every copy
// is a full chunk. Waits are bounded: a warp whose wait runs out raises the
// CTA's abort flag, every wait gives up once the flag is up, the CTA leaves
// at the next round barrier after waiting (bounded) for its copies in flight,
// and the call's status word records the error for the host.
#include <algorithm>
#include <cstdint>
#include <mutex>
#include <vector>

#include "async_copy.cuh"
#include "device_common.cuh"
#include "forest.cuh"
#include "tmem.cuh"
#include "cluster.cuh"

namespace mlk::cuda {
namespace {

constexpr int kTeams = 4;                              // teams of R threads, one 64-tree block each at a time
constexpr int kTrees = 4;                              // trees per chunk = trees one thread walks side by side
constexpr int kChunksPerBlock = kTreeBlock / kTrees;   // 16
constexpr int kHeapSmemLimit = 227 * 1024;
constexpr int kMaxSlotBits = 10;
static_assert(kTreeBlock % kTrees == 0, "chunks never straddle a block of 64 trees");

__host__ __device__ constexpr int record_bytes(int depth, bool leaf32) { return heap_record_size(depth, leaf32); }

// Shared memory layout (byte offsets): header (mbarriers [team][2] at 0,
// buffer-done counters [team][2] at 64, fills issued [team][2] at 96, abort
// flag at 128) | keys [slots][R] int32 | block partials [2][team][R] double |
// first buffers of the four teams | second buffers of the four teams.
struct Layout {
    int keys, parts, ring0, ring1, total;
};

// `partials` rows of partial sums: 2 * kTeams (two rounds of four blocks)
// for heap_kernel, one per 64-tree block for the staged kernel.
__host__ __device__ inline Layout layout_of(int slots, int depth, bool leaf32, int rows, int partials = 2 * kTeams) {
    Layout l{};
    l.keys = 256;
    l.parts = l.keys + align128(slots * rows * 4);
    l.ring0 = l.parts + align128(partials * rows * 8);
    const int chunk = kTrees * record_bytes(depth, leaf32);
    l.ring1 = l.ring0 + align128(kTeams * chunk);
    l.total = l.ring1 + align128(kTeams * chunk);
    return l;
}

// One tree walked exactly for one row: the packed compare where the high
// bits differ, the reference's comparison of the prepared double with the
// file threshold (exact_right) where they tie. Returns the heap index of the
// leaf reached. Only trees whose fast walk met a tie come here.
template <int D, int R, typename XT>
__device__ __forceinline__ uint32_t walk_exact(const ForestArgs& a, const HeapArgs& h, uint32_t base, uint32_t col,
                                            uint32_t mask, int tree, const XT* __restrict__ x, long long row,
                                            long long batch) {
    constexpr int kSplits = (1 << D) - 1;
    uint32_t i = 0;
    for (int d = 0; d < D; ++d) {
        const uint32_t n = lds_u32(base + 4 * i);
        const int k = lds_s32(col + (n & mask) * (R * 4));
        bool right = k > static_cast<int>(n);
        if (static_cast<uint32_t>(k ^ static_cast<int>(n)) <= mask && tree < a.T) {
            const int node = __ldg(h.node_ids + static_cast<size_t>(tree) * kSplits + i);
            if (node >= 0) right = exact_right(a, x, row, batch, node);
        }
        i = 2 * i + (right ? 2u : 1u);
    }
    return i;
}

// Walks the kTrees trees of the chunk at shared address `buf` (file trees
// tree0 .. tree0 + kTrees - 1) for one row; v[t] receives tree t's leaf value.
template <int D, int R, bool LEAF32, typename XT>
__device__ __forceinline__ void walk_leaves(const ForestArgs& a, const HeapArgs& h, uint32_t buf, uint32_t col,
                                            uint32_t mask, int tree0, const XT* x, long long row, long long batch,
                                            double (&v)[kTrees]) {
    constexpr int kRec = record_bytes(D, LEAF32);
    uint32_t p[kTrees], go_left[kTrees];
    bool tie[kTrees];
#pragma unroll
    for (int t = 0; t < kTrees; ++t) {
        p[t] = buf + t * kRec;
        go_left[t] = 4u - p[t];  // left child of the split at byte address q: 2q + go_left
        tie[t] = false;
    }
#pragma unroll
    for (int d = 0; d < D; ++d) {
        uint32_t n[kTrees];
        int k[kTrees];
#pragma unroll
        for (int t = 0; t < kTrees; ++t) n[t] = lds_u32(p[t]);
#pragma unroll
        for (int t = 0; t < kTrees; ++t) k[t] = lds_s32(col + (n[t] & mask) * (R * 4));
#pragma unroll
        for (int t = 0; t < kTrees; ++t) {
            tie[t] |= k[t] == static_cast<int>(n[t]);
            p[t] = 2 * p[t] + go_left[t] + (k[t] > static_cast<int>(n[t]) ? 4u : 0u);
        }
    }
    bool any = false;
#pragma unroll
    for (int t = 0; t < kTrees; ++t) any |= tie[t];
    if (__any_sync(0xffffffffu, any)) {
#pragma unroll
        for (int t = 0; t < kTrees; ++t) {
            if (tie[t]) {
                const uint32_t base = buf + t * kRec;
                p[t] = base + 4 * walk_exact<D, R>(a, h, base, col, mask, tree0 + t, x, row, batch);
            }
        }
    }
    // Heap index i >= 2^D - 1 sits at byte base + 4i; its leaf value (leaf
    // i - (2^D - 1) after the 2^D words) at base + 4i + 4 for float32
    // leaves, at 2(base + 4i) - base + 8 - 4 * 2^D for float64 ones.
#pragma unroll
    for (int t = 0; t < kTrees; ++t) {
        v[t] = LEAF32 ? lds_leaf(p[t] + 4u, true) : lds_leaf(2u * p[t] + go_left[t] + (4u - (4u << D)), false);
    }
}

// Walks a chunk and adds the leaves of its first `live` trees, in order, to `part`.
template <int D, int R, bool LEAF32, typename XT>
__device__ __forceinline__ void walk_chunk(const ForestArgs& a, const HeapArgs& h, uint32_t buf, uint32_t col,
                                           uint32_t mask, int chunk, int live, const XT* x, long long row,
                                           long long batch, double& part) {
    double v[kTrees];
    walk_leaves<D, R, LEAF32>(a, h, buf, col, mask, chunk * kTrees, x, row, batch, v);
#pragma unroll
    for (int t = 0; t < kTrees; ++t) {
        if (t < live) part = __dadd_rn(part, v[t]);
    }
}

template <int D, int R, bool LEAF32, typename XT>
__global__ void __launch_bounds__(kTeams * R, 1) heap_kernel(const __grid_constant__ ForestArgs a, const __grid_constant__ HeapArgs h,
                                                          const XT* __restrict__ x, long long batch,
                                                          double* __restrict__ out) {
    constexpr int kChunkBytes = kTrees * record_bytes(D, LEAF32);
    constexpr int kWarpsPerTeam = R / 32;
    extern __shared__ __align__(128) unsigned char smem[];
    const Layout L = layout_of(a.slots, D, LEAF32, R);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem);                // [team][buffer]
    unsigned* done = reinterpret_cast<unsigned*>(smem + 64);         // [team][buffer]: warps done, cumulative
    unsigned* fills = reinterpret_cast<unsigned*>(smem + 96);        // [team][buffer]: copies issued
    volatile int* abort = reinterpret_cast<volatile int*>(smem + 128);
    int* keys = reinterpret_cast<int*>(smem + L.keys);
    double* parts = reinterpret_cast<double*>(smem + L.parts);

    const int tid = threadIdx.x;
    const int team = tid / R, r = tid % R;
    const int warp = tid >> 5, lane = tid & 31;
    const bool producer = r == 0;  // issues the team's first two copies of a row group
    const int chunks = (a.T + kTrees - 1) / kTrees;
    const int blocks = (a.T + kTreeBlock - 1) / kTreeBlock;
    const int rounds = (blocks + kTeams - 1) / kTeams;
    const long long groups = (batch + R - 1) / R;
    const size_t row_bytes = static_cast<size_t>(a.F) * sizeof(XT);
    const uint32_t mask = (1u << h.slot_bits) - 1u;
    // The team's chunks in walking order: blocks team, team + 4, ...; the
    // q-th is chunk_at(q), and n_team of them per row group.
    int n_team = 0;
    for (int b = team; b < blocks; b += kTeams) n_team += min(kChunksPerBlock, chunks - b * kChunksPerBlock);
    auto chunk_at = [&](int q) {
        return (team + kTeams * (q / kChunksPerBlock)) * kChunksPerBlock + q % kChunksPerBlock;
    };
    const uint32_t buf0 = smem_u32(smem + L.ring0) + team * kChunkBytes;
    const uint32_t buf1 = smem_u32(smem + L.ring1) + team * kChunkBytes;
    uint64_t* team_bar = bar + 2 * team;

    if (tid == 0) {
        for (int b = 0; b < 2 * kTeams; ++b) {
            mbar_init(&bar[b]);
            done[b] = 0u;
            fills[b] = 0u;
        }
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        if (blockIdx.x < groups) {
            const long long r0 = static_cast<long long>(blockIdx.x) * R;
            prefetch_l2(x + r0 * a.F, static_cast<size_t>(min(static_cast<long long>(R), batch - r0)) * row_bytes);
        }
    }
    __syncthreads();

    // Buffer b's k-th fill completes its barrier's phase k: every thread of
    // the team keeps the parity of the next fill it waits for; `fills`
    // counts those issued (to wait out copies in flight before an early exit).
    uint32_t phase = 0u;  // bit b: parity of the next fill of buffer b (a register, not an indexed array)
    auto issue = [&](int q) {
        if (a.skip_copies) return;  // fault injection: the wait for this chunk runs out
        const int b = q & 1;
        bulk_load(b ? buf1 : buf0, h.trees + static_cast<size_t>(chunk_at(q)) * kChunkBytes, kChunkBytes,
                  &team_bar[b]);
        atomicAdd(&fills[2 * team + b], 1u);
    };
    if (producer && blockIdx.x < groups) {
        if (n_team > 0) issue(0);
        if (n_team > 1) issue(1);
    }

    const uint32_t col = smem_u32(keys) + r * 4;  // this row's key column
    for (long long g = blockIdx.x; g < groups; g += gridDim.x) {
        const long long row0 = g * R;
        const long long row = row0 + r;
        {
            // Prepare: thread (team, r) builds the keys of row r for the team's
            // quarter of the features (even-sized, so vector loads stay aligned).
            const int per = ((a.F + kTeams - 1) / kTeams + 7) & ~7;
            const int f_begin = min(a.F, team * per), f_end = min(a.F, f_begin + per);
            prepare_own_row<R>(a, x, row, batch, keys + r, f_begin, f_end, static_cast<int>(mask));
            if (team == 0) keys[a.pad_slot * R + r] = INT_MIN;
        }
        __syncthreads();
        if (tid == 0 && g + gridDim.x < groups) {  // the next group's rows into L2 while this one walks
            const long long r1 = row0 + static_cast<long long>(gridDim.x) * R;
            prefetch_l2(x + r1 * a.F, static_cast<size_t>(min(static_cast<long long>(R), batch - r1)) * row_bytes);
        }

        double acc = 0.0;  // team 0: the row's sum over the rounds done
        bool bad = false;  // the CTA is aborting (uniform after each round barrier)
        int q = 0;         // position in the team's chunk list
        for (int k = 0; k < rounds; ++k) {
            const int block = team + kTeams * k;
            if (block < blocks) {
                const int c0 = block * kChunksPerBlock;
                const int cn = min(kChunksPerBlock, chunks - c0);
                double part = (block == 0 && !a.mean) ? __ldg(a.base) : 0.0;
                for (int c = 0; c < cn; ++c, ++q) {
                    const int b = q & 1;
                    // Warp-uniform: the walk's votes need every lane. Once the
                    // CTA is aborting no wait is trusted: a warp whose own wait
                    // ran out has lost count of the barrier's phases, and a
                    // wait on the other parity would return at once.
                    const bool ok = __all_sync(0xffffffffu, !*abort && mbar_wait(&team_bar[b], (phase >> b) & 1u,
                                                                                 a.wait_ns, abort));
                    phase ^= 1u << b;
                    if (ok) {
                        walk_chunk<D, R, LEAF32>(a, h, b ? buf1 : buf0, col, mask, c0 + c,
                                                 min(kTrees, a.T - (c0 + c) * kTrees), x, row, batch, part);
                    } else if (lane == 0) {
                        *abort = 1;
                    }
                    __syncwarp();
                    if (lane == 0) {
                        // This warp's reads of buffer b are done; the team's
                        // last warp to get here refills it.
                        __threadfence_block();
                        const unsigned before = atomicAdd(&done[2 * team + b], 1u);
                        if (before % kWarpsPerTeam == kWarpsPerTeam - 1 && q + 2 < n_team && !*abort) {
                            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                            issue(q + 2);
                        }
                    }
                }
                parts[((k & 1) * kTeams + team) * R + r] = part;
            }
            if (__syncthreads_or(*abort)) {
                bad = true;
                break;
            }
            if (team == 0) {
#pragma unroll
                for (int j = 0; j < kTeams; ++j) {
                    const int blk = kTeams * k + j;
                    if (blk < blocks) {
                        const double v = parts[((k & 1) * kTeams + j) * R + r];
                        acc = blk == 0 ? v : __dadd_rn(acc, v);
                    }
                }
            }
        }
        if (bad) {
            // Leave no bulk copy in flight into shared memory: wait (bounded)
            // for the last copy issued to each buffer, then stop.
            if (producer) {
                if (team == 0) atomicExch(a.status, 1);
                for (int b = 0; b < 2; ++b) {
                    const unsigned n = fills[2 * team + b];
                    if (n > 0) mbar_wait(&team_bar[b], (n - 1u) & 1u, a.wait_ns);
                }
            }
            return;
        }
        if (team == 0 && row < batch) {
            double v[1] = {acc};
            if (a.mean) {
                const int n = __ldg(a.counts);
                v[0] = __dadd_rn(__ldg(a.base), n ? __ddiv_rn(v[0], static_cast<double>(n)) : 0.0);
            }
            apply_link<1>(a, v, 1);
            out[row] = v[0];
        }
        // Every team passed the last round's barrier, so both buffers are
        // free: start the next group's first two chunks.
        if (producer && g + gridDim.x < groups) {
            if (n_team > 0) issue(0);
            if (n_team > 1) issue(1);
        }
        __syncthreads();  // keys and partials are rewritten by the next group
    }
}

// ---------------------------------------------------------------------------
// Staged complete-tree kernel: heap_kernel's walk with the prepare taken off
// the walkers' path. Beside the four teams of 128 walker threads (warps
// 0..15) run four producer warps (16..19), one thread per row of the group:
// while the walkers walk row group g, the producers read the rows of the
// CTA's next group and write their keys into tensor memory, lane = row of
// the group, column = slot (the pad slot, always INT_MIN, is not staged).
// At the start of a group every walker copies its own row's keys for a
// quarter of the slots from its TMEM lane (a warp's rows are exactly the 32
// lanes its quarter of TMEM holds) into the shared key table. Two mbarriers
// hand the stage over: `full` (one arrival per producer warp: the group's
// keys are in TMEM) and `empty` (one per walker warp: copied out, the stage
// may be overwritten). Each is waited on with the time bound and abort flag
// of the chunk waits. Every 64-tree block's partial sums have their own row
// of shared memory, so the walkers meet once per group (a named barrier of
// the 512 walkers; the producers never take part), after which team 0 adds
// the blocks in order. The CTA allocates the
// stage's TMEM columns once and frees them on every way out, after a last
// barrier of all 640 threads. Only for 128 rows per CTA and models whose pad
// slot is at most 512 (the stage fits 512 columns); one CTA per SM (its
// registers), launched one per SM.
// ---------------------------------------------------------------------------
constexpr int kStageRows = 128;
constexpr int kWalkers = kTeams * kStageRows;  // 512
constexpr int kProducerWarps = 4;              // one per quarter of TMEM's 128 lanes
constexpr int kStagedThreads = kWalkers + 32 * kProducerWarps;
constexpr int kMaxStageCols = 512;

// The walkers' barrier (named barrier 1, the 512 walker threads only);
// returns whether any walker passed a nonzero `v`.
__device__ __forceinline__ bool walkers_sync_or(int v) {
    int any;
    asm volatile(
        "{ .reg .pred p, q; setp.ne.s32 q, %1, 0; bar.red.or.pred p, 1, %2, q; selp.s32 %0, 1, 0, p; }"
        : "=r"(any)
        : "r"(v), "n"(kWalkers)
        : "memory");
    return any != 0;
}
__device__ __forceinline__ void walkers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kWalkers) : "memory"); }

// Rows of partial sums the staged kernel keeps: one per 64-tree block.
__host__ __device__ inline int stage_partials(int trees) {
    return max(2 * kTeams, (trees + kTreeBlock - 1) / kTreeBlock);
}

// TMEM columns a model's stage takes: the smallest power of two, at least
// 32, holding slots 0 .. pad_slot - 1; 0 when it needs more than 512.
__host__ __device__ inline int stage_cols(int pad_slot) {
    int c = 32;
    while (c < pad_slot) c *= 2;
    return c <= kMaxStageCols ? c : 0;
}

template <int D, bool LEAF32, typename XT>
__global__ void __launch_bounds__(kStagedThreads, 1) heap_staged_kernel(const __grid_constant__ ForestArgs a, const __grid_constant__ HeapArgs h,
                                                                        const XT* __restrict__ x, long long batch,
                                                                        double* __restrict__ out, int cols) {
    constexpr int R = kStageRows;
    constexpr int kChunkBytes = kTrees * record_bytes(D, LEAF32);
    constexpr int kWarpsPerTeam = R / 32;
    extern __shared__ __align__(128) unsigned char smem[];
    const Layout L = layout_of(a.slots, D, LEAF32, R, stage_partials(a.T));
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem);                // [team][buffer]
    unsigned* done = reinterpret_cast<unsigned*>(smem + 64);         // [team][buffer]: warps done, cumulative
    unsigned* fills = reinterpret_cast<unsigned*>(smem + 96);        // [team][buffer]: copies issued
    volatile int* abort = reinterpret_cast<volatile int*>(smem + 128);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + 136);        // stage written (producer warps)
    uint64_t* empty = reinterpret_cast<uint64_t*>(smem + 144);       // stage copied out (walker warps)
    uint32_t* stage_addr = reinterpret_cast<uint32_t*>(smem + 152);  // TMEM address of the stage
    int* keys = reinterpret_cast<int*>(smem + L.keys);
    double* parts = reinterpret_cast<double*>(smem + L.parts);

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const long long groups = (batch + R - 1) / R;
    const size_t row_bytes = static_cast<size_t>(a.F) * sizeof(XT);
    const uint32_t mask = (1u << h.slot_bits) - 1u;
    const int staged = a.pad_slot;  // slots 0 .. staged - 1 go through TMEM

    if (tid == 0) {
        for (int b = 0; b < 2 * kTeams; ++b) {
            mbar_init(&bar[b]);
            done[b] = 0u;
            fills[b] = 0u;
        }
        mbar_init(full, kProducerWarps);
        mbar_init(empty, kWalkers / 32);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        if (blockIdx.x < groups) {
            const long long r0 = static_cast<long long>(blockIdx.x) * R;
            prefetch_l2(x + r0 * a.F, static_cast<size_t>(min(static_cast<long long>(R), batch - r0)) * row_bytes);
        }
    }
    if (warp == kWalkers / 32) tmem_alloc(stage_addr, static_cast<uint32_t>(cols));
    tmem_fence_before_sync();
    __syncthreads();
    tmem_fence_after_sync();
    const uint32_t stage = *stage_addr;

    if (tid >= kWalkers) {
        // Producer: row p of every group this CTA takes, into TMEM lane p.
        const int p = tid - kWalkers;
        const uint32_t lane_base = stage + (static_cast<uint32_t>(p & ~31) << 16);
        int it = 0;
        for (long long g = blockIdx.x; g < groups; g += gridDim.x, ++it) {
            if (it > 0) {
                // The walkers have copied the previous group out of the stage.
                const bool ok = __all_sync(0xffffffffu, !*abort && mbar_wait(empty, (it - 1) & 1, a.wait_ns, abort));
                if (!ok) {
                    if (lane == 0) *abort = 1;
                    break;
                }
                tmem_fence_after_sync();
            }
            prepare_row_with(a, x, g * R + p, batch, 0, a.F, [&](int f, int k, bool nan, bool zero) {
                const int4 s = __ldg(a.slot_of + f);
                auto tag = [mask](int key, int slot) { return (key & ~static_cast<int>(mask)) | (slot & static_cast<int>(mask)); };
                if (s.x >= 0) tmem_st1(lane_base + s.x, tag(nan ? INT_MAX : k, s.x));
                if (s.y >= 0) tmem_st1(lane_base + s.y, tag(nan ? INT_MIN : k, s.y));
                if (s.z >= 0) tmem_st1(lane_base + s.z, tag(zero ? INT_MAX : k, s.z));
                if (s.w >= 0) tmem_st1(lane_base + s.w, tag(zero ? INT_MIN : k, s.w));
            });
            tmem_wait_st();
            tmem_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(full);
            if (p == 0 && g + gridDim.x < groups) {  // the rows of the next group this CTA prepares, into L2
                const long long r1 = (g + gridDim.x) * R;
                prefetch_l2(x + r1 * a.F, static_cast<size_t>(min(static_cast<long long>(R), batch - r1)) * row_bytes);
            }
        }
    } else {
        const int team = tid / R, r = tid % R;
        const bool issuer = r == 0;  // issues the team's first two copies of a row group
        const int chunks = (a.T + kTrees - 1) / kTrees;
        const int blocks = (a.T + kTreeBlock - 1) / kTreeBlock;
        int n_team = 0;
        for (int b = team; b < blocks; b += kTeams) n_team += min(kChunksPerBlock, chunks - b * kChunksPerBlock);
        auto chunk_at = [&](int q) {
            return (team + kTeams * (q / kChunksPerBlock)) * kChunksPerBlock + q % kChunksPerBlock;
        };
        const uint32_t buf0 = smem_u32(smem + L.ring0) + team * kChunkBytes;
        const uint32_t buf1 = smem_u32(smem + L.ring1) + team * kChunkBytes;
        uint64_t* team_bar = bar + 2 * team;
        const uint32_t lane_base = stage + (static_cast<uint32_t>(r & ~31) << 16);

        uint32_t phase = 0u;  // bit b: parity of the next fill of buffer b (a register, not an indexed array)
        auto issue = [&](int q) {
            if (a.skip_copies) return;  // fault injection: the wait for this chunk runs out
            const int b = q & 1;
            bulk_load(b ? buf1 : buf0, h.trees + static_cast<size_t>(chunk_at(q)) * kChunkBytes, kChunkBytes,
                      &team_bar[b]);
            atomicAdd(&fills[2 * team + b], 1u);
        };
        if (issuer && blockIdx.x < groups) {
            if (n_team > 0) issue(0);
            if (n_team > 1) issue(1);
        }

        const uint32_t col = smem_u32(keys) + r * 4;  // this row's key column
        bool bad = false;                              // the CTA is aborting (uniform after each walkers' barrier)
        int it = 0;
        for (long long g = blockIdx.x; g < groups; g += gridDim.x, ++it) {
            const long long row = g * R + r;
            {
                // Keys of this group: this row's staged slots c, c + 1, ...
                // (16 at a time, the team's quarter) from TMEM into the table.
                const bool ok = __all_sync(0xffffffffu, !*abort && mbar_wait(full, it & 1, a.wait_ns, abort));
                if (ok) {
                    tmem_fence_after_sync();
                    for (int c = 16 * team; c < staged; c += 16 * kTeams) {
                        int v[16];
                        tmem_ld16(lane_base + static_cast<uint32_t>(c), v);
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            if (c + j < staged) keys[(c + j) * R + r] = v[j];
                        }
                    }
                    if (team == 0) keys[a.pad_slot * R + r] = INT_MIN;
                    tmem_fence_before_sync();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(empty);
                } else if (lane == 0) {
                    *abort = 1;
                }
            }
            if (walkers_sync_or(*abort)) {
                bad = true;
                break;
            }

            // Every block's partial has its own row of `parts`: the teams
            // meet once per group, after all their blocks.
            int q = 0;  // position in the team's chunk list
            for (int block = team; block < blocks; block += kTeams) {
                const int c0 = block * kChunksPerBlock;
                const int cn = min(kChunksPerBlock, chunks - c0);
                double part = (block == 0 && !a.mean) ? __ldg(a.base) : 0.0;
                for (int c = 0; c < cn; ++c, ++q) {
                    const int b = q & 1;
                    const bool ok = __all_sync(0xffffffffu, !*abort && mbar_wait(&team_bar[b], (phase >> b) & 1u,
                                                                                 a.wait_ns, abort));
                    phase ^= 1u << b;
                    if (ok) {
                        walk_chunk<D, R, LEAF32>(a, h, b ? buf1 : buf0, col, mask, c0 + c,
                                                 min(kTrees, a.T - (c0 + c) * kTrees), x, row, batch, part);
                    } else if (lane == 0) {
                        *abort = 1;
                    }
                    __syncwarp();
                    if (lane == 0) {
                        __threadfence_block();
                        const unsigned before = atomicAdd(&done[2 * team + b], 1u);
                        if (before % kWarpsPerTeam == kWarpsPerTeam - 1 && q + 2 < n_team && !*abort) {
                            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                            issue(q + 2);
                        }
                    }
                }
                parts[block * R + r] = part;
            }
            if (walkers_sync_or(*abort)) {
                bad = true;
                break;
            }
            if (team == 0 && row < batch) {
                double acc = parts[r];  // blocks in order: the reference's association
                for (int blk = 1; blk < blocks; ++blk) acc = __dadd_rn(acc, parts[blk * R + r]);
                double v[1] = {acc};
                if (a.mean) {
                    const int n = __ldg(a.counts);
                    v[0] = __dadd_rn(__ldg(a.base), n ? __ddiv_rn(v[0], static_cast<double>(n)) : 0.0);
                }
                apply_link<1>(a, v, 1);
                out[row] = v[0];
            }
            if (issuer && g + gridDim.x < groups) {
                if (n_team > 0) issue(0);
                if (n_team > 1) issue(1);
            }
            walkers_sync();  // keys and partials are rewritten by the next group
        }
        if (bad && issuer) {
            // Leave no bulk copy in flight into shared memory: wait (bounded)
            // for the last copy issued to each buffer.
            if (team == 0) atomicExch(a.status, 1);
            for (int b = 0; b < 2; ++b) {
                const unsigned n = fills[2 * team + b];
                if (n > 0) mbar_wait(&team_bar[b], (n - 1u) & 1u, a.wait_ns);
            }
        }
    }
    // Every TMEM access of the CTA is done: free the stage.
    tmem_fence_before_sync();
    __syncthreads();
    if (warp == kWalkers / 32) {
        tmem_fence_after_sync();
        tmem_dealloc(stage, static_cast<uint32_t>(cols));
    }
}

// ---------------------------------------------------------------------------
// Tree-parallel kernel for small batches (at most kLatencyRows rows), where
// the row-streaming kernel would give one CTA the whole ensemble. CTA
// (b, g) takes the 64-tree block b for the (at most) 8 rows of group g, so a
// one-row call of 1000 trees runs 16 CTAs and a 64-row call 128. It builds
// the group's key tables in shared memory (every load of a round in flight
// at once), then each thread walks one tree of the block for two rows
// (lane = tree), reading the split words straight from the L2-resident tree
// records: a small call pays no copy of the trees into shared memory, only
// the dependent loads of its walks, two chains per thread. Leaf values meet
// in shared memory, where one thread per row adds the block's 64 leaves in
// tree order (block 0 onto the base score) into `bpart`
// ([block][kLatencyRows]). The last CTA of the row group to finish (a
// device-scope counter, no waiting) adds the block sums in block order and
// applies the link: the reference's association (trees.cpp:303-388).
// `count` ([row groups]) starts at zero and that last CTA sets it back to
// zero.
// ---------------------------------------------------------------------------
constexpr int kLatencyRows = 64;
constexpr int kGroupRows = 8;                              // rows per CTA
constexpr int kLatencyThreads = 256;                       // 64 trees x 4 row pairs
constexpr int kRowPairs = kLatencyThreads / kTreeBlock;    // 4: thread walks rows p and p + 4
constexpr int kSumBatch = 16;                              // final sum: global loads in flight per thread
static_assert(kGroupRows == 2 * kRowPairs, "each thread walks two rows");
static_assert(kLatencyRows / kGroupRows <= kLatencyCounters, "one counter per row group");

__host__ __device__ inline int latency_smem(int slots, int depth, bool leaf32) {
    return 128 + align128(slots * kGroupRows * 4) + kTreeBlock * kGroupRows * 8;
}

// One split word of tree record `rec` (global memory, read through L1).
__device__ __forceinline__ uint32_t split_word(const unsigned char* rec, uint32_t i) {
    return __ldg(reinterpret_cast<const uint32_t*>(rec) + i);
}

// Heap index of the leaf tree `tree` (record `rec`) reaches for the row whose
// key column is `col` ([slot][kGroupRows]); ties of the packed compare are
// decided on the double (exact_right), as in walk_exact.
template <int D, typename XT>
__device__ __forceinline__ uint32_t walk_global(const ForestArgs& a, const HeapArgs& h, const unsigned char* rec,
                                                const int* col, uint32_t mask, int tree, const XT* x, long long row,
                                                long long batch, bool exact) {
    constexpr int kSplits = (1 << D) - 1;
    uint32_t i = 0;
#pragma unroll
    for (int d = 0; d < D; ++d) {
        const uint32_t n = split_word(rec, i);
        const int k = col[(n & mask) * kGroupRows];
        bool right = k > static_cast<int>(n);
        if (exact && k == static_cast<int>(n)) {
            const int node = __ldg(h.node_ids + static_cast<size_t>(tree) * kSplits + i);
            if (node >= 0) right = exact_right(a, x, row, batch, node);
        }
        i = 2 * i + (right ? 2u : 1u);
    }
    return i;
}

template <int D, bool LEAF32, typename XT>
__global__ void __launch_bounds__(kLatencyThreads) latency_kernel(const __grid_constant__ ForestArgs a, const __grid_constant__ HeapArgs h,
                                                                  const XT* __restrict__ x, long long batch,
                                                                  double* __restrict__ out, double* bpart, int* count) {
    constexpr int kRec = record_bytes(D, LEAF32);
    constexpr int kSplits = (1 << D) - 1;
    constexpr int kPerThread = 8;  // values one thread loads per round of the prepare
    extern __shared__ __align__(128) unsigned char smem[];
    int* flag = reinterpret_cast<int*>(smem);
    int* keys = reinterpret_cast<int*>(smem + 128);  // [slot][kGroupRows]
    double* leafv = reinterpret_cast<double*>(smem + 128 + align128(a.slots * kGroupRows * 4));  // [tree][row]

    const int tid = threadIdx.x;
    const int blocks = (a.T + kTreeBlock - 1) / kTreeBlock;
    const int block = blockIdx.x % blocks, group = blockIdx.x / blocks;
    const long long row0 = static_cast<long long>(kGroupRows) * group;
    const int rows = static_cast<int>(min(static_cast<long long>(kGroupRows), batch - row0));
    const int t0 = block * kTreeBlock;
    const int nt = min(kTreeBlock, a.T - t0);
    const uint32_t mask = (1u << h.slot_bits) - 1u;

    // Keys of the group's rows: value i is (row row0 + i / F, feature i % F);
    // rows past the batch keep whatever the table holds (their walks read
    // in-bounds shared memory; their leaves are never added).
    const int values = rows * a.F;
    for (int i0 = tid; i0 < values; i0 += kPerThread * kLatencyThreads) {
        double v[kPerThread], mean[kPerThread], scale[kPerThread];
        int4 slot[kPerThread];
#pragma unroll
        for (int j = 0; j < kPerThread; ++j) {
            const int i = i0 + j * kLatencyThreads;
            const int f = i % a.F;
            const bool live = i < values;
            v[j] = live ? load_x(x + (row0 + i / a.F) * a.F + f) : 0.0;
            slot[j] = live ? __ldg(a.slot_of + f) : make_int4(-1, -1, -1, -1);
            mean[j] = (live && a.standardize) ? __ldg(a.pre_mean + f) : 0.0;
            scale[j] = (live && a.standardize) ? __ldg(a.pre_scale + f) : 1.0;
        }
#pragma unroll
        for (int j = 0; j < kPerThread; ++j) {
            const int i = i0 + j * kLatencyThreads;
            if (i < values) {
                put_keys<kGroupRows>(a, keys + i / a.F, slot[j], finish(a, v[j], mean[j], scale[j]),
                                     static_cast<int>(mask));
            }
        }
    }
    if (tid < kGroupRows) keys[a.pad_slot * kGroupRows + tid] = INT_MIN;
    __syncthreads();

    // Walks: thread (pair, lane) takes tree t0 + tid % 64 for rows pair and
    // pair + 4 of the group, two independent chains of dependent loads.
    const int local = tid % kTreeBlock, pair = tid / kTreeBlock;
    const int tree = t0 + local;
    if (local < nt && pair < rows) {
        const unsigned char* rec = h.trees + static_cast<size_t>(tree) * kRec;
        const int ra = pair, rb = pair + kRowPairs;
        const bool two = rb < rows;
        const int* ca = keys + ra;
        const int* cb = keys + rb;
        uint32_t ia = 0, ib = 0;
        bool tie = false;
#pragma unroll
        for (int d = 0; d < D; ++d) {
            const uint32_t na = split_word(rec, ia);
            const uint32_t nb = split_word(rec, ib);
            const int ka = ca[(na & mask) * kGroupRows];
            const int kb = cb[(nb & mask) * kGroupRows];
            tie |= ka == static_cast<int>(na) || (two && kb == static_cast<int>(nb));
            ia = 2 * ia + (ka > static_cast<int>(na) ? 2u : 1u);
            ib = 2 * ib + (kb > static_cast<int>(nb) ? 2u : 1u);
        }
        if (tie) {
            ia = walk_global<D>(a, h, rec, ca, mask, tree, x, row0 + ra, batch, true);
            if (two) ib = walk_global<D>(a, h, rec, cb, mask, tree, x, row0 + rb, batch, true);
        }
        auto leaf = [&](uint32_t i) {
            const unsigned char* at = rec + (4 << D);
            const uint32_t l = i - kSplits;
            return LEAF32 ? static_cast<double>(__ldg(reinterpret_cast<const float*>(at) + l))
                          : __ldg(reinterpret_cast<const double*>(at) + l);
        };
        leafv[local * kGroupRows + ra] = leaf(ia);
        if (two) leafv[local * kGroupRows + rb] = leaf(ib);
    }
    __syncthreads();
    if (tid < rows) {
        double acc = (block == 0 && !a.mean) ? __ldg(a.base) : 0.0;
        for (int j0 = 0; j0 < nt; j0 += 8) {
            double v[8];  // the loads together, the adds in order
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = j0 + j < nt ? leafv[(j0 + j) * kGroupRows + tid] : 0.0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (j0 + j < nt) acc = __dadd_rn(acc, v[j]);
            }
        }
        __stcg(bpart + static_cast<size_t>(block) * kLatencyRows + row0 + tid, acc);
        __threadfence();
    }
    __syncthreads();
    if (tid == 0) {
        *flag = atomicAdd(&count[group], 1) == blocks - 1;
        if (*flag) count[group] = 0;  // every CTA of the group has counted: ready for the next launch
    }
    __syncthreads();
    if (!*flag || tid >= rows) return;
    // Last CTA of the row group: the block sums in order, then mean and link.
    const long long row = row0 + tid;
    double v[1] = {__ldcg(bpart + row)};
    for (int b0 = 1; b0 < blocks; b0 += kSumBatch) {
        double p[kSumBatch];
#pragma unroll
        for (int j = 0; j < kSumBatch; ++j) {
            p[j] = b0 + j < blocks ? __ldcg(bpart + static_cast<size_t>(b0 + j) * kLatencyRows + row) : 0.0;
        }
#pragma unroll
        for (int j = 0; j < kSumBatch; ++j) {
            if (b0 + j < blocks) v[0] = __dadd_rn(v[0], p[j]);
        }
    }
    if (a.mean) {
        const int n = __ldg(a.counts);
        v[0] = __dadd_rn(__ldg(a.base), n ? __ddiv_rn(v[0], static_cast<double>(n)) : 0.0);
    }
    apply_link<1>(a, v, 1);
    out[row] = v[0];
}


// ---------------------------------------------------------------------------
// Cluster form of the small-batch kernel, for forests of at most
// kClusterBlocks 64-tree blocks: the CTAs of one row group (one per block)
// form a thread-block cluster. CTA 0 of the cluster reads the group's rows
// once (uncached: in the host-call path they are read straight from the
// pinned staging buffer, so the call's graph has no copy node) and pushes
// them into every CTA's shared memory; after a cluster barrier each CTA
// builds the keys, walks its 64 trees as latency_kernel does and pushes its
// block sum into CTA 0's shared memory; after a second barrier CTA 0 adds the
// block sums in block order, applies the link and stores the rows' results.
// No device scratch, counter or fence. Requests whose copies would total more
// than kClusterPush values let every CTA read the rows itself instead.
// ---------------------------------------------------------------------------
constexpr int kClusterBlocks = 16;
constexpr int kClusterPush = 6144;

__device__ __forceinline__ double load_uncached(const double* p) {
    double v;
    asm volatile("ld.global.cv.f64 %0, [%1];" : "=d"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ double load_uncached(const float* p) {
    float v;
    asm volatile("ld.global.cv.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
    return static_cast<double>(v);
}

// Shared memory: pad | keys [slot][row] | leaf values [tree][row] | rows
// [row][F] (doubles) | block sums [block][row] (used in CTA 0).
__host__ __device__ inline int latency_cluster_smem(int slots, int F) {
    return 128 + align128(slots * kGroupRows * 4) + kTreeBlock * kGroupRows * 8 + align128(kGroupRows * F * 8) +
           kClusterBlocks * kGroupRows * 8;
}

template <int D, bool LEAF32, typename XT>
__global__ void __launch_bounds__(kLatencyThreads) latency_cluster_kernel(const __grid_constant__ ForestArgs a,
                                                                          const __grid_constant__ HeapArgs h,
                                                                          const XT* __restrict__ x, long long batch,
                                                                          double* __restrict__ out) {
    constexpr int kRec = record_bytes(D, LEAF32);
    constexpr int kSplits = (1 << D) - 1;
    extern __shared__ __align__(128) unsigned char smem[];
    int* keys = reinterpret_cast<int*>(smem + 128);  // [slot][kGroupRows]
    double* leafv = reinterpret_cast<double*>(smem + 128 + align128(a.slots * kGroupRows * 4));  // [tree][row]
    double* xs = leafv + kTreeBlock * kGroupRows;                                                 // [row][F]
    double* bsum = reinterpret_cast<double*>(reinterpret_cast<unsigned char*>(xs) + align128(kGroupRows * a.F * 8));

    const int tid = threadIdx.x;
    const int blocks = (a.T + kTreeBlock - 1) / kTreeBlock;  // the cluster's size
    const int block = blockIdx.x % blocks, group = blockIdx.x / blocks;
    const long long row0 = static_cast<long long>(kGroupRows) * group;
    const int rows = static_cast<int>(min(static_cast<long long>(kGroupRows), batch - row0));
    const int t0 = block * kTreeBlock;
    const int nt = min(kTreeBlock, a.T - t0);
    const uint32_t mask = (1u << h.slot_bits) - 1u;
    const int values = rows * a.F;
    const XT* xr = x + row0 * a.F;

    if (values * (blocks - 1) <= kClusterPush) {
        if (block == 0) {
            for (int i = tid; i < values; i += kLatencyThreads) {
                const double v = load_uncached(xr + i);
                xs[i] = v;
                const uint32_t at = smem_u32(xs + i);
                for (int j = 1; j < blocks; ++j) st_cluster_f64(cluster_map(at, j), v);
            }
        }
    } else {
        for (int i = tid; i < values; i += kLatencyThreads) xs[i] = load_x(xr + i);
    }
    cluster_sync();  // the rows are in every CTA

    for (int i = tid; i < values; i += kLatencyThreads) {
        const int f = i % a.F;
        const double mean = a.standardize ? __ldg(a.pre_mean + f) : 0.0;
        const double scale = a.standardize ? __ldg(a.pre_scale + f) : 1.0;
        put_keys<kGroupRows>(a, keys + i / a.F, __ldg(a.slot_of + f), finish(a, xs[i], mean, scale),
                             static_cast<int>(mask));
    }
    if (tid < kGroupRows) keys[a.pad_slot * kGroupRows + tid] = INT_MIN;
    __syncthreads();

    // Walks: thread (pair, lane) takes tree t0 + tid % 64 for rows pair and
    // pair + 4 of the group, reading the L2-resident records.
    const int local = tid % kTreeBlock, pair = tid / kTreeBlock;
    const int tree = t0 + local;
    if (local < nt && pair < rows) {
        const unsigned char* rec = h.trees + static_cast<size_t>(tree) * kRec;
        const int ra = pair, rb = pair + kRowPairs;
        const bool two = rb < rows;
        const int* ca = keys + ra;
        const int* cb = keys + rb;
        uint32_t ia = 0, ib = 0;
        bool tie = false;
#pragma unroll
        for (int d = 0; d < D; ++d) {
            const uint32_t na = split_word(rec, ia);
            const uint32_t nb = split_word(rec, ib);
            const int ka = ca[(na & mask) * kGroupRows];
            const int kb = cb[(nb & mask) * kGroupRows];
            tie |= ka == static_cast<int>(na) || (two && kb == static_cast<int>(nb));
            ia = 2 * ia + (ka > static_cast<int>(na) ? 2u : 1u);
            ib = 2 * ib + (kb > static_cast<int>(nb) ? 2u : 1u);
        }
        if (tie) {
            ia = walk_global<D>(a, h, rec, ca, mask, tree, x, row0 + ra, batch, true);
            if (two) ib = walk_global<D>(a, h, rec, cb, mask, tree, x, row0 + rb, batch, true);
        }
        auto leaf = [&](uint32_t i) {
            const unsigned char* at = rec + (4 << D);
            const uint32_t l = i - kSplits;
            return LEAF32 ? static_cast<double>(__ldg(reinterpret_cast<const float*>(at) + l))
                          : __ldg(reinterpret_cast<const double*>(at) + l);
        };
        leafv[local * kGroupRows + ra] = leaf(ia);
        if (two) leafv[local * kGroupRows + rb] = leaf(ib);
    }
    __syncthreads();
    if (tid < rows) {
        double acc = (block == 0 && !a.mean) ? __ldg(a.base) : 0.0;
        for (int j0 = 0; j0 < nt; j0 += 8) {
            double v[8];  // the loads together, the adds in order
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = j0 + j < nt ? leafv[(j0 + j) * kGroupRows + tid] : 0.0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (j0 + j < nt) acc = __dadd_rn(acc, v[j]);
            }
        }
        st_cluster_f64(cluster_map(smem_u32(bsum + block * kGroupRows + tid), 0), acc);
    }
    cluster_sync();  // every block sum is in CTA 0
    if (block != 0 || tid >= rows) return;
    double v[1] = {bsum[tid]};
    for (int b = 1; b < blocks; ++b) v[0] = __dadd_rn(v[0], bsum[b * kGroupRows + tid]);
    if (a.mean) {
        const int n = __ldg(a.counts);
        v[0] = __dadd_rn(__ldg(a.base), n ? __ddiv_rn(v[0], static_cast<double>(n)) : 0.0);
    }
    apply_link<1>(a, v, 1);
    out[row0 + tid] = v[0];
}

template <int D, bool LEAF32, typename XT>
void* latency_of() {
    return reinterpret_cast<void*>(&latency_kernel<D, LEAF32, XT>);
}

template <int D>
void* pick_latency_leaf(bool leaf32, bool f64) {
    if (leaf32) return f64 ? latency_of<D, true, double>() : latency_of<D, true, float>();
    return f64 ? latency_of<D, false, double>() : latency_of<D, false, float>();
}

template <int D>
void* pick_latency_cluster_leaf(bool leaf32, bool f64) {
    if (leaf32) {
        return f64 ? reinterpret_cast<void*>(&latency_cluster_kernel<D, true, double>)
                   : reinterpret_cast<void*>(&latency_cluster_kernel<D, true, float>);
    }
    return f64 ? reinterpret_cast<void*>(&latency_cluster_kernel<D, false, double>)
               : reinterpret_cast<void*>(&latency_cluster_kernel<D, false, float>);
}

void* pick_latency_cluster(int depth, bool leaf32, bool f64) {
    switch (depth) {
        case 1: return pick_latency_cluster_leaf<1>(leaf32, f64);
        case 2: return pick_latency_cluster_leaf<2>(leaf32, f64);
        case 3: return pick_latency_cluster_leaf<3>(leaf32, f64);
        case 4: return pick_latency_cluster_leaf<4>(leaf32, f64);
        case 5: return pick_latency_cluster_leaf<5>(leaf32, f64);
        case 6: return pick_latency_cluster_leaf<6>(leaf32, f64);
        case 7: return pick_latency_cluster_leaf<7>(leaf32, f64);
        case 8: return pick_latency_cluster_leaf<8>(leaf32, f64);
    }
    return nullptr;
}

void* pick_latency(int depth, bool leaf32, bool f64) {
    switch (depth) {
        case 1: return pick_latency_leaf<1>(leaf32, f64);
        case 2: return pick_latency_leaf<2>(leaf32, f64);
        case 3: return pick_latency_leaf<3>(leaf32, f64);
        case 4: return pick_latency_leaf<4>(leaf32, f64);
        case 5: return pick_latency_leaf<5>(leaf32, f64);
        case 6: return pick_latency_leaf<6>(leaf32, f64);
        case 7: return pick_latency_leaf<7>(leaf32, f64);
        case 8: return pick_latency_leaf<8>(leaf32, f64);
    }
    return nullptr;
}

template <int D, int R, bool LEAF32, typename XT>
void* heap_of() {
    return reinterpret_cast<void*>(&heap_kernel<D, R, LEAF32, XT>);
}

template <int D, int R>
void* pick_leaf(bool leaf32, bool f64) {
    if (leaf32) return f64 ? heap_of<D, R, true, double>() : heap_of<D, R, true, float>();
    return f64 ? heap_of<D, R, false, double>() : heap_of<D, R, false, float>();
}

template <int D>
void* pick_rows(int rows, bool leaf32, bool f64) {
    switch (rows) {
        case 128: return pick_leaf<D, 128>(leaf32, f64);
        case 64: return pick_leaf<D, 64>(leaf32, f64);
        case 32: return pick_leaf<D, 32>(leaf32, f64);
    }
    return nullptr;
}

template <int D>
void* pick_staged_leaf(bool leaf32, bool f64) {
    if (leaf32) {
        return f64 ? reinterpret_cast<void*>(&heap_staged_kernel<D, true, double>)
                   : reinterpret_cast<void*>(&heap_staged_kernel<D, true, float>);
    }
    return f64 ? reinterpret_cast<void*>(&heap_staged_kernel<D, false, double>)
               : reinterpret_cast<void*>(&heap_staged_kernel<D, false, float>);
}

void* pick_staged(int depth, bool leaf32, bool f64) {
    switch (depth) {
        case 1: return pick_staged_leaf<1>(leaf32, f64);
        case 2: return pick_staged_leaf<2>(leaf32, f64);
        case 3: return pick_staged_leaf<3>(leaf32, f64);
        case 4: return pick_staged_leaf<4>(leaf32, f64);
        case 5: return pick_staged_leaf<5>(leaf32, f64);
        case 6: return pick_staged_leaf<6>(leaf32, f64);
        case 7: return pick_staged_leaf<7>(leaf32, f64);
        case 8: return pick_staged_leaf<8>(leaf32, f64);
    }
    return nullptr;
}

void* pick_heap(int depth, int rows, bool leaf32, bool f64) {
    switch (depth) {
        case 1: return pick_rows<1>(rows, leaf32, f64);
        case 2: return pick_rows<2>(rows, leaf32, f64);
        case 3: return pick_rows<3>(rows, leaf32, f64);
        case 4: return pick_rows<4>(rows, leaf32, f64);
        case 5: return pick_rows<5>(rows, leaf32, f64);
        case 6: return pick_rows<6>(rows, leaf32, f64);
        case 7: return pick_rows<7>(rows, leaf32, f64);
        case 8: return pick_rows<8>(rows, leaf32, f64);
    }
    return nullptr;
}

}  // namespace

int heap_record_bytes(int depth, bool leaf32) { return record_bytes(depth, leaf32); }

int heap_chunk_trees() { return kTrees; }

int heap_slot_bits(int slots) {
    int bits = 1;
    while ((1 << bits) < slots) ++bits;
    return bits;
}

// The most rows per CTA (128, 64, 32) whose key tables, partials and team
// buffers fit; false when none do or the slot index needs more than
// kMaxSlotBits bits of the split word.
bool heap_plan(int slots, int depth, bool leaf32, int& rows, int& buffers) {
    if (depth < 1 || depth > 8 || heap_slot_bits(slots) > kMaxSlotBits) return false;
    for (int r : {128, 64, 32}) {
        if (layout_of(slots, depth, leaf32, r).total <= kHeapSmemLimit) {
            rows = r;
            buffers = 2;
            return true;
        }
    }
    return false;
}

namespace {

// Rows per CTA of a complete-tree launch: the plan's, halved while the batch
// would leave SMs idle.
int heap_rows(const DevForest& f, long long batch) {
    int rows = f.heap.rows;
    while (rows > 32 && (batch + rows - 1) / rows < f.sm_count) rows /= 2;
    return rows;
}

}  // namespace

// 128 rows per CTA: the staged kernel, whose producer warps prepare the next
// group's keys in TMEM while the walkers walk. Its 640 threads take most of
// an SM's registers, so it runs one CTA per SM and its TMEM allocation never
// waits for another CTA's.
bool heap_staged(const DevForest& f, long long batch) {
    return heap_rows(f, batch) == kStageRows && stage_cols(f.args.pad_slot) > 0 &&
           layout_of(f.args.slots, f.heap.depth, f.heap.leaf32, kStageRows, stage_partials(f.args.T)).total <=
               kHeapSmemLimit;
}

bool launch_heap(const DevForest& f, int dtype, const void* x, long long batch, double* out, cudaStream_t stream,
                 std::string& err) {
    const HeapArgs& h = f.heap;
    const bool f64 = dtype == 2;
    const int rows = heap_rows(f, batch);
    const int cols = stage_cols(f.args.pad_slot);
    const bool staged = heap_staged(f, batch);
    void* k = staged ? pick_staged(h.depth, h.leaf32, f64) : pick_heap(h.depth, rows, h.leaf32, f64);
    if (!k) {
        err = "no complete-tree kernel for this model";
        return false;
    }
    const int smem =
        layout_of(f.args.slots, h.depth, h.leaf32, rows, staged ? stage_partials(f.args.T) : 2 * kTeams).total;
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
    const long long groups = (batch + rows - 1) / rows;
    const int per_sm = staged ? 1 : std::max(1, kHeapSmemLimit / (smem + 1024));
    const int grid = static_cast<int>(std::min<long long>(groups, static_cast<long long>(f.sm_count) * per_sm));
    ForestArgs a = f.args;
    HeapArgs hh = h;
    hh.rows = rows;
    int stage = cols;
    void* args[] = {&a, &hh, const_cast<void**>(&x), &batch, &out, &stage};
    const cudaError_t e = cudaLaunchKernel(k, grid, staged ? kStagedThreads : kTeams * rows, args, smem, stream);
    if (e != cudaSuccess) {
        err = std::string("complete-tree kernel launch: ") + cudaGetErrorString(e);
        return false;
    }
    return true;
}

size_t latency_scratch_bytes(const DevForest& f) {
    if (f.heap.depth <= 0) return 0;
    const size_t blocks = static_cast<size_t>((f.args.T + kTreeBlock - 1) / kTreeBlock);
    return blocks * kLatencyRows * sizeof(double) + kLatencyCounters * sizeof(int);
}

// The tree-parallel kernel takes batches of at most kLatencyRows rows when
// the key tables of 32 rows and a whole 64-tree block fit shared memory.
bool latency_fits(const DevForest& f, long long batch) {
    const HeapArgs& h = f.heap;
    if (h.depth <= 0 || batch > kLatencyRows) return false;
    return latency_smem(f.args.slots, h.depth, h.leaf32) <= kHeapSmemLimit;
}

// Which form of the small-batch kernel a call of `batch` rows runs: 0 the
// counter form (latency_kernel), 1 the cluster form with every CTA reading
// the rows, 2 the cluster form with CTA 0 reading them once (the rows may
// then sit in pinned host memory). The cluster form needs at most
// kClusterBlocks blocks and a GPU that can place such a cluster (checked once
// per kernel and device).
int latency_form(const DevForest& f, int dtype, long long batch) {
    const HeapArgs& h = f.heap;
    const int blocks = (f.args.T + kTreeBlock - 1) / kTreeBlock;
    if (!latency_fits(f, batch) || blocks > kClusterBlocks) return 0;
    const int smem = latency_cluster_smem(f.args.slots, f.args.F);
    if (smem > kHeapSmemLimit) return 0;
    void* k = pick_latency_cluster(h.depth, h.leaf32, dtype == 2);
    if (!k) return 0;
    // (kernel, device, cluster size, shared memory) -> whether the GPU can place it
    struct Known {
        void* kernel;
        int device, blocks, smem;
        bool can;
    };
    static std::mutex mu;
    static std::vector<Known> known;
    bool can = false;
    {
        std::lock_guard<std::mutex> lock(mu);
        auto it = std::find_if(known.begin(), known.end(), [&](const Known& e) {
            return e.kernel == k && e.device == f.device && e.blocks == blocks && e.smem == smem;
        });
        if (it != known.end()) {
            can = it->can;
        } else {
            cudaLaunchConfig_t cfg = {};
            cudaLaunchAttribute attr[1];
            cfg.gridDim = dim3(static_cast<unsigned>(blocks));
            cfg.blockDim = dim3(kLatencyThreads);
            cfg.dynamicSmemBytes = static_cast<size_t>(smem);
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = static_cast<unsigned>(blocks);
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            int clusters = 0;
            can = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kHeapSmemLimit) == cudaSuccess &&
                  (blocks <= 8 ||
                   cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) &&
                  cudaOccupancyMaxActiveClusters(&clusters, k, &cfg) == cudaSuccess && clusters >= 1;
            cudaGetLastError();
            known.push_back(Known{k, f.device, blocks, smem, can});
        }
    }
    if (!can) return 0;
    const long long rows = std::min<long long>(batch, kGroupRows);
    return rows * f.args.F * (blocks - 1) <= kClusterPush ? 2 : 1;
}

bool launch_latency(const DevForest& f, int dtype, const void* x, long long batch, double* out, cudaStream_t stream,
                    std::string& err, void* scratch, int* counters) {
    const HeapArgs& h = f.heap;
    if (latency_form(f, dtype, batch) > 0) {
        void* k = pick_latency_cluster(h.depth, h.leaf32, dtype == 2);
        const int blocks = (f.args.T + kTreeBlock - 1) / kTreeBlock;
        const int groups = static_cast<int>((batch + kGroupRows - 1) / kGroupRows);
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        cfg.gridDim = dim3(static_cast<unsigned>(blocks * groups));
        cfg.blockDim = dim3(kLatencyThreads);
        cfg.dynamicSmemBytes = static_cast<size_t>(latency_cluster_smem(f.args.slots, f.args.F));
        cfg.stream = stream;
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = static_cast<unsigned>(blocks);
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        ForestArgs a = f.args;
        HeapArgs hh = h;
        void* args[] = {&a, &hh, const_cast<void**>(&x), &batch, &out};
        const cudaError_t e = cudaLaunchKernelExC(&cfg, k, args);
        if (e != cudaSuccess) {
            err = std::string("small-batch kernel launch: ") + cudaGetErrorString(e);
            return false;
        }
        return true;
    }
    void* k = pick_latency(h.depth, h.leaf32, dtype == 2);
    if (!k) {
        err = "no small-batch complete-tree kernel for this model";
        return false;
    }
    const int smem = latency_smem(f.args.slots, h.depth, h.leaf32);
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
    const int blocks = (f.args.T + kTreeBlock - 1) / kTreeBlock;
    const int groups = static_cast<int>((batch + kGroupRows - 1) / kGroupRows);
    double* bpart = static_cast<double*>(scratch);
    // The kernel leaves its counters at zero: a dedicated zeroed buffer needs
    // no clearing, counters in the shared scratch do.
    int* count = counters ? counters : reinterpret_cast<int*>(bpart + static_cast<size_t>(blocks) * kLatencyRows);
    cudaError_t e = counters ? cudaSuccess : cudaMemsetAsync(count, 0, kLatencyCounters * sizeof(int), stream);
    if (e != cudaSuccess) {
        err = std::string("cudaMemsetAsync: ") + cudaGetErrorString(e);
        return false;
    }
    ForestArgs a = f.args;
    HeapArgs hh = h;
    void* args[] = {&a, &hh, const_cast<void**>(&x), &batch, &out, &bpart, &count};
    e = cudaLaunchKernel(k, blocks * groups, kLatencyThreads, args, smem, stream);
    if (e != cudaSuccess) {
        err = std::string("small-batch kernel launch: ") + cudaGetErrorString(e);
        return false;
    }
    return true;
}
}  // namespace mlk::cuda
