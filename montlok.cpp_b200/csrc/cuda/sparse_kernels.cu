// Multi-output predict kernel for sm_100a: 2..8 outputs (LightGBM / XGBoost
// multiclass), trees of any shape whose records fit shared memory.
//
// Work split. A CTA owns R rows for the whole ensemble and runs one team of R
// threads (one per row) per output: team k walks the trees whose output is
// k, in tree order. The reference's association (trees.cpp:366-388) is per
// output: block 0 of 64 trees adds onto the base score, every later block
// sums from 0.0 and is then added (a block without trees of output k adds
// 0.0). A team therefore meets every tree of its output in order and needs
// nothing from the other teams; at the end the outputs meet in shared memory
// for the link (softmax needs all of them).
//
// Keys. The row's key table holds one entry per (feature, missing kind): kind
// 0 treats NaN as missing, kind 1 NaN and LightGBM's zero band (|v| <=
// 1e-35f). A missing value has key 0; any other value the order-preserving
// unsigned key u = (key32 ^ 0x80000000) | mask (>= 1). A split word is
//
//     W = (U_T & ~mask) | (slot << 1) | c          (U_T = T ^ 0x80000000)
//
// with c = 1 when missing values go right. A step computes v = u - c and
// goes right when v > W (unsigned): for a present value v keeps u's high
// bits, so the compare is the threshold test; a missing value with c = 1
// wraps to 0xFFFFFFFF and goes right, with c = 0 stays 0 and goes left. When
// v and W agree in their high bits the tree is walked again with those
// splits decided exactly (exact_right, the reference's comparison of the
// prepared double), as in the complete-tree kernel; missing values never tie.
//
// Trees. A tree record is a 16-byte header (block of the tree, depth, live)
// and its nodes in breadth-first order with the two children of a split
// adjacent, each node 8 bytes {W, byte offset to its left child}; a leaf is
// {(leaf + 1) << slot_bits | pad slot << 1, 0}: the pad slot's key is always
// 0, so a leaf never goes right and the walk stays on it. The leaf values
// (float32 when every leaf is exactly a float) follow the nodes. Records of
// one output are contiguous and padded to whole chunks with inert trees (one
// leaf, not live). Each team streams its records through two chunk buffers
// with bulk async copies and the protocol of the complete-tree kernel: the
// last warp done with a buffer refills it two chunks ahead, waits are
// bounded, a CTA-wide abort flag ends every wait.
#include <algorithm>
#include <cstdint>
#include <mutex>
#include <vector>

#include "async_copy.cuh"
#include "device_common.cuh"
#include "forest.cuh"

namespace mlk::cuda {
namespace {

constexpr int kTrees = 2;                  // trees per chunk = trees one thread walks side by side
constexpr int kMaxTeams = 8;               // outputs
constexpr int kTile = 4;                   // features per transpose tile in the prepare
constexpr int kTileBytes = 32 * (kTile + 1) * 8;
constexpr int kSmemLimit = 227 * 1024;
constexpr int kHeader = 384;               // mbarriers, counters, abort flag

// Shared memory: header | keys [slots][R] | outputs [K][R] double | first
// buffers of the K teams | second buffers (the prepare's tiles until the
// second chunk is issued).
struct Layout {
    int keys, outs, ring0, ring1, total;
};

__host__ __device__ inline Layout layout_of(int slots, int teams, int record, int rows) {
    Layout l{};
    l.keys = kHeader;
    l.outs = l.keys + align128(slots * rows * 4);
    l.ring0 = l.outs + align128(teams * rows * 8);
    const int chunk = kTrees * record;
    l.ring1 = l.ring0 + align128(teams * chunk);
    const int tiles = teams * (rows / 32) * kTileBytes;
    l.total = l.ring1 + align128(max(teams * chunk, tiles));
    return l;
}

// Keys of one prepared value into its feature's slots (kind 0, kind 1).
template <int STRIDE>
__device__ __forceinline__ void put_sparse_keys(const ForestArgs& a, unsigned* col, int2 s, double v, unsigned low) {
    const bool nan = v != v;
    const bool zero = nan || fabs(v) <= kZeroThr;
    const int k = a.cast_f32 ? key32(__double2float_rn(v)) : key32(__double2float_rd(v));
    const unsigned u = (static_cast<unsigned>(k) ^ 0x80000000u) | low;
    if (s.x >= 0) col[s.x * STRIDE] = nan ? 0u : u;
    if (s.y >= 0) col[s.y * STRIDE] = zero ? 0u : u;
}

// Keys of the 32 rows row0 .. row0 + 31 for features [f_begin, f_end) (the
// transpose of the complete-tree kernel's prepare: kTile features of all 32
// rows per step, the next two steps' loads in flight).
template <int STRIDE, typename XT>
__device__ void prepare_rows(const ForestArgs& a, const SparseArgs& s, const XT* __restrict__ x, long long row0,
                             long long batch, unsigned* keys, double* tile, int lane, int f_begin, int f_end,
                             unsigned low) {
    constexpr int kPerLoad = 32 / kTile;
    const int sub = lane / kTile, f_in = lane % kTile;
    auto load = [&](int f0, double (&v)[kTile]) {
        const int feat = f0 + f_in;
#pragma unroll
        for (int i = 0; i < kTile; ++i) {
            const long long row = row0 + i * kPerLoad + sub;
            v[i] = (feat < f_end && row < batch) ? load_x(x + row * a.F + feat) : 0.0;
        }
    };
    auto stage = [&](int f0, const double (&v)[kTile]) {
        const int feat = f0 + f_in;
        double mean = 0.0, scale = 1.0;
        if (a.standardize && feat < f_end) {
            mean = __ldg(a.pre_mean + feat);
            scale = __ldg(a.pre_scale + feat);
        }
#pragma unroll
        for (int i = 0; i < kTile; ++i) {
            const long long row = row0 + i * kPerLoad + sub;
            tile[(i * kPerLoad + sub) * (kTile + 1) + f_in] =
                (feat < f_end && row < batch) ? finish(a, v[i], mean, scale) : 0.0;
        }
    };
    auto keys_of = [&](int f0) {
        __syncwarp();
        const int nf = min(kTile, f_end - f0);
        for (int j = 0; j < nf; ++j) {
            put_sparse_keys<STRIDE>(a, keys + lane, __ldg(s.slot_of + f0 + j), tile[lane * (kTile + 1) + j], low);
        }
        __syncwarp();
    };
    double even[kTile], odd[kTile];
    load(f_begin, even);
    load(f_begin + kTile, odd);
    for (int f0 = f_begin; f0 < f_end; f0 += 2 * kTile) {
        stage(f0, even);
        load(f0 + 2 * kTile, even);
        keys_of(f0);
        if (f0 + kTile < f_end) {
            stage(f0 + kTile, odd);
            load(f0 + 3 * kTile, odd);
            keys_of(f0 + kTile);
        }
    }
}

// One tree walked exactly for one row: the packed compare where the high
// bits differ, exact_right where they tie. Returns the byte address of the
// leaf reached.
template <int R, typename XT>
__device__ __noinline__ uint32_t walk_exact(const ForestArgs& a, const SparseArgs& s, uint32_t base, uint32_t col,
                                            uint32_t mask, int depth, int record, const XT* __restrict__ x,
                                            long long row, long long batch) {
    uint32_t p = base + 16;
    for (int d = 0; d < depth; ++d) {
        const uint2 n = lds_v2(p);
        const uint32_t u = lds_u32(col + (n.x & (mask - 1u)) * (R * 2));
        const uint32_t v = u - (n.x & 1u);
        bool right = v > n.x;
        if ((v ^ n.x) <= mask) {
            const int node = __ldg(s.node_ids + static_cast<size_t>(record) * s.node_max + ((p - base - 16) >> 3));
            if (node >= 0) right = exact_right(a, x, row, batch, node);
        }
        p += n.y + (right ? 8u : 0u);
    }
    return p;
}

template <int R, int TEAMS, bool LEAF32, typename XT>
__global__ void __launch_bounds__(TEAMS * R, 1) sparse_kernel(const __grid_constant__ ForestArgs a, const __grid_constant__ SparseArgs s,
                                                                   const XT* __restrict__ x, long long batch,
                                                                   double* __restrict__ out) {
    constexpr int kWarpsPerTeam = R / 32;
    extern __shared__ __align__(128) unsigned char smem[];
    const int K = s.teams;
    const int record = s.record;
    const int chunk_bytes = kTrees * record;
    const Layout L = layout_of(s.slots, K, record, R);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem);          // [team][buffer]
    unsigned* done = reinterpret_cast<unsigned*>(smem + 128);   // [team][buffer]
    unsigned* fills = reinterpret_cast<unsigned*>(smem + 192);  // [team][buffer]
    volatile int* abort = reinterpret_cast<volatile int*>(smem + 256);
    unsigned* keys = reinterpret_cast<unsigned*>(smem + L.keys);
    double* outs = reinterpret_cast<double*>(smem + L.outs);

    const int tid = threadIdx.x;
    const int team = tid / R, r = tid % R;
    const int warp = tid >> 5, lane = tid & 31;
    const bool producer = r == 0;
    const int chunks = s.chunks[team];
    const unsigned char* stream = s.trees + static_cast<size_t>(s.offset[team]) * record;
    const int blocks = (a.T + kTreeBlock - 1) / kTreeBlock;
    const long long groups = (batch + R - 1) / R;
    const size_t row_bytes = static_cast<size_t>(a.F) * sizeof(XT);
    const uint32_t mask = (1u << s.slot_bits) - 1u;
    const uint32_t buf0 = smem_u32(smem + L.ring0) + team * chunk_bytes;
    const uint32_t buf1 = smem_u32(smem + L.ring1) + team * chunk_bytes;
    uint64_t* team_bar = bar + 2 * team;

    if (tid == 0) {
        for (int b = 0; b < 2 * kMaxTeams; ++b) {
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

    uint32_t phase = 0u;  // bit b: parity of the next fill of buffer b (a register, not an indexed array)
    auto issue = [&](int q) {
        if (a.skip_copies) return;  // fault injection: the wait for this chunk runs out
        const int b = q & 1;
        bulk_load(b ? buf1 : buf0, stream + static_cast<size_t>(q) * chunk_bytes, static_cast<uint32_t>(chunk_bytes),
                  &team_bar[b]);
        atomicAdd(&fills[2 * team + b], 1u);
    };
    if (producer && chunks > 0 && blockIdx.x < groups) issue(0);

    const uint32_t col = smem_u32(keys) + r * 4;
    const int nodes_bytes = 16 + s.node_max * 8;
    for (long long g = blockIdx.x; g < groups; g += gridDim.x) {
        const long long row0 = g * R;
        const long long row = row0 + r;
        {
            const int slice = warp % kWarpsPerTeam;
            const int per = (a.F + K - 1) / K;
            const int f_begin = min(a.F, team * per), f_end = min(a.F, f_begin + per);
            double* tile = reinterpret_cast<double*>(smem + L.ring1 + warp * kTileBytes);
            prepare_rows<R>(a, s, x, row0 + slice * 32, batch, keys + slice * 32, tile, lane, f_begin, f_end, mask);
            if (team == 0) keys[s.pad_slot * R + slice * 32 + lane] = 0u;
        }
        __syncthreads();
        if (producer && chunks > 1) issue(1);
        if (tid == 0 && g + gridDim.x < groups) {
            const long long r1 = row0 + static_cast<long long>(gridDim.x) * R;
            prefetch_l2(x + r1 * a.F, static_cast<size_t>(min(static_cast<long long>(R), batch - r1)) * row_bytes);
        }

        // The output's sum: block 0 adds onto the base, block b > 0 into
        // `part`, which is added when the next block starts.
        double acc = a.mean ? 0.0 : __ldg(a.base + team);
        double part = 0.0;
        int cur = 0;
        for (int q = 0; q < chunks; ++q) {
            const int b = q & 1;
            // Once the CTA is aborting no wait is trusted: a warp whose own
            // wait ran out has lost count of the barrier's phases, and a wait
            // on the other parity would return at once.
            const bool ok = __all_sync(0xffffffffu, !*abort && mbar_wait(&team_bar[b], (phase >> b) & 1u, a.wait_ns,
                                                                         abort));
            phase ^= 1u << b;
            if (ok) {
                const uint32_t buf = b ? buf1 : buf0;
                int4 hdr[kTrees];
                uint32_t p[kTrees];
                bool tie[kTrees];
                int depth = 0;
#pragma unroll
                for (int t = 0; t < kTrees; ++t) {
                    hdr[t] = lds_v4(buf + t * record);  // block, depth, live
                    depth = max(depth, hdr[t].y);
                    p[t] = buf + t * record + 16;
                    tie[t] = false;
                }
                // Unrolled by 4 (c4, depth 12: 16.2 ms per 1M rows against
                // 16.9 unrolled by 2, 17.5 by 1, 17.0 by 6, 16.7 by 8).
#pragma unroll 4
                for (int d = 0; d < depth; ++d) {
                    uint2 n[kTrees];
                    uint32_t u[kTrees];
#pragma unroll
                    for (int t = 0; t < kTrees; ++t) n[t] = lds_v2(p[t]);
#pragma unroll
                    for (int t = 0; t < kTrees; ++t) u[t] = lds_u32(col + (n[t].x & (mask - 1u)) * (R * 2));
#pragma unroll
                    for (int t = 0; t < kTrees; ++t) {
                        const uint32_t v = u[t] - (n[t].x & 1u);
                        tie[t] |= (v ^ n[t].x) <= mask;
                        p[t] += n[t].y + (v > n[t].x ? 8u : 0u);
                    }
                }
                bool any = false;
#pragma unroll
                for (int t = 0; t < kTrees; ++t) any |= tie[t];
                if (__any_sync(0xffffffffu, any)) {
#pragma unroll
                    for (int t = 0; t < kTrees; ++t) {
                        if (tie[t]) {
                            p[t] = walk_exact<R>(a, s, buf + t * record, col, mask, hdr[t].y,
                                                 s.offset[team] + q * kTrees + t, x, row, batch);
                        }
                    }
                }
#pragma unroll
                for (int t = 0; t < kTrees; ++t) {
                    if (hdr[t].z) {
                        const uint32_t leaf = (lds_u32(p[t]) >> s.slot_bits) - 1u;
                        const double value =
                            lds_leaf(buf + t * record + nodes_bytes + leaf * (LEAF32 ? 4u : 8u), LEAF32);
                        const int blk = hdr[t].x;
                        if (blk != cur) {
                            if (cur >= 1) acc = __dadd_rn(acc, part);
                            if (blk > cur + 1) acc = __dadd_rn(acc, 0.0);  // blocks without this output's trees
                            part = 0.0;
                            cur = blk;
                        }
                        if (blk == 0) acc = __dadd_rn(acc, value);
                        else part = __dadd_rn(part, value);
                    }
                }
            } else if (lane == 0) {
                *abort = 1;
            }
            __syncwarp();
            if (lane == 0) {
                __threadfence_block();
                const unsigned before = atomicAdd(&done[2 * team + b], 1u);
                if (before % kWarpsPerTeam == kWarpsPerTeam - 1 && q + 2 < chunks && !*abort) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    issue(q + 2);
                }
            }
        }
        if (cur >= 1) acc = __dadd_rn(acc, part);
        if (blocks - 1 > cur) acc = __dadd_rn(acc, 0.0);
        outs[team * R + r] = acc;
        if (__syncthreads_or(*abort)) {
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
            double v[kMaxTeams];
#pragma unroll
            for (int k = 0; k < kMaxTeams; ++k) {
                v[k] = 0.0;
                if (k < K) {
                    v[k] = outs[k * R + r];
                    if (a.mean) {
                        const int n = __ldg(a.counts + k);
                        v[k] = __dadd_rn(__ldg(a.base + k), n ? __ddiv_rn(v[k], static_cast<double>(n)) : 0.0);
                    }
                }
            }
            apply_link<kMaxTeams>(a, v, K);
#pragma unroll
            for (int k = 0; k < kMaxTeams; ++k) {
                if (k < K) out[row * K + k] = v[k];
            }
        }
        if (producer && chunks > 0 && g + gridDim.x < groups) issue(0);
        __syncthreads();  // keys and outputs are rewritten by the next group
    }
}

template <int R, int TEAMS, bool LEAF32, typename XT>
void* sparse_of() {
    return reinterpret_cast<void*>(&sparse_kernel<R, TEAMS, LEAF32, XT>);
}

// TEAMS bounds the outputs a launch may have (5 or 8): the register budget
// per thread follows from TEAMS * R threads per CTA.
template <int R, int TEAMS>
void* pick_leaf(bool leaf32, bool f64) {
    if (leaf32) return f64 ? sparse_of<R, TEAMS, true, double>() : sparse_of<R, TEAMS, true, float>();
    return f64 ? sparse_of<R, TEAMS, false, double>() : sparse_of<R, TEAMS, false, float>();
}

template <int TEAMS>
void* pick_rows(int rows, bool leaf32, bool f64) {
    switch (rows) {
        case 96: return pick_leaf<96, TEAMS>(leaf32, f64);
        case 64: return pick_leaf<64, TEAMS>(leaf32, f64);
        case 32: return pick_leaf<32, TEAMS>(leaf32, f64);
    }
    return nullptr;
}

void* pick_sparse(int teams, int rows, bool leaf32, bool f64) {
    return teams <= 5 ? pick_rows<5>(rows, leaf32, f64) : pick_rows<8>(rows, leaf32, f64);
}

}  // namespace

int sparse_chunk_trees() { return kTrees; }

// The most rows per CTA (96, 64, 32) whose key tables, outputs and team
// buffers fit shared memory; false when none do.
bool sparse_plan(int slots, int teams, int record, int& rows) {
    if (teams < 2 || teams > kMaxTeams) return false;
    for (int r : {96, 64, 32}) {
        if (layout_of(slots, teams, record, r).total <= kSmemLimit) {
            rows = r;
            return true;
        }
    }
    return false;
}

bool launch_sparse(const DevForest& f, int dtype, const void* x, long long batch, double* out, cudaStream_t stream,
                   std::string& err) {
    SparseArgs ss = f.sparse;
    // Fewer rows per CTA while the batch would leave SMs idle.
    while (ss.rows > 32 && (batch + ss.rows - 1) / ss.rows < f.sm_count) ss.rows = ss.rows == 96 ? 64 : 32;
    const SparseArgs& s = ss;
    void* k = pick_sparse(s.teams, s.rows, s.leaf32, dtype == 2);
    if (!k) {
        err = "no multi-output kernel for this model";
        return false;
    }
    const int smem = layout_of(s.slots, s.teams, s.record, s.rows).total;
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
    const long long groups = (batch + s.rows - 1) / s.rows;
    const int grid = static_cast<int>(std::min<long long>(groups, static_cast<long long>(f.sm_count)));
    ForestArgs a = f.args;
    void* args[] = {&a, &ss, const_cast<void**>(&x), &batch, &out};
    const cudaError_t e = cudaLaunchKernel(k, grid, s.teams * s.rows, args, smem, stream);
    if (e != cudaSuccess) {
        err = std::string("multi-output kernel launch: ") + cudaGetErrorString(e);
        return false;
    }
    return true;
}

}  // namespace mlk::cuda
