// Latency engine: a resident kernel that answers small host-buffer predicts
// (at most kEngineRows rows) without a launch or a copy per call. It is the
// GPU counterpart of the reference's latency threads (montlok_set_latency_
// threads, src/core/runtime.cpp:300-420): workers that stay up, wait on a
// mailbox and split a small batch's 64-tree blocks, whose sums are then added
// in block order (trees.cpp:303-362).
//
// Each CTA of the engine owns one 64-tree block of a complete-tree forest and
// keeps its tree records in shared memory for its whole life, so a walk is
// eight shared loads. The calling thread writes the request's rows into a
// mailbox in pinned host memory and posts its number and row count in one
// 64-bit word. Thread 0 of CTA 0 polls that word (system-scope acquire loads;
// the only poller of the bus) and CTA 0 reads the rows over the bus in 16-byte
// loads. Engines of at most kClusterBlocks blocks run as one thread-block
// cluster: CTA 0 pushes the rows into every CTA's shared memory (or, for
// large requests, through device memory) and wakes each CTA with a remote
// mbarrier arrival; every CTA builds the rows' keys, walks its 64 trees for
// each row (one thread per tree and row pair), adds the leaves in tree order
// and pushes its block sum into CTA 0's shared memory, arriving on CTA 0's
// barrier; CTA 0 adds the block sums in block order and applies the link.
// Larger engines are a cooperative launch whose CTAs meet through device
// memory: CTA 0 relays the rows and publishes the post word with a release
// store the others poll; the last CTA to finish (an acquire-release counter,
// no waiting) loads the block sums sixteen at a time and adds them in order.
// Either way each row's answer is written into the mailbox as one 16-byte
// record with the request's number; the caller spins on those numbers.
//
// Every wait is bounded. An engine CTA exits when the host asks (stop), when
// CTA 0 has seen no request for kEngineIdleNs (it tells the others: a quit
// flag, or in the cluster a pushed order to leave; they also leave on their
// own after a longer wait) or after kEnginePolls polls; the cluster form's
// CTAs leave through a cluster barrier. The host starts the engine on demand
// (a cluster launch when the GPU can place it, else a cooperative launch; if
// neither can start the call takes the graph path), relaunches it when it has
// exited, and gives up on a request after kEngineTimeoutNs with
// MONTLOK_ERROR_INTERNAL.
#include <atomic>
#include <chrono>
#include <cstring>
#include <memory>
#include <string>
#include <thread>

#include "async_copy.cuh"
#include "cluster.cuh"
#include "device_common.cuh"
#include "engine.cuh"
#include "forest.cuh"

namespace mlk::cuda {
namespace {

constexpr int kEngineThreads = 256;                     // 64 trees x 4 row pairs
constexpr int kEnginePairs = kEngineThreads / kTreeBlock;
constexpr unsigned long long kEngineIdleNs = 200000000ull;  // an engine idle this long exits
constexpr long long kEnginePolls = 1ll << 24;               // hard cap on one wait's polls
constexpr long long kEngineTimeoutNs = 2000000000ll;        // a request unanswered this long fails
constexpr long long kEngineCheckNs = 20000000ll;            // when the host first checks the engine
static_assert(kEngineRows == 2 * kEnginePairs, "each thread walks two rows");

// The mailbox, in pinned host memory the engine reads and writes over the bus.
// A request is posted as one 64-bit store of its number (low half) and rows
// (high half), so one bus read brings both.
struct Mailbox {
    unsigned long long post;  // host: rows << 32 | number of the latest request
    unsigned int stop;        // host: exit now
    unsigned int unused;
};

__host__ __device__ inline unsigned long long post_word(unsigned int seq, int rows) {
    return static_cast<unsigned long long>(static_cast<unsigned int>(rows)) << 32 | seq;
}

// One row's answer, written with a single 16-byte store: the caller reads
// `value` once `seq` shows its request's number, so the engine needs no
// system-wide fence before publishing.
struct alignas(16) Answer {
    double value;
    unsigned long long seq;
};

__device__ __forceinline__ unsigned int load_acquire_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long load_acquire_sys64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// A request value read past any cache: the host rewrites these each call.
__device__ __forceinline__ double load_fresh(const double* p) {
    double v;
    asm volatile("ld.global.cv.f64 %0, [%1];" : "=d"(v) : "l"(p) : "memory");
    return v;
}

constexpr int kClusterBlocks = 16;  // engines of at most this many blocks run as one thread-block cluster
// The cluster form pushes a request's rows into every CTA's shared memory when
// the copies total at most this many values (c5: requests of 1 or 2 rows);
// larger requests go through device memory once (CTA 0's port would carry
// every copy).
constexpr int kPushValues = 6144;

// Shared memory: control words and the cluster form's two mbarriers | the
// block's tree records | keys [slot][row] | rows [row][F] | leaf values
// [tree][row] | per feature its slots (int4), preprocessing mean and scale
// (copied once, so a request reads no constant from global memory) | the
// cluster form's block sums [block][row] (used in CTA 0).
__host__ __device__ inline int engine_smem(int slots, int F, int record) {
    return 128 + kTreeBlock * record + align128(slots * kEngineRows * 4) + align128(kEngineRows * F * 8) +
           kTreeBlock * kEngineRows * 8 + align128(F * 32) + kClusterBlocks * kEngineRows * 8;
}


// The split decided on the double for a float64 model whose keys tied (the
// rows sit in shared memory: `xs` [row][F]).
__device__ __forceinline__ bool exact_split(const ForestArgs& a, const double* xs, int row, int node) {
    const int feat = __ldg(a.feature + node);
    const double t = __ldg(a.threshold + node);
    const double mean = a.standardize ? __ldg(a.pre_mean + feat) : 0.0;
    const double scale = a.standardize ? __ldg(a.pre_scale + feat) : 1.0;
    const double v = finish(a, xs[row * a.F + feat], mean, scale);
    return a.le ? (v > t) : !(v < t);
}

// Device-memory side of a request: the rows CTA 0 copied from the mailbox,
// and the words it publishes them with.
struct Relay {
    unsigned long long go;  // rows << 32 | number of the request whose rows are in `x`
    int count;              // CTAs done with the current request
    int quit;               // 1: every CTA leaves
};

__device__ __forceinline__ unsigned long long load_acquire_gpu64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void store_release_gpu64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Counts this CTA done (release: its block sums, stored before the CTA
// barrier, are published with it; acquire: the last CTA sees every other
// CTA's); returns the count before.
__device__ __forceinline__ int count_done(int* p) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(p) : "memory");
    return old;
}

// Release at cluster scope: the CTA's stores before its barrier reach the
// waiter with the arrival.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}
// Waits for phase `parity` of a local mbarrier that CTAs of the cluster
// arrive on; false after `limit_ns`.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, unsigned long long limit_ns) {
    if (mbar_try_cluster(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (long long polls = 0; polls < kEnginePolls; ++polls) {
        if (mbar_try_cluster(bar, parity)) return true;
        if (global_ns() - t0 > limit_ns) return false;
    }
    return false;
}

// CLUSTER: the engine's CTAs form one thread-block cluster (at most
// kClusterBlocks). CTA 0 pushes a request's rows and control words into every
// CTA's shared memory and wakes it with a remote arrival on its `rows_bar`;
// each CTA pushes its block sums into CTA 0's `bsum` and arrives on CTA 0's
// `sum_bar`, on which CTA 0 waits before adding them in block order. No
// device-memory relay, counter or reload of the sums. Without CLUSTER the
// CTAs meet through device memory (`relay`, `bpart`). An engine CTA leaves
// only through a cluster barrier, so no CTA leaves while another may still
// write into its shared memory.
template <int D, bool LEAF32, bool CLUSTER>
__global__ void __launch_bounds__(kEngineThreads, 1)
    engine_kernel(const __grid_constant__ ForestArgs a, const __grid_constant__ HeapArgs h, Mailbox* box, const double* x, double* out, double* bpart,
                  double* xd, Relay* relay, unsigned int first) {
    Answer* answers = reinterpret_cast<Answer*>(out);
    constexpr int kRec = heap_record_size(D, LEAF32);
    constexpr int kSplits = (1 << D) - 1;
    extern __shared__ __align__(128) unsigned char smem[];
    volatile unsigned int* ctl = reinterpret_cast<volatile unsigned int*>(smem);  // request, exit/last, rows, ok
    uint64_t* rows_bar = reinterpret_cast<uint64_t*>(smem + 64);                 // cluster: a request's rows are in
    uint64_t* sum_bar = reinterpret_cast<uint64_t*>(smem + 72);                  // cluster, CTA 0: every block summed
    unsigned char* trees = smem + 128;
    int* keys = reinterpret_cast<int*>(trees + kTreeBlock * kRec);  // [slot][kEngineRows]
    double* xs = reinterpret_cast<double*>(reinterpret_cast<unsigned char*>(keys) +
                                           align128(a.slots * kEngineRows * 4));  // [row][F]
    double* leafv = reinterpret_cast<double*>(reinterpret_cast<unsigned char*>(xs) +
                                              align128(kEngineRows * a.F * 8));   // [tree][row]
    int4* slot_of = reinterpret_cast<int4*>(leafv + kTreeBlock * kEngineRows);  // [F]
    double* pre = reinterpret_cast<double*>(slot_of + a.F);                     // [F] mean, scale
    double* bsum = reinterpret_cast<double*>(reinterpret_cast<unsigned char*>(slot_of) + align128(a.F * 32));  // [block][row]

    const int tid = threadIdx.x;
    const int blocks = gridDim.x, block = blockIdx.x;
    const int t0 = block * kTreeBlock;
    const int nt = min(kTreeBlock, a.T - t0);
    const uint32_t mask = (1u << h.slot_bits) - 1u;
    volatile int* quit = &relay->quit;

    // The block's tree records, once for the engine's life.
    {
        const int4* src = reinterpret_cast<const int4*>(h.trees + static_cast<size_t>(t0) * kRec);
        int4* dst = reinterpret_cast<int4*>(trees);
        for (int i = tid; i < nt * kRec / 16; i += kEngineThreads) dst[i] = __ldg(src + i);
        for (int f = tid; f < a.F; f += kEngineThreads) {
            slot_of[f] = __ldg(a.slot_of + f);
            pre[2 * f] = a.standardize ? __ldg(a.pre_mean + f) : 0.0;
            pre[2 * f + 1] = a.standardize ? __ldg(a.pre_scale + f) : 1.0;
        }
    }
    if constexpr (CLUSTER) {
        if (tid == 0) {
            mbar_init(rows_bar, 1);
            mbar_init(sum_bar, static_cast<uint32_t>(blocks));
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        __syncthreads();
        cluster_sync();  // every CTA's barriers exist before any remote arrival
    } else {
        __syncthreads();
    }

    unsigned int mine = first;
    uint32_t n = 0;  // requests this engine has served (the phase of its barriers)
    for (;;) {
        // CTA 0 waits on the mailbox in host memory (the only poller of the
        // bus); every wait is bounded.
        if (block == 0) {
            if (tid == 0) {
                unsigned int cmd = 0, seq = mine;
                unsigned long long word = 0;
                const unsigned long long since = global_ns();
                for (long long polls = 0;; ++polls) {
                    word = load_acquire_sys64(&box->post);
                    seq = static_cast<unsigned int>(word);
                    if (seq != mine) break;
                    // `stop` (a second bus read) is looked at every 256th poll
                    // only, so a poll is one bus round trip.
                    if ((!CLUSTER && *quit) || polls >= kEnginePolls ||
                        ((polls & 255) == 255 && load_acquire_sys(&box->stop))) {
                        cmd = 1;
                        break;
                    }
                    // CTA 0 decides when the engine has idled long enough.
                    if (global_ns() - since > kEngineIdleNs) {
                        cmd = 1;
                        break;
                    }
                    __nanosleep(32);
                }
                if (!CLUSTER && cmd) atomicExch(&relay->quit, 1);
                ctl[0] = seq;
                ctl[1] = cmd;
                ctl[2] = static_cast<unsigned int>(min(kEngineRows, max(1, static_cast<int>(word >> 32))));
            }
            __syncthreads();
        } else if constexpr (CLUSTER) {
            // CTA 0 pushes the request (or the order to leave) and arrives;
            // the bound is a safety net far beyond CTA 0's idle limit.
            if (tid == 0 && !mbar_wait_cluster(rows_bar, n & 1u, 4 * kEngineIdleNs)) ctl[1] = 1;
            __syncthreads();
        } else {
            if (tid == 0) {
                unsigned int cmd = 0, seq = mine;
                unsigned long long word = 0;
                const unsigned long long since = global_ns();
                for (long long polls = 0;; ++polls) {
                    word = load_acquire_gpu64(&relay->go);
                    seq = static_cast<unsigned int>(word);
                    if (seq != mine) break;
                    if (*quit || polls >= kEnginePolls || global_ns() - since > 2 * kEngineIdleNs) {
                        cmd = 1;
                        break;
                    }
                    __nanosleep(16);
                }
                ctl[0] = seq;
                ctl[1] = cmd;
                ctl[2] = static_cast<unsigned int>(min(kEngineRows, max(1, static_cast<int>(word >> 32))));
            }
            __syncthreads();
        }
        const unsigned int cmd = ctl[1];
        const unsigned int seq = ctl[0];
        const int rows = static_cast<int>(ctl[2]);
        const int values = rows * a.F;
        const bool push = CLUSTER && values * (blocks - 1) <= kPushValues;
        if (block == 0) {
            if (!cmd) {
                // Rows from host memory in 16-byte reads, into this CTA's
                // table and (cluster) every other CTA's, or (no cluster)
                // relayed through device memory.
                // Four reads in flight per thread before any store (each read
                // is a bus round trip).
                constexpr int kInFlight = 4;
                const int pairs = (values + 1) / 2;
                for (int i0 = tid; i0 < pairs; i0 += kInFlight * kEngineThreads) {
                    double2 v[kInFlight];
#pragma unroll
                    for (int u = 0; u < kInFlight; ++u) {
                        const int i = i0 + u * kEngineThreads;
                        if (i < pairs) {
                            asm volatile("ld.global.cv.v2.f64 {%0, %1}, [%2];"
                                         : "=d"(v[u].x), "=d"(v[u].y)
                                         : "l"(x + 2 * i)
                                         : "memory");
                        }
                    }
#pragma unroll
                    for (int u = 0; u < kInFlight; ++u) {
                        const int i = i0 + u * kEngineThreads;
                        if (i >= pairs) break;
                        xs[2 * i] = v[u].x;
                        if (2 * i + 1 < values) xs[2 * i + 1] = v[u].y;
                        if (push) {
                            // pairs are 16-byte aligned ([row][F] doubles); the
                            // odd value past the end lands in the table's slack
                            const uint32_t at = smem_u32(xs + 2 * i);
                            for (int j = 1; j < blocks; ++j) st_cluster_v2f64(cluster_map(at, j), v[u].x, v[u].y);
                        } else {
                            xd[2 * i] = v[u].x;
                            if (2 * i + 1 < values) xd[2 * i + 1] = v[u].y;
                        }
                    }
                }
            }
            __syncthreads();
            if constexpr (CLUSTER) {
                if (tid >= 1 && tid < blocks) {
                    const uint32_t c = cluster_map(smem_u32(const_cast<unsigned int*>(ctl)), tid);
                    st_cluster_u32(c, seq);
                    st_cluster_u32(c + 4, cmd);
                    st_cluster_u32(c + 8, static_cast<unsigned int>(rows));
                    mbar_arrive_remote(cluster_map(smem_u32(rows_bar), tid));
                }
            } else if (tid == 0 && !cmd) {
                // Release: the rows stored into `xd` before the barrier go with it.
                store_release_gpu64(&relay->go, post_word(seq, rows));
            }
        } else if (!push) {
            // Rows relayed through device memory: published by the release
            // store (no cluster) or the cluster-scope arrival CTA 0 made
            // after storing them.
            if (!cmd) {
                for (int i = tid; i < values; i += kEngineThreads) xs[i] = __ldcg(xd + i);
            }
            __syncthreads();
        }
        if (cmd) break;
        for (int i = tid; i < values; i += kEngineThreads) {
            const int f = i % a.F;
            put_keys<kEngineRows>(a, keys + i / a.F, slot_of[f], finish(a, xs[i], pre[2 * f], pre[2 * f + 1]),
                                  static_cast<int>(mask));
        }
        if (tid < kEngineRows) keys[a.pad_slot * kEngineRows + tid] = INT_MIN;
        __syncthreads();

        // Thread (pair, local) walks tree t0 + local for rows pair and pair + 4.
        const int local = tid % kTreeBlock, pair = tid / kTreeBlock;
        if (local < nt && pair < rows) {
            const uint32_t base = smem_u32(trees + local * kRec);
            // Heap index of the leaf row r reaches; `exact` decides tied
            // splits on the double, `tie` reports whether any split tied.
            auto walk = [&](int r, bool exact, bool& tie) {
                const uint32_t col = smem_u32(keys + r);
                uint32_t i = 0;
#pragma unroll
                for (int d = 0; d < D; ++d) {
                    const uint32_t n = lds_u32(base + 4 * i);
                    const int k = lds_s32(col + (n & mask) * (kEngineRows * 4));
                    bool right = k > static_cast<int>(n);
                    if (k == static_cast<int>(n)) {
                        tie = true;
                        if (exact) {
                            const int node = __ldg(h.node_ids + static_cast<size_t>(t0 + local) * kSplits + i);
                            if (node >= 0) right = exact_split(a, xs, r, node);
                        }
                    }
                    i = 2 * i + (right ? 2u : 1u);
                }
                return i;
            };
            for (int r = pair; r < rows; r += kEnginePairs) {
                bool tie = false;
                uint32_t i = walk(r, false, tie);
                if (tie) i = walk(r, true, tie);
                const uint32_t leaf = i - kSplits;  // leaves follow the 2^D split words
                leafv[local * kEngineRows + r] = lds_leaf(base + (4u << D) + leaf * (LEAF32 ? 4u : 8u), LEAF32);
            }
        }
        __syncthreads();
        if (tid < rows) {
            double acc = (block == 0 && !a.mean) ? __ldg(a.base) : 0.0;
            for (int j = 0; j < nt; ++j) acc = __dadd_rn(acc, leafv[j * kEngineRows + tid]);
            if constexpr (CLUSTER) {
                st_cluster_f64(cluster_map(smem_u32(bsum + block * kEngineRows + tid), 0), acc);
            } else {
                __stcg(bpart + static_cast<size_t>(block) * kEngineRows + tid, acc);
            }
        }
        __syncthreads();
        bool last;
        if constexpr (CLUSTER) {
            if (tid == 0) mbar_arrive_remote(cluster_map(smem_u32(sum_bar), 0));
            last = block == 0;
            if (last) {
                if (tid == 0) ctl[3] = mbar_wait_cluster(sum_bar, n & 1u, kEngineIdleNs) ? 1u : 0u;
                __syncthreads();
                if (!ctl[3]) {
                    // A block never reported: tell every CTA to leave (the
                    // host restarts the engine and the request stays posted).
                    if (tid >= 1 && tid < blocks) {
                        const uint32_t c = cluster_map(smem_u32(const_cast<unsigned int*>(ctl)), tid);
                        st_cluster_u32(c + 4, 1u);
                        mbar_arrive_remote(cluster_map(smem_u32(rows_bar), tid));
                    }
                    break;
                }
            }
        } else {
            if (tid == 0) {
                const bool is_last = count_done(&relay->count) == blocks - 1;
                if (is_last) relay->count = 0;  // every CTA has counted this request
                ctl[1] = is_last;
            }
            __syncthreads();
            last = ctl[1] != 0;
        }
        if (last) {
            if (tid < rows) {
                // The block sums, 16 loads in flight at a time, added in
                // block order.
                constexpr int kBatch = 16;
                double v[1] = {0.0};
                for (int b0 = 0; b0 < blocks; b0 += kBatch) {
                    double t[kBatch];
#pragma unroll
                    for (int j = 0; j < kBatch; ++j) {
                        if constexpr (CLUSTER) {
                            t[j] = b0 + j < blocks ? bsum[(b0 + j) * kEngineRows + tid] : 0.0;
                        } else {
                            t[j] = b0 + j < blocks ? __ldcg(bpart + static_cast<size_t>(b0 + j) * kEngineRows + tid) : 0.0;
                        }
                    }
#pragma unroll
                    for (int j = 0; j < kBatch; ++j) {
                        if (b0 + j < blocks) v[0] = b0 + j == 0 ? t[j] : __dadd_rn(v[0], t[j]);
                    }
                }
                if (a.mean) {
                    const int c = __ldg(a.counts);
                    v[0] = __dadd_rn(__ldg(a.base), c ? __ddiv_rn(v[0], static_cast<double>(c)) : 0.0);
                }
                apply_link<1>(a, v, 1);
                const unsigned long long tag = seq;
                asm volatile("st.global.v2.b64 [%0], {%1, %2};" ::"l"(answers + tid),
                             "l"(__double_as_longlong(v[0])), "l"(tag)
                             : "memory");
            }
        }
        mine = seq;
        ++n;
        __syncthreads();  // every thread has read this request's control words before they are rewritten
    }
    if constexpr (CLUSTER) cluster_sync();
}

template <int D, bool LEAF32>
void* engine_of(bool cluster) {
    return cluster ? reinterpret_cast<void*>(&engine_kernel<D, LEAF32, true>)
                   : reinterpret_cast<void*>(&engine_kernel<D, LEAF32, false>);
}

void* pick_engine(int depth, bool leaf32, bool cluster) {
    switch (depth) {
        case 1: return leaf32 ? engine_of<1, true>(cluster) : engine_of<1, false>(cluster);
        case 2: return leaf32 ? engine_of<2, true>(cluster) : engine_of<2, false>(cluster);
        case 3: return leaf32 ? engine_of<3, true>(cluster) : engine_of<3, false>(cluster);
        case 4: return leaf32 ? engine_of<4, true>(cluster) : engine_of<4, false>(cluster);
        case 5: return leaf32 ? engine_of<5, true>(cluster) : engine_of<5, false>(cluster);
        case 6: return leaf32 ? engine_of<6, true>(cluster) : engine_of<6, false>(cluster);
        case 7: return leaf32 ? engine_of<7, true>(cluster) : engine_of<7, false>(cluster);
        case 8: return leaf32 ? engine_of<8, true>(cluster) : engine_of<8, false>(cluster);
    }
    return nullptr;
}

bool checked(cudaError_t e, const char* what, std::string& err) {
    if (e == cudaSuccess) return true;
    err = std::string(what) + " failed: " + cudaGetErrorString(e);
    cudaGetLastError();
    return false;
}

long long now_ns() {
    return std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now().time_since_epoch())
        .count();
}

}  // namespace

struct LatencyEngine {
    unsigned long long forest = 0;
    int device = 0;
    int blocks = 0, F = 0, K = 0;
    cudaStream_t stream = nullptr;
    unsigned char* host = nullptr;  // mailbox, then kEngineRows * F inputs, then kEngineRows * K outputs
    unsigned char* mapped = nullptr;
    void* dev = nullptr;            // block sums, relayed rows, then the Relay words
    unsigned int seq = 0;
    bool launched = false;
    bool cluster = false;  // running as one thread-block cluster

    Mailbox* box() const { return reinterpret_cast<Mailbox*>(host); }
    double* x_host() const { return reinterpret_cast<double*>(host + 64); }
    Answer* out_host() const { return reinterpret_cast<Answer*>(host + 64 + kEngineRows * F * 8); }

    ~LatencyEngine() {
        if (host) {
            reinterpret_cast<volatile unsigned int*>(&box()->stop)[0] = 1;
            if (stream) cudaStreamSynchronize(stream);  // the engine sees `stop` at its next poll
        }
        if (stream) cudaStreamDestroy(stream);
        if (dev) cudaFree(dev);
        if (host) cudaFreeHost(host);
    }
};

void destroy_engine(LatencyEngine* e) { delete e; }

bool engine_fits(const DevForest& f, long long batch) {
    if (f.heap.depth <= 0 || batch < 1 || batch > kEngineRows || f.args.K != 1) return false;
    const int blocks = (f.args.T + kTreeBlock - 1) / kTreeBlock;
    const int smem = engine_smem(f.args.slots, f.args.F, heap_record_bytes(f.heap.depth, f.heap.leaf32));
    return blocks <= f.sm_count && smem <= 227 * 1024;
}

// Starts (or restarts) the engine of `e` for forest `f`; `first` is the
// request number the engine treats as already answered.
// An engine of at most kClusterBlocks blocks runs as one thread-block
// cluster when the GPU can place it; otherwise as a cooperative launch.
static bool engine_launch(const DevForest& f, LatencyEngine& e, unsigned int first, std::string& err) {
    const int smem = engine_smem(f.args.slots, f.args.F, heap_record_bytes(f.heap.depth, f.heap.leaf32));
    bool cluster = e.blocks <= kClusterBlocks;
    void* kc = pick_engine(f.heap.depth, f.heap.leaf32 != 0, true);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    if (cluster && kc) {
        cfg.gridDim = dim3(static_cast<unsigned>(e.blocks));
        cfg.blockDim = dim3(kEngineThreads);
        cfg.dynamicSmemBytes = static_cast<size_t>(smem);
        cfg.stream = e.stream;
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = static_cast<unsigned>(e.blocks);
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int clusters = 0;
        cluster = cudaFuncSetAttribute(kc, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) == cudaSuccess &&
                  (e.blocks <= 8 ||
                   cudaFuncSetAttribute(kc, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) &&
                  cudaOccupancyMaxActiveClusters(&clusters, kc, &cfg) == cudaSuccess && clusters >= 1;
        cudaGetLastError();
    } else {
        cluster = false;
    }
    void* k = cluster ? kc : pick_engine(f.heap.depth, f.heap.leaf32 != 0, false);
    if (!k || (!cluster && !checked(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                                    "cudaFuncSetAttribute", err))) {
        if (!k) err = "no latency engine for this model";
        return false;
    }
    double* bpart = static_cast<double*>(e.dev);
    double* xd = bpart + static_cast<size_t>(e.blocks) * kEngineRows;
    Relay* relay = reinterpret_cast<Relay*>(xd + static_cast<size_t>(kEngineRows) * e.F);
    // The relay starts at the request the engine treats as answered.
    const Relay start{first, 0, 0};
    if (!checked(cudaMemcpyAsync(relay, &start, sizeof start, cudaMemcpyHostToDevice, e.stream), "cudaMemcpyAsync",
                 err) ||
        !checked(cudaStreamSynchronize(e.stream), "cudaStreamSynchronize", err)) {
        return false;
    }
    e.box()->stop = 0;
    Mailbox* box = reinterpret_cast<Mailbox*>(e.mapped);
    const double* x = reinterpret_cast<const double*>(e.mapped + 64);
    double* out = reinterpret_cast<double*>(e.mapped + 64 + kEngineRows * e.F * 8);
    ForestArgs a = f.args;
    HeapArgs h = f.heap;
    void* args[] = {&a, &h, &box, &x, &out, &bpart, &xd, &relay, &first};
    const cudaError_t launched = cluster ? cudaLaunchKernelExC(&cfg, k, args)
                                         : cudaLaunchCooperativeKernel(k, e.blocks, kEngineThreads, args, smem, e.stream);
    if (!checked(launched, "latency engine launch", err)) return false;
    e.launched = true;
    e.cluster = cluster;
    return true;
}

int engine_predict(const DevForest& f, LatencyEngine*& slot, int dtype, const void* x, size_t batch, double* out,
                   std::string& err) {
    if (!engine_fits(f, static_cast<long long>(batch))) return -1;
    if (slot && slot->forest != f.uid) {
        delete slot;  // one engine per thread and device: the newest model wins
        slot = nullptr;
    }
    if (!slot) {
        auto e = std::make_unique<LatencyEngine>();
        e->forest = f.uid;
        e->device = f.device;
        e->blocks = (f.args.T + kTreeBlock - 1) / kTreeBlock;
        e->F = f.args.F;
        e->K = f.args.K;
        const size_t bytes = 64 + static_cast<size_t>(kEngineRows) * (e->F * 8 + e->K * sizeof(Answer));
        void* host = nullptr;
        if (!checked(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking), "cudaStreamCreate", err) ||
            !checked(cudaHostAlloc(&host, bytes, cudaHostAllocMapped), "cudaHostAlloc", err)) {
            return kEngineFailed;
        }
        e->host = static_cast<unsigned char*>(host);
        std::memset(e->host, 0, bytes);
        void* mapped = nullptr;
        if (!checked(cudaHostGetDevicePointer(&mapped, host, 0), "cudaHostGetDevicePointer", err) ||
            !checked(cudaMalloc(&e->dev, (static_cast<size_t>(e->blocks) + e->F) * kEngineRows * 8 + sizeof(Relay)),
                     "cudaMalloc", err)) {
            return kEngineFailed;
        }
        e->mapped = static_cast<unsigned char*>(mapped);
        slot = e.release();
    }
    LatencyEngine& e = *slot;
    const bool running = e.launched && cudaStreamQuery(e.stream) == cudaErrorNotReady;
    cudaGetLastError();
    if (!running) {
        if (e.launched && !checked(cudaStreamSynchronize(e.stream), "latency engine", err)) return kEngineFailed;
        if (!engine_launch(f, e, e.seq, err)) return -1;  // e.g. not enough SMs free: take the graph path
    }
    // Post the request: rows first, then its number (x86 keeps the stores in
    // order, and the engine reads the number with acquire semantics).
    double* xh = e.x_host();
    const size_t values = batch * static_cast<size_t>(e.F);
    if (dtype == 1) {
        for (size_t i = 0; i < values; ++i) xh[i] = static_cast<const float*>(x)[i];
    } else {
        std::memcpy(xh, x, values * sizeof(double));
    }
    volatile Mailbox* box = e.box();
    const unsigned int seq = ++e.seq;
    std::atomic_thread_fence(std::memory_order_seq_cst);
    box->post = post_word(seq, static_cast<int>(batch));  // one aligned 64-bit store
    const long long posted = now_ns();
    long long checked_at = posted + kEngineCheckNs;
    volatile Answer* answers = e.out_host();
    auto answered = [&] {
        for (size_t r = 0; r < batch; ++r) {
            if (answers[r].seq != seq) return false;
        }
        return true;
    };
    for (unsigned spins = 0; !answered(); ++spins) {
        if ((spins & 1023u) != 1023u) continue;
        const long long t = now_ns();
        if (t > posted + kEngineTimeoutNs) {
            box->stop = 1;
            err = "the latency engine did not answer within 2 s";
            return kEngineFailed;
        }
        if (t > checked_at) {
            checked_at = t + kEngineCheckNs;
            // An engine that left (idle, or racing this request) is restarted;
            // the request stays posted and is answered by the new one.
            if (cudaStreamQuery(e.stream) != cudaErrorNotReady) {
                cudaGetLastError();
                if (!checked(cudaStreamSynchronize(e.stream), "latency engine", err) ||
                    !engine_launch(f, e, seq - 1, err)) {
                    return kEngineFailed;
                }
            }
        }
        std::this_thread::yield();
    }
    std::atomic_thread_fence(std::memory_order_acquire);
    for (size_t r = 0; r < batch; ++r) out[r] = answers[r].value;
    return 0;
}

}  // namespace mlk::cuda
