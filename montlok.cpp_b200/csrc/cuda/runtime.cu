// Host side of the CUDA layer: device replicas of a forest, per-thread
// workspaces (streams, device buffers, pinned staging) and the pipelined
// host-buffer predict behind montlok_model_predict.
//
// Host-buffer calls split the rows into chunks and alternate two streams:
// while one chunk's kernel runs, the next chunk's input is copied host ->
// device on the other stream (straight from the caller's memory when it is
// pinned, else through a pinned staging buffer) and the previous chunk's
// results come back device -> host. Pageable float64 rows of a model that
// casts its features to float32 (and has no preprocessing) are rounded to
// float32 while they are staged, halving the bytes on the bus. Staging runs
// on a pool of host threads. Each calling thread has its own workspace per
// device, so concurrent calls on one model never share buffers.
//
// MONTLOK_FAULT_INJECT=alloc|copy|launch makes the next device allocation,
// copy or launch of a call fail as if CUDA had failed; tests use it to check
// that failures surface as MONTLOK_ERROR_INTERNAL with a message.
// MONTLOK_FAULT_INJECT=wait launches the kernels with their tree copies
// switched off and a 2 ms wait limit, so every wait on a copy runs out: the
// kernels give up cleanly (no copy is in flight) and set the call's status
// word, which the host reports as MONTLOK_ERROR_INTERNAL.
#include <algorithm>
#include <atomic>
#include <cfenv>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <functional>
#include <map>
#include <mutex>
#include <memory>
#include <string>
#include <thread>
#include <type_traits>
#include <vector>

#include "async_copy.cuh"
#include "engine.cuh"
#include "forest.cuh"
#include "mlk_cuda.h"

namespace mlk::cuda {
namespace {

constexpr int kInternal = 7;
constexpr int kInvalid = 1;
constexpr size_t kChunkBytes = size_t{64} << 20;  // input bytes per pipelined chunk

std::atomic<int> g_copy_threads{0};  // 0: every hardware thread
std::atomic<int> g_latency_engine{0};  // nonzero: small host calls go to the calling thread's latency engine

int copy_threads() {
    const int n = g_copy_threads.load(std::memory_order_relaxed);
    return std::max(1, n > 0 ? n : static_cast<int>(std::thread::hardware_concurrency()));
}

void put_error(char* err, size_t errlen, const std::string& message) {
    if (!err || errlen == 0) return;
    const size_t n = std::min(errlen - 1, message.size());
    std::memcpy(err, message.data(), n);
    err[n] = '\0';
}

bool injected(const char* what) {
    const char* v = std::getenv("MONTLOK_FAULT_INJECT");
    return v && std::strcmp(v, what) == 0;
}

constexpr unsigned long long kInjectedWaitNs = 2000000ull;

// The kernel arguments of one call: the forest's, with the call's status
// word and, under MONTLOK_FAULT_INJECT=wait, no tree copies and a short wait.
DevForest call_forest(const DevForest& f, int* status, bool fault_wait) {
    DevForest g = f;
    g.args.status = status;
    if (fault_wait) {
        g.args.skip_copies = 1;
        g.args.wait_ns = kInjectedWaitNs;
    }
    return g;
}

bool ok(cudaError_t e, const char* what, std::string& err) {
    if (e == cudaSuccess) return true;
    err = std::string(what) + " failed: " + cudaGetErrorString(e);
    cudaGetLastError();
    return false;
}

// Restores the calling thread's current device on scope exit.
class DeviceGuard {
public:
    explicit DeviceGuard(int device) {
        if (cudaGetDevice(&previous_) != cudaSuccess) previous_ = -1;
        if (previous_ != device) cudaSetDevice(device);
    }
    ~DeviceGuard() {
        int now = -1;
        if (previous_ >= 0 && cudaGetDevice(&now) == cudaSuccess && now != previous_) cudaSetDevice(previous_);
    }

private:
    int previous_ = -1;
};

bool device_alloc(void** p, size_t bytes, std::string& err) {
    if (injected("alloc")) {
        err = "cudaMalloc failed: injected fault (MONTLOK_FAULT_INJECT=alloc)";
        return false;
    }
    return ok(cudaMalloc(p, bytes), "cudaMalloc", err);
}

bool host_alloc(void** p, size_t bytes, std::string& err) {
    if (injected("alloc")) {
        err = "cudaMallocHost failed: injected fault (MONTLOK_FAULT_INJECT=alloc)";
        return false;
    }
    return ok(cudaMallocHost(p, bytes), "cudaMallocHost", err);
}

bool copy_async(void* dst, const void* src, size_t bytes, cudaMemcpyKind kind, cudaStream_t s, std::string& err) {
    if (bytes == 0) return true;
    if (injected("copy")) {
        err = "cudaMemcpyAsync failed: injected fault (MONTLOK_FAULT_INJECT=copy)";
        return false;
    }
    return ok(cudaMemcpyAsync(dst, src, bytes, kind, s), "cudaMemcpyAsync", err);
}

// Host worker threads for staging: a job is split into parts that the pool's
// threads and the calling thread take one at a time, and the caller returns
// when every part is done. Several callers (one per device) share the pool;
// since callers work on their own jobs too, a job finishes even if no worker
// is free (or, after a fork, none exists). Workers start from the default
// floating-point environment (round to nearest, no flush to zero).
class HostPool {
public:
    static HostPool& get() {
        static HostPool* pool = new HostPool();  // never destroyed: workers may be blocked at exit
        return *pool;
    }

    void run(size_t parts, const std::function<void(size_t)>& fn) {
        if (parts <= 1) {
            if (parts == 1) fn(0);
            return;
        }
        auto job = std::make_shared<Job>();
        job->fn = &fn;
        job->parts = parts;
        {
            std::lock_guard<std::mutex> lock(mu_);
            jobs_.push_back(job);
        }
        cv_.notify_all();
        work(*job);
        std::unique_lock<std::mutex> lock(mu_);
        done_cv_.wait(lock, [&] { return job->done.load() == job->parts; });
    }

private:
    struct Job {
        const std::function<void(size_t)>* fn = nullptr;
        size_t parts = 0;
        std::atomic<size_t> next{0};
        std::atomic<size_t> done{0};
    };

    HostPool() {
        const unsigned n = std::max(1u, std::thread::hardware_concurrency()) - 1;
        for (unsigned i = 0; i < std::min(n, 255u); ++i) std::thread([this] { loop(); }).detach();
    }

    // Takes parts of `job` until none is left.
    void work(Job& job) {
        for (size_t i; (i = job.next.fetch_add(1)) < job.parts;) {
            (*job.fn)(i);
            if (job.done.fetch_add(1) + 1 == job.parts) {
                std::lock_guard<std::mutex> lock(mu_);
                done_cv_.notify_all();
            }
        }
    }

    void loop() {
        std::fesetenv(FE_DFL_ENV);
        for (;;) {
            std::shared_ptr<Job> job;
            {
                std::unique_lock<std::mutex> lock(mu_);
                cv_.wait(lock, [&] {
                    while (!jobs_.empty() && jobs_.front()->next.load() >= jobs_.front()->parts) jobs_.pop_front();
                    return !jobs_.empty();
                });
                job = jobs_.front();
            }
            work(*job);
        }
    }

    std::mutex mu_;
    std::condition_variable cv_, done_cv_;
    std::deque<std::shared_ptr<Job>> jobs_;
};

// Splits [0, n) into at most copy_threads() ranges of at least `grain` and
// runs fn(lo, hi) on each through the pool.
void host_parallel(size_t n, size_t grain, const std::function<void(size_t, size_t)>& fn) {
    const size_t parts = std::min<size_t>(static_cast<size_t>(copy_threads()), std::max<size_t>(1, n / grain));
    const size_t step = (n + parts - 1) / parts;
    HostPool::get().run(parts, [&](size_t i) {
        const size_t lo = i * step, hi = std::min(n, lo + step);
        if (lo < hi) fn(lo, hi);
    });
}

// memcpy split over the worker threads for large blocks.
void host_copy(void* dst, const void* src, size_t bytes) {
    host_parallel(bytes, size_t{4} << 20, [&](size_t lo, size_t hi) {
        std::memcpy(static_cast<char*>(dst) + lo, static_cast<const char*>(src) + lo, hi - lo);
    });
}

// dst[i] = (float)src[i] for n values, split over the worker threads.
void host_narrow(float* dst, const double* src, size_t n) {
    host_parallel(n, size_t{512} << 10, [&](size_t lo, size_t hi) {
        for (size_t i = lo; i < hi; ++i) dst[i] = static_cast<float>(src[i]);
    });
}

// Whether this thread converts double to float as the kernels' cast does:
// round to nearest even, subnormal results kept (no flush to zero).
bool narrowing_exact() {
    volatile double up = 1.0 + 0x3p-25, down = 1.0 + 0x1p-25, tiny = 1e-40;
    return static_cast<float>(up) == 1.0f + 0x1p-23f && static_cast<float>(down) == 1.0f &&
           static_cast<float>(tiny) != 0.0f && static_cast<float>(-static_cast<double>(up)) == -(1.0f + 0x1p-23f);
}

// A device buffer that only grows; zeroed when (re)allocated, which the
// small-batch kernel's self-resetting counters rely on.
struct DeviceBuffer {
    void* p = nullptr;
    size_t cap = 0;
    bool reserve(size_t bytes, std::string& err) {
        if (bytes <= cap) return true;
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
        if (!device_alloc(&p, bytes, err) || !ok(cudaMemset(p, 0, bytes), "cudaMemset", err)) return false;
        cap = bytes;
        return true;
    }
    ~DeviceBuffer() {
        if (p) cudaFree(p);
    }
};

struct PinnedBuffer {
    void* p = nullptr;
    size_t cap = 0;
    bool reserve(size_t bytes, std::string& err) {
        if (bytes <= cap) return true;
        if (p) cudaFreeHost(p);
        p = nullptr;
        cap = 0;
        if (!host_alloc(&p, bytes, err)) return false;
        cap = bytes;
        return true;
    }
    ~PinnedBuffer() {
        if (p) cudaFreeHost(p);
    }
};

// A small host-buffer predict captured as a CUDA graph (input copy, kernel,
// output copy) for one forest, input type and row count, over the buffers
// it was captured with.
struct CachedGraph {
    unsigned long long forest = 0;
    int dtype = 0;
    size_t batch = 0;
    const void* buffers[5] = {};
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    cudaGraphNode_t input_copy = nullptr;  // the host -> device copy, re-pointed at pinned caller inputs
    const void* input = nullptr;           // where that copy reads now
    unsigned long long used = 0;
};

constexpr size_t kCounterBytes = 2 * kLatencyCounters * sizeof(int);  // a workspace's counters: one block per stream

struct Workspace {
    cudaStream_t stream[2] = {nullptr, nullptr};
    // The status word of this thread's host calls (mapped pinned memory): the
    // kernels set it when a wait on their tree copies runs out; cleared
    // before every call and read after it.
    int* status_host = nullptr;
    int* status_dev = nullptr;
    DeviceBuffer dx[2], dout[2], scratch;
    // The small-batch kernel's counters, one block of kLatencyCounters per
    // stream: zero between launches, nothing else uses them. Always this
    // size (never reallocated), since cached graphs hold its address.
    DeviceBuffer counters;
    PinnedBuffer hx[2], hout[2];
    std::vector<CachedGraph> graphs;
    unsigned long long tick = 0;
    LatencyEngine* engine = nullptr;  // this thread's resident small-call kernel, when latency threads are on
    ~Workspace() {
        destroy_engine(engine);
        for (auto& g : graphs) {
            if (g.exec) cudaGraphExecDestroy(g.exec);
            if (g.graph) cudaGraphDestroy(g.graph);
        }
        for (auto s : stream) {
            if (s) cudaStreamDestroy(s);
        }
        if (status_host) cudaFreeHost(status_host);
    }
};

Workspace* workspace(int device, std::string& err) {
    thread_local std::map<int, std::unique_ptr<Workspace>> spaces;
    auto& w = spaces[device];
    if (!w) {
        auto fresh = std::make_unique<Workspace>();
        for (auto& s : fresh->stream) {
            if (!ok(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate", err)) return nullptr;
        }
        void* word = nullptr;
        if (!ok(cudaHostAlloc(&word, sizeof(int), cudaHostAllocMapped), "cudaHostAlloc", err)) return nullptr;
        fresh->status_host = static_cast<int*>(word);
        *fresh->status_host = 0;
        if (!ok(cudaHostGetDevicePointer(reinterpret_cast<void**>(&fresh->status_dev), word, 0),
                "cudaHostGetDevicePointer", err)) {
            return nullptr;
        }
        w = std::move(fresh);
    }
    return w.get();
}

constexpr size_t kGraphRows = 4096;  // host-buffer predicts of at most this many rows replay a graph
constexpr size_t kGraphCache = 8;    // graphs kept per workspace

// A predict of at most kGraphRows rows from and to host memory: the input is
// copied into the workspace's pinned staging buffer (or, when the caller's
// input is pinned already, the graph's copy reads it in place), a cached
// graph of (host -> device copy, kernel) runs on the workspace's first
// stream, the kernel storing its results into pinned host memory directly,
// and the result is copied out. When the small-batch kernel runs in its
// cluster form with one CTA reading the rows (latency_form 2), the kernel
// reads them straight from the pinned staging buffer and the graph is one
// kernel node. (The counter form reading them over the bus from every CTA
// was slower than the copy: 21.5 and 30.6 us against 18.1 and 22.1 for 1 and
// 8 rows.) The graph is captured on the first call with this forest, input
// type and row count (or after a staging buffer grew), so later calls of the
// same shape pay one graph launch instead of separate stream operations and
// kernel launches.
int run_small(const DevForest& base, int dtype, const void* x, int x_kind, size_t batch, double* out, char* err,
              size_t errlen) {
    std::string e;
    DeviceGuard guard(base.device);
    Workspace* w = workspace(base.device, e);
    if (!w) {
        put_error(err, errlen, e);
        return kInternal;
    }
    const bool fault_wait = injected("wait");
    const DevForest f = call_forest(base, w->status_dev, fault_wait);
    *reinterpret_cast<volatile int*>(w->status_host) = 0;
    const size_t in_bytes = batch * static_cast<size_t>(f.args.F) * (dtype == 1 ? 4 : 8);
    const size_t out_bytes = batch * static_cast<size_t>(f.args.K) * sizeof(double);
    const size_t scratch = scratch_bytes(f, static_cast<long long>(batch));
    if (!w->counters.reserve(kCounterBytes, e) || !w->dx[0].reserve(in_bytes, e) ||
        !w->hx[0].reserve(in_bytes, e) ||
        !w->hout[0].reserve(out_bytes, e) || (scratch && !w->scratch.reserve(scratch, e))) {
        put_error(err, errlen, e);
        return kInternal;
    }
    cudaStream_t st = w->stream[0];
    // No copy when the kernel's first CTA reads the rows from the pinned
    // staging buffer over the bus: the graph is one kernel node.
    const bool direct = latency_form(f, dtype, static_cast<long long>(batch)) == 2;
    const void* kernel_x = direct ? w->hx[0].p : w->dx[0].p;
    const void* buffers[5] = {w->dx[0].p, nullptr, w->hx[0].p, w->hout[0].p, scratch ? w->scratch.p : nullptr};
    CachedGraph* g = nullptr;
    for (auto& c : w->graphs) {
        if (c.forest == f.uid && c.dtype == dtype && c.batch == batch && std::equal(buffers, buffers + 5, c.buffers)) {
            g = &c;
        }
    }
    if (fault_wait) {
        // The injected launch is never cached: run it on the stream directly.
        std::memcpy(w->hx[0].p, x, in_bytes);
        bool good = copy_async(w->dx[0].p, w->hx[0].p, in_bytes, cudaMemcpyHostToDevice, st, e) &&
                    launch_forest(f, dtype, w->dx[0].p, static_cast<long long>(batch),
                                  static_cast<double*>(w->hout[0].p), nullptr, st, e,
                                  scratch ? static_cast<int*>(w->scratch.p) : nullptr,
                                  static_cast<int*>(w->counters.p)) &&
                    ok(cudaStreamSynchronize(st), "cudaStreamSynchronize", e);
        if (good && *reinterpret_cast<volatile int*>(w->status_host) != 0) {
            e = "a predict kernel gave up waiting for its tree data (bounded wait ran out)";
            good = false;
        }
        if (!good) {
            put_error(err, errlen, e);
            return kInternal;
        }
        std::memcpy(out, w->hout[0].p, out_bytes);
        return 0;
    }
    if (!g) {
        bool good = ok(cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed), "cudaStreamBeginCapture", e);
        if (good) {
            good = direct || copy_async(w->dx[0].p, w->hx[0].p, in_bytes, cudaMemcpyHostToDevice, st, e);
            if (good && injected("launch")) {
                e = "kernel launch failed: injected fault (MONTLOK_FAULT_INJECT=launch)";
                good = false;
            }
            // The kernel stores the results straight into the pinned staging
            // buffer (host memory the device addresses directly).
            good = good && launch_forest(f, dtype, kernel_x, static_cast<long long>(batch),
                                         static_cast<double*>(w->hout[0].p), nullptr, st, e,
                                         scratch ? static_cast<int*>(w->scratch.p) : nullptr,
                                         static_cast<int*>(w->counters.p));
            cudaGraph_t graph = nullptr;
            const cudaError_t end = cudaStreamEndCapture(st, &graph);
            if (good) good = ok(end, "cudaStreamEndCapture", e);
            cudaGraphExec_t exec = nullptr;
            if (good) good = ok(cudaGraphInstantiate(&exec, graph, 0), "cudaGraphInstantiate", e);
            cudaGraphNode_t input_copy = nullptr;
            if (good) {
                size_t n = 0;
                cudaGraphGetNodes(graph, nullptr, &n);
                std::vector<cudaGraphNode_t> nodes(n);
                if (n && cudaGraphGetNodes(graph, nodes.data(), &n) == cudaSuccess) {
                    for (auto node : nodes) {
                        cudaGraphNodeType type;
                        if (cudaGraphNodeGetType(node, &type) == cudaSuccess && type == cudaGraphNodeTypeMemcpy) {
                            input_copy = node;
                        }
                    }
                }
            }
            cudaGetLastError();
            if (good) {
                if (w->graphs.size() >= kGraphCache) {
                    auto oldest = std::min_element(w->graphs.begin(), w->graphs.end(),
                                                   [](const CachedGraph& a, const CachedGraph& b) { return a.used < b.used; });
                    cudaGraphExecDestroy(oldest->exec);
                    cudaGraphDestroy(oldest->graph);
                    w->graphs.erase(oldest);
                }
                CachedGraph c;
                c.forest = f.uid;
                c.dtype = dtype;
                c.batch = batch;
                std::copy(buffers, buffers + 5, c.buffers);
                c.graph = graph;
                c.exec = exec;
                c.input_copy = input_copy;
                c.input = w->hx[0].p;
                w->graphs.push_back(c);
                g = &w->graphs.back();
            } else if (graph) {
                cudaGraphDestroy(graph);
            }
        }
        if (!good) {
            put_error(err, errlen, e);
            return kInternal;
        }
    }
    g->used = ++w->tick;
    const void* src = (x_kind == MLK_PTR_PINNED && g->input_copy) ? x : w->hx[0].p;
    if (src != g->input) {
        if (!ok(cudaGraphExecMemcpyNodeSetParams1D(g->exec, g->input_copy, w->dx[0].p, src, in_bytes,
                                                   cudaMemcpyHostToDevice),
                "cudaGraphExecMemcpyNodeSetParams1D", e)) {
            put_error(err, errlen, e);
            return kInternal;
        }
        g->input = src;
    }
    if (src != x) std::memcpy(w->hx[0].p, x, in_bytes);
    bool good = ok(cudaGraphLaunch(g->exec, st), "cudaGraphLaunch", e) &&
                ok(cudaStreamSynchronize(st), "cudaStreamSynchronize", e);
    if (good) std::memcpy(out, w->hout[0].p, out_bytes);
    if (good && *reinterpret_cast<volatile int*>(w->status_host) != 0) {
        e = "a predict kernel gave up waiting for its tree data (bounded wait ran out)";
        good = false;
    }
    if (!good) {
        put_error(err, errlen, e);
        return kInternal;
    }
    return 0;
}

// A pending chunk whose results sit in a pinned staging buffer.
struct Pending {
    bool live = false;
    size_t bytes = 0;
    void* dst = nullptr;
};

template <typename Out>
int run_host(const DevForest& base, int dtype, const void* x, size_t batch, Out* out, size_t out_per_row,
             bool leaves, char* err, size_t errlen) {
    std::string e;
    DeviceGuard guard(base.device);
    Workspace* w = workspace(base.device, e);
    if (!w) {
        put_error(err, errlen, e);
        return kInternal;
    }
    const DevForest f = call_forest(base, w->status_dev, injected("wait"));
    *reinterpret_cast<volatile int*>(w->status_host) = 0;
    const size_t elem = dtype == 1 ? 4 : 8;
    const size_t row_in = static_cast<size_t>(f.args.F) * elem;
    const size_t row_out = out_per_row * sizeof(Out);
    size_t chunk = std::max<size_t>(1024, kChunkBytes / std::max<size_t>(row_in, 1));
    chunk = std::min(chunk, batch);

    int kx = MLK_PTR_PAGEABLE, ko = MLK_PTR_PAGEABLE, dev = -1;
    mlk_cuda_pointer_kind(x, &kx, &dev);
    mlk_cuda_pointer_kind(out, &ko, &dev);
    const bool pin_x = kx == MLK_PTR_PINNED, pin_out = ko == MLK_PTR_PINNED;
    const bool dev_x = kx == MLK_PTR_DEVICE, dev_out = ko == MLK_PTR_DEVICE;
    if constexpr (std::is_same_v<Out, double>) {
        if (!leaves && !dev_x && !dev_out && batch <= static_cast<size_t>(kEngineRows)) {
            if (g_latency_engine.load(std::memory_order_relaxed) > 0) {
                const int served = engine_predict(base, w->engine, dtype, x, batch, out, e);
                if (served == 0) return 0;
                if (served != -1) {
                    put_error(err, errlen, e);
                    return kInternal;
                }
            } else if (w->engine) {
                destroy_engine(w->engine);  // latency threads were turned off: release the SMs
                w->engine = nullptr;
            }
        }
        if (!leaves && batch <= kGraphRows && !dev_x && !dev_out) {
            return run_small(base, dtype, x, kx, batch, out, err, errlen);
        }
    }
    // A model that casts features to float32 and has no preprocessing uses
    // only the float32 value of each double (trees.cpp:275), so pageable rows
    // are rounded to float32 while they are staged: the staging writes and
    // the bytes on the bus halve, and the float-input kernels give the same
    // bits. Pinned rows go to the device as they are: the bus reads them as
    // fast as the host threads would convert them.
    const bool narrow = dtype == 2 && !dev_x && !pin_x && f.args.cast_f32 && !f.args.standardize && !f.args.clip &&
                        narrowing_exact();
    const int kernel_dtype = narrow ? 1 : dtype;
    const size_t row_dev = narrow ? static_cast<size_t>(f.args.F) * 4 : row_in;

    // Chunks are `chunk` rows but the last one, which may take another kernel.
    // The two streams' kernels may run at the same time, so each stream has
    // its own half of the scratch (key tables, small-batch sums) and of the
    // counters.
    const size_t tail = batch % chunk;
    const size_t scratch = (std::max(scratch_bytes(f, static_cast<long long>(chunk)),
                                     tail ? scratch_bytes(f, static_cast<long long>(tail)) : size_t{0}) +
                            255) & ~size_t{255};
    if ((scratch && !w->scratch.reserve(2 * scratch, e)) || !w->counters.reserve(kCounterBytes, e)) {
        put_error(err, errlen, e);
        return kInternal;
    }
    for (int s = 0; s < 2; ++s) {
        if ((!dev_x && !w->dx[s].reserve(chunk * row_dev, e)) || (!dev_out && !w->dout[s].reserve(chunk * row_out, e)) ||
            (!dev_x && !pin_x && !w->hx[s].reserve(chunk * row_dev, e)) ||
            (!dev_out && !pin_out && !w->hout[s].reserve(chunk * row_out, e))) {
            put_error(err, errlen, e);
            return kInternal;
        }
    }
    Pending pending[2];
    auto drain = [&](int s) -> bool {
        if (!pending[s].live) return true;
        if (!ok(cudaStreamSynchronize(w->stream[s]), "cudaStreamSynchronize", e)) return false;
        std::memcpy(pending[s].dst, w->hout[s].p, pending[s].bytes);
        pending[s].live = false;
        return true;
    };
    bool good = true;
    size_t c = 0;
    for (size_t r0 = 0; r0 < batch && good; r0 += chunk, ++c) {
        const int s = static_cast<int>(c & 1);
        const size_t rows = std::min(chunk, batch - r0);
        cudaStream_t st = w->stream[s];
        // The staging buffers of stream s are reused: wait for its last chunk.
        if (pending[s].live) {
            good = drain(s);
        } else if (c >= 2 && !pin_x && !dev_x) {
            good = ok(cudaStreamSynchronize(st), "cudaStreamSynchronize", e);
        }
        if (!good) break;
        const char* src = static_cast<const char*>(x) + r0 * row_in;
        const void* dsrc = src;
        if (!dev_x) {
            if (narrow) {
                host_narrow(static_cast<float*>(w->hx[s].p), reinterpret_cast<const double*>(src), rows * f.args.F);
                src = static_cast<const char*>(w->hx[s].p);
            } else if (!pin_x) {
                host_copy(w->hx[s].p, src, rows * row_in);
                src = static_cast<const char*>(w->hx[s].p);
            }
            good = copy_async(w->dx[s].p, src, rows * row_dev, cudaMemcpyHostToDevice, st, e);
            dsrc = w->dx[s].p;
        }
        if (!good) break;
        void* dst_dev = dev_out ? static_cast<void*>(out + r0 * out_per_row) : w->dout[s].p;
        if (injected("launch")) {
            e = "kernel launch failed: injected fault (MONTLOK_FAULT_INJECT=launch)";
            good = false;
            break;
        }
        int* own_scratch = scratch ? reinterpret_cast<int*>(static_cast<char*>(w->scratch.p) + s * scratch) : nullptr;
        good = launch_forest(f, kernel_dtype, dsrc, static_cast<long long>(rows), leaves ? nullptr : static_cast<double*>(dst_dev),
                             leaves ? static_cast<int*>(dst_dev) : nullptr, st, e, own_scratch,
                             static_cast<int*>(w->counters.p) + s * kLatencyCounters);
        if (!good) break;
        if (!dev_out) {
            if (pin_out) {
                good = copy_async(out + r0 * out_per_row, dst_dev, rows * row_out, cudaMemcpyDeviceToHost, st, e);
            } else {
                good = copy_async(w->hout[s].p, dst_dev, rows * row_out, cudaMemcpyDeviceToHost, st, e);
                pending[s] = Pending{true, rows * row_out, out + r0 * out_per_row};
            }
        }
    }
    for (int s = 0; s < 2; ++s) {
        if (good) good = drain(s);
        if (good) good = ok(cudaStreamSynchronize(w->stream[s]), "cudaStreamSynchronize", e);
        else cudaStreamSynchronize(w->stream[s]);
    }
    if (good && *reinterpret_cast<volatile int*>(w->status_host) != 0) {
        e = "a predict kernel gave up waiting for its tree data (bounded wait ran out)";
        good = false;
    }
    if (!good) {
        put_error(err, errlen, e);
        return kInternal;
    }
    return 0;
}

// Builds and uploads the deep-tree records of `v` into f.deep (left unset
// when the record or leaf numbers do not fit 31 bits). A record is a split,
// its two children's split words and the four exits below them, so one
// 32-byte load decides two levels; a child that is a leaf gets the pad word
// (never goes right) and both its exits name it. Records are laid out tree by
// tree in breadth-first order. False only on a CUDA error.
bool upload_deep(const mlk_forest_view* v, DevForest& f, std::string& e) {
    const int T = v->trees;
    const int slot_bits = heap_slot_bits(v->slots);
    const uint32_t mask = (1u << slot_bits) - 1u;
    const uint32_t pad = static_cast<uint32_t>(v->pad_slot);
    constexpr uint32_t kLeaf = 0x80000000u;
    constexpr size_t kMaxRecords = size_t{1} << 26;  // 2 GB; shared subtrees unfolded further use the generic kernel
    std::vector<uint32_t> words;  // 8 per record
    std::vector<int32_t> ids;     // 3 per record: file node of the top, left and right split, -1 for none
    std::vector<int32_t> queue;   // file node at the top of each record
    std::vector<int32_t> level;   // record steps from the tree's root to each record
    std::vector<uint32_t> roots(static_cast<size_t>(T));
    std::vector<int32_t> steps(static_cast<size_t>(T), 0);
    std::vector<double> leaves;
    bool f32 = true, fits = true;
    auto split_word = [&](int node) {
        const int32_t* w = &v->node_words[static_cast<size_t>(node) * 4];
        return (static_cast<uint32_t>(w[0]) & ~mask) | static_cast<uint32_t>(w[1]);
    };
    // The exit to `node` from a record `depth` steps below the root.
    auto exit_to = [&](int node, int depth, int32_t& need) -> uint32_t {
        if (v->feature[node] >= 0) {
            const size_t r = queue.size();
            if (r >= kMaxRecords) fits = false;
            queue.push_back(node);
            level.push_back(depth);
            return static_cast<uint32_t>(r);
        }
        need = std::max(need, depth);
        const size_t leaf = leaves.size();
        if (leaf >= kLeaf) fits = false;
        const double value = v->leaf_value[node];
        leaves.push_back(value);
        f32 = f32 && static_cast<double>(static_cast<float>(value)) == value;
        return kLeaf | static_cast<uint32_t>(leaf);
    };
    for (int t = 0; t < T && fits; ++t) {
        int32_t& need = steps[static_cast<size_t>(t)];
        size_t i = queue.size();
        roots[static_cast<size_t>(t)] = exit_to(v->roots[t], 0, need);
        for (; i < queue.size() && fits; ++i) {
            const int a = queue[i];
            const int depth = level[i] + 1;
            const int32_t* wa = &v->node_words[static_cast<size_t>(a) * 4];
            uint32_t rec[8] = {split_word(a), pad, pad, 0u, 0u, 0u, 0u, 0u};
            int32_t id[3] = {a, -1, -1};
            for (int side = 0; side < 2; ++side) {
                const int c = wa[2 + side];
                if (v->feature[c] >= 0) {
                    const int32_t* wc = &v->node_words[static_cast<size_t>(c) * 4];
                    rec[1 + side] = split_word(c);
                    id[1 + side] = c;
                    rec[4 + 2 * side] = exit_to(wc[2], depth, need);
                    rec[5 + 2 * side] = exit_to(wc[3], depth, need);
                } else {
                    rec[4 + 2 * side] = rec[5 + 2 * side] = exit_to(c, depth, need);
                }
            }
            words.insert(words.end(), rec, rec + 8);
            ids.insert(ids.end(), id, id + 3);
        }
    }
    if (!fits) return true;
    std::vector<float> leaves32;
    if (f32) leaves32.assign(leaves.begin(), leaves.end());
    const size_t leaf_bytes = f32 ? leaves32.size() * 4 : leaves.size() * 8;
    const void* leaf_src = f32 ? static_cast<const void*>(leaves32.data()) : static_cast<const void*>(leaves.data());
    void* dnodes = nullptr;
    void* dleaves = nullptr;
    void* droots = nullptr;
    void* dsteps = nullptr;
    void* dids = nullptr;
    const size_t word_bytes = words.size() * 4, id_bytes = ids.size() * 4;
    if (!device_alloc(&dnodes, std::max<size_t>(word_bytes, 32), e) ||
        !ok(cudaMemcpy(dnodes, words.data(), word_bytes, cudaMemcpyHostToDevice), "cudaMemcpy", e) ||
        !device_alloc(&dleaves, std::max<size_t>(leaf_bytes, 16), e) ||
        !ok(cudaMemcpy(dleaves, leaf_src, leaf_bytes, cudaMemcpyHostToDevice), "cudaMemcpy", e) ||
        !device_alloc(&droots, roots.size() * 4, e) ||
        !ok(cudaMemcpy(droots, roots.data(), roots.size() * 4, cudaMemcpyHostToDevice), "cudaMemcpy", e) ||
        !device_alloc(&dsteps, steps.size() * 4, e) ||
        !ok(cudaMemcpy(dsteps, steps.data(), steps.size() * 4, cudaMemcpyHostToDevice), "cudaMemcpy", e) ||
        !device_alloc(&dids, std::max<size_t>(id_bytes, 16), e) ||
        !ok(cudaMemcpy(dids, ids.data(), id_bytes, cudaMemcpyHostToDevice), "cudaMemcpy", e)) {
        for (void* p : {dnodes, dleaves, droots, dsteps, dids}) {
            if (p) cudaFree(p);
        }
        return false;
    }
    for (void* p : {dnodes, dleaves, droots, dsteps, dids}) f.blocks[f.nblocks++] = p;
    DeepArgs& d = f.deep;
    d.slot_bits = slot_bits;
    d.leaf32 = f32;
    d.records = static_cast<const uint32_t*>(dnodes);
    d.leaves = dleaves;
    d.roots = static_cast<const uint32_t*>(droots);
    d.steps = static_cast<const int*>(dsteps);
    d.node_ids = static_cast<const int*>(dids);
    return true;
}

// Builds and uploads the multi-output records of `v` into f.sparse (left
// unset, teams 0, when the model does not fit the kernel). A split reads the
// key of (feature, missing kind): kind 1 for LightGBM's zero missing type,
// kind 0 otherwise; missing values go right (c = 1) for the NaN-right and
// zero-right variants. False only on a CUDA error.
bool upload_sparse(const mlk_forest_view* v, DevForest& f, std::string& e) {
    const int F = v->features, K = v->outputs, T = v->trees;
    // Variant slot -> (feature, variant).
    std::vector<int> slot_feature(static_cast<size_t>(v->slots), -1), slot_variant(static_cast<size_t>(v->slots), -1);
    for (int feat = 0; feat < F; ++feat) {
        for (int var = 0; var < 4; ++var) {
            const int s = v->slot_of[feat * 4 + var];
            if (s >= 0) {
                slot_feature[static_cast<size_t>(s)] = feat;
                slot_variant[static_cast<size_t>(s)] = var;
            }
        }
    }
    // (feature, kind) slots in kind-major order, then the pad slot.
    std::vector<int2> slot_of(static_cast<size_t>(F), make_int2(-1, -1));
    int slots = 0;
    for (int kind = 0; kind < 2; ++kind) {
        for (int feat = 0; feat < F; ++feat) {
            bool used = false;
            for (int var = 2 * kind; var < 2 * kind + 2; ++var) used = used || v->slot_of[feat * 4 + var] >= 0;
            if (used) (kind ? slot_of[static_cast<size_t>(feat)].y : slot_of[static_cast<size_t>(feat)].x) = slots++;
        }
    }
    const int pad = slots++;
    const int slot_bits = heap_slot_bits(2 * slots);
    const uint32_t mask = (1u << slot_bits) - 1u;
    // Breadth-first layout of every tree, children of a split adjacent.
    struct Laid {
        std::vector<int32_t> order;  // file node of each position
        std::vector<int32_t> rel;    // positions to the left child, 0 for leaves
        int leaves = 0;
    };
    std::vector<Laid> laid(static_cast<size_t>(T));
    int node_max = 1, leaf_max = 1;
    bool f32 = true;
    constexpr size_t kMaxNodes = 1 << 16;
    for (int t = 0; t < T; ++t) {
        Laid& l = laid[static_cast<size_t>(t)];
        l.order.push_back(v->roots[t]);
        for (size_t i = 0; i < l.order.size(); ++i) {
            const int node = l.order[i];
            if (v->feature[node] >= 0) {
                l.rel.push_back(static_cast<int32_t>(l.order.size() - i));
                l.order.push_back(v->node_words[static_cast<size_t>(node) * 4 + 2]);
                l.order.push_back(v->node_words[static_cast<size_t>(node) * 4 + 3]);
                if (l.order.size() > kMaxNodes) return true;  // shared subtrees unfolded too far: no sparse view
            } else {
                l.rel.push_back(0);
                ++l.leaves;
                const double value = v->leaf_value[node];
                f32 = f32 && static_cast<double>(static_cast<float>(value)) == value;
            }
        }
        node_max = std::max(node_max, static_cast<int>(l.order.size()));
        leaf_max = std::max(leaf_max, l.leaves);
    }
    if (static_cast<uint64_t>(leaf_max + 1) >= (uint64_t{1} << (32 - slot_bits))) return true;
    const int record = (16 + node_max * 8 + leaf_max * (f32 ? 4 : 8) + 15) & ~15;
    int rows = 0;
    if (!sparse_plan(slots, K, record, rows)) return true;
    // Records output by output, each list padded to whole chunks.
    const int chunk = sparse_chunk_trees();
    std::vector<std::vector<int>> lists(static_cast<size_t>(K));
    for (int t = 0; t < T; ++t) lists[static_cast<size_t>(v->tree_output[t])].push_back(t);
    SparseArgs& s = f.sparse;
    int records = 0;
    for (int k = 0; k < K; ++k) {
        s.offset[k] = records;
        const int n = static_cast<int>(lists[static_cast<size_t>(k)].size());
        s.chunks[k] = (n + chunk - 1) / chunk;
        records += s.chunks[k] * chunk;
    }
    std::vector<unsigned char> host(static_cast<size_t>(records) * record, 0);
    std::vector<int32_t> ids(static_cast<size_t>(records) * node_max, -1);
    const uint32_t leaf_low = static_cast<uint32_t>(pad) << 1;
    for (int k = 0; k < K; ++k) {
        const auto& list = lists[static_cast<size_t>(k)];
        for (int j = 0; j < s.chunks[k] * chunk; ++j) {
            const size_t at = static_cast<size_t>(s.offset[k] + j);
            unsigned char* rec = host.data() + at * record;
            int32_t* hdr = reinterpret_cast<int32_t*>(rec);
            uint32_t* nodes = reinterpret_cast<uint32_t*>(rec + 16);
            unsigned char* leaves = rec + 16 + static_cast<size_t>(node_max) * 8;
            if (j >= static_cast<int>(list.size())) {  // inert: one leaf of 0.0, never added
                nodes[0] = (1u << slot_bits) | leaf_low;
                continue;
            }
            const int t = list[static_cast<size_t>(j)];
            const Laid& l = laid[static_cast<size_t>(t)];
            hdr[0] = t / 64;
            hdr[1] = v->depth[t];
            hdr[2] = 1;
            int leaf = 0;
            for (size_t i = 0; i < l.order.size(); ++i) {
                const int node = l.order[i];
                if (v->feature[node] >= 0) {
                    const int32_t* w = &v->node_words[static_cast<size_t>(node) * 4];
                    const int var = slot_variant[static_cast<size_t>(w[1])];
                    const int feat = slot_feature[static_cast<size_t>(w[1])];
                    const int2 fs = slot_of[static_cast<size_t>(feat)];
                    const int sl = var >= 2 ? fs.y : fs.x;
                    const uint32_t c = (var == 0 || var == 2) ? 1u : 0u;  // NaN-right, zero-right
                    nodes[2 * i] = ((static_cast<uint32_t>(w[0]) ^ 0x80000000u) & ~mask) |
                                   (static_cast<uint32_t>(sl) << 1) | c;
                    nodes[2 * i + 1] = static_cast<uint32_t>(l.rel[i]) * 8u;
                    ids[at * node_max + i] = node;
                } else {
                    nodes[2 * i] = (static_cast<uint32_t>(leaf + 1) << slot_bits) | leaf_low;
                    nodes[2 * i + 1] = 0u;
                    const double value = v->leaf_value[node];
                    if (f32) {
                        const float fv = static_cast<float>(value);
                        std::memcpy(leaves + static_cast<size_t>(leaf) * 4, &fv, 4);
                    } else {
                        std::memcpy(leaves + static_cast<size_t>(leaf) * 8, &value, 8);
                    }
                    ++leaf;
                }
            }
        }
    }
    void* trees = nullptr;
    void* dids = nullptr;
    void* dslots = nullptr;
    if (!device_alloc(&trees, host.size(), e) ||
        !ok(cudaMemcpy(trees, host.data(), host.size(), cudaMemcpyHostToDevice), "cudaMemcpy", e) ||
        !device_alloc(&dids, ids.size() * 4, e) ||
        !ok(cudaMemcpy(dids, ids.data(), ids.size() * 4, cudaMemcpyHostToDevice), "cudaMemcpy", e) ||
        !device_alloc(&dslots, slot_of.size() * sizeof(int2), e) ||
        !ok(cudaMemcpy(dslots, slot_of.data(), slot_of.size() * sizeof(int2), cudaMemcpyHostToDevice), "cudaMemcpy",
            e)) {
        if (trees) cudaFree(trees);
        if (dids) cudaFree(dids);
        if (dslots) cudaFree(dslots);
        s = SparseArgs{};
        return false;
    }
    f.blocks[f.nblocks++] = trees;
    f.blocks[f.nblocks++] = dids;
    f.blocks[f.nblocks++] = dslots;
    s.teams = K;
    s.rows = rows;
    s.leaf32 = f32;
    s.slot_bits = slot_bits;
    s.node_max = node_max;
    s.record = record;
    s.slots = slots;
    s.pad_slot = pad;
    s.trees = static_cast<const unsigned char*>(trees);
    s.node_ids = static_cast<const int*>(dids);
    s.slot_of = static_cast<const int2*>(dslots);
    return true;
}

}  // namespace
}  // namespace mlk::cuda

using mlk::cuda::DevForest;
using mlk::cuda::put_error;

extern "C" {

void mlk_cuda_set_copy_threads(int threads) { mlk::cuda::g_copy_threads.store(std::max(1, threads)); }

void mlk_cuda_set_latency_engine(int on) { mlk::cuda::g_latency_engine.store(on); }

int mlk_cuda_device_count(int* count, char* err, size_t errlen) {
    *count = 0;
    const cudaError_t e = cudaGetDeviceCount(count);
    if (e != cudaSuccess) {
        cudaGetLastError();
        *count = 0;
        put_error(err, errlen, std::string("no CUDA device is available: ") + cudaGetErrorString(e));
        return mlk::cuda::kInternal;
    }
    if (*count == 0) {
        put_error(err, errlen, "no CUDA device is available");
        return mlk::cuda::kInternal;
    }
    return 0;
}

int mlk_cuda_current_device(int* device, char* err, size_t errlen) {
    const cudaError_t e = cudaGetDevice(device);
    if (e != cudaSuccess) {
        cudaGetLastError();
        put_error(err, errlen, std::string("cudaGetDevice failed: ") + cudaGetErrorString(e));
        return mlk::cuda::kInternal;
    }
    return 0;
}

int mlk_cuda_pointer_kind(const void* p, int* kind, int* device) {
    *kind = MLK_PTR_PAGEABLE;
    if (device) *device = -1;
    cudaPointerAttributes attr{};
    if (!p || cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged) {
        *kind = MLK_PTR_DEVICE;
        if (device) *device = attr.device;
    } else if (attr.type == cudaMemoryTypeHost) {
        *kind = MLK_PTR_PINNED;
    }
    return 0;
}

int mlk_cuda_forest_device(const mlk_dev_forest* forest) { return forest->f.device; }

int mlk_cuda_forest_upload(int device, const mlk_forest_view* v, mlk_dev_forest** out, char* err, size_t errlen) {
    using namespace mlk::cuda;
    *out = nullptr;
    std::string e;
    DeviceGuard guard(device);
    auto holder = std::make_unique<mlk_dev_forest>();
    DevForest& f = holder->f;
    static std::atomic<unsigned long long> next_uid{1};
    f.uid = next_uid.fetch_add(1);
    f.device = device;
    if (!ok(cudaDeviceGetAttribute(&f.sm_count, cudaDevAttrMultiProcessorCount, device), "cudaDeviceGetAttribute", e)) {
        put_error(err, errlen, e);
        return kInternal;
    }
    // One allocation; every array 256-byte aligned inside it.
    struct Part {
        const void* src;
        size_t bytes;
        size_t at;
    };
    std::vector<Part> parts;
    size_t total = 0;
    auto add = [&](const void* src, size_t bytes) {
        parts.push_back(Part{src, bytes, total});
        total += (bytes + 255) & ~size_t{255};
        return parts.size() - 1;
    };
    const size_t n = static_cast<size_t>(v->nodes), T = static_cast<size_t>(v->trees);
    const size_t F = static_cast<size_t>(v->features), K = static_cast<size_t>(v->outputs);
    const size_t i_nodes = add(v->node_words, n * 16), i_leaf = add(v->leaf_value, n * 8);
    const size_t i_roots = add(v->roots, T * 4), i_depth = add(v->depth, T * 4), i_out = add(v->tree_output, T * 4);
    const size_t i_slot = add(v->slot_of, F * 16), i_base = add(v->base, K * 8), i_counts = add(v->counts, K * 4);
    const size_t i_thr = add(v->threshold, n * 8), i_feat = add(v->feature, n * 4);
    const size_t i_mean = v->standardize ? add(v->pre_mean, F * 8) : SIZE_MAX;
    const size_t i_scale = v->standardize ? add(v->pre_scale, F * 8) : SIZE_MAX;
    std::vector<unsigned char> staging(total, 0);
    for (const Part& p : parts) {
        if (p.bytes) std::memcpy(staging.data() + p.at, p.src, p.bytes);
    }
    void* block = nullptr;
    if (!device_alloc(&block, std::max<size_t>(total, 256), e) ||
        !ok(cudaMemcpy(block, staging.data(), total, cudaMemcpyHostToDevice), "cudaMemcpy", e)) {
        if (block) cudaFree(block);
        put_error(err, errlen, e);
        return kInternal;
    }
    f.blocks[f.nblocks++] = block;
    auto at = [&](size_t i) { return static_cast<unsigned char*>(block) + parts[i].at; };
    ForestArgs& a = f.args;
    a.F = v->features;
    a.K = v->outputs;
    a.T = v->trees;
    a.slots = v->slots;
    a.pad_slot = v->pad_slot;
    a.le = v->decision_le;
    a.cast_f32 = v->cast_f32;
    a.mean = v->mean;
    a.link = v->link;
    a.sigmoid_scale = v->sigmoid_scale;
    a.standardize = v->standardize;
    a.clip = v->clip;
    a.lo = v->clip_lo;
    a.hi = v->clip_hi;
    a.pre_mean = v->standardize ? reinterpret_cast<const double*>(at(i_mean)) : nullptr;
    a.pre_scale = v->standardize ? reinterpret_cast<const double*>(at(i_scale)) : nullptr;
    a.nodes = reinterpret_cast<const int4*>(at(i_nodes));
    a.leaf_value = reinterpret_cast<const double*>(at(i_leaf));
    a.roots = reinterpret_cast<const int*>(at(i_roots));
    a.depth = reinterpret_cast<const int*>(at(i_depth));
    a.tree_output = reinterpret_cast<const int*>(at(i_out));
    a.slot_of = reinterpret_cast<const int4*>(at(i_slot));
    a.base = reinterpret_cast<const double*>(at(i_base));
    a.counts = reinterpret_cast<const int*>(at(i_counts));
    a.threshold = reinterpret_cast<const double*>(at(i_thr));
    a.feature = reinterpret_cast<const int*>(at(i_feat));
    // The status word of device-buffer calls (host-buffer calls use their
    // workspace's): mapped pinned memory, so the host reads it without a
    // copy; montlok_model_device_status reads and clears it.
    void* status = nullptr;
    if (!ok(cudaHostAlloc(&status, sizeof(int), cudaHostAllocMapped), "cudaHostAlloc", e) ||
        !ok(cudaHostGetDevicePointer(reinterpret_cast<void**>(&a.status), status, 0), "cudaHostGetDevicePointer", e)) {
        if (status) cudaFreeHost(status);
        cudaFree(block);
        put_error(err, errlen, e);
        return kInternal;
    }
    f.status_host = static_cast<int*>(status);
    *f.status_host = 0;
    a.wait_ns = kWaitLimitNs;
    a.skip_copies = 0;
    // Complete-tree records: [2^d split words, the last unused] [2^d leaves],
    // 16-byte aligned; a split word is (T & ~mask) | slot.
    const int D = v->complete_depth;
    int rows = 0, buffers = 0;
    if (D > 0 && T > 0 && heap_plan(v->slots, D, v->heap_leaf_f32 != 0, rows, buffers)) {
        const bool f32 = v->heap_leaf_f32 != 0;
        const size_t splits = (size_t{1} << D) - 1, leaves = size_t{1} << D;
        const size_t rec = static_cast<size_t>(heap_record_bytes(D, f32));
        // Whole chunks: the tail is inert trees (every split goes left, to
        // leaves of 0.0), which the kernel walks but never adds.
        const size_t chunk = static_cast<size_t>(heap_chunk_trees());
        const size_t padded = (T + chunk - 1) / chunk * chunk;
        // The split word keeps as few low bits for the slot as the slots the
        // words name need (the pad slot only when padding splits or inert
        // trees exist): every bit left to the threshold halves the ties.
        int32_t top_slot = padded > T ? v->pad_slot : 0;
        for (size_t i = 0; i < T * splits; ++i) top_slot = std::max(top_slot, v->heap_words[2 * i + 1]);
        const int slot_bits = heap_slot_bits(top_slot + 1);
        const uint32_t mask = (1u << slot_bits) - 1u;
        std::vector<unsigned char> host(padded * rec, 0);
        for (size_t t = 0; t < padded; ++t) {
            uint32_t* w = reinterpret_cast<uint32_t*>(host.data() + t * rec);
            const int32_t* src = t < T ? v->heap_words + t * splits * 2 : nullptr;
            for (size_t i = 0; i < splits; ++i) {
                const int32_t thr = src ? src[2 * i] : INT32_MAX;
                const int32_t slot = src ? src[2 * i + 1] : v->pad_slot;
                w[i] = (static_cast<uint32_t>(thr) & ~mask) | static_cast<uint32_t>(slot);
            }
        }
        for (size_t t = 0; t < T; ++t) {
            unsigned char* r = host.data() + t * rec + (size_t{4} << D);
            for (size_t j = 0; j < leaves; ++j) {
                const double value = v->heap_leaf[t * leaves + j];
                if (f32) {
                    const float fv = static_cast<float>(value);
                    std::memcpy(r + j * 4, &fv, 4);
                } else {
                    std::memcpy(r + j * 8, &value, 8);
                }
            }
        }
        void* trees = nullptr;
        void* ids = nullptr;
        if (!device_alloc(&trees, host.size(), e) ||
            !ok(cudaMemcpy(trees, host.data(), host.size(), cudaMemcpyHostToDevice), "cudaMemcpy", e) ||
            !device_alloc(&ids, T * splits * 4, e) ||
            !ok(cudaMemcpy(ids, v->heap_node_id, T * splits * 4, cudaMemcpyHostToDevice), "cudaMemcpy", e)) {
            if (trees) cudaFree(trees);
            if (ids) cudaFree(ids);
            cudaFreeHost(status);
            cudaFree(block);
            put_error(err, errlen, e);
            return kInternal;
        }
        f.blocks[f.nblocks++] = trees;
        f.blocks[f.nblocks++] = ids;
        f.heap.depth = D;
        f.heap.rows = rows;
        f.heap.buffers = buffers;
        f.heap.leaf32 = f32;
        f.heap.slot_bits = slot_bits;
        f.heap.trees = static_cast<const unsigned char*>(trees);
        f.heap.node_ids = static_cast<const int*>(ids);
    }
    // Deep-tree nodes (deep_kernels.cu) for single-output models the
    // complete-tree layout does not take.
    if (f.heap.depth == 0 && v->outputs == 1 && T > 0 && deep_fits(v->slots)) {
        if (!upload_deep(v, f, e)) {
            cudaFreeHost(status);
            for (int i = 0; i < f.nblocks; ++i) cudaFree(f.blocks[i]);
            put_error(err, errlen, e);
            return kInternal;
        }
    }
    // Multi-output records (sparse_kernels.cu) for 2..8 outputs.
    if (f.heap.depth == 0 && v->outputs >= 2 && v->outputs <= 8 && T > 0) {
        if (!upload_sparse(v, f, e)) {
            cudaFreeHost(status);
            for (int i = 0; i < f.nblocks; ++i) cudaFree(f.blocks[i]);
            put_error(err, errlen, e);
            return kInternal;
        }
    }
    if (!prepare_kernels(f, e)) {
        cudaFreeHost(status);
        for (int i = 0; i < f.nblocks; ++i) cudaFree(f.blocks[i]);
        put_error(err, errlen, e);
        return kInternal;
    }
    *out = holder.release();
    return 0;
}

void mlk_cuda_forest_release(mlk_dev_forest* forest) {
    if (!forest) return;
    {
        mlk::cuda::DeviceGuard guard(forest->f.device);
        for (int i = 0; i < forest->f.nblocks; ++i) cudaFree(forest->f.blocks[i]);
        if (forest->f.status_host) cudaFreeHost(forest->f.status_host);
    }
    delete forest;
}

namespace {

// The device-buffer calls' scratch comes from a memory pool of the library's
// own per device, which keeps up to kPoolKeep bytes mapped across
// synchronisations (the default pool returns its memory at every
// synchronisation, so a caller that synchronises after each small call would
// pay a fresh mapping per call). Null when the pool cannot be made: calls then
// use the default pool.
constexpr uint64_t kPoolKeep = uint64_t{256} << 20;

cudaMemPool_t scratch_pool(int device) {
    static std::mutex mu;
    static std::map<int, cudaMemPool_t> pools;
    std::lock_guard<std::mutex> lock(mu);
    auto it = pools.find(device);
    if (it != pools.end()) return it->second;
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = device;
    cudaMemPool_t pool = nullptr;
    if (cudaMemPoolCreate(&pool, &props) == cudaSuccess) {
        uint64_t keep = kPoolKeep;
        if (cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep) != cudaSuccess) {
            cudaMemPoolDestroy(pool);
            pool = nullptr;
        }
    } else {
        pool = nullptr;
    }
    cudaGetLastError();
    pools[device] = pool;
    return pool;
}

}  // namespace

static int device_call(const mlk_dev_forest* forest, int dtype, const void* x, size_t batch, double* out,
                       int32_t* leaves, void* stream, char* err, size_t errlen) {
    using namespace mlk::cuda;
    if (batch == 0) return 0;
    std::string e;
    DeviceGuard guard(forest->f.device);
    const size_t scratch = scratch_bytes(forest->f, static_cast<long long>(batch));
    void* tmp = nullptr;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (scratch) {
        cudaMemPool_t pool = scratch_pool(forest->f.device);
        const cudaError_t a = pool ? cudaMallocFromPoolAsync(&tmp, scratch, pool, st) : cudaMallocAsync(&tmp, scratch, st);
        if (!ok(a, "cudaMallocAsync", e)) {
            put_error(err, errlen, e);
            return kInternal;
        }
    }
    bool good = true;
    if (injected("launch")) {
        e = "kernel launch failed: injected fault (MONTLOK_FAULT_INJECT=launch)";
        good = false;
    } else {
        const DevForest f = call_forest(forest->f, forest->f.args.status, injected("wait"));
        good = launch_forest(f, dtype, x, static_cast<long long>(batch), out, leaves, st, e, static_cast<int*>(tmp));
    }
    if (tmp) cudaFreeAsync(tmp, st);
    if (!good) {
        put_error(err, errlen, e);
        return kInternal;
    }
    return 0;
}

int mlk_cuda_predict_device(const mlk_dev_forest* forest, int dtype, const void* x, size_t batch, double* out,
                            void* stream, char* err, size_t errlen) {
    return device_call(forest, dtype, x, batch, out, nullptr, stream, err, errlen);
}

int mlk_cuda_leaves_device(const mlk_dev_forest* forest, int dtype, const void* x, size_t batch, int32_t* leaves,
                           void* stream, char* err, size_t errlen) {
    return device_call(forest, dtype, x, batch, nullptr, leaves, stream, err, errlen);
}

int mlk_cuda_predict_host(const mlk_dev_forest* forest, int dtype, const void* x, size_t batch, double* out,
                          char* err, size_t errlen) {
    if (batch == 0) return 0;
    return mlk::cuda::run_host<double>(forest->f, dtype, x, batch, out, static_cast<size_t>(forest->f.args.K), false,
                                       err, errlen);
}

int mlk_cuda_forest_status(const mlk_dev_forest* forest, int clear) {
    volatile int* word = forest->f.status_host;
    if (!word) return 0;
    const int value = *word;
    if (clear && value) *word = 0;
    return value;
}

int mlk_cuda_leaves_host(const mlk_dev_forest* forest, int dtype, const void* x, size_t batch, int32_t* leaves,
                         char* err, size_t errlen) {
    if (batch == 0) return 0;
    return mlk::cuda::run_host<int32_t>(forest->f, dtype, x, batch, leaves, static_cast<size_t>(forest->f.args.T),
                                        true, err, errlen);
}

}  // extern "C"
