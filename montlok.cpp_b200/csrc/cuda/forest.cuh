// Device-side forest and the kernel launchers (internal to csrc/cuda).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>

namespace mlk::cuda {

// Everything a kernel needs, passed by value as a kernel parameter.
struct ForestArgs {
    int F, K, T, slots, pad_slot;
    int le, cast_f32, mean, link;
    double sigmoid_scale;
    int standardize, clip;
    double lo, hi;
    const double* pre_mean;
    const double* pre_scale;
    const int4* nodes;          // [nodes]: T, slot, left, right
    const double* leaf_value;   // [nodes]
    const int* roots;           // [T]
    const int* depth;           // [T]
    const int* tree_output;     // [T]
    const int4* slot_of;        // [F]: slot per variant, -1 when unused
    const double* base;         // [K]
    const int* counts;          // [K]
    const double* threshold;    // [nodes]
    const int* feature;         // [nodes]
    // Per call: the mapped host word a kernel sets to 1 when a wait on its
    // tree copies runs out (then its rows are not written), how long such a
    // wait may take, and a fault-injection switch that makes the kernels
    // issue no tree copy at all, so every wait runs out (tests only).
    int* status;
    unsigned long long wait_ns;
    int skip_copies;
};

// Complete-tree layout (heap_kernels.cu); depth 0 when the model has none.
struct HeapArgs {
    int depth, rows, leaf32, buffers;
    int slot_bits;               // low bits of a split word holding the slot
    const unsigned char* trees;  // whole chunks of heap_record_bytes(depth, leaf32) records, inert trees last
    const int* node_ids;         // [T * (2^depth - 1)]: file node of each heap split, -1 for padding
};

// Multi-output layout (sparse_kernels.cu); teams 0 when the model has none.
struct SparseArgs {
    int teams;                   // outputs: one team of `rows` threads per output
    int rows;                    // rows per CTA
    int leaf32;
    int slot_bits;               // low bits of a split word: slot << 1 | missing-goes-right
    int node_max;                // nodes per tree record
    int record;                  // bytes per tree record
    int slots;                   // key table rows: (feature, missing kind) pairs and the pad slot
    int pad_slot;                // slot whose key is always 0 (leaves)
    int offset[8];               // first record of output k's trees
    int chunks[8];               // chunks of output k
    const unsigned char* trees;  // records, output by output, each padded to whole chunks
    const int* node_ids;         // [records * node_max]: file node of each split, -1 for leaves
    const int2* slot_of;         // [F]: slot of (feature, NaN missing), (feature, NaN or zero missing)
};

// Bytes of one complete-tree record of depth `depth`: 2^depth split words of
// 4 bytes (the last unused), then 2^depth leaf values, 16-byte aligned.
__host__ __device__ constexpr int heap_record_size(int depth, bool leaf32) {
    return ((4 << depth) + (1 << depth) * (leaf32 ? 4 : 8) + 15) & ~15;
}

// Deep-tree layout (deep_kernels.cu); nodes null when the model has none.
inline constexpr int kTreeBlock = 64;  // trees per partial sum (the reference sums in 64-tree blocks)

struct DeepArgs {
    int slot_bits;            // low bits of a split word holding the slot
    int leaf32;               // leaf values are float32
    const uint32_t* records;  // 8 words per record: {W top, W left, W right, 0, exits LL, LR, RL, RR}
    const void* leaves;       // leaf values, indexed by an exit with the top bit set
    const uint32_t* roots;    // [T]: exit to each tree's root
    const int* steps;         // [T]: records on the longest root-to-leaf walk
    const int* node_ids;      // [3 * records]: file node of each record's three splits, -1 for none
};

struct DevForest {
    unsigned long long uid = 0;  // distinct for every forest uploaded by this process
    int device = 0;
    int sm_count = 0;
    ForestArgs args{};
    HeapArgs heap{};
    SparseArgs sparse{};
    DeepArgs deep{};
    int* status_host = nullptr;  // the status word as the host sees it
    void* blocks[20] = {};  // device allocations, freed with the forest
    int nblocks = 0;
};

// Queues one predict (out != nullptr) or leaf-index (leaves != nullptr) pass
// over device buffers on `stream`. `scratch` holds scratch_bytes(f, batch) bytes of
// device memory (nullptr when that is 0). `counters`, when given, is a buffer
// of at least kLatencyCounters ints that is zero and that only these
// launches use (they leave it zero); without it the small-batch kernel's
// counters live in `scratch` and are cleared on the stream first. Returns
// false with `err` set.
inline constexpr int kLatencyCounters = 8;
bool launch_forest(const DevForest& f, int dtype, const void* x, long long batch, double* out, int* leaves,
                   cudaStream_t stream, std::string& err, int* scratch, int* counters = nullptr);

// Device scratch a launch of `batch` rows needs: key tables in global memory
// when a warp's table exceeds shared memory (models with thousands of
// features), one per resident warp; then, for batches the small-batch
// complete-tree kernel takes, its per-tree leaf values and block sums.
size_t scratch_bytes(const DevForest& f, long long batch);

// One-time per-device kernel attributes (dynamic shared memory limits).
bool prepare_kernels(const DevForest& f, std::string& err);

// Complete-tree kernels: rows per CTA and chunk buffers that fit shared
// memory (false: none), bytes of one tree record, trees per chunk, launch.
bool heap_plan(int slots, int depth, bool leaf32, int& rows, int& buffers);
int heap_record_bytes(int depth, bool leaf32);
int heap_chunk_trees();
int heap_slot_bits(int slots);

// Tree-parallel complete-tree kernel for small batches: device scratch it
// needs, whether it takes `batch` rows, launch (`scratch` holds
// latency_scratch_bytes(f) bytes).
size_t latency_scratch_bytes(const DevForest& f);
bool latency_fits(const DevForest& f, long long batch);
// 0: the counter form; 1, 2: the cluster form (2: CTA 0 reads the rows once,
// so they may be in pinned host memory).
int latency_form(const DevForest& f, int dtype, long long batch);
bool launch_latency(const DevForest& f, int dtype, const void* x, long long batch, double* out, cudaStream_t stream,
                    std::string& err, void* scratch, int* counters);
bool launch_heap(const DevForest& f, int dtype, const void* x, long long batch, double* out, cudaStream_t stream,
                 std::string& err);
// Whether launch_heap runs the staged variant (keys prepared in TMEM by
// producer warps while the walkers walk) for `batch` rows.
bool heap_staged(const DevForest& f, long long batch);

// Deep-tree kernel (one output): whether a model's key tables fit, launch.
bool deep_fits(int slots);
bool launch_deep(const DevForest& f, int dtype, const void* x, long long batch, double* out, cudaStream_t stream,
                 std::string& err);

// Multi-output kernel: trees per chunk, rows per CTA that fit (false: none),
// launch.
int sparse_chunk_trees();
bool sparse_plan(int slots, int teams, int record, int& rows);
bool launch_sparse(const DevForest& f, int dtype, const void* x, long long batch, double* out, cudaStream_t stream,
                   std::string& err);

}  // namespace mlk::cuda

// The opaque handle of mlk_cuda.h: one device replica of a forest.
struct mlk_dev_forest {
    mlk::cuda::DevForest f;
};
