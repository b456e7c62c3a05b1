// The latency engine (engine_kernels.cu): a resident kernel that answers
// small host-buffer predicts without a launch or copy per call.
#pragma once

#include <cstddef>
#include <string>

#include "forest.cuh"

namespace mlk::cuda {

inline constexpr int kEngineRows = 8;     // rows a request may hold
inline constexpr int kEngineFailed = 7;   // MONTLOK_ERROR_INTERNAL

struct LatencyEngine;
void destroy_engine(LatencyEngine* engine);

// Whether the engine can answer `batch` rows of this forest (complete trees,
// one output, at most kEngineRows rows, a CTA per 64-tree block that fits).
bool engine_fits(const DevForest& f, long long batch);

// Predicts through the calling thread's engine `slot` (created, started or
// replaced as needed). Returns 0 when `out` is written, -1 when the engine
// cannot serve the call (the caller takes another path), or kEngineFailed
// with `err` set.
int engine_predict(const DevForest& f, LatencyEngine*& slot, int dtype, const void* x, size_t batch, double* out,
                   std::string& err);

}  // namespace mlk::cuda
