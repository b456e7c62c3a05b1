// Device helpers shared by the tree kernels: keys, preprocess, the row
// transpose into key tables, the exact float64 split, and the link math.
#pragma once

#include <climits>
#include <cstdint>

#include "forest.cuh"

namespace mlk::cuda {

inline constexpr int kMaxOut = 8;      // outputs held in registers per pass
inline constexpr int kIlp = 4;         // trees one lane walks side by side
inline constexpr int kStage = 33;      // padded row length of the transpose tile
inline constexpr int kStageBytes = 32 * kStage * 8;
inline constexpr double kZeroThr = static_cast<double>(1e-35f);  // LightGBM kZeroThreshold

__host__ __device__ constexpr int align16(int n) { return (n + 15) & ~15; }
__host__ __device__ constexpr int key_bytes(int slots) { return align16(slots * 32 * 4); }

__device__ __forceinline__ int key32(float v) {
    const unsigned b = __float_as_uint(v);
    const int m = static_cast<int>(b & 0x7fffffffu);
    return (b >> 31) ? -m : m;
}

__device__ __forceinline__ double load_x(const float* p) { return static_cast<double>(__ldg(p)); }
__device__ __forceinline__ double load_x(const double* p) { return __ldg(p); }

// Preprocess and cast of one raw value (reference runtime.cpp:532-552 and the
// cast of trees.cpp:275); std::max/std::min written out so NaN stays NaN.
__device__ __forceinline__ double finish(const ForestArgs& a, double v, double mean, double scale) {
    if (a.standardize) v = __ddiv_rn(__dsub_rn(v, mean), scale);
    if (a.clip) {
        v = (v < a.lo) ? a.lo : v;
        v = (a.hi < v) ? a.hi : v;
    }
    if (a.cast_f32) v = static_cast<double>(__double2float_rn(v));
    return v;
}

// Writes the keys of one prepared value into every slot (variant) its
// feature uses. With a nonzero `mask` (the packed-word kernels, whose split
// words are (T & ~mask) | slot) every key keeps only its high bits and
// carries its own slot in the low ones, (key & ~mask) | slot: a key read
// for a split then has the split word's low bits, so `key > word` compares
// the high bits alone and `key == word` is exactly a tie of the high bits.
__device__ __forceinline__ void key_of(const ForestArgs& a, double v, int& k, bool& nan, bool& zero);
template <int STRIDE>
__device__ __forceinline__ void put_made_keys(int* col, int4 s, int k, bool nan, bool zero, int mask);

template <int STRIDE>
__device__ __forceinline__ void put_keys(const ForestArgs& a, int* col, int4 s, double v, int mask = 0) {
    int k;
    bool nan, zero;
    key_of(a, v, k, nan, zero);
    put_made_keys<STRIDE>(col, s, k, nan, zero, mask);
}

// Builds the key table columns of 32 rows starting at row0: the warp reads
// TILE features of all 32 rows at a time, coalesced (TILE consecutive values
// per row), stages them in a padded [32][TILE + 1] tile, and then each lane
// (one row) turns its TILE values into keys. `keys` points at the warp's first
// column; slot s of the lane's row is keys[s * STRIDE + lane].
template <int STRIDE, int TILE, typename XT>
__device__ void prepare_group(const ForestArgs& a, const XT* __restrict__ x, long long row0, long long batch,
                              int* keys, double* stage, int lane, int f_begin = 0, int f_end = -1,
                              bool pad = true) {
    static_assert(TILE == 16 || TILE == 32, "tiles of 16 or 32 features");
    constexpr int kPerLoad = 32 / TILE;  // rows covered by one warp-wide load
    const int sub = lane / TILE, f_in = lane % TILE;
    if (f_end < 0) f_end = a.F;
    for (int f0 = f_begin; f0 < f_end; f0 += TILE) {
        const int feat = f0 + f_in;
        const bool live = feat < f_end;
        double mean = 0.0, scale = 1.0;
        if (live && a.standardize) {
            mean = __ldg(a.pre_mean + feat);
            scale = __ldg(a.pre_scale + feat);
        }
        // All loads of the tile first, so their latencies overlap.
        double raw[32 / kPerLoad];
#pragma unroll
        for (int i = 0; i < 32 / kPerLoad; ++i) {
            const long long row = row0 + i * kPerLoad + sub;
            raw[i] = (live && row < batch) ? load_x(x + row * a.F + feat) : 0.0;
        }
#pragma unroll
        for (int i = 0; i < 32 / kPerLoad; ++i) {
            const long long row = row0 + i * kPerLoad + sub;
            stage[(i * kPerLoad + sub) * (TILE + 1) + f_in] = (live && row < batch) ? finish(a, raw[i], mean, scale) : 0.0;
        }
        __syncwarp();
        const int nf = min(TILE, f_end - f0);
        for (int j = 0; j < nf; ++j) {
            put_keys<STRIDE>(a, keys + lane, __ldg(a.slot_of + f0 + j), stage[lane * (TILE + 1) + j]);
        }
        __syncwarp();
    }
    if (pad) keys[a.pad_slot * STRIDE + lane] = INT_MIN;
    __syncwarp();
}

// The key of one prepared value (see put_keys) with its NaN and LightGBM
// zero-band flags. A float32-cast model's value is a float: its key is exact.
// A float64 model keys RD32(v) and decides ties on the double (exact_right).
__device__ __forceinline__ void key_of(const ForestArgs& a, double v, int& k, bool& nan, bool& zero) {
    if (a.cast_f32) {
        const float f = __double2float_rn(v);
        nan = f != f;
        zero = nan || fabsf(f) <= 1e-35f;  // the float compare of kZeroThr's exact value
        k = key32(f);
    } else {
        nan = v != v;
        zero = nan || fabs(v) <= kZeroThr;
        k = key32(__double2float_rd(v));
    }
}

// put_keys with the key already made.
template <int STRIDE>
__device__ __forceinline__ void put_made_keys(int* col, int4 s, int k, bool nan, bool zero, int mask) {
    auto tag = [mask](int key, int slot) { return (key & ~mask) | (slot & mask); };
    if (s.x >= 0) col[s.x * STRIDE] = tag(nan ? INT_MAX : k, s.x);
    if (s.y >= 0) col[s.y * STRIDE] = tag(nan ? INT_MIN : k, s.y);
    if (s.z >= 0) col[s.z * STRIDE] = tag(zero ? INT_MAX : k, s.z);
    if (s.w >= 0) col[s.w * STRIDE] = tag(zero ? INT_MIN : k, s.w);
}

// Keys of one row, this lane's, for features [f_begin, f_end), written to
// col[slot * STRIDE]. The lane reads its own row eight values at a time, with
// 16-byte vector loads when the rows are 16-byte aligned (the warp's 32 lanes
// read 32 rows; the second half of each 32-byte sector comes from L1), so no
// shared-memory transpose is needed; each value is prepared once (the float32
// cast and key straight from the double when the model has no preprocessing)
// and its key written to every variant slot its feature uses. Rows at or past
// `batch` are prepared as 0.0: their walks read in-bounds shared memory and
// their results are never stored.
//
// prepare_row_with is the same walk over the row with the keys handed to
// put(feature, key, nan, zero) instead; the loop is warp-uniform when
// f_begin and f_end are, so put may hold warp-collective instructions.
template <typename XT, typename Put>
__device__ __forceinline__ void prepare_row_with(const ForestArgs& a, const XT* __restrict__ x, long long row,
                                                 long long batch, int f_begin, int f_end, Put&& put) {
    constexpr int kBatch = 8;
    constexpr int kVec = 16 / static_cast<int>(sizeof(XT));  // values per 16-byte load
    const bool live = row < batch;
    const XT* p = x + (live ? row : 0ll) * a.F;
    const bool plain = !a.standardize && !a.clip;
    const bool vec = a.F % kVec == 0 && f_begin % kVec == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    for (int f0 = f_begin; f0 < f_end; f0 += kBatch) {
        const int n = min(kBatch, f_end - f0);
        double v[kBatch];
        if (vec && n == kBatch) {
            if constexpr (sizeof(XT) == 8) {
#pragma unroll
                for (int i = 0; i < kBatch / 2; ++i) {
                    const double2 t = __ldg(reinterpret_cast<const double2*>(p + f0) + i);
                    v[2 * i] = t.x;
                    v[2 * i + 1] = t.y;
                }
            } else {
#pragma unroll
                for (int i = 0; i < kBatch / 4; ++i) {
                    const float4 t = __ldg(reinterpret_cast<const float4*>(p + f0) + i);
                    v[4 * i] = t.x;
                    v[4 * i + 1] = t.y;
                    v[4 * i + 2] = t.z;
                    v[4 * i + 3] = t.w;
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < kBatch; ++i) v[i] = i < n ? load_x(p + f0 + i) : 0.0;
        }
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
            if (i < n) {
                const int f = f0 + i;
                double val = live ? v[i] : 0.0;
                if (!plain) {
                    const double mean = a.standardize ? __ldg(a.pre_mean + f) : 0.0;
                    const double scale = a.standardize ? __ldg(a.pre_scale + f) : 1.0;
                    val = finish(a, val, mean, scale);
                }
                int k;
                bool nan, zero;
                key_of(a, val, k, nan, zero);
                put(f, k, nan, zero);
            }
        }
    }
}

template <int STRIDE, typename XT>
__device__ void prepare_own_row(const ForestArgs& a, const XT* __restrict__ x, long long row, long long batch, int* col,
                                int f_begin, int f_end, int mask) {
    prepare_row_with(a, x, row, batch, f_begin, f_end, [&](int f, int k, bool nan, bool zero) {
        put_made_keys<STRIDE>(col, __ldg(a.slot_of + f), k, nan, zero, mask);
    });
}

inline constexpr int kPrepTile = 4;                               // features per transpose tile
inline constexpr int kPrepTileBytes = 32 * (kPrepTile + 1) * 8;  // one warp's tile

// Keys of the 32 rows row0 .. row0 + 31 for features [f_begin, f_end): the
// warp reads kPrepTile features of all 32 rows per step (four coalesced loads of
// 8 rows x kPrepTile values; the next two steps' loads are in flight meanwhile),
// stages them in `tile` ([32][kPrepTile + 1] doubles) and each lane turns its own
// row's values into keys, column `lane` of the [slot][STRIDE] table at `keys`.
template <int STRIDE, typename XT>
__device__ void prepare_rows(const ForestArgs& a, const XT* __restrict__ x, long long row0, long long batch, int* keys,
                             double* tile, int lane, int f_begin, int f_end, int mask) {
    constexpr int kPerLoad = 32 / kPrepTile;  // rows covered by one warp-wide load
    const int sub = lane / kPrepTile, f_in = lane % kPrepTile;
    auto load = [&](int f0, double (&v)[kPrepTile]) {
        const int feat = f0 + f_in;
#pragma unroll
        for (int i = 0; i < kPrepTile; ++i) {
            const long long row = row0 + i * kPerLoad + sub;
            v[i] = (feat < f_end && row < batch) ? load_x(x + row * a.F + feat) : 0.0;
        }
    };
    auto stage = [&](int f0, const double (&v)[kPrepTile]) {
        const int feat = f0 + f_in;
        double mean = 0.0, scale = 1.0;
        if (a.standardize && feat < f_end) {
            mean = __ldg(a.pre_mean + feat);
            scale = __ldg(a.pre_scale + feat);
        }
#pragma unroll
        for (int i = 0; i < kPrepTile; ++i) {
            const long long row = row0 + i * kPerLoad + sub;
            tile[(i * kPerLoad + sub) * (kPrepTile + 1) + f_in] =
                (feat < f_end && row < batch) ? finish(a, v[i], mean, scale) : 0.0;
        }
    };
    auto keys_of = [&](int f0) {
        __syncwarp();
        const int nf = min(kPrepTile, f_end - f0);
        for (int j = 0; j < nf; ++j) {
            put_keys<STRIDE>(a, keys + lane, __ldg(a.slot_of + f0 + j), tile[lane * (kPrepTile + 1) + j], mask);
        }
        __syncwarp();
    };
    double even[kPrepTile], odd[kPrepTile];
    load(f_begin, even);
    load(f_begin + kPrepTile, odd);
    for (int f0 = f_begin; f0 < f_end; f0 += 2 * kPrepTile) {
        stage(f0, even);
        load(f0 + 2 * kPrepTile, even);
        keys_of(f0);
        if (f0 + kPrepTile < f_end) {
            stage(f0 + kPrepTile, odd);
            load(f0 + 3 * kPrepTile, odd);
            keys_of(f0 + kPrepTile);
        }
    }
}

// The split decided on doubles, for a float64 model whose keys tied.
template <typename XT>
__device__ __noinline__ bool exact_right(const ForestArgs& a, const XT* __restrict__ x, long long row,
                                         long long batch, int idx) {
    const int feat = __ldg(a.feature + idx);
    const double t = __ldg(a.threshold + idx);
    double v = 0.0;  // padding rows were prepared as 0.0
    if (row < batch) {
        double mean = 0.0, scale = 1.0;
        if (a.standardize) {
            mean = __ldg(a.pre_mean + feat);
            scale = __ldg(a.pre_scale + feat);
        }
        v = finish(a, load_x(x + row * a.F + feat), mean, scale);
    }
    return a.le ? (v > t) : !(v < t);
}

// ---------------------------------------------------------------------------
// Link functions: the reference's exp (kernels.hpp:220-253) — clamp to
// [-708, 708], n = round(x / ln 2) through the 1.5 * 2^52 shifter, Cody-Waite
// reduction r = (x - n ln2_hi) - n ln2_lo, exp(r) - 1 by the degree-13 Taylor
// series in Horner form, and 2^n assembled in the exponent bits.
// ---------------------------------------------------------------------------

__device__ __forceinline__ double vexp(double x) {
    constexpr double kInvLn2 = 1.4426950408889634074;
    constexpr double kLn2Hi = 6.93147180369123816490e-01;
    constexpr double kLn2Lo = 1.90821492927058770002e-10;
    constexpr double kShifter = 6755399441055744.0;
    constexpr double c[13] = {
        1.0 / 6227020800.0, 1.0 / 479001600.0, 1.0 / 39916800.0, 1.0 / 3628800.0, 1.0 / 362880.0,
        1.0 / 40320.0,      1.0 / 5040.0,      1.0 / 720.0,      1.0 / 120.0,     1.0 / 24.0,
        1.0 / 6.0,          0.5,               1.0,
    };
    x = (x < -708.0) ? -708.0 : x;
    x = (x > 708.0) ? 708.0 : x;
    const double shifted = __dadd_rn(__dmul_rn(x, kInvLn2), kShifter);
    const double n = __dsub_rn(shifted, kShifter);
    const double r = __dsub_rn(__dsub_rn(x, __dmul_rn(n, kLn2Hi)), __dmul_rn(n, kLn2Lo));
    double p = c[0];
#pragma unroll
    for (int i = 1; i < 13; ++i) p = __dadd_rn(__dmul_rn(p, r), c[i]);
    p = __dadd_rn(__dmul_rn(p, r), 1.0);
    const unsigned long long bits = static_cast<unsigned long long>(__double_as_longlong(shifted)) -
                                    static_cast<unsigned long long>(__double_as_longlong(kShifter));
    return __dmul_rn(p, __longlong_as_double(static_cast<long long>((bits + 1023ull) << 52)));
}

template <int KC>
__device__ __forceinline__ void apply_link(const ForestArgs& a, double (&v)[KC], int kc) {
    if (a.link == 1) {
#pragma unroll
        for (int j = 0; j < KC; ++j) {
            if (j < kc) {
                const double s = __dmul_rn(v[j], a.sigmoid_scale);
                v[j] = __ddiv_rn(1.0, __dadd_rn(1.0, vexp(__dsub_rn(0.0, s))));
            }
        }
    } else if (a.link == 3) {
#pragma unroll
        for (int j = 0; j < KC; ++j) {
            if (j < kc) v[j] = vexp(v[j]);
        }
    } else if (a.link == 2) {
        double peak = v[0];
#pragma unroll
        for (int j = 1; j < KC; ++j) {
            if (j < kc) peak = (peak < v[j]) ? v[j] : peak;
        }
        double total = 0.0;
#pragma unroll
        for (int j = 0; j < KC; ++j) {
            if (j < kc) {
                v[j] = vexp(__dsub_rn(v[j], peak));
                total = __dadd_rn(total, v[j]);
            }
        }
#pragma unroll
        for (int j = 0; j < KC; ++j) {
            if (j < kc) v[j] = __ddiv_rn(v[j], total);
        }
    }
}

}  // namespace mlk::cuda
