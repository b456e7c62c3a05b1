// The tree_ensemble family: validation (same checks, order and statuses as
// the reference constructor, src/core/trees.cpp:70-156) and compilation into
// the image the CUDA kernels read.
//
// Decision rule. The reference decides a split with leaf()
// (src/core/trees.cpp:411-430): NaN takes the default branch unless the
// missing mode is 0 (then NaN reads as 0.0); mode 2 also sends |v| <= 1e-35f
// to the default branch; otherwise left when v <= t ("le") or v < t ("lt").
// The GPU evaluates the same rule as one signed 32-bit compare,
//
//     go right  <=>  key(prepared value) > T
//
// where key() maps a float to an int32 in the order of the reals (-0 and +0
// both to 0), and the prepared row holds, per feature, up to four variants
// that fold the missing rules into the key:
//
//     kNanRight   NaN -> INT32_MAX   (NaN must go right)
//     kNanLeft    NaN -> INT32_MIN   (NaN must go left)
//     kZeroRight  NaN and |v| <= 1e-35f -> INT32_MAX
//     kZeroLeft   NaN and |v| <= 1e-35f -> INT32_MIN
//
// A split reads the variant of its own rule: mode 1 and 2 by the default
// side, mode 0 by where 0.0 goes. Thresholds become:
//
//   float32 features ("feature_cast": "f32"): the value is a float, so
//     le:  v >  t  <=>  v > RD32(t)    T = key(RD32(t))
//     lt:  v >= t  <=>  v >= RU32(t)   T = key(RU32(t)) - 1
//   (RD32/RU32 round a double down/up to float; -inf < t < inf or not, both
//   hold, which keeps infinite thresholds exact).
//
//   float64 features: the prepared value is RD32(v) and T = key(RD32(t)).
//   Unequal keys order v and t exactly; equal keys (v and t in the same
//   float32 interval, rare for real data) fall back to comparing the doubles,
//   which the kernel reads from the input.
//
// NaN keys are INT32_MAX/INT32_MIN and every T lies in
// [key(-inf) - 1, key(+inf)], so NaN never ties and always goes its way.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>

#include "runtime.hpp"

namespace mlk {

namespace {

constexpr double kZero = static_cast<double>(1e-35f);  // LightGBM's kZeroThreshold
constexpr int32_t kNeverRight = std::numeric_limits<int32_t>::max();

int32_t key32(float v) noexcept {
    uint32_t bits;
    std::memcpy(&bits, &v, 4);
    const uint32_t magnitude = bits & 0x7FFFFFFFu;
    return (bits >> 31) ? -static_cast<int32_t>(magnitude) : static_cast<int32_t>(magnitude);
}

float round_down32(double t) noexcept {
    float f = static_cast<float>(t);
    if (static_cast<double>(f) > t) f = std::nextafter(f, -std::numeric_limits<float>::infinity());
    return f;
}

float round_up32(double t) noexcept {
    float f = static_cast<float>(t);
    if (static_cast<double>(f) < t) f = std::nextafter(f, std::numeric_limits<float>::infinity());
    return f;
}

// Which prepared-row variant a split reads (see the file comment).
int variant_of(uint8_t flags, double t, bool le) noexcept {
    const unsigned mode = (flags >> 1) & 3u;
    const bool default_left = (flags & 1u) != 0;
    if (mode == 0) {
        const bool zero_goes_right = le ? (0.0 > t) : !(0.0 < t);
        return zero_goes_right ? kNanRight : kNanLeft;
    }
    if (mode == 1) return default_left ? kNanLeft : kNanRight;
    return default_left ? kZeroLeft : kZeroRight;
}

// The complete-tree view of a single-output forest no deeper than 8 levels
// (see ForestImage). A leaf above the last level becomes splits that always
// go left (T = INT32_MAX, never exceeded) down to copies of itself.
void build_heap_view(ForestImage& img) {
    constexpr int kMaxDepth = 8;
    if (img.outputs != 1) return;
    int D = 1;
    for (const int32_t d : img.depth) D = std::max(D, static_cast<int>(d));
    if (D > kMaxDepth) return;
    const size_t splits = (size_t{1} << D) - 1, leaves = size_t{1} << D, T = static_cast<size_t>(img.trees);
    img.heap_words.assign(T * splits * 2, 0);
    img.heap_node_id.assign(T * splits, -1);
    img.heap_leaf.assign(T * leaves, 0.0);
    img.heap_leaf_id.assign(T * leaves, -1);
    bool f32 = true;
    struct Item {
        size_t heap;
        int level;
        int32_t node;
    };
    std::vector<Item> stack;
    for (size_t t = 0; t < T; ++t) {
        stack.assign(1, Item{0, 0, img.roots[t]});
        while (!stack.empty()) {
            const Item it = stack.back();
            stack.pop_back();
            const bool split = img.feature[static_cast<size_t>(it.node)] >= 0;
            if (it.level == D) {  // a real leaf: depth D bounds every path
                const double v = img.leaf_value[static_cast<size_t>(it.node)];
                img.heap_leaf[t * leaves + (it.heap - splits)] = v;
                img.heap_leaf_id[t * leaves + (it.heap - splits)] = it.node;
                f32 = f32 && static_cast<double>(static_cast<float>(v)) == v;
                continue;
            }
            int32_t* w = &img.heap_words[(t * splits + it.heap) * 2];
            if (split) {
                const int32_t* nw = &img.node_words[static_cast<size_t>(it.node) * 4];
                w[0] = nw[0];
                w[1] = nw[1];
                img.heap_node_id[t * splits + it.heap] = it.node;
                stack.push_back(Item{2 * it.heap + 2, it.level + 1, nw[3]});
                stack.push_back(Item{2 * it.heap + 1, it.level + 1, nw[2]});
            } else {
                w[0] = kNeverRight;
                w[1] = img.pad_slot;
                stack.push_back(Item{2 * it.heap + 2, it.level + 1, it.node});
                stack.push_back(Item{2 * it.heap + 1, it.level + 1, it.node});
            }
        }
    }
    img.complete_depth = D;
    img.heap_leaf_f32 = f32;
}

}  // namespace

std::unique_ptr<ForestImage> build_forest(const Archive& a, const json::Value& spec, const json::Value& config,
                                          size_t features, size_t sequence) {
    if (sequence > 1) fail(Status::Shape, "tree_ensemble models are tabular: inputs.sequence must be 0 or 1");
    auto img = std::make_unique<ForestImage>();
    const json::Value* outputs = spec.find("outputs");
    const size_t K = json_size(*outputs, "size", 1);
    img->features = static_cast<int32_t>(features);
    img->outputs = static_cast<int32_t>(K);

    const std::string decision = json_string(config, "decision", "le");
    if (decision != "le" && decision != "lt") fail(Status::Format, "tree_ensemble decision must be \"le\" or \"lt\"");
    img->decision_le = decision == "le";
    const std::string cast = json_string(config, "feature_cast", "f64");
    if (cast != "f64" && cast != "f32") fail(Status::Format, "feature_cast must be \"f64\" or \"f32\"");
    img->cast_f32 = cast == "f32";
    const std::string aggregate = json_string(config, "aggregate", "sum");
    if (aggregate != "sum" && aggregate != "mean") fail(Status::Format, "aggregate must be \"sum\" or \"mean\"");
    img->mean = aggregate == "mean";
    const std::string link = json_string(config, "link", "identity");
    if (link == "identity") img->link = Link::Identity;
    else if (link == "sigmoid") img->link = Link::Sigmoid;
    else if (link == "softmax") img->link = Link::Softmax;
    else if (link == "exp") img->link = Link::Exp;
    else fail(Status::Unsupported, "unknown tree_ensemble link \"" + link + "\"");
    img->sigmoid_scale = json_double(config, "sigmoid_scale", 1.0);

    img->base.assign(K, 0.0);
    if (const json::Value* base = config.find("base_score"); base && !base->is_null()) {
        if (base->is_number()) {
            std::fill(img->base.begin(), img->base.end(), base->as_number());
        } else if (base->is_array() && base->as_array().size() == K) {
            for (size_t k = 0; k < K; ++k) img->base[k] = base->as_array()[k].as_number();
        } else {
            fail(Status::Format, "base_score must be a number or one number per output");
        }
    }

    const std::string p = json_string(config, "tensors", "trees");
    std::vector<int32_t> roots = a.i32(p + ".root", {-1});
    std::vector<int32_t> tree_output = a.i32(p + ".output", {static_cast<int64_t>(roots.size())});
    std::vector<int32_t> feature = a.i32(p + ".feature", {-1});
    const auto n = static_cast<int64_t>(feature.size());
    std::vector<double> threshold = a.f64(p + ".threshold", {n});
    const std::vector<int32_t> left = a.i32(p + ".left", {n});
    const std::vector<int32_t> right = a.i32(p + ".right", {n});
    const std::vector<double> value = a.f64(p + ".value", {n});
    std::vector<uint8_t> flags = a.u8(p + ".flags", {n});
    if (roots.empty() || feature.empty()) fail(Status::Format, "tree_ensemble needs at least one tree");
    if (n > std::numeric_limits<int32_t>::max() / 4) fail(Status::Unsupported, "tree_ensemble has too many nodes");

    for (int64_t i = 0; i < n; ++i) {
        const auto self = static_cast<int32_t>(i);
        if (feature[i] >= 0) {
            if (static_cast<size_t>(feature[i]) >= features) {
                fail(Status::Shape, "node " + std::to_string(i) + " splits on feature " + std::to_string(feature[i]) +
                                        " of " + std::to_string(features));
            }
            if (left[i] <= self || right[i] <= self || left[i] >= n || right[i] >= n) {
                fail(Status::Format, "node " + std::to_string(i) + " must point to later nodes");
            }
            if (std::isnan(threshold[i])) fail(Status::Format, "node " + std::to_string(i) + " has a NaN threshold");
            if (((flags[i] >> 1) & 3u) == 3u) fail(Status::Format, "node " + std::to_string(i) + " has bad flags");
        } else if (!std::isfinite(value[i])) {
            fail(Status::Format, "leaf " + std::to_string(i) + " has a non-finite value");
        }
    }
    img->counts.assign(K, 0);
    for (size_t t = 0; t < roots.size(); ++t) {
        if (roots[t] < 0 || roots[t] >= n) fail(Status::Format, "tree " + std::to_string(t) + " root is out of range");
        if (tree_output[t] < 0 || static_cast<size_t>(tree_output[t]) >= K) {
            fail(Status::Format, "tree " + std::to_string(t) + " adds to a missing output");
        }
        ++img->counts[static_cast<size_t>(tree_output[t])];
    }
    if (img->link == Link::Softmax && K < 2) fail(Status::Format, "softmax needs at least two outputs");
    if (features > static_cast<size_t>(std::numeric_limits<int32_t>::max() / kVariants - 1)) {
        fail(Status::Unsupported, "tree_ensemble has too many features for the GPU layout");
    }

    // Slots: every (feature, variant) some split reads, variant-major.
    const size_t F = features;
    std::vector<uint8_t> used(F * kVariants, 0);
    std::vector<int8_t> node_variant(static_cast<size_t>(n), 0);
    for (int64_t i = 0; i < n; ++i) {
        if (feature[i] < 0) continue;
        const int v = variant_of(flags[i], threshold[i], img->decision_le);
        node_variant[i] = static_cast<int8_t>(v);
        used[static_cast<size_t>(feature[i]) * kVariants + v] = 1;
    }
    img->slot_of.assign(F * kVariants, -1);
    int32_t next = 0;
    for (int v = 0; v < kVariants; ++v) {
        for (size_t f = 0; f < F; ++f) {
            if (used[f * kVariants + v]) img->slot_of[f * kVariants + v] = next++;
        }
    }
    img->pad_slot = next++;
    img->slots = next;

    // Nodes.
    img->nodes = static_cast<int32_t>(n);
    img->trees = static_cast<int32_t>(roots.size());
    img->node_words.resize(static_cast<size_t>(n) * 4);
    img->leaf_value.assign(static_cast<size_t>(n), 0.0);
    for (int64_t i = 0; i < n; ++i) {
        int32_t* w = &img->node_words[static_cast<size_t>(i) * 4];
        if (feature[i] < 0) {
            w[0] = kNeverRight;
            w[1] = img->pad_slot;
            w[2] = w[3] = static_cast<int32_t>(i);
            img->leaf_value[i] = value[i];
            continue;
        }
        const double t = threshold[i];
        int32_t T;
        if (!img->cast_f32) T = key32(round_down32(t));
        else if (img->decision_le) T = key32(round_down32(t));
        else T = key32(round_up32(t)) - 1;
        w[0] = T;
        w[1] = img->slot_of[static_cast<size_t>(feature[i]) * kVariants + node_variant[i]];
        w[2] = left[i];
        w[3] = right[i];
    }

    // Longest root-to-leaf path of every tree (children come after parents).
    std::vector<int32_t> height(static_cast<size_t>(n), 0);
    for (int64_t i = n - 1; i >= 0; --i) {
        if (feature[i] >= 0) height[i] = 1 + std::max(height[left[i]], height[right[i]]);
    }
    img->depth.resize(roots.size());
    for (size_t t = 0; t < roots.size(); ++t) img->depth[t] = height[roots[t]];
    img->roots = std::move(roots);
    img->tree_output = std::move(tree_output);
    img->threshold = std::move(threshold);
    img->feature = std::move(feature);
    img->flags = std::move(flags);
    build_heap_view(*img);
    return img;
}

}  // namespace mlk
