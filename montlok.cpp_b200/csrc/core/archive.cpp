// Model files. A .montlok file is a safetensors container: eight bytes of
// little-endian header length, a JSON header naming each tensor's dtype,
// shape and byte range (relative to the end of the header), then the tensor
// bytes; the model spec is the JSON text stored as __metadata__["montlok"].
//
// Loading copies the file into memory and checks it in three steps, each
// failure a montlok status the reference loader also returns for it (format
// errors, or UNSUPPORTED for a dtype or schema this build does not read):
//   1. the container: the length field and the header's bounds;
//   2. every tensor entry, in header order: its fields, dtype, rank, extents
//      and byte range, and that the range holds exactly shape x dtype bytes;
//   3. the spec: present, a JSON object, schema "montlok.model/1".
// After that, no tensor view can point outside the file.
#include <cstdio>
#include <cstring>
#include <limits>

#include "runtime.hpp"

namespace mlk {

namespace {

constexpr uint64_t kMaxHeader = uint64_t{64} << 20;  // header bytes a model may use
constexpr size_t kMaxRank = 8;
constexpr const char* kSchema = "montlok.model/1";

struct DTypeInfo {
    const char* tag;
    DType dtype;
    size_t width;
};

constexpr DTypeInfo kDTypes[] = {
    {"F64", DType::F64, 8}, {"F32", DType::F32, 4}, {"I64", DType::I64, 8},
    {"I32", DType::I32, 4}, {"U8", DType::U8, 1},   {"BOOL", DType::Bool, 1},
};

const DTypeInfo* dtype_named(std::string_view tag) noexcept {
    for (const DTypeInfo& d : kDTypes) {
        if (tag == d.tag) return &d;
    }
    return nullptr;
}

const DTypeInfo& info(DType dtype) noexcept {
    for (const DTypeInfo& d : kDTypes) {
        if (d.dtype == dtype) return d;
    }
    return kDTypes[0];
}

std::string dims(const std::vector<int64_t>& shape) {
    std::string text = "(";
    for (size_t i = 0; i < shape.size(); ++i) {
        if (i) text += ",";
        text += shape[i] < 0 ? std::string("*") : std::to_string(shape[i]);
    }
    return text + ")";
}

std::vector<uint8_t> read_file(const std::string& path) {
    std::FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) fail(Status::Io, "model file " + path + " could not be opened");
    std::vector<uint8_t> bytes;
    uint8_t block[1 << 16];
    size_t got;
    while ((got = std::fread(block, 1, sizeof block, f)) > 0) bytes.insert(bytes.end(), block, block + got);
    const bool bad = std::ferror(f) != 0;
    std::fclose(f);
    if (bad) fail(Status::Io, "model file " + path + " could not be read");
    return bytes;
}

// A tensor entry of the header, checked against the data region.
Tensor decode_entry(const std::string& name, const json::Value& entry, const uint8_t* data, size_t data_size) {
    auto bad = [&](const std::string& why) { fail(Status::Format, "tensor \"" + name + "\": " + why); };
    if (!entry.is_object()) bad("its header entry is not an object");
    const json::Value* dtype = entry.find("dtype");
    const json::Value* shape = entry.find("shape");
    const json::Value* range = entry.find("data_offsets");
    if (!(dtype && dtype->is_string() && shape && shape->is_array() && range && range->is_array())) {
        bad("the entry needs a string dtype and shape and data_offsets arrays");
    }
    const DTypeInfo* d = dtype_named(dtype->as_string());
    if (!d) fail(Status::Unsupported, "tensor \"" + name + "\": dtype " + dtype->as_string() + " is not supported");
    if (shape->as_array().size() > kMaxRank) bad("more than 8 dimensions");

    Tensor t;
    t.name = name;
    t.dtype = d->dtype;
    size_t elements = 1;
    int64_t lo = 0, hi = 0;
    try {
        for (const json::Value& extent : shape->as_array()) {
            const int64_t n = extent.as_int();
            if (n < 0) bad("a negative extent");
            if (n != 0 && elements > std::numeric_limits<size_t>::max() / static_cast<size_t>(n)) {
                bad("more elements than memory can hold");
            }
            elements *= static_cast<size_t>(n);
            t.shape.push_back(n);
        }
        if (range->as_array().size() != 2) bad("data_offsets must be [begin, end]");
        lo = range->as_array()[0].as_int();
        hi = range->as_array()[1].as_int();
    } catch (const Error&) {
        throw;
    } catch (const std::exception& e) {
        bad(e.what());
    }
    if (lo < 0 || hi < lo || static_cast<uint64_t>(hi) > data_size) bad("data_offsets fall outside the file");
    t.data = data + lo;
    t.nbytes = static_cast<size_t>(hi - lo);
    if (elements > std::numeric_limits<size_t>::max() / d->width || elements * d->width != t.nbytes) {
        bad("its byte range does not hold shape x dtype bytes");
    }
    return t;
}

// Element i of a tensor whose elements are stored as `From`.
template <typename From>
From element(const Tensor& t, size_t i) noexcept {
    From v;
    std::memcpy(&v, t.data + i * sizeof(From), sizeof(From));
    return v;
}

}  // namespace

size_t Tensor::numel() const noexcept {
    size_t n = 1;
    for (const int64_t d : shape) n *= static_cast<size_t>(d);
    return n;
}

std::string Tensor::describe() const { return "\"" + name + "\" " + info(dtype).tag + dims(shape); }

std::shared_ptr<const Archive> Archive::from_file(const std::string& path) {
    auto archive = std::shared_ptr<Archive>(new Archive());
    archive->bytes_ = read_file(path);
    archive->parse();
    return archive;
}

std::shared_ptr<const Archive> Archive::from_bytes(const void* data, size_t size) {
    if (!data && size) fail(Status::InvalidArgument, "null model buffer");
    auto archive = std::shared_ptr<Archive>(new Archive());
    archive->bytes_.resize(size);
    if (size) std::memcpy(archive->bytes_.data(), data, size);
    archive->parse();
    return archive;
}

void Archive::parse() {
    // 1. The container.
    if (bytes_.size() < 8) fail(Status::Format, "not a model file: too short for a safetensors header");
    uint64_t header_bytes = 0;
    for (int i = 7; i >= 0; --i) header_bytes = (header_bytes << 8) | bytes_[static_cast<size_t>(i)];
    if (header_bytes > kMaxHeader || header_bytes > bytes_.size() - 8) {
        fail(Status::Format, "not a model file: the safetensors header length is impossible");
    }
    const uint8_t* data = bytes_.data() + 8 + header_bytes;
    const size_t data_size = bytes_.size() - 8 - static_cast<size_t>(header_bytes);
    json::Value header;
    try {
        header = json::Value::parse(
            std::string_view(reinterpret_cast<const char*>(bytes_.data() + 8), static_cast<size_t>(header_bytes)));
    } catch (const std::exception& e) {
        fail(Status::Format, std::string("safetensors header: ") + e.what());
    }
    if (!header.is_object()) fail(Status::Format, "safetensors header must be a JSON object");

    // 2. The tensors, in header order.
    const json::Value* metadata = nullptr;
    for (const auto& [name, entry] : header.as_object()) {
        if (name == "__metadata__") {
            metadata = &entry;
        } else {
            tensors_.push_back(decode_entry(name, entry, data, data_size));
        }
    }

    // 3. The spec.
    const json::Value* text = metadata && metadata->is_object() ? metadata->find("montlok") : nullptr;
    if (!metadata || !metadata->is_object()) fail(Status::Format, "not a montlok model: the file has no metadata");
    if (!text || !text->is_string()) fail(Status::Format, "not a montlok model: metadata has no \"montlok\" spec");
    spec_text_ = text->as_string();
    try {
        spec_ = json::Value::parse(spec_text_);
    } catch (const std::exception& e) {
        fail(Status::Format, std::string("model spec: ") + e.what());
    }
    if (!spec_.is_object()) fail(Status::Format, "model spec must be a JSON object");
    const json::Value* schema = spec_.find("schema");
    if (!schema || !schema->is_string() || schema->as_string() != kSchema) {
        fail(Status::Unsupported, std::string("model spec schema is not ") + kSchema);
    }
}

const Tensor* Archive::find(std::string_view name) const noexcept {
    for (const Tensor& t : tensors_) {
        if (t.name == name) return &t;
    }
    return nullptr;
}

const Tensor& Archive::checked(std::string_view name, const std::vector<int64_t>& shape) const {
    const Tensor* t = find(name);
    if (!t) fail(Status::Format, "model file lacks tensor \"" + std::string(name) + "\"");
    bool same = t->shape.size() == shape.size();
    for (size_t i = 0; same && i < shape.size(); ++i) same = shape[i] < 0 || shape[i] == t->shape[i];
    if (!same) fail(Status::Shape, "tensor " + t->describe() + " should have shape " + dims(shape));
    return *t;
}

std::vector<double> Archive::f64(std::string_view name, const std::vector<int64_t>& shape) const {
    const Tensor& t = checked(name, shape);
    std::vector<double> out(t.numel());
    switch (t.dtype) {
        case DType::F64:
            for (size_t i = 0; i < out.size(); ++i) out[i] = element<double>(t, i);
            break;
        case DType::F32:
            for (size_t i = 0; i < out.size(); ++i) out[i] = element<float>(t, i);
            break;
        default: fail(Status::Format, "tensor " + t.describe() + " should hold F64 or F32 values");
    }
    return out;
}

std::vector<int32_t> Archive::i32(std::string_view name, const std::vector<int64_t>& shape) const {
    const Tensor& t = checked(name, shape);
    std::vector<int32_t> out(t.numel());
    switch (t.dtype) {
        case DType::I32:
            for (size_t i = 0; i < out.size(); ++i) out[i] = element<int32_t>(t, i);
            break;
        case DType::I64:
            for (size_t i = 0; i < out.size(); ++i) {
                const int64_t v = element<int64_t>(t, i);
                if (v != static_cast<int32_t>(v)) fail(Status::Format, "tensor " + t.describe() + " overflows int32");
                out[i] = static_cast<int32_t>(v);
            }
            break;
        default: fail(Status::Format, "tensor " + t.describe() + " should hold I32 or I64 values");
    }
    return out;
}

std::vector<uint8_t> Archive::u8(std::string_view name, const std::vector<int64_t>& shape) const {
    const Tensor& t = checked(name, shape);
    if (t.dtype != DType::U8 && t.dtype != DType::Bool) {
        fail(Status::Format, "tensor " + t.describe() + " should hold U8 values");
    }
    return std::vector<uint8_t>(t.data, t.data + t.nbytes);
}

// Spec fields with a fallback when absent or null.

size_t json_size(const json::Value& object, std::string_view key, size_t fallback) {
    const json::Value* v = object.find(key);
    if (!v || v->is_null()) return fallback;
    auto bad = [&] { fail(Status::Format, "spec field \"" + std::string(key) + "\" must be a non-negative integer"); };
    int64_t n = -1;
    try {
        n = v->as_int();
    } catch (const std::exception&) {
        bad();
    }
    if (n < 0) bad();
    return static_cast<size_t>(n);
}

double json_double(const json::Value& object, std::string_view key, double fallback) {
    const json::Value* v = object.find(key);
    if (!v || v->is_null()) return fallback;
    if (!v->is_number()) fail(Status::Format, "spec field \"" + std::string(key) + "\" must be a number");
    return v->as_number();
}

std::string json_string(const json::Value& object, std::string_view key, const std::string& fallback) {
    const json::Value* v = object.find(key);
    if (!v || v->is_null()) return fallback;
    if (!v->is_string()) fail(Status::Format, "spec field \"" + std::string(key) + "\" must be a string");
    return v->as_string();
}

}  // namespace mlk
