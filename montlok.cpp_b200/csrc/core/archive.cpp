// safetensors reader. An 8-byte little-endian header length, the JSON header,
// then tensor bytes addressed by "data_offsets" relative to the header's end;
// the model spec is the JSON string __metadata__["montlok"]. Every offset,
// dtype, rank and byte size is checked before use, with the statuses of the
// reference reader (src/core/archive.cpp:105-188), so a damaged file is an
// error and never an out-of-range read.
#include <cstring>
#include <fstream>
#include <limits>

#include "runtime.hpp"

namespace mlk {

namespace {

constexpr uint64_t kHeaderLimit = uint64_t{64} << 20;
constexpr size_t kRankLimit = 8;

bool dtype_of(const std::string& tag, DType& out) noexcept {
    static const struct {
        const char* tag;
        DType dtype;
    } table[] = {{"F64", DType::F64}, {"F32", DType::F32}, {"I64", DType::I64},
                 {"I32", DType::I32}, {"U8", DType::U8},   {"BOOL", DType::Bool}};
    for (const auto& row : table) {
        if (tag == row.tag) {
            out = row.dtype;
            return true;
        }
    }
    return false;
}

size_t width(DType d) noexcept {
    switch (d) {
        case DType::F64:
        case DType::I64: return 8;
        case DType::F32:
        case DType::I32: return 4;
        case DType::U8:
        case DType::Bool: return 1;
    }
    return 0;
}

const char* tag_of(DType d) noexcept {
    switch (d) {
        case DType::F64: return "F64";
        case DType::F32: return "F32";
        case DType::I64: return "I64";
        case DType::I32: return "I32";
        case DType::U8: return "U8";
        case DType::Bool: return "BOOL";
    }
    return "?";
}

std::string shape_string(const std::vector<int64_t>& shape) {
    std::string s = "[";
    for (size_t i = 0; i < shape.size(); ++i) s += (i ? ", " : "") + std::to_string(shape[i]);
    return s + "]";
}

}  // namespace

size_t Tensor::numel() const noexcept {
    size_t n = 1;
    for (const int64_t d : shape) n *= static_cast<size_t>(d);
    return n;
}

std::string Tensor::describe() const { return name + " " + tag_of(dtype) + shape_string(shape); }

std::shared_ptr<const Archive> Archive::from_file(const std::string& path) {
    std::ifstream file(path, std::ios::binary | std::ios::ate);
    if (!file) fail(Status::Io, "cannot open model file: " + path);
    const std::streamoff end = file.tellg();
    if (end < 0) fail(Status::Io, "cannot size model file: " + path);
    auto archive = std::shared_ptr<Archive>(new Archive());
    archive->bytes_.resize(static_cast<size_t>(end));
    file.seekg(0);
    if (end > 0 && !file.read(reinterpret_cast<char*>(archive->bytes_.data()), end)) {
        fail(Status::Io, "cannot read model file: " + path);
    }
    archive->parse();
    return archive;
}

std::shared_ptr<const Archive> Archive::from_bytes(const void* data, size_t size) {
    if (!data && size) fail(Status::InvalidArgument, "null model buffer");
    auto archive = std::shared_ptr<Archive>(new Archive());
    const auto* p = static_cast<const uint8_t*>(data);
    archive->bytes_.assign(p, p + size);
    archive->parse();
    return archive;
}

void Archive::parse() {
    const size_t size = bytes_.size();
    const uint8_t* b = bytes_.data();
    if (size < 8) fail(Status::Format, "not a safetensors file: shorter than 8 bytes");
    uint64_t head = 0;
    for (int i = 0; i < 8; ++i) head |= static_cast<uint64_t>(b[i]) << (8 * i);
    if (head > kHeaderLimit || head > size - 8) fail(Status::Format, "not a safetensors file: header length out of range");
    const size_t data_at = 8 + static_cast<size_t>(head);
    const size_t data_size = size - data_at;

    json::Value header;
    try {
        header = json::Value::parse(std::string_view(reinterpret_cast<const char*>(b + 8), static_cast<size_t>(head)));
    } catch (const std::exception& e) {
        fail(Status::Format, std::string("safetensors header: ") + e.what());
    }
    if (!header.is_object()) fail(Status::Format, "safetensors header is not a JSON object");

    const json::Value* meta = nullptr;
    for (const auto& [name, entry] : header.as_object()) {
        if (name == "__metadata__") {
            meta = &entry;
            continue;
        }
        if (!entry.is_object()) fail(Status::Format, "tensor entry is not an object: " + name);
        const json::Value* dtype = entry.find("dtype");
        const json::Value* shape = entry.find("shape");
        const json::Value* offsets = entry.find("data_offsets");
        if (!dtype || !dtype->is_string() || !shape || !shape->is_array() || !offsets || !offsets->is_array()) {
            fail(Status::Format, "tensor entry lacks dtype/shape/data_offsets: " + name);
        }
        Tensor t;
        t.name = name;
        if (!dtype_of(dtype->as_string(), t.dtype)) {
            fail(Status::Unsupported, "tensor " + name + " has unsupported dtype " + dtype->as_string());
        }
        if (shape->as_array().size() > kRankLimit) fail(Status::Format, "tensor rank above 8: " + name);
        size_t count = 1;
        try {
            for (const auto& d : shape->as_array()) {
                const int64_t extent = d.as_int();
                if (extent < 0) fail(Status::Format, "negative extent in tensor " + name);
                if (extent > 0 && count > std::numeric_limits<size_t>::max() / static_cast<size_t>(extent)) {
                    fail(Status::Format, "tensor too large: " + name);
                }
                count *= static_cast<size_t>(extent);
                t.shape.push_back(extent);
            }
            if (offsets->as_array().size() != 2) fail(Status::Format, "data_offsets must have two entries: " + name);
            const int64_t lo = offsets->as_array()[0].as_int();
            const int64_t hi = offsets->as_array()[1].as_int();
            if (lo < 0 || hi < lo || static_cast<uint64_t>(hi) > data_size) {
                fail(Status::Format, "data_offsets out of range: " + name);
            }
            t.data = b + data_at + static_cast<size_t>(lo);
            t.nbytes = static_cast<size_t>(hi - lo);
        } catch (const Error&) {
            throw;
        } catch (const std::exception& e) {
            fail(Status::Format, "tensor " + name + ": " + e.what());
        }
        if (count > std::numeric_limits<size_t>::max() / width(t.dtype) || count * width(t.dtype) != t.nbytes) {
            fail(Status::Format, "tensor " + name + " byte size does not match its shape");
        }
        tensors_.push_back(std::move(t));
    }

    if (!meta || !meta->is_object()) fail(Status::Format, "not a montlok model: no __metadata__");
    const json::Value* text = meta->find("montlok");
    if (!text || !text->is_string()) fail(Status::Format, "not a montlok model: __metadata__.montlok is missing");
    spec_text_ = text->as_string();
    try {
        spec_ = json::Value::parse(spec_text_);
    } catch (const std::exception& e) {
        fail(Status::Format, std::string("model spec: ") + e.what());
    }
    if (!spec_.is_object()) fail(Status::Format, "model spec is not a JSON object");
    const json::Value* schema = spec_.find("schema");
    if (!schema || !schema->is_string() || schema->as_string() != "montlok.model/1") {
        fail(Status::Unsupported, "model spec schema must be \"montlok.model/1\"");
    }
}

const Tensor* Archive::find(std::string_view name) const noexcept {
    for (const auto& t : tensors_) {
        if (t.name == name) return &t;
    }
    return nullptr;
}

const Tensor& Archive::checked(std::string_view name, const std::vector<int64_t>& shape) const {
    const Tensor* t = find(name);
    if (!t) fail(Status::Format, "model file has no tensor named " + std::string(name));
    bool ok = t->shape.size() == shape.size();
    for (size_t i = 0; ok && i < shape.size(); ++i) ok = shape[i] < 0 || shape[i] == t->shape[i];
    if (!ok) fail(Status::Shape, "tensor " + t->describe() + " does not have shape " + shape_string(shape));
    return *t;
}

std::vector<double> Archive::f64(std::string_view name, const std::vector<int64_t>& shape) const {
    const Tensor& t = checked(name, shape);
    std::vector<double> out(t.numel());
    if (t.dtype == DType::F64) {
        if (t.nbytes) std::memcpy(out.data(), t.data, t.nbytes);
    } else if (t.dtype == DType::F32) {
        for (size_t i = 0; i < out.size(); ++i) {
            float v;
            std::memcpy(&v, t.data + 4 * i, 4);
            out[i] = v;
        }
    } else {
        fail(Status::Format, "tensor " + t.describe() + " must be F64 or F32");
    }
    return out;
}

std::vector<int32_t> Archive::i32(std::string_view name, const std::vector<int64_t>& shape) const {
    const Tensor& t = checked(name, shape);
    std::vector<int32_t> out(t.numel());
    if (t.dtype == DType::I32) {
        if (t.nbytes) std::memcpy(out.data(), t.data, t.nbytes);
    } else if (t.dtype == DType::I64) {
        for (size_t i = 0; i < out.size(); ++i) {
            int64_t v;
            std::memcpy(&v, t.data + 8 * i, 8);
            if (v < std::numeric_limits<int32_t>::min() || v > std::numeric_limits<int32_t>::max()) {
                fail(Status::Format, "tensor " + t.describe() + " has values outside int32");
            }
            out[i] = static_cast<int32_t>(v);
        }
    } else {
        fail(Status::Format, "tensor " + t.describe() + " must be I32 or I64");
    }
    return out;
}

std::vector<uint8_t> Archive::u8(std::string_view name, const std::vector<int64_t>& shape) const {
    const Tensor& t = checked(name, shape);
    if (t.dtype != DType::U8 && t.dtype != DType::Bool) fail(Status::Format, "tensor " + t.describe() + " must be U8");
    return std::vector<uint8_t>(t.data, t.data + t.nbytes);
}

size_t json_size(const json::Value& object, std::string_view key, size_t fallback) {
    const json::Value* v = object.find(key);
    if (!v || v->is_null()) return fallback;
    int64_t n = 0;
    try {
        n = v->as_int();
    } catch (const std::exception&) {
        fail(Status::Format, "\"" + std::string(key) + "\" must be a non-negative integer");
    }
    if (n < 0) fail(Status::Format, "\"" + std::string(key) + "\" must be a non-negative integer");
    return static_cast<size_t>(n);
}

double json_double(const json::Value& object, std::string_view key, double fallback) {
    const json::Value* v = object.find(key);
    if (!v || v->is_null()) return fallback;
    if (!v->is_number()) fail(Status::Format, "\"" + std::string(key) + "\" must be a number");
    return v->as_number();
}

std::string json_string(const json::Value& object, std::string_view key, const std::string& fallback) {
    const json::Value* v = object.find(key);
    if (!v || v->is_null()) return fallback;
    if (!v->is_string()) fail(Status::Format, "\"" + std::string(key) + "\" must be a string");
    return v->as_string();
}

}  // namespace mlk
