// JSON values for safetensors headers and model specs.
//
// The parser accepts RFC 8259 documents only and additionally refuses what a
// model file must never contain, so that the same files are accepted as by
// the reference loader: an object that names a member twice, a \u escape
// that is half of a surrogate pair, a raw control character inside a string,
// containers nested more than 128 deep, and numbers that overflow (or
// underflow) a double. A number counts as an integer when it is integral and
// at most 2^53 in magnitude.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <string_view>
#include <utility>
#include <variant>
#include <vector>

namespace mlk::json {

class Value;
using Array = std::vector<Value>;
using Object = std::vector<std::pair<std::string, Value>>;  // members in document order

class Value {
public:
    enum class Kind : uint8_t { Null, Bool, Number, String, Array, Object };

    Value() = default;
    explicit Value(bool b) : data_(b) {}
    explicit Value(double x) : data_(x) {}
    explicit Value(std::string s) : data_(std::move(s)) {}
    explicit Value(Array items) : data_(std::make_shared<const json::Array>(std::move(items))) {}
    explicit Value(Object members) : data_(std::make_shared<const json::Object>(std::move(members))) {}

    // Parses one whole document; throws std::runtime_error with the byte
    // offset of the first problem.
    static Value parse(std::string_view text);

    Kind kind() const noexcept { return static_cast<Kind>(data_.index()); }
    bool is_null() const noexcept { return kind() == Kind::Null; }
    bool is_bool() const noexcept { return kind() == Kind::Bool; }
    bool is_number() const noexcept { return kind() == Kind::Number; }
    bool is_string() const noexcept { return kind() == Kind::String; }
    bool is_array() const noexcept { return kind() == Kind::Array; }
    bool is_object() const noexcept { return kind() == Kind::Object; }

    // Each throws std::runtime_error when the value is of another kind.
    bool as_bool() const;
    double as_number() const;
    int64_t as_int() const;  // integral and |x| <= 2^53, else throws
    const std::string& as_string() const;
    const Array& as_array() const;
    const Object& as_object() const;

    // The member named `key` of an object; nullptr when absent or not an object.
    const Value* find(std::string_view key) const noexcept;

private:
    // Alternatives in the order of Kind.
    std::variant<std::monostate, bool, double, std::string, std::shared_ptr<const json::Array>,
                 std::shared_ptr<const json::Object>>
        data_;
};

}  // namespace mlk::json
