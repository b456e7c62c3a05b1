// Strict JSON (RFC 8259) values for safetensors headers and model specs.
//
// Acceptance follows the reference loader (montlok.cpp src/core/json.cpp):
// duplicate member names, unpaired surrogates, control characters in strings,
// nesting deeper than 128 and numbers that do not fit a finite double are
// errors; integers are "exact" when integral with magnitude <= 2^53.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <string_view>
#include <utility>
#include <vector>

namespace mlk::json {

class Value;
using Array = std::vector<Value>;
using Object = std::vector<std::pair<std::string, Value>>;

class Value {
public:
    enum class Kind : uint8_t { Null, Bool, Number, String, Array, Object };

    Value() = default;

    // Parses a whole document; throws std::runtime_error naming the byte
    // offset of the first problem.
    static Value parse(std::string_view text);

    Kind kind() const noexcept { return kind_; }
    bool is_null() const noexcept { return kind_ == Kind::Null; }
    bool is_bool() const noexcept { return kind_ == Kind::Bool; }
    bool is_number() const noexcept { return kind_ == Kind::Number; }
    bool is_string() const noexcept { return kind_ == Kind::String; }
    bool is_array() const noexcept { return kind_ == Kind::Array; }
    bool is_object() const noexcept { return kind_ == Kind::Object; }

    // Each throws std::runtime_error when the value has another kind.
    bool as_bool() const;
    double as_number() const;
    int64_t as_int() const;  // integral and |x| <= 2^53, else throws
    const std::string& as_string() const;
    const Array& as_array() const;
    const Object& as_object() const;

    // The member named `key` of an object; nullptr when absent or not an object.
    const Value* find(std::string_view key) const noexcept;

private:
    friend class Reader;
    Kind kind_ = Kind::Null;
    bool flag_ = false;
    double number_ = 0;
    std::string text_;
    std::shared_ptr<const Array> items_;
    std::shared_ptr<const Object> members_;
};

}  // namespace mlk::json
