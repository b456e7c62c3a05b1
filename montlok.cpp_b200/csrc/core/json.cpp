#include "json.hpp"

#include <cmath>
#include <cstdlib>
#include <locale>
#include <sstream>
#include <stdexcept>

namespace mlk::json {

namespace {

const char* kind_text(Value::Kind k) noexcept {
    switch (k) {
        case Value::Kind::Null: return "null";
        case Value::Kind::Bool: return "bool";
        case Value::Kind::Number: return "number";
        case Value::Kind::String: return "string";
        case Value::Kind::Array: return "array";
        case Value::Kind::Object: return "object";
    }
    return "?";
}

[[noreturn]] void wrong_kind(Value::Kind want, Value::Kind have) {
    throw std::runtime_error(std::string("JSON value is ") + kind_text(have) + ", expected " + kind_text(want));
}

void put_utf8(std::string& out, uint32_t c) {
    if (c < 0x80) {
        out += static_cast<char>(c);
    } else if (c < 0x800) {
        out += static_cast<char>(0xC0 | (c >> 6));
        out += static_cast<char>(0x80 | (c & 0x3F));
    } else if (c < 0x10000) {
        out += static_cast<char>(0xE0 | (c >> 12));
        out += static_cast<char>(0x80 | ((c >> 6) & 0x3F));
        out += static_cast<char>(0x80 | (c & 0x3F));
    } else {
        out += static_cast<char>(0xF0 | (c >> 18));
        out += static_cast<char>(0x80 | ((c >> 12) & 0x3F));
        out += static_cast<char>(0x80 | ((c >> 6) & 0x3F));
        out += static_cast<char>(0x80 | (c & 0x3F));
    }
}

}  // namespace

// A recursive-descent reader over one document.
class Reader {
public:
    explicit Reader(std::string_view s) : s_(s) {}

    Value document() {
        blank();
        Value v = value(0);
        blank();
        if (i_ != s_.size()) error("trailing characters");
        return v;
    }

private:
    static constexpr int kDeepest = 128;

    [[noreturn]] void error(const char* what) const {
        throw std::runtime_error("invalid JSON at byte " + std::to_string(i_) + ": " + what);
    }

    bool at_end() const noexcept { return i_ >= s_.size(); }
    char peek() const noexcept { return s_[i_]; }

    void blank() noexcept {
        while (!at_end() && (peek() == ' ' || peek() == '\t' || peek() == '\n' || peek() == '\r')) ++i_;
    }

    bool take(char c) noexcept {
        if (!at_end() && peek() == c) {
            ++i_;
            return true;
        }
        return false;
    }

    void word(std::string_view w) {
        if (s_.compare(i_, w.size(), w) != 0) error("unexpected token");
        i_ += w.size();
    }

    Value value(int depth) {
        if (depth > kDeepest) error("nesting too deep");
        if (at_end()) error("unexpected end");
        Value v;
        switch (peek()) {
            case 'n': word("null"); return v;
            case 't':
                word("true");
                v.kind_ = Value::Kind::Bool;
                v.flag_ = true;
                return v;
            case 'f':
                word("false");
                v.kind_ = Value::Kind::Bool;
                return v;
            case '"':
                v.kind_ = Value::Kind::String;
                v.text_ = string();
                return v;
            case '[': return array(depth);
            case '{': return object(depth);
            default: return number();
        }
    }

    void digits() noexcept {
        while (!at_end() && peek() >= '0' && peek() <= '9') ++i_;
    }

    Value number() {
        const size_t begin = i_;
        take('-');
        if (at_end()) error("bad number");
        if (peek() == '0') {
            ++i_;
        } else if (peek() >= '1' && peek() <= '9') {
            digits();
        } else {
            error("bad number");
        }
        if (take('.')) {
            const size_t d = i_;
            digits();
            if (i_ == d) error("bad fraction");
        }
        if (!at_end() && (peek() == 'e' || peek() == 'E')) {
            ++i_;
            if (!take('+')) take('-');
            const size_t d = i_;
            digits();
            if (i_ == d) error("bad exponent");
        }
        // The grammar is checked; the conversion is locale-independent.
        std::istringstream in(std::string(s_.substr(begin, i_ - begin)));
        in.imbue(std::locale::classic());
        double x = 0;
        in >> x;
        if (in.fail() || !std::isfinite(x)) error("number out of range");
        Value v;
        v.kind_ = Value::Kind::Number;
        v.number_ = x;
        return v;
    }

    uint32_t hex4() {
        if (i_ + 4 > s_.size()) error("bad unicode escape");
        uint32_t c = 0;
        for (int k = 0; k < 4; ++k) {
            const char h = s_[i_++];
            c <<= 4;
            if (h >= '0' && h <= '9') c |= static_cast<uint32_t>(h - '0');
            else if (h >= 'a' && h <= 'f') c |= static_cast<uint32_t>(h - 'a' + 10);
            else if (h >= 'A' && h <= 'F') c |= static_cast<uint32_t>(h - 'A' + 10);
            else error("bad unicode escape");
        }
        return c;
    }

    std::string string() {
        ++i_;
        std::string out;
        for (;;) {
            if (at_end()) error("unterminated string");
            const auto c = static_cast<unsigned char>(s_[i_++]);
            if (c == '"') return out;
            if (c < 0x20) error("control character in string");
            if (c != '\\') {
                out += static_cast<char>(c);
                continue;
            }
            if (at_end()) error("unterminated escape");
            const char e = s_[i_++];
            switch (e) {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {
                    uint32_t c1 = hex4();
                    if (c1 >= 0xDC00 && c1 <= 0xDFFF) error("unpaired surrogate");
                    if (c1 >= 0xD800 && c1 <= 0xDBFF) {
                        if (!(take('\\') && take('u'))) error("unpaired surrogate");
                        const uint32_t c2 = hex4();
                        if (c2 < 0xDC00 || c2 > 0xDFFF) error("unpaired surrogate");
                        c1 = 0x10000 + ((c1 - 0xD800) << 10) + (c2 - 0xDC00);
                    }
                    put_utf8(out, c1);
                    break;
                }
                default: error("bad escape");
            }
        }
    }

    Value array(int depth) {
        ++i_;
        auto items = std::make_shared<Array>();
        blank();
        if (!take(']')) {
            for (;;) {
                blank();
                items->push_back(value(depth + 1));
                blank();
                if (take(']')) break;
                if (!take(',')) error("expected ',' or ']'");
            }
        }
        Value v;
        v.kind_ = Value::Kind::Array;
        v.items_ = std::move(items);
        return v;
    }

    Value object(int depth) {
        ++i_;
        auto members = std::make_shared<Object>();
        blank();
        if (!take('}')) {
            for (;;) {
                blank();
                if (at_end() || peek() != '"') error("expected member name");
                std::string key = string();
                for (const auto& m : *members) {
                    if (m.first == key) error("duplicate member name");
                }
                blank();
                if (!take(':')) error("expected ':'");
                blank();
                Value item = value(depth + 1);
                members->emplace_back(std::move(key), std::move(item));
                blank();
                if (take('}')) break;
                if (!take(',')) error("expected ',' or '}'");
            }
        }
        Value v;
        v.kind_ = Value::Kind::Object;
        v.members_ = std::move(members);
        return v;
    }

    std::string_view s_;
    size_t i_ = 0;
};

Value Value::parse(std::string_view text) { return Reader(text).document(); }

bool Value::as_bool() const {
    if (kind_ != Kind::Bool) wrong_kind(Kind::Bool, kind_);
    return flag_;
}

double Value::as_number() const {
    if (kind_ != Kind::Number) wrong_kind(Kind::Number, kind_);
    return number_;
}

int64_t Value::as_int() const {
    const double x = as_number();
    if (std::nearbyint(x) != x || std::fabs(x) > 9007199254740992.0) {
        throw std::runtime_error("JSON number is not an exact integer");
    }
    return static_cast<int64_t>(x);
}

const std::string& Value::as_string() const {
    if (kind_ != Kind::String) wrong_kind(Kind::String, kind_);
    return text_;
}

const Array& Value::as_array() const {
    if (kind_ != Kind::Array) wrong_kind(Kind::Array, kind_);
    return *items_;
}

const Object& Value::as_object() const {
    if (kind_ != Kind::Object) wrong_kind(Kind::Object, kind_);
    return *members_;
}

const Value* Value::find(std::string_view key) const noexcept {
    if (kind_ != Kind::Object) return nullptr;
    for (const auto& m : *members_) {
        if (m.first == key) return &m.second;
    }
    return nullptr;
}

}  // namespace mlk::json
