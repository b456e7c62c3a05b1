// JSON parser: a tokenizer and a table of open containers (no recursion, so
// deep documents cannot exhaust the stack; the depth limit is a rule of the
// format, not of this implementation).
#include "json.hpp"

#include <charconv>
#include <clocale>
#include <cmath>
#include <cstdlib>
#include <stdexcept>
#include <unordered_set>

namespace mlk::json {

namespace {

constexpr size_t kMaxDepth = 128;  // a value may sit inside at most 128 containers

[[noreturn]] void reject(size_t at, const std::string& why) {
    throw std::runtime_error("malformed JSON (offset " + std::to_string(at) + "): " + why);
}

enum class Tok : uint8_t { End, BeginObject, EndObject, BeginArray, EndArray, Colon, Comma, Str, Num, True, False, Null };

// Splits the text into tokens; string tokens are unescaped into `text`,
// number tokens converted into `number`.
class Tokenizer {
public:
    explicit Tokenizer(std::string_view s) : s_(s) {}

    size_t offset() const noexcept { return start_; }

    Tok next(std::string& text, double& number) {
        while (pos_ < s_.size() && (s_[pos_] == ' ' || s_[pos_] == '\n' || s_[pos_] == '\r' || s_[pos_] == '\t')) {
            ++pos_;
        }
        start_ = pos_;
        if (pos_ == s_.size()) return Tok::End;
        const char c = s_[pos_];
        switch (c) {
            case '{': ++pos_; return Tok::BeginObject;
            case '}': ++pos_; return Tok::EndObject;
            case '[': ++pos_; return Tok::BeginArray;
            case ']': ++pos_; return Tok::EndArray;
            case ':': ++pos_; return Tok::Colon;
            case ',': ++pos_; return Tok::Comma;
            case '"': read_string(text); return Tok::Str;
            case 't': literal("true"); return Tok::True;
            case 'f': literal("false"); return Tok::False;
            case 'n': literal("null"); return Tok::Null;
            default:
                if (c == '-' || (c >= '0' && c <= '9')) {
                    number = read_number();
                    return Tok::Num;
                }
                reject(pos_, std::string("unexpected character '") + c + "'");
        }
    }

private:
    void literal(std::string_view word) {
        if (s_.substr(pos_, word.size()) != word) reject(pos_, "unknown literal");
        pos_ += word.size();
    }

    size_t run_of_digits() noexcept {
        const size_t from = pos_;
        while (pos_ < s_.size() && s_[pos_] >= '0' && s_[pos_] <= '9') ++pos_;
        return pos_ - from;
    }

    // number = [-] (0 | [1-9][0-9]*) [. [0-9]+] [(e|E) [+|-] [0-9]+]
    double read_number() {
        const size_t from = pos_;
        if (s_[pos_] == '-') ++pos_;
        if (pos_ < s_.size() && s_[pos_] == '0') {
            ++pos_;
        } else if (run_of_digits() == 0) {
            reject(from, "a number needs digits");
        }
        if (pos_ < s_.size() && s_[pos_] == '.') {
            ++pos_;
            if (run_of_digits() == 0) reject(from, "a number needs digits after '.'");
        }
        if (pos_ < s_.size() && (s_[pos_] == 'e' || s_[pos_] == 'E')) {
            ++pos_;
            if (pos_ < s_.size() && (s_[pos_] == '+' || s_[pos_] == '-')) ++pos_;
            if (run_of_digits() == 0) reject(from, "a number needs exponent digits");
        }
        double x = 0.0;
        const char* first = s_.data() + from;
        const char* last = s_.data() + pos_;
        const auto [end, ec] = std::from_chars(first, last, x);
        if (ec == std::errc::result_out_of_range) {
            // Too large, or too small: a number below the smallest subnormal
            // reads as the C library reads it (0 or the subnormal), as the
            // reference loader does; only overflow is an error.
            static const locale_t c_locale = newlocale(LC_ALL_MASK, "C", nullptr);
            const std::string token(first, last);
            x = strtod_l(token.c_str(), nullptr, c_locale);
        } else if (ec != std::errc() || end != last) {
            reject(from, "not a number");
        }
        if (!std::isfinite(x)) reject(from, "number does not fit a double");
        return x;
    }

    unsigned hex_unit() {
        if (s_.size() - pos_ < 4) reject(pos_, "short \\u escape");
        unsigned u = 0;
        for (int i = 0; i < 4; ++i) {
            const char h = s_[pos_++];
            const int d = (h >= '0' && h <= '9') ? h - '0'
                        : (h >= 'a' && h <= 'f') ? h - 'a' + 10
                        : (h >= 'A' && h <= 'F') ? h - 'A' + 10
                                                 : -1;
            if (d < 0) reject(pos_ - 1, "bad hex digit in \\u escape");
            u = u * 16 + static_cast<unsigned>(d);
        }
        return u;
    }

    static void append_utf8(std::string& out, unsigned cp) {
        if (cp < 0x80) {
            out.push_back(static_cast<char>(cp));
            return;
        }
        // Lead byte and continuation bytes, 6 payload bits each.
        const int tail = cp < 0x800 ? 1 : cp < 0x10000 ? 2 : 3;
        static const unsigned char lead[] = {0, 0xC0, 0xE0, 0xF0};
        out.push_back(static_cast<char>(lead[tail] | (cp >> (6 * tail))));
        for (int k = tail - 1; k >= 0; --k) out.push_back(static_cast<char>(0x80 | ((cp >> (6 * k)) & 0x3F)));
    }

    void read_string(std::string& out) {
        out.clear();
        const size_t open = pos_++;
        for (;;) {
            if (pos_ >= s_.size()) reject(open, "string never closed");
            const auto c = static_cast<unsigned char>(s_[pos_++]);
            if (c == '"') return;
            if (c < 0x20) reject(pos_ - 1, "raw control character in string");
            if (c != '\\') {
                out.push_back(static_cast<char>(c));
                continue;
            }
            if (pos_ >= s_.size()) reject(open, "string never closed");
            const char e = s_[pos_++];
            static const std::string_view simple = "\"\\/bfnrt", meaning = "\"\\/\b\f\n\r\t";
            if (const size_t k = simple.find(e); k != std::string_view::npos) {
                out.push_back(meaning[k]);
                continue;
            }
            if (e != 'u') reject(pos_ - 1, "unknown escape");
            unsigned cp = hex_unit();
            if (cp >= 0xDC00 && cp <= 0xDFFF) reject(pos_ - 6, "low surrogate without a high one");
            if (cp >= 0xD800 && cp <= 0xDBFF) {
                if (s_.substr(pos_, 2) != "\\u") reject(pos_, "high surrogate without a low one");
                pos_ += 2;
                const unsigned low = hex_unit();
                if (low < 0xDC00 || low > 0xDFFF) reject(pos_ - 6, "high surrogate without a low one");
                cp = 0x10000 + (((cp & 0x3FF) << 10) | (low & 0x3FF));
            }
            append_utf8(out, cp);
        }
    }

    std::string_view s_;
    size_t pos_ = 0, start_ = 0;
};

// A container being filled: its members so far (objects also keep the
// names seen and the name waiting for its value).
struct Open {
    bool object;
    Array items;
    Object members;
    std::unordered_set<std::string> names;
    std::string name;
};

}  // namespace

Value Value::parse(std::string_view text) {
    Tokenizer tokens(text);
    std::vector<Open> open;
    std::string str;
    double num = 0.0;
    Value root;
    bool have_root = false;

    // Where the grammar stands, per the innermost container: just opened,
    // after a member name, after ':' or ',', or after a complete value.
    enum class At { Start, Opened, Name, Colon, Comma, Value };
    At at = At::Start;

    // Hands a finished value to the innermost container, or makes it the root.
    auto deliver = [&](Value v) {
        if (open.empty()) {
            root = std::move(v);
            have_root = true;
        } else if (open.back().object) {
            open.back().members.emplace_back(std::move(open.back().name), std::move(v));
        } else {
            open.back().items.push_back(std::move(v));
        }
        at = At::Value;
    };

    for (;;) {
        const Tok t = tokens.next(str, num);
        const size_t where = tokens.offset();
        if (have_root) {
            if (t != Tok::End) reject(where, "text after the document");
            return root;
        }
        const bool in_object = !open.empty() && open.back().object;
        const bool value_ok = at == At::Start || at == At::Colon || (!in_object && (at == At::Opened || at == At::Comma));
        const bool too_deep = open.size() > kMaxDepth;  // for a value arriving now
        switch (t) {
            case Tok::End: reject(where, "document ends early");
            case Tok::BeginObject:
            case Tok::BeginArray:
                if (!value_ok) reject(where, "a value is not allowed here");
                if (too_deep) reject(where, "containers nested too deep");
                open.push_back(Open{t == Tok::BeginObject, {}, {}, {}, {}});
                at = At::Opened;
                break;
            case Tok::EndObject:
            case Tok::EndArray: {
                const bool closes_object = t == Tok::EndObject;
                if (open.empty() || open.back().object != closes_object || !(at == At::Opened || at == At::Value)) {
                    reject(where, "unexpected closing bracket");
                }
                Open done = std::move(open.back());
                open.pop_back();
                deliver(done.object ? Value(std::move(done.members)) : Value(std::move(done.items)));
                break;
            }
            case Tok::Colon:
                if (!in_object || at != At::Name) reject(where, "unexpected ':'");
                at = At::Colon;
                break;
            case Tok::Comma:
                if (open.empty() || at != At::Value) reject(where, "unexpected ','");
                at = At::Comma;
                break;
            case Tok::Str:
                if (in_object && (at == At::Opened || at == At::Comma)) {
                    if (!open.back().names.insert(str).second) reject(where, "member \"" + str + "\" named twice");
                    open.back().name = str;
                    at = At::Name;
                    break;
                }
                if (!value_ok) reject(where, "a value is not allowed here");
                if (too_deep) reject(where, "containers nested too deep");
                deliver(Value(str));
                break;
            case Tok::Num:
            case Tok::True:
            case Tok::False:
            case Tok::Null:
                if (!value_ok) reject(where, "a value is not allowed here");
                if (too_deep) reject(where, "containers nested too deep");
                deliver(t == Tok::Num ? Value(num) : t == Tok::Null ? Value() : Value(t == Tok::True));
                break;
        }
    }
}

namespace {

const char* kind_name(Value::Kind k) noexcept {
    static const char* names[] = {"null", "a boolean", "a number", "a string", "an array", "an object"};
    return names[static_cast<int>(k)];
}

[[noreturn]] void not_a(Value::Kind want, Value::Kind got) {
    throw std::runtime_error(std::string("expected ") + kind_name(want) + " in JSON, found " + kind_name(got));
}

}  // namespace

bool Value::as_bool() const {
    if (!is_bool()) not_a(Kind::Bool, kind());
    return std::get<bool>(data_);
}

double Value::as_number() const {
    if (!is_number()) not_a(Kind::Number, kind());
    return std::get<double>(data_);
}

int64_t Value::as_int() const {
    const double x = as_number();
    constexpr double kExact = 9007199254740992.0;  // 2^53
    if (!(std::fabs(x) <= kExact) || std::trunc(x) != x) throw std::runtime_error("JSON number is not an integer");
    return static_cast<int64_t>(x);
}

const std::string& Value::as_string() const {
    if (!is_string()) not_a(Kind::String, kind());
    return std::get<std::string>(data_);
}

const Array& Value::as_array() const {
    if (!is_array()) not_a(Kind::Array, kind());
    return *std::get<std::shared_ptr<const Array>>(data_);
}

const Object& Value::as_object() const {
    if (!is_object()) not_a(Kind::Object, kind());
    return *std::get<std::shared_ptr<const Object>>(data_);
}

const Value* Value::find(std::string_view key) const noexcept {
    if (!is_object()) return nullptr;
    for (const auto& [name, value] : *std::get<std::shared_ptr<const Object>>(data_)) {
        if (name == key) return &value;
    }
    return nullptr;
}

}  // namespace mlk::json
