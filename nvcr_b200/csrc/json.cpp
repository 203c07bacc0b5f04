#include "json.hpp"

#include <cerrno>
#include <cstdlib>
#include <cstring>

namespace nvcr_sm100::json {

const Value* Value::get(std::string_view key) const {
    if (kind != Kind::object) return nullptr;
    auto found = members.find(key);
    return found == members.end() ? nullptr : &found->second;
}

namespace {

constexpr int max_depth = 64;

class Reader {
public:
    explicit Reader(std::string_view text) : s_(text) {}

    Result<Value> document() {
        auto value = read(0);
        if (!value) return value;
        skip();
        if (at_ < s_.size()) return bad("trailing characters after the document");
        return value;
    }

private:
    std::string_view s_;
    std::size_t at_{0};

    Error bad(const std::string& what) const {
        return fail(Code::invalid_argument, "JSON: " + what + " at byte " + std::to_string(at_));
    }

    void skip() {
        while (at_ < s_.size() && (s_[at_] == ' ' || s_[at_] == '\t' || s_[at_] == '\n' || s_[at_] == '\r')) ++at_;
    }

    bool eat(char c) {
        skip();
        if (at_ < s_.size() && s_[at_] == c) {
            ++at_;
            return true;
        }
        return false;
    }

    Result<Value> read(int depth) {
        if (depth > max_depth) return bad("nesting is too deep");
        skip();
        if (at_ >= s_.size()) return bad("unexpected end");
        const char c = s_[at_];
        if (c == '{') return object(depth);
        if (c == '[') return array(depth);
        if (c == '"') {
            auto text = string();
            if (!text) return text.error();
            Value v;
            v.kind = Value::Kind::string;
            v.text = std::move(text.value());
            return v;
        }
        if (c == 't') return literal("true", Value::Kind::boolean, true);
        if (c == 'f') return literal("false", Value::Kind::boolean, false);
        if (c == 'n') return literal("null", Value::Kind::null, false);
        if (c == '-' || (c >= '0' && c <= '9')) return number();
        return bad("unexpected character");
    }

    Result<Value> literal(std::string_view word, Value::Kind kind, bool flag) {
        if (s_.substr(at_, word.size()) != word) return bad("invalid literal");
        at_ += word.size();
        Value v;
        v.kind = kind;
        v.boolean = flag;
        return v;
    }

    Result<Value> object(int depth) {
        ++at_;
        Value v;
        v.kind = Value::Kind::object;
        if (eat('}')) return v;
        while (true) {
            skip();
            if (at_ >= s_.size() || s_[at_] != '"') return bad("object key must be a string");
            auto key = string();
            if (!key) return key.error();
            if (!eat(':')) return bad("missing ':' after an object key");
            auto member = read(depth + 1);
            if (!member) return member;
            if (v.members.count(key.value()) != 0) return bad("duplicate object key '" + key.value() + "'");
            v.members.emplace(std::move(key.value()), std::move(member.value()));
            if (eat('}')) return v;
            if (!eat(',')) return bad("missing ',' between object members");
        }
    }

    Result<Value> array(int depth) {
        ++at_;
        Value v;
        v.kind = Value::Kind::array;
        if (eat(']')) return v;
        while (true) {
            auto item = read(depth + 1);
            if (!item) return item;
            v.items.push_back(std::move(item.value()));
            if (eat(']')) return v;
            if (!eat(',')) return bad("missing ',' between array items");
        }
    }

    static void append_utf8(std::string& out, std::uint32_t code) {
        if (code < 0x80) {
            out.push_back(static_cast<char>(code));
        } else if (code < 0x800) {
            out.push_back(static_cast<char>(0xC0 | (code >> 6)));
            out.push_back(static_cast<char>(0x80 | (code & 0x3F)));
        } else if (code < 0x10000) {
            out.push_back(static_cast<char>(0xE0 | (code >> 12)));
            out.push_back(static_cast<char>(0x80 | ((code >> 6) & 0x3F)));
            out.push_back(static_cast<char>(0x80 | (code & 0x3F)));
        } else {
            out.push_back(static_cast<char>(0xF0 | (code >> 18)));
            out.push_back(static_cast<char>(0x80 | ((code >> 12) & 0x3F)));
            out.push_back(static_cast<char>(0x80 | ((code >> 6) & 0x3F)));
            out.push_back(static_cast<char>(0x80 | (code & 0x3F)));
        }
    }

    Result<std::uint32_t> hex4() {
        if (at_ + 4 > s_.size()) return bad("short \\u escape");
        std::uint32_t code = 0;
        for (int i = 0; i < 4; ++i) {
            const char h = s_[at_++];
            code <<= 4;
            if (h >= '0' && h <= '9') code |= static_cast<std::uint32_t>(h - '0');
            else if (h >= 'a' && h <= 'f') code |= static_cast<std::uint32_t>(h - 'a' + 10);
            else if (h >= 'A' && h <= 'F') code |= static_cast<std::uint32_t>(h - 'A' + 10);
            else return bad("invalid \\u escape");
        }
        return code;
    }

    Result<std::string> string() {
        ++at_;  // opening quote
        std::string out;
        while (true) {
            if (at_ >= s_.size()) return bad("unterminated string");
            const char c = s_[at_++];
            if (c == '"') return out;
            if (static_cast<unsigned char>(c) < 0x20) return bad("control character in a string");
            if (c != '\\') {
                out.push_back(c);
                continue;
            }
            if (at_ >= s_.size()) return bad("unterminated escape");
            const char e = s_[at_++];
            switch (e) {
            case '"': out.push_back('"'); break;
            case '\\': out.push_back('\\'); break;
            case '/': out.push_back('/'); break;
            case 'b': out.push_back('\b'); break;
            case 'f': out.push_back('\f'); break;
            case 'n': out.push_back('\n'); break;
            case 'r': out.push_back('\r'); break;
            case 't': out.push_back('\t'); break;
            case 'u': {
                auto code = hex4();
                if (!code) return code.error();
                std::uint32_t value = code.value();
                if (value >= 0xD800 && value <= 0xDBFF) {
                    if (at_ + 2 > s_.size() || s_[at_] != '\\' || s_[at_ + 1] != 'u') return bad("lone surrogate");
                    at_ += 2;
                    auto low = hex4();
                    if (!low) return low.error();
                    if (low.value() < 0xDC00 || low.value() > 0xDFFF) return bad("invalid surrogate pair");
                    value = 0x10000 + ((value - 0xD800) << 10) + (low.value() - 0xDC00);
                } else if (value >= 0xDC00 && value <= 0xDFFF) {
                    return bad("lone surrogate");
                }
                append_utf8(out, value);
                break;
            }
            default:
                return bad("invalid escape");
            }
        }
    }

    Result<Value> number() {
        const std::size_t start = at_;
        bool integral = true;
        if (s_[at_] == '-') ++at_;
        if (at_ >= s_.size() || !(s_[at_] >= '0' && s_[at_] <= '9')) return bad("invalid number");
        if (s_[at_] == '0' && at_ + 1 < s_.size() && s_[at_ + 1] >= '0' && s_[at_ + 1] <= '9') {
            return bad("leading zero in a number");
        }
        while (at_ < s_.size() && s_[at_] >= '0' && s_[at_] <= '9') ++at_;
        if (at_ < s_.size() && s_[at_] == '.') {
            integral = false;
            ++at_;
            if (at_ >= s_.size() || !(s_[at_] >= '0' && s_[at_] <= '9')) return bad("invalid fraction");
            while (at_ < s_.size() && s_[at_] >= '0' && s_[at_] <= '9') ++at_;
        }
        if (at_ < s_.size() && (s_[at_] == 'e' || s_[at_] == 'E')) {
            integral = false;
            ++at_;
            if (at_ < s_.size() && (s_[at_] == '+' || s_[at_] == '-')) ++at_;
            if (at_ >= s_.size() || !(s_[at_] >= '0' && s_[at_] <= '9')) return bad("invalid exponent");
            while (at_ < s_.size() && s_[at_] >= '0' && s_[at_] <= '9') ++at_;
        }
        const std::string token(s_.substr(start, at_ - start));
        Value v;
        v.kind = Value::Kind::number;
        // strtod is correctly rounded in glibc and locale-independent here
        // because the token holds only digits, sign, '.', and exponent.
        v.number = std::strtod(token.c_str(), nullptr);
        if (integral) {
            errno = 0;
            char* end = nullptr;
            const long long parsed = std::strtoll(token.c_str(), &end, 10);
            if (errno == 0 && end != nullptr && *end == '\0') v.integer = parsed;
        }
        return v;
    }
};

}  // namespace

Result<Value> parse(std::string_view document) { return Reader(document).document(); }

}  // namespace nvcr_sm100::json
