#pragma once

// Minimal JSON reader for pack manifests (OpWorks include/runtime/json.cuh
// API: json::parse, Value::at / find / as_* / is_null). Recursive descent over
// the whole manifest string; numbers keep both a double and, when integral,
// an exact int64 (tensor offsets exceed 2^53 only in absurd packs, which the
// pack reader rejects anyway).

#include <cstdint>
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace opworks::json {

class Value {
  public:
    enum class Kind { kNull, kBool, kNumber, kString, kArray, kObject };
    using Array = std::vector<Value>;
    using Object = std::map<std::string, Value>;

    Value() = default;
    static Value null() { return Value(); }

    Kind kind() const { return kind_; }
    bool is_null() const { return kind_ == Kind::kNull; }

    bool as_bool() const {
        expect(Kind::kBool, "bool");
        return b_;
    }
    double as_number() const {
        expect(Kind::kNumber, "number");
        return num_;
    }
    int64_t as_int() const {
        expect(Kind::kNumber, "number");
        if (!integral_)
            throw std::runtime_error("json: expected an integer");
        return int_;
    }
    const std::string &as_string() const {
        expect(Kind::kString, "string");
        return str_;
    }
    const Array &as_array() const {
        expect(Kind::kArray, "array");
        return *arr_;
    }
    const Object &as_object() const {
        expect(Kind::kObject, "object");
        return *obj_;
    }
    const Value &at(const std::string &key) const {
        const Value *v = find(key);
        if (!v)
            throw std::runtime_error("json: missing key '" + key + "'");
        return *v;
    }
    const Value *find(const std::string &key) const {
        if (kind_ != Kind::kObject)
            return nullptr;
        auto it = obj_->find(key);
        return it == obj_->end() ? nullptr : &it->second;
    }

  private:
    friend class Parser;
    void expect(Kind k, const char *what) const {
        if (kind_ != k)
            throw std::runtime_error(std::string("json: expected ") + what);
    }
    Kind kind_ = Kind::kNull;
    bool b_ = false;
    double num_ = 0.0;
    int64_t int_ = 0;
    bool integral_ = false;
    std::string str_;
    std::shared_ptr<Array> arr_;
    std::shared_ptr<Object> obj_;
};

class Parser {
  public:
    explicit Parser(const std::string &s) : s_(s) {}

    Value parse_document() {
        Value v = parse_value(0);
        skip_ws();
        if (i_ != s_.size())
            fail("trailing characters");
        return v;
    }

  private:
    [[noreturn]] void fail(const char *msg) const {
        throw std::runtime_error(std::string("json: ") + msg + " at offset " + std::to_string(i_));
    }
    void skip_ws() {
        while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t'))
            ++i_;
    }
    bool consume(const char *lit) {
        size_t n = 0;
        while (lit[n])
            ++n;
        if (s_.compare(i_, n, lit) == 0) {
            i_ += n;
            return true;
        }
        return false;
    }

    Value parse_value(int depth) {
        if (depth > 64)
            fail("nesting too deep");
        skip_ws();
        if (i_ >= s_.size())
            fail("unexpected end");
        Value v;
        const char c = s_[i_];
        if (c == '{') {
            ++i_;
            v.kind_ = Value::Kind::kObject;
            v.obj_ = std::make_shared<Value::Object>();
            skip_ws();
            if (i_ < s_.size() && s_[i_] == '}') {
                ++i_;
                return v;
            }
            while (true) {
                skip_ws();
                if (i_ >= s_.size() || s_[i_] != '"')
                    fail("expected key");
                std::string key = parse_string();
                skip_ws();
                if (i_ >= s_.size() || s_[i_] != ':')
                    fail("expected ':'");
                ++i_;
                (*v.obj_)[key] = parse_value(depth + 1);
                skip_ws();
                if (i_ < s_.size() && s_[i_] == ',') {
                    ++i_;
                    continue;
                }
                if (i_ < s_.size() && s_[i_] == '}') {
                    ++i_;
                    return v;
                }
                fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            ++i_;
            v.kind_ = Value::Kind::kArray;
            v.arr_ = std::make_shared<Value::Array>();
            skip_ws();
            if (i_ < s_.size() && s_[i_] == ']') {
                ++i_;
                return v;
            }
            while (true) {
                v.arr_->push_back(parse_value(depth + 1));
                skip_ws();
                if (i_ < s_.size() && s_[i_] == ',') {
                    ++i_;
                    continue;
                }
                if (i_ < s_.size() && s_[i_] == ']') {
                    ++i_;
                    return v;
                }
                fail("expected ',' or ']'");
            }
        }
        if (c == '"') {
            v.kind_ = Value::Kind::kString;
            v.str_ = parse_string();
            return v;
        }
        if (consume("true")) {
            v.kind_ = Value::Kind::kBool;
            v.b_ = true;
            return v;
        }
        if (consume("false")) {
            v.kind_ = Value::Kind::kBool;
            return v;
        }
        if (consume("null"))
            return v;
        return parse_number();
    }

    std::string parse_string() {
        ++i_; // opening quote
        std::string out;
        while (i_ < s_.size() && s_[i_] != '"') {
            char c = s_[i_++];
            if (c == '\\') {
                if (i_ >= s_.size())
                    fail("bad escape");
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
                    if (i_ + 4 > s_.size())
                        fail("bad \\u escape");
                    const unsigned cp = static_cast<unsigned>(std::strtoul(s_.substr(i_, 4).c_str(), nullptr, 16));
                    i_ += 4;
                    if (cp < 0x80) {
                        out += static_cast<char>(cp);
                    } else if (cp < 0x800) {
                        out += static_cast<char>(0xC0 | (cp >> 6));
                        out += static_cast<char>(0x80 | (cp & 0x3F));
                    } else {
                        out += static_cast<char>(0xE0 | (cp >> 12));
                        out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
                        out += static_cast<char>(0x80 | (cp & 0x3F));
                    }
                    break;
                }
                default: fail("bad escape");
                }
            } else {
                out += c;
            }
        }
        if (i_ >= s_.size())
            fail("unterminated string");
        ++i_;
        return out;
    }

    Value parse_number() {
        const size_t start = i_;
        if (i_ < s_.size() && (s_[i_] == '-' || s_[i_] == '+'))
            ++i_;
        bool integral = true;
        while (i_ < s_.size()) {
            const char c = s_[i_];
            if (c >= '0' && c <= '9') {
                ++i_;
            } else if (c == '.' || c == 'e' || c == 'E' || c == '-' || c == '+') {
                integral = false;
                ++i_;
            } else {
                break;
            }
        }
        if (i_ == start)
            fail("unexpected character");
        const std::string tok = s_.substr(start, i_ - start);
        Value v;
        v.kind_ = Value::Kind::kNumber;
        char *end = nullptr;
        v.num_ = std::strtod(tok.c_str(), &end);
        if (end == tok.c_str())
            fail("bad number");
        if (integral) {
            v.integral_ = true;
            v.int_ = std::strtoll(tok.c_str(), nullptr, 10);
        } else if (v.num_ == static_cast<double>(static_cast<int64_t>(v.num_))) {
            v.integral_ = true;
            v.int_ = static_cast<int64_t>(v.num_);
        }
        return v;
    }

    const std::string &s_;
    size_t i_ = 0;
};

inline Value parse(const std::string &text) { return Parser(text).parse_document(); }

} // namespace opworks::json
