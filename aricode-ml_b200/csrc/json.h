// json.h — minimal JSON DOM for reading the launch plan (objects, arrays,
// strings, numbers, booleans, null). Throws std::runtime_error on malformed input.
#pragma once
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace b2json {

struct Value {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    double num = 0.0;
    std::string str;
    std::vector<Value> arr;
    std::map<std::string, Value> obj;

    bool is_null() const { return kind == Null; }
    bool has(const std::string& k) const { return kind == Object && obj.count(k) && !obj.at(k).is_null(); }
    const Value& operator[](const std::string& k) const {
        static const Value null_v;
        if (kind != Object) throw std::runtime_error("plan: expected an object for key '" + k + "'");
        auto it = obj.find(k);
        return it == obj.end() ? null_v : it->second;
    }
    const Value& operator[](size_t i) const {
        if (kind != Array || i >= arr.size()) throw std::runtime_error("plan: array index out of range");
        return arr[i];
    }
    size_t size() const { return kind == Array ? arr.size() : (kind == Object ? obj.size() : 0); }
    double as_num(const char* what = "") const {
        if (kind != Number) throw std::runtime_error(std::string("plan: expected a number ") + what);
        return num;
    }
    long long as_int(const char* what = "") const { return (long long)as_num(what); }
    const std::string& as_str(const char* what = "") const {
        if (kind != String) throw std::runtime_error(std::string("plan: expected a string ") + what);
        return str;
    }
    bool as_bool() const { return kind == Bool ? b : (kind == Number ? num != 0 : false); }
};

class Parser {
  public:
    explicit Parser(const std::string& s) : s_(s) {}
    Value parse() {
        Value v = value();
        ws();
        if (i_ != s_.size()) fail("trailing characters");
        return v;
    }

  private:
    const std::string& s_;
    size_t i_ = 0;

    [[noreturn]] void fail(const char* m) {
        throw std::runtime_error(std::string("plan JSON: ") + m + " at offset " + std::to_string(i_));
    }
    void ws() { while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_; }
    bool lit(const char* w) {
        size_t n = std::char_traits<char>::length(w);
        if (s_.compare(i_, n, w) == 0) { i_ += n; return true; }
        return false;
    }
    Value value() {
        ws();
        if (i_ >= s_.size()) fail("unexpected end");
        Value v;
        char c = s_[i_];
        if (c == '{') {
            v.kind = Value::Object; ++i_; ws();
            if (i_ < s_.size() && s_[i_] == '}') { ++i_; return v; }
            for (;;) {
                ws();
                Value k = value();
                if (k.kind != Value::String) fail("object key must be a string");
                ws();
                if (i_ >= s_.size() || s_[i_] != ':') fail("expected ':'");
                ++i_;
                v.obj[k.str] = value();
                ws();
                if (i_ < s_.size() && s_[i_] == ',') { ++i_; continue; }
                if (i_ < s_.size() && s_[i_] == '}') { ++i_; return v; }
                fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            v.kind = Value::Array; ++i_; ws();
            if (i_ < s_.size() && s_[i_] == ']') { ++i_; return v; }
            for (;;) {
                v.arr.push_back(value());
                ws();
                if (i_ < s_.size() && s_[i_] == ',') { ++i_; continue; }
                if (i_ < s_.size() && s_[i_] == ']') { ++i_; return v; }
                fail("expected ',' or ']'");
            }
        }
        if (c == '"') {
            v.kind = Value::String; ++i_;
            while (i_ < s_.size() && s_[i_] != '"') {
                if (s_[i_] == '\\') {
                    ++i_;
                    if (i_ >= s_.size()) fail("bad escape");
                    char e = s_[i_];
                    if (e == 'n') v.str += '\n'; else if (e == 't') v.str += '\t';
                    else if (e == 'u') { v.str += '?'; i_ += 4; }
                    else v.str += e;
                    ++i_;
                } else {
                    v.str += s_[i_++];
                }
            }
            if (i_ >= s_.size()) fail("unterminated string");
            ++i_;
            return v;
        }
        if (lit("true")) { v.kind = Value::Bool; v.b = true; return v; }
        if (lit("false")) { v.kind = Value::Bool; v.b = false; return v; }
        if (lit("null")) { v.kind = Value::Null; return v; }
        if (lit("NaN") || lit("Infinity")) fail("non-finite numbers are not valid JSON");
        char* end = nullptr;
        v.kind = Value::Number;
        v.num = std::strtod(s_.c_str() + i_, &end);
        if (end == s_.c_str() + i_) fail("unexpected character");
        i_ = (size_t)(end - s_.c_str());
        return v;
    }
};

inline Value parse(const std::string& s) { return Parser(s).parse(); }

}  // namespace b2json
