// utils.h — schedule rules of the heteromm deploy layer (B200 build).
//
// Interface of the reference's deploy/utils.h: ScheduleConfig holds three
// lists of interval rules, read from a JSON file shaped like deploy/schedule.json,
// and returns the kernel names ("cpu" / "gpu" / "fpga") of the first rule whose
// upper bounds (-1: unbounded) admit the given sizes; no matching rule throws
// std::runtime_error.  The reference reads the file with a vendored third-party
// JSON library; this build carries its own small reader (JsonValue below) and
// names it `json` so `ScheduleConfig::load_from_json(json)` keeps its spelling.
// Two fixes: get_build_memory_config takes the one size its rule has (the
// reference's caller passes two, memory_manager.h:304), and rules whose
// `config` lists are shorter than their step count are rejected on load (the
// reference would index past them).
#ifndef HETEROMM_B200_DEPLOY_UTILS_H_
#define HETEROMM_B200_DEPLOY_UTILS_H_

#include <cerrno>
#include <cstdint>
#include <cstdlib>
#include <fstream>
#include <limits>
#include <sstream>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace heteromm {
namespace deploy {

// A parsed JSON document (RFC 8259): null, boolean, number, string, array or
// object.  Parsing rejects anything outside the grammar with
// std::runtime_error naming the byte offset; nesting is limited to 256 levels.
class JsonValue {
public:
    enum class Kind { Null, Bool, Number, String, Array, Object };

    static JsonValue parse(const std::string& text) {
        Parser p{text, 0};
        p.skip_ws();
        JsonValue v = p.value(0);
        p.skip_ws();
        if (p.i != text.size()) p.fail("trailing characters after the document");
        return v;
    }

    Kind kind() const { return kind_; }
    bool is_null() const { return kind_ == Kind::Null; }
    bool is_array() const { return kind_ == Kind::Array; }
    bool is_object() const { return kind_ == Kind::Object; }

    // Object member access; a later duplicate key wins.
    bool contains(const std::string& key) const { return find(key) != nullptr; }
    const JsonValue& operator[](const std::string& key) const {
        if (kind_ != Kind::Object) throw std::runtime_error("json: not an object (key '" + key + "')");
        const JsonValue* v = find(key);
        if (!v) throw std::runtime_error("json: missing key '" + key + "'");
        return *v;
    }
    const JsonValue& operator[](const char* key) const { return (*this)[std::string(key)]; }

    // Array element access and iteration (arrays only).
    const JsonValue& operator[](size_t i) const {
        if (kind_ != Kind::Array) throw std::runtime_error("json: not an array");
        if (i >= arr_.size()) throw std::runtime_error("json: array index out of range");
        return arr_[i];
    }
    const JsonValue& operator[](int i) const {
        if (i < 0) throw std::runtime_error("json: negative array index");
        return (*this)[static_cast<size_t>(i)];
    }
    size_t size() const {
        return kind_ == Kind::Array ? arr_.size() : kind_ == Kind::Object ? obj_.size() : 0;
    }
    std::vector<JsonValue>::const_iterator begin() const { return array_ref().begin(); }
    std::vector<JsonValue>::const_iterator end() const { return array_ref().end(); }

    // Typed reads: int (an integral number in int range), long long, double,
    // bool, std::string; anything else throws std::runtime_error.
    template <typename T>
    T get() const;

private:
    struct Parser {
        const std::string& s;
        size_t i;

        [[noreturn]] void fail(const char* what) const {
            throw std::runtime_error(std::string("json: ") + what + " at byte " + std::to_string(i));
        }
        void skip_ws() {
            while (i < s.size() && (s[i] == ' ' || s[i] == '\t' || s[i] == '\n' || s[i] == '\r')) ++i;
        }
        bool eat(const char* lit) {
            size_t n = 0;
            while (lit[n]) ++n;
            if (s.compare(i, n, lit) != 0) return false;
            i += n;
            return true;
        }
        JsonValue value(int depth) {
            if (depth > 256) fail("nesting deeper than 256 levels");
            if (i >= s.size()) fail("unexpected end of input");
            JsonValue v;
            const char c = s[i];
            if (c == '{') {
                v.kind_ = Kind::Object;
                ++i;
                skip_ws();
                if (i < s.size() && s[i] == '}') { ++i; return v; }
                for (;;) {
                    skip_ws();
                    if (i >= s.size() || s[i] != '"') fail("expected a string key");
                    std::string key = string();
                    skip_ws();
                    if (i >= s.size() || s[i] != ':') fail("expected ':'");
                    ++i;
                    skip_ws();
                    v.obj_.emplace_back(std::move(key), value(depth + 1));
                    skip_ws();
                    if (i < s.size() && s[i] == ',') { ++i; continue; }
                    if (i < s.size() && s[i] == '}') { ++i; return v; }
                    fail("expected ',' or '}'");
                }
            }
            if (c == '[') {
                v.kind_ = Kind::Array;
                ++i;
                skip_ws();
                if (i < s.size() && s[i] == ']') { ++i; return v; }
                for (;;) {
                    skip_ws();
                    v.arr_.push_back(value(depth + 1));
                    skip_ws();
                    if (i < s.size() && s[i] == ',') { ++i; continue; }
                    if (i < s.size() && s[i] == ']') { ++i; return v; }
                    fail("expected ',' or ']'");
                }
            }
            if (c == '"') {
                v.kind_ = Kind::String;
                v.str_ = string();
                return v;
            }
            if (eat("true")) { v.kind_ = Kind::Bool; v.b_ = true; return v; }
            if (eat("false")) { v.kind_ = Kind::Bool; v.b_ = false; return v; }
            if (eat("null")) return v;
            if (c == '-' || (c >= '0' && c <= '9')) return number();
            fail("unexpected character");
        }
        static bool digit(char c) { return c >= '0' && c <= '9'; }
        JsonValue number() {
            const size_t start = i;
            bool integral = true;
            if (s[i] == '-') ++i;
            if (i >= s.size() || !digit(s[i])) fail("malformed number");
            if (s[i] == '0') ++i;
            else while (i < s.size() && digit(s[i])) ++i;
            if (i < s.size() && s[i] == '.') {
                integral = false;
                ++i;
                if (i >= s.size() || !digit(s[i])) fail("malformed number");
                while (i < s.size() && digit(s[i])) ++i;
            }
            if (i < s.size() && (s[i] == 'e' || s[i] == 'E')) {
                integral = false;
                ++i;
                if (i < s.size() && (s[i] == '+' || s[i] == '-')) ++i;
                if (i >= s.size() || !digit(s[i])) fail("malformed number");
                while (i < s.size() && digit(s[i])) ++i;
            }
            const std::string text = s.substr(start, i - start);
            JsonValue v;
            v.kind_ = Kind::Number;
            v.num_ = std::strtod(text.c_str(), nullptr);
            if (integral) {
                errno = 0;
                const long long x = std::strtoll(text.c_str(), nullptr, 10);
                v.integral_ = errno != ERANGE;
                v.int_ = x;
            }
            return v;
        }
        unsigned hex4() {
            if (i + 4 > s.size()) fail("short \\u escape");
            unsigned u = 0;
            for (int k = 0; k < 4; ++k) {
                const char h = s[i++];
                u <<= 4;
                if (h >= '0' && h <= '9') u |= (unsigned)(h - '0');
                else if (h >= 'a' && h <= 'f') u |= (unsigned)(h - 'a' + 10);
                else if (h >= 'A' && h <= 'F') u |= (unsigned)(h - 'A' + 10);
                else fail("bad hex digit in \\u escape");
            }
            return u;
        }
        static void utf8(std::string& out, unsigned cp) {
            if (cp < 0x80) {
                out += (char)cp;
            } else if (cp < 0x800) {
                out += (char)(0xC0 | (cp >> 6));
                out += (char)(0x80 | (cp & 0x3F));
            } else if (cp < 0x10000) {
                out += (char)(0xE0 | (cp >> 12));
                out += (char)(0x80 | ((cp >> 6) & 0x3F));
                out += (char)(0x80 | (cp & 0x3F));
            } else {
                out += (char)(0xF0 | (cp >> 18));
                out += (char)(0x80 | ((cp >> 12) & 0x3F));
                out += (char)(0x80 | ((cp >> 6) & 0x3F));
                out += (char)(0x80 | (cp & 0x3F));
            }
        }
        std::string string() {
            ++i;   // opening quote
            std::string out;
            for (;;) {
                if (i >= s.size()) fail("unterminated string");
                const char c = s[i++];
                if (c == '"') return out;
                if ((unsigned char)c < 0x20) fail("control character in a string");
                if (c != '\\') { out += c; continue; }
                if (i >= s.size()) fail("unterminated escape");
                const char e = s[i++];
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
                        unsigned cp = hex4();
                        if (cp >= 0xD800 && cp < 0xDC00) {   // high surrogate: a low one follows
                            if (!eat("\\u")) fail("lone high surrogate");
                            const unsigned lo = hex4();
                            if (lo < 0xDC00 || lo >= 0xE000) fail("bad low surrogate");
                            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                        } else if (cp >= 0xDC00 && cp < 0xE000) {
                            fail("lone low surrogate");
                        }
                        utf8(out, cp);
                        break;
                    }
                    default: fail("unknown escape");
                }
            }
        }
    };

    const JsonValue* find(const std::string& key) const {
        if (kind_ != Kind::Object) return nullptr;
        for (auto it = obj_.rbegin(); it != obj_.rend(); ++it)
            if (it->first == key) return &it->second;
        return nullptr;
    }
    const std::vector<JsonValue>& array_ref() const {
        if (kind_ != Kind::Array) throw std::runtime_error("json: not an array");
        return arr_;
    }

    Kind kind_ = Kind::Null;
    bool b_ = false;
    double num_ = 0.0;
    bool integral_ = false;
    long long int_ = 0;
    std::string str_;
    std::vector<JsonValue> arr_;
    std::vector<std::pair<std::string, JsonValue>> obj_;
};

template <>
inline long long JsonValue::get<long long>() const {
    if (kind_ != Kind::Number || !integral_) throw std::runtime_error("json: expected an integer");
    return int_;
}
template <>
inline int JsonValue::get<int>() const {
    const long long v = get<long long>();
    if (v < std::numeric_limits<int>::min() || v > std::numeric_limits<int>::max())
        throw std::runtime_error("json: integer out of int range");
    return (int)v;
}
template <>
inline double JsonValue::get<double>() const {
    if (kind_ != Kind::Number) throw std::runtime_error("json: expected a number");
    return num_;
}
template <>
inline bool JsonValue::get<bool>() const {
    if (kind_ != Kind::Bool) throw std::runtime_error("json: expected a boolean");
    return b_;
}
template <>
inline std::string JsonValue::get<std::string>() const {
    if (kind_ != Kind::String) throw std::runtime_error("json: expected a string");
    return str_;
}

using json = JsonValue;

// sched rule: first matching (reference utils.h:14-37)
struct BuildMemoryRule {
    int retrieved_data_max;   // upper bound of the retrieved_data size (-1: unbounded)
    std::string config;       // kernel of build_memory
};

struct ManageMemoryAndApplyRule {
    int retrieved_data_max;   // -1: unbounded
    int memory_max;           // -1: unbounded
    int query;
    int output;
    std::vector<std::string> config;   // kernels of compute_score, memory_retrieval, apply_memory
};

struct BuildAndApplyMemoryRule {
    int retrieved_data_max;   // -1: unbounded
    int query;
    int output;
    std::vector<std::string> config;   // kernels of the four steps
};

class ScheduleConfig {
public:
    std::vector<BuildMemoryRule> build_memory_rules;
    std::vector<ManageMemoryAndApplyRule> manage_memory_and_apply_rules;
    std::vector<BuildAndApplyMemoryRule> build_and_apply_memory_rules;

    ScheduleConfig() = default;

    static ScheduleConfig load_from_file(const std::string& filepath) {
        std::ifstream file(filepath);
        if (!file.is_open()) throw std::runtime_error("Failed to open schedule file: " + filepath);
        std::stringstream text;
        text << file.rdbuf();
        return load_from_string(text.str());
    }

    static ScheduleConfig load_from_string(const std::string& text) {
        return load_from_json(json::parse(text));
    }

    static ScheduleConfig load_from_json(const json& j) {
        ScheduleConfig config;
        if (j.contains("build_memory")) {
            for (const auto& item : j["build_memory"]) {
                BuildMemoryRule rule;
                rule.retrieved_data_max = item["retrieved_data"].get<int>();
                rule.config = item["config"].get<std::string>();
                config.build_memory_rules.push_back(rule);
            }
        }
        if (j.contains("manage_memory_and_apply")) {
            for (const auto& item : j["manage_memory_and_apply"]) {
                ManageMemoryAndApplyRule rule;
                rule.retrieved_data_max = item["retrieved_data"].get<int>();
                rule.memory_max = item["memory"].get<int>();
                rule.query = item["query"].get<int>();
                rule.output = item["output"].get<int>();
                rule.config = names(item["config"], 3, "manage_memory_and_apply");
                config.manage_memory_and_apply_rules.push_back(rule);
            }
        }
        if (j.contains("build_and_apply_memory")) {
            for (const auto& item : j["build_and_apply_memory"]) {
                BuildAndApplyMemoryRule rule;
                rule.retrieved_data_max = item["retrieved_data"].get<int>();
                rule.query = item["query"].get<int>();
                rule.output = item["output"].get<int>();
                rule.config = names(item["config"], 4, "build_and_apply_memory");
                config.build_and_apply_memory_rules.push_back(rule);
            }
        }
        return config;
    }

    std::string get_build_memory_config(int retrieved_data) const {
        for (const auto& rule : build_memory_rules)
            if (rule.retrieved_data_max == -1 || retrieved_data <= rule.retrieved_data_max)
                return rule.config;
        throw std::runtime_error("No matching build_memory rule found");
    }

    std::vector<std::string> get_manage_memory_and_apply_config(int retrieved_data, int memory) const {
        for (const auto& rule : manage_memory_and_apply_rules) {
            const bool match_retrieved =
                rule.retrieved_data_max == -1 || retrieved_data <= rule.retrieved_data_max;
            const bool match_memory = rule.memory_max == -1 || memory <= rule.memory_max;
            if (match_retrieved && match_memory) return rule.config;
        }
        throw std::runtime_error("No matching manage_memory_and_apply rule found");
    }

    std::vector<std::string> get_build_and_apply_memory_config(int retrieved_data) const {
        for (const auto& rule : build_and_apply_memory_rules)
            if (rule.retrieved_data_max == -1 || retrieved_data <= rule.retrieved_data_max)
                return rule.config;
        throw std::runtime_error("No matching build_and_apply_memory rule found");
    }

private:
    static std::vector<std::string> names(const json& list, size_t need, const char* what) {
        std::vector<std::string> out;
        for (const auto& x : list) out.push_back(x.get<std::string>());
        if (out.size() < need)
            throw std::runtime_error(std::string("schedule: a ") + what + " rule needs " +
                                     std::to_string(need) + " kernel names");
        return out;
    }
};

}  // namespace deploy
}  // namespace heteromm

#endif  // HETEROMM_B200_DEPLOY_UTILS_H_
