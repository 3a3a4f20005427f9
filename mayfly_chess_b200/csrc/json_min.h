// A minimal JSON reader for the weight file's header (objects, arrays, strings, numbers, true/false/null).
// Throws std::runtime_error with the byte offset on malformed input.
#pragma once
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace mf {

struct JVal {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    double num = 0.0;
    std::string str;
    std::vector<JVal> arr;
    std::map<std::string, JVal> obj;

    const JVal* get(const std::string& k) const
    {
        auto it = obj.find(k);
        return (kind == Obj && it != obj.end()) ? &it->second : nullptr;
    }
};

class JParser {
public:
    explicit JParser(const std::string& s) : s_(s) {}

    JVal parse()
    {
        JVal v = value();
        ws();
        if (i_ != s_.size()) fail("trailing characters");
        return v;
    }

private:
    const std::string& s_;
    size_t i_ = 0;

    [[noreturn]] void fail(const char* why) const
    {
        throw std::runtime_error(std::string("bad JSON header (") + why + ") at byte " + std::to_string(i_));
    }
    void ws()
    {
        while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_;
    }
    bool eat(char c)
    {
        ws();
        if (i_ < s_.size() && s_[i_] == c) {
            ++i_;
            return true;
        }
        return false;
    }
    void expect(char c)
    {
        if (!eat(c)) fail("unexpected character");
    }
    std::string string()
    {
        expect('"');
        std::string out;
        while (i_ < s_.size() && s_[i_] != '"') {
            char c = s_[i_++];
            if (c == '\\') {
                if (i_ >= s_.size()) fail("unterminated escape");
                char e = s_[i_++];
                switch (e) {
                    case 'n': out += '\n'; break;
                    case 't': out += '\t'; break;
                    case 'r': out += '\r'; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'u': {
                        if (i_ + 4 > s_.size()) fail("short \\u escape");
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
                    default: out += e;
                }
            } else {
                out += c;
            }
        }
        if (i_ >= s_.size()) fail("unterminated string");
        ++i_;
        return out;
    }
    JVal value()
    {
        ws();
        if (i_ >= s_.size()) fail("unexpected end");
        JVal v;
        const char c = s_[i_];
        if (c == '{') {
            ++i_;
            v.kind = JVal::Obj;
            if (eat('}')) return v;
            do {
                ws();
                std::string k = string();
                expect(':');
                v.obj[k] = value();
            } while (eat(','));
            expect('}');
        } else if (c == '[') {
            ++i_;
            v.kind = JVal::Arr;
            if (eat(']')) return v;
            do {
                v.arr.push_back(value());
            } while (eat(','));
            expect(']');
        } else if (c == '"') {
            v.kind = JVal::Str;
            v.str = string();
        } else if (s_.compare(i_, 4, "true") == 0) {
            i_ += 4;
            v.kind = JVal::Bool;
            v.b = true;
        } else if (s_.compare(i_, 5, "false") == 0) {
            i_ += 5;
            v.kind = JVal::Bool;
        } else if (s_.compare(i_, 4, "null") == 0) {
            i_ += 4;
        } else {
            const char* start = s_.c_str() + i_;
            char* end = nullptr;
            v.num = std::strtod(start, &end);
            if (end == start) fail("not a value");
            v.kind = JVal::Num;
            i_ += static_cast<size_t>(end - start);
        }
        return v;
    }
};

}  // namespace mf
