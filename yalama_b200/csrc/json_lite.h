// Minimal JSON reader for the two documents the engine parses itself: a
// safetensors header (include/safetensors.h:37-78 in the reference parses it
// with nlohmann::json) and an HF config.json (src/ConfigManager.cpp:389-471).
// Objects, arrays, strings (with escapes), numbers, true/false/null.
#pragma once
#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace ylm {

struct JVal
{
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    double num = 0;
    std::string str;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj; // insertion order kept

    const JVal *get(const std::string &k) const
    {
        for (auto &kv : obj)
            if (kv.first == k)
                return &kv.second;
        return nullptr;
    }
    bool has(const std::string &k) const { return get(k) != nullptr; }
    double as_num() const
    {
        if (kind == Num)
            return num;
        if (kind == Bool)
            return b ? 1 : 0;
        throw std::runtime_error("json: number expected");
    }
};

class JParser
{
  public:
    explicit JParser(const std::string &s) : s_(s) {}
    JVal parse()
    {
        JVal v = value();
        ws();
        if (i_ != s_.size())
            throw std::runtime_error("json: trailing characters");
        return v;
    }

  private:
    const std::string &s_;
    size_t i_ = 0;

    void ws()
    {
        while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\t' || s_[i_] == '\r'))
            i_++;
    }
    char peek()
    {
        ws();
        if (i_ >= s_.size())
            throw std::runtime_error("json: unexpected end");
        return s_[i_];
    }
    void expect(char c)
    {
        if (peek() != c)
            throw std::runtime_error(std::string("json: expected ") + c);
        i_++;
    }
    JVal value()
    {
        char c = peek();
        if (c == '{')
            return object();
        if (c == '[')
            return array();
        if (c == '"')
        {
            JVal v;
            v.kind = JVal::Str;
            v.str = string();
            return v;
        }
        if (s_.compare(i_, 4, "true") == 0)
        {
            i_ += 4;
            JVal v;
            v.kind = JVal::Bool;
            v.b = true;
            return v;
        }
        if (s_.compare(i_, 5, "false") == 0)
        {
            i_ += 5;
            JVal v;
            v.kind = JVal::Bool;
            return v;
        }
        if (s_.compare(i_, 4, "null") == 0)
        {
            i_ += 4;
            return JVal();
        }
        return number();
    }
    JVal object()
    {
        JVal v;
        v.kind = JVal::Obj;
        expect('{');
        if (peek() == '}')
        {
            i_++;
            return v;
        }
        for (;;)
        {
            if (peek() != '"')
                throw std::runtime_error("json: key expected");
            std::string k = string();
            expect(':');
            v.obj.emplace_back(std::move(k), value());
            char c = peek();
            i_++;
            if (c == '}')
                return v;
            if (c != ',')
                throw std::runtime_error("json: , or } expected");
        }
    }
    JVal array()
    {
        JVal v;
        v.kind = JVal::Arr;
        expect('[');
        if (peek() == ']')
        {
            i_++;
            return v;
        }
        for (;;)
        {
            v.arr.push_back(value());
            char c = peek();
            i_++;
            if (c == ']')
                return v;
            if (c != ',')
                throw std::runtime_error("json: , or ] expected");
        }
    }
    std::string string()
    {
        expect('"');
        std::string out;
        while (i_ < s_.size() && s_[i_] != '"')
        {
            char c = s_[i_++];
            if (c == '\\')
            {
                if (i_ >= s_.size())
                    break;
                char e = s_[i_++];
                switch (e)
                {
                case 'n': out += '\n'; break;
                case 't': out += '\t'; break;
                case 'r': out += '\r'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'u':
                {
                    if (i_ + 4 > s_.size())
                        throw std::runtime_error("json: bad \\u escape");
                    unsigned cp = std::stoul(s_.substr(i_, 4), nullptr, 16);
                    i_ += 4;
                    if (cp < 0x80)
                        out += (char)cp;
                    else if (cp < 0x800)
                    {
                        out += (char)(0xC0 | (cp >> 6));
                        out += (char)(0x80 | (cp & 0x3F));
                    }
                    else
                    {
                        out += (char)(0xE0 | (cp >> 12));
                        out += (char)(0x80 | ((cp >> 6) & 0x3F));
                        out += (char)(0x80 | (cp & 0x3F));
                    }
                    break;
                }
                default: out += e;
                }
            }
            else
                out += c;
        }
        if (i_ >= s_.size())
            throw std::runtime_error("json: unterminated string");
        i_++;
        return out;
    }
    JVal number()
    {
        size_t st = i_;
        while (i_ < s_.size() && (isdigit((unsigned char)s_[i_]) || s_[i_] == '-' || s_[i_] == '+' || s_[i_] == '.' ||
                                  s_[i_] == 'e' || s_[i_] == 'E'))
            i_++;
        if (st == i_)
            throw std::runtime_error("json: value expected");
        JVal v;
        v.kind = JVal::Num;
        v.num = std::stod(s_.substr(st, i_ - st));
        return v;
    }
};

inline JVal json_parse(const std::string &s) { return JParser(s).parse(); }

} // namespace ylm
