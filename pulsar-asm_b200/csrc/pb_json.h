// pb_json.h -- minimal JSON reader for the .lfm3q8 header (objects, arrays,
// strings with simple escapes, numbers, true/false/null). The reference scans
// the same header by hand (lfm3_nanode.cu:1445-1526); a real parser rejects a
// malformed record instead of reading a neighbour's field.
#pragma once
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace pbjson {

struct Value {
  enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
  bool b = false;
  double num = 0;
  long long inum = 0;
  bool is_int = false;
  std::string str;
  std::vector<Value> arr;
  std::vector<std::pair<std::string, Value>> obj;
  const Value* get(const char* key) const {
    if (kind != OBJ) return nullptr;
    for (auto& kv : obj) if (kv.first == key) return &kv.second;
    return nullptr;
  }
  double as_num(double def) const { return kind == NUM ? num : def; }
  long long as_int(long long def) const { return kind == NUM ? (is_int ? inum : (long long)num) : def; }
};

class Parser {
 public:
  Parser(const char* s, size_t n) : p_(s), e_(s + n) {}
  bool parse(Value& v) {
    ws();
    if (!value(v, 0)) return false;
    ws();
    return p_ == e_ || *p_ == '\0';
  }
  const char* error() const { return err_; }

 private:
  const char* p_;
  const char* e_;
  const char* err_ = "";
  void ws() { while (p_ < e_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) p_++; }
  bool fail(const char* m) { err_ = m; return false; }
  bool lit(const char* s) {
    size_t n = strlen(s);
    if ((size_t)(e_ - p_) < n || memcmp(p_, s, n)) return false;
    p_ += n;
    return true;
  }
  bool string(std::string& out) {
    if (p_ >= e_ || *p_ != '"') return fail("expected string");
    p_++;
    while (p_ < e_ && *p_ != '"') {
      char c = *p_++;
      if (c == '\\') {
        if (p_ >= e_) return fail("bad escape");
        char d = *p_++;
        switch (d) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            if (e_ - p_ < 4) return fail("bad \\u");
            unsigned cp = (unsigned)strtoul(std::string(p_, 4).c_str(), nullptr, 16);
            p_ += 4;
            if (cp < 0x80) out += (char)cp;
            else if (cp < 0x800) { out += (char)(0xc0 | (cp >> 6)); out += (char)(0x80 | (cp & 0x3f)); }
            else { out += (char)(0xe0 | (cp >> 12)); out += (char)(0x80 | ((cp >> 6) & 0x3f)); out += (char)(0x80 | (cp & 0x3f)); }
            break;
          }
          default: out += d;
        }
      } else {
        out += c;
      }
    }
    if (p_ >= e_) return fail("unterminated string");
    p_++;
    return true;
  }
  bool value(Value& v, int depth) {
    if (depth > 64) return fail("nesting too deep");
    ws();
    if (p_ >= e_) return fail("unexpected end");
    char c = *p_;
    if (c == '{') {
      v.kind = Value::OBJ;
      p_++;
      ws();
      if (p_ < e_ && *p_ == '}') { p_++; return true; }
      while (true) {
        ws();
        std::string k;
        if (!string(k)) return false;
        ws();
        if (p_ >= e_ || *p_ != ':') return fail("expected ':'");
        p_++;
        Value child;
        if (!value(child, depth + 1)) return false;
        v.obj.emplace_back(std::move(k), std::move(child));
        ws();
        if (p_ < e_ && *p_ == ',') { p_++; continue; }
        if (p_ < e_ && *p_ == '}') { p_++; return true; }
        return fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      v.kind = Value::ARR;
      p_++;
      ws();
      if (p_ < e_ && *p_ == ']') { p_++; return true; }
      while (true) {
        Value child;
        if (!value(child, depth + 1)) return false;
        v.arr.push_back(std::move(child));
        ws();
        if (p_ < e_ && *p_ == ',') { p_++; continue; }
        if (p_ < e_ && *p_ == ']') { p_++; return true; }
        return fail("expected ',' or ']'");
      }
    }
    if (c == '"') { v.kind = Value::STR; return string(v.str); }
    if (lit("true")) { v.kind = Value::BOOL; v.b = true; return true; }
    if (lit("false")) { v.kind = Value::BOOL; v.b = false; return true; }
    if (lit("null")) { v.kind = Value::NUL; return true; }
    if (c == '-' || (c >= '0' && c <= '9')) {
      const char* s = p_;
      bool frac = false;
      if (*p_ == '-') p_++;
      while (p_ < e_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' ||
                         *p_ == '+' || *p_ == '-')) {
        if (*p_ == '.' || *p_ == 'e' || *p_ == 'E') frac = true;
        p_++;
      }
      std::string tok(s, p_ - s);
      v.kind = Value::NUM;
      v.num = strtod(tok.c_str(), nullptr);
      v.is_int = !frac;
      if (!frac) v.inum = strtoll(tok.c_str(), nullptr, 10);
      return true;
    }
    return fail("unexpected character");
  }
};

}  // namespace pbjson
