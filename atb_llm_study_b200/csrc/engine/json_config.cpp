#include "engine/json_config.h"

#include <cmath>
#include <cstdlib>
#include <fstream>
#include <sstream>

namespace b200llm {

namespace {

struct Parser {
  const std::string& s;
  size_t i = 0;
  std::string err;
  int depth = 0;

  explicit Parser(const std::string& t) : s(t) {}

  void ws() {
    while (i < s.size() && (s[i] == ' ' || s[i] == '\t' || s[i] == '\n' || s[i] == '\r')) ++i;
  }
  bool fail(const char* m) {
    if (err.empty()) err = std::string(m) + " at offset " + std::to_string(i);
    return false;
  }
  bool lit(const char* w) {
    size_t n = std::char_traits<char>::length(w);
    if (s.compare(i, n, w) != 0) return fail("bad literal");
    i += n;
    return true;
  }
  static void put_utf8(std::string& o, unsigned cp) {
    if (cp < 0x80) {
      o += (char)cp;
    } else if (cp < 0x800) {
      o += (char)(0xC0 | (cp >> 6));
      o += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      o += (char)(0xE0 | (cp >> 12));
      o += (char)(0x80 | ((cp >> 6) & 0x3F));
      o += (char)(0x80 | (cp & 0x3F));
    } else {
      o += (char)(0xF0 | (cp >> 18));
      o += (char)(0x80 | ((cp >> 12) & 0x3F));
      o += (char)(0x80 | ((cp >> 6) & 0x3F));
      o += (char)(0x80 | (cp & 0x3F));
    }
  }
  bool hex4(unsigned& v) {
    if (i + 4 > s.size()) return fail("short \\u escape");
    v = 0;
    for (int k = 0; k < 4; ++k) {
      char c = s[i++];
      v <<= 4;
      if (c >= '0' && c <= '9') v |= (unsigned)(c - '0');
      else if (c >= 'a' && c <= 'f') v |= (unsigned)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= (unsigned)(c - 'A' + 10);
      else return fail("bad hex digit");
    }
    return true;
  }
  bool string(std::string& o) {
    if (s[i] != '"') return fail("expected string");
    ++i;
    while (i < s.size()) {
      char c = s[i++];
      if (c == '"') return true;
      if (c != '\\') {
        o += c;
        continue;
      }
      if (i >= s.size()) break;
      char e = s[i++];
      switch (e) {
        case '"': o += '"'; break;
        case '\\': o += '\\'; break;
        case '/': o += '/'; break;
        case 'b': o += '\b'; break;
        case 'f': o += '\f'; break;
        case 'n': o += '\n'; break;
        case 'r': o += '\r'; break;
        case 't': o += '\t'; break;
        case 'u': {
          unsigned cp;
          if (!hex4(cp)) return false;
          if (cp >= 0xD800 && cp < 0xDC00 && i + 6 <= s.size() && s[i] == '\\' && s[i + 1] == 'u') {
            i += 2;
            unsigned lo;
            if (!hex4(lo)) return false;
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          put_utf8(o, cp);
          break;
        }
        default: return fail("bad escape");
      }
    }
    return fail("unterminated string");
  }
  bool value(JsonValue& v) {
    if (++depth > 256) return fail("nesting too deep");
    ws();
    if (i >= s.size()) return fail("unexpected end");
    bool ok = true;
    char c = s[i];
    if (c == '{') {
      v.kind = JsonValue::Object;
      ++i;
      ws();
      if (i < s.size() && s[i] == '}') {
        ++i;
      } else {
        while (true) {
          ws();
          std::string k;
          if (i >= s.size() || !string(k)) { ok = false; break; }
          ws();
          if (i >= s.size() || s[i] != ':') { ok = fail("expected ':'"); break; }
          ++i;
          JsonValue child;
          if (!value(child)) { ok = false; break; }
          v.obj[k] = std::move(child);
          ws();
          if (i < s.size() && s[i] == ',') { ++i; continue; }
          if (i < s.size() && s[i] == '}') { ++i; break; }
          ok = fail("expected ',' or '}'");
          break;
        }
      }
    } else if (c == '[') {
      v.kind = JsonValue::Array;
      ++i;
      ws();
      if (i < s.size() && s[i] == ']') {
        ++i;
      } else {
        while (true) {
          JsonValue child;
          if (!value(child)) { ok = false; break; }
          v.arr.push_back(std::move(child));
          ws();
          if (i < s.size() && s[i] == ',') { ++i; continue; }
          if (i < s.size() && s[i] == ']') { ++i; break; }
          ok = fail("expected ',' or ']'");
          break;
        }
      }
    } else if (c == '"') {
      v.kind = JsonValue::String;
      ok = string(v.str);
    } else if (c == 't') {
      v.kind = JsonValue::Bool;
      v.b = true;
      ok = lit("true");
    } else if (c == 'f') {
      v.kind = JsonValue::Bool;
      ok = lit("false");
    } else if (c == 'n') {
      ok = lit("null");
    } else {
      const char* b = s.c_str() + i;
      char* e = nullptr;
      v.num = std::strtod(b, &e);
      if (e == b) {
        ok = fail("bad number");
      } else {
        v.kind = JsonValue::Number;
        i += (size_t)(e - b);
      }
    }
    --depth;
    return ok;
  }
};

}  // namespace

bool JsonValue::Parse(const std::string& text, JsonValue& out, std::string* err) {
  Parser p(text);
  out = JsonValue();
  bool ok = p.value(out);
  if (ok) {
    p.ws();
    if (p.i != text.size()) ok = p.fail("trailing characters");
  }
  if (!ok && err) *err = p.err;
  return ok;
}

JsonConfig JsonConfig::Parse(const std::string& json_str) {
  auto v = std::make_shared<JsonValue>();
  if (!JsonValue::Parse(json_str, *v)) return JsonConfig();
  return JsonConfig(v);
}

JsonConfig JsonConfig::Load(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return JsonConfig();
  std::stringstream ss;
  ss << f.rdbuf();
  return Parse(ss.str());
}

const JsonValue* JsonConfig::Find(const std::string& key) const {
  if (!IsValid()) return nullptr;
  auto it = root_->obj.find(key);
  return it == root_->obj.end() ? nullptr : &it->second;
}

bool JsonConfig::HasKey(const std::string& key) const {
  const JsonValue* v = Find(key);
  return v && v->kind != JsonValue::Null;
}

int JsonConfig::GetInt(const std::string& key, int default_val) const {
  const JsonValue* v = Find(key);
  return (v && v->kind == JsonValue::Number) ? (int)v->num : default_val;
}

int64_t JsonConfig::GetInt64(const std::string& key, int64_t default_val) const {
  const JsonValue* v = Find(key);
  return (v && v->kind == JsonValue::Number) ? (int64_t)v->num : default_val;
}

float JsonConfig::GetFloat(const std::string& key, float default_val) const {
  const JsonValue* v = Find(key);
  return (v && v->kind == JsonValue::Number) ? (float)v->num : default_val;
}

std::string JsonConfig::GetString(const std::string& key, const std::string& default_val) const {
  const JsonValue* v = Find(key);
  return (v && v->kind == JsonValue::String) ? v->str : default_val;
}

bool JsonConfig::GetBool(const std::string& key, bool default_val) const {
  const JsonValue* v = Find(key);
  return (v && v->kind == JsonValue::Bool) ? v->b : default_val;
}

std::vector<int> JsonConfig::GetIntArray(const std::string& key) const {
  std::vector<int> out;
  const JsonValue* v = Find(key);
  if (v && v->kind == JsonValue::Array)
    for (auto& e : v->arr)
      if (e.kind == JsonValue::Number) out.push_back((int)e.num);
  return out;
}

std::vector<float> JsonConfig::GetFloatArray(const std::string& key) const {
  std::vector<float> out;
  const JsonValue* v = Find(key);
  if (v && v->kind == JsonValue::Array)
    for (auto& e : v->arr)
      if (e.kind == JsonValue::Number) out.push_back((float)e.num);
  return out;
}

JsonConfig JsonConfig::GetSubConfig(const std::string& key) const {
  const JsonValue* v = Find(key);
  if (!v || v->kind != JsonValue::Object) return JsonConfig();
  return JsonConfig(std::shared_ptr<const JsonValue>(root_, v));
}

}  // namespace b200llm
