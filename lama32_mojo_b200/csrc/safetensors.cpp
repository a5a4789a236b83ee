// Minimal safetensors reader — see safetensors.h.  A small recursive-descent
// JSON parser covering what the headers and index.json use (objects, arrays,
// strings with escapes, integers, and skipping of any other value).
#include "safetensors.h"

#include <stdio.h>
#include <string.h>
#include <sys/stat.h>

#include <set>

namespace q8 {
namespace {

struct Json {
  enum Kind { NUL, NUM, STR, ARR, OBJ, BOOL } kind = NUL;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
  const Json* get(const std::string& k) const {
    for (auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct Parser {
  const char* p;
  const char* e;
  std::string err;
  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool fail(const char* m) {
    if (err.empty()) err = m;
    return false;
  }
  bool str(std::string& out) {
    if (p >= e || *p != '"') return fail("expected string");
    ++p;
    out.clear();
    while (p < e && *p != '"') {
      if (*p == '\\') {
        ++p;
        if (p >= e) return fail("bad escape");
        char c = *p++;
        switch (c) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            if (e - p < 4) return fail("bad \\u escape");
            unsigned v = 0;
            for (int i = 0; i < 4; ++i) {
              char h = *p++;
              v <<= 4;
              if (h >= '0' && h <= '9') v |= h - '0';
              else if (h >= 'a' && h <= 'f') v |= h - 'a' + 10;
              else if (h >= 'A' && h <= 'F') v |= h - 'A' + 10;
              else return fail("bad hex digit");
            }
            if (v < 0x80) out += (char)v;
            else if (v < 0x800) { out += (char)(0xC0 | (v >> 6)); out += (char)(0x80 | (v & 63)); }
            else { out += (char)(0xE0 | (v >> 12)); out += (char)(0x80 | ((v >> 6) & 63)); out += (char)(0x80 | (v & 63)); }
            break;
          }
          default: out += c;
        }
      } else {
        out += *p++;
      }
    }
    if (p >= e) return fail("unterminated string");
    ++p;
    return true;
  }
  bool value(Json& v, int depth) {
    if (depth > 64) return fail("nesting too deep");
    ws();
    if (p >= e) return fail("unexpected end");
    char c = *p;
    if (c == '{') {
      v.kind = Json::OBJ;
      ++p;
      ws();
      if (p < e && *p == '}') { ++p; return true; }
      while (true) {
        ws();
        std::string k;
        if (!str(k)) return false;
        ws();
        if (p >= e || *p != ':') return fail("expected ':'");
        ++p;
        Json child;
        if (!value(child, depth + 1)) return false;
        v.obj.emplace_back(std::move(k), std::move(child));
        ws();
        if (p < e && *p == ',') { ++p; continue; }
        if (p < e && *p == '}') { ++p; return true; }
        return fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      v.kind = Json::ARR;
      ++p;
      ws();
      if (p < e && *p == ']') { ++p; return true; }
      while (true) {
        Json child;
        if (!value(child, depth + 1)) return false;
        v.arr.push_back(std::move(child));
        ws();
        if (p < e && *p == ',') { ++p; continue; }
        if (p < e && *p == ']') { ++p; return true; }
        return fail("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v.kind = Json::STR;
      return str(v.str);
    }
    if (c == '-' || (c >= '0' && c <= '9')) {
      v.kind = Json::NUM;
      char* endp = nullptr;
      std::string tmp(p, std::min<size_t>(64, e - p));
      v.num = strtod(tmp.c_str(), &endp);
      if (endp == tmp.c_str()) return fail("bad number");
      p += (endp - tmp.c_str());
      return true;
    }
    if (e - p >= 4 && !strncmp(p, "true", 4)) { v.kind = Json::BOOL; v.num = 1; p += 4; return true; }
    if (e - p >= 5 && !strncmp(p, "false", 5)) { v.kind = Json::BOOL; p += 5; return true; }
    if (e - p >= 4 && !strncmp(p, "null", 4)) { v.kind = Json::NUL; p += 4; return true; }
    return fail("unexpected character");
  }
};

bool parse_json(const std::string& s, Json& out, std::string& err) {
  Parser ps{s.data(), s.data() + s.size(), {}};
  if (!ps.value(out, 0)) {
    err = "json: " + ps.err;
    return false;
  }
  return true;
}

bool read_file(const std::string& path, std::string& out, std::string& err) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) {
    err = "cannot open " + path;
    return false;
  }
  fseek(f, 0, SEEK_END);
  long n = ftell(f);
  fseek(f, 0, SEEK_SET);
  out.resize(n > 0 ? (size_t)n : 0);
  if (n > 0 && fread(&out[0], 1, (size_t)n, f) != (size_t)n) {
    fclose(f);
    err = "short read " + path;
    return false;
  }
  fclose(f);
  return true;
}

}  // namespace

bool safetensors_parse_header(const std::string& json, const std::string& path, int64_t data_start,
                              std::map<std::string, TensorInfo>& out, std::string& err) {
  Json h;
  if (!parse_json(json, h, err)) return false;
  if (h.kind != Json::OBJ) {
    err = "header is not an object: " + path;
    return false;
  }
  for (auto& kv : h.obj) {
    if (kv.first == "__metadata__") continue;
    const Json& m = kv.second;
    const Json* dt = m.get("dtype");
    const Json* sh = m.get("shape");
    const Json* of = m.get("data_offsets");
    if (!dt || dt->kind != Json::STR || !sh || sh->kind != Json::ARR || !of || of->kind != Json::ARR ||
        of->arr.size() != 2) {
      err = "malformed entry " + kv.first + " in " + path;
      return false;
    }
    TensorInfo ti;
    ti.name = kv.first;
    ti.dtype = dt->str;
    ti.path = path;
    for (auto& d : sh->arr) {
      if (d.kind != Json::NUM || d.num < 0) {
        err = "bad shape for " + kv.first;
        return false;
      }
      ti.shape.push_back((int64_t)d.num);
    }
    if (of->arr[0].kind != Json::NUM || of->arr[1].kind != Json::NUM || of->arr[1].num < of->arr[0].num) {
      err = "bad data_offsets for " + kv.first;
      return false;
    }
    ti.begin = data_start + (int64_t)of->arr[0].num;
    ti.end = data_start + (int64_t)of->arr[1].num;
    out[ti.name] = std::move(ti);
  }
  return true;
}

static bool scan_file(const std::string& path, std::map<std::string, TensorInfo>& out, std::string& err) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) {
    err = "cannot open " + path;
    return false;
  }
  uint64_t n = 0;
  if (fread(&n, 8, 1, f) != 1 || n == 0 || n > (1ull << 31)) {
    fclose(f);
    err = "bad header length in " + path;
    return false;
  }
  std::string hdr(n, '\0');
  if (fread(&hdr[0], 1, n, f) != n) {
    fclose(f);
    err = "truncated header in " + path;
    return false;
  }
  fseek(f, 0, SEEK_END);
  const int64_t fsize = ftell(f);
  fclose(f);
  std::map<std::string, TensorInfo> part;
  if (!safetensors_parse_header(hdr, path, 8 + (int64_t)n, part, err)) return false;
  for (auto& kv : part) {
    if (kv.second.end > fsize) {
      err = "tensor " + kv.first + " extends past end of " + path + " (truncated file?)";
      return false;
    }
    out[kv.first] = kv.second;
  }
  return true;
}

bool safetensors_scan(const std::string& dir, std::map<std::string, TensorInfo>& out, std::string& err) {
  const std::string idx = dir + "/model.safetensors.index.json";
  struct stat st;
  std::vector<std::string> shards;
  if (stat(idx.c_str(), &st) == 0) {
    std::string txt;
    if (!read_file(idx, txt, err)) return false;
    Json j;
    if (!parse_json(txt, j, err)) return false;
    const Json* wm = j.get("weight_map");
    if (!wm || wm->kind != Json::OBJ) {
      err = "index.json has no weight_map";
      return false;
    }
    std::set<std::string> seen;
    for (auto& kv : wm->obj) {
      if (kv.second.kind != Json::STR) continue;
      if (seen.insert(kv.second.str).second) shards.push_back(dir + "/" + kv.second.str);
    }
  } else {
    shards.push_back(dir + "/model.safetensors");
  }
  for (auto& s : shards)
    if (!scan_file(s, out, err)) return false;
  return true;
}

}  // namespace q8
