// Operator policy registry (host C++), the B200 backend's equivalent of the
// reference's Rust policy core (crates/fireprot-core/src/registry.rs:95-268)
// behind the same JSON-in / JSON-out protocol as its CPython bridge
// (crates/fireprot-bridge/src/lib.rs:86-125):
//  - candidates per operation sorted by priority (desc), then name, then
//    version (registry.rs:118-124); the first supporting candidate wins;
//  - a capability callback returns supported / rejected-with-reason; an
//    error inside it rejects only that candidate (registry.rs:173-190);
//  - per-signature cache, cleared by every (un)registration;
//  - selection counts keyed by (operation, implementation) including
//    "native" when nothing matched, and the last decision per signature
//    (registry.rs:195-259);
//  - an interrupted callback (status -1) aborts the resolution without
//    caching it or touching counts (registry.rs:144-149).
// Signatures arrive as canonical JSON (sorted keys) and are used verbatim as
// cache keys; only "operation" is read from them.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

extern "C" {
// Capability callback: return 1 = supported, 0 = rejected (reason written
// into `reason`, NUL-terminated, at most `cap` bytes), -1 = interrupted.
typedef int (*fpb_capability_fn)(const char* signature_json, void* user, char* reason,
                                 size_t cap);
}

namespace {

struct Impl {
  std::string operation, name, version;
  int priority = 0;
  fpb_capability_fn fn = nullptr;
  void* user = nullptr;
};

struct Rejection {
  std::string implementation, reason;
};

struct Selection {
  bool has_impl = false;
  std::string operation, name, version;
  int priority = 0;
  std::vector<Rejection> rejected;
};

std::string json_escape(const std::string& s) {
  std::string o;
  o.reserve(s.size() + 8);
  for (unsigned char c : s) {
    switch (c) {
      case '"': o += "\\\""; break;
      case '\\': o += "\\\\"; break;
      case '\n': o += "\\n"; break;
      case '\r': o += "\\r"; break;
      case '\t': o += "\\t"; break;
      default:
        if (c < 0x20) {
          char b[8];
          std::snprintf(b, sizeof(b), "\\u%04x", c);
          o += b;
        } else {
          o += static_cast<char>(c);
        }
    }
  }
  return o;
}

// Minimal reader for top-level string / integer fields of a flat JSON object.
bool skip_ws(const char*& p) {
  while (*p == ' ' || *p == '\n' || *p == '\t' || *p == '\r') ++p;
  return *p != 0;
}

bool read_string(const char*& p, std::string& out) {
  if (*p != '"') return false;
  ++p;
  out.clear();
  while (*p && *p != '"') {
    if (*p == '\\') {
      ++p;
      switch (*p) {
        case 'n': out += '\n'; break;
        case 't': out += '\t'; break;
        case 'r': out += '\r'; break;
        case 'b': out += '\b'; break;
        case 'f': out += '\f'; break;
        case 'u': {
          unsigned v = 0;
          for (int i = 1; i <= 4 && p[i]; ++i) {
            const char h = p[i];
            v = v * 16 + (h >= '0' && h <= '9' ? h - '0' : (h | 32) - 'a' + 10);
          }
          p += 4;
          if (v < 0x80) out += static_cast<char>(v);
          else if (v < 0x800) {
            out += static_cast<char>(0xC0 | (v >> 6));
            out += static_cast<char>(0x80 | (v & 0x3F));
          } else {
            out += static_cast<char>(0xE0 | (v >> 12));
            out += static_cast<char>(0x80 | ((v >> 6) & 0x3F));
            out += static_cast<char>(0x80 | (v & 0x3F));
          }
          break;
        }
        default: out += *p;
      }
      ++p;
    } else {
      out += *p++;
    }
  }
  if (*p != '"') return false;
  ++p;
  return true;
}

// Skip any JSON value (object, array, string, number, literal).
bool skip_value(const char*& p) {
  skip_ws(p);
  if (*p == '"') {
    std::string tmp;
    return read_string(p, tmp);
  }
  if (*p == '{' || *p == '[') {
    const char open = *p, close = open == '{' ? '}' : ']';
    int depth = 0;
    while (*p) {
      if (*p == '"') {
        std::string tmp;
        if (!read_string(p, tmp)) return false;
        continue;
      }
      if (*p == open) ++depth;
      if (*p == close && --depth == 0) {
        ++p;
        return true;
      }
      ++p;
    }
    return false;
  }
  while (*p && *p != ',' && *p != '}' && *p != ']') ++p;
  return true;
}

// Top-level fields of a flat object as raw text (strings unescaped).
bool parse_fields(const char* json, std::map<std::string, std::string>& out) {
  const char* p = json;
  if (!skip_ws(p) || *p != '{') return false;
  ++p;
  while (skip_ws(p)) {
    if (*p == '}') return true;
    std::string key;
    if (!read_string(p, key)) return false;
    skip_ws(p);
    if (*p != ':') return false;
    ++p;
    skip_ws(p);
    if (*p == '"') {
      std::string v;
      if (!read_string(p, v)) return false;
      out[key] = v;
    } else {
      const char* s = p;
      if (!skip_value(p)) return false;
      out[key] = std::string(s, p - s);
    }
    skip_ws(p);
    if (*p == ',') ++p;
  }
  return false;
}

struct Registry {
  std::mutex mu;
  std::map<std::string, std::vector<Impl>> candidates;
  std::map<std::string, Selection> cache;
  std::map<std::pair<std::string, std::string>, unsigned long long> counts;
  std::map<std::string, Selection> last_decisions;
};

std::string selection_json(const Selection& s, bool cache_hit) {
  std::string o = "{\"implementation\": ";
  if (s.has_impl) {
    char pr[32];
    std::snprintf(pr, sizeof(pr), "%d", s.priority);
    o += "{\"operation\": \"" + json_escape(s.operation) + "\", \"name\": \"" +
         json_escape(s.name) + "\", \"version\": \"" + json_escape(s.version) +
         "\", \"priority\": " + pr + "}";
  } else {
    o += "null";
  }
  o += ", \"rejected\": [";
  for (size_t i = 0; i < s.rejected.size(); ++i) {
    if (i) o += ", ";
    o += "{\"implementation\": \"" + json_escape(s.rejected[i].implementation) +
         "\", \"reason\": \"" + json_escape(s.rejected[i].reason) + "\"}";
  }
  o += "], \"cache_hit\": ";
  o += cache_hit ? "true" : "false";
  o += "}";
  return o;
}

int write_out(const std::string& s, char* out, size_t cap) {
  if (!out || s.size() + 1 > cap) return -(int)(s.size() + 1);
  std::memcpy(out, s.c_str(), s.size() + 1);
  return 0;
}

}  // namespace

extern "C" {

void* fpb_registry_new(void) { return new (std::nothrow) Registry(); }

void fpb_registry_free(void* reg) { delete static_cast<Registry*>(reg); }

// metadata: {"operation": ..., "name": ..., "priority": int, "version": ...}
// Returns 0, 2 (empty identity), 3 (duplicate name), 4 (bad JSON / args).
int fpb_registry_register(void* reg, const char* metadata_json, fpb_capability_fn fn,
                          void* user) {
  auto* r = static_cast<Registry*>(reg);
  if (!r || !metadata_json || !fn) return 4;
  std::map<std::string, std::string> f;
  if (!parse_fields(metadata_json, f)) return 4;
  Impl im;
  im.operation = f["operation"];
  im.name = f["name"];
  im.version = f["version"];
  const auto trim_empty = [](const std::string& s) {
    return s.find_first_not_of(" \t\n\r") == std::string::npos;
  };
  if (trim_empty(im.operation) || trim_empty(im.name) || trim_empty(im.version)) return 2;
  im.priority = f.count("priority") ? std::atoi(f["priority"].c_str()) : 0;
  im.fn = fn;
  im.user = user;
  std::lock_guard<std::mutex> lk(r->mu);
  auto& v = r->candidates[im.operation];
  for (auto& c : v)
    if (c.name == im.name) return 3;
  v.push_back(im);
  std::stable_sort(v.begin(), v.end(), [](const Impl& a, const Impl& b) {
    if (a.priority != b.priority) return a.priority > b.priority;
    if (a.name != b.name) return a.name < b.name;
    return a.version < b.version;
  });
  r->cache.clear();
  return 0;
}

// Returns 0, or 5 when the implementation is unknown.
int fpb_registry_unregister(void* reg, const char* operation, const char* name) {
  auto* r = static_cast<Registry*>(reg);
  if (!r || !operation || !name) return 4;
  std::lock_guard<std::mutex> lk(r->mu);
  auto it = r->candidates.find(operation);
  if (it == r->candidates.end()) return 5;
  auto& v = it->second;
  for (size_t i = 0; i < v.size(); ++i) {
    if (v[i].name == name) {
      v.erase(v.begin() + i);
      r->cache.clear();
      return 0;
    }
  }
  return 5;
}

// Resolve a signature (canonical JSON). Writes the selection JSON
// {"implementation": {...}|null, "rejected": [...], "cache_hit": bool}.
// Returns 0, 4 (bad JSON), 6 (a callback was interrupted: nothing cached or
// counted), or -(bytes needed) when `cap` is too small.
int fpb_registry_resolve(void* reg, const char* signature_json, char* out, size_t cap) {
  auto* r = static_cast<Registry*>(reg);
  if (!r || !signature_json) return 4;
  std::map<std::string, std::string> f;
  if (!parse_fields(signature_json, f) || !f.count("operation")) return 4;
  const std::string key(signature_json);
  std::lock_guard<std::mutex> lk(r->mu);
  Selection sel;
  bool hit = false;
  auto c = r->cache.find(key);
  if (c != r->cache.end()) {
    sel = c->second;
    hit = true;
  } else {
    auto it = r->candidates.find(f["operation"]);
    if (it != r->candidates.end()) {
      for (const Impl& im : it->second) {
        char reason[1024];
        reason[0] = 0;
        const int ok = im.fn(signature_json, im.user, reason, sizeof(reason));
        if (ok < 0) return 6;
        if (ok > 0) {
          sel.has_impl = true;
          sel.operation = im.operation;
          sel.name = im.name;
          sel.version = im.version;
          sel.priority = im.priority;
          break;
        }
        sel.rejected.push_back({im.name, reason[0] ? reason : "capability returned false"});
      }
    }
    r->cache[key] = sel;
  }
  const std::string name = sel.has_impl ? sel.name : "native";
  auto& cnt = r->counts[{f["operation"], name}];
  if (cnt != ~0ull) ++cnt;
  r->last_decisions[key] = sel;
  return write_out(selection_json(sel, hit), out, cap);
}

// Manifest: {"implementations": {op: [{name, priority, version}]},
// "selection_counts": [{operation, implementation, count}],
// "decisions": [{signature, selected, rejected}]} (registry.rs:218-259).
int fpb_registry_manifest(void* reg, char* out, size_t cap) {
  auto* r = static_cast<Registry*>(reg);
  if (!r) return 4;
  std::lock_guard<std::mutex> lk(r->mu);
  std::string o = "{\"implementations\": {";
  bool first = true;
  for (auto& kv : r->candidates) {
    if (!first) o += ", ";
    first = false;
    o += "\"" + json_escape(kv.first) + "\": [";
    for (size_t i = 0; i < kv.second.size(); ++i) {
      char pr[32];
      std::snprintf(pr, sizeof(pr), "%d", kv.second[i].priority);
      if (i) o += ", ";
      o += "{\"name\": \"" + json_escape(kv.second[i].name) + "\", \"priority\": " + pr +
           ", \"version\": \"" + json_escape(kv.second[i].version) + "\"}";
    }
    o += "]";
  }
  o += "}, \"selection_counts\": [";
  first = true;
  for (auto& kv : r->counts) {
    char cn[32];
    std::snprintf(cn, sizeof(cn), "%llu", kv.second);
    if (!first) o += ", ";
    first = false;
    o += "{\"operation\": \"" + json_escape(kv.first.first) + "\", \"implementation\": \"" +
         json_escape(kv.first.second) + "\", \"count\": " + cn + "}";
  }
  o += "], \"decisions\": [";
  first = true;
  for (auto& kv : r->last_decisions) {
    if (!first) o += ", ";
    first = false;
    o += "{\"signature\": " + kv.first + ", \"selected\": \"" +
         json_escape(kv.second.has_impl ? kv.second.name : "native") + "\", \"rejected\": [";
    for (size_t i = 0; i < kv.second.rejected.size(); ++i) {
      if (i) o += ", ";
      o += "{\"implementation\": \"" + json_escape(kv.second.rejected[i].implementation) +
           "\", \"reason\": \"" + json_escape(kv.second.rejected[i].reason) + "\"}";
    }
    o += "]}";
  }
  o += "]}";
  return write_out(o, out, cap);
}

int fpb_registry_clear_runtime_state(void* reg) {
  auto* r = static_cast<Registry*>(reg);
  if (!r) return 4;
  std::lock_guard<std::mutex> lk(r->mu);
  r->cache.clear();
  r->counts.clear();
  r->last_decisions.clear();
  return 0;
}

}  // extern "C"
