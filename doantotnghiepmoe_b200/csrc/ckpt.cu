// Merged-INT8 checkpoint reader: the safetensors shards written by the
// reference's converter (tools/prepare_olmoe.py:85-94), indexed the way the
// reference's TensorIndex does it (src/safetensors.rs:90-181):
//
//   * every `*.safetensors` file of the directory, in sorted path order;
//   * 8-byte little-endian header length, at most 100,000,000, the header a
//     JSON object starting with '{';
//   * entries {dtype: U8|I8|F16|BF16|F32, shape: [..], data_offsets: [b, e]}
//     with no other fields; `__metadata__` must map strings to strings;
//   * duplicate names (in one header or across shards), shape or byte-count
//     overflow, offsets that disagree with shape x dtype size, data past the
//     end of the file, gaps or overlaps between tensors, and bytes that no
//     tensor covers are all rejected.
//
// Tensor payloads are read on demand with pread.  Host code only: the device
// upload of a layer (moe_load_layer) lives with the handle in moe_abi.cu.
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>
#include <dirent.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "ckpt.h"

namespace moe {
namespace {

constexpr uint64_t kMaxHeaderBytes = 100000000ull;

// Minimal JSON reader for safetensors headers: objects, arrays, strings
// (with escapes), non-negative integers.  Anything else is an error.
struct Json {
  const char *p, *end;
  std::string err;

  void ws() {
    while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool fail(const char *m) {
    if (err.empty()) err = m;
    return false;
  }
  bool lit(char c) {
    ws();
    if (p < end && *p == c) {
      ++p;
      return true;
    }
    return false;
  }
  static void utf8(std::string &o, uint32_t cp) {
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
  bool hex4(uint32_t &v) {
    if (end - p < 4) return fail("truncated \\u escape");
    v = 0;
    for (int i = 0; i < 4; ++i, ++p) {
      const char c = *p;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
      else return fail("bad \\u escape");
    }
    return true;
  }
  bool str(std::string &o) {
    o.clear();
    if (!lit('"')) return fail("expected a string");
    while (p < end) {
      const char c = *p++;
      if (c == '"') return true;
      if ((unsigned char)c < 0x20) return fail("control character in string");
      if (c != '\\') {
        o += c;
        continue;
      }
      if (p >= end) break;
      const char x = *p++;
      switch (x) {
        case '"': o += '"'; break;
        case '\\': o += '\\'; break;
        case '/': o += '/'; break;
        case 'b': o += '\b'; break;
        case 'f': o += '\f'; break;
        case 'n': o += '\n'; break;
        case 'r': o += '\r'; break;
        case 't': o += '\t'; break;
        case 'u': {
          uint32_t cp;
          if (!hex4(cp)) return false;
          if (cp >= 0xD800 && cp < 0xDC00) {  // surrogate pair
            uint32_t lo;
            if (end - p < 2 || p[0] != '\\' || p[1] != 'u') return fail("lone surrogate");
            p += 2;
            if (!hex4(lo) || lo < 0xDC00 || lo >= 0xE000) return fail("bad surrogate pair");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          } else if (cp >= 0xDC00 && cp < 0xE000) {
            return fail("lone surrogate");
          }
          utf8(o, cp);
          break;
        }
        default: return fail("bad escape");
      }
    }
    return fail("unterminated string");
  }
  bool u64(uint64_t &v) {
    ws();
    if (p >= end || *p < '0' || *p > '9') return fail("expected a non-negative integer");
    if (*p == '0' && p + 1 < end && p[1] >= '0' && p[1] <= '9') return fail("leading zero");
    v = 0;
    while (p < end && *p >= '0' && *p <= '9') {
      const uint64_t d = (uint64_t)(*p++ - '0');
      if (v > (UINT64_MAX - d) / 10) return fail("integer overflow");
      v = v * 10 + d;
    }
    if (p < end && (*p == '.' || *p == 'e' || *p == 'E')) return fail("expected an integer");
    return true;
  }
  bool u64_array(std::vector<uint64_t> &out) {
    out.clear();
    if (!lit('[')) return fail("expected an array");
    if (lit(']')) return true;
    do {
      uint64_t v;
      if (!u64(v)) return false;
      out.push_back(v);
    } while (lit(','));
    if (!lit(']')) return fail("expected ']'");
    return true;
  }
};

int dtype_code(const std::string &s) {
  if (s == "U8") return MOE_DT_U8;
  if (s == "I8") return MOE_DT_I8;
  if (s == "F16") return MOE_DT_F16;
  if (s == "BF16") return MOE_DT_BF16;
  if (s == "F32") return MOE_DT_F32;
  return -1;
}

}  // namespace

size_t dtype_bytes(int dt) {
  switch (dt) {
    case MOE_DT_U8:
    case MOE_DT_I8: return 1;
    case MOE_DT_F16:
    case MOE_DT_BF16: return 2;
    case MOE_DT_F32: return 4;
    default: return 0;
  }
}

}  // namespace moe

using namespace moe;

struct moe_ckpt {
  std::vector<int> fds;
  std::vector<std::string> paths;
  std::map<std::string, CkptTensor> tensors;
};

namespace {

void put_err(char *err, size_t len, const std::string &m) {
  if (err && len) snprintf(err, len, "%s", m.c_str());
}

// One shard: header checks and entries (src/safetensors.rs:112-181).
bool add_shard(moe_ckpt *c, const std::string &path, std::string &why) {
  const int fd = open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0) {
    why = path + ": cannot open";
    return false;
  }
  struct stat st {};
  if (fstat(fd, &st) != 0) {
    close(fd);
    why = path + ": cannot stat";
    return false;
  }
  const uint64_t file_len = (uint64_t)st.st_size;
  uint8_t prefix[8];
  if (file_len < 8 || pread(fd, prefix, 8, 0) != 8) {
    close(fd);
    why = path + ": invalid Safetensors header length";
    return false;
  }
  uint64_t header_len = 0;
  for (int i = 7; i >= 0; --i) header_len = (header_len << 8) | prefix[i];
  if (header_len == 0 || header_len > kMaxHeaderBytes || header_len + 8 > file_len) {
    close(fd);
    why = path + ": invalid Safetensors header length";
    return false;
  }
  const uint64_t start = header_len + 8;
  std::string header(header_len, '\0');
  if (pread(fd, &header[0], header_len, 8) != (ssize_t)header_len) {
    close(fd);
    why = path + ": short header read";
    return false;
  }
  auto bad = [&](const std::string &m) {
    close(fd);
    why = path + ": " + m;
    return false;
  };
  if (header[0] != '{') return bad("header must start with '{'");
  Json j{header.data(), header.data() + header.size(), {}};
  if (!j.lit('{')) return bad("header must start with '{'");
  const int shard = (int)c->fds.size();
  std::vector<std::pair<uint64_t, uint64_t>> ranges;
  std::map<std::string, CkptTensor> local;
  bool seen_meta = false;
  if (!j.lit('}')) {
    do {
      std::string name;
      if (!j.str(name)) return bad(j.err);
      if (!j.lit(':')) return bad("expected ':'");
      if (name == "__metadata__") {
        if (seen_meta) return bad("duplicate tensor: __metadata__");
        seen_meta = true;
        if (!j.lit('{')) return bad("__metadata__ must map strings to strings");
        if (!j.lit('}')) {
          do {  // a repeated metadata key keeps its last value, as a map would
            std::string k, v;
            if (!j.str(k) || !j.lit(':') || !j.str(v))
              return bad("__metadata__ must map strings to strings");
          } while (j.lit(','));
          if (!j.lit('}')) return bad("expected '}'");
        }
        continue;
      }
      if (local.count(name)) return bad("duplicate tensor: " + name);
      if (!j.lit('{')) return bad(name + ": expected a descriptor object");
      std::string dts;
      std::vector<uint64_t> shape, offs;
      bool has_dt = false, has_shape = false, has_offs = false;
      if (!j.lit('}')) {
        do {
          std::string field;
          if (!j.str(field) || !j.lit(':')) return bad(name + ": " + j.err);
          if (field == "dtype" && !has_dt) {
            if (!j.str(dts)) return bad(name + ": " + j.err);
            has_dt = true;
          } else if (field == "shape" && !has_shape) {
            if (!j.u64_array(shape)) return bad(name + ": " + j.err);
            has_shape = true;
          } else if (field == "data_offsets" && !has_offs) {
            if (!j.u64_array(offs)) return bad(name + ": " + j.err);
            has_offs = true;
          } else {
            return bad(name + ": unknown or repeated field " + field);
          }
        } while (j.lit(','));
        if (!j.lit('}')) return bad(name + ": expected '}'");
      }
      if (!has_dt || !has_shape || !has_offs) return bad(name + ": missing field");
      const int dt = dtype_code(dts);
      if (dt < 0) return bad(name + ": unknown dtype " + dts);
      if (offs.size() != 2) return bad(name + ": data_offsets must hold two numbers");
      uint64_t elems = 1;
      for (uint64_t d : shape) {
        if (d != 0 && elems > UINT64_MAX / d) return bad("tensor shape overflow");
        elems *= d;
      }
      const uint64_t sz = dtype_bytes(dt);
      if (elems > UINT64_MAX / sz) return bad("tensor byte length overflow");
      const uint64_t bytes = elems * sz;
      const uint64_t b = offs[0], e = offs[1];
      if (e < b || e > file_len - start || e - b != bytes)
        return bad(name + ": invalid tensor offsets or shape");
      ranges.emplace_back(b, e);
      CkptTensor t;
      t.dtype = dt;
      t.shape.assign(shape.begin(), shape.end());
      t.bytes = bytes;
      t.shard = shard;
      t.offset = start + b;
      local.emplace(name, std::move(t));
    } while (j.lit(','));
    if (!j.lit('}')) return bad("expected '}' at the end of the header");
  }
  j.ws();
  if (j.p != j.end) return bad("trailing bytes after the header object");
  std::sort(ranges.begin(), ranges.end());
  uint64_t cursor = 0;
  for (auto &r : ranges) {
    if (r.first != cursor) return bad("tensor data has gaps or overlaps");
    cursor = r.second;
  }
  if (cursor != file_len - start) return bad("unindexed tensor data");
  for (auto &kv : local)
    if (c->tensors.count(kv.first)) return bad("duplicate tensor across shards: " + kv.first);
  for (auto &kv : local) c->tensors.emplace(kv.first, kv.second);
  c->fds.push_back(fd);
  c->paths.push_back(path);
  return true;
}

}  // namespace

namespace moe {

const CkptTensor *ckpt_find(const moe_ckpt *c, const std::string &name) {
  auto it = c->tensors.find(name);
  return it == c->tensors.end() ? nullptr : &it->second;
}

bool ckpt_read(const moe_ckpt *c, const CkptTensor &t, void *dst) {
  uint8_t *d = static_cast<uint8_t *>(dst);
  uint64_t done = 0;
  while (done < t.bytes) {
    const uint64_t want = std::min<uint64_t>(t.bytes - done, 1ull << 30);
    const ssize_t got = pread(c->fds[t.shard], d + done, want, (off_t)(t.offset + done));
    if (got <= 0) return false;
    done += (uint64_t)got;
  }
  return true;
}

}  // namespace moe

extern "C" moe_status moe_ckpt_open(const char *dir, moe_ckpt **out, char *err, size_t err_len) {
  if (!dir || !out) return MOE_ERR_INVALID;
  *out = nullptr;
  DIR *d = opendir(dir);
  if (!d) {
    put_err(err, err_len, std::string(dir) + ": cannot open directory");
    return MOE_ERR_INVALID;
  }
  std::vector<std::string> paths;
  while (dirent *ent = readdir(d)) {
    const std::string n = ent->d_name;
    if (n.size() > 12 && n.compare(n.size() - 12, 12, ".safetensors") == 0)
      paths.push_back(std::string(dir) + "/" + n);
  }
  closedir(d);
  std::sort(paths.begin(), paths.end());
  if (paths.empty()) {
    put_err(err, err_len, "no .safetensors shards found");
    return MOE_ERR_INVALID;
  }
  auto *c = new moe_ckpt();
  for (const auto &p : paths) {
    std::string why;
    if (!add_shard(c, p, why)) {
      put_err(err, err_len, why);
      moe_ckpt_close(c);
      return MOE_ERR_INVALID;
    }
  }
  *out = c;
  return MOE_OK;
}

extern "C" void moe_ckpt_close(moe_ckpt *c) {
  if (!c) return;
  for (int fd : c->fds) close(fd);
  delete c;
}

extern "C" int moe_ckpt_num_tensors(const moe_ckpt *c) { return c ? (int)c->tensors.size() : 0; }

extern "C" moe_status moe_ckpt_tensor_info(const moe_ckpt *c, const char *name, int *dtype,
                                           int *ndim, int64_t *shape, size_t *bytes) {
  if (!c || !name) return MOE_ERR_INVALID;
  const CkptTensor *t = ckpt_find(c, name);
  if (!t) return MOE_ERR_INVALID;
  if (dtype) *dtype = t->dtype;
  if (ndim) *ndim = (int)t->shape.size();
  if (shape)
    for (size_t i = 0; i < t->shape.size() && i < 8; ++i) shape[i] = t->shape[i];
  if (bytes) *bytes = (size_t)t->bytes;
  return MOE_OK;
}

extern "C" moe_status moe_ckpt_read(const moe_ckpt *c, const char *name, void *dst,
                                    size_t dst_bytes) {
  if (!c || !name || !dst) return MOE_ERR_INVALID;
  const CkptTensor *t = ckpt_find(c, name);
  if (!t || t->bytes > dst_bytes) return MOE_ERR_INVALID;
  return ckpt_read(c, *t, dst) ? MOE_OK : MOE_ERR_INVALID;
}
