// gb_gguf.cpp -- GGUF v2/v3 reader (memory image or mmap'd file) and writer.
// Reader: the checks and layout of gguf.Parse (gguf/gguf.go:62-130) and
// gguf.Open (gguf/open_unix.go:13). Writer: gguf/writer.go:141 WriteTo
// (version 3, tensors aligned to general.alignment, default 32).
#include <fcntl.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "gb_internal.h"

namespace {

struct Reader {
  const uint8_t *b;
  size_t len, pos = 0;
  const char *err = nullptr;
  bool need(uint64_t n) {
    if (err) return false;
    if (n > len || pos + n > len) {
      err = "gguf: truncated header";
      return false;
    }
    return true;
  }
  uint64_t le(int n) {
    if (!need((uint64_t)n)) return 0;
    uint64_t v = 0;
    for (int i = 0; i < n; i++) v |= (uint64_t)b[pos + i] << (8 * i);
    pos += (size_t)n;
    return v;
  }
  std::string str() {
    uint64_t n = le(8);
    if (n > len || !need(n)) {
      if (!err) err = "gguf: bad string length";
      return std::string();
    }
    std::string s((const char *)b + pos, (size_t)n);
    pos += (size_t)n;
    return s;
  }
  // gguf/gguf.go:401 typed
  bool typed(int t, GbValue &v, int depth) {
    v.type = t;
    uint64_t x;
    switch (t) {
      case 0: v.u = le(1); break;
      case 1: v.u = (uint64_t)(int64_t)(int8_t)le(1); break;
      case 2: v.u = le(2); break;
      case 3: v.u = (uint64_t)(int64_t)(int16_t)le(2); break;
      case 4: v.u = le(4); break;
      case 5: v.u = (uint64_t)(int64_t)(int32_t)le(4); break;
      case 6: { uint32_t u = (uint32_t)le(4); float f; memcpy(&f, &u, 4); v.f = f; break; }
      case 7: v.u = le(1) != 0; break;
      case 8: v.s = str(); break;
      case 10: v.u = le(8); break;
      case 11: v.u = le(8); break;
      case 12: { x = le(8); double d; memcpy(&d, &x, 8); v.f = d; break; }
      case 9: {
        v.elem = (int)le(4);
        uint64_t n = le(8);
        if (n > len) { err = "gguf: bad array length"; return false; }
        if (depth > 16) { err = "gguf: arrays nested too deep"; return false; }
        for (uint64_t i = 0; i < n && !err; i++) {
          GbValue e;
          if (!typed(v.elem, e, depth + 1)) return false;
          v.arr.push_back(std::move(e));
        }
        break;
      }
      default: err = "gguf: unknown value type"; return false;
    }
    return err == nullptr;
  }
};

}  // namespace

GbGguf::~GbGguf() {
  if (map) munmap(map, map_len);
}

const GbValue *GbGguf::get(const std::string &k) const {
  for (auto &p : kv)
    if (p.first == k) return &p.second;
  return nullptr;
}
// gguf/gguf.go:154 Uint: any integer type, else def.
uint64_t GbGguf::get_uint(const std::string &k, uint64_t def) const {
  const GbValue *v = get(k);
  return v && v->is_int() ? v->u : def;
}
// gguf/gguf.go:162 Float: float32 or float64, else def.
double GbGguf::get_float(const std::string &k, double def) const {
  const GbValue *v = get(k);
  return v && (v->type == 6 || v->type == 12) ? v->f : def;
}
std::string GbGguf::get_string(const std::string &k, const std::string &def) const {
  const GbValue *v = get(k);
  return v && v->type == 8 ? v->s : def;
}
const GbTensor *GbGguf::tensor(const std::string &name) const {
  for (auto &t : tensors)
    if (t.name == name) return &t;
  return nullptr;
}

GbGguf *gb_gguf_parse(const uint8_t *data, size_t len) {
  Reader r{data, len};
  GbGguf *f = new GbGguf();
  f->data = data;
  f->len = len;
  const char *msg = nullptr;
  uint64_t n_t = 0, n_kv = 0;
  if (r.le(4) != 0x46554747u) { msg = r.err ? r.err : "gguf: bad magic"; goto fail; }
  f->version = (uint32_t)r.le(4);
  if (r.err) { msg = r.err; goto fail; }
  if (f->version < 2 || f->version > 3) { msg = "gguf: unsupported version"; goto fail; }
  n_t = r.le(8);
  n_kv = r.le(8);
  if (r.err) { msg = r.err; goto fail; }
  if (n_kv > len || n_t > len) { msg = "gguf: corrupt header counts"; goto fail; }
  for (uint64_t i = 0; i < n_kv; i++) {
    std::string key = r.str();
    int t = (int)r.le(4);
    GbValue v;
    if (r.err || !r.typed(t, v, 0)) { msg = r.err ? r.err : "gguf: bad value"; goto fail; }
    if (key == "general.alignment") {
      f->alignment = (uint32_t)(v.is_int() || v.type == 7 ? v.u : 0);
      if (f->alignment == 0 || (f->alignment & (f->alignment - 1)) != 0) {
        msg = "gguf: bad alignment"; goto fail;
      }
    }
    f->kv.emplace_back(std::move(key), std::move(v));
  }
  for (uint64_t i = 0; i < n_t; i++) {
    GbTensor t;
    t.name = r.str();
    uint32_t nd = (uint32_t)r.le(4);
    if (r.err) { msg = r.err; goto fail; }
    if (nd > 4) { msg = "gguf: tensor has more than 4 dims"; goto fail; }
    for (uint32_t j = 0; j < nd; j++) t.dims.push_back(r.le(8));
    t.type = (int)r.le(4);
    t.offset = r.le(8);
    if (r.err) { msg = r.err; goto fail; }
    // The reference knows every ggml type's size; this build decodes the
    // subset with kernels and rejects the rest up front.
    if (gb_block_size(t.type) == 0) { msg = "gguf: unsupported tensor type"; goto fail; }
    if (f->tensor(t.name)) { msg = "gguf: duplicate tensor"; goto fail; }
    f->tensors.push_back(std::move(t));
  }
  f->data_offset = (r.pos + f->alignment - 1) & ~(uint64_t)(f->alignment - 1);
  for (auto &t : f->tensors) {
    uint64_t ne = t.numel();
    t.bytes = t.dims.empty() || t.dims[0] == 0
                  ? 0
                  : (uint64_t)gb_row_bytes(t.type, (int64_t)t.dims[0]) * (ne / t.dims[0]);
    uint64_t end = f->data_offset + t.offset + t.bytes;
    if (t.offset % f->alignment != 0 || end > len) { msg = "gguf: tensor data out of range"; goto fail; }
    t.data = data + f->data_offset + t.offset;
  }
  return f;
fail:
  gb_fail(GB_ERR_IO, "%s", msg ? msg : "gguf: parse error");
  delete f;
  return nullptr;
}

// gguf/open_unix.go:13 Open: mmap the file read-only and parse it.
GbGguf *gb_gguf_open(const char *path) {
  int fd = open(path, O_RDONLY);
  if (fd < 0) {
    gb_fail(GB_ERR_IO, "gguf: open %s: cannot open file", path);
    return nullptr;
  }
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size <= 0) {
    close(fd);
    gb_fail(GB_ERR_IO, "gguf: %s: empty or unreadable", path);
    return nullptr;
  }
  void *m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (m == MAP_FAILED) {
    gb_fail(GB_ERR_IO, "gguf: mmap %s failed", path);
    return nullptr;
  }
  GbGguf *f = gb_gguf_parse((const uint8_t *)m, (size_t)st.st_size);
  if (!f) {
    munmap(m, (size_t)st.st_size);
    return nullptr;
  }
  f->map = m;
  f->map_len = (size_t)st.st_size;
  return f;
}

// ---- writer (gguf/writer.go) ----------------------------------------------

void GbGgufWriter::set_u32(const std::string &k, uint32_t v) {
  GbValue x;
  x.type = 4;
  x.u = v;
  kv.emplace_back(k, x);
}
void GbGgufWriter::set_f32(const std::string &k, float v) {
  GbValue x;
  x.type = 6;
  x.f = v;
  kv.emplace_back(k, x);
}
void GbGgufWriter::set_str(const std::string &k, const std::string &v) {
  GbValue x;
  x.type = 8;
  x.s = v;
  kv.emplace_back(k, x);
}

// gguf/writer.go:103 AddTensor: shape row-major; data exactly RowBytes*rows
// (or empty, for a tensor whose bytes are filled in after layout()).
int GbGgufWriter::add_tensor(const std::string &name, const std::vector<int> &shape, int type,
                             std::vector<uint8_t> &&data) {
  if (gb_block_size(type) == 0) return gb_fail(GB_ERR_INVALID, "gguf: unknown type %d", type);
  if (shape.empty()) return gb_fail(GB_ERR_INVALID, "gguf: tensor %s has no dims", name.c_str());
  T t;
  t.name = name;
  uint64_t n = 1;
  for (size_t i = 0; i < shape.size(); i++) {
    t.dims.insert(t.dims.begin(), (uint64_t)shape[i]);
    n *= (uint64_t)shape[i];
  }
  int inner = shape.back();
  if (inner % gb_block_size(type) != 0)
    return gb_fail(GB_ERR_INVALID, "gguf: tensor %s: inner dim %d not a multiple of the block",
                   name.c_str(), inner);
  t.bytes = (uint64_t)gb_row_bytes(type, inner) * (n / (uint64_t)inner);
  if (!data.empty() && data.size() != t.bytes)
    return gb_fail(GB_ERR_INVALID, "gguf: tensor %s: %zu bytes, want %llu", name.c_str(),
                   data.size(), (unsigned long long)t.bytes);
  t.type = type;
  t.data = std::move(data);
  tensors.push_back(std::move(t));
  return GB_OK;
}

namespace {
struct Out {
  std::vector<uint8_t> b;
  void le(uint64_t v, int n) {
    for (int i = 0; i < n; i++) b.push_back((uint8_t)(v >> (8 * i)));
  }
  void str(const std::string &s) {
    le(s.size(), 8);
    b.insert(b.end(), s.begin(), s.end());
  }
  void pad(uint32_t a) {
    while (b.size() % a) b.push_back(0);
  }
  void typed(const GbValue &v) {
    switch (v.type) {
      case 0: case 1: case 7: le(v.u, 1); break;
      case 2: case 3: le(v.u, 2); break;
      case 4: case 5: le(v.u, 4); break;
      case 10: case 11: le(v.u, 8); break;
      case 6: { float f = (float)v.f; uint32_t u; memcpy(&u, &f, 4); le(u, 4); break; }
      case 12: { uint64_t u; memcpy(&u, &v.f, 8); le(u, 8); break; }
      case 8: str(v.s); break;
      case 9:
        le((uint64_t)v.elem, 4);
        le(v.arr.size(), 8);
        for (auto &e : v.arr) typed(e);
        break;
    }
  }
};
}  // namespace

// gguf/writer.go:141-166: header bytes up to the aligned data section, and
// each tensor's offset inside the data section.
std::vector<uint8_t> GbGgufWriter::layout(std::vector<uint64_t> *offsets,
                                          uint64_t *total) const {
  Out o;
  o.le(0x46554747u, 4);
  o.le(3, 4);
  o.le(tensors.size(), 8);
  o.le(kv.size(), 8);
  for (auto &p : kv) {
    o.str(p.first);
    o.le((uint64_t)p.second.type, 4);
    o.typed(p.second);
  }
  uint64_t off = 0;
  offsets->clear();
  for (auto &t : tensors) {
    o.str(t.name);
    o.le(t.dims.size(), 4);
    for (auto d : t.dims) o.le(d, 8);
    o.le((uint64_t)t.type, 4);
    o.le(off, 8);
    offsets->push_back(off);
    off = (off + t.bytes + alignment - 1) / alignment * alignment;
  }
  o.pad(alignment);
  *total = o.b.size() + off;
  return std::move(o.b);
}

// gguf/writer.go:141 WriteTo, into one contiguous image.
std::vector<uint8_t> GbGgufWriter::write() const {
  std::vector<uint64_t> offs;
  uint64_t total = 0;
  std::vector<uint8_t> img = layout(&offs, &total);
  size_t hdr = img.size();
  img.resize((size_t)total, 0);
  for (size_t i = 0; i < tensors.size(); i++)
    if (!tensors[i].data.empty())
      memcpy(img.data() + hdr + offs[i], tensors[i].data.data(), tensors[i].data.size());
  return img;
}

// ---- C ABI over the reader ---------------------------------------------------
struct gb_gguf {
  GbGguf *f = nullptr;
};

extern "C" {

int gb_gguf_parse(const void *data, size_t len, gb_gguf **out) {
  gb_clear_error();
  if (!data || !out) return gb_fail(GB_ERR_INVALID, "gguf: null argument");
  GbGguf *f = gb_gguf_parse((const uint8_t *)data, len);
  if (!f) return GB_ERR_IO;
  *out = new gb_gguf{f};
  return GB_OK;
}

int gb_gguf_open(const char *path, gb_gguf **out) {
  gb_clear_error();
  if (!path || !out) return gb_fail(GB_ERR_INVALID, "gguf: null argument");
  GbGguf *f = gb_gguf_open(path);
  if (!f) return GB_ERR_IO;
  *out = new gb_gguf{f};
  return GB_OK;
}

int gb_gguf_close(gb_gguf *f) {
  gb_clear_error();
  if (f) {
    delete f->f;
    delete f;
  }
  return GB_OK;
}

int gb_gguf_header(const gb_gguf *f, uint32_t *version, uint32_t *alignment, int *n_kv, int *n_tensors) {
  gb_clear_error();
  if (!f) return gb_fail(GB_ERR_INVALID, "gguf: null handle");
  if (version) *version = f->f->version;
  if (alignment) *alignment = f->f->alignment;
  if (n_kv) *n_kv = (int)f->f->kv.size();
  if (n_tensors) *n_tensors = (int)f->f->tensors.size();
  return GB_OK;
}

uint64_t gb_gguf_uint(const gb_gguf *f, const char *key, uint64_t def) {
  return f && key ? f->f->get_uint(key, def) : def;
}

double gb_gguf_float(const gb_gguf *f, const char *key, double def) {
  return f && key ? f->f->get_float(key, def) : def;
}

int gb_gguf_string(const gb_gguf *f, const char *key, const char *def, char *out, int cap) {
  gb_clear_error();
  if (!f || !key || !out || cap <= 0) return gb_fail(GB_ERR_INVALID, "gguf: bad arguments");
  std::string s = f->f->get_string(key, def ? def : "");
  snprintf(out, (size_t)cap, "%s", s.c_str());
  return GB_OK;
}

const char *gb_gguf_key(const gb_gguf *f, int i, int *value_type) {
  if (!f || i < 0 || i >= (int)f->f->kv.size()) return nullptr;
  if (value_type) *value_type = f->f->kv[(size_t)i].second.type;
  return f->f->kv[(size_t)i].first.c_str();
}

int gb_gguf_array_len(const gb_gguf *f, const char *key, int *elem_type) {
  const GbValue *v = f && key ? f->f->get(key) : nullptr;
  if (!v || v->type != 9) return 0;
  if (elem_type) *elem_type = v->elem;
  return (int)v->arr.size();
}

// gguf/gguf.go:259 Value.Float64 of element j.
double gb_gguf_array_float(const gb_gguf *f, const char *key, int j) {
  const GbValue *v = f && key ? f->f->get(key) : nullptr;
  if (!v || v->type != 9 || j < 0 || j >= (int)v->arr.size()) return 0;
  const GbValue &e = v->arr[(size_t)j];
  if (e.type == 6 || e.type == 12) return e.f;
  if (e.is_int()) return (double)(int64_t)e.u;
  return 0;
}

int gb_gguf_array_string(const gb_gguf *f, const char *key, int j, char *out, int cap) {
  gb_clear_error();
  const GbValue *v = f && key ? f->f->get(key) : nullptr;
  if (!v || v->type != 9 || v->elem != 8 || j < 0 || j >= (int)v->arr.size() || !out || cap <= 0)
    return gb_fail(GB_ERR_INVALID, "gguf: no string element %d in %s", j, key ? key : "");
  snprintf(out, (size_t)cap, "%s", v->arr[(size_t)j].s.c_str());
  return GB_OK;
}

int gb_gguf_tensor(const gb_gguf *f, const char *name, int *type, int *ndims, uint64_t dims[4],
                   uint64_t *offset, uint64_t *nbytes, const void **data) {
  gb_clear_error();
  if (!f || !name) return gb_fail(GB_ERR_INVALID, "gguf: null argument");
  const GbTensor *t = f->f->tensor(name);
  if (!t) return gb_fail(GB_ERR_INVALID, "gguf: no tensor %s", name);
  if (type) *type = t->type;
  if (ndims) *ndims = (int)t->dims.size();
  if (dims)
    for (size_t i = 0; i < 4; i++) dims[i] = i < t->dims.size() ? t->dims[i] : 0;
  if (offset) *offset = t->offset;
  if (nbytes) *nbytes = t->bytes;
  if (data) *data = t->data;
  return GB_OK;
}

const char *gb_gguf_tensor_at(const gb_gguf *f, int i) {
  if (!f || i < 0 || i >= (int)f->f->tensors.size()) return nullptr;
  return f->f->tensors[(size_t)i].name.c_str();
}

}  // extern "C"
