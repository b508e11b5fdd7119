// safetensors.cpp -- reader of MLX-format safetensors model directories.
//
// Replaces the weight-loading half of higgs-models: collect_safetensors_files
// (crates/higgs-models/src/lib.rs:688-707: model.safetensors.index.json's
// weight_map, else a single model.safetensors), Array::load_safetensors
// (lib.rs:612-616) and the quantized key remap (remap_quantized_key,
// lib.rs:709-723).  Files are memory-mapped; a tensor (or a 2-D slice of it,
// for tensor-parallel shards) is copied straight from the mapping into a
// caller-owned host or device buffer, so a rank reads only its own shard.
//
// File format (the published safetensors layout): an 8-byte little-endian
// header length N, N bytes of JSON {name: {"dtype", "shape", "data_offsets":
// [begin, end]}, "__metadata__": {...}}, then the data; offsets are relative to
// the end of the header.
#include <fcntl.h>
#include <stdint.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <vector>

#include "common.cuh"

using higgs::fail;

namespace {

// ---- a minimal JSON reader (objects, arrays, strings, numbers, literals) ----
struct JVal {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  double num = 0.0;
  int64_t inum = 0;  // exact value of an integer literal
  bool is_int = false;
  std::string str;
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;
  const JVal* get(const std::string& k) const {
    for (auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

class JParser {
 public:
  JParser(const char* p, size_t n) : p_(p), e_(p + n) {}
  bool parse(JVal* out) {
    if (!value(out, 0)) return false;
    ws();
    return p_ == e_;
  }

 private:
  const char* p_;
  const char* e_;
  void ws() {
    while (p_ < e_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
  }
  bool lit(const char* s) {
    const size_t n = strlen(s);
    if ((size_t)(e_ - p_) < n || memcmp(p_, s, n) != 0) return false;
    p_ += n;
    return true;
  }
  bool string(std::string* s) {
    if (p_ >= e_ || *p_ != '"') return false;
    ++p_;
    while (p_ < e_ && *p_ != '"') {
      if (*p_ == '\\') {
        if (++p_ >= e_) return false;
        const char c = *p_++;
        switch (c) {
          case 'n': s->push_back('\n'); break;
          case 't': s->push_back('\t'); break;
          case 'r': s->push_back('\r'); break;
          case 'b': s->push_back('\b'); break;
          case 'f': s->push_back('\f'); break;
          case 'u': {  // \uXXXX: keep ASCII, otherwise a placeholder byte
            if (e_ - p_ < 4) return false;
            unsigned v = 0;
            for (int i = 0; i < 4; ++i) {
              const char h = p_[i];
              v = v * 16 + (unsigned)(h >= '0' && h <= '9' ? h - '0'
                                      : h >= 'a' && h <= 'f' ? h - 'a' + 10
                                      : h >= 'A' && h <= 'F' ? h - 'A' + 10 : 0);
            }
            p_ += 4;
            s->push_back(v < 128 ? (char)v : '?');
            break;
          }
          default: s->push_back(c);
        }
      } else {
        s->push_back(*p_++);
      }
    }
    if (p_ >= e_) return false;
    ++p_;
    return true;
  }
  bool value(JVal* v, int depth) {
    if (depth > 64) return false;
    ws();
    if (p_ >= e_) return false;
    const char c = *p_;
    if (c == '{') {
      ++p_;
      v->kind = JVal::Obj;
      ws();
      if (p_ < e_ && *p_ == '}') {
        ++p_;
        return true;
      }
      for (;;) {
        ws();
        std::string k;
        if (!string(&k)) return false;
        ws();
        if (p_ >= e_ || *p_ != ':') return false;
        ++p_;
        JVal x;
        if (!value(&x, depth + 1)) return false;
        v->obj.emplace_back(std::move(k), std::move(x));
        ws();
        if (p_ < e_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < e_ && *p_ == '}') {
          ++p_;
          return true;
        }
        return false;
      }
    }
    if (c == '[') {
      ++p_;
      v->kind = JVal::Arr;
      ws();
      if (p_ < e_ && *p_ == ']') {
        ++p_;
        return true;
      }
      for (;;) {
        JVal x;
        if (!value(&x, depth + 1)) return false;
        v->arr.push_back(std::move(x));
        ws();
        if (p_ < e_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < e_ && *p_ == ']') {
          ++p_;
          return true;
        }
        return false;
      }
    }
    if (c == '"') {
      v->kind = JVal::Str;
      return string(&v->str);
    }
    if (lit("true")) {
      v->kind = JVal::Bool;
      v->num = 1;
      return true;
    }
    if (lit("false")) {
      v->kind = JVal::Bool;
      return true;
    }
    if (lit("null")) return true;
    // number
    const char* s = p_;
    bool integral = true;
    if (p_ < e_ && (*p_ == '-' || *p_ == '+')) ++p_;
    while (p_ < e_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' ||
                       *p_ == '-' || *p_ == '+')) {
      if (*p_ == '.' || *p_ == 'e' || *p_ == 'E') integral = false;
      ++p_;
    }
    if (p_ == s) return false;
    const std::string t(s, p_);
    v->kind = JVal::Num;
    v->num = strtod(t.c_str(), nullptr);
    v->is_int = integral;
    if (integral) v->inum = strtoll(t.c_str(), nullptr, 10);
    return true;
  }
};

bool read_file(const std::string& path, std::string* out) {
  const int fd = open(path.c_str(), O_RDONLY);
  if (fd < 0) return false;
  struct stat st;
  if (fstat(fd, &st) != 0) {
    close(fd);
    return false;
  }
  out->resize((size_t)st.st_size);
  size_t got = 0;
  while (got < out->size()) {
    const ssize_t r = read(fd, &(*out)[got], out->size() - got);
    if (r <= 0) break;
    got += (size_t)r;
  }
  close(fd);
  return got == out->size();
}

struct Mapped {
  void* base = nullptr;
  size_t size = 0;
  size_t data_off = 0;  // 8 + header length
  ~Mapped() {
    if (base) munmap(base, size);
  }
};

struct TensorEntry {
  std::string name;       // as stored
  std::string canonical;  // with ".inner" segments removed (lib.rs:709-723 in reverse)
  int dtype = -1;
  size_t elem = 0;
  std::vector<int64_t> shape;
  int file = 0;
  size_t begin = 0, end = 0;  // absolute offsets in the mapping
};

int dtype_code(const std::string& s, size_t* elem) {
  if (s == "U32") return *elem = 4, HIGGS_DTYPE_U32;
  if (s == "I32") return *elem = 4, HIGGS_DTYPE_U32;  // same bits for packed codes
  if (s == "BF16") return *elem = 2, HIGGS_DTYPE_BF16;
  if (s == "F32") return *elem = 4, HIGGS_DTYPE_F32;
  if (s == "F16") return *elem = 2, HIGGS_DTYPE_F16;
  return -1;
}

// "a.inner.weight" -> "a.weight": the reference loader tries the flat MLX name
// first and then the name with ".inner" inserted; both name the same tensor.
std::string canonical_name(const std::string& k) {
  std::string out = k;
  const std::string seg = ".inner.";
  size_t p;
  while ((p = out.find(seg)) != std::string::npos) out.erase(p, seg.size() - 1);
  return out;
}

}  // namespace

struct higgs_safetensors {
  std::vector<std::unique_ptr<Mapped>> files;
  std::vector<TensorEntry> tensors;
  std::map<std::string, int> by_name;  // canonical and stored names
};

static int map_file(const std::string& path, higgs_safetensors* st) {
  const int fd = open(path.c_str(), O_RDONLY);
  if (fd < 0) return fail(HIGGS_ERR_INVALID_ARG, "safetensors: cannot open " + path);
  struct stat sb;
  if (fstat(fd, &sb) != 0 || sb.st_size < 8) {
    close(fd);
    return fail(HIGGS_ERR_INVALID_ARG, "safetensors: " + path + " is too short");
  }
  void* base = mmap(nullptr, (size_t)sb.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (base == MAP_FAILED) return fail(HIGGS_ERR_INVALID_ARG, "safetensors: cannot map " + path);
  auto m = std::make_unique<Mapped>();
  m->base = base;
  m->size = (size_t)sb.st_size;
  uint64_t hlen = 0;
  memcpy(&hlen, base, 8);  // little-endian on every supported host
  if (hlen > m->size - 8) return fail(HIGGS_ERR_INVALID_ARG, "safetensors: bad header length in " + path);
  m->data_off = 8 + (size_t)hlen;
  JVal root;
  JParser jp(static_cast<const char*>(base) + 8, (size_t)hlen);
  if (!jp.parse(&root) || root.kind != JVal::Obj)
    return fail(HIGGS_ERR_INVALID_ARG, "safetensors: bad header JSON in " + path);
  const int fi = (int)st->files.size();
  for (auto& kv : root.obj) {
    if (kv.first == "__metadata__") continue;
    const JVal& t = kv.second;
    const JVal* dt = t.get("dtype");
    const JVal* sh = t.get("shape");
    const JVal* off = t.get("data_offsets");
    if (!dt || dt->kind != JVal::Str || !sh || sh->kind != JVal::Arr || !off || off->kind != JVal::Arr ||
        off->arr.size() != 2)
      return fail(HIGGS_ERR_INVALID_ARG, "safetensors: bad entry '" + kv.first + "' in " + path);
    TensorEntry e;
    e.name = kv.first;
    e.canonical = canonical_name(kv.first);
    e.dtype = dtype_code(dt->str, &e.elem);
    if (e.dtype < 0)
      return fail(HIGGS_ERR_UNSUPPORTED, "safetensors: dtype " + dt->str + " of '" + kv.first + "'");
    size_t n = 1;
    for (auto& d : sh->arr) {
      if (d.kind != JVal::Num || !d.is_int || d.inum < 0)
        return fail(HIGGS_ERR_INVALID_ARG, "safetensors: bad shape of '" + kv.first + "'");
      e.shape.push_back(d.inum);
      n *= (size_t)d.inum;
    }
    if (e.shape.size() > 8) return fail(HIGGS_ERR_UNSUPPORTED, "safetensors: rank > 8 for '" + kv.first + "'");
    const int64_t b = off->arr[0].inum, en = off->arr[1].inum;
    if (b < 0 || en < b || (size_t)(en - b) != n * e.elem || m->data_off + (size_t)en > m->size)
      return fail(HIGGS_ERR_INVALID_ARG, "safetensors: bad data offsets of '" + kv.first + "'");
    e.file = fi;
    e.begin = m->data_off + (size_t)b;
    e.end = m->data_off + (size_t)en;
    st->tensors.push_back(std::move(e));
  }
  st->files.push_back(std::move(m));
  return HIGGS_OK;
}

extern "C" int higgs_safetensors_open(const char* model_dir, higgs_safetensors** out) {
  if (!model_dir || !out) return fail(HIGGS_ERR_INVALID_ARG, "higgs_safetensors_open: null argument");
  *out = nullptr;
  const std::string dir(model_dir);
  std::vector<std::string> paths;
  std::string idx;
  if (read_file(dir + "/model.safetensors.index.json", &idx)) {
    JVal root;
    JParser jp(idx.data(), idx.size());
    const JVal* wm = nullptr;
    if (!jp.parse(&root) || !(wm = root.get("weight_map")) || wm->kind != JVal::Obj)
      return fail(HIGGS_ERR_INVALID_ARG, "higgs_safetensors_open: bad model.safetensors.index.json");
    std::set<std::string> files;
    for (auto& kv : wm->obj) {
      if (kv.second.kind != JVal::Str || kv.second.str.find('/') != std::string::npos)
        return fail(HIGGS_ERR_INVALID_ARG, "higgs_safetensors_open: bad weight_map entry '" + kv.first + "'");
      files.insert(kv.second.str);
    }
    for (auto& f : files) paths.push_back(dir + "/" + f);
  } else {
    struct stat sb;
    if (stat((dir + "/model.safetensors").c_str(), &sb) != 0)
      return fail(HIGGS_ERR_INVALID_ARG, "higgs_safetensors_open: no safetensors files found in " + dir);
    paths.push_back(dir + "/model.safetensors");
  }
  auto st = std::make_unique<higgs_safetensors>();
  for (auto& p : paths)
    if (int rc = map_file(p, st.get())) return rc;
  std::sort(st->tensors.begin(), st->tensors.end(),
            [](const TensorEntry& a, const TensorEntry& b) { return a.name < b.name; });
  for (int i = 0; i < (int)st->tensors.size(); ++i) {
    const TensorEntry& e = st->tensors[i];
    if (!st->by_name.emplace(e.name, i).second)
      return fail(HIGGS_ERR_INVALID_ARG, "higgs_safetensors_open: tensor '" + e.name + "' stored twice");
    st->by_name.emplace(e.canonical, i);
  }
  *out = st.release();
  return HIGGS_OK;
}

extern "C" int higgs_safetensors_close(higgs_safetensors* st) {
  delete st;
  return HIGGS_OK;
}

extern "C" int higgs_safetensors_count(const higgs_safetensors* st) {
  return st ? (int)st->tensors.size() : 0;
}

extern "C" int higgs_safetensors_find(const higgs_safetensors* st, const char* name) {
  if (!st || !name) return -1;
  auto it = st->by_name.find(name);
  if (it == st->by_name.end()) it = st->by_name.find(canonical_name(name));
  return it == st->by_name.end() ? -1 : it->second;
}

extern "C" int higgs_safetensors_info(const higgs_safetensors* st, int i, const char** name,
                                      int* dtype, int* ndim, int64_t* shape) {
  if (!st || i < 0 || i >= (int)st->tensors.size())
    return fail(HIGGS_ERR_INVALID_ARG, "higgs_safetensors_info: bad tensor index");
  const TensorEntry& e = st->tensors[i];
  if (name) *name = e.canonical.c_str();
  if (dtype) *dtype = e.dtype;
  if (ndim) *ndim = (int)e.shape.size();
  if (shape)
    for (size_t d = 0; d < e.shape.size(); ++d) shape[d] = e.shape[d];
  return HIGGS_OK;
}

extern "C" int higgs_safetensors_read(higgs_ctx* ctx, const higgs_safetensors* st, int i, int64_t row0,
                                      int64_t rows, int64_t col0, int64_t cols, void* dst,
                                      int dst_on_device, void* stream) {
  if (!st || !dst || i < 0 || i >= (int)st->tensors.size())
    return fail(HIGGS_ERR_INVALID_ARG, "higgs_safetensors_read: bad argument");
  const TensorEntry& e = st->tensors[i];
  const int64_t ncols = e.shape.empty() ? 1 : e.shape.back();
  int64_t nrows = 1;
  for (size_t d = 0; d + 1 < e.shape.size(); ++d) nrows *= e.shape[d];
  if (row0 < 0 || rows < 0 || col0 < 0 || cols < 0 || row0 + rows > nrows || col0 + cols > ncols)
    return fail(HIGGS_ERR_INVALID_ARG, "higgs_safetensors_read: slice outside '" + e.name + "'");
  if (rows == 0 || cols == 0) return HIGGS_OK;
  const char* src = static_cast<const char*>(st->files[e.file]->base) + e.begin +
                    ((size_t)row0 * (size_t)ncols + (size_t)col0) * e.elem;
  const size_t pitch = (size_t)ncols * e.elem, width = (size_t)cols * e.elem;
  if (!dst_on_device) {
    char* d = static_cast<char*>(dst);
    for (int64_t r = 0; r < rows; ++r) memcpy(d + (size_t)r * width, src + (size_t)r * pitch, width);
    return HIGGS_OK;
  }
  if (!ctx) return fail(HIGGS_ERR_INVALID_ARG, "higgs_safetensors_read: a device copy needs a context");
  HG_DEVICE(ctx);
  HG_CUDA(cudaMemcpy2DAsync(dst, width, src, pitch, width, (size_t)rows, cudaMemcpyHostToDevice,
                            (cudaStream_t)stream));
  // complete before returning: the caller may close the mapping right after
  HG_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  return HIGGS_OK;
}
