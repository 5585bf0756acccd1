// model_files.cu -- host-side readers of the two weight containers the denoiser loads:
// GGUF v3 (the format of crates/sketchpad-convert/src/gguf.rs:351-470, whose Q8_0 and K-quant
// tensors feed sp_q8_0_repack_host / sp_kquant_repack_host) and safetensors (the format of
// crates/sketchpad-convert/src/loader.rs:60-90, plus F8_E4M3 tensors for the FP8 linears).
// Files are memory-mapped read-only; tensor bytes are returned as pointers into the map.
// Host code only: nothing here touches a GPU.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"

namespace sp {
namespace {

struct TensorRec {
  std::string name;
  int type = -1;  // sp_tensor_type
  std::vector<int64_t> dims;  // row-major (slowest first)
  uint64_t offset = 0;        // from the start of the file
  uint64_t nbytes = 0;
};

struct ModelFile {
  int fd = -1;
  const uint8_t* map = nullptr;
  size_t size = 0;
  int container = 0;  // SP_CONTAINER_*
  std::vector<TensorRec> tensors;
  std::unordered_map<std::string, int64_t> by_name;
  std::vector<std::string> meta_keys;
  ~ModelFile() {
    if (map) munmap(const_cast<uint8_t*>(map), size);
    if (fd >= 0) close(fd);
  }
};

// ---------------------------------------------------------------------------- GGUF
// ggml type ids with their (block elements, block bytes) -- gguf.rs:18-38, :130-166
bool ggml_block(uint32_t t, int* elems, int* bytes) {
  struct E { uint32_t id; int n, b; };
  static const E table[] = {{0, 1, 4},     {1, 1, 2},      {2, 32, 18},    {3, 32, 20},
                            {6, 32, 22},   {7, 32, 24},    {8, 32, 34},    {10, 256, 84},
                            {11, 256, 110}, {12, 256, 144}, {13, 256, 176}, {14, 256, 210},
                            {16, 256, 66}, {17, 256, 74},  {18, 256, 98},  {19, 256, 50},
                            {20, 32, 18},  {21, 256, 110}, {22, 256, 82},  {23, 256, 136},
                            {29, 256, 56}};
  for (const E& e : table)
    if (e.id == t) {
      *elems = e.n;
      *bytes = e.b;
      return true;
    }
  return false;
}

struct Cursor {
  const uint8_t* p;
  size_t n, pos = 0;
  bool ok = true;
  bool take(void* dst, size_t k) {
    if (!ok || k > n - pos) return ok = false;
    std::memcpy(dst, p + pos, k);
    pos += k;
    return true;
  }
  uint32_t u32() { uint32_t v = 0; take(&v, 4); return v; }
  uint64_t u64() { uint64_t v = 0; take(&v, 8); return v; }
  std::string str() {
    const uint64_t len = u64();
    if (!ok || len > n - pos) { ok = false; return {}; }
    std::string s(reinterpret_cast<const char*>(p + pos), (size_t)len);
    pos += (size_t)len;
    return s;
  }
  bool skip(uint64_t k) {
    if (!ok || k > n - pos) return ok = false;
    pos += (size_t)k;
    return true;
  }
};

// skips one metadata value of type t (gguf.rs:320-345: 0..12, arrays recursive)
bool skip_value(Cursor& c, uint32_t t, int depth) {
  static const int fixed[13] = {1, 1, 2, 2, 4, 4, 4, 1, -1, -2, 8, 8, 8};
  if (t > 12 || depth > 8) return false;
  if (fixed[t] > 0) return c.skip((uint64_t)fixed[t]);
  if (t == 8) { c.str(); return c.ok; }
  const uint32_t et = c.u32();
  const uint64_t count = c.u64();
  if (!c.ok) return false;
  if (et <= 12 && fixed[et] > 0) {
    if (count > (c.n - c.pos) / (uint64_t)fixed[et]) return c.ok = false;
    return c.skip(count * (uint64_t)fixed[et]);
  }
  for (uint64_t i = 0; i < count; ++i)
    if (!skip_value(c, et, depth + 1)) return false;
  return true;
}

int parse_gguf(ModelFile& f) {
  Cursor c{f.map, f.size};
  const uint32_t magic = c.u32(), version = c.u32();
  if (magic != 0x46554747u) return set_error(SP_ERR_INVALID_ARG, "not a GGUF file");
  // the reference reads version 3 only (gguf.rs:366-369)
  if (version != 3) return set_error(SP_ERR_INVALID_ARG, "unsupported GGUF version %u", version);
  const uint64_t ntensors = c.u64(), nkv = c.u64();
  if (!c.ok || ntensors > (1u << 24) || nkv > (1u << 24))
    return set_error(SP_ERR_INVALID_ARG, "GGUF header is truncated or implausible");
  for (uint64_t i = 0; i < nkv; ++i) {
    std::string key = c.str();
    const uint32_t t = c.u32();
    if (!c.ok || !skip_value(c, t, 0))
      return set_error(SP_ERR_INVALID_ARG, "GGUF metadata entry %llu is malformed",
                       (unsigned long long)i);
    f.meta_keys.push_back(std::move(key));
  }
  std::vector<uint64_t> rel;
  for (uint64_t i = 0; i < ntensors; ++i) {
    TensorRec r;
    r.name = c.str();
    const uint32_t nd = c.u32();
    if (!c.ok || nd == 0 || nd > 8) return set_error(SP_ERR_INVALID_ARG, "GGUF tensor %llu: bad rank",
                                                     (unsigned long long)i);
    r.dims.resize(nd);
    for (uint32_t d = 0; d < nd; ++d) r.dims[d] = (int64_t)c.u64();
    const uint32_t t = c.u32();
    const uint64_t off = c.u64();
    if (!c.ok) return set_error(SP_ERR_INVALID_ARG, "GGUF tensor table is truncated");
    int be = 0, bb = 0;
    if (!ggml_block(t, &be, &bb))
      return set_error(SP_ERR_DTYPE, "GGUF tensor '%s': unsupported ggml type %u", r.name.c_str(), t);
    // innermost dimension first on disk; reversed to row-major as the reference does
    // (gguf.rs:392-395)
    std::vector<int64_t> rev(r.dims.rbegin(), r.dims.rend());
    r.dims = rev;
    uint64_t elems = 1;
    for (int64_t d : r.dims) {
      if (d <= 0 || (uint64_t)d > (1ull << 40) || elems > (1ull << 40) / (uint64_t)d)
        return set_error(SP_ERR_SHAPE, "GGUF tensor '%s': bad dimension", r.name.c_str());
      elems *= (uint64_t)d;
    }
    if (elems % (uint64_t)be) return set_error(SP_ERR_SHAPE, "GGUF tensor '%s': %llu elements are "
                                               "not whole blocks", r.name.c_str(),
                                               (unsigned long long)elems);
    r.nbytes = elems / (uint64_t)be * (uint64_t)bb;
    r.type = t == 0 ? SP_T_F32 : t == 1 ? SP_T_F16 : SP_T_GGML_BASE + (int)t;
    rel.push_back(off);
    f.tensors.push_back(std::move(r));
  }
  // tensor data start: the header end rounded up to 32 bytes (gguf.rs:15, :406)
  const uint64_t base = (c.pos + 31) & ~uint64_t(31);
  for (size_t i = 0; i < f.tensors.size(); ++i) {
    TensorRec& r = f.tensors[i];
    if (base > f.size || rel[i] > f.size - base)
      return set_error(SP_ERR_SHAPE, "GGUF tensor '%s' starts past the end of the file",
                       r.name.c_str());
    r.offset = base + rel[i];
    if (r.nbytes > f.size - r.offset)
      return set_error(SP_ERR_SHAPE, "GGUF tensor '%s' runs past the end of the file",
                       r.name.c_str());
  }
  return SP_OK;
}

// ---------------------------------------------------------------------------- safetensors
// The header is a JSON object {name: {"dtype": s, "shape": [..], "data_offsets": [b, e]},
// "__metadata__": {..}}; a small recursive-descent reader covers what it may contain.
struct Json {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
  const Json* get(const char* k) const {
    for (const auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct JsonReader {
  const char* s;
  size_t n, i = 0;
  bool ok = true;
  void ws() { while (i < n && (s[i] == ' ' || s[i] == '\t' || s[i] == '\n' || s[i] == '\r')) ++i; }
  bool lit(const char* w) {
    const size_t k = std::strlen(w);
    if (n - i < k || std::memcmp(s + i, w, k)) return ok = false;
    i += k;
    return true;
  }
  std::string string() {
    std::string out;
    if (i >= n || s[i] != '"') { ok = false; return out; }
    ++i;
    while (i < n && s[i] != '"') {
      char ch = s[i++];
      if (ch == '\\') {
        if (i >= n) { ok = false; return out; }
        const char e = s[i++];
        switch (e) {
          case 'n': ch = '\n'; break;
          case 't': ch = '\t'; break;
          case 'r': ch = '\r'; break;
          case 'b': ch = '\b'; break;
          case 'f': ch = '\f'; break;
          case 'u': {  // \uXXXX as UTF-8 (tensor names are ASCII in practice)
            if (n - i < 4) { ok = false; return out; }
            unsigned cp = 0;
            for (int h = 0; h < 4; ++h) {  // no exceptions may leave this library
              const char d = s[i + h];
              const int v = d >= '0' && d <= '9' ? d - '0'
                            : d >= 'a' && d <= 'f' ? d - 'a' + 10
                            : d >= 'A' && d <= 'F' ? d - 'A' + 10 : -1;
              if (v < 0) { ok = false; return out; }
              cp = cp * 16 + (unsigned)v;
            }
            i += 4;
            if (cp < 0x80) { out += (char)cp; }
            else if (cp < 0x800) { out += (char)(0xC0 | (cp >> 6)); out += (char)(0x80 | (cp & 0x3F)); }
            else { out += (char)(0xE0 | (cp >> 12)); out += (char)(0x80 | ((cp >> 6) & 0x3F));
                   out += (char)(0x80 | (cp & 0x3F)); }
            continue;
          }
          default: ch = e;  // \" \\ \/
        }
      }
      out += ch;
    }
    if (i >= n) { ok = false; return out; }
    ++i;
    return out;
  }
  Json value(int depth) {
    Json v;
    ws();
    if (!ok || i >= n || depth > 32) { ok = false; return v; }
    const char c = s[i];
    if (c == '{') {
      v.kind = Json::Obj;
      ++i;
      ws();
      if (i < n && s[i] == '}') { ++i; return v; }
      while (ok) {
        ws();
        std::string k = string();
        ws();
        if (!ok || i >= n || s[i] != ':') { ok = false; break; }
        ++i;
        Json x = value(depth + 1);
        v.obj.emplace_back(std::move(k), std::move(x));
        ws();
        if (i < n && s[i] == ',') { ++i; continue; }
        if (i < n && s[i] == '}') { ++i; break; }
        ok = false;
      }
    } else if (c == '[') {
      v.kind = Json::Arr;
      ++i;
      ws();
      if (i < n && s[i] == ']') { ++i; return v; }
      while (ok) {
        v.arr.push_back(value(depth + 1));
        ws();
        if (i < n && s[i] == ',') { ++i; continue; }
        if (i < n && s[i] == ']') { ++i; break; }
        ok = false;
      }
    } else if (c == '"') {
      v.kind = Json::Str;
      v.str = string();
    } else if (c == 't') {
      v.kind = Json::Bool; v.num = 1; lit("true");
    } else if (c == 'f') {
      v.kind = Json::Bool; lit("false");
    } else if (c == 'n') {
      lit("null");
    } else {
      v.kind = Json::Num;
      const size_t j = i;
      while (i < n && (std::strchr("+-0123456789.eE", s[i]) != nullptr)) ++i;
      if (i == j) { ok = false; return v; }
      v.num = std::strtod(std::string(s + j, i - j).c_str(), nullptr);
    }
    return v;
  }
};

int safetensors_type(const std::string& d, int* elem) {
  struct E { const char* name; int type, size; };
  static const E table[] = {{"F64", SP_T_F64, 8},  {"F32", SP_T_F32, 4},  {"F16", SP_T_F16, 2},
                            {"BF16", SP_T_BF16, 2}, {"F8_E4M3", SP_T_F8_E4M3, 1},
                            {"F8_E5M2", SP_T_F8_E5M2, 1}, {"I64", SP_T_I64, 8},
                            {"I32", SP_T_I32, 4},  {"I16", SP_T_I16, 2},  {"I8", SP_T_I8, 1},
                            {"U8", SP_T_U8, 1},    {"BOOL", SP_T_BOOL, 1}};
  for (const E& e : table)
    if (d == e.name) {
      *elem = e.size;
      return e.type;
    }
  return -1;
}

int parse_safetensors(ModelFile& f) {
  if (f.size < 8) return set_error(SP_ERR_INVALID_ARG, "file too small for safetensors");
  uint64_t hlen = 0;
  std::memcpy(&hlen, f.map, 8);
  if (hlen > f.size - 8 || hlen > (100u << 20))
    return set_error(SP_ERR_INVALID_ARG, "safetensors header length %llu is implausible",
                     (unsigned long long)hlen);
  JsonReader jr{reinterpret_cast<const char*>(f.map + 8), (size_t)hlen};
  const Json root = jr.value(0);
  if (!jr.ok || root.kind != Json::Obj)
    return set_error(SP_ERR_INVALID_ARG, "safetensors header is not a JSON object");
  const uint64_t base = 8 + hlen;
  for (const auto& kv : root.obj) {
    if (kv.first == "__metadata__") {
      for (const auto& m : kv.second.obj) f.meta_keys.push_back(m.first);
      continue;
    }
    const Json& t = kv.second;
    const Json* dt = t.get("dtype");
    const Json* sh = t.get("shape");
    const Json* off = t.get("data_offsets");
    if (!dt || dt->kind != Json::Str || !sh || sh->kind != Json::Arr || !off ||
        off->kind != Json::Arr || off->arr.size() != 2)
      return set_error(SP_ERR_INVALID_ARG, "safetensors entry '%s' is malformed", kv.first.c_str());
    TensorRec r;
    r.name = kv.first;
    int es = 0;
    r.type = safetensors_type(dt->str, &es);
    if (r.type < 0)
      return set_error(SP_ERR_DTYPE, "safetensors tensor '%s': unknown dtype %s", r.name.c_str(),
                       dt->str.c_str());
    uint64_t elems = 1;
    if (sh->arr.size() > 8)
      return set_error(SP_ERR_SHAPE, "safetensors tensor '%s': rank above 8", r.name.c_str());
    auto whole = [](const Json& v) {  // a non-negative integer JSON number below 2^53
      return v.kind == Json::Num && v.num >= 0 && v.num < 9007199254740992.0 &&
             v.num == (double)(uint64_t)v.num;
    };
    for (const Json& d : sh->arr) {
      if (!whole(d) || d.num > (double)(1ull << 40) || elems > (1ull << 40) / ((uint64_t)d.num + 1))
        return set_error(SP_ERR_SHAPE, "safetensors tensor '%s': bad shape", r.name.c_str());
      r.dims.push_back((int64_t)d.num);
      elems *= (uint64_t)d.num;
    }
    if (!whole(off->arr[0]) || !whole(off->arr[1]))
      return set_error(SP_ERR_SHAPE, "safetensors tensor '%s': bad data_offsets", r.name.c_str());
    const uint64_t b = (uint64_t)off->arr[0].num, e = (uint64_t)off->arr[1].num;
    if (e < b || e - b != elems * (uint64_t)es || e > f.size - base)
      return set_error(SP_ERR_SHAPE, "safetensors tensor '%s': offsets [%llu, %llu) do not match "
                       "its shape or the file", r.name.c_str(), (unsigned long long)b,
                       (unsigned long long)e);
    r.offset = base + b;
    r.nbytes = e - b;
    f.tensors.push_back(std::move(r));
  }
  return SP_OK;
}

ModelFile* as_file(void* h) { return static_cast<ModelFile*>(h); }

}  // namespace
}  // namespace sp

extern "C" {

int sp_model_open(const char* path, void** file_out) {
  using namespace sp;
  clear_error();
  if (!path || !file_out) return set_error(SP_ERR_INVALID_ARG, "model open: null argument");
  *file_out = nullptr;
  auto* f = new ModelFile();
  f->fd = open(path, O_RDONLY | O_CLOEXEC);
  struct stat st;
  if (f->fd < 0 || fstat(f->fd, &st) != 0 || st.st_size <= 0) {
    delete f;
    return set_error(SP_ERR_INVALID_ARG, "cannot open '%s'", path);
  }
  f->size = (size_t)st.st_size;
  void* m = mmap(nullptr, f->size, PROT_READ, MAP_PRIVATE, f->fd, 0);
  if (m == MAP_FAILED) {
    delete f;
    return set_error(SP_ERR_INVALID_ARG, "cannot map '%s'", path);
  }
  f->map = static_cast<const uint8_t*>(m);
  uint32_t magic = 0;
  if (f->size >= 4) std::memcpy(&magic, f->map, 4);
  f->container = magic == 0x46554747u ? SP_CONTAINER_GGUF : SP_CONTAINER_SAFETENSORS;
  int rc;
  try {  // nothing may throw across the C ABI (allocation failure on a hostile header)
    rc = f->container == SP_CONTAINER_GGUF ? parse_gguf(*f) : parse_safetensors(*f);
  } catch (...) {
    rc = set_error(SP_ERR_INVALID_ARG, "'%s' could not be parsed", path);
  }
  if (rc != SP_OK) {
    delete f;
    return rc;
  }
  for (size_t i = 0; i < f->tensors.size(); ++i) f->by_name[f->tensors[i].name] = (int64_t)i;
  *file_out = f;
  return SP_OK;
}

int sp_model_close(void* file) {
  sp::clear_error();
  if (!file) return sp::set_error(SP_ERR_INVALID_ARG, "model close: null handle");
  delete sp::as_file(file);
  return SP_OK;
}

int sp_model_info(void* file, int* container_out, int64_t* tensor_count_out,
                  int64_t* meta_count_out) {
  sp::clear_error();
  if (!file || !container_out || !tensor_count_out || !meta_count_out)
    return sp::set_error(SP_ERR_INVALID_ARG, "model info: null argument");
  const sp::ModelFile* f = sp::as_file(file);
  *container_out = f->container;
  *tensor_count_out = (int64_t)f->tensors.size();
  *meta_count_out = (int64_t)f->meta_keys.size();
  return SP_OK;
}

int sp_model_meta_key(void* file, int64_t index, char* name_out, size_t name_cap) {
  sp::clear_error();
  if (!file || !name_out || name_cap == 0) return sp::set_error(SP_ERR_INVALID_ARG, "meta key: null argument");
  const sp::ModelFile* f = sp::as_file(file);
  if (index < 0 || index >= (int64_t)f->meta_keys.size())
    return sp::set_error(SP_ERR_INVALID_ARG, "meta key: index out of range");
  const std::string& k = f->meta_keys[(size_t)index];
  if (k.size() + 1 > name_cap) return sp::set_error(SP_ERR_INVALID_ARG, "meta key: buffer too small");
  std::memcpy(name_out, k.c_str(), k.size() + 1);
  return SP_OK;
}

int sp_model_tensor_info(void* file, int64_t index, char* name_out, size_t name_cap,
                         int* type_out, int* ndims_out, int64_t dims_out[8],
                         uint64_t* nbytes_out) {
  sp::clear_error();
  if (!file || !name_out || name_cap == 0 || !type_out || !ndims_out || !dims_out || !nbytes_out)
    return sp::set_error(SP_ERR_INVALID_ARG, "tensor info: null argument");
  const sp::ModelFile* f = sp::as_file(file);
  if (index < 0 || index >= (int64_t)f->tensors.size())
    return sp::set_error(SP_ERR_INVALID_ARG, "tensor info: index out of range");
  const sp::TensorRec& r = f->tensors[(size_t)index];
  if (r.name.size() + 1 > name_cap)
    return sp::set_error(SP_ERR_INVALID_ARG, "tensor info: name buffer too small");
  std::memcpy(name_out, r.name.c_str(), r.name.size() + 1);
  *type_out = r.type;
  *ndims_out = (int)r.dims.size();
  for (int i = 0; i < 8; ++i) dims_out[i] = i < (int)r.dims.size() ? r.dims[i] : 0;
  *nbytes_out = r.nbytes;
  return SP_OK;
}

int sp_model_find(void* file, const char* name, int64_t* index_out) {
  sp::clear_error();
  if (!file || !name || !index_out) return sp::set_error(SP_ERR_INVALID_ARG, "find: null argument");
  const sp::ModelFile* f = sp::as_file(file);
  auto it = f->by_name.find(name);
  if (it == f->by_name.end()) return sp::set_error(SP_ERR_INVALID_ARG, "tensor '%s' not found", name);
  *index_out = it->second;
  return SP_OK;
}

int sp_model_tensor_data(void* file, int64_t index, const uint8_t** data_out) {
  sp::clear_error();
  if (!file || !data_out) return sp::set_error(SP_ERR_INVALID_ARG, "tensor data: null argument");
  const sp::ModelFile* f = sp::as_file(file);
  if (index < 0 || index >= (int64_t)f->tensors.size())
    return sp::set_error(SP_ERR_INVALID_ARG, "tensor data: index out of range");
  *data_out = f->map + f->tensors[(size_t)index].offset;
  return SP_OK;
}

}  // extern "C"
