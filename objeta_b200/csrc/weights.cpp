// weights.cpp -- safetensors weights for the expert path: ModelWeights
// (crates/objeta-parser/src/lib.rs:97-330) as a C++ mmap loader whose tensors
// can be pinned for DMA and fed to the expert cache or copied to the device.
//
// A file is [u64 header length][JSON header][data]; the header maps tensor
// names to {dtype, shape, data_offsets: [begin, end)} relative to the data
// start, plus an ignored "__metadata__" object.  A directory is every
// *.safetensors file in it, in file-name order (later files win on
// duplicate names, as the reference's HashMap insert does).
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <dirent.h>
#include <map>
#include <string>
#include <vector>

#include "objb_common.h"

namespace objb {
namespace {

struct Tensor {
  int dtype;  // OBJB_DTYPE_*
  std::vector<size_t> shape;
  size_t file;     // index into files
  size_t offset;   // absolute byte offset in the file
  size_t nbytes;
  size_t nelem;
};

struct MappedFile {
  void* base = nullptr;   // what tensor pointers are taken from (the mapping, or the pinned slab)
  void* map = nullptr;    // the mmap
  size_t size = 0;
  bool registered = false;  // the mapping itself is pinned
  void* slab = nullptr;     // pinned copy when the mapping cannot be registered
};

int dtype_from_str(const std::string& s) {
  if (s == "F32" || s == "FLOAT32") return OBJB_DTYPE_F32;
  if (s == "F16" || s == "FLOAT16") return OBJB_DTYPE_F16;
  if (s == "BF16" || s == "BFLOAT16") return OBJB_DTYPE_BF16;
  if (s == "I64" || s == "INT64") return OBJB_DTYPE_I64;
  if (s == "I32" || s == "INT32") return OBJB_DTYPE_I32;
  if (s == "I8" || s == "INT8") return OBJB_DTYPE_I8;
  if (s == "U8" || s == "UINT8") return OBJB_DTYPE_U8;
  if (s == "F8_E8M0") return OBJB_DTYPE_F8_E8M0;
  if (s == "F8_E4M3") return OBJB_DTYPE_F8_E4M3;
  if (s == "BOOL") return OBJB_DTYPE_BOOL;
  return -1;
}

size_t dtype_size(int d) {
  switch (d) {
    case OBJB_DTYPE_F32:
    case OBJB_DTYPE_I32: return 4;
    case OBJB_DTYPE_F16:
    case OBJB_DTYPE_BF16: return 2;
    case OBJB_DTYPE_I64: return 8;
    default: return 1;
  }
}

// A small JSON reader for the safetensors header: objects, arrays, strings
// (with escapes), numbers, true / false / null.
struct Json {
  const char* p;
  const char* end;
  std::string error;

  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool fail(const std::string& m) {
    if (error.empty()) error = m;
    return false;
  }
  bool expect(char c) {
    ws();
    if (p >= end || *p != c) return fail(std::string("expected '") + c + "'");
    ++p;
    return true;
  }
  bool string(std::string* out) {
    ws();
    if (p >= end || *p != '"') return fail("expected a string");
    ++p;
    out->clear();
    while (p < end && *p != '"') {
      if (*p == '\\') {
        if (++p >= end) return fail("unterminated escape");
        const char c = *p++;
        if (c == 'u') {
          if (end - p < 4) return fail("short \\u escape");
          unsigned v = 0;
          for (int i = 0; i < 4; ++i) {
            const char h = *p++;
            v = v * 16 + (h >= '0' && h <= '9' ? h - '0' : h >= 'a' && h <= 'f' ? h - 'a' + 10
                                                          : h >= 'A' && h <= 'F' ? h - 'A' + 10 : 0);
          }
          if (v < 0x80) {
            out->push_back(static_cast<char>(v));
          } else if (v < 0x800) {
            out->push_back(static_cast<char>(0xC0 | (v >> 6)));
            out->push_back(static_cast<char>(0x80 | (v & 0x3F)));
          } else {
            out->push_back(static_cast<char>(0xE0 | (v >> 12)));
            out->push_back(static_cast<char>(0x80 | ((v >> 6) & 0x3F)));
            out->push_back(static_cast<char>(0x80 | (v & 0x3F)));
          }
        } else {
          out->push_back(c == 'n' ? '\n' : c == 't' ? '\t' : c == 'r' ? '\r' : c == 'b' ? '\b' : c == 'f' ? '\f' : c);
        }
      } else {
        out->push_back(*p++);
      }
    }
    if (p >= end) return fail("unterminated string");
    ++p;
    return true;
  }
  bool number(size_t* out) {
    ws();
    if (p >= end || *p < '0' || *p > '9') return fail("expected a non-negative integer");
    size_t v = 0;
    while (p < end && *p >= '0' && *p <= '9') {
      const size_t d = static_cast<size_t>(*p++ - '0');
      if (v > (SIZE_MAX - d) / 10) return fail("integer overflow");
      v = v * 10 + d;
    }
    *out = v;
    return true;
  }
  bool skip_value(int depth = 0) {
    ws();
    if (depth > 64) return fail("nesting too deep");
    if (p >= end) return fail("unexpected end");
    if (*p == '"') {
      std::string s;
      return string(&s);
    }
    if (*p == '{' || *p == '[') {
      const char close = *p == '{' ? '}' : ']';
      const bool obj = *p == '{';
      ++p;
      ws();
      if (p < end && *p == close) {
        ++p;
        return true;
      }
      for (;;) {
        if (obj) {
          std::string k;
          if (!string(&k) || !expect(':')) return false;
        }
        if (!skip_value(depth + 1)) return false;
        ws();
        if (p < end && *p == ',') {
          ++p;
          continue;
        }
        return expect(close);
      }
    }
    while (p < end && *p != ',' && *p != '}' && *p != ']' && *p != ' ' && *p != '\n') ++p;  // literal
    return true;
  }
  bool size_array(std::vector<size_t>* out) {
    if (!expect('[')) return false;
    out->clear();
    ws();
    if (p < end && *p == ']') {
      ++p;
      return true;
    }
    for (;;) {
      size_t v;
      if (!number(&v)) return false;
      out->push_back(v);
      ws();
      if (p < end && *p == ',') {
        ++p;
        continue;
      }
      return expect(']');
    }
  }
};

}  // namespace
}  // namespace objb

struct objb_weights {
  std::vector<objb::MappedFile> files;
  std::map<std::string, objb::Tensor> index;
  std::vector<const std::string*> names;  // sorted, for enumeration
};

namespace objb {
namespace {

int parse_file(objb_weights* w, const std::string& path) {
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) return OBJB_FAIL(OBJB_ERR_IO, "open safetensors", path + ": " + std::strerror(errno));
  struct stat st;
  if (fstat(fd, &st) != 0) {
    ::close(fd);
    return OBJB_FAIL(OBJB_ERR_IO, "stat safetensors", path);
  }
  const size_t size = static_cast<size_t>(st.st_size);
  if (size < 8) {
    ::close(fd);
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "parse safetensors header", path + ": file too short");
  }
  void* base = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (base == MAP_FAILED) return OBJB_FAIL(OBJB_ERR_IO, "mmap safetensors", path + ": " + std::strerror(errno));
  const size_t fi = w->files.size();
  MappedFile mf;
  mf.base = base;
  mf.map = base;
  mf.size = size;
  w->files.push_back(mf);
  uint64_t hlen = 0;
  std::memcpy(&hlen, base, 8);  // little-endian u64
  if (hlen > size - 8)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "parse safetensors header", path + ": header length exceeds file size");
  const char* h = static_cast<const char*>(base) + 8;
  const size_t data_start = 8 + static_cast<size_t>(hlen);
  Json js{h, h + hlen, {}};
  if (!js.expect('{')) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "parse safetensors header", "invalid header JSON: " + js.error);
  js.ws();
  if (js.p < js.end && *js.p == '}') return OBJB_OK;
  for (;;) {
    std::string name;
    if (!js.string(&name) || !js.expect(':'))
      return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "parse safetensors header", "invalid header JSON: " + js.error);
    if (name == "__metadata__") {
      if (!js.skip_value())
        return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "parse safetensors header", "invalid header JSON: " + js.error);
    } else {
      Tensor t{};
      t.file = fi;
      std::string dtype;
      bool have_d = false, have_s = false, have_o = false;
      std::vector<size_t> offs;
      if (!js.expect('{'))
        return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "parse safetensors header", "invalid tensor entry for '" + name + "'");
      for (;;) {
        std::string key;
        if (!js.string(&key) || !js.expect(':'))
          return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "parse safetensors header", "invalid tensor entry for '" + name + "'");
        bool ok;
        if (key == "dtype") {
          ok = js.string(&dtype);
          have_d = true;
        } else if (key == "shape") {
          ok = js.size_array(&t.shape);
          have_s = true;
        } else if (key == "data_offsets") {
          ok = js.size_array(&offs);
          have_o = true;
        } else {
          ok = js.skip_value();
        }
        if (!ok)
          return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "parse safetensors header",
                           "invalid tensor entry for '" + name + "': " + js.error);
        js.ws();
        if (js.p < js.end && *js.p == ',') {
          ++js.p;
          continue;
        }
        if (!js.expect('}'))
          return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "parse safetensors header", "invalid tensor entry for '" + name + "'");
        break;
      }
      if (!have_d || !have_s || !have_o || offs.size() != 2 || offs[1] < offs[0])
        return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "parse safetensors header",
                         "invalid tensor entry for '" + name + "': missing dtype, shape or data_offsets");
      t.dtype = dtype_from_str(dtype);
      if (t.dtype < 0)
        return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "parse safetensors header", "Unknown dtype: " + dtype);
      t.nelem = 1;
      for (size_t d : t.shape) t.nelem *= d;
      t.nbytes = offs[1] - offs[0];
      t.offset = data_start + offs[0];
      if (t.offset + t.nbytes > size || t.offset + t.nbytes < t.offset)
        return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "parse safetensors header",
                         "tensor '" + name + "' data lies outside the file");
      w->index[name] = t;
    }
    js.ws();
    if (js.p < js.end && *js.p == ',') {
      ++js.p;
      continue;
    }
    if (!js.expect('}')) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "parse safetensors header", "invalid header JSON: " + js.error);
    break;
  }
  return OBJB_OK;
}

const Tensor* find(objb_weights* w, const char* name) {
  if (!w || !name) return nullptr;
  auto it = w->index.find(name);
  return it == w->index.end() ? nullptr : &it->second;
}

int missing(const char* name) {
  return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "get tensor", std::string("missing tensor: ") + (name ? name : "(null)"));
}

// half_to_f32 (objeta-parser lib.rs:285-310): subnormals as m * 2^-24.
float half_to_f32(uint16_t h) {
  const uint32_t sign = h >> 15, exp = (h >> 10) & 0x1F, man = h & 0x3FF;
  if (exp == 0) {
    if (man == 0) {
      uint32_t b = sign << 31;
      float f;
      std::memcpy(&f, &b, 4);
      return f;
    }
    const float v = static_cast<float>(man) * std::ldexp(1.0f, 1 - 15 - 10);
    return sign ? -v : v;
  }
  if (exp == 31) {
    if (man == 0) {
      uint32_t b = (sign << 31) | 0x7F800000u;
      float f;
      std::memcpy(&f, &b, 4);
      return f;
    }
    return NAN;
  }
  uint32_t b = (sign << 31) | ((exp + (127 - 15)) << 23) | (man << 13);
  float f;
  std::memcpy(&f, &b, 4);
  return f;
}

}  // namespace
}  // namespace objb

using namespace objb;

extern "C" {

int objb_weights_open(const char* path, objb_weights** out) {
  clear_error();
  if (!path || !out) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_weights_open", "null argument");
  *out = nullptr;
  struct stat st;
  if (stat(path, &st) != 0) return OBJB_FAIL(OBJB_ERR_IO, "open safetensors", std::string(path) + ": " + std::strerror(errno));
  auto* w = new objb_weights();
  int rc = OBJB_OK;
  if (S_ISDIR(st.st_mode)) {
    std::vector<std::string> files;
    DIR* d = opendir(path);
    if (!d) {
      delete w;
      return OBJB_FAIL(OBJB_ERR_IO, "read shard directory", path);
    }
    while (dirent* e = readdir(d)) {
      const std::string n = e->d_name;
      if (n.size() > 12 && n.compare(n.size() - 12, 12, ".safetensors") == 0) files.push_back(n);
    }
    closedir(d);
    std::sort(files.begin(), files.end());
    for (const auto& f : files) {
      rc = parse_file(w, std::string(path) + "/" + f);
      if (rc != OBJB_OK) break;
    }
  } else {
    rc = parse_file(w, path);
  }
  if (rc != OBJB_OK) {
    objb_weights_close(w);
    return rc;
  }
  for (const auto& kv : w->index) w->names.push_back(&kv.first);
  *out = w;
  return OBJB_OK;
}

void objb_weights_close(objb_weights* w) {
  if (!w) return;
  for (auto& f : w->files) {
    if (f.registered) cudaHostUnregister(f.map);
    if (f.slab) cudaFreeHost(f.slab);
    if (f.map) munmap(f.map, f.size);
  }
  delete w;
}

int objb_weights_count(objb_weights* w, size_t* n) {
  clear_error();
  if (!w || !n) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_weights_count", "null argument");
  *n = w->index.size();
  return OBJB_OK;
}

int objb_weights_name_at(objb_weights* w, size_t i, const char** name) {
  clear_error();
  if (!w || !name || i >= w->names.size())
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_weights_name_at", "index out of range");
  *name = w->names[i]->c_str();
  return OBJB_OK;
}

int objb_weights_info(objb_weights* w, const char* name, objb_tensor_info* info) {
  clear_error();
  const Tensor* t = find(w, name);
  if (!t) return missing(name);
  if (!info) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_weights_info", "null output");
  info->dtype = t->dtype;
  info->ndim = static_cast<int>(std::min<size_t>(t->shape.size(), 8));
  for (int i = 0; i < 8; ++i) info->shape[i] = i < info->ndim ? t->shape[i] : 0;
  info->offset = t->offset;
  info->nbytes = t->nbytes;
  info->nelem = t->nelem;
  return OBJB_OK;
}

int objb_weights_raw(objb_weights* w, const char* name, const void** data, size_t* nbytes) {
  clear_error();
  const Tensor* t = find(w, name);
  if (!t) return missing(name);
  if (!data || !nbytes) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_weights_raw", "null output");
  *data = static_cast<const uint8_t*>(w->files[t->file].base) + t->offset;
  *nbytes = t->nbytes;
  return OBJB_OK;
}

int objb_weights_get_f32(objb_weights* w, const char* name, float* out, size_t out_len) {
  clear_error();
  const Tensor* t = find(w, name);
  if (!t) return missing(name);
  const uint8_t* raw = static_cast<const uint8_t*>(w->files[t->file].base) + t->offset;
  const size_t es = dtype_size(t->dtype);
  const size_t n = t->nbytes / es;
  if (t->dtype != OBJB_DTYPE_F32 && t->dtype != OBJB_DTYPE_F16 && t->dtype != OBJB_DTYPE_BF16)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "get tensor as f32", "cannot convert dtype to f32");
  if (!out || out_len < n)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "get tensor as f32",
                     "output holds " + std::to_string(out_len) + " values, tensor has " + std::to_string(n));
  for (size_t i = 0; i < n; ++i) {
    if (t->dtype == OBJB_DTYPE_F32) {
      std::memcpy(&out[i], raw + 4 * i, 4);
    } else {
      uint16_t h;
      std::memcpy(&h, raw + 2 * i, 2);
      if (t->dtype == OBJB_DTYPE_F16) {
        out[i] = half_to_f32(h);
      } else {
        const uint32_t b = static_cast<uint32_t>(h) << 16;  // bf16_to_f32 (lib.rs:334-337)
        std::memcpy(&out[i], &b, 4);
      }
    }
  }
  return OBJB_OK;
}

int objb_weights_pin(objb_weights* w) {
  clear_error();
  if (!w) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_weights_pin", "null weights");
  const size_t page = static_cast<size_t>(sysconf(_SC_PAGESIZE));
  for (auto& f : w->files) {
    if (f.registered || f.slab || !f.size) continue;
    // The mapping itself when the platform can pin read-only file memory;
    // otherwise a pinned slab holding a copy of the file.
    const size_t span = (f.size + page - 1) / page * page;
    if (cudaHostRegister(f.map, span, cudaHostRegisterReadOnly | cudaHostRegisterPortable) == cudaSuccess) {
      f.registered = true;
      continue;
    }
    (void)cudaGetLastError();
    void* slab = nullptr;
    OBJB_CUDA(cudaHostAlloc(&slab, f.size, cudaHostAllocPortable), "allocate pinned weight slab");
    std::memcpy(slab, f.map, f.size);
    f.slab = slab;
    f.base = slab;
  }
  return OBJB_OK;
}

int objb_weights_to_device(objb_weights* w, const char* name, void* d_dst, size_t dst_bytes, objb_stream_t stream) {
  clear_error();
  const Tensor* t = find(w, name);
  if (!t) return missing(name);
  if (!d_dst || dst_bytes < t->nbytes)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "copy tensor to device", "destination smaller than the tensor");
  const void* src = static_cast<const uint8_t*>(w->files[t->file].base) + t->offset;
  OBJB_CUDA(cudaMemcpyAsync(d_dst, src, t->nbytes, cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream)),
            "copy tensor to device");
  return OBJB_OK;
}

}  // extern "C"
