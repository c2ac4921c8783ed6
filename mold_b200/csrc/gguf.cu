// GGUF file reader and model loaders (host code).
//
// Replaces the weight source of the hot path: `quantized_var_builder::VarBuilder::from_gguf`
// (flux/pipeline.rs:976; tensor names as read at flux/pipeline.rs:255-276 and
// qwen_image/quantized_transformer.rs:577-1040) and the city96 embedding patch
// (flux/pipeline.rs:254-330: fine-tune GGUFs without img_in / time_in / vector_in / guidance_in
// take those tensors from another FLUX GGUF).
//
// File layout (GGUF v2 / v3, little endian): u32 magic "GGUF", u32 version, u64 tensor count,
// u64 metadata count; metadata = (string key, u32 type, value)*; tensor infos = (string name,
// u32 n_dims, u64 dims[n_dims] (dims[0] innermost), u32 ggml type, u64 offset)*; tensor data
// starts at the first multiple of `general.alignment` (default 32) after the infos, each
// tensor at data start + offset. Strings are u64 length + bytes. The file is memory-mapped and
// each tensor's bytes are handed to the model's set_tensor (one host-to-device copy).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>
#include <map>
#include <set>
#include <string>
#include <vector>

#include "internal.h"

namespace mb {
namespace {

struct GgufTensor {
  std::string name;
  std::vector<uint64_t> dims;
  int type;
  uint64_t offset;  // from the data section start
};

struct GgufFile {
  int fd = -1;
  const uint8_t* map = nullptr;
  size_t size = 0;
  uint32_t version = 0;
  uint64_t data_start = 0;
  std::vector<GgufTensor> tensors;
  std::string error;

  ~GgufFile() {
    if (map) munmap((void*)map, size);
    if (fd >= 0) close(fd);
  }
};

// Element bytes of the metadata value types (0 = variable / not a scalar).
int scalar_bytes(uint32_t t) {
  switch (t) {
    case 0: case 1: case 7: return 1;   // u8, i8, bool
    case 2: case 3: return 2;           // u16, i16
    case 4: case 5: case 6: return 4;   // u32, i32, f32
    case 10: case 11: case 12: return 8;  // u64, i64, f64
    default: return 0;
  }
}

struct Cursor {
  const uint8_t* p;
  const uint8_t* end;
  bool ok = true;
  template <typename T>
  T get() {
    T v{};
    if (p + sizeof(T) > end) {
      ok = false;
      return v;
    }
    memcpy(&v, p, sizeof(T));
    p += sizeof(T);
    return v;
  }
  std::string str() {
    const uint64_t n = get<uint64_t>();
    if (!ok || n > (uint64_t)(end - p)) {
      ok = false;
      return {};
    }
    std::string s((const char*)p, (size_t)n);
    p += n;
    return s;
  }
  void skip_value(uint32_t type, int depth = 0) {
    if (!ok) return;
    if (type == 8) {  // string
      str();
    } else if (type == 9) {  // array: u32 element type, u64 count, elements
      const uint32_t et = get<uint32_t>();
      const uint64_t n = get<uint64_t>();
      if (!ok || depth > 4) {
        ok = false;
        return;
      }
      const int b = scalar_bytes(et);
      if (b > 0) {
        if (n > (uint64_t)(end - p) / (uint64_t)b) {
          ok = false;
          return;
        }
        p += n * (uint64_t)b;
      } else {
        for (uint64_t i = 0; i < n && ok; i++) skip_value(et, depth + 1);
      }
    } else {
      const int b = scalar_bytes(type);
      if (b == 0 || p + b > end) {
        ok = false;
        return;
      }
      p += b;
    }
  }
};

// bytes of a tensor of `type` with dims (dims[0] innermost); 0 if unsupported
uint64_t tensor_bytes(int type, const std::vector<uint64_t>& dims) {
  if (dims.empty()) return 0;
  uint64_t rows = 1;
  for (size_t i = 1; i < dims.size(); i++) rows *= dims[i];
  const int64_t rb = row_bytes_of(type, (int64_t)dims[0]);
  return rb > 0 ? rows * (uint64_t)rb : 0;
}

mb_status open_gguf(const char* path, GgufFile& f) {
  MB_CHECK(path, MB_ERR_INVALID, "path is NULL");
  f.fd = open(path, O_RDONLY);
  MB_CHECK(f.fd >= 0, MB_ERR_INVALID, std::string("cannot open GGUF file ") + path);
  struct stat st;
  MB_CHECK(fstat(f.fd, &st) == 0 && st.st_size > 24, MB_ERR_INVALID, std::string("not a GGUF file: ") + path);
  f.size = (size_t)st.st_size;
  void* m = mmap(nullptr, f.size, PROT_READ, MAP_PRIVATE, f.fd, 0);
  MB_CHECK(m != MAP_FAILED, MB_ERR_INVALID, std::string("cannot map GGUF file ") + path);
  f.map = (const uint8_t*)m;
  Cursor c{f.map, f.map + f.size};
  const uint32_t magic = c.get<uint32_t>();
  MB_CHECK(magic == 0x46554747u, MB_ERR_INVALID, std::string("bad GGUF magic in ") + path);
  f.version = c.get<uint32_t>();
  MB_CHECK(f.version == 2 || f.version == 3, MB_ERR_UNSUPPORTED,
           "GGUF version " + std::to_string(f.version) + " is not supported (2 or 3)");
  const uint64_t n_tensors = c.get<uint64_t>(), n_kv = c.get<uint64_t>();
  MB_CHECK(c.ok && n_tensors < (1u << 24) && n_kv < (1u << 24), MB_ERR_INVALID, "corrupt GGUF header");
  uint64_t alignment = 32;
  for (uint64_t i = 0; i < n_kv && c.ok; i++) {
    const std::string key = c.str();
    const uint32_t type = c.get<uint32_t>();
    if (key == "general.alignment" && type == 4) {
      alignment = c.get<uint32_t>();
    } else {
      c.skip_value(type);
    }
  }
  MB_CHECK(c.ok, MB_ERR_INVALID, "corrupt GGUF metadata");
  MB_CHECK(alignment > 0 && (alignment & (alignment - 1)) == 0, MB_ERR_INVALID, "bad general.alignment");
  f.tensors.resize((size_t)n_tensors);
  for (uint64_t i = 0; i < n_tensors && c.ok; i++) {
    GgufTensor& t = f.tensors[i];
    t.name = c.str();
    const uint32_t nd = c.get<uint32_t>();
    if (nd == 0 || nd > 4) {
      c.ok = false;
      break;
    }
    t.dims.resize(nd);
    for (uint32_t d = 0; d < nd; d++) t.dims[d] = c.get<uint64_t>();
    t.type = (int)c.get<uint32_t>();
    t.offset = c.get<uint64_t>();
  }
  MB_CHECK(c.ok, MB_ERR_INVALID, "corrupt GGUF tensor table");
  const uint64_t hdr = (uint64_t)(c.p - f.map);
  f.data_start = (hdr + alignment - 1) / alignment * alignment;
  for (const GgufTensor& t : f.tensors) {
    const uint64_t nb = tensor_bytes(t.type, t.dims);
    MB_CHECK(nb == 0 || f.data_start + t.offset + nb <= f.size, MB_ERR_INVALID,
             "GGUF tensor " + t.name + " extends past the end of the file");
  }
  return MB_OK;
}

// Loads every tensor of `f` the model knows (`want` names) through `set`; returns how many.
template <typename Set>
mb_status load_into(const GgufFile& f, const std::set<std::string>* only, Set set, int* loaded, int* skipped) {
  for (const GgufTensor& t : f.tensors) {
    if (only && !only->count(t.name)) continue;
    const uint64_t nb = tensor_bytes(t.type, t.dims);
    if (nb == 0) {
      ++*skipped;
      continue;
    }
    uint64_t rows = 1;
    for (size_t i = 1; i < t.dims.size(); i++) rows *= t.dims[i];
    const mb_status s = set(t.name.c_str(), t.type, (int64_t)rows, (int64_t)t.dims[0], f.map + f.data_start + t.offset,
                            (size_t)nb);
    if (s == MB_ERR_INVALID && std::string(mb_last_error()).find("unknown") != std::string::npos) {
      ++*skipped;  // a tensor this model does not read
      continue;
    }
    if (s != MB_OK) return s;
    ++*loaded;
  }
  return MB_OK;
}

const char* kFluxEmbeddings[] = {"img_in.weight", "img_in.bias", "time_in.in_layer.weight", "time_in.in_layer.bias",
                                 "time_in.out_layer.weight", "time_in.out_layer.bias", "vector_in.in_layer.weight",
                                 "vector_in.in_layer.bias", "vector_in.out_layer.weight", "vector_in.out_layer.bias",
                                 "guidance_in.in_layer.weight", "guidance_in.in_layer.bias",
                                 "guidance_in.out_layer.weight", "guidance_in.out_layer.bias"};

}  // namespace
}  // namespace mb

using namespace mb;

extern "C" {

mb_status mb_gguf_inspect(const char* path, char* buf, size_t buflen, int64_t* n_tensors) {
  MB_CHECK(buf && buflen > 0, MB_ERR_INVALID, "buf is NULL");
  GgufFile f;
  const mb_status s = open_gguf(path, f);
  if (s != MB_OK) return s;
  std::string out;
  for (const GgufTensor& t : f.tensors) {
    out += t.name + "\t" + std::to_string(t.type);
    for (size_t d = t.dims.size(); d-- > 0;) out += "\t" + std::to_string(t.dims[d]);  // outermost first
    out += "\n";
  }
  const size_t n = out.size() < buflen - 1 ? out.size() : buflen - 1;
  memcpy(buf, out.data(), n);
  buf[n] = 0;
  if (n_tensors) *n_tensors = (int64_t)f.tensors.size();
  return MB_OK;
}

mb_status mb_flux_load_gguf(mb_flux* m, const char* path, const char* embeddings_path, int* n_loaded) {
  MB_CHECK(m && path, MB_ERR_INVALID, "NULL argument");
  int loaded = 0, skipped = 0;
  {
    GgufFile f;
    const mb_status s = open_gguf(path, f);
    if (s != MB_OK) return s;
    auto set = [&](const char* n, int t, int64_t r, int64_t c, const void* d, size_t nb) {
      return mb_flux_set_tensor(m, n, t, r, c, d, nb, 0);
    };
    const mb_status ls = load_into(f, nullptr, set, &loaded, &skipped);
    if (ls != MB_OK) return ls;
  }
  if (embeddings_path) {
    // city96 patch: embedding tensors the main file lacks come from a complete FLUX GGUF
    std::vector<char> miss(1 << 20);
    mb_flux_missing(m, miss.data(), miss.size());
    std::set<std::string> want;
    for (const char* e : kFluxEmbeddings)
      if (strstr(miss.data(), (std::string(e) + "\n").c_str())) want.insert(e);
    if (!want.empty()) {
      GgufFile f;
      const mb_status s = open_gguf(embeddings_path, f);
      if (s != MB_OK) return s;
      auto set = [&](const char* n, int t, int64_t r, int64_t c, const void* d, size_t nb) {
        return mb_flux_set_tensor(m, n, t, r, c, d, nb, 0);
      };
      const mb_status ls = load_into(f, &want, set, &loaded, &skipped);
      if (ls != MB_OK) return ls;
    }
  }
  if (n_loaded) *n_loaded = loaded;
  return MB_OK;
}

mb_status mb_qwen_load_gguf(mb_qwen* m, const char* path, int* n_loaded) {
  MB_CHECK(m && path, MB_ERR_INVALID, "NULL argument");
  GgufFile f;
  const mb_status s = open_gguf(path, f);
  if (s != MB_OK) return s;
  int loaded = 0, skipped = 0;
  auto set = [&](const char* n, int t, int64_t r, int64_t c, const void* d, size_t nb) {
    return mb_qwen_set_tensor(m, n, t, r, c, d, nb, 0);
  };
  const mb_status ls = load_into(f, nullptr, set, &loaded, &skipped);
  if (ls != MB_OK) return ls;
  if (n_loaded) *n_loaded = loaded;
  return MB_OK;
}

}  // extern "C"
