// st_loader.cu — weights straight from a safetensors checkpoint to device int8.
//
// The reference engine mmaps its checkpoints read-only (safetensors.c,
// iro_st_load), quantises the DiT's 96 projection matrices on the host at
// init (dit.c:235-259 calling ops.c:259-293), then drops the fp32 pages it no
// longer needs (generate.c:543-556 through iro_st_drop_prefix,
// safetensors.c:525-552).  Here the fp32 bytes go from the mapping to the
// device and are quantised there by the same kernel as
// iro_int8_dev_weight_quantize, so the codes, scales and column sums are the
// host quantiser's bit for bit; page dropping keeps the reference's rule.
//
// Format (safetensors): an 8-byte little-endian header length, a JSON object
// {"name": {"dtype": "F32", "shape": [...], "data_offsets": [begin, end]},
// "__metadata__": {...}}, then the data; offsets are relative to the data.
#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <string>
#include <vector>

#include "quantize.cuh"

// The reference engine links its own iro_st_* loader (safetensors.c); these
// entry points are iro_st_file_* so both can live in one binary.

struct IroStFile {
  int fd = -1;
  uint8_t* map = nullptr;
  size_t size = 0;
  size_t data_start = 0;
  struct Entry {
    std::string name;
    int dtype = 0;
    int ndims = 0;
    uint64_t shape[8] = {0};
    uint64_t begin = 0, end = 0;
  };
  std::vector<Entry> tensors;
};

namespace {

// dtype codes in the order of irodori.h's IroDType.
int dtype_code(const std::string& s) {
  static const char* const names[] = {"F32", "F16", "BF16", "I64", "I32", "I16", "I8", "U8", "BOOL"};
  for (int i = 0; i < 9; i++)
    if (s == names[i]) return i;
  return 9;  // unknown
}

int dtype_size(int code) {
  static const int sizes[] = {4, 2, 2, 8, 4, 2, 1, 1, 1};
  return code >= 0 && code < 9 ? sizes[code] : 0;
}

// A small recursive-descent reader for the header JSON.
struct Json {
  const char* p;
  const char* e;
  bool ok = true;

  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) p++;
  }
  bool eat(char c) {
    ws();
    if (p < e && *p == c) {
      p++;
      return true;
    }
    return false;
  }
  bool str(std::string& out) {
    ws();
    if (p >= e || *p != '"') return ok = false;
    p++;
    out.clear();
    while (p < e && *p != '"') {
      if (*p == '\\') {
        if (++p >= e) return ok = false;
        const char c = *p;
        if (c == 'u') {  // keep the escape verbatim: names here are ASCII
          out += "\\u";
          p++;
          continue;
        }
        out += c == 'n' ? '\n' : c == 't' ? '\t' : c == 'r' ? '\r' : c == 'b' ? '\b' : c == 'f' ? '\f' : c;
        p++;
        continue;
      }
      out += *p++;
    }
    if (p >= e) return ok = false;
    p++;
    return true;
  }
  bool u64(uint64_t& v) {
    ws();
    if (p >= e || *p < '0' || *p > '9') return ok = false;
    v = 0;
    while (p < e && *p >= '0' && *p <= '9') {
      const uint64_t d = (uint64_t)(*p - '0');
      if (v > (UINT64_MAX - d) / 10) return ok = false;
      v = v * 10 + d;
      p++;
    }
    return true;
  }
  // Skip any value (metadata may hold strings, numbers, nested objects).
  bool skip() {
    ws();
    if (p >= e) return ok = false;
    if (*p == '"') {
      std::string t;
      return str(t);
    }
    if (*p == '{' || *p == '[') {
      const char close = *p == '{' ? '}' : ']';
      p++;
      if (eat(close)) return true;
      do {
        if (close == '}') {
          std::string k;
          if (!str(k) || !eat(':')) return ok = false;
        }
        if (!skip()) return false;
      } while (eat(','));
      return eat(close) ? true : (ok = false);
    }
    while (p < e && *p != ',' && *p != '}' && *p != ']') p++;  // number, true, false, null
    return true;
  }
};

bool parse_header(IroStFile* f, const char* js, size_t n) {
  Json j{js, js + n};
  if (!j.eat('{')) return false;
  if (j.eat('}')) return true;
  do {
    std::string key;
    if (!j.str(key) || !j.eat(':')) return false;
    if (key == "__metadata__") {
      if (!j.skip()) return false;
      continue;
    }
    IroStFile::Entry t;
    t.name = key;
    bool have_dtype = false, have_shape = false, have_off = false;
    if (!j.eat('{')) return false;
    if (!j.eat('}')) {
      do {
        std::string field;
        if (!j.str(field) || !j.eat(':')) return false;
        if (field == "dtype") {
          std::string d;
          if (!j.str(d)) return false;
          t.dtype = dtype_code(d);
          have_dtype = true;
        } else if (field == "shape") {
          if (!j.eat('[')) return false;
          if (!j.eat(']')) {
            do {
              uint64_t v;
              if (t.ndims >= 8 || !j.u64(v)) return false;
              t.shape[t.ndims++] = v;
            } while (j.eat(','));
            if (!j.eat(']')) return false;
          }
          have_shape = true;
        } else if (field == "data_offsets") {
          if (!j.eat('[') || !j.u64(t.begin) || !j.eat(',') || !j.u64(t.end) || !j.eat(']'))
            return false;
          have_off = true;
        } else if (!j.skip()) {
          return false;
        }
      } while (j.eat(','));
      if (!j.eat('}')) return false;
    }
    if (!have_dtype || !have_shape || !have_off) return false;
    f->tensors.push_back(t);
  } while (j.eat(','));
  return j.eat('}') && j.ok;
}

const IroStFile::Entry* find(const IroStFile* f, const char* name) {
  if (!f || !name) return nullptr;
  for (const auto& t : f->tensors)
    if (t.name == name) return &t;
  return nullptr;
}

}  // namespace

using namespace iro;

extern "C" {

void iro_st_file_close(IroStFile* f) {
  if (!f) return;
  if (f->map) munmap(f->map, f->size);
  if (f->fd >= 0) close(f->fd);
  delete f;
}

int iro_st_file_open(IroStFile** out, const char* path) {
  if (!out || !path) return IRO_ERR_INVALID;
  *out = nullptr;
  IroStFile* f = new IroStFile();
  f->fd = open(path, O_RDONLY);
  struct stat sb;
  if (f->fd < 0 || fstat(f->fd, &sb) != 0 || sb.st_size < 8) {
    iro_st_file_close(f);
    return IRO_ERR_INVALID;
  }
  f->size = (size_t)sb.st_size;
  void* m = mmap(nullptr, f->size, PROT_READ, MAP_PRIVATE, f->fd, 0);
  if (m == MAP_FAILED) {
    iro_st_file_close(f);
    return IRO_ERR_INVALID;
  }
  f->map = static_cast<uint8_t*>(m);
  uint64_t hlen = 0;
  for (int i = 7; i >= 0; i--) hlen = (hlen << 8) | f->map[i];
  if (hlen > f->size - 8 || !parse_header(f, reinterpret_cast<const char*>(f->map) + 8, hlen)) {
    iro_st_file_close(f);
    return IRO_ERR_INVALID;
  }
  f->data_start = 8 + (size_t)hlen;
  // Every tensor's bytes must lie inside the file and match its geometry.
  for (const auto& t : f->tensors) {
    uint64_t numel = 1;
    for (int d = 0; d < t.ndims; d++) numel *= t.shape[d];
    const int es = dtype_size(t.dtype);
    if (t.end < t.begin || t.end > f->size - f->data_start ||
        (es && t.end - t.begin != numel * (uint64_t)es)) {
      iro_st_file_close(f);
      return IRO_ERR_INVALID;
    }
  }
  *out = f;
  return IRO_OK;
}

int iro_st_file_count(const IroStFile* f) { return f ? (int)f->tensors.size() : IRO_ERR_INVALID; }

const char* iro_st_file_name(const IroStFile* f, int i) {
  return f && i >= 0 && i < (int)f->tensors.size() ? f->tensors[i].name.c_str() : nullptr;
}

int iro_st_file_tensor(const IroStFile* f, const char* name, int* dtype, int* ndims, uint64_t* shape,
                  uint64_t* nbytes) {
  const IroStFile::Entry* t = find(f, name);
  if (!t) return IRO_ERR_INVALID;
  if (dtype) *dtype = t->dtype;
  if (ndims) *ndims = t->ndims;
  if (shape)
    for (int d = 0; d < t->ndims; d++) shape[d] = t->shape[d];
  if (nbytes) *nbytes = t->end - t->begin;
  return IRO_OK;
}

const void* iro_st_file_data(const IroStFile* f, const char* name) {
  const IroStFile::Entry* t = find(f, name);
  return t ? f->map + f->data_start + t->begin : nullptr;
}

uint64_t iro_st_file_drop_prefix(const IroStFile* f, const char* prefix) {
  // safetensors.c:525-552: the page-aligned span covering every tensor with
  // this name prefix, clipped to the mapping, released with MADV_DONTNEED.
  if (!f || !f->map || !prefix || !*prefix) return 0;
  const size_t plen = strlen(prefix);
  uintptr_t first = UINTPTR_MAX, last = 0;
  for (const auto& t : f->tensors) {
    if (t.name.compare(0, plen, prefix) != 0) continue;
    const uintptr_t b = (uintptr_t)(f->map + f->data_start + t.begin);
    const uintptr_t en = b + (uintptr_t)(t.end - t.begin);
    if (b < first) first = b;
    if (en > last) last = en;
  }
  if (first == UINTPTR_MAX || last <= first) return 0;
  const long ps = sysconf(_SC_PAGESIZE);
  if (ps <= 0) return 0;
  const uintptr_t page = (uintptr_t)ps;
  const uintptr_t mb = (uintptr_t)f->map, me = mb + f->size;
  uintptr_t ab = first & ~(page - 1u);
  uintptr_t ae = (last + page - 1u) & ~(page - 1u);
  if (ab < mb) ab = mb;
  if (ae > me) ae = me;
  if (ae <= ab || madvise(reinterpret_cast<void*>(ab), ae - ab, MADV_DONTNEED) != 0) return 0;
  return (uint64_t)(ae - ab);
}

int iro_int8_dev_weight_from_st(IroInt8DevWeight* dst, const IroStFile* f, const char* name,
                                int transposed, const char* bias_name) {
  if (!dst) return IRO_ERR_INVALID;
  memset(dst, 0, sizeof(*dst));
  const IroStFile::Entry* t = find(f, name);
  if (!t || t->dtype != 0 || t->ndims != 2 || t->shape[0] == 0 || t->shape[1] == 0 ||
      t->shape[0] > 0x7fffffffULL || t->shape[1] > 0x7fffffffULL)
    return IRO_ERR_INVALID;
  // [N, K] row-major, or [K, N] for the transposed form (ops.c:295-306).
  const int N = (int)(transposed ? t->shape[1] : t->shape[0]);
  const int K = (int)(transposed ? t->shape[0] : t->shape[1]);
  const IroStFile::Entry* b = nullptr;
  if (bias_name) {
    b = find(f, bias_name);
    if (!b || b->dtype != 0 || b->ndims != 1 || b->shape[0] != (uint64_t)N) return IRO_ERR_INVALID;
  }
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  const size_t nk = (size_t)N * K;
  const size_t wbytes = (nk * sizeof(float) + 255) / 256 * 256;
  float* base = static_cast<float*>(
      arena_get(c, wbytes * (transposed ? 2 : 1) + sizeof(float) * (size_t)N, &st));
  if (!base) return st;
  float* w_dev = base;
  float* src = w_dev;
  float* bias_dev = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(base) +
                                             wbytes * (transposed ? 2 : 1));
  cudaStream_t s = c->stream;
  cudaError_t e = cudaMemcpyAsync(w_dev, f->map + f->data_start + t->begin, nk * sizeof(float),
                                  cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess && b)
    e = cudaMemcpyAsync(bias_dev, f->map + f->data_start + b->begin, sizeof(float) * (size_t)N,
                        cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return map_cuda(e);
  }
  if (transposed) {
    src = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(base) + wbytes);
    st = transpose_f32_launch(w_dev, K, N, src, s);
    if (st) return st;
  }
  // Same kernel and numerics as iro_int8_dev_weight_quantize; synchronises
  // the stream before returning (the scratch is reused by the next call).
  return iro_int8_dev_weight_quantize(dst, src, N, K, b ? bias_dev : nullptr, nullptr);
}

}  // extern "C"
