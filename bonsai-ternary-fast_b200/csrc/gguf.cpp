// GGUF (v2/v3) tensor access and the load path for PTQ1_0 weights: file ->
// mmap -> pinned staging -> GPU repack into the panel layout. The reference's
// load path is bd::Gguf (ref/bonsai-decoder/src/gguf.cpp) + GpuDecoder::upload_mat
// (src/cuda/gpu_decoder.cu:284-300); this reader is written from the public GGUF
// layout:
//   u32 magic "GGUF", u32 version, u64 tensor_count, u64 kv_count,
//   kv_count x { string key, u32 value type, value },
//   tensor_count x { string name, u32 n_dims, u64 ne[n_dims], u32 type, u64 offset },
//   data section at the header end rounded up to general.alignment (default 32);
//   strings are u64 length + bytes; arrays are u32 element type + u64 count + elements.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "btf_b200.h"
#include "gguf_meta.h"

namespace btf {
int fail(int status, const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);
}  // namespace btf

namespace {

constexpr uint32_t kGgufMagic = 0x46554747u;  // "GGUF"
constexpr uint32_t kTypePtq1_0 = 143;

struct Tensor {
  std::string name;
  int n_dims = 0;
  int64_t ne[4] = {1, 1, 1, 1};
  uint32_t type = 0;
  uint64_t offset = 0;
  uint64_t bytes = 0;
};

struct File {
  std::map<std::string, btf::gguf::Value> kv;
  int fd = -1;
  const uint8_t* map = nullptr;
  size_t size = 0;
  uint32_t version = 0;
  uint64_t alignment = 32;
  uint64_t data_start = 0;
  std::vector<Tensor> tensors;
  ~File() {
    if (map) munmap(const_cast<uint8_t*>(map), size);
    if (fd >= 0) close(fd);
  }
};

// Bounds-checked little-endian reader over the mapped header.
struct Reader {
  const uint8_t* p;
  size_t n, pos = 0;
  bool ok = true;
  bool need(size_t k) {
    if (!ok || k > n - pos) ok = false;
    return ok;
  }
  template <class T>
  T get() {
    T v{};
    if (need(sizeof(T))) {
      std::memcpy(&v, p + pos, sizeof(T));
      pos += sizeof(T);
    }
    return v;
  }
  std::string str() {
    const uint64_t len = get<uint64_t>();
    if (!ok || !need(len)) return {};
    std::string s(reinterpret_cast<const char*>(p + pos), len);
    pos += len;
    return s;
  }
  void skip(uint64_t k) {
    if (need(k)) pos += k;
  }
};

// Bytes of one scalar of a metadata value type (0 for strings and arrays).
size_t scalar_bytes(uint32_t t) {
  switch (t) {
    case 0: case 1: case 7: return 1;   // u8, i8, bool
    case 2: case 3: return 2;           // u16, i16
    case 4: case 5: case 6: return 4;   // u32, i32, f32
    case 10: case 11: case 12: return 8;  // u64, i64, f64
    default: return 0;
  }
}

// Reads one scalar of metadata type t (u8, i8, u16, i16, u32, i32, f32, bool,
// u64, i64, f64) into the integer or the float slot of v.
void read_scalar(Reader& r, uint32_t t, int64_t& i, double& f) {
  switch (t) {
    case 0: i = r.get<uint8_t>(); break;
    case 1: i = r.get<int8_t>(); break;
    case 2: i = r.get<uint16_t>(); break;
    case 3: i = r.get<int16_t>(); break;
    case 4: i = r.get<uint32_t>(); break;
    case 5: i = r.get<int32_t>(); break;
    case 6: f = r.get<float>(); break;
    case 7: i = r.get<uint8_t>() != 0; break;
    case 10: i = (int64_t)r.get<uint64_t>(); break;
    case 11: i = r.get<int64_t>(); break;
    case 12: f = r.get<double>(); break;
    default: r.ok = false;
  }
  if (t != 6 && t != 12) f = (double)i;
  else i = (f > -9.2e18 && f < 9.2e18) ? (int64_t)f : 0;  // NaN or out of range: no integer view
}

// Reads one metadata value (scalars, strings and one level of arrays).
btf::gguf::Value read_value(Reader& r, uint32_t type) {
  btf::gguf::Value v;
  v.type = type;
  if (type == 8) {  // string
    v.s = r.str();
  } else if (type == 9) {  // array
    const uint32_t et = r.get<uint32_t>();
    const uint64_t count = r.get<uint64_t>();
    v.elem_type = et;
    if (et == 8) {
      if (count > r.n - r.pos) r.ok = false;  // every string takes at least its 8-byte length
      for (uint64_t i = 0; i < count && r.ok; ++i) v.as.push_back(r.str());
    } else if (const size_t eb = scalar_bytes(et)) {
      if (count > (r.n - r.pos) / eb) {
        r.ok = false;
      } else {
        v.ai.resize(count);
        v.af.resize(count);
        for (uint64_t i = 0; i < count && r.ok; ++i) read_scalar(r, et, v.ai[i], v.af[i]);
      }
    } else {
      r.ok = false;  // nested arrays are not part of the format this reader accepts
    }
  } else {
    read_scalar(r, type, v.i, v.f);
  }
  return v;
}

// Data bytes of a tensor for the types this library reads; 0 if unknown.
uint64_t tensor_bytes(uint32_t type, int64_t n_elem, int64_t ne0) {
  switch (type) {
    case 0: return (uint64_t)n_elem * 4;                                   // f32
    case 1: case 30: return (uint64_t)n_elem * 2;                          // f16, bf16
    case 8: return ne0 % 32 ? 0 : (uint64_t)(n_elem / 32) * 34;           // q8_0
    case kTypePtq1_0: return ne0 % 128 ? 0 : (uint64_t)(n_elem / 128) * 28;
    default: return 0;
  }
}

int parse(File& f) {
  Reader r{f.map, f.size};
  if (r.get<uint32_t>() != kGgufMagic) return btf::fail(BTF_ERR_ARG, "btf_gguf_open: not a GGUF file");
  f.version = r.get<uint32_t>();
  if (f.version < 2 || f.version > 3) return btf::fail(BTF_ERR_UNSUPPORTED, "btf_gguf_open: GGUF version %u", f.version);
  const uint64_t n_tensors = r.get<uint64_t>(), n_kv = r.get<uint64_t>();
  // every key/value takes at least 12 bytes (empty key, type), every tensor entry at least 32
  // (empty name, n_dims, one ne, type, offset): counts beyond what the file holds are malformed
  if (!r.ok || n_tensors > (1u << 24) || n_kv > (1u << 24) || n_kv > (r.n - r.pos) / 12 ||
      n_tensors > (r.n - r.pos) / 32)
    return btf::fail(BTF_ERR_ARG, "btf_gguf_open: bad header");
  for (uint64_t i = 0; i < n_kv && r.ok; ++i) {
    const std::string key = r.str();
    const uint32_t type = r.get<uint32_t>();
    btf::gguf::Value v = read_value(r, type);
    if (r.ok && key == "general.alignment" && type != 8 && type != 9 && v.i > 0) f.alignment = (uint64_t)v.i;
    if (r.ok) f.kv[key] = std::move(v);
  }
  f.tensors.resize(n_tensors);
  for (uint64_t i = 0; i < n_tensors && r.ok; ++i) {
    Tensor& t = f.tensors[i];
    t.name = r.str();
    const uint32_t nd = r.get<uint32_t>();
    if (nd < 1 || nd > 4) {
      r.ok = false;
      break;
    }
    t.n_dims = (int)nd;
    int64_t n_elem = 1;
    for (uint32_t d = 0; d < nd; ++d) {
      t.ne[d] = (int64_t)r.get<uint64_t>();
      if (t.ne[d] <= 0 || t.ne[d] > (int64_t(1) << 40) || n_elem > (int64_t(1) << 50) / t.ne[d]) r.ok = false;
      else n_elem *= t.ne[d];
    }
    t.type = r.get<uint32_t>();
    t.offset = r.get<uint64_t>();
    t.bytes = tensor_bytes(t.type, n_elem, t.ne[0]);
  }
  if (!r.ok) return btf::fail(BTF_ERR_ARG, "btf_gguf_open: truncated or malformed header");
  if (f.alignment == 0 || (f.alignment & (f.alignment - 1)) || f.alignment > (uint64_t(1) << 30))
    return btf::fail(BTF_ERR_ARG, "btf_gguf_open: bad alignment");
  f.data_start = (r.pos + f.alignment - 1) / f.alignment * f.alignment;
  for (const Tensor& t : f.tensors)
    if (f.data_start > f.size || t.offset > f.size - f.data_start || t.bytes > f.size - f.data_start - t.offset)
      return btf::fail(BTF_ERR_ARG, "btf_gguf_open: tensor %s lies beyond the file", t.name.c_str());
  return BTF_OK;
}

}  // namespace

namespace btf {
namespace gguf {
const Value* meta(const void* handle, const std::string& key) {
  if (!handle) return nullptr;
  const File& f = *static_cast<const File*>(handle);
  const auto it = f.kv.find(key);
  return it == f.kv.end() ? nullptr : &it->second;
}
}  // namespace gguf
}  // namespace btf

extern "C" {

int btf_gguf_open(const char* path, void** handle) {
  if (!path || !handle) return btf::fail(BTF_ERR_ARG, "btf_gguf_open: null argument");
  *handle = nullptr;
  File* f = new File;
  f->fd = open(path, O_RDONLY);
  struct stat st;
  if (f->fd < 0 || fstat(f->fd, &st) != 0 || st.st_size < 24) {
    delete f;
    return btf::fail(BTF_ERR_ARG, "btf_gguf_open: cannot open %s", path);
  }
  f->size = (size_t)st.st_size;
  void* m = mmap(nullptr, f->size, PROT_READ, MAP_PRIVATE, f->fd, 0);
  if (m == MAP_FAILED) {
    delete f;
    return btf::fail(BTF_ERR_ARG, "btf_gguf_open: mmap failed for %s", path);
  }
  f->map = static_cast<const uint8_t*>(m);
  if (int rc = parse(*f)) {
    delete f;
    return rc;
  }
  *handle = f;
  return BTF_OK;
}

int btf_gguf_close(void* handle) {
  delete static_cast<File*>(handle);
  return BTF_OK;
}

int64_t btf_gguf_tensor_count(const void* handle) {
  return handle ? (int64_t) static_cast<const File*>(handle)->tensors.size() : -1;
}

int64_t btf_gguf_find(const void* handle, const char* name) {
  if (!handle || !name) return -1;
  const File* f = static_cast<const File*>(handle);
  for (size_t i = 0; i < f->tensors.size(); ++i)
    if (f->tensors[i].name == name) return (int64_t)i;
  return -1;
}

int btf_gguf_tensor(const void* handle, int64_t index, btf_gguf_tensor_info* out) {
  const File* f = static_cast<const File*>(handle);
  if (!f || !out || index < 0 || index >= (int64_t)f->tensors.size())
    return btf::fail(BTF_ERR_ARG, "btf_gguf_tensor: bad handle or index");
  const Tensor& t = f->tensors[(size_t)index];
  out->name = t.name.c_str();
  out->n_dims = t.n_dims;
  for (int d = 0; d < 4; ++d) out->ne[d] = t.ne[d];
  out->type = t.type;
  out->data = f->map + f->data_start + t.offset;
  out->bytes = t.bytes;
  return BTF_OK;
}

int btf_gguf_load_panels(const void* handle, int64_t index, void* panels, int64_t staging_bytes, void* stream) {
  const File* f = static_cast<const File*>(handle);
  if (!f || index < 0 || index >= (int64_t)f->tensors.size())
    return btf::fail(BTF_ERR_ARG, "btf_gguf_load_panels: bad handle or index");
  return btf_gguf_load_panels_rows(handle, index, 0, f->tensors[(size_t)index].ne[1], panels, staging_bytes, stream);
}

int btf_gguf_load_panels_rows(const void* handle, int64_t index, int64_t row0, int64_t rows, void* panels,
                              int64_t staging_bytes, void* stream) {
  const File* f = static_cast<const File*>(handle);
  if (!f || !panels || index < 0 || index >= (int64_t)f->tensors.size())
    return btf::fail(BTF_ERR_ARG, "btf_gguf_load_panels: bad handle, index or panel buffer");
  const Tensor& t = f->tensors[(size_t)index];
  if (t.type != kTypePtq1_0 || t.n_dims != 2)
    return btf::fail(BTF_ERR_UNSUPPORTED, "btf_gguf_load_panels: %s is not a 2-D PTQ1_0 tensor", t.name.c_str());
  const int64_t K = t.ne[0], NT = t.ne[1];
  if (K % 128) return btf::fail(BTF_ERR_ARG, "btf_gguf_load_panels: %s width %lld is not a multiple of 128", t.name.c_str(), (long long)K);
  if (row0 < 0 || row0 % 8 || rows <= 0 || row0 + rows > NT)
    return btf::fail(BTF_ERR_ARG, "btf_gguf_load_panels: rows [%lld, %lld) of %lld (row0 a multiple of 8)",
                     (long long)row0, (long long)(row0 + rows), (long long)NT);
  const int64_t N = rows;  // the rows loaded, written from panel row group 0
  const int64_t row_bytes = K / 128 * 28, S = (K + 1023) / 1024;
  const int64_t rows_per = btf::gguf::staging_rows(K, N, staging_bytes);
  const size_t stage = (size_t)(rows_per * row_bytes);
  const uint8_t* src = f->map + f->data_start + t.offset + row0 * row_bytes;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // two pinned staging buffers, read by the repack kernel over the bus (mapped)
  void* buf[2] = {nullptr, nullptr};
  cudaEvent_t ev[2] = {nullptr, nullptr};
  int rc = BTF_OK;
  cudaError_t e = cudaSuccess;
  for (int i = 0; i < 2 && e == cudaSuccess; ++i) {
    e = cudaHostAlloc(&buf[i], stage, cudaHostAllocMapped);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming);
  }
  if (e != cudaSuccess) rc = btf::cuda_fail(e, "btf_gguf_load_panels: staging");
  int slot = 0;
  for (int64_t r0 = 0; r0 < N && rc == BTF_OK; r0 += rows_per, slot ^= 1) {
    const int64_t nr = std::min(rows_per, N - r0);
    if ((e = cudaEventSynchronize(ev[slot])) != cudaSuccess) {  // this buffer's previous repack is done
      rc = btf::cuda_fail(e, "btf_gguf_load_panels: staging wait");
      break;
    }
    std::memcpy(buf[slot], src + r0 * row_bytes, (size_t)(nr * row_bytes));
    uint8_t* dst = static_cast<uint8_t*>(panels) + (r0 / 8) * S * BTF_PANEL_BYTES;
    if ((rc = btf_repack_panels(buf[slot], nr, K, dst, stream)) != BTF_OK) break;
    if ((e = cudaEventRecord(ev[slot], st)) != cudaSuccess) rc = btf::cuda_fail(e, "btf_gguf_load_panels: record");
  }
  if ((e = cudaStreamSynchronize(st)) != cudaSuccess && rc == BTF_OK) rc = btf::cuda_fail(e, "btf_gguf_load_panels");
  for (int i = 0; i < 2; ++i) {
    if (ev[i]) cudaEventDestroy(ev[i]);
    if (buf[i]) cudaFreeHost(buf[i]);
  }
  return rc;
}

}  // extern "C"
