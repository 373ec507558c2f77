// gguf.cpp — zero-copy GGUF reader (replaces GGUFModel, src/model/gguf.rs:125-195).
//
// The file is memory-mapped read-only; tensor data is returned as pointers into the
// mapping. Differences from the reference, all deliberate:
//  * UINT8 / INT8 metadata values are read as 1 byte (the GGUF format). The reference
//    reads 4 bytes for them (gguf.rs:100-101), which desynchronises the parser on any
//    file that has such a key.
//  * Every read is bounds-checked; a truncated or malformed file returns RRR_ERR_IO
//    instead of panicking, and unknown value types are an error (the reference skips one
//    byte, gguf.rs:115).
//  * Tensor byte sizes follow the same per-type table (gguf.rs:173-195).
//  * Uploads go through reusable pinned staging (two buffers, host copies from the mapping
//    by several threads, cudaMemcpyAsync on a copy stream, each DMA overlapping the host
//    copy of the next chunk) instead of per-tensor synchronous copies from pageable
//    memory; rrr_gguf_load places many tensors in one device allocation.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <map>
#include <string>
#include <thread>
#include <vector>

#include "capi_internal.h"

using namespace rrr;

namespace {

struct Meta {
  uint32_t type = 0;  // GGUF value type
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0.0;
  bool is_int = false, is_uint = false, is_float = false, is_str = false, is_array = false;
  std::string s;
};

struct Tensor {
  std::string name;
  int n_dims = 0;
  uint64_t shape[4] = {1, 1, 1, 1};
  uint32_t type = 0;
  uint64_t offset = 0;
  uint64_t n_bytes = 0;
};

struct Reader {
  const uint8_t* p;
  size_t n, pos = 0;
  bool ok = true;
  bool take(void* dst, size_t k) {
    if (!ok || k > n - pos) return ok = false;
    std::memcpy(dst, p + pos, k);
    pos += k;
    return true;
  }
  uint8_t u8() { uint8_t v = 0; take(&v, 1); return v; }
  uint16_t u16() { uint16_t v = 0; take(&v, 2); return v; }
  uint32_t u32() { uint32_t v = 0; take(&v, 4); return v; }
  uint64_t u64() { uint64_t v = 0; take(&v, 8); return v; }
  std::string str() {
    const uint64_t len = u64();
    if (!ok || len > n - pos) { ok = false; return std::string(); }
    std::string s(reinterpret_cast<const char*>(p + pos), (size_t)len);
    pos += (size_t)len;
    return s;
  }
};

// Reads one value of GGUF type `t` (gguf.rs:93-117 with the corrections above).
bool read_value(Reader& r, uint32_t t, Meta& m, int depth) {
  m.type = t;
  switch (t) {
    case 0: m.u = r.u8(); m.is_uint = true; break;
    case 1: m.i = (int8_t)r.u8(); m.is_int = true; break;
    case 2: m.u = r.u16(); m.is_uint = true; break;
    case 3: m.i = (int16_t)r.u16(); m.is_int = true; break;
    case 4: m.u = r.u32(); m.is_uint = true; break;
    case 5: m.i = (int32_t)r.u32(); m.is_int = true; break;
    case 6: { uint32_t b = r.u32(); float f; std::memcpy(&f, &b, 4); m.f = f; m.is_float = true; break; }
    case 7: m.u = r.u8() != 0; m.is_uint = true; break;
    case 8: m.s = r.str(); m.is_str = true; break;
    case 9: {
      if (depth > 4) return false;
      const uint32_t at = r.u32();
      const uint64_t len = r.u64();
      if (!r.ok || len > r.n) return false;
      m.is_array = true;
      m.u = len;
      for (uint64_t k = 0; k < len && r.ok; ++k) {
        Meta e;
        if (!read_value(r, at, e, depth + 1)) return false;
      }
      break;
    }
    case 10: m.u = r.u64(); m.is_uint = true; break;
    case 11: m.i = (int64_t)r.u64(); m.is_int = true; break;
    case 12: { uint64_t b = r.u64(); double d; std::memcpy(&d, &b, 8); m.f = d; m.is_float = true; break; }
    default: return false;
  }
  return r.ok;
}

// Bytes of a tensor of `n` elements (gguf.rs:177-190); 0 for an unknown type.
uint64_t type_bytes(uint32_t t, uint64_t n) {
  switch (t) {
    case 0: return n * 4;
    case 1: return n * 2;
    case 2: return (n / 32) * 18;
    case 3: return (n / 32) * 20;
    case 6: return (n / 32) * 22;
    case 7: return (n / 32) * 24;
    case 8: return (n / 32) * 34;
    case 9: return (n / 32) * 36;
    case 12: return (n / 256) * 144;
    case 13: return (n / 256) * 176;
    case 14: return (n / 256) * 210;
    default: return 0;
  }
}

}  // namespace

// Pinned staging of the uploads: two host buffers, a copy stream and an event per buffer.
struct Staging {
  static constexpr size_t kChunk = 32u << 20;  // bytes per staged copy
  static constexpr int kThreads = 8;           // host threads copying out of the mapping
  void* pinned[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  cudaStream_t stream = nullptr;
  int device = -1;
};

struct rrr_gguf {
  Staging staging;
  int fd = -1;
  const uint8_t* map = nullptr;
  size_t size = 0;
  uint32_t version = 0;
  uint64_t data_offset = 0;
  std::map<std::string, Meta> meta;
  std::vector<Tensor> tensors;
  std::map<std::string, size_t> by_name;
};

static int fill_tensor(rrr_gguf* g, size_t i, rrr_gguf_tensor* out) {
  const Tensor& t = g->tensors[i];
  out->name = t.name.c_str();
  out->n_dims = t.n_dims;
  for (int k = 0; k < 4; ++k) out->shape[k] = t.shape[k];
  out->type = t.type;
  out->offset = t.offset;
  out->n_bytes = t.n_bytes;
  out->data = g->map + g->data_offset + t.offset;
  return RRR_OK;
}

extern "C" {

int rrr_gguf_open(const char* path, rrr_gguf** out) {
  if (!path || !out) return set_error(nullptr, RRR_ERR_INVALID_ARG, "rrr_gguf_open: null argument");
  *out = nullptr;
  const int fd = ::open(path, O_RDONLY);
  if (fd < 0) return set_error(nullptr, RRR_ERR_IO, "rrr_gguf_open: cannot open %s", path);
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 24) {
    ::close(fd);
    return set_error(nullptr, RRR_ERR_IO, "rrr_gguf_open: %s is too small to be GGUF", path);
  }
  void* m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  if (m == MAP_FAILED) {
    ::close(fd);
    return set_error(nullptr, RRR_ERR_IO, "rrr_gguf_open: mmap failed for %s", path);
  }
  rrr_gguf* g = new rrr_gguf();
  g->fd = fd;
  g->map = static_cast<const uint8_t*>(m);
  g->size = (size_t)st.st_size;
  Reader r{g->map, g->size};
  auto fail = [&](const char* why) {
    rrr_gguf_close(g);
    return set_error(nullptr, RRR_ERR_IO, "rrr_gguf_open: %s (%s)", why, path);
  };
  if (r.u32() != 0x46554747u) return fail("bad magic (not GGUF)");
  g->version = r.u32();
  if (g->version < 2) return fail("GGUF version 1 is not supported");
  const uint64_t n_tensors = r.u64(), n_kv = r.u64();
  if (!r.ok || n_tensors > g->size || n_kv > g->size) return fail("truncated header");
  for (uint64_t k = 0; k < n_kv; ++k) {
    std::string key = r.str();
    const uint32_t t = r.u32();
    Meta mv;
    if (!r.ok || !read_value(r, t, mv, 0)) return fail("malformed metadata");
    g->meta[key] = mv;
  }
  for (uint64_t k = 0; k < n_tensors; ++k) {
    Tensor t;
    t.name = r.str();
    const uint32_t nd = r.u32();
    if (!r.ok || nd > 4) return fail("malformed tensor info");
    t.n_dims = (int)nd;
    uint64_t ne = 1;
    for (uint32_t d = 0; d < nd; ++d) {
      t.shape[d] = r.u64();
      ne *= t.shape[d];
    }
    t.type = r.u32();
    t.offset = r.u64();
    if (!r.ok) return fail("truncated tensor info");
    t.n_bytes = type_bytes(t.type, ne);
    if (t.n_bytes == 0 && ne != 0) return fail("tensor of an unsupported type");
    g->by_name[t.name] = g->tensors.size();
    g->tensors.push_back(t);
  }
  uint64_t align = 32;
  auto it = g->meta.find("general.alignment");
  if (it != g->meta.end() && (it->second.is_uint || it->second.is_int)) {
    const uint64_t a = it->second.is_uint ? it->second.u : (uint64_t)it->second.i;
    if (a > 0) align = a;
  }
  g->data_offset = (r.pos + align - 1) / align * align;
  for (const Tensor& t : g->tensors)
    if (g->data_offset + t.offset + t.n_bytes > g->size) return fail("tensor data past end of file");
  *out = g;
  return RRR_OK;
}

int rrr_gguf_close(rrr_gguf* g) {
  if (!g) return RRR_OK;
  Staging& st = g->staging;
  if (st.stream) {
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(st.device);
    cudaStreamSynchronize(st.stream);
    cudaStreamDestroy(st.stream);
    for (int b = 0; b < 2; ++b) {
      if (st.done[b]) cudaEventDestroy(st.done[b]);
      if (st.pinned[b]) cudaFreeHost(st.pinned[b]);
    }
    cudaSetDevice(cur);
  }
  if (g->map) munmap(const_cast<uint8_t*>(g->map), g->size);
  if (g->fd >= 0) ::close(g->fd);
  delete g;
  return RRR_OK;
}

int rrr_gguf_n_tensors(rrr_gguf* g, int64_t* n) {
  if (!g || !n) return set_error(nullptr, RRR_ERR_INVALID_ARG, "rrr_gguf_n_tensors: null argument");
  *n = (int64_t)g->tensors.size();
  return RRR_OK;
}

int rrr_gguf_tensor_at(rrr_gguf* g, int64_t i, rrr_gguf_tensor* out) {
  if (!g || !out) return set_error(nullptr, RRR_ERR_INVALID_ARG, "rrr_gguf_tensor_at: null argument");
  if (i < 0 || (size_t)i >= g->tensors.size())
    return set_error(nullptr, RRR_ERR_INVALID_ARG, "rrr_gguf_tensor_at: index %lld out of range",
                     (long long)i);
  return fill_tensor(g, (size_t)i, out);
}

int rrr_gguf_find_tensor(rrr_gguf* g, const char* name, rrr_gguf_tensor* out) {
  if (!g || !name || !out) return set_error(nullptr, RRR_ERR_INVALID_ARG, "rrr_gguf_find_tensor: null argument");
  auto it = g->by_name.find(name);
  if (it == g->by_name.end())
    return set_error(nullptr, RRR_ERR_INVALID_ARG, "Tensor not found: %s", name);
  return fill_tensor(g, it->second, out);
}

int rrr_gguf_meta_u64(rrr_gguf* g, const char* key, uint64_t* out) {
  if (!g || !key || !out) return set_error(nullptr, RRR_ERR_INVALID_ARG, "rrr_gguf_meta_u64: null argument");
  auto it = g->meta.find(key);
  if (it == g->meta.end() || !(it->second.is_uint || it->second.is_int) || it->second.type == 7)
    return set_error(nullptr, RRR_ERR_INVALID_ARG, "metadata %s is missing or not an integer", key);
  *out = it->second.is_uint ? it->second.u : (uint64_t)it->second.i;
  return RRR_OK;
}

int rrr_gguf_meta_f32(rrr_gguf* g, const char* key, float* out) {
  if (!g || !key || !out) return set_error(nullptr, RRR_ERR_INVALID_ARG, "rrr_gguf_meta_f32: null argument");
  auto it = g->meta.find(key);
  if (it == g->meta.end() || !it->second.is_float)
    return set_error(nullptr, RRR_ERR_INVALID_ARG, "metadata %s is missing or not a float", key);
  *out = (float)it->second.f;
  return RRR_OK;
}

int rrr_gguf_meta_str(rrr_gguf* g, const char* key, const char** out) {
  if (!g || !key || !out) return set_error(nullptr, RRR_ERR_INVALID_ARG, "rrr_gguf_meta_str: null argument");
  auto it = g->meta.find(key);
  if (it == g->meta.end() || !it->second.is_str)
    return set_error(nullptr, RRR_ERR_INVALID_ARG, "metadata %s is missing or not a string", key);
  *out = it->second.s.c_str();
  return RRR_OK;
}

int rrr_gguf_version(rrr_gguf* g, uint32_t* v) {
  if (!g || !v) return set_error(nullptr, RRR_ERR_INVALID_ARG, "rrr_gguf_version: null argument");
  *v = g->version;
  return RRR_OK;
}

int rrr_gguf_data_offset(rrr_gguf* g, uint64_t* off) {
  if (!g || !off) return set_error(nullptr, RRR_ERR_INVALID_ARG, "rrr_gguf_data_offset: null argument");
  *off = g->data_offset;
  return RRR_OK;
}

int rrr_gguf_upload(rrr_ctx* ctx, rrr_gguf* g, const char* name, void** dptr, uint64_t* n_bytes) {
  if (!name) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_gguf_upload: null argument");
  uint64_t nb = 0;
  const int rc = rrr_gguf_load(ctx, g, &name, 1, dptr, &nb, nullptr);
  if (rc == RRR_OK && n_bytes) *n_bytes = nb;
  return rc;
}

int rrr_gguf_load(rrr_ctx* ctx, rrr_gguf* g, const char* const* names, int n, void** dptrs,
                  uint64_t* n_bytes, double* seconds) {
  if (!ctx) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null context");
  if (!g || !names || !dptrs || n < 1) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_gguf_load: bad arguments");
  for (int i = 0; i < n; ++i) dptrs[i] = nullptr;
  std::vector<rrr_gguf_tensor> ts(n);
  std::vector<size_t> offs(n);
  size_t total = 0;
  for (int i = 0; i < n; ++i) {
    if (!names[i] || rrr_gguf_find_tensor(g, names[i], &ts[i]) != RRR_OK)
      return set_error(ctx, RRR_ERR_INVALID_ARG, "Tensor not found: %s", names[i] ? names[i] : "(null)");
    offs[i] = total;
    total += (ts[i].n_bytes + 255) & ~(uint64_t)255;  // 256-byte aligned tensors
  }
  int rc = bind_device(ctx);
  if (rc) return rc;
  const auto t0 = std::chrono::steady_clock::now();
  Staging& st = g->staging;
  cudaError_t e = cudaSuccess;
  if (st.device != ctx->device) {
    // first upload on this device: pinned buffers, events, a copy stream (kept until close)
    if (st.stream) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_gguf_load: the file's staging belongs to another device");
    for (int b = 0; b < 2 && e == cudaSuccess; ++b) {
      e = cudaHostAlloc(&st.pinned[b], Staging::kChunk, cudaHostAllocDefault);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&st.done[b], cudaEventDisableTiming);
    }
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&st.stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_gguf_load: staging");
    st.device = ctx->device;
  }
  void* arena = nullptr;
  e = cudaMalloc(&arena, total ? total : 256);
  if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_gguf_load: cudaMalloc");
  char* base = static_cast<char*>(arena);
  int b = 0;
  bool used[2] = {false, false};
  for (int i = 0; i < n && e == cudaSuccess; ++i) {
    const uint8_t* src = static_cast<const uint8_t*>(ts[i].data);
    for (uint64_t done = 0; done < ts[i].n_bytes && e == cudaSuccess;) {
      const size_t len = (size_t)std::min<uint64_t>(Staging::kChunk, ts[i].n_bytes - done);
      // the buffer's previous DMA must have finished before it is overwritten
      if (used[b]) e = cudaEventSynchronize(st.done[b]);
      if (e != cudaSuccess) break;
      char* dst = static_cast<char*>(st.pinned[b]);
      const uint8_t* from = src + done;
      const size_t part = (len + Staging::kThreads - 1) / Staging::kThreads;
      std::vector<std::thread> th;
      for (int k = 1; k < Staging::kThreads && (size_t)k * part < len; ++k)
        th.emplace_back([=] { memcpy(dst + k * part, from + k * part, std::min(part, len - k * part)); });
      memcpy(dst, from, std::min(part, len));
      for (auto& t : th) t.join();
      e = cudaMemcpyAsync(base + offs[i] + done, dst, len, cudaMemcpyHostToDevice, st.stream);
      if (e == cudaSuccess) e = cudaEventRecord(st.done[b], st.stream);
      used[b] = true;
      done += len;
      b ^= 1;
    }
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(st.stream);
  if (e != cudaSuccess) {
    cudaStreamSynchronize(st.stream);
    cudaFree(arena);
    return cuda_error(ctx, e, "rrr_gguf_load: copy");
  }
  for (int i = 0; i < n; ++i) {
    dptrs[i] = base + offs[i];
    if (n_bytes) n_bytes[i] = ts[i].n_bytes;
  }
  if (seconds)
    *seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  return RRR_OK;
}

}  // extern "C"
