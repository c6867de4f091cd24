// Host codecs of the runtime library (C ABI, bound from Python with ctypes):
//
//  * safetensors  - read F32 / BF16 / F16 tensors as fp32, write F32 (reference core/model/src/checkpoint.rs:27-216).
//                   Header JSON keys sorted, padded with spaces to 8 bytes, data laid out in header order.
//  * zstd         - libzstd.so.1 opened with dlopen (the image ships the runtime library but no header;
//                   the handful of entry points used here are declared locally).
//  * SparseDelta  - the reference's delta wire format: zstd(JSON {indices, values, shapes, scales, config})
//                   (compression.rs:92-104, 262-290, 429-441), encoded/decoded without a JSON DOM for the
//                   big index / value arrays.
//  * DTZ1         - this framework's binary delta format (flat indices + int8 + per-block scales).
//  * shard assignment - SipHash-1-3 (Rust DefaultHasher, keys 0,0) + splitmix64 Fisher-Yates
//                   (core/model/src/training.rs:229-279), bit-exact with the reference.
#include <dlfcn.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "json.hpp"

#define DT_API extern "C" __attribute__((visibility("default")))

namespace {

thread_local std::string g_err;
int set_err(const std::string& s) {
  g_err = s;
  return -1;
}

// ───────────────────────────── half conversions ─────────────────────────────
float bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
float f16_to_f32(uint16_t h) {
  uint32_t sign = (h >> 15) & 1, exp = (h >> 10) & 0x1F, man = h & 0x3FF, out;
  if (exp == 0) {
    if (man == 0) {
      out = sign << 31;
    } else {
      int e = -1;
      do { man <<= 1; ++e; } while (!(man & 0x400));
      man &= 0x3FF;
      out = (sign << 31) | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 0x1F) {
    out = (sign << 31) | (0xFFu << 23) | (man << 13);
  } else {
    out = (sign << 31) | ((exp - 15 + 127) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &out, 4);
  return f;
}

// ───────────────────────────── zstd via dlopen ─────────────────────────────
struct Zstd {
  void* h = nullptr;
  size_t (*compress)(void*, size_t, const void*, size_t, int) = nullptr;
  size_t (*decompress)(void*, size_t, const void*, size_t) = nullptr;
  size_t (*bound)(size_t) = nullptr;
  unsigned (*is_error)(size_t) = nullptr;
  const char* (*err_name)(size_t) = nullptr;
  unsigned long long (*content_size)(const void*, size_t) = nullptr;
  void* (*create_dctx)() = nullptr;
  size_t (*free_dctx)(void*) = nullptr;
  size_t (*decompress_stream)(void*, void*, void*) = nullptr;
  size_t (*dstream_out_size)() = nullptr;
};
Zstd g_z;
std::once_flag g_z_once;

bool zstd_ok() {
  std::call_once(g_z_once, [] {
    const char* names[] = {"libzstd.so.1", "libzstd.so"};
    for (const char* n : names) {
      g_z.h = dlopen(n, RTLD_NOW | RTLD_LOCAL);
      if (g_z.h) break;
    }
    if (!g_z.h) return;
    g_z.compress = (decltype(g_z.compress))dlsym(g_z.h, "ZSTD_compress");
    g_z.decompress = (decltype(g_z.decompress))dlsym(g_z.h, "ZSTD_decompress");
    g_z.bound = (decltype(g_z.bound))dlsym(g_z.h, "ZSTD_compressBound");
    g_z.is_error = (decltype(g_z.is_error))dlsym(g_z.h, "ZSTD_isError");
    g_z.err_name = (decltype(g_z.err_name))dlsym(g_z.h, "ZSTD_getErrorName");
    g_z.content_size = (decltype(g_z.content_size))dlsym(g_z.h, "ZSTD_getFrameContentSize");
    g_z.create_dctx = (decltype(g_z.create_dctx))dlsym(g_z.h, "ZSTD_createDStream");
    g_z.free_dctx = (decltype(g_z.free_dctx))dlsym(g_z.h, "ZSTD_freeDStream");
    g_z.decompress_stream = (decltype(g_z.decompress_stream))dlsym(g_z.h, "ZSTD_decompressStream");
    g_z.dstream_out_size = (decltype(g_z.dstream_out_size))dlsym(g_z.h, "ZSTD_DStreamOutSize");
  });
  return g_z.compress && g_z.decompress && g_z.bound && g_z.is_error;
}

struct ZInBuf { const void* src; size_t size; size_t pos; };
struct ZOutBuf { void* dst; size_t size; size_t pos; };

bool zstd_decompress_all(const uint8_t* src, size_t n, std::string& out, std::string& err) {
  if (!zstd_ok()) { err = "libzstd.so.1 not available"; return false; }
  unsigned long long cs = g_z.content_size ? g_z.content_size(src, n) : 0ULL - 1;
  const unsigned long long UNKNOWN = 0ULL - 1, ERR = 0ULL - 2;
  if (cs != UNKNOWN && cs != ERR) {
    out.resize(cs);
    size_t r = g_z.decompress(&out[0], cs, src, n);
    if (g_z.is_error(r)) { err = g_z.err_name(r); return false; }
    out.resize(r);
    return true;
  }
  if (!g_z.create_dctx || !g_z.decompress_stream) { err = "zstd: unknown frame size and no streaming API"; return false; }
  void* ds = g_z.create_dctx();
  size_t chunk = g_z.dstream_out_size ? g_z.dstream_out_size() : (1 << 17);
  ZInBuf in{src, n, 0};
  std::vector<char> buf(chunk);
  out.clear();
  while (in.pos < in.size) {
    ZOutBuf o{buf.data(), chunk, 0};
    size_t r = g_z.decompress_stream(ds, &o, &in);
    if (g_z.is_error(r)) { err = g_z.err_name(r); g_z.free_dctx(ds); return false; }
    out.append(buf.data(), o.pos);
    if (r == 0 && in.pos >= in.size) break;
  }
  g_z.free_dctx(ds);
  return true;
}

// ───────────────────────────── small buffers handed to Python ─────────────────────────────
struct Blob {
  std::string data;
};

// ───────────────────────────── SipHash-1-3 / splitmix64 ─────────────────────────────
inline uint64_t rotl(uint64_t x, int b) { return (x << b) | (x >> (64 - b)); }
struct Sip13 {
  uint64_t v0, v1, v2, v3;
  uint64_t tail = 0;
  int ntail = 0;
  uint64_t len = 0;
  Sip13() {
    v0 = 0x736f6d6570736575ULL;
    v1 = 0x646f72616e646f6dULL;
    v2 = 0x6c7967656e657261ULL;
    v3 = 0x7465646279746573ULL;
  }
  void round() {
    v0 += v1; v1 = rotl(v1, 13); v1 ^= v0; v0 = rotl(v0, 32);
    v2 += v3; v3 = rotl(v3, 16); v3 ^= v2;
    v0 += v3; v3 = rotl(v3, 21); v3 ^= v0;
    v2 += v1; v1 = rotl(v1, 17); v1 ^= v2; v2 = rotl(v2, 32);
  }
  void word(uint64_t m) {
    v3 ^= m;
    round();
    v0 ^= m;
  }
  void write(const uint8_t* p, size_t n) {
    len += n;
    for (size_t i = 0; i < n; ++i) {
      tail |= (uint64_t)p[i] << (8 * ntail);
      if (++ntail == 8) {
        word(tail);
        tail = 0;
        ntail = 0;
      }
    }
  }
  uint64_t finish() {
    uint64_t b = ((len & 0xff) << 56) | tail;
    word(b);
    v2 ^= 0xff;
    round(); round(); round();
    return v0 ^ v1 ^ v2 ^ v3;
  }
};
inline uint64_t splitmix64(uint64_t s) {
  s += 0x9e3779b97f4a7c15ULL;
  uint64_t z = s;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}

}  // namespace

// ───────────────────────────── error / blob API ─────────────────────────────
DT_API const char* dtr_last_error() { return g_err.c_str(); }
DT_API long long dtr_blob_size(void* b) { return b ? (long long)static_cast<Blob*>(b)->data.size() : 0; }
DT_API const void* dtr_blob_data(void* b) { return b ? static_cast<Blob*>(b)->data.data() : nullptr; }
DT_API void dtr_blob_free(void* b) { delete static_cast<Blob*>(b); }

// ───────────────────────────── zstd ─────────────────────────────
DT_API int dtr_zstd_available() { return zstd_ok() ? 1 : 0; }

DT_API void* dtr_zstd_compress(const void* src, long long n, int level) {
  if (!zstd_ok()) { set_err("libzstd.so.1 not available"); return nullptr; }
  auto* b = new Blob;
  size_t cap = g_z.bound((size_t)n);
  b->data.resize(cap);
  size_t r = g_z.compress(&b->data[0], cap, src, (size_t)n, level);
  if (g_z.is_error(r)) { set_err(g_z.err_name(r)); delete b; return nullptr; }
  b->data.resize(r);
  return b;
}

DT_API void* dtr_zstd_decompress(const void* src, long long n) {
  auto* b = new Blob;
  std::string err;
  if (!zstd_decompress_all((const uint8_t*)src, (size_t)n, b->data, err)) { set_err(err); delete b; return nullptr; }
  return b;
}

// ───────────────────────────── shard assignment ─────────────────────────────
DT_API unsigned long long dtr_siphash13(const void* data, long long n) {
  Sip13 h;
  h.write((const uint8_t*)data, (size_t)n);
  return h.finish();
}

DT_API unsigned long long dtr_splitmix64(unsigned long long s) { return splitmix64(s); }

// Gaussian test matrix of the low-rank compressor (reference lowrank.rs:54-80): n x r values (row-major),
// state = m * 0x9e3779b97f4a7c15 + n + r, each draw replaces the state by splitmix64 of it; pairs of
// draws give u1 = lo32 / 2^32 + 1e-10, u2 = lo32 / 2^32 and the value sqrt(-2 ln u1) cos(2 pi u2) (f64).
DT_API void dtr_lowrank_omega(long long m, long long n, long long r, double* out) {
  uint64_t st = (uint64_t)m * 0x9e3779b97f4a7c15ULL + (uint64_t)n + (uint64_t)r;
  const long long cnt = n * r;
  for (long long i = 0; i < cnt; ++i) {
    st = splitmix64(st);
    const double u1 = (double)(st & 0xFFFFFFFFULL) / 4294967296.0 + 1e-10;
    st = splitmix64(st);
    const double u2 = (double)(st & 0xFFFFFFFFULL) / 4294967296.0;
    out[i] = std::sqrt(-2.0 * std::log(u1)) * std::cos(2.0 * M_PI * u2);
  }
}

// Rust `format!("{}:{}", version, node_id).hash()` / `version.hash()` on DefaultHasher (SipHash-1-3,
// keys 0,0): a str hashes its bytes followed by 0xff, a u64 its 8 little-endian bytes.
DT_API unsigned long long dtr_hash_str(const char* s) {
  Sip13 h;
  h.write((const uint8_t*)s, strlen(s));
  uint8_t ff = 0xff;
  h.write(&ff, 1);
  return h.finish();
}
DT_API unsigned long long dtr_hash_u64(unsigned long long v) {
  Sip13 h;
  uint8_t b[8];
  for (int i = 0; i < 8; ++i) b[i] = (uint8_t)(v >> (8 * i));
  h.write(b, 8);
  return h.finish();
}

// out must hold min(shards_per_node, total_shards) entries; returns that count.
DT_API long long dtr_shard_assignment(const char* node_id, unsigned long long version, long long total_shards,
                                      long long shards_per_node, long long* out) {
  long long count = std::min(shards_per_node, total_shards);
  std::string key = std::to_string(version) + ":" + node_id;
  uint64_t node_seed = dtr_hash_str(key.c_str());
  uint64_t global_seed = dtr_hash_u64(version);
  std::vector<long long> all(total_shards);
  for (long long i = 0; i < total_shards; ++i) all[i] = i;
  uint64_t st = global_seed;
  for (long long i = total_shards - 1; i >= 1; --i) {
    st = splitmix64(st);
    long long j = (long long)(st % (uint64_t)(i + 1));
    std::swap(all[i], all[j]);
  }
  st = node_seed;
  for (long long i = total_shards - 1; i >= 1; --i) {
    st = splitmix64(st);
    long long j = (long long)(st % (uint64_t)(i + 1));
    std::swap(all[i], all[j]);
  }
  for (long long i = 0; i < count; ++i) out[i] = all[i];
  return count;
}

// ───────────────────────────── safetensors ─────────────────────────────
struct StTensor {
  std::string name, dtype;
  std::vector<int64_t> shape;
  uint64_t begin, end;
};
struct StFile {
  std::vector<StTensor> tensors;
  std::string metadata_json;
  const uint8_t* data = nullptr;  // start of the byte buffer
  size_t data_size = 0;
  void* map = nullptr;
  size_t map_size = 0;
  std::string owned;  // when loaded from memory
};

static int parse_st(StFile* f, const uint8_t* buf, size_t n) {
  if (n < 8) return set_err("safetensors: file too small");
  uint64_t hlen = 0;
  for (int i = 0; i < 8; ++i) hlen |= (uint64_t)buf[i] << (8 * i);
  if (hlen > n - 8) return set_err("safetensors: header length out of range");
  dtj::Value h;
  try {
    h = dtj::parse((const char*)buf + 8, hlen);
  } catch (std::exception& e) {
    return set_err(std::string("safetensors header: ") + e.what());
  }
  if (h.kind != dtj::Value::Obj) return set_err("safetensors: header is not an object");
  f->data = buf + 8 + hlen;
  f->data_size = n - 8 - hlen;
  for (auto& kv : *h.o) {
    if (kv.first == "__metadata__") {
      f->metadata_json = dtj::dump(kv.second);
      continue;
    }
    StTensor t;
    t.name = kv.first;
    t.dtype = kv.second.at("dtype").s;
    for (auto& d : *kv.second.at("shape").a) t.shape.push_back(d.as_int());
    auto& off = *kv.second.at("data_offsets").a;
    t.begin = (uint64_t)off[0].as_int();
    t.end = (uint64_t)off[1].as_int();
    if (t.end < t.begin || t.end > f->data_size) return set_err("safetensors: bad data_offsets for " + t.name);
    f->tensors.push_back(std::move(t));
  }
  return 0;
}

DT_API void* dtr_st_open(const char* path) {
  int fd = open(path, O_RDONLY);
  if (fd < 0) { set_err(std::string("open ") + path + ": " + strerror(errno)); return nullptr; }
  struct stat sb;
  fstat(fd, &sb);
  size_t n = (size_t)sb.st_size;
  void* m = n ? mmap(nullptr, n, PROT_READ, MAP_PRIVATE, fd, 0) : nullptr;
  close(fd);
  if (n && m == MAP_FAILED) { set_err("mmap failed"); return nullptr; }
  auto* f = new StFile;
  f->map = m;
  f->map_size = n;
  if (parse_st(f, (const uint8_t*)m, n)) {
    if (m) munmap(m, n);
    delete f;
    return nullptr;
  }
  return f;
}

DT_API void* dtr_st_open_bytes(const void* data, long long n) {
  auto* f = new StFile;
  f->owned.assign((const char*)data, (size_t)n);
  if (parse_st(f, (const uint8_t*)f->owned.data(), f->owned.size())) { delete f; return nullptr; }
  return f;
}

DT_API void dtr_st_close(void* h) {
  auto* f = static_cast<StFile*>(h);
  if (!f) return;
  if (f->map) munmap(f->map, f->map_size);
  delete f;
}

DT_API int dtr_st_count(void* h) { return (int)static_cast<StFile*>(h)->tensors.size(); }
DT_API const char* dtr_st_name(void* h, int i) { return static_cast<StFile*>(h)->tensors[i].name.c_str(); }
DT_API const char* dtr_st_dtype(void* h, int i) { return static_cast<StFile*>(h)->tensors[i].dtype.c_str(); }
DT_API int dtr_st_ndim(void* h, int i) { return (int)static_cast<StFile*>(h)->tensors[i].shape.size(); }
DT_API long long dtr_st_dim(void* h, int i, int d) { return static_cast<StFile*>(h)->tensors[i].shape[d]; }
DT_API const char* dtr_st_metadata(void* h) { return static_cast<StFile*>(h)->metadata_json.c_str(); }

// Decode tensor i to fp32 into out (numel entries). Returns numel or -1.
DT_API long long dtr_st_read_f32(void* h, int i, float* out, long long cap) {
  auto* f = static_cast<StFile*>(h);
  const StTensor& t = f->tensors[i];
  const uint8_t* p = f->data + t.begin;
  size_t nb = t.end - t.begin;
  long long n;
  if (t.dtype == "F32") {
    n = (long long)(nb / 4);
    if (n > cap) return set_err("output too small");
    memcpy(out, p, (size_t)n * 4);
  } else if (t.dtype == "BF16" || t.dtype == "F16") {
    n = (long long)(nb / 2);
    if (n > cap) return set_err("output too small");
    bool bf = t.dtype == "BF16";
    for (long long k = 0; k < n; ++k) {
      uint16_t v = (uint16_t)(p[2 * k] | (p[2 * k + 1] << 8));
      out[k] = bf ? bf16_to_f32(v) : f16_to_f32(v);
    }
  } else {
    return set_err("unsupported dtype " + t.dtype);
  }
  return n;
}

// Serialize fp32 tensors. names/ndims/dims are flattened arrays (dims concatenated). If path is null the
// bytes are returned as a Blob handle through *blob_out.
DT_API int dtr_st_save(const char* path, int count, const char* const* names, const int* ndims,
                       const long long* dims, const float* const* data, const char* metadata_json,
                       void** blob_out) {
  std::vector<int> order(count);
  for (int i = 0; i < count; ++i) order[i] = i;
  std::sort(order.begin(), order.end(), [&](int a, int b) { return strcmp(names[a], names[b]) < 0; });
  std::vector<size_t> dim_off(count);
  size_t acc = 0;
  for (int i = 0; i < count; ++i) { dim_off[i] = acc; acc += ndims[i]; }
  std::string hdr = "{";
  bool first = true;
  if (metadata_json && *metadata_json) {
    hdr += "\"__metadata__\":";
    hdr += metadata_json;
    first = false;
  }
  uint64_t off = 0;
  std::vector<uint64_t> nbytes(count);
  for (int k = 0; k < count; ++k) {
    int i = order[k];
    uint64_t numel = 1;
    for (int d = 0; d < ndims[i]; ++d) numel *= (uint64_t)dims[dim_off[i] + d];
    nbytes[i] = numel * 4;
    if (!first) hdr += ",";
    first = false;
    dtj::dump_string(names[i], hdr);
    hdr += ":{\"dtype\":\"F32\",\"shape\":[";
    for (int d = 0; d < ndims[i]; ++d) {
      if (d) hdr += ",";
      hdr += std::to_string(dims[dim_off[i] + d]);
    }
    hdr += "],\"data_offsets\":[" + std::to_string(off) + "," + std::to_string(off + nbytes[i]) + "]}";
    off += nbytes[i];
  }
  hdr += "}";
  while (hdr.size() % 8) hdr += ' ';
  uint64_t hl = hdr.size();
  char lenb[8];
  for (int i = 0; i < 8; ++i) lenb[i] = (char)(hl >> (8 * i));
  if (path) {
    std::string tmp = std::string(path) + ".tmp";
    FILE* fp = fopen(tmp.c_str(), "wb");
    if (!fp) return set_err(std::string("open ") + tmp + ": " + strerror(errno));
    bool ok = fwrite(lenb, 1, 8, fp) == 8 && fwrite(hdr.data(), 1, hdr.size(), fp) == hdr.size();
    for (int k = 0; k < count && ok; ++k) {
      int i = order[k];
      ok = fwrite(data[i], 1, nbytes[i], fp) == nbytes[i];
    }
    if (fclose(fp) != 0) ok = false;
    if (!ok) { unlink(tmp.c_str()); return set_err("write failed"); }
    if (rename(tmp.c_str(), path) != 0) return set_err(std::string("rename: ") + strerror(errno));
    return 0;
  }
  auto* b = new Blob;
  b->data.reserve(8 + hdr.size() + off);
  b->data.append(lenb, 8);
  b->data += hdr;
  for (int k = 0; k < count; ++k) {
    int i = order[k];
    b->data.append((const char*)data[i], nbytes[i]);
  }
  *blob_out = b;
  return 0;
}

// ───────────────────────────── SparseDelta JSON (reference format) ─────────────────────────────
// Encoder input: per tensor name, shape, kept indices (u32, ascending) and values (f32), optional
// per-tensor scale; config_json is the CompressionConfig object text.
DT_API void* dtr_sparse_delta_encode(int count, const char* const* names, const int* ndims, const long long* dims,
                                     const long long* nkept, const unsigned* const* indices,
                                     const float* const* values, const float* scales, const char* config_json,
                                     int zstd_level) {
  std::string out;
  size_t total = 0;
  for (int i = 0; i < count; ++i) total += (size_t)nkept[i];
  out.reserve(total * 22 + 4096);
  out += "{\"indices\":{";
  for (int i = 0; i < count; ++i) {
    if (i) out += ',';
    dtj::dump_string(names[i], out);
    out += ":[";
    for (long long k = 0; k < nkept[i]; ++k) {
      if (k) out += ',';
      out += std::to_string(indices[i][k]);
    }
    out += ']';
  }
  out += "},\"values\":{";
  for (int i = 0; i < count; ++i) {
    if (i) out += ',';
    dtj::dump_string(names[i], out);
    out += ":[";
    for (long long k = 0; k < nkept[i]; ++k) {
      if (k) out += ',';
      dtj::dump_double((double)values[i][k], out);
    }
    out += ']';
  }
  out += "},\"shapes\":{";
  size_t doff = 0;
  for (int i = 0; i < count; ++i) {
    if (i) out += ',';
    dtj::dump_string(names[i], out);
    out += ":[";
    for (int d = 0; d < ndims[i]; ++d) {
      if (d) out += ',';
      out += std::to_string(dims[doff + d]);
    }
    doff += ndims[i];
    out += ']';
  }
  out += "},\"scales\":";
  if (scales) {
    out += '{';
    for (int i = 0; i < count; ++i) {
      if (i) out += ',';
      dtj::dump_string(names[i], out);
      out += ':';
      dtj::dump_double((double)scales[i], out);
    }
    out += '}';
  } else {
    out += "null";
  }
  out += ",\"config\":";
  out += (config_json && *config_json) ? config_json : "null";
  out += '}';
  if (zstd_level <= 0) {
    auto* b = new Blob;
    b->data = std::move(out);
    return b;
  }
  return dtr_zstd_compress(out.data(), (long long)out.size(), zstd_level);
}

// Decoder: (optionally zstd) SparseDelta JSON -> dense fp32 per tensor. Returns a handle with
// accessors below. Low-rank JSON ({"tensors": {...}, "rank": r}) is detected and reported.
struct DecodedDelta {
  std::vector<std::string> names;
  std::vector<std::vector<int64_t>> shapes;
  std::vector<std::vector<float>> dense;
  std::string config_json;
  int lowrank = 0;
  std::string raw_json;
};

static int decode_sparse(const std::string& js, DecodedDelta* dd) {
  dtj::Value v;
  try {
    v = dtj::parse(js);
  } catch (std::exception& e) {
    return set_err(std::string("delta json: ") + e.what());
  }
  if (v.find("tensors") && v.find("rank")) {
    dd->lowrank = 1;
    dd->raw_json = js;
    return 0;
  }
  const dtj::Value* shapes = v.find("shapes");
  const dtj::Value* idx = v.find("indices");
  const dtj::Value* vals = v.find("values");
  if (!shapes || !idx || !vals) return set_err("delta json: missing indices/values/shapes");
  if (const dtj::Value* c = v.find("config")) dd->config_json = dtj::dump(*c);
  for (auto& kv : *shapes->o) {
    dd->names.push_back(kv.first);
    std::vector<int64_t> sh;
    int64_t numel = 1;
    for (auto& d : *kv.second.a) { sh.push_back(d.as_int()); numel *= d.as_int(); }
    dd->shapes.push_back(sh);
    std::vector<float> flat((size_t)numel, 0.f);
    const dtj::Value* ii = idx->find(kv.first);
    const dtj::Value* vv = vals->find(kv.first);
    if (ii && vv) {
      size_t n = std::min(ii->a->size(), vv->a->size());
      for (size_t k = 0; k < n; ++k) {
        int64_t j = (*ii->a)[k].as_int();
        if (j < 0 || j >= numel) return set_err("delta json: index out of range in " + kv.first);
        flat[(size_t)j] = (float)(*vv->a)[k].num();
      }
    }
    dd->dense.push_back(std::move(flat));
  }
  return 0;
}

DT_API void* dtr_delta_decode(const void* data, long long n) {
  auto* dd = new DecodedDelta;
  std::string js;
  const uint8_t* p = (const uint8_t*)data;
  bool is_zstd = n >= 4 && p[0] == 0x28 && p[1] == 0xB5 && p[2] == 0x2F && p[3] == 0xFD;
  if (is_zstd) {
    std::string err;
    if (!zstd_decompress_all(p, (size_t)n, js, err)) { set_err("zstd decompression failed: " + err); delete dd; return nullptr; }
  } else {
    js.assign((const char*)data, (size_t)n);  // raw-JSON fallback (aggregation.rs:504-513)
  }
  if (decode_sparse(js, dd)) { delete dd; return nullptr; }
  return dd;
}
DT_API void dtr_delta_free(void* h) { delete static_cast<DecodedDelta*>(h); }
DT_API int dtr_delta_is_lowrank(void* h) { return static_cast<DecodedDelta*>(h)->lowrank; }
DT_API const char* dtr_delta_raw_json(void* h) { return static_cast<DecodedDelta*>(h)->raw_json.c_str(); }
DT_API int dtr_delta_count(void* h) { return (int)static_cast<DecodedDelta*>(h)->names.size(); }
DT_API const char* dtr_delta_name(void* h, int i) { return static_cast<DecodedDelta*>(h)->names[i].c_str(); }
DT_API int dtr_delta_ndim(void* h, int i) { return (int)static_cast<DecodedDelta*>(h)->shapes[i].size(); }
DT_API long long dtr_delta_dim(void* h, int i, int d) { return static_cast<DecodedDelta*>(h)->shapes[i][d]; }
DT_API const float* dtr_delta_data(void* h, int i) { return static_cast<DecodedDelta*>(h)->dense[i].data(); }
DT_API long long dtr_delta_numel(void* h, int i) { return (long long)static_cast<DecodedDelta*>(h)->dense[i].size(); }
DT_API const char* dtr_delta_config(void* h) { return static_cast<DecodedDelta*>(h)->config_json.c_str(); }

// ───────────────────────────── DTZ1 binary delta ─────────────────────────────
// Layout (little endian): "DTZ1" | u32 flags (1 = int8) | u32 block | u64 total_params | u64 count |
// u32 idx[count] | (int8 q[count] + pad to 4 + f32 scales[ceil(count/block)]) or f32 values[count],
// optionally zstd-compressed as a whole (detected by the zstd magic).
DT_API void* dtr_dtz_encode(long long total_params, long long count, const int* idx, const signed char* q,
                            const float* scales, const float* values, int block, int zstd_level) {
  std::string out;
  auto put32 = [&](uint32_t v) { out.append((const char*)&v, 4); };
  auto put64 = [&](uint64_t v) { out.append((const char*)&v, 8); };
  out += "DTZ1";
  put32(q ? 1u : 0u);
  put32((uint32_t)block);
  put64((uint64_t)total_params);
  put64((uint64_t)count);
  out.append((const char*)idx, (size_t)count * 4);
  if (q) {
    out.append((const char*)q, (size_t)count);
    while (out.size() % 4) out += '\0';
    long long nb = block > 0 ? (count + block - 1) / block : 0;
    out.append((const char*)scales, (size_t)nb * 4);
  } else {
    out.append((const char*)values, (size_t)count * 4);
  }
  if (zstd_level <= 0) {
    auto* b = new Blob;
    b->data = std::move(out);
    return b;
  }
  return dtr_zstd_compress(out.data(), (long long)out.size(), zstd_level);
}

// Decode DTZ1 (optionally zstd) into a dense fp32 vector of total_params entries (blob of floats).
DT_API void* dtr_dtz_decode_dense(const void* data, long long n) {
  std::string raw;
  const uint8_t* p = (const uint8_t*)data;
  if (n >= 4 && p[0] == 0x28 && p[1] == 0xB5 && p[2] == 0x2F && p[3] == 0xFD) {
    std::string err;
    if (!zstd_decompress_all(p, (size_t)n, raw, err)) { set_err(err); return nullptr; }
  } else {
    raw.assign((const char*)data, (size_t)n);
  }
  if (raw.size() < 28 || memcmp(raw.data(), "DTZ1", 4) != 0) { set_err("not a DTZ1 delta"); return nullptr; }
  uint32_t flags, block;
  uint64_t total, count;
  memcpy(&flags, raw.data() + 4, 4);
  memcpy(&block, raw.data() + 8, 4);
  memcpy(&total, raw.data() + 12, 8);
  memcpy(&count, raw.data() + 20, 8);
  size_t off = 28;
  if (raw.size() < off + count * 4) { set_err("DTZ1 truncated"); return nullptr; }
  const uint32_t* idx = (const uint32_t*)(raw.data() + off);
  off += count * 4;
  auto* b = new Blob;
  b->data.assign(total * 4, '\0');
  float* dense = (float*)&b->data[0];
  if (flags & 1) {
    const int8_t* q = (const int8_t*)(raw.data() + off);
    off += count;
    off = (off + 3) & ~size_t(3);
    const float* sc = (const float*)(raw.data() + off);
    uint64_t nb = block ? (count + block - 1) / block : 0;
    if (raw.size() < off + nb * 4) { set_err("DTZ1 truncated"); delete b; return nullptr; }
    for (uint64_t k = 0; k < count; ++k) {
      if (idx[k] >= total) { set_err("DTZ1 index out of range"); delete b; return nullptr; }
      dense[idx[k]] = (float)q[k] * sc[k / block];
    }
  } else {
    const float* v = (const float*)(raw.data() + off);
    if (raw.size() < off + count * 4) { set_err("DTZ1 truncated"); delete b; return nullptr; }
    for (uint64_t k = 0; k < count; ++k) {
      if (idx[k] >= total) { set_err("DTZ1 index out of range"); delete b; return nullptr; }
      dense[idx[k]] = v[k];
    }
  }
  return b;
}
