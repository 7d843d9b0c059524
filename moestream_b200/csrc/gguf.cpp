// GGUF expert source: slot fills read straight from the model file.
//
// The reference fills a slot by pread-ing one expert's bytes out of the GGUF
// the model was loaded from (src/llama-moestream.cpp:1230-1263 do_read /
// run_reads_parallel), with the file offsets taken from llama.cpp's loader
// and a few metadata integers read from the header by key suffix
// (:601-693 gguf_kv_int). It opens every shard of a split GGUF, named
// "<base>-NNNNN-of-MMMMM.gguf" (:571-598), refuses to run when one is
// missing (:1455-1466), and checks before the first read that every expert
// tensor ends inside its shard (:1478-1506).
//
// This library has no model loader to take the offsets from, so it parses
// the GGUF header itself (format version 2 and 3, little-endian): the
// key-value section, the tensor table and the aligned data section of every
// shard. All tensors are checked against their shard's size at open. Reads
// are pread loops spread over threads that take experts off a shared atomic
// counter, one thread set per call; a short read is an error (the reference
// leaves the rest of the destination as it was). A fill reads into pinned
// host memory owned by the handle (two halves used in turn, so that the
// reads of one call overlap the copies of the previous one) and hands it to
// msb_fill_slots_async.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "msb_internal.h"

using msb::fail;

namespace {

// ggml type id -> (elements per block, bytes per block); 0 = unknown id.
// The values are the GGUF format's published type sizes.
struct TypeSize { int blck; int bytes; };
TypeSize type_size(int t) {
  switch (t) {
    case 0: return {1, 4};       // F32
    case 1: return {1, 2};       // F16
    case 2: return {32, 18};     // Q4_0
    case 3: return {32, 20};     // Q4_1
    case 6: return {32, 22};     // Q5_0
    case 7: return {32, 24};     // Q5_1
    case 8: return {32, 34};     // Q8_0
    case 9: return {32, 40};     // Q8_1
    case 10: return {256, 84};   // Q2_K
    case 11: return {256, 110};  // Q3_K
    case 12: return {256, 144};  // Q4_K
    case 13: return {256, 176};  // Q5_K
    case 14: return {256, 210};  // Q6_K
    case 15: return {256, 292};  // Q8_K
    case 16: return {256, 66};   // IQ2_XXS
    case 17: return {256, 74};   // IQ2_XS
    case 18: return {256, 98};   // IQ3_XXS
    case 19: return {256, 50};   // IQ1_S
    case 20: return {32, 18};    // IQ4_NL
    case 21: return {256, 110};  // IQ3_S
    case 22: return {256, 82};   // IQ2_S
    case 23: return {256, 136};  // IQ4_XS
    case 24: return {1, 1};      // I8
    case 25: return {1, 2};      // I16
    case 26: return {1, 4};      // I32
    case 27: return {1, 8};      // I64
    case 28: return {1, 8};      // F64
    case 29: return {256, 56};   // IQ1_M
    case 30: return {1, 2};      // BF16
    case 34: return {256, 54};   // TQ1_0
    case 35: return {256, 66};   // TQ2_0
    case 39: return {32, 17};    // MXFP4
    default: return {0, 0};
  }
}

// GGUF value types.
enum : uint32_t {
  kU8 = 0, kI8, kU16, kI16, kU32, kI32, kF32, kBool, kString, kArray, kU64, kI64, kF64
};
constexpr int kMaxArrayDepth = 4;

// Sequential reader over one file with a 1 MiB buffer (headers hold large
// token arrays; one syscall per value would dominate the open).
class Reader {
 public:
  Reader(int fd, uint64_t size) : fd_(fd), size_(size), buf_(1 << 20) {}
  uint64_t pos() const { return pos_; }
  uint64_t left() const { return size_ - pos_; }
  bool get(void *dst, uint64_t n) {
    uint8_t *d = static_cast<uint8_t *>(dst);
    while (n) {
      if (pos_ < start_ || pos_ >= start_ + len_) {
        if (!refill()) return false;
      }
      const uint64_t at = pos_ - start_;
      const uint64_t take = std::min<uint64_t>(n, len_ - at);
      std::memcpy(d, buf_.data() + at, take);
      d += take; n -= take; pos_ += take;
    }
    return true;
  }
  bool skip(uint64_t n) {
    if (n > left()) return false;
    pos_ += n;
    return true;
  }
  template <class T> bool val(T &v) { return get(&v, sizeof v); }
  bool str(std::string &s, uint64_t max_len) {
    uint64_t n;
    if (!val(n) || n > max_len || n > left()) return false;
    s.resize(n);
    return n == 0 || get(&s[0], n);
  }
  bool skip_str() {
    uint64_t n;
    return val(n) && skip(n);
  }

 private:
  bool refill() {
    if (pos_ >= size_) return false;
    const uint64_t want = std::min<uint64_t>(buf_.size(), size_ - pos_);
    uint64_t got = 0;
    while (got < want) {
      const ssize_t r = pread(fd_, buf_.data() + got, want - got, off_t(pos_ + got));
      if (r < 0 && errno == EINTR) continue;
      if (r <= 0) break;
      got += uint64_t(r);
    }
    if (got == 0) return false;
    start_ = pos_;
    len_ = got;
    return true;
  }
  int fd_;
  uint64_t size_, pos_ = 0, start_ = 0, len_ = 0;
  std::vector<uint8_t> buf_;
};

bool fixed_size(uint32_t t, uint64_t &n) {
  static const uint8_t kSize[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
  if (t > kF64 || t == kString || t == kArray) return false;
  n = kSize[t];
  return true;
}

bool is_int(uint32_t t) {
  return t == kU8 || t == kI8 || t == kU16 || t == kI16 || t == kU32 || t == kI32 ||
         t == kU64 || t == kI64;
}

int64_t int_of(uint32_t t, const uint8_t *b) {
  switch (t) {
    case kU8: return *b;
    case kI8: return int8_t(*b);
    case kU16: { uint16_t v; std::memcpy(&v, b, 2); return v; }
    case kI16: { int16_t v; std::memcpy(&v, b, 2); return v; }
    case kU32: { uint32_t v; std::memcpy(&v, b, 4); return v; }
    case kI32: { int32_t v; std::memcpy(&v, b, 4); return v; }
    case kU64: { uint64_t v; std::memcpy(&v, b, 8); return int64_t(v); }
    default: { int64_t v; std::memcpy(&v, b, 8); return v; }
  }
}

bool skip_value(Reader &r, uint32_t t, int depth) {
  if (t == kString) return r.skip_str();
  if (t == kArray) {
    uint32_t et;
    uint64_t n;
    if (depth >= kMaxArrayDepth || !r.val(et) || !r.val(n)) return false;
    uint64_t sz;
    if (fixed_size(et, sz)) return n <= r.left() / std::max<uint64_t>(sz, 1) && r.skip(n * sz);
    for (uint64_t i = 0; i < n; ++i)
      if (!skip_value(r, et, depth + 1)) return false;
    return true;
  }
  uint64_t sz;
  return fixed_size(t, sz) && r.skip(sz);
}

struct Kv {
  std::string key;
  uint32_t type;
  int64_t ival;   // integer types only
};

struct Tensor {
  std::string name;
  int type;
  int n_dims;
  int64_t ne[4];
  int32_t shard;
  uint64_t offset;  // absolute, within the shard
  int64_t nbytes;
};

// Shard list of a split GGUF: a path ending in "-NNNNN-of-MMMMM.gguf" with
// 1 <= NNNNN <= MMMMM < 1000 names all MMMMM files; anything else is one file
// (the reference's rule, src/llama-moestream.cpp:580-597).
std::vector<std::string> shard_paths(const std::string &path) {
  if (path.size() > 20) {
    const std::string tail = path.substr(path.size() - 20);
    int a = 0, b = 0;
    char end[8] = {0};
    if (std::sscanf(tail.c_str(), "-%5d-of-%5d%7s", &a, &b, end) == 3 &&
        std::strcmp(end, ".gguf") == 0 && a >= 1 && b >= 1 && a <= b && b < 1000) {
      std::vector<std::string> v;
      const std::string base = path.substr(0, path.size() - 20);
      for (int i = 1; i <= b; ++i) {
        char suf[32];
        std::snprintf(suf, sizeof suf, "-%05d-of-%05d.gguf", i, b);
        v.push_back(base + suf);
      }
      return v;
    }
  }
  return {path};
}

}  // namespace

struct msb_gguf_s {
  std::vector<std::string> paths;
  std::vector<int> fds;
  std::vector<uint64_t> sizes;
  std::vector<Kv> kvs;         // key-value section of the first shard
  std::vector<Tensor> tensors; // every shard's, in file order
  struct Stage {
    uint8_t *host = nullptr;
    size_t bytes = 0;
    cudaEvent_t done = nullptr;
    int device = -1;
    bool pending = false;
  } stage[2];
  int next_stage = 0;

  ~msb_gguf_s() {
    for (Stage &s : stage) {
      if (s.pending) cudaEventSynchronize(s.done);
      if (s.done) cudaEventDestroy(s.done);
      if (s.host) cudaFreeHost(s.host);
    }
    for (int fd : fds)
      if (fd >= 0) close(fd);
  }
};

namespace {

// Parses one shard's header; appends its tensors (and, for shard 0, its
// key-value pairs). Returns MSB_OK or a failure with the reason.
int parse_shard(msb_gguf_s *g, int32_t shard) {
  const std::string &path = g->paths[size_t(shard)];
  Reader r(g->fds[size_t(shard)], g->sizes[size_t(shard)]);
  char magic[4];
  uint32_t version;
  uint64_t n_tensor, n_kv;
  if (!r.get(magic, 4) || std::memcmp(magic, "GGUF", 4) != 0)
    return fail(MSB_ERR_INVALID, "gguf: %s: not a GGUF file (bad magic)", path.c_str());
  if (!r.val(version) || (version != 2 && version != 3))
    return fail(MSB_ERR_UNSUPPORTED, "gguf: %s: format version %u is not supported (2 or 3)",
                path.c_str(), version);
  if (!r.val(n_tensor) || !r.val(n_kv))
    return fail(MSB_ERR_INVALID, "gguf: %s: truncated header", path.c_str());
  // Every tensor record and key takes at least 8 bytes: bounds the counts.
  if (n_tensor > r.left() / 8 || n_kv > r.left() / 8)
    return fail(MSB_ERR_INVALID, "gguf: %s: implausible counts (%llu tensors, %llu keys)",
                path.c_str(), (unsigned long long)n_tensor, (unsigned long long)n_kv);
  uint64_t alignment = 32;
  for (uint64_t i = 0; i < n_kv; ++i) {
    Kv kv;
    if (!r.str(kv.key, 1u << 20) || !r.val(kv.type))
      return fail(MSB_ERR_INVALID, "gguf: %s: truncated key-value pair %llu", path.c_str(),
                  (unsigned long long)i);
    kv.ival = 0;
    if (is_int(kv.type)) {
      uint64_t sz;
      uint8_t b[8];
      fixed_size(kv.type, sz);
      if (!r.get(b, sz))
        return fail(MSB_ERR_INVALID, "gguf: %s: truncated value of %s", path.c_str(),
                    kv.key.c_str());
      kv.ival = int_of(kv.type, b);
    } else if (!skip_value(r, kv.type, 0)) {
      return fail(MSB_ERR_INVALID, "gguf: %s: bad value of %s (type %u)", path.c_str(),
                  kv.key.c_str(), kv.type);
    }
    if (kv.key == "general.alignment") {
      if (kv.type != kU32 || kv.ival <= 0 || (kv.ival & (kv.ival - 1)))
        return fail(MSB_ERR_INVALID, "gguf: %s: general.alignment must be a power of two",
                    path.c_str());
      alignment = uint64_t(kv.ival);
    }
    if (shard == 0) g->kvs.push_back(std::move(kv));
  }
  const size_t first = g->tensors.size();
  for (uint64_t i = 0; i < n_tensor; ++i) {
    Tensor t;
    uint32_t n_dims, type;
    if (!r.str(t.name, 1u << 16) || !r.val(n_dims))
      return fail(MSB_ERR_INVALID, "gguf: %s: truncated tensor record %llu", path.c_str(),
                  (unsigned long long)i);
    if (n_dims < 1 || n_dims > 4)
      return fail(MSB_ERR_INVALID, "gguf: %s: tensor %s has %u dimensions", path.c_str(),
                  t.name.c_str(), n_dims);
    t.n_dims = int(n_dims);
    for (int d = 0; d < 4; ++d) t.ne[d] = 1;
    for (uint32_t d = 0; d < n_dims; ++d) {
      uint64_t v;
      if (!r.val(v) || v > (uint64_t(1) << 40))
        return fail(MSB_ERR_INVALID, "gguf: %s: tensor %s: bad dimension", path.c_str(),
                    t.name.c_str());
      t.ne[d] = int64_t(v);
    }
    uint64_t off;
    if (!r.val(type) || !r.val(off))
      return fail(MSB_ERR_INVALID, "gguf: %s: truncated tensor record %s", path.c_str(),
                  t.name.c_str());
    t.type = int(type);
    const TypeSize ts = type_size(t.type);
    if (ts.blck == 0)
      return fail(MSB_ERR_UNSUPPORTED, "gguf: %s: tensor %s has unknown type %d", path.c_str(),
                  t.name.c_str(), t.type);
    if (t.ne[0] % ts.blck)
      return fail(MSB_ERR_INVALID, "gguf: %s: tensor %s: row of %lld is not whole blocks",
                  path.c_str(), t.name.c_str(), (long long)t.ne[0]);
    if (off % alignment)
      return fail(MSB_ERR_INVALID, "gguf: %s: tensor %s: offset %llu is not aligned to %llu",
                  path.c_str(), t.name.c_str(), (unsigned long long)off,
                  (unsigned long long)alignment);
    const unsigned __int128 nb = (unsigned __int128)(t.ne[0] / ts.blck) * ts.bytes * t.ne[1] *
                                 t.ne[2] * t.ne[3];
    if (nb > (unsigned __int128)(uint64_t(1) << 62))
      return fail(MSB_ERR_INVALID, "gguf: %s: tensor %s is too large", path.c_str(),
                  t.name.c_str());
    t.nbytes = int64_t(nb);
    t.offset = off;  // relative until the data section is known
    t.shard = shard;
    g->tensors.push_back(std::move(t));
  }
  const uint64_t data = (r.pos() + alignment - 1) / alignment * alignment;
  for (size_t i = first; i < g->tensors.size(); ++i) {
    Tensor &t = g->tensors[i];
    t.offset += data;
    if (t.offset < data || t.offset + uint64_t(t.nbytes) > g->sizes[size_t(shard)])
      return fail(MSB_ERR_INVALID,
                  "gguf: %s: tensor %s ends past the end of the file (needs %llu, size %llu)",
                  path.c_str(), t.name.c_str(),
                  (unsigned long long)(t.offset + uint64_t(t.nbytes)),
                  (unsigned long long)g->sizes[size_t(shard)]);
  }
  return MSB_OK;
}

const Kv *find_kv(const msb_gguf_s *g, const char *suffix) {
  const size_t sl = std::strlen(suffix);
  for (const Kv &kv : g->kvs)
    if (kv.key.size() >= sl && kv.key.compare(kv.key.size() - sl, sl, suffix) == 0)
      return &kv;
  return nullptr;
}

int64_t expert_bytes_of(const Tensor &t) { return t.nbytes / t.ne[2]; }

// Reads experts[i] of tensor t into dst[i] with up to n_threads threads.
int read_experts(const msb_gguf_s *g, const Tensor &t, int32_t n, const int32_t *experts,
                 void *const *dst, int32_t n_threads) {
  const uint64_t eb = uint64_t(expert_bytes_of(t));
  for (int32_t i = 0; i < n; ++i)
    if (experts[i] < 0 || experts[i] >= t.ne[2] || !dst[i])
      return fail(MSB_ERR_INVALID, "gguf: %s: expert %d of %lld (or a null destination)",
                  t.name.c_str(), experts[i], (long long)t.ne[2]);
  const int fd = g->fds[size_t(t.shard)];
  std::atomic<int32_t> next{0}, bad{-1};
  std::atomic<int> err{0};
  auto worker = [&] {
    for (;;) {
      const int32_t i = next.fetch_add(1);
      if (i >= n) return;
      uint8_t *d = static_cast<uint8_t *>(dst[i]);
      const uint64_t at = t.offset + uint64_t(experts[i]) * eb;
      uint64_t done = 0;
      while (done < eb) {
        const ssize_t r = pread(fd, d + done, eb - done, off_t(at + done));
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) {
          int32_t none = -1;
          bad.compare_exchange_strong(none, i);
          err.store(r < 0 ? errno : 0);
          return;
        }
        done += uint64_t(r);
      }
    }
  };
  const int nt = std::max(1, std::min<int>(n_threads, n));
  if (nt == 1) {
    worker();
  } else {
    std::vector<std::thread> th;
    th.reserve(size_t(nt));
    for (int i = 0; i < nt; ++i) th.emplace_back(worker);
    for (std::thread &x : th) x.join();
  }
  if (bad.load() >= 0) {
    const int e = err.load();
    return fail(MSB_ERR_IO, "gguf: %s: short read of expert %d from %s%s%s", t.name.c_str(),
                experts[bad.load()], g->paths[size_t(t.shard)].c_str(), e ? ": " : "",
                e ? std::strerror(e) : "");
  }
  return MSB_OK;
}

}  // namespace

extern "C" {

int msb_gguf_open(const char *path, msb_gguf_t *out) {
  MSB_CHECK_ARG(path && *path && out, "msb_gguf_open: null argument");
  *out = nullptr;
  msb_gguf_s *g = new (std::nothrow) msb_gguf_s();
  if (!g) return fail(MSB_ERR_NOMEM, "msb_gguf_open: out of memory");
  g->paths = shard_paths(path);
  for (const std::string &p : g->paths) {
    const int fd = open(p.c_str(), O_RDONLY | O_CLOEXEC);
    struct stat st;
    if (fd < 0 || fstat(fd, &st) != 0) {
      const int e = errno;
      if (fd >= 0) close(fd);
      const bool split = g->paths.size() > 1;
      const int rc = fail(MSB_ERR_IO, "gguf: cannot open %s%s: %s", p.c_str(),
                          split ? " (a split GGUF needs every shard)" : "", std::strerror(e));
      delete g;
      return rc;
    }
    g->fds.push_back(fd);
    g->sizes.push_back(uint64_t(st.st_size));
  }
  for (int32_t s = 0; s < int32_t(g->paths.size()); ++s) {
    const int rc = parse_shard(g, s);
    if (rc != MSB_OK) {
      delete g;
      return rc;
    }
  }
  const Kv *count = find_kv(g, "split.count");
  if (count && is_int(count->type) && count->ival > 1 &&
      count->ival != int64_t(g->paths.size())) {
    const std::string p = g->paths[0];
    const long long want = count->ival;
    delete g;
    return fail(MSB_ERR_INVALID,
                "gguf: %s is shard 1 of %lld; open it by its -00001-of-%05lld.gguf name",
                p.c_str(), want, want);
  }
  *out = g;
  return MSB_OK;
}

int msb_gguf_close(msb_gguf_t g) {
  delete g;
  return MSB_OK;
}

int32_t msb_gguf_shard_count(msb_gguf_t g) { return g ? int32_t(g->paths.size()) : 0; }

int64_t msb_gguf_tensor_count(msb_gguf_t g) { return g ? int64_t(g->tensors.size()) : 0; }

int msb_gguf_tensor_info(msb_gguf_t g, int64_t index, msb_gguf_tensor_t *out) {
  MSB_CHECK_ARG(g && out, "msb_gguf_tensor_info: null argument");
  MSB_CHECK_ARG(index >= 0 && index < int64_t(g->tensors.size()),
                "msb_gguf_tensor_info: index %lld of %zu", (long long)index, g->tensors.size());
  const Tensor &t = g->tensors[size_t(index)];
  out->name = t.name.c_str();
  out->type = t.type;
  out->n_dims = t.n_dims;
  for (int d = 0; d < 4; ++d) out->ne[d] = t.ne[d];
  out->shard = t.shard;
  out->offset = t.offset;
  out->nbytes = t.nbytes;
  return MSB_OK;
}

int64_t msb_gguf_find_tensor(msb_gguf_t g, const char *name) {
  if (!g || !name) return -1;
  for (size_t i = 0; i < g->tensors.size(); ++i)
    if (g->tensors[i].name == name) return int64_t(i);
  return -1;
}

int64_t msb_gguf_expert_tensor(msb_gguf_t g, int32_t layer, int role) {
  static const char *kRole[3] = {"gate", "up", "down"};
  if (!g || layer < 0 || role < 0 || role > 2) return -1;
  char name[64];
  std::snprintf(name, sizeof name, "blk.%d.ffn_%s_exps.weight", layer, kRole[role]);
  const int64_t i = msb_gguf_find_tensor(g, name);
  if (i < 0 || g->tensors[size_t(i)].n_dims != 3) return -1;
  return i;
}

int msb_gguf_kv_int(msb_gguf_t g, const char *key_suffix, int64_t *value) {
  MSB_CHECK_ARG(g && key_suffix && value, "msb_gguf_kv_int: null argument");
  const size_t sl = std::strlen(key_suffix);
  for (const Kv &kv : g->kvs) {
    if (kv.key.size() < sl || kv.key.compare(kv.key.size() - sl, sl, key_suffix) != 0) continue;
    if (!is_int(kv.type)) continue;
    *value = kv.ival;
    return MSB_OK;
  }
  return fail(MSB_ERR_INVALID, "gguf: no integer key ending in \"%s\"", key_suffix);
}

uint64_t msb_gguf_bytes_per_slot(msb_gguf_t g) {
  if (!g) return 0;
  uint64_t total = 0;
  for (const Tensor &t : g->tensors) {
    const char *nm = t.name.c_str();
    if (std::strncmp(nm, "blk.", 4) != 0 || t.ne[2] <= 1) continue;
    if (!std::strstr(nm, ".ffn_gate_exps.weight") && !std::strstr(nm, ".ffn_up_exps.weight") &&
        !std::strstr(nm, ".ffn_down_exps.weight"))
      continue;
    total += uint64_t(expert_bytes_of(t));
  }
  return total;
}

int msb_gguf_read_experts(msb_gguf_t g, int64_t tensor, int32_t n, const int32_t *experts,
                          void *const *dst_host, int32_t n_threads) {
  MSB_CHECK_ARG(g && n >= 0 && (n == 0 || (experts && dst_host)),
                "msb_gguf_read_experts: null argument");
  MSB_CHECK_ARG(tensor >= 0 && tensor < int64_t(g->tensors.size()),
                "msb_gguf_read_experts: tensor %lld of %zu", (long long)tensor,
                g->tensors.size());
  msb::clear_error();
  return n ? read_experts(g, g->tensors[size_t(tensor)], n, experts, dst_host, n_threads)
           : MSB_OK;
}

int msb_gguf_fill_slots_async(msb_gguf_t g, int64_t tensor, msb_pool_t pool, int32_t n,
                              const int32_t *experts, const int32_t *slots, int32_t n_threads,
                              void *stream) {
  MSB_CHECK_ARG(g && pool && n >= 0 && (n == 0 || (experts && slots)),
                "msb_gguf_fill_slots_async: null argument");
  MSB_CHECK_ARG(tensor >= 0 && tensor < int64_t(g->tensors.size()),
                "msb_gguf_fill_slots_async: tensor %lld of %zu", (long long)tensor,
                g->tensors.size());
  if (n == 0) return MSB_OK;
  const Tensor &t = g->tensors[size_t(tensor)];
  msb_pool_info_t info;
  int rc = msb_pool_get_info(pool, &info);
  if (rc != MSB_OK) return rc;
  if (t.n_dims != 3 || t.type != info.wtype || t.ne[0] != info.K || t.ne[1] != info.N)
    return fail(MSB_ERR_INVALID,
                "gguf: %s (type %d, %lld x %lld) does not match the pool (type %d, K %lld, N %lld)",
                t.name.c_str(), t.type, (long long)t.ne[0], (long long)t.ne[1], info.wtype,
                (long long)info.K, (long long)info.N);
  const size_t eb = size_t(expert_bytes_of(t));
  const size_t need = eb * size_t(n);
  msb_gguf_s::Stage &s = g->stage[g->next_stage];
  g->next_stage ^= 1;
  // The half about to be rewritten may still feed the copies of an earlier call.
  if (s.pending) {
    MSB_CUDA_TRY(cudaEventSynchronize(s.done));
    s.pending = false;
  }
  if (s.bytes < need) {
    if (s.host) cudaFreeHost(s.host);
    s.host = nullptr;
    s.bytes = 0;
    if (cudaHostAlloc(&s.host, need, cudaHostAllocPortable) != cudaSuccess) {
      s.host = nullptr;
      return fail(MSB_ERR_NOMEM, "gguf: pinned staging of %zu bytes failed", need);
    }
    s.bytes = need;
  }
  if (s.device != info.device) {
    if (s.done) cudaEventDestroy(s.done);
    s.done = nullptr;
    MSB_CUDA_TRY(cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming));
    s.device = info.device;
  }
  std::vector<void *> dst(static_cast<size_t>(n));
  for (int32_t i = 0; i < n; ++i) dst[size_t(i)] = s.host + size_t(i) * eb;
  msb::clear_error();
  rc = read_experts(g, t, n, experts, dst.data(), n_threads);
  if (rc != MSB_OK) return rc;
  rc = msb_fill_slots_async(pool, n, slots, dst.data(), stream);
  if (rc != MSB_OK) return rc;
  MSB_CUDA_TRY(cudaEventRecord(s.done, static_cast<cudaStream_t>(stream)));
  s.pending = true;
  return MSB_OK;
}

}  // extern "C"
