// fw_codec.cu -- compressed expert containers (the reference's storage
// format for streamed experts: tools/build_sequential_shuffle_container.py,
// read by src/compressed_overlap.rs).
//
// A container file holds one independent zstd frame per (layer, expert),
// each at a page-aligned offset; a JSON manifest lists the records:
//   {layer, expert, offset, compressed_bytes, physical_bytes, frame_sha256,
//    source_sha256}
// with "exact_transform": "bf16_even_bytes_then_odd_bytes_per_expert" (the
// frame decompresses to the expert's gate_up then down bytes, byte-shuffled:
// every even byte of the source, then every odd byte), "codec" zstandard,
// "source_bytes_per_expert", "page_bytes" and "container_file".
//
// Loading splits the work where it runs best: the host decompresses the
// frames (libzstd, loaded at run time; several experts at once on worker
// threads) and checks the SHA-256 of frame and source when asked; the GPU
// un-shuffles the bytes (k_unshuffle_bf16, HBM-bound byte interleave) and
// the tiled re-layout places the expert in the layer's bank
// (fw_moe_load_expert).
#include <dlfcn.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include <cuda_runtime.h>

#include "fw_json.h"
#include "fw_kernels.h"
#include "fwmoe.h"

namespace {

using fw::json::Json;
using fw::json::JsonReader;
using fw::json::member;

// ---- SHA-256 (FIPS 180-4) --------------------------------------------------------

constexpr uint32_t kSha256K[64] = {
    0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
    0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
    0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
    0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
    0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
    0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
    0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
    0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};

class Sha256 {
 public:
  Sha256() {
    static const uint32_t h0[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                                   0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
    std::memcpy(h_, h0, sizeof h_);
  }
  void update(const uint8_t* p, size_t n) {
    bits_ += static_cast<uint64_t>(n) * 8;
    if (fill_ > 0) {
      const size_t take = std::min(n, 64 - fill_);
      std::memcpy(buf_ + fill_, p, take);
      fill_ += take;
      p += take;
      n -= take;
      if (fill_ < 64) return;
      block(buf_);
      fill_ = 0;
    }
    for (; n >= 64; p += 64, n -= 64) block(p);
    std::memcpy(buf_, p, n);
    fill_ = n;
  }
  std::string hex() {
    const uint64_t bits = bits_;
    const uint8_t one = 0x80, zero = 0;
    update(&one, 1);
    while (fill_ != 56) update(&zero, 1);
    uint8_t len[8];
    for (int i = 0; i < 8; ++i) len[i] = static_cast<uint8_t>(bits >> (56 - 8 * i));
    update(len, 8);
    char out[65];
    for (int i = 0; i < 8; ++i) std::snprintf(out + 8 * i, 9, "%08x", h_[i]);
    return std::string(out, 64);
  }

 private:
  uint32_t h_[8];
  uint8_t buf_[64];
  size_t fill_ = 0;
  uint64_t bits_ = 0;

  static uint32_t rotr(uint32_t x, int r) { return (x >> r) | (x << (32 - r)); }
  void block(const uint8_t* p) {
    uint32_t w[64];
    for (int i = 0; i < 16; ++i)
      w[i] = (static_cast<uint32_t>(p[4 * i]) << 24) | (static_cast<uint32_t>(p[4 * i + 1]) << 16) |
             (static_cast<uint32_t>(p[4 * i + 2]) << 8) | p[4 * i + 3];
    for (int i = 16; i < 64; ++i) {
      const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
      const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h_[0], b = h_[1], c = h_[2], d = h_[3], e = h_[4], f = h_[5], g = h_[6], h = h_[7];
    for (int i = 0; i < 64; ++i) {
      const uint32_t t1 = h + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + kSha256K[i] + w[i];
      const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
      h = g;
      g = f;
      f = e;
      e = d + t1;
      d = c;
      c = b;
      b = a;
      a = t1 + t2;
    }
    h_[0] += a;
    h_[1] += b;
    h_[2] += c;
    h_[3] += d;
    h_[4] += e;
    h_[5] += f;
    h_[6] += g;
    h_[7] += h;
  }
};

std::string sha256_hex(const uint8_t* p, size_t n) {
  Sha256 s;
  s.update(p, n);
  return s.hex();
}

// SHA-256 of the un-shuffled source, fed straight from the shuffled bytes
// (source byte 2i = shuffled[i], byte 2i+1 = shuffled[n/2 + i]).
std::string sha256_unshuffled(const uint8_t* shuffled, size_t n) {
  Sha256 s;
  const size_t half = n / 2;
  uint8_t buf[4096];
  for (size_t i = 0; i < half;) {
    const size_t m = std::min(half - i, sizeof buf / 2);
    for (size_t j = 0; j < m; ++j) {
      buf[2 * j] = shuffled[i + j];
      buf[2 * j + 1] = shuffled[half + i + j];
    }
    s.update(buf, 2 * m);
    i += m;
  }
  return s.hex();
}

// ---- libzstd (loaded at run time) ------------------------------------------------

struct ZstdApi {
  bool ok = false;
  char why[160] = {};
  size_t (*decompress)(void*, size_t, const void*, size_t) = nullptr;
  unsigned (*is_error)(size_t) = nullptr;
  const char* (*error_name)(size_t) = nullptr;
  unsigned long long (*frame_content_size)(const void*, size_t) = nullptr;
};

const ZstdApi& zstd() {
  static ZstdApi z;
  static std::once_flag once;
  std::call_once(once, [] {
    void* lib = dlopen("libzstd.so.1", RTLD_NOW | RTLD_LOCAL);
    if (lib == nullptr) {
      std::snprintf(z.why, sizeof z.why, "libzstd.so.1 not loadable: %s", dlerror());
      return;
    }
    z.decompress = reinterpret_cast<decltype(z.decompress)>(dlsym(lib, "ZSTD_decompress"));
    z.is_error = reinterpret_cast<decltype(z.is_error)>(dlsym(lib, "ZSTD_isError"));
    z.error_name = reinterpret_cast<decltype(z.error_name)>(dlsym(lib, "ZSTD_getErrorName"));
    z.frame_content_size =
        reinterpret_cast<decltype(z.frame_content_size)>(dlsym(lib, "ZSTD_getFrameContentSize"));
    if (!z.decompress || !z.is_error || !z.error_name || !z.frame_content_size) {
      std::snprintf(z.why, sizeof z.why, "libzstd.so.1 lacks an entry point this library needs");
      return;
    }
    z.ok = true;
  });
  return z;
}

// ---- manifest and container ------------------------------------------------------

struct Record {
  int layer = 0, expert = 0;
  uint64_t offset = 0, compressed = 0, physical = 0;
  std::string frame_sha256, source_sha256;
};

bool read_text(const std::string& path, std::string* out) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (f == nullptr) return false;
  char buf[1 << 16];
  size_t n;
  while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) out->append(buf, n);
  const bool ok = std::ferror(f) == 0;
  std::fclose(f);
  return ok;
}

bool is_hex64(const std::string& s) {
  if (s.size() != 64) return false;
  for (char c : s)
    if (!((c >= '0' && c <= '9') || (c >= 'a' && c <= 'f'))) return false;
  return true;
}

bool get_uint(const Json& o, const char* key, uint64_t* v) {
  const Json* m = member(o, key);
  if (m == nullptr || m->kind != Json::Number || !m->is_uint) return false;
  *v = m->u;
  return true;
}

class Container {
 public:
  ~Container() {
    if (map_ != nullptr) munmap(map_, size_);
  }
  // Parse and check the manifest, map the container file.
  bool open(const std::string& manifest_path, uint64_t source_bytes, std::string* err) {
    std::string text;
    if (!read_text(manifest_path, &text)) {
      *err = manifest_path + ": cannot read";
      return false;
    }
    Json root;
    std::string jerr;
    if (!JsonReader(text.data(), text.size()).parse(&root, &jerr) || root.kind != Json::Object) {
      *err = "codec manifest: " + (jerr.empty() ? std::string("not an object") : jerr);
      return false;
    }
    const Json* tr = member(root, "exact_transform");
    if (tr == nullptr || tr->kind != Json::String || tr->s != "bf16_even_bytes_then_odd_bytes_per_expert") {
      *err = "codec manifest: unsupported exact_transform";
      return false;
    }
    const Json* codec = member(root, "codec");
    const Json* name = codec != nullptr && codec->kind == Json::Object ? member(*codec, "name") : nullptr;
    if (name == nullptr || name->kind != Json::String || name->s != "zstandard") {
      *err = "codec manifest: unsupported codec";
      return false;
    }
    uint64_t per = 0, page = 0;
    if (!get_uint(root, "source_bytes_per_expert", &per) || per != source_bytes) {
      *err = "codec manifest: source_bytes_per_expert does not match the block's expert size";
      return false;
    }
    if (!get_uint(root, "page_bytes", &page) || page == 0) {
      *err = "codec manifest: invalid page_bytes";
      return false;
    }
    source_bytes_ = per;
    const Json* file = member(root, "container_file");
    if (file == nullptr || file->kind != Json::String || file->s.empty() || file->s.find('/') != std::string::npos ||
        file->s == "." || file->s == "..") {
      *err = "codec manifest: container_file must be one path component";
      return false;
    }
    const size_t slash = manifest_path.rfind('/');
    const std::string dir = slash == std::string::npos ? std::string(".") : manifest_path.substr(0, slash);
    const std::string path = dir + "/" + file->s;
    const Json* recs = member(root, "records");
    if (recs == nullptr || recs->kind != Json::Array) {
      *err = "codec manifest: records missing";
      return false;
    }
    const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0) {
      *err = path + ": cannot open";
      return false;
    }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size <= 0) {
      ::close(fd);
      *err = path + ": cannot stat or empty";
      return false;
    }
    size_ = static_cast<size_t>(st.st_size);
    void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) {
      *err = path + ": cannot map";
      return false;
    }
    map_ = static_cast<unsigned char*>(m);
    for (const Json& r : recs->items) {
      Record rec;
      uint64_t layer = 0, expert = 0;
      const Json* fh = r.kind == Json::Object ? member(r, "frame_sha256") : nullptr;
      const Json* sh = r.kind == Json::Object ? member(r, "source_sha256") : nullptr;
      if (r.kind != Json::Object || !get_uint(r, "layer", &layer) || !get_uint(r, "expert", &expert) ||
          !get_uint(r, "offset", &rec.offset) || !get_uint(r, "compressed_bytes", &rec.compressed) ||
          !get_uint(r, "physical_bytes", &rec.physical) || fh == nullptr || fh->kind != Json::String ||
          !is_hex64(fh->s) || sh == nullptr || sh->kind != Json::String || !is_hex64(sh->s) || layer > 1u << 20 ||
          expert > 1u << 20) {
        *err = "codec manifest: invalid record";
        return false;
      }
      rec.layer = static_cast<int>(layer);
      rec.expert = static_cast<int>(expert);
      rec.frame_sha256 = fh->s;
      rec.source_sha256 = sh->s;
      if (rec.compressed == 0 || rec.physical < rec.compressed || rec.offset % page != 0 || rec.physical % page != 0 ||
          rec.offset > size_ || rec.physical > size_ - rec.offset) {
        *err = "codec record " + std::to_string(rec.layer) + ":" + std::to_string(rec.expert) +
               ": frame outside the container or not page-aligned";
        return false;
      }
      records_.push_back(rec);
    }
    return true;
  }

  const std::vector<Record>& records() const { return records_; }
  uint64_t source_bytes() const { return source_bytes_; }

  // Decompress one record into out (source_bytes); checks the frame and,
  // when `verify`, both hashes.  Thread-safe.
  bool decode(const Record& r, bool verify, uint8_t* out, std::string* err) const {
    const ZstdApi& z = zstd();
    if (!z.ok) {
      *err = z.why;
      return false;
    }
    const uint8_t* frame = map_ + r.offset;
    const std::string id = std::to_string(r.layer) + ":" + std::to_string(r.expert);
    if (verify && sha256_hex(frame, r.compressed) != r.frame_sha256) {
      *err = "codec record " + id + ": frame hash mismatch";
      return false;
    }
    if (z.frame_content_size(frame, r.compressed) != source_bytes_) {
      *err = "codec record " + id + ": frame content size is not the expert size";
      return false;
    }
    const size_t n = z.decompress(out, source_bytes_, frame, r.compressed);
    if (z.is_error(n) || n != source_bytes_) {
      *err = "codec record " + id + ": " + (z.is_error(n) ? z.error_name(n) : "short frame");
      return false;
    }
    if (verify && sha256_unshuffled(out, n) != r.source_sha256) {
      *err = "codec record " + id + ": source hash mismatch";
      return false;
    }
    return true;
  }

 private:
  unsigned char* map_ = nullptr;
  size_t size_ = 0;
  uint64_t source_bytes_ = 0;
  std::vector<Record> records_;
};

// Records of `layer` (all when layer < 0), decoded `threads` at a time;
// `consume(record, bytes)` runs on the calling thread in record order.
template <typename Consume>
bool decode_records(const Container& c, int layer, bool verify, std::string* err, Consume consume) {
  std::vector<const Record*> todo;
  for (const Record& r : c.records())
    if (layer < 0 || r.layer == layer) todo.push_back(&r);
  const size_t hw = std::max(1u, std::thread::hardware_concurrency());
  const size_t threads = std::min<size_t>(std::min<size_t>(hw, 16), std::max<size_t>(todo.size(), 1));
  std::vector<std::vector<uint8_t>> bufs(threads, std::vector<uint8_t>(c.source_bytes()));
  for (size_t b = 0; b < todo.size(); b += threads) {
    const size_t n = std::min(threads, todo.size() - b);
    std::vector<std::string> errs(n);
    std::vector<char> ok(n, 0);
    std::vector<std::thread> pool;
    for (size_t i = 0; i < n; ++i)
      pool.emplace_back([&, i] { ok[i] = c.decode(*todo[b + i], verify, bufs[i].data(), &errs[i]) ? 1 : 0; });
    for (auto& t : pool) t.join();
    for (size_t i = 0; i < n; ++i) {
      if (!ok[i]) {
        *err = errs[i];
        return false;
      }
      if (!consume(*todo[b + i], bufs[i].data())) return false;
    }
  }
  return true;
}

thread_local char g_codec_msg[512];
int codec_fail(int code, const std::string& msg) {
  std::snprintf(g_codec_msg, sizeof g_codec_msg, "%s", msg.c_str());
  return fw::record_error(code, g_codec_msg);
}

// out[i] = bf16 with low byte in[i] and high byte in[n + i] (n elements):
// 16 elements per step, two 16-byte loads and two 16-byte stores.
__global__ void k_unshuffle_bf16(const uint8_t* in, long long n, uint16_t* out) {
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long i0 = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if ((n & 15) == 0) {
    for (long long v = i0; v < n / 16; v += stride) {
      const uint4 lo = *reinterpret_cast<const uint4*>(in + 16 * v);
      const uint4 hi = *reinterpret_cast<const uint4*>(in + n + 16 * v);
      const uint32_t l[4] = {lo.x, lo.y, lo.z, lo.w}, h[4] = {hi.x, hi.y, hi.z, hi.w};
      uint32_t o[8];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        o[2 * q] = __byte_perm(l[q], h[q], 0x5140);      // lo0 hi0 lo1 hi1
        o[2 * q + 1] = __byte_perm(l[q], h[q], 0x7362);  // lo2 hi2 lo3 hi3
      }
      uint4* dst = reinterpret_cast<uint4*>(out + 16 * v);
      dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
      dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
    }
    return;
  }
  for (long long i = i0; i < n; i += stride)
    out[i] = static_cast<uint16_t>(in[i] | (static_cast<uint16_t>(in[n + i]) << 8));
}

}  // namespace

extern "C" {

int fw_codec_container_check(const char* manifest, int32_t layer, uint64_t source_bytes_per_expert,
                             int32_t verify, int32_t* records) {
  if (manifest == nullptr || records == nullptr) return codec_fail(FW_EINVAL, "null argument");
  Container c;
  std::string err;
  if (!c.open(manifest, source_bytes_per_expert, &err)) return codec_fail(FW_EINVAL, err);
  int count = 0;
  if (!decode_records(c, layer, verify != 0, &err, [&](const Record&, const uint8_t*) {
        ++count;
        return true;
      }))
    return codec_fail(FW_EINVAL, err);
  *records = count;
  return FW_OK;
}

int fw_moe_load_expert_container(fw_moe* h, int32_t layer, const char* manifest, int32_t container_layer,
                                 int32_t verify, int32_t* loaded) {
  if (h == nullptr || manifest == nullptr || loaded == nullptr) return codec_fail(FW_EINVAL, "null argument");
  fw_moe_config cfg{};
  if (int rc = fw_moe_get_config(h, &cfg); rc != FW_OK) return rc;
  const uint64_t I = cfg.intermediate, H = cfg.hidden;
  const uint64_t source = 3 * H * I * 2;  // gate_up [2I][H] then down [H][I], bf16
  Container c;
  std::string err;
  if (!c.open(manifest, source, &err)) return codec_fail(FW_EINVAL, err);
  const fw::HandlePlace ep = fw::handle_place(h);
  if (cudaSetDevice(ep.device) != cudaSuccess) return codec_fail(FW_ECUDA, "cudaSetDevice");
  uint8_t* d_shuffled = nullptr;
  uint16_t* d_expert = nullptr;
  if (cudaMalloc(&d_shuffled, source) != cudaSuccess || cudaMalloc(&d_expert, source) != cudaSuccess) {
    cudaFree(d_shuffled);
    return codec_fail(FW_ENOMEM, "codec staging buffers");
  }
  int count = 0, rc = FW_OK;
  const bool ok = decode_records(c, container_layer, verify != 0, &err, [&](const Record& r, const uint8_t* bytes) {
    if (r.expert >= cfg.experts) {
      err = "codec record expert " + std::to_string(r.expert) + " out of range";
      return false;
    }
    if (r.expert % ep.world != ep.rank) return true;  // held by another rank
    // copy and un-shuffle in order on one stream, complete before the load
    cudaError_t e = cudaMemcpyAsync(d_shuffled, bytes, source, cudaMemcpyHostToDevice, cudaStreamLegacy);
    if (e == cudaSuccess) {
      const long long n = static_cast<long long>(source / 2);
      k_unshuffle_bf16<<<148 * 4, 256, 0, cudaStreamLegacy>>>(d_shuffled, n, d_expert);
      e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(cudaStreamLegacy);
    if (e != cudaSuccess) {
      err = std::string("codec un-shuffle: ") + cudaGetErrorString(e);
      rc = FW_ECUDA;
      return false;
    }
    const int lrc = fw_moe_load_expert(h, layer, r.expert, d_expert, d_expert + 2 * I * H);
    if (lrc != FW_OK) {
      err = fw_last_error();
      rc = lrc;
      return false;
    }
    ++count;
    return true;
  });
  cudaFree(d_shuffled);
  cudaFree(d_expert);
  if (!ok) return codec_fail(rc != FW_OK ? rc : FW_EINVAL, err);
  *loaded = count;
  return FW_OK;
}

}  // extern "C"
