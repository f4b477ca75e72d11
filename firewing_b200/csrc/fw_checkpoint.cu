// fw_checkpoint.cu -- safetensors checkpoint loading for the block's weights
// (host code).
//
// A checkpoint is a directory holding model.safetensors.index.json (its
// "weight_map" names the shard file of every tensor) and the shards, or a
// single .safetensors file.  Shards are memory-mapped read-only and checked
// as the reference checks them (src/checkpoint_catalog.rs:146-253):
//   - at least 16 bytes; an 8-byte little-endian header length in
//     (0, 16 MiB] that fits in the file; the header a JSON object;
//   - "__metadata__", when present, an object;
//   - per tensor: a known dtype, a non-empty shape without zero dimensions,
//     two data offsets with end - start = the shape's byte count and end
//     within the payload; no duplicate names; no overlapping ranges.
// An index may only name shards by a single relative path component, every
// indexed tensor must be in its shard, and every shard tensor indexed
// (src/checkpoint_catalog.rs:356-393).  Tensors the block reads must be BF16
// with the shape the handle's configuration implies (src/expert.rs:362-512).
// The per-expert banks are read in place from the mapping: under expert
// parallelism only this rank's experts are copied to the device.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "fw_json.h"
#include "fw_kernels.h"
#include "fwmoe.h"

namespace {

using fw::json::Json;
using fw::json::JsonReader;
using fw::json::member;

// ---- shards --------------------------------------------------------------------

// Element size of a safetensors dtype (0: unknown), as the reference's
// dtype_bytes (src/checkpoint_catalog.rs:135-143).
size_t dtype_bytes(const std::string& t) {
  if (t == "BOOL" || t == "U8" || t == "I8" || t == "F8_E4M3" || t == "F8_E4M3FN" || t == "F8_E5M2") return 1;
  if (t == "U16" || t == "I16" || t == "F16" || t == "BF16") return 2;
  if (t == "U32" || t == "I32" || t == "F32") return 4;
  if (t == "U64" || t == "I64" || t == "F64") return 8;
  return 0;
}

struct TensorMeta {
  std::string dtype;
  std::vector<uint64_t> shape;
  uint64_t start = 0, end = 0;  // within the payload
};

class Shard {
 public:
  ~Shard() {
    if (map_ != nullptr) munmap(map_, size_);
  }
  // Map and validate `path`; false with a message in *err.
  bool open(const std::string& path, std::string* err) {
    const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0) {
      *err = path + ": cannot open";
      return false;
    }
    struct stat st;
    if (fstat(fd, &st) != 0) {
      ::close(fd);
      *err = path + ": cannot stat";
      return false;
    }
    size_ = static_cast<size_t>(st.st_size);
    if (size_ < 16) {
      ::close(fd);
      *err = path + " is too short";
      return false;
    }
    void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) {
      *err = path + ": cannot map";
      return false;
    }
    map_ = static_cast<unsigned char*>(m);
    uint64_t header = 0;
    for (int i = 7; i >= 0; --i) header = (header << 8) | map_[i];
    if (header == 0 || header > 16ull * 1024 * 1024 || 8 + header > size_) {
      *err = "invalid safetensors header in " + path;
      return false;
    }
    payload_ = 8 + header;
    Json root;
    std::string jerr;
    if (!JsonReader(reinterpret_cast<const char*>(map_ + 8), header).parse(&root, &jerr)) {
      *err = path + " header: " + jerr;
      return false;
    }
    if (root.kind != Json::Object) {
      *err = "safetensors header is not an object";
      return false;
    }
    const uint64_t payload_bytes = size_ - payload_;
    std::vector<std::pair<std::pair<uint64_t, uint64_t>, std::string>> ranges;
    for (const auto& kv : root.members) {
      const std::string& name = kv.first;
      const Json& item = kv.second;
      if (name == "__metadata__") {
        if (item.kind != Json::Object) {
          *err = "safetensors __metadata__ is not an object";
          return false;
        }
        continue;
      }
      if (item.kind != Json::Object) {
        *err = name + ": tensor entry is not an object";
        return false;
      }
      const Json* dt = member(item, "dtype");
      if (dt == nullptr || dt->kind != Json::String) {
        *err = name + ": missing dtype";
        return false;
      }
      const size_t eb = dtype_bytes(dt->s);
      if (eb == 0) {
        *err = name + ": unknown dtype";
        return false;
      }
      const Json* sh = member(item, "shape");
      if (sh == nullptr || sh->kind != Json::Array) {
        *err = name + ": missing shape";
        return false;
      }
      TensorMeta t;
      t.dtype = dt->s;
      uint64_t bytes = eb;
      for (const Json& d : sh->items) {
        if (d.kind != Json::Number || !d.is_uint) {
          *err = name + ": invalid shape";
          return false;
        }
        if (d.u == 0) {
          *err = name + ": empty shape";
          return false;
        }
        if (bytes > UINT64_MAX / d.u) {
          *err = "tensor size overflow";
          return false;
        }
        bytes *= d.u;
        t.shape.push_back(d.u);
      }
      if (t.shape.empty()) {
        *err = name + ": empty shape";
        return false;
      }
      const Json* off = member(item, "data_offsets");
      if (off == nullptr || off->kind != Json::Array) {
        *err = name + ": missing offsets";
        return false;
      }
      if (off->items.size() != 2) {
        *err = name + ": invalid offsets";
        return false;
      }
      const Json &s0 = off->items[0], &s1 = off->items[1];
      if (s0.kind != Json::Number || !s0.is_uint) {
        *err = name + ": invalid start";
        return false;
      }
      if (s1.kind != Json::Number || !s1.is_uint) {
        *err = name + ": invalid end";
        return false;
      }
      t.start = s0.u;
      t.end = s1.u;
      if (t.end < t.start || t.end - t.start != bytes || t.end > payload_bytes) {
        *err = name + ": payload layout mismatch";
        return false;
      }
      ranges.push_back({{t.start, t.end}, name});
      if (!tensors_.emplace(name, std::move(t)).second) {
        *err = "duplicate tensor " + name;
        return false;
      }
    }
    std::sort(ranges.begin(), ranges.end());
    uint64_t previous_end = 0;
    for (const auto& r : ranges) {
      if (r.first.first < previous_end) {
        *err = "overlapping tensor " + r.second;
        return false;
      }
      previous_end = r.first.second;
    }
    return true;
  }

  const TensorMeta* find(const std::string& name) const {
    const auto it = tensors_.find(name);
    return it == tensors_.end() ? nullptr : &it->second;
  }
  const std::map<std::string, TensorMeta>& tensors() const { return tensors_; }
  const unsigned char* payload(const TensorMeta& t) const { return map_ + payload_ + t.start; }

 private:
  unsigned char* map_ = nullptr;
  size_t size_ = 0;
  uint64_t payload_ = 0;
  std::map<std::string, TensorMeta> tensors_;
};

bool is_dir(const std::string& p) {
  struct stat st;
  return stat(p.c_str(), &st) == 0 && S_ISDIR(st.st_mode);
}

// One path component, not "." or ".." (the reference's safe_relative).
bool safe_relative(const std::string& name) {
  return !name.empty() && name.find('/') == std::string::npos && name != "." && name != "..";
}

bool read_file(const std::string& path, std::string* out) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (f == nullptr) return false;
  char buf[1 << 16];
  size_t n;
  while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) out->append(buf, n);
  const bool ok = std::ferror(f) == 0;
  std::fclose(f);
  return ok;
}

// A checkpoint: an index and its shards, or one file.
class Checkpoint {
 public:
  bool open(const std::string& path, std::string* err) {
    if (!is_dir(path)) {
      auto s = std::make_unique<Shard>();
      if (!s->open(path, err)) return false;
      for (const auto& kv : s->tensors()) weight_map_[kv.first] = "";
      shards_[""] = std::move(s);
      return true;
    }
    std::string text;
    const std::string index = path + "/model.safetensors.index.json";
    if (!read_file(index, &text)) {
      *err = index + ": cannot read";
      return false;
    }
    Json root;
    std::string jerr;
    if (!JsonReader(text.data(), text.size()).parse(&root, &jerr) || root.kind != Json::Object) {
      *err = "checkpoint index: " + (jerr.empty() ? std::string("not an object") : jerr);
      return false;
    }
    const Json* wm = member(root, "weight_map");
    if (wm == nullptr || wm->kind != Json::Object) {
      *err = "checkpoint index has no weight_map";
      return false;
    }
    for (const auto& kv : wm->members) {
      if (kv.second.kind != Json::String || !safe_relative(kv.second.s)) {
        *err = "unbound checkpoint shard: " + (kv.second.kind == Json::String ? kv.second.s : kv.first);
        return false;
      }
      weight_map_[kv.first] = kv.second.s;
    }
    for (const auto& kv : weight_map_) {
      if (shards_.count(kv.second)) continue;
      auto s = std::make_unique<Shard>();
      if (!s->open(path + "/" + kv.second, err)) return false;
      shards_[kv.second] = std::move(s);
    }
    for (const auto& kv : weight_map_)
      if (shards_[kv.second]->find(kv.first) == nullptr) {
        *err = "indexed tensor absent: " + kv.first;
        return false;
      }
    for (const auto& sh : shards_)
      for (const auto& t : sh.second->tensors()) {
        const auto it = weight_map_.find(t.first);
        if (it == weight_map_.end() || it->second != sh.first) {
          *err = "unindexed tensor in " + sh.first + ": " + t.first;
          return false;
        }
      }
    return true;
  }

  const TensorMeta* meta(const std::string& name) const {
    const auto it = weight_map_.find(name);
    return it == weight_map_.end() ? nullptr : shards_.at(it->second)->find(name);
  }

  // A BF16 tensor of exactly `shape`; its payload in the mapping.
  const uint16_t* bf16(const std::string& name, const std::vector<uint64_t>& shape, std::string* err) const {
    const auto it = weight_map_.find(name);
    if (it == weight_map_.end()) {
      *err = "tensor absent from checkpoint: " + name;
      return nullptr;
    }
    const Shard& s = *shards_.at(it->second);
    const TensorMeta* t = s.find(name);
    if (t->dtype != "BF16") {
      *err = name + ": expected BF16, got " + t->dtype;
      return nullptr;
    }
    if (t->shape != shape) {
      *err = name + ": shape mismatch";
      return nullptr;
    }
    const unsigned char* p = s.payload(*t);
    if ((reinterpret_cast<uintptr_t>(p) & 1u) != 0) {
      *err = name + ": BF16 payload is unaligned";
      return nullptr;
    }
    return reinterpret_cast<const uint16_t*>(p);
  }

 private:
  std::map<std::string, std::string> weight_map_;  // tensor -> shard file ("" for a single file)
  std::map<std::string, std::unique_ptr<Shard>> shards_;
};

thread_local char g_ckpt_msg[512];
int ckpt_fail(int code, const std::string& msg) {
  std::snprintf(g_ckpt_msg, sizeof g_ckpt_msg, "%s", msg.c_str());
  return fw::record_error(code, g_ckpt_msg);
}

}  // namespace

extern "C" {

int fw_safetensors_tensor_info(const char* file, const char* tensor, char dtype[16], int64_t shape[8],
                               int32_t* rank, uint64_t* offset, uint64_t* bytes) {
  if (file == nullptr || tensor == nullptr || dtype == nullptr || shape == nullptr || rank == nullptr ||
      offset == nullptr || bytes == nullptr)
    return ckpt_fail(FW_EINVAL, "null argument");
  Shard s;
  std::string err;
  if (!s.open(file, &err)) return ckpt_fail(FW_EINVAL, err);
  const TensorMeta* t = s.find(tensor);
  if (t == nullptr) return ckpt_fail(FW_EINVAL, std::string("tensor absent from shard: ") + tensor);
  if (t->shape.size() > 8) return ckpt_fail(FW_EINVAL, "tensor rank above 8");
  std::snprintf(dtype, 16, "%s", t->dtype.c_str());
  *rank = static_cast<int32_t>(t->shape.size());
  for (size_t i = 0; i < t->shape.size(); ++i) shape[i] = static_cast<int64_t>(t->shape[i]);
  *offset = t->start;
  *bytes = t->end - t->start;
  return FW_OK;
}

int fw_moe_load_layer_safetensors(fw_moe* h, int32_t layer, const char* checkpoint, const char* prefix) {
  if (h == nullptr || checkpoint == nullptr || prefix == nullptr) return ckpt_fail(FW_EINVAL, "null argument");
  fw_moe_config c{};
  if (int rc = fw_moe_get_config(h, &c); rc != FW_OK) return rc;
  Checkpoint ck;
  std::string err;
  if (!ck.open(checkpoint, &err)) return ckpt_fail(FW_EINVAL, err);
  const uint64_t E = c.experts, H = c.hidden, I = c.intermediate, Is = c.shared_intermediate;
  const std::string p(prefix);
  const uint16_t* router = ck.bf16(p + ".gate.weight", {E, H}, &err);
  const uint16_t* gate_up = router ? ck.bf16(p + ".experts.gate_up_proj", {E, 2 * I, H}, &err) : nullptr;
  const uint16_t* down = gate_up ? ck.bf16(p + ".experts.down_proj", {E, H, I}, &err) : nullptr;
  const uint16_t* sg = down ? ck.bf16(p + ".shared_expert.gate_proj.weight", {Is, H}, &err) : nullptr;
  const uint16_t* su = sg ? ck.bf16(p + ".shared_expert.up_proj.weight", {Is, H}, &err) : nullptr;
  const uint16_t* sd = su ? ck.bf16(p + ".shared_expert.down_proj.weight", {H, Is}, &err) : nullptr;
  const uint16_t* sgw = sd ? ck.bf16(p + ".shared_expert_gate.weight", {1, H}, &err) : nullptr;
  if (sgw == nullptr) return ckpt_fail(FW_EINVAL, err);
  return fw_moe_load_layer(h, layer, router, gate_up, down, sg, su, sd, sgw, nullptr);
}

int fw_moe_load_hc_safetensors(fw_moe* h, int32_t layer, const char* checkpoint, const char* prefix) {
  if (h == nullptr || checkpoint == nullptr || prefix == nullptr) return ckpt_fail(FW_EINVAL, "null argument");
  fw_moe_config c{};
  if (int rc = fw_moe_get_config(h, &c); rc != FW_OK) return rc;
  Checkpoint ck;
  std::string err;
  if (!ck.open(checkpoint, &err)) return ckpt_fail(FW_EINVAL, err);
  const uint64_t HH = 4ull * c.hidden;
  const std::string p(prefix);
  // The low rank comes from the checkpoint: input_mix_weight_down is [LR][4H].
  const TensorMeta* md = ck.meta(p + ".input_mix_weight_down.weight");
  if (md == nullptr || md->shape.size() != 2)
    return ckpt_fail(FW_EINVAL, p + ".input_mix_weight_down.weight: absent or not two-dimensional");
  const uint64_t lowrank = md->shape[0];
  const uint16_t* norm = ck.bf16(p + ".hc_norm.weight", {HH}, &err);
  const uint16_t* down = norm ? ck.bf16(p + ".input_mix_weight_down.weight", {lowrank, HH}, &err) : nullptr;
  const uint16_t* up = down ? ck.bf16(p + ".input_mix_weight_up.weight", {HH, lowrank}, &err) : nullptr;
  const uint16_t* inject = up ? ck.bf16(p + ".block_inject_weight.weight", {4, HH}, &err) : nullptr;
  if (inject == nullptr) return ckpt_fail(FW_EINVAL, err);
  return fw_moe_load_hc(h, layer, static_cast<int32_t>(lowrank), norm, down, up, inject);
}

}  // extern "C"
