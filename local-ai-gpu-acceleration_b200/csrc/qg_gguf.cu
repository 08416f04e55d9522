// qg_gguf.cu -- GGUF header and tensor-table reader (host code): the ingest side of the
// resident packs.  Follows the reference's probe (runtime/apps/gguf_probe/main.cpp:124-631):
// magic "GGUF", version, tensor and metadata counts, metadata key/value pairs (typed
// values and arrays skipped; general.alignment and general.architecture kept), tensor
// infos (name, dims, ggml type, offset relative to the data section), data section at the
// end of the tensor infos aligned up to general.alignment (default 32), tensor spans from
// the sorted offsets, and the same validation: a supported type, a block-aligned element
// count, a span that holds the expected bytes with padding below the alignment.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <new>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/qgemv_b200.h"

namespace {

struct BlockType {
  uint64_t block_size, type_size;
  const char* name;
};

// ggml type ids of the probe's table (gguf_probe/main.cpp:196-207).
const std::unordered_map<uint32_t, BlockType>& block_types() {
  static const std::unordered_map<uint32_t, BlockType> t = {
      {0u, {1u, 4u, "F32"}},     {1u, {1u, 2u, "F16"}},      {8u, {32u, 34u, "Q8_0"}},
      {12u, {256u, 144u, "Q4_K"}}, {13u, {256u, 176u, "Q5_K"}}, {21u, {256u, 110u, "IQ3_S"}},
      {22u, {256u, 82u, "IQ2_S"}},
  };
  return t;
}

struct Tensor {
  std::string name;
  std::vector<uint64_t> dims;
  uint32_t type = 0;
  uint64_t offset = 0;
  uint64_t span = 0;
  uint64_t expected = 0;
  bool valid = false;
};

class Reader {
 public:
  explicit Reader(FILE* f) : f_(f) {}
  bool ok() const { return ok_; }
  template <typename T>
  T pod() {
    T v{};
    if (ok_ && std::fread(&v, sizeof(T), 1, f_) != 1) ok_ = false;
    return v;
  }
  std::string str() {
    const uint64_t n = pod<uint64_t>();
    if (!ok_ || n > (1ull << 30)) {
      ok_ = false;
      return {};
    }
    std::string s(n, '\0');
    if (n > 0 && std::fread(s.data(), 1, n, f_) != n) ok_ = false;
    return s;
  }
  void skip(uint64_t n) {
    if (ok_ && std::fseek(f_, static_cast<long>(n), SEEK_CUR) != 0) ok_ = false;
  }
  // metadata value types (gguf_probe/main.cpp:22-36)
  void skip_value(uint32_t type, int depth = 0) {
    switch (type) {
      case 0: case 1: case 7: skip(1); break;
      case 2: case 3: skip(2); break;
      case 4: case 5: case 6: skip(4); break;
      case 10: case 11: case 12: skip(8); break;
      case 8: (void)str(); break;
      case 9: {
        const uint32_t item = pod<uint32_t>();
        const uint64_t n = pod<uint64_t>();
        if (depth > 4) {
          ok_ = false;
          break;
        }
        for (uint64_t i = 0; i < n && ok_; ++i) skip_value(item, depth + 1);
        break;
      }
      default: ok_ = false;
    }
  }
  uint64_t tell() const { return static_cast<uint64_t>(std::ftell(f_)); }

 private:
  FILE* f_;
  bool ok_ = true;
};

}  // namespace

struct qg_gguf_s {
  FILE* file = nullptr;
  uint32_t version = 0;
  uint64_t metadata_count = 0;
  uint64_t info_end = 0;
  uint64_t data_offset = 0;
  uint64_t alignment = 32;
  uint64_t file_size = 0;
  std::string architecture;
  std::vector<Tensor> tensors;  // in file order of the tensor infos
};

extern "C" {

cudaError_t qg_gguf_open(const char* path, qg_gguf* out) {
  if (path == nullptr || out == nullptr) return cudaErrorInvalidValue;
  *out = nullptr;
  FILE* f = std::fopen(path, "rb");
  if (f == nullptr) return cudaErrorFileNotFound;
  auto* g = new (std::nothrow) qg_gguf_s();
  if (g == nullptr) {
    std::fclose(f);
    return cudaErrorMemoryAllocation;
  }
  g->file = f;
  std::fseek(f, 0, SEEK_END);
  g->file_size = static_cast<uint64_t>(std::ftell(f));
  std::fseek(f, 0, SEEK_SET);
  Reader in(f);
  char magic[4] = {};
  const bool magic_ok = std::fread(magic, 1, 4, f) == 4 && std::memcmp(magic, "GGUF", 4) == 0;
  g->version = in.pod<uint32_t>();
  const uint64_t tensor_count = in.pod<uint64_t>();
  g->metadata_count = in.pod<uint64_t>();
  if (!magic_ok || !in.ok() || tensor_count > (1ull << 24)) {
    qg_gguf_close(g);
    return cudaErrorInvalidValue;
  }
  for (uint64_t i = 0; i < g->metadata_count && in.ok(); ++i) {
    const std::string key = in.str();
    const uint32_t type = in.pod<uint32_t>();
    if (key == "general.alignment" && type == 4u) {
      g->alignment = in.pod<uint32_t>();
    } else if (key == "general.architecture" && type == 8u) {
      g->architecture = in.str();
    } else {
      in.skip_value(type);
    }
  }
  g->tensors.resize(tensor_count);
  for (uint64_t i = 0; i < tensor_count && in.ok(); ++i) {
    Tensor& t = g->tensors[i];
    t.name = in.str();
    const uint32_t n_dims = in.pod<uint32_t>();
    if (n_dims > 8u) {
      qg_gguf_close(g);
      return cudaErrorInvalidValue;
    }
    for (uint32_t d = 0; d < n_dims; ++d) t.dims.push_back(in.pod<uint64_t>());
    t.type = in.pod<uint32_t>();
    t.offset = in.pod<uint64_t>();
  }
  if (!in.ok() || g->alignment == 0u) {
    qg_gguf_close(g);
    return cudaErrorInvalidValue;
  }
  g->info_end = in.tell();
  g->data_offset = (g->info_end + g->alignment - 1u) / g->alignment * g->alignment;
  // spans from the offsets in ascending order; the last runs to the end of the file
  std::vector<size_t> order(tensor_count);
  for (size_t i = 0; i < order.size(); ++i) order[i] = i;
  std::sort(order.begin(), order.end(),
            [&](size_t a, size_t b) { return g->tensors[a].offset < g->tensors[b].offset; });
  const uint64_t data_bytes = g->file_size > g->data_offset ? g->file_size - g->data_offset : 0u;
  for (size_t k = 0; k < order.size(); ++k) {
    Tensor& t = g->tensors[order[k]];
    const uint64_t next = k + 1 < order.size() ? g->tensors[order[k + 1]].offset : data_bytes;
    t.span = next >= t.offset ? next - t.offset : 0u;
    const auto it = block_types().find(t.type);
    uint64_t elements = 1;
    for (const uint64_t d : t.dims) elements *= d;
    if (it == block_types().end() || elements % it->second.block_size != 0u) continue;
    t.expected = elements / it->second.block_size * it->second.type_size;
    t.valid = t.span >= t.expected && t.span - t.expected < g->alignment;
  }
  *out = g;
  return cudaSuccess;
}

cudaError_t qg_gguf_summary(qg_gguf g, qg_gguf_info* info) {
  if (g == nullptr || info == nullptr) return cudaErrorInvalidValue;
  std::memset(info, 0, sizeof(*info));
  info->version = g->version;
  info->tensor_count = g->tensors.size();
  info->metadata_count = g->metadata_count;
  info->tensor_info_end_offset = g->info_end;
  info->tensor_data_offset = g->data_offset;
  info->tensor_data_alignment = g->alignment;
  for (const Tensor& t : g->tensors) {
    if (block_types().count(t.type) != 0u) ++info->supported_tensors;
    if (t.valid) ++info->valid_tensors;
    info->expected_data_bytes += t.expected;
  }
  std::snprintf(info->architecture, sizeof(info->architecture), "%s", g->architecture.c_str());
  return cudaSuccess;
}

cudaError_t qg_gguf_tensor(qg_gguf g, uint64_t index, qg_gguf_tensor_info* out) {
  if (g == nullptr || out == nullptr || index >= g->tensors.size()) return cudaErrorInvalidValue;
  const Tensor& t = g->tensors[index];
  std::memset(out, 0, sizeof(*out));
  std::snprintf(out->name, sizeof(out->name), "%s", t.name.c_str());
  out->ggml_type = t.type;
  out->n_dims = static_cast<uint32_t>(std::min<size_t>(t.dims.size(), 4));
  for (uint32_t d = 0; d < out->n_dims; ++d) out->dims[d] = t.dims[d];
  out->offset = t.offset;
  out->absolute_offset = g->data_offset + t.offset;
  out->span_bytes = t.span;
  out->data_bytes = t.expected;
  out->valid = t.valid ? 1u : 0u;
  const auto it = block_types().find(t.type);
  if (it != block_types().end()) {
    out->block_size = static_cast<uint32_t>(it->second.block_size);
    out->type_size = static_cast<uint32_t>(it->second.type_size);
  }
  return cudaSuccess;
}

cudaError_t qg_gguf_find(qg_gguf g, const char* name, uint64_t* index) {
  if (g == nullptr || name == nullptr || index == nullptr) return cudaErrorInvalidValue;
  for (size_t i = 0; i < g->tensors.size(); ++i) {
    if (g->tensors[i].name == name) {
      *index = i;
      return cudaSuccess;
    }
  }
  return cudaErrorInvalidSymbol;
}

cudaError_t qg_gguf_read(qg_gguf g, uint64_t index, void* dst, uint64_t bytes) {
  if (g == nullptr || dst == nullptr || index >= g->tensors.size()) return cudaErrorInvalidValue;
  const Tensor& t = g->tensors[index];
  if (!t.valid || bytes != t.expected) return cudaErrorInvalidValue;
  if (std::fseek(g->file, static_cast<long>(g->data_offset + t.offset), SEEK_SET) != 0 ||
      std::fread(dst, 1, bytes, g->file) != bytes) {
    return cudaErrorUnknown;
  }
  return cudaSuccess;
}

cudaError_t qg_gguf_close(qg_gguf g) {
  if (g == nullptr) return cudaSuccess;
  if (g->file != nullptr) std::fclose(g->file);
  delete g;
  return cudaSuccess;
}

}  // extern "C"
