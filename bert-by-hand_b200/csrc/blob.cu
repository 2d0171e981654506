// Single-file weight blob: the reference ships one fp16 file per tensor
// (scripts/dump_weights.py:69-94 writes weights/<HF key>.bin; src/model/weights.h:88-107
// opens them one by one). This packs them into one file that loads with one read and one
// host->device copy, and checks what it loads.
//
// Layout (little-endian):
//   0   char[4]  "BBHW"
//   4   u32      version (1)
//   8   u32      layers
//   12  u32      tensor count (= bbh_num_tensors(layers))
//   16  u64      data offset (4096-aligned)
//   24  u64      data bytes
//   32  u64      FNV-1a 64 of the data bytes
//   40  per tensor: u32 name length, name bytes, u64 numel, u64 offset from the data start
//       (256-byte aligned), in the catalogue order of bbh_tensor_name()
//   data: fp16 tensors, nn.Linear (out, in) row-major, as in the per-tensor files.
#include "internal.h"
#include "../../include/bbh.h"

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

namespace {

constexpr char kMagic[4] = {'B', 'B', 'H', 'W'};
constexpr uint32_t kVersion = 1;

uint64_t fnv1a(const uint8_t* p, size_t n) {
  uint64_t h = 1469598103934665603ull;
  for (size_t i = 0; i < n; ++i) {
    h ^= p[i];
    h *= 1099511628211ull;
  }
  return h;
}

template <typename T>
void put(std::vector<uint8_t>& b, T v) {
  const size_t o = b.size();
  b.resize(o + sizeof(T));
  std::memcpy(b.data() + o, &v, sizeof(T));
}

struct Reader {
  const uint8_t* p;
  size_t n, at = 0;
  template <typename T>
  bool get(T* v) {
    if (at + sizeof(T) > n) return false;
    std::memcpy(v, p + at, sizeof(T));
    at += sizeof(T);
    return true;
  }
};

// Parses and checks a blob in memory; on success tensor i starts at data + offs[i].
int parse(const std::vector<uint8_t>& file, const std::string& what, int* layers_out,
          std::vector<uint64_t>* offs_out) {
  Reader r{file.data(), file.size()};
  char magic[4];
  uint32_t version = 0, layers = 0, count = 0;
  uint64_t data_off = 0, data_bytes = 0, sum = 0;
  if (!r.get(&magic) || std::memcmp(magic, kMagic, 4) != 0)
    return bbh::internal_fail(BBH_ERR_IO, what + ": not a weight blob (bad magic)");
  if (!r.get(&version) || version != kVersion)
    return bbh::internal_fail(BBH_ERR_IO, what + ": unsupported blob version " + std::to_string(version));
  if (!r.get(&layers) || !r.get(&count) || !r.get(&data_off) || !r.get(&data_bytes) || !r.get(&sum))
    return bbh::internal_fail(BBH_ERR_IO, what + ": truncated header");
  if (bbh_num_tensors(static_cast<int>(layers)) == 0 || count != static_cast<uint32_t>(bbh_num_tensors(int(layers))))
    return bbh::internal_fail(BBH_ERR_IO, what + ": bad layer count " + std::to_string(layers) + " / tensor count " +
                                              std::to_string(count));
  if (data_off > file.size() || data_bytes > file.size() - data_off)
    return bbh::internal_fail(BBH_ERR_IO, what + ": truncated data (" + std::to_string(file.size()) + " bytes)");
  std::vector<uint64_t> offs(count);
  for (uint32_t i = 0; i < count; ++i) {
    uint32_t len = 0;
    uint64_t numel = 0, off = 0;
    if (!r.get(&len) || r.at + len > r.n) return bbh::internal_fail(BBH_ERR_IO, what + ": truncated tensor table");
    const std::string name(reinterpret_cast<const char*>(r.p + r.at), len);
    r.at += len;
    if (!r.get(&numel) || !r.get(&off)) return bbh::internal_fail(BBH_ERR_IO, what + ": truncated tensor table");
    const char* want = bbh_tensor_name(int(layers), int(i));
    if (name != want)
      return bbh::internal_fail(BBH_ERR_IO, what + ": tensor " + std::to_string(i) + " is '" + name +
                                                "', expected '" + want + "'");
    if (int64_t(numel) != bbh_tensor_numel(int(layers), int(i)) || off % 256 || off + numel * 2 > data_bytes)
      return bbh::internal_fail(BBH_ERR_IO, what + ": tensor '" + name + "' has a bad size or offset");
    offs[i] = data_off + off;
  }
  if (r.at > data_off) return bbh::internal_fail(BBH_ERR_IO, what + ": tensor table overlaps the data");
  if (fnv1a(file.data() + data_off, data_bytes) != sum)
    return bbh::internal_fail(BBH_ERR_IO, what + ": checksum mismatch (corrupt data)");
  *layers_out = int(layers);
  *offs_out = std::move(offs);
  return BBH_OK;
}

int read_all(const char* path, std::vector<uint8_t>* out) {
  FILE* f = std::fopen(path, "rb");
  if (!f) return bbh::internal_fail(BBH_ERR_IO, std::string("cannot open ") + path);
  std::fseek(f, 0, SEEK_END);
  const long size = std::ftell(f);
  std::fseek(f, 0, SEEK_SET);
  out->resize(size > 0 ? size_t(size) : 0);
  const size_t got = out->empty() ? 0 : std::fread(out->data(), 1, out->size(), f);
  std::fclose(f);
  if (got != out->size()) return bbh::internal_fail(BBH_ERR_IO, std::string("short read of ") + path);
  return BBH_OK;
}

}  // namespace

extern "C" {

int bbh_weights_pack(const char* dir, int layers, const char* blob_path) {
  if (!dir || !blob_path || bbh_num_tensors(layers) == 0)
    return bbh::internal_fail(BBH_ERR_ARG, "bbh_weights_pack: bad arguments");
  const int count = bbh_num_tensors(layers);
  std::vector<uint8_t> data;
  std::vector<uint64_t> offs(static_cast<size_t>(count));
  for (int i = 0; i < count; ++i) {
    const std::string path = std::string(dir) + "/" + bbh_tensor_name(layers, i) + ".bin";
    const size_t bytes = size_t(bbh_tensor_numel(layers, i)) * 2;
    offs[size_t(i)] = data.size();
    data.resize(data.size() + ((bytes + 255) & ~size_t(255)), 0);
    FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) return bbh::internal_fail(BBH_ERR_IO, "cannot open " + path);
    const size_t got = std::fread(data.data() + offs[size_t(i)], 1, bytes, f);
    std::fclose(f);
    if (got != bytes)
      return bbh::internal_fail(BBH_ERR_IO, path + ": expected " + std::to_string(bytes) + " bytes, got " +
                                                std::to_string(got));
  }
  std::vector<uint8_t> head;
  head.insert(head.end(), kMagic, kMagic + 4);
  put<uint32_t>(head, kVersion);
  put<uint32_t>(head, uint32_t(layers));
  put<uint32_t>(head, uint32_t(count));
  const size_t patch = head.size();
  put<uint64_t>(head, 0);  // data offset, patched below
  put<uint64_t>(head, data.size());
  put<uint64_t>(head, fnv1a(data.data(), data.size()));
  for (int i = 0; i < count; ++i) {
    const std::string name = bbh_tensor_name(layers, i);
    put<uint32_t>(head, uint32_t(name.size()));
    head.insert(head.end(), name.begin(), name.end());
    put<uint64_t>(head, uint64_t(bbh_tensor_numel(layers, i)));
    put<uint64_t>(head, offs[size_t(i)]);
  }
  const uint64_t data_off = (head.size() + 4095) & ~uint64_t(4095);
  std::memcpy(head.data() + patch, &data_off, 8);
  head.resize(data_off, 0);
  FILE* f = std::fopen(blob_path, "wb");
  if (!f) return bbh::internal_fail(BBH_ERR_IO, std::string("cannot create ") + blob_path);
  const bool ok = std::fwrite(head.data(), 1, head.size(), f) == head.size() &&
                  std::fwrite(data.data(), 1, data.size(), f) == data.size();
  const bool closed = std::fclose(f) == 0;
  if (!ok || !closed) return bbh::internal_fail(BBH_ERR_IO, std::string("short write of ") + blob_path);
  return BBH_OK;
}

int bbh_blob_check(const char* blob_path, int* layers) {
  if (!blob_path || !layers) return bbh::internal_fail(BBH_ERR_ARG, "bbh_blob_check: bad arguments");
  std::vector<uint8_t> file;
  int rc = read_all(blob_path, &file);
  if (rc) return rc;
  std::vector<uint64_t> offs;
  return parse(file, blob_path, layers, &offs);
}

int bbh_weights_load_blob(const char* blob_path, int device, bbh_weights** out) {
  if (!blob_path || !out) return bbh::internal_fail(BBH_ERR_ARG, "bbh_weights_load_blob: bad arguments");
  std::vector<uint8_t> file;
  int rc = read_all(blob_path, &file);
  if (rc) return rc;
  int layers = 0;
  std::vector<uint64_t> offs;
  rc = parse(file, blob_path, &layers, &offs);
  if (rc) return rc;
  std::vector<const uint16_t*> ptrs(offs.size());
  for (size_t i = 0; i < offs.size(); ++i) ptrs[i] = reinterpret_cast<const uint16_t*>(file.data() + offs[i]);
  return bbh_weights_from_host(ptrs.data(), layers, device, out);
}

}  // extern "C"
