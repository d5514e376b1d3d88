// k3x_reader.cpp -- reader for K3X v1 checkpoint containers (.k3x), the
// reference runtime's weight format, restricted to what the MoE path needs:
// open with the checks of k3x::Reader::open (runtime/src/reader.cpp:420-702,
// same ErrorCode values), find tensors by id, read their data and auxiliary
// extents (reader.cpp:749-778). Layout (converter/k3x_converter/format.py):
// a 4096-byte superblock ("K3XCHKPT", version 1.0, directory offsets, CRC32C
// of its first 4092 bytes, directory and root SHA-256), the tensor ("TENS",
// 128-byte records), layer ("LAYR", 64) and expert ("EXPT", 64) directories
// and a 256-byte model config, every extent 4096-aligned. MXFP4 records are
// UINT8 data (packed E2M1) with an E8M0 auxiliary extent.
#include "k3x_reader.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <fstream>
#include <limits>
#include <unordered_set>
#include <utility>

#include "sidecar.h"  // crc32c

namespace glm5x {
namespace {

constexpr uint64_t kBlock = 4096;
constexpr uint64_t kTensorRecord = 128, kLayerRecord = 64, kExpertRecord = 64;
constexpr uint64_t kConfigBytes = 256;

uint64_t le(const uint8_t* p, int n) {
  uint64_t v = 0;
  for (int i = 0; i < n; ++i) v |= (uint64_t)p[i] << (8 * i);
  return v;
}
bool all_zero(const uint8_t* p, size_t n) {
  for (size_t i = 0; i < n; ++i)
    if (p[i]) return false;
  return true;
}
bool range_valid(uint64_t offset, uint64_t length, uint64_t limit) {
  return offset <= limit && length <= limit - offset;
}

int read_raw(const std::string& path, uint64_t offset, uint64_t length, std::vector<uint8_t>* out) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return kK3xIo;
  out->resize(length);
  f.seekg((std::streamoff)offset);
  f.read(reinterpret_cast<char*>(out->data()), (std::streamsize)length);
  if ((uint64_t)f.gcount() != length) return kK3xTruncated;
  return kK3xOk;
}

// directory header "<4sIQ" = (tag, record size, count) then the records
bool directory_count(const std::vector<uint8_t>& d, const char* tag, uint64_t record,
                     uint64_t* count) {
  if (d.size() < 16 || std::memcmp(d.data(), tag, 4) != 0 || le(d.data() + 4, 4) != record)
    return false;
  const uint64_t n = le(d.data() + 8, 8);
  if (n > (d.size() - 16) / record || d.size() != 16 + n * record) return false;
  *count = n;
  return true;
}

// ---------------------------------------------------------------- SHA-256
// FIPS 180-4. The round constants and initial hash words are, as the standard
// defines them, the first 32 fractional bits of the cube roots of the first
// 64 primes and of the square roots of the first 8; they are computed here.
struct Sha256Tables {
  uint32_t k[64], h0[8];
  Sha256Tables() {
    int primes[64], n = 0;
    for (int c = 2; n < 64; ++c) {
      bool prime = true;
      for (int d = 2; d * d <= c; ++d)
        if (c % d == 0) prime = false;
      if (prime) primes[n++] = c;
    }
    auto frac32 = [](long double r) {
      return (uint32_t)std::floor((r - std::floor(r)) * 4294967296.0L);
    };
    for (int i = 0; i < 64; ++i) k[i] = frac32(std::cbrt((long double)primes[i]));
    for (int i = 0; i < 8; ++i) h0[i] = frac32(std::sqrt((long double)primes[i]));
  }
};
const Sha256Tables& sha_tables() {
  static const Sha256Tables t;
  return t;
}
uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

struct Sha256 {
  uint32_t h[8];
  uint8_t buf[64];
  size_t fill = 0;
  uint64_t total = 0;
  Sha256() { std::memcpy(h, sha_tables().h0, sizeof h); }
  void block(const uint8_t* p) {
    const uint32_t* k = sha_tables().k;
    uint32_t w[64];
    for (int i = 0; i < 16; ++i)
      w[i] = ((uint32_t)p[4 * i] << 24) | ((uint32_t)p[4 * i + 1] << 16) |
             ((uint32_t)p[4 * i + 2] << 8) | p[4 * i + 3];
    for (int i = 16; i < 64; ++i) {
      const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
      const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int i = 0; i < 64; ++i) {
      const uint32_t t1 = hh + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) +
                          k[i] + w[i];
      const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
      hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
    }
    h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
  }
  void update(const uint8_t* p, size_t n) {
    total += n;
    while (n) {
      const size_t take = std::min(n, (size_t)64 - fill);
      std::memcpy(buf + fill, p, take);
      fill += take;
      p += take;
      n -= take;
      if (fill == 64) {
        block(buf);
        fill = 0;
      }
    }
  }
  void finish(uint8_t out[32]) {
    const uint64_t bits = total * 8;
    const uint8_t one = 0x80, zero = 0;
    update(&one, 1);
    while (fill != 56) update(&zero, 1);
    uint8_t len[8];
    for (int i = 0; i < 8; ++i) len[i] = (uint8_t)(bits >> (56 - 8 * i));
    update(len, 8);
    for (int i = 0; i < 8; ++i)
      for (int j = 0; j < 4; ++j) out[4 * i + j] = (uint8_t)(h[i] >> (24 - 8 * j));
  }
};

}  // namespace

void sha256(const uint8_t* data, size_t n, uint8_t out[32]) {
  Sha256 s;
  s.update(data, n);
  s.finish(out);
}

uint64_t fnv1a64(const char* name) {
  uint64_t h = 0xCBF29CE484222325ull;
  for (const unsigned char* p = reinterpret_cast<const unsigned char*>(name); *p; ++p) {
    h ^= *p;
    h *= 0x100000001B3ull;
  }
  return h;
}

const K3xTensor* k3x_find(const K3xFile& f, uint64_t id) {
  for (const K3xTensor& t : f.tensors)
    if (t.tensor_id == id) return &t;
  return nullptr;
}

int k3x_read_extent(const K3xFile& f, uint64_t offset, uint64_t length, uint8_t* dst,
                    std::string* msg) {
  if (!length || !range_valid(offset, length, f.file_length)) {
    *msg = "extent outside the file";
    return kK3xInvalidExtent;
  }
  std::ifstream s(f.path, std::ios::binary);
  if (!s) {
    *msg = f.path;
    return kK3xIo;
  }
  s.seekg((std::streamoff)offset);
  s.read(reinterpret_cast<char*>(dst), (std::streamsize)length);
  if ((uint64_t)s.gcount() != length) {
    *msg = "short read";
    return kK3xTruncated;
  }
  return kK3xOk;
}

int k3x_open(const char* path, bool verify, K3xFile* out, std::string* msg) {
  auto fail = [&](int st, const char* what) {
    *msg = what;
    return st;
  };
  K3xFile f;
  f.path = path;
  {
    std::ifstream s(path, std::ios::binary | std::ios::ate);
    if (!s) return fail(kK3xTruncated, "cannot size the file");
    f.file_length = (uint64_t)s.tellg();
  }
  if (f.file_length < kBlock) return fail(kK3xTruncated, "shorter than the superblock");
  std::vector<uint8_t> sb;
  int st = read_raw(f.path, 0, kBlock, &sb);
  if (st) return fail(st, "superblock read");
  const uint8_t* b = sb.data();
  if (std::memcmp(b, "K3XCHKPT", 8) != 0) return fail(kK3xBadMagic, "K3XCHKPT");
  if (le(b + 8, 2) != 1 || le(b + 10, 2) != 0 || le(b + 12, 4) != kBlock || le(b + 16, 4) != kBlock)
    return fail(kK3xUnsupportedVersion, "superblock version / layout");
  if (crc32c(b, 4092) != (uint32_t)le(b + 4092, 4))
    return fail(kK3xSuperblockCrc, "superblock CRC32C");
  if (le(b + 24, 8) != 0) return fail(kK3xUnsupportedRequiredFeature, "required features");
  if (!all_zero(b + 232, 4092 - 232)) return fail(kK3xInvalidDirectory, "superblock reserved bytes");
  const uint32_t state = (uint32_t)le(b + 20, 4);
  uint64_t v[10];
  for (int i = 0; i < 10; ++i) v[i] = le(b + 88 + 8 * i, 8);
  if (state != 1 || v[9] != f.file_length) return fail(kK3xTruncated, "state or file length");
  for (int r = 0; r < 4; ++r)
    if (v[2 * r] % kBlock || !range_valid(v[2 * r], v[2 * r + 1], f.file_length))
      return fail(kK3xInvalidExtent, "directory extent");
  std::vector<uint8_t> tdir, ldir, edir, cfg;
  if (read_raw(f.path, v[0], v[1], &tdir) || read_raw(f.path, v[2], v[3], &ldir) ||
      read_raw(f.path, v[4], v[5], &edir) || read_raw(f.path, v[6], v[7], &cfg) ||
      cfg.size() != kConfigBytes)
    return fail(kK3xInvalidDirectory, "directory read");
  uint64_t nt = 0, nl = 0, ne = 0;
  if (!directory_count(tdir, "TENS", kTensorRecord, &nt) ||
      !directory_count(ldir, "LAYR", kLayerRecord, &nl) ||
      !directory_count(edir, "EXPT", kExpertRecord, &ne) || le(cfg.data() + 8, 4) != nl ||
      !all_zero(cfg.data() + 112, kConfigBytes - 112) || (le(cfg.data() + 108, 4) & ~3ull))
    return fail(kK3xInvalidDirectory, "directory headers");
  std::vector<std::pair<uint64_t, uint64_t>> ranges{{0, kBlock}};
  for (int r = 0; r < 4; ++r) ranges.emplace_back(v[2 * r], v[2 * r] + v[2 * r + 1]);
  std::unordered_set<uint64_t> ids;
  for (uint64_t i = 0; i < nt; ++i) {
    const uint8_t* r = tdir.data() + 16 + i * kTensorRecord;
    K3xTensor t;
    t.tensor_id = le(r, 8);
    t.dtype = (uint16_t)le(r + 12, 2);
    t.quantization = (uint16_t)le(r + 14, 2);
    t.rank = r[16];
    t.layer_id = (int32_t)(uint32_t)le(r + 20, 4);
    t.expert_id = (int32_t)(uint32_t)le(r + 24, 4);
    for (int d = 0; d < 4; ++d) t.dims[d] = le(r + 32 + 8 * d, 8);
    t.data_offset = le(r + 64, 8);
    t.data_length = le(r + 72, 8);
    t.logical_length = le(r + 80, 8);
    t.auxiliary_offset = le(r + 88, 8);
    t.auxiliary_length = le(r + 96, 8);
    t.data_crc32c = (uint32_t)le(r + 104, 4);
    t.auxiliary_crc32c = (uint32_t)le(r + 108, 4);
    if (t.rank > 4 || (t.dtype != 1 && t.dtype != 2 && t.dtype != 3) || t.quantization > 1 ||
        le(r + 8, 4) != 0 || r[17] != 0 || le(r + 18, 2) != 0 || le(r + 28, 4) != 0 ||
        !all_zero(r + 112, kTensorRecord - 112) || !ids.insert(t.tensor_id).second)
      return fail(kK3xInvalidDirectory, "tensor record");
    for (int d = t.rank; d < 4; ++d)
      if (t.dims[d]) return fail(kK3xInvalidDirectory, "tensor dimensions");
    const bool plain = (t.dtype == 1 || t.dtype == 3) && t.quantization == 0 &&
                       t.auxiliary_length == 0 && t.auxiliary_offset == 0 &&
                       t.auxiliary_crc32c == 0;
    const bool mxfp4 = t.dtype == 2 && t.quantization == 1 && t.auxiliary_length != 0;
    if (!t.data_length || !t.logical_length || (!plain && !mxfp4))
      return fail(kK3xInvalidDirectory, "tensor kind");
    const std::pair<uint64_t, uint64_t> ext[2] = {{t.data_offset, t.data_length},
                                                  {t.auxiliary_offset, t.auxiliary_length}};
    for (const auto& [off, len] : ext) {
      if (!len) {
        if (off) return fail(kK3xInvalidExtent, "empty extent with an offset");
      } else {
        if (off % kBlock || !range_valid(off, len, f.file_length))
          return fail(kK3xInvalidExtent, "tensor extent");
        ranges.emplace_back(off, off + len);
      }
    }
    f.tensors.push_back(t);
  }
  const int64_t experts_cfg = (int64_t)le(cfg.data() + 48, 4);
  for (const K3xTensor& t : f.tensors)
    if (t.layer_id < -1 || t.layer_id >= (int64_t)nl || t.expert_id < -1 ||
        t.expert_id >= experts_cfg || (t.expert_id >= 0 && t.layer_id < 0))
      return fail(kK3xInvalidDirectory, "tensor layer / expert");
  for (uint64_t i = 0; i < nl; ++i) {
    const uint8_t* r = ldir.data() + 16 + i * kLayerRecord;
    const uint64_t index = le(r, 4), attn = le(r + 4, 2), ffn = le(r + 6, 2);
    const uint64_t first_t = le(r + 8, 4), count_t = le(r + 12, 4);
    const uint64_t first_e = le(r + 16, 4), count_e = le(r + 20, 4);
    if (index != i || (attn != 1 && attn != 2) || (ffn != 1 && ffn != 2) || le(r + 28, 4) != 0 ||
        !all_zero(r + 32, kLayerRecord - 32) || first_t > nt || count_t > nt - first_t ||
        first_e > ne || count_e > ne - first_e)
      return fail(kK3xInvalidDirectory, "layer record");
    for (uint64_t t = first_t; t < first_t + count_t; ++t)
      if (f.tensors[t].layer_id != (int32_t)i) return fail(kK3xInvalidDirectory, "layer tensors");
  }
  std::unordered_set<uint64_t> orders;
  for (uint64_t i = 0; i < ne; ++i) {
    const uint8_t* r = edir.data() + 16 + i * kExpertRecord;
    const uint64_t layer = le(r, 4), expert = le(r + 4, 4), order = le(r + 8, 4);
    if (layer >= nl || (int64_t)expert >= experts_cfg || order >= ne ||
        !orders.insert(order).second || le(r + 12, 4) != 0 || !all_zero(r + 48, kExpertRecord - 48))
      return fail(kK3xInvalidDirectory, "expert record");
    for (int o = 16; o <= 32; o += 8) {
      const K3xTensor* t = k3x_find(f, le(r + o, 8));
      const bool native_mxfp4 = t && t->dtype == 2 && t->quantization == 1;
      const bool staged_bf16 = t && t->dtype == 3 && t->quantization == 0 &&
                               t->auxiliary_length == 0 && t->auxiliary_offset == 0 &&
                               t->auxiliary_crc32c == 0;
      if (!t || t->layer_id != (int32_t)layer || t->expert_id != (int32_t)expert ||
          (!native_mxfp4 && !staged_bf16))
        return fail(kK3xInvalidDirectory, "expert tensors");
    }
  }
  for (uint64_t l = 0; l < nl; ++l) {
    const uint8_t* r = ldir.data() + 16 + l * kLayerRecord;
    const uint64_t first = le(r + 16, 4), count = le(r + 20, 4);
    for (uint64_t e = first; e < first + count; ++e)
      if (le(edir.data() + 16 + e * kExpertRecord, 4) != l)
        return fail(kK3xInvalidDirectory, "layer experts");
  }
  std::sort(ranges.begin(), ranges.end());
  for (size_t i = 1; i < ranges.size(); ++i)
    if (ranges[i].first < ranges[i - 1].second) return fail(kK3xInvalidExtent, "overlapping extents");
  if (verify) {
    std::vector<uint8_t> buf;
    for (const K3xTensor& t : f.tensors) {
      if (read_raw(f.path, t.data_offset, t.data_length, &buf) ||
          crc32c(buf.data(), buf.size()) != t.data_crc32c)
        return fail(kK3xDataCrc, "tensor data CRC32C");
      if (t.auxiliary_length &&
          (read_raw(f.path, t.auxiliary_offset, t.auxiliary_length, &buf) ||
           crc32c(buf.data(), buf.size()) != t.auxiliary_crc32c))
        return fail(kK3xAuxiliaryCrc, "tensor auxiliary CRC32C");
    }
    Sha256 dsha;
    for (const auto* d : {&tdir, &ldir, &edir, &cfg}) dsha.update(d->data(), d->size());
    uint8_t digest[32];
    dsha.finish(digest);
    if (std::memcmp(digest, b + 168, 32) != 0) return fail(kK3xDirectorySha, "directory SHA-256");
    // root: the whole file with the root digest and the superblock CRC zeroed
    std::ifstream s(f.path, std::ios::binary);
    if (!s) return fail(kK3xIo, "root read");
    Sha256 rsha;
    std::vector<uint8_t> chunk(1 << 20);
    for (uint64_t pos = 0; pos < f.file_length;) {
      const uint64_t n = std::min<uint64_t>(chunk.size(), f.file_length - pos);
      s.read(reinterpret_cast<char*>(chunk.data()), (std::streamsize)n);
      if ((uint64_t)s.gcount() != n) return fail(kK3xTruncated, "root read");
      for (const auto& [lo, hi] : {std::pair<uint64_t, uint64_t>{200, 232}, {4092, 4096}}) {
        const uint64_t l = std::max(lo, pos), h = std::min(hi, pos + n);
        if (l < h) std::memset(chunk.data() + (l - pos), 0, h - l);
      }
      rsha.update(chunk.data(), n);
      pos += n;
    }
    rsha.finish(digest);
    if (std::memcmp(digest, b + 200, 32) != 0) return fail(kK3xRootSha, "root SHA-256");
  }
  *out = std::move(f);
  return kK3xOk;
}

}  // namespace glm5x
