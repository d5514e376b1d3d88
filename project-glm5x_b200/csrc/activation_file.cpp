// activation_file.cpp -- GLM5XACT BF16 activation batch files, the hidden-state
// hand-off between the reference's Python layer and its C++ runtime
// (reader: runtime/src/glm5x_activation.cpp:13-111; writer:
// converter/glm5x_converter/activation.py:13-57).
//
// Layout (little endian): a 40-byte header struct "<8sIIIIHHQI" =
// ("GLM5XACT", version 1, header bytes 40, token_count, hidden_size, dtype 3
// (BF16), reserved 0, payload bytes = tokens * hidden * 2, CRC32C of the
// payload), then the row-major BF16 [tokens, hidden] payload. The reader
// rejects what the reference's reader rejects, with the same status codes.
#include "activation_file.h"

#include <cstdio>
#include <cstring>
#include <fstream>
#include <limits>

#include "sidecar.h"

namespace glm5x {
namespace {

constexpr char kMagic[8] = {'G', 'L', 'M', '5', 'X', 'A', 'C', 'T'};
constexpr uint32_t kVersion = 1;
constexpr uint32_t kHeaderBytes = 40;
constexpr uint16_t kBf16Dtype = 3;

uint32_t le32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
uint64_t le64(const uint8_t* p) { return (uint64_t)le32(p) | ((uint64_t)le32(p + 4) << 32); }
void put32(uint8_t* p, uint32_t v) {
  for (int i = 0; i < 4; ++i) p[i] = (uint8_t)(v >> (8 * i));
}
void put64(uint8_t* p, uint64_t v) {
  put32(p, (uint32_t)v);
  put32(p + 4, (uint32_t)(v >> 32));
}

}  // namespace

int read_activation_header(const char* path, uint32_t expected_tokens, uint32_t expected_hidden,
                           ActivationHeader* out, std::string* msg) {
  std::ifstream f(path, std::ios::binary | std::ios::ate);
  if (!f) {
    *msg = path;
    return kSidecarIo;
  }
  const std::streamoff end = f.tellg();
  if (end < 0 || (uint64_t)end < kHeaderBytes) {
    *msg = "activation header";
    return kSidecarTruncated;
  }
  uint8_t h[kHeaderBytes];
  f.seekg(0, std::ios::beg);
  if (!f.read(reinterpret_cast<char*>(h), kHeaderBytes)) {
    *msg = "activation header read";
    return kSidecarIo;
  }
  if (std::memcmp(h, kMagic, 8) != 0) {
    *msg = "GLM5XACT";
    return kSidecarMagic;
  }
  const uint16_t dtype = (uint16_t)(h[24] | (h[25] << 8));
  const uint16_t reserved = (uint16_t)(h[26] | (h[27] << 8));
  if (le32(h + 8) != kVersion || le32(h + 12) != kHeaderBytes || dtype != kBf16Dtype ||
      reserved != 0) {
    *msg = "activation header";
    return kSidecarVersion;
  }
  const uint32_t tokens = le32(h + 16), hidden = le32(h + 20);
  const uint64_t payload = le64(h + 28);
  if (tokens == 0 || hidden == 0 || (expected_tokens && tokens != expected_tokens) ||
      (expected_hidden && hidden != expected_hidden) ||
      payload != (uint64_t)tokens * hidden * 2u || (uint64_t)end != kHeaderBytes + payload) {
    *msg = "activation dimensions";
    return kSidecarExtent;
  }
  out->tokens = tokens;
  out->hidden = hidden;
  out->payload_bytes = payload;
  out->crc = le32(h + 36);
  return kSidecarOk;
}

int read_activation(const char* path, uint32_t expected_tokens, uint32_t expected_hidden,
                    ActivationHeader* hdr, uint16_t* out, uint64_t out_elems, std::string* msg) {
  int st = read_activation_header(path, expected_tokens, expected_hidden, hdr, msg);
  if (st != kSidecarOk) return st;
  if (out_elems < hdr->payload_bytes / 2) {
    *msg = "activation buffer smaller than the payload";
    return kSidecarExtent;
  }
  std::ifstream f(path, std::ios::binary);
  f.seekg(kHeaderBytes, std::ios::beg);
  if (!f || !f.read(reinterpret_cast<char*>(out), (std::streamsize)hdr->payload_bytes)) {
    *msg = "activation payload read";
    return kSidecarIo;
  }
  if (crc32c(reinterpret_cast<const uint8_t*>(out), hdr->payload_bytes) != hdr->crc) {
    *msg = "activation payload";
    return kSidecarDataCrc;
  }
  return kSidecarOk;
}

int write_activation(const char* path, const uint16_t* data, uint32_t tokens, uint32_t hidden,
                     std::string* msg) {
  if (tokens == 0 || hidden == 0) {
    *msg = "activation tensor dimensions must be non-zero";
    return kSidecarExtent;
  }
  const uint64_t payload = (uint64_t)tokens * hidden * 2u;
  uint8_t h[kHeaderBytes];
  std::memcpy(h, kMagic, 8);
  put32(h + 8, kVersion);
  put32(h + 12, kHeaderBytes);
  put32(h + 16, tokens);
  put32(h + 20, hidden);
  h[24] = (uint8_t)kBf16Dtype;
  h[25] = 0;
  h[26] = h[27] = 0;
  put64(h + 28, payload);
  put32(h + 36, crc32c(reinterpret_cast<const uint8_t*>(data), payload));
  // written beside the destination, then renamed over it (the writer's
  // atomic replace)
  const std::string dst(path), tmp = dst + ".tmp";
  {
    std::ofstream f(tmp, std::ios::binary | std::ios::trunc);
    if (!f || !f.write(reinterpret_cast<const char*>(h), kHeaderBytes) ||
        !f.write(reinterpret_cast<const char*>(data), (std::streamsize)payload) || !f.flush()) {
      std::remove(tmp.c_str());
      *msg = "activation write";
      return kSidecarIo;
    }
  }
  if (std::rename(tmp.c_str(), dst.c_str()) != 0) {
    std::remove(tmp.c_str());
    *msg = "activation rename";
    return kSidecarIo;
  }
  return kSidecarOk;
}

}  // namespace glm5x
