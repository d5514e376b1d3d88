// sidecar.h -- packed expert sidecar reader (.pn4 / .pm4).
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace glm5x {

enum SidecarStatus {
  kSidecarOk = 0,
  kSidecarIo = 1,
  kSidecarMagic = 2,
  kSidecarVersion = 3,
  kSidecarTruncated = 7,
  kSidecarDirectory = 8,
  kSidecarExtent = 9,
  kSidecarDataCrc = 10,
  kSidecarAuxCrc = 11,
  kSidecarState = 16,
};

struct SidecarRole {
  int64_t rows = 0, cols = 0, group_size = 0;
  int64_t packed_offset = 0, packed_bytes = 0;
  int64_t scale_offset = 0, scale_bytes = 0;
  float global_scale = 1.0f;  // NVFP4 only
};

struct Sidecar {
  int precision = 0;  // 0 NVFP4, 1 MXFP4
  std::string source_digest;
  SidecarRole roles[3];  // gate, up, down
  std::vector<uint8_t> payload;
};

// CRC-32C (Castagnoli), the checksum google_crc32c computes.
uint32_t crc32c(const uint8_t* data, size_t n);

// Reads and checks one sidecar. precision: 0 NVFP4, 1 MXFP4, -1 either (the
// file's format string decides); source_digest: the expected source_digest,
// or NULL for none. Returns a SidecarStatus (values equal k3x::ErrorCode /
// glm5x_status) and, on failure, a message led by the reference's error code.
int read_sidecar(const char* path, int precision, const char* source_digest, Sidecar* out,
                 std::string* msg);

}  // namespace glm5x
