// k3x_reader.h -- K3X v1 checkpoint containers (.k3x), read for the MoE path.
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace glm5x {

// Status values are k3x::ErrorCode's (runtime/include/k3x/status.hpp:9-30).
enum K3xStatus {
  kK3xOk = 0,
  kK3xIo = 1,
  kK3xBadMagic = 2,
  kK3xUnsupportedVersion = 3,
  kK3xUnsupportedRequiredFeature = 4,
  kK3xSuperblockCrc = 6,
  kK3xTruncated = 7,
  kK3xInvalidDirectory = 8,
  kK3xInvalidExtent = 9,
  kK3xDataCrc = 10,
  kK3xAuxiliaryCrc = 11,
  kK3xDirectorySha = 12,
  kK3xRootSha = 13,
  kK3xTensorNotFound = 14,
};

// One 128-byte tensor record (converter/k3x_converter/format.py:155-210).
struct K3xTensor {
  uint64_t tensor_id = 0;
  uint16_t dtype = 0, quantization = 0;  // dtype 1 FP32, 2 UINT8, 3 BF16; quantization 1 MXFP4
  uint8_t rank = 0;
  int32_t layer_id = -1, expert_id = -1;
  uint64_t dims[4] = {0, 0, 0, 0};
  uint64_t data_offset = 0, data_length = 0, logical_length = 0;
  uint64_t auxiliary_offset = 0, auxiliary_length = 0;
  uint32_t data_crc32c = 0, auxiliary_crc32c = 0;
};

struct K3xFile {
  std::string path;
  uint64_t file_length = 0;
  std::vector<K3xTensor> tensors;
};

// FNV-1a 64 of a tensor name: the tensor ids the converter writes
// (format.py:49-54) and the runtime looks experts up by (runtime/src/model.cpp:540).
uint64_t fnv1a64(const char* name);

// SHA-256 (FIPS 180-4) of data.
void sha256(const uint8_t* data, size_t n, uint8_t out[32]);

// Opens and validates like k3x::Reader::open (runtime/src/reader.cpp:420-702);
// verify = the checksums mode (every extent's CRC32C, the directory and root
// SHA-256), else metadata only.
int k3x_open(const char* path, bool verify, K3xFile* out, std::string* msg);
const K3xTensor* k3x_find(const K3xFile& f, uint64_t tensor_id);
// Reads [offset, offset + length) of the file (length > 0, inside the file).
int k3x_read_extent(const K3xFile& f, uint64_t offset, uint64_t length, uint8_t* dst,
                    std::string* msg);

}  // namespace glm5x
