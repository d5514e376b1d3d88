// activation_file.h -- GLM5XACT BF16 activation batch files.
#pragma once
#include <cstdint>
#include <string>

namespace glm5x {

struct ActivationHeader {
  uint32_t tokens = 0, hidden = 0;
  uint64_t payload_bytes = 0;
  uint32_t crc = 0;
};

// Each returns a SidecarStatus (values equal k3x::ErrorCode / glm5x_status).
// expected_tokens / expected_hidden = 0 accept any extent.
int read_activation_header(const char* path, uint32_t expected_tokens, uint32_t expected_hidden,
                           ActivationHeader* out, std::string* msg);
int read_activation(const char* path, uint32_t expected_tokens, uint32_t expected_hidden,
                    ActivationHeader* hdr, uint16_t* out, uint64_t out_elems, std::string* msg);
int write_activation(const char* path, const uint16_t* data, uint32_t tokens, uint32_t hidden,
                     std::string* msg);

}  // namespace glm5x
