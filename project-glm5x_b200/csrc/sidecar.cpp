// sidecar.cpp -- reader for the reference's packed expert sidecars
// (reference/glm5x_ref/packed_cache.py:24-27, 192-205, 327-404, 407-504).
//
// File layout: struct "<8sII" = ("GLM5XPI4", version 1, json_len), then
// json_len bytes of compact sorted-key JSON, then the payload. The JSON holds
// {"format": "glm5x-<precision>-expert-v1", "payload_bytes", "roles": [gate,
// up, down], "source_digest"}; every role has shape, packed/qparams offsets,
// sizes and CRC32C values (NVFP4 adds scale_bytes and global_scale_bytes = 4;
// its qparams are the blocked E4M3 scales followed by the FP32 global).
#include "sidecar.h"

#include "../../include/glm5x_moe.h"

#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace glm5x {

// ------------------------------------------------------------------ CRC32C
// Slicing-by-8 tables of the Castagnoli polynomial (reflected 0x82F63B78),
// built once in a function-local static: C++11 makes its initialization
// thread-safe, so sidecars, .k3x files and activation files may be read from
// several host threads at once.
namespace {
struct Crc32cTables {
  uint32_t t[8][256];
  Crc32cTables() {
    for (uint32_t i = 0; i < 256; ++i) {
      uint32_t c = i;
      for (int k = 0; k < 8; ++k) c = (c & 1) ? (c >> 1) ^ 0x82F63B78u : c >> 1;
      t[0][i] = c;
    }
    for (uint32_t i = 0; i < 256; ++i)
      for (int s = 1; s < 8; ++s) t[s][i] = (t[s - 1][i] >> 8) ^ t[0][t[s - 1][i] & 0xff];
  }
};

const Crc32cTables& crc_tables() {
  static const Crc32cTables tables;
  return tables;
}
}  // namespace

uint32_t crc32c(const uint8_t* data, size_t n) {
  const auto& crc32c_table = crc_tables().t;
  uint32_t c = 0xFFFFFFFFu;
  while (n >= 8) {
    uint64_t v;
    std::memcpy(&v, data, 8);
    v ^= c;
    c = crc32c_table[7][v & 0xff] ^ crc32c_table[6][(v >> 8) & 0xff] ^
        crc32c_table[5][(v >> 16) & 0xff] ^ crc32c_table[4][(v >> 24) & 0xff] ^
        crc32c_table[3][(v >> 32) & 0xff] ^ crc32c_table[2][(v >> 40) & 0xff] ^
        crc32c_table[1][(v >> 48) & 0xff] ^ crc32c_table[0][v >> 56];
    data += 8;
    n -= 8;
  }
  while (n--) c = crc32c_table[0][(c ^ *data++) & 0xff] ^ (c >> 8);
  return c ^ 0xFFFFFFFFu;
}

// ------------------------------------------------------------------ JSON
namespace {
struct Json {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  double num = 0;
  bool b = false;
  std::string str;
  std::vector<Json> arr;
  std::map<std::string, Json> obj;
  const Json* get(const char* k) const {
    auto it = obj.find(k);
    return it == obj.end() ? nullptr : &it->second;
  }
};

struct Parser {
  const char* p;
  const char* end;
  bool ok = true;
  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\t' || *p == '\r')) ++p;
  }
  Json value() {
    ws();
    Json j;
    if (p >= end) {
      ok = false;
      return j;
    }
    if (*p == '{') {
      j.kind = Json::Obj;
      ++p;
      ws();
      if (p < end && *p == '}') {
        ++p;
        return j;
      }
      while (ok) {
        ws();
        Json k = value();
        if (k.kind != Json::Str) {
          ok = false;
          break;
        }
        ws();
        if (p >= end || *p != ':') {
          ok = false;
          break;
        }
        ++p;
        j.obj[k.str] = value();
        ws();
        if (p < end && *p == ',') {
          ++p;
          continue;
        }
        if (p < end && *p == '}') {
          ++p;
          break;
        }
        ok = false;
      }
    } else if (*p == '[') {
      j.kind = Json::Arr;
      ++p;
      ws();
      if (p < end && *p == ']') {
        ++p;
        return j;
      }
      while (ok) {
        j.arr.push_back(value());
        ws();
        if (p < end && *p == ',') {
          ++p;
          continue;
        }
        if (p < end && *p == ']') {
          ++p;
          break;
        }
        ok = false;
      }
    } else if (*p == '"') {
      j.kind = Json::Str;
      ++p;
      while (p < end && *p != '"') {
        if (*p == '\\' && p + 1 < end) ++p;
        j.str.push_back(*p++);
      }
      if (p >= end) ok = false; else ++p;
    } else if (!std::strncmp(p, "true", 4)) {
      j.kind = Json::Bool;
      j.b = true;
      p += 4;
    } else if (!std::strncmp(p, "false", 5)) {
      j.kind = Json::Bool;
      p += 5;
    } else if (!std::strncmp(p, "null", 4)) {
      p += 4;
    } else {
      j.kind = Json::Num;
      char* e = nullptr;
      j.num = std::strtod(p, &e);
      if (e == p) ok = false;
      p = e;
    }
    return j;
  }
};

bool get_int(const Json& o, const char* k, int64_t* v) {
  const Json* j = o.get(k);
  if (!j || j->kind != Json::Num) return false;
  *v = static_cast<int64_t>(j->num);
  return true;
}
}  // namespace

// Checks in the order of GLM5XPackedExpertCache.get / _decode_role
// (packed_cache.py:518-545, 407-423, 476-479), so a file with several faults
// reports the one the reference meets first. Each message starts with the
// reference's error code name.
int read_sidecar(const char* path, int precision, const char* source_digest, Sidecar* out,
                 std::string* msg) {
  auto fail = [&](int status, const char* code, const std::string& what) {
    *msg = std::string(code) + ": " + what;
    return status;
  };
  std::ifstream f(path, std::ios::binary);
  if (!f) return fail(kSidecarIo, "GLM5X_PACKED_CACHE_IO", std::string("cannot open ") + path);
  std::vector<uint8_t> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  if (bytes.size() < 16)
    return fail(kSidecarTruncated, "GLM5X_PACKED_CACHE_HEADER", "shorter than its 16-byte header");
  if (std::memcmp(bytes.data(), "GLM5XPI4", 8) != 0)
    return fail(kSidecarMagic, "GLM5X_PACKED_CACHE_FORMAT", "magic is not GLM5XPI4");
  uint32_t version, json_len;
  std::memcpy(&version, bytes.data() + 8, 4);
  std::memcpy(&json_len, bytes.data() + 12, 4);
  if (version != 1)
    return fail(kSidecarVersion, "GLM5X_PACKED_CACHE_FORMAT", "unsupported version");
  if (16ull + json_len > bytes.size())
    return fail(kSidecarDirectory, "GLM5X_PACKED_CACHE_METADATA", "metadata runs past the file");
  Parser ps{reinterpret_cast<const char*>(bytes.data() + 16),
            reinterpret_cast<const char*>(bytes.data() + 16 + json_len)};
  Json meta = ps.value();
  ps.ws();
  if (!ps.ok || ps.p != ps.end || meta.kind != Json::Obj)
    return fail(kSidecarDirectory, "GLM5X_PACKED_CACHE_METADATA", "metadata is not a JSON object");
  const Json* fmt = meta.get("format");
  int found = -1;
  if (fmt && fmt->kind == Json::Str) {
    if (fmt->str == "glm5x-nvfp4-expert-v1") found = 0;
    else if (fmt->str == "glm5x-mxfp4-expert-v1") found = 1;
  }
  if (found < 0 || (precision >= 0 && found != precision))
    return fail(kSidecarState, "GLM5X_PACKED_CACHE_FORMAT",
                precision == 1 ? "format is not glm5x-mxfp4-expert-v1"
                : precision == 0 ? "format is not glm5x-nvfp4-expert-v1"
                                 : "format is neither glm5x-nvfp4-expert-v1 nor -mxfp4-");
  out->precision = found;
  const Json* digest = meta.get("source_digest");
  out->source_digest = digest && digest->kind == Json::Str ? digest->str : std::string();
  if (source_digest && (!digest || digest->kind != Json::Str || digest->str != source_digest))
    return fail(kSidecarState, "GLM5X_PACKED_CACHE_SOURCE_MISMATCH",
                "source_digest differs from the expected one");
  const Json* roles = meta.get("roles");
  if (!roles || roles->kind != Json::Arr || roles->arr.size() != 3)
    return fail(kSidecarDirectory, "GLM5X_PACKED_CACHE_ROLES", "roles is not a list of three");
  int64_t payload_bytes = -1;
  const size_t base = 16ull + json_len;
  if (!get_int(meta, "payload_bytes", &payload_bytes) ||
      base + static_cast<uint64_t>(payload_bytes) != bytes.size() || payload_bytes < 0)
    return fail(kSidecarExtent, "GLM5X_PACKED_CACHE_PAYLOAD_EXTENT",
                "payload size differs from payload_bytes");
  out->payload.assign(bytes.begin() + base, bytes.end());
  for (int r = 0; r < 3; ++r) {
    const Json& role = roles->arr[r];
    SidecarRole& dst = out->roles[r];
    const Json* shape = role.kind == Json::Obj ? role.get("shape") : nullptr;
    int64_t po, pb, qo, qb, pcrc, qcrc, group = 0;
    if (!shape || shape->kind != Json::Arr || shape->arr.size() != 2 ||
        shape->arr[0].kind != Json::Num || shape->arr[1].kind != Json::Num ||
        !get_int(role, "packed_offset", &po) || !get_int(role, "packed_bytes", &pb) ||
        !get_int(role, "qparams_offset", &qo) || !get_int(role, "qparams_bytes", &qb) ||
        !get_int(role, "packed_crc32c", &pcrc) || !get_int(role, "qparams_crc32c", &qcrc) ||
        !get_int(role, "group_size", &group))
      return fail(kSidecarDirectory, "GLM5X_PACKED_CACHE_ROLES", "role metadata incomplete");
    dst.rows = static_cast<int64_t>(shape->arr[0].num);
    dst.cols = static_cast<int64_t>(shape->arr[1].num);
    dst.group_size = group;
    if (po < 0 || pb < 0 || qo < 0 || qb < 0 || po + pb > payload_bytes ||
        qo + qb > payload_bytes)
      return fail(kSidecarExtent, "GLM5X_PACKED_CACHE_PAYLOAD_EXTENT",
                  "role section outside the payload");
    const uint8_t* pp = out->payload.data() + po;
    const uint8_t* qp = out->payload.data() + qo;
    if (crc32c(pp, pb) != static_cast<uint32_t>(pcrc))
      return fail(kSidecarDataCrc, "GLM5X_PACKED_CACHE_PACKED_CRC", "packed CRC32C mismatch");
    if (crc32c(qp, qb) != static_cast<uint32_t>(qcrc))
      return fail(kSidecarAuxCrc, "GLM5X_PACKED_CACHE_QPARAM_CRC", "qparams CRC32C mismatch");
    dst.packed_offset = po;
    dst.packed_bytes = pb;
    if (found == 0) {
      int64_t sb = 0, gb = 0;
      if (!get_int(role, "scale_bytes", &sb) || !get_int(role, "global_scale_bytes", &gb) ||
          sb + gb != qb || gb != 4)
        return fail(kSidecarExtent, "GLM5X_PACKED_CACHE_NVFP4_QPARAM_EXTENT",
                    "scale_bytes + global_scale_bytes differs from qparams_bytes");
      dst.scale_offset = qo;
      dst.scale_bytes = sb;
      std::memcpy(&dst.global_scale, qp + sb, 4);
    } else {
      dst.scale_offset = qo;
      dst.scale_bytes = qb;
      dst.global_scale = 1.0f;
    }
    // the reference reshapes the sections to packed_shape / qparams_shape
    // (a mismatch raises there); the sizes a matrix of this shape needs
    if (dst.rows <= 0 || dst.cols <= 0 || dst.cols % 2 || pb != dst.rows * dst.cols / 2)
      return fail(kSidecarExtent, "GLM5X_PACKED_CACHE_PAYLOAD_EXTENT",
                  "packed bytes do not match the role's shape");
  }
  return 0;
}

}  // namespace glm5x

// ------------------------------------------------------------------ C ABI
// The host-only half of glm5x_moe_load_sidecar (no device, no engine).
namespace glm5x {
void set_last_error(const char* msg);
}

struct glm5x_sidecar {
  glm5x::Sidecar sc;
};

extern "C" {

glm5x_status glm5x_sidecar_open(const char* path, int32_t precision, const char* source_digest,
                                glm5x_sidecar** out) {
  if (!path || !out || precision < -1 || precision > 1) {
    glm5x::set_last_error("sidecar open: null argument or precision outside {-1, 0, 1}");
    return GLM5X_INVALID_STATE;
  }
  *out = nullptr;
  auto* h = new glm5x_sidecar;
  std::string msg;
  const int rc = glm5x::read_sidecar(path, precision, source_digest, &h->sc, &msg);
  if (rc != 0) {
    glm5x::set_last_error(msg.c_str());
    delete h;
    return static_cast<glm5x_status>(rc);
  }
  *out = h;
  return GLM5X_OK;
}

void glm5x_sidecar_close(glm5x_sidecar* h) { delete h; }

glm5x_status glm5x_sidecar_get_role(const glm5x_sidecar* h, int32_t role, glm5x_sidecar_role* out) {
  if (!h || !out || role < 0 || role > 2) {
    glm5x::set_last_error("sidecar role: null argument or role outside [0, 2]");
    return GLM5X_INVALID_STATE;
  }
  const glm5x::SidecarRole& r = h->sc.roles[role];
  out->precision = h->sc.precision;
  out->rows = r.rows;
  out->cols = r.cols;
  out->group_size = r.group_size;
  out->packed = h->sc.payload.data() + r.packed_offset;
  out->packed_bytes = r.packed_bytes;
  out->scales = h->sc.payload.data() + r.scale_offset;
  out->scale_bytes = r.scale_bytes;
  out->global_scale = r.global_scale;
  return GLM5X_OK;
}

glm5x_status glm5x_sidecar_path(const char* root, int32_t layer, int32_t expert,
                                int32_t precision, char* buf, size_t capacity) {
  if (!root || !buf || layer < 0 || expert < 0 || (precision != 0 && precision != 1)) {
    glm5x::set_last_error("GLM5X_PACKED_CACHE_KEY: negative layer / expert or bad precision");
    return GLM5X_INVALID_STATE;
  }
  const int n = std::snprintf(buf, capacity, "%s/layer-%04d-expert-%04d.%s", root, layer, expert,
                              precision == 0 ? "pn4" : "pm4");
  if (n < 0 || static_cast<size_t>(n) >= capacity) {
    glm5x::set_last_error("sidecar path: buffer too small");
    return GLM5X_INVALID_EXTENT;
  }
  return GLM5X_OK;
}

}  // extern "C"

