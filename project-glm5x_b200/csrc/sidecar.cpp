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

#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace glm5x {

// ------------------------------------------------------------------ CRC32C
static uint32_t crc32c_table[8][256];
static bool crc_init_done = false;

static void crc_init() {
  for (uint32_t i = 0; i < 256; ++i) {
    uint32_t c = i;
    for (int k = 0; k < 8; ++k) c = (c & 1) ? (c >> 1) ^ 0x82F63B78u : c >> 1;
    crc32c_table[0][i] = c;
  }
  for (uint32_t i = 0; i < 256; ++i)
    for (int t = 1; t < 8; ++t)
      crc32c_table[t][i] = (crc32c_table[t - 1][i] >> 8) ^ crc32c_table[0][crc32c_table[t - 1][i] & 0xff];
  crc_init_done = true;
}

uint32_t crc32c(const uint8_t* data, size_t n) {
  if (!crc_init_done) crc_init();
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

int read_sidecar(const char* path, Sidecar* out, std::string* msg) {
  std::ifstream f(path, std::ios::binary);
  if (!f) {
    *msg = std::string("cannot open sidecar ") + path;
    return kSidecarIo;
  }
  std::vector<uint8_t> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  if (bytes.size() < 16) {
    *msg = "sidecar shorter than its header";
    return kSidecarTruncated;
  }
  if (std::memcmp(bytes.data(), "GLM5XPI4", 8) != 0) {
    *msg = "sidecar magic is not GLM5XPI4";
    return kSidecarMagic;
  }
  uint32_t version, json_len;
  std::memcpy(&version, bytes.data() + 8, 4);
  std::memcpy(&json_len, bytes.data() + 12, 4);
  if (version != 1) {
    *msg = "unsupported sidecar version";
    return kSidecarVersion;
  }
  if (16ull + json_len > bytes.size()) {
    *msg = "sidecar metadata truncated";
    return kSidecarTruncated;
  }
  Parser ps{reinterpret_cast<const char*>(bytes.data() + 16),
            reinterpret_cast<const char*>(bytes.data() + 16 + json_len)};
  Json meta = ps.value();
  if (!ps.ok || meta.kind != Json::Obj) {
    *msg = "sidecar metadata is not a JSON object";
    return kSidecarExtent;
  }
  const Json* fmt = meta.get("format");
  const Json* roles = meta.get("roles");
  int64_t payload_bytes = 0;
  if (!fmt || fmt->kind != Json::Str || !roles || roles->kind != Json::Arr ||
      roles->arr.size() != 3 || !get_int(meta, "payload_bytes", &payload_bytes)) {
    *msg = "sidecar metadata lacks format/roles/payload_bytes";
    return kSidecarExtent;
  }
  if (fmt->str == "glm5x-nvfp4-expert-v1")
    out->precision = 0;
  else if (fmt->str == "glm5x-mxfp4-expert-v1")
    out->precision = 1;
  else {
    *msg = "unsupported sidecar format " + fmt->str;
    return kSidecarExtent;
  }
  const size_t base = 16ull + json_len;
  if (base + static_cast<uint64_t>(payload_bytes) != bytes.size()) {
    *msg = "sidecar payload size mismatch";
    return kSidecarTruncated;
  }
  out->payload.assign(bytes.begin() + base, bytes.end());
  for (int r = 0; r < 3; ++r) {
    const Json& role = roles->arr[r];
    SidecarRole& dst = out->roles[r];
    const Json* shape = role.get("shape");
    int64_t po, pb, qo, qb, pcrc, qcrc, group = 0;
    if (!shape || shape->kind != Json::Arr || shape->arr.size() != 2 ||
        !get_int(role, "packed_offset", &po) || !get_int(role, "packed_bytes", &pb) ||
        !get_int(role, "qparams_offset", &qo) || !get_int(role, "qparams_bytes", &qb) ||
        !get_int(role, "packed_crc32c", &pcrc) || !get_int(role, "qparams_crc32c", &qcrc)) {
      *msg = "sidecar role metadata incomplete";
      return kSidecarExtent;
    }
    get_int(role, "group_size", &group);
    dst.rows = static_cast<int64_t>(shape->arr[0].num);
    dst.cols = static_cast<int64_t>(shape->arr[1].num);
    dst.group_size = group;
    if (po < 0 || pb < 0 || qo < 0 || qb < 0 || po + pb > payload_bytes ||
        qo + qb > payload_bytes || dst.rows <= 0 || dst.cols <= 0 ||
        pb != dst.rows * dst.cols / 2) {
      *msg = "sidecar role extents out of range";
      return kSidecarExtent;
    }
    const uint8_t* pp = out->payload.data() + po;
    const uint8_t* qp = out->payload.data() + qo;
    if (crc32c(pp, pb) != static_cast<uint32_t>(pcrc)) {
      *msg = "sidecar packed CRC32C mismatch";
      return kSidecarDataCrc;
    }
    if (crc32c(qp, qb) != static_cast<uint32_t>(qcrc)) {
      *msg = "sidecar qparams CRC32C mismatch";
      return kSidecarAuxCrc;
    }
    dst.packed_offset = po;
    dst.packed_bytes = pb;
    if (out->precision == 0) {
      int64_t sb = 0, gb = 0;
      if (!get_int(role, "scale_bytes", &sb) || !get_int(role, "global_scale_bytes", &gb) ||
          gb != 4 || sb + gb != qb) {
        *msg = "NVFP4 qparams extent mismatch";
        return kSidecarExtent;
      }
      dst.scale_offset = qo;
      dst.scale_bytes = sb;
      std::memcpy(&dst.global_scale, qp + sb, 4);
    } else {
      dst.scale_offset = qo;
      dst.scale_bytes = qb;
      dst.global_scale = 1.0f;
    }
  }
  return 0;
}

}  // namespace glm5x
