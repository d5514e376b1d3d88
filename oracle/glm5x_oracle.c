/*
 * glm5x_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's CPU algorithms for the routed-expert
 * MoE path (rsb1813/project-glm5x). Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / --impl reference legs may load this library, and
 * only as the checker; the product path never calls it.
 *
 * Parity pinning: tests/golden/ holds fixtures produced by the reference's own
 * Python modules (tests/golden/make_golden.py) and the reference's C++ sources
 * compiled into oracle/_ref (oracle/Makefile); tests/test_oracle_golden.py
 * checks every function below against both.
 *
 * Reference citations are paths inside the reference project.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* E2M1 codebook in the reference's index order
 * (reference/glm5x_ref/nvfp4.py:10-13, reference/k3x_ref/mxfp4.py:7-26). */
static const float ORC_E2M1[16] = {0.0f,  0.5f,  1.0f,  1.5f,  2.0f,  3.0f,
                                   4.0f,  6.0f,  -0.0f, -0.5f, -1.0f, -1.5f,
                                   -2.0f, -3.0f, -4.0f, -6.0f};

static const float ORC_NVFP4_FACTORS[9] = {0.5f,  0.625f, 0.75f, 0.875f, 1.0f,
                                           1.125f, 1.25f, 1.5f,  2.0f};

float orc_e2m1_value(int code) { return ORC_E2M1[code & 15]; }

/* argmin_i |v - codebook[i]| with the first index winning ties: torch.argmin
 * semantics used at nvfp4.py:150-152,168-170 and mxfp4.py:77-79,91-93. */
int orc_e2m1_encode(float v) {
  float best = fabsf(v - ORC_E2M1[0]);
  int best_i = 0;
  for (int i = 1; i < 16; ++i) {
    const float d = fabsf(v - ORC_E2M1[i]);
    if (d < best) {
      best = d;
      best_i = i;
    }
  }
  return best_i;
}

/* float -> float8_e4m3fn, round-to-nearest-even, saturating to 448 (the
 * reference always clamps into [2^-6, 448] before the cast, nvfp4.py:131-134,
 * 139-144, so saturation never changes a reference result). */
uint8_t orc_e4m3_encode(float x) {
  uint32_t b;
  memcpy(&b, &x, 4);
  const uint32_t sign = (b >> 24) & 0x80u;
  b &= 0x7fffffffu;
  if (b == 0) return (uint8_t)sign;
  if (b >= 0x7f800000u) return (uint8_t)(sign | 0x7e); /* inf/nan: saturate */
  const int exp = (int)(b >> 23) - 127;
  if (exp < -6) {
    /* subnormal E4M3: m * 2^-9, m in [0, 8]; m == 8 is the smallest normal */
    const float q = x < 0 ? -x * 512.0f : x * 512.0f;
    const float m = nearbyintf(q); /* default rounding mode: nearest-even */
    return (uint8_t)(sign | (uint8_t)m);
  }
  const uint32_t rounded = (b + 0x7ffffu + ((b >> 20) & 1u)) & ~0xfffffu;
  const int e = (int)(rounded >> 23) - 127;
  const uint32_t mant = (rounded >> 20) & 7u;
  if (e > 8 || (e == 8 && mant == 7)) return (uint8_t)(sign | 0x7e);
  return (uint8_t)(sign | (uint32_t)((e + 7) << 3) | mant);
}

float orc_e4m3_decode(uint8_t c) {
  const int e = (c >> 3) & 15;
  const int m = c & 7;
  float v;
  if (e == 15 && m == 7) return NAN;
  if (e == 0)
    v = ldexpf((float)m, -9);
  else
    v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
  return (c & 0x80) ? -v : v;
}

/* ---------------------------------------------------------------------- */
/* NVFP4 (16-element blocks, E4M3 block scale, FP32 global scale)          */
/* ---------------------------------------------------------------------- */

/* Sum of 16 squared errors in the order torch 2.x's CPU reduction uses for a
 * contiguous 16-wide `mean(dim=-1)` (eight interleaved lanes, folded in
 * order); it only decides exact near-ties of the MSE candidate search
 * (nvfp4.py:153-156). */
static float orc_sum16(const float* sq) {
  float lane[8];
  for (int j = 0; j < 8; ++j) lane[j] = sq[j] + sq[j + 8];
  float s = lane[0];
  for (int j = 1; j < 8; ++j) s = s + lane[j];
  return s;
}

/* _quantize_payload (reference/glm5x_ref/nvfp4.py:101-177).
 * src: [rows, cols] FP32. packed: [rows, cols/2]. scales: row-major
 * [rows, cols/16] E4M3 bytes (NOT blocked). Returns 0 on success. */
int orc_nvfp4_quantize(const float* src, int64_t rows, int64_t cols, int mse,
                       uint8_t* packed, uint8_t* scales, float* global_out) {
  if (rows <= 0 || cols <= 0 || cols % 16 || cols % 2) return -1;
  const int64_t nb = cols / 16;
  float maximum = 0.0f;
  for (int64_t i = 0; i < rows * cols; ++i) {
    if (!isfinite(src[i])) return -2;
    const float a = fabsf(src[i]);
    if (a > maximum) maximum = a;
  }
  /* nvfp4.py:127-130: max(maximum / (448*6), 1e-12) in FP32 */
  float g = maximum / 2688.0f;
  if (!(g >= 1e-12f)) g = 1e-12f;
  const float six_g = 6.0f * g;
  const float tiny = 0.015625f; /* torch.finfo(float8_e4m3fn).tiny = 2^-6 */
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t b = 0; b < nb; ++b) {
      const float* x = src + r * cols + b * 16;
      float bmax = 0.0f;
      for (int i = 0; i < 16; ++i) {
        const float a = fabsf(x[i]);
        if (a > bmax) bmax = a;
      }
      float base = bmax / six_g; /* nvfp4.py:131-134 */
      if (base < tiny) base = tiny;
      if (base > 448.0f) base = 448.0f;
      uint8_t codes[16];
      uint8_t sel_byte;
      if (mse) {
        /* nvfp4.py:139-163 */
        float best_err = 0.0f;
        int best = -1;
        uint8_t best_codes[16];
        uint8_t best_byte = 0;
        for (int c = 0; c < 9; ++c) {
          float cand = base * ORC_NVFP4_FACTORS[c];
          if (cand < tiny) cand = tiny;
          if (cand > 448.0f) cand = 448.0f;
          const uint8_t cbyte = orc_e4m3_encode(cand);
          const float cs = orc_e4m3_decode(cbyte);
          const float denom = cs * g;
          uint8_t cc[16];
          float sq[16];
          for (int i = 0; i < 16; ++i) {
            const int code = orc_e2m1_encode(x[i] / denom);
            cc[i] = (uint8_t)code;
            const float rec = ORC_E2M1[code] * denom;
            const float d = rec - x[i];
            sq[i] = d * d;
          }
          const float err = orc_sum16(sq) / 16.0f;
          if (best < 0 || err < best_err) {
            best = c;
            best_err = err;
            memcpy(best_codes, cc, 16);
            best_byte = cbyte;
          }
        }
        memcpy(codes, best_codes, 16);
        sel_byte = best_byte;
      } else {
        /* nvfp4.py:164-170 */
        sel_byte = orc_e4m3_encode(base);
        const float denom = orc_e4m3_decode(sel_byte) * g;
        for (int i = 0; i < 16; ++i) codes[i] = (uint8_t)orc_e2m1_encode(x[i] / denom);
      }
      scales[r * nb + b] = sel_byte;
      uint8_t* p = packed + r * (cols / 2) + b * 8;
      for (int i = 0; i < 8; ++i) p[i] = (uint8_t)(codes[2 * i] | (codes[2 * i + 1] << 4));
    }
  }
  *global_out = g;
  return 0;
}

/* _to_blocked (nvfp4.py:23-40): row-major [rows, cols] scale bytes -> the
 * 128x4 tiled layout (flattened (32,16) chunks, zero padding). */
int64_t orc_blocked_size(int64_t rows, int64_t cols) {
  return ((rows + 127) / 128) * ((cols + 3) / 4) * 512;
}

void orc_to_blocked(const uint8_t* rm, int64_t rows, int64_t cols, uint8_t* out) {
  const int64_t rb = (rows + 127) / 128, cb = (cols + 3) / 4;
  memset(out, 0, (size_t)(rb * cb * 512));
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c) {
      const int64_t chunk = (r / 128) * cb + c / 4;
      const int64_t rr = r % 128;
      out[chunk * 512 + (rr % 32) * 16 + (rr / 32) * 4 + (c % 4)] = rm[r * cols + c];
    }
}

/* _from_blocked (nvfp4.py:43-55) */
void orc_from_blocked(const uint8_t* bl, int64_t rows, int64_t cols, uint8_t* rm) {
  const int64_t cb = (cols + 3) / 4;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c) {
      const int64_t chunk = (r / 128) * cb + c / 4;
      const int64_t rr = r % 128;
      rm[r * cols + c] = bl[chunk * 512 + (rr % 32) * 16 + (rr / 32) * 4 + (c % 4)];
    }
}

/* dequantize_nvfp4 (nvfp4.py:201-217): E2M1 value * (float(E4M3) * global). */
void orc_nvfp4_dequantize(const uint8_t* packed, const uint8_t* blocked, float g,
                          int64_t rows, int64_t cols, float* out) {
  const int64_t nb = cols / 16, cb = (nb + 3) / 4;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c) {
      const int64_t b = c / 16;
      const int64_t chunk = (r / 128) * cb + b / 4;
      const int64_t rr = r % 128;
      const uint8_t sb = blocked[chunk * 512 + (rr % 32) * 16 + (rr / 32) * 4 + (b % 4)];
      const float s = orc_e4m3_decode(sb) * g;
      const uint8_t byte = packed[r * (cols / 2) + c / 2];
      const int code = (c & 1) ? (byte >> 4) : (byte & 15);
      out[r * cols + c] = ORC_E2M1[code] * s;
    }
}

/* ---------------------------------------------------------------------- */
/* MXFP4 (32-element groups, E8M0 scale)                                   */
/* ---------------------------------------------------------------------- */

/* encode_mxfp4 (reference/k3x_ref/mxfp4.py:31-107). Scales are row-major
 * [rows * cols / group] bytes. Returns 0, or -1 (shape), -2 (non-finite),
 * -3 (exponent > 126). */
int orc_mxfp4_encode(const float* src, int64_t rows, int64_t cols, int group, int mse,
                     uint8_t* packed, uint8_t* scales) {
  static const int offsets[7] = {-4, -3, -2, -1, 0, 1, 2};
  if (rows <= 0 || cols <= 0 || group <= 0 || cols % group || cols % 2) return -1;
  const int64_t ng = rows * cols / group;
  for (int64_t i = 0; i < rows * cols; ++i)
    if (!isfinite(src[i])) return -2;
  for (int64_t gi = 0; gi < ng; ++gi) {
    const float* x = src + gi * group;
    float m = 0.0f;
    for (int i = 0; i < group; ++i) {
      const float a = fabsf(x[i]);
      if (a > m) m = a;
    }
    int e;
    if (m > 0.0f) {
      /* mxfp4.py:62: torch.ceil(torch.log2(max / 6.0)) in FP32 */
      const float l = log2f(m / 6.0f);
      const float ce = ceilf(l);
      if (ce > 126.0f) return -3;
      e = (int)ce;
      if (e < -127) e = -127;
    } else {
      e = -127;
    }
    int sel_e = e;
    uint8_t codes[64];
    if (group > 64) return -1;
    if (mse) {
      /* mxfp4.py:80-97 */
      float best_err = 0.0f;
      int best = -1;
      for (int c = 0; c < 7; ++c) {
        int ce = e + offsets[c];
        if (ce < -127) ce = -127;
        if (ce > 126) ce = 126;
        const float sc = ldexpf(1.0f, ce);
        uint8_t cc[64];
        double unused = 0;
        (void)unused;
        float sum = 0.0f;
        float sq[64];
        for (int i = 0; i < group; ++i) {
          const int code = orc_e2m1_encode(x[i] / sc);
          cc[i] = (uint8_t)code;
          const float d = ORC_E2M1[code] * sc - x[i];
          sq[i] = d * d;
        }
        /* mean over the group (dim=1 of a [G, group, 7] view: strided, summed
         * in index order) */
        for (int i = 0; i < group; ++i) sum += sq[i];
        const float err = sum / (float)group;
        if (best < 0 || err < best_err) {
          best = c;
          best_err = err;
          memcpy(codes, cc, (size_t)group);
          sel_e = ce;
        }
      }
    } else {
      const float sc = ldexpf(1.0f, e);
      for (int i = 0; i < group; ++i) codes[i] = (uint8_t)orc_e2m1_encode(x[i] / sc);
    }
    scales[gi] = (uint8_t)(sel_e + 127);
    for (int i = 0; i < group / 2; ++i)
      packed[gi * (group / 2) + i] = (uint8_t)(codes[2 * i] | (codes[2 * i + 1] << 4));
  }
  return 0;
}

/* decode_mxfp4 (mxfp4.py:110-144; runtime/src/ops.cpp:40-63): rejects 0xFF. */
int orc_mxfp4_decode(const uint8_t* packed, const uint8_t* scales, int64_t rows,
                     int64_t cols, int group, float* out) {
  if (rows <= 0 || cols <= 0 || group <= 0 || cols % group || cols % 2) return -1;
  const int64_t n = rows * cols;
  for (int64_t i = 0; i < n / group; ++i)
    if (scales[i] == 0xff) return -4;
  for (int64_t i = 0; i < n; ++i) {
    const uint8_t byte = packed[i / 2];
    const int code = (i & 1) ? (byte >> 4) : (byte & 15);
    out[i] = ldexpf(ORC_E2M1[code], (int)scales[i / group] - 127);
  }
  return 0;
}

/* ---------------------------------------------------------------------- */
/* Routing                                                                 */
/* ---------------------------------------------------------------------- */

/* select_routing, natural mode (runtime/src/routing_policy.cpp:31-159):
 * stable descending sort on score+bias (ties keep the lower expert index),
 * natural top-k, weights = score / sum(scores of the selected, summed in
 * slot order). Returns 0, or -1 on the reference's validation failures. */
int orc_select_routing(const float* scores, const float* bias, int n, int k,
                       int32_t* ids, float* weights) {
  if (n <= 0 || k <= 0 || k > n) return -1;
  float* adj = (float*)malloc(sizeof(float) * (size_t)n);
  int32_t* order = (int32_t*)malloc(sizeof(int32_t) * (size_t)n);
  for (int i = 0; i < n; ++i) {
    if (!isfinite(scores[i]) || scores[i] < 0.0f || scores[i] > 1.0f || !isfinite(bias[i])) {
      free(adj);
      free(order);
      return -1;
    }
    adj[i] = scores[i] + bias[i];
    if (!isfinite(adj[i])) {
      free(adj);
      free(order);
      return -1;
    }
    order[i] = i;
  }
  /* stable insertion of the top k: an element moves ahead only when strictly
   * greater, matching std::stable_sort with `adjusted[l] > adjusted[r]`. */
  for (int i = 1; i < n; ++i) {
    const int32_t v = order[i];
    int j = i - 1;
    while (j >= 0 && adj[v] > adj[order[j]]) {
      order[j + 1] = order[j];
      --j;
    }
    order[j + 1] = v;
  }
  float denom = 0.0f;
  for (int s = 0; s < k; ++s) denom += scores[order[s]];
  if (!isfinite(denom) || denom <= 0.0f) {
    free(adj);
    free(order);
    return -1;
  }
  for (int s = 0; s < k; ++s) {
    ids[s] = order[s];
    weights[s] = scores[order[s]] / denom;
  }
  free(adj);
  free(order);
  return 0;
}

/* build_learned_routes (runtime/src/cuda_glm5x_real_expert_bench.cpp:287-328):
 * sequential FP32 dot product for each logit, sigmoid 1/(1+exp(-l)), natural
 * select_routing, contribution = weight * routed_scale. hidden [T,H],
 * router [E,H], bias [E]; outputs logits [T,E] (may be NULL), ids/weights
 * [T,k]. */
int orc_route_tokens(const float* hidden, const float* router, const float* bias,
                     int64_t T, int64_t H, int E, int k, float routed_scale,
                     float* logits, int32_t* ids, float* weights) {
  float* scores = (float*)malloc(sizeof(float) * (size_t)E);
  for (int64_t t = 0; t < T; ++t) {
    const float* x = hidden + t * H;
    for (int e = 0; e < E; ++e) {
      const float* w = router + (int64_t)e * H;
      float logit = 0.0f;
      for (int64_t i = 0; i < H; ++i) logit += x[i] * w[i];
      if (logits) logits[t * E + e] = logit;
      scores[e] = 1.0f / (1.0f + expf(-logit));
    }
    const int rc = orc_select_routing(scores, bias, E, k, ids + t * k, weights + t * k);
    if (rc) {
      free(scores);
      return rc;
    }
    for (int s = 0; s < k; ++s) weights[t * k + s] = weights[t * k + s] * routed_scale;
  }
  free(scores);
  return 0;
}

/* select_routing with a Top-K policy (runtime/src/routing_policy.cpp:31-159):
 * mode 0 natural, 1 fixed (fixed_k), 2 adaptive (k must be 16), floor_k the
 * quality floor. Validation as routing_policy.cpp:41-70; the decision
 * scalars in the reference's FP32 operation order (:89-150). Outputs:
 * ids[k] / weights[k] in natural order with -1 / 0 past the selected K,
 * sel[2] = (selected K, quality floor escalated), diag[4] = (normalized
 * entropy, entropy effective support, selected cumulative mass, boundary
 * confidence). Returns 0, or -1 where the reference fails. */
static int orc_in_ladder(int k) { return k == 4 || k == 6 || k == 8 || k == 12 || k == 16; }

static float orc_boundary_confidence(const float* p, int k, int selected) {
  if (selected >= k) return 1.0f;
  float gap = p[selected - 1] - p[selected];
  if (gap < 0.0f) gap = 0.0f;
  const float top = p[0] > 1.17549435e-38f ? p[0] : 1.17549435e-38f;
  return gap / top;
}

static int orc_choose_adaptive(const float* p, int k, int floor_k, float support,
                               float mass_target, float min_gap) {
  const float eps = 1.0e-5f;
  float cumulative = 0.0f;
  for (int slot = 0; slot < k; ++slot) {
    cumulative += p[slot];
    const int candidate = slot + 1;
    if (!orc_in_ladder(candidate) || candidate < floor_k) continue;
    const float confidence = orc_boundary_confidence(p, k, candidate);
    if (cumulative + eps >= mass_target && (float)candidate + eps >= support &&
        confidence + eps >= min_gap)
      return candidate;
  }
  return k;
}

int orc_select_routing_policy(const float* scores, const float* bias, int n, int k, int mode,
                              int fixed_k, float mass_target, float min_gap, int floor_k,
                              int32_t* ids, float* weights, int32_t* sel, float* diag) {
  if (n <= 0 || k <= 0 || k > n || k > 16) return -1;
  if (!isfinite(mass_target) || mass_target <= 0.0f || mass_target > 1.0f ||
      !isfinite(min_gap) || min_gap < 0.0f || min_gap > 1.0f)
    return -1;
  if (floor_k != 0 && (!orc_in_ladder(floor_k) || (mode != 0 && floor_k > k))) return -1;
  if (mode == 1 && (!orc_in_ladder(fixed_k) || fixed_k > k)) return -1;
  if (mode == 2 && k != 16) return -1;
  if (mode < 0 || mode > 2) return -1;
  int32_t order[16];
  float top[16];
  int32_t nat[16];
  float nat_w[16];
  /* the natural order and weights of the natural Top-k */
  if (orc_select_routing(scores, bias, n, k, nat, nat_w)) return -1;
  for (int s = 0; s < k; ++s) {
    order[s] = nat[s];
    top[s] = scores[nat[s]];
  }
  float denom = 0.0f;
  for (int s = 0; s < k; ++s) denom += top[s];
  float p[16];
  float entropy = 0.0f;
  for (int s = 0; s < k; ++s) {
    p[s] = top[s] / denom;
    if (p[s] > 0.0f) entropy -= p[s] * logf(p[s]);
  }
  const float support = expf(entropy);
  int selected = k, unfloored = k;
  if (mode == 1) {
    unfloored = fixed_k;
    selected = fixed_k > floor_k ? fixed_k : floor_k;
  } else if (mode == 2) {
    unfloored = orc_choose_adaptive(p, k, 0, support, mass_target, min_gap);
    selected = orc_choose_adaptive(p, k, floor_k, support, mass_target, min_gap);
  }
  float sdenom = 0.0f;
  for (int s = 0; s < selected; ++s) sdenom += top[s];
  if (!isfinite(sdenom) || sdenom <= 0.0f) return -1;
  for (int s = 0; s < k; ++s) {
    ids[s] = s < selected ? order[s] : -1;
    weights[s] = s < selected ? top[s] / sdenom : 0.0f;
  }
  if (sel) {
    sel[0] = selected;
    sel[1] = selected > unfloored;
  }
  if (diag) {
    float mass = 0.0f;
    for (int s = 0; s < selected; ++s) mass += p[s];
    diag[0] = k == 1 ? 0.0f : entropy / logf((float)k);
    diag[1] = support;
    diag[2] = mass;
    diag[3] = orc_boundary_confidence(p, k, selected);
  }
  return 0;
}

/* verify_greedy_target_block (runtime/src/speculative.cpp:8-21, 75-113):
 * candidates[n] after `anchor`, targets[n_targets]. Returns 0 (committed[0 ..
 * *accepted] filled), 9 (invalid extent) or 16 (invalid state). */
int orc_verify_greedy_target_block(uint32_t anchor, const uint32_t* candidates, int n,
                                   int max_draft, uint32_t vocab, const uint32_t* targets,
                                   int n_targets, int* accepted, uint32_t* committed) {
  if (vocab == 0 || anchor >= vocab || n > max_draft) return 9;
  for (int i = 0; i < n; ++i)
    if (candidates[i] >= vocab) return 9;
  if (n_targets == 0 || n_targets - 1 != n) return 9;
  for (int i = 0; i < n_targets; ++i)
    if (targets[i] >= vocab) return 16;
  int a = 0;
  for (; a < n; ++a) {
    if (candidates[a] != targets[a]) break;
    committed[a] = candidates[a];
  }
  committed[a] = a < n ? targets[a] : targets[n_targets - 1];
  *accepted = a;
  return 0;
}

/* ---------------------------------------------------------------------- */
/* Dense SwiGLU expert (CPU reference path)                                */
/* ---------------------------------------------------------------------- */

/* CpuBackend::dense_situ_mlp(..., MlpActivation::silu)
 * (runtime/src/backend_cpu.cpp:23-46, 107-128; runtime/src/ops.cpp:32-38):
 * every projection is a double-accumulated dot product rounded to FP32, the
 * activation is gate * (1 / (1 + exp(-gate))) * up in FP32. */
void orc_dense_silu_mlp(const float* x, const float* gate, const float* up,
                        const float* down, int64_t H, int64_t I, float* out) {
  float* act = (float*)malloc(sizeof(float) * (size_t)I);
  for (int64_t r = 0; r < I; ++r) {
    double sg = 0.0, su = 0.0;
    const float* wg = gate + r * H;
    const float* wu = up + r * H;
    for (int64_t c = 0; c < H; ++c) {
      sg += (double)wg[c] * x[c];
      su += (double)wu[c] * x[c];
    }
    const float g = (float)sg, u = (float)su;
    const float sig = 1.0f / (1.0f + expf(-g));
    act[r] = g * sig * u;
  }
  for (int64_t r = 0; r < H; ++r) {
    double s = 0.0;
    const float* wd = down + r * I;
    for (int64_t c = 0; c < I; ++c) s += (double)wd[c] * act[c];
    out[r] = (float)s;
  }
  free(act);
}

/* FP32-input matrix product with double accumulation, out[m, n] =
 * sum_k a[m, k] * b[n, k]; the dequant-matmul oracle's inner product
 * (mxfp4_matmul, runtime/src/ops.cpp:65-84). */
void orc_matmul_nt(const float* a, const float* b, int64_t M, int64_t N, int64_t K,
                   float* out) {
  for (int64_t m = 0; m < M; ++m)
    for (int64_t n = 0; n < N; ++n) {
      double s = 0.0;
      const float* pa = a + m * K;
      const float* pb = b + n * K;
      for (int64_t kk = 0; kk < K; ++kk) s += (double)pa[kk] * pb[kk];
      out[m * N + n] = (float)s;
    }
}
