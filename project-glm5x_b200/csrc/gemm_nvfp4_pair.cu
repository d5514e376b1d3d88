// gemm_nvfp4_pair.cu -- grouped NVFP4 GEMM on CTA pairs (tcgen05 cta_group::2).
//
// Same contract and epilogues as gemm_nvfp4.cu (the reference's NVFP4
// projections, reference/glm5x_ref/nvfp4.py:220-233 / nvfp4_batched.py:64-151,
// with SwiGLU and the routing weight fused), for token tiles up to 256 rows.
// A cluster of two CTAs on neighbouring SMs computes a 256-weight-row x
// N-token tile with M = 256 MMAs: each CTA loads its own 128 weight rows and
// half of the N token rows, so per FLOP each SM moves two thirds of the bytes
// a single-CTA 128 x 256 tile moves. Each CTA also loads its weight rows'
// scale chunks and all N rows' scale chunks (the MMA reads every column's
// scales from each CTA's own TMEM).
//
// Roles (per CTA, 512 threads, four warpgroups):
//   warp 0     this CTA's TMA loads of its weight rows and token rows,
//              counted on the leader CTA's full barrier, plus its scale
//              chunks (bulk copies on its own full_sf barrier);
//   warp 1     TMEM (pair allocation); in the leader it issues the pair MMAs
//              once both CTAs' operands have landed and both CTAs' scales are
//              in TMEM, and its commits arrive on both CTAs' barriers;
//   warps 2-5  scale staging into this CTA's TMEM with tcgen05.st (one warp
//              per lane quadrant), then an arrive on the leader's full
//              barrier: a stage's full barrier completes when the operand
//              bytes of both CTAs have landed and all eight staging warps
//              have arrived, so the MMA thread waits once per stage (each
//              wait costs the single issuing thread ~70 cycles even when the
//              barrier is already complete);
//   warps 8-15 epilogue: drain this CTA's accumulator half to registers,
//              signal the leader, then SwiGLU / routing weight and stores.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "glm5x_kernels.cuh"
#include "glm5x_ptx.cuh"

namespace glm5x {
namespace {

constexpr int kPM = 256;           // weight rows per pair tile (128 per CTA)
constexpr int kBN = 256;           // token rows per pair tile (up to 128 per CTA)
constexpr int kBK = 128;           // K bytes per stage (256 FP4)
constexpr int kChunk = 512;        // one 128-row x 4-scale chunk
constexpr int kEpiWarps = 8;
constexpr int kEpiWarp0 = 8;
constexpr int kThreads = 512;
constexpr uint32_t kRegsLow = 80;
constexpr uint32_t kRegsEpi = 176;
static_assert(256 * kRegsLow + 256 * kRegsEpi <= 65536, "register split");
constexpr int kStages = 5;
// Stage loads in each CTA: 0 = warp 0 issues everything; 1 = warp 6 takes
// the token rows; 2 = warp 6 takes the scale chunks (one issuing thread
// streams copies at a lower rate than two).
#ifndef G5_PAIR_SPLIT
#define G5_PAIR_SPLIT 0
#endif
constexpr int kABytes = 128 * kBK;           // this CTA's weight rows
constexpr int kBBytes = 128 * kBK;           // this CTA's token rows
constexpr int kSfaBytes = 4 * kChunk;
constexpr int kSfbBytes = 2 * 4 * kChunk;    // both 128-row scale blocks of the tile
constexpr int kStageBytes = ((kABytes + kBBytes + kSfaBytes + kSfbBytes + 1023) / 1024) * 1024;
constexpr int kSfaCols = 16, kSfbCols = 32;
constexpr int kSfBase = kBN;                 // one accumulator of kBN columns
constexpr int kTmemCols = 512;
static_assert(kSfBase + kStages * (kSfaCols + kSfbCols) <= kTmemCols, "TMEM budget");
constexpr int kMaxSeg = 260;
constexpr size_t kSmem = (size_t)kStages * kStageBytes + 1024 + 256;
static_assert((3 * kStages + 3) * 8 + 4 <= 256, "barrier area");

struct PairTile {
  int seg, m2, row_start, n_valid;
};

// The tile list of one launch, held in shared memory: per segment its
// token-tile prefix, row count and first row, and the group boundaries of
// the tile order.
//
// Order. gt == 0: segment-major (a segment's weight tiles in turn, each
// with its token tiles next to one another). gt > 0: the segments are cut
// into groups by where their first token tile falls (group g holds the
// segments whose tile prefix is in [g * gt, (g + 1) * gt)), and a group's
// tiles run weight-tile-major: weight tile 0 of every segment in the group,
// then weight tile 1, and so on. Routed loads are skewed (at config 5 an
// expert gets 0 to ~900 rows), so in segment order the pairs running at
// one time work on two or three experts: all light ones (their weights
// streamed from HBM for a few rows, the tensor pipe idle) or all heavy ones
// (weights reused from L2, HBM idle). In group order they run the same
// weight tile of tens of experts, light and heavy together, and HBM and the
// tensor pipe are busy at the same time; a group's token rows (gt tiles of
// at most 256 rows) stay in L2 across its weight tiles, and each
// (segment, weight tile) slab is still read once, by the pairs that run its
// token tiles side by side.
//
// Decoding. A tile's segment comes from a table of every token tile's
// segment (seg_tt, built at launch when the launch has at most kMaxTT token
// tiles) instead of binary searches: one lookup against ~9 dependent
// shared-memory loads per search, which the MMA-issuing thread otherwise
// paid (~2000 cycles per tile with two searches) between tiles. 768 entries
// cover every launch of up to ~17k tokens per GPU at top-8 of 256 experts
// (C5's 8192 tokens make ~450 token tiles); larger launches search.
constexpr int kMaxTT = 768;
struct PairMap {
  int32_t ntp[kMaxSeg + 1], cnt[kMaxSeg], start[kMaxSeg + 1], gseg[kMaxSeg + 2];
  uint16_t seg_tt[kMaxTT];
  int nseg, m2_tiles, gt, table;
};
// the down projection's epilogue stages 8 token rows x 32 features of BF16 y
// per epilogue warp (512 bytes) to store them as 16-byte pieces
template <int EPI>
constexpr int kYStageBytes = EPI == 1 ? kEpiWarps * 512 : 16;
static_assert(kSmem + sizeof(PairMap) + kYStageBytes<1> + 128 <= 232448,
              "shared memory budget");

// largest s in [lo, hi) with ntp[s] <= key (ntp non-decreasing, ntp[lo] <= key)
__device__ __forceinline__ int seg_search(const int32_t* __restrict__ ntp, int lo, int hi,
                                          int key) {
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (ntp[mid] <= key) lo = mid; else hi = mid;
  }
  return lo;
}

// Every thread of the CTA; ends with the map complete and visible.
__device__ __forceinline__ void load_pair_map(PairMap& m, const GemmParams& p, int m2_tiles) {
  for (int i = threadIdx.x; i <= p.nseg; i += blockDim.x) {
    m.ntp[i] = p.ntile_prefix[i];
    m.start[i] = p.seg_start[i];
    if (i < p.nseg) m.cnt[i] = p.seg_count[i];
  }
  __syncthreads();
  const int nt = m.ntp[p.nseg];
  int gt = p.tile_group;
  if (gt > nt) gt = nt > 0 ? nt : 1;  // one group: weight-tile-major over all segments
  // at most kMaxSeg + 1 groups (their kMaxSeg + 2 boundaries fit gseg)
  if (gt > 0 && (nt + gt - 1) / gt > kMaxSeg + 1) gt = (nt + kMaxSeg) / (kMaxSeg + 1);
  if (gt > 0) {
    const int groups = (nt + gt - 1) / gt;
    for (int g = threadIdx.x; g <= groups; g += blockDim.x) {
      // first segment whose tile prefix reaches g * gt (nseg if none)
      int lo = 0, hi = p.nseg;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (m.ntp[mid] >= g * gt) hi = mid; else lo = mid + 1;
      }
      m.gseg[g] = lo;
    }
  }
  const bool table = nt <= kMaxTT;
  if (table)
    for (int sg = threadIdx.x; sg < p.nseg; sg += blockDim.x)
      for (int tt = m.ntp[sg]; tt < m.ntp[sg + 1]; ++tt) m.seg_tt[tt] = (uint16_t)sg;
  if (threadIdx.x == 0) {
    m.nseg = p.nseg;
    m.m2_tiles = m2_tiles;
    m.gt = gt;
    m.table = table ? 1 : 0;
  }
  __syncthreads();
}

__device__ __forceinline__ bool decode_pair_tile(int tile, const PairMap& m, PairTile& ti) {
  const int key = tile / m.m2_tiles;
  int s = m.table ? (int)m.seg_tt[key] : seg_search(m.ntp, 0, m.nseg, key);
  int n;
  if (m.gt > 0) {
    const int g = m.ntp[s] / m.gt;
    const int gs = m.gseg[g], ge = m.gseg[g + 1];
    const int base = m.ntp[gs], gnt = m.ntp[ge] - base;
    if (gnt <= 0) return false;
    const int local = tile - m.m2_tiles * base;
    ti.m2 = local / gnt;
    const int tt = base + (local - ti.m2 * gnt);
    s = m.table ? (int)m.seg_tt[tt] : seg_search(m.ntp, gs, ge, tt);
    n = tt - m.ntp[s];
  } else {
    const int nt = m.ntp[s + 1] - m.ntp[s];
    if (nt <= 0) return false;
    const int local = tile - m.m2_tiles * m.ntp[s];
    ti.m2 = local / nt;
    n = local - ti.m2 * nt;
  }
  ti.seg = s;
  ti.row_start = m.start[s] + n * kBN;
  const int left = m.cnt[s] - n * kBN;
  ti.n_valid = left < kBN ? left : kBN;
  return ti.n_valid > 0;
}

__device__ __forceinline__ uint16_t f2bf(float x) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

__device__ __forceinline__ float shfl_idx_ordered(float v, int src) {
  float r;
  asm volatile("shfl.sync.idx.b32 %0, %1, %2, 0x1f, 0xffffffff;" : "=f"(r) : "f"(v), "r"(src));
  return r;
}

// two floats rounded to BF16 (nearest even) in one word, lo in the low half
__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Epilogue warps 8-15 of both CTAs: drain this CTA's accumulator half to
// registers, hand it back to the leader, then SwiGLU (EPI 0, BF16 h and the
// slab amax) or the routing weight (EPI 1, BF16 y) and the stores.
template <int EPI>
__device__ __forceinline__ void pair_epilogue(const GemmParams& p, uint32_t tmem_base,
                                              uint64_t* tfull, uint64_t* tempty, int pair,
                                              int npairs, int total_tiles, const PairMap& s_map,
                                              uint32_t rank, int warp, int lane,
                                              uint8_t* ystage) {
    const int q = warp & 3;
    const int half_cols = (warp - kEpiWarp0) >> 2;
    const uint32_t lead_tempty = mapa_shared(smem_u32(tempty), 0);
    uint32_t acc_phase = 0;
    for (int tile = pair; tile < total_tiles; tile += npairs) {
      PairTile ti;
      if (!decode_pair_tile(tile, s_map, ti)) continue;
      if (!mbar_wait_cluster(tfull, acc_phase, p.err)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(32 * q) << 16);
      // drain to registers and hand the accumulator back before the math
      constexpr int kChunks = kBN / 64;
      uint32_t v[kChunks][32];
#pragma unroll
      for (int i = 0; i < kChunks; ++i)
        if (32 * half_cols + 64 * i < ti.n_valid) {
          if (EPI == 0) {
            tmem_ld_32x32b_x32(t_row + 32 * half_cols + 64 * i, v[i]);
          } else {
            tmem_ld_16x256b_x4(t_row + 32 * half_cols + 64 * i, v[i]);
            tmem_ld_16x256b_x4(t_row + (16u << 16) + 32 * half_cols + 64 * i, v[i] + 16);
          }
        }
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < kChunks; ++i) reg_fence(v[i]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster_relaxed(lead_tempty);
      acc_phase ^= 1u;
      const int m_tile = 2 * ti.m2 + (int)rank;  // this CTA's 128-row weight tile
      const float bscale = p.b_global[ti.seg];
      if (EPI == 0) {
        const float s_gate = bscale * p.a_global[2 * ti.seg];
        const float s_up = bscale * p.a_global[2 * ti.seg + 1];
        const bool lo = lane < 16;
        const int j = m_tile * 64 + 16 * q + (lane & 15);
        const int hcols = p.M_per / 2;
        float amax = 0.0f;
#pragma unroll
        for (int ch = 0; ch < kChunks; ++ch) {
          const int c0 = 32 * half_cols + 64 * ch;
          if (c0 >= ti.n_valid) break;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float send = __uint_as_float(lo ? v[ch][i + 16] : v[ch][i]);
            const float recv = __shfl_xor_sync(0xffffffffu, send, 16);
            const float gate = lo ? __uint_as_float(v[ch][i]) * s_gate : recv * s_gate;
            const float up = lo ? recv * s_up : __uint_as_float(v[ch][i + 16]) * s_up;
            const int col = c0 + i + (lo ? 0 : 16);
            if (col < ti.n_valid) {
              const float h = __fdividef(gate, 1.0f + __expf(-gate)) * up;
              const uint16_t hb = f2bf(h);
              amax = fmaxf(amax, fabsf(__uint_as_float((uint32_t)hb << 16)));
              p.out[(size_t)(ti.row_start + col) * hcols + j] = hb;
            }
          }
        }
        for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if (lane == 0 && amax > 0.0f)
          atomicMax(reinterpret_cast<unsigned int*>(p.h_amax + ti.seg), __float_as_uint(amax));
      } else {
        // v[ch] holds columns c0 .. c0 + 31 of this quadrant's 32 lanes as
        // 16x8 fragments (lanes 0-15 in v[ch][0..15], lanes 16-31 in
        // v[ch][16..31]): each thread has two neighbouring token columns of
        // four output features. Eight tokens at a time go through the warp's
        // 512-byte staging area (token row c: 32 features, 64 bytes, its
        // 16-byte piece m in slot m ^ ((c >> 1) & 3), so neither the
        // transposing stores nor the reads below meet a bank conflict), and
        // each lane then stores 16 bytes (8 features of one token) of y.
        const float scale = bscale * p.a_global[ti.seg];
        const uint32_t sbuf = smem_u32(ystage) + (uint32_t)(warp - kEpiWarp0) * 512u;
        const int sr = lane & 7, sm = lane >> 3;
        const uint32_t st_addr = sbuf + sr * 64 + 16 * (sm ^ ((sr >> 1) & 3));
        const int lr = lane >> 2;
        const uint32_t ld_addr = sbuf + lr * 64 + 16 * ((lane & 3) ^ ((lr >> 1) & 3));
        const int ycol = m_tile * 128 + 32 * q + 8 * (lane & 3);
#pragma unroll
        for (int ch = 0; ch < kChunks; ++ch) {
          const int c0 = 32 * half_cols + 64 * ch;
          if (c0 >= ti.n_valid) break;
          const float wmine =
              c0 + lane < ti.n_valid ? p.row_weight[ti.row_start + c0 + lane] * scale : 0.0f;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int cj = c0 + 8 * j;
            if (cj >= ti.n_valid) break;
            // volatile: kept in order with the staging stores, so the
            // compiler does not hoist every piece's weights at once (which
            // spilled next to the 128 accumulator registers)
            const float w0 = shfl_idx_ordered(wmine, 8 * j + 2 * (lane & 3));
            const float w1 = shfl_idx_ordered(wmine, 8 * j + 2 * (lane & 3) + 1);
            const uint32_t* a = v[ch] + 4 * j;
            const uint32_t* b = v[ch] + 16 + 4 * j;
            stmatrix_x4_trans(st_addr,
                              bf16x2_rn(__uint_as_float(a[0]) * w0, __uint_as_float(a[1]) * w1),
                              bf16x2_rn(__uint_as_float(a[2]) * w0, __uint_as_float(a[3]) * w1),
                              bf16x2_rn(__uint_as_float(b[0]) * w0, __uint_as_float(b[1]) * w1),
                              bf16x2_rn(__uint_as_float(b[2]) * w0, __uint_as_float(b[3]) * w1));
            __syncwarp();
            uint4 y;
            asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(y.x), "=r"(y.y), "=r"(y.z), "=r"(y.w)
                         : "r"(ld_addr)
                         : "memory");
            if (cj + lr < ti.n_valid)
              *reinterpret_cast<uint4*>(p.out + (size_t)(ti.row_start + cj + lr) * p.M_per +
                                        ycol) = y;
            __syncwarp();
          }
        }
      }
    }
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    nvfp4_pair_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                           const __grid_constant__ CUtensorMap tmap_b32,
                           const __grid_constant__ CUtensorMap tmap_b64,
                           const __grid_constant__ CUtensorMap tmap_b128, const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);  // leader's used
  uint64_t* empty = full + kStages;
  uint64_t* full_sf = empty + kStages;
  uint64_t* tfull = full_sf + kStages;
  uint64_t* tempty = tfull + 1;            // leader's used
  uint64_t* drained = tempty + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drained + 1);
  __shared__ PairMap s_map;
  __shared__ __align__(128) uint8_t s_ystage[kYStageBytes<EPI>];

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int m2_tiles = p.M_per / kPM;
  const int ks_count = p.K / 256;
  const int kc_per_rb = p.K / 64;

  load_pair_map(s_map, p, m2_tiles);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      // the leader producer(s)' expect-tx arrivals + 4 staging warps in each CTA
      mbar_init(&full[s], (G5_PAIR_SPLIT == 1 ? 2 : 1) + 8);
      mbar_init(&empty[s], 1);
      mbar_init(&full_sf[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, 2 * kEpiWarps);  // one arrive per epilogue warp of each CTA
    mbar_init(drained, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer's barriers exist before anyone signals them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int total_tiles = m2_tiles * s_map.ntp[p.nseg];

  if (warp < kEpiWarp0) {
  regs_dealloc<kRegsLow>();
  if (warp == 0 || warp == 6) {
    // ------------------------------------------------------ TMA producer(s)
    const bool do_a = warp == 0;
    const bool do_b = G5_PAIR_SPLIT == 1 ? warp == 6 : warp == 0;
    const bool do_sf = G5_PAIR_SPLIT == 2 ? warp == 6 : warp == 0;
    if (lane == 0 && (do_a || do_b || do_sf)) {
      tma_prefetch_desc(&tmap_a);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = pair; tile < total_tiles && ok; tile += npairs) {
        PairTile ti;
        if (!decode_pair_tile(tile, s_map, ti)) continue;
        const int n_mma = (ti.n_valid + 15) & ~15;
        const int half = n_mma / 2;  // token rows held by each CTA (multiple of 8)
        const int box = half <= 32 ? 32 : (half <= 64 ? 64 : 128);
        const CUtensorMap* mb = box == 32 ? &tmap_b32 : (box == 64 ? &tmap_b64 : &tmap_b128);
        const int sfb_ch = n_mma > 128 ? 2 : 1;
        const int a_row = ti.seg * p.M_per + ti.m2 * kPM + (int)rank * 128;
        const uint8_t* sfa = p.sfa + (size_t)(a_row / 128) * kc_per_rb * kChunk;
        const uint8_t* sfb = p.sfb + (size_t)(ti.row_start / 128) * kc_per_rb * kChunk;
        const uint32_t cta_bytes = (do_a ? kABytes : 0) + (do_b ? box * kBK : 0);
        const uint32_t sf_bytes = kSfaBytes + sfb_ch * 4 * kChunk;
        for (int ks = 0; ks < ks_count; ++ks) {
          if (!mbar_wait_cluster(&empty[stage], phase ^ 1u, p.err)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * kStageBytes;
          uint8_t* sb = sa + kABytes;
          uint8_t* ssfa = sb + kBBytes;
          uint8_t* ssfb = ssfa + kSfaBytes;
          const uint32_t lead_full = mapa_shared(smem_u32(&full[stage]), 0);
          if (do_sf) {
            mbar_arrive_expect_tx(&full_sf[stage], sf_bytes);
            bulk_load(ssfa, sfa + (size_t)ks * 4 * kChunk, kSfaBytes, &full_sf[stage]);
            for (int h = 0; h < sfb_ch; ++h)
              bulk_load(ssfb + h * 4 * kChunk, sfb + ((size_t)h * kc_per_rb + ks * 4) * kChunk,
                        4 * kChunk, &full_sf[stage]);
          }
          if (leader && cta_bytes) mbar_arrive_expect_tx(&full[stage], 2 * cta_bytes);
          if (do_a) tma_load_2d_pair(sa, &tmap_a, lead_full, ks * kBK, a_row);
          if (do_b)
            tma_load_2d_pair(sb, mb, lead_full, ks * kBK, ti.row_start + (int)rank * half);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA (leader)
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int tile = pair; tile < total_tiles && ok; tile += npairs) {
        PairTile ti;
        if (!decode_pair_tile(tile, s_map, ti)) continue;
        const uint32_t n_mma = (uint32_t)((ti.n_valid + 15) & ~15);
        const uint32_t idesc = idesc_fp4(kPM, n_mma, 0, 0, 0);
        if (!mbar_wait_cluster(tempty, acc_phase ^ 1u, p.err)) break;
        tc_fence_after();
        for (int ks = 0; ks < ks_count; ++ks) {
          if (!mbar_wait_cluster(&full[stage], phase, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* sa = smem + stage * kStageBytes;
          const uint8_t* sb = sa + kABytes;
          const uint32_t sfa_col = tmem_base + kSfBase + stage * (kSfaCols + kSfbCols);
          const uint32_t sfb_col = sfa_col + kSfaCols;
          const uint32_t a_addr = smem_u32(sa), b_addr = smem_u32(sb);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            mma_nvfp4_pair(tmem_base, desc_kmajor_sw128(a_addr + 32 * c),
                           desc_kmajor_sw128(b_addr + 32 * c), idesc, sfa_col + 4 * c,
                           sfb_col + 8 * c, (ks | c) != 0 ? 1u : 0u);
          tc_commit_pair(&empty[stage], 0x3);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit_pair(tfull, 0x3);
        acc_phase ^= 1u;
      }
      tc_commit_pair(drained, 0x1);
      mbar_wait(drained, 0, p.err);
    }
    __syncwarp();
  } else if (warp < 6) {
    // ------------------------------------------------------ scale staging
    // (both CTAs; the layout tcgen05.cp.32x128b.warpx4 writes)
    const int q = warp & 3;
    const uint32_t t_lane = tmem_base + ((uint32_t)(32 * q) << 16);
    const uint32_t lead_ready0 = mapa_shared(smem_u32(&full[0]), 0);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int tile = pair; tile < total_tiles && ok; tile += npairs) {
      PairTile ti;
      if (!decode_pair_tile(tile, s_map, ti)) continue;
      const bool two_blocks = ((ti.n_valid + 15) & ~15) > 128;
      for (int ks = 0; ks < ks_count; ++ks) {
        if (!mbar_wait(&full_sf[stage], phase, p.err)) {
          ok = false;
          break;
        }
        const uint8_t* ssfa = smem + stage * kStageBytes + kABytes + kBBytes;
        const uint8_t* ssfb = ssfa + kSfaBytes;
        const uint32_t sfa_col = kSfBase + stage * (kSfaCols + kSfbCols);
        const uint32_t sfb_col = sfa_col + kSfaCols;
        uint32_t r[kSfaCols];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 v = *reinterpret_cast<const uint4*>(ssfa + c * kChunk + lane * 16);
          r[4 * c] = v.x; r[4 * c + 1] = v.y; r[4 * c + 2] = v.z; r[4 * c + 3] = v.w;
        }
#pragma unroll
        for (int o = 0; o < kSfaCols; o += 8) tmem_st_32x32b_x8(t_lane + sfa_col + o, r + o);
        // chunk c of 128-row block h -> columns 8c + 4h
        uint32_t rb[kSfbCols];
#pragma unroll
        for (int g = 0; g < kSfbCols / 4; ++g) {
          const int c = g / 2, h = g % 2;
          uint4 v = make_uint4(0u, 0u, 0u, 0u);
          if (h == 0 || two_blocks)
            v = *reinterpret_cast<const uint4*>(ssfb + (h * 4 + c) * kChunk + lane * 16);
          rb[4 * g] = v.x; rb[4 * g + 1] = v.y; rb[4 * g + 2] = v.z; rb[4 * g + 3] = v.w;
        }
#pragma unroll
        for (int o = 0; o < kSfbCols; o += 8) tmem_st_32x32b_x8(t_lane + sfb_col + o, rb + o);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster_relaxed(lead_ready0 + stage * 8u);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  }
  } else {
    // ------------------------------------------------------ epilogue (both CTAs)
    regs_alloc<kRegsEpi>();
    pair_epilogue<EPI>(p, tmem_base, tfull, tempty, pair, npairs, total_tiles, s_map, rank,
                       warp, lane, s_ystage);
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA frees TMEM or exits while its peer may still signal it
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, kTmemCols);
}

// ---------------------------------------------------------------------------
// Wide-stage form (WIDE): a stage covers 512 of K (two 256-K chunks), so the
// leader's MMA thread waits once, issues eight MMAs and commits once per
// stage. Every tcgen05 instruction and every barrier wait costs that single
// thread about 90 cycles, which holds the 256-K form at ~690 cycles a stage
// against ~540 of tensor work for a full tile. Three operand stages of 64 KB
// (both chunks' weight rows and token rows, no scales) fill the shared
// memory; the block scales travel on their own two-slot ring (12 KB a slot)
// into one of two TMEM scale slots (96 columns each). Copy threads per CTA:
// warp 0 the weight rows, warp 6 the token rows, warp 7 the scale chunks (one
// TMA-issuing thread streams about 50 bytes per SM cycle, two about 100).
// The staging warps write a stage's scales once the MMAs of the stage two
// back have finished (its commit), since those read the same TMEM slot.
constexpr int kWChunks = 2;                                   // 256-K chunks per stage
constexpr int kWStages = 3;
constexpr int kWStageBytes = kWChunks * (kABytes + kBBytes);  // 64 KB
constexpr int kWSfSlots = 2;
constexpr int kWSfaBytes = kWChunks * kSfaBytes;              // [chunk][4 x 512 B]
constexpr int kWSfbBytes = kWChunks * kSfbBytes;              // [block][chunk][4 x 512 B]
constexpr int kWSfSlotBytes = kWSfaBytes + kWSfbBytes;        // 12 KB
constexpr int kWChunkCols = kSfaCols + kSfbCols;              // 48 TMEM columns per chunk
constexpr int kWSfCols = kWChunks * kWChunkCols;              // 96
constexpr size_t kWSmem =
    (size_t)kWStages * kWStageBytes + kWSfSlots * kWSfSlotBytes + 1024 + 256;
static_assert(kSfBase + kWSfSlots * kWSfCols <= kTmemCols, "TMEM budget (wide)");
static_assert((2 * kWStages + 2 * kWSfSlots + 3) * 8 + 4 <= 256, "barrier area (wide)");
// PairMap, the tile row-count ring, the y staging area and its alignment
static_assert(kWSmem + sizeof(PairMap) + 32 + kYStageBytes<1> + 128 <= 232448,
              "shared memory budget (wide)");

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    nvfp4_pair_gemm_wide_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                const __grid_constant__ CUtensorMap tmap_b32,
                                const __grid_constant__ CUtensorMap tmap_b64,
                                const __grid_constant__ CUtensorMap tmap_b128,
                                const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sf_ring = smem + kWStages * kWStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sf_ring + kWSfSlots * kWSfSlotBytes);  // leader's
  uint64_t* empty = full + kWStages;
  uint64_t* full_sf = empty + kWStages;
  uint64_t* sf_free = full_sf + kWSfSlots;
  uint64_t* tfull = sf_free + kWSfSlots;
  uint64_t* tempty = tfull + 1;  // leader's used
  uint64_t* drained = tempty + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drained + 1);
  __shared__ PairMap s_map;
  __shared__ __align__(128) uint8_t s_ystage[kYStageBytes<EPI>];
  // each tile's row count, from the leader's weight-copy thread (which decodes
  // the tile anyway) to the MMA thread: written before the tile's first
  // expect-tx arrival on the full barrier the MMA thread then waits on, read
  // after that wait; eight tiles deep (the copy thread runs at most three
  // stages ahead of the MMAs)
  __shared__ int32_t s_tile_n[8];

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int m2_tiles = p.M_per / kPM;
  const int chunks = p.K / 256;
  const int wstages = (chunks + kWChunks - 1) / kWChunks;
  const int kc_per_rb = p.K / 64;

  load_pair_map(s_map, p, m2_tiles);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kWStages; ++s) {
      // the leader's two operand copy threads' expect-tx arrivals + 4 staging
      // warps in each CTA
      mbar_init(&full[s], 2 + 8);
      mbar_init(&empty[s], 1);
    }
    for (int t = 0; t < kWSfSlots; ++t) {
      mbar_init(&full_sf[t], 1);
      mbar_init(&sf_free[t], 4);  // this CTA's staging warps
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, 2 * kEpiWarps);
    mbar_init(drained, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer's barriers exist before anyone signals them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int total_tiles = m2_tiles * s_map.ntp[p.nseg];

  if (warp < kEpiWarp0) {
  regs_dealloc<kRegsLow>();
  if (warp == 0 || warp == 6) {
    // ------------------------------------------------------ operand copies
    // (warp 0: this CTA's 128 weight rows; warp 6: its half of the token rows)
    if (lane == 0) {
      const bool do_a = warp == 0;
      if (do_a) tma_prefetch_desc(&tmap_a);
      int stage = 0, k = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = pair; tile < total_tiles && ok; tile += npairs, ++k) {
        PairTile ti;
        if (!decode_pair_tile(tile, s_map, ti)) ti.n_valid = 0;  // (every tile decodes)
        if (do_a && leader) s_tile_n[k & 7] = ti.n_valid;
        const int n_mma = (ti.n_valid + 15) & ~15;
        const int half = n_mma / 2;  // token rows held by each CTA (multiple of 8)
        const int box = half <= 32 ? 32 : (half <= 64 ? 64 : 128);
        const CUtensorMap* mb = box == 32 ? &tmap_b32 : (box == 64 ? &tmap_b64 : &tmap_b128);
        const int a_row = ti.seg * p.M_per + ti.m2 * kPM + (int)rank * 128;
        const int b_row = ti.row_start + (int)rank * half;
        const uint32_t chunk_bytes = do_a ? (uint32_t)kABytes : (uint32_t)(box * kBK);
        for (int w = 0; w < wstages; ++w) {
          const int c0 = w * kWChunks;
          const int nc = chunks - c0 < kWChunks ? chunks - c0 : kWChunks;
          if (!mbar_wait_cluster(&empty[stage], phase ^ 1u, p.err)) {
            ok = false;
            break;
          }
          uint8_t* dst = smem + stage * kWStageBytes + (do_a ? 0 : kWChunks * kABytes);
          const uint32_t lead_full = mapa_shared(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2u * (uint32_t)nc * chunk_bytes);
          for (int h = 0; h < nc; ++h) {
            if (do_a)
              tma_load_2d_pair(dst + h * kABytes, &tmap_a, lead_full, (c0 + h) * kBK, a_row);
            else
              tma_load_2d_pair(dst + h * kBBytes, mb, lead_full, (c0 + h) * kBK, b_row);
          }
          if (++stage == kWStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 7) {
    // ------------------------------------------------------ scale copies
    // (this CTA's weight rows' chunks and every token row's chunks)
    if (lane == 0) {
      int slot = 0;
      uint32_t sphase = 0;
      bool ok = true;
      for (int tile = pair; tile < total_tiles && ok; tile += npairs) {
        PairTile ti;
        if (!decode_pair_tile(tile, s_map, ti)) continue;
        const int n_mma = (ti.n_valid + 15) & ~15;
        const int sfb_ch = n_mma > 128 ? 2 : 1;
        const int a_row = ti.seg * p.M_per + ti.m2 * kPM + (int)rank * 128;
        const uint8_t* sfa = p.sfa + (size_t)(a_row / 128) * kc_per_rb * kChunk;
        const uint8_t* sfb = p.sfb + (size_t)(ti.row_start / 128) * kc_per_rb * kChunk;
        for (int w = 0; w < wstages; ++w) {
          const int c0 = w * kWChunks;
          const int nc = chunks - c0 < kWChunks ? chunks - c0 : kWChunks;
          if (!mbar_wait(&sf_free[slot], sphase ^ 1u, p.err)) {
            ok = false;
            break;
          }
          uint8_t* ssfa = sf_ring + slot * kWSfSlotBytes;
          uint8_t* ssfb = ssfa + kWSfaBytes;
          const uint32_t piece = (uint32_t)nc * 4u * kChunk;  // nc chunks of one 128-row block
          mbar_arrive_expect_tx(&full_sf[slot], piece * (uint32_t)(1 + sfb_ch));
          bulk_load(ssfa, sfa + (size_t)c0 * 4 * kChunk, piece, &full_sf[slot]);
          for (int h = 0; h < sfb_ch; ++h)
            bulk_load(ssfb + h * (kWSfbBytes / 2), sfb + ((size_t)h * kc_per_rb + c0 * 4) * kChunk,
                      piece, &full_sf[slot]);
          if (++slot == kWSfSlots) {
            slot = 0;
            sphase ^= 1u;
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA (leader)
    if (leader && lane == 0) {
      int stage = 0, slot = 0, k = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      const uint64_t desc_a0 = desc_kmajor_sw128(smem_u32(smem));
      // every tile index below total_tiles decodes to a tile, so the MMA
      // thread only counts them and takes each tile's row count from the
      // weight-copy thread (s_tile_n) after the tile's first full wait
      for (int tile = pair; tile < total_tiles && ok; tile += npairs, ++k) {
        uint32_t idesc = 0;
        for (int w = 0; w < wstages; ++w) {
          const int nc = chunks - w * kWChunks < kWChunks ? chunks - w * kWChunks : kWChunks;
          if (!mbar_wait_cluster(&full[stage], phase, p.err)) {
            ok = false;
            break;
          }
          if (w == 0) {
            const uint32_t n_mma = (uint32_t)((s_tile_n[k & 7] + 15) & ~15);
            idesc = idesc_fp4(kPM, n_mma, 0, 0, 0);
            if (!mbar_wait_cluster(tempty, acc_phase ^ 1u, p.err)) {
              ok = false;
              break;
            }
          }
          tc_fence_after();
          // a descriptor's start address is in 16-byte units in its low bits
          // (shared addresses stay below 256 KB, so adding never carries out)
          const uint64_t da = desc_a0 + (uint64_t)(stage * (kWStageBytes >> 4));
          const uint64_t db = da + (uint64_t)((kWChunks * kABytes) >> 4);
          const uint32_t sf_col = tmem_base + kSfBase + slot * kWSfCols;
#pragma unroll
          for (int h = 0; h < kWChunks; ++h) {
            if (h >= nc) break;
#pragma unroll
            for (int c = 0; c < 4; ++c)
              mma_nvfp4_pair(tmem_base, da + (uint64_t)((h * kABytes + 32 * c) >> 4),
                             db + (uint64_t)((h * kBBytes + 32 * c) >> 4), idesc,
                             sf_col + h * kWChunkCols + 4 * c,
                             sf_col + h * kWChunkCols + kSfaCols + 8 * c,
                             (w | h | c) != 0 ? 1u : 0u);
          }
          tc_commit_pair(&empty[stage], 0x3);
          if (++stage == kWStages) {
            stage = 0;
            phase ^= 1u;
          }
          if (++slot == kWSfSlots) slot = 0;
        }
        if (!ok) break;
        tc_commit_pair(tfull, 0x3);
        acc_phase ^= 1u;
      }
      tc_commit_pair(drained, 0x1);
      mbar_wait(drained, 0, p.err);
    }
    __syncwarp();
  } else if (warp < 6) {
    // ------------------------------------------------------ scale staging
    // (both CTAs; the layout tcgen05.cp.32x128b.warpx4 writes)
    const int q = warp & 3;
    const uint32_t t_lane = tmem_base + ((uint32_t)(32 * q) << 16);
    const uint32_t lead_full0 = mapa_shared(smem_u32(&full[0]), 0);
    int slot = 0, g = 0;
    uint32_t sphase = 0;
    bool ok = true;
    for (int tile = pair; tile < total_tiles && ok; tile += npairs) {
      PairTile ti;
      if (!decode_pair_tile(tile, s_map, ti)) continue;
      const bool two_blocks = ((ti.n_valid + 15) & ~15) > 128;
      for (int w = 0; w < wstages; ++w, ++g) {
        const int nc = chunks - w * kWChunks < kWChunks ? chunks - w * kWChunks : kWChunks;
        if (!mbar_wait(&full_sf[slot], sphase, p.err)) {
          ok = false;
          break;
        }
        // the TMEM slot's previous stage (two back) has finished its MMAs
        if (g >= kWSfSlots) {
          const int gp = g - kWSfSlots;
          if (!mbar_wait(&empty[gp % kWStages], (uint32_t)((gp / kWStages) & 1), p.err)) {
            ok = false;
            break;
          }
        }
        const uint8_t* ssfa = sf_ring + slot * kWSfSlotBytes;
        const uint8_t* ssfb = ssfa + kWSfaBytes;
        const uint32_t col0 = kSfBase + slot * kWSfCols;
        for (int h = 0; h < nc; ++h) {
          uint32_t r[kSfaCols];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint4 v =
                *reinterpret_cast<const uint4*>(ssfa + (h * 4 + c) * kChunk + lane * 16);
            r[4 * c] = v.x; r[4 * c + 1] = v.y; r[4 * c + 2] = v.z; r[4 * c + 3] = v.w;
          }
#pragma unroll
          for (int o = 0; o < kSfaCols; o += 8)
            tmem_st_32x32b_x8(t_lane + col0 + h * kWChunkCols + o, r + o);
          // chunk c of 128-row block hb -> columns 8c + 4hb
          uint32_t rb[kSfbCols];
#pragma unroll
          for (int gg = 0; gg < kSfbCols / 4; ++gg) {
            const int c = gg / 2, hb = gg % 2;
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (hb == 0 || two_blocks)
              v = *reinterpret_cast<const uint4*>(ssfb + hb * (kWSfbBytes / 2) +
                                                  (h * 4 + c) * kChunk + lane * 16);
            rb[4 * gg] = v.x; rb[4 * gg + 1] = v.y; rb[4 * gg + 2] = v.z; rb[4 * gg + 3] = v.w;
          }
#pragma unroll
          for (int o = 0; o < kSfbCols; o += 8)
            tmem_st_32x32b_x8(t_lane + col0 + h * kWChunkCols + kSfaCols + o, rb + o);
        }
        tmem_st_wait();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sf_free[slot]);  // the ring slot may be refilled
        tc_fence_before();
        if (lane == 0) mbar_arrive_cluster_relaxed(lead_full0 + (g % kWStages) * 8u);
        if (++slot == kWSfSlots) {
          slot = 0;
          sphase ^= 1u;
        }
      }
    }
  }
  } else {
    regs_alloc<kRegsEpi>();
    pair_epilogue<EPI>(p, tmem_base, tfull, tempty, pair, npairs, total_tiles, s_map, rank,
                       warp, lane, s_ystage);
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA frees TMEM or exits while its peer may still signal it
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, kTmemCols);
}

template <int EPI, int WIDE>
cudaError_t launch_pair(const CUtensorMap* ta, const CUtensorMap* tb, const GemmParams& p,
                        int grid, cudaStream_t st) {
  auto kern = WIDE ? nvfp4_pair_gemm_wide_kernel<EPI> : nvfp4_pair_gemm_kernel<EPI>;
  const size_t smem = WIDE ? kWSmem : kSmem;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // setmaxnreg.inc waits until the block's launch registers cover the split
  cudaFuncAttributes fa{};
  e = cudaFuncGetAttributes(&fa, kern);
  if (e != cudaSuccess) return e;
  if ((size_t)fa.numRegs * kThreads < 256u * (kRegsLow + kRegsEpi)) return cudaErrorInvalidConfiguration;
  return cudaLaunchKernelEx(&cfg, kern, *ta, tb[0], tb[1], tb[2], p);
}

}  // namespace

int nvfp4_pair_gemm_grid(int num_sms) {
  // as many CTA pairs as can be resident at once (clusters of two SMs)
  auto kern = nvfp4_pair_gemm_kernel<0>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem) !=
      cudaSuccess)
    return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)num_sms);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess) return 0;
  return 2 * clusters;
}

cudaError_t launch_nvfp4_pair_gemm(int epi, const CUtensorMap* tmap_a, const CUtensorMap* tmap_b,
                                   const CUtensorMap* tmap_sfa, const CUtensorMap* tmap_sfb,
                                   const GemmParams& p, int grid, cudaStream_t st, int wide) {
  (void)tmap_sfa;
  (void)tmap_sfb;
  if (p.nseg > kMaxSeg || p.K % 256 || p.M_per % kPM || grid < 2 || grid % 2)
    return cudaErrorInvalidValue;
  if (wide)
    return epi == 0 ? launch_pair<0, 1>(tmap_a, tmap_b, p, grid, st)
                    : launch_pair<1, 1>(tmap_a, tmap_b, p, grid, st);
  return epi == 0 ? launch_pair<0, 0>(tmap_a, tmap_b, p, grid, st)
                  : launch_pair<1, 0>(tmap_a, tmap_b, p, grid, st);
}

}  // namespace glm5x
