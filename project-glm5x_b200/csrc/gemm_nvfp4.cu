// gemm_nvfp4.cu -- persistent grouped NVFP4 GEMM on tcgen05 block-scaled MMA.
//
// Replaces the reference's expert projections: the cuBLASLt NVFP4
// torch._scaled_mm calls (reference/glm5x_ref/nvfp4.py:220-233, 294-335;
// grouped form reference/glm5x_ref/nvfp4_batched.py:64-151) and the SIMT
// MXFP4 grid (runtime/cuda/mxfp4.cu:67-104), with SwiGLU
// (runtime/cuda/situ.cu:51-75, layer10_moe.py:730) fused into the gate/up
// epilogue and the routing weight (layer10_moe.py:843-846) fused into the
// down epilogue.
//
// Structure (one CTA per SM, 512 threads = four warpgroups):
//   warp 0      TMA producer: weight tile (128 rows x 256 K) and activation
//               tile (BN rows x 256 K), both 128B-swizzled, plus the four
//               512-byte scale chunks of each operand by bulk copy.
//   warp 1      TMEM owner and MMA issuer: four kind::mxf4nvf4 block16 MMAs
//               (K = 64 each) per stage accumulate into TMEM.
//   warps 2-5   scale staging, one per 32-lane TMEM quadrant: each stage's
//               scale chunks go from shared memory through registers into
//               that stage's TMEM scale columns with tcgen05.st (the layout a
//               32x128b.warpx4 tcgen05.cp would write). Done by tcgen05.cp
//               from the MMA thread, the copies execute in the tensor pipe
//               between the MMAs and cost about a third of its time; from
//               these warps they overlap the MMAs.
//   warps 8-15  epilogue: two warps per 32-lane TMEM quadrant, alternating
//               32-column chunks of the 128 x n accumulator. Each warp drains
//               its columns to registers, hands the TMEM buffer back, then
//               scales by the two global scales, applies the fused
//               activation and stores BF16.
//   warps 6, 7  idle. The first two warpgroups give registers to the two
//               epilogue warpgroups (setmaxnreg).
// Weights are the M side (swap-AB): M = 128 weight rows per tile, N = the
// expert's tokens (<= BN), so the decode regime (a few tokens per expert)
// still uses full 128-row MMAs. Tiles are enumerated expert-major, then
// weight tile, then token tile, so CTAs sharing a weight or token tile run at
// the same time and hit L2.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "glm5x_kernels.cuh"
#include "glm5x_ptx.cuh"

// Build-time tuning: L2 prefetch of the next tile's operands (measured to
// raise DRAM traffic without speeding the GEMM up, so off) and loading only
// the activation rows a tile needs (in 32/64/128-row pieces).
#ifndef G5_GEMM_L2_PREFETCH
#define G5_GEMM_L2_PREFETCH 0
#endif
#ifndef G5_GEMM_B_PIECES
#define G5_GEMM_B_PIECES 1
#endif
// Threads issuing the stage loads: 1 = warp 0 issues scales, weights and
// activations; 2 = warp 6 takes the activation rows; 3 = warp 6 the weight
// rows and warp 7 the activation rows; 4 = warp 6 takes the scale chunks.
#ifndef G5_GEMM_PRODUCERS
#define G5_GEMM_PRODUCERS 2
#endif

namespace glm5x {

namespace {

constexpr int kBM = 128;          // weight rows per tile
constexpr int kBKBytes = 128;     // K bytes per stage (256 FP4 values)
constexpr int kChunkBytes = 512;  // one 128-row x 4-scale chunk
constexpr int kEpiWarps = 8;      // two warps per TMEM lane quadrant
constexpr int kEpiWarp0 = 8;      // first epilogue warp (warpgroups 2 and 3)
constexpr int kSfWarp0 = 2;       // scale-staging warps 2..5
constexpr int kThreads = 512;
// setmaxnreg split of the 64K registers: 256 x 80 + 256 x 176 = 65536
constexpr uint32_t kRegsLow = 80;
constexpr uint32_t kRegsEpi = 176;
static_assert(256 * kRegsLow + 256 * kRegsEpi <= 65536, "register split");
constexpr int kMaxSeg = 260;      // segments (local experts + shared) per launch

// MX = 0: NVFP4 (E4M3 scale per 16, kind::mxf4nvf4 block16, one 4-scale
// chunk per K = 64 MMA). MX = 1: MXFP4 (E8M0 scale per 32, kind::mxf4 block32,
// one chunk per two MMAs, which pick its scale bytes 0-1 or 2-3 by the scale
// id) with four B rows per token (the residual terms of the activation).
// MH = 2 (narrow token tiles): a tile covers 256 weight rows as two 128-row
// halves, each with its own M = 128 MMAs and accumulator; one stage carries
// both halves' weight rows against the same token rows, so every barrier
// wait, stage hand-off and tile switch moves twice the weight bytes.
template <int BN, int MX, int MH = 1>
struct Cfg {
  static constexpr int kSfbCh = BN > 128 ? 2 : 1;  // 128-row scale blocks per tile
  static constexpr int kAcc = BN > 128 ? 1 : 2;    // TMEM accumulator buffers
  static constexpr int kCh = MX ? 2 : 4;           // scale chunks per 128 rows per stage
  static constexpr int kABytes = MH * kBM * kBKBytes;
  static constexpr int kBBytes = BN * kBKBytes;
  static constexpr int kSfaBytes = MH * kCh * kChunkBytes;
  static constexpr int kSfbBytes = kSfbCh * kCh * kChunkBytes;
  static constexpr int kStageBytes =
      ((kABytes + kBBytes + kSfaBytes + kSfbBytes + 1023) / 1024) * 1024;
  // two-half tiles: as many stages as fit (at most 5)
  static constexpr int kStagesFit = (232448 - 1536 - 3 * 4 * (kMaxSeg + 1)) / kStageBytes;
  static constexpr int kStages =
      MH == 2 ? (kStagesFit < 5 ? kStagesFit : 5)
              : (BN > 128 ? 4 : (BN > 64 ? 5 : (BN > 32 ? 6 : 8)));
  static constexpr int kSfaCols = 4 * kCh * MH;       // half h's chunk c at 4 * kCh * h + 4c
  static constexpr int kSfbCols = 4 * kCh * kSfbCh;   // chunk c of block h at 4 * kSfbCh * c + 4 * h
  static constexpr int kSfBase = kAcc * MH * BN;
  static constexpr int kStageSfCols = kSfaCols + kSfbCols;
  static constexpr int kTmemCols = 512;
  static_assert(kSfBase + kStages * kStageSfCols <= kTmemCols, "TMEM budget");
  static constexpr size_t kSmem = (size_t)kStages * kStageBytes + 1024 + 512;
  static_assert((4 * kStages + 2 * kAcc + 1) * 8 + 4 <= 512, "barrier area");
  static_assert(kSmem + 3 * 4 * (kMaxSeg + 1) <= 232448, "shared memory budget");
};

struct TileInfo {
  int seg, m_tile, row_start, n_valid;
};

__device__ __forceinline__ bool decode_tile(int tile, int m_tiles, int nseg, int bn,
                                            const int32_t* __restrict__ ntp,
                                            const int32_t* __restrict__ cnt,
                                            const int32_t* __restrict__ start, TileInfo& ti) {
  const int key = tile / m_tiles;
  int lo = 0, hi = nseg;  // largest s with ntp[s] <= key
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (ntp[mid] <= key) lo = mid; else hi = mid;
  }
  const int s = lo;
  const int nt = ntp[s + 1] - ntp[s];
  if (nt <= 0) return false;
  const int local = tile - m_tiles * ntp[s];
  const int m = local / nt, n = local % nt;
  ti.seg = s;
  ti.m_tile = m;
  // tiles narrower than 128 rows each own a 128-row block (tile_stride 128)
  ti.row_start = start[s] + n * (bn < 128 ? 128 : bn);
  const int left = cnt[s] - n * bn;
  ti.n_valid = left < bn ? left : bn;
  return true;
}

__device__ __forceinline__ uint16_t f2bf(float x) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

// TM = 1 (token-major, down projection of large batches, BN = 256): the MMA's
// M side is 128 token rows and its N side 256 weight rows, so each epilogue
// thread holds one token's consecutive output features and stores them in
// 16-byte pieces; tiles enumerate 128-token tiles fastest within a 256-row
// weight tile. A / SFA are the token rows, B / SFB the weights.
template <int BN, int EPI, int MX, int TM, int MH>
__global__ void __launch_bounds__(kThreads, 1)
    nvfp4_grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                              const __grid_constant__ CUtensorMap tmap_b32,
                              const __grid_constant__ CUtensorMap tmap_b64,
                              const __grid_constant__ CUtensorMap tmap_b128, const GemmParams p) {
  using C = Cfg<BN, MX, MH>;
  static_assert(MH == 1 || (!TM && BN <= 64), "two weight halves: narrow token tiles only");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* sf_ready = empty + C::kStages;
  uint64_t* full_sf = sf_ready + C::kStages;  // a stage's scale chunks landed
  uint64_t* tfull = full_sf + C::kStages;
  uint64_t* tempty = tfull + C::kAcc;
  uint64_t* drained = tempty + C::kAcc;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drained + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  static_assert(!TM || (BN == 256 && EPI == 1 && !MX), "token-major: down projection, BN 256");
  const int m_tiles = TM ? p.M_per / 256 : p.M_per / (kBM * MH);
  constexpr int kTileRows = TM ? 128 : BN;  // token rows per tile
  const int ks_count = p.K / 256;
  const int kc_per_rb = p.K / (MX ? 128 : 64);  // scale chunks per 128-row block
  __shared__ int32_t s_ntp[kMaxSeg + 1], s_cnt[kMaxSeg], s_start[kMaxSeg + 1];

  // Token-tile prefix: from the permutation (tiles of its width), or, when
  // this launch's tiles differ from it (TM, or a wider-than-128 width the
  // permutation did not use; segments are contiguous 128-aligned rows then),
  // counted here.
  const bool own_prefix = TM || p.ntile_prefix == nullptr;
  for (int i = threadIdx.x; i <= p.nseg; i += blockDim.x) {
    if (!own_prefix) s_ntp[i] = p.ntile_prefix[i];
    s_start[i] = p.seg_start[i];
    if (i < p.nseg) s_cnt[i] = p.seg_count[i];
  }
  if (own_prefix) {
    __syncthreads();
    if (threadIdx.x == 0) {
      int acc = 0;
      for (int i = 0; i < p.nseg; ++i) {
        s_ntp[i] = acc;
        acc += (s_cnt[i] + kTileRows - 1) / kTileRows;
      }
      s_ntp[p.nseg] = acc;
    }
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], (G5_GEMM_PRODUCERS == 2 || G5_GEMM_PRODUCERS == 3) ? 2 : 1);
      mbar_init(&empty[s], 1);
      mbar_init(&sf_ready[s], 4);
      mbar_init(&full_sf[s], 1);
    }
    for (int a = 0; a < C::kAcc; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpiWarps);  // one arrive per epilogue warp
    }
    mbar_init(drained, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b32);
    tma_prefetch_desc(&tmap_b64);
    tma_prefetch_desc(&tmap_b128);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int total_tiles = m_tiles * s_ntp[p.nseg];
  if (warp < kEpiWarp0) {
  // the producer, MMA and staging warpgroups give registers back together
  regs_dealloc<kRegsLow>();
  if (warp == 0 || warp == 6 || warp == 7) {
    // ------------------------------------------------------ TMA producer(s)
    const int role = warp == 0 ? 0 : warp - 5;
    constexpr int kP = G5_GEMM_PRODUCERS;
    const bool do_sf = kP == 4 ? role == 1 : role == 0;
    const bool do_a = kP == 3 ? role == 1 : role == 0;
    const bool do_b = (kP == 1 || kP == 4) ? role == 0 : role == kP - 1;
    if (lane == 0 && (do_sf || do_a || do_b)) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      const size_t a_row_bytes = (size_t)p.K / 2;
      // L2 prefetch of one tile's weight rows + scales and activation rows
      auto prefetch_tile = [&](int tile) {
        TileInfo tp;
        if (tile >= total_tiles ||
            !decode_tile(tile, m_tiles, p.nseg, kTileRows, s_ntp, s_cnt, s_start, tp))
          return;
        const size_t a_row = (size_t)tp.seg * p.M_per + (size_t)tp.m_tile * kBM;
        const uint8_t* a = p.a_packed + a_row * a_row_bytes;
        const uint32_t a_bytes = (uint32_t)(kBM * a_row_bytes);
        for (uint32_t off = 0; off < a_bytes; off += 65536u)
          l2_prefetch(a + off, a_bytes - off < 65536u ? a_bytes - off : 65536u);
        l2_prefetch(p.sfa + (a_row / 128) * kc_per_rb * kChunkBytes, kc_per_rb * kChunkBytes);
        const uint32_t b_bytes = (uint32_t)(((tp.n_valid + 31) & ~31) * a_row_bytes);
        l2_prefetch(p.b_packed + (size_t)tp.row_start * a_row_bytes, b_bytes);
      };
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        TileInfo ti;
        if (!decode_tile(tile, m_tiles, p.nseg, kTileRows, s_ntp, s_cnt, s_start, ti)) continue;
        if (G5_GEMM_L2_PREFETCH && role == 0) prefetch_tile(tile + gridDim.x);
        // TM: A = the 128 token rows, B = 256 weight rows
        const int w_row = ti.seg * p.M_per + ti.m_tile * (TM ? 256 : kBM * MH);
        const int a_row = TM ? ti.row_start : w_row;
        const int b_row = TM ? w_row : ti.row_start;
        const int sfb_ch = TM ? 2 : (ti.n_valid > 128 ? 2 : 1);
        const uint8_t* sfa = p.sfa + (size_t)(a_row / 128) * kc_per_rb * kChunkBytes;
        const uint8_t* sfb = p.sfb + (size_t)(b_row / 128) * kc_per_rb * kChunkBytes;
        // activation rows in pieces: rows [0, 128) and [128, n), each rounded
        // up to 32 rows and loaded with the 32/64/128-row box that fits
        const int b_rows = TM ? 256 : ti.n_valid;
        const int rows0 = G5_GEMM_B_PIECES ? (b_rows < 128 ? b_rows : 128) : (BN < 128 ? BN : 128);
        const int rows1 = G5_GEMM_B_PIECES ? b_rows - rows0 : (BN > 128 ? BN - 128 : 0);
        const int box0 = rows0 <= 32 ? 32 : (rows0 <= 64 ? 64 : 128);
        const int box1 = rows1 <= 0 ? 0 : (rows1 <= 32 ? 32 : (rows1 <= 64 ? 64 : 128));
        const CUtensorMap* m0 = box0 == 32 ? &tmap_b32 : (box0 == 64 ? &tmap_b64 : &tmap_b128);
        const CUtensorMap* m1 = box1 == 32 ? &tmap_b32 : (box1 == 64 ? &tmap_b64 : &tmap_b128);
        const uint32_t bytes =
            (do_a ? (uint32_t)C::kABytes : 0u) + (do_b ? (uint32_t)(box0 + box1) * kBKBytes : 0u);
        const uint32_t sf_bytes = C::kSfaBytes + sfb_ch * C::kCh * kChunkBytes;
        for (int ks = 0; ks < ks_count; ++ks) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.err)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * C::kStageBytes;
          uint8_t* sb = sa + C::kABytes;
          uint8_t* ssfa = sb + C::kBBytes;
          uint8_t* ssfb = ssfa + C::kSfaBytes;
          // scale chunks first, on their own barrier: the staging warps move
          // them into TMEM while the operand tiles are still landing
          if (do_sf) {
            mbar_arrive_expect_tx(&full_sf[stage], sf_bytes);
#pragma unroll
            for (int h = 0; h < MH; ++h)  // one 128-row scale block per weight half
              bulk_load(ssfa + h * C::kCh * kChunkBytes,
                        sfa + ((size_t)h * kc_per_rb + ks * C::kCh) * kChunkBytes,
                        C::kCh * kChunkBytes, &full_sf[stage]);
            for (int h = 0; h < sfb_ch; ++h)
              bulk_load(ssfb + h * C::kCh * kChunkBytes,
                        sfb + ((size_t)h * kc_per_rb + ks * C::kCh) * kChunkBytes,
                        C::kCh * kChunkBytes, &full_sf[stage]);
          }
          if (bytes) mbar_arrive_expect_tx(&full[stage], bytes);
          if (do_a) {
#pragma unroll
            for (int h = 0; h < MH; ++h)
              tma_load_2d(sa + h * kBM * kBKBytes, &tmap_a, &full[stage], ks * kBKBytes,
                          a_row + h * kBM);
          }
          if (do_b) {
            tma_load_2d(sb, m0, &full[stage], ks * kBKBytes, b_row);
            if (box1)
              tma_load_2d(sb + 128 * kBKBytes, m1, &full[stage], ks * kBKBytes, b_row + 128);
          }
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        TileInfo ti;
        if (!decode_tile(tile, m_tiles, p.nseg, kTileRows, s_ntp, s_cnt, s_start, ti)) continue;
        const uint32_t n_mma = TM ? 256u : (uint32_t)((ti.n_valid + 7) / 8 * 8);
        const uint32_t idesc = idesc_fp4(kBM, n_mma, 0, 0, 0);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, p.err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * MH * BN;
        for (int ks = 0; ks < ks_count; ++ks) {
          // operands landed (full) and this stage's scales are in TMEM
          if (!mbar_wait(&full[stage], phase, p.err) ||
              !mbar_wait(&sf_ready[stage], phase, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* sa = smem + stage * C::kStageBytes;
          const uint8_t* sb = sa + C::kABytes;
          const uint32_t sfa_col = tmem_base + C::kSfBase + stage * C::kStageSfCols;
          const uint32_t sfb_col = sfa_col + C::kSfaCols;
          const uint32_t a_addr = smem_u32(sa), b_addr = smem_u32(sb);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
#pragma unroll
            for (int h = 0; h < MH; ++h) {
              const uint32_t a_h = a_addr + h * kBM * kBKBytes;
              const uint32_t sfa_h = sfa_col + 4 * C::kCh * h;
              if (MX) {
                // chunk c / 2; scale bytes 0-1 (id 0) or 2-3 (id 2) of each column,
                // given in the address's top bits and in the descriptor
                const uint32_t id = (uint32_t)(c & 1) * 2u;
                mma_mxfp4(d_tmem + h * BN, desc_kmajor_sw128(a_h + 32 * c),
                          desc_kmajor_sw128(b_addr + 32 * c), idesc_fp4(kBM, n_mma, 1, id, id),
                          (sfa_h + 4 * (c >> 1)) | (id << 30),
                          (sfb_col + 4 * C::kSfbCh * (c >> 1)) | (id << 30),
                          (ks | c) != 0 ? 1u : 0u);
              } else {
                mma_nvfp4(d_tmem + h * BN, desc_kmajor_sw128(a_h + 32 * c),
                          desc_kmajor_sw128(b_addr + 32 * c), idesc, sfa_h + 4 * c,
                          sfb_col + 4 * C::kSfbCh * c, (ks | c) != 0 ? 1u : 0u);
              }
            }
          }
          tc_commit(&empty[stage]);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&tfull[acc]);
        if (++acc == C::kAcc) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // every MMA this thread issued has completed once `drained` flips
      tc_commit(drained);
      mbar_wait(drained, 0, p.err);
    }
    __syncwarp();
  } else if (warp < kSfWarp0 + 4) {
    // ------------------------------------------------------ scale staging
    // Lane l of the warp owning quadrant q writes, for every scale chunk of
    // the stage, the chunk's 16 bytes at l * 16 into four consecutive TMEM
    // columns of lane 32q + l: the layout tcgen05.cp.32x128b.warpx4 writes
    // (every quadrant gets the same 32 x 16 bytes).
    const int q = warp & 3;
    const uint32_t t_lane = tmem_base + ((uint32_t)(32 * q) << 16);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
      TileInfo ti;
      if (!decode_tile(tile, m_tiles, p.nseg, kTileRows, s_ntp, s_cnt, s_start, ti)) continue;
      const bool two_blocks = TM || ti.n_valid > 128;
      for (int ks = 0; ks < ks_count; ++ks) {
        if (!mbar_wait(&full_sf[stage], phase, p.err)) {
          ok = false;
          break;
        }
        const uint8_t* ssfa = smem + stage * C::kStageBytes + C::kABytes + C::kBBytes;
        const uint8_t* ssfb = ssfa + C::kSfaBytes;
        const uint32_t sfa_col = C::kSfBase + stage * C::kStageSfCols;
        const uint32_t sfb_col = sfa_col + C::kSfaCols;
        // SFA: chunk c (of half c / kCh) -> columns 4c..4c+3
        uint32_t r[C::kSfaCols];
#pragma unroll
        for (int c = 0; c < C::kCh * MH; ++c) {
          const uint4 v = *reinterpret_cast<const uint4*>(ssfa + c * kChunkBytes + lane * 16);
          r[4 * c] = v.x; r[4 * c + 1] = v.y; r[4 * c + 2] = v.z; r[4 * c + 3] = v.w;
        }
#pragma unroll
        for (int o = 0; o < C::kSfaCols; o += 8) tmem_st_32x32b_x8(t_lane + sfa_col + o, r + o);
        // SFB: chunk c of 128-row block h -> columns 4 * kSfbCh * c + 4h
        uint32_t rb[C::kSfbCols];
#pragma unroll
        for (int g = 0; g < C::kSfbCols / 4; ++g) {
          const int c = g / C::kSfbCh, h = g % C::kSfbCh;
          uint4 v = make_uint4(0u, 0u, 0u, 0u);
          if (h == 0 || two_blocks)
            v = *reinterpret_cast<const uint4*>(ssfb + (h * C::kCh + c) * kChunkBytes + lane * 16);
          rb[4 * g] = v.x; rb[4 * g + 1] = v.y; rb[4 * g + 2] = v.z; rb[4 * g + 3] = v.w;
        }
#pragma unroll
        for (int o = 0; o < C::kSfbCols; o += 8) tmem_st_32x32b_x8(t_lane + sfb_col + o, rb + o);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_relaxed(&sf_ready[stage]);
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  }
  } else {
    // ------------------------------------------------------ epilogue
    regs_alloc<kRegsEpi>();
    const int q = warp & 3;                         // TMEM lane quadrant this warp may access
    const int half = (warp - kEpiWarp0) >> 2;       // which alternate 32-column chunks
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x) {
      TileInfo ti;
      if (!decode_tile(tile, m_tiles, p.nseg, kTileRows, s_ntp, s_cnt, s_start, ti)) continue;
      if (!mbar_wait(&tfull[acc], acc_phase, p.err)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(32 * q) << 16) + acc * MH * BN;
      // Drain this warp's columns of the accumulator into registers and hand
      // the TMEM buffer back before any math or store, so the next tile's
      // MMAs overlap this tile's epilogue even with a single buffer.
      constexpr int kChunks = (BN + 63) / 64;
      uint32_t vv[MH][kChunks][32];
#pragma unroll
      for (int h = 0; h < MH; ++h)
#pragma unroll
        for (int i = 0; i < kChunks; ++i)
          if (TM || 32 * half + 64 * i < ti.n_valid)
            tmem_ld_32x32b_x32(t_row + h * BN + 32 * half + 64 * i, vv[h][i]);
      tmem_ld_wait();
#pragma unroll
      for (int h = 0; h < MH; ++h)
#pragma unroll
        for (int i = 0; i < kChunks; ++i) reg_fence(vv[h][i]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_relaxed(&tempty[acc]);
#pragma unroll
      for (int h = 0; h < MH; ++h) {
        // weight half h: 128-row m-tile mt of the expert
        const int mt = ti.m_tile * MH + h;
        auto& v = vv[h];
        const float bscale = p.b_global[ti.seg];
        if (TM) {
          // lane = token row 32q + lane of the tile; a chunk = 32 consecutive
          // output features of that token, stored as four 16-byte pieces
          const int r = 32 * q + lane;
          if (r < ti.n_valid) {
            const float w = p.row_weight[ti.row_start + r] * (bscale * p.a_global[ti.seg]);
            uint16_t* yrow = p.out + (size_t)(ti.row_start + r) * p.M_per + mt * 256;
  #pragma unroll
            for (int ch = 0; ch < kChunks; ++ch) {
              const int c0 = 32 * half + 64 * ch;
              uint32_t pk[16];
  #pragma unroll
              for (int i = 0; i < 16; ++i) {
                const __nv_bfloat162 b2 = __floats2bfloat162_rn(
                    __uint_as_float(v[ch][2 * i]) * w, __uint_as_float(v[ch][2 * i + 1]) * w);
                pk[i] = *reinterpret_cast<const uint32_t*>(&b2);
              }
              uint4* dst = reinterpret_cast<uint4*>(yrow + c0);
  #pragma unroll
              for (int i = 0; i < 4; ++i)
                dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
            }
          }
        } else if (MX && EPI == 0) {
          // Columns 4r..4r+3 of a chunk are the four terms of the chunk's token
          // r (r = 0..7): their sum is the token's product. Lanes l < 16 hold
          // gate rows and compute h for tokens 0-3, lanes l + 16 the matching up
          // rows and tokens 4-7; one swap per token pair. h goes to the token's
          // term-0 row.
          const float s_gate = bscale * p.a_global[2 * ti.seg];
          const float s_up = bscale * p.a_global[2 * ti.seg + 1];
          const bool lo = lane < 16;
          const int j = mt * (kBM / 2) + 16 * q + (lane & 15);
          const int hcols = p.M_per / 2;
  #pragma unroll
          for (int ch = 0; ch < kChunks; ++ch) {
            const int c0 = 32 * half + 64 * ch;
            if (c0 >= ti.n_valid) break;
            float t[8];
  #pragma unroll
            for (int r = 0; r < 8; ++r)
              t[r] = (__uint_as_float(v[ch][4 * r]) + __uint_as_float(v[ch][4 * r + 1])) +
                     (__uint_as_float(v[ch][4 * r + 2]) + __uint_as_float(v[ch][4 * r + 3]));
  #pragma unroll
            for (int r = 0; r < 4; ++r) {
              const float recv = __shfl_xor_sync(0xffffffffu, lo ? t[r + 4] : t[r], 16);
              const float gate = (lo ? t[r] : recv) * s_gate;
              const float up = (lo ? recv : t[r + 4]) * s_up;
              const int col = c0 + 4 * (r + (lo ? 0 : 4));
              if (col < ti.n_valid)
                p.out[(size_t)(ti.row_start + col) * hcols + j] =
                    f2bf(__fdividef(gate, 1.0f + __expf(-gate)) * up);
            }
          }
        } else if (MX) {
          // four term columns per token; routing weight of the term-0 row
          const float scale = bscale * p.a_global[ti.seg];
          const int o = mt * kBM + 32 * q + lane;
  #pragma unroll
          for (int ch = 0; ch < kChunks; ++ch) {
            const int c0 = 32 * half + 64 * ch;
            if (c0 >= ti.n_valid) break;
            const float wmine = lane < 8 && c0 + 4 * lane < ti.n_valid
                                    ? p.row_weight[ti.row_start + c0 + 4 * lane] * scale
                                    : 0.0f;
  #pragma unroll
            for (int r = 0; r < 8; ++r) {
              const float w = __shfl_sync(0xffffffffu, wmine, r);
              const float t = (__uint_as_float(v[ch][4 * r]) + __uint_as_float(v[ch][4 * r + 1])) +
                              (__uint_as_float(v[ch][4 * r + 2]) + __uint_as_float(v[ch][4 * r + 3]));
              if (c0 + 4 * r < ti.n_valid)
                p.out[(size_t)(ti.row_start + c0 + 4 * r) * p.M_per + o] = f2bf(t * w);
            }
          }
        } else if (EPI == 0) {
          // Rows 32q..32q+15 of the tile are gate rows, 32q+16..32q+31 the
          // matching up rows. For columns (i, i+16) of a chunk, lanes l and
          // l^16 swap one value so that every lane computes one h.
          const float s_gate = bscale * p.a_global[2 * ti.seg];
          const float s_up = bscale * p.a_global[2 * ti.seg + 1];
          const bool lo = lane < 16;
          const int j = mt * (kBM / 2) + 16 * q + (lane & 15);
          const int hcols = p.M_per / 2;
          float amax = 0.0f;
  #pragma unroll
          for (int ch = 0; ch < kChunks; ++ch) {
            const int c0 = 32 * half + 64 * ch;
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
          const float scale = bscale * p.a_global[ti.seg];
          const int o = mt * kBM + 32 * q + lane;
  #pragma unroll
          for (int ch = 0; ch < kChunks; ++ch) {
            const int c0 = 32 * half + 64 * ch;
            if (c0 >= ti.n_valid) break;
            const float wmine =
                c0 + lane < ti.n_valid ? p.row_weight[ti.row_start + c0 + lane] * scale : 0.0f;
  #pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float w = __shfl_sync(0xffffffffu, wmine, i);
              if (c0 + i < ti.n_valid)
                p.out[(size_t)(ti.row_start + c0 + i) * p.M_per + o] =
                    f2bf(__uint_as_float(v[ch][i]) * w);
            }
          }
        }
      }
      if (++acc == C::kAcc) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::kTmemCols);
}

template <int BN, int EPI, int MX, int TM = 0, int MH = 1>
cudaError_t launch_impl(const CUtensorMap* ta, const CUtensorMap* tb, const GemmParams& p,
                        int num_sms, cudaStream_t st) {
  using C = Cfg<BN, MX, MH>;
  auto kern = nvfp4_grouped_gemm_kernel<BN, EPI, MX, TM, MH>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)C::kSmem);
  if (e != cudaSuccess) return e;
  // setmaxnreg.inc waits until the block's launch registers cover the split;
  // refuse a build whose launch register count could not.
  cudaFuncAttributes fa{};
  e = cudaFuncGetAttributes(&fa, kern);
  if (e != cudaSuccess) return e;
  if ((size_t)fa.numRegs * kThreads < 256u * (kRegsLow + kRegsEpi)) return cudaErrorInvalidConfiguration;
  kern<<<num_sms, kThreads, C::kSmem, st>>>(*ta, tb[0], tb[1], tb[2], p);
  return cudaGetLastError();
}

}  // namespace

size_t nvfp4_gemm_smem_bytes(int bn) {
  switch (bn) {
    case 32: return Cfg<32, 0>::kSmem;
    case 64: return Cfg<64, 0>::kSmem;
    case 128: return Cfg<128, 0>::kSmem;
    case 256: return Cfg<256, 0>::kSmem;
  }
  return 0;
}

cudaError_t launch_nvfp4_grouped_gemm(int bn, int epi, const CUtensorMap* tmap_a,
                                      const CUtensorMap* tmap_b, const GemmParams& p,
                                      int num_sms, cudaStream_t st, int mxfp4, int weight_rows) {
  if (p.nseg > kMaxSeg || p.K % 256 || p.M_per % kBM) return cudaErrorInvalidValue;
  if (epi == 2) {
    // token-major down projection (tmap_a: token rows, box 128; tmap_b[2]:
    // weight rows, box 128)
    if (mxfp4 || p.M_per % 256) return cudaErrorInvalidValue;
    return launch_impl<256, 1, 0, 1>(tmap_a, tmap_b, p, num_sms, st);
  }
  if (weight_rows == 256 && bn <= 64) {
    // 256 weight rows per tile in two halves (narrow token tiles)
    if (p.M_per % 256) return cudaErrorInvalidValue;
#define G5_CASE2(BN_)                                                                   \
  case BN_:                                                                             \
    if (mxfp4)                                                                          \
      return epi == 0 ? launch_impl<BN_, 0, 1, 0, 2>(tmap_a, tmap_b, p, num_sms, st)    \
                      : launch_impl<BN_, 1, 1, 0, 2>(tmap_a, tmap_b, p, num_sms, st);   \
    return epi == 0 ? launch_impl<BN_, 0, 0, 0, 2>(tmap_a, tmap_b, p, num_sms, st)      \
                    : launch_impl<BN_, 1, 0, 0, 2>(tmap_a, tmap_b, p, num_sms, st);
    switch (bn) {
      G5_CASE2(32)
      G5_CASE2(64)
    }
#undef G5_CASE2
    return cudaErrorInvalidValue;
  }
#define G5_CASE(BN_)                                                                     \
  case BN_:                                                                              \
    if (mxfp4)                                                                           \
      return epi == 0 ? launch_impl<BN_, 0, 1>(tmap_a, tmap_b, p, num_sms, st)           \
                      : launch_impl<BN_, 1, 1>(tmap_a, tmap_b, p, num_sms, st);          \
    return epi == 0 ? launch_impl<BN_, 0, 0>(tmap_a, tmap_b, p, num_sms, st)             \
                    : launch_impl<BN_, 1, 0>(tmap_a, tmap_b, p, num_sms, st);
  switch (bn) {
    G5_CASE(32)
    G5_CASE(64)
    G5_CASE(128)
    G5_CASE(256)
  }
#undef G5_CASE
  return cudaErrorInvalidValue;
}

}  // namespace glm5x
