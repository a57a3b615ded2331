// gemm_fp8fp4_pair.cuh — the FP8 x FP4 block-scaled GEMM of gemm_fp8fp4.cuh on CTA pairs.
//
// Same recipe and operands (tests/a8w4.py:29-30, :48): out = bf16(sum_k x * sfa * w * sfw)
// with e4m3 tokens, e2m1 weights and power-of-two scales per 128 (tokens) / 32 (weights)
// K elements, run as tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale.
//
// Why pairs. The tensor core reads its operands from shared memory: a 128 x 128 x 32
// UMMA step reads 8 KB (64 wavefronts of 128 B) for 0.5 M MACs, and a block-scaled UMMA
// of N=128 occupies the pipe for ~91 cycles against 64 of math (N=256: 128 cycles,
// full rate). A CTA pair runs one M=256 x N=256 UMMA: each CTA holds 128 weight rows and
// 128 tokens, and per 128-K group an SM moves 32 KB in by TMA and 32 KB out to the
// tensor core for 4.2 M MACs, at the full fp8 rate.
//
// Scale factors go straight into TMEM. Copying them from shared memory with tcgen05.cp
// costs ~290 cycles of copy bandwidth per 32x128b.warpx4 copy (measured: one copy per
// four N=256 UMMAs hides, three add ~360 cycles), and a group needs three (weights'
// 128 rows, tokens' 256 columns), which bounded the kernel. Instead four converter warps
// per CTA, one per TMEM lane quarter, write the UE8M0 words with tcgen05.st, each warp
// its own lane quarter: the MMA's quarter q reads row r's word at lane 32q + r % 32,
// column r / 32, so every warp writes the same words (rows r0 + 32c for its lane r0)
// into its quarter. Weights: 4 columns per group (A, 128 rows of this CTA); tokens: 8
// (B, all 256 tokens of the pair tile, needed in both CTAs). The MMA's a_sf_id /
// b_sf_id select the byte, i.e. the K block of each K=32 UMMA; a token's scale is per
// 128-K group, so its byte is repeated four times.
//
// The fp32 scales arrive by TMA in blocks of 8 K groups (wide box rows: the TMA engine
// moves about one box row per cycle whatever its width), double-buffered and one block
// ahead: the CTA's 128 weight rows (box {32, 128} of sfw, 128-byte swizzled so that the
// converter lanes, 32 rows at the same group, hit distinct banks) and the pair tile's
// 256 tokens (box {8, 256} of sfa). Each converter lane first gathers its rows' words for
// the whole block into registers, then writes the block group by group. The TMEM scale
// ring holds two blocks. Converters fill a block,
// then signal rank 0 once (a release at cluster scope: a memory barrier of ~2000
// cycles, so once per block, not per group); rank 0's issuer frees a block's ring slot
// with a commit after its last group. Rows past M / N and groups past K load as zero
// scales (2^-127) next to zero-filled data, so they add exactly zero.
//
// TMEM per CTA: one 256-column accumulator (its 128 weight rows x 256 tokens) plus the
// 192-column scale ring; the epilogue drains the accumulator to registers, frees it,
// then converts and stores.
//
// Roles (512 threads per CTA): warp 0 TMA producer, warp 1 UMMA issuer (rank 0), warp 2
// TMEM allocator, warp 3 idle, warps 4-7 scale converters, warps 8-15 epilogue.
#pragma once

#include "gemm_fp8fp4.cuh"
#include "sm100.cuh"

namespace arcb {
namespace fp8fp4pair {

using a8w4::kGroupK;
using a8w4::kUmmaK;
using fp8fp4::kHalfRows;
using fp8fp4::kTokBytes;
using fp8fp4::kWBytes;
using fp8fp4::kWTxBytes;

constexpr uint32_t kTileW = 256;   // weight rows per pair tile (UMMA M)
constexpr uint32_t kTileT = 256;   // tokens per pair tile (UMMA N)
constexpr uint32_t kStages = 5;    // one 128-K group each
constexpr uint32_t kThreads = 512;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kEpiWarps = 8;
constexpr uint32_t kBlk = 8;                           // K groups per scale block
constexpr uint32_t kSfCol = kTileT;                    // scale ring follows the accumulator
constexpr uint32_t kSfGroup = 12;                      // columns per group: weights 4, tokens 8
constexpr uint32_t kSfSlot = kBlk * kSfGroup;          // columns per block
constexpr uint32_t kSfwBytes = kHalfRows * kBlk * 16;  // fp32 x 4 per weight row and group
constexpr uint32_t kSfaBytes = kTileT * kBlk * 4;      // fp32 per token row and group
// Register shares per warpgroup (setmaxnreg): producer / issuer / allocator warps and the
// converters drop to kRegsCtl / kRegsConv, the epilogue (128 packed columns) rises to
// kRegsHigh, out of kLaunchRegs per thread at launch.
constexpr uint32_t kRegsCtl = 72, kRegsConv = 120, kRegsHigh = 160, kLaunchRegs = 128;
static_assert(kSfCol + 2 * kSfSlot <= kTmemCols, "accumulator and scale ring fit in TMEM");
static_assert(128 * kRegsCtl + 128 * kRegsConv + 256 * kRegsHigh <= kThreads * kLaunchRegs, "register shares");

struct Params {
  CUtensorMap tm_tok;  // x viewed [G][M][128] e4m3, box {128, 128, 1}, SW128
  CUtensorMap tm_w;    // wp viewed [G][N][128 codes] (16U4_ALIGN16B), box {128, 128, 1}, SW128
  CUtensorMap tm_sfw;  // sfw [N][K/32] fp32, box {32, 128}, SW128
  CUtensorMap tm_sfa;  // sfa [M][K/128] fp32, box {8, 256}
  uint16_t* out;
  uint32_t M, N, G, ldc;
  uint32_t tiles_m, tiles_n, num_tiles;  // pair tiles
};

struct alignas(1024) Smem {
  uint8_t tok[kStages][kTokBytes];     // this CTA's 128 tokens, e4m3, SW128
  uint8_t w[kStages][kWBytes];         // this CTA's 128 weight rows, padded e2m1, SW128
  uint8_t sfw_raw[2][kHalfRows * 128];  // fp32 weight scales of a block: [slot][row][group x 16 B], SW128
  float4 sfa_raw[2][kTileT][2];          // fp32 token scales of a block: [slot][token][groups 0-3, 4-7]
  uint64_t full[kStages];              // rank 0: pair TMA bytes of a stage
  uint64_t mma_done[kStages];          // each CTA: the stage's UMMAs retired
  uint64_t sf_loaded[2];               // each CTA: a block's fp32 scales landed
  uint64_t raw_free[2];                // each CTA: the converters read a block's fp32 scales
  uint64_t sf_ready[2];                // rank 0: both CTAs wrote a block's scales to TMEM
  uint64_t sf_free[2];                 // each CTA: the UMMAs of a block's ring slot retired
  uint64_t tile_full;                  // each CTA: accumulator complete
  uint64_t tmem_empty;                 // rank 0: both epilogues drained the accumulator
  uint64_t drain;                      // rank 0: every pair UMMA retired
  uint32_t tmem_base;
  uint32_t abort;
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;
static_assert(kSmemBytes <= 232448, "shared memory fits in 227 KB");

__device__ __forceinline__ void tile_coords(const Params& p, uint32_t t, uint32_t& m0, uint32_t& n0) {
  constexpr uint32_t kBand = 4;  // token tiles per band: their tokens stay in L2 while weights stream
  const uint32_t band = t / (kBand * p.tiles_n);
  const uint32_t rem = t - band * kBand * p.tiles_n;
  const uint32_t m_first = band * kBand;
  const uint32_t m_cnt = min(kBand, p.tiles_m - m_first);
  m0 = (m_first + rem % m_cnt) * kTileT;
  n0 = (rem / m_cnt) * kTileW;
}

// Pair block-scaled UMMA: M = 256 (idesc), A = E2M1, B = E4M3, UE8M0 scales.
__host__ __device__ constexpr uint32_t idesc_pair(uint32_t k) {
  return (k << 4) | (5u << 7) | ((kTileT >> 3) << 17) | (1u << 23) | ((kTileW >> 4) << 24) | (k << 29);
}

__device__ __forceinline__ void umma_mxf8f6f4_pair(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                   uint32_t sfa, uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t"
      "}"
      :
      : "r"(d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
      : "memory");
}

__global__ void __launch_bounds__(kThreads, 1) gemm_fp8fp4_pair_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>(smem_raw + smem_align_pad(smem_raw));
  const uint32_t warp = warp_idx_sync();
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t rank = cluster_ctarank();
  const uint32_t pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;
  volatile uint32_t* abort = &s.abort;
  auto stage_parity = [](uint32_t i) { return (i / kStages) & 1u; };

  // Probe stamps (probe build only, rank 0), stages 4..11: 0-7 UMMAs issued, 24-31 loads
  // issued; 8-15 scale blocks 0..7 in TMEM; 32-35 tiles 0..3 drained; 56 entry, 57
  // prologue done.
  if (threadIdx.x == 0 && rank == 0) probe_mark(56);
  pdl_launch_dependents();
  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_tok);
      tma_prefetch_desc(&p.tm_w);
      tma_prefetch_desc(&p.tm_sfw);
      tma_prefetch_desc(&p.tm_sfa);
    }
    for (uint32_t i = lane; i < kStages; i += 32) {
      mbar_init(&s.full[i], 1);  // rank 0's producer, with both CTAs' bytes
      mbar_init(&s.mma_done[i], 1);
    }
    for (uint32_t i = lane; i < 2; i += 32) {
      mbar_init(&s.sf_loaded[i], 1);
      mbar_init(&s.raw_free[i], 4);  // the 4 converter warps
      mbar_init(&s.sf_ready[i], 2);  // one converter thread per CTA
      mbar_init(&s.sf_free[i], 1);
    }
    if (lane == 0) {
      mbar_init(&s.tile_full, 1);
      mbar_init(&s.tmem_empty, 2 * kEpiWarps);
      mbar_init(&s.drain, 1);
      s.abort = 0;
    }
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc_pair(&s.tmem_base, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before_sync();
  cluster_sync_all();  // both CTAs' barriers exist before any remote arrive or TMA
  tc_fence_after_sync();
  const uint32_t tmem_base = s.tmem_base;
  pdl_wait();
  if (threadIdx.x == 0 && rank == 0) probe_mark(57);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    regs_release<kRegsCtl>();
    if (lane == 0) {
      uint32_t i = 0, blk = 0;  // stages and scale blocks issued
      bool ok = true;
      const uint32_t full0 = map_to_rank(&s.full[0], 0);
      // Scale blocks run one block ahead of the operand stages, with their own cursor
      // (the next block can belong to the next tile): block b+1 is issued when the
      // stages reach block b, into the raw slot the converters released after block b-1.
      uint32_t sb_t = pair, sb_g0 = 0;
      auto issue_scale_block = [&]() -> bool {
        if (sb_t >= p.num_tiles) return true;
        const uint32_t slot = blk & 1u;
        if (blk >= 2 && !mbar_wait(&s.raw_free[slot], ((blk >> 1) - 1u) & 1u, abort, kStatusTimeoutProducer)) {
          return false;
        }
        uint32_t m0s, n0s;
        tile_coords(p, sb_t, m0s, n0s);
        mbar_arrive_expect_tx(&s.sf_loaded[slot], kSfwBytes + kSfaBytes);
        tma_load_2d(&p.tm_sfw, &s.sf_loaded[slot], s.sfw_raw[slot], int32_t(4 * sb_g0),
                    int32_t(n0s + rank * kHalfRows), kCacheEvictNormal);
        tma_load_2d(&p.tm_sfa, &s.sf_loaded[slot], s.sfa_raw[slot], int32_t(sb_g0), int32_t(m0s), kCacheEvictLast);
        ++blk;
        if ((sb_g0 += kBlk) >= p.G) {
          sb_g0 = 0;
          sb_t += num_pairs;
        }
        return true;
      };
      ok = issue_scale_block();
      for (uint32_t t = pair; ok && t < p.num_tiles; t += num_pairs) {
        uint32_t m0, n0;
        tile_coords(p, t, m0, n0);
        const uint32_t own_t = m0 + rank * 128u, own_w = n0 + rank * kHalfRows;
        for (uint32_t g = 0; g < p.G; ++g, ++i) {
          const uint32_t st = i % kStages;
          if (i >= kStages && !mbar_wait(&s.mma_done[st], stage_parity(i) ^ 1u, abort, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          if (rank == 0 && i - 4u < 8u) probe_mark(24 + i - 4u);
          if (g % kBlk == 0 && !issue_scale_block()) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&s.full[st], 2 * (kTokBytes + kWTxBytes));
          tma_load_3d_pair(&p.tm_tok, full0 + st * 8u, s.tok[st], 0, int32_t(own_t), int32_t(g), kCacheEvictLast);
          tma_load_3d_pair(&p.tm_w, full0 + st * 8u, s.w[st], 0, int32_t(own_w), int32_t(g), kCacheEvictNormal);
        }
      }
      // Own scale loads land on own barriers: drain them. The pair loads complete on
      // rank 0's barriers, which rank 0 drains for both CTAs.
      for (uint32_t b = blk > 2u ? blk - 2u : 0u; b < blk; ++b) mbar_drain(&s.sf_loaded[b & 1u], (b >> 1) & 1u);
      if (rank == 0) {
        const uint32_t n_drain = i < kStages ? i : kStages;
        for (uint32_t j = i - n_drain; j < i; ++j) mbar_drain(&s.full[j % kStages], stage_parity(j));
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer (rank 0)
    regs_release<kRegsCtl>();
    if (rank == 0 && lane == 0) {
      uint32_t i = 0, ti = 0, blk = 0;
      bool ok = true;
      for (uint32_t t = pair; ok && t < p.num_tiles; t += num_pairs, ++ti) {
        if (ti > 0 && !mbar_wait(&s.tmem_empty, (ti - 1u) & 1u, abort, kStatusTimeoutMma)) break;
        tc_fence_after_sync();
        for (uint32_t g = 0; g < p.G; ++g, ++i) {
          const uint32_t st = i % kStages;
          const uint32_t slot = blk & 1u, gb = g % kBlk;
          const uint32_t t_ld = mbar_test(&s.full[st], stage_parity(i));
          if ((gb == 0 && !mbar_wait(&s.sf_ready[slot], (blk >> 1) & 1u, abort, kStatusTimeoutMma)) ||
              (t_ld == 0u && !mbar_wait(&s.full[st], stage_parity(i), abort, kStatusTimeoutMma))) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t sfa = tmem_base + kSfCol + slot * kSfSlot + gb * kSfGroup, sfb = sfa + 4u;
          const uint64_t adesc = make_sw128_kmajor_desc(s.w[st]);
          const uint64_t bdesc = make_sw128_kmajor_desc(s.tok[st]);
#pragma unroll
          for (uint32_t k = 0; k < kGroupK / kUmmaK; ++k) {
            umma_mxf8f6f4_pair(tmem_base, desc_advance(adesc, k * kUmmaK), desc_advance(bdesc, k * kUmmaK),
                               idesc_pair(k), sfa, sfb, (g | k) != 0u ? 1u : 0u);
          }
          umma_commit_pair(&s.mma_done[st], 0x3);
          if (gb == kBlk - 1 || g + 1 == p.G) {
            umma_commit_pair(&s.sf_free[slot], 0x3);  // the block's ring slot may be rewritten
            ++blk;
          }
          if (i - 4u < 8u) probe_mark(i - 4u);
        }
        if (ok) umma_commit_pair(&s.tile_full, 0x3);
      }
      umma_commit_pair(&s.drain, 0x1);
      mbar_drain(&s.drain, 0);
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------ scale converters
    // Warp 4 + q writes TMEM lane quarter q; lane r0 holds the words of weight rows
    // r0 + 32c (c < 4) and tokens r0 + 32c (c < 8).
    regs_release<kRegsConv>();
    const uint32_t q = warp & 3u;
    const uint32_t lane_base = tmem_base + ((q * 32u) << 16);
    const uint32_t ready0[2] = {map_to_rank(&s.sf_ready[0], 0), map_to_rank(&s.sf_ready[1], 0)};
    uint32_t blk = 0;
    bool ok = true;
    for (uint32_t t = pair; ok && t < p.num_tiles; t += num_pairs) {
      for (uint32_t g0 = 0; g0 < p.G; g0 += kBlk, ++blk) {
        const uint32_t slot = blk & 1u, n = min(kBlk, p.G - g0);
        // The block's fp32 scales landed, and the UMMAs that read the ring slot's previous
        // block retired (rank 0's commit after that block's last group).
        if (!mbar_wait_all2(&s.sf_loaded[slot], (blk >> 1) & 1u, 0u, &s.sf_free[slot], ((blk >> 1) - 1u) & 1u,
                            blk >= 2 ? 0u : 1u, abort, kStatusTimeoutScales)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        using fp8fp4::ue8m0;
        // Per half block (4 groups): gather the words of weight rows lane + 32c (c < 4)
        // (row-swizzled 16-byte chunks: conflict-free) and the bytes of tokens lane + 32c
        // (c < 8, four groups per float4) into registers, then write the 4 groups.
        const uint32_t col0 = lane_base + kSfCol + slot * kSfSlot;
#pragma unroll
        for (uint32_t hb = 0; hb < 2; ++hb) {
          uint32_t wa[4][4], tb[8];
#pragma unroll
          for (uint32_t c = 0; c < 4; ++c) {
            const uint32_t row = lane + 32u * c;
            const uint8_t* rp = s.sfw_raw[slot] + row * 128u;
#pragma unroll
            for (uint32_t j = 0; j < 4; ++j) {
              const float4 v = *reinterpret_cast<const float4*>(rp + (((4u * hb + j) ^ (row & 7u)) << 4));
              wa[c][j] = ue8m0(v.x) | (ue8m0(v.y) << 8) | (ue8m0(v.z) << 16) | (ue8m0(v.w) << 24);
            }
          }
#pragma unroll
          for (uint32_t c = 0; c < 8; ++c) {
            const float4 v = s.sfa_raw[slot][lane + 32u * c][hb];
            tb[c] = ue8m0(v.x) | (ue8m0(v.y) << 8) | (ue8m0(v.z) << 16) | (ue8m0(v.w) << 24);
          }
#pragma unroll
          for (uint32_t j = 0; j < 4; ++j) {
            const uint32_t gb = 4u * hb + j;
            if (gb < n) {
              const uint32_t wa4[4] = {wa[0][j], wa[1][j], wa[2][j], wa[3][j]};
              uint32_t wb[8];
#pragma unroll
              for (uint32_t c = 0; c < 8; ++c) wb[c] = ((tb[c] >> (8u * j)) & 0xFFu) * 0x01010101u;
              tmem_st_32x32b_x4(col0 + gb * kSfGroup, wa4);
              tmem_st_32x32b_x8(col0 + gb * kSfGroup + 4u, wb);
            }
          }
        }
        tmem_st_wait();
        // The raw slot's next block arrives by TMA (async proxy): order this warp's
        // generic reads of it before the release.
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.raw_free[slot]);  // the raw slot may take the block after next
        tc_fence_before_sync();
        named_barrier_sync(2, 128);  // the four lane quarters of the block are written
        if (warp == 4 && lane == 0) {
          mbar_arrive_cluster(ready0[slot]);
          if (rank == 0 && blk < 8u) probe_mark(8 + blk);
        }
      }
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    // Warp pair (w, w+4) shares TMEM lane quarter w % 4: tokens 0-127 and 128-255.
    regs_claim<kRegsHigh>();
    const uint32_t q = warp & 3u;
    const uint32_t c0 = ((warp - 8u) >> 2) * 128u;
    const uint32_t empty0 = map_to_rank(&s.tmem_empty, 0);
    uint32_t ti = 0;
    for (uint32_t t = pair; t < p.num_tiles; t += num_pairs, ++ti) {
      uint32_t m0, n0;
      tile_coords(p, t, m0, n0);
      if (!mbar_wait_all2(&s.tile_full, ti & 1u, 0u, &s.tile_full, 0u, 1u, abort, kStatusTimeoutEpilogue)) break;
      tc_fence_after_sync();
      uint32_t packed[64];
      const uint32_t t_row = tmem_base + ((q * 32u) << 16) + c0;
#pragma unroll
      for (uint32_t cc = 0; cc < 128; cc += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + cc, r);
        tmem_ld_wait();
#pragma unroll
        for (uint32_t j = 0; j < 16; ++j) packed[cc / 2 + j] = fp8fp4::pack_bf16x2(r[2 * j], r[2 * j + 1]);
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(empty0);
      if (threadIdx.x == 256 && rank == 0 && ti < 4u) probe_mark(32 + ti);
      const uint32_t n = n0 + rank * kHalfRows + q * 32u + lane;
      const uint32_t m_first = m0 + c0;
      if (n < p.N && m_first < p.M) {
        const uint32_t m_cnt = min(128u, p.M - m_first);
        uint16_t* o = p.out + size_t(m_first) * p.ldc + n;
#pragma unroll
        for (uint32_t j = 0; j < 128; ++j) {
          if (j < m_cnt) *o = uint16_t(packed[j / 2] >> (16u * (j & 1u)));
          o += p.ldc;
        }
      }
    }
  } else {
    regs_release<kRegsCtl>();
  }

  tc_fence_before_sync();
  cluster_sync_all();
  if (warp == 2) {
    tc_fence_after_sync();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

}  // namespace fp8fp4pair
}  // namespace arcb
