// gemm_fp8fp4_pair.cuh — the FP8 x FP4 block-scaled GEMM of gemm_fp8fp4.cuh on CTA pairs.
//
// Same recipe and operands (tests/a8w4.py:29-30, :48): out = bf16(sum_k x * sfa * w * sfw)
// with e4m3 tokens, e2m1 weights and power-of-two scales per 128 (tokens) / 32 (weights)
// K elements, run as tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale.
//
// Why pairs. The tensor core reads its operands from shared memory: a 128 x 128 x 32
// UMMA step reads 8 KB (64 wavefronts of 128 B) for 0.5 M MACs, about one wavefront per
// cycle at the fp8 rate, so a one-CTA kernel saturates shared memory before the tensor
// pipe once the TMA writes (and any other shared traffic) are added; ncu showed the TC
// pipe's shared wavefronts at 45 % and LSU's at 32 % of peak with the tensor pipe 48 %
// active. A CTA pair runs one M=256 x N=256 UMMA: each CTA holds 128 weight rows and
// 128 tokens, and per 128-K group an SM moves 32 KB in by TMA and 32 KB out to the
// tensor core for 4.2 M MACs, half the shared-memory bytes per MAC.
//
// Scale factors. The fp32 scales come in by TMA as well (no per-thread copies: those
// cost one shared-memory wavefront per thread): per stage the weight scales of the
// CTA's 128 rows (box {4, 128} of sfw) and the token scales of all 256 tokens of the
// pair tile (box {4 groups, 256} of sfa; the MMA needs the B scales of the whole N in
// both CTAs, its A scales per CTA). Four converter warps per CTA turn them into UE8M0
// chunks (layout as in gemm_fp8fp4.cuh) and arrive on rank 0's stage barrier; rank 0's
// issuer copies them with tcgen05.cp.cta_group::2 (each CTA's chunks into its own TMEM)
// before the stage's UMMAs. Rows past M / N load as zero scales (2^-127) next to
// zero-filled data, so they add exactly zero.
//
// TMEM per CTA: one 256-column accumulator (its 128 weight rows x 256 tokens) plus 12
// scale columns per stage; the epilogue drains the accumulator to registers, frees it,
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
constexpr uint32_t kSfCol = kTileT;                  // scale columns follow the accumulator
constexpr uint32_t kSfSlot = 12;                     // per stage: weights 4, tokens 8
constexpr uint32_t kSfwBytes = kHalfRows * 16;       // fp32 x 4 per weight row
constexpr uint32_t kSfaBytes = kTileT * 16;          // fp32 x 4 groups per token row
constexpr uint32_t kRegsLow = 96, kRegsHigh = 160, kLaunchRegs = 128;
static_assert(kSfCol + kStages * kSfSlot <= kTmemCols, "scale-factor slots fit in TMEM");
static_assert(256 * kRegsLow + 256 * kRegsHigh <= kThreads * kLaunchRegs, "register shares");

struct Params {
  CUtensorMap tm_tok;  // x viewed [G][M][128] e4m3, box {128, 128, 1}, SW128
  CUtensorMap tm_w;    // wp viewed [G][N][128 codes] (16U4_ALIGN16B), box {128, 128, 1}, SW128
  CUtensorMap tm_sfw;  // sfw [N][K/32] fp32, box {4, 128}
  CUtensorMap tm_sfa;  // sfa [M][K/128] fp32, box {4, 256}
  uint16_t* out;
  uint32_t M, N, G, ldc;
  uint32_t tiles_m, tiles_n, num_tiles;  // pair tiles
};

struct alignas(1024) Smem {
  uint8_t tok[kStages][kTokBytes];     // this CTA's 128 tokens, e4m3, SW128
  uint8_t w[kStages][kWBytes];         // this CTA's 128 weight rows, padded e2m1, SW128
  float4 sfw_raw[kStages][kHalfRows];  // fp32 scales of the stage's group, per weight row
  float4 sfa_raw[kStages][kTileT];     // fp32 scales of 4 groups, per token row
  uint32_t sf[kStages][3][128];        // UE8M0 chunks: weights, tokens 0-127, tokens 128-255
  uint64_t full[kStages];              // rank 0: pair TMA bytes + 8 converter warps
  uint64_t sf_loaded[kStages];         // each CTA: its fp32 scales landed
  uint64_t mma_done[kStages];          // each CTA: the stage's UMMAs retired
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

// Each CTA of the pair: its own 32 x 128-bit chunk (same offset) -> its own TMEM,
// broadcast to the four lane quarters.
__device__ __forceinline__ void tmem_cp_pair_32x128b_warpx4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
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

  // Probe stamps (probe build only, rank 0), stages 4..11: 0-7 UMMAs issued, 8-15 scale
  // chunks written, 24-31 loads issued; 32-35 tiles 0..3 drained; 56 entry, 57 prologue.
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
      mbar_init(&s.full[i], 1 + 2 * 4);  // rank 0's producer (with the bytes) + 4 converter warps per CTA
      mbar_init(&s.sf_loaded[i], 1);
      mbar_init(&s.mma_done[i], 1);
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
    regs_release<kRegsLow>();
    if (lane == 0) {
      uint32_t i = 0;
      bool ok = true;
      for (uint32_t t = pair; ok && t < p.num_tiles; t += num_pairs) {
        uint32_t m0, n0;
        tile_coords(p, t, m0, n0);
        for (uint32_t g = 0; g < p.G; ++g, ++i) {
          const uint32_t st = i % kStages;
          if (i >= kStages && !mbar_wait(&s.mma_done[st], stage_parity(i) ^ 1u, abort, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          if (rank == 0 && i - 4u < 8u) probe_mark(24 + i - 4u);
          const uint32_t full0 = map_to_rank(&s.full[st], 0);
          if (rank == 0) mbar_arrive_expect_tx(&s.full[st], 2 * (kTokBytes + kWTxBytes));
          const uint32_t own_t = m0 + rank * 128u, own_w = n0 + rank * kHalfRows;
          tma_load_3d_pair(&p.tm_tok, full0, s.tok[st], 0, int32_t(own_t), int32_t(g), kCacheEvictLast);
          tma_load_3d_pair(&p.tm_w, full0, s.w[st], 0, int32_t(own_w), int32_t(g), kCacheEvictNormal);
          mbar_arrive_expect_tx(&s.sf_loaded[st], kSfwBytes + kSfaBytes);
          tma_load_2d(&p.tm_sfw, &s.sf_loaded[st], s.sfw_raw[st], int32_t(4 * g), int32_t(own_w),
                      kCacheEvictNormal);
          tma_load_2d(&p.tm_sfa, &s.sf_loaded[st], s.sfa_raw[st], int32_t(g & ~3u), int32_t(m0),
                      kCacheEvictLast);
        }
      }
      // Own scale loads land on own barriers: drain them. The pair loads complete on
      // rank 0's barriers, which rank 0 drains for both CTAs.
      const uint32_t n_drain = i < kStages ? i : kStages;
      for (uint32_t j = i - n_drain; j < i; ++j) {
        mbar_drain(&s.sf_loaded[j % kStages], stage_parity(j));
        if (rank == 0) mbar_drain(&s.full[j % kStages], stage_parity(j));
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer (rank 0)
    regs_release<kRegsLow>();
    if (rank == 0 && lane == 0) {
      uint32_t i = 0, ti = 0;
      bool ok = true;
      for (uint32_t t = pair; ok && t < p.num_tiles; t += num_pairs, ++ti) {
        if (ti > 0 && !mbar_wait(&s.tmem_empty, (ti - 1u) & 1u, abort, kStatusTimeoutMma)) break;
        tc_fence_after_sync();
        for (uint32_t g = 0; g < p.G; ++g, ++i) {
          const uint32_t st = i % kStages;
          if (!mbar_wait(&s.full[st], stage_parity(i), abort, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t sfa = tmem_base + kSfCol + st * kSfSlot, sfb = sfa + 4u;
#pragma unroll
          for (uint32_t c = 0; c < 3; ++c) {
            tmem_cp_pair_32x128b_warpx4(sfa + 4u * c, fp8fp4::make_chunk_desc(s.sf[st][c]));
          }
          const uint64_t adesc = make_sw128_kmajor_desc(s.w[st]);
          const uint64_t bdesc = make_sw128_kmajor_desc(s.tok[st]);
#pragma unroll
          for (uint32_t k = 0; k < kGroupK / kUmmaK; ++k) {
            umma_mxf8f6f4_pair(tmem_base, desc_advance(adesc, k * kUmmaK), desc_advance(bdesc, k * kUmmaK),
                               idesc_pair(k), sfa, sfb, (g | k) != 0u ? 1u : 0u);
          }
          umma_commit_pair(&s.mma_done[st], 0x3);
          if (i - 4u < 8u) probe_mark(i - 4u);
        }
        if (ok) umma_commit_pair(&s.tile_full, 0x3);
      }
      umma_commit_pair(&s.drain, 0x1);
      mbar_drain(&s.drain, 0);
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------ scale converters
    // Thread ut: weight row ut of this CTA, token rows ut and ut + 128 of the pair tile.
    regs_release<kRegsLow>();
    const uint32_t ut = threadIdx.x - 128u;
    const uint32_t widx = (ut & 31u) * 4u + (ut >> 5);
    const uint32_t full0_base = map_to_rank(&s.full[0], 0);
    uint32_t i = 0;
    for (uint32_t t = pair; t < p.num_tiles; t += num_pairs) {
      bool ok = true;
      for (uint32_t g = 0; g < p.G; ++g, ++i) {
        const uint32_t st = i % kStages;
        if (!mbar_wait_all2(&s.sf_loaded[st], stage_parity(i), 0u, &s.sf_loaded[st], 0u, 1u, abort,
                            kStatusTimeoutScales)) {
          ok = false;
          break;
        }
        const float4 v = s.sfw_raw[st][ut];
        const float* a0 = reinterpret_cast<const float*>(&s.sfa_raw[st][ut]);
        const float* a1 = reinterpret_cast<const float*>(&s.sfa_raw[st][ut + 128u]);
        using fp8fp4::ue8m0;
        s.sf[st][0][widx] = ue8m0(v.x) | (ue8m0(v.y) << 8) | (ue8m0(v.z) << 16) | (ue8m0(v.w) << 24);
        s.sf[st][1][widx] = ue8m0(a0[g & 3u]) * 0x01010101u;
        s.sf[st][2][widx] = ue8m0(a1[g & 3u]) * 0x01010101u;
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(full0_base + st * 8u);
        if (rank == 0 && ut == 0 && i - 4u < 8u) probe_mark(8 + i - 4u);
      }
      if (!ok) break;
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
    regs_release<kRegsLow>();
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
