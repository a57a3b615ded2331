// gemm_bf16_pair.cuh — bf16 x bf16 -> bf16 GEMM on CTA pairs, C[M,N] = A[M,K] . B[N,K]^T
// (the NT layout of the reference's arc.matmul, arc/mm.py:71-79).
//
// Why pairs. Per 64-wide K block a CTA with a 128 x 256 tile moves 96 KB through its
// shared memory: 48 KB written by TMA and 48 KB read by the tensor core (A 16 KB + B
// 32 KB). At 128 B per cycle that is ~750 cycles against ~512 cycles of bf16 MMA work,
// which caps a single-CTA kernel near 70 % of the tensor peak (the one-CTA kernel in
// gemm_bf16.cuh measures 0.74). With cta_group::2 two CTAs of a cluster run one
// 256 x 256 UMMA: each holds 128 rows of A and 128 rows (N/2) of B, so per K block and
// SM 32 KB are written and 32 KB read for the same 128 x 256 x 64 MACs, 64 KB instead
// of 96 KB.
//
// Roles (256 threads per CTA, both CTAs of the pair):
//   warp 0   TMA producer: own A rows (128 x 64) and own B rows (128 x 64), SW128; the
//            bytes complete on rank 0's stage barrier
//   warp 1   rank 0 only: UMMA issuer, 4 x tcgen05.mma.cta_group::2 M=256 N=256 K=16
//            per K block; completions go to both CTAs (stage free, accumulator full)
//   warp 2   TMEM allocator (512 columns in each CTA: two 256-column accumulators)
//   warp 3   idle
//   warps 4-7 epilogue, per CTA: its 128 rows x 256 columns, tcgen05.ld 32 columns ->
//            bf16 -> 64B-swizzled smem -> TMA store; frees the accumulator on rank 0
#pragma once

#include "gemm_bf16.cuh"
#include "sm100.cuh"

namespace arcb {
namespace bf16pair {

using bf16::BK;
using bf16::kEpiCols;
using bf16::kUmmaK;

constexpr uint32_t kRowsPerCta = 128;  // A rows (and B rows) per CTA
constexpr uint32_t kTileM = 256;       // pair tile
constexpr uint32_t kTileN = 256;
constexpr uint32_t kStages = 6;
constexpr uint32_t kNumThreads = 256;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kBandM = 8;  // m-blocks per raster band (L2 reuse of B tiles)
constexpr uint32_t kStageBytes = 2 * kRowsPerCta * BK * 2;  // A + B of one CTA

struct alignas(1024) Smem {
  uint8_t a[kStages][kRowsPerCta * BK * 2];
  uint8_t b[kStages][kRowsPerCta * BK * 2];
  uint8_t cd[2][kRowsPerCta * kEpiCols * 2];
  uint64_t full[kStages];    // rank 0: both CTAs' TMA bytes of a stage
  uint64_t empty[kStages];   // each CTA: its stage was consumed by the pair UMMAs
  uint64_t tmem_full[2];     // each CTA: accumulator complete
  uint64_t tmem_empty[2];    // rank 0: both CTAs' epilogues drained the accumulator
  uint64_t drain;            // rank 0: every pair UMMA retired
  uint32_t tmem_base;
  uint32_t abort;
  uint32_t epi_ok;
};

constexpr size_t kSmemBytes = sizeof(Smem) + 1024;
static_assert(kSmemBytes <= 232448, "shared memory fits in 227 KB");

struct Params {
  CUtensorMap tm_a;  // [M][K] bf16, box {64, 128}, SW128
  CUtensorMap tm_b;  // [N][K] bf16, box {64, 128}, SW128
  CUtensorMap tm_c;  // [M][N] bf16, box {32, 128}, SW64
  uint32_t M, N, K;
  uint32_t tiles_m, tiles_n, num_tiles, num_kb;  // pair tiles of 256 x 256
};

__device__ __forceinline__ void tile_coords(const Params& p, uint32_t t, uint32_t& mb, uint32_t& nb) {
  const uint32_t band = t / (kBandM * p.tiles_n);
  const uint32_t rem = t - band * kBandM * p.tiles_n;
  const uint32_t m_first = band * kBandM;
  const uint32_t m_cnt = min(kBandM, p.tiles_m - m_first);
  mb = m_first + rem % m_cnt;
  nb = rem / m_cnt;
}

__global__ void __launch_bounds__(kNumThreads, 1) gemm_bf16_pair_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>(smem_raw + smem_align_pad(smem_raw));
  const uint32_t warp = warp_idx_sync();
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t rank = cluster_ctarank();
  const uint32_t pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;
  volatile uint32_t* abort = &s.abort;

  pdl_launch_dependents();
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tm_a);
    tma_prefetch_desc(&p.tm_b);
    tma_prefetch_desc(&p.tm_c);
    for (uint32_t i = 0; i < kStages; ++i) {
      mbar_init(&s.full[i], 1);  // rank 0's producer arrives with the pair's byte count
      mbar_init(&s.empty[i], 1);
    }
    for (uint32_t i = 0; i < 2; ++i) {
      mbar_init(&s.tmem_full[i], 1);
      mbar_init(&s.tmem_empty[i], 8);  // 4 epilogue warps x 2 CTAs
    }
    mbar_init(&s.drain, 1);
    s.abort = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc_pair(&s.tmem_base, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before_sync();
  cluster_sync_all();  // both CTAs' barriers exist before any remote arrive or TMA
  tc_fence_after_sync();
  pdl_wait();
  const uint32_t tmem_base = s.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, issued = 0;
      const uint32_t row0 = rank * kRowsPerCta;
      for (uint32_t t = pair; t < p.num_tiles; t += num_pairs) {
        uint32_t mb, nb;
        tile_coords(p, t, mb, nb);
        bool ok = true;
        for (uint32_t kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&s.empty[stage], phase ^ 1u, abort, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          const uint32_t full0 = map_to_rank(&s.full[stage], 0);
          if (rank == 0) mbar_arrive_expect_tx(&s.full[stage], 2 * kStageBytes);
          tma_load_2d_pair(&p.tm_a, full0, s.a[stage], int32_t(kb * BK), int32_t(mb * kTileM + row0),
                           kCacheEvictNormal);
          tma_load_2d_pair(&p.tm_b, full0, s.b[stage], int32_t(kb * BK), int32_t(nb * kTileN + row0),
                           kCacheEvictNormal);
          ++issued;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
      }
      // Loads still in flight land on rank 0's barriers; rank 0 waits for them there
      // (its UMMA issuer consumed every stage it issued, or the CTA aborted), and the
      // closing cluster barrier keeps this CTA's shared memory alive until then. Rank 0
      // drains its own stage barriers.
      if (rank == 0) {
        const uint32_t n_drain = issued < kStages ? issued : kStages;
        for (uint32_t i = issued - n_drain; i < issued; ++i) {
          mbar_drain(&s.full[i % kStages], (i / kStages) & 1u);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer (rank 0)
    if (rank == 0 && lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kTileM, kTileN);
      uint32_t stage = 0, phase = 0, local = 0;
      bool ok = true;
      for (uint32_t t = pair; t < p.num_tiles && ok; t += num_pairs, ++local) {
        const uint32_t acc = local & 1u;
        const uint32_t acc_phase = (local >> 1) & 1u;
        if (!mbar_wait(&s.tmem_empty[acc], acc_phase ^ 1u, abort, kStatusTimeoutMma)) break;
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * kTileN;
        for (uint32_t kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&s.full[stage], phase, abort, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint64_t adesc = make_sw128_kmajor_desc(s.a[stage]);
          const uint64_t bdesc = make_sw128_kmajor_desc(s.b[stage]);
#pragma unroll
          for (uint32_t k = 0; k < BK / kUmmaK; ++k) {
            umma_bf16_pair(d_tmem, desc_advance(adesc, k * kUmmaK * 2), desc_advance(bdesc, k * kUmmaK * 2),
                           idesc, (kb | k) != 0u ? 1u : 0u);
          }
          umma_commit_pair(&s.empty[stage], 0x3);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit_pair(&s.tmem_full[acc], 0x3);
      }
      // Every pair UMMA must retire before either CTA releases TMEM or exits.
      umma_commit_pair(&s.drain, 0x1);
      mbar_drain(&s.drain, 0);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const uint32_t q = warp & 3u;
    const uint32_t et = threadIdx.x - 128;
    const uint32_t row = q * 32 + lane;
    const uint32_t empty0[2] = {map_to_rank(&s.tmem_empty[0], 0), map_to_rank(&s.tmem_empty[1], 0)};
    uint32_t local = 0, chunk_ctr = 0;
    for (uint32_t t = pair; t < p.num_tiles; t += num_pairs, ++local) {
      uint32_t mb, nb;
      tile_coords(p, t, mb, nb);
      const uint32_t acc = local & 1u;
      const uint32_t acc_phase = (local >> 1) & 1u;
      if (et == 0) {
        s.epi_ok = mbar_wait(&s.tmem_full[acc], acc_phase, abort, kStatusTimeoutEpilogue) ? 1u : 0u;
      }
      named_barrier_sync(1, 128);
      if (*reinterpret_cast<volatile uint32_t*>(&s.epi_ok) == 0u) break;
      tc_fence_after_sync();
      const uint32_t m0 = mb * kTileM + rank * kRowsPerCta;
      const uint32_t t_row = tmem_base + ((q * 32u) << 16) + acc * kTileN;
#pragma unroll 1
      for (uint32_t c = 0; c < kTileN / kEpiCols; ++c, ++chunk_ctr) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c * kEpiCols, r);
        tmem_ld_wait();
        if (c == kTileN / kEpiCols - 1) {
          tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(empty0[acc]);
        }
        uint32_t packed[16];
#pragma unroll
        for (uint32_t i = 0; i < 16; ++i) {
          packed[i] = pack_bf16x2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
        }
        const uint32_t buf = chunk_ctr & 1u;
        if (et == 0) tma_store_wait_read<1>();
        named_barrier_sync(1, 128);
        uint8_t* cd = s.cd[buf] + row * (kEpiCols * 2);
        const uint32_t sw = (row >> 1) & 3u;  // SWIZZLE_64B: 16-byte chunk j -> j ^ sw
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
          *reinterpret_cast<uint4*>(cd + ((j ^ sw) << 4)) =
              make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
        }
        fence_proxy_async_smem();
        named_barrier_sync(1, 128);
        const uint32_t n0 = nb * kTileN + c * kEpiCols;
        // Boxes wholly past M or N (a pair tile's second half at the edge) are skipped.
        if (et == 0 && m0 < p.M && n0 < p.N) {
          tma_store_2d(&p.tm_c, s.cd[buf], int32_t(n0), int32_t(m0));
        }
        if (et == 0) tma_store_commit();
      }
    }
    if (et == 0) tma_store_wait_all<0>();
  }

  // Both CTAs stay resident until the pair's last UMMA retired (rank 0's drain) and
  // both epilogues finished with TMEM; then each frees its TMEM columns.
  tc_fence_before_sync();
  cluster_sync_all();
  if (warp == 2) {
    tc_fence_after_sync();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

}  // namespace bf16pair
}  // namespace arcb
