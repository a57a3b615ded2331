// gemm_bf16.cuh — bf16 x bf16 -> bf16 GEMM, C[M,N] = A[M,K] . B[N,K]^T (both K-major,
// the "NT" layout of the reference's arc.matmul, arc/mm.py:71-79).
//
// The reference kernel (arc/include/mm.cuh:31-216) runs one 128x128 tile per CTA,
// with a single TMEM accumulator and an epilogue that starts only after the last
// MMA. This kernel is persistent instead: each CTA walks a strided list of 128x256
// output tiles, and the accumulator is double-buffered in TMEM (2 x 256 fp32
// columns) so the epilogue of tile i drains while the tensor core already runs
// tile i+1.
//
// Roles (256 threads):
//   warp 0   TMA producer: A tile 128x64 and B tile 256x64 per K block (SW128)
//   warp 1   UMMA issuer: 4 x tcgen05.mma kind::f16 M=128 N=256 K=16 per K block
//   warp 2   TMEM allocator (512 columns)
//   warp 3   idle
//   warps 4-7 epilogue: tcgen05.ld 32 columns -> bf16 -> 64B-swizzled smem -> TMA store
#pragma once

#include "sm100.cuh"

namespace arcb {
namespace bf16 {

constexpr uint32_t BM = 128;
constexpr uint32_t BN = 256;
constexpr uint32_t BK = 64;  // one 128-byte swizzle row of bf16
constexpr uint32_t kStages = 4;
constexpr uint32_t kUmmaK = 16;
constexpr uint32_t kEpiCols = 32;  // output columns per store chunk
constexpr uint32_t kNumThreads = 256;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kBandM = 8;  // m-blocks per raster band (L2 reuse of B tiles)

struct alignas(1024) Smem {
  uint8_t a[kStages][BM * BK * 2];
  uint8_t b[kStages][BN * BK * 2];
  uint8_t cd[2][BM * kEpiCols * 2];
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  uint32_t abort;
  uint32_t epi_ok;  // result of the epilogue's single waiter, broadcast by a named barrier
};

constexpr size_t kSmemBytes = sizeof(Smem) + 1024;  // + slack for manual alignment

struct Params {
  CUtensorMap tm_a;  // [M][K] bf16, box {64, 128}, SW128
  CUtensorMap tm_b;  // [N][K] bf16, box {64, 256}, SW128
  CUtensorMap tm_c;  // [M][N] bf16, box {32, 128}, SW64
  uint32_t M, N, K;
  uint32_t tiles_m, tiles_n, num_tiles, num_kb;
};

__device__ __forceinline__ void tile_coords(const Params& p, uint32_t t, uint32_t& mb,
                                            uint32_t& nb) {
  const uint32_t band = t / (kBandM * p.tiles_n);
  const uint32_t rem = t - band * kBandM * p.tiles_n;
  const uint32_t m_first = band * kBandM;
  const uint32_t m_cnt = min(kBandM, p.tiles_m - m_first);
  mb = m_first + rem % m_cnt;
  nb = rem / m_cnt;
}

__global__ void __launch_bounds__(kNumThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>(smem_raw + smem_align_pad(smem_raw));
  const uint32_t warp = warp_idx_sync();
  const uint32_t lane = threadIdx.x & 31u;
  volatile uint32_t* abort = &s.abort;

  pdl_launch_dependents();
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tm_a);
    tma_prefetch_desc(&p.tm_b);
    tma_prefetch_desc(&p.tm_c);
    for (uint32_t i = 0; i < kStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (uint32_t i = 0; i < 2; ++i) {
      mbar_init(&s.tmem_full[i], 1);
      mbar_init(&s.tmem_empty[i], 4);  // one arrive per epilogue warp
    }
    mbar_init(&s.drain, 1);
    s.abort = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(&s.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  // The prologue above may overlap the previous grid in the stream (programmatic
  // dependent launch); global memory is only touched after it has completed.
  pdl_wait();
  const uint32_t tmem_base = s.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, issued = 0;
      const uint32_t tx = (BM + BN) * BK * 2;
      for (uint32_t t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
        uint32_t mb, nb;
        tile_coords(p, t, mb, nb);
        bool ok = true;
        for (uint32_t kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&s.empty[stage], phase ^ 1u, abort, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&s.full[stage], tx);
          tma_load_2d(&p.tm_a, &s.full[stage], s.a[stage], int32_t(kb * BK), int32_t(mb * BM),
                      kCacheEvictNormal);
          tma_load_2d(&p.tm_b, &s.full[stage], s.b[stage], int32_t(kb * BK), int32_t(nb * BN),
                      kCacheEvictNormal);
          ++issued;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
      }
      // Let every load still in flight land before the CTA can exit.
      const uint32_t n_drain = issued < kStages ? issued : kStages;
      for (uint32_t i = issued - n_drain; i < issued; ++i) {
        mbar_drain(&s.full[i % kStages], (i / kStages) & 1u);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      uint32_t stage = 0, phase = 0, local = 0;
      bool ok = true;
      for (uint32_t t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, ++local) {
        const uint32_t acc = local & 1u;
        const uint32_t acc_phase = (local >> 1) & 1u;
        if (!mbar_wait(&s.tmem_empty[acc], acc_phase ^ 1u, abort, kStatusTimeoutMma)) break;
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * BN;
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
            umma_bf16(d_tmem, desc_advance(adesc, k * kUmmaK * 2), desc_advance(bdesc, k * kUmmaK * 2),
                      idesc, (kb | k) != 0u ? 1u : 0u);
          }
          umma_commit(&s.empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit(&s.tmem_full[acc]);
      }
      // Every MMA issued by this thread must retire before TMEM is released.
      umma_commit(&s.drain);
      mbar_drain(&s.drain, 0);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    const uint32_t q = warp & 3u;           // TMEM lane quarter
    const uint32_t et = threadIdx.x - 128;  // 0..127
    const uint32_t row = q * 32 + lane;     // row within the tile
    uint32_t local = 0, chunk_ctr = 0;
    for (uint32_t t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++local) {
      uint32_t mb, nb;
      tile_coords(p, t, mb, nb);
      const uint32_t acc = local & 1u;
      const uint32_t acc_phase = (local >> 1) & 1u;
      // One thread waits; the named barrier hands its verdict to all four warps so
      // that they leave the loop together (bar.sync needs every one of them).
      if (et == 0) {
        s.epi_ok = mbar_wait(&s.tmem_full[acc], acc_phase, abort, kStatusTimeoutEpilogue) ? 1u : 0u;
      }
      named_barrier_sync(1, 128);
      if (*reinterpret_cast<volatile uint32_t*>(&s.epi_ok) == 0u) break;
      tc_fence_after_sync();
      const uint32_t t_row = tmem_base + ((q * 32u) << 16) + acc * BN;
#pragma unroll 1
      for (uint32_t c = 0; c < BN / kEpiCols; ++c, ++chunk_ctr) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c * kEpiCols, r);
        tmem_ld_wait();
        if (c == BN / kEpiCols - 1) {
          // Accumulator fully read: hand the buffer back to the MMA warp.
          tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s.tmem_empty[acc]);
        }
        uint32_t packed[16];
#pragma unroll
        for (uint32_t i = 0; i < 16; ++i) {
          packed[i] = pack_bf16x2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
        }
        const uint32_t buf = chunk_ctr & 1u;
        // The store issued two chunks ago from this buffer must have read it.
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
        if (et == 0) {
          tma_store_2d(&p.tm_c, s.cd[buf], int32_t(nb * BN + c * kEpiCols), int32_t(mb * BM));
          tma_store_commit();
        }
      }
    }
    if (et == 0) tma_store_wait_all<0>();
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace bf16
}  // namespace arcb
