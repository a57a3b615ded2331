// gemm_fp8fp4.cuh — FP8 (e4m3) activations x FP4 (e2m1) weights with UE8M0 block scales.
//
// The recipe of the reference's A8W4 test (tests/a8w4.py:29-30, the call at :48):
//   a  = (x  [M][K] e4m3,       sfa [M][K/128] fp32 powers of two)   recipe_a = (1, 128)
//   b  = (wp [N][K/2] e2m1 x2,  sfw [N][K/32]  fp32 powers of two)   recipe_b = (1, 32)
//   out[m,n] = bf16( sum_k x[m,k] sfa[m,k/128] * w[n,k] sfw[n,k/32] )
// with the packing of the reference's quantizers (arc/testing/quant.py:51-84: e2m1 code =
// magnitude index | sign << 3, two codes per byte, even k in the low nibble).
//
// Unlike the int8 x int4 recipe, every scale is a power of two applied per 32-wide K
// block, which is exactly what the block-scaled tensor-core MMA does in hardware
// (tcgen05.mma kind::mxf8f6f4.block_scale, UE8M0 scale factors read from TMEM). So
// one fp32 accumulator covers the whole K range of a tile and the epilogue runs once
// per tile.
//
// Orientation as in gemm_a8w4.cuh: weights are the UMMA A operand (128 rows -> TMEM
// lanes), tokens the B operand (BT columns).
//   * e2m1 -> e4m3 in the unpack warpgroup (every e2m1 value is exact in e4m3), into
//     the 128-byte-swizzled K-major layout of an 8-bit UMMA operand;
//   * scale factors: the same warps write them into TMEM with tcgen05.st. For both
//     operands, row r's four UE8M0 bytes (one per 32-wide K block of a 128-K group)
//     form one 32-bit word. The MMA's 32-lane sub-partition q reads row r's word from
//     lane 32q + r % 32, column slot + r / 32, so the word goes to column r / 32 of
//     lane r % 32 in every lane quarter: the thread at lane 32q + r0 writes the words
//     of rows r0, r0+32, r0+64, r0+96 into columns 0..3. The MMA's a_sf_id / b_sf_id
//     select the byte, i.e. the K block of each K=32 UMMA. (Layout established on
//     B200 with single-UMMA probes of known scale patterns.)
//   * the activation scale is per 128-K group, so its byte is repeated four times.
//
// Roles (512 threads, as in the int8 kernel): warp 0 TMA producer, warp 1 UMMA issuer,
// warp 2 TMEM allocator, warp 3 idle, warps 4-7 unpack + scale factors, warps 8-15
// epilogue (TMEM -> bf16 -> global, once per tile).
#pragma once

#include "gemm_a8w4.cuh"
#include "sm100.cuh"

namespace arcb {
namespace fp8fp4 {

using a8w4::kGroupK;
using a8w4::kPackedRow;
using a8w4::kRows;
using a8w4::kUmmaK;
using a8w4::Work;

constexpr uint32_t kGps = 2;        // K-groups per pipeline step
constexpr uint32_t kUnpacked = 2;   // unpacked weight stages (steps)
constexpr uint32_t kLoadStages = 3;
constexpr uint32_t kDoneRing = 8;
constexpr uint32_t kBT = 128;       // tokens per tile (UMMA N)
constexpr uint32_t kSfCol = 2 * kBT;  // first TMEM column of the scale-factor slots
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kThreads = 512;

struct Params {
  CUtensorMap tm_tok;  // x [M][K] e4m3 (u8 view), box {128, BT}, SW128
  CUtensorMap tm_wp;   // wp [N][K/2] u8, box {128, 128} (two groups), SW128
  const float* sfa;    // [M][K/128]
  const float* sfw;    // [N][K/32]
  uint16_t* out;
  uint32_t M, N, K, G;
  uint32_t ldsfa, ldsfw, ldc;
  uint32_t R;          // weight rows per tile (128)
  uint32_t tiles_m, tiles_n, num_tiles;
};

struct alignas(1024) Smem {
  uint8_t w[kUnpacked][kGps][kRows * kGroupK];      // e4m3, SW128 (UMMA A)
  uint8_t tok[kLoadStages][kGps][kBT * kGroupK];    // e4m3, SW128 (UMMA B)
  uint8_t wp[kLoadStages][kRows * kPackedRow * kGps];  // packed e2m1, SW128
  uint64_t load_full[kLoadStages];
  uint64_t w_full[kUnpacked];
  uint64_t mma_done[kDoneRing];
  uint32_t xch[2][kGps][2][kRows];                  // scale words, [step parity][group][A/B][row]
  uint64_t tile_full[2];
  uint64_t tmem_empty[2];
  uint64_t xch_full[2];                             // 4 unpack warps wrote xch[b]
  uint32_t tmem_base;
  uint32_t abort;
};

__device__ __forceinline__ uint32_t done_parity(uint32_t si) { return (si / kDoneRing) & 1u; }

// Work decomposition: the same tile order as the int8 kernel.
__device__ __forceinline__ bool next_tile(const Params& p, uint32_t& cursor, Work& w) {
  const uint32_t t = blockIdx.x + cursor * gridDim.x;
  if (t >= p.num_tiles) return false;
  ++cursor;
  constexpr uint32_t kBand = 4;
  const uint32_t band = t / (kBand * p.tiles_n);
  const uint32_t rem = t - band * kBand * p.tiles_n;
  const uint32_t m_first = band * kBand;
  const uint32_t m_cnt = min(kBand, p.tiles_m - m_first);
  w.m0 = (m_first + rem % m_cnt) * kBT;
  w.n0 = (rem / m_cnt) * p.R;
  w.g_begin = 0;
  w.g_end = p.G;
  return true;
}

// Four e2m1 codes (nibbles of the low 16 bits of x, k ascending) -> four e4m3 bytes.
// Magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6} come from an 8-byte table through one byte
// permute; the sign (code bit 3) through a second permute of {0x00, 0x80}.
__device__ __forceinline__ uint32_t e2m1x4_to_e4m3(uint32_t x) {
  const uint32_t mag = __byte_perm(0x3C383000u, 0x4C484440u, x & 0x7777u);
  const uint32_t sgn = __byte_perm(0x00008000u, 0u, (x >> 3) & 0x1111u);
  return mag | sgn;
}

// 16 packed bytes (32 codes) -> 32 e4m3 bytes as two 16-byte chunks.
__device__ __forceinline__ void expand_e2m1x32(const uint4& x, uint4& lo, uint4& hi) {
  lo = make_uint4(e2m1x4_to_e4m3(x.x), e2m1x4_to_e4m3(x.x >> 16), e2m1x4_to_e4m3(x.y),
                  e2m1x4_to_e4m3(x.y >> 16));
  hi = make_uint4(e2m1x4_to_e4m3(x.z), e2m1x4_to_e4m3(x.z >> 16), e2m1x4_to_e4m3(x.w),
                  e2m1x4_to_e4m3(x.w >> 16));
}

// UE8M0 byte of a power-of-two fp32 scale (its biased exponent).
__device__ __forceinline__ uint32_t ue8m0(float s) { return (__float_as_uint(s) >> 23) & 0xFFu; }

// Block-scaled instruction descriptor: E4M3 x E4M3, UE8M0 scales, M=128, N=kBT, and the
// scale byte (K block) k of both operands.
__host__ __device__ constexpr uint32_t idesc_mxf8(uint32_t k) {
  return (k << 4) | ((kBT >> 3) << 17) | (1u << 23) | ((kRows >> 4) << 24) | (k << 29);
}

__device__ __forceinline__ void umma_mxf8(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t sfa, uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t"
      "}"
      :
      : "r"(d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
      : "memory");
}

__device__ __forceinline__ void tmem_st_32x32b_x4(uint32_t taddr, const uint32_t (&v)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr),
               "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3])
               : "memory");
}

// TMEM column of the scale-factor slot of (unpacked stage u, group h): A at +0, B at +4.
__device__ __forceinline__ uint32_t sf_col(uint32_t u, uint32_t h) { return kSfCol + (u * kGps + h) * 8u; }

__global__ void __launch_bounds__(kThreads, 1) gemm_fp8fp4_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>(smem_raw + smem_align_pad(smem_raw));
  const uint32_t warp = warp_idx_sync();
  const uint32_t lane = threadIdx.x & 31u;
  volatile uint32_t* abort = &s.abort;
  const uint32_t steps_per_tile = (p.G + kGps - 1) / kGps;

  // Probe stamps (probe build only), steps 4..11: 0-7 UMMAs issued, 8-15 unpack waits
  // passed, 16-23 stage unpacked, 24-31 loads issued; 32-35 tiles 0..3 drained by the
  // epilogue; 56 entry, 57 prologue done.
  if (threadIdx.x == 0) probe_mark(56);
  pdl_launch_dependents();
  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_tok);
      tma_prefetch_desc(&p.tm_wp);
    }
    for (uint32_t i = lane; i < kLoadStages; i += 32) mbar_init(&s.load_full[i], 1);
    for (uint32_t i = lane; i < kUnpacked; i += 32) mbar_init(&s.w_full[i], 4);
    for (uint32_t i = lane; i < kDoneRing; i += 32) mbar_init(&s.mma_done[i], 1);
    for (uint32_t i = lane; i < 2; i += 32) {
      mbar_init(&s.tile_full[i], 1);
      mbar_init(&s.tmem_empty[i], 8);  // the 8 epilogue warps
      mbar_init(&s.xch_full[i], 4);    // the 4 unpack warps
    }
    if (lane == 0) s.abort = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(&s.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = s.tmem_base;
  pdl_wait();
  if (threadIdx.x == 0) probe_mark(57);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t stage = 0, si = 0, cursor = 0;
      Work w;
      bool ok = true;
      while (ok && next_tile(p, cursor, w)) {
        for (uint32_t t = 0; t < steps_per_tile; ++t, ++si) {
          if (si >= kLoadStages &&
              !mbar_wait(&s.mma_done[(si - kLoadStages) % kDoneRing], done_parity(si - kLoadStages),
                         abort, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          const uint32_t g0 = w.g_begin + t * kGps;
          const uint32_t real = min(kGps, w.g_end - g0);
          if (si - 4u < 8u) probe_mark(24 + si - 4u);
          mbar_arrive_expect_tx(&s.load_full[stage], real * kBT * kGroupK + kRows * kPackedRow * kGps);
#pragma unroll
          for (uint32_t h = 0; h < kGps; ++h) {
            if (h < real) {
              tma_load_2d(&p.tm_tok, &s.load_full[stage], s.tok[stage][h], int32_t((g0 + h) * kGroupK),
                          int32_t(w.m0), kCacheEvictLast);
            }
          }
          tma_load_2d(&p.tm_wp, &s.load_full[stage], s.wp[stage], int32_t(g0 * kPackedRow),
                      int32_t(w.n0), kCacheEvictFirst);
          if (++stage == kLoadStages) stage = 0;
        }
      }
      const uint32_t n_drain = si < kLoadStages ? si : kLoadStages;
      for (uint32_t i = si - n_drain; i < si; ++i) {
        mbar_drain(&s.load_full[i % kLoadStages], (i / kLoadStages) & 1u);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, us = 0, uphase = 0, si = 0, ti = 0, cursor = 0;
      Work w;
      bool ok = true;
      while (ok && next_tile(p, cursor, w)) {
        const uint32_t acc = ti & 1u;
        if (ti >= 2 && !mbar_wait(&s.tmem_empty[acc], ((ti >> 1) - 1u) & 1u, abort, kStatusTimeoutMma)) {
          break;
        }
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * kBT;
        for (uint32_t t = 0; t < steps_per_tile; ++t, ++si) {
          const uint32_t t_w = mbar_test(&s.w_full[us], uphase);
          const uint32_t t_ld = mbar_test(&s.load_full[stage], phase);
          if ((t_w == 0u && !mbar_wait(&s.w_full[us], uphase, abort, kStatusTimeoutMma)) ||
              (t_ld == 0u && !mbar_wait(&s.load_full[stage], phase, abort, kStatusTimeoutMma))) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t real = min(kGps, w.g_end - (w.g_begin + t * kGps));
#pragma unroll
          for (uint32_t h = 0; h < kGps; ++h) {
            if (h >= real) break;
            const uint64_t adesc = make_sw128_kmajor_desc(s.w[us][h]);
            const uint64_t bdesc = make_sw128_kmajor_desc(s.tok[stage][h]);
            const uint32_t sfa = tmem_base + sf_col(us, h);
#pragma unroll
            for (uint32_t k = 0; k < kGroupK / kUmmaK; ++k) {
              umma_mxf8(d_tmem, desc_advance(adesc, k * kUmmaK), desc_advance(bdesc, k * kUmmaK),
                        idesc_mxf8(k), sfa, sfa + 4u, (t | h | k) != 0u ? 1u : 0u);
            }
          }
          umma_commit(&s.mma_done[si % kDoneRing]);
          if (si - 4u < 8u) probe_mark(si - 4u);
          if (++stage == kLoadStages) {
            stage = 0;
            phase ^= 1u;
          }
          if (++us == kUnpacked) {
            us = 0;
            uphase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&s.tile_full[acc]);
        ++ti;
      }
      if (si > 0u) mbar_drain(&s.mma_done[(si - 1u) % kDoneRing], done_parity(si - 1u));
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------ unpack + scale factors
    const uint32_t ut = threadIdx.x - 128;  // 0..127 = this thread's TMEM lane
    const uint32_t lane_addr = ((ut & ~31u) << 16);
    const uint32_t c16 = ut & 3u;
    uint32_t stage = 0, phase = 0, us = 0, si = 0;
    Work w;
    bool ok = true;
    const uint32_t r0 = ut & 31u;
    // Scale words. The TMEM layout needs, in every lane quarter, lane r0 holding the
    // words of rows r0 + 32c (c = 0..3). Each thread loads only its own row ut (weights:
    // 32 contiguous bytes; tokens: two floats), one step ahead of use; the four warps
    // then trade words through s.xch, guarded by the bounded mbarrier xch_full.
    struct Sf {
      uint32_t wa[kGps], wb[kGps];
    };
    auto load_sf = [&](const Work& ww, uint32_t tt, Sf& f) {
      const uint32_t n = ww.n0 + ut, m = ww.m0 + ut;
      const uint32_t g0 = ww.g_begin + tt * kGps;
#pragma unroll
      for (uint32_t h = 0; h < kGps; ++h) {
        const uint32_t g = g0 + h;
        f.wa[h] = 0x7F7F7F7Fu;
        f.wb[h] = 0x7F7F7F7Fu;
        if (g < ww.g_end) {
          if (n < p.N) {
            const float4 v = __ldg(reinterpret_cast<const float4*>(p.sfw + size_t(n) * p.ldsfw) + g);
            f.wa[h] = ue8m0(v.x) | (ue8m0(v.y) << 8) | (ue8m0(v.z) << 16) | (ue8m0(v.w) << 24);
          }
          if (m < p.M) f.wb[h] = ue8m0(__ldg(p.sfa + size_t(m) * p.ldsfa + g)) * 0x01010101u;
        }
      }
    };
    Work wn;
    uint32_t cursor_n = 0, tn = 0;
    bool have = next_tile(p, cursor_n, wn);
    Sf cur, nxt;
    if (have) load_sf(wn, 0, cur);
    while (ok && have) {
      w = wn;
      for (uint32_t t = 0; t < steps_per_tile; ++t) {
        // Publish this step's words of row ut.
        const uint32_t xb = si & 1u;
#pragma unroll
        for (uint32_t h = 0; h < kGps; ++h) {
          s.xch[xb][h][0][ut] = cur.wa[h];
          s.xch[xb][h][1][ut] = cur.wb[h];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.xch_full[xb]);
        // Position of the next step (possibly in the next tile) and its scales.
        tn = t + 1;
        bool more = true;
        if (tn == steps_per_tile) {
          tn = 0;
          more = next_tile(p, cursor_n, wn);
        }
        if (more) load_sf(tn == 0 ? wn : w, tn, nxt);
        const uint32_t t1 = mbar_test(&s.load_full[stage], phase);
        const uint32_t t2 = si >= kUnpacked ? mbar_test(&s.mma_done[(si - kUnpacked) % kDoneRing],
                                                        done_parity(si - kUnpacked))
                                            : 1u;
        if (!mbar_wait_all2(&s.load_full[stage], phase, t1, &s.mma_done[(si - kUnpacked) % kDoneRing],
                            done_parity(si - kUnpacked), t2, abort, kStatusTimeoutUnpack)) {
          ok = false;
          break;
        }
        if (ut == 0 && si - 4u < 8u) probe_mark(8 + si - 4u);
        tc_fence_after_sync();
        // Same lane mapping as the int8 kernel's unpack (conflict-free with the
        // 128-byte swizzle of the packed tile).
        const uint8_t* src = s.wp[stage];
        uint4 x[8];
#pragma unroll
        for (uint32_t i = 0; i < 8; ++i) {
          const uint32_t r = (i & 3u) * 32u + (ut >> 2), j = (i >> 2) * 4u + c16;
          x[i] = *reinterpret_cast<const uint4*>(src + r * (kGps * kPackedRow) + ((j ^ (r & 7u)) << 4));
        }
#pragma unroll
        for (uint32_t i = 0; i < 8; ++i) {
          const uint32_t r = (i & 3u) * 32u + (ut >> 2);
          uint4 lo, hi;
          expand_e2m1x32(x[i], lo, hi);
          uint8_t* row = s.w[us][i >> 2] + r * kGroupK;
          *reinterpret_cast<uint4*>(row + (((2u * c16) ^ (r & 7u)) << 4)) = lo;
          *reinterpret_cast<uint4*>(row + (((2u * c16 + 1u) ^ (r & 7u)) << 4)) = hi;
        }
        // The four warps' words of this step: lane r0 takes rows r0 + 32c.
        if (!mbar_wait_all2(&s.xch_full[xb], (si >> 1) & 1u, 0u, &s.xch_full[xb], 0u, 1u, abort,
                            kStatusTimeoutUnpack)) {
          ok = false;
          break;
        }
#pragma unroll
        for (uint32_t h = 0; h < kGps; ++h) {
          uint32_t va[4], vb[4];
#pragma unroll
          for (uint32_t c = 0; c < 4; ++c) {
            va[c] = s.xch[xb][h][0][r0 + 32u * c];
            vb[c] = s.xch[xb][h][1][r0 + 32u * c];
          }
          tmem_st_32x32b_x4(tmem_base + lane_addr + sf_col(us, h), va);
          tmem_st_32x32b_x4(tmem_base + lane_addr + sf_col(us, h) + 4u, vb);
        }
        tmem_st_wait();
        fence_proxy_async_smem();
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.w_full[us]);
        if (ut == 0 && si - 4u < 8u) probe_mark(16 + si - 4u);
        if (++stage == kLoadStages) {
          stage = 0;
          phase ^= 1u;
        }
        if (++us == kUnpacked) us = 0;
        ++si;
        cur = nxt;
        if (tn == 0) {
          have = more;
          break;  // the tile is done; `wn` holds the next one
        }
      }
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------ epilogue (per tile)
    const uint32_t ew = warp - 8;
    const uint32_t q = ew & 3u, hh = ew >> 2;
    const uint32_t nl = q * 32 + lane;
    const uint32_t col0 = hh * (kBT / 2);
    uint32_t ti = 0, cursor = 0;
    Work w;
    while (next_tile(p, cursor, w)) {
      const uint32_t acc = ti & 1u;
      if (!mbar_wait_all2(&s.tile_full[acc], (ti >> 1) & 1u, 0u, &s.tile_full[acc], 0u, 1u, abort,
                          kStatusTimeoutEpilogue)) {
        break;
      }
      tc_fence_after_sync();
      uint32_t r[kBT / 2];
      const uint32_t t_row = tmem_base + ((q * 32u) << 16) + acc * kBT + col0;
      tmem_ld_32x32b_x32(t_row, *reinterpret_cast<uint32_t(*)[32]>(r));
      tmem_ld_32x32b_x32(t_row + 32u, *reinterpret_cast<uint32_t(*)[32]>(r + 32));
      tmem_ld_wait();
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.tmem_empty[acc]);
      if (threadIdx.x == 256 && ti < 4u) probe_mark(32 + ti);
      const uint32_t n = w.n0 + nl;
      if (nl < p.R && n < p.N) {
        uint16_t* o = p.out + n;
#pragma unroll
        for (uint32_t j = 0; j < kBT / 2; ++j) {
          const uint32_t mm = w.m0 + col0 + j;
          if (mm < p.M) o[size_t(mm) * p.ldc] = __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(r[j])));
        }
      }
      ++ti;
    }
  } else if (warp == 2 || warp == 3) {
    // TMEM allocator / idle.
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace fp8fp4
}  // namespace arcb
