// gemm_a8w4.cuh — int8 activations x packed int4 weights, K-group-128 scales.
//
//   P[m,n,g] = sum_{k=128g}^{128g+127} A[m,k] * W[n,k]                (int32, exact)
//   out[m,n] = bf16( sa[m] * sum_g f32(sb[n,g]) * P[m,n,g] )           (fp32 math)
//
// A  : [M][K] int8 row-major (lda bytes), sa: [M] fp32 per-token scale
// Wp : [N][K/2] uint8, two int4 codes per byte along K, LOW nibble = even k
//      (the packing convention of the reference's quantizer,
//       arc/testing/quant.py:82-83: packed = c[2j] & 0xF | (c[2j+1] & 0xF) << 4)
// sb : [N][K/128] bf16 per-(column, K-group) weight scale, out: [M][N] bf16
//
// The reference's role for this op is a third-party FP8xFP4 GEMM called at
// tests/a8w4.py:48,70; this kernel implements the int8 x int4 recipe with the same
// (data, scale)-pair calling shape.
//
// Orientation ("swap AB", as the reference's bf16 kernel does at
// arc/include/mm.cuh:148-149): the unpacked weight tile is the UMMA M operand
// (128 weight rows -> 128 TMEM lanes) and the token tile is the UMMA N operand
// (BT tokens -> BT TMEM columns). A thread of the epilogue therefore owns one output
// column n: the weight scale sb[n,g] is one scalar per thread per group, and the
// per-token scale sa[m] is applied once per tile.
//
// int4 -> int8: each nibble is placed in the HIGH half of its byte, so the int8
// operand holds 16*w exactly (two's complement) with no sign-extension work; the
// accumulator holds 16*P (|16P| <= 16*128*127*8 < 2^22, exact in int32 and fp32) and
// the factor 1/16 is folded into the (exact) scale multiply.
//
// Roles (256 + 128*EWG threads):
//   warp 0        TMA producer: token tile [BT x 128 B] (SW128) + packed weight tile
//                 [R x 64 B] per K-group into stage s of an LS-stage ring
//   warp 1        UMMA issuer: 4 x tcgen05.mma kind::i8 M=128 N=BT K=32 per group into
//                 one of two TMEM accumulators (a fresh int32 partial per group, on
//                 top of the bias described at kBiasBits); two commits per group
//   warp 2        TMEM allocator
//   warp 3        idle
//   warps 4-7     unpack warpgroup: packed smem -> int8 SW128 smem in the same stage
//   warps 8-...   epilogue warpgroup(s): tcgen05.ld partial, re-arm the bias, fp32
//                 scale-accumulate on packed f32x2 pairs
//
// Work decomposition: persistent CTAs stride over (token tile, weight tile) pairs;
// each tile covers all K-groups and is stored through TMA. Decode-sized M (<= 32)
// uses the dedicated kernel in gemm_a8w4_decode.cuh instead.
#pragma once

#include "sm100.cuh"

namespace arcb {
namespace a8w4 {

constexpr uint32_t kRows = 128;        // UMMA M: weight rows per tile (TMEM lanes)
constexpr uint32_t kGroupK = 128;      // K elements per scale group = one 128-byte row
constexpr uint32_t kPackedRow = 64;    // bytes of packed int4 per row per group
constexpr uint32_t kUmmaK = 32;        // K per kind::i8 UMMA (32 bytes)
// Accumulator bias. Between uses every int32 accumulator column in TMEM holds
// kBiasBits, the bit pattern of kBiasF = 1.5 * 2^23, and the UMMAs of a K-group
// accumulate onto it. Since |16 P| < 2^22, the int32 sum kBiasBits + 16P is exactly
// the bit pattern of the float kBiasF + 16P, so a partial is read back as a float with
// no int->float conversion instruction (those issue on a quarter-rate pipe and would
// cap the kernel far below the tensor rate).
constexpr uint32_t kBiasBits = 0x4B400000u;
constexpr float kBiasF = 12582912.0f;
// The epilogue accumulates s_g * (kBiasF + 16P_g) and removes the accumulated bias
// sum every kBiasFlush groups: 1 + 1/kBiasFlush fp32 operations per element and
// group, with the running value never more than kBiasFlush biased terms away from the
// result (rounding error ~2^-9 of a typical partial's scale, far below a bf16 ulp).
constexpr uint32_t kBiasFlush = 4;

struct Params {
  CUtensorMap tm_tok;  // A  [M][K] u8 view of int8, box {128, BT}, SW128
  CUtensorMap tm_wp;   // Wp [N][K/2] u8, box {64, R}, no swizzle
  CUtensorMap tm_out;  // out [M][N] bf16, box {128, BT}, no swizzle
  const float* sa;
  const uint16_t* sb;
  uint16_t* out;
  int32_t* partials;   // optional [M][N][G] dump of the exact int32 group partials
  uint32_t M, N, K, G;
  uint32_t ldsb;       // elements between sb rows
  uint32_t ldc;        // elements between out rows
  uint32_t R;          // valid weight rows per tile (multiple of 8, <= 128)
  uint32_t tiles_m, tiles_n, num_tiles;
};

template <uint32_t BT, uint32_t EWG, uint32_t LS>
struct Cfg {
  static_assert(BT == 16 || BT == 32 || BT == 64 || BT == 128, "token tile");
  static_assert(EWG == 1 || EWG == 2, "epilogue warpgroups");
  static constexpr uint32_t kStages = LS;
  static constexpr uint32_t kThreads = 256 + 128 * EWG;
  static constexpr uint32_t kCols = BT / EWG;               // columns per epilogue thread
  static constexpr uint32_t kChunk = kCols < 32 ? kCols : 32;
  static constexpr uint32_t kTmemCols = (2 * BT) < 32 ? 32 : 2 * BT;
  static constexpr uint32_t kTokBytes = BT * kGroupK;
  static constexpr uint32_t kWpBytes = kRows * kPackedRow;
  static constexpr uint32_t kWBytes = kRows * kGroupK;
  static_assert(kCols % 8 == 0 && kChunk % 2 == 0, "epilogue column split");
};

// One ring of LS stages; stage s holds the token tile, the packed weight tile and
// its unpacked int8 copy of the same K-group, so a single UMMA commit per group
// (`consumed`) frees all three.
template <uint32_t BT, uint32_t EWG, uint32_t LS>
struct alignas(1024) Smem {
  using C = Cfg<BT, EWG, LS>;
  uint8_t w[LS][C::kWBytes];                    // unpacked int8, SW128 (UMMA A)
  uint8_t tok[LS][C::kTokBytes];                // tokens, SW128 (UMMA B)
  uint8_t wp[LS][C::kWpBytes];                  // packed int4 straight from TMA
  uint8_t out[BT * kRows * 2];                  // output staging [BT][128] bf16
  float sa[BT];
  uint64_t load_full[LS];                       // TMA bytes landed (tokens + packed W)
  uint64_t unpack_full[LS];                     // 4 unpack warps wrote w[s]
  uint64_t consumed[LS];                        // UMMAs of stage s finished reading it
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  uint32_t abort;
  uint32_t unpack_ok;
  uint32_t epi_ok;
};

// ---------------------------------------------------------------------------------
// Work decomposition
// ---------------------------------------------------------------------------------
struct Work {
  uint32_t m0, n0, g_begin, g_end;
};

// Tile order for the persistent decomposition: weight tiles of one band of token
// tiles first (the token tiles of a band stay L2-resident while the weights stream).
__device__ __forceinline__ void tile_of(const Params& p, uint32_t t, uint32_t& mt, uint32_t& nt) {
  constexpr uint32_t kBand = 4;
  const uint32_t band = t / (kBand * p.tiles_n);
  const uint32_t rem = t - band * kBand * p.tiles_n;
  const uint32_t m_first = band * kBand;
  const uint32_t m_cnt = min(kBand, p.tiles_m - m_first);
  mt = m_first + rem % m_cnt;
  nt = rem / m_cnt;
}

template <uint32_t BT>
__device__ __forceinline__ bool next_work(const Params& p, uint32_t& cursor, Work& w) {
  const uint32_t t = blockIdx.x + cursor * gridDim.x;
  if (t >= p.num_tiles) return false;
  ++cursor;
  uint32_t mt, nt;
  tile_of(p, t, mt, nt);
  w.m0 = mt * BT;
  w.n0 = nt * p.R;
  w.g_begin = 0;
  w.g_end = p.G;
  return true;
}

// int4 pair-packed bytes -> int8 with each code in the high nibble (value 16*w).
// x holds 4 packed bytes (8 codes, k = 0..7 with the even k in each low nibble).
__device__ __forceinline__ uint2 expand_int4x8(uint32_t x) {
  const uint32_t even = (x << 4) & 0xF0F0F0F0u;  // byte j: code k=2j   in bits 7:4
  const uint32_t odd = x & 0xF0F0F0F0u;          // byte j: code k=2j+1 in bits 7:4
  return make_uint2(__byte_perm(even, odd, 0x5140), __byte_perm(even, odd, 0x7362));
}

// ---------------------------------------------------------------------------------
// Kernel
// ---------------------------------------------------------------------------------
template <uint32_t BT, uint32_t EWG, uint32_t LS>
__global__ void __launch_bounds__(Cfg<BT, EWG, LS>::kThreads, 1)
    gemm_a8w4_kernel(const __grid_constant__ Params p) {
  using C = Cfg<BT, EWG, LS>;
  using S_t = Smem<BT, EWG, LS>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  S_t& s = *reinterpret_cast<S_t*>(smem_raw + smem_align_pad(smem_raw));
  const uint32_t warp = warp_idx_sync();
  const uint32_t lane = threadIdx.x & 31u;
  volatile uint32_t* abort = &s.abort;

  pdl_launch_dependents();
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tm_tok);
    tma_prefetch_desc(&p.tm_wp);
    tma_prefetch_desc(&p.tm_out);
    for (uint32_t i = 0; i < LS; ++i) {
      mbar_init(&s.load_full[i], 1);
      mbar_init(&s.unpack_full[i], 4);  // one arrive per unpack warp
      mbar_init(&s.consumed[i], 1);     // UMMA commit
    }
    for (uint32_t i = 0; i < 2; ++i) {
      mbar_init(&s.tmem_full[i], 1);
      mbar_init(&s.tmem_empty[i], 4 * EWG);
    }
    mbar_init(&s.drain, 1);
    s.abort = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(&s.tmem_base, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = s.tmem_base;
  if (warp >= 8) {
    // Arm both accumulators with the bias before the first UMMA may touch them.
    const uint32_t ew = warp - 8;
    const uint32_t row = tmem_base + (((ew & 3u) * 32u) << 16) + (ew >> 2) * C::kCols;
#pragma unroll
    for (uint32_t b = 0; b < 2; ++b) {
#pragma unroll
      for (uint32_t c = 0; c < C::kCols; c += 8) tmem_st_32x32b_x8_fill(row + b * BT + c, kBiasBits);
    }
    tmem_st_wait();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  // The prologue above may overlap the previous grid in the stream (programmatic
  // dependent launch); global memory is only touched after it has completed.
  pdl_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, issued = 0, cursor = 0;
      const uint32_t tx = C::kTokBytes + p.R * kPackedRow;
      Work w;
      bool ok = true;
      while (ok && next_work<BT>(p, cursor, w)) {
        for (uint32_t g = w.g_begin; g < w.g_end; ++g) {
          if (!mbar_wait(&s.consumed[stage], phase ^ 1u, abort, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&s.load_full[stage], tx);
          tma_load_2d(&p.tm_tok, &s.load_full[stage], s.tok[stage], int32_t(g * kGroupK),
                      int32_t(w.m0), kCacheEvictLast);
          tma_load_2d(&p.tm_wp, &s.load_full[stage], s.wp[stage], int32_t(g * kPackedRow),
                      int32_t(w.n0), kCacheEvictFirst);
          ++issued;
          if (++stage == LS) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      const uint32_t n_drain = issued < LS ? issued : LS;
      for (uint32_t i = issued - n_drain; i < issued; ++i) {
        mbar_drain(&s.load_full[i % LS], (i / LS) & 1u);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_s8_s32(kRows, BT);
      uint32_t stage = 0, phase = 0, gi = 0, cursor = 0;
      Work w;
      bool ok = true;
      while (ok && next_work<BT>(p, cursor, w)) {
        for (uint32_t g = w.g_begin; g < w.g_end; ++g, ++gi) {
          const uint32_t acc = gi & 1u;
          const uint32_t acc_phase = (gi >> 1) & 1u;
          if (!mbar_wait(&s.tmem_empty[acc], acc_phase ^ 1u, abort, kStatusTimeoutMma) ||
              !mbar_wait(&s.unpack_full[stage], phase, abort, kStatusTimeoutMma) ||
              !mbar_wait(&s.load_full[stage], phase, abort, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint64_t adesc = make_sw128_kmajor_desc(s.w[stage]);
          const uint64_t bdesc = make_sw128_kmajor_desc(s.tok[stage]);
          const uint32_t d_tmem = tmem_base + acc * BT;
          // Every UMMA accumulates: the group starts from the bias the epilogue left.
#pragma unroll
          for (uint32_t k = 0; k < kGroupK / kUmmaK; ++k) {
            umma_s8(d_tmem, desc_advance(adesc, k * kUmmaK), desc_advance(bdesc, k * kUmmaK), idesc,
                    1u);
          }
          umma_commit(&s.consumed[stage]);
          umma_commit(&s.tmem_full[acc]);
          if (++stage == LS) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      umma_commit(&s.drain);
      mbar_drain(&s.drain, 0);
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------ unpack warpgroup
    const uint32_t ut = threadIdx.x - 128;  // 0..127
    uint32_t stage = 0, phase = 0, cursor = 0;
    Work w;
    bool ok = true;
    while (ok && next_work<BT>(p, cursor, w)) {
      for (uint32_t g = w.g_begin; g < w.g_end; ++g) {
        if (ut == 0) {
          // Packed tile landed, and the UMMAs that read w[stage] last time are done.
          s.unpack_ok = (mbar_wait(&s.load_full[stage], phase, abort, kStatusTimeoutUnpack) &&
                         mbar_wait(&s.consumed[stage], phase ^ 1u, abort, kStatusTimeoutUnpack))
                            ? 1u
                            : 0u;
        }
        named_barrier_sync(2, 128);
        if (*reinterpret_cast<volatile uint32_t*>(&s.unpack_ok) == 0u) {
          ok = false;
          break;
        }
        const uint8_t* src = s.wp[stage];
        uint8_t* dst = s.w[stage];
        // 1024 chunks of 8 packed bytes -> 16 int8; thread ut handles chunk id = i*128+ut.
        // Reads: a warp covers 256 contiguous bytes. Writes: the 8 threads of a
        // quarter-warp fill one 128-byte swizzled row.
#pragma unroll
        for (uint32_t i = 0; i < 8; ++i) {
          const uint32_t id = i * 128u + ut;
          const uint32_t r = id >> 3, c = id & 7u;
          const uint2 x = *reinterpret_cast<const uint2*>(src + r * kPackedRow + c * 8u);
          const uint2 lo = expand_int4x8(x.x);
          const uint2 hi = expand_int4x8(x.y);
          *reinterpret_cast<uint4*>(dst + r * kGroupK + (((c ^ (r & 7u)) << 4))) =
              make_uint4(lo.x, lo.y, hi.x, hi.y);
        }
        fence_proxy_async_smem();
        __syncwarp();
        // The warp's reads of wp[stage] are complete here, so this arrival (through
        // the UMMA commit on `consumed`) is also what lets the producer refill it.
        if (lane == 0) mbar_arrive(&s.unpack_full[stage]);
        if (++stage == LS) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------ epilogue
    const uint32_t ew = warp - 8;            // 0 .. 4*EWG-1
    const uint32_t q = ew & 3u;              // TMEM lane quarter
    const uint32_t h = ew >> 2;              // column block of this warpgroup
    const uint32_t et = threadIdx.x - 256;   // 0 .. 128*EWG-1
    const uint32_t nl = q * 32 + lane;       // weight row (output column) within the tile
    const uint32_t col0 = h * C::kCols;      // first token column of this thread
    const uint32_t n_epi = 128 * EWG;
    constexpr uint32_t kPairs = C::kCols / 2;
    uint32_t gi = 0, cursor = 0;
    Work w;
    bool ok = true;
    while (ok && next_work<BT>(p, cursor, w)) {
      const uint32_t n = w.n0 + nl;
      const bool n_valid = (nl < p.R) && (n < p.N);
      uint64_t acc[kPairs];
#pragma unroll
      for (uint32_t j = 0; j < kPairs; ++j) acc[j] = 0ull;
      float bias_sum = 0.f;

      // Weight scale of the first group, then one group ahead.
      float s_next = 0.f;
      if (n_valid && w.g_begin < w.g_end) {
        s_next = bf16_bits_to_float(__ldg(p.sb + size_t(n) * p.ldsb + w.g_begin));
      }
      for (uint32_t g = w.g_begin; g < w.g_end; ++g, ++gi) {
        const float s_g = s_next * 0.0625f;  // 1/16 undoes the high-nibble placement
        if (n_valid && g + 1 < w.g_end) {
          s_next = bf16_bits_to_float(__ldg(p.sb + size_t(n) * p.ldsb + g + 1));
        }
        const uint64_t s2 = f32x2_pack(s_g, s_g);
        const uint32_t acc_b = gi & 1u;
        const uint32_t acc_phase = (gi >> 1) & 1u;
        if (et == 0) {
          s.epi_ok =
              mbar_wait(&s.tmem_full[acc_b], acc_phase, abort, kStatusTimeoutEpilogue) ? 1u : 0u;
        }
        named_barrier_sync(1, n_epi);
        if (*reinterpret_cast<volatile uint32_t*>(&s.epi_ok) == 0u) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t t_row = tmem_base + ((q * 32u) << 16) + acc_b * BT + col0;
#pragma unroll
        for (uint32_t c0 = 0; c0 < C::kCols; c0 += C::kChunk) {
          uint32_t r[C::kChunk];
          if constexpr (C::kChunk == 16) {
            tmem_ld_32x32b_x16(t_row + c0, r);
          } else {
            tmem_ld_32x32b_x32(t_row + c0, r);
          }
          tmem_ld_wait();
          if (c0 + C::kChunk == C::kCols) {
            // Every column of this thread has been read: re-arm the bias, then hand
            // the accumulator back to the UMMA issuer.
#pragma unroll
            for (uint32_t c = 0; c < C::kCols; c += 8) tmem_st_32x32b_x8_fill(t_row + c, kBiasBits);
            tmem_st_wait();
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.tmem_empty[acc_b]);
          }
#pragma unroll
          for (uint32_t j = 0; j < C::kChunk; j += 2) {
            acc[(c0 + j) / 2] = f32x2_fma(f32x2_pack(__uint_as_float(r[j]), __uint_as_float(r[j + 1])),
                                          s2, acc[(c0 + j) / 2]);
          }
          if (p.partials != nullptr && n_valid) {
#pragma unroll
            for (uint32_t j = 0; j < C::kChunk; ++j) {
              const uint32_t m = w.m0 + col0 + c0 + j;
              if (m < p.M) {
                p.partials[(size_t(m) * p.N + n) * p.G + g] =
                    static_cast<int32_t>(r[j] - kBiasBits) >> 4;
              }
            }
          }
        }
        bias_sum += s_g * kBiasF;  // exact: 8 significant bits times 2
        if ((g - w.g_begin) % kBiasFlush == kBiasFlush - 1u || g + 1 == w.g_end) {
          const uint64_t nb = f32x2_pack(-bias_sum, -bias_sum);
#pragma unroll
          for (uint32_t j = 0; j < kPairs; ++j) acc[j] = f32x2_add(acc[j], nb);
          bias_sum = 0.f;
        }
      }
      if (!ok) break;

      {
        // ---- scale by sa, stage [BT][128] bf16, one TMA store per tile.
        if (et < BT) s.sa[et] = (w.m0 + et < p.M) ? __ldg(p.sa + w.m0 + et) : 0.f;
        if (et == 0) tma_store_wait_read<0>();  // previous tile's store has read s.out
        named_barrier_sync(1, n_epi);
        uint16_t* o = reinterpret_cast<uint16_t*>(s.out);
#pragma unroll
        for (uint32_t j = 0; j < kPairs; ++j) {
          float a0, a1;
          f32x2_unpack(acc[j], a0, a1);
          o[(col0 + 2 * j) * kRows + nl] =
              __bfloat16_as_ushort(__float2bfloat16_rn(a0 * s.sa[col0 + 2 * j]));
          o[(col0 + 2 * j + 1) * kRows + nl] =
              __bfloat16_as_ushort(__float2bfloat16_rn(a1 * s.sa[col0 + 2 * j + 1]));
        }
        fence_proxy_async_smem();
        named_barrier_sync(1, n_epi);
        if (et == 0) {
          tma_store_2d(&p.tm_out, s.out, int32_t(w.n0), int32_t(w.m0));
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
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

}  // namespace a8w4
}  // namespace arcb
