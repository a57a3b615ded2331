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
// Work moves through the pipeline in STEPS of two K-groups (kGps): one load stage,
// one unpacked stage, one commit and one accumulator pair per step, so every
// mbarrier hand-off (~250 cycles between warps on B200) is paid once per 256 K.
//
// Roles (256 + 128*EWG threads):
//   warp 0        TMA producer: per step two token boxes [BT x 128 B] (SW128) and one
//                 packed weight box [128 x 128 B] (both groups) into an LS-stage ring
//   warp 1        UMMA issuer: per group 4 x tcgen05.mma kind::i8 M=128 N=BT K=32 into
//                 its own TMEM accumulator (a fresh int32 partial per group, on top of
//                 the bias described at kBiasBits), then ONE commit per step
//   warp 2        TMEM allocator
//   warp 3        idle
//   warps 4-7     unpack warpgroup: packed smem -> int8 SW128 smem (kUnpacked-stage ring)
//   warps 8-...   epilogue warpgroup(s): tcgen05.ld partials, re-arm the bias, fp32
//                 scale-accumulate on packed f32x2 pairs, bf16 stores to global
//
// Synchronisation: the per-step commit lands on mma_done[si % 8] (si counts the CTA's
// steps). It tells the producer that load stage si % LS is free again (waited LS
// steps later), the unpack warps that unpacked stage si % kUnpacked is free
// (kUnpacked steps later) and the epilogue that accumulator pair si % 2 holds the
// step's partials. Each waiter is at most one phase behind the barrier it tests,
// which the bounds LS, kUnpacked <= 8 and 2 accumulator pairs < 8 guarantee.
//
// Work decomposition: persistent CTAs stride over (token tile, weight tile) pairs;
// each tile covers all K-groups. Decode-sized M (<= 32) uses the dedicated kernel in
// gemm_a8w4_decode.cuh instead.
#pragma once

#include "sm100.cuh"

namespace arcb {
namespace a8w4 {

constexpr uint32_t kRows = 128;        // UMMA M: weight rows per tile (TMEM lanes)
constexpr uint32_t kGroupK = 128;      // K elements per scale group = one 128-byte row
constexpr uint32_t kPackedRow = 64;    // bytes of packed int4 per row per group
constexpr uint32_t kUmmaK = 32;        // K per kind::i8 UMMA (32 bytes)
constexpr uint32_t kGps = 2;           // K-groups per pipeline step
constexpr uint32_t kUnpacked = 2;      // unpacked weight stages (steps)
constexpr uint32_t kAccPairs = 2;      // TMEM accumulator pairs (steps in flight)
constexpr uint32_t kDoneRing = 8;      // per-step completion barriers

// Accumulator bias. Between uses every int32 accumulator column in TMEM holds
// kBiasBits, the bit pattern of kBiasF = 1.5 * 2^23, and the UMMAs of a K-group
// accumulate onto it. Since |16 P| < 2^22, the int32 sum kBiasBits + 16P is exactly
// the bit pattern of the float kBiasF + 16P, so a partial is read back as a float with
// no int->float conversion instruction.
constexpr uint32_t kBiasBits = 0x4B400000u;
constexpr float kBiasF = 12582912.0f;
// The epilogue accumulates s_g * (kBiasF + 16P_g) and removes the accumulated bias
// sum every kBiasFlush groups: 1 + 1/kBiasFlush fp32 operations per element and
// group, with the running value never more than kBiasFlush biased terms away from the
// result (rounding error ~2^-9 of a typical partial's scale, far below a bf16 ulp).
constexpr uint32_t kBiasFlush = 4;
static_assert(kBiasFlush % kGps == 0, "flush on step boundaries");

struct Params {
  CUtensorMap tm_tok;  // A  [M][K] u8 view of int8, box {128, BT}, SW128
  CUtensorMap tm_wp;   // Wp [N][K/2] u8, box {128, 128} (two groups), SW128
  const float* sa;
  const uint16_t* sb;
  uint16_t* out;
  int32_t* partials;   // optional [M][N][G] dump of the exact int32 group partials
  uint32_t M, N, K, G;
  uint32_t ldsb;       // elements between sb rows
  uint32_t ldc;        // elements between out rows
  uint32_t R;          // weight rows per tile (128)
  uint32_t tiles_m, tiles_n, num_tiles;
  uint32_t split;      // Wp in the pre-packed layout (expand_piece)
};

template <uint32_t BT, uint32_t EWG, uint32_t LS>
struct Cfg {
  static_assert(BT == 64 || BT == 128, "token tile");
  static_assert(EWG == 1 || EWG == 2, "epilogue warpgroups");
  static_assert(LS >= 2 && LS <= kDoneRing && kUnpacked <= kDoneRing && kAccPairs < kDoneRing,
                "each waiter must stay within one phase of its completion barrier");
  static constexpr uint32_t kThreads = 256 + 128 * EWG;
  static constexpr uint32_t kCols = BT / EWG;               // columns per epilogue thread
  static constexpr uint32_t kChunk = 32;                    // TMEM columns per load
  static constexpr uint32_t kTmemCols = kAccPairs * kGps * BT;  // 256 or 512
  static constexpr uint32_t kTokBytes = BT * kGroupK;       // one group's token box
  static constexpr uint32_t kWpBytes = kRows * kPackedRow * kGps;
  static constexpr uint32_t kWBytes = kRows * kGroupK;      // one group's unpacked tile
  // Register budget: the producer/UMMA and unpack warpgroups drop to kRegsLow and
  // the epilogue warpgroup(s) rise to kRegsHigh, out of kLaunchRegs per thread at
  // launch (the most 1 CTA/SM allows; the host checks the compiled count).
  static constexpr uint32_t kLaunchRegs = EWG == 2 ? 128 : 168;
  static constexpr bool kSplitRegs = true;
  static constexpr uint32_t kRegsLow = EWG == 2 ? 80 : 112;
  static constexpr uint32_t kRegsHigh = EWG == 2 ? 176 : 232;
  static_assert(256 * kRegsLow + 128 * EWG * kRegsHigh <= kThreads * kLaunchRegs,
                "register shares exceed the launch budget");
  static_assert(kCols % kChunk == 0, "epilogue column split");
};

template <uint32_t BT, uint32_t EWG, uint32_t LS>
struct alignas(1024) Smem {
  using C = Cfg<BT, EWG, LS>;
  uint8_t w[kUnpacked][kGps][C::kWBytes];       // unpacked int8, SW128 (UMMA A)
  uint8_t tok[LS][kGps][C::kTokBytes];          // tokens, SW128 (UMMA B)
  uint8_t wp[LS][C::kWpBytes];                  // packed int4 [128 rows][2 x 64 B], SW128
  uint64_t load_full[LS];                       // TMA bytes landed (tokens + packed W)
  uint64_t w_full[kUnpacked];                   // 4 unpack warps wrote w[u]
  uint64_t mma_done[kDoneRing];                 // the UMMAs of step si retired
  uint64_t tmem_empty[kAccPairs];               // epilogue read accumulator pair a
  uint32_t tmem_base;
  uint32_t abort;
};

// Parity of the completion of mma_done that belongs to step si.
__device__ __forceinline__ uint32_t done_parity(uint32_t si) { return (si / kDoneRing) & 1u; }

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

// One 16-byte piece of a weight row (32 codes, k = 32q .. 32q+31) -> its 32 int8 codes
// (16*w) as two 16-byte chunks, k ascending: lo = k 0..15, hi = k 16..31.
// split == 0: the reference's packing (byte j = codes 2j | 2j+1 << 4).
// split != 0: the pre-packed layout (byte j = codes j | j+16 << 4, arc_a8w4_prepack_weights),
// where both chunks are a mask (and a shift) of the piece, with no byte permutes.
__device__ __forceinline__ void expand_piece(const uint4& x, uint32_t split, uint4& lo, uint4& hi) {
  if (split) {
    lo = make_uint4((x.x << 4) & 0xF0F0F0F0u, (x.y << 4) & 0xF0F0F0F0u, (x.z << 4) & 0xF0F0F0F0u,
                    (x.w << 4) & 0xF0F0F0F0u);
    hi = make_uint4(x.x & 0xF0F0F0F0u, x.y & 0xF0F0F0F0u, x.z & 0xF0F0F0F0u, x.w & 0xF0F0F0F0u);
  } else {
    const uint2 a = expand_int4x8(x.x), b = expand_int4x8(x.y);
    const uint2 c = expand_int4x8(x.z), d = expand_int4x8(x.w);
    lo = make_uint4(a.x, a.y, b.x, b.y);
    hi = make_uint4(c.x, c.y, d.x, d.y);
  }
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
  const uint32_t steps_per_tile = (p.G + kGps - 1) / kGps;

  // Probe stamps (probe build only): steady-state steps 4..11 of the first tile.
  //   0-7 UMMA waits passed   8-15 partials seen by the epilogue   16-23 accumulator
  //   pair released   24-31 unpack waits passed   32-39 stage unpacked   40-47 loads
  //   issued   48-55 step accumulated   56 entry   57 prologue done   59 exit
  if (threadIdx.x == 0) probe_mark(56);
  pdl_launch_dependents();
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tm_tok);
    tma_prefetch_desc(&p.tm_wp);
    for (uint32_t i = 0; i < LS; ++i) mbar_init(&s.load_full[i], 1);
    for (uint32_t i = 0; i < kUnpacked; ++i) mbar_init(&s.w_full[i], 4);  // one per unpack warp
    for (uint32_t i = 0; i < kDoneRing; ++i) mbar_init(&s.mma_done[i], 1);  // UMMA commit
    for (uint32_t i = 0; i < kAccPairs; ++i) mbar_init(&s.tmem_empty[i], 4 * EWG);
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
    // Arm every accumulator with the bias before the first UMMA may touch it.
    const uint32_t ew = warp - 8;
    const uint32_t row = tmem_base + (((ew & 3u) * 32u) << 16) + (ew >> 2) * C::kCols;
#pragma unroll
    for (uint32_t b = 0; b < kAccPairs * kGps; ++b) {
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
  if (threadIdx.x == 0) probe_mark(57);

  // Register moves sit inside each role's branch, so that the compiler gives every
  // role's code the budget of that role.
  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if constexpr (C::kSplitRegs) regs_release<C::kRegsLow>();
    if (lane == 0) {
      uint32_t stage = 0, si = 0, cursor = 0;
      Work w;
      bool ok = true;
      while (ok && next_work<BT>(p, cursor, w)) {
        for (uint32_t t = 0; t < steps_per_tile; ++t, ++si) {
          // Stage `stage` last served step si - LS; its UMMAs (which ran after the
          // unpack warps had read the packed half) must have retired.
          if (si >= LS && !mbar_wait(&s.mma_done[(si - LS) % kDoneRing], done_parity(si - LS),
                                     abort, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          if (si - 4u < 8u) probe_mark(40 + si - 4u);
          const uint32_t g0 = w.g_begin + t * kGps;
          // The last step of an odd group count has one real group: its second token
          // box is not loaded (the packed box is partly in bounds and is credited in
          // full, zero fill included).
          const uint32_t real = min(kGps, w.g_end - g0);
          mbar_arrive_expect_tx(&s.load_full[stage], real * C::kTokBytes + C::kWpBytes);
#pragma unroll
          for (uint32_t h = 0; h < kGps; ++h) {
            if (h < real) {
              tma_load_2d(&p.tm_tok, &s.load_full[stage], s.tok[stage][h],
                          int32_t((g0 + h) * kGroupK), int32_t(w.m0), kCacheEvictLast);
            }
          }
          tma_load_2d(&p.tm_wp, &s.load_full[stage], s.wp[stage], int32_t(g0 * kPackedRow),
                      int32_t(w.n0), kCacheEvictFirst);
          if (++stage == LS) stage = 0;
        }
      }
      // Let the loads still in flight land before the CTA may exit.
      const uint32_t n_drain = si < LS ? si : LS;
      for (uint32_t i = si - n_drain; i < si; ++i) {
        mbar_drain(&s.load_full[i % LS], (i / LS) & 1u);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    if constexpr (C::kSplitRegs) regs_release<C::kRegsLow>();
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_s8_s32(kRows, BT);
      uint32_t stage = 0, phase = 0, us = 0, uphase = 0, si = 0, cursor = 0;
      Work w;
      bool ok = true;
      while (ok && next_work<BT>(p, cursor, w)) {
        for (uint32_t t = 0; t < steps_per_tile; ++t, ++si) {
          const uint32_t pair = si % kAccPairs;
          const uint32_t acc_parity = (si / kAccPairs - 1u) & 1u;
          // Test all three first (their latencies overlap), block only on the others.
          const uint32_t t_acc = si >= kAccPairs ? mbar_test(&s.tmem_empty[pair], acc_parity) : 1u;
          const uint32_t t_w = mbar_test(&s.w_full[us], uphase);
          const uint32_t t_ld = mbar_test(&s.load_full[stage], phase);
          if ((t_acc == 0u && !mbar_wait(&s.tmem_empty[pair], acc_parity, abort, kStatusTimeoutMma)) ||
              (t_w == 0u && !mbar_wait(&s.w_full[us], uphase, abort, kStatusTimeoutMma)) ||
              (t_ld == 0u && !mbar_wait(&s.load_full[stage], phase, abort, kStatusTimeoutMma))) {
            ok = false;
            break;
          }
          if (si - 4u < 8u) probe_mark(si - 4u);
          tc_fence_after_sync();
          // A group past K (odd group count) is skipped: its accumulator keeps the bias
          // for the next tile, and the epilogue skips it too.
          const uint32_t real = min(kGps, w.g_end - (w.g_begin + t * kGps));
#pragma unroll
          for (uint32_t h = 0; h < kGps; ++h) {
            if (h >= real) break;
            const uint64_t adesc = make_sw128_kmajor_desc(s.w[us][h]);
            const uint64_t bdesc = make_sw128_kmajor_desc(s.tok[stage][h]);
            const uint32_t d_tmem = tmem_base + (pair * kGps + h) * BT;
            // Every UMMA accumulates: the group starts from the bias the epilogue left.
#pragma unroll
            for (uint32_t k = 0; k < kGroupK / kUmmaK; ++k) {
              umma_s8(d_tmem, desc_advance(adesc, k * kUmmaK), desc_advance(bdesc, k * kUmmaK),
                      idesc, 1u);
            }
          }
          umma_commit(&s.mma_done[si % kDoneRing]);
          if (++stage == LS) {
            stage = 0;
            phase ^= 1u;
          }
          if (++us == kUnpacked) {
            us = 0;
            uphase ^= 1u;
          }
        }
      }
      // The last commit covers every UMMA this thread issued.
      if (si > 0u) mbar_drain(&s.mma_done[(si - 1u) % kDoneRing], done_parity(si - 1u));
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------ unpack warpgroup
    if constexpr (C::kSplitRegs) regs_release<C::kRegsLow>();
    const uint32_t ut = threadIdx.x - 128;  // 0..127
    uint32_t stage = 0, phase = 0, us = 0, si = 0, cursor = 0;
    // Each warp waits for itself (no warpgroup barrier per step). The packed stage is
    // [128 rows][kGps x 64 B], landed by TMA with the 128-byte swizzle (16-byte chunk
    // j of row r at position j ^ (r & 7)). Load i of thread ut covers chunk id =
    // i*128 + ut: group h = id / 512, row r = (id % 512) / 4, K quarter c = id % 4,
    // i.e. 32 codes that become swizzled int8 chunks 2c and 2c+1 of row r of unpacked
    // tile h. A quarter-warp handles two consecutive rows of one group: its loads hit
    // 8 distinct chunk positions and its stores the even and the odd chunks of the
    // two rows, so neither has bank conflicts.
    static_assert(kGps == 2, "unpack lane mapping assumes two groups per step");
    const uint32_t c16 = ut & 3u;
    Work w;
    bool ok = true;
    while (ok && next_work<BT>(p, cursor, w)) {
      for (uint32_t t = 0; t < steps_per_tile; ++t, ++si) {
        // Packed tile landed, and the UMMAs that read w[us] last time have retired
        // (both tested at once).
        const uint32_t t1 = mbar_test(&s.load_full[stage], phase);
        const uint32_t t2 = si >= kUnpacked ? mbar_test(&s.mma_done[(si - kUnpacked) % kDoneRing],
                                                        done_parity(si - kUnpacked))
                                            : 1u;
        if (!mbar_wait_all2(&s.load_full[stage], phase, t1,
                             &s.mma_done[(si - kUnpacked) % kDoneRing], done_parity(si - kUnpacked), t2,
                             abort, kStatusTimeoutUnpack)) {
          ok = false;
          break;
        }
        if (ut == 0 && si - 4u < 8u) probe_mark(24 + si - 4u);
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
          expand_piece(x[i], p.split, lo, hi);
          uint8_t* row = s.w[us][i >> 2] + r * kGroupK;
          *reinterpret_cast<uint4*>(row + (((2u * c16) ^ (r & 7u)) << 4)) = lo;
          *reinterpret_cast<uint4*>(row + (((2u * c16 + 1u) ^ (r & 7u)) << 4)) = hi;
        }
        fence_proxy_async_smem();
        __syncwarp();
        // The warp's reads of wp[stage] completed before this arrival, and the UMMAs
        // of this step (whose commit frees the load stage) wait for it.
        if (lane == 0) mbar_arrive(&s.w_full[us]);
        if (ut == 0 && si - 4u < 8u) probe_mark(32 + si - 4u);
        if (++stage == LS) {
          stage = 0;
          phase ^= 1u;
        }
        if (++us == kUnpacked) us = 0;
      }
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------ epilogue
    if constexpr (C::kSplitRegs) regs_claim<C::kRegsHigh>();
    const uint32_t ew = warp - 8;            // 0 .. 4*EWG-1
    const uint32_t q = ew & 3u;              // TMEM lane quarter
    const uint32_t hh = ew >> 2;             // column block of this warpgroup
    const uint32_t et = threadIdx.x - 256;   // 0 .. 128*EWG-1
    const uint32_t nl = q * 32 + lane;       // weight row (output column) within the tile
    const uint32_t col0 = hh * C::kCols;     // first token column of this thread
    constexpr uint32_t kPairs = C::kCols / 2;
    // Vector scale loads need 16-byte-aligned 8-group chunks in every row.
    const bool vec_sb = (p.G % 8u == 0u) && (p.ldsb % 8u == 0u) &&
                        ((reinterpret_cast<uintptr_t>(p.sb) & 15u) == 0u);
    uint32_t si = 0, cursor = 0;
    uint32_t pre = 0;  // step si's partials seen complete by an early test
    Work w;
    bool ok = true;
    while (ok && next_work<BT>(p, cursor, w)) {
      const uint32_t n = w.n0 + nl;
      const bool n_valid = (nl < p.R) && (n < p.N);
      uint64_t acc[kPairs];
#pragma unroll
      for (uint32_t j = 0; j < kPairs; ++j) acc[j] = 0ull;
      float bias_sum = 0.f;

      // Weight scales. A scale fetched only one group ahead would expose a full L2
      // latency every group, so with 16-byte-aligned rows (the usual case) the
      // scales come in 8-group vectors two windows ahead: `win0` holds the scales
      // of the next groups (consumed 16 bits at a time), `win1` the 8 after those.
      const uint16_t* sb_row = p.sb + size_t(n) * p.ldsb;
      uint4 win0 = make_uint4(0, 0, 0, 0), win1 = make_uint4(0, 0, 0, 0);
      float s_next = 0.f;
      if (n_valid && w.g_begin < w.g_end) {
        if (vec_sb) {
          win0 = __ldg(reinterpret_cast<const uint4*>(sb_row + w.g_begin));
          if (w.g_begin + 8u < w.g_end) win1 = __ldg(reinterpret_cast<const uint4*>(sb_row + w.g_begin + 8u));
        } else {
          s_next = bf16_bits_to_float(__ldg(sb_row + w.g_begin));
        }
      }
      for (uint32_t t = 0; t < steps_per_tile; ++t, ++si) {
        const uint32_t pair = si % kAccPairs;
        if (!mbar_wait_all2(&s.mma_done[si % kDoneRing], done_parity(si), pre,
                             &s.mma_done[si % kDoneRing], done_parity(si), 1u, abort,
                             kStatusTimeoutEpilogue)) {
          ok = false;
          break;
        }
        if (et == 0 && si - 4u < 8u) probe_mark(8 + si - 4u);
        tc_fence_after_sync();
#pragma unroll
        for (uint32_t h = 0; h < kGps; ++h) {
          const uint32_t g = w.g_begin + t * kGps + h;
          if (g >= w.g_end) break;  // past K: uniform across the CTA
          float s_g;
          if (vec_sb) {
            s_g = __uint_as_float(win0.x << 16) * 0.0625f;  // 1/16: high-nibble placement
            win0.x = __funnelshift_r(win0.x, win0.y, 16);
            win0.y = __funnelshift_r(win0.y, win0.z, 16);
            win0.z = __funnelshift_r(win0.z, win0.w, 16);
            win0.w >>= 16;
            if (((g - w.g_begin) & 7u) == 7u) {
              win0 = win1;
              if (n_valid && g + 9u < w.g_end) {
                win1 = __ldg(reinterpret_cast<const uint4*>(sb_row + g + 9u));
              }
            }
          } else {
            s_g = s_next * 0.0625f;
            if (n_valid && g + 1 < w.g_end) s_next = bf16_bits_to_float(__ldg(sb_row + g + 1));
          }
          const uint64_t s2 = f32x2_pack(s_g, s_g);
          const uint32_t t_row = tmem_base + ((q * 32u) << 16) + (pair * kGps + h) * BT + col0;
          // All of this thread's columns of the group in one wait; the bias re-arm is
          // issued right away and overlaps the arithmetic.
          uint32_t r[C::kCols];
#pragma unroll
          for (uint32_t c0 = 0; c0 < C::kCols; c0 += C::kChunk) {
            tmem_ld_32x32b_x32(t_row + c0, *reinterpret_cast<uint32_t(*)[32]>(r + c0));
          }
          // Ask early whether the next step's partials are ready; the answer arrives
          // while the loads are in flight.
          if (h == 0) pre = mbar_test(&s.mma_done[(si + 1u) % kDoneRing], done_parity(si + 1u));
          tmem_ld_wait();
#pragma unroll
          for (uint32_t c = 0; c < C::kCols; c += 8) tmem_st_32x32b_x8_fill(t_row + c, kBiasBits);
#pragma unroll
          for (uint32_t j = 0; j < C::kCols; j += 2) {
            acc[j / 2] = f32x2_fma(f32x2_pack(__uint_as_float(r[j]), __uint_as_float(r[j + 1])), s2,
                                   acc[j / 2]);
          }
          if (p.partials != nullptr && n_valid) {
#pragma unroll
            for (uint32_t j = 0; j < C::kCols; ++j) {
              const uint32_t m = w.m0 + col0 + j;
              if (m < p.M) {
                p.partials[(size_t(m) * p.N + n) * p.G + g] =
                    static_cast<int32_t>(r[j] - kBiasBits) >> 4;
              }
            }
          }
          bias_sum += s_g * kBiasF;  // exact: 8 significant bits times 2
        }
        // Both accumulators of the pair are read and re-armed: hand them back.
        tmem_st_wait();
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.tmem_empty[pair]);
        if (et == 0 && si - 4u < 8u) probe_mark(16 + si - 4u);
        if ((t * kGps) % kBiasFlush == kBiasFlush - kGps || t + 1 == steps_per_tile) {
          const uint64_t nb = f32x2_pack(-bias_sum, -bias_sum);
#pragma unroll
          for (uint32_t j = 0; j < kPairs; ++j) acc[j] = f32x2_add(acc[j], nb);
          bias_sum = 0.f;
        }
        if (et == 0 && si - 4u < 8u) probe_mark(48 + si - 4u);
      }
      if (!ok) break;

      // ---- scale by sa and store: for each token m the 32 lanes of a warp write 32
      // consecutive columns (64 contiguous bytes).
      if (n_valid) {
        uint16_t* o = p.out + n;
#pragma unroll
        for (uint32_t j = 0; j < kPairs; ++j) {
          float a0, a1;
          f32x2_unpack(acc[j], a0, a1);
          const uint32_t m = w.m0 + col0 + 2 * j;
          if (m < p.M) {
            o[size_t(m) * p.ldc] = __bfloat16_as_ushort(__float2bfloat16_rn(a0 * __ldg(p.sa + m)));
          }
          if (m + 1 < p.M) {
            o[size_t(m + 1) * p.ldc] =
                __bfloat16_as_ushort(__float2bfloat16_rn(a1 * __ldg(p.sa + m + 1)));
          }
        }
      }
    }
  } else {
    // Warps 2-3 (TMEM allocator, idle) share the producer's warpgroup.
    if constexpr (C::kSplitRegs) regs_release<C::kRegsLow>();
  }

  tc_fence_before_sync();
  __syncthreads();
  if (threadIdx.x == 0) probe_mark(59);
  if (warp == 2) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

}  // namespace a8w4
}  // namespace arcb
