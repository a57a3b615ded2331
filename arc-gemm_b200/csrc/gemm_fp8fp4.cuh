// gemm_fp8fp4.cuh — FP8 (e4m3) activations x FP4 (e2m1) weights with UE8M0 block scales.
//
// The recipe of the reference's A8W4 test (tests/a8w4.py:29-30, the call at :48):
//   a  = (x  [M][K] e4m3,       sfa [M][K/128] fp32 powers of two)   recipe_a = (1, 128)
//   b  = (wp [N][K/2] e2m1 x2,  sfw [N][K/32]  fp32 powers of two)   recipe_b = (1, 32)
//   out[m,n] = bf16( sum_k x[m,k] sfa[m,k/128] * w[n,k] sfw[n,k/32] )
// with the packing of the reference's quantizers (arc/testing/quant.py:51-84: e2m1 code =
// magnitude index | sign << 3, two codes per byte, even k in the low nibble).
//
// Every scale is a power of two applied per 32-wide K block, which is what the
// block-scaled tensor-core MMA does in hardware (tcgen05.mma kind::mxf8f6f4.block_scale
// with UE8M0 scale factors in TMEM), and that MMA takes E2M1 directly as one operand
// next to E4M3 as the other. So the kernel is a plain TMA -> UMMA pipeline:
//   * weights (UMMA A, 128-row halves -> TMEM lanes) load through a tensor map of type
//     16U4_ALIGN16B: the packed codes are read from global memory as they are (64 B per
//     row per 128-K group) and land in shared memory as 8-byte runs of 16 codes padded
//     to 16 bytes, the layout the MMA reads for a 4-bit operand of kind::mxf8f6f4, in
//     the same 128-byte swizzle as the e4m3 token tile (UMMA B, 128 tokens);
//   * scale factors: four converter warps turn the fp32 scales of a K group into UE8M0
//     bytes and write them to a 512-byte shared-memory chunk per 128 rows of each
//     operand, then arrive on the stage's load barrier next to the TMA bytes; the UMMA
//     issuer copies each chunk into TMEM with tcgen05.cp (32x128b.warpx4) right before
//     the group's UMMAs (same thread, so the copy is ordered before them).
//     Chunk layout (the one the MMA reads through the copy's broadcast to all four lane
//     quarters): byte 16*r0 + 4*c + j holds row 32c + r0's scale of K block j, so the
//     MMA's lane quarter q finds row r's four bytes at lane 32q + r % 32, column r / 32.
//     The MMA's a_sf_id / b_sf_id pick the byte of each K=32 UMMA. The activation scale
//     is per 128-K group, so its byte is repeated four times.
//
// Two tile shapes (template parameter H = weight halves of 128 rows):
//   * H = 2 (large M): 256 weights x 128 tokens per CTA, two UMMAs (M=128) per K step
//     sharing the token operand. Per 128-K group the CTA reads 32 KB from L2 for 4.2 M
//     MACs, half the bytes per MAC of a 128 x 128 tile: at 128 x 128 the kernel was
//     bound by the L2 -> SM bytes it could keep in flight. TMEM then holds one
//     accumulator (256 columns) plus the scale slots, so the epilogue drains it first
//     and releases it before converting and storing.
//   * H = 1 (small M): 128 x 128 tiles (twice as many CTAs for the few tiles of a
//     decode batch), two groups per stage, double-buffered accumulators.
// In both the single issuing thread waits on one barrier per 8 UMMAs: on B200 even a
// test of a completed mbarrier phase takes ~180 cycles, which at 4 UMMAs per wait
// bounded the kernel.
//
// Roles (512 threads): warp 0 TMA producer, warp 1 UMMA issuer, warp 2 TMEM allocator,
// warp 3 idle, warps 4-7 scale converters, warps 8-15 epilogue (TMEM -> bf16 -> global
// once per tile; two warps per TMEM lane quarter).
#pragma once

#include "gemm_a8w4.cuh"
#include "sm100.cuh"

namespace arcb {
namespace fp8fp4 {

using a8w4::kGroupK;
using a8w4::kUmmaK;
using a8w4::Work;

constexpr uint32_t kBT = 128;        // tokens per tile (UMMA N)
constexpr uint32_t kHalfRows = 128;  // weight rows per UMMA (M)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kThreads = 512;
constexpr uint32_t kEpiWarps = 8;
constexpr uint32_t kSfAhead = 2;     // scale fetches (stages) in flight per converter thread
constexpr uint32_t kSfBufs = kSfAhead + 1;
constexpr uint32_t kTokBytes = kBT * kGroupK;            // e4m3 token tile of one group
constexpr uint32_t kWBytes = kHalfRows * kGroupK;        // padded e2m1 half tile in smem
constexpr uint32_t kWTxBytes = kHalfRows * kGroupK / 2;  // its transaction bytes (packed)

template <uint32_t H>
struct Cfg {
  static constexpr uint32_t kH = H;
  static constexpr uint32_t kRows = H * kHalfRows;        // weight rows per tile
  static constexpr uint32_t kGps = H == 1 ? 2 : 1;        // 128-K groups per stage
  static constexpr uint32_t kStages = H == 1 ? 3 : 4;
  static constexpr uint32_t kAccBufs = H == 1 ? 2 : 1;
  static constexpr uint32_t kAccCols = H * kBT;           // one accumulator (all halves)
  static constexpr uint32_t kSfCol = kAccBufs * kAccCols;  // first scale-slot column
  static constexpr uint32_t kSfSlot = (H + 1) * 4;         // columns per group: H weight chunks + tokens
  static_assert(kSfCol + kStages * kGps * kSfSlot <= kTmemCols, "scale-factor slots fit in TMEM");
  // H = 2 moves registers to the epilogue (it holds 128 packed columns while it drains
  // the single accumulator): warpgroups 0-1 drop to kRegsLow, 2-3 rise to kRegsHigh,
  // out of kLaunchRegs per thread at launch (the host checks the compiled count).
  static constexpr bool kSplitRegs = H == 2;
  static constexpr uint32_t kLaunchRegs = 128;
  static constexpr uint32_t kRegsLow = 96;
  static constexpr uint32_t kRegsHigh = 160;
  static_assert(256 * kRegsLow + 256 * kRegsHigh <= kThreads * kLaunchRegs,
                "register shares exceed the launch budget");
};

struct Params {
  CUtensorMap tm_tok;  // x viewed [G][M][128] e4m3, box {128, BT, groups per stage}, SW128
  CUtensorMap tm_w;    // wp viewed [G][N][128 codes] (16U4_ALIGN16B), box {128, rows, groups}, SW128
  const float* sfa;    // [M][K/128]
  const float* sfw;    // [N][K/32]
  uint16_t* out;
  uint32_t M, N, K, G;
  uint32_t ldsfa, ldsfw, ldc;
  uint32_t tiles_m, tiles_n, num_tiles;
  // K split (S > 1, for problems with fewer tiles than SMs): the S CTAs of a tile each
  // take gs consecutive K groups (a multiple of the groups per stage), write their fp32
  // partial to ws[split][m][n] and count themselves in counters[tile]; the last one
  // sums the S partials in split order (deterministic), stores the bf16 tile and
  // resets its counter to zero for the next call.
  uint32_t S, gs;
  float* ws;
  uint32_t* counters;
};

template <uint32_t H>
struct alignas(1024) Smem {
  using C = Cfg<H>;
  uint8_t tok[C::kStages][C::kGps][kTokBytes];     // e4m3, SW128 (UMMA B)
  uint8_t w[C::kStages][C::kGps][H][kWBytes];      // e2m1 in 16-byte containers of 16 codes, SW128
  uint32_t sf[C::kStages][C::kGps][H + 1][128];    // UE8M0 chunks: [..][weight halves, tokens][4*r0 + c]
  float4 sfw_stage[kSfBufs][C::kGps][C::kRows];    // fp32 weight scales of a stage
  float sfa_stage[kSfBufs][C::kGps][kBT];          // fp32 token scales of a stage
  uint64_t load_full[C::kStages];                  // TMA bytes + the 4 converter warps
  uint64_t mma_done[C::kStages];
  uint64_t tile_full[C::kAccBufs];
  uint64_t tmem_empty[C::kAccBufs];
  uint32_t tmem_base;
  uint32_t abort;
  uint32_t last;  // K split: this CTA was the last of its tile
};
static_assert(sizeof(Smem<1>) + 1024 <= 232448, "shared memory (with alignment slack) fits in 227 KB");
static_assert(sizeof(Smem<2>) + 1024 <= 232448, "shared memory (with alignment slack) fits in 227 KB");

// Asynchronous global -> shared copies (zero-filled when `valid` is false).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(valid ? 16u : 0u)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(valid ? 4u : 0u)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Work decomposition: bands of 4 token tiles sweep all weight tiles, so a wave of CTAs
// shares a few token tiles and each weight tile is read by up to 4 neighbouring CTAs.
// With a K split, work item t is split t % S of tile t / S (the splits of a tile are
// neighbours in launch order, so they run at the same time).
template <uint32_t H>
__device__ __forceinline__ bool next_tile(const Params& p, uint32_t& cursor, Work& w) {
  const uint32_t item = blockIdx.x + cursor * gridDim.x;
  if (item >= p.num_tiles * p.S) return false;
  ++cursor;
  const uint32_t t = item / p.S, split = item - t * p.S;
  constexpr uint32_t kBand = 4;
  const uint32_t band = t / (kBand * p.tiles_n);
  const uint32_t rem = t - band * kBand * p.tiles_n;
  const uint32_t m_first = band * kBand;
  const uint32_t m_cnt = min(kBand, p.tiles_m - m_first);
  w.m0 = (m_first + rem % m_cnt) * kBT;
  w.n0 = (rem / m_cnt) * Cfg<H>::kRows;
  w.g_begin = split * p.gs;
  w.g_end = min(p.G, w.g_begin + p.gs);
  return true;
}

// UE8M0 byte of a power-of-two fp32 scale (its biased exponent).
__device__ __forceinline__ uint32_t ue8m0(float s) { return (__float_as_uint(s) >> 23) & 0xFFu; }

// Block-scaled instruction descriptor: A = E2M1 (format 5), B = E4M3 (0), UE8M0 scales
// (bit 23), M = 128, N = kBT, scale byte (K block) k of both operands (bits 4-5, 29-30).
__host__ __device__ constexpr uint32_t idesc_mxf4x8(uint32_t k) {
  return (k << 4) | (5u << 7) | ((kBT >> 3) << 17) | (1u << 23) | ((kHalfRows >> 4) << 24) | (k << 29);
}

__device__ __forceinline__ void umma_mxf8f6f4(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
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

// Shared-memory descriptor of a 32-row x 16-byte chunk stored row after row (no
// swizzle, K-major): core matrices of 8 rows x 16 B stacked along M 128 B apart (stride
// offset); one core matrix along K, so the leading offset is not used.
__device__ __forceinline__ uint64_t make_chunk_desc(const void* smem) {
  const uint32_t addr = smem_u32(smem);
  uint64_t desc = 0;
  desc |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
  desc |= static_cast<uint64_t>(1u) << 16;
  desc |= static_cast<uint64_t>(128u >> 4) << 32;
  desc |= static_cast<uint64_t>(1u) << 46;
  return desc;  // layout bits 61-63 = 0: no swizzle
}

// Shared memory -> TMEM: 32 rows x 128 bits into lanes 0..31 of every lane quarter
// (columns taddr .. taddr+3). Asynchronous; ordered before later tcgen05.mma of the
// same thread and tracked by its tcgen05.commit.
__device__ __forceinline__ void tmem_cp_32x128b_warpx4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16x2(uint32_t lo, uint32_t hi) {
  return uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(lo)))) |
         (uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(hi)))) << 16);
}

template <uint32_t H>
__global__ void __launch_bounds__(kThreads, 1) gemm_fp8fp4_kernel(const __grid_constant__ Params p) {
  using C = Cfg<H>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem<H>& s = *reinterpret_cast<Smem<H>*>(smem_raw + smem_align_pad(smem_raw));
  const uint32_t warp = warp_idx_sync();
  const uint32_t lane = threadIdx.x & 31u;
  volatile uint32_t* abort = &s.abort;
  auto stage_parity = [](uint32_t i) { return (i / C::kStages) & 1u; };

  // Probe stamps (probe build only), pipeline stages 4..11: 0-7 UMMAs issued, 8-15
  // scale chunks written, 24-31 loads issued; 32-35 tiles 0..3 drained by the
  // epilogue; 56 entry, 57 prologue done.
  if (threadIdx.x == 0) probe_mark(56);
  pdl_launch_dependents();
  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_tok);
      tma_prefetch_desc(&p.tm_w);
    }
    for (uint32_t i = lane; i < C::kStages; i += 32) {
      mbar_init(&s.load_full[i], 1 + 4);  // producer (with the TMA bytes) + 4 converter warps
      mbar_init(&s.mma_done[i], 1);
    }
    for (uint32_t i = lane; i < C::kAccBufs; i += 32) {
      mbar_init(&s.tile_full[i], 1);
      mbar_init(&s.tmem_empty[i], kEpiWarps);
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
    if constexpr (C::kSplitRegs) regs_release<C::kRegsLow>();
    if (lane == 0) {
      uint32_t i = 0, cursor = 0;
      Work w;
      bool ok = true;
      while (ok && next_tile<H>(p, cursor, w)) {
        for (uint32_t g = w.g_begin; g < w.g_end; g += C::kGps, ++i) {
          const uint32_t st = i % C::kStages;
          if (i >= C::kStages &&
              !mbar_wait(&s.mma_done[st], stage_parity(i) ^ 1u, abort, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          if (i - 4u < 8u) probe_mark(24 + i - 4u);
          // A group past K (odd group count) is zero-filled and adds exactly zero; rows
          // past M or N are zero-filled too. The box bytes count in full either way.
          mbar_arrive_expect_tx(&s.load_full[st], C::kGps * (kTokBytes + H * kWTxBytes));
          tma_load_3d(&p.tm_tok, &s.load_full[st], s.tok[st], 0, int32_t(w.m0), int32_t(g), kCacheEvictLast);
          tma_load_3d(&p.tm_w, &s.load_full[st], s.w[st], 0, int32_t(w.n0), int32_t(g), kCacheEvictNormal);
        }
      }
      const uint32_t n_drain = i < C::kStages ? i : C::kStages;
      for (uint32_t j = i - n_drain; j < i; ++j) mbar_drain(&s.load_full[j % C::kStages], stage_parity(j));
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    if constexpr (C::kSplitRegs) regs_release<C::kRegsLow>();
    if (lane == 0) {
      uint32_t i = 0, ti = 0, cursor = 0;
      Work w;
      bool ok = true;
      while (ok && next_tile<H>(p, cursor, w)) {
        const uint32_t acc = ti % C::kAccBufs;
        const uint32_t use = ti / C::kAccBufs;  // earlier uses of this accumulator
        if (use > 0 && !mbar_wait(&s.tmem_empty[acc], (use - 1u) & 1u, abort, kStatusTimeoutMma)) break;
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * C::kAccCols;
        for (uint32_t g = w.g_begin; g < w.g_end; g += C::kGps, ++i) {
          const uint32_t st = i % C::kStages;
          if (!mbar_wait(&s.load_full[st], stage_parity(i), abort, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
#pragma unroll
          for (uint32_t gs = 0; gs < C::kGps; ++gs) {
            const uint32_t sf0 = tmem_base + C::kSfCol + (st * C::kGps + gs) * C::kSfSlot;
            const uint32_t sfb = sf0 + 4u * H;
#pragma unroll
            for (uint32_t h = 0; h <= H; ++h) tmem_cp_32x128b_warpx4(sf0 + 4u * h, make_chunk_desc(s.sf[st][gs][h]));
            const uint64_t bdesc = make_sw128_kmajor_desc(s.tok[st][gs]);
#pragma unroll
            for (uint32_t k = 0; k < kGroupK / kUmmaK; ++k) {
#pragma unroll
              for (uint32_t h = 0; h < H; ++h) {
                umma_mxf8f6f4(d_tmem + h * kBT, desc_advance(make_sw128_kmajor_desc(s.w[st][gs][h]), k * kUmmaK),
                              desc_advance(bdesc, k * kUmmaK), idesc_mxf4x8(k), sf0 + 4u * h, sfb,
                              (g != w.g_begin || gs != 0u || k != 0u) ? 1u : 0u);
              }
            }
          }
          umma_commit(&s.mma_done[st]);
          if (i - 4u < 8u) probe_mark(i - 4u);
        }
        if (!ok) break;
        umma_commit(&s.tile_full[acc]);
        ++ti;
      }
      if (i > 0u) mbar_drain(&s.mma_done[(i - 1u) % C::kStages], stage_parity(i - 1u));
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------ scale converters
    // Thread ut owns weight rows ut + 128h and token row ut: it fetches their fp32 scales
    // kSfAhead stages ahead with cp.async (into its own staging slots only), converts
    // them to UE8M0 words and stores the words at their places in the stage's chunks
    // once the stage is free (its previous UMMAs retired).
    if constexpr (C::kSplitRegs) regs_release<C::kRegsLow>();
    const uint32_t ut = threadIdx.x - 128u;
    const uint32_t widx = (ut & 31u) * 4u + (ut >> 5);
    struct Pos {
      Work w;
      uint32_t g, cursor;
      bool valid;
    };
    auto advance = [&](Pos& q) {
      if (q.valid && (q.g += C::kGps) >= q.w.g_end) {
        q.valid = next_tile<H>(p, q.cursor, q.w);
        q.g = q.w.g_begin;
      }
    };
    auto fetch = [&](const Pos& q, uint32_t b) {
#pragma unroll
      for (uint32_t gs = 0; gs < C::kGps; ++gs) {
        const uint32_t g = q.g + gs;
        const bool gv = q.valid && g < q.w.g_end;
#pragma unroll
        for (uint32_t h = 0; h < H; ++h) {
          const uint32_t n = q.w.n0 + h * kHalfRows + ut;
          const bool nv = gv && n < p.N;
          cp_async16(&s.sfw_stage[b][gs][h * kHalfRows + ut], p.sfw + (nv ? size_t(n) * p.ldsfw + 4u * g : 0), nv);
        }
        const bool mv = gv && q.w.m0 + ut < p.M;
        cp_async4(&s.sfa_stage[b][gs][ut], p.sfa + (mv ? size_t(q.w.m0 + ut) * p.ldsfa + g : 0), mv);
      }
      cp_async_commit();
    };
    Pos cur{}, ahead{};
    cur.valid = next_tile<H>(p, cur.cursor, cur.w);
    cur.g = cur.w.g_begin;
    ahead = cur;
    for (uint32_t b = 0; b < kSfAhead; ++b) {
      fetch(ahead, b);
      advance(ahead);
    }
    uint32_t i = 0;
    while (cur.valid) {
      const uint32_t st = i % C::kStages, b = i % kSfBufs;
      cp_async_wait<kSfAhead - 1>();
      // Rows past M / N and groups past K get scale 1 (their data is zero-filled).
      uint32_t word_w[C::kGps][H], word_a[C::kGps];
#pragma unroll
      for (uint32_t gs = 0; gs < C::kGps; ++gs) {
        const bool gv = cur.g + gs < cur.w.g_end;
#pragma unroll
        for (uint32_t h = 0; h < H; ++h) {
          const float4 v = s.sfw_stage[b][gs][h * kHalfRows + ut];
          word_w[gs][h] = gv && cur.w.n0 + h * kHalfRows + ut < p.N
                              ? (ue8m0(v.x) | (ue8m0(v.y) << 8) | (ue8m0(v.z) << 16) | (ue8m0(v.w) << 24))
                              : 0x7F7F7F7Fu;
        }
        word_a[gs] = gv && cur.w.m0 + ut < p.M ? ue8m0(s.sfa_stage[b][gs][ut]) * 0x01010101u : 0x7F7F7F7Fu;
      }
      // Buffer (i + kSfAhead) % kSfBufs was read one iteration ago, not now.
      fetch(ahead, (i + kSfAhead) % kSfBufs);
      advance(ahead);
      if (i >= C::kStages && !mbar_wait_all2(&s.mma_done[st], stage_parity(i) ^ 1u, 0u, &s.mma_done[st], 0u,
                                             1u, abort, kStatusTimeoutScales)) {
        break;
      }
#pragma unroll
      for (uint32_t gs = 0; gs < C::kGps; ++gs) {
#pragma unroll
        for (uint32_t h = 0; h < H; ++h) s.sf[st][gs][h][widx] = word_w[gs][h];
        s.sf[st][gs][H][widx] = word_a[gs];
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.load_full[st]);
      if (ut == 0 && i - 4u < 8u) probe_mark(8 + i - 4u);
      advance(cur);
      ++i;
    }
    cp_async_wait<0>();
  } else if (warp >= 8) {
    // ------------------------------------------------------------ epilogue (per tile)
    // H = 2: warp pair (w, w+4) splits the two weight halves, 128 token columns each.
    // H = 1: the pair splits the 128 token columns of the one half, 64 each.
    if constexpr (C::kSplitRegs) regs_claim<C::kRegsHigh>();
    constexpr uint32_t kCols = H == 2 ? kBT : kBT / 2;
    const uint32_t q = warp & 3u;
    const uint32_t sel = (warp - 8u) >> 2;
    const uint32_t h = H == 2 ? sel : 0u;
    const uint32_t c0 = H == 2 ? 0u : sel * kCols;
    const uint32_t nl = h * kHalfRows + q * 32 + lane;
    uint32_t ti = 0, cursor = 0;
    Work w;
    while (next_tile<H>(p, cursor, w)) {
      const uint32_t acc = ti % C::kAccBufs;
      const uint32_t use = ti / C::kAccBufs;
      if (!mbar_wait_all2(&s.tile_full[acc], use & 1u, 0u, &s.tile_full[acc], 0u, 1u, abort,
                          kStatusTimeoutEpilogue)) {
        break;
      }
      tc_fence_after_sync();
      const uint32_t t_row = tmem_base + ((q * 32u) << 16) + acc * C::kAccCols + h * kBT + c0;
      const uint32_t n = w.n0 + nl;
      const uint32_t m_first = w.m0 + c0;
      if (p.S > 1) {
        // K split: this CTA's fp32 partial goes to ws[split] (only rows m < M), then
        // the last CTA of the tile reduces.
        const uint32_t split = w.g_begin / p.gs;
        const bool mine = n < p.N && m_first < p.M;
        const uint32_t m_cnt = mine ? min(kCols, p.M - m_first) : 0u;
        float* wp_ = p.ws + (size_t(split) * p.M + m_first) * p.N + n;
#pragma unroll
        for (uint32_t cc = 0; cc < kCols; cc += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + cc, r);
          tmem_ld_wait();
          if (cc < m_cnt) {
#pragma unroll
            for (uint32_t j = 0; j < 32; ++j) {
              if (cc + j < m_cnt) wp_[size_t(cc + j) * p.N] = __uint_as_float(r[j]);
            }
          }
        }
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.tmem_empty[acc]);
        __threadfence();  // the partial is visible device-wide before this CTA is counted
        named_barrier_sync(2, 32 * kEpiWarps);
        const uint32_t tile = (blockIdx.x + (cursor - 1u) * gridDim.x) / p.S;
        if (threadIdx.x == 256) s.last = atomicAdd(p.counters + tile, 1u) == p.S - 1u ? 1u : 0u;
        named_barrier_sync(2, 32 * kEpiWarps);
        if (*reinterpret_cast<volatile uint32_t*>(&s.last) != 0u) {
          __threadfence();
          // 32 rows at a time, split-major: each split's 32 loads are independent, so
          // the reduction costs ~S L2 round trips, not S x rows.
          for (uint32_t cc = 0; cc < m_cnt; cc += 32) {
            float sum[32];
#pragma unroll
            for (uint32_t j = 0; j < 32; ++j) sum[j] = 0.f;
            for (uint32_t r = 0; r < p.S; ++r) {
              const float* src = p.ws + (size_t(r) * p.M + m_first + cc) * p.N + n;
              // Unpredicated loads (rows past m_cnt re-read the last valid row) so that
              // all 32 are in flight together.
              float v[32];
#pragma unroll
              for (uint32_t j = 0; j < 32; ++j) v[j] = __ldcg(src + size_t(min(cc + j, m_cnt - 1u) - cc) * p.N);
#pragma unroll
              for (uint32_t j = 0; j < 32; ++j) sum[j] += v[j];
            }
#pragma unroll
            for (uint32_t j = 0; j < 32; ++j) {
              if (cc + j < m_cnt) {
                p.out[size_t(m_first + cc + j) * p.ldc + n] = __bfloat16_as_ushort(__float2bfloat16_rn(sum[j]));
              }
            }
          }
          if (threadIdx.x == 256) p.counters[tile] = 0u;  // ready for the next call
        }
        ++ti;
        continue;
      }
      uint32_t packed[kCols / 2];
      // 32 columns at a time, so the raw and the packed values fit in registers.
#pragma unroll
      for (uint32_t cc = 0; cc < kCols; cc += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + cc, r);
        tmem_ld_wait();
#pragma unroll
        for (uint32_t j = 0; j < 16; ++j) packed[cc / 2 + j] = pack_bf16x2(r[2 * j], r[2 * j + 1]);
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.tmem_empty[acc]);
      if (threadIdx.x == 256 && ti < 4u) probe_mark(32 + ti);
      if (n < p.N && m_first < p.M) {
        const uint32_t m_cnt = min(kCols, p.M - m_first);
        uint16_t* o = p.out + size_t(m_first) * p.ldc + n;
#pragma unroll
        for (uint32_t j = 0; j < kCols; ++j) {
          if (j < m_cnt) *o = uint16_t(packed[j / 2] >> (16u * (j & 1u)));
          o += p.ldc;
        }
      }
      ++ti;
    }
  } else {
    // Warps 2-3: TMEM allocator / idle.
    if constexpr (C::kSplitRegs) regs_release<C::kRegsLow>();
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
