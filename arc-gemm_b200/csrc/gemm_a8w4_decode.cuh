// gemm_a8w4_decode.cuh — A8W4 GEMM for decode-sized M (<= 32 tokens).
//
// Same arithmetic and operand formats as gemm_a8w4.cuh (int8 tokens x int4 weights
// placed in the high nibble, exact int32 group partials, fp32 scale epilogue), with a
// decomposition built for streaming the weight matrix once at HBM speed, inside a
// stream of back-to-back launches:
//
// * Every weight tile is 128 rows (TMEM lanes). With S > 1 (2 or 4) the S CTAs of a
//   cluster split the tile's K-groups and push fp32 partials to the CTA that finishes
//   each row slice through distributed shared memory (one wave, no global scratch);
//   with S == 1 CTAs are persistent over weight tiles.
// * Small footprint, so that the CTAs of the NEXT launch in the stream are resident
//   while this one runs: <= ~105 KiB of shared memory, 384 threads and 256 TMEM
//   columns per CTA (two CTAs fit on an SM). The next launch starts at once
//   (programmatic dependent launch) and, when the caller states that the weights are
//   not written by the preceding kernel (Params::static_weights), streams its weights
//   and weight scales and unpacks them BEFORE griddepcontrol.wait. Only the tokens,
//   the token scales and the output wait for the preceding grid.
// * Weights move in stages of two K-groups: one TMA box of 128 rows x 128 bytes
//   (128-byte swizzle). Each thread of the four unpack warps owns one row of a stage and
//   reads all of it into registers; it writes the first group's 128 int8 codes into a
//   TMEM slot (one tcgen05.st of 32 columns; the UMMA then takes A from TMEM) and the
//   second group's back into the same 128 bytes of shared memory, in the swizzled
//   K-major layout the UMMA reads A from. So the four ring stages hold all eight
//   K-groups of a decode CTA, unpacked, before the tokens arrive, in 64 KiB of shared
//   memory plus 128 TMEM columns.
// * Two UMMA issuer warps take alternate stages (one tcgen05.mma issuing thread needs
//   ~61 cycles per small UMMA; two keep the tensor pipe near its ~40-cycle floor for
//   N <= 32, measured on this pool's B200s). A stage is 8 UMMAs, one commit each for
//   the epilogue, the weight stage and the token stage.
// * Four epilogue warps read a stage's two int32 partials with one tcgen05.ld (one
//   TMEM lane = one output column), scale them by sb[n,g] and accumulate in fp32
//   registers. Every hand-off between roles is paid once per stage, not per group.
//
// Roles (512 threads): warp 0 TMA producer, warps 1 and 3 UMMA issuers (even / odd
// stages), warp 2 TMEM allocator, warps 4-7 and 12-15 unpack (even / odd stages: a
// stage's unpack is mostly latency, ~0.5 us per 16 KiB), warps 8-11 epilogue (warps
// 4+q, 12+q and 8+q own TMEM lanes 32q..32q+31). Registers (setmaxnreg): 64 per thread
// at launch (two CTAs per SM), the producer / issuer / allocator warpgroup drops to 40,
// the epilogue rises to 80 (BT=16) or 88 (BT=32).
//
// Every wait is bounded (sm100.cuh: mbar_wait); a timeout sets a status bit, lets the
// CTA's roles leave their loops and still pass every barrier they share.
#pragma once

#include "gemm_a8w4.cuh"
#include "sm100.cuh"

namespace arcb {
namespace a8w4dec {

using a8w4::expand_piece;
using a8w4::kGroupK;
using a8w4::kPackedRow;
using a8w4::kRows;

constexpr uint32_t kThreads = 512;
constexpr uint32_t kLaunchRegs = 64;  // 2 CTAs per SM
constexpr uint32_t kRegsUnpack = 64;
// The control warpgroup's share (producer, UMMA issuers, TMEM allocator: one lane each
// works); BT = 32 hands 8 of its registers on to the epilogue.
template <uint32_t BT>
__host__ __device__ constexpr uint32_t regs_ctl() { return BT == 16 ? 40u : 32u; }
// The epilogue's share: its BT running sums plus one stage's 32 partials and the scales.
template <uint32_t BT>
__host__ __device__ constexpr uint32_t regs_epi() { return BT == 16 ? 80u : 96u; }
static_assert(128 * (regs_ctl<16>() + 2 * kRegsUnpack + regs_epi<16>()) <= kThreads * kLaunchRegs, "register shares");
static_assert(128 * (regs_ctl<32>() + 2 * kRegsUnpack + regs_epi<32>()) <= kThreads * kLaunchRegs, "register shares");
constexpr uint32_t kTmemCols = 256;   // half an SM's TMEM: two CTAs share one SM
constexpr uint32_t kGps = 2;          // K-groups per load stage (one 128-byte box row)
constexpr uint32_t kWStageBytes = kRows * kGps * kPackedRow;  // 16 KiB of packed weights
constexpr uint32_t kWStages = 4;
constexpr uint32_t kMaxPeers = 8;     // GPUs of a fused all-gather
constexpr uint32_t kEpiThread0 = 256; // first thread of the epilogue warps

struct Params {
  CUtensorMap tm_tok;  // A as [G][M][128] u8 (3-D), box {128, BT, 2}, SW128
  CUtensorMap tm_wp;   // Wp [N][K/2] u8, box {128 B, 128 rows}, SW128
  CUtensorMap tm_out;  // out [M][N] bf16, box {128 / S, BT}, no swizzle
  const float* sa;
  const uint16_t* sb;
  int32_t* partials;   // optional [M][N][G] int32 dump
  uint32_t M, N, K, G;
  uint32_t ldsb;
  uint32_t S;          // CTAs per cluster along K: 1 (persistent tiles), 2 or 4
  uint32_t num_items;  // weight tiles of 128 rows
  uint32_t split;      // Wp in the pre-packed layout (a8w4::expand_piece)
  uint32_t static_weights;  // Wp and sb are not written by the preceding kernel
  uint32_t sb_vec;     // sb rows 16-byte aligned with G % 8 == 0: 8 scales per load
  // Fused all-gather (peers > 0): every output tile is stored into each rank's output
  // through tm_peer[i], the [M][N] column window of rank i's gathered [M][world*N] output
  // that this rank owns (peer memory over NVLink; TMA stores only). tm_out is then unused.
  uint32_t peers;
  CUtensorMap tm_peer[kMaxPeers];
  // Barrier of the fused all-gather folded into the kernel (bar_world > 0): bar_flags[i]
  // is rank i's flag array (the layout of peer_barrier.cuh plus word world + 1, this
  // rank's count of CTAs done). The last CTA to finish runs the barrier, so one launch
  // per step both gathers and synchronises.
  uint32_t* bar_flags[kMaxPeers];
  uint32_t bar_world, bar_rank;
  uint64_t bar_timeout_ns;
};

template <uint32_t BT>
struct Cfg {
  static_assert(BT == 16 || BT == 32, "decode token tile");
  static constexpr uint32_t kTokTile = BT * kGroupK;        // one group's token box
  static constexpr uint32_t kTokStage = kGps * kTokTile;    // 4 or 8 KiB
  static constexpr uint32_t kTStages = BT == 16 ? 4 : 3;
  // TMEM: columns [0, 128) hold the first group of each weight stage (32 columns per
  // group), then kDStages accumulator slots of one stage (2 x BT columns) each.
  static constexpr uint32_t kDBase = kWStages * 32;
  static constexpr uint32_t kDStages = BT == 16 ? 4 : 2;
  static_assert(kDBase + kDStages * 2 * BT <= kTmemCols, "TMEM budget");
  // Stream mode: kStreamA weight slots of one stage (both groups, 64 columns) first, then
  // kStreamD accumulator slots. Three weight slots let a stage's unpack wait for the
  // UMMAs of the stage three back rather than two (BT=16; BT=32 has room for two).
  static constexpr uint32_t kStreamA = BT == 16 ? 3 : 2;
  static constexpr uint32_t kStreamDBase = kStreamA * 64;
  static constexpr uint32_t kStreamD = 2;
  static_assert(kStreamDBase + kStreamD * 2 * BT <= kTmemCols, "TMEM budget (stream mode)");
};

template <uint32_t BT>
struct alignas(1024) Smem {
  using C = Cfg<BT>;
  // Packed weights [128 rows][2 groups x 64 B], SW128; after the unpack the second
  // group's int8 codes [128 rows][128 B] in the same bytes (SW128 K-major, UMMA A).
  uint8_t wring[kWStages][kWStageBytes];
  uint8_t tring[C::kTStages][C::kTokStage];     // tokens [2 groups][BT][128 B], SW128
  float recv[kRows * BT];                       // [src][128 / S][BT] partials from the peers
  uint64_t w_full[kWStages];
  uint64_t w_empty[kWStages];                   // the stage's UMMAs retired
  uint64_t a_full[kWStages];                    // the stage is unpacked
  uint64_t a_empty[C::kStreamA];                // stream mode: a TMEM stage slot's UMMAs retired
  uint64_t t_full[C::kTStages];
  uint64_t t_empty[C::kTStages];
  uint64_t mma_done[C::kDStages];               // a stage's UMMAs retired
  uint64_t tmem_empty[C::kDStages];             // its accumulators were read
  uint64_t drain;
  uint64_t recv_full;                           // peers' partials landed (S > 1)
  uint32_t tmem_base;
  uint32_t abort;
#if defined(ARC_PROBE)
  unsigned long long stamps[kProbeSlots];  // probe build: this CTA's stamps, copied out at teardown
#endif
};

// Probe stamp (probe build only): %clock64 into shared memory, a few cycles, so that the
// stamps barely move the pipeline they time. The CTA copies them to the attached probe
// buffer when it ends (sm100.cuh: g_arc_probe, one row of kProbeSlots per CTA). Stamps
// of different warps may come from different SM sub-partitions' counters: compare a
// warp's stamps with its own.
template <uint32_t BT>
__device__ __forceinline__ void stamp(Smem<BT>& s, uint32_t slot) {
#if defined(ARC_PROBE)
  unsigned long long t;
  asm volatile("mov.u64 %0, %%clock64;" : "=l"(t));
  if (slot < kProbeSlots) s.stamps[slot] = t;
#else
  (void)s;
  (void)slot;
#endif
}

// The sequence of load stages one CTA works through: `items` weight tiles of `ng`
// K-groups each (one tile for S > 1), in stages of two consecutive groups of one tile
// (a tile with an odd group count ends with a one-group stage), flattened.
struct Walk {
  uint32_t g0, ng, spi, items;
  uint32_t S;  // CTAs of the cluster along K (1: persistent tiles, no split)
  __device__ __forceinline__ Walk(const Params& p, uint32_t cluster) : S(cluster) {
    if (S > 1) {
      const uint32_t r = blockIdx.x % S;
      g0 = r * p.G / S;
      ng = (r + 1) * p.G / S - g0;
      items = 1;
    } else {
      g0 = 0;
      ng = p.G;
      items = blockIdx.x < p.num_items ? (p.num_items - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    }
    spi = (ng + 1) / 2;
  }
  __device__ __forceinline__ uint32_t stages() const { return items * spi; }
  __device__ __forceinline__ uint32_t n0(const Params& p, uint32_t k) const {
    return (S > 1 ? blockIdx.x / S : blockIdx.x + k * gridDim.x) * kRows;
  }
  // Stage t covers groups 2j and 2j + 1 (if 2j + 1 < ng) of tile k, with k = t / spi and
  // j = t % spi. Loops keep (k, j) as a cursor and step it, instead of dividing.
  __device__ __forceinline__ void advance(uint32_t& k, uint32_t& j, uint32_t step) const {
    j += step;
    while (j >= spi) {
      j -= spi;
      ++k;
    }
  }
  __device__ __forceinline__ bool has_second(uint32_t j) const { return 2u * j + 1u < ng; }
};

// Every lane of the warp waits; the warp proceeds only if all of them succeeded,
// so a timeout can never split a warp in front of a .sync.aligned instruction.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile uint32_t* abort,
                                          uint32_t err) {
  const bool ok = mbar_wait(bar, parity, abort, err);
  return __all_sync(0xffffffffu, ok);
}
// The same, polling (mbar_wait_poll): for the waits on the critical path after the tokens.
__device__ __forceinline__ bool warp_wait_poll(uint64_t* bar, uint32_t parity, volatile uint32_t* abort,
                                               uint32_t err) {
  const bool ok = mbar_wait_poll(bar, parity, abort, err);
  return __all_sync(0xffffffffu, ok);
}

// acc[c] = fma(16P[c], s, acc[c]) for the BT int32 partials r[off .. off+BT). An int32 16P
// (|16P| < 2^22) becomes a float with two full-rate operations instead of a conversion:
// bits(16P) + bits(1.5 * 2^23) is the float 1.5 * 2^23 + 16P exactly, and subtracting
// 1.5 * 2^23 leaves 16P exactly (the same value a conversion gives).
template <uint32_t BT>
__device__ __forceinline__ void accumulate(float (&acc)[BT], const uint32_t (&r)[32], uint32_t off, float s) {
#pragma unroll
  for (uint32_t c = 0; c < BT; ++c) {
    acc[c] = fmaf(__uint_as_float(r[off + c] + 0x4B400000u) - 12582912.0f, s, acc[c]);
  }
}

// bf16 scale j (0..7) of an 8-scale window, as fp32.
__device__ __forceinline__ float window_scale(const uint4& w, uint32_t j) {
  const uint32_t word = (j & 4u) ? ((j & 2u) ? w.w : w.z) : ((j & 2u) ? w.y : w.x);
  return __uint_as_float((j & 1u) ? (word & 0xFFFF0000u) : (word << 16));
}

// STREAM: stream mode, for CTAs with more load stages than the ring holds: both groups
// of a stage are unpacked into TMEM (Cfg::kStreamA stage slots of 64 columns), so a ring
// stage is free as soon as it has been read and the loads run ahead of the UMMAs.
// Otherwise (chunk mode) the second group stays in the ring stage, unpacked in place,
// until its UMMAs. DUMP: write the exact int32 group partials (a debugging aid) to
// p.partials. SK: CTAs of the cluster along K (p.S: 1, 2 or 4). GATHER: fused
// all-gather (p.peers > 0). The host picks the instantiation; each compiles only its own
// code.
template <uint32_t BT, bool STREAM, bool DUMP, uint32_t SK, bool GATHER>
__global__ void __launch_bounds__(kThreads, 2)
    gemm_a8w4_decode_kernel(const __grid_constant__ Params p) {
  using C = Cfg<BT>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem<BT>& s = *reinterpret_cast<Smem<BT>*>(smem_raw + smem_align_pad(smem_raw));
  const uint32_t warp = warp_idx_sync();
  const uint32_t lane = threadIdx.x & 31u;
  volatile uint32_t* abort = &s.abort;

#if defined(ARC_PROBE)
  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < kProbeSlots; ++i) s.stamps[i] = 0ull;
  }
#endif
  if (threadIdx.x == 0) stamp(s, 0);  // kernel entry
  pdl_launch_dependents();
  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_tok);
      tma_prefetch_desc(&p.tm_wp);
      tma_prefetch_desc(&p.tm_out);
    }
    // The barrier inits are spread over the warp's lanes (each is a shared-memory
    // operation with a long latency).
    for (uint32_t i = lane; i < kWStages; i += 32) {
      mbar_init(&s.w_full[i], 1);
      // Freed by the stage's issuer (chunk mode) or by the four unpack warps (stream mode).
      mbar_init(&s.w_empty[i], STREAM ? 4 : 1);
      mbar_init(&s.a_full[i], 4);   // the four warps of the stage's unpack warpgroup
    }
    for (uint32_t i = lane; i < C::kStreamA; i += 32) mbar_init(&s.a_empty[i], 1);
    for (uint32_t i = lane; i < C::kTStages; i += 32) {
      mbar_init(&s.t_full[i], 1);
      mbar_init(&s.t_empty[i], 1);
    }
    for (uint32_t i = lane; i < C::kDStages; i += 32) {
      mbar_init(&s.mma_done[i], 1);
      mbar_init(&s.tmem_empty[i], 4);  // the four epilogue warps
    }
    if (lane == 0) {
      mbar_init(&s.drain, 2);
      mbar_init(&s.recv_full, 1);
      s.abort = 0;
    }
    fence_barrier_init();
    __syncwarp();
    if (lane == 0 && SK > 1) {
      // Armed before the cluster barrier below, so every peer's bulk copy lands on a
      // barrier that already expects it.
      mbar_arrive_expect_tx(&s.recv_full, (SK - 1) * (kRows / SK) * BT * 4u);
    }
  }
  if (warp == 2) {
    tmem_alloc(&s.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  if (SK > 1) cluster_sync_all();  // every CTA's barriers exist before any exchange
  if (threadIdx.x == 0) stamp(s, 1);  // prologue done
  const uint32_t tmem_base = s.tmem_base;
  const Walk wk(p, SK);
  const uint32_t ns = wk.stages();
  // Accumulator slots of the mode: a power of two, stage t uses slot t & dmask.
  const uint32_t dsh = STREAM ? 1u : (C::kDStages == 4 ? 2u : 1u);
  const uint32_t dmask = (1u << dsh) - 1u;
  const uint32_t dbase = STREAM ? C::kStreamDBase : C::kDBase;

  // Register moves sit inside each role's branch, so that the compiler gives every
  // role's code the budget of that role.
  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    regs_release<regs_ctl<BT>()>();
    // Weight stages run up to kWStages ahead of token stages; with static weights the
    // first kWStages are issued before the wait for the preceding grid.
    if (lane == 0) {
      uint32_t wi = 0, ti = 0;  // weight / token stages issued
      uint32_t wk_k = 0, wk_j = 0, tk_j = 0;  // (tile, stage) of the next weight / token stage
      bool ok = true;
      auto issue_w = [&](uint32_t t) -> bool {
        const uint32_t slot = t % kWStages;
        if (t >= kWStages &&
            !mbar_wait(&s.w_empty[slot], ((t / kWStages) & 1u) ^ 1u, abort, kStatusTimeoutProducer)) {
          return false;
        }
        mbar_arrive_expect_tx(&s.w_full[slot], kWStageBytes);
        tma_load_2d(&p.tm_wp, &s.w_full[slot], s.wring[slot], int32_t((wk.g0 + 2u * wk_j) * kPackedRow),
                    int32_t(wk.n0(p, wk_k)), kCacheEvictFirst);
        wk.advance(wk_k, wk_j, 1);
        return true;
      };
      if (p.static_weights) {
        while (ok && wi < ns && wi < kWStages) ok = issue_w(wi++);
        stamp(s, 2);  // weights issued ahead of the wait
      }
      // Tokens (and, without static_weights, everything) only after the preceding grid.
      pdl_wait();
      stamp(s, 3);  // preceding grid complete
      for (uint32_t t = 0; ok && t < ns; ++t) {
        while (ok && wi < ns && wi < t + kWStages) ok = issue_w(wi++);
        if (!ok) break;
        const uint32_t slot = t % C::kTStages;
        if (t >= C::kTStages && !mbar_wait(&s.t_empty[slot], ((t / C::kTStages) & 1u) ^ 1u, abort,
                                           kStatusTimeoutProducer)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&s.t_full[slot], C::kTokStage);
        tma_load_3d(&p.tm_tok, &s.t_full[slot], s.tring[slot], 0, 0, int32_t(wk.g0 + 2u * tk_j), kCacheEvictLast);
        if (++tk_j == wk.spi) tk_j = 0;
        ++ti;
      }
      // Every load issued lands before the CTA may exit.
      for (uint32_t t = wi - (wi < kWStages ? wi : kWStages); t < wi; ++t) {
        mbar_drain(&s.w_full[t % kWStages], (t / kWStages) & 1u);
      }
      for (uint32_t t = ti - (ti < C::kTStages ? ti : C::kTStages); t < ti; ++t) {
        mbar_drain(&s.t_full[t % C::kTStages], (t / C::kTStages) & 1u);
      }
      stamp(s, 10);  // producer drained
    }
  } else if (warp == 1 || warp == 3) {
    // ------------------------------------------------------------ UMMA issuers
    regs_release<regs_ctl<BT>()>();
    // Issuer q takes the stages t with t % 2 == q. A stage: four K=32 UMMAs of its first
    // group (A from TMEM) and four of its second (A from the unpacked shared-memory
    // stage), B from the stage's token tiles, into the accumulator pair of slot
    // t % kDStages; then one commit each for the epilogue, the weight stage (ring slot
    // and TMEM A slot free again) and the token stage.
    if (lane == 0) {
      // Every wait below depends on the tokens, so it starts after the preceding grid:
      // a long predecessor can then never run a bounded wait out.
      pdl_wait();
      const uint32_t q = warp == 1 ? 0u : 1u;
      constexpr uint32_t idesc = idesc_s8_s32(kRows, BT);
      const uint64_t tdesc0 = make_sw128_kmajor_desc(s.tring);
      const uint64_t wdesc0 = make_sw128_kmajor_desc(s.wring);
      bool ok = true;
      uint32_t ck = 0, cj = 0;  // (tile, stage) of stage t
      wk.advance(ck, cj, q);
      for (uint32_t t = q; ok && t < ns; t += 2, wk.advance(ck, cj, 2)) {
        const uint32_t ts = t % C::kTStages, ws = t % kWStages, ds = t & dmask;
        // A slot of the stage: the ring slot (chunk mode) or one of two TMEM stage slots.
        const uint32_t as = STREAM ? (t % C::kStreamA) : ws;
        const uint32_t a_par = STREAM ? ((t / C::kStreamA) & 1u) : ((t / kWStages) & 1u);
        // The three tests are issued together (each costs ~200 cycles even when complete).
        const uint32_t t_t = mbar_test(&s.t_full[ts], (t / C::kTStages) & 1u);
        const uint32_t t_a = mbar_test(&s.a_full[as], a_par);
        const uint32_t t_d = t <= dmask ? 1u : mbar_test(&s.tmem_empty[ds], ((t >> dsh) & 1u) ^ 1u);
        if ((t_t == 0u && !mbar_wait_poll(&s.t_full[ts], (t / C::kTStages) & 1u, abort, kStatusTimeoutMma)) ||
            (t_a == 0u && !mbar_wait_poll(&s.a_full[as], a_par, abort, kStatusTimeoutMma)) ||
            (t_d == 0u &&
             !mbar_wait_poll(&s.tmem_empty[ds], ((t >> dsh) & 1u) ^ 1u, abort, kStatusTimeoutMma))) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        stamp(s, 24 + (t & 7u));  // stage's waits passed
        const uint32_t d = tmem_base + dbase + ds * 2u * BT;
        const uint32_t a = tmem_base + as * (STREAM ? 64u : 32u);
        const uint64_t b = desc_advance(tdesc0, ts * C::kTokStage);
        // The two groups' K steps alternate, so consecutive UMMAs accumulate into
        // different TMEM columns and the tensor pipe never waits on the previous one.
        const bool two = wk.has_second(cj);
        const uint64_t w = desc_advance(wdesc0, ws * kWStageBytes);
        const uint64_t b2 = desc_advance(b, C::kTokTile);
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
          umma_s8_tmem_a(d, a + 8u * j, desc_advance(b, 32 * j), idesc, j > 0 ? 1u : 0u);
          if (two) {
            if (STREAM) {
              umma_s8_tmem_a(d + BT, a + 32u + 8u * j, desc_advance(b2, 32 * j), idesc, j > 0 ? 1u : 0u);
            } else {
              umma_s8(d + BT, desc_advance(w, 32 * j), desc_advance(b2, 32 * j), idesc, j > 0 ? 1u : 0u);
            }
          }
        }
        umma_commit(&s.mma_done[ds]);
        // The slot-release commits only where a later stage reloads the slot (each
        // tcgen05 instruction costs the issuer tens of cycles).
        if (t + (STREAM ? C::kStreamA : kWStages) < ns) umma_commit(STREAM ? &s.a_empty[as] : &s.w_empty[ws]);
        if (t + C::kTStages < ns) umma_commit(&s.t_empty[ts]);
        stamp(s, 16 + (t & 15u));  // stage issued
      }
      umma_commit(&s.drain);
      mbar_drain(&s.drain, 0);
      stamp(s, 11 + q);  // every UMMA of this issuer retired
    }
  } else if ((warp >= 4 && warp < 8) || warp >= 12) {
    // ------------------------------------------------------------ unpack warps
    // Thread = row nl of the stage (TMEM lane nl). The row's 128 packed bytes (two
    // groups, 16-byte chunks placed by the 128-byte swizzle) go to registers; the first
    // group's 128 int8 codes to TMEM columns [32 * slot, +32), the second's back into the
    // row's 128 bytes in the K-major SW128 layout.
    const uint32_t nl = (warp & 3u) * 32 + lane;
    const uint32_t lane_addr = ((warp & 3u) * 32u) << 16;
    const uint32_t sw = nl & 7u;
    const uint32_t ug = warp >= 12 ? 1u : 0u;  // unpack warpgroup: stages t with t % 2 == ug
    bool ok = true;
    // With static weights the stages that fit the A slots are unpacked before the
    // preceding grid is waited for; every later wait depends on the UMMAs, hence on the
    // tokens.
    const uint32_t pre = STREAM ? C::kStreamA : kWStages;
    bool waited = !p.static_weights;
    if (waited) pdl_wait();
    uint32_t uk = 0, uj = 0;  // (tile, stage) of stage t
    wk.advance(uk, uj, ug);
    for (uint32_t t = ug; ok && t < ns; t += 2, wk.advance(uk, uj, 2)) {
      if (!waited && t >= pre) {
        pdl_wait();
        waited = true;
      }
      const uint32_t ws = t % kWStages;
      const uint32_t as = STREAM ? (t % C::kStreamA) : ws;
      if (!warp_wait(&s.w_full[ws], (t / kWStages) & 1u, abort, kStatusTimeoutUnpack) ||
          (STREAM && t >= C::kStreamA &&
           !warp_wait(&s.a_empty[as], ((t / C::kStreamA) & 1u) ^ 1u, abort, kStatusTimeoutUnpack))) {
        ok = false;
        break;
      }
      if (STREAM) tc_fence_after_sync();  // the TMEM slot's previous UMMAs have retired
      uint8_t* row = s.wring[ws] + nl * (kGps * kPackedRow);
      uint4 x[8];
#pragma unroll
      for (uint32_t c = 0; c < 8; ++c) x[c] = *reinterpret_cast<const uint4*>(row + ((c ^ sw) << 4));
#pragma unroll
      for (uint32_t h = 0; h < 2; ++h) {  // two 16-column halves of the group (fewer live registers)
        uint32_t v[16];
#pragma unroll
        for (uint32_t c = 0; c < 2; ++c) {
          uint4 lo, hi;
          expand_piece(x[2 * h + c], p.split, lo, hi);
          v[8 * c + 0] = lo.x;
          v[8 * c + 1] = lo.y;
          v[8 * c + 2] = lo.z;
          v[8 * c + 3] = lo.w;
          v[8 * c + 4] = hi.x;
          v[8 * c + 5] = hi.y;
          v[8 * c + 6] = hi.z;
          v[8 * c + 7] = hi.w;
        }
        tmem_st_32x32b_x16(tmem_base + lane_addr + as * (STREAM ? 64u : 32u) + 16u * h, v);
      }
      if (wk.has_second(uj)) {
        if (STREAM) {
          // Second group: TMEM columns [64 * slot + 32, +32).
#pragma unroll
          for (uint32_t h = 0; h < 2; ++h) {
            uint32_t v[16];
#pragma unroll
            for (uint32_t c = 0; c < 2; ++c) {
              uint4 lo, hi;
              expand_piece(x[4 + 2 * h + c], p.split, lo, hi);
              v[8 * c + 0] = lo.x;
              v[8 * c + 1] = lo.y;
              v[8 * c + 2] = lo.z;
              v[8 * c + 3] = lo.w;
              v[8 * c + 4] = hi.x;
              v[8 * c + 5] = hi.y;
              v[8 * c + 6] = hi.z;
              v[8 * c + 7] = hi.w;
            }
            tmem_st_32x32b_x16(tmem_base + lane_addr + as * 64u + 32u + 16u * h, v);
          }
        } else {
          // K-major SW128: 16-byte chunk u (k = 16u .. 16u+15) of row nl at (u ^ (nl & 7)).
#pragma unroll
          for (uint32_t c = 0; c < 4; ++c) {
            uint4 lo, hi;
            expand_piece(x[4 + c], p.split, lo, hi);
            *reinterpret_cast<uint4*>(row + (((2u * c) ^ sw) << 4)) = lo;
            *reinterpret_cast<uint4*>(row + (((2u * c + 1u) ^ sw) << 4)) = hi;
          }
          fence_proxy_async_smem();
        }
      }
      tmem_st_wait();
      tc_fence_before_sync();
      // Stream mode frees the ring stage for a TMA reload (async proxy): order this
      // warp's generic reads of it first.
      if (STREAM) fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s.a_full[as]);
        if (STREAM) mbar_arrive(&s.w_empty[ws]);  // the stage has been read: reload it
      }
      if ((warp & 7u) == 4u && lane == 0 && t + 2 >= (ns < pre ? ns : pre) && t < pre) stamp(s, 4);  // pre-wait stages unpacked
    }
  } else if (warp >= 8 && warp < 12) {
    // ------------------------------------------------------------ epilogue warps
    regs_claim<regs_epi<BT>()>();
    const uint32_t qw = warp - 8;
    const uint32_t et = threadIdx.x - kEpiThread0;  // 0..127
    const uint32_t nl = qw * 32 + lane;             // row of the tile = TMEM lane
    const uint32_t lane_addr = (qw * 32u) << 16;
    bool ok = true;
    bool cl_arrived = false;  // arrived at the end-of-kernel cluster barrier (S > 1)

    // Weight scales of this row for the current tile, 8 K-groups per window: the
    // current window and the next one are in registers.
    uint32_t n = wk.n0(p, 0) + nl;
    bool n_valid = n < p.N;
    const uint16_t* sb_row = p.sb + size_t(n_valid ? n : 0) * p.ldsb;
    const bool vec = p.sb_vec != 0u && (wk.g0 & 7u) == 0u;
    auto load_window = [&](uint32_t w) -> uint4 {
      uint4 r = make_uint4(0u, 0u, 0u, 0u);
      if (!n_valid || 8u * w >= wk.ng) return r;
      const uint16_t* src = sb_row + wk.g0 + 8u * w;
      if (vec) return __ldg(reinterpret_cast<const uint4*>(src));
      uint32_t h[8];
#pragma unroll
      for (uint32_t j = 0; j < 8; ++j) h[j] = 8u * w + j < wk.ng ? __ldg(src + j) : 0u;
      return make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16), h[6] | (h[7] << 16));
    };
    // With static weights the scales are loaded before the wait for the preceding grid.
    if (!p.static_weights) pdl_wait();
    uint4 win_cur = ns > 0 ? load_window(0) : make_uint4(0u, 0u, 0u, 0u);
    uint4 win_nxt = ns > 0 ? load_window(1) : win_cur;
    if (p.static_weights) pdl_wait();  // token scales and outputs only after the preceding grid
    // Lane c holds token c's scale (BT <= 32). Waited for here, where the tokens are
    // still on their way, rather than at its first use at the end of the tile.
    float sa_lane = lane < p.M ? __ldg(p.sa + lane) : 0.f;
    asm volatile("" : "+f"(sa_lane));

    float acc[BT];
#pragma unroll
    for (uint32_t j = 0; j < BT; ++j) acc[j] = 0.f;
    uint32_t k = 0, ej = 0;  // (tile, stage) of stage t
    for (uint32_t t = 0; t < ns; ++t, wk.advance(k, ej, 1)) {
      const uint32_t gi = 2u * ej;
      const bool second = gi + 1u < wk.ng;
      if (gi == 0 && k > 0) {  // next tile of a persistent CTA
        n = wk.n0(p, k) + nl;
        n_valid = n < p.N;
        sb_row = p.sb + size_t(n_valid ? n : 0) * p.ldsb;
        win_cur = load_window(0);
        win_nxt = load_window(1);
#pragma unroll
        for (uint32_t j = 0; j < BT; ++j) acc[j] = 0.f;
      } else if (gi > 0 && (gi & 7u) == 0u) {
        win_cur = win_nxt;
        win_nxt = load_window(gi / 8u + 1u);
      }
      const uint32_t ds = t & dmask;
      if (ok) ok = warp_wait_poll(&s.mma_done[ds], (t >> dsh) & 1u, abort, kStatusTimeoutEpilogue);
      if (ok) {
        tc_fence_after_sync();
        const uint32_t dcol = tmem_base + lane_addr + dbase + ds * 2u * BT;
        // 1/16 undoes the high-nibble placement of the weights.
        const float s0 = window_scale(win_cur, gi & 7u) * 0.0625f;
        const float s1 = second ? window_scale(win_cur, (gi + 1u) & 7u) * 0.0625f : 0.f;
        uint32_t r[32];
        tmem_ld_32x32b_x32(dcol, r);  // BT=16: both groups; BT=32: the first
        tmem_ld_wait();
        if constexpr (BT == 16) {
          tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s.tmem_empty[ds]);
          accumulate<16>(acc, r, 0, s0);
          if (second) accumulate<16>(acc, r, 16, s1);
        } else {
          accumulate<32>(acc, r, 0, s0);
          if (DUMP && n_valid) {
            const uint32_t g = wk.g0 + gi;
#pragma unroll
            for (uint32_t c = 0; c < 32; ++c) {
              if (c < p.M) p.partials[(size_t(c) * p.N + n) * p.G + g] = static_cast<int32_t>(r[c]) >> 4;
            }
          }
          if (second) {
            tmem_ld_32x32b_x32(dcol + 32u, r);
            tmem_ld_wait();
          }
          tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s.tmem_empty[ds]);
          if (second) accumulate<32>(acc, r, 0, s1);
        }
        if (DUMP && n_valid) {
          // r holds the second group's partials (BT=32), or both groups' (BT=16).
          const uint32_t g = wk.g0 + gi;
#pragma unroll
          for (uint32_t c = 0; c < BT; ++c) {
            if (c < p.M) {
              if constexpr (BT == 16) p.partials[(size_t(c) * p.N + n) * p.G + g] = static_cast<int32_t>(r[c]) >> 4;
              if (second) {
                p.partials[(size_t(c) * p.N + n) * p.G + g + 1] =
                    static_cast<int32_t>(r[BT == 16 ? 16 + c : c]) >> 4;
              }
            }
          }
        }
        if (qw == 0 && lane == 0) stamp(s, 48 + (t & 15u));  // stage accumulated
      }
      if (gi + 2u < wk.ng) continue;

      // ---------------------------------------------------------- tile complete
      const uint32_t n0 = wk.n0(p, k);
      if constexpr (SK == 1) {
        // Whole K range here: scale by sa, stage the [BT][128] bf16 tile, one TMA store.
        uint16_t* tile = reinterpret_cast<uint16_t*>(s.recv);  // recv is unused when S == 1
        if (et == 0) tma_store_wait_read<0>();  // the previous tile's store has read it
        named_barrier_sync(1, 128);
#pragma unroll
        for (uint32_t c = 0; c < BT; ++c) {
          const float sa_c = __shfl_sync(0xffffffffu, sa_lane, c);
          tile[c * kRows + nl] = __bfloat16_as_ushort(__float2bfloat16_rn(acc[c] * sa_c));
        }
        fence_proxy_async_smem();
        named_barrier_sync(1, 128);
        if (et == 0 && *abort == 0u) {
          if (!GATHER) {
            tma_store_2d(&p.tm_out, tile, int32_t(n0), 0);
          } else {
            for (uint32_t i = 0; i < p.peers; ++i) tma_store_2d(&p.tm_peer[i], tile, int32_t(n0), 0);
          }
          tma_store_commit();
        }
      } else {
        // K split over the S-CTA cluster; rank r finishes rows [r*128/S, (r+1)*128/S).
        // Every row's partial is staged as send[row][token] in the (now idle) weight
        // ring. A warp's 32 rows lie in one rank's slice: a warp of a peer's slice ships
        // its rows with one bulk copy into recv[this rank] of that peer as soon as they
        // are staged. Then all 128 threads sum the owned slice in rank order and one TMA
        // store writes it.
        const uint32_t rank = blockIdx.x % SK;
        constexpr uint32_t rows_per = kRows / (SK > 1 ? SK : 1);
        float* send = reinterpret_cast<float*>(s.wring);
        uint16_t* tile = reinterpret_cast<uint16_t*>(&s.wring[0][0] + kRows * BT * 4u);
        float4* dst = reinterpret_cast<float4*>(send + nl * BT);
#pragma unroll
        for (uint32_t c = 0; c < BT; c += 4) dst[c / 4] = make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
        const uint32_t owner = qw * 32u / rows_per;  // rank whose slice holds this warp's rows
        if (owner != rank) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && *abort == 0u) {
            // rows qw*32.. are rows (qw*32) % rows_per.. of the owner's slice
            bulk_copy_to_peer(map_to_rank(s.recv + (rank * rows_per + (qw * 32u) % rows_per) * BT, owner),
                              reinterpret_cast<const float*>(dst) - lane * BT, 32u * BT * 4u,
                              map_to_rank(&s.recv_full, owner));
          }
        }
        if (et == 0) stamp(s, 5);  // partials staged
        const bool got = warp_wait_poll(&s.recv_full, 0, abort, kStatusTimeoutEpilogue);
        // Every copy into this CTA has landed: arriving now lets the end-of-kernel
        // cluster barrier complete while the slice is summed and stored.
        __syncwarp();
        cluster_arrive_relaxed();
        cl_arrived = true;
        named_barrier_sync(1, 128);  // the owned rows staged by other warps are visible
        if (et == 0) stamp(s, 6);  // peer partials landed
        if (got) {
          const float sa_mine = __shfl_sync(0xffffffffu, sa_lane, lane % BT);  // token et % BT
          const float* own = send + rank * rows_per * BT;
          for (uint32_t e = et; e < rows_per * BT; e += 128) {
            const uint32_t rr = e / BT, c = e % BT;  // c == et % BT: sa_mine is its scale
            float sum = 0.f;
            for (uint32_t src = 0; src < SK; ++src) {  // fixed order: deterministic
              sum += src == rank ? own[e] : s.recv[src * rows_per * BT + e];
            }
            tile[c * rows_per + rr] = __bfloat16_as_ushort(__float2bfloat16_rn(sum * sa_mine));
          }
        }
        if (et == 0) stamp(s, 8);  // owned slice summed
        fence_proxy_async_smem();
        named_barrier_sync(1, 128);
        if (et == 0) stamp(s, 9);  // tile complete
        if (et == 0 && *abort == 0u) {
          if (!GATHER) {
            tma_store_2d(&p.tm_out, tile, int32_t(n0 + rank * rows_per), 0);
          } else {
            for (uint32_t i = 0; i < p.peers; ++i) {
              tma_store_2d(&p.tm_peer[i], tile, int32_t(n0 + rank * rows_per), 0);
            }
          }
          tma_store_commit();
          stamp(s, 7);  // output store issued
        }
      }
    }
    if (SK > 1 && !cl_arrived) {  // no tile completed here (not reached with a valid plan)
      __syncwarp();
      cluster_arrive_relaxed();
    }
    // The stores must have read their shared-memory tile before the CTA exits; their
    // global writes complete with the grid.
    if (et == 0) {
      if (GATHER && p.bar_world > 0) {
        tma_store_wait_all<0>();  // every store (into every rank's output) performed
      } else {
        tma_store_wait_read<0>();
      }
    }
    if (GATHER && p.bar_world > 0 && qw == 0) {
      // Folded barrier: the CTA that completes the count announces this rank's next epoch
      // in every rank's flags and waits for every rank's (bounded), as peer_barrier.cuh
      // does in a launch of its own.
      const uint32_t world = p.bar_world;
      uint32_t* counter = p.bar_flags[p.bar_rank] + world + 1;
      uint32_t last = 0;
      if (lane == 0) {
        __threadfence_system();  // this CTA's peer stores before its count
        last = atomicAdd(counter, 1u) + 1u == gridDim.x ? 1u : 0u;
        if (last) {
          *counter = 0u;           // ready for the next launch
          __threadfence_system();  // every CTA's stores before the announcement
        }
      }
      if (__shfl_sync(0xffffffffu, last, 0)) {
        uint32_t* epochs = p.bar_flags[p.bar_rank] + world;
        const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(epochs) + 1u;
        if (lane < world) {
          asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p.bar_flags[lane] + p.bar_rank), "r"(epoch)
                       : "memory");
          const uint32_t* f = p.bar_flags[p.bar_rank] + lane;
          const uint64_t start = globaltimer_ns();
#pragma unroll 1
          for (uint32_t it = 0;; ++it) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
            if (static_cast<int32_t>(v - epoch) >= 0) break;
            if ((it & 63u) == 63u && globaltimer_ns() - start > p.bar_timeout_ns) {
              atomicOr(&g_arc_status, kStatusTimeoutPeer);
              break;
            }
            __nanosleep(64);
          }
        }
        __syncwarp();
        if (lane == 0) *epochs = epoch;
      }
    }
  } else {
    regs_release<regs_ctl<BT>()>();  // warp 2 (TMEM allocator) shares the producer's warpgroup
  }

  if (SK > 1) {
    // No CTA leaves while a peer's bulk copy may still read its shared memory (or write
    // into it): every thread arrives when its role is done, the epilogue threads after
    // their recv_full wait. The copies' data is ordered by the transaction counts, so
    // the arrival orders nothing (relaxed).
    __syncwarp();
    if (warp < 8 || warp >= 12) cluster_arrive_relaxed();  // the epilogue warps have arrived
    cluster_wait();
    if (threadIdx.x == 0) stamp(s, 14);  // end-of-kernel cluster barrier passed
  }

  tc_fence_before_sync();
  __syncthreads();
  if (threadIdx.x == 0) stamp(s, 15);  // teardown
#if defined(ARC_PROBE)
  if (warp < 2) {
    named_barrier_sync(3, 64);
    unsigned long long* buf = g_arc_probe;
    if (buf != nullptr) buf[blockIdx.x * kProbeSlots + threadIdx.x] = s.stamps[threadIdx.x];
  }
#endif
  if (warp == 2) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace a8w4dec
}  // namespace arcb
