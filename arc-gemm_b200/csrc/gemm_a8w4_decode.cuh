// gemm_a8w4_decode.cuh — A8W4 GEMM for decode-sized M (<= 32 tokens).
//
// Same arithmetic and operand formats as gemm_a8w4.cuh (int8 tokens x int4 weights
// placed in the high nibble, exact int32 group partials, fp32 scale epilogue), but a
// decomposition built for streaming the weight matrix once at HBM speed:
//
// * A CTA owns R weight rows (R <= 128, a multiple of 8) and a K-group range. With
//   S > 1 (2 or 4) the CTAs of a cluster split K and push fp32 partials to the CTA
//   that finishes each row through distributed shared memory (the grid is then
//   exactly one wave); with S == 1 CTAs are persistent over weight tiles. The count
//   of tcgen05.mma instructions per CTA (four per K-group, each costing tens of
//   cycles to issue whatever its N) is what the K split spreads out.
// * Loads are wide: one ring stage holds GPS (2, 4 or 8) consecutive K-groups, fetched
//   with two TMA instructions — the packed weights as one [R x GPS*64 B] box (a u32
//   view, so a box row spans GPS groups) and the token tiles as one 3-D box
//   [GPS][BT][128 B] in the 128-byte swizzle layout the UMMA B operand expects.
// * Eight unpack warps split a stage by rows (each reads whole contiguous rows) and
//   write every group into its own unpacked slot. Slots are packed R rows apart:
//   the UMMA reads 128 rows from a slot base, rows >= R fall into the next slot and
//   only feed TMEM lanes that are never read. With up to 16 slots a CTA rarely has
//   to wait for a slot to be released (the wait is on the UMMA completion of the
//   group that used the slot before).
// * Every K-group gets its own TMEM accumulator slot (512 / BT of them), so the
//   tensor core never waits for the epilogue to drain a buffer.
// * Programmatic dependent launch: the prologue (barrier init, TMEM allocation,
//   descriptor prefetch) overlaps the previous kernel in the stream;
//   griddepcontrol.wait precedes every global-memory access.
//
// Roles (512 threads): warp 0 TMA producer, warp 1 UMMA issuer, warp 2 TMEM
// allocator, warp 3 idle, warps 4-11 unpack, warps 12-15 epilogue (warp 12+q reads
// TMEM lanes 32q..32q+31, i.e. weight rows 32q..; warps whose rows are all >= R only
// take part in the barriers).
#pragma once

#include "gemm_a8w4.cuh"
#include "sm100.cuh"

namespace arcb {
namespace a8w4dec {

using a8w4::expand_piece;
using a8w4::kGroupK;
using a8w4::kPackedRow;
using a8w4::kRows;
using a8w4::kUmmaK;

constexpr uint32_t kUnpackWarps = 8;
constexpr uint32_t kEpiWarps = 4;
constexpr uint32_t kThreads = 32 * (4 + kUnpackWarps + kEpiWarps);
constexpr uint32_t kMaxStages = 8;
constexpr uint32_t kRingBytes = 88 * 1024;
constexpr uint32_t kSlotBytes = 112 * 1024;  // unpacked slots, R*128 bytes apart
constexpr uint32_t kMaxSlots = 16;
constexpr uint32_t kScaleLookahead = 8;
constexpr uint32_t kMaxPeers = 8;  // GPUs of a fused all-gather

struct Params {
  CUtensorMap tm_tok;  // A as [G][M][128] u8 (3-D), box {128, BT, GPS}, SW128
  CUtensorMap tm_wp;   // Wp as [N][K/8] u32, box {16*GPS, R}, no swizzle
  CUtensorMap tm_out;  // out [M][N] bf16, box {R / S, BT}, no swizzle
  const float* sa;
  const uint16_t* sb;
  uint16_t* out;
  int32_t* partials;   // optional [M][N][G] int32 dump
  uint32_t M, N, K, G;
  uint32_t ldsb, ldc;
  uint32_t R;          // weight rows per tile
  uint32_t S;          // CTAs per cluster along K: 1 (persistent tiles), 2 or 4
  uint32_t num_items;  // weight tiles
  uint32_t gps;        // K-groups per ring stage (2, 4 or 8)
  uint32_t stages;     // ring depth (<= kMaxStages)
  uint32_t stage_bytes;
  uint32_t tok_bytes;  // token part of a stage: gps * BT * 128
  uint32_t slots;      // unpacked slots (<= kMaxSlots)
  uint32_t slot_stride;  // R * 128 (a multiple of 1024)
  // Fused all-gather (peers > 0): every output tile is stored into each rank's output
  // through tm_peer[i], the [M][N] column window of rank i's gathered [M][world*N] output
  // that this rank owns (peer memory over NVLink; TMA stores only). tm_out is then unused.
  uint32_t peers;
  uint32_t split;  // Wp in the pre-packed layout (a8w4::expand_piece)
  CUtensorMap tm_peer[kMaxPeers];
};

template <uint32_t BT>
struct Cfg {
  static_assert(BT == 16 || BT == 32, "decode token tile");
  static constexpr uint32_t kTokTile = BT * kGroupK;
  static constexpr uint32_t kTmemSlots = 512 / BT;
};

template <uint32_t BT>
struct alignas(1024) Smem {
  using C = Cfg<BT>;
  // Unpacked slots first: a UMMA on the last slot reads up to 16 KB past its base,
  // which stays inside this CTA's shared memory (the ring that follows).
  uint8_t slots[kSlotBytes];
  uint8_t ring[kRingBytes];                  // stages: [GPS token tiles | R x GPS*64 B]
  float recv[kRows * BT];                    // [src][R/S][BT] partials from the peers
  uint64_t load_full[kMaxStages];
  uint64_t load_empty[kMaxStages];
  uint64_t unpacked[kMaxStages];             // stage fully unpacked (one arrive per warp)
  uint64_t mma_done[C::kTmemSlots];
  uint64_t tmem_empty[C::kTmemSlots];
  uint64_t drain;
  uint64_t recv_full;                        // peers' partials landed (S > 1)
  uint32_t tmem_base;
  uint32_t abort;
};

struct Item {
  uint32_t n0, g0, g1;
};

__device__ __forceinline__ bool get_item(const Params& p, uint32_t idx, Item& it) {
  if (p.S > 1) {
    if (idx != 0) return false;
    const uint32_t rank = blockIdx.x % p.S;
    it.n0 = (blockIdx.x / p.S) * p.R;
    it.g0 = rank * p.G / p.S;
    it.g1 = (rank + 1) * p.G / p.S;
    return true;
  }
  const uint32_t t = blockIdx.x + idx * gridDim.x;
  if (t >= p.num_items) return false;
  it.n0 = t * p.R;
  it.g0 = 0;
  it.g1 = p.G;
  return true;
}

// Every lane of the warp waits; the warp proceeds only if all of them succeeded,
// so a timeout can never split a warp in front of a .sync.aligned instruction.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile uint32_t* abort,
                                          uint32_t err) {
  const bool ok = mbar_wait(bar, parity, abort, err);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void st_dsmem_f32x4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}

template <uint32_t BT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_a8w4_decode_kernel(const __grid_constant__ Params p) {
  using C = Cfg<BT>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem<BT>& s = *reinterpret_cast<Smem<BT>*>(smem_raw + smem_align_pad(smem_raw));
  const uint32_t warp = warp_idx_sync();
  const uint32_t lane = threadIdx.x & 31u;
  volatile uint32_t* abort = &s.abort;
  const uint32_t epi_warps = (p.R + 31) / 32;

  if (threadIdx.x == 0) probe_mark(0);  // kernel entry
  pdl_launch_dependents();
  if (warp == 0) {
    // The ~90 barrier inits are spread over the warp's lanes (each is a shared-memory
    // operation with a long latency).
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_tok);
      tma_prefetch_desc(&p.tm_wp);
      tma_prefetch_desc(&p.tm_out);
    }
    for (uint32_t i = lane; i < p.stages; i += 32) {
      mbar_init(&s.load_full[i], 1);
      mbar_init(&s.load_empty[i], kUnpackWarps + 1);  // each unpack warp + the UMMA commit
      mbar_init(&s.unpacked[i], kUnpackWarps);
    }
    for (uint32_t i = lane; i < C::kTmemSlots; i += 32) {
      mbar_init(&s.mma_done[i], 1);
      mbar_init(&s.tmem_empty[i], epi_warps);
    }
    if (lane == 0) {
      mbar_init(&s.drain, 1);
      mbar_init(&s.recv_full, 1);
      s.abort = 0;
    }
    fence_barrier_init();
    __syncwarp();
    if (lane == 0 && p.S > 1) {
      // Armed before the cluster barrier below, so every peer's bulk copy lands on a
      // barrier that already expects it.
      mbar_arrive_expect_tx(&s.recv_full, (p.S - 1) * (p.R / p.S) * BT * 4u);
    }
  }
  if (warp == 2) {
    tmem_alloc(&s.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  if (p.S > 1) cluster_sync_all();  // every CTA's barriers exist before any exchange
  if (threadIdx.x == 0) probe_mark(1);  // prologue done
  // Everything above overlaps the previous grid; nothing below may run before it
  // has completed and its writes are visible.
  pdl_wait();
  if (threadIdx.x == 0) probe_mark(2);  // previous grid complete
  bool cl_arrived = false;  // this thread's arrival on the end-of-kernel cluster barrier
  const uint32_t tmem_base = s.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint32_t tx = p.tok_bytes + p.R * p.gps * kPackedRow;
      uint32_t q = 0;  // stages issued
      Item it;
      bool ok = true;
      for (uint32_t idx = 0; ok && get_item(p, idx, it); ++idx) {
        for (uint32_t g = it.g0; g < it.g1; g += p.gps, ++q) {
          const uint32_t st = q % p.stages;
          // The first fill of each stage needs no wait (a wait on a fresh barrier still
          // costs ~240 cycles of this thread's time before the first load goes out).
          if (q >= p.stages && !mbar_wait(&s.load_empty[st], ((q / p.stages) & 1u) ^ 1u, abort,
                                          kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* base = s.ring + st * p.stage_bytes;
          mbar_arrive_expect_tx(&s.load_full[st], tx);
          tma_load_3d(&p.tm_tok, &s.load_full[st], base, 0, 0, int32_t(g), kCacheEvictLast);
          tma_load_2d(&p.tm_wp, &s.load_full[st], base + p.tok_bytes,
                      int32_t(g * (kPackedRow / 4)), int32_t(it.n0), kCacheEvictFirst);
        }
      }
      probe_mark(3);  // every load issued
      const uint32_t n_drain = q < p.stages ? q : p.stages;
      for (uint32_t j = q - n_drain; j < q; ++j) {
        mbar_drain(&s.load_full[j % p.stages], (j / p.stages) & 1u);
      }
      probe_mark(10);  // producer drained
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    // One thread issues everything. tcgen05.mma issue costs tens of cycles of this
    // thread's own instruction latency, so the loop keeps ring/slot positions as
    // wrapping counters (no division) and derives descriptors by adding offsets.
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_s8_s32(kRows, BT);
      const uint64_t slot_desc0 = make_sw128_kmajor_desc(s.slots);
      const uint64_t ring_desc0 = make_sw128_kmajor_desc(s.ring);
      uint32_t st = 0, st_ph = 0;   // ring stage and its phase parity
      uint32_t ts = 0, ts_ph = 0;   // TMEM accumulator slot and its phase parity
      uint32_t sl = 0;              // unpacked slot
      uint32_t q = 0, i = 0;        // stages / groups consumed (probe only)
      Item it;
      bool ok = true;
      for (uint32_t idx = 0; ok && get_item(p, idx, it); ++idx) {
        for (uint32_t g0 = it.g0; ok && g0 < it.g1; g0 += p.gps, ++q) {
          // Both tested at once (a test costs ~180 cycles even when complete).
          const uint32_t t_ld = mbar_test(&s.load_full[st], st_ph);
          const uint32_t t_up = mbar_test(&s.unpacked[st], st_ph);
          if ((t_ld == 0u && !mbar_wait(&s.load_full[st], st_ph, abort, kStatusTimeoutMma)) ||
              (t_up == 0u && !mbar_wait(&s.unpacked[st], st_ph, abort, kStatusTimeoutMma))) {
            ok = false;
            break;
          }
          probe_mark(8 + (q & 7u));  // stage landed and unpacked
          tc_fence_after_sync();
          const uint64_t tok_desc = desc_advance(ring_desc0, st * p.stage_bytes);
          const uint32_t n_in = min(p.gps, it.g1 - g0);
#pragma unroll 1
          for (uint32_t j = 0; j < n_in; ++j, ++i) {
            // A TMEM slot is waited for only when it has been used before.
            if (i >= C::kTmemSlots &&
                !mbar_wait(&s.tmem_empty[ts], ts_ph ^ 1u, abort, kStatusTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after_sync();
            const uint64_t adesc = desc_advance(slot_desc0, sl * p.slot_stride);
            const uint64_t bdesc = desc_advance(tok_desc, j * C::kTokTile);
            const uint32_t d = tmem_base + ts * BT;
            umma_s8(d, adesc, bdesc, idesc, 0u);
            umma_s8(d, desc_advance(adesc, 32), desc_advance(bdesc, 32), idesc, 1u);
            umma_s8(d, desc_advance(adesc, 64), desc_advance(bdesc, 64), idesc, 1u);
            umma_s8(d, desc_advance(adesc, 96), desc_advance(bdesc, 96), idesc, 1u);
            // One commit per group: the epilogue waits on it, and so does the unpack
            // warp that next writes this group's unpacked slot.
            umma_commit(&s.mma_done[ts]);
            probe_mark(32 + (i & 15u));  // group issued to the tensor core
            if (++ts == C::kTmemSlots) {
              ts = 0;
              ts_ph ^= 1u;
            }
            if (++sl == p.slots) sl = 0;
          }
          if (ok) umma_commit(&s.load_empty[st]);  // token tiles of the stage consumed
          if (++st == p.stages) {
            st = 0;
            st_ph ^= 1u;
          }
        }
      }
      umma_commit(&s.drain);
      mbar_drain(&s.drain, 0);
      probe_mark(11);  // every UMMA retired
    }
  } else if (warp >= 4 && warp < 4 + kUnpackWarps) {
    // ------------------------------------------------------------ unpack warps
    // A stage row is gps*64 bytes; a lane converts one 16-byte piece (32 codes of
    // one group) into two 16-byte int8 chunks of that group's slot row.
    const uint32_t u = warp - 4;
    const uint32_t row_bytes = p.gps * kPackedRow;
    const uint32_t lanes_per_row = row_bytes / 16u;     // 16 or 32
    const uint32_t rows_per_pass = 32u / lanes_per_row; // 2 or 1
    const uint32_t piece = lane % lanes_per_row;
    const uint32_t jl = piece >> 2;                     // group within the stage
    const uint32_t quarter = piece & 3u;                // 32-wide K quarter of the group
    const uint32_t row0 = u * rows_per_pass + lane / lanes_per_row;
    const uint32_t row_step = kUnpackWarps * rows_per_pass;
    uint32_t q = 0, i = 0;
    Item it;
    bool ok = true;
    for (uint32_t idx = 0; ok && get_item(p, idx, it); ++idx) {
      for (uint32_t g0 = it.g0; ok && g0 < it.g1; g0 += p.gps, ++q) {
        const uint32_t st = q % p.stages;
        const uint32_t n_in = min(p.gps, it.g1 - g0);
        if (!warp_wait(&s.load_full[st], (q / p.stages) & 1u, abort, kStatusTimeoutUnpack)) {
          ok = false;
          break;
        }
        // The slots this stage fills are free once the UMMAs of the groups that used
        // them last (p.slots groups earlier) have completed. Those groups' TMEM slots
        // cannot have been reused since: their successors come after this unpack.
        for (uint32_t j = 0; ok && j < n_in; ++j) {
          const uint32_t gi = i + j;
          if (gi >= p.slots) {
            const uint32_t prev = gi - p.slots;
            ok = warp_wait(&s.mma_done[prev % C::kTmemSlots], (prev / C::kTmemSlots) & 1u, abort,
                           kStatusTimeoutUnpack);
          }
        }
        if (!ok) break;
        const uint8_t* packed = s.ring + st * p.stage_bytes + p.tok_bytes;
        if (jl < n_in) {
          uint8_t* slot = s.slots + ((i + jl) % p.slots) * p.slot_stride;
#pragma unroll 2
          for (uint32_t r = row0; r < p.R; r += row_step) {
            const uint4 x = *reinterpret_cast<const uint4*>(packed + r * row_bytes + piece * 16u);
            uint4 lo, hi;
            expand_piece(x, p.split, lo, hi);
            uint8_t* dst = slot + r * kGroupK;
            const uint32_t sw = r & 7u;
            *reinterpret_cast<uint4*>(dst + (((2u * quarter) ^ sw) << 4)) = lo;
            *reinterpret_cast<uint4*>(dst + (((2u * quarter + 1u) ^ sw) << 4)) = hi;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&s.unpacked[st]);
          mbar_arrive(&s.load_empty[st]);
          if (u == 0) probe_mark(16 + (q & 15u));  // stage unpacked by warp 0
        }
        i += n_in;
      }
    }
  } else if (warp >= 4 + kUnpackWarps) {
    // ------------------------------------------------------------ epilogue warps
    // All four warps walk the same items and meet at the same named barriers; warps
    // whose TMEM lanes hold no valid row (and any warp after a failed wait) skip the
    // arithmetic but not the barriers.
    const uint32_t qw = warp - (4 + kUnpackWarps);
    const uint32_t et = threadIdx.x - 32 * (4 + kUnpackWarps);  // 0..127
    const bool active = qw < epi_warps;
    const uint32_t nl = qw * 32 + lane;
    // Lane c holds token c's scale (BT <= 32); loaded now, far from its use.
    float sa_lane = lane < p.M ? __ldg(p.sa + lane) : 0.f;
    asm volatile("" : "+f"(sa_lane));
    const float sa_mine = __shfl_sync(0xffffffffu, sa_lane, lane % BT);  // token et % BT
    uint32_t i = 0;
    Item it;
    bool ok = true;
    for (uint32_t idx = 0; get_item(p, idx, it); ++idx) {
      const uint32_t n = it.n0 + nl;
      const bool n_valid = nl < p.R && n < p.N;
      const uint16_t* sb_row = p.sb + size_t(n_valid ? n : 0) * p.ldsb;
      float acc[BT];
#pragma unroll
      for (uint32_t j = 0; j < BT; ++j) acc[j] = 0.f;
      const uint32_t ng = it.g1 - it.g0;
      if (active && ok) {
        float sreg[kScaleLookahead];
#pragma unroll
        for (uint32_t v = 0; v < kScaleLookahead; ++v) {
          sreg[v] = (n_valid && it.g0 + v < it.g1) ? bf16_bits_to_float(__ldg(sb_row + it.g0 + v))
                                                   : 0.f;
        }
        for (uint32_t jb = 0; ok && jb < ng; jb += kScaleLookahead) {
#pragma unroll
          for (uint32_t v = 0; v < kScaleLookahead; ++v) {
            const uint32_t j = jb + v;
            if (j >= ng) break;
            const uint32_t ts = i % C::kTmemSlots;
            const float s_g = sreg[v] * 0.0625f;  // 1/16 undoes the high-nibble placement
            if (n_valid && j + kScaleLookahead < ng) {
              sreg[v] = bf16_bits_to_float(__ldg(sb_row + it.g0 + j + kScaleLookahead));
            }
            if (!warp_wait(&s.mma_done[ts], (i / C::kTmemSlots) & 1u, abort,
                           kStatusTimeoutEpilogue)) {
              ok = false;
              break;
            }
            tc_fence_after_sync();
            uint32_t r[BT];
            if constexpr (BT == 16) {
              tmem_ld_32x32b_x16(tmem_base + ((qw * 32u) << 16) + ts * BT, r);
            } else {
              tmem_ld_32x32b_x32(tmem_base + ((qw * 32u) << 16) + ts * BT, r);
            }
            tmem_ld_wait();
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.tmem_empty[ts]);
#pragma unroll
            for (uint32_t c = 0; c < BT; ++c) {
              acc[c] = fmaf(static_cast<float>(static_cast<int32_t>(r[c])), s_g, acc[c]);
            }
            if (qw == 0 && lane == 0) probe_mark(48 + (i & 15u));  // group accumulated
            if (p.partials != nullptr && n_valid) {
              const uint32_t g = it.g0 + j;
#pragma unroll
              for (uint32_t c = 0; c < BT; ++c) {
                if (c < p.M) {
                  p.partials[(size_t(c) * p.N + n) * p.G + g] = static_cast<int32_t>(r[c]) >> 4;
                }
              }
            }
            ++i;
          }
        }
      }

      if (p.S == 1) {
        // Whole K range here: scale by sa, stage the [BT][R] bf16 tile, one TMA store.
        uint16_t* tile = reinterpret_cast<uint16_t*>(s.recv);  // recv is unused when S == 1
        if (et == 0) tma_store_wait_read<0>();  // the previous item's store has read the tile
        named_barrier_sync(1, 128);
        // Every lane takes part in the shuffle (a warp can hold valid and invalid
        // rows when R is not a multiple of 32); only the store is predicated.
#pragma unroll
        for (uint32_t c = 0; c < BT; ++c) {
          const float sa_c = __shfl_sync(0xffffffffu, sa_lane, c);
          if (active && nl < p.R) {
            tile[c * p.R + nl] = __bfloat16_as_ushort(__float2bfloat16_rn(acc[c] * sa_c));
          }
        }
        fence_proxy_async_smem();
        named_barrier_sync(1, 128);
        if (et == 0 && *abort == 0u) {
          if (p.peers == 0) {
            tma_store_2d(&p.tm_out, tile, int32_t(it.n0), 0);
          } else {
            for (uint32_t i = 0; i < p.peers; ++i) tma_store_2d(&p.tm_peer[i], tile, int32_t(it.n0), 0);
          }
          tma_store_commit();
        }
      } else {
        // K split over the S-CTA cluster; rank r finishes rows [r*R/S, (r+1)*R/S).
        // Every row's partial is staged in send[owner][row][token] (the unpacked
        // slots are idle: every UMMA has completed), the peers' parts are shipped as
        // one bulk copy per peer into recv[this rank], then all 128 threads sum the
        // owned slice in rank order and one TMA store writes it.
        const uint32_t rank = blockIdx.x % p.S;
        const uint32_t rows_per = p.R / p.S;
        float* send = reinterpret_cast<float*>(s.slots);
        uint16_t* tile = reinterpret_cast<uint16_t*>(s.slots + p.R * BT * 4u);
        if (active && nl < p.R) {
          const uint32_t owner = nl / rows_per;
          float4* dst = reinterpret_cast<float4*>(send + (owner * rows_per + nl - owner * rows_per) * BT);
#pragma unroll
          for (uint32_t c = 0; c < BT; c += 4) {
            dst[c / 4] = make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
          }
        }
        fence_proxy_async_smem();
        named_barrier_sync(1, 128);
        if (et == 0 && *abort == 0u) {
          probe_mark(4);  // partials staged
          for (uint32_t o = 0; o < p.S; ++o) {
            if (o == rank) continue;
            bulk_copy_to_peer(map_to_rank(s.recv + rank * rows_per * BT, o),
                              send + o * rows_per * BT, rows_per * BT * 4u,
                              map_to_rank(&s.recv_full, o));
          }
        }
        const bool got = warp_wait(&s.recv_full, 0, abort, kStatusTimeoutEpilogue);
        if (et == 0) probe_mark(5);  // peer partials landed
        // Nothing targets this CTA's shared memory any more: announce it now and wait at
        // the end, so the cluster barrier overlaps the reduction and the store.
        if (!cl_arrived) {
          __syncwarp();
          cluster_arrive();
          cl_arrived = true;
        }
        if (got) {
          const float* own = send + rank * rows_per * BT;
          for (uint32_t e = et; e < rows_per * BT; e += 128) {
            const uint32_t rr = e / BT, c = e % BT;  // c == et % BT: sa_mine is its scale
            float sum = 0.f;
            for (uint32_t src = 0; src < p.S; ++src) {  // fixed order: deterministic
              sum += src == rank ? own[e] : s.recv[src * rows_per * BT + e];
            }
            tile[c * rows_per + rr] = __bfloat16_as_ushort(__float2bfloat16_rn(sum * sa_mine));
          }
        }
        fence_proxy_async_smem();
        named_barrier_sync(1, 128);
        if (et == 0 && *abort == 0u) {
          if (p.peers == 0) {
            tma_store_2d(&p.tm_out, tile, int32_t(it.n0 + rank * rows_per), 0);
          } else {
            for (uint32_t i = 0; i < p.peers; ++i) {
              tma_store_2d(&p.tm_peer[i], tile, int32_t(it.n0 + rank * rows_per), 0);
            }
          }
          tma_store_commit();
          probe_mark(6);  // output store issued
        }
      }
    }
    if (et == 0) tma_store_wait_all<0>();
  }

  if (warp == 4 && lane == 0) probe_mark(12);  // unpack warp 0 done
  if (threadIdx.x == 64) probe_mark(15);  // TMEM allocator warp reached the end
  if (p.S > 1) {
    // No CTA leaves while a bulk copy may still target its shared memory: owners
    // arrive only after their recv_full wait (or its timeout), every other thread
    // when its role is done.
    __syncwarp();
    if (!cl_arrived) cluster_arrive();
    cluster_wait();
    if (threadIdx.x == 0) probe_mark(14);  // end-of-kernel cluster barrier passed
  }

  tc_fence_before_sync();
  __syncthreads();
  if (threadIdx.x == 0) probe_mark(7);  // teardown
  if (warp == 2) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace a8w4dec
}  // namespace arcb
