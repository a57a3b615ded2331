// prepack.cuh — int4 weight pre-pack: the reference's packing -> the kernels' expand layout.
//
// The reference packs two int4 codes per byte along K, the even k in the low nibble
// (arc/testing/quant.py:82-83). Expanding that to int8 takes two byte permutes per 8 codes
// (a8w4::expand_int4x8). The pre-packed layout keeps every 16-byte piece of a row (32
// codes, k = 32q .. 32q+31) in place and only reorders the nibbles inside it: byte j holds
// code j in its low nibble and code j+16 in its high nibble. The unpack warps then get the
// piece's 32 int8 codes with one mask per word (high nibbles) and one shift + mask (low
// nibbles). Shapes, strides and scales are unchanged, so a pre-packed matrix is a drop-in
// replacement for Wp wherever the GEMM is told its layout.
//
// The pass reads and writes every byte once: HBM-bound, 2 * N * K/2 bytes per call.
#pragma once

#include "gemm_a8w4.cuh"

namespace arcb {
namespace prepack {

// One 16-byte piece, reference packing -> pre-packed layout.
__device__ __forceinline__ uint4 split_piece(const uint4& x) {
  const uint2 e0 = a8w4::expand_int4x8(x.x);  // codes 0..7   in the high nibbles
  const uint2 e1 = a8w4::expand_int4x8(x.y);  // codes 8..15
  const uint2 e2 = a8w4::expand_int4x8(x.z);  // codes 16..23
  const uint2 e3 = a8w4::expand_int4x8(x.w);  // codes 24..31
  return make_uint4((e0.x >> 4) | e2.x, (e0.y >> 4) | e2.y, (e1.x >> 4) | e3.x, (e1.y >> 4) | e3.y);
}

constexpr uint32_t kThreads = 256;
constexpr uint32_t kUnroll = 4;  // pieces in flight per thread

// dst may equal src (in place): every piece is read and written by the same thread.
__global__ void __launch_bounds__(kThreads) prepack_w4_kernel(const uint4* src, uint4* dst, uint64_t pieces) {
  const uint64_t span = uint64_t(kThreads) * kUnroll;
  for (uint64_t base = uint64_t(blockIdx.x) * span; base < pieces; base += uint64_t(gridDim.x) * span) {
    uint4 x[kUnroll];
#pragma unroll
    for (uint32_t u = 0; u < kUnroll; ++u) {
      const uint64_t i = base + u * kThreads + threadIdx.x;
      if (i < pieces) x[u] = src[i];
    }
#pragma unroll
    for (uint32_t u = 0; u < kUnroll; ++u) {
      const uint64_t i = base + u * kThreads + threadIdx.x;
      if (i < pieces) dst[i] = split_piece(x[u]);
    }
  }
}

}  // namespace prepack
}  // namespace arcb
