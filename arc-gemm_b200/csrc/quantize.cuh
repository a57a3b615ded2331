// quantize.cuh — per-token int8 quantisation of bf16 activations on the GPU.
//
//   amax[m] = max(max_k |x[m,k]|, 1e-4)      sa[m] = amax[m] / 127   (fp32)
//   q[m,k]  = clamp(round_half_even(x[m,k] / sa[m]), -127, 127)     (int8)
//
// This is the step in front of the A8W4 GEMM: its (q, sa) pair is the GEMM's
// activation operand. The arithmetic is the host quantizer's
// (arc/quant.py: per_token_cast_to_int8), which follows the reference's
// per-token cast (arc/testing/quant.py:30-48) with the int8 recipe: same amax clamp,
// fp32 division and round-half-even, so the two agree bit for bit.
//
// One CTA of kThreads per token row. A row of up to kThreads * 8 * kRegVecs
// elements stays in registers between the max and the quantisation pass; longer rows
// are read a second time (from L2). Loads and stores are 16 and 8 bytes wide when
// the rows allow it. The kernel is HBM-bound: 2 bytes read and 1 written per element.
#pragma once

#include "sm100.cuh"

namespace arcb {
namespace quant {

constexpr uint32_t kThreads = 256;
constexpr uint32_t kRegVecs = 8;  // 8-element vectors per thread kept in registers

struct Params {
  const uint16_t* x;  // bf16 [M][ldx]
  int8_t* q;          // [M][ldq]
  float* sa;          // [M]
  uint32_t M, K, ldx, ldq;
  uint32_t vec;       // 1: 16-byte loads / 8-byte stores are aligned for every row
};

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

__device__ __forceinline__ float absmax8(const uint4& v) {
  float m = fabsf(bf16_lo(v.x));
  m = fmaxf(m, fabsf(bf16_hi(v.x)));
  m = fmaxf(m, fabsf(bf16_lo(v.y)));
  m = fmaxf(m, fabsf(bf16_hi(v.y)));
  m = fmaxf(m, fabsf(bf16_lo(v.z)));
  m = fmaxf(m, fabsf(bf16_hi(v.z)));
  m = fmaxf(m, fabsf(bf16_lo(v.w)));
  return fmaxf(m, fabsf(bf16_hi(v.w)));
}

__device__ __forceinline__ int32_t quant1(float v, float sa) {
  const float r = rintf(v / sa);  // IEEE division, round half to even
  return static_cast<int32_t>(fminf(fmaxf(r, -127.f), 127.f));
}

__device__ __forceinline__ uint32_t pack4(int32_t a, int32_t b, int32_t c, int32_t d) {
  return (static_cast<uint32_t>(a) & 0xFFu) | ((static_cast<uint32_t>(b) & 0xFFu) << 8) |
         ((static_cast<uint32_t>(c) & 0xFFu) << 16) | ((static_cast<uint32_t>(d) & 0xFFu) << 24);
}

__device__ __forceinline__ uint2 quant8(const uint4& v, float sa) {
  return make_uint2(pack4(quant1(bf16_lo(v.x), sa), quant1(bf16_hi(v.x), sa), quant1(bf16_lo(v.y), sa),
                          quant1(bf16_hi(v.y), sa)),
                    pack4(quant1(bf16_lo(v.z), sa), quant1(bf16_hi(v.z), sa), quant1(bf16_lo(v.w), sa),
                          quant1(bf16_hi(v.w), sa)));
}

__global__ void __launch_bounds__(kThreads) quantize_int8_per_token_kernel(const __grid_constant__ Params p) {
  __shared__ float warp_max[kThreads / 32];
  // The next kernel (the GEMM) may start its prologue now; it waits for this grid's
  // completion before it reads q and sa.
  pdl_launch_dependents();
  pdl_wait();  // x may come from the previous kernel in the stream
  const uint32_t t = threadIdx.x;
  const uint16_t* xr = p.x + size_t(blockIdx.x) * p.ldx;
  int8_t* qr = p.q + size_t(blockIdx.x) * p.ldq;

  float amax = 0.f;
  uint4 regs[kRegVecs];
  const uint32_t nvec = p.vec ? p.K / 8u : 0u;
  if (p.vec) {
#pragma unroll
    for (uint32_t i = 0; i < kRegVecs; ++i) {
      const uint32_t v = t + i * kThreads;
      regs[i] = v < nvec ? __ldg(reinterpret_cast<const uint4*>(xr) + v) : make_uint4(0, 0, 0, 0);
      amax = fmaxf(amax, absmax8(regs[i]));
    }
    for (uint32_t v = t + kRegVecs * kThreads; v < nvec; v += kThreads) {
      amax = fmaxf(amax, absmax8(__ldg(reinterpret_cast<const uint4*>(xr) + v)));
    }
  } else {
    for (uint32_t k = t; k < p.K; k += kThreads) amax = fmaxf(amax, fabsf(bf16_lo(__ldg(xr + k))));
  }
#pragma unroll
  for (uint32_t off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  if ((t & 31u) == 0u) warp_max[t / 32] = amax;
  __syncthreads();
  amax = warp_max[0];
#pragma unroll
  for (uint32_t w = 1; w < kThreads / 32; ++w) amax = fmaxf(amax, warp_max[w]);
  const float sa = fmaxf(amax, 1e-4f) / 127.f;
  if (t == 0) p.sa[blockIdx.x] = sa;

  if (p.vec) {
#pragma unroll
    for (uint32_t i = 0; i < kRegVecs; ++i) {
      const uint32_t v = t + i * kThreads;
      if (v < nvec) reinterpret_cast<uint2*>(qr)[v] = quant8(regs[i], sa);
    }
    for (uint32_t v = t + kRegVecs * kThreads; v < nvec; v += kThreads) {
      reinterpret_cast<uint2*>(qr)[v] = quant8(__ldg(reinterpret_cast<const uint4*>(xr) + v), sa);
    }
  } else {
    for (uint32_t k = t; k < p.K; k += kThreads) {
      qr[k] = static_cast<int8_t>(quant1(bf16_lo(__ldg(xr + k)), sa));
    }
  }
}

}  // namespace quant
}  // namespace arcb
