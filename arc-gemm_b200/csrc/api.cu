// api.cu — host side of libarcb200.so: argument checks, TMA descriptor encoding,
// work decomposition and kernel launches behind the C ABI of include/arc_b200.h.
//
// The reference's equivalent is the generated TVM-FFI shim in arc/mm.py:17-49 plus
// the descriptor helper arc/include/ptx/tma.cuh:19-74. Differences by design:
// errors are returned (never exit()), tensor maps take explicit leading dimensions,
// and the tile/stage configuration is chosen per shape instead of being fixed at
// (128,128,128)x3 (arc/mm.py:64).
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "arc_b200.h"
#include "gemm_a8w4.cuh"
#include "gemm_bf16.cuh"
#include "sm100.cuh"

namespace {

constexpr int kVersion = 100;  // 0.1.0

thread_local char g_last_error[512] = "";

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_fail(cudaError_t err, const char* what) {
  return fail(ARC_ERR_CUDA, "%s: %s (%d)", what, cudaGetErrorString(err), static_cast<int>(err));
}

// ---------------------------------------------------------------------------------
// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda link).
// ---------------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}

// 2-D row-major matrix [rows][cols] with `ld` elements between rows.
int encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t elem_bytes, const void* ptr,
              uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_cols, uint32_t box_rows,
              CUtensorMapSwizzle swizzle, const char* what) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(ARC_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * elem_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, dtype, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return fail(ARC_ERR_CUDA, "cuTensorMapEncodeTiled(%s) failed with CUresult %d", what,
                static_cast<int>(r));
  }
  return ARC_OK;
}

// ---------------------------------------------------------------------------------
// Per-device facts and one-time kernel attributes.
// ---------------------------------------------------------------------------------
constexpr int kMaxDevices = 64;

struct DeviceState {
  std::once_flag once;
  int status = ARC_OK;
  int sms = 0;
};
DeviceState g_dev[kMaxDevices];

template <typename Kernel>
cudaError_t allow_smem(Kernel k, size_t bytes) {
  return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(bytes));
}

template <uint32_t BT, uint32_t EWG, uint32_t LS, bool kSplit>
constexpr size_t a8w4_smem_bytes() {
  return sizeof(arcb::a8w4::Smem<BT, EWG, LS, kSplit>) + 1024;
}

// The kernel instantiations the dispatcher can pick.
#define ARC_A8W4_VARIANTS(X) \
  X(16, 1, 8, true)          \
  X(32, 1, 8, true)          \
  X(64, 1, 5, false)         \
  X(128, 2, 4, false)

int init_device(int dev) {
  DeviceState& st = g_dev[dev];
  std::call_once(st.once, [&] {
    cudaDeviceProp prop;
    cudaError_t e = cudaGetDeviceProperties(&prop, dev);
    if (e != cudaSuccess) {
      st.status = cuda_fail(e, "cudaGetDeviceProperties");
      return;
    }
    if (prop.major != 10 || prop.minor != 0) {
      st.status = fail(ARC_ERR_NO_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a",
                       dev, prop.major, prop.minor);
      return;
    }
    st.sms = prop.multiProcessorCount;
    e = allow_smem(arcb::bf16::gemm_bf16_kernel, arcb::bf16::kSmemBytes);
#define ARC_SET_ATTR(BT, EWG, LS, SPLIT)                                              \
  if (e == cudaSuccess) {                                                             \
    e = allow_smem(arcb::a8w4::gemm_a8w4_kernel<BT, EWG, LS, SPLIT>,                  \
                   a8w4_smem_bytes<BT, EWG, LS, SPLIT>());                            \
  }
    ARC_A8W4_VARIANTS(ARC_SET_ATTR)
#undef ARC_SET_ATTR
    if (e != cudaSuccess) st.status = cuda_fail(e, "cudaFuncSetAttribute");
  });
  if (st.status != ARC_OK) {
    // Re-state the stored failure for this thread.
    return fail(st.status, "device %d failed to initialise (first error reported earlier)", dev);
  }
  return ARC_OK;
}

int current_device(int* dev) {
  const cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (*dev < 0 || *dev >= kMaxDevices) return fail(ARC_ERR_NO_DEVICE, "device %d out of range", *dev);
  return init_device(*dev);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

uint32_t ceil_div(uint32_t a, uint32_t b) { return (a + b - 1) / b; }

// ---------------------------------------------------------------------------------
// A8W4 work decomposition
// ---------------------------------------------------------------------------------
// Decode-sized problems (M <= 32) stream the weights once: the plan chooses a tile
// height R (multiple of 8, <= 128) and a K-split S so that ceil(N/R)*S CTAs fill the
// SMs in as few waves as possible, scored by the bytes the busiest SM streams plus a
// fixed per-wave cost. Larger M uses persistent token x weight tiles.
int plan_a8w4(int M, int N, int K, int sms, arc_a8w4_plan_t* plan) {
  const uint32_t G = static_cast<uint32_t>(K) / arcb::a8w4::kGroupK;
  if (M <= 32) {
    const uint32_t bt = M <= 16 ? 16u : 32u;
    // One "row-group" = 64 bytes of packed weights. ~1400 of them is roughly the
    // per-SM streaming time of a kernel launch's fixed overhead.
    constexpr double kWaveCost = 1400.0;
    double best = 1e300;
    arc_a8w4_plan_t bp{};
    for (uint32_t R = 128; R >= 64; R -= 8) {
      const uint32_t tiles = ceil_div(static_cast<uint32_t>(N), R);
      for (uint32_t S = 1; S <= arcb::a8w4::kMaxSplit; S *= 2) {
        if (S > G || (R % S) != 0) continue;
        const uint32_t ctas = tiles * S;
        const uint32_t waves = ceil_div(ctas, static_cast<uint32_t>(sms));
        const double cost = waves * (static_cast<double>(R) * ceil_div(G, S) + kWaveCost);
        if (cost < best - 1e-9) {
          best = cost;
          bp.split = 1;
          bp.token_tile = static_cast<int>(bt);
          bp.weight_rows = static_cast<int>(R);
          bp.k_split = static_cast<int>(S);
          bp.grid = static_cast<int>(ctas);
          bp.load_stages = 8;
        }
      }
    }
    *plan = bp;
    return ARC_OK;
  }
  const uint32_t bt = M <= 64 ? 64u : 128u;
  const uint32_t tiles = ceil_div(static_cast<uint32_t>(M), bt) *
                         ceil_div(static_cast<uint32_t>(N), arcb::a8w4::kRows);
  plan->split = 0;
  plan->token_tile = static_cast<int>(bt);
  plan->weight_rows = static_cast<int>(arcb::a8w4::kRows);
  plan->k_split = 1;
  plan->grid = static_cast<int>(tiles < static_cast<uint32_t>(sms) ? tiles : sms);
  plan->load_stages = bt == 64 ? 5 : 4;
  return ARC_OK;
}

template <uint32_t BT, uint32_t EWG, uint32_t LS, bool kSplit>
cudaError_t launch_a8w4(const arcb::a8w4::Params& p, uint32_t grid, uint32_t cluster,
                        cudaStream_t stream) {
  using C = arcb::a8w4::Cfg<BT, EWG, LS, kSplit>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(C::kThreads, 1, 1);
  cfg.dynamicSmemBytes = a8w4_smem_bytes<BT, EWG, LS, kSplit>();
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (kSplit) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, arcb::a8w4::gemm_a8w4_kernel<BT, EWG, LS, kSplit>, p);
}

}  // namespace

// =================================================================================
// C ABI
// =================================================================================
extern "C" {

int arc_version(void) { return kVersion; }

const char* arc_status_string(int status) {
  switch (status) {
    case ARC_OK: return "ok";
    case ARC_ERR_INVALID_ARGUMENT: return "invalid argument";
    case ARC_ERR_UNSUPPORTED: return "unsupported shape, alignment or recipe";
    case ARC_ERR_CUDA: return "CUDA error";
    case ARC_ERR_NO_DEVICE: return "no usable sm_100 device";
    case ARC_ERR_DEVICE_TIMEOUT: return "a kernel abandoned a wait (device timeout)";
    default: return "unknown status";
  }
}

const char* arc_last_error(void) { return g_last_error; }

int arc_matmul_bf16(const void* A, const void* B, void* C, int M, int N, int K, int lda, int ldb,
                    int ldc, cudaStream_t stream) {
  g_last_error[0] = '\0';
  if (A == nullptr || B == nullptr || C == nullptr) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_matmul_bf16: null pointer");
  }
  if (M <= 0 || N <= 0 || K <= 0) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_matmul_bf16: sizes must be positive (M=%d N=%d K=%d)",
                M, N, K);
  }
  if (lda < K || ldb < K || ldc < N) {
    return fail(ARC_ERR_INVALID_ARGUMENT,
                "arc_matmul_bf16: leading dimensions too small (lda=%d ldb=%d ldc=%d)", lda, ldb,
                ldc);
  }
  if (!aligned16(A) || !aligned16(B) || !aligned16(C) || (lda % 8) || (ldb % 8) || (ldc % 8)) {
    return fail(ARC_ERR_UNSUPPORTED,
                "arc_matmul_bf16: pointers must be 16-byte aligned and leading dimensions "
                "multiples of 8");
  }
  int dev = 0;
  if (int st = current_device(&dev)) return st;
  namespace B16 = arcb::bf16;
  B16::Params p;
  if (int st = encode_2d(&p.tm_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, A, K, M, lda, B16::BK,
                         B16::BM, CU_TENSOR_MAP_SWIZZLE_128B, "A")) {
    return st;
  }
  if (int st = encode_2d(&p.tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, B, K, N, ldb, B16::BK,
                         B16::BN, CU_TENSOR_MAP_SWIZZLE_128B, "B")) {
    return st;
  }
  if (int st = encode_2d(&p.tm_c, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, C, N, M, ldc,
                         B16::kEpiCols, B16::BM, CU_TENSOR_MAP_SWIZZLE_64B, "C")) {
    return st;
  }
  p.M = M;
  p.N = N;
  p.K = K;
  p.tiles_m = ceil_div(M, B16::BM);
  p.tiles_n = ceil_div(N, B16::BN);
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.num_kb = ceil_div(K, B16::BK);
  const uint32_t grid = p.num_tiles < static_cast<uint32_t>(g_dev[dev].sms)
                            ? p.num_tiles
                            : static_cast<uint32_t>(g_dev[dev].sms);
  B16::gemm_bf16_kernel<<<grid, B16::kNumThreads, B16::kSmemBytes, stream>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gemm_bf16_kernel launch");
  return ARC_OK;
}

int arc_a8w4_describe_plan(int M, int N, int K, int num_sms, arc_a8w4_plan_t* plan) {
  if (plan == nullptr || M <= 0 || N <= 0 || K <= 0 || num_sms <= 0) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_a8w4_describe_plan: bad argument");
  }
  if (K % static_cast<int>(arcb::a8w4::kGroupK) != 0) {
    return fail(ARC_ERR_UNSUPPORTED, "arc_a8w4_describe_plan: K must be a multiple of 128");
  }
  return plan_a8w4(M, N, K, num_sms, plan);
}

int arc_a8w4_gemm(const int8_t* A, const float* sa, const uint8_t* Wp, const uint16_t* sb,
                  uint16_t* C, int M, int N, int K, int group, cudaStream_t stream,
                  int32_t* partials_dbg) {
  g_last_error[0] = '\0';
  if (A == nullptr || sa == nullptr || Wp == nullptr || sb == nullptr || C == nullptr) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_a8w4_gemm: null pointer");
  }
  if (M <= 0 || N <= 0 || K <= 0) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_a8w4_gemm: sizes must be positive (M=%d N=%d K=%d)",
                M, N, K);
  }
  if (group != static_cast<int>(arcb::a8w4::kGroupK)) {
    return fail(ARC_ERR_UNSUPPORTED, "arc_a8w4_gemm: only group == 128 is supported (got %d)",
                group);
  }
  if (K % group != 0) {
    return fail(ARC_ERR_UNSUPPORTED, "arc_a8w4_gemm: K (%d) must be a multiple of %d", K, group);
  }
  if (N % 8 != 0) {
    return fail(ARC_ERR_UNSUPPORTED, "arc_a8w4_gemm: N (%d) must be a multiple of 8", N);
  }
  if (!aligned16(A) || !aligned16(Wp) || !aligned16(C) ||
      (reinterpret_cast<uintptr_t>(sa) & 3u) || (reinterpret_cast<uintptr_t>(sb) & 1u)) {
    return fail(ARC_ERR_UNSUPPORTED,
                "arc_a8w4_gemm: A, Wp and C must be 16-byte aligned (sa 4-byte, sb 2-byte)");
  }
  int dev = 0;
  if (int st = current_device(&dev)) return st;

  arc_a8w4_plan_t plan;
  plan_a8w4(M, N, K, g_dev[dev].sms, &plan);
  const uint32_t BT = static_cast<uint32_t>(plan.token_tile);
  const uint32_t R = static_cast<uint32_t>(plan.weight_rows);

  namespace Q = arcb::a8w4;
  Q::Params p;
  if (int st = encode_2d(&p.tm_tok, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, A, K, M, K, Q::kGroupK, BT,
                         CU_TENSOR_MAP_SWIZZLE_128B, "A")) {
    return st;
  }
  if (int st = encode_2d(&p.tm_wp, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, Wp, K / 2, N, K / 2,
                         Q::kPackedRow, R, CU_TENSOR_MAP_SWIZZLE_NONE, "Wp")) {
    return st;
  }
  if (!plan.split) {
    if (int st = encode_2d(&p.tm_out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, C, N, M, N, Q::kRows,
                           BT, CU_TENSOR_MAP_SWIZZLE_NONE, "C")) {
      return st;
    }
  } else {
    memset(&p.tm_out, 0, sizeof(p.tm_out));
  }
  p.sa = sa;
  p.sb = sb;
  p.out = C;
  p.partials = partials_dbg;
  p.M = M;
  p.N = N;
  p.K = K;
  p.G = K / group;
  p.ldsb = p.G;
  p.ldc = N;
  p.R = R;
  p.S = plan.k_split;
  p.tiles_m = ceil_div(M, BT);
  p.tiles_n = ceil_div(N, R);
  p.num_tiles = p.tiles_m * p.tiles_n;

  cudaError_t e = cudaErrorInvalidConfiguration;
  if (plan.split) {
    const uint32_t grid = p.num_tiles * p.S;
    if (BT == 16) e = launch_a8w4<16, 1, 8, true>(p, grid, p.S, stream);
    else e = launch_a8w4<32, 1, 8, true>(p, grid, p.S, stream);
  } else {
    const uint32_t grid = static_cast<uint32_t>(plan.grid);
    if (BT == 64) e = launch_a8w4<64, 1, 5, false>(p, grid, 1, stream);
    else e = launch_a8w4<128, 2, 4, false>(p, grid, 1, stream);
  }
  if (e != cudaSuccess) return cuda_fail(e, "gemm_a8w4_kernel launch");
  return ARC_OK;
}

int arc_device_status(int device, uint32_t* status, int clear) {
  if (status == nullptr) return fail(ARC_ERR_INVALID_ARGUMENT, "arc_device_status: null pointer");
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (device != prev && (e = cudaSetDevice(device)) != cudaSuccess) {
    return cuda_fail(e, "cudaSetDevice");
  }
  e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(status, arcb::g_arc_status, sizeof(uint32_t));
  if (e == cudaSuccess && clear) {
    const uint32_t zero = 0;
    e = cudaMemcpyToSymbol(arcb::g_arc_status, &zero, sizeof(uint32_t));
  }
  if (device != prev) cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "arc_device_status");
  return ARC_OK;
}

}  // extern "C"
