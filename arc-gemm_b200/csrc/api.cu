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
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "arc_b200.h"
#include "gemm_a8w4.cuh"
#include "gemm_bf16_pair.cuh"
#include "gemm_a8w4_decode.cuh"
#include "gemm_fp8fp4.cuh"
#include "gemm_fp8fp4_pair.cuh"
#include "peer_barrier.cuh"
#include "prepack.cuh"
#include "quantize.cuh"
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

// Packed e2m1 codes [N][K/2 bytes] viewed as [G][N][128 codes] of type 16U4_ALIGN16B:
// group g's weight tile is the box {128, rows, groups} at (0, n0, g); in shared memory
// every 16 codes (8 bytes) are padded to 16 bytes, so a 128-code row takes 128 bytes
// and the 128-byte swizzle applies as for an 8-bit tile. Needs a 32-byte aligned base
// and K % 64 == 0 (row stride a multiple of 32 bytes).
int encode_e2m1_3d(CUtensorMap* map, const void* ptr, uint64_t N, uint64_t K, uint32_t box_rows,
                   uint32_t box_groups) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(ARC_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[3] = {128, N, K / 128};
  const cuuint64_t strides[2] = {K / 2, 64};
  const cuuint32_t box[3] = {128, box_rows, box_groups};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 3, const_cast<void*>(ptr), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return fail(ARC_ERR_CUDA, "cuTensorMapEncodeTiled(e2m1 weights 3-D) failed with CUresult %d",
                static_cast<int>(r));
  }
  return ARC_OK;
}

// A [M][K] byte matrix viewed as [G][M][128]: group g's token tile is the 3-D box
// {128, rows, groups} at (0, m0, g), landing as consecutive [rows][128] tiles.
int encode_tokens_3d(CUtensorMap* map, const void* ptr, uint64_t M, uint64_t K, uint32_t box_rows,
                     uint32_t box_groups) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(ARC_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[3] = {128, M, K / 128};
  const cuuint64_t strides[2] = {K, 128};
  const cuuint32_t box[3] = {128, box_rows, box_groups};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(ptr), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return fail(ARC_ERR_CUDA, "cuTensorMapEncodeTiled(tokens 3-D) failed with CUresult %d",
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
  int max_clusters2 = 0;  // co-resident 2-CTA clusters of the decode kernel
  int max_clusters4 = 0;  // co-resident 4-CTA clusters of the decode kernel
  int max_bf16_pairs = 0;  // co-resident CTA pairs of the bf16 pair kernel
  int max_fp8fp4_pairs = 0;  // co-resident CTA pairs of the FP8 x FP4 pair kernel
};
DeviceState g_dev[kMaxDevices];

template <typename Kernel>
cudaError_t allow_smem(Kernel k, size_t bytes) {
  return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(bytes));
}

template <uint32_t BT, uint32_t EWG, uint32_t LS>
constexpr size_t a8w4_smem_bytes() {
  return sizeof(arcb::a8w4::Smem<BT, EWG, LS>) + 1024;
}

template <uint32_t BT>
constexpr size_t decode_smem_bytes() {
  return sizeof(arcb::a8w4dec::Smem<BT>) + 1024;
}

// The decode instantiations the dispatcher can launch: token tile x stream mode x cluster size,
// each plain, with the partials dump, or with the fused all-gather.
#define ARC_DECODE_VARIANTS_MODE(X, BT, STR, SK) \
  X(BT, STR, false, SK, false)                   \
  X(BT, STR, true, SK, false)                    \
  X(BT, STR, false, SK, true)
#define ARC_DECODE_VARIANTS_BT(X, BT)                                                            \
  ARC_DECODE_VARIANTS_MODE(X, BT, false, 1) ARC_DECODE_VARIANTS_MODE(X, BT, false, 2)              \
  ARC_DECODE_VARIANTS_MODE(X, BT, false, 4) ARC_DECODE_VARIANTS_MODE(X, BT, true, 1)               \
  ARC_DECODE_VARIANTS_MODE(X, BT, true, 2) ARC_DECODE_VARIANTS_MODE(X, BT, true, 4)
#define ARC_DECODE_VARIANTS(X) ARC_DECODE_VARIANTS_BT(X, 16) ARC_DECODE_VARIANTS_BT(X, 32)
constexpr int kDecodeVariants = 36;

// Decode stream mode: some CTA of the plan has more load stages (two K-groups each) than
// the weight ring holds.
bool decode_stream(int G, int S, int num_items, int grid) {
  const int ng_max = (G + S - 1) / S;
  const int items_max = S > 1 ? 1 : (num_items + grid - 1) / grid;
  return items_max * ((ng_max + 1) / 2) > static_cast<int>(arcb::a8w4dec::kWStages);
}

// The persistent-tile instantiations the dispatcher can pick (M > 32).
#define ARC_A8W4_VARIANTS(X) \
  X(64, 1, 4)                \
  X(128, 2, 3)

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
    if (e == cudaSuccess) e = allow_smem(arcb::bf16pair::gemm_bf16_pair_kernel, arcb::bf16pair::kSmemBytes);
    // The persistent kernel moves registers between its warpgroups (setmaxnreg); the
    // shares are sized for a launch count of Cfg::kLaunchRegs per thread, and a
    // different compiled count could leave an increase waiting, so refuse it.
    bool regs_ok = true;
#define ARC_SET_ATTR(BT, EWG, LS)                                                     \
  if (e == cudaSuccess) {                                                             \
    e = allow_smem(arcb::a8w4::gemm_a8w4_kernel<BT, EWG, LS>,                         \
                   a8w4_smem_bytes<BT, EWG, LS>());                                   \
  }                                                                                   \
  if (e == cudaSuccess) {                                                             \
    cudaFuncAttributes fa;                                                            \
    e = cudaFuncGetAttributes(&fa, arcb::a8w4::gemm_a8w4_kernel<BT, EWG, LS>);        \
    if (e == cudaSuccess &&                                                           \
        fa.numRegs != static_cast<int>(arcb::a8w4::Cfg<BT, EWG, LS>::kLaunchRegs)) {  \
      regs_ok = false;                                                                \
    }                                                                                 \
  }
    ARC_A8W4_VARIANTS(ARC_SET_ATTR)
#undef ARC_SET_ATTR
    if (e == cudaSuccess && !regs_ok) {
      st.status = fail(ARC_ERR_UNSUPPORTED,
                       "gemm_a8w4_kernel was compiled with an unexpected register count");
      return;
    }
    // The decode kernels (token tile x chunk / stream mode) also move registers between
    // warpgroups (64 per thread at launch, two CTAs per SM).
    {
      namespace D = arcb::a8w4dec;
      const void* kerns[kDecodeVariants];
      size_t smems[kDecodeVariants];
      int nk = 0;
#define ARC_DECODE_KERN(BT, STR, DUMP, SK, GATHER)                                        \
  kerns[nk] = reinterpret_cast<const void*>(D::gemm_a8w4_decode_kernel<BT, STR, DUMP, SK, GATHER>); \
  smems[nk++] = decode_smem_bytes<BT>();
      ARC_DECODE_VARIANTS(ARC_DECODE_KERN)
#undef ARC_DECODE_KERN
      for (int v = 0; v < nk && e == cudaSuccess; ++v) {
        const size_t smem = smems[v];
        e = cudaFuncSetAttribute(kerns[v], cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        cudaFuncAttributes fa;
        if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, kerns[v]);
        if (e == cudaSuccess && fa.numRegs != static_cast<int>(D::kLaunchRegs)) {
          st.status = fail(ARC_ERR_UNSUPPORTED, "gemm_a8w4_decode_kernel was compiled with an unexpected register count");
          return;
        }
      }
    }
    if (e == cudaSuccess) {
      e = allow_smem(arcb::fp8fp4::gemm_fp8fp4_kernel<1>, sizeof(arcb::fp8fp4::Smem<1>) + 1024);
    }
    if (e == cudaSuccess) {
      e = allow_smem(arcb::fp8fp4::gemm_fp8fp4_kernel<2>, sizeof(arcb::fp8fp4::Smem<2>) + 1024);
    }
    if (e == cudaSuccess) {
      e = allow_smem(arcb::fp8fp4pair::gemm_fp8fp4_pair_kernel, arcb::fp8fp4pair::kSmemBytes);
    }
    if (e == cudaSuccess) {
      cudaFuncAttributes fa;
      e = cudaFuncGetAttributes(&fa, arcb::fp8fp4pair::gemm_fp8fp4_pair_kernel);
      if (e == cudaSuccess && fa.numRegs != static_cast<int>(arcb::fp8fp4pair::kLaunchRegs)) {
        st.status = fail(ARC_ERR_UNSUPPORTED,
                         "gemm_fp8fp4_pair_kernel was compiled with an unexpected register count");
        return;
      }
    }
    if (e == cudaSuccess) {
      cudaFuncAttributes fa;
      e = cudaFuncGetAttributes(&fa, arcb::fp8fp4::gemm_fp8fp4_kernel<2>);
      if (e == cudaSuccess && fa.numRegs != static_cast<int>(arcb::fp8fp4::Cfg<2>::kLaunchRegs)) {
        st.status = fail(ARC_ERR_UNSUPPORTED,
                         "gemm_fp8fp4_kernel was compiled with an unexpected register count");
        return;
      }
    }
    if (e != cudaSuccess) {
      st.status = cuda_fail(e, "cudaFuncSetAttribute");
      return;
    }
    // How many 2- and 4-CTA clusters of the (larger) decode variant fit at once.
    for (uint32_t size : {2u, 4u}) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(size * st.sms, 1, 1);
      cfg.blockDim = dim3(arcb::a8w4dec::kThreads, 1, 1);
      cfg.dynamicSmemBytes = decode_smem_bytes<32>();
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = size;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, arcb::a8w4dec::gemm_a8w4_decode_kernel<32, false, false, 4, false>, &cfg) !=
          cudaSuccess) {
        cudaGetLastError();  // clear; plans then avoid clusters of this size
        n = 0;
      }
      (size == 2 ? st.max_clusters2 : st.max_clusters4) = n;
    }
    {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(st.sms, 1, 1);
      cfg.blockDim = dim3(arcb::bf16pair::kNumThreads, 1, 1);
      cfg.dynamicSmemBytes = arcb::bf16pair::kSmemBytes;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, arcb::bf16pair::gemm_bf16_pair_kernel, &cfg) != cudaSuccess) {
        cudaGetLastError();  // clear; bf16 GEMMs then use the one-CTA kernel
        n = 0;
      }
      st.max_bf16_pairs = n;
    }
    {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(st.sms, 1, 1);
      cfg.blockDim = dim3(arcb::fp8fp4pair::kThreads, 1, 1);
      cfg.dynamicSmemBytes = arcb::fp8fp4pair::kSmemBytes;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, arcb::fp8fp4pair::gemm_fp8fp4_pair_kernel, &cfg) != cudaSuccess) {
        cudaGetLastError();  // clear; FP8 x FP4 GEMMs then use the one-CTA kernels
        n = 0;
      }
      st.max_fp8fp4_pairs = n;
    }
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
constexpr uint32_t kDecodeMaxM = 32;
// K-groups per tile from which a decode problem is long enough to be bound by HBM rather
// than by the launch chain: its plans may use both CTA slots of an SM.
constexpr uint32_t kDecodeLongG = 64;

// Decode-sized problems (M <= 32) stream the weights once, in 128-row tiles. A plan is a
// K split S in {1, 2, 4}: S > 1 runs one wave of S-CTA clusters that reduce on chip
// (every CTA streams 1/S of a tile's K-groups); S == 1 runs persistent CTAs over whole
// tiles. The largest S whose grid stays within one CTA per SM is taken, so that the next
// launch in the stream finds a free slot on every SM (two decode CTAs fit on one SM) and
// overlaps this one; each CTA's UMMA issue (four per K-group) shrinks with S.
//
// ARC_DECODE_PLAN="128:S[:grid]" (tuning and tests only) forces the K split, and for
// S == 1 optionally caps the grid (so that CTAs walk several tiles); it is ignored unless
// it is valid for the shape and device.
bool decode_override(uint32_t tiles, uint32_t G, int sms, int max_c2, int max_c4, arc_a8w4_plan_t* plan);

void decode_plan(uint32_t bt, uint32_t S, uint32_t grid, arc_a8w4_plan_t* plan) {
  plan->split = S > 1 ? 1 : 0;
  plan->token_tile = static_cast<int>(bt);
  plan->weight_rows = static_cast<int>(arcb::a8w4::kRows);
  plan->k_split = static_cast<int>(S);
  plan->grid = static_cast<int>(grid);
  plan->load_stages = static_cast<int>(arcb::a8w4dec::kWStages);
  plan->groups_per_stage = static_cast<int>(arcb::a8w4dec::kGps);
}

int plan_a8w4(int M, int N, int K, int sms, int max_c2, int max_c4, arc_a8w4_plan_t* plan) {
  const uint32_t G = static_cast<uint32_t>(K) / arcb::a8w4::kGroupK;
  if (M <= static_cast<int>(kDecodeMaxM)) {
    const uint32_t bt = M <= 16 ? 16u : 32u;
    const uint32_t tiles = ceil_div(static_cast<uint32_t>(N), arcb::a8w4::kRows);
    if (decode_override(tiles, G, sms, max_c2, max_c4, plan)) {
      plan->token_tile = static_cast<int>(bt);
      return ARC_OK;
    }
    // Short problems keep one CTA per SM (the next launch's CTAs take the other slot);
    // long ones (many K-groups per tile) may use both slots: twice the CTAs streaming.
    const uint32_t slots = static_cast<uint32_t>(sms) * (G >= kDecodeLongG ? 2u : 1u);
    for (uint32_t S : {4u, 2u}) {
      const int cap = S == 2 ? max_c2 : max_c4;
      if (S <= G && tiles * S <= slots && tiles <= static_cast<uint32_t>(cap)) {
        decode_plan(bt, S, tiles * S, plan);
        return ARC_OK;
      }
    }
    decode_plan(bt, 1, tiles < slots ? tiles : slots, plan);
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
  plan->load_stages = bt == 64 ? 4 : 3;
  plan->groups_per_stage = static_cast<int>(arcb::a8w4::kGps);
  return ARC_OK;
}

bool decode_override(uint32_t tiles, uint32_t G, int sms, int max_c2, int max_c4, arc_a8w4_plan_t* plan) {
  const char* env = getenv("ARC_DECODE_PLAN");
  unsigned R = 0, S = 0, grid_cap = 0;
  if (env == nullptr || sscanf(env, "%u:%u:%u", &R, &S, &grid_cap) < 2) return false;
  if (R != arcb::a8w4::kRows || !(S == 1 || S == 2 || S == 4) || S > G) return false;
  if (S > 1 && tiles > static_cast<uint32_t>(S == 2 ? max_c2 : max_c4)) return false;
  uint32_t grid = S > 1 ? tiles * S : (tiles < static_cast<uint32_t>(sms) ? tiles : static_cast<uint32_t>(sms));
  if (S == 1 && grid_cap > 0 && grid_cap < grid) grid = grid_cap;
  decode_plan(16, S, grid, plan);
  return true;
}

// Launch with programmatic stream serialization (PDL) and an optional cluster.
template <typename Kern, typename P>
cudaError_t launch_ex(Kern kernel, const P& p, uint32_t grid, uint32_t threads, size_t smem,
                      uint32_t cluster, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  uint32_t n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = 1;
  ++n;
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

// Launch the decode instantiation of the mode (stream or chunk) and of the partials dump.
// The fused-gather entry points pass no partials buffer, so the gather instantiations
// carry no dump.
template <uint32_t BT, bool STR, uint32_t SK>
cudaError_t launch_decode_mode(const arcb::a8w4dec::Params& p, uint32_t grid, uint32_t S, bool dump, bool gather,
                               cudaStream_t stream) {
  namespace D = arcb::a8w4dec;
  auto k = gather ? D::gemm_a8w4_decode_kernel<BT, STR, false, SK, true>
                  : (dump ? D::gemm_a8w4_decode_kernel<BT, STR, true, SK, false>
                          : D::gemm_a8w4_decode_kernel<BT, STR, false, SK, false>);
  return launch_ex(k, p, grid, D::kThreads, decode_smem_bytes<BT>(), S, stream);
}
template <uint32_t BT>
cudaError_t launch_decode(const arcb::a8w4dec::Params& p, uint32_t grid, uint32_t S, bool str, bool dump,
                          cudaStream_t stream) {
  const bool gather = p.peers > 0;
  if (str) {
    return S == 4 ? launch_decode_mode<BT, true, 4>(p, grid, S, dump, gather, stream)
         : S == 2 ? launch_decode_mode<BT, true, 2>(p, grid, S, dump, gather, stream)
                  : launch_decode_mode<BT, true, 1>(p, grid, S, dump, gather, stream);
  }
  return S == 4 ? launch_decode_mode<BT, false, 4>(p, grid, S, dump, gather, stream)
       : S == 2 ? launch_decode_mode<BT, false, 2>(p, grid, S, dump, gather, stream)
                : launch_decode_mode<BT, false, 1>(p, grid, S, dump, gather, stream);
}


// bf16 kernel choice. CTA pairs (256 x 256 tiles, half the shared-memory traffic per
// MAC) once the pair tiles give every co-resident pair one; one CTA per 128 x 256 tile
// below that (e.g. 2048^3: 64 pair tiles would leave 20 SMs idle, 128 one-CTA tiles
// fill as many). ARC_BF16_CTAS=1|2 forces one (tests and tuning).
int choose_bf16(int dev, int M, int N, bool* pairs) {
  const uint32_t max_pairs = static_cast<uint32_t>(g_dev[dev].max_bf16_pairs);
  *pairs = max_pairs > 0 && static_cast<uint32_t>(ceil_div(M, 256) * ceil_div(N, 256)) >= max_pairs;
  if (const char* env = getenv("ARC_BF16_CTAS")) {
    const int v = atoi(env);
    if (v != 1 && v != 2) {
      return fail(ARC_ERR_INVALID_ARGUMENT, "ARC_BF16_CTAS must be 1 or 2 (got '%s')", env);
    }
    if (v == 2 && max_pairs == 0) {
      return fail(ARC_ERR_UNSUPPORTED, "ARC_BF16_CTAS=2: no CTA pair of the bf16 kernel fits on this device");
    }
    *pairs = v == 2;
  }
  return ARC_OK;
}

// FP8 x FP4 kernel choice (variant 0: 128-row tiles, 1: 256-row tiles, 2: CTA pairs).
// Pairs on 256 x 256 tiles (full-rate N=256 UMMAs, half the shared-memory bytes per MAC)
// when the pair tiles give every co-resident pair one and K % 512 == 0 (the token-scale
// tensor map needs a 16-byte row pitch); else one CTA per 256-row weight tile when
// those fill the SMs; else 128-row tiles (twice the CTAs, e.g. for decode batches).
// ARC_FP8FP4_KERNEL=128|256|pair forces one (tests and tuning).
int choose_fp8fp4(int dev, int M, int N, int K, bool sfa_aligned16, int* variant) {
  const uint32_t sms = static_cast<uint32_t>(g_dev[dev].sms);
  const uint32_t max_pairs = static_cast<uint32_t>(g_dev[dev].max_fp8fp4_pairs);
  const bool pairs_ok = max_pairs > 0 && K % 512 == 0 && sfa_aligned16;
  *variant = ceil_div(M, 128) * ceil_div(N, 256) >= sms ? 1 : 0;
  if (pairs_ok && ceil_div(M, 256) * ceil_div(N, 256) >= max_pairs) *variant = 2;
  if (const char* env = getenv("ARC_FP8FP4_KERNEL")) {
    if (strcmp(env, "pair") == 0) {
      if (!pairs_ok) {
        return fail(ARC_ERR_UNSUPPORTED,
                    "ARC_FP8FP4_KERNEL=pair needs K %% 512 == 0, a 16-byte aligned sfa and a co-resident CTA pair");
      }
      *variant = 2;
    } else if (strcmp(env, "128") == 0) {
      *variant = 0;
    } else if (strcmp(env, "256") == 0) {
      *variant = 1;
    } else {
      return fail(ARC_ERR_INVALID_ARGUMENT, "ARC_FP8FP4_KERNEL must be 128, 256 or pair (got '%s')", env);
    }
  }
  return ARC_OK;
}

// K split of the one-CTA FP8 x FP4 kernel for problems with fewer 128 x 128 tiles than
// SMs (decode batches): S CTAs per tile (2, 4 or 8, all resident in one wave), each
// taking gs K groups (a multiple of 2, the groups per stage). Workspace: one uint32
// counter per tile in a fixed 4 KB head (a split problem has fewer tiles than SMs), then
// S fp32 partials of [M][N]. The head never holds partials, so one workspace serves
// problems of any shape in turn: the kernel leaves every counter at zero.
constexpr size_t kSplitCounterBytes = 4096;
struct SplitPlan {
  uint32_t S, gs;
  size_t partial_offset, bytes;
};
SplitPlan fp8fp4_split_plan(int dev, int M, int N, int K) {
  SplitPlan sp{1, static_cast<uint32_t>(K / 128), 0, 0};
  const uint32_t sms = static_cast<uint32_t>(g_dev[dev].sms);
  const uint32_t G = static_cast<uint32_t>(K / 128);
  const uint32_t tiles = static_cast<uint32_t>(ceil_div(M, 128) * ceil_div(N, 128));
  uint32_t S = 1;
  for (uint32_t c : {8u, 4u, 2u}) {
    if (tiles * c <= sms && G >= 2 * c) {
      S = c;
      break;
    }
  }
  if (const char* env = getenv("ARC_FP8FP4_SPLIT")) {  // tests and tuning
    const int v = atoi(env);
    if (v >= 1 && v <= 16 && static_cast<uint32_t>(v) * 2 <= G) S = static_cast<uint32_t>(v);
  }
  if (S <= 1) return sp;
  uint32_t gs = (G + S - 1) / S;
  gs += gs & 1u;
  S = (G + gs - 1) / gs;  // no empty splits
  if (S <= 1) return sp;
  sp.S = S;
  sp.gs = gs;
  if (size_t(tiles) * sizeof(uint32_t) > kSplitCounterBytes) return SplitPlan{1, G, 0, 0};
  sp.partial_offset = kSplitCounterBytes;
  sp.bytes = kSplitCounterBytes + size_t(S) * M * N * sizeof(float);
  return sp;
}

// Argument checks of the FP8 x FP4 entry points (host only: no device call, nothing enqueued).
int fp8fp4_check(const uint8_t* A, const float* sfa, const uint8_t* Wp, const float* sfw, const uint16_t* C,
                 int M, int N, int K) {
  if (A == nullptr || sfa == nullptr || Wp == nullptr || sfw == nullptr || C == nullptr) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_fp8_fp4_gemm: null pointer");
  }
  if (M <= 0 || N <= 0 || K <= 0) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_fp8_fp4_gemm: sizes must be positive (M=%d N=%d K=%d)",
                M, N, K);
  }
  if (K % 128 != 0 || N % 8 != 0) {
    return fail(ARC_ERR_UNSUPPORTED, "arc_fp8_fp4_gemm: need K %% 128 == 0 and N %% 8 == 0 (N=%d K=%d)",
                N, K);
  }
  if (!aligned16(A) || (reinterpret_cast<uintptr_t>(Wp) & 31u) || !aligned16(C) || !aligned16(sfw) ||
      (reinterpret_cast<uintptr_t>(sfa) & 3u)) {
    return fail(ARC_ERR_UNSUPPORTED,
                "arc_fp8_fp4_gemm: A, C and sfw must be 16-byte aligned, Wp 32-byte (sfa 4-byte)");
  }
  return ARC_OK;
}

int fp8fp4_gemm(const uint8_t* A, const float* sfa, const uint8_t* Wp, const float* sfw, uint16_t* C,
                int M, int N, int K, void* workspace, size_t workspace_bytes, cudaStream_t stream);
int a8w4_gemm(const int8_t* A, const float* sa, const uint8_t* Wp, const uint16_t* sb, uint16_t* C, int M,
              int N, int K, int group, cudaStream_t stream, int32_t* partials_dbg, uint16_t* const* outs,
              int world, int rank, uint32_t flags, uint32_t* const* bar_flags = nullptr);

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

int arc_kernel_name(int op, int M, int N, int K, char* name, int len) {
  g_last_error[0] = '\0';
  if (name == nullptr || len <= 0 || M <= 0 || N <= 0 || K <= 0) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_kernel_name: bad argument");
  }
  int dev = 0;
  if (int st = current_device(&dev)) return st;
  const char* kernel = nullptr;
  if (op == ARC_OP_MATMUL_BF16) {
    bool pairs = false;
    if (int st = choose_bf16(dev, M, N, &pairs)) return st;
    kernel = pairs ? "gemm_bf16_pair_kernel" : "gemm_bf16_kernel";
  } else if (op == ARC_OP_A8W4) {
    if (K % static_cast<int>(arcb::a8w4::kGroupK) != 0) {
      return fail(ARC_ERR_UNSUPPORTED, "arc_kernel_name: K must be a multiple of 128");
    }
    arc_a8w4_plan_t plan;
    plan_a8w4(M, N, K, g_dev[dev].sms, g_dev[dev].max_clusters2, g_dev[dev].max_clusters4, &plan);
    if (M <= static_cast<int>(kDecodeMaxM)) {
      const bool str = decode_stream(K / static_cast<int>(arcb::a8w4::kGroupK), plan.k_split,
                                     ceil_div(N, static_cast<int>(arcb::a8w4::kRows)), plan.grid);
      // As ncu lists them: gemm_a8w4_decode_kernel<BT, STREAM, DUMP, cluster size, GATHER>.
      static const char* kNames[2][2][3] = {
          {{"gemm_a8w4_decode_kernel<16, 0, 0, 1, 0>", "gemm_a8w4_decode_kernel<16, 0, 0, 2, 0>",
            "gemm_a8w4_decode_kernel<16, 0, 0, 4, 0>"},
           {"gemm_a8w4_decode_kernel<16, 1, 0, 1, 0>", "gemm_a8w4_decode_kernel<16, 1, 0, 2, 0>",
            "gemm_a8w4_decode_kernel<16, 1, 0, 4, 0>"}},
          {{"gemm_a8w4_decode_kernel<32, 0, 0, 1, 0>", "gemm_a8w4_decode_kernel<32, 0, 0, 2, 0>",
            "gemm_a8w4_decode_kernel<32, 0, 0, 4, 0>"},
           {"gemm_a8w4_decode_kernel<32, 1, 0, 1, 0>", "gemm_a8w4_decode_kernel<32, 1, 0, 2, 0>",
            "gemm_a8w4_decode_kernel<32, 1, 0, 4, 0>"}}};
      kernel = kNames[plan.token_tile == 16 ? 0 : 1][str ? 1 : 0][plan.k_split == 4 ? 2 : plan.k_split == 2 ? 1 : 0];
    } else {
      kernel = plan.token_tile == 64 ? "gemm_a8w4_kernel<64,1,4>" : "gemm_a8w4_kernel<128,2,3>";
    }
  } else if (op == ARC_OP_FP8_FP4) {
    int variant = 0;
    if (int st = choose_fp8fp4(dev, M, N, K, true, &variant)) return st;
    kernel = variant == 2 ? "gemm_fp8fp4_pair_kernel"
                          : (variant == 1 ? "gemm_fp8fp4_kernel<2>" : "gemm_fp8fp4_kernel<1>");
  } else {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_kernel_name: unknown op %d", op);
  }
  snprintf(name, static_cast<size_t>(len), "%s", kernel);
  return ARC_OK;
}

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
  const uint32_t sms = static_cast<uint32_t>(g_dev[dev].sms);
  const uint32_t max_pairs = static_cast<uint32_t>(g_dev[dev].max_bf16_pairs);
  bool pairs = false;
  if (int st = choose_bf16(dev, M, N, &pairs)) return st;
  if (pairs) {
    namespace P2 = arcb::bf16pair;
    P2::Params p;
    if (int st = encode_2d(&p.tm_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, A, K, M, lda, P2::BK,
                           P2::kRowsPerCta, CU_TENSOR_MAP_SWIZZLE_128B, "A")) {
      return st;
    }
    if (int st = encode_2d(&p.tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, B, K, N, ldb, P2::BK,
                           P2::kRowsPerCta, CU_TENSOR_MAP_SWIZZLE_128B, "B")) {
      return st;
    }
    if (int st = encode_2d(&p.tm_c, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, C, N, M, ldc,
                           P2::kEpiCols, P2::kRowsPerCta, CU_TENSOR_MAP_SWIZZLE_64B, "C")) {
      return st;
    }
    p.M = M;
    p.N = N;
    p.K = K;
    p.tiles_m = ceil_div(M, P2::kTileM);
    p.tiles_n = ceil_div(N, P2::kTileN);
    p.num_tiles = p.tiles_m * p.tiles_n;
    p.num_kb = ceil_div(K, P2::BK);
    // One wave of co-resident pairs strides over the pair tiles.
    const uint32_t grid = 2 * (p.num_tiles < max_pairs ? p.num_tiles : max_pairs);
    const cudaError_t e =
        launch_ex(P2::gemm_bf16_pair_kernel, p, grid, P2::kNumThreads, P2::kSmemBytes, 2, stream);
    if (e != cudaSuccess) return cuda_fail(e, "gemm_bf16_pair_kernel launch");
    return ARC_OK;
  }
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
  const uint32_t grid = p.num_tiles < sms ? p.num_tiles : sms;
  const cudaError_t e =
      launch_ex(B16::gemm_bf16_kernel, p, grid, B16::kNumThreads, B16::kSmemBytes, 1, stream);
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
  // Without a device: two decode CTAs fit on an SM, and clusters of 2 and 4 tile the
  // SMs completely.
  return plan_a8w4(M, N, K, num_sms, num_sms, num_sms / 2, plan);
}

int arc_a8w4_gemm(const int8_t* A, const float* sa, const uint8_t* Wp, const uint16_t* sb,
                  uint16_t* C, int M, int N, int K, int group, cudaStream_t stream,
                  int32_t* partials_dbg) {
  g_last_error[0] = '\0';
  return a8w4_gemm(A, sa, Wp, sb, C, M, N, K, group, stream, partials_dbg, nullptr, 0, 0, 0u);
}

int arc_a8w4_gemm_ex(const int8_t* A, const float* sa, const uint8_t* Wp, const uint16_t* sb, uint16_t* C,
                     int M, int N, int K, int group, unsigned flags, cudaStream_t stream, int32_t* partials_dbg) {
  g_last_error[0] = '\0';
  if (flags & ~(ARC_A8W4_PREPACKED | ARC_A8W4_STATIC_WEIGHTS)) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_a8w4_gemm_ex: unknown flags 0x%x", flags);
  }
  if ((flags & ARC_A8W4_PREPACKED) && partials_dbg != nullptr) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_a8w4_gemm_ex: no partials dump with pre-packed weights");
  }
  return a8w4_gemm(A, sa, Wp, sb, C, M, N, K, group, stream, partials_dbg, nullptr, 0, 0, flags);
}

int arc_a8w4_gemm_prepacked(const int8_t* A, const float* sa, const uint8_t* Wq, const uint16_t* sb,
                            uint16_t* C, int M, int N, int K, int group, cudaStream_t stream) {
  g_last_error[0] = '\0';
  return a8w4_gemm(A, sa, Wq, sb, C, M, N, K, group, stream, nullptr, nullptr, 0, 0, ARC_A8W4_PREPACKED);
}

int arc_a8w4_prepack_weights(const uint8_t* Wp, uint8_t* Wq, int N, int K, cudaStream_t stream) {
  g_last_error[0] = '\0';
  if (Wp == nullptr || Wq == nullptr) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_a8w4_prepack_weights: null pointer");
  }
  if (N <= 0 || K <= 0) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_a8w4_prepack_weights: sizes must be positive (N=%d K=%d)", N, K);
  }
  if (K % 32 != 0) {
    return fail(ARC_ERR_UNSUPPORTED, "arc_a8w4_prepack_weights: K (%d) must be a multiple of 32", K);
  }
  if (!aligned16(Wp) || !aligned16(Wq)) {
    return fail(ARC_ERR_UNSUPPORTED, "arc_a8w4_prepack_weights: Wp and Wq must be 16-byte aligned");
  }
  const uint64_t bytes = uint64_t(N) * uint64_t(K / 2);
  const uintptr_t src = reinterpret_cast<uintptr_t>(Wp), dst = reinterpret_cast<uintptr_t>(Wq);
  if (src != dst && src < dst + bytes && dst < src + bytes) {
    return fail(ARC_ERR_INVALID_ARGUMENT,
                "arc_a8w4_prepack_weights: Wq overlaps Wp without being the same buffer");
  }
  int dev = 0;
  if (int st = current_device(&dev)) return st;
  namespace PP = arcb::prepack;
  const uint64_t pieces = bytes / 16u;
  const uint64_t per_block = uint64_t(PP::kThreads) * PP::kUnroll;
  const uint64_t want = (pieces + per_block - 1) / per_block;
  const uint64_t cap = uint64_t(g_dev[dev].sms) * 8u;  // 8 resident 256-thread blocks per SM
  const uint32_t grid = static_cast<uint32_t>(want < cap ? want : cap);
  PP::prepack_w4_kernel<<<grid, PP::kThreads, 0, stream>>>(reinterpret_cast<const uint4*>(Wp),
                                                           reinterpret_cast<uint4*>(Wq), pieces);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "prepack_w4_kernel launch");
  return ARC_OK;
}

int arc_a8w4_gemm_gather_ex(const int8_t* A, const float* sa, const uint8_t* Wp, const uint16_t* sb,
                            uint16_t* const* outs, int world, int rank, int M, int N, int K, unsigned flags,
                            cudaStream_t stream) {
  g_last_error[0] = '\0';
  if (flags & ~ARC_A8W4_STATIC_WEIGHTS) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_a8w4_gemm_gather_ex: unsupported flags 0x%x", flags);
  }
  if (outs == nullptr || world < 1 || world > static_cast<int>(arcb::peer::kMaxPeers) || rank < 0 ||
      rank >= world) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_a8w4_gemm_gather: bad outs / world (%d) / rank (%d)", world,
                rank);
  }
  for (int i = 0; i < world; ++i) {
    if (outs[i] == nullptr || !aligned16(outs[i])) {
      return fail(ARC_ERR_INVALID_ARGUMENT, "arc_a8w4_gemm_gather: output %d is null or not 16-byte aligned", i);
    }
  }
  if (M <= 0 || M > static_cast<int>(kDecodeMaxM)) {
    return fail(ARC_ERR_UNSUPPORTED,
                "arc_a8w4_gemm_gather: the fused all-gather covers decode batches (1 <= M <= %u, got %d)",
                kDecodeMaxM, M);
  }
  if (N <= 0 || N % 8 != 0) {
    return fail(ARC_ERR_UNSUPPORTED, "arc_a8w4_gemm_gather: N (%d) must be a positive multiple of 8", N);
  }
  return a8w4_gemm(A, sa, Wp, sb, outs[rank] + size_t(rank) * N, M, N, K, 128, stream, nullptr, outs, world,
                   rank, flags);
}

int arc_a8w4_gemm_gather(const int8_t* A, const float* sa, const uint8_t* Wp, const uint16_t* sb,
                         uint16_t* const* outs, int world, int rank, int M, int N, int K,
                         cudaStream_t stream) {
  return arc_a8w4_gemm_gather_ex(A, sa, Wp, sb, outs, world, rank, M, N, K, 0u, stream);
}

int arc_a8w4_gemm_gather_sync(const int8_t* A, const float* sa, const uint8_t* Wp, const uint16_t* sb,
                              uint16_t* const* outs, uint32_t* const* bar_flags, int world, int rank, int M,
                              int N, int K, unsigned flags, cudaStream_t stream) {
  g_last_error[0] = '\0';
  if (bar_flags == nullptr || world < 1 || world > static_cast<int>(arcb::peer::kMaxPeers)) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_a8w4_gemm_gather_sync: bad flags / world (%d)", world);
  }
  for (int i = 0; i < world; ++i) {
    if (bar_flags[i] == nullptr || (reinterpret_cast<uintptr_t>(bar_flags[i]) & 3u)) {
      return fail(ARC_ERR_INVALID_ARGUMENT, "arc_a8w4_gemm_gather_sync: flag array %d is null or misaligned", i);
    }
  }
  if (flags & ~ARC_A8W4_STATIC_WEIGHTS) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_a8w4_gemm_gather_sync: unsupported flags 0x%x", flags);
  }
  if (outs == nullptr || rank < 0 || rank >= world) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_a8w4_gemm_gather_sync: bad outs / rank (%d)", rank);
  }
  for (int i = 0; i < world; ++i) {
    if (outs[i] == nullptr || !aligned16(outs[i])) {
      return fail(ARC_ERR_INVALID_ARGUMENT, "arc_a8w4_gemm_gather_sync: output %d is null or not 16-byte aligned", i);
    }
  }
  if (M <= 0 || M > static_cast<int>(kDecodeMaxM)) {
    return fail(ARC_ERR_UNSUPPORTED,
                "arc_a8w4_gemm_gather_sync: the fused all-gather covers decode batches (1 <= M <= %u, got %d)",
                kDecodeMaxM, M);
  }
  if (N <= 0 || N % 8 != 0) {
    return fail(ARC_ERR_UNSUPPORTED, "arc_a8w4_gemm_gather_sync: N (%d) must be a positive multiple of 8", N);
  }
  return a8w4_gemm(A, sa, Wp, sb, outs[rank] + size_t(rank) * N, M, N, K, 128, stream, nullptr, outs, world,
                   rank, flags, bar_flags);
}

int arc_ipc_export(const void* ptr, void* handle, uint64_t* offset) {
  g_last_error[0] = '\0';
  if (ptr == nullptr || handle == nullptr || offset == nullptr) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_ipc_export: null pointer");
  }
  using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static AddressRangeFn range_fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      range_fn = reinterpret_cast<AddressRangeFn>(f);
    }
  });
  if (range_fn == nullptr) return fail(ARC_ERR_CUDA, "cuMemGetAddressRange is unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range_fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_ipc_export: %p is not device memory", ptr);
  }
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return ARC_OK;
}

int arc_ipc_open(const void* handle, uint64_t offset, void** ptr, void** base) {
  g_last_error[0] = '\0';
  if (handle == nullptr || ptr == nullptr || base == nullptr) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_ipc_open: null pointer");
  }
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* b = nullptr;
  // Opened in the current device's context: its kernels are the ones that access the
  // mapping, and the flag enables peer access from it to the owner's GPU.
  const cudaError_t e = cudaIpcOpenMemHandle(&b, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  *base = b;
  *ptr = static_cast<uint8_t*>(b) + offset;
  return ARC_OK;
}

int arc_ipc_close(void* base) {
  g_last_error[0] = '\0';
  if (base == nullptr) return fail(ARC_ERR_INVALID_ARGUMENT, "arc_ipc_close: null pointer");
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
  return ARC_OK;
}

int arc_peer_barrier(uint32_t* const* flags, int world, int rank, cudaStream_t stream) {
  return arc_peer_barrier_ex(flags, world, rank, arcb::kWaitTimeoutNs, stream);
}

int arc_peer_barrier_ex(uint32_t* const* flags, int world, int rank, uint64_t timeout_ns, cudaStream_t stream) {
  g_last_error[0] = '\0';
  if (timeout_ns == 0 || timeout_ns > arcb::kWaitTimeoutNs) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_peer_barrier_ex: timeout must be in (0, 2 s]");
  }
  if (flags == nullptr || world < 1 || world > static_cast<int>(arcb::peer::kMaxPeers) || rank < 0 ||
      rank >= world) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_peer_barrier: bad flags / world (%d) / rank (%d)", world, rank);
  }
  arcb::peer::BarrierParams b = {};
  for (int i = 0; i < world; ++i) {
    if (flags[i] == nullptr || (reinterpret_cast<uintptr_t>(flags[i]) & 3u)) {
      return fail(ARC_ERR_INVALID_ARGUMENT, "arc_peer_barrier: flag array %d is null or misaligned", i);
    }
    b.flags[i] = flags[i];
  }
  b.world = static_cast<uint32_t>(world);
  b.rank = static_cast<uint32_t>(rank);
  b.timeout_ns = timeout_ns;
  int dev = 0;
  if (int st = current_device(&dev)) return st;
  const cudaError_t e = launch_ex(arcb::peer::peer_barrier_kernel, b, 1, 32, 0, 1, stream);
  if (e != cudaSuccess) return cuda_fail(e, "peer_barrier_kernel launch");
  return ARC_OK;
}

}  // extern "C"

namespace {

int a8w4_gemm(const int8_t* A, const float* sa, const uint8_t* Wp, const uint16_t* sb, uint16_t* C, int M,
              int N, int K, int group, cudaStream_t stream, int32_t* partials_dbg, uint16_t* const* outs,
              int world, int rank, uint32_t flags, uint32_t* const* bar_flags) {
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
  plan_a8w4(M, N, K, g_dev[dev].sms, g_dev[dev].max_clusters2, g_dev[dev].max_clusters4, &plan);
  const uint32_t BT = static_cast<uint32_t>(plan.token_tile);
  const uint32_t R = static_cast<uint32_t>(plan.weight_rows);
  const uint32_t G = static_cast<uint32_t>(K / group);
  cudaError_t e = cudaErrorInvalidConfiguration;
  if (M <= static_cast<int>(kDecodeMaxM)) {
    namespace D = arcb::a8w4dec;
    D::Params p;
    if (int st = encode_tokens_3d(&p.tm_tok, A, M, K, BT, D::kGps)) return st;
    // Packed weights [N][K/2] bytes; a box row is two K-groups (128 bytes), swizzled.
    if (int st = encode_2d(&p.tm_wp, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, Wp, K / 2, N, K / 2,
                           D::kGps * arcb::a8w4::kPackedRow, arcb::a8w4::kRows, CU_TENSOR_MAP_SWIZZLE_128B,
                           "Wp")) {
      return st;
    }
    const uint32_t S = static_cast<uint32_t>(plan.k_split);
    // The output: C [M][N], or with a fused all-gather this rank's [M][N] column window of
    // every rank's [M][world*N] output (row pitch world*N).
    const uint32_t ldo = outs != nullptr ? static_cast<uint32_t>(N * world) : static_cast<uint32_t>(N);
    if (int st = encode_2d(&p.tm_out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, C, N, M, ldo, R / S, BT,
                           CU_TENSOR_MAP_SWIZZLE_NONE, "C")) {
      return st;
    }
    p.peers = 0;
    if (outs != nullptr) {
      for (int i = 0; i < world; ++i) {
        if (int st = encode_2d(&p.tm_peer[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                               outs[i] + size_t(rank) * N, N, M, ldo, R / S, BT, CU_TENSOR_MAP_SWIZZLE_NONE,
                               "peer output")) {
          return st;
        }
      }
      p.peers = static_cast<uint32_t>(world);
    }
    p.bar_world = 0;
    p.bar_rank = 0;
    p.bar_timeout_ns = arcb::kWaitTimeoutNs;
    if (bar_flags != nullptr) {
      for (int i = 0; i < world; ++i) p.bar_flags[i] = bar_flags[i];
      p.bar_world = static_cast<uint32_t>(world);
      p.bar_rank = static_cast<uint32_t>(rank);
    }
    p.sa = sa;
    p.sb = sb;
    p.partials = partials_dbg;
    p.M = M;
    p.N = N;
    p.K = K;
    p.G = G;
    p.ldsb = G;
    p.S = S;
    p.num_items = ceil_div(N, R);
    p.split = (flags & ARC_A8W4_PREPACKED) ? 1u : 0u;
    p.static_weights = (flags & ARC_A8W4_STATIC_WEIGHTS) ? 1u : 0u;
    p.sb_vec = (G % 8 == 0 && aligned16(sb)) ? 1u : 0u;
    const uint32_t grid = static_cast<uint32_t>(plan.grid);
    const bool str = decode_stream(static_cast<int>(G), static_cast<int>(S), static_cast<int>(p.num_items),
                                   static_cast<int>(grid));
    const bool dump = partials_dbg != nullptr;
    e = BT == 16 ? launch_decode<16>(p, grid, S, str, dump, stream) : launch_decode<32>(p, grid, S, str, dump, stream);
    if (e != cudaSuccess) return cuda_fail(e, "gemm_a8w4_decode_kernel launch");
    return ARC_OK;
  }

  namespace Q = arcb::a8w4;
  Q::Params p;
  if (int st = encode_2d(&p.tm_tok, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, A, K, M, K, Q::kGroupK, BT,
                         CU_TENSOR_MAP_SWIZZLE_128B, "A")) {
    return st;
  }
  if (int st = encode_2d(&p.tm_wp, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, Wp, K / 2, N, K / 2,
                         Q::kPackedRow * Q::kGps, R, CU_TENSOR_MAP_SWIZZLE_128B, "Wp")) {
    return st;
  }
  p.sa = sa;
  p.sb = sb;
  p.out = C;
  p.partials = partials_dbg;
  p.M = M;
  p.N = N;
  p.K = K;
  p.G = G;
  p.ldsb = G;
  p.ldc = N;
  p.R = R;
  p.tiles_m = ceil_div(M, BT);
  p.tiles_n = ceil_div(N, R);
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.split = (flags & ARC_A8W4_PREPACKED) ? 1u : 0u;
  const uint32_t grid = static_cast<uint32_t>(plan.grid);
  if (BT == 64) {
    e = launch_ex(Q::gemm_a8w4_kernel<64, 1, 4>, p, grid, Q::Cfg<64, 1, 4>::kThreads,
                  a8w4_smem_bytes<64, 1, 4>(), 1, stream);
  } else {
    e = launch_ex(Q::gemm_a8w4_kernel<128, 2, 3>, p, grid, Q::Cfg<128, 2, 3>::kThreads,
                  a8w4_smem_bytes<128, 2, 3>(), 1, stream);
  }
  if (e != cudaSuccess) return cuda_fail(e, "gemm_a8w4_kernel launch");
  return ARC_OK;
}

}  // namespace

extern "C" {

int arc_fp8_fp4_gemm(const uint8_t* A, const float* sfa, const uint8_t* Wp, const float* sfw,
                     uint16_t* C, int M, int N, int K, cudaStream_t stream) {
  g_last_error[0] = '\0';
  return fp8fp4_gemm(A, sfa, Wp, sfw, C, M, N, K, nullptr, 0, stream);
}

int arc_fp8_fp4_workspace_bytes(int M, int N, int K, size_t* bytes) {
  g_last_error[0] = '\0';
  if (bytes == nullptr || M <= 0 || N <= 0 || K <= 0 || K % 128 != 0) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_fp8_fp4_workspace_bytes: bad argument");
  }
  int dev = 0;
  if (int st = current_device(&dev)) return st;
  int variant = 0;
  if (int st = choose_fp8fp4(dev, M, N, K, true, &variant)) return st;
  *bytes = variant == 0 ? fp8fp4_split_plan(dev, M, N, K).bytes : 0;
  return ARC_OK;
}

int arc_fp8_fp4_gemm_ws(const uint8_t* A, const float* sfa, const uint8_t* Wp, const float* sfw,
                        uint16_t* C, int M, int N, int K, void* workspace, size_t workspace_bytes,
                        cudaStream_t stream) {
  g_last_error[0] = '\0';
  if (workspace != nullptr && (reinterpret_cast<uintptr_t>(workspace) & 255u)) {
    return fail(ARC_ERR_UNSUPPORTED, "arc_fp8_fp4_gemm_ws: the workspace must be 256-byte aligned");
  }
  return fp8fp4_gemm(A, sfa, Wp, sfw, C, M, N, K, workspace, workspace_bytes, stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------------
// Allocation-free FP8 x FP4 GEMM. Some callers cannot hand this library a workspace:
// plugins whose host framework budgets every byte of device memory itself and offers
// the operator nothing beyond its input and output tensors, and hosts that must not call
// cudaMalloc on the request path (it can synchronise the device and its latency is not
// bounded). For them the K split's scratch lives in a fixed device array built into the
// library, 4 MiB on every GPU that loads it, held until the process exits. Shapes whose
// split would need more run without the split (no scratch).
// ---------------------------------------------------------------------------------
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;

struct NoAllocScratch {
  std::once_flag once;
  cudaError_t err = cudaSuccess;
  void* ptr = nullptr;  // device address of the array on this device
};
NoAllocScratch g_noalloc[kMaxDevices];

}  // namespace

// In host code this name is a host-side stand-in, not a device address; the device
// address comes from cudaGetSymbolAddress, once per device, with that device current.
static __device__ __align__(256) unsigned char g_fp8fp4_noalloc_scratch[kNoAllocScratchBytes];

extern "C" int arc_fp8_fp4_gemm_noalloc(const uint8_t* A, const float* sfa, const uint8_t* Wp,
                                        const float* sfw, uint16_t* C, int M, int N, int K,
                                        cudaStream_t stream) {
  g_last_error[0] = '\0';
  // Every argument is checked before anything is put on the stream.
  if (int st = fp8fp4_check(A, sfa, Wp, sfw, C, M, N, K)) return st;
  int dev = 0;
  if (int st = current_device(&dev)) return st;
  int variant = 0;
  if (int st = choose_fp8fp4(dev, M, N, K, aligned16(sfa), &variant)) return st;
  const size_t need = variant == 0 ? fp8fp4_split_plan(dev, M, N, K).bytes : 0;
  // No K split for this shape, or one whose partials would not fit the built-in array:
  // the unsplit kernel, which needs no scratch at all.
  if (need == 0 || need > kNoAllocScratchBytes) {
    return fp8fp4_gemm(A, sfa, Wp, sfw, C, M, N, K, nullptr, 0, stream);
  }
  NoAllocScratch& sc = g_noalloc[dev];
  std::call_once(sc.once, [&sc] {
    sc.err = cudaGetSymbolAddress(&sc.ptr, g_fp8fp4_noalloc_scratch);
    if (sc.err != cudaSuccess) cudaGetLastError();
  });
  if (sc.err != cudaSuccess || sc.ptr == nullptr) {
    return cuda_fail(sc.err != cudaSuccess ? sc.err : cudaErrorInvalidSymbol,
                     "arc_fp8_fp4_gemm_noalloc: cudaGetSymbolAddress of the built-in scratch");
  }
  // The array keeps the previous call's contents: the tile counters must start at zero.
  const cudaError_t e = cudaMemsetAsync(sc.ptr, 0, kSplitCounterBytes, stream);
  if (e != cudaSuccess) return cuda_fail(e, "arc_fp8_fp4_gemm_noalloc: clearing the scratch counters");
  return fp8fp4_gemm(A, sfa, Wp, sfw, C, M, N, K, sc.ptr, kNoAllocScratchBytes, stream);
}

namespace {

int fp8fp4_gemm(const uint8_t* A, const float* sfa, const uint8_t* Wp, const float* sfw, uint16_t* C,
                int M, int N, int K, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (int st = fp8fp4_check(A, sfa, Wp, sfw, C, M, N, K)) return st;
  int dev = 0;
  if (int st = current_device(&dev)) return st;
  namespace F = arcb::fp8fp4;
  const uint32_t sms = static_cast<uint32_t>(g_dev[dev].sms);
  // Kernel choice. CTA pairs on 256 x 256 tiles (half the shared-memory bytes per MAC)
  // when the pair tiles give every pair one and K % 512 == 0 (the token-scale tensor map
  // needs a 16-byte row pitch); else one CTA per 256-row weight tile when those fill the
  // SMs; else 128-row tiles (twice the CTAs, e.g. for decode batches).
  // ARC_FP8FP4_KERNEL=128|256|pair forces one (tests and tuning).
  const uint32_t max_pairs = static_cast<uint32_t>(g_dev[dev].max_fp8fp4_pairs);
  int variant = 0;
  if (int st = choose_fp8fp4(dev, M, N, K, aligned16(sfa), &variant)) return st;
  const uint32_t rows = variant == 1 ? 256u : 128u;
  if (variant == 2) {
    namespace FP = arcb::fp8fp4pair;
    FP::Params q;
    if (int st = encode_tokens_3d(&q.tm_tok, A, M, K, 128, 1)) return st;
    if (int st = encode_e2m1_3d(&q.tm_w, Wp, N, K, 128, 1)) return st;
    if (int st = encode_2d(&q.tm_sfw, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, sfw, K / 32, N, K / 32,
                           4 * FP::kBlk, 128, CU_TENSOR_MAP_SWIZZLE_128B, "sfw")) {
      return st;
    }
    if (int st = encode_2d(&q.tm_sfa, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, sfa, K / 128, M, K / 128,
                           FP::kBlk, 256, CU_TENSOR_MAP_SWIZZLE_NONE, "sfa")) {
      return st;
    }
    q.out = C;
    q.M = M;
    q.N = N;
    q.G = static_cast<uint32_t>(K) / F::kGroupK;
    q.ldc = N;
    q.tiles_m = ceil_div(M, FP::kTileT);
    q.tiles_n = ceil_div(N, FP::kTileW);
    q.num_tiles = q.tiles_m * q.tiles_n;
    const uint32_t grid = 2 * (q.num_tiles < max_pairs ? q.num_tiles : max_pairs);
    const cudaError_t e = launch_ex(FP::gemm_fp8fp4_pair_kernel, q, grid, FP::kThreads, FP::kSmemBytes, 2, stream);
    if (e != cudaSuccess) return cuda_fail(e, "gemm_fp8fp4_pair_kernel launch");
    return ARC_OK;
  }
  F::Params p;
  const uint32_t gps = rows == 256 ? F::Cfg<2>::kGps : F::Cfg<1>::kGps;
  if (int st = encode_tokens_3d(&p.tm_tok, A, M, K, F::kBT, gps)) return st;
  if (int st = encode_e2m1_3d(&p.tm_w, Wp, N, K, rows, gps)) return st;
  p.sfa = sfa;
  p.sfw = sfw;
  p.out = C;
  p.M = M;
  p.N = N;
  p.K = K;
  p.G = static_cast<uint32_t>(K) / F::kGroupK;
  p.ldsfa = static_cast<uint32_t>(K) / 128u;
  p.ldsfw = static_cast<uint32_t>(K) / 32u;
  p.ldc = N;
  p.tiles_m = ceil_div(M, F::kBT);
  p.tiles_n = ceil_div(N, rows);
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.S = 1;
  p.gs = p.G;
  p.ws = nullptr;
  p.counters = nullptr;
  if (variant == 0 && workspace != nullptr) {
    const SplitPlan sp = fp8fp4_split_plan(dev, M, N, K);
    if (sp.S > 1 && workspace_bytes >= sp.bytes) {
      p.S = sp.S;
      p.gs = sp.gs;
      p.counters = static_cast<uint32_t*>(workspace);
      p.ws = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + sp.partial_offset);
    }
  }
  const uint32_t items = p.num_tiles * p.S;
  const uint32_t grid = items < sms ? items : sms;
  const cudaError_t e =
      rows == 256 ? launch_ex(F::gemm_fp8fp4_kernel<2>, p, grid, F::kThreads, sizeof(F::Smem<2>) + 1024, 1, stream)
                  : launch_ex(F::gemm_fp8fp4_kernel<1>, p, grid, F::kThreads, sizeof(F::Smem<1>) + 1024, 1, stream);
  if (e != cudaSuccess) return cuda_fail(e, "gemm_fp8fp4_kernel launch");
  return ARC_OK;
}

}  // namespace

extern "C" {

int arc_quantize_int8(const void* x, int8_t* q, float* sa, int M, int K, int ldx, int ldq,
                      cudaStream_t stream) {
  g_last_error[0] = '\0';
  if (x == nullptr || q == nullptr || sa == nullptr) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_quantize_int8: null pointer");
  }
  if (M <= 0 || K <= 0 || ldx < K || ldq < K) {
    return fail(ARC_ERR_INVALID_ARGUMENT,
                "arc_quantize_int8: need M, K >= 1, ldx >= K, ldq >= K (M=%d K=%d ldx=%d ldq=%d)", M,
                K, ldx, ldq);
  }
  if ((reinterpret_cast<uintptr_t>(x) & 1u) || (reinterpret_cast<uintptr_t>(sa) & 3u)) {
    return fail(ARC_ERR_UNSUPPORTED, "arc_quantize_int8: x must be 2-byte and sa 4-byte aligned");
  }
  int dev = 0;
  if (int st = current_device(&dev)) return st;
  arcb::quant::Params p;
  p.x = static_cast<const uint16_t*>(x);
  p.q = q;
  p.sa = sa;
  p.M = static_cast<uint32_t>(M);
  p.K = static_cast<uint32_t>(K);
  p.ldx = static_cast<uint32_t>(ldx);
  p.ldq = static_cast<uint32_t>(ldq);
  p.vec = (K % 8 == 0 && ldx % 8 == 0 && ldq % 8 == 0 && aligned16(x) &&
           (reinterpret_cast<uintptr_t>(q) & 7u) == 0u)
              ? 1u
              : 0u;
  const cudaError_t e = launch_ex(arcb::quant::quantize_int8_per_token_kernel, p,
                                  static_cast<uint32_t>(M), arcb::quant::kThreads, 0, 1, stream);
  if (e != cudaSuccess) return cuda_fail(e, "quantize_int8_per_token_kernel launch");
  return ARC_OK;
}

int arc_probe_attach(void* buffer, size_t bytes) {
#if defined(ARC_PROBE)
  if (buffer != nullptr && bytes < sizeof(unsigned long long) * arcb::kProbeSlots) {
    return fail(ARC_ERR_INVALID_ARGUMENT, "arc_probe_attach: buffer smaller than one CTA's stamps");
  }
  unsigned long long* ptr = static_cast<unsigned long long*>(buffer);
  const cudaError_t e = cudaMemcpyToSymbol(arcb::g_arc_probe, &ptr, sizeof(ptr));
  if (e != cudaSuccess) return cuda_fail(e, "arc_probe_attach");
  return ARC_OK;
#else
  (void)buffer;
  (void)bytes;
  return fail(ARC_ERR_UNSUPPORTED, "arc_probe_attach: library built without ARC_PROBE");
#endif
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
