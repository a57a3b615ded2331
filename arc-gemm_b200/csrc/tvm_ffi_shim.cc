// tvm_ffi_shim.cc — TVM-FFI typed exports of the GEMMs (libarcb200_tvm_ffi.so).
//
// The reference binds its GEMM as a TVM-FFI typed function: arc/mm.py:30 defines
// `void matmul(TensorView a, TensorView b, TensorView out)`, arc/mm.py:48 exports it with
// TVM_FFI_DLL_EXPORT_TYPED_FUNC, and arc/mm.py:38 launches on the stream that
// TVMFFIEnvGetStream returns for the output's device. This file gives this library the
// same binding over its C ABI (include/arc_b200.h), so a caller that loads the
// reference's module with tvm_ffi.load_module can load this one instead:
//
//   matmul(a, b, out)                       bf16 a [M, K], b [N, K], out [M, N]
//   a8w4_matmul(a, sa, w, sb, out)          the int8 x int4 recipe: a int8 [M, K],
//                                           sa f32 [M], w uint8 [N, K/2], sb bf16
//                                           [N, K/128], out bf16 [M, N]
//   fp8_fp4_gemm_nt(a, sfa, w, sfw, out)    the reference's A8W4 recipe (tests/a8w4.py:48)
//
// Every tensor must be a contiguous CUDA tensor of the stated type on one device. The
// call makes that device current, launches on its TVM-FFI environment stream and
// returns without synchronising. A bad argument or a nonzero arc_status_t raises (the
// reference exits the process on CUDA errors, arc/include/common.cuh:8-28).
#include <cuda_runtime_api.h>

#include <tvm/ffi/container/tensor.h>
#include <tvm/ffi/error.h>
#include <tvm/ffi/extra/c_env_api.h>
#include <tvm/ffi/function.h>

#include "arc_b200.h"

namespace arc_tvm {

using tvm::ffi::TensorView;

void expect(const TensorView& t, const char* name, uint8_t code, uint8_t bits, int ndim, int device_id) {
  if (t.device().device_type != kDLCUDA) {
    TVM_FFI_THROW(ValueError) << name << " must be a CUDA tensor (there is no CPU path)";
  }
  if (device_id >= 0 && t.device().device_id != device_id) {
    TVM_FFI_THROW(ValueError) << name << " is on CUDA device " << t.device().device_id << ", expected "
                              << device_id;
  }
  if (t.dtype().code != code || t.dtype().bits != bits || t.dtype().lanes != 1) {
    TVM_FFI_THROW(TypeError) << name << " has the wrong dtype";
  }
  if (t.ndim() != ndim) TVM_FFI_THROW(ValueError) << name << " must have " << ndim << " dimensions";
  int64_t expect_stride = 1;
  for (int d = ndim - 1; d >= 0; --d) {
    if (t.size(d) > 1 && t.stride(d) != expect_stride) {
      TVM_FFI_THROW(ValueError) << name << " must be contiguous";
    }
    expect_stride *= t.size(d);
  }
}

void* ptr(const TensorView& t) { return static_cast<char*>(t.data_ptr()) + t.byte_offset(); }

void check(int status, const char* what) {
  if (status != ARC_OK) {
    TVM_FFI_THROW(RuntimeError) << what << ": " << arc_status_string(status) << ": " << arc_last_error();
  }
}

// Makes the tensors' device current for the duration of a call.
class DeviceScope {
 public:
  explicit DeviceScope(int device) {
    if (cudaGetDevice(&prev_) != cudaSuccess) {
      cudaGetLastError();
      TVM_FFI_THROW(RuntimeError) << "cudaGetDevice failed";
    }
    if (prev_ != device && cudaSetDevice(device) != cudaSuccess) {
      cudaGetLastError();
      TVM_FFI_THROW(RuntimeError) << "cudaSetDevice(" << device << ") failed";
    }
  }
  ~DeviceScope() { cudaSetDevice(prev_); }

 private:
  int prev_ = 0;
};

cudaStream_t stream_of(const TensorView& t) {
  return static_cast<cudaStream_t>(TVMFFIEnvGetStream(t.device().device_type, t.device().device_id));
}

int as_int(int64_t v, const char* what) {
  if (v <= 0 || v > INT32_MAX) TVM_FFI_THROW(ValueError) << what << " out of range";
  return static_cast<int>(v);
}

void matmul(TensorView a, TensorView b, TensorView out) {
  const int dev = out.device().device_id;
  expect(a, "a", kDLBfloat, 16, 2, dev);
  expect(b, "b", kDLBfloat, 16, 2, dev);
  expect(out, "out", kDLBfloat, 16, 2, dev);
  const int M = as_int(a.size(0), "M"), K = as_int(a.size(1), "K"), N = as_int(b.size(0), "N");
  if (b.size(1) != K) TVM_FFI_THROW(ValueError) << "Inner dimensions must match";
  if (out.size(0) != M || out.size(1) != N) TVM_FFI_THROW(ValueError) << "out must be [M, N]";
  DeviceScope scope(dev);
  check(arc_matmul_bf16(ptr(a), ptr(b), ptr(out), M, N, K, K, K, N, stream_of(out)), "matmul");
}

void a8w4_matmul(TensorView a, TensorView sa, TensorView w, TensorView sb, TensorView out) {
  const int dev = out.device().device_id;
  expect(a, "a", kDLInt, 8, 2, dev);
  expect(sa, "sa", kDLFloat, 32, 1, dev);
  expect(w, "w", kDLUInt, 8, 2, dev);
  expect(sb, "sb", kDLBfloat, 16, 2, dev);
  expect(out, "out", kDLBfloat, 16, 2, dev);
  const int M = as_int(a.size(0), "M"), K = as_int(a.size(1), "K"), N = as_int(w.size(0), "N");
  if (w.size(1) * 2 != K) TVM_FFI_THROW(ValueError) << "Inner dimensions must match: w must be [N, K/2]";
  if (K % 128 != 0) TVM_FFI_THROW(ValueError) << "K must be a multiple of 128";
  if (sa.size(0) != M || sb.size(0) != N || sb.size(1) != K / 128) {
    TVM_FFI_THROW(ValueError) << "sa must be [M] and sb [N, K/128]";
  }
  if (out.size(0) != M || out.size(1) != N) TVM_FFI_THROW(ValueError) << "out must be [M, N]";
  DeviceScope scope(dev);
  check(arc_a8w4_gemm(static_cast<const int8_t*>(ptr(a)), static_cast<const float*>(ptr(sa)),
                      static_cast<const uint8_t*>(ptr(w)), static_cast<const uint16_t*>(ptr(sb)),
                      static_cast<uint16_t*>(ptr(out)), M, N, K, 128, stream_of(out), nullptr),
        "a8w4_matmul");
}

void fp8_fp4_gemm_nt(TensorView a, TensorView sfa, TensorView w, TensorView sfw, TensorView out) {
  const int dev = out.device().device_id;
  expect(a, "a", kDLFloat8_e4m3fn, 8, 2, dev);
  expect(sfa, "sfa", kDLFloat, 32, 2, dev);
  expect(w, "w", kDLUInt, 8, 2, dev);
  expect(sfw, "sfw", kDLFloat, 32, 2, dev);
  expect(out, "out", kDLBfloat, 16, 2, dev);
  const int M = as_int(a.size(0), "M"), K = as_int(a.size(1), "K"), N = as_int(w.size(0), "N");
  if (w.size(1) * 2 != K) TVM_FFI_THROW(ValueError) << "Inner dimensions must match: w must be [N, K/2]";
  if (K % 128 != 0) TVM_FFI_THROW(ValueError) << "K must be a multiple of 128";
  if (sfa.size(0) != M || sfa.size(1) != K / 128 || sfw.size(0) != N || sfw.size(1) != K / 32) {
    TVM_FFI_THROW(ValueError) << "sfa must be [M, K/128] and sfw [N, K/32]";
  }
  if (out.size(0) != M || out.size(1) != N) TVM_FFI_THROW(ValueError) << "out must be [M, N]";
  DeviceScope scope(dev);
  check(arc_fp8_fp4_gemm(static_cast<const uint8_t*>(ptr(a)), static_cast<const float*>(ptr(sfa)),
                         static_cast<const uint8_t*>(ptr(w)), static_cast<const float*>(ptr(sfw)),
                         static_cast<uint16_t*>(ptr(out)), M, N, K, stream_of(out)),
        "fp8_fp4_gemm_nt");
}

}  // namespace arc_tvm

TVM_FFI_DLL_EXPORT_TYPED_FUNC(matmul, arc_tvm::matmul);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(a8w4_matmul, arc_tvm::a8w4_matmul);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(fp8_fp4_gemm_nt, arc_tvm::fp8_fp4_gemm_nt);
