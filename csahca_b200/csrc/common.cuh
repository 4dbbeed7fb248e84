// Shared device helpers for the csahca_b200 kernels (sm_100a only).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/csahca_b200.h"

namespace csahca {

// ---------------------------------------------------------------- element types
template <typename T> struct Elem;
template <> struct Elem<float> {
  static constexpr int kVec = 4;  // elements per 16-byte vector
  __device__ static __forceinline__ void widen(const uint4& v, float* f) {
    f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
  }
  __device__ static __forceinline__ float to_f(float x) { return x; }
  __device__ static __forceinline__ float from_f(float x) { return x; }
};
template <> struct Elem<__half> {
  static constexpr int kVec = 8;
  __device__ static __forceinline__ void widen(const uint4& v, float* f) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) { float2 t = __half22float2(h[i]); f[2 * i] = t.x; f[2 * i + 1] = t.y; }
  }
  __device__ static __forceinline__ float to_f(__half x) { return __half2float(x); }
  __device__ static __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};
template <> struct Elem<__nv_bfloat16> {
  static constexpr int kVec = 8;
  __device__ static __forceinline__ void widen(const uint4& v, float* f) {
    // bf16 -> f32 is a 16-bit shift of the bit pattern (exact).
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
  __device__ static __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ static __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

// Row geometry of a [.., D] row split in 16-byte vectors across a warp.
//   kNV  vectors per row, kLPT lanes sharing one row, kTPS rows per warp step,
//   kVPL vectors per lane per row.
template <typename T, int D>
struct RowGeom {
  static constexpr int kVec = Elem<T>::kVec;
  static constexpr int kNV = D / kVec;
  static_assert(D % kVec == 0, "row must be a whole number of 16-byte vectors");
  static_assert(kNV <= 32 ? (32 % kNV == 0) : (kNV % 32 == 0), "unsupported head_dim");
  static constexpr int kLPT = kNV <= 32 ? kNV : 32;
  static constexpr int kTPS = 32 / kLPT;
  static constexpr int kVPL = kNV <= 32 ? 1 : kNV / 32;
  static constexpr int kFPL = kVPL * kVec;  // floats per lane
};

// ---------------------------------------------------------------- memory helpers
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

__device__ __forceinline__ float warp_sum_xor(float v, int from, int to) {
  for (int o = from; o < to; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Order-preserving 32-bit key of a float (larger float -> larger key; NaN above +inf).
__device__ __forceinline__ uint32_t float_order_key(float f) {
  uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// ---------------------------------------------------------------- device error word
// Kernels receive a pointer to the per-device error word (owned by capi.cu) and
// set it, instead of trapping, when a bounded wait gives up or an index falls
// outside its buffer; csahca_read_device_error() reads and clears it.
enum DeviceError : int {
  kErrNone = 0,
  kErrWaitTimeout = 1,
  kErrSlotOutOfRange = 2,
};

__device__ __forceinline__ void report_device_error(int* err, int code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

constexpr float kLog2e = 1.4426950408889634f;

}  // namespace csahca

// ---------------------------------------------------------------- host helpers
#define CSAHCA_RETURN_IF_CUDA(expr)                                   \
  do {                                                                \
    cudaError_t _e = (expr);                                          \
    if (_e != cudaSuccess) return csahca_set_cuda_error(_e, #expr);   \
  } while (0)

int csahca_set_cuda_error(cudaError_t e, const char* what);
int csahca_set_arg_error(const char* msg);
int csahca_set_unsupported(const char* msg);
// Device address of the current device's error word (nullptr if unavailable).
int* csahca_device_error_ptr();
// Number of SMs of the current device (cached per device).
int csahca_num_sms();
