// Shared helpers for the mzoo_b200 sm_100a kernels: status codes, error strings,
// launch checks, bit-exact scalar rounding helpers and small PTX wrappers.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "../../include/mzb200.h"

namespace mzb {

// Thread-local message of the last failing C-ABI call (read through mzb_last_error).
void set_error(const char* fmt, ...);

#define MZB_REQUIRE(cond, code, ...)          \
  do {                                        \
    if (!(cond)) {                            \
      ::mzb::set_error(__VA_ARGS__);          \
      return (code);                          \
    }                                         \
  } while (0)

// Launch-error check after a kernel launch (configuration errors only; never syncs).
inline int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
    return MZB_ERR_LAUNCH;
  }
  return MZB_OK;
}

inline int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// ---------------------------------------------------------------- element access

template <int DT> struct Elem;
template <> struct Elem<MZB_F32> {
  using T = float;
  static __device__ __forceinline__ float load(const T v) { return v; }
  static __device__ __forceinline__ T store(float v) { return v; }
};
template <> struct Elem<MZB_BF16> {
  using T = __nv_bfloat16;
  static __device__ __forceinline__ float load(const T v) { return __bfloat162float(v); }
  static __device__ __forceinline__ T store(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Elem<MZB_F16> {
  using T = __half;
  static __device__ __forceinline__ float load(const T v) { return __half2float(v); }
  static __device__ __forceinline__ T store(float v) { return __float2half_rn(v); }
};

// ---------------------------------------------------------------- exact rounding helpers

// 2^ceil(log2 t) through the exponent bits (exponent - 127 + (mantissa != 0)), the
// ue8m0 scale rounding of mzoo's `_pow2_ceil_scale`.
__device__ __forceinline__ float pow2_ceil(float t) {
  uint32_t b = __float_as_uint(t);
  int e = int((b >> 23) & 0xFF) - 127 + ((b & 0x7FFFFF) != 0);
  // 2^e for e in [-149, 128]; build it exactly (subnormal range included)
  if (e >= -126) return __uint_as_float(uint32_t(e + 127) << 23);
  return __uint_as_float(1u << (e + 149));
}

// torch.clamp semantics: NaN passes through.
__device__ __forceinline__ float clamp_nan(float v, float lo, float hi) {
  return v < lo ? lo : (v > hi ? hi : v);
}

// float -> e4m3fn -> float with torch's cast semantics: round-to-nearest-even, NaN for
// |v| > 464 (values in (464, 480) round onto the NaN code, >= 480 saturate to NaN).
__device__ __forceinline__ float e4m3_round(float v) {
  float a = fabsf(v);
  if (!(a <= 464.0f)) return __uint_as_float(0x7fffffffu);
  __nv_fp8_storage_t q = __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
  __half_raw h = __nv_cvt_fp8_to_halfraw(q, __NV_E4M3);
  return __half2float(__half(h));
}

__device__ __forceinline__ float e4m3_to_float(uint8_t q) {
  __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)q, __NV_E4M3);
  return __half2float(__half(h));
}

// e2m1 code (sign in bit 3) of a pre-clamped value, mzoo's `_e2m1_codes` thresholds:
// ties at 0.25/1.25/2.5/5.0 round down, at 0.75/1.75/3.5 round up.
__device__ __forceinline__ float e2m1_value(float q) {
  float m = fabsf(q);
  float v = (m > 5.0f) ? 6.0f : (m >= 3.5f) ? 4.0f : (m > 2.5f) ? 3.0f : (m >= 1.75f) ? 2.0f
          : (m > 1.25f) ? 1.5f : (m >= 0.75f) ? 1.0f : (m > 0.25f) ? 0.5f : 0.0f;
  // code 8 (negative zero) maps to +0.0 in mzoo's table
  return (signbit(q) && v != 0.0f) ? -v : v;
}

// Two values onto the e2m1 grid {0, .5, 1, 1.5, 2, 3, 4, 6} with the hardware conversion
// (round to nearest, ties to the even code -- the same choices as the thresholds above: ties
// at 0.25/1.25/2.5/5.0 go to codes 0/2/4/6 below, at 0.75/1.75/3.5 to codes 2/4/6 above --
// saturating at 6), then back through f16x2.  mzoo's table gives +0.0 for -0 and its
// thresholds give 0 for NaN; both are applied explicitly.  Inputs are pre-clamped to [-6, 6].
__device__ __forceinline__ void e2m1_value2(float q0, float q1, float& r0, float& r1) {
  uint32_t h2;
  asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %2, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}"
      : "=r"(h2)
      : "f"(q0), "f"(q1));
  const __half2 hh = *reinterpret_cast<const __half2*>(&h2);
  const float2 f = __half22float2(hh);
  r0 = isnan(q0) ? 0.0f : __fadd_rn(f.x, 0.0f);
  r1 = isnan(q1) ? 0.0f : __fadd_rn(f.y, 0.0f);
}

// ---------------------------------------------------------------- PTX helpers

// 2^x on the SFU (ex2.approx, relative error ~2^-22; -inf -> +0).  Softmax numerators only.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (sm_100 FFMA2): two independent fp32 FMAs per instruction, each
// rounded exactly as fmaf.
__device__ __forceinline__ uint64_t pack_f32x2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ uint64_t ffma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ float2 unpack_f32x2(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

}  // namespace mzb
