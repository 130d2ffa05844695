// Quantised KV-cache storage of the DeepSeek-V4.1 attention: pack bf16 latents into the
// cache formats and unpack them back to the bf16 values the attention kernels consume.
//
// Formats (src/mzoo/layers/attn/csa_attn/README.md:215-235; tickets/0010-csa2-fp-cache.md):
//   window cache: e4m3 codes [rows, D] + one ue8m0 scale byte per 32 channels [rows, D/32]
//                 (the biased exponent: scale = 2^(byte - 127));
//   main cache:   e2m1 codes packed two per byte, low nibble first [rows, D/2] + one e4m3
//                 scale byte per 16 channels [rows, D/16].
// The values are bit-identical to the model's fake quantisers
// (archs/dsv4/modeling_deepseek_v41.py:359-402, :668-683): `_fake_quant_fp8_block(x, 32)`
// and `_fake_quant_fp4_block(x, 16, e4m3_scales=True)` -- unpack(pack(x)) equals them
// exactly, scales included (clamp floors, e2m1 ties, -0 -> +0 on dequant).
//
// HBM-bound: one pass over x and the codes.  Pack: one lane per channel, the block amax by
// xor-shuffles inside the warp (32-channel blocks: a warp, 16-channel blocks: half a warp).
#include "common.cuh"

namespace mzb {
namespace kvc {

struct Args {
  const __nv_bfloat16* x;
  uint8_t* codes;        // pack output / unpack input
  uint8_t* scales;
  __nv_bfloat16* out;    // unpack output
  long long rows;
  int D;
};

// torch.amax semantics for the block max: a NaN anywhere makes it NaN
__device__ __forceinline__ float nan_max(float a, float b) {
  return (isnan(a) || isnan(b)) ? __uint_as_float(0x7fffffffu) : fmaxf(a, b);
}

// 2^(byte - 127), exactly (byte 0 is the subnormal 2^-127)
__device__ __forceinline__ float ue8m0_value(uint32_t byte) {
  return byte ? __uint_as_float(byte << 23) : __uint_as_float(1u << 22);
}

// ---------------------------------------------------------------- window cache (fp8 / ue8m0 / 32)

__global__ void pack_fp8_kernel(Args a) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // element index
  const long long n = a.rows * a.D;
  const bool own = i < n;
  const float v = own ? __bfloat162float(a.x[i]) : 0.0f;
  float am = fabsf(v);
  for (int o = 16; o; o >>= 1) am = nan_max(am, __shfl_xor_sync(0xffffffffu, am, o));
  if (!own) return;
  // `_pow2_ceil_scale(amax.clamp_min(1e-4) * (1 / 448))`: 2^(exponent field - 127 + (mantissa != 0))
  const float t = __fmul_rn(am < 1e-4f ? 1e-4f : am, 1.0f / 448.0f);
  const uint32_t b = __float_as_uint(t);
  const int ebyte = int((b >> 23) & 0xFF) + ((b & 0x7FFFFF) ? 1 : 0);  // k + 127
  const float s = pow2_ceil(t);
  const float q = clamp_nan(__fdiv_rn(v, s), -448.0f, 448.0f);
  a.codes[i] = uint8_t(__nv_cvt_float_to_fp8(q, __NV_SATFINITE, __NV_E4M3));
  if ((threadIdx.x & 31) == 0) a.scales[i >> 5] = uint8_t(ebyte);
}

__global__ void unpack_fp8_kernel(Args a) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.rows * a.D) return;
  const float s = ue8m0_value(a.scales[i >> 5]);
  a.out[i] = __float2bfloat16_rn(__fmul_rn(e4m3_to_float(a.codes[i]), s));
}

// ---------------------------------------------------------------- main cache (e2m1 / e4m3 / 16)

// e2m1 code of a pre-clamped value (sign in bit 3), `_e2m1_codes`' thresholds: ties at
// 0.25 / 1.25 / 2.5 / 5.0 round down, at 0.75 / 1.75 / 3.5 round up; NaN -> 0 | sign.
__device__ __forceinline__ uint32_t e2m1_code(float q) {
  const float m = fabsf(q);
  const uint32_t c = (m > 5.0f) ? 7u : (m >= 3.5f) ? 6u : (m > 2.5f) ? 5u : (m >= 1.75f) ? 4u
                   : (m > 1.25f) ? 3u : (m >= 0.75f) ? 2u : (m > 0.25f) ? 1u : 0u;
  return c | (signbit(q) ? 8u : 0u);
}

__global__ void pack_fp4_kernel(Args a) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long n = a.rows * a.D;
  const bool own = i < n;
  const float v = own ? __bfloat162float(a.x[i]) : 0.0f;
  float am = fabsf(v);
  for (int o = 8; o; o >>= 1) am = nan_max(am, __shfl_xor_sync(0xffffffffu, am, o));  // 16-lane blocks
  // `(amax.clamp_min(6 * 2**-9) / 6).to(float8_e4m3fn)`
  const float t = __fdiv_rn(am < 6.0f * 0x1p-9f ? 6.0f * 0x1p-9f : am, 6.0f);
  const float s = e4m3_round(t);
  const uint32_t code = e2m1_code(clamp_nan(__fdiv_rn(v, s), -6.0f, 6.0f));
  const uint32_t hi = __shfl_down_sync(0xffffffffu, code, 1);
  if (!own) return;
  if ((i & 1) == 0) a.codes[i >> 1] = uint8_t(code | (hi << 4));
  if ((threadIdx.x & 15) == 0)
    a.scales[i >> 4] = isnan(s) ? uint8_t(0x7F) : uint8_t(__nv_cvt_float_to_fp8(t, __NV_SATFINITE, __NV_E4M3));
}

__global__ void unpack_fp4_kernel(Args a) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.rows * a.D) return;
  const uint32_t byte = a.codes[i >> 1];
  const uint32_t code = (i & 1) ? (byte >> 4) : (byte & 0xF);
  // mzoo's e2m1 table; code 8 (negative zero) is +0.0 in it
  const float mag = (code & 7u) == 0 ? 0.0f
                  : (code & 7u) == 1 ? 0.5f : (code & 7u) == 2 ? 1.0f : (code & 7u) == 3 ? 1.5f
                  : (code & 7u) == 4 ? 2.0f : (code & 7u) == 5 ? 3.0f : (code & 7u) == 6 ? 4.0f : 6.0f;
  const float val = (code & 8u) && mag != 0.0f ? -mag : mag;
  a.out[i] = __float2bfloat16_rn(__fmul_rn(val, e4m3_to_float(a.scales[i >> 4])));
}

static int launch(void (*k)(Args), const Args& a, const char* what, cudaStream_t st) {
  const long long n = a.rows * a.D;
  if (n == 0) return MZB_OK;
  k<<<unsigned((n + 255) / 256), 256, 0, st>>>(a);
  return launch_status(what);
}

}  // namespace kvc
}  // namespace mzb

using namespace mzb;

extern "C" int mzb_kv_pack_fp8(const void* x, uint8_t* codes, uint8_t* scales, int64_t rows, int D, void* stream) {
  MZB_REQUIRE(rows >= 0 && D > 0 && D % 32 == 0, MZB_ERR_SHAPE, "kv_pack_fp8: D=%d must be a multiple of 32", D);
  kvc::Args a{static_cast<const __nv_bfloat16*>(x), codes, scales, nullptr, rows, D};
  return kvc::launch(kvc::pack_fp8_kernel, a, "kv_pack_fp8", static_cast<cudaStream_t>(stream));
}

extern "C" int mzb_kv_unpack_fp8(const uint8_t* codes, const uint8_t* scales, void* out, int64_t rows, int D,
                                 void* stream) {
  MZB_REQUIRE(rows >= 0 && D > 0 && D % 32 == 0, MZB_ERR_SHAPE, "kv_unpack_fp8: D=%d must be a multiple of 32", D);
  kvc::Args a{nullptr, const_cast<uint8_t*>(codes), const_cast<uint8_t*>(scales), static_cast<__nv_bfloat16*>(out),
              rows, D};
  return kvc::launch(kvc::unpack_fp8_kernel, a, "kv_unpack_fp8", static_cast<cudaStream_t>(stream));
}

extern "C" int mzb_kv_pack_fp4(const void* x, uint8_t* codes, uint8_t* scales, int64_t rows, int D, void* stream) {
  MZB_REQUIRE(rows >= 0 && D > 0 && D % 16 == 0, MZB_ERR_SHAPE, "kv_pack_fp4: D=%d must be a multiple of 16", D);
  kvc::Args a{static_cast<const __nv_bfloat16*>(x), codes, scales, nullptr, rows, D};
  return kvc::launch(kvc::pack_fp4_kernel, a, "kv_pack_fp4", static_cast<cudaStream_t>(stream));
}

extern "C" int mzb_kv_unpack_fp4(const uint8_t* codes, const uint8_t* scales, void* out, int64_t rows, int D,
                                 void* stream) {
  MZB_REQUIRE(rows >= 0 && D > 0 && D % 16 == 0, MZB_ERR_SHAPE, "kv_unpack_fp4: D=%d must be a multiple of 16", D);
  kvc::Args a{nullptr, const_cast<uint8_t*>(codes), const_cast<uint8_t*>(scales), static_cast<__nv_bfloat16*>(out),
              rows, D};
  return kvc::launch(kvc::unpack_fp4_kernel, a, "kv_unpack_fp4", static_cast<cudaStream_t>(stream));
}
