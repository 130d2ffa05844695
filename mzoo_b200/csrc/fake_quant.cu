// Fake-quant (quantise -> dequantise) kernels, bit-exact with mzoo's torch rules.
//
// Reference: src/mzoo/archs/owlet1/quant.py:49-86 (`_fake_quant_fp4_block`,
// `_fake_quant_fp8_block`), identical to src/mzoo/archs/dsv4/modeling_deepseek_v41.py:343-402,
// 613-630. Plus the two rules BASELINE config 5 asks for (OCP MXFP4 floor-scale and FP8
// per-tile absmax), which mzoo does not implement.
//
// HBM-bound, one pass: every thread owns one 16-byte vector of one block; the G threads of
// a block (G = block / vector elements, a power of two <= 32, always inside one warp)
// reduce the block's amax with xor-shuffles, then each thread rounds its own elements.
// The grid is a multiple of the SM count and walks the tensor in warp-uniform strides so
// every shuffle has its full warp.
#include "common.cuh"

namespace mzb {

enum Fp4Rule { FP4_UE8M0 = 0, FP4_E4M3 = 1, FP4_OCP = 2 };
enum Fp8Rule { FP8_UE8M0 = 0, FP8_ABSMAX = 1 };

// The rule is a template parameter: every per-element choice below is made at compile time.
template <int RULE>
struct Fp4Op {
  static constexpr int rule = RULE;
  __device__ __forceinline__ float scale(float amax) const {
    if (rule == FP4_E4M3) {
      return e4m3_round(__fdiv_rn(fmaxf(amax, 6.0f * 0x1p-9f), 6.0f));
    } else if (rule == FP4_UE8M0) {
      return pow2_ceil(__fmul_rn(fmaxf(amax, 6.0f * 0x1p-126f), 1.0f / 6.0f));
    } else {  // OCP MX: 2^(floor(log2 amax) - 2), e8m0 exponent clamped to [-127, 127]
      if (!(amax > 0.0f)) return 1.0f;
      uint32_t b = __float_as_uint(amax);
      int ef = int((b >> 23) & 0xFF);
      int fl = ef > 0 ? ef - 127 : (31 - __clz(int(b & 0x7FFFFF))) - 149;
      int e = max(-127, min(127, fl - 2));
      return e >= -126 ? __uint_as_float(uint32_t(e + 127) << 23) : __uint_as_float(1u << (e + 149));
    }
  }
  // Power-of-two scales (ue8m0 and OCP rules, 2^-127..2^127): 1/s is an exactly
  // representable float, so x * (1/s) is the same correctly rounded value as x / s.
  __device__ __forceinline__ bool pow2() const { return rule != FP4_E4M3; }
  __device__ __forceinline__ float apply(float x, float s, float inv) const {
    float q = clamp_nan(pow2() ? __fmul_rn(x, inv) : __fdiv_rn(x, s), -6.0f, 6.0f);
    return __fmul_rn(e2m1_value(q), s);
  }
  // The clamp to [-6, 6] of `apply` is left to the conversion: `satfinite` saturates
  // |q| > 6 (infinities included) to the largest code, 6, which is what rounding the
  // clamped value gives, and a NaN q is mapped to 0 from q itself.
  __device__ __forceinline__ void apply2(float x0, float x1, float s, float inv, float& r0, float& r1) const {
    const float q0 = pow2() ? __fmul_rn(x0, inv) : __fdiv_rn(x0, s);
    const float q1 = pow2() ? __fmul_rn(x1, inv) : __fdiv_rn(x1, s);
    float v0, v1;
    e2m1_value2(q0, q1, v0, v1);
    r0 = __fmul_rn(v0, s);
    r1 = __fmul_rn(v1, s);
  }
};

template <int RULE>
struct Fp8Op {
  static constexpr int rule = RULE;
  __device__ __forceinline__ float scale(float amax) const {
    if (rule == FP8_UE8M0) return pow2_ceil(__fmul_rn(fmaxf(amax, 1e-4f), 1.0f / 448.0f));
    float s = __fdiv_rn(amax, 448.0f);
    return s > 0.0f ? s : 1.0f;
  }
  __device__ __forceinline__ bool pow2() const { return rule == FP8_UE8M0; }
  __device__ __forceinline__ float apply(float x, float s, float inv) const {
    float q = clamp_nan(pow2() ? __fmul_rn(x, inv) : __fdiv_rn(x, s), -448.0f, 448.0f);
    return __fmul_rn(e4m3_round(q), s);
  }
  __device__ __forceinline__ void apply2(float x0, float x1, float s, float inv, float& r0, float& r1) const {
    r0 = apply(x0, s, inv);
    r1 = apply(x1, s, inv);
  }
};

// NaN-propagating |x| max, like torch's amax (a NaN anywhere makes the block amax NaN).
__device__ __forceinline__ float amax_step(float a, float v) {
  return (isnan(a) || isnan(v)) ? __uint_as_float(0x7fffffffu) : fmaxf(a, fabsf(v));
}

// The same over eight bf16 values in their packed form: |x| by clearing the sign bits, then
// NaN-propagating bf16x2 maxima (bf16 -> f32 is exact, so the maximum is the same value);
// three packed instructions in place of eight conversions and eight scalar steps.
__device__ __forceinline__ float bf16x8_amax(const uint4 w) {
  uint32_t m;
  asm("{\n\t.reg .b32 a, b, c, d;\n\t"
      "and.b32 a, %1, 0x7FFF7FFF;\n\t"
      "and.b32 b, %2, 0x7FFF7FFF;\n\t"
      "and.b32 c, %3, 0x7FFF7FFF;\n\t"
      "and.b32 d, %4, 0x7FFF7FFF;\n\t"
      "max.NaN.bf16x2 a, a, b;\n\t"
      "max.NaN.bf16x2 c, c, d;\n\t"
      "max.NaN.bf16x2 %0, a, c;\n\t}"
      : "=r"(m)
      : "r"(w.x), "r"(w.y), "r"(w.z), "r"(w.w));
  const float lo = __uint_as_float(m << 16), hi = __uint_as_float(m & 0xFFFF0000u);
  return (isnan(lo) || isnan(hi)) ? __uint_as_float(0x7fffffffu) : fmaxf(lo, hi);
}

template <int DT, int G, class Op>
__global__ void __launch_bounds__(256) fq_vec_kernel(const void* __restrict__ x_, void* __restrict__ y_,
                                                      int64_t total_threads, Op op) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int V = 16 / sizeof(T);  // elements per thread
  const T* __restrict__ x = static_cast<const T*>(x_);
  T* __restrict__ y = static_cast<T*>(y_);
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  // two vectors per thread per pass, both loads issued before either is used (one load in
  // flight per thread left the kernel latency-bound at ~3.5 TB/s)
  constexpr int U = 2;
  for (int64_t base = warp * 32; base < total_threads; base += nwarps * 32 * U) {
    int64_t t[U];
    bool active[U];
    uint4 raw[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      t[u] = base + int64_t(u) * nwarps * 32 + lane;
      active[u] = t[u] < total_threads;
      raw[u] = active[u] ? __ldg(reinterpret_cast<const uint4*>(x) + t[u]) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float v[V];
      float amax = 0.0f;
      const T* e = reinterpret_cast<const T*>(&raw[u]);
#pragma unroll
      for (int i = 0; i < V; ++i) v[i] = E::load(e[i]);
      if constexpr (DT == MZB_BF16) {
        amax = bf16x8_amax(raw[u]);
      } else {
#pragma unroll
        for (int i = 0; i < V; ++i) amax = amax_step(amax, v[i]);
      }
#pragma unroll
      for (int off = 1; off < G; off <<= 1) {
        float o = __shfl_xor_sync(0xffffffffu, amax, off);
        amax = (isnan(amax) || isnan(o)) ? __uint_as_float(0x7fffffffu) : fmaxf(amax, o);
      }
      if (active[u]) {
        const float s = op.scale(amax);
        const float inv = op.pow2() ? __frcp_rn(s) : 0.0f;  // exact for a power of two
        uint4 out;
        T* o = reinterpret_cast<T*>(&out);
#pragma unroll
        for (int i = 0; i < V; i += 2) {
          float r0, r1;
          op.apply2(v[i], v[i + 1], s, inv, r0, r1);
          o[i] = E::store(r0);
          o[i + 1] = E::store(r1);
        }
        reinterpret_cast<uint4*>(y)[t[u]] = out;
      }
    }
  }
}

// Any block size / alignment: one thread per block, scalar loads (shape support, not speed).
template <int DT, class Op>
__global__ void fq_scalar_kernel(const void* __restrict__ x_, void* __restrict__ y_, int64_t nblocks,
                                 int block, Op op) {
  using E = Elem<DT>;
  using T = typename E::T;
  const T* x = static_cast<const T*>(x_);
  T* y = static_cast<T*>(y_);
  for (int64_t b = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; b < nblocks;
       b += int64_t(gridDim.x) * blockDim.x) {
    const T* xb = x + b * block;
    float amax = 0.0f;
    for (int i = 0; i < block; ++i) amax = amax_step(amax, E::load(xb[i]));
    const float s = op.scale(amax);
    const float inv = op.pow2() ? __frcp_rn(s) : 0.0f;
    for (int i = 0; i < block; ++i) y[b * block + i] = E::store(op.apply(E::load(xb[i]), s, inv));
  }
}

template <int DT, class Op>
static int launch_fq(const void* x, void* y, int64_t numel, int block, Op op, cudaStream_t st) {
  using T = typename Elem<DT>::T;
  constexpr int V = 16 / sizeof(T);
  const int64_t nblocks = numel / block;
  const bool aligned = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (reinterpret_cast<uintptr_t>(y) % 16 == 0);
  const int g = block / V;
  const bool vec = aligned && block % V == 0 && g >= 1 && g <= 32 && (g & (g - 1)) == 0;
  if (numel == 0) return MZB_OK;
  if (vec) {
    const int64_t threads = numel / V;
    int64_t blocks = (threads + 255) / 256;
    const int64_t cap = int64_t(num_sms()) * 8;
    if (blocks > cap) blocks = cap;
    switch (g) {
#define MZB_FQ_CASE(GG) \
  case GG: fq_vec_kernel<DT, GG, Op><<<int(blocks), 256, 0, st>>>(x, y, threads, op); break;
      MZB_FQ_CASE(1) MZB_FQ_CASE(2) MZB_FQ_CASE(4) MZB_FQ_CASE(8) MZB_FQ_CASE(16) MZB_FQ_CASE(32)
#undef MZB_FQ_CASE
    }
  } else {
    int64_t blocks = (nblocks + 255) / 256;
    const int64_t cap = int64_t(num_sms()) * 8;
    if (blocks > cap) blocks = cap;
    fq_scalar_kernel<DT, Op><<<int(blocks), 256, 0, st>>>(x, y, nblocks, block, op);
  }
  return launch_status("fake_quant");
}

template <class Op>
static int dispatch_fq(const void* x, void* y, int64_t rows, int64_t n, int dtype, int block, Op op,
                       cudaStream_t st) {
  MZB_REQUIRE(rows >= 0 && n >= 0, MZB_ERR_SHAPE, "fake_quant: negative shape rows=%lld n=%lld",
              (long long)rows, (long long)n);
  MZB_REQUIRE(block >= 1, MZB_ERR_SHAPE, "fake_quant: block_size must be >= 1, got %d", block);
  MZB_REQUIRE(n % block == 0, MZB_ERR_SHAPE,
              "fake_quant: last dim %lld not divisible by block_size %d (the caller returns x unchanged)",
              (long long)n, block);
  const int64_t numel = rows * n;
  switch (dtype) {
    case MZB_F32: return launch_fq<MZB_F32>(x, y, numel, block, op, st);
    case MZB_BF16: return launch_fq<MZB_BF16>(x, y, numel, block, op, st);
    case MZB_F16: return launch_fq<MZB_F16>(x, y, numel, block, op, st);
  }
  set_error("fake_quant: unsupported dtype code %d", dtype);
  return MZB_ERR_UNSUPPORTED;
}

}  // namespace mzb

extern "C" int mzb_fq_fp4(const void* x, void* y, int64_t rows, int64_t n, int dtype, int block_size,
                          int rule, void* stream) {
  MZB_REQUIRE(rule >= 0 && rule <= 2, MZB_ERR_UNSUPPORTED, "mzb_fq_fp4: unknown rule %d", rule);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rule == mzb::FP4_UE8M0) return mzb::dispatch_fq(x, y, rows, n, dtype, block_size, mzb::Fp4Op<mzb::FP4_UE8M0>{}, st);
  if (rule == mzb::FP4_E4M3) return mzb::dispatch_fq(x, y, rows, n, dtype, block_size, mzb::Fp4Op<mzb::FP4_E4M3>{}, st);
  return mzb::dispatch_fq(x, y, rows, n, dtype, block_size, mzb::Fp4Op<mzb::FP4_OCP>{}, st);
}

extern "C" int mzb_fq_fp8(const void* x, void* y, int64_t rows, int64_t n, int dtype, int block_size,
                          int rule, void* stream) {
  MZB_REQUIRE(rule >= 0 && rule <= 1, MZB_ERR_UNSUPPORTED, "mzb_fq_fp8: unknown rule %d", rule);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rule == mzb::FP8_UE8M0) return mzb::dispatch_fq(x, y, rows, n, dtype, block_size, mzb::Fp8Op<mzb::FP8_UE8M0>{}, st);
  return mzb::dispatch_fq(x, y, rows, n, dtype, block_size, mzb::Fp8Op<mzb::FP8_ABSMAX>{}, st);
}
