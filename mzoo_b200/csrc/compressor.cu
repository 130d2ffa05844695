// Compressor producer step, fused after the two fp32 projections: gated softmax pool of
// `ratio` tokens, RMSNorm, and the compressed-cache entry (RoPE + MXFP4 fake quant).
//
// Reference: src/mzoo/archs/dsv4/modeling_deepseek_v41.py
//   :318-340  DeepseekV41Compressor.forward -- kv = x W_kv^T, gate = x W_gate^T in fp32;
//             latent = sum_r kv_r * softmax_r(gate_r) per channel (fp32), cast to the model
//             dtype, RMSNorm; ratio 1: no gate, the projection itself
//   :58-63    DeepseekV41RMSNorm -- x fp32 * rsqrt(mean(x^2) + eps), cast, times the weight
//   :405-425  apply_rotary_pos_emb -- adjacent (even, odd) pairs of the trailing rope
//             channels rotated as complex numbers in fp32, cast back
//   :745-753  the cache entry: rotate the latent, then _fake_quant_fp4_block(block 16,
//             e4m3 scales)
// The projections are plain GEMMs (the library's); this kernel reads their fp32 outputs
// once and writes both the pre-RoPE latent (the indexer's input, :509-510) and the cache
// entry, instead of the reference's chain of separate elementwise passes.
//
// One CTA per group (batch, g); thread t owns channels [4t, 4t + 4) (16-byte loads of every
// token row of the group), so a rope pair and a quarter of a 16-channel quant block stay in
// one thread.  Groups of up to RMAX tokens load all their kv and gate rows into registers
// first (one DRAM round trip); longer groups loop over the rows three times (max, sum,
// weighted sum; the later passes hit L1).  The softmax uses expf and a division, as torch's; the RMS variance is a CTA
// reduction in fp32.  Rope and fake quant use explicitly rounded operations, so they are
// bit-exact given the bf16 latent.  Model dtype bf16 (latent, weight, outputs).
#include "common.cuh"

namespace mzb {
namespace comp {

constexpr int MAXT = 1024;
constexpr int RMAX = 4;  // groups up to this many tokens keep all their rows in registers

__device__ __forceinline__ float bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

struct Args {
  const float* kv;        // [B, G*ratio, D]
  const float* gate;      // [B, G*ratio, D] or null (ratio 1)
  const __nv_bfloat16* w; // [D] RMSNorm weight
  const float* cosv;      // [B, G, rope/2] or null (no cache entry)
  const float* sinv;
  __nv_bfloat16* latent;  // [B, G, D]
  __nv_bfloat16* cache;   // [B, G, D] or null
  int G, ratio, D, rope;
  float eps;
};

__global__ void __launch_bounds__(MAXT) compress_kernel(Args a) {
  __shared__ float red[32];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int c0 = 4 * t;
  const bool own = c0 < a.D;
  const long long row = blockIdx.x;  // b * G + g
  const long long b = row / a.G, g = row % a.G;
  const long long tok0 = (b * a.G + g) * a.ratio;  // first token row of the group
  float v[4] = {0.f, 0.f, 0.f, 0.f};
  if (own) {
    if (a.gate == nullptr) {
      const float4 x = *reinterpret_cast<const float4*>(a.kv + tok0 * a.D + c0);
      v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
    } else if (a.ratio <= RMAX) {
      // short groups: every row of kv and gate loaded up front (one DRAM round trip), then
      // the same operations in the same order as the general path below
      float4 gr[RMAX], kr[RMAX];
#pragma unroll
      for (int r = 0; r < RMAX; ++r) {
        if (r < a.ratio) {
          gr[r] = *reinterpret_cast<const float4*>(a.gate + (tok0 + r) * a.D + c0);
          kr[r] = *reinterpret_cast<const float4*>(a.kv + (tok0 + r) * a.D + c0);
        }
      }
      float m[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY}, s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int r = 0; r < RMAX; ++r)
        if (r < a.ratio) {
          m[0] = fmaxf(m[0], gr[r].x); m[1] = fmaxf(m[1], gr[r].y); m[2] = fmaxf(m[2], gr[r].z); m[3] = fmaxf(m[3], gr[r].w);
        }
#pragma unroll
      for (int r = 0; r < RMAX; ++r)
        if (r < a.ratio) {
          s[0] += expf(gr[r].x - m[0]); s[1] += expf(gr[r].y - m[1]); s[2] += expf(gr[r].z - m[2]); s[3] += expf(gr[r].w - m[3]);
        }
#pragma unroll
      for (int r = 0; r < RMAX; ++r)
        if (r < a.ratio) {
          const float gg[4] = {gr[r].x, gr[r].y, gr[r].z, gr[r].w}, kk[4] = {kr[r].x, kr[r].y, kr[r].z, kr[r].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) v[j] = __fadd_rn(v[j], __fmul_rn(kk[j], expf(gg[j] - m[j]) / s[j]));
        }
    } else {
      // softmax over the group's tokens per channel: max, exp(g - max), sum, divide
      float m[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      for (int r = 0; r < a.ratio; ++r) {
        const float4 gv = *reinterpret_cast<const float4*>(a.gate + (tok0 + r) * a.D + c0);
        m[0] = fmaxf(m[0], gv.x); m[1] = fmaxf(m[1], gv.y); m[2] = fmaxf(m[2], gv.z); m[3] = fmaxf(m[3], gv.w);
      }
      float s[4] = {0.f, 0.f, 0.f, 0.f};
      for (int r = 0; r < a.ratio; ++r) {
        const float4 gv = *reinterpret_cast<const float4*>(a.gate + (tok0 + r) * a.D + c0);
        s[0] += expf(gv.x - m[0]); s[1] += expf(gv.y - m[1]); s[2] += expf(gv.z - m[2]); s[3] += expf(gv.w - m[3]);
      }
      // as torch: the softmax weights first (exp / sum), then sum_r kv_r * w_r (the group's
      // rows are re-read from L1)
      for (int r = 0; r < a.ratio; ++r) {
        const float4 gv = *reinterpret_cast<const float4*>(a.gate + (tok0 + r) * a.D + c0);
        const float4 kv = *reinterpret_cast<const float4*>(a.kv + (tok0 + r) * a.D + c0);
        const float gg[4] = {gv.x, gv.y, gv.z, gv.w}, kk[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = __fadd_rn(v[j], __fmul_rn(kk[j], expf(gg[j] - m[j]) / s[j]));
      }
    }
  }
  // cast to the model dtype, RMSNorm over D channels
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[j] = own ? bf(v[j]) : 0.f;
    ss = fmaf(v[j], v[j], ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float x = lane < (blockDim.x >> 5) ? red[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    if (lane == 0) red[0] = x;
  }
  __syncthreads();
  const float inv = 1.0f / sqrtf(red[0] / float(a.D) + a.eps);
  float y[4];
  if (own) {
    const uint2 wr = *reinterpret_cast<const uint2*>(a.w + c0);
    const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wr);
    const float2 w01 = __bfloat1622float2(w2[0]), w23 = __bfloat1622float2(w2[1]);
    const float wv[4] = {w01.x, w01.y, w23.x, w23.y};
#pragma unroll
    for (int j = 0; j < 4; ++j) y[j] = bf(__fmul_rn(wv[j], bf(v[j] * inv)));
    __nv_bfloat162 o0 = __floats2bfloat162_rn(y[0], y[1]), o1 = __floats2bfloat162_rn(y[2], y[3]);
    uint2 ov;
    ov.x = *reinterpret_cast<uint32_t*>(&o0);
    ov.y = *reinterpret_cast<uint32_t*>(&o1);
    *reinterpret_cast<uint2*>(a.latent + row * a.D + c0) = ov;
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) y[j] = 0.f;
  }
  if (a.cache == nullptr) return;  // uniform over the CTA
  // the cache entry: rope on the trailing channels (pairs inside this thread), then the
  // 16-channel e2m1 quant-dequant with an e4m3 scale (4 lanes per block)
  const int r0 = a.D - a.rope;
  if (own && c0 >= r0) {
    const float* cs = a.cosv + row * (a.rope / 2) + (c0 - r0) / 2;
    const float* sn = a.sinv + row * (a.rope / 2) + (c0 - r0) / 2;
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const float e = y[2 * p], o = y[2 * p + 1], c = cs[p], s = sn[p];
      y[2 * p] = bf(__fsub_rn(__fmul_rn(e, c), __fmul_rn(o, s)));
      y[2 * p + 1] = bf(__fadd_rn(__fmul_rn(e, s), __fmul_rn(o, c)));
    }
  }
  float am = fmaxf(fmaxf(fabsf(y[0]), fabsf(y[1])), fmaxf(fabsf(y[2]), fabsf(y[3])));
  am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
  am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
  if (!own) return;
  const float sc = e4m3_round(__fdiv_rn(fmaxf(am, 6.0f * 0x1p-9f), 6.0f));
  float q[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) q[j] = __fmul_rn(e2m1_value(clamp_nan(__fdiv_rn(y[j], sc), -6.0f, 6.0f)), sc);
  __nv_bfloat162 q0 = __floats2bfloat162_rn(q[0], q[1]), q1 = __floats2bfloat162_rn(q[2], q[3]);
  uint2 qv;
  qv.x = *reinterpret_cast<uint32_t*>(&q0);
  qv.y = *reinterpret_cast<uint32_t*>(&q1);
  *reinterpret_cast<uint2*>(a.cache + row * a.D + c0) = qv;
}

}  // namespace comp
}  // namespace mzb

using namespace mzb;

extern "C" int mzb_compress(const float* kv, const float* gate, const void* norm_w, const float* cos_v,
                            const float* sin_v, void* latent, void* cache, int64_t B, int64_t G, int ratio, int D,
                            int rope_dim, float eps, void* stream) {
  MZB_REQUIRE(B >= 0 && G >= 0 && ratio >= 1 && B * G < (int64_t(1) << 31), MZB_ERR_SHAPE,
              "compress: bad sizes B=%lld G=%lld ratio=%d", (long long)B, (long long)G, ratio);
  MZB_REQUIRE(D >= 16 && D % 16 == 0 && D / 4 <= comp::MAXT, MZB_ERR_UNSUPPORTED,
              "compress: head_dim %d must be a multiple of 16 (the fp4 block) and at most %d", D, 4 * comp::MAXT);
  MZB_REQUIRE(ratio == 1 || gate != nullptr, MZB_ERR_SHAPE, "compress: ratio %d > 1 needs the gate projection",
              ratio);
  MZB_REQUIRE(cache == nullptr || (cos_v && sin_v && rope_dim >= 0 && rope_dim % 4 == 0 && rope_dim <= D),
              MZB_ERR_SHAPE, "compress: the cache entry needs cos / sin and a rope_dim (multiple of 4, <= D), got %d",
              rope_dim);
  MZB_REQUIRE(B * G == 0 || (kv && norm_w && latent), MZB_ERR_SHAPE, "compress: kv, norm weight and latent required");
  MZB_REQUIRE(((reinterpret_cast<uintptr_t>(kv) | reinterpret_cast<uintptr_t>(gate)) & 15) == 0, MZB_ERR_ALIGN,
              "compress: kv / gate must be 16-byte aligned");
  MZB_REQUIRE(((reinterpret_cast<uintptr_t>(latent) | reinterpret_cast<uintptr_t>(cache) |
                reinterpret_cast<uintptr_t>(norm_w)) & 7) == 0,
              MZB_ERR_ALIGN, "compress: latent, cache and the norm weight must be 8-byte aligned");
  if (B * G == 0) return MZB_OK;
  comp::Args a{kv, gate, static_cast<const __nv_bfloat16*>(norm_w), cos_v, sin_v,
               static_cast<__nv_bfloat16*>(latent), static_cast<__nv_bfloat16*>(cache), int(G), ratio, D,
               cache ? rope_dim : 0, eps};
  const int threads = ((D / 4 + 31) / 32) * 32;
  comp::compress_kernel<<<unsigned(B * G), threads, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return launch_status("compress");
}
