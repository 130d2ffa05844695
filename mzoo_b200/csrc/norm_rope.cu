// Fused RMSNorm + RoPE prologue of q / kv, forward and backward (one pass over the rows).
//
// Reference: src/mzoo/layers/attn/norm_rope.py (the fused TileLang kernels `make_fwd`
// :52-110 / `make_bwd` :113-180 and their contract `qk_norm_rope_eager` :37-44, which is
// the model's `DeepseekV41RMSNorm.forward` then `apply_rotary_pos_emb`,
// archs/dsv4/modeling_deepseek_v41.py:49-63, :405-425).
//
//   rstd = 1 / sqrt(mean(x^2) + eps) (fp32);  y = bf16(w * bf16(x * rstd))
//   nope channels pass, each (even, odd) pair of the trailing rope_dim channels rotates:
//   y_e' = bf16(e*cos - o*sin), y_o' = bf16(e*sin + o*cos) (fp32, products rounded separately)
//
// Backward (the reference's closed form, bf16 casts treated as identity): dxn = the
// inverse rotation of dy, g = w * dxn, dx = rstd * (g - x * rstd^2 * mean(g * x)),
// dw = sum_rows dxn * x * rstd.
//
// Layout: rows = B*S*H of D bf16 channels (BSHD), row r belongs to token r / H; cos / sin
// [tokens, rope_dim / 2] fp32.  HBM-bound: one 16-byte vector (8 channels) per lane, a row
// on 16 lanes (D <= 128, two rows per warp) or a whole warp (D = 256); each warp issues
// the loads of two such row groups (with their cos / sin vectors) before any math, then
// strides over the rows; 3-4 blocks of 256 threads per SM.  dw: each block accumulates its rows' contributions per channel in registers and
// writes one partial row; a second kernel sums the partials in a fixed order
// (deterministic, no atomics).
#include "common.cuh"

namespace mzb {
namespace nr {

constexpr int THREADS = 256;

struct Args {
  const __nv_bfloat16* x;
  const __nv_bfloat16* w;
  const float* cos;
  const float* sin;
  const __nv_bfloat16* dy;
  __nv_bfloat16* out;  // forward: y; backward: dx
  float* rstd;
  float* dw_part;      // [parts, D]
  float* dw;           // [D]
  long long rows;
  int heads, rope_dim, parts;
  float eps;
};

__device__ __forceinline__ void unpack8(const uint4 v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 b = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&b);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ float bf16_round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

template <int D>
struct Geo {
  static constexpr int CH = D / 8;                // 16-byte chunks per row
  static constexpr int LPR = D <= 128 ? 16 : 32;  // lanes per row
  static constexpr int RPW = 32 / LPR;            // rows per warp
};

// sum over the LPR lanes holding one row
template <int LPR>
__device__ __forceinline__ float row_sum(float v) {
#pragma unroll
  for (int o = LPR / 2; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

constexpr int U = 2;  // row groups per warp iteration: their loads are all issued before any math

// cos / sin of the 4 pairs in channel chunk `sub` of a row of token `tok` (16-byte vectors
// when the chunk is entirely rope and the pair index is 4-aligned; scalar otherwise)
__device__ __forceinline__ void load_cs(const Args& a, int D, int sub, long long tok, float (&c)[4], float (&s)[4]) {
  const int nope = D - a.rope_dim, half = a.rope_dim / 2, d0 = sub * 8;
  if (d0 + 8 <= nope) return;
  if (d0 >= nope && ((d0 - nope) & 7) == 0 && (half & 3) == 0) {
    const int j0 = (d0 - nope) >> 1;
    const float4 cv = __ldg(reinterpret_cast<const float4*>(a.cos + tok * half + j0));
    const float4 sv = __ldg(reinterpret_cast<const float4*>(a.sin + tok * half + j0));
    c[0] = cv.x; c[1] = cv.y; c[2] = cv.z; c[3] = cv.w;
    s[0] = sv.x; s[1] = sv.y; s[2] = sv.z; s[3] = sv.w;
    return;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = d0 + 2 * i;
    if (d >= nope) {
      c[i] = __ldg(a.cos + tok * half + ((d - nope) >> 1));
      s[i] = __ldg(a.sin + tok * half + ((d - nope) >> 1));
    }
  }
}

template <int D>
__global__ void __launch_bounds__(THREADS, 4) fwd_kernel(Args a) {
  using G = Geo<D>;
  const int lane = threadIdx.x & 31, sub = lane % G::LPR, slot = lane / G::LPR;
  const long long gw = (long long)(blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nw = (long long)(gridDim.x * blockDim.x) >> 5;
  const bool has = sub < G::CH;
  const int nope = D - a.rope_dim, d0 = sub * 8;
  const bool rope = has && d0 + 8 > nope;
  float wv[8];
  if (has) unpack8(__ldg(reinterpret_cast<const uint4*>(a.w) + sub), wv);
  for (long long rb = gw * G::RPW * U; rb < a.rows; rb += nw * G::RPW * U) {
    uint4 raw[U];
    float cs[U][4], sn[U][4];
#pragma unroll
    for (int u = 0; u < U; ++u) {  // every load of the U rows first
      const long long r = rb + u * G::RPW + slot;
      raw[u] = make_uint4(0, 0, 0, 0);
      if (has && r < a.rows) {
        raw[u] = __ldg(reinterpret_cast<const uint4*>(a.x + r * D) + sub);
        if (rope) load_cs(a, D, sub, r / a.heads, cs[u], sn[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long long r = rb + u * G::RPW + slot;
      const bool act = has && r < a.rows;
      float v[8];
      unpack8(raw[u], v);
      float ss = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(v[i], v[i], ss);
      ss = row_sum<G::LPR>(ss);
      const float rstd = rsqrtf(ss / float(D) + a.eps);
      if (!act) continue;
      float y[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = bf16_round(__fmul_rn(wv[i], bf16_round(__fmul_rn(v[i], rstd))));
      if (rope) {  // nope is even: a pair never straddles chunks
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (d0 + 2 * i >= nope) {
            const float c = cs[u][i], s = sn[u][i], e = y[2 * i], o = y[2 * i + 1];
            y[2 * i] = __fsub_rn(__fmul_rn(e, c), __fmul_rn(o, s));
            y[2 * i + 1] = __fadd_rn(__fmul_rn(e, s), __fmul_rn(o, c));
          }
        }
      }
      reinterpret_cast<uint4*>(a.out + r * D)[sub] = pack8(y);
      if (sub == 0) a.rstd[r] = rstd;
    }
  }
}

template <int D>
__global__ void __launch_bounds__(THREADS, 3) bwd_kernel(Args a) {
  using G = Geo<D>;
  __shared__ float red[THREADS / 32 * 2][D];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sub = lane % G::LPR, slot = lane / G::LPR;
  const long long gw = (long long)(blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nw = (long long)(gridDim.x * blockDim.x) >> 5;
  const bool has = sub < G::CH;
  const int nope = D - a.rope_dim, d0 = sub * 8;
  const bool rope = has && d0 + 8 > nope;
  float wv[8], dwa[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (has) unpack8(__ldg(reinterpret_cast<const uint4*>(a.w) + sub), wv);
  for (long long rb = gw * G::RPW * U; rb < a.rows; rb += nw * G::RPW * U) {
    uint4 rx[U], rdy[U];
    float rs[U], cs[U][4], sn[U][4];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long long r = rb + u * G::RPW + slot;
      rx[u] = rdy[u] = make_uint4(0, 0, 0, 0);
      rs[u] = 0.0f;
      if (has && r < a.rows) {
        rx[u] = __ldg(reinterpret_cast<const uint4*>(a.x + r * D) + sub);
        rdy[u] = __ldg(reinterpret_cast<const uint4*>(a.dy + r * D) + sub);
        rs[u] = __ldg(a.rstd + r);
        if (rope) load_cs(a, D, sub, r / a.heads, cs[u], sn[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long long r = rb + u * G::RPW + slot;
      const bool act = has && r < a.rows;
      float xv[8], dxn[8];
      unpack8(rx[u], xv);
      unpack8(rdy[u], dxn);
      if (rope) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (d0 + 2 * i >= nope) {
            const float c = cs[u][i], s = sn[u][i], e = dxn[2 * i], o = dxn[2 * i + 1];
            dxn[2 * i] = fmaf(e, c, o * s);
            dxn[2 * i + 1] = fmaf(o, c, -e * s);
          }
        }
      }
      float g[8], dot = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        g[i] = act ? wv[i] * dxn[i] : 0.0f;
        dot = fmaf(g[i], xv[i], dot);
      }
      dot = row_sum<G::LPR>(dot) / float(D);
      if (!act) continue;
      const float rstd = rs[u], k2 = rstd * rstd * dot;
      float dx[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        dx[i] = rstd * (g[i] - xv[i] * k2);
        dwa[i] = fmaf(dxn[i] * xv[i], rstd, dwa[i]);
      }
      reinterpret_cast<uint4*>(a.out + r * D)[sub] = pack8(dx);
    }
  }
  // this block's dw: per (warp, row slot) partials in shared memory, summed in a fixed order
  if (has) {
#pragma unroll
    for (int i = 0; i < 8; ++i) red[warp * G::RPW + slot][sub * 8 + i] = dwa[i];
  }
  __syncthreads();
  for (int d = threadIdx.x; d < D; d += THREADS) {
    float s = 0.0f;
    for (int k = 0; k < THREADS / 32 * G::RPW; ++k) s += red[k][d];
    a.dw_part[(long long)blockIdx.x * D + d] = s;
  }
}

// dw[d] = sum over the partial rows: one block per channel, each thread a strided subset
// of the partials, then a fixed-order tree over the threads (deterministic).
__global__ void __launch_bounds__(THREADS) dw_reduce_kernel(Args a, int D) {
  __shared__ float red[THREADS];
  const int d = blockIdx.x;
  float s = 0.0f;
  for (int p = threadIdx.x; p < a.parts; p += THREADS) s += a.dw_part[(long long)p * D + d];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int o = THREADS / 2; o; o >>= 1) {
    if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) a.dw[d] = red[0];
}

static int grid_for(long long rows, int D) {
  const int rpw = (D <= 128 ? 2 : 1) * U;
  const long long blocks = (rows + (THREADS / 32) * rpw - 1) / ((THREADS / 32) * rpw);
  const long long cap = (long long)num_sms() * 8;
  return int(blocks < cap ? (blocks < 1 ? 1 : blocks) : cap);
}

static int check(const void* x, const void* w, const void* out, long long rows, int heads, int dim, int rope_dim) {
  MZB_REQUIRE(dim == 64 || dim == 96 || dim == 128 || dim == 256, MZB_ERR_UNSUPPORTED,
              "norm_rope: head dim must be 64, 96, 128 or 256, got %d", dim);
  MZB_REQUIRE(rope_dim >= 0 && rope_dim <= dim && rope_dim % 2 == 0 && (dim - rope_dim) % 2 == 0, MZB_ERR_SHAPE,
              "norm_rope: rope_dim %d must be even and at most the head dim %d", rope_dim, dim);
  MZB_REQUIRE(rows >= 0 && heads >= 1 && rows % heads == 0, MZB_ERR_SHAPE,
              "norm_rope: rows %lld must be a multiple of heads %d", rows, heads);
  MZB_REQUIRE(reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(out) % 16 == 0,
              MZB_ERR_ALIGN, "norm_rope: x, w and the output must be 16-byte aligned");
  return MZB_OK;
}

}  // namespace nr
}  // namespace mzb

using namespace mzb;

extern "C" int mzb_norm_rope_fwd(const void* x, const void* w, const float* cos, const float* sin, void* out,
                                 float* rstd, int64_t rows, int heads, int dim, int rope_dim, float eps,
                                 void* stream) {
  if (int e = nr::check(x, w, out, rows, heads, dim, rope_dim)) return e;
  if (rows == 0) return MZB_OK;
  MZB_REQUIRE(rope_dim == 0 || (cos && sin), MZB_ERR_SHAPE, "norm_rope: cos / sin required when rope_dim > 0");
  nr::Args a{};
  a.x = static_cast<const __nv_bfloat16*>(x); a.w = static_cast<const __nv_bfloat16*>(w);
  a.cos = cos; a.sin = sin; a.out = static_cast<__nv_bfloat16*>(out); a.rstd = rstd;
  a.rows = rows; a.heads = heads; a.rope_dim = rope_dim; a.eps = eps;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = nr::grid_for(rows, dim);
  switch (dim) {
    case 64: nr::fwd_kernel<64><<<grid, nr::THREADS, 0, st>>>(a); break;
    case 96: nr::fwd_kernel<96><<<grid, nr::THREADS, 0, st>>>(a); break;
    case 128: nr::fwd_kernel<128><<<grid, nr::THREADS, 0, st>>>(a); break;
    default: nr::fwd_kernel<256><<<grid, nr::THREADS, 0, st>>>(a); break;
  }
  return launch_status("norm_rope_fwd");
}

extern "C" int mzb_norm_rope_bwd_parts(int64_t rows, int dim) {
  if (rows <= 0) return 1;
  return nr::grid_for(rows, dim);
}

extern "C" int mzb_norm_rope_bwd(const void* x, const void* dy, const void* w, const float* rstd, const float* cos,
                                 const float* sin, void* dx, float* dw_part, float* dw, int64_t rows, int heads,
                                 int dim, int rope_dim, int parts, void* stream) {
  if (int e = nr::check(x, w, dx, rows, heads, dim, rope_dim)) return e;
  MZB_REQUIRE(reinterpret_cast<uintptr_t>(dy) % 16 == 0, MZB_ERR_ALIGN, "norm_rope: dy must be 16-byte aligned");
  MZB_REQUIRE(dw_part && dw, MZB_ERR_SHAPE, "norm_rope: needs the dw workspace and output");
  MZB_REQUIRE(rope_dim == 0 || (cos && sin), MZB_ERR_SHAPE, "norm_rope: cos / sin required when rope_dim > 0");
  const int grid = nr::grid_for(rows, dim);
  MZB_REQUIRE(parts >= grid, MZB_ERR_SHAPE, "norm_rope: dw workspace holds %d partial rows, %d needed", parts, grid);
  nr::Args a{};
  a.x = static_cast<const __nv_bfloat16*>(x); a.w = static_cast<const __nv_bfloat16*>(w);
  a.dy = static_cast<const __nv_bfloat16*>(dy); a.cos = cos; a.sin = sin;
  a.out = static_cast<__nv_bfloat16*>(dx); a.rstd = const_cast<float*>(rstd); a.dw_part = dw_part; a.dw = dw;
  a.rows = rows; a.heads = heads; a.rope_dim = rope_dim; a.parts = rows > 0 ? grid : 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rows > 0) {
    switch (dim) {
      case 64: nr::bwd_kernel<64><<<grid, nr::THREADS, 0, st>>>(a); break;
      case 96: nr::bwd_kernel<96><<<grid, nr::THREADS, 0, st>>>(a); break;
      case 128: nr::bwd_kernel<128><<<grid, nr::THREADS, 0, st>>>(a); break;
      default: nr::bwd_kernel<256><<<grid, nr::THREADS, 0, st>>>(a); break;
    }
    if (int r = launch_status("norm_rope_bwd")) return r;
  }
  nr::dw_reduce_kernel<<<dim, nr::THREADS, 0, st>>>(a, dim);
  return launch_status("norm_rope_dw_reduce");
}
