// Shared-latent MQA attention backward (swa_attn / csa2_attn), tcgen05 kernels.
//
// Reference: src/mzoo/layers/attn/swa_attn/bwd.py:79-119 (preprocess, bwd_kv, bwd_dq) and
// csa2_attn/bwd.py:67-130 + bwd_dq.py:60-187 (dQ plus the fp32-atomic scatter of dmain_kv).
// With P the softmax (sink column included through lse), delta = rowsum(dO * O):
//   dS = P * (dO V^T - delta),  dQ = scale dS K,  dK = scale dS^T Q,  dV = P^T dO,
//   K == V: dKV = dK + dV;  gathered rows: dmain[idx] += dK_g + dV_g (fp32 atomics, so not
//   bit-reproducible run to run, as in the reference).
//
// Kernels (one CTA per tile, persistent):
//   preprocess  delta and lse*log2(e) per packed row, into 128-row-padded buffers
//   dkv         key owner: 128 window keys; loops over the query tiles that see them;
//               S^T = K Q^T and dP^T = V dO^T in TMEM; two compute warpgroups (thread =
//               key; warps 4-7 query columns [0, 64), warps 8-11 [64, 128)) turn them into
//               P^T, dS^T and store them back into TMEM as bf16, each half packed into the
//               front of its own columns, which the TS MMAs dV += P^T dO, dK += dS^T Q
//               read as their A operand.
//   dq          query owner: 128 rows; loops over window tiles then gathered tiles;
//               S = Q K^T, dP = dO V^T; dS -> TMEM (A of dQ += dS K); gathered tiles also
//               keep dS and P in shared memory for dM = dS^T Q + P^T dO, scattered into
//               dmain by the compute warps with fp32 atomics.  Window-only (separate V):
//               warps 8-11 take the upper key half of every tile and copy each item's Q /
//               dO rows into the unused dM columns, so S and dP are TS MMAs issued per key
//               half and software-pipelined across the two warpgroups.
// Column visibility (window run, or a token's valid gathered slots) is one mask word per
// 32 columns, built per tile.  D = 256 (K == V): the key owner keeps one Q/dO stage and a
// merged dK + dV accumulator; the query owner uses 64-key tiles and forms the gathered-row
// gradient transposed (dM^T, channels in TMEM lanes).
#include "tc.cuh"

namespace mzb {
namespace attnb {

constexpr float LOG2E = 1.4426950408889634f;

__device__ __forceinline__ void st_shared16(uint8_t* p, const uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(p)), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 ld_shared16(const uint8_t* p) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_u32(p))
               : "memory");
  return v;
}
// bits [lo, hi] of a 32-bit word (empty when hi < lo; lo, hi clipped to [0, 31])
__device__ __forceinline__ uint32_t run_bits(int lo, int hi) {
  lo = max(lo, 0);
  hi = min(hi, 31);
  return lo > hi ? 0u : ((0xFFFFFFFFu >> (31 - (hi - lo))) << lo);
}
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

struct Args {
  const __nv_bfloat16* o;
  const __nv_bfloat16* dout;
  const float* lse;      // [B, S*H] natural log
  float* delta;          // [B, Rpad] workspace
  float* lse2;           // [B, Rpad] workspace (lse * log2 e)
  const __nv_bfloat16* main_kv;
  const int32_t* idx;
  __nv_bfloat16* dq;     // [B, S*H, D]
  __nv_bfloat16* dk;     // [B, S, D]  (dK + dV when K == V)
  __nv_bfloat16* dv;     // [B, S, D] or null
  float* dmain;          // [B, G, D] fp32 accumulator (zeroed by the caller) or null
  float* dkv_part;       // [splits, B, S, 2, D] fp32 partial dK (scaled) | dV per query-loop split
  int B, S, H, D, window, G, topk, Rpad, hshift, splits;
  float scale, scale_log2;
  int* err;
};

// ------------------------------------------------------------------ preprocess
// Four lanes per packed row, each reading D / 32 16-byte vectors of O and dO (all in flight).
template <int D>
__global__ void __launch_bounds__(256) preprocess_kernel(Args a) {
  constexpr int NV = D / 8 / 4;  // 16-byte vectors per lane
  const long long row = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 2;
  const int sub = threadIdx.x & 3;
  const long long R = (long long)a.S * a.H, nrows = (long long)a.B * a.Rpad;
  const bool in = row < nrows;  // lanes past the end still take part in the shuffles
  const long long b = in ? row / a.Rpad : 0, r = in ? row % a.Rpad : 0;
  float d = 0.0f, l2 = 0.0f;
  if (in && r < R) {
    const uint4* op = reinterpret_cast<const uint4*>(a.o + (b * R + r) * D);
    const uint4* gp = reinterpret_cast<const uint4*>(a.dout + (b * R + r) * D);
    uint4 ov[NV], gv[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      ov[v] = __ldg(op + sub + 4 * v);
      gv[v] = __ldg(gp + sub + 4 * v);
    }
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const __nv_bfloat162* o2 = reinterpret_cast<const __nv_bfloat162*>(&ov[v]);
      const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv[v]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 of = __bfloat1622float2(o2[i]), gf = __bfloat1622float2(g2[i]);
        d = fmaf(of.x, gf.x, d);
        d = fmaf(of.y, gf.y, d);
      }
    }
    l2 = a.lse[b * R + r] * LOG2E;
  }
  d += __shfl_xor_sync(0xffffffffu, d, 1);
  d += __shfl_xor_sync(0xffffffffu, d, 2);
  if (in && sub == 0) {
    a.delta[b * a.Rpad + r] = d;
    a.lse2[b * a.Rpad + r] = l2;
  }
}

// ------------------------------------------------------------------ dkv (key owner)
template <int D, bool SEP_V>
struct KvCfg {
  static constexpr int DB = D / 64;
  static constexpr int T_BYTES = 128 * D * 2;  // one 128-row tile of Q, dO, K or V
  static constexpr int STAGE = 2 * T_BYTES + 1024;  // Q, dO, lse2[128], delta[128]
  // D = 256 (K == V only): one Q/dO stage fits the shared memory, and dK and dV share one
  // accumulator (scale * dS^T Q + P^T dO) so that S and dP still fit in TMEM
  static constexpr bool MERGE = D == 256;
  static constexpr int NST = MERGE ? 1 : 2;
  static constexpr int TILE_BYTES = (SEP_V ? 2 : 1) * T_BYTES + NST * STAGE;
  static constexpr int SMEM = TILE_BYTES + 256;
  static constexpr int C_DK = 0, C_DV = MERGE ? 0 : D, C_S = MERGE ? D : 2 * D, C_DP = C_S + 128;
  static_assert(C_DP + 128 <= 512, "TMEM");
  static_assert(SMEM <= 232448, "smem");
  static_assert(!(MERGE && SEP_V), "a separate V needs D <= 128");
};

// Packed bf16 column of query column c (even) of P^T / dS^T within the S / dP region: each
// half of the 128 columns is packed into the front of its own 64 columns, so the two compute
// warpgroups never store over columns the other one has still to read.
__device__ __forceinline__ int pt_col(int c) { return c / 2 + (c >= 64 ? 32 : 0); }

// S_FULL / PT_FULL per query half h (columns [64 h, 64 h + 64)): S_FULL + h, PT_FULL + h
enum KvBar { KV_FULL = 0, KV_EMPTY, QD_FULL, QD_FULL1, QD_EMPTY, QD_EMPTY1, S_FULL, S_FULL1, PT_FULL, PT_FULL1,
             O_DONE, ACC_EMPTY, KV_NBAR };

struct KvItem {
  int b, kt, k0, sp, nq;  // nq query tiles in this split (may be 0)
  int q_lo, total, s0;    // the key tile's query tiles [q_lo, q_lo + total); this split's first step
};

// Query tile of step i of an item.  A key tile's query tiles are visited rotated, step
// s0 + i taking the tile q_lo + ((s0 + i - q_lo) mod total): every key tile with the full
// window (total equal for all of them) then reads, at the same step, the tile whose index is
// congruent to that step, so the ~window/128 + 1 key tiles that share a query tile -- issued
// in the same wave of items -- read it at about the same time and L2 serves the repeats
// (visited in plain order, adjacent key tiles reach a tile 128*H/128 steps apart, and every
// query row came from DRAM once per key tile).  The split's sum does not depend on the order
// beyond fp32 rounding; the order is fixed, so results stay deterministic.
__device__ __forceinline__ int kv_qtile(const KvItem& m, int i) {
  int r = (m.s0 + i - m.q_lo) % m.total;
  if (r < 0) r += m.total;
  return m.q_lo + r;
}

// Item = (key tile, batch, split of the query loop): the reference's split query loop
// (swa_attn/bwd.py:66 pick_splits) so every SM has work; partials are summed by
// dkv_finalize_kernel in a fixed order (deterministic).
__device__ __forceinline__ KvItem kv_item(const Args& a, int it) {
  KvItem m;
  m.sp = it % a.splits;
  const int rest = it / a.splits;
  m.b = rest % a.B;
  m.kt = rest / a.B;
  m.k0 = m.kt * 128;
  const int k1 = min(a.S - 1, m.k0 + 127);
  const int tmax = min(a.S - 1, k1 + a.window - 1);
  const int q_lo = (m.k0 << a.hshift) / 128, q_hi = (((tmax + 1) << a.hshift) - 1) / 128;
  const int total = q_hi - q_lo + 1;
  const int per = (total + a.splits - 1) / a.splits;
  const int s0 = min(total, m.sp * per), s1 = min(total, s0 + per);
  m.q_lo = q_lo;
  m.total = total;
  m.s0 = s0;
  m.nq = s1 - s0;
  return m;
}

template <int D, bool SEP_V>
__global__ void __launch_bounds__(384, 1)
    dkv_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdo,
               const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv, Args a) {
  using C = KvCfg<D, SEP_V>;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* ks = smem;
  uint8_t* vs = SEP_V ? smem + C::T_BYTES : smem;
  uint8_t* st0 = smem + (SEP_V ? 2 : 1) * C::T_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::TILE_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::TILE_BYTES + 8 * KV_NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::TILE_BYTES + 8 * KV_NBAR + 4);
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) atomicExch(a.err, MZB_ERR_ALIGN);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < KV_NBAR; ++i) tc::mbar_init(&bars[i], (i == PT_FULL || i == PT_FULL1 || i == ACC_EMPTY) ? 4 : 1);
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, 512);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const int n_kt = (a.S + 127) / 128;
  const int items = a.B * n_kt * a.splits;
  auto stage = [&](int s) { return st0 + s * C::STAGE; };

  if (warp == 0) {
    if (lane == 0) {
      int g = 0, ii = 0;
      for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x) {
        const KvItem m = kv_item(a, it);
        if (m.nq == 0) continue;
        if (!tc::mbar_wait(&bars[KV_EMPTY], (ii & 1) ^ 1, a.err, 401)) { *abort_flag = 1; break; }
        ++ii;
        tc::mbar_expect_tx(&bars[KV_FULL], (SEP_V ? 2 : 1) * C::T_BYTES);
        for (int cb = 0; cb < C::DB; ++cb) {
          tc::tma_load_3d(ks + cb * 128 * 128, &tk, &bars[KV_FULL], cb * 64, m.k0, m.b);
          if (SEP_V) tc::tma_load_3d(vs + cb * 128 * 128, &tv, &bars[KV_FULL], cb * 64, m.k0, m.b);
        }
        bool ok = true;
        for (int i = 0; i < m.nq; ++i, ++g) {
          const int s = g % C::NST, ph = (g / C::NST) & 1;
          if (!tc::mbar_wait(&bars[QD_EMPTY + s], ph ^ 1, a.err, 402)) { ok = false; break; }
          uint8_t* sp = stage(s);
          const int qt = kv_qtile(m, i);
          tc::mbar_expect_tx(&bars[QD_FULL + s], 2 * C::T_BYTES + 1024);
          for (int cb = 0; cb < C::DB; ++cb) {
            tc::tma_load_3d(sp + cb * 128 * 128, &tq, &bars[QD_FULL + s], cb * 64, qt * 128, m.b);
            tc::tma_load_3d(sp + C::T_BYTES + cb * 128 * 128, &tdo, &bars[QD_FULL + s], cb * 64, qt * 128, m.b);
          }
          tc::bulk_load(sp + 2 * C::T_BYTES, a.lse2 + (long long)m.b * a.Rpad + qt * 128, 512, &bars[QD_FULL + s]);
          tc::bulk_load(sp + 2 * C::T_BYTES + 512, a.delta + (long long)m.b * a.Rpad + qt * 128, 512,
                        &bars[QD_FULL + s]);
        }
        if (!ok) { *abort_flag = 1; break; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // S^T / dP^T and the dV / dK MMAs go in query halves h (columns / rows [64 h, 64 h + 64)),
      // software-pipelined: for tile i the order is TS_lo(i), S_lo(i+1) + dP_lo(i+1),
      // TS_hi(i), S_hi(i+1) + dP_hi(i+1), so while one compute warpgroup turns its half of
      // tile i+1 into P^T / dS^T the tensor core runs the other half's MMAs.  Each S / dP
      // half MMA is issued after the TS MMAs that read that half's packed columns (one
      // thread, in order).
      const uint32_t idesc_s = tc::make_idesc(128, 64, 1, 1);
      const uint32_t idesc_acc = tc::make_idesc(128, D, 1, 1, false, true);
      const uint32_t k_base = smem_u32(ks), v_base = smem_u32(vs);
      const uint64_t kd = tc::make_sdesc<128>(k_base, 16, 1024), vd = tc::make_sdesc<128>(v_base, 16, 1024);
      // S^T(h) = K Q_h^T and dP^T(h) = V dO_h^T of stage s (query rows 64 h.. of the tile)
      auto issue_sdp = [&](int s, int h) {
        const uint32_t q_base = smem_u32(stage(s)), do_base = q_base + C::T_BYTES;
        const uint64_t qd = tc::make_sdesc<128>(q_base + h * 8192, 16, 1024);
        const uint64_t dod = tc::make_sdesc<128>(do_base + h * 8192, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int cb = kk >> 2, off = (kk & 3) * 32;
          tc::mma_ss<0>(tmem + C::C_S + 64 * h, tc::sdesc_add(kd, cb * 16384 + off),
                        tc::sdesc_add(qd, cb * 16384 + off), idesc_s, kk > 0);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int cb = kk >> 2, off = (kk & 3) * 32;
          tc::mma_ss<0>(tmem + C::C_DP + 64 * h, tc::sdesc_add(vd, cb * 16384 + off),
                        tc::sdesc_add(dod, cb * 16384 + off), idesc_s, kk > 0);
        }
        tc::mma_commit(&bars[S_FULL + h]);
      };
      // dV += P^T(h) dO_h, dK += dS^T(h) Q_h over the half's 64 query rows (16 per step)
      auto issue_ts = [&](int s, int h, bool first) {
        const uint32_t q_base = smem_u32(stage(s)), do_base = q_base + C::T_BYTES;
        const uint64_t q_mn = tc::make_sdesc<128>(q_base, 16384, 1024);
        const uint64_t do_mn = tc::make_sdesc<128>(do_base, 16384, 1024);
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          const int kk = 4 * h + k4;
          const uint32_t acc = (first && kk == 0) ? 0u : 1u;
          const int pc = pt_col(16 * kk);
          tc::mma_ts(tmem + C::C_DV, tmem + C::C_S + pc, tc::sdesc_add(do_mn, kk * 2048), idesc_acc, acc);
          tc::mma_ts(tmem + C::C_DK, tmem + C::C_DP + pc, tc::sdesc_add(q_mn, kk * 2048), idesc_acc,
                     C::MERGE ? 1u : acc);
        }
      };
      int g = 0, ii = -1;
      for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x) {
        const KvItem m = kv_item(a, it);
        if (m.nq == 0) continue;
        ++ii;
        if (!tc::mbar_wait(&bars[KV_FULL], ii & 1, a.err, 410)) { *abort_flag = 1; break; }
        bool ok = true;
        {  // both halves of the item's first tile
          const int s = g % C::NST, ph = (g / C::NST) & 1;
          if (!tc::mbar_wait(&bars[QD_FULL + s], ph, a.err, 411)) ok = false;
          if (ok) {
            tc::fence_after_sync();
            issue_sdp(s, 0);
            issue_sdp(s, 1);
          }
        }
        for (int i = 0; i < m.nq && ok; ++i, ++g) {
          const int s = g % C::NST;
          const int s1 = (g + 1) % C::NST, ph1 = ((g + 1) / C::NST) & 1;
          const bool more = i + 1 < m.nq;
          if (i == 0 && !tc::mbar_wait(&bars[ACC_EMPTY], (ii & 1) ^ 1, a.err, 412)) { ok = false; break; }
          if (!tc::mbar_wait(&bars[PT_FULL], g & 1, a.err, 413)) { ok = false; break; }  // half 0 of tile i
          tc::fence_after_sync();
          issue_ts(s, 0, i == 0);
          // with one Q / dO stage (D = 256) tile i + 1 loads only after this tile's TS MMAs
          // release the stage, so its S^T / dP^T wait for them
          if (more && C::NST > 1) {
            if (!tc::mbar_wait(&bars[QD_FULL + s1], ph1, a.err, 411)) { ok = false; break; }
            tc::fence_after_sync();
            issue_sdp(s1, 0);
          }
          if (!tc::mbar_wait(&bars[PT_FULL1], g & 1, a.err, 414)) { ok = false; break; }
          tc::fence_after_sync();
          issue_ts(s, 1, false);
          tc::mma_commit(&bars[QD_EMPTY + s]);
          if (more) {
            if (C::NST == 1) {
              if (!tc::mbar_wait(&bars[QD_FULL + s1], ph1, a.err, 411)) { ok = false; break; }
              tc::fence_after_sync();
              issue_sdp(s1, 0);
            }
            issue_sdp(s1, 1);
          }
          if (i == m.nq - 1) {
            tc::mma_commit(&bars[O_DONE]);
            tc::mma_commit(&bars[KV_EMPTY]);
          }
        }
        if (!ok) { *abort_flag = 1; break; }
      }
    }
  } else if (warp >= 4) {
    // two compute warpgroups on the same keys (TMEM lane = key within the tile, quarter =
    // warp % 4): warps 4-7 take query columns [0, 64), warps 8-11 [64, 128)
    const int sw = warp & 3, row = sw * 32 + lane;
    const bool second = warp >= 8;
    const int cbeg = second ? 64 : 0, cend = cbeg + 64;
    const float sl = a.scale_log2;
    int g = 0, ii = -1;
    for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x) {
      const KvItem m = kv_item(a, it);
      const int j = m.k0 + row;
      float* part = a.dkv_part + (((long long)m.sp * a.B + m.b) * a.S + j) * 2 * D;
      if (m.nq == 0) {  // this split has no query tiles: contribute zeros
        if (j < a.S && !second)
          for (int c = 0; c < 2 * D; c += 4) *reinterpret_cast<float4*>(part + c) = make_float4(0.f, 0.f, 0.f, 0.f);
        continue;
      }
      ++ii;
      bool ok = true;
      for (int i = 0; i < m.nq; ++i, ++g) {
        const int s = g % C::NST;
        if (!tc::mbar_wait(&bars[S_FULL + (second ? 1 : 0)], g & 1, a.err, 420)) { ok = false; break; }
        tc::fence_after_sync();
        const float* l2 = reinterpret_cast<const float*>(stage(s) + 2 * C::T_BYTES);
        const float* dl = l2 + 128;
        const int tb = (kv_qtile(m, i) * 128) >> a.hshift;  // token of column 0
        // key j is seen by the tile's columns (packed rows of tokens t, j <= t < j + window,
        // t < S): one run [clo, chi] of columns, turned into one mask word per 32 columns
        int clo = 1, chi = 0;
        if (j < a.S) {
          clo = (j - tb) * a.H;
          chi = (min(j + a.window - 1, a.S - 1) - tb + 1) * a.H - 1;
        }
        const bool warp_full = __all_sync(0xffffffffu, clo <= 0 && chi >= 127);
#pragma unroll 1
        for (int c0 = cbeg; c0 < cend; c0 += 32) {
          uint32_t sv[32], dv[32];
          tc::tmem_ld32(tc::taddr(tmem, sw * 32, C::C_S + c0), sv);
          tc::tmem_ld32(tc::taddr(tmem, sw * 32, C::C_DP + c0), dv);
          const uint32_t mw = warp_full ? 0xFFFFFFFFu : run_bits(clo - c0, chi - c0);
          const float4* l24 = reinterpret_cast<const float4*>(l2 + c0);
          const float4* dl4 = reinterpret_cast<const float4*>(dl + c0);
          tc::tmem_wait_ld();
          tc::reg_after_wait(sv);
          tc::reg_after_wait(dv);
          uint32_t pp[16], dd[16];
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4) {
            const float4 L = l24[q4], Dl = dl4[q4];
            const float lv[4] = {L.x, L.y, L.z, L.w}, dlv[4] = {Dl.x, Dl.y, Dl.z, Dl.w};
            float p2[4], d2[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int c = 4 * q4 + e;  // column within the chunk
              float p = fast_exp2(fmaf(__uint_as_float(sv[c]), sl, -lv[e]));
              if (!warp_full) p = (mw >> c) & 1u ? p : 0.0f;
              p2[e] = p;
              d2[e] = p * (__uint_as_float(dv[c]) - dlv[e]);
              if (C::MERGE) d2[e] *= a.scale;  // the merged accumulator takes scale * dS
            }
            pp[2 * q4] = pack_bf16(p2[0], p2[1]);
            pp[2 * q4 + 1] = pack_bf16(p2[2], p2[3]);
            dd[2 * q4] = pack_bf16(d2[0], d2[1]);
            dd[2 * q4 + 1] = pack_bf16(d2[2], d2[3]);
          }
          tc::tmem_st16(tc::taddr(tmem, sw * 32, C::C_S + pt_col(c0)), pp);
          tc::tmem_st16(tc::taddr(tmem, sw * 32, C::C_DP + pt_col(c0)), dd);
        }
        tc::tmem_wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bars[PT_FULL + (second ? 1 : 0)]);
      }
      if (!ok) { *abort_flag = 1; break; }
      if (second) continue;  // the first warpgroup writes the partial dK / dV
      if (!tc::mbar_wait(&bars[O_DONE], ii & 1, a.err, 421)) { *abort_flag = 1; break; }
      tc::fence_after_sync();
#pragma unroll 1
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t kv[32], vv[32];
        tc::tmem_ld32(tc::taddr(tmem, sw * 32, C::C_DK + c0), kv);
        if (!C::MERGE) tc::tmem_ld32(tc::taddr(tmem, sw * 32, C::C_DV + c0), vv);
        tc::tmem_wait_ld();
        if (C::MERGE) {  // dK + dV in one accumulator, the scale already applied: partial dV = 0
          if (j < a.S) {
#pragma unroll
            for (int q = 0; q < 32; q += 4) {
              *reinterpret_cast<float4*>(part + c0 + q) = make_float4(
                  __uint_as_float(kv[q]), __uint_as_float(kv[q + 1]), __uint_as_float(kv[q + 2]), __uint_as_float(kv[q + 3]));
              *reinterpret_cast<float4*>(part + D + c0 + q) = make_float4(0.f, 0.f, 0.f, 0.f);
            }
          }
        } else if (j < a.S) {
#pragma unroll
          for (int q = 0; q < 32; q += 4) {
            *reinterpret_cast<float4*>(part + c0 + q) =
                make_float4(__uint_as_float(kv[q]) * a.scale, __uint_as_float(kv[q + 1]) * a.scale,
                            __uint_as_float(kv[q + 2]) * a.scale, __uint_as_float(kv[q + 3]) * a.scale);
            *reinterpret_cast<float4*>(part + D + c0 + q) =
                make_float4(__uint_as_float(vv[q]), __uint_as_float(vv[q + 1]), __uint_as_float(vv[q + 2]),
                            __uint_as_float(vv[q + 3]));
          }
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&bars[ACC_EMPTY]);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_free(tmem, 512);
  }
}

// Sum the per-split partials in split order: dk = sum dK (+ sum dV when K == V), dv = sum dV.
__global__ void dkv_finalize_kernel(Args a, int sep_v) {
  const long long n = (long long)a.B * a.S * a.D;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / a.D;
    const int d = int(i % a.D);
    float k = 0.0f, v = 0.0f;
    for (int sp = 0; sp < a.splits; ++sp) {
      const float* p = a.dkv_part + ((long long)sp * a.B * a.S + row) * 2 * a.D;
      k += p[d];
      v += p[a.D + d];
    }
    if (sep_v) {
      a.dk[i] = __float2bfloat16_rn(k);
      a.dv[i] = __float2bfloat16_rn(v);
    } else {
      a.dk[i] = __float2bfloat16_rn(k + v);
    }
  }
}

// ------------------------------------------------------------------ dq (query owner)
template <int D, bool SEP_V>
struct QCfg {
  static constexpr int DB = D / 64;
  // D = 256: 64-key K/V tiles, and the gathered-row gradient is formed transposed (dM^T =
  // Q^T dS + dO^T P, d in the TMEM lanes, two 128-channel halves of KT columns) so that
  // the dQ accumulator (256 columns), S, dP and dM^T fit in TMEM together
  static constexpr bool WIDE = D == 256;
  static constexpr int KT = WIDE ? 64 : 128;     // keys per K/V tile
  static constexpr int T_BYTES = 128 * D * 2;    // Q / dO tile (128 packed rows)
  static constexpr int KV_BYTES = KT * D * 2;
  static constexpr int KV_STAGE = (SEP_V ? 2 : 1) * KV_BYTES;
  static constexpr int STAGES = 2;
  static constexpr int P_BYTES = 128 * KT * 2;   // dS / P tile [rows][KT keys] bf16 (gathered tiles)
  static constexpr int NP = SEP_V ? 0 : 2;       // dS and P copies (csa2 only)
  static constexpr int TILE_BYTES = 2 * T_BYTES + STAGES * KV_STAGE + NP * P_BYTES;
  static constexpr int SMEM = TILE_BYTES + 512;
  static constexpr int C_DQ = 0, C_S = D, C_DP = D + KT, C_DM = D + 2 * KT;
  // window-only (separate V): warps 8-11 are free, so the columns of each key tile are split
  // over two compute warpgroups, each packing its dS into the front of its own S half; the
  // unused dM columns hold the item's Q and dO rows (bf16 pairs), the TMEM A operands of the
  // S and dP MMAs, so shared memory carries only K / V operands for them and the Q / dO
  // buffer is free for the next item as soon as it has been copied
  static constexpr bool SPLIT = SEP_V;
  static constexpr int C_QT = C_DM, C_DOT = C_DM + D / 2;
  static_assert(C_DP + KT <= 512 && (SEP_V || C_DM + (WIDE ? 2 * KT : D) <= 512), "TMEM");
  static_assert(!SPLIT || C_DOT + D / 2 <= 512, "TMEM");
  static_assert(SMEM <= 232448, "smem");
  static_assert(!(WIDE && SEP_V), "a separate V needs D <= 128");
};

// S_FULL_Q / DS_FULL cover the whole key tile, or with SPLIT its first half of keys;
// S_FULL_Q1 / DS_FULL1 the second half, QT_FULL the item's Q / dO rows in TMEM (SPLIT only)
enum QBar { Q_FULL = 0, Q_EMPTY, S_FULL_Q, DS_FULL, DM_FULL, DM_EMPTY, QO_DONE, QACC_EMPTY, KVW_FULL,
            KVG_FULL = KVW_FULL + 2, KVQ_EMPTY = KVG_FULL + 2, S_FULL_Q1 = KVQ_EMPTY + 2, DS_FULL1, QT_FULL,
            Q_NBAR };

struct QItem {
  int b, qt, t0, t1, kt0, n_win, n_gat, gtiles, tq_valid;
};

template <int KT>
__device__ __forceinline__ QItem q_item(const Args& a, int it, int n_qt) {
  QItem m;
  m.b = it % a.B;
  m.qt = n_qt - 1 - it / a.B;
  const int tq = 128 / a.H;
  m.t0 = m.qt * tq;
  m.t1 = min(a.S, m.t0 + tq) - 1;
  m.tq_valid = m.t1 - m.t0 + 1;
  const int lo = max(0, m.t0 - a.window + 1);
  m.kt0 = lo / KT;
  m.n_win = m.t1 / KT - m.kt0 + 1;
  m.gtiles = (a.main_kv && a.topk > 0 && a.G > 0) ? (a.topk + KT - 1) / KT : 0;
  m.n_gat = m.gtiles * m.tq_valid;
  return m;
}

template <int D, bool SEP_V>
__global__ void __launch_bounds__(384, 1)
    dq_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdo,
              const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv, Args a) {
  using C = QCfg<D, SEP_V>;
  constexpr int KT = C::KT;
  constexpr int KB = KT * 128;  // bytes of one 64-channel column block of a K/V tile
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* qs = smem;
  uint8_t* dos = smem + C::T_BYTES;
  uint8_t* kvs = smem + 2 * C::T_BYTES;
  uint8_t* dss = kvs + C::STAGES * C::KV_STAGE;  // csa2: dS tile then P tile
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::TILE_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::TILE_BYTES + 8 * Q_NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::TILE_BYTES + 8 * Q_NBAR + 4);
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) atomicExch(a.err, MZB_ERR_ALIGN);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < Q_NBAR; ++i) {
      uint32_t c = 1;
      if (i == DS_FULL || i == DS_FULL1 || i == QT_FULL || i == DM_EMPTY || i == KVG_FULL || i == KVG_FULL + 1)
        c = 4;
      if (i == QACC_EMPTY) c = C::SPLIT ? 8 : 4;  // with SPLIT both warpgroups store half of dQ
      if (i == Q_EMPTY && C::SPLIT) c = 4;        // released by the warps that copy Q / dO to TMEM
      tc::mbar_init(&bars[i], c);
    }
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, 512);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const int tqn = 128 / a.H;
  const int n_qt = (a.S + tqn - 1) / tqn;
  const int items = a.B * n_qt;

  if (warp == 0) {
    if (lane == 0) {
      int g = 0, ii = 0;
      for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x, ++ii) {
        const QItem m = q_item<KT>(a, it, n_qt);
        if (!tc::mbar_wait(&bars[Q_EMPTY], (ii & 1) ^ 1, a.err, 501)) { *abort_flag = 1; break; }
        tc::mbar_expect_tx(&bars[Q_FULL], 2 * C::T_BYTES);
        for (int cb = 0; cb < C::DB; ++cb) {
          tc::tma_load_3d(qs + cb * 16384, &tq, &bars[Q_FULL], cb * 64, m.qt * 128, m.b);
          tc::tma_load_3d(dos + cb * 16384, &tdo, &bars[Q_FULL], cb * 64, m.qt * 128, m.b);
        }
        bool ok = true;
        for (int j = 0; j < m.n_win + m.n_gat; ++j, ++g) {
          const int st = g & 1, ph = (g >> 1) & 1;
          if (j >= m.n_win) continue;
          if (!tc::mbar_wait(&bars[KVQ_EMPTY + st], ph ^ 1, a.err, 502)) { ok = false; break; }
          uint8_t* kt = kvs + st * C::KV_STAGE;
          tc::mbar_expect_tx(&bars[KVW_FULL + st], C::KV_STAGE);
          for (int cb = 0; cb < C::DB; ++cb) {
            tc::tma_load_3d(kt + cb * KB, &tk, &bars[KVW_FULL + st], cb * 64, (m.kt0 + j) * KT, m.b);
            if (SEP_V)
              tc::tma_load_3d(kt + C::KV_BYTES + cb * KB, &tv, &bars[KVW_FULL + st], cb * 64, (m.kt0 + j) * KT, m.b);
          }
        }
        if (!ok) { *abort_flag = 1; break; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc_s = tc::make_idesc(128, KT, 1, 1);
      const uint32_t idesc_dq = tc::make_idesc(128, D, 1, 1, false, true);
      const uint32_t idesc_dm = tc::make_idesc(128, C::WIDE ? KT : D, 1, 1, true, true);
      const uint32_t q_base = smem_u32(qs), do_base = smem_u32(dos), kv_base = smem_u32(kvs);
      const uint32_t ds_base = smem_u32(dss), p_base = ds_base + C::P_BYTES;
      int g = 0, ii = 0, gm = 0;
      int uses_w[2] = {0, 0}, uses_g[2] = {0, 0};
      for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x, ++ii) {
        const QItem m = q_item<KT>(a, it, n_qt);
        const int n = m.n_win + m.n_gat;
        if (!tc::mbar_wait(&bars[C::SPLIT ? QT_FULL : Q_FULL], ii & 1, a.err, 510)) { *abort_flag = 1; break; }
        bool ok = true;
        if constexpr (C::SPLIT) {
          // window tiles only (a separate V excludes gathered rows).  S / dP and dQ += dS K run
          // in halves of KT / 2 keys, one per compute warpgroup; the next tile's S / dP half is
          // issued as soon as its warpgroup has packed dS of this tile, so it computes while
          // the other warpgroup works
          const uint32_t idesc_h = tc::make_idesc(128, KT / 2, 1, 1);
          tc::fence_after_sync();
          auto kv_wait = [&](int gg) {
            if (!tc::mbar_wait(&bars[KVW_FULL + (gg & 1)], (gg >> 1) & 1, a.err, 511)) return false;
            tc::fence_after_sync();
            return true;
          };
          auto issue_s = [&](int gg, int h) {
            const uint32_t kb = kv_base + (gg & 1) * C::KV_STAGE + h * (KT / 2) * 128;
            const uint64_t kd = tc::make_sdesc<128>(kb, 16, 1024), vd = tc::make_sdesc<128>(kb + C::KV_BYTES, 16, 1024);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const int cb = kk >> 2, off = (kk & 3) * 32;
              tc::mma_ts(tmem + C::C_S + h * (KT / 2), tmem + C::C_QT + kk * 8, tc::sdesc_add(kd, cb * KB + off),
                         idesc_h, kk > 0 ? 1u : 0u);
            }
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const int cb = kk >> 2, off = (kk & 3) * 32;
              tc::mma_ts(tmem + C::C_DP + h * (KT / 2), tmem + C::C_DOT + kk * 8, tc::sdesc_add(vd, cb * KB + off),
                         idesc_h, kk > 0 ? 1u : 0u);
            }
            tc::mma_commit(&bars[h ? S_FULL_Q1 : S_FULL_Q]);
          };
          auto issue_dq = [&](int gg, int h, bool first) {
            const uint64_t k_mn = tc::make_sdesc<128>(kv_base + (gg & 1) * C::KV_STAGE, KB, 1024);
#pragma unroll
            for (int k4 = 0; k4 < KT / 32; ++k4) {  // 16 keys per step; half h's packed dS columns
              const uint32_t ds_col = C::C_S + h * (KT / 2) + k4 * 8;
              tc::mma_ts(tmem + C::C_DQ, tmem + ds_col, tc::sdesc_add(k_mn, (h * (KT / 32) + k4) * 2048), idesc_dq,
                         (first && k4 == 0) ? 0u : 1u);
            }
          };
          if (n > 0) {
            if (kv_wait(g)) {
              issue_s(g, 0);
              issue_s(g, 1);
            } else {
              ok = false;
            }
          }
          for (int j = 0; ok && j < n; ++j, ++g) {
            const bool more = j + 1 < n;
            if (j == 0 && !tc::mbar_wait(&bars[QACC_EMPTY], (ii & 1) ^ 1, a.err, 512)) { ok = false; break; }
            if (!tc::mbar_wait(&bars[DS_FULL], g & 1, a.err, 513)) { ok = false; break; }
            tc::fence_after_sync();
            issue_dq(g, 0, j == 0);
            if (more) {
              if (!kv_wait(g + 1)) { ok = false; break; }
              issue_s(g + 1, 0);
            }
            if (!tc::mbar_wait(&bars[DS_FULL1], g & 1, a.err, 515)) { ok = false; break; }
            tc::fence_after_sync();
            issue_dq(g, 1, false);
            tc::mma_commit(&bars[KVQ_EMPTY + (g & 1)]);
            if (more)
              issue_s(g + 1, 1);
            else
              tc::mma_commit(&bars[QO_DONE]);
          }
          if (!ok) { *abort_flag = 1; break; }
          continue;
        }
        for (int j = 0; j < n; ++j, ++g) {
          const int st = g & 1;
          const bool win = j < m.n_win;
          const int par = win ? (uses_w[st]++ & 1) : (uses_g[st]++ & 1);
          if (!tc::mbar_wait(&bars[(win ? KVW_FULL : KVG_FULL) + st], par, a.err, 511)) { ok = false; break; }
          tc::fence_after_sync();
          const uint32_t kb = kv_base + st * C::KV_STAGE, vb = kb + (SEP_V ? C::KV_BYTES : 0);
          // descriptors once per tile; the unrolled loops add constant offsets
          const uint64_t qd = tc::make_sdesc<128>(q_base, 16, 1024), dod = tc::make_sdesc<128>(do_base, 16, 1024);
          const uint64_t kd = tc::make_sdesc<128>(kb, 16, 1024), vd = tc::make_sdesc<128>(vb, 16, 1024);
          const uint64_t k_mn = tc::make_sdesc<128>(kb, KB, 1024);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int cb = kk >> 2, off = (kk & 3) * 32;
            tc::mma_ss<0>(tmem + C::C_S, tc::sdesc_add(qd, cb * 16384 + off), tc::sdesc_add(kd, cb * KB + off),
                          idesc_s, kk > 0);
          }
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int cb = kk >> 2, off = (kk & 3) * 32;
            tc::mma_ss<0>(tmem + C::C_DP, tc::sdesc_add(dod, cb * 16384 + off), tc::sdesc_add(vd, cb * KB + off),
                          idesc_s, kk > 0);
          }
          tc::mma_commit(&bars[S_FULL_Q]);
          if (j == 0 && !tc::mbar_wait(&bars[QACC_EMPTY], (ii & 1) ^ 1, a.err, 512)) { ok = false; break; }
          if (!tc::mbar_wait(&bars[DS_FULL], g & 1, a.err, 513)) { ok = false; break; }
          tc::fence_after_sync();
#pragma unroll
          for (int kk = 0; kk < KT / 16; ++kk) {  // KT keys, 16 per step: dQ += dS K
            const uint32_t ds_col = C::C_S + kk * 8;  // (SPLIT kernels take the pipelined path above)
            tc::mma_ts(tmem + C::C_DQ, tmem + ds_col, tc::sdesc_add(k_mn, kk * 2048), idesc_dq,
                       (j == 0 && kk == 0) ? 0u : 1u);
          }
          if (!win) {
            if (!tc::mbar_wait(&bars[DM_EMPTY], (gm & 1) ^ 1, a.err, 514)) { ok = false; break; }
            const uint64_t ds_mn = tc::make_sdesc<128>(ds_base, 16384, 1024);
            const uint64_t p_mn = tc::make_sdesc<128>(p_base, 16384, 1024);
            const uint64_t q_mn = tc::make_sdesc<128>(q_base, 16384, 1024);
            const uint64_t do_mn = tc::make_sdesc<128>(do_base, 16384, 1024);
            if (C::WIDE) {
              // dM^T[d, key] for d in half h: A = Q^T / dO^T (channels 128h.., MN-major),
              // B = dS / P [rows][keys] (MN-major), K = the 128 query rows
#pragma unroll
              for (int h = 0; h < 2; ++h) {
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                  tc::mma_ss<0>(tmem + C::C_DM + h * KT, tc::sdesc_add(q_mn, 2 * h * 16384 + kk * 2048),
                                tc::sdesc_add(ds_mn, kk * 2048), idesc_dm, kk > 0);
                  tc::mma_ss<0>(tmem + C::C_DM + h * KT, tc::sdesc_add(do_mn, 2 * h * 16384 + kk * 2048),
                                tc::sdesc_add(p_mn, kk * 2048), idesc_dm, 1u);
                }
              }
            } else {
#pragma unroll
              for (int kk = 0; kk < 8; ++kk) {  // 128 query rows: dM = dS^T Q + P^T dO
                tc::mma_ss<0>(tmem + C::C_DM, tc::sdesc_add(ds_mn, kk * 2048), tc::sdesc_add(q_mn, kk * 2048), idesc_dm,
                              kk > 0);
                tc::mma_ss<0>(tmem + C::C_DM, tc::sdesc_add(p_mn, kk * 2048), tc::sdesc_add(do_mn, kk * 2048), idesc_dm,
                              1u);
              }
            }
            tc::mma_commit(&bars[DM_FULL]);
            ++gm;
          }
          tc::mma_commit(&bars[KVQ_EMPTY + st]);
          if (j == n - 1) {
            tc::mma_commit(&bars[Q_EMPTY]);
            tc::mma_commit(&bars[QO_DONE]);
          }
        }
        if (!ok) { *abort_flag = 1; break; }
      }
    }
  } else if ((warp >= 4 && warp < 8) || (C::SPLIT && warp >= 8)) {
    // compute warps: rows r of the tile (TMEM lane quarter = warp % 4); with SPLIT the first
    // warpgroup takes key columns [0, KT/2) and the second [KT/2, KT)
    const int sw = warp & 3, r = sw * 32 + lane;
    const bool second = C::SPLIT && warp >= 8;
    const int cbeg = second ? KT / 2 : 0, cend = (C::SPLIT && !second) ? KT / 2 : KT;
    const float sl = a.scale_log2;
    // dQ columns [c_lo, c_hi) of item mm (index iim) -> bf16 rows; frees the accumulator
    auto store_dq = [&](const QItem& mm, int iim, int c_lo, int c_hi) {
      if (!tc::mbar_wait(&bars[QO_DONE], iim & 1, a.err, 522)) return false;
      tc::fence_after_sync();
      const bool ok_row = mm.t0 + r / a.H < a.S;
      const long long grow = (long long)mm.qt * 128 + r;
#pragma unroll 1
      for (int c0 = c_lo; c0 < c_hi; c0 += 32) {
        uint32_t qv[32];
        tc::tmem_ld32(tc::taddr(tmem, sw * 32, C::C_DQ + c0), qv);
        tc::tmem_wait_ld();
        if (ok_row) {
          uint4* dst = reinterpret_cast<uint4*>(a.dq + ((long long)mm.b * a.S * a.H + grow) * D + c0);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            dst[q] = make_uint4(pack_bf16(__uint_as_float(qv[8 * q]) * a.scale, __uint_as_float(qv[8 * q + 1]) * a.scale),
                                pack_bf16(__uint_as_float(qv[8 * q + 2]) * a.scale, __uint_as_float(qv[8 * q + 3]) * a.scale),
                                pack_bf16(__uint_as_float(qv[8 * q + 4]) * a.scale, __uint_as_float(qv[8 * q + 5]) * a.scale),
                                pack_bf16(__uint_as_float(qv[8 * q + 6]) * a.scale, __uint_as_float(qv[8 * q + 7]) * a.scale));
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&bars[QACC_EMPTY]);
      return true;
    };
    // SPLIT: row r of a 128-row bf16 tile in shared memory (64-channel blocks of 128-byte rows,
    // 16-byte chunks swizzled by r % 8) -> TMEM lane r, columns col.. as bf16 pairs
    auto rows_to_tmem = [&](const uint8_t* src, int col) {
#pragma unroll
      for (int cb = 0; cb < C::DB; ++cb) {
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          uint32_t v[16];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int ch = h2 * 4 + c;
            const uint4 x = ld_shared16(src + cb * 16384 + r * 128 + ((ch ^ (r & 7)) * 16));
            v[4 * c] = x.x;
            v[4 * c + 1] = x.y;
            v[4 * c + 2] = x.z;
            v[4 * c + 3] = x.w;
          }
          tc::tmem_st16(tc::taddr(tmem, sw * 32, col + cb * 32 + h2 * 16), v);
        }
      }
    };
    QItem prev{};
    int g = 0, ii = 0, gm = 0;
    for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x, ++ii) {
      const QItem m = q_item<KT>(a, it, n_qt);
      const int n = m.n_win + m.n_gat;
      const int tr = r / a.H, t = m.t0 + tr;
      const bool row_ok = t < a.S;
      const long long grow = (long long)m.qt * 128 + r;
      const float l2 = a.lse2[(long long)m.b * a.Rpad + grow];
      const float dl = a.delta[(long long)m.b * a.Rpad + grow];
      if (C::SPLIT && second) {
        // this item's Q and dO rows into TMEM: every S / dP MMA of the previous item has
        // completed (this warpgroup saw its last S_FULL_Q1), and the shared-memory buffer is
        // released for the next item's rows at once; then the previous item's upper dQ half
        if (!tc::mbar_wait(&bars[Q_FULL], ii & 1, a.err, 523)) { *abort_flag = 1; break; }
        tc::fence_after_sync();
        rows_to_tmem(qs, C::C_QT);
        rows_to_tmem(dos, C::C_DOT);
        tc::tmem_wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) {
          tc::mbar_arrive(&bars[QT_FULL]);
          tc::mbar_arrive(&bars[Q_EMPTY]);
        }
        if (ii > 0 && !store_dq(prev, ii - 1, D / 2, D)) { *abort_flag = 1; break; }
      }
      bool ok = true;
      for (int j = 0; j < n; ++j, ++g) {
        const bool win = j < m.n_win;
        int k0 = 0, wlo = 0, whi = -1, gtok = -1, e0 = 0;
        uint32_t gmask[KT / 32];
#pragma unroll
        for (int w = 0; w < KT / 32; ++w) gmask[w] = 0u;
        if (win) {
          k0 = (m.kt0 + j) * KT;
          wlo = max(0, t - a.window + 1) - k0;
          whi = t - k0;
        } else {
          const int gj = j - m.n_win;
          gtok = gj / m.gtiles;
          e0 = (gj % m.gtiles) * KT;
          const int32_t* irow = a.idx + ((long long)m.b * a.S + (m.t0 + gtok)) * a.topk;
#pragma unroll
          for (int w = 0; w < KT / 32; ++w) {
            const int e = e0 + w * 32 + lane;
            bool v = false;
            if (e < a.topk) {
              const int gi = irow[e];
              v = gi >= 0 && gi < a.G;
            }
            gmask[w] = __ballot_sync(0xffffffffu, v);
          }
        }
        const bool full = row_ok && win && wlo <= 0 && whi >= KT - 1;
        const bool warp_full = __all_sync(0xffffffffu, full);
        if (!tc::mbar_wait(&bars[second ? S_FULL_Q1 : S_FULL_Q], g & 1, a.err, 520)) { ok = false; break; }
        tc::fence_after_sync();
if constexpr (C::SPLIT) {
          // window tiles only: both 32-column chunks of this warpgroup's key half in flight at
          // once, so the half costs one TMEM load round trip (this step is on the critical
          // path between the two halves' MMAs)
          uint32_t sv0[32], dv0[32], sv1[32], dv1[32];
          tc::tmem_ld32(tc::taddr(tmem, sw * 32, C::C_S + cbeg), sv0);
          tc::tmem_ld32(tc::taddr(tmem, sw * 32, C::C_DP + cbeg), dv0);
          tc::tmem_ld32(tc::taddr(tmem, sw * 32, C::C_S + cbeg + 32), sv1);
          tc::tmem_ld32(tc::taddr(tmem, sw * 32, C::C_DP + cbeg + 32), dv1);
          uint32_t mw0 = 0xFFFFFFFFu, mw1 = 0xFFFFFFFFu;
          if (!warp_full) {
            mw0 = row_ok ? run_bits(wlo - cbeg, whi - cbeg) : 0u;
            mw1 = row_ok ? run_bits(wlo - cbeg - 32, whi - cbeg - 32) : 0u;
          }
          tc::tmem_wait_ld();
          tc::reg_after_wait(sv0);
          tc::reg_after_wait(dv0);
          tc::reg_after_wait(sv1);
          tc::reg_after_wait(dv1);
          auto chunk = [&](const int c0, const uint32_t mw, uint32_t(&sv)[32], uint32_t(&dv)[32]) {
            uint32_t dd[16];
#pragma unroll
            for (int q = 0; q < 16; ++q) {
              const int c = 2 * q;
              const float p0 = (mw >> c) & 1u ? fast_exp2(fmaf(__uint_as_float(sv[c]), sl, -l2)) : 0.0f;
              const float p1 = (mw >> (c + 1)) & 1u ? fast_exp2(fmaf(__uint_as_float(sv[c + 1]), sl, -l2)) : 0.0f;
              dd[q] = pack_bf16(p0 * (__uint_as_float(dv[c]) - dl), p1 * (__uint_as_float(dv[c + 1]) - dl));
            }
            tc::tmem_st16(tc::taddr(tmem, sw * 32, second ? C::C_S + KT / 2 + (c0 - KT / 2) / 2 : C::C_S + c0 / 2), dd);
          };
          chunk(cbeg, mw0, sv0, dv0);
          chunk(cbeg + 32, mw1, sv1, dv1);
        } else {
  #pragma unroll 1
          for (int c0 = cbeg; c0 < cend; c0 += 32) {
            uint32_t sv[32], dv[32];
            tc::tmem_ld32(tc::taddr(tmem, sw * 32, C::C_S + c0), sv);
            tc::tmem_ld32(tc::taddr(tmem, sw * 32, C::C_DP + c0), dv);
            // this row's valid columns of the chunk as bits (window run, or its gathered slots)
            uint32_t mw = 0xFFFFFFFFu;
            if (!warp_full) {
              mw = 0u;
              if (row_ok) mw = win ? run_bits(wlo - c0, whi - c0) : (tr == gtok ? gmask[c0 >> 5] : 0u);
            }
            tc::tmem_wait_ld();
            tc::reg_after_wait(sv);
            tc::reg_after_wait(dv);
            // P and dS overwrite S and dP in place; only gathered tiles pack the extra copies
  #pragma unroll
            for (int c = 0; c < 32; ++c) {
              const float p = (mw >> c) & 1u ? fast_exp2(fmaf(__uint_as_float(sv[c]), sl, -l2)) : 0.0f;
              sv[c] = __float_as_uint(p);
              dv[c] = __float_as_uint(p * (__uint_as_float(dv[c]) - dl));
            }
            uint32_t dd[16];
  #pragma unroll
            for (int q = 0; q < 16; ++q) dd[q] = pack_bf16(__uint_as_float(dv[2 * q]), __uint_as_float(dv[2 * q + 1]));
            tc::tmem_st16(tc::taddr(tmem, sw * 32, second ? C::C_S + KT / 2 + (c0 - KT / 2) / 2 : C::C_S + c0 / 2), dd);
            if (!win) {  // keep scale*dS (dK carries the softmax scale) and P in smem for the gathered-row gradient
              uint8_t* dsr = dss + (c0 >> 6) * 16384 + r * 128;
              uint8_t* pr = dsr + C::P_BYTES;
              auto ds2 = [&](int c) {
                return pack_bf16(__uint_as_float(dv[c]) * a.scale, __uint_as_float(dv[c + 1]) * a.scale);
              };
              auto pp2 = [&](int c) { return pack_bf16(__uint_as_float(sv[c]), __uint_as_float(sv[c + 1])); };
  #pragma unroll
              for (int q = 0; q < 4; ++q) {
                const int ch = ((c0 & 63) >> 3) + q;
                const int c = 8 * q;
                st_shared16(dsr + ((ch ^ (r & 7)) * 16), make_uint4(ds2(c), ds2(c + 2), ds2(c + 4), ds2(c + 6)));
                st_shared16(pr + ((ch ^ (r & 7)) * 16), make_uint4(pp2(c), pp2(c + 2), pp2(c + 4), pp2(c + 6)));
              }
            }
          }
        }
        tc::tmem_wait_st();
        if (!win) tc::fence_async_smem();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bars[second ? DS_FULL1 : DS_FULL]);
        if (!win && !second) {
          if (!tc::mbar_wait(&bars[DM_FULL], gm & 1, a.err, 521)) { ok = false; break; }
          tc::fence_after_sync();
          if (C::WIDE) {
            // dM^T (thread = channel d of each half, column = key slot) -> fp32 atomics into
            // dmain; the 32 lanes of a warp add to 32 consecutive channels of one row
            const int32_t* irow = a.idx + ((long long)m.b * a.S + (m.t0 + gtok)) * a.topk;
            int gl[KT / 32];
#pragma unroll
            for (int w = 0; w < KT / 32; ++w) {
              const int e = e0 + w * 32 + lane;
              gl[w] = e < a.topk ? irow[e] : -1;
            }
#pragma unroll 1
            for (int h = 0; h < 2; ++h) {
              const int d = h * 128 + sw * 32 + lane;
#pragma unroll 1
              for (int c0 = 0; c0 < KT; c0 += 32) {
                uint32_t mv[32];
                tc::tmem_ld32(tc::taddr(tmem, sw * 32, C::C_DM + h * KT + c0), mv);
                tc::tmem_wait_ld();
#pragma unroll
                for (int q = 0; q < 32; ++q) {
                  const int gi = __shfl_sync(0xffffffffu, gl[c0 >> 5], q);
                  if (gi >= 0 && gi < a.G) atomicAdd(a.dmain + ((long long)m.b * a.G + gi) * D + d, __uint_as_float(mv[q]));
                }
              }
            }
          } else {
            // dM rows (thread = key slot of the tile) -> fp32 atomics into dmain
            const int e = e0 + r;
            int gi = -1;
            if (e < a.topk) gi = a.idx[((long long)m.b * a.S + (m.t0 + gtok)) * a.topk + e];
            const bool v = gi >= 0 && gi < a.G;
            float* dst = a.dmain + ((long long)m.b * a.G + (v ? gi : 0)) * D;
#pragma unroll 1
            for (int c0 = 0; c0 < D; c0 += 32) {
              uint32_t mv[32];
              tc::tmem_ld32(tc::taddr(tmem, sw * 32, C::C_DM + c0), mv);
              tc::tmem_wait_ld();
              if (v) {
#pragma unroll
                for (int q = 0; q < 32; ++q) atomicAdd(dst + c0 + q, __uint_as_float(mv[q]));
              }
            }
          }
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&bars[DM_EMPTY]);
          ++gm;
        }
      }
      if (!ok) { *abort_flag = 1; break; }
      if (second) {  // the upper dQ half of this item is stored at the start of the next one
        prev = m;
        continue;
      }
      if (!store_dq(m, ii, 0, C::SPLIT ? D / 2 : D)) { *abort_flag = 1; break; }
    }
    // the last item's upper dQ half
    if (C::SPLIT && second && ii > 0 && !*abort_flag && !store_dq(prev, ii - 1, D / 2, D)) *abort_flag = 1;
  } else if (warp >= 8) {
    // gathered-row producers (csa2): main_kv rows -> the K stage (K == V)
    const int t = threadIdx.x - 256, row = t;  // 128 rows, one per thread
    int g = 0;
    for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x) {
      const QItem m = q_item<KT>(a, it, n_qt);
      const int n = m.n_win + m.n_gat;
      bool ok = true;
      for (int j = 0; j < n; ++j, ++g) {
        if (j < m.n_win) continue;
        const int st = g & 1, ph = (g >> 1) & 1;
        // KT rows of D channels: 128 / KT threads per row, 16-byte vectors [q0, q0 + NQ)
        constexpr int TPR = 128 / KT, NQ = D / 8 / TPR;
        const int kr = row / TPR, q0 = (row % TPR) * NQ;
        const int gj = j - m.n_win, gtok = gj / m.gtiles, e = (gj % m.gtiles) * KT + kr;
        int gi = -1;
        if (e < a.topk) gi = a.idx[((long long)m.b * a.S + (m.t0 + gtok)) * a.topk + e];
        const bool v = gi >= 0 && gi < a.G;
        const uint4* src = reinterpret_cast<const uint4*>(a.main_kv + ((long long)m.b * a.G + (v ? gi : 0)) * D) + q0;
        uint4 raw[NQ];
#pragma unroll
        for (int q = 0; q < NQ; ++q) raw[q] = v ? __ldg(src + q) : make_uint4(0, 0, 0, 0);
        if (!tc::mbar_wait(&bars[KVQ_EMPTY + st], ph ^ 1, a.err, 530)) { ok = false; break; }
        uint8_t* kt = kvs + st * C::KV_STAGE;
#pragma unroll
        for (int qq = 0; qq < NQ; ++qq) {
          const int q = q0 + qq;
          st_shared16(kt + (q >> 3) * KB + kr * 128 + (((q & 7) ^ (kr & 7)) * 16), raw[qq]);
        }
        tc::fence_async_smem();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bars[KVG_FULL + st]);
      }
      if (!ok) { *abort_flag = 1; break; }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_free(tmem, 512);
  }
}

template <int D, bool SEP_V>
int launch(const void* q, const void* kv, const void* v, const Args& a, cudaStream_t st) {
  CUtensorMap tq, tdo, tk, tv;
  const uint32_t box[3] = {64, 128, 1};
  {
    const uint64_t dims[3] = {uint64_t(D), uint64_t(a.S) * a.H, uint64_t(a.B)};
    const uint64_t str[2] = {uint64_t(D) * 2, uint64_t(a.S) * a.H * D * 2};
    if (int r = encode_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, q, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return r;
    if (int r = encode_tmap(&tdo, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a.dout, dims, str, box,
                            CU_TENSOR_MAP_SWIZZLE_128B))
      return r;
  }
  {
    const uint64_t dims[3] = {uint64_t(D), uint64_t(a.S), uint64_t(a.B)};
    const uint64_t str[2] = {uint64_t(D) * 2, uint64_t(a.S) * D * 2};
    if (int r = encode_tmap(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, kv, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return r;
    if (int r = encode_tmap(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, SEP_V ? v : kv, dims, str, box,
                            CU_TENSOR_MAP_SWIZZLE_128B))
      return r;
  }
  const long long rows = (long long)a.B * a.Rpad;
  preprocess_kernel<D><<<unsigned((rows * 4 + 255) / 256), 256, 0, st>>>(a);
  if (int r = launch_status("attn_bwd_preprocess")) return r;

  auto kkv = dkv_kernel<D, SEP_V>;
  if (cudaFuncSetAttribute(kkv, cudaFuncAttributeMaxDynamicSharedMemorySize, KvCfg<D, SEP_V>::SMEM) != cudaSuccess)
    return launch_status("attn_bwd_dkv(smem attr)");
  const int kv_items = a.B * ((a.S + 127) / 128) * a.splits;
  kkv<<<kv_items < num_sms() ? kv_items : num_sms(), 384, KvCfg<D, SEP_V>::SMEM, st>>>(tq, tdo, tk, tv, a);
  if (int r = launch_status("attn_bwd_dkv")) return r;
  {
    const long long n = (long long)a.B * a.S * a.D;
    long long blocks = (n + 255) / 256;
    if (blocks > 8LL * num_sms()) blocks = 8LL * num_sms();
    dkv_finalize_kernel<<<unsigned(blocks), 256, 0, st>>>(a, SEP_V ? 1 : 0);
    if (int r = launch_status("attn_bwd_dkv_finalize")) return r;
  }

  auto kq = dq_kernel<D, SEP_V>;
  if (cudaFuncSetAttribute(kq, cudaFuncAttributeMaxDynamicSharedMemorySize, QCfg<D, SEP_V>::SMEM) != cudaSuccess)
    return launch_status("attn_bwd_dq(smem attr)");
  constexpr int KT = QCfg<D, SEP_V>::KT;
  if (KT != 128) {  // the query-owner kernel reads KT-row K / V tiles
    const uint32_t kbox[3] = {64, uint32_t(KT), 1};
    const uint64_t dims[3] = {uint64_t(D), uint64_t(a.S), uint64_t(a.B)};
    const uint64_t str[2] = {uint64_t(D) * 2, uint64_t(a.S) * D * 2};
    if (int r = encode_tmap(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, kv, dims, str, kbox, CU_TENSOR_MAP_SWIZZLE_128B))
      return r;
    if (int r = encode_tmap(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, SEP_V ? v : kv, dims, str, kbox,
                            CU_TENSOR_MAP_SWIZZLE_128B))
      return r;
  }
  const int tqn = 128 / a.H;
  const int q_items = a.B * ((a.S + tqn - 1) / tqn);
  kq<<<q_items < num_sms() ? q_items : num_sms(), 384, QCfg<D, SEP_V>::SMEM, st>>>(tq, tdo, tk, tv, a);
  return launch_status("attn_bwd_dq");
}

}  // namespace attnb
}  // namespace mzb

using namespace mzb;

extern "C" int mzb_attn_bwd_splits(int64_t B, int64_t S, int H, int window) {
  // query-loop splits of the key-owner kernel: ~4 items per SM (the reference targets 768
  // CTAs, swa_attn/bwd.py:57-76), at most 16, never more than the query tiles of a key tile
  const int n_kt = int((S + 127) / 128);
  const long long q_tiles = ((long long)(127 + window) * H + 127) / 128 + 1;
  int sp = int((4LL * num_sms() + B * n_kt - 1) / (B * n_kt));
  if (sp > 16) sp = 16;
  if (sp > q_tiles) sp = int(q_tiles);
  return sp < 1 ? 1 : sp;
}

extern "C" int mzb_attn_bwd(const void* q, const void* kv, const void* v, const void* main_kv, const int32_t* indices,
                            const void* o, const float* lse, const void* dout, void* dq, void* dk, void* dv,
                            float* dmain_f32, float* delta_ws, float* lse2_ws, float* dkv_part_ws, int splits,
                            int64_t B, int64_t S, int H, int D, int window, int64_t G, int topk, float softmax_scale,
                            int* err, void* stream) {
  MZB_REQUIRE(B >= 1 && S >= 1 && window >= 1 && topk >= 0 && G >= 0, MZB_ERR_SHAPE, "attn_bwd: bad sizes");
  MZB_REQUIRE(H >= 1 && H <= 128 && 128 % H == 0, MZB_ERR_UNSUPPORTED, "attn_bwd: heads must divide 128, got %d",
              H);
  MZB_REQUIRE(D == 64 || D == 128 || D == 256, MZB_ERR_UNSUPPORTED, "attn_bwd: head dim %d not built (64, 128, 256)",
              D);
  const bool sep = v != nullptr && v != kv;
  MZB_REQUIRE(!(sep && D == 256), MZB_ERR_UNSUPPORTED, "attn_bwd: a separate V needs head dim <= 128");
  const bool gathered = main_kv != nullptr && topk > 0 && G > 0;
  MZB_REQUIRE(!(sep && gathered), MZB_ERR_UNSUPPORTED, "attn_bwd: a separate V only for the window-only kernel");
  MZB_REQUIRE(!gathered || dmain_f32 != nullptr, MZB_ERR_SHAPE, "attn_bwd: gathered rows need a dmain accumulator");
  MZB_REQUIRE(err && delta_ws && lse2_ws && dkv_part_ws, MZB_ERR_SHAPE, "attn_bwd: needs err and workspaces");
  MZB_REQUIRE(splits >= 1 && splits <= 64, MZB_ERR_SHAPE, "attn_bwd: splits must be in [1, 64], got %d", splits);
  attnb::Args a{};
  a.o = static_cast<const __nv_bfloat16*>(o);
  a.dout = static_cast<const __nv_bfloat16*>(dout);
  a.lse = lse;
  a.delta = delta_ws;
  a.lse2 = lse2_ws;
  a.main_kv = gathered ? static_cast<const __nv_bfloat16*>(main_kv) : nullptr;
  a.idx = gathered ? indices : nullptr;
  a.dq = static_cast<__nv_bfloat16*>(dq);
  a.dk = static_cast<__nv_bfloat16*>(dk);
  a.dv = sep ? static_cast<__nv_bfloat16*>(dv) : nullptr;
  a.dmain = gathered ? dmain_f32 : nullptr;
  a.B = int(B); a.S = int(S); a.H = H; a.D = D; a.window = window; a.G = gathered ? int(G) : 0;
  a.topk = gathered ? topk : 0;
  a.Rpad = int(((S * H + 127) / 128) * 128);
  a.dkv_part = dkv_part_ws;
  a.splits = splits;
  a.hshift = __builtin_ctz(unsigned(H));
  a.scale = softmax_scale;
  a.scale_log2 = softmax_scale * attnb::LOG2E;
  a.err = err;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (D == 64) return sep ? attnb::launch<64, true>(q, kv, v, a, st) : attnb::launch<64, false>(q, kv, v, a, st);
  if (D == 256) return attnb::launch<256, false>(q, kv, v, a, st);
  return sep ? attnb::launch<128, true>(q, kv, v, a, st) : attnb::launch<128, false>(q, kv, v, a, st);
}
