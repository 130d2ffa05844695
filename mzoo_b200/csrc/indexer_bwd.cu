// Lightning-indexer backward (bf16 q/k, fp32 w and dL): dq, dk, dw.
//
// Reference: src/mzoo/layers/attn/indexer/bwd.py:38-133 (`index_score_bwd`, `bwd`):
//   r = q . k (recomputed), d = dL masked to the group-causal visible keys (masked entries
//   contribute nothing whatever they hold), scale = Di^-1/2:
//   dw[s,h] = sum_t relu(r) * scale * d,   dr = d * w * scale * [r > 0],
//   dq[s,h,:] = sum_t dr * k[t,:],          dk[t,:] = sum_{s,h} dr * q[s,h,:]
//
// Two tcgen05 kernels, both with keys in the MMA M dimension and (token, head) query rows
// in N exactly like the forward score kernel (indexer.cu):
//   dq_dw   query owner: per key tile R = K Q^T in TMEM; the epilogue warps (thread = key)
//           form dr and the relu-weighted dL, reduce dw over keys with warp reduce-scatter
//           + shared-memory atomics, and stage dr (bf16) in shared memory so that
//           dq += dr^T K runs as two M=128 MMAs with an MN-major A operand.
//   dk      key owner: loops over the query blocks that see its 128 keys; dr is written
//           back into TMEM as bf16 and dk += dr Q runs as a TS MMA (A from TMEM).  No
//           atomics (the reference accumulates dk with fp32 atomics; this is deterministic).
#include "tc.cuh"

namespace mzb {
namespace ibwd {

constexpr int NTHREADS = 384;
constexpr int BM = 128;

template <int DI>
struct Cfg {
  static constexpr int DB = DI / 64;           // 64-channel column blocks of q / k rows
  // (token, head) rows per query block: 256, or 128 for Di = 256 (q, two k stages and dr
  // then fill the shared memory, and dq's 256 fp32 columns the upper half of TMEM)
  static constexpr int NMAX = DI == 256 ? 128 : 256;
  static constexpr int Q_BYTES = NMAX * DI * 2;
  static constexpr int K_BYTES = BM * DI * 2;
  static constexpr int DR_BYTES = BM * NMAX * 2;  // dr tile [key][(token, head)] bf16
  static constexpr int SMEM_A = Q_BYTES + 2 * K_BYTES + DR_BYTES + NMAX * 4 * 5 + 512;  // + w, 4 dw partials
  static constexpr int SMEM_B = 2 * Q_BYTES + K_BYTES + 2 * NMAX * 4 + 512;
  static_assert(SMEM_A <= 232448 && SMEM_B <= 232448, "smem");
};

struct Args {
  const float* w;    // [B, S, Hi]
  const float* dl;   // [B, S, T]
  __nv_bfloat16* dq; // [B, S, Hi, Di]
  __nv_bfloat16* dk; // [B, T, Di]
  float* dw;         // [B, S, Hi]
  int B, S, T, Hi, Tq, N, ratio;
  long long q_offset;
  float scale;
  int* err;
};

__device__ __forceinline__ int vis_keys(const Args& a, int s) {
  long long v = (a.q_offset + s + 1) / a.ratio;
  return v < 0 ? 0 : (v > a.T ? a.T : int(v));
}

__device__ __forceinline__ void st_shared16(uint8_t* p, const uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(p)), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// ------------------------------------------------------------------ dq + dw (query owner)
enum ABar { A_Q_FULL = 0, A_Q_EMPTY, A_K_FULL, A_K_FULL1, A_K_EMPTY, A_K_EMPTY1, A_R_FULL, A_DR_FULL, A_DQ_DONE,
            A_DQ_EMPTY, A_NBAR };

template <int DI>
__global__ void __launch_bounds__(NTHREADS, 1)
    dq_dw_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk, Args a) {
  using C = Cfg<DI>;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* qs = smem;
  uint8_t* ks = qs + C::Q_BYTES;
  uint8_t* drs = ks + 2 * C::K_BYTES;
  float* wsm = reinterpret_cast<float*>(drs + C::DR_BYTES);
  float* dwsm = wsm + C::NMAX;  // [4 lane quarters][NMAX] partial sums: each column is owned by one
                                // warpgroup, each (quarter, column) by one warp -> no atomics
  uint64_t* bars = reinterpret_cast<uint64_t*>(dwsm + 4 * C::NMAX);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + A_NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) atomicExch(a.err, MZB_ERR_ALIGN);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < A_NBAR; ++i) tc::mbar_init(&bars[i], (i == A_DR_FULL || i == A_DQ_EMPTY) ? 8 : 1);
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, 512);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const int n_tb = (a.S + a.Tq - 1) / a.Tq;
  const int items = a.B * n_tb;
  auto tiles_of = [&](int tb) {
    const int s_last = min((tb + 1) * a.Tq, a.S) - 1;
    return (vis_keys(a, s_last) + BM - 1) / BM;
  };
  constexpr int C_R = 0, C_DQ = 256;
  static_assert(C_DQ + (C::NMAX / 128) * DI <= 512, "TMEM");

  if (warp == 0) {
    if (lane == 0) {
      int g = 0, ii = 0;
      for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x) {
        const int tb = n_tb - 1 - it / a.B, b = it % a.B;
        const int n = tiles_of(tb);
        if (n == 0) continue;  // no visible key: the epilogue writes zeros
        if (!tc::mbar_wait(&bars[A_Q_EMPTY], (ii & 1) ^ 1, a.err, 601)) { *abort_flag = 1; break; }
        ++ii;
        tc::mbar_expect_tx(&bars[A_Q_FULL], uint32_t(a.N) * DI * 2);
        for (int cb = 0; cb < C::DB; ++cb)
          tc::tma_load_3d(qs + cb * C::NMAX * 128, &tq, &bars[A_Q_FULL], cb * 64, tb * a.Tq * a.Hi, b);
        bool ok = true;
        for (int kt = 0; kt < n; ++kt, ++g) {
          const int st = g & 1, ph = (g >> 1) & 1;
          if (!tc::mbar_wait(&bars[A_K_EMPTY + st], ph ^ 1, a.err, 602)) { ok = false; break; }
          tc::mbar_expect_tx(&bars[A_K_FULL + st], C::K_BYTES);
          for (int cb = 0; cb < C::DB; ++cb)
            tc::tma_load_3d(ks + st * C::K_BYTES + cb * BM * 128, &tk, &bars[A_K_FULL + st], cb * 64, kt * BM, b);
        }
        if (!ok) { *abort_flag = 1; break; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc_r = tc::make_idesc(BM, a.N, 1, 1);
      const uint32_t idesc_dq = tc::make_idesc(128, DI, 1, 1, true, true);
      const uint32_t q_base = smem_u32(qs), k_base = smem_u32(ks), dr_base = smem_u32(drs);
      int g = 0, ii = -1;
      for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x) {
        const int tb = n_tb - 1 - it / a.B;
        const int n = tiles_of(tb);
        if (n == 0) continue;
        ++ii;
        if (!tc::mbar_wait(&bars[A_Q_FULL], ii & 1, a.err, 610)) { *abort_flag = 1; break; }
        bool ok = true;
        for (int kt = 0; kt < n; ++kt, ++g) {
          const int st = g & 1, ph = (g >> 1) & 1;
          if (!tc::mbar_wait(&bars[A_K_FULL + st], ph, a.err, 611)) { ok = false; break; }
          tc::fence_after_sync();
          const uint32_t kb = k_base + st * C::K_BYTES;
#pragma unroll
          for (int kk = 0; kk < DI / 16; ++kk) {
            const int cb = kk >> 2, off = (kk & 3) * 32;
            tc::mma_ss<0>(tmem + C_R, tc::make_sdesc<128>(kb + cb * BM * 128 + off, 16, 1024),
                          tc::make_sdesc<128>(q_base + cb * C::NMAX * 128 + off, 16, 1024), idesc_r, kk > 0);
          }
          tc::mma_commit(&bars[A_R_FULL]);
          if (kt == 0 && !tc::mbar_wait(&bars[A_DQ_EMPTY], (ii & 1) ^ 1, a.err, 612)) { ok = false; break; }
          if (!tc::mbar_wait(&bars[A_DR_FULL], g & 1, a.err, 613)) { ok = false; break; }
          tc::fence_after_sync();
          // dq[rows of half hb] += dr^T K  (M = 128 rows, K = 128 keys, N = Di)
#pragma unroll
          for (int hb = 0; hb < 2; ++hb) {
            if (hb * 128 >= a.N) break;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              tc::mma_ss<0>(tmem + C_DQ + hb * DI, tc::make_sdesc<128>(dr_base + 2 * hb * 16384 + kk * 2048, 16384, 1024),
                            tc::make_sdesc<128>(kb + kk * 2048, BM * 128, 1024), idesc_dq, (kt > 0 || kk > 0) ? 1u : 0u);
          }
          tc::mma_commit(&bars[A_K_EMPTY + st]);
          if (kt == n - 1) {
            tc::mma_commit(&bars[A_Q_EMPTY]);
            tc::mma_commit(&bars[A_DQ_DONE]);
          }
        }
        if (!ok) { *abort_flag = 1; break; }
      }
    }
  } else if (warp >= 4) {
    const int et = threadIdx.x - 128;   // 0..255
    const int quarter = warp & 3;       // TMEM lane quarter
    const int wg = (warp - 4) >> 2;     // token parity handled by this warpgroup
    const int row = quarter * 32 + lane;  // key within the tile
    int g = 0, ii = -1;
    for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x) {
      const int tb = n_tb - 1 - it / a.B, b = it % a.B;
      const int s0 = tb * a.Tq;
      const int n = tiles_of(tb);
      if (n > 0) ++ii;
      // weights and dw accumulators of this block
      for (int i = et; i < C::NMAX; i += 256) {
        const int s = s0 + i / a.Hi;
        wsm[i] = (i < a.N && s < a.S) ? a.w[((long long)b * a.S + s) * a.Hi + i % a.Hi] : 0.0f;
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) dwsm[qq * C::NMAX + i] = 0.0f;
      }
      tc::bar_sync(1, 256);
      bool ok = true;
      for (int kt = 0; kt < n; ++kt, ++g) {
        const int t = kt * BM + row;
        if (!tc::mbar_wait(&bars[A_R_FULL], g & 1, a.err, 620)) { ok = false; break; }
        tc::fence_after_sync();
        for (int tt = wg; tt < a.Tq; tt += 2) {
          const int s = s0 + tt;
          float d = 0.0f;
          if (s < a.S && t < vis_keys(a, s)) d = a.dl[((long long)b * a.S + s) * a.T + t] * a.scale;
          for (int h0 = 0; h0 < a.Hi; h0 += 16) {
            const int c0 = tt * a.Hi + h0;  // column = (token, head)
            uint32_t rv[16];
            tc::tmem_ld16(tc::taddr(tmem, quarter * 32, C_R + c0), rv);
            tc::tmem_wait_ld();
            float dwv[16];
            uint32_t pk[8];
#pragma unroll
            for (int i = 0; i < 16; i += 2) {
              const float r0 = __uint_as_float(rv[i]), r1 = __uint_as_float(rv[i + 1]);
              dwv[i] = fmaxf(r0, 0.0f) * d;
              dwv[i + 1] = fmaxf(r1, 0.0f) * d;
              pk[i / 2] = pack_bf16(r0 > 0.0f ? d * wsm[c0 + i] : 0.0f, r1 > 0.0f ? d * wsm[c0 + i + 1] : 0.0f);
            }
            // dr -> smem tile [key][column], 64-column blocks, 128-byte swizzle
            uint8_t* rowp = drs + (c0 >> 6) * 16384 + row * 128;
            const int ch0 = (c0 & 63) >> 3;
            st_shared16(rowp + (((ch0) ^ (row & 7)) * 16), make_uint4(pk[0], pk[1], pk[2], pk[3]));
            st_shared16(rowp + (((ch0 + 1) ^ (row & 7)) * 16), make_uint4(pk[4], pk[5], pk[6], pk[7]));
            // dw: reduce the 16 columns over the warp's 32 keys (reduce-scatter), then smem atomics
#pragma unroll
            for (int step = 8; step >= 1; step >>= 1) {
              const bool upper = lane & step;
#pragma unroll
              for (int i = 0; i < step; ++i) {
                const float send = upper ? dwv[i] : dwv[i + step];
                const float recv = __shfl_xor_sync(0xffffffffu, send, step);
                dwv[i] = (upper ? dwv[i + step] : dwv[i]) + recv;
              }
            }
            // lane l now holds column (l & 15)'s partial over the 16 lanes sharing bit 4
            const float other = __shfl_xor_sync(0xffffffffu, dwv[0], 16);
            if (lane < 16) dwsm[quarter * C::NMAX + c0 + lane] += dwv[0] + other;
          }
        }
        tc::fence_async_smem();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bars[A_DR_FULL]);
      }
      if (!ok) { *abort_flag = 1; break; }
      if (n == 0) {  // nothing visible: dq = 0, dw = 0
        for (int i = et; i < a.N * DI; i += 256) {
          const int rr = i / DI, s = s0 + rr / a.Hi;
          if (s < a.S) a.dq[(((long long)b * a.S + s) * a.Hi + rr % a.Hi) * DI + i % DI] = __float2bfloat16_rn(0.0f);
        }
      } else {
        if (!tc::mbar_wait(&bars[A_DQ_DONE], ii & 1, a.err, 621)) { *abort_flag = 1; break; }
        tc::fence_after_sync();
        // thread (quarter, lane) of warpgroup wg owns packed row wg*128 + row (the second
        // warpgroup has no rows, and no accumulator columns, when NMAX = 128)
        const int rr = wg * 128 + row;
        const int s = s0 + rr / a.Hi;
        if (wg * 128 < C::NMAX) {
          for (int c0 = 0; c0 < DI; c0 += 16) {
            uint32_t v[16];
            tc::tmem_ld16(tc::taddr(tmem, quarter * 32, C_DQ + wg * DI + c0), v);
            tc::tmem_wait_ld();
            if (rr < a.N && s < a.S) {
              uint4* dst = reinterpret_cast<uint4*>(a.dq + (((long long)b * a.S + s) * a.Hi + rr % a.Hi) * DI + c0);
              dst[0] = make_uint4(pack_bf16(__uint_as_float(v[0]), __uint_as_float(v[1])),
                                  pack_bf16(__uint_as_float(v[2]), __uint_as_float(v[3])),
                                  pack_bf16(__uint_as_float(v[4]), __uint_as_float(v[5])),
                                  pack_bf16(__uint_as_float(v[6]), __uint_as_float(v[7])));
              dst[1] = make_uint4(pack_bf16(__uint_as_float(v[8]), __uint_as_float(v[9])),
                                  pack_bf16(__uint_as_float(v[10]), __uint_as_float(v[11])),
                                  pack_bf16(__uint_as_float(v[12]), __uint_as_float(v[13])),
                                  pack_bf16(__uint_as_float(v[14]), __uint_as_float(v[15])));
            }
          }
        }
      }
      tc::fence_before_sync();
      tc::bar_sync(1, 256);  // every dw partial of this block landed
      for (int i = et; i < a.N; i += 256) {
        const int s = s0 + i / a.Hi;
        const float v = ((dwsm[i] + dwsm[C::NMAX + i]) + dwsm[2 * C::NMAX + i]) + dwsm[3 * C::NMAX + i];
        if (s < a.S) a.dw[((long long)b * a.S + s) * a.Hi + i % a.Hi] = v;
      }
      __syncwarp();
      if (lane == 0 && n > 0) tc::mbar_arrive(&bars[A_DQ_EMPTY]);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_free(tmem, 512);
  }
}

// ------------------------------------------------------------------ dk (key owner)
enum BBar { B_K_FULL = 0, B_K_EMPTY, B_Q_FULL, B_Q_FULL1, B_Q_EMPTY, B_Q_EMPTY1, B_R_FULL, B_DR_FULL, B_DK_DONE,
            B_DK_EMPTY, B_NBAR };

template <int DI>
__global__ void __launch_bounds__(NTHREADS, 1)
    dk_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk, Args a) {
  using C = Cfg<DI>;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* ks = smem;
  uint8_t* qs = ks + C::K_BYTES;  // 2 stages
  float* wsm = reinterpret_cast<float*>(qs + 2 * C::Q_BYTES);  // 2 stages x NMAX
  uint64_t* bars = reinterpret_cast<uint64_t*>(wsm + 2 * C::NMAX);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + B_NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) atomicExch(a.err, MZB_ERR_ALIGN);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < B_NBAR; ++i) tc::mbar_init(&bars[i], (i == B_DR_FULL || i == B_DK_EMPTY) ? 8 : 1);
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, 512);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const int n_kt = (a.T + BM - 1) / BM;
  const int n_tb = (a.S + a.Tq - 1) / a.Tq;
  const int items = a.B * n_kt;
  // query blocks that see key tile kt: the first block whose last token sees key kt*128
  auto first_tb = [&](int kt) {
    int lo = 0, hi = n_tb;  // smallest tb with vis(last token of tb) > kt*BM
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      const int s_last = min((mid + 1) * a.Tq, a.S) - 1;
      if (vis_keys(a, s_last) > kt * BM) hi = mid; else lo = mid + 1;
    }
    return lo;
  };
  // R (NMAX columns), dk accumulator (DI), packed bf16 dr (NMAX / 2): 0 / 256 / 384, or
  // 0 / 256 / 128 when NMAX = 128 and DI = 256
  constexpr int C_R = 0, C_DK = 256, C_DR = C::NMAX == 256 ? 384 : 128;
  static_assert(C_DK + DI <= 512 && (C_DR + C::NMAX / 2 <= C_DK || C_DR >= C_DK + DI), "TMEM");

  if (warp == 0) {
    if (lane == 0) {
      int g = 0, ii = 0;
      for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x) {
        const int kt = it / a.B, b = it % a.B;
        const int tb0 = first_tb(kt);
        if (tb0 >= n_tb) continue;
        if (!tc::mbar_wait(&bars[B_K_EMPTY], (ii & 1) ^ 1, a.err, 701)) { *abort_flag = 1; break; }
        ++ii;
        tc::mbar_expect_tx(&bars[B_K_FULL], C::K_BYTES);
        for (int cb = 0; cb < C::DB; ++cb)
          tc::tma_load_3d(ks + cb * BM * 128, &tk, &bars[B_K_FULL], cb * 64, kt * BM, b);
        bool ok = true;
        for (int tb = tb0; tb < n_tb; ++tb, ++g) {
          const int st = g & 1, ph = (g >> 1) & 1;
          if (!tc::mbar_wait(&bars[B_Q_EMPTY + st], ph ^ 1, a.err, 702)) { ok = false; break; }
          tc::mbar_expect_tx(&bars[B_Q_FULL + st], uint32_t(a.N) * DI * 2);
          for (int cb = 0; cb < C::DB; ++cb)
            tc::tma_load_3d(qs + st * C::Q_BYTES + cb * C::NMAX * 128, &tq, &bars[B_Q_FULL + st], cb * 64,
                            tb * a.Tq * a.Hi, b);
        }
        if (!ok) { *abort_flag = 1; break; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc_r = tc::make_idesc(BM, a.N, 1, 1);
      const uint32_t idesc_dk = tc::make_idesc(BM, DI, 1, 1, false, true);
      const uint32_t k_base = smem_u32(ks), q_base = smem_u32(qs);
      int g = 0, ii = -1;
      for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x) {
        const int kt = it / a.B;
        const int tb0 = first_tb(kt);
        if (tb0 >= n_tb) continue;
        ++ii;
        if (!tc::mbar_wait(&bars[B_K_FULL], ii & 1, a.err, 710)) { *abort_flag = 1; break; }
        bool ok = true;
        for (int tb = tb0; tb < n_tb; ++tb, ++g) {
          const int st = g & 1, ph = (g >> 1) & 1;
          if (!tc::mbar_wait(&bars[B_Q_FULL + st], ph, a.err, 711)) { ok = false; break; }
          tc::fence_after_sync();
          const uint32_t qb = q_base + st * C::Q_BYTES;
#pragma unroll
          for (int kk = 0; kk < DI / 16; ++kk) {
            const int cb = kk >> 2, off = (kk & 3) * 32;
            tc::mma_ss<0>(tmem + C_R, tc::make_sdesc<128>(k_base + cb * BM * 128 + off, 16, 1024),
                          tc::make_sdesc<128>(qb + cb * C::NMAX * 128 + off, 16, 1024), idesc_r, kk > 0);
          }
          tc::mma_commit(&bars[B_R_FULL]);
          if (tb == tb0 && !tc::mbar_wait(&bars[B_DK_EMPTY], (ii & 1) ^ 1, a.err, 712)) { ok = false; break; }
          if (!tc::mbar_wait(&bars[B_DR_FULL], g & 1, a.err, 713)) { ok = false; break; }
          tc::fence_after_sync();
          // dk += dr Q: A = dr [keys x rows] from TMEM (bf16 pairs in R's columns), K = rows
          for (int kk = 0; kk < a.N / 16; ++kk)
            tc::mma_ts(tmem + C_DK, tmem + C_DR + kk * 8, tc::make_sdesc<128>(qb + kk * 2048, C::NMAX * 128, 1024),
                       idesc_dk, (tb > tb0 || kk > 0) ? 1u : 0u);
          tc::mma_commit(&bars[B_Q_EMPTY + st]);
          if (tb == n_tb - 1) {
            tc::mma_commit(&bars[B_DK_DONE]);
            tc::mma_commit(&bars[B_K_EMPTY]);
          }
        }
        if (!ok) { *abort_flag = 1; break; }
      }
    }
  } else if (warp >= 4) {
    const int quarter = warp & 3, wg = (warp - 4) >> 2, row = quarter * 32 + lane;
    int g = 0, ii = -1;
    for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x) {
      const int kt = it / a.B, b = it % a.B;
      const int tb0 = first_tb(kt);
      const int t = kt * BM + row;
      if (tb0 >= n_tb) {  // no query sees these keys: dk = 0
        if (wg == 0 && t < a.T)
          for (int c = 0; c < DI; ++c) a.dk[((long long)b * a.T + t) * DI + c] = __float2bfloat16_rn(0.0f);
        continue;
      }
      ++ii;
      bool ok = true;
      for (int tb = tb0; tb < n_tb; ++tb, ++g) {
        const int s0 = tb * a.Tq;
        if (!tc::mbar_wait(&bars[B_R_FULL], g & 1, a.err, 720)) { ok = false; break; }
        tc::fence_after_sync();
        // columns (token, head): warpgroup wg takes columns [wg*N/2, (wg+1)*N/2)
        const int half = a.N >> 1, hs = __ffs(a.Hi) - 1;
        for (int c0 = wg * half; c0 < (wg + 1) * half; c0 += 32) {
          uint32_t rv[32];
          tc::tmem_ld32(tc::taddr(tmem, quarter * 32, C_R + c0), rv);
          tc::tmem_wait_ld();
          // a 32-column chunk spans at most two tokens (Hi >= 16)
          const int sa = s0 + (c0 >> hs), sb = s0 + ((c0 + 31) >> hs);
          float da = 0.0f, db = 0.0f;
          if (sa < a.S && t < vis_keys(a, sa)) da = a.dl[((long long)b * a.S + sa) * a.T + t] * a.scale;
          if (sb < a.S && t < vis_keys(a, sb)) db = a.dl[((long long)b * a.S + sb) * a.T + t] * a.scale;
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            float v2[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int c = c0 + i + e;
              const int s = s0 + (c >> hs);
              const float d = s == sa ? da : db;
              const float w = s < a.S ? a.w[((long long)b * a.S + s) * a.Hi + (c & (a.Hi - 1))] : 0.0f;
              v2[e] = __uint_as_float(rv[i + e]) > 0.0f ? d * w : 0.0f;
            }
            pk[i / 2] = pack_bf16(v2[0], v2[1]);
          }
          tc::tmem_st16(tc::taddr(tmem, quarter * 32, C_DR + c0 / 2), pk);
        }
        tc::tmem_wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bars[B_DR_FULL]);
      }
      if (!ok) { *abort_flag = 1; break; }
      if (!tc::mbar_wait(&bars[B_DK_DONE], ii & 1, a.err, 721)) { *abort_flag = 1; break; }
      tc::fence_after_sync();
      for (int c0 = wg * (DI / 2); c0 < (wg + 1) * (DI / 2); c0 += 16) {
        uint32_t v[16];
        tc::tmem_ld16(tc::taddr(tmem, quarter * 32, C_DK + c0), v);
        tc::tmem_wait_ld();
        if (t < a.T) {
          uint4* dst = reinterpret_cast<uint4*>(a.dk + ((long long)b * a.T + t) * DI + c0);
          dst[0] = make_uint4(pack_bf16(__uint_as_float(v[0]), __uint_as_float(v[1])),
                              pack_bf16(__uint_as_float(v[2]), __uint_as_float(v[3])),
                              pack_bf16(__uint_as_float(v[4]), __uint_as_float(v[5])),
                              pack_bf16(__uint_as_float(v[6]), __uint_as_float(v[7])));
          dst[1] = make_uint4(pack_bf16(__uint_as_float(v[8]), __uint_as_float(v[9])),
                              pack_bf16(__uint_as_float(v[10]), __uint_as_float(v[11])),
                              pack_bf16(__uint_as_float(v[12]), __uint_as_float(v[13])),
                              pack_bf16(__uint_as_float(v[14]), __uint_as_float(v[15])));
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&bars[B_DK_EMPTY]);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_free(tmem, 512);
  }
}

template <int DI>
int launch(const void* q, const void* k, const Args& a, cudaStream_t st) {
  using C = Cfg<DI>;
  CUtensorMap tq, tk;
  {
    const uint64_t dims[3] = {uint64_t(DI), uint64_t(a.S) * a.Hi, uint64_t(a.B)};
    const uint64_t str[2] = {uint64_t(DI) * 2, uint64_t(a.S) * a.Hi * DI * 2};
    const uint32_t box[3] = {64, uint32_t(a.N), 1};
    if (int r = encode_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, q, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return r;
  }
  {
    const uint64_t dims[3] = {uint64_t(DI), uint64_t(a.T), uint64_t(a.B)};
    const uint64_t str[2] = {uint64_t(DI) * 2, uint64_t(a.T) * DI * 2};
    const uint32_t box[3] = {64, uint32_t(BM), 1};
    if (int r = encode_tmap(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, k, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return r;
  }
  auto ka = dq_dw_kernel<DI>;
  auto kb = dk_kernel<DI>;
  if (cudaFuncSetAttribute(ka, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_A) != cudaSuccess ||
      cudaFuncSetAttribute(kb, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_B) != cudaSuccess)
    return launch_status("indexer_bwd(smem attr)");
  const int n_tb = (a.S + a.Tq - 1) / a.Tq;
  const int ia = a.B * n_tb, ib = a.B * ((a.T + BM - 1) / BM);
  ka<<<ia < num_sms() ? ia : num_sms(), NTHREADS, C::SMEM_A, st>>>(tq, tk, a);
  if (int r = launch_status("indexer_bwd_dq_dw")) return r;
  kb<<<ib < num_sms() ? ib : num_sms(), NTHREADS, C::SMEM_B, st>>>(tq, tk, a);
  return launch_status("indexer_bwd_dk");
}

}  // namespace ibwd
}  // namespace mzb

using namespace mzb;

extern "C" int mzb_indexer_bwd(const void* q, const void* k, const float* w, const float* dl, void* dq, void* dk,
                               float* dw, int64_t B, int64_t S, int64_t T, int Hi, int Di, int ratio, int64_t q_offset,
                               float scale, int* err, void* stream) {
  MZB_REQUIRE(B >= 1 && S >= 1 && T >= 1, MZB_ERR_SHAPE, "indexer_bwd: bad shape (an empty key axis is the caller's)");
  MZB_REQUIRE(Di == 64 || Di == 128 || Di == 256, MZB_ERR_UNSUPPORTED,
              "indexer_bwd: index head dim %d not built (64, 128, 256)", Di);
  const int nmax = Di == 256 ? 128 : 256;  // (token, head) rows per query block
  MZB_REQUIRE(Hi >= 16 && Hi <= nmax && Hi % 16 == 0 && nmax % Hi == 0, MZB_ERR_SHAPE,
              "indexer_bwd: index heads must divide %d and be a multiple of 16 (pad with zero weights), got %d", nmax,
              Hi);
  MZB_REQUIRE(ratio >= 1 && err != nullptr, MZB_ERR_SHAPE, "indexer_bwd: bad ratio or missing error word");
  ibwd::Args a{};
  a.w = w; a.dl = dl;
  a.dq = static_cast<__nv_bfloat16*>(dq);
  a.dk = static_cast<__nv_bfloat16*>(dk);
  a.dw = dw;
  a.B = int(B); a.S = int(S); a.T = int(T); a.Hi = Hi;
  a.Tq = nmax / Hi; a.N = nmax;
  a.ratio = ratio; a.q_offset = q_offset; a.scale = scale; a.err = err;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (Di == 64) return ibwd::launch<64>(q, k, a, st);
  return Di == 128 ? ibwd::launch<128>(q, k, a, st) : ibwd::launch<256>(q, k, a, st);
}
