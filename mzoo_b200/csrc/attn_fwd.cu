// Shared-latent MQA attention forward with packed (token, head) rows: the sliding-window
// kernel (`swa_attn`) and the window + gathered top-k kernel (`csa2_attn`), bf16 in, fp32
// accumulate, bf16 out, natural-log lse.
//
// Reference: src/mzoo/layers/attn/swa_attn/fwd.py:55-208 and csa2_attn/fwd.py:70-286:
//   rows = q.view(B, S*H, D) (T_q = 128 / H tokens x H heads per tile), keys of the window
//   t-W < k <= t (self included), then per token its gathered main_kv[indices[t, :]] rows
//   (index outside [0, G) = empty; duplicates count twice; only that token's rows see them),
//   one online softmax over both, optional per-head sink (denominator only), scale D^-1/2.
//   K == V (the shared latent) by default; a distinct V (where K and V
//   are quantised differently) is accepted for the window-only kernel.
//
// tcgen05 kernel, one CTA per 128-row query tile, persistent over tiles:
//   warp 0      TMA: Q tile, window K (and V) tiles into a ring of stages
//   warp 1      TMEM allocation + the MMA-issuing thread
//   warps 4-7   softmax, lazy O correction, epilogue (thread = row = TMEM lane); column
//               visibility as one mask word per 32 columns per tile
//   warps 8-11  gathered-tile producers (ld.global of main_kv rows -> swizzled smem), or,
//               without gathered rows, the O / lse epilogue while the softmax warps start
//               the next tile
//   warps 12-15 (separate V, D <= 128 only) a second softmax warpgroup on the upper half of
//               each tile's key columns; the pair of warps on one TMEM lane quarter swaps
//               partial row maxima through TMEM columns [X_COL, X_COL + 4) under a count-2
//               mbarrier, and the upper half's row sum reaches the epilogue the same way;
//               there warps 8-11 also copy each item's Q rows into TMEM one item ahead, so
//               QK^T is a TS MMA and the Q buffer is free for the next item at once
// S = Q K^T (M=128 rows, N=NK keys) and O += P V (N=D) accumulate in TMEM; P (bf16) is
// written back into its S buffer and read from there as the A operand of the PV MMA, so
// shared memory carries only Q, K and V.  MMA order QK_0, QK_1, PV_0, QK_2, PV_1, ...
#include "tc.cuh"

namespace mzb {
namespace attn {

constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;

// Row finish, written with explicitly rounded operations so that the softmax warps and the
// separate epilogue warps (window-only kernel) produce the same bits: msl = m * scale_log2,
// optional sink term in the denominator, lse in natural log.
__device__ __forceinline__ float row_sum_with_sink(float lsum, float msl, const float* sinks, int h) {
  return sinks ? __fadd_rn(lsum, exp2f(__fsub_rn(__fmul_rn(sinks[h], LOG2E), msl))) : lsum;
}
__device__ __forceinline__ float row_lse(float msl, float lsum) { return __fmul_rn(__fadd_rn(msl, log2f(lsum)), LN2); }

template <int D, bool SEP_V>
struct Cfg {
  static constexpr int NK = D == 256 ? 64 : 128;  // keys per tile
  static constexpr int DB = D / 64;               // 64-channel column blocks
  static constexpr int Q_BYTES = 128 * D * 2;
  static constexpr int K_BYTES = NK * D * 2;
  static constexpr int STAGE_BYTES = K_BYTES * (SEP_V ? 2 : 1);
  static constexpr int STAGES = SEP_V ? (D == 256 ? 2 : 3) : 4;  // K (+ V) ring depth
  static constexpr int TILE_BYTES = Q_BYTES + STAGES * STAGE_BYTES;
  static constexpr int MISC = 512 + 4 * 128 * 4;  // barriers; 2 x (row max, row sum) handoff
  static constexpr int SMEM = TILE_BYTES + MISC;
  static constexpr int S_COL0 = D;  // O in columns [0, D), S buffers after it
  // separate V (window only) at D <= 128: a second softmax warpgroup (warps 12-15) takes the
  // upper half of every key tile's columns; the two halves exchange their row maxima, and
  // hand the second half's row sum to the epilogue, through TMEM columns [X_COL, X_COL + 6)
  static constexpr bool SPLIT = SEP_V && D <= 128;
  static constexpr int NT = SPLIT ? 512 : 384;
  static constexpr int NQ = SPLIT ? NK / 64 : NK / 32;  // 32-column chunks per softmax warp
  static constexpr int X_COL = D + 2 * NK;
  static_assert(!SPLIT || X_COL + 6 <= 512, "TMEM budget");
  // SPLIT: the item's Q rows (bf16 pairs, the TS operand layout) in the last D / 2 columns;
  // S = Q K^T then reads only K from shared memory, and the Q buffer is free for the next
  // item once warps 8-11 have copied it
  static constexpr int C_QT = 512 - D / 2;
  static_assert(!SPLIT || X_COL + 6 <= C_QT, "TMEM budget");
  // P (bf16) goes back into its own S buffer: the 32-bit column of keys (c, c + 1) is
  // pt_col(c); each column half [0, NK/2), [NK/2, NK) packs into the front of its own
  // columns, so the two softmax warpgroups never store over S columns the other still reads
  static __device__ __forceinline__ int pt_col(int c) { return c / 2 + (c >= NK / 2 ? NK / 4 : 0); }
  static_assert(SMEM <= 232448, "shared memory budget");
  static_assert(D + 2 * NK <= 512, "TMEM budget");
};

struct Args {
  const __nv_bfloat16* main_kv;  // [B, G, D] gathered source (csa2) or null
  const int32_t* idx;            // [B, S, topk] or null
  const float* sinks;            // [H] or null
  __nv_bfloat16* o;              // [B, S*H, D]
  float* lse;                    // [B, S*H]
  int B, S, H, window, G, topk;
  float scale_log2;
  int* err;
};

// O_FINAL: commit after an item's last PV, waited on by the epilogue with the item parity
// (two PVs can still be in flight there, so O_DONE's parity would alias an older phase).
// QK_DONE: commit after an item's last QK^T; QT_FULL: the item's Q rows are in TMEM (SPLIT).
enum Bar { Q_FULL = 0, Q_EMPTY, O_DONE, O_EMPTY, S_FULL, S_FULL1, S_EMPTY, S_EMPTY1, P_FULL, P_FULL1, KV_FULL_W,
           KV_FULL_G = KV_FULL_W + 4, KV_EMPTY = KV_FULL_G + 4, O_FINAL = KV_EMPTY + 4, EPI_FULL, MX,
           QK_DONE = MX + 4, QT_FULL, NBAR };

__device__ __forceinline__ void st_shared16(uint8_t* p, const uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(p)), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Per item (query tile): window tile range and the number of gathered tiles.
struct Item {
  int b, qt, t0, t1, kt0, n_win, n_gat, tq_valid;
};

template <int NK>
__device__ __forceinline__ Item make_item(const Args& a, int it, int n_qt) {
  Item m;
  m.b = it % a.B;
  m.qt = n_qt - 1 - it / a.B;  // heavy (late) tiles first
  const int tq = 128 / a.H;
  m.t0 = m.qt * tq;
  m.t1 = min(a.S, m.t0 + tq) - 1;
  m.tq_valid = m.t1 - m.t0 + 1;
  const int lo = max(0, m.t0 - a.window + 1);
  m.kt0 = lo / NK;
  m.n_win = m.t1 / NK - m.kt0 + 1;
  const int gt = (a.main_kv && a.topk > 0 && a.G > 0) ? (a.topk + NK - 1) / NK : 0;
  m.n_gat = gt * m.tq_valid;
  return m;
}

template <int D, bool SEP_V>
__global__ void __launch_bounds__(Cfg<D, SEP_V>::NT, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, Args a) {
  using C = Cfg<D, SEP_V>;
  constexpr int NK = C::NK;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* qs = smem;
  uint8_t* kvs = qs + C::Q_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::TILE_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::TILE_BYTES + 8 * NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::TILE_BYTES + 8 * NBAR + 4);
  // window-only kernel: the softmax warps hand each item's row statistics (max in the
  // exp2 domain, sum) to warps 8-11, which write O and lse while the next item runs
  float* stats = reinterpret_cast<float*>(smem + C::TILE_BYTES + 512);  // [2][2][128]
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) atomicExch(a.err, MZB_ERR_ALIGN);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NBAR; ++i) {
      uint32_t c = 1;
      if (i == O_EMPTY) c = 4;
      if (i == S_EMPTY || i == S_EMPTY1 || i == P_FULL || i == P_FULL1 || i == EPI_FULL) c = C::SPLIT ? 8 : 4;
      if (i >= MX && i < MX + 4) c = 2;  // the two softmax warps of one TMEM lane quarter
      if (i == QT_FULL || (i == Q_EMPTY && C::SPLIT)) c = 4;  // warps 8-11 copy Q to TMEM
      if (i >= KV_FULL_G && i < KV_EMPTY) c = 4;
      tc::mbar_init(&bars[i], c);
    }
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, 512);
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&tq);
    tc::prefetch_tmap(&tk);
    if (SEP_V) tc::prefetch_tmap(&tv);
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  const int tqn = 128 / a.H;
  const int n_qt = (a.S + tqn - 1) / tqn;
  const int items = a.B * n_qt;
  const bool epi_warps = a.main_kv == nullptr;  // no gathered rows: warps 8-11 are free

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int g = 0, ii = 0;
      for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x, ++ii) {
        const Item m = make_item<NK>(a, it, n_qt);
        if (!tc::mbar_wait(&bars[Q_EMPTY], (ii & 1) ^ 1, a.err, 301)) { *abort_flag = 1; break; }
        tc::mbar_expect_tx(&bars[Q_FULL], C::Q_BYTES);
        for (int cb = 0; cb < C::DB; ++cb) tc::tma_load_3d(qs + cb * 128 * 128, &tq, &bars[Q_FULL], cb * 64, m.qt * 128, m.b);
        bool ok = true;
        for (int j = 0; j < m.n_win + m.n_gat; ++j, ++g) {
          const int st = g % C::STAGES, ph = (g / C::STAGES) & 1;
          if (j >= m.n_win) continue;  // gathered tiles: warps 8-11
          if (!tc::mbar_wait(&bars[KV_EMPTY + st], ph ^ 1, a.err, 302)) { ok = false; break; }
          uint8_t* kt = kvs + st * C::STAGE_BYTES;
          tc::mbar_expect_tx(&bars[KV_FULL_W + st], C::STAGE_BYTES);
          for (int cb = 0; cb < C::DB; ++cb) {
            tc::tma_load_3d(kt + cb * NK * 128, &tk, &bars[KV_FULL_W + st], cb * 64, (m.kt0 + j) * NK, m.b);
            if (SEP_V)
              tc::tma_load_3d(kt + C::K_BYTES + cb * NK * 128, &tv, &bars[KV_FULL_W + st], cb * 64, (m.kt0 + j) * NK,
                              m.b);
          }
        }
        if (!ok) { *abort_flag = 1; break; }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc_qk = tc::make_idesc(128, NK, 1, 1);
      const uint32_t idesc_pv = tc::make_idesc(128, D, 1, 1, false, true);
      const uint32_t q_base = smem_u32(qs), kv_base = smem_u32(kvs);
      // descriptors built once per tile/buffer; unrolled loops add constant offsets (one
      // thread issues every MMA, so per-MMA descriptor arithmetic would throttle issue)
      const uint64_t qd = tc::make_sdesc<128>(q_base, 16, 1024);
      int g = 0, ii = 0;
      int uses_w[4] = {0, 0, 0, 0}, uses_g[4] = {0, 0, 0, 0};
      auto pv = [&](int gg, bool first, int item) -> bool {
        const int st = gg % C::STAGES, pb = gg & 1;
        if (first && !tc::mbar_wait(&bars[O_EMPTY], (item & 1) ^ 1, a.err, 311)) return false;
        if (!tc::mbar_wait(&bars[P_FULL + pb], (gg >> 1) & 1, a.err, 312)) return false;
        tc::fence_after_sync();
        const uint32_t vb = kv_base + st * C::STAGE_BYTES + (SEP_V ? C::K_BYTES : 0);
        const uint64_t vd = tc::make_sdesc<128>(vb, NK * 128, 1024);
#pragma unroll
        for (int jj = 0; jj < NK / 16; ++jj)  // O += P V, P (A operand) from the S buffer in TMEM
          tc::mma_ts(tmem, tmem + C::S_COL0 + pb * NK + C::pt_col(16 * jj), tc::sdesc_add(vd, jj * 16 * 128),
                     idesc_pv, (first && jj == 0) ? 0u : 1u);
        tc::mma_commit(&bars[KV_EMPTY + st]);
        tc::mma_commit(&bars[O_DONE]);
        return true;
      };
      for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x, ++ii) {
        const Item m = make_item<NK>(a, it, n_qt);
        const int n = m.n_win + m.n_gat;
        if (!tc::mbar_wait(&bars[C::SPLIT ? QT_FULL : Q_FULL], ii & 1, a.err, 310)) { *abort_flag = 1; break; }
        bool ok = true;
        for (int j = 0; j < n; ++j, ++g) {
          const int st = g % C::STAGES, sb = g & 1;
          const bool win = j < m.n_win;
          const int par = win ? (uses_w[st]++ & 1) : (uses_g[st]++ & 1);
          if (!tc::mbar_wait(&bars[(win ? KV_FULL_W : KV_FULL_G) + st], par, a.err, 313) ||
              !tc::mbar_wait(&bars[S_EMPTY + sb], ((g >> 1) & 1) ^ 1, a.err, 314)) { ok = false; break; }
          tc::fence_after_sync();
          const uint32_t kb = kv_base + st * C::STAGE_BYTES;
          const uint64_t kd = tc::make_sdesc<128>(kb, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int cb = kk >> 2, off = (kk & 3) * 32;
            if constexpr (C::SPLIT)
              tc::mma_ts(tmem + C::S_COL0 + sb * NK, tmem + C::C_QT + kk * 8, tc::sdesc_add(kd, cb * NK * 128 + off),
                         idesc_qk, kk > 0 ? 1u : 0u);
            else
              tc::mma_ss<0>(tmem + C::S_COL0 + sb * NK, tc::sdesc_add(qd, cb * 128 * 128 + off),
                            tc::sdesc_add(kd, cb * NK * 128 + off), idesc_qk, kk > 0 ? 1u : 0u);
          }
          tc::mma_commit(&bars[S_FULL + sb]);
          if (j == n - 1) tc::mma_commit(&bars[C::SPLIT ? QK_DONE : Q_EMPTY]);
          if (j >= 1 && !pv(g - 1, j == 1, ii)) { ok = false; break; }
        }
        if (!ok || !pv(g - 1, n == 1, ii)) { *abort_flag = 1; break; }
        tc::mma_commit(&bars[O_FINAL]);
      }
    }
  } else if ((warp >= 4 && warp < 8) || (C::SPLIT && warp >= 12)) {
    // ---------------------------------------------------------------- softmax / epilogue
    const int sw = warp & 3, r = sw * 32 + lane;
    const bool wg2 = C::SPLIT && warp >= 12;  // second softmax warpgroup: upper column half
    const int q0 = wg2 ? C::NQ : 0;           // first 32-column chunk of this warp
    const int oc0 = wg2 ? D / 2 : 0, oc1 = C::SPLIT ? oc0 + D / 2 : D;  // O columns it rescales
    const float sl = a.scale_log2;
    int g = 0, ii = 0;
    for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x, ++ii) {
      const Item m = make_item<NK>(a, it, n_qt);
      const int n = m.n_win + m.n_gat;
      const int tr = r / a.H;          // token of this row within the tile
      const int t = m.t0 + tr;         // absolute token
      const int h = r % a.H;
      const bool row_ok = t < a.S;
      const int gtiles = m.n_gat / max(1, m.tq_valid);
      float mrow = -1e30f, lsum = 0.0f;
      bool ok = true;
      for (int j = 0; j < n; ++j, ++g) {
        const int sb = g & 1;
        // column validity of this tile for this row
        const bool win = j < m.n_win;
        int k0 = 0, wlo = 0, whi = -1, gtok = -1;
        uint32_t gm[NK / 32];
        if (win) {
          k0 = (m.kt0 + j) * NK;
          wlo = max(0, t - a.window + 1) - k0;  // valid columns [wlo, whi]
          whi = t - k0;
        } else {
          const int gj = j - m.n_win;
          gtok = gj / gtiles;
          const int e0 = (gj % gtiles) * NK;
          const int32_t* irow = a.idx + ((long long)m.b * a.S + (m.t0 + gtok)) * a.topk;
#pragma unroll
          for (int w = 0; w < NK / 32; ++w) {
            const int e = e0 + w * 32 + lane;
            bool v = false;
            if (e < a.topk) {
              const int gi = irow[e];
              v = gi >= 0 && gi < a.G;
            }
            gm[w] = __ballot_sync(0xffffffffu, v);
          }
        }
        if (!tc::mbar_wait(&bars[S_FULL + sb], (g >> 1) & 1, a.err, 320)) { ok = false; break; }
        tc::fence_after_sync();
        const uint32_t sbase = tc::taddr(tmem, sw * 32, C::S_COL0 + sb * NK);
        // column validity of this row as bits, built once per tile (window: the run
        // [wlo, whi]; gathered: this token's valid slots); a warp whose rows all see the
        // whole tile takes the mask-free loops
        const bool full = row_ok && win && wlo <= 0 && whi >= NK - 1;
        const bool warp_full = __all_sync(0xffffffffu, full);
        uint32_t mw[C::NQ];
#pragma unroll
        for (int q = 0; q < C::NQ; ++q) {
          const int qa = q0 + q;
          uint32_t w = 0u;
          if (row_ok) {
            if (win) {
              const int lo = max(wlo - 32 * qa, 0), hi = min(whi - 32 * qa, 31);
              w = lo > hi ? 0u : ((0xFFFFFFFFu >> (31 - (hi - lo))) << lo);
            } else if (!C::SPLIT && tr == gtok) {  // (no gathered tiles with a separate V)
              w = gm[q];
            }
          }
          mw[q] = w;
        }
        // the whole S row (this warp's columns) behind one TMEM wait; P overwrites it in place
        // below, and the next QK^T into this buffer is issued only after this tile's PV, which
        // the in-order tensor pipe finishes first
        uint32_t sv[C::NQ][32];
#pragma unroll
        for (int q = 0; q < C::NQ; ++q) tc::tmem_ld32(sbase + 32 * (q0 + q), sv[q]);
        tc::tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < C::NQ; ++q) tc::reg_after_wait(sv[q]);
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bars[S_EMPTY + sb]);
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        if (warp_full) {
#pragma unroll
          for (int q = 0; q < C::NQ; ++q)
#pragma unroll
            for (int i = 0; i < 32; ++i) mx[i & 3] = fmaxf(mx[i & 3], __uint_as_float(sv[q][i]));
        } else {
#pragma unroll
          for (int q = 0; q < C::NQ; ++q)
#pragma unroll
            for (int i = 0; i < 32; ++i)
              mx[i & 3] = fmaxf(mx[i & 3], (mw[q] >> i) & 1u ? __uint_as_float(sv[q][i]) : -INFINITY);
        }
        float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
        if (C::SPLIT) {
          // the pair's two partial maxima (double-buffered by tile parity) -> the same max in both
          const uint32_t xa = tc::taddr(tmem, sw * 32, C::X_COL + (g & 1) * 2);
          tc::tmem_st1(xa + (wg2 ? 1 : 0), __float_as_uint(mt));
          tc::tmem_wait_st();
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&bars[MX + sw]);
          if (!tc::mbar_wait(&bars[MX + sw], g & 1, a.err, 324)) { ok = false; break; }
          tc::fence_after_sync();
          uint32_t other = tc::tmem_ld1(xa + (wg2 ? 0 : 1));
          tc::tmem_wait_ld();
          tc::reg_after_wait1(other);
          mt = fmaxf(mt, __uint_as_float(other));
        }
        const bool need = mt * sl > mrow * sl + 8.0f;
        const float m_new = need ? mt : mrow;
        const float alpha = fast_exp2((mrow - m_new) * sl);
        const float ms = m_new * sl;
        float ps4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int q = 0; q < C::NQ; ++q) {
          const int c0 = 32 * (q0 + q);
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float p0 = fast_exp2(fmaf(__uint_as_float(sv[q][2 * i]), sl, -ms));
            float p1 = fast_exp2(fmaf(__uint_as_float(sv[q][2 * i + 1]), sl, -ms));
            if (!warp_full) {
              p0 = (mw[q] >> (2 * i)) & 1u ? p0 : 0.0f;
              p1 = (mw[q] >> (2 * i + 1)) & 1u ? p1 : 0.0f;
            }
            ps4[i & 3] += p0 + p1;
            pk[i] = pack_bf16(p0, p1);
          }
          tc::tmem_st16(sbase + C::pt_col(c0), pk);  // S of these keys is already in registers
        }
        const float psum = (ps4[0] + ps4[1]) + (ps4[2] + ps4[3]);
        lsum = lsum * alpha + psum;
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          if (!tc::mbar_wait(&bars[O_DONE], (g - 1) & 1, a.err, 321)) { ok = false; break; }
          tc::fence_after_sync();
#pragma unroll
          for (int c0 = oc0; c0 < oc1; c0 += 32) {
            uint32_t ov[32];
            tc::tmem_ld32(tc::taddr(tmem, sw * 32, c0), ov);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
            tc::tmem_st32(tc::taddr(tmem, sw * 32, c0), ov);
          }
          tc::tmem_wait_st();
        }
        mrow = m_new;
        tc::tmem_wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bars[P_FULL + sb]);
      }
      if (!ok) { *abort_flag = 1; break; }
      if (epi_warps) {
        float* st = stats + (ii & 1) * 256;
        if (wg2) {  // the upper half's row sum goes through TMEM (item parity)
          tc::tmem_st1(tc::taddr(tmem, sw * 32, C::X_COL + 4 + (ii & 1)), __float_as_uint(lsum));
          tc::tmem_wait_st();
          tc::fence_before_sync();
        } else {
          st[r] = __fmul_rn(mrow, sl);
          st[128 + r] = lsum;
        }
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bars[EPI_FULL]);
        continue;
      }
      if (!tc::mbar_wait(&bars[O_FINAL], ii & 1, a.err, 322)) { *abort_flag = 1; break; }
      tc::fence_after_sync();
      const float msl = __fmul_rn(mrow, sl);
      lsum = row_sum_with_sink(lsum, msl, a.sinks, h);
      const float inv = 1.0f / lsum;
      const long long grow = (long long)m.qt * 128 + r;  // packed row within the batch
      if (row_ok) {
        __nv_bfloat16* orow = a.o + ((long long)m.b * a.S * a.H + grow) * D;
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t ov[32];
          tc::tmem_ld32(tc::taddr(tmem, sw * 32, c0), ov);
          tc::tmem_wait_ld();
          uint4* dst = reinterpret_cast<uint4*>(orow + c0);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            dst[q] = make_uint4(pack_bf16(__uint_as_float(ov[8 * q]) * inv, __uint_as_float(ov[8 * q + 1]) * inv),
                                pack_bf16(__uint_as_float(ov[8 * q + 2]) * inv, __uint_as_float(ov[8 * q + 3]) * inv),
                                pack_bf16(__uint_as_float(ov[8 * q + 4]) * inv, __uint_as_float(ov[8 * q + 5]) * inv),
                                pack_bf16(__uint_as_float(ov[8 * q + 6]) * inv, __uint_as_float(ov[8 * q + 7]) * inv));
        }
        a.lse[(long long)m.b * a.S * a.H + grow] = row_lse(msl, lsum);
      } else {
        // keep the warp-collective TMEM loads uniform: rows past S read and discard
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t ov[32];
          tc::tmem_ld32(tc::taddr(tmem, sw * 32, c0), ov);
          tc::tmem_wait_ld();
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&bars[O_EMPTY]);
    }
  } else if (warp >= 8 && epi_warps) {
    // ---------------------------------------------------------------- epilogue (window-only)
    const int sw = warp - 8, r = sw * 32 + lane;  // TMEM lane quarter warp % 4, as the softmax
    // SPLIT: Q of item number k (shared tile, 64-channel blocks of 128-byte rows with 16-byte
    // chunks swizzled by row % 8) -> TMEM lane r, columns C_QT.. as bf16 pairs; the previous
    // item's QK^T MMAs have completed (QK_DONE), and the shared buffer is released at once
    auto q_to_tmem = [&](int k) {
      if (!tc::mbar_wait(&bars[Q_FULL], k & 1, a.err, 324)) return false;
      if (k > 0 && !tc::mbar_wait(&bars[QK_DONE], (k - 1) & 1, a.err, 325)) return false;
      tc::fence_after_sync();
#pragma unroll
      for (int cb = 0; cb < C::DB; ++cb) {
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          uint32_t v[16];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int ch = h2 * 4 + c;
            uint4 x;
            asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(x.x), "=r"(x.y), "=r"(x.z), "=r"(x.w)
                         : "r"(smem_u32(qs + cb * 128 * 128 + r * 128 + ((ch ^ (r & 7)) * 16)))
                         : "memory");
            v[4 * c] = x.x;
            v[4 * c + 1] = x.y;
            v[4 * c + 2] = x.z;
            v[4 * c + 3] = x.w;
          }
          tc::tmem_st16(tc::taddr(tmem, sw * 32, C::C_QT + cb * 32 + h2 * 16), v);
        }
      }
      tc::tmem_wait_st();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) {
        tc::mbar_arrive(&bars[QT_FULL]);
        tc::mbar_arrive(&bars[Q_EMPTY]);
      }
      return true;
    };
    if (C::SPLIT && (int)blockIdx.x < items && !q_to_tmem(0)) *abort_flag = 1;
    int ii = 0;
    for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x, ++ii) {
      const Item m = make_item<NK>(a, it, n_qt);
      const int t = m.t0 + r / a.H, h = r % a.H;
      const bool row_ok = t < a.S;
      // the next item's Q first: its QK^T can start while this item's O is written
      if (C::SPLIT && it + (int)gridDim.x < items && !q_to_tmem(ii + 1)) { *abort_flag = 1; break; }
      if (!tc::mbar_wait(&bars[EPI_FULL], ii & 1, a.err, 323) ||
          !tc::mbar_wait(&bars[O_FINAL], ii & 1, a.err, 322)) { *abort_flag = 1; break; }
      tc::fence_after_sync();
      const float* st = stats + (ii & 1) * 256;
      const float msl = st[r];
      float lraw = st[128 + r];
      if (C::SPLIT) {  // add the upper column half's row sum (fixed order)
        uint32_t l2 = tc::tmem_ld1(tc::taddr(tmem, sw * 32, C::X_COL + 4 + (ii & 1)));
        tc::tmem_wait_ld();
        tc::reg_after_wait1(l2);
        lraw = __fadd_rn(lraw, __uint_as_float(l2));
      }
      const float lsum = row_sum_with_sink(lraw, msl, a.sinks, h);
      const float inv = 1.0f / lsum;
      const long long grow = (long long)m.qt * 128 + r;  // packed row within the batch
      __nv_bfloat16* orow = a.o + ((long long)m.b * a.S * a.H + grow) * D;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t ov[32];
        tc::tmem_ld32(tc::taddr(tmem, sw * 32, c0), ov);
        tc::tmem_wait_ld();
        tc::reg_after_wait(ov);
        if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c0);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            dst[q] = make_uint4(pack_bf16(__uint_as_float(ov[8 * q]) * inv, __uint_as_float(ov[8 * q + 1]) * inv),
                                pack_bf16(__uint_as_float(ov[8 * q + 2]) * inv, __uint_as_float(ov[8 * q + 3]) * inv),
                                pack_bf16(__uint_as_float(ov[8 * q + 4]) * inv, __uint_as_float(ov[8 * q + 5]) * inv),
                                pack_bf16(__uint_as_float(ov[8 * q + 6]) * inv, __uint_as_float(ov[8 * q + 7]) * inv));
        }
      }
      if (row_ok) a.lse[(long long)m.b * a.S * a.H + grow] = row_lse(msl, lsum);
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&bars[O_EMPTY]);
    }
  } else if (warp >= 8) {
    // ---------------------------------------------------------------- gathered-tile producers
    const int t = threadIdx.x - 256;  // 0..127
    constexpr int TPR = 128 / NK;     // threads per row
    constexpr int CPT = D / 8 / TPR;  // 16-byte chunks per thread
    const int row = t / TPR, sub = t % TPR;
    int g = 0;
    for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x) {
      const Item m = make_item<NK>(a, it, n_qt);
      const int n = m.n_win + m.n_gat;
      const int gtiles = m.n_gat / max(1, m.tq_valid);
      bool ok = true;
      for (int j = 0; j < n; ++j, ++g) {
        if (j < m.n_win) continue;
        const int st = g % C::STAGES, ph = (g / C::STAGES) & 1;
        const int gj = j - m.n_win, gtok = gj / gtiles, e = (gj % gtiles) * NK + row;
        int gi = -1;
        if (e < a.topk) gi = a.idx[((long long)m.b * a.S + (m.t0 + gtok)) * a.topk + e];
        const bool v = gi >= 0 && gi < a.G;
        const uint4* src = reinterpret_cast<const uint4*>(a.main_kv + ((long long)m.b * a.G + (v ? gi : 0)) * D);
        uint4 raw[CPT];
#pragma unroll
        for (int q = 0; q < CPT; ++q) raw[q] = v ? __ldg(src + sub * CPT + q) : make_uint4(0, 0, 0, 0);
        if (!tc::mbar_wait(&bars[KV_EMPTY + st], ph ^ 1, a.err, 330)) { ok = false; break; }
        uint8_t* kt = kvs + st * C::STAGE_BYTES;
#pragma unroll
        for (int q = 0; q < CPT; ++q) {
          const int ch = sub * CPT + q;  // chunk within the row (8 bf16 each)
          const int cb = ch >> 3, c16 = ch & 7;
          st_shared16(kt + cb * NK * 128 + row * 128 + ((c16 ^ (row & 7)) * 16), raw[q]);
        }
        tc::fence_async_smem();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bars[KV_FULL_G + st]);
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
int launch(const void* q, const void* k, const void* v, const Args& a, cudaStream_t st) {
  using C = Cfg<D, SEP_V>;
  CUtensorMap tq, tk, tv;
  {
    const uint64_t dims[3] = {uint64_t(D), uint64_t(a.S) * a.H, uint64_t(a.B)};
    const uint64_t str[2] = {uint64_t(D) * 2, uint64_t(a.S) * a.H * D * 2};
    const uint32_t box[3] = {64, 128, 1};
    if (int r = encode_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, q, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return r;
  }
  const uint64_t dims[3] = {uint64_t(D), uint64_t(a.S), uint64_t(a.B)};
  const uint64_t str[2] = {uint64_t(D) * 2, uint64_t(a.S) * D * 2};
  const uint32_t box[3] = {64, uint32_t(C::NK), 1};
  if (int r = encode_tmap(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, k, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
    return r;
  if (int r = encode_tmap(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, SEP_V ? v : k, dims, str, box,
                          CU_TENSOR_MAP_SWIZZLE_128B))
    return r;
  auto kern = attn_fwd_kernel<D, SEP_V>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
    return launch_status("attn_fwd(smem attr)");
  const int n_qt = (a.S + 128 / a.H - 1) / (128 / a.H);
  const int items = a.B * n_qt;
  const int grid = items < num_sms() ? items : num_sms();
  kern<<<grid, C::NT, C::SMEM, st>>>(tq, tk, tv, a);
  return launch_status("attn_fwd");
}

}  // namespace attn
}  // namespace mzb

using namespace mzb;

extern "C" int mzb_attn_fwd(const void* q, const void* kv, const void* v, const void* main_kv, const int32_t* indices,
                            const float* sinks, void* o, float* lse, int64_t B, int64_t S, int H, int D, int window,
                            int64_t G, int topk, float softmax_scale, int* err, void* stream) {
  MZB_REQUIRE(B >= 1 && S >= 1 && window >= 1 && topk >= 0 && G >= 0, MZB_ERR_SHAPE,
              "attn_fwd: bad sizes B=%lld S=%lld window=%d topk=%d G=%lld", (long long)B, (long long)S, window, topk,
              (long long)G);
  MZB_REQUIRE(H >= 1 && H <= 128 && 128 % H == 0, MZB_ERR_UNSUPPORTED,
              "attn_fwd: heads must divide 128 (packed 128-row tiles), got %d", H);
  MZB_REQUIRE(D == 64 || D == 128 || D == 256, MZB_ERR_UNSUPPORTED, "attn_fwd: unsupported head dim %d", D);
  MZB_REQUIRE(v == nullptr || v == kv || main_kv == nullptr || topk == 0, MZB_ERR_UNSUPPORTED,
              "attn_fwd: a separate V is supported for the window-only kernel");
  MZB_REQUIRE(err != nullptr, MZB_ERR_SHAPE, "attn_fwd: needs an error word");
  MZB_REQUIRE(S * H * D < (int64_t(1) << 40), MZB_ERR_SHAPE, "attn_fwd: too large");
  attn::Args a{};
  a.main_kv = static_cast<const __nv_bfloat16*>(main_kv);
  a.idx = indices;
  a.sinks = sinks;
  a.o = static_cast<__nv_bfloat16*>(o);
  a.lse = lse;
  a.B = int(B); a.S = int(S); a.H = H; a.window = window; a.G = int(G); a.topk = topk;
  if (!main_kv || topk == 0 || G == 0) { a.main_kv = nullptr; a.topk = 0; }
  a.scale_log2 = softmax_scale * attn::LOG2E;
  a.err = err;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool sep = v != nullptr && v != kv;
  switch (D) {
    case 64: return sep ? attn::launch<64, true>(q, kv, v, a, st) : attn::launch<64, false>(q, kv, v, a, st);
    case 128: return sep ? attn::launch<128, true>(q, kv, v, a, st) : attn::launch<128, false>(q, kv, v, a, st);
    default: return sep ? attn::launch<256, true>(q, kv, v, a, st) : attn::launch<256, false>(q, kv, v, a, st);
  }
}
