// Lightning indexer: score GEMM on tcgen05 tensor cores and exact top-k selection.
//
// Reference: src/mzoo/layers/attn/indexer/fwd.py:48-132 (`index_score`, `fwd`),
// indexer/attn.py:67-81 (`attn`: topk on the score matrix), golden_ref.py:213-243
// (`indexer_scores`, `topk_indices`), and the model's absolute-position form
// archs/dsv4/modeling_deepseek_v41.py:555-556 (`compress_lens = (position_ids + 1) // ratio`).
//
//   score[b,s,t] = scale * sk[b,t] * sum_h (w[b,s,h] * sq[b,s,h]) * relu(q[b,s,h,:] . k[b,t,:])
//   visible iff t < (q_offset + s + 1) // ratio, else -inf
//
// (bf16 mode: sq = sk = 1, scale = Di^-1/2 -- the reference kernel; fp8 mode: e4m3 codes
// with fp32 per-(token, head) / per-key scales, scale = 1 -- BASELINE config 2.)
//
// Kernel 1 (`score_kernel`): keys in the MMA M dimension (128 per tile), (token, head)
// query rows in N (up to 256 = T_q tokens x Hi heads), so the per-token head reduction is
// a per-thread loop over TMEM columns.  Persistent CTAs, one per SM; warp 0 issues TMA
// loads (K tiles in a 4-stage ring, Q tiles double-buffered), warp 1 issues tcgen05.mma
// into two TMEM accumulators, warps 4-11 run the relu * weight reduction epilogue and
// store fp32 scores.  The key loop stops at the block's causal frontier.
//
// Kernel 2 (`topk_kernel`): one CTA per query row.  The fp32 tensor-core scores carry a
// rounding error bounded by delta = eps * A_s * max_t B_t, with
// A_s = sum_h |w sq| * ||q_h||_2 and B_t = |scale| sk_t ||k_t||_2 (Cauchy-Schwarz on the
// dot products plus the fp32 reductions).  A radix select finds the approximate k-th
// score theta; keys above theta + 2 delta are certainly selected, keys below
// theta - 2 delta certainly not, and the few in between are re-scored EXACTLY in fp64
// (e4m3 and bf16 products are exact in fp64, the 8-bit-code sums are exact too) and
// ranked by (score desc, index asc).  The selected indices are written in ascending
// order, -1 padded.  The result therefore equals the top-k of the canonical fp64 score
//   c_h = w*sq (exact), dot_h = sum_i q*k (fp64, sequential), p_h = c_h*max(dot_h, 0),
//   acc = ((p_0 + p_1) + ...) + p_{Hi-1}, score = (acc * sk) * scale,
// with ties to the lower index -- which is what the CPU oracle computes.
#include "tc.cuh"

namespace mzb {
namespace idx {

constexpr int BM = 128;  // keys per tile = MMA M
constexpr int NTHREADS = 384;
constexpr int EPI_WARP0 = 4;
constexpr int NEPI = 256;
constexpr int KB_PARTS = 16;  // per-batch partial maxima of B_t

template <bool FP8, int DI>
struct Cfg {
  static constexpr int EB = FP8 ? 1 : 2;
  static constexpr int R = DI * EB;  // bytes per row
  static constexpr int SW = (R % 128 == 0) ? 128 : ((R % 64 == 0) ? 64 : 32);
  static constexpr int NCB = R / SW;
  static constexpr int KSTEPS = R / 32;  // 32 bytes of K per MMA (K=16 bf16, K=32 e4m3)
  static constexpr int NMAX = (R <= 256) ? 256 : 128;
  static constexpr int Q_BYTES = NMAX * R;
  static constexpr int K_BYTES = BM * R;
  static constexpr int BUDGET = 200 * 1024;
  static constexpr int Q_BUFS = (2 * Q_BYTES + 2 * K_BYTES <= BUDGET) ? 2 : 1;
  static constexpr int KS_RAW = (BUDGET - Q_BUFS * Q_BYTES) / K_BYTES;
  static constexpr int K_STAGES = KS_RAW > 4 ? 4 : KS_RAW;
  static constexpr int TMEM_COLS = 2 * NMAX;
  static constexpr int SMEM = Q_BUFS * Q_BYTES + K_STAGES * K_BYTES + NMAX * 4 + 256 + 1024;
  static_assert(R % 32 == 0, "row bytes must be a multiple of 32");
  static_assert(K_STAGES >= 2, "smem budget");
};

struct ScoreArgs {
  const float* w;
  const float* sq;
  const float* sk;
  const int32_t* q_pos;  // [B*S] absolute positions, or null (q_offset + s)
  float* scores;
  int B, S, T, Hi, Tq, N;
  int ratio;
  long long q_offset;
  float scale;
  int write_tail;
  int* err;
};

__device__ __forceinline__ int visible_keys(long long q_offset, long long s, int ratio, int T) {
  long long v = (q_offset + s + 1) / ratio;
  return v < 0 ? 0 : (v > T ? T : int(v));
}

// Visible keys of query (b, s): position q_pos[b*S+s] when given, else q_offset + s.
__device__ __forceinline__ int visible_of(const int32_t* q_pos, long long q_offset, int b, int S, int s, int ratio,
                                          int T) {
  if (q_pos) return visible_keys(0, (long long)q_pos[(long long)b * S + s], ratio, T);
  return visible_keys(q_offset, s, ratio, T);
}

template <bool FP8, int DI>
__global__ void __launch_bounds__(NTHREADS, 1)
    score_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk, ScoreArgs a) {
  using C = Cfg<FP8, DI>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = smem;
  uint8_t* ks = qs + C::Q_BUFS * C::Q_BYTES;
  float* cw = reinterpret_cast<float*>(ks + C::K_STAGES * C::K_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(cw + C::NMAX);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 2;
  uint64_t* k_full = bars + 4;
  uint64_t* k_empty = k_full + C::K_STAGES;
  uint64_t* acc_full = k_empty + C::K_STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&q_full[i], 1);
      tc::mbar_init(&q_empty[i], 1);
      tc::mbar_init(&acc_full[i], 1);
      tc::mbar_init(&acc_empty[i], NEPI / 32);
    }
    for (int i = 0; i < C::K_STAGES; ++i) {
      tc::mbar_init(&k_full[i], 1);
      tc::mbar_init(&k_empty[i], 1);
    }
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, C::TMEM_COLS);
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&tq);
    tc::prefetch_tmap(&tk);
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  const int n_tb = (a.S + a.Tq - 1) / a.Tq;
  const int items = a.B * n_tb;
  auto item_tiles = [&](int tb, int b) {
    int vis = 0;
    for (int s = tb * a.Tq; s < min((tb + 1) * a.Tq, a.S); ++s)
      vis = max(vis, visible_of(a.q_pos, a.q_offset, b, a.S, s, a.ratio, a.T));
    return (vis + BM - 1) / BM;
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int ks_i = 0, ks_ph = 0, qi = 0;
      uint32_t k_issued = 0, k_par[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      uint32_t q_issued = 0, q_par[2] = {0, 0};
      for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x) {
        const int tb = n_tb - 1 - it / a.B, b = it % a.B;
        const int qb = qi % C::Q_BUFS, qpar = (qi / C::Q_BUFS) & 1;
        if (!tc::mbar_wait(&q_empty[qb], qpar ^ 1, a.err, 101)) { *abort_flag = 1; break; }
        tc::mbar_expect_tx(&q_full[qb], uint32_t(a.N) * C::R);
        for (int cb = 0; cb < C::NCB; ++cb)
          tc::tma_load_3d(qs + qb * C::Q_BYTES + cb * C::NMAX * C::SW, &tq, &q_full[qb], cb * C::SW / C::EB,
                          tb * a.Tq * a.Hi, b);
        q_issued |= 1u << qb;
        q_par[qb] = qpar;
        const int n_kt = item_tiles(tb, b);
        for (int kt = 0; kt < n_kt; ++kt) {
          if (!tc::mbar_wait(&k_empty[ks_i], ks_ph ^ 1, a.err, 102)) { *abort_flag = 1; break; }
          tc::mbar_expect_tx(&k_full[ks_i], C::K_BYTES);
          for (int cb = 0; cb < C::NCB; ++cb)
            tc::tma_load_3d(ks + ks_i * C::K_BYTES + cb * BM * C::SW, &tk, &k_full[ks_i], cb * C::SW / C::EB,
                            kt * BM, b);
          k_issued |= 1u << ks_i;
          k_par[ks_i] = ks_ph;
          if (++ks_i == C::K_STAGES) { ks_i = 0; ks_ph ^= 1; }
        }
        ++qi;
      }
      if (*abort_flag) {  // drain this CTA's own copies before the CTA (and its smem) goes away
        for (int i = 0; i < C::K_STAGES; ++i)
          if (k_issued >> i & 1) tc::mbar_wait(&k_full[i], k_par[i], nullptr, 0);
        for (int i = 0; i < 2; ++i)
          if (q_issued >> i & 1) tc::mbar_wait(&q_full[i], q_par[i], nullptr, 0);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t kFmt = FP8 ? 0 : 1;
      const uint32_t idesc = tc::make_idesc(BM, a.N, kFmt, kFmt);
      int ks_i = 0, ks_ph = 0, acc = 0, acc_ph = 0, qi = 0;
      for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x) {
        const int tb = n_tb - 1 - it / a.B, b = it % a.B;
        const int qb = qi % C::Q_BUFS, qpar = (qi / C::Q_BUFS) & 1;
        if (!tc::mbar_wait(&q_full[qb], qpar, a.err, 103)) { *abort_flag = 1; break; }
        const uint32_t q_base = smem_u32(qs + qb * C::Q_BYTES);
        const int n_kt = item_tiles(tb, b);
        for (int kt = 0; kt < n_kt; ++kt) {
          if (!tc::mbar_wait(&acc_empty[acc], acc_ph ^ 1, a.err, 104)) { *abort_flag = 1; break; }
          if (!tc::mbar_wait(&k_full[ks_i], ks_ph, a.err, 105)) { *abort_flag = 1; break; }
          tc::fence_after_sync();
          const uint32_t k_base = smem_u32(ks + ks_i * C::K_BYTES);
          const uint32_t d = tmem + uint32_t(acc * C::NMAX);
#pragma unroll
          for (int kk = 0; kk < C::KSTEPS; ++kk) {
            const int byte = kk * 32, cb = byte / C::SW, off = byte % C::SW;
            const uint64_t ad = tc::make_sdesc<C::SW>(k_base + cb * BM * C::SW + off, 16, 8 * C::SW);
            const uint64_t bd = tc::make_sdesc<C::SW>(q_base + cb * C::NMAX * C::SW + off, 16, 8 * C::SW);
            tc::mma_ss<FP8 ? 1 : 0>(d, ad, bd, idesc, kk > 0);
          }
          tc::mma_commit(&k_empty[ks_i]);
          tc::mma_commit(&acc_full[acc]);
          if (++ks_i == C::K_STAGES) { ks_i = 0; ks_ph ^= 1; }
          acc ^= 1;
          if (acc == 0) acc_ph ^= 1;
        }
        tc::mma_commit(&q_empty[qb]);
        ++qi;
      }
    }
  } else if (warp >= EPI_WARP0) {
    // ---------------------------------------------------------------- epilogue
    const int et = threadIdx.x - EPI_WARP0 * 32;  // 0..255
    const int quarter = warp & 3;
    const int wg = (warp - EPI_WARP0) >> 2;  // 0/1: even / odd tokens
    const int row = quarter * 32 + lane;     // key row inside the tile
    int acc = 0, acc_ph = 0;
    for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x) {
      const int tb = n_tb - 1 - it / a.B, b = it % a.B;
      const int s0 = tb * a.Tq;
      tc::bar_sync(1, NEPI);
      for (int i = et; i < a.N; i += NEPI) {
        const int s = s0 + i / a.Hi, h = i % a.Hi;
        float c = 0.0f;
        if (s < a.S) {
          const size_t o = (size_t(b) * a.S + s) * a.Hi + h;
          c = a.w[o] * (a.sq ? a.sq[o] : 1.0f);
        }
        cw[i] = c;
      }
      tc::bar_sync(1, NEPI);
      const int n_kt = item_tiles(tb, b);
      for (int kt = 0; kt < n_kt; ++kt) {
        if (!tc::mbar_wait(&acc_full[acc], acc_ph, a.err, 106)) { *abort_flag = 1; break; }
        tc::fence_after_sync();
        const int j = kt * BM + row;
        const float skj = (j < a.T) ? (a.sk ? a.sk[size_t(b) * a.T + j] : 1.0f) * a.scale : 0.0f;
        const uint32_t tbase = tc::taddr(tmem, quarter * 32, acc * C::NMAX);
        for (int t = wg; t < a.Tq; t += 2) {
          float sum = 0.0f;
          for (int h0 = 0; h0 < a.Hi; h0 += 64) {
            uint32_t r[4][16];
            const int nch = min(4, (a.Hi - h0) >> 4);
#pragma unroll
            for (int c = 0; c < 4; ++c)
              if (c < nch) tc::tmem_ld16(tbase + t * a.Hi + h0 + c * 16, r[c]);
            tc::tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              if (c < nch) {
                const float4* cwp = reinterpret_cast<const float4*>(cw + t * a.Hi + h0 + c * 16);
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                  const float4 cc = cwp[q4];
                  sum = fmaf(fmaxf(__uint_as_float(r[c][q4 * 4 + 0]), 0.0f), cc.x, sum);
                  sum = fmaf(fmaxf(__uint_as_float(r[c][q4 * 4 + 1]), 0.0f), cc.y, sum);
                  sum = fmaf(fmaxf(__uint_as_float(r[c][q4 * 4 + 2]), 0.0f), cc.z, sum);
                  sum = fmaf(fmaxf(__uint_as_float(r[c][q4 * 4 + 3]), 0.0f), cc.w, sum);
                }
              }
            }
          }
          const int s = s0 + t;
          if (s < a.S && j < a.T) {
            const int vis = visible_of(a.q_pos, a.q_offset, b, a.S, s, a.ratio, a.T);
            a.scores[(size_t(b) * a.S + s) * a.T + j] = (j < vis) ? sum * skj : -INFINITY;
          }
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&acc_empty[acc]);
        acc ^= 1;
        if (acc == 0) acc_ph ^= 1;
      }
      if (a.write_tail) {  // keys no token of this block can see
        const int t0 = n_kt * BM;
        for (int t = 0; t < a.Tq; ++t) {
          const int s = s0 + t;
          if (s >= a.S) break;
          float* rowp = a.scores + (size_t(b) * a.S + s) * a.T;
          for (int j = t0 + et; j < a.T; j += NEPI) rowp[j] = -INFINITY;
        }
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_free(tmem, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------- top-k

struct TopkArgs {
  const float* scores;
  const uint8_t* q;
  const uint8_t* k;
  const float* w;
  const float* sq;
  const float* sk;
  const float* kbmax;  // [B, KB_PARTS]
  const int32_t* q_pos;
  int32_t* out;
  int B, S, T, Hi, Di, topk, ratio;
  long long q_offset;
  float scale, eps;
  int fp8;
  int* err;
};

constexpr int TK_THREADS = 256;
constexpr int CAND_MAX = 2048;

__device__ __forceinline__ uint32_t f2key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

__device__ __forceinline__ float elem_f(const uint8_t* p, int i, int fp8) {
  if (fp8) return e4m3_to_float(p[i]);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

// B_t = |scale| * sk_t * ||k_t||_2, partial maxima per (batch, part).
__global__ void kbound_kernel(TopkArgs a) {
  const int b = blockIdx.x, part = blockIdx.y;
  const int eb = a.fp8 ? 1 : 2;
  float m = 0.0f;
  const int per = (a.T + KB_PARTS - 1) / KB_PARTS;
  const int t_lo = part * per, t_hi = min(a.T, t_lo + per);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int t = t_lo + warp; t < t_hi; t += blockDim.x >> 5) {
    const uint8_t* kr = a.k + (size_t(b) * a.T + t) * a.Di * eb;
    float ss = 0.0f;
    for (int i = lane; i < a.Di; i += 32) {
      const float v = elem_f(kr, i, a.fp8);
      ss = fmaf(v, v, ss);
    }
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float sk = a.sk ? a.sk[size_t(b) * a.T + t] : 1.0f;
    m = fmaxf(m, fabsf(a.scale) * fabsf(sk) * sqrtf(ss));
  }
  __shared__ float red[32];
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float r = 0.0f;
    for (int i = 0; i < int(blockDim.x >> 5); ++i) r = fmaxf(r, red[i]);
    const_cast<float*>(a.kbmax)[b * KB_PARTS + part] = r;
  }
}

__global__ void __launch_bounds__(TK_THREADS) topk_kernel(TopkArgs a) {
  extern __shared__ uint8_t sm[];
  const int row = blockIdx.x;  // b * S + s
  const int b = row / a.S, s = row % a.S;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int32_t* out = a.out + size_t(row) * a.topk;
  const int V = visible_of(a.q_pos, a.q_offset, b, a.S, s, a.ratio, a.T);
  if (V <= a.topk) {
    for (int i = tid; i < a.topk; i += TK_THREADS) out[i] = i < V ? i : -1;
    return;
  }
  const int eb = a.fp8 ? 1 : 2;
  const int qstride = a.Di * eb + 4;  // padded rows: lane-varying heads hit different banks
  // smem carve-up
  uint32_t* keys = reinterpret_cast<uint32_t*>(sm);                        // V
  uint32_t* sel = keys + V;                                                // ceil(V/32)
  const int nsel = (V + 31) >> 5;
  int* cand = reinterpret_cast<int*>(sel + nsel);                          // CAND_MAX
  double* exact = reinterpret_cast<double*>(                               // CAND_MAX
      (reinterpret_cast<uintptr_t>(cand + CAND_MAX) + 7) & ~uintptr_t(7));
  double* pbuf = exact + CAND_MAX;                                         // 8 warps x Hi
  double* cq = pbuf + 8 * a.Hi;                                            // Hi
  uint8_t* qrow = reinterpret_cast<uint8_t*>(cq + a.Hi);                   // Hi x qstride
  __shared__ int hist[256];
  __shared__ uint32_t sh_prefix, sh_kk;
  __shared__ int n_in, n_cand, sh_scan[TK_THREADS];
  __shared__ float sh_A;

  const float* srow = a.scores + size_t(row) * a.T;
  for (int j = tid; j < V; j += TK_THREADS) keys[j] = f2key(srow[j]);
  for (int i = tid; i < nsel; i += TK_THREADS) sel[i] = 0u;
  // stage the query row and its exact weights; A_s = sum_h |c_h| ||q_h||
  const uint8_t* qg = a.q + size_t(row) * a.Hi * a.Di * eb;
  for (int i = tid; i < a.Hi * a.Di * eb; i += TK_THREADS) {
    const int h = i / (a.Di * eb), o = i % (a.Di * eb);
    qrow[h * qstride + o] = qg[i];
  }
  for (int h = tid; h < a.Hi; h += TK_THREADS) {
    const size_t o = size_t(row) * a.Hi + h;
    cq[h] = double(a.w[o]) * double(a.sq ? a.sq[o] : 1.0f);
  }
  if (tid == 0) { sh_A = 0.0f; n_in = 0; n_cand = 0; }
  __syncthreads();
  {
    float part = 0.0f;
    for (int h = warp; h < a.Hi; h += TK_THREADS / 32) {
      float ss = 0.0f;
      for (int i = lane; i < a.Di; i += 32) {
        const float v = elem_f(qrow + h * qstride, i, a.fp8);
        ss = fmaf(v, v, ss);
      }
      for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      part += float(fabs(cq[h])) * sqrtf(ss);
    }
    if (lane == 0) atomicAdd(&sh_A, part);
  }
  // radix select: the topk-th largest key (MSB-first, 8-bit digits)
  uint32_t prefix = 0, mask = 0, kk = a.topk;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = tid; i < 256; i += TK_THREADS) hist[i] = 0;
    __syncthreads();
    for (int j = tid; j < V; j += TK_THREADS) {
      const uint32_t kx = keys[j];
      if ((kx & mask) == prefix) atomicAdd(&hist[(kx >> shift) & 255], 1);
    }
    __syncthreads();
    if (warp == 0) {
      // lane l owns bins 255-8l .. 248-8l (descending)
      int cnt[8], tot = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) { cnt[i] = hist[255 - 8 * lane - i]; tot += cnt[i]; }
      int incl = tot;
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      const int excl = incl - tot;
      if (excl < int(kk) && int(kk) <= incl) {
        int run = excl;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (run < int(kk) && int(kk) <= run + cnt[i]) {
            sh_prefix = prefix | (uint32_t(255 - 8 * lane - i) << shift);
            sh_kk = kk - run;
          }
          run += cnt[i];
        }
      }
    }
    __syncthreads();
    prefix = sh_prefix;
    kk = sh_kk;
    mask |= 255u << shift;
  }
  const float theta = key2f(prefix);
  float kbm = 0.0f;
  for (int i = 0; i < KB_PARTS; ++i) kbm = fmaxf(kbm, a.kbmax[b * KB_PARTS + i]);
  const float delta = a.eps * sh_A * kbm * 1.0001f;
  const float hi_thr = __fadd_ru(theta, 2.0f * delta), lo_thr = __fsub_rd(theta, 2.0f * delta);
  for (int j = tid; j < V; j += TK_THREADS) {
    const float v = key2f(keys[j]);
    if (v > hi_thr) {
      atomicOr(&sel[j >> 5], 1u << (j & 31));
      atomicAdd(&n_in, 1);
    } else if (v >= lo_thr) {
      const int c = atomicAdd(&n_cand, 1);
      if (c < CAND_MAX) cand[c] = j;
    }
  }
  __syncthreads();
  const int nin = n_in, nc = n_cand;
  const int need = a.topk - nin;
  if (nc > CAND_MAX || need < 0 || need > nc) {
    if (tid == 0) atomicExch(a.err, MZB_ERR_BOUND);
    for (int i = tid; i < a.topk; i += TK_THREADS) out[i] = -1;
    return;
  }
  // exact fp64 re-scoring, one warp per candidate; lane l owns heads l, l+32, ...
  for (int c = warp; c < nc; c += TK_THREADS / 32) {
    const int j = cand[c];
    const uint8_t* kr = a.k + (size_t(b) * a.T + j) * a.Di * eb;
    for (int h = lane; h < a.Hi; h += 32) {
      const uint8_t* qh = qrow + h * qstride;
      double dot = 0.0;
      for (int i = 0; i < a.Di; ++i) dot = fma(double(elem_f(qh, i, a.fp8)), double(elem_f(kr, i, a.fp8)), dot);
      pbuf[warp * a.Hi + h] = __dmul_rn(cq[h], dot > 0.0 ? dot : 0.0);
    }
    __syncwarp();
    if (lane == 0) {
      double acc = 0.0;
      for (int h = 0; h < a.Hi; ++h) acc = __dadd_rn(acc, pbuf[warp * a.Hi + h]);
      const double skj = a.sk ? double(a.sk[size_t(b) * a.T + j]) : 1.0;
      exact[c] = __dmul_rn(__dmul_rn(acc, skj), double(a.scale));
    }
    __syncwarp();
  }
  __syncthreads();
  // rank candidates by (score desc, index asc); keep the best `need`
  for (int c = tid; c < nc; c += TK_THREADS) {
    const double e = exact[c];
    const int j = cand[c];
    int rank = 0;
    for (int o = 0; o < nc; ++o) {
      const double f = exact[o];
      rank += (f > e) || (f == e && cand[o] < j);
    }
    if (rank < need) atomicOr(&sel[j >> 5], 1u << (j & 31));
  }
  __syncthreads();
  // ascending compaction of the selected bits
  const int per = (nsel + TK_THREADS - 1) / TK_THREADS;
  const int w0 = tid * per, w1 = min(nsel, w0 + per);
  int cnt = 0;
  for (int i = w0; i < w1; ++i) cnt += __popc(sel[i]);
  sh_scan[tid] = cnt;
  __syncthreads();
  for (int o = 1; o < TK_THREADS; o <<= 1) {
    const int v = tid >= o ? sh_scan[tid - o] : 0;
    __syncthreads();
    sh_scan[tid] += v;
    __syncthreads();
  }
  int pos = sh_scan[tid] - cnt;
  for (int i = w0; i < w1; ++i) {
    uint32_t bits = sel[i];
    while (bits) {
      const int bit = __ffs(bits) - 1;
      bits &= bits - 1;
      if (pos < a.topk) out[pos] = i * 32 + bit;
      ++pos;
    }
  }
  const int total = sh_scan[TK_THREADS - 1];
  for (int i = total + tid; i < a.topk; i += TK_THREADS) out[i] = -1;
}

static size_t topk_smem(int T, int Hi, int Di, int eb) {
  size_t V = size_t(T);
  size_t bytes = V * 4 + ((V + 31) / 32) * 4 + CAND_MAX * 4 + 8;
  bytes += CAND_MAX * 8 + 8 * Hi * 8 + Hi * 8 + size_t(Hi) * (Di * eb + 4) + 16;
  return bytes;
}

template <bool FP8, int DI>
static int launch_scores(const void* q, const void* k, const ScoreArgs& a, cudaStream_t st) {
  using C = Cfg<FP8, DI>;
  CUtensorMap tq, tk;
  const CUtensorMapDataType dt = FP8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const CUtensorMapSwizzle swz = C::SW == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : (C::SW == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
  {
    const uint64_t dims[3] = {uint64_t(DI), uint64_t(a.S) * a.Hi, uint64_t(a.B)};
    const uint64_t str[2] = {uint64_t(C::R), uint64_t(a.S) * a.Hi * C::R};
    const uint32_t box[3] = {uint32_t(C::SW / C::EB), uint32_t(a.N), 1};
    int e = encode_tmap(&tq, dt, 3, q, dims, str, box, swz);
    if (e) return e;
  }
  {
    const uint64_t dims[3] = {uint64_t(DI), uint64_t(a.T), uint64_t(a.B)};
    const uint64_t str[2] = {uint64_t(C::R), uint64_t(a.T) * C::R};
    const uint32_t box[3] = {uint32_t(C::SW / C::EB), uint32_t(BM), 1};
    int e = encode_tmap(&tk, dt, 3, k, dims, str, box, swz);
    if (e) return e;
  }
  auto kern = score_kernel<FP8, DI>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
    return launch_status("indexer_scores(smem attr)");
  const int n_tb = (a.S + a.Tq - 1) / a.Tq;
  const int items = a.B * n_tb;
  const int grid = items < num_sms() ? items : num_sms();
  kern<<<grid, NTHREADS, C::SMEM, st>>>(tq, tk, a);
  return launch_status("indexer_scores");
}

}  // namespace idx
}  // namespace mzb

using namespace mzb;

static int indexer_common_checks(const void* q, const void* k, int64_t B, int64_t S, int64_t T, int Hi, int Di,
                                 int dtype, int ratio) {
  MZB_REQUIRE(dtype == MZB_BF16 || dtype == MZB_E4M3, MZB_ERR_UNSUPPORTED,
              "indexer: q/k must be bf16 or e4m3 (dtype code %d)", dtype);
  MZB_REQUIRE(B >= 1 && S >= 1 && T >= 0, MZB_ERR_SHAPE, "indexer: bad shape B=%lld S=%lld T=%lld",
              (long long)B, (long long)S, (long long)T);
  MZB_REQUIRE(Hi >= 16 && Hi <= 256 && Hi % 16 == 0, MZB_ERR_SHAPE,
              "indexer: index heads must be a multiple of 16 in [16, 256] (pad with zero weights), got %d", Hi);
  MZB_REQUIRE(ratio >= 1, MZB_ERR_SHAPE, "indexer: compress_ratio must be >= 1, got %d", ratio);
  MZB_REQUIRE(reinterpret_cast<uintptr_t>(q) % 16 == 0 && reinterpret_cast<uintptr_t>(k) % 16 == 0, MZB_ERR_ALIGN,
              "indexer: q/k must be 16-byte aligned");
  MZB_REQUIRE(S * Hi < (int64_t(1) << 31) && B * S * T < (int64_t(1) << 40), MZB_ERR_SHAPE, "indexer: too large");
  (void)Di;
  return MZB_OK;
}

extern "C" int mzb_indexer_scores(const void* q, const void* k, const float* w, const float* sq, const float* sk,
                                  const int32_t* q_pos, float* scores, int64_t B, int64_t S, int64_t T, int Hi,
                                  int Di, int dtype, int ratio, int64_t q_offset, float scale, int write_tail,
                                  int* err, void* stream) {
  int e = indexer_common_checks(q, k, B, S, T, Hi, Di, dtype, ratio);
  if (e) return e;
  MZB_REQUIRE(dtype == MZB_BF16 || (sq && sk), MZB_ERR_SHAPE, "indexer: fp8 inputs need sq and sk scales");
  if (T == 0) return MZB_OK;
  idx::ScoreArgs a{};
  a.w = w; a.sq = sq; a.sk = sk; a.q_pos = q_pos; a.scores = scores;
  a.B = int(B); a.S = int(S); a.T = int(T); a.Hi = Hi;
  const int nmax = (Di * (dtype == MZB_E4M3 ? 1 : 2) <= 256) ? 256 : 128;
  a.Tq = nmax / Hi;
  MZB_REQUIRE(a.Tq >= 1, MZB_ERR_SHAPE, "indexer: Hi=%d too large for Di=%d", Hi, Di);
  a.N = a.Tq * Hi;
  a.ratio = ratio; a.q_offset = q_offset; a.scale = scale; a.write_tail = write_tail; a.err = err;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == MZB_E4M3) {
    switch (Di) {
      case 64: return idx::launch_scores<true, 64>(q, k, a, st);
      case 128: return idx::launch_scores<true, 128>(q, k, a, st);
    }
  } else {
    switch (Di) {
      case 32: return idx::launch_scores<false, 32>(q, k, a, st);
      case 64: return idx::launch_scores<false, 64>(q, k, a, st);
      case 96: return idx::launch_scores<false, 96>(q, k, a, st);
      case 128: return idx::launch_scores<false, 128>(q, k, a, st);
      case 256: return idx::launch_scores<false, 256>(q, k, a, st);
    }
  }
  set_error("indexer: unsupported index head dim %d for dtype code %d", Di, dtype);
  return MZB_ERR_UNSUPPORTED;
}

extern "C" int mzb_indexer_topk(const float* scores, const void* q, const void* k, const float* w, const float* sq,
                                const float* sk, const int32_t* q_pos, float* kbmax_ws, int32_t* out, int64_t B,
                                int64_t S, int64_t T,
                                int Hi, int Di, int dtype, int ratio, int64_t q_offset, float scale, int topk,
                                float eps, int* err, void* stream) {
  int e = indexer_common_checks(q, k, B, S, T, Hi, Di, dtype, ratio);
  if (e) return e;
  MZB_REQUIRE(topk >= 1, MZB_ERR_SHAPE, "indexer topk: topk must be >= 1, got %d", topk);
  MZB_REQUIRE(err != nullptr, MZB_ERR_SHAPE, "indexer topk: needs an error word");
  MZB_REQUIRE(dtype == MZB_BF16 || (sq && sk), MZB_ERR_SHAPE, "indexer: fp8 inputs need sq and sk scales");
  const int eb = dtype == MZB_E4M3 ? 1 : 2;
  const size_t smem = idx::topk_smem(int(T), Hi, Di, eb);
  MZB_REQUIRE(smem <= 200 * 1024, MZB_ERR_UNSUPPORTED, "indexer topk: T=%lld needs %zu B of shared memory",
              (long long)T, smem);
  idx::TopkArgs a{};
  a.scores = scores; a.q = static_cast<const uint8_t*>(q); a.k = static_cast<const uint8_t*>(k);
  a.w = w; a.sq = sq; a.sk = sk; a.q_pos = q_pos; a.kbmax = kbmax_ws; a.out = out;
  a.B = int(B); a.S = int(S); a.T = int(T); a.Hi = Hi; a.Di = Di; a.topk = topk; a.ratio = ratio;
  a.q_offset = q_offset; a.scale = scale; a.eps = eps; a.fp8 = dtype == MZB_E4M3; a.err = err;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (T > 0) {
    idx::kbound_kernel<<<dim3(unsigned(B), idx::KB_PARTS), 256, 0, st>>>(a);
    if (int r = launch_status("indexer_kbound")) return r;
  }
  if (cudaFuncSetAttribute(idx::topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
    return launch_status("indexer_topk(smem attr)");
  idx::topk_kernel<<<unsigned(B * S), idx::TK_THREADS, smem, st>>>(a);
  return launch_status("indexer_topk");
}
