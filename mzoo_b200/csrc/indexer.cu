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
// into two TMEM accumulators, the epilogue warpgroups run the relu * weight reduction and
// store fp32 scores (modes below: one warpgroup per accumulator, or with 64 heads and
// four-token blocks two per accumulator, two tokens each).  The key loop stops at the
// block's causal frontier; with few (batch, query block) pairs (decode) every CTA takes an
// equal share of all visible key tiles so every SM gets the same work.
//
// Keys are either dense rows [B, T] or, for a paged KV cache (decode), rows of 64-key
// pages [P, 64] reached through a page table [B, max_pages] (`key_row`); the score kernel
// then loads each 128-key tile as its two 64-row pages.
//
// Kernel 2 (`topk_kernel`): one CTA per query row.  The fp32 tensor-core scores carry a
// rounding error bounded by delta = eps * A_s * max_t B_t, with
// A_s = sum_h |w sq| * ||q_h||_2 and B_t = |scale| sk_t ||k_t||_2 (Cauchy-Schwarz on the
// dot products plus the fp32 reductions; both factors come from `bound_kernel`).  A
// histogram over linear bins of a sampled score range, then an exact rank (or radix
// select) inside the cut bin, finds the approximate k-th score theta; keys above
// theta + 2 delta are certainly selected, keys below
// theta - 2 delta certainly not, and the few in between are re-scored EXACTLY in fp64
// (e4m3 and bf16 products are exact in fp64, the 8-bit-code sums are exact too) and
// ranked by (score desc, index asc).  The selected indices are written in ascending
// order, -1 padded.  The result therefore equals the top-k of the canonical fp64 score
//   c_h = w*sq (exact), dot_h = sum_i q*k (fp64, sequential), p_h = c_h*max(dot_h, 0),
//   acc = ((p_0 + p_1) + ...) + p_{Hi-1}, score = (acc * sk) * scale,
// with ties to the lower index -- which is what the CPU oracle computes.
#include <algorithm>

#include "tc.cuh"

namespace mzb {
namespace idx {

constexpr int BM = 128;  // keys per tile = MMA M
constexpr int NTHREADS = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int EPI_WARP0 = 2;   // epilogue warp w reads TMEM lanes 32 * (w % 4): warps 2-5 and 6-9
                               // each cover all four lane quarters
constexpr int KB_PARTS = 16;  // per-batch partial maxima of B_t
constexpr int BAL_MAX = 512;  // (batch, query block) units of the tile-balanced split
constexpr int SK_RING = 16;   // paged keys: per-tile key-scale slots in shared memory
constexpr int BARS_BYTES = 512;  // mbarriers, TMEM slot and abort flag
// Accumulator buffers in TMEM: two of NMAX columns, or four of 128 when a tile's query
// columns fit in 128 (decode: one token x 64 heads) -- small MMAs complete quickly but each
// buffer waits for the epilogue's TMEM read, so more buffers keep the MMA issuing.
__host__ __device__ constexpr int score_accs(int n) { return n <= 128 ? 4 : 2; }
constexpr int PREF_BYTES = 2304;  // tile prefix [BAL_MAX + 1] ints, rounded up to 256
static_assert((BAL_MAX + 1) * 4 <= PREF_BYTES, "prefix area");
static_assert(SK_RING > 12 && (SK_RING & (SK_RING - 1)) == 0, "scale ring: more slots than K stages + accumulators");

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
  // paged keys (decode: one query, a long key stream per unit) keep up to 8 tiles in flight
  static constexpr int K_STAGES_PAGED = KS_RAW > 8 ? 8 : KS_RAW;
  static constexpr int TMEM_COLS = 2 * NMAX;
  // dense keys: tiles, weights, barriers, tile prefix; paged keys add the key-scale ring
  static constexpr int SMEM =
      Q_BUFS * Q_BYTES + K_STAGES * K_BYTES + 8 * NMAX * 4 + BARS_BYTES + (BAL_MAX + 1) * 4 + 1024;
  static constexpr int SMEM_PAGED =
      Q_BUFS * Q_BYTES + K_STAGES_PAGED * K_BYTES + 8 * NMAX * 4 + BARS_BYTES + PREF_BYTES + SK_RING * BM * 4 + 1024;
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
  int kc, n_kc;  // key tiles per chunk, chunks per (batch, query block)
  int bal;       // 1: each CTA takes a contiguous 1/grid share of all key tiles (few units)
  const int32_t* k_pt;  // [B, k_ptw] page table of 64-key pages, or null (dense keys)
  int k_ptw, k_npages;
  int sk_ring;  // paged keys with 16-byte aligned scales: the TMA warp copies each tile's
                // 128 key scales into a shared-memory ring next to its key tile
  int* err;
};

// 32-bit load issued where written (asm volatile keeps the compiler from sinking a
// look-ahead load down to its first use).
__device__ __forceinline__ int ld_nc_s32(const int32_t* p) {
  int v;
  asm volatile("ld.global.nc.b32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// Row of key t of batch b: dense [B, T] rows, or through the page table of 64-key pages.
// Page ids are clamped into the pool: keys past a sequence's length are only ever masked,
// whatever its table holds there, so their (clamped) reads just have to stay in bounds.
__device__ __forceinline__ long long key_row(const int32_t* pt, int ptw, int npages, int T, int b, int t) {
  if (!pt) return (long long)b * T + t;
  const int pi = min(t >> 6, ptw - 1);  // a tile's second page may lie past the table's last column
  int pg = __ldg(pt + (long long)b * ptw + pi);
  pg = pg < 0 ? 0 : (pg >= npages ? npages - 1 : pg);
  return (long long)pg * 64 + (t & 63);
}

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

// Epilogue modes: 0 the generic head loop; 1 the 64-head indexer's (packed FMAs, one TMEM
// wait per token) with warpgroup g draining the accumulator buffers of parity g, i.e.
// alternate tiles, all tokens; 2 the same for four-token blocks with four warpgroups that
// each take one token of every tile (a buffer is released after four 16-column loads, so
// the MMA of the tile two ahead is not held up by a longer chain of loads).
__host__ __device__ constexpr int score_nthreads(int mode) { return mode == 2 ? NTHREADS + 256 : NTHREADS; }

template <bool FP8, int DI, int MODE, bool PAGED>
__global__ void __launch_bounds__(score_nthreads(MODE), 1)
    score_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk, ScoreArgs a) {
  using C = Cfg<FP8, DI>;
  constexpr int KST = PAGED ? C::K_STAGES_PAGED : C::K_STAGES;  // key stages in the ring
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = smem;
  uint8_t* ks = qs + C::Q_BUFS * C::Q_BYTES;
  float* cw = reinterpret_cast<float*>(ks + KST * C::K_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(cw + 8 * C::NMAX);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 2;
  uint64_t* k_full = bars + 4;
  uint64_t* k_empty = k_full + KST;
  uint64_t* acc_empty = k_empty + KST;  // [4]
  uint64_t* sk_full = acc_empty + 4;  // [SK_RING]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sk_full + SK_RING);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* pref = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(bars) + BARS_BYTES);  // [units + 1] tile prefix
  float* sks = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + BARS_BYTES + PREF_BYTES);  // [SK_RING][BM]
  // 4 x 128 columns need NMAX = 256; n_acc <= K_STAGES for the epilogue's k_empty wait
  const int n_acc = (MODE == 2 || C::NMAX != 256 || KST < 4) ? 2 : score_accs(a.N);
  const int acc_cols = n_acc == 4 ? 128 : C::NMAX;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&q_full[i], 1);
      tc::mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < 4; ++i) {
      tc::mbar_init(&acc_empty[i], MODE == 2 ? 16 : 4);  // the warps of the warpgroup(s) of buffer i
    }
    for (int i = 0; i < SK_RING; ++i) tc::mbar_init(&sk_full[i], 1);
    for (int i = 0; i < KST; ++i) {
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
  const int n_tb = (a.S + a.Tq - 1) / a.Tq;
  const int units = a.B * n_tb;  // (batch, query block) pairs
  auto unit_tiles = [&](int b, int tb) {  // key tiles a query block sees
    int vis = 0;
    for (int s = tb * a.Tq; s < min((tb + 1) * a.Tq, a.S); ++s)
      vis = max(vis, visible_of(a.q_pos, a.q_offset, b, a.S, s, a.ratio, a.T));
    return (vis + BM - 1) / BM;
  };
  if (a.bal) {
    // tile prefix over units (u = b * n_tb + tb): pref[u] tiles before u.  Every thread
    // counts one unit's tiles (position loads all in flight at once), then warp 2 scans.
    for (int u = threadIdx.x; u < units; u += blockDim.x) pref[u + 1] = unit_tiles(u / n_tb, u % n_tb);
    __syncthreads();
  }
  if (a.bal && warp == 2) {
    int run = 0;
    for (int u0 = 0; u0 < units; u0 += 32) {
      const int u = u0 + lane;
      const int nt = u < units ? pref[u + 1] : 0;
      __syncwarp();
      int incl = nt;
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      if (u < units) pref[u + 1] = run + incl;
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) pref[0] = 0;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  // item = (key chunk, query block, batch); chunk-major so full chunks go first
  const int items = a.B * n_tb * a.n_kc;
  struct Item {
    int tb, b, kc, k0, k1;
  };
  auto item_of = [&](int it) {
    Item r;
    r.kc = it / (a.B * n_tb);
    const int rem = it % (a.B * n_tb);
    r.tb = n_tb - 1 - rem / a.B;
    r.b = rem % a.B;
    const int n_kt = unit_tiles(r.b, r.tb);
    r.k0 = r.kc * a.kc;
    r.k1 = min(n_kt, r.k0 + a.kc);
    return r;
  };
  // Tile-balanced split (few units, e.g. decode): this CTA takes key tiles [lo, hi) of the
  // units' tiles laid end to end, as pieces (unit, k0, k1); units' lengths differ widely, so
  // a round-robin of fixed chunks would leave some CTAs with far more tiles than others.
  long long lo = 0, hi = 0;
  int u_first = 0;
  if (a.bal) {
    const long long total = pref[units];
    lo = total * blockIdx.x / gridDim.x;
    hi = total * (blockIdx.x + 1) / gridDim.x;
    int l = 0, h = units;  // first unit whose tiles end after lo
    while (l < h) {
      const int mid = (l + h) >> 1;
      if (pref[mid + 1] > lo) h = mid; else l = mid + 1;
    }
    u_first = l;
  }
  // the k-th work item of this CTA
  auto get_item = [&](int k, Item& r) -> bool {
    if (!a.bal) {
      const int it = blockIdx.x + k * gridDim.x;
      if (it >= items) return false;
      r = item_of(it);
      return true;
    }
    const int u = u_first + k;
    if (u >= units || pref[u] >= hi) return false;
    r.b = u / n_tb;
    r.tb = u % n_tb;
    r.k0 = int((lo > pref[u] ? lo : (long long)pref[u]) - pref[u]);
    r.k1 = int((hi < pref[u + 1] ? hi : (long long)pref[u + 1]) - pref[u]);
    r.kc = 1;  // the -inf tail of a unit is written in a separate pass in this mode
    return true;
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int ks_i = 0, ks_ph = 0, qi = 0;
      uint32_t k_issued = 0, k_par[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      uint32_t n_tiles = 0, sk_issued = 0, sk_par[SK_RING] = {};
      uint32_t q_issued = 0, q_par[2] = {0, 0};
      for (int k = 0; !*abort_flag; ++k) {
        Item m;
        if (!get_item(k, m)) break;
        if (m.k0 >= m.k1) continue;
        const int qb = qi % C::Q_BUFS, qpar = (qi / C::Q_BUFS) & 1;
        if (!tc::mbar_wait(&q_empty[qb], qpar ^ 1, a.err, 101)) { *abort_flag = 1; break; }
        tc::mbar_expect_tx(&q_full[qb], uint32_t(a.N) * C::R);
        for (int cb = 0; cb < C::NCB; ++cb)
          tc::tma_load_3d(qs + qb * C::Q_BYTES + cb * C::NMAX * C::SW, &tq, &q_full[qb], cb * C::SW / C::EB,
                          m.tb * a.Tq * a.Hi, m.b);
        q_issued |= 1u << qb;
        q_par[qb] = qpar;
        // paged keys: each tile's two page ids are requested two tiles before its loads are
        // issued (this one thread issues every load, so a page-table read per tile on its
        // path would cap the key stream at one L2 round trip per tile)
        const int32_t* ptrow = PAGED ? a.k_pt + (long long)m.b * a.k_ptw : nullptr;
        auto page_id = [&](int t) { return ld_nc_s32(ptrow + min(t >> 6, a.k_ptw - 1)); };
        int pc0 = 0, pc1 = 0, pn0 = 0, pn1 = 0;  // raw page ids of tiles kt and kt + 1
        if (PAGED) {
          pc0 = page_id(m.k0 * BM);
          pc1 = page_id(m.k0 * BM + 64);
          if (m.k0 + 1 < m.k1) {
            pn0 = page_id((m.k0 + 1) * BM);
            pn1 = page_id((m.k0 + 1) * BM + 64);
          }
        }
        for (int kt = m.k0; kt < m.k1; ++kt) {
          int pf0 = 0, pf1 = 0;  // tile kt + 2
          if (PAGED && kt + 2 < m.k1) {
            pf0 = page_id((kt + 2) * BM);
            pf1 = page_id((kt + 2) * BM + 64);
          }
          auto row_of = [&](int pg) { return (pg < 0 ? 0 : (pg >= a.k_npages ? a.k_npages - 1 : pg)) * 64; };
          const int r0 = row_of(pc0), r1 = row_of(pc1);
          pc0 = pn0; pc1 = pn1; pn0 = pf0; pn1 = pf1;
          if (!tc::mbar_wait(&k_empty[ks_i], ks_ph ^ 1, a.err, 102)) { *abort_flag = 1; break; }
          tc::mbar_expect_tx(&k_full[ks_i], C::K_BYTES);
          if constexpr (PAGED) {  // two 64-key pages (2D map over the page pool's rows)
            for (int cb = 0; cb < C::NCB; ++cb) {
              uint8_t* dst = ks + ks_i * C::K_BYTES + cb * BM * C::SW;
              tc::tma_load_2d(dst, &tk, &k_full[ks_i], cb * C::SW / C::EB, r0);
              tc::tma_load_2d(dst + 64 * C::SW, &tk, &k_full[ks_i], cb * C::SW / C::EB, r1);
            }
            if (a.sk_ring) {
              // The tile's key scales (two 256-byte page rows).  Slot reuse is safe without an
              // empty barrier: this copy waited (k_empty above) for the MMA of the tile
              // KST back, which waited for the epilogue to release the tile n_acc (<= 4)
              // before that, and the epilogue reads a tile's scales before releasing it -- so
              // every tile up to KST + 4 back has been read, and SK_RING > KST + 4.
              const int si = int(n_tiles % SK_RING);
              tc::mbar_expect_tx(&sk_full[si], 2 * 64 * 4);
              tc::bulk_load(sks + si * BM, a.sk + r0, 64 * 4, &sk_full[si]);
              tc::bulk_load(sks + si * BM + 64, a.sk + r1, 64 * 4, &sk_full[si]);
              sk_issued |= 1u << si;
              sk_par[si] = (n_tiles / SK_RING) & 1u;
            }
          } else {
            for (int cb = 0; cb < C::NCB; ++cb)
              tc::tma_load_3d(ks + ks_i * C::K_BYTES + cb * BM * C::SW, &tk, &k_full[ks_i], cb * C::SW / C::EB,
                              kt * BM, m.b);
          }
          k_issued |= 1u << ks_i;
          k_par[ks_i] = ks_ph;
          if (++ks_i == KST) { ks_i = 0; ks_ph ^= 1; }
          ++n_tiles;
        }
        ++qi;
      }
      if (*abort_flag) {  // drain this CTA's own copies before the CTA (and its smem) goes away
        for (int i = 0; i < KST; ++i)
          if (k_issued >> i & 1) tc::mbar_wait(&k_full[i], k_par[i], nullptr, 0);
        for (int i = 0; i < 2; ++i)
          if (q_issued >> i & 1) tc::mbar_wait(&q_full[i], q_par[i], nullptr, 0);
        if constexpr (PAGED)
          for (int i = 0; i < SK_RING; ++i)
            if (sk_issued >> i & 1) tc::mbar_wait(&sk_full[i], sk_par[i], nullptr, 0);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t kFmt = FP8 ? 0 : 1;
      const uint32_t idesc = tc::make_idesc(BM, a.N, kFmt, kFmt);
      // Descriptors of stage / buffer 0 built once; per MMA only constant offsets are added
      // (this one thread issues every MMA: building each descriptor from its address cost
      // more issue time than the small decode MMAs themselves)
      const uint64_t kd0 = tc::make_sdesc<C::SW>(smem_u32(ks), 16, 8 * C::SW);
      const uint64_t qd0 = tc::make_sdesc<C::SW>(smem_u32(qs), 16, 8 * C::SW);
      int ks_i = 0, ks_ph = 0, acc = 0, acc_ph = 0, qi = 0;
      for (int k = 0; !*abort_flag; ++k) {
        Item m;
        if (!get_item(k, m)) break;
        if (m.k0 >= m.k1) continue;
        const int qb = qi % C::Q_BUFS, qpar = (qi / C::Q_BUFS) & 1;
        if (!tc::mbar_wait(&q_full[qb], qpar, a.err, 103)) { *abort_flag = 1; break; }
        const uint64_t qdesc = tc::sdesc_add(qd0, uint32_t(qb * C::Q_BYTES));
        for (int kt = m.k0; kt < m.k1; ++kt) {
          if (!tc::mbar_wait(&acc_empty[acc], acc_ph ^ 1, a.err, 104)) { *abort_flag = 1; break; }
          if (!tc::mbar_wait(&k_full[ks_i], ks_ph, a.err, 105)) { *abort_flag = 1; break; }
          tc::fence_after_sync();
          const uint64_t kdesc = tc::sdesc_add(kd0, uint32_t(ks_i * C::K_BYTES));
          const uint32_t d = tmem + uint32_t(acc * acc_cols);
#pragma unroll
          for (int kk = 0; kk < C::KSTEPS; ++kk) {
            const int byte = kk * 32, cb = byte / C::SW, off = byte % C::SW;
            tc::mma_ss<FP8 ? 1 : 0>(d, tc::sdesc_add(kdesc, cb * BM * C::SW + off),
                                    tc::sdesc_add(qdesc, cb * C::NMAX * C::SW + off), idesc, kk > 0);
          }
          // one commit per tile: k_empty both frees the key stage and tells the epilogue the
          // accumulator is complete (it waits on that stage's barrier, below)
          tc::mma_commit(&k_empty[ks_i]);
          if (++ks_i == KST) { ks_i = 0; ks_ph ^= 1; }
          if (++acc == n_acc) { acc = 0; acc_ph ^= 1; }
        }
        tc::mma_commit(&q_empty[qb]);
        ++qi;
      }
    }
  } else if (warp >= EPI_WARP0) {
    // ---------------------------------------------------------------- epilogue
    // Each warp keeps its own copy of the weights c = w * sq of the tokens it sums.
    constexpr int NEPI_M = score_nthreads(MODE) - EPI_WARP0 * 32;
    const int et = threadIdx.x - EPI_WARP0 * 32;  // 0..NEPI_M-1
    const int ew = warp - EPI_WARP0;
    const int quarter = warp & 3;  // TMEM lanes 32 * (warp % 4) ...
    const int wg = ew >> 2;
    const int bwg = wg;                    // modes 0 / 1: the parity of the buffers this warpgroup drains
    const int th = MODE == 2 ? wg : 0;     // MODE 2: token th of the block, every tile
    const int row = quarter * 32 + lane;  // key row inside the tile
    constexpr int CWN = MODE == 2 ? 64 : C::NMAX;  // weights per warp
    float* cwp = cw + ew * CWN;
    uint32_t tcount = 0;
    auto write_tail = [&](int b, int tb) {  // keys no token of this block can see
      const int s0 = tb * a.Tq;
      const int n_kt = unit_tiles(b, tb);
      for (int t = 0; t < a.Tq; ++t) {
        const int s = s0 + t;
        if (s >= a.S) break;
        float* rowp = a.scores + (size_t(b) * a.S + s) * a.T;
        for (int j = n_kt * BM + et; j < a.T; j += NEPI_M) rowp[j] = -INFINITY;
      }
    };
    if (a.bal && a.write_tail)
      for (int u = blockIdx.x; u < units; u += gridDim.x) write_tail(u / n_tb, u % n_tb);
    for (int k = 0; !*abort_flag; ++k) {
      Item m;
      if (!get_item(k, m)) break;
      const int s0 = m.tb * a.Tq;
      if (a.write_tail && m.kc == 0) write_tail(m.b, m.tb);
      if (m.k0 >= m.k1) continue;
      const int tq_n = min(a.Tq, a.S - s0);  // real tokens in this block
      const int t0 = MODE == 2 ? min(th, tq_n) : 0, t1 = MODE == 2 ? min(th + 1, tq_n) : tq_n;
      for (int i = lane; i < (MODE == 2 ? 64 : a.N); i += 32) {
        const int ci = (MODE == 2 ? th * 64 : 0) + i;  // column (token, head) of the block
        const int s = s0 + ci / a.Hi, h = ci % a.Hi;
        float c = 0.0f;
        if (s < a.S) {
          const size_t o = (size_t(m.b) * a.S + s) * a.Hi + h;
          c = a.w[o] * (a.sq ? a.sq[o] : 1.0f);
        }
        cwp[i] = c;
      }
      // visible keys of token t, held by lane t (Tq <= 16)
      const int vis_l = lane < tq_n ? visible_of(a.q_pos, a.q_offset, m.b, a.S, s0 + lane, a.ratio, a.T) : 0;
      __syncwarp();
      bool ok = true;
      for (int kt = m.k0; kt < m.k1; ++kt, ++tcount) {
        // tile tcount: buffer tcount % n_acc, its (tcount / n_acc)-th use; buffers alternate
        // between the warpgroups (two buffers each when there are four)
        const int acc = int(tcount % uint32_t(n_acc));
        if (MODE != 2 && (acc & 1) != bwg) continue;
        // the key scale does not depend on the MMA: load it before waiting
        const int j = kt * BM + row;
        float skj;
        if (PAGED && a.sk_ring) {  // paged keys: from the ring the TMA warp filled (read before the release)
          const int si = int(tcount % SK_RING);
          if (!tc::mbar_wait(&sk_full[si], (tcount / SK_RING) & 1u, a.err, 107)) { ok = false; break; }
          skj = (j < a.T) ? sks[si * BM + row] * a.scale : 0.0f;
        } else {
          skj = (j < a.T) ? (a.sk ? __ldg(a.sk + key_row(PAGED ? a.k_pt : nullptr, a.k_ptw, a.k_npages, a.T, m.b, j))
                                  : 1.0f) * a.scale
                          : 0.0f;
        }
        // the tile's MMAs are complete when its key stage's k_empty phase completes (the one
        // commit per tile).  That phase cannot be overtaken before this wait: the stage's next
        // completion needs the MMA of tile tcount + K_STAGES, which waits for this
        // accumulator's release (n_acc <= K_STAGES, K_STAGES >= 2), and each buffer's tiles are
        // drained in order.
        if (!tc::mbar_wait(&k_empty[tcount % uint32_t(KST)], (tcount / uint32_t(KST)) & 1u, a.err,
                           106)) { ok = false; break; }
        tc::fence_after_sync();
        const uint32_t tbase = tc::taddr(tmem, quarter * 32, acc * acc_cols);
        bool released = false;
        if constexpr (MODE >= 1) {  // the DeepSeek-V4 indexer: 64 columns per token, packed FMAs
          // Per token, both 32-column TMEM loads go out behind one wait; the buffer is released
          // as soon as the last token's columns are in registers, so the MMA can refill it
          // while they are summed.
          auto release = [&]() {
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&acc_empty[acc]);
            released = true;
          };
          uint64_t sum4[4];  // 8 independent fp32 sums of the current token
          auto half = [&](const uint32_t (&r)[32], int u) {  // u = 2 t + (half of token t)
            const int t = u >> 1;
            if ((u & 1) == 0) sum4[0] = sum4[1] = sum4[2] = sum4[3] = 0ull;
            const float4* cq4 = reinterpret_cast<const float4*>(cwp + (u - 2 * t0) * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float4 c0 = cq4[2 * i], c1 = cq4[2 * i + 1];
              sum4[0] = ffma_f32x2(pack_f32x2(fmaxf(__uint_as_float(r[8 * i + 0]), 0.0f),
                                              fmaxf(__uint_as_float(r[8 * i + 1]), 0.0f)),
                                   pack_f32x2(c0.x, c0.y), sum4[0]);
              sum4[1] = ffma_f32x2(pack_f32x2(fmaxf(__uint_as_float(r[8 * i + 2]), 0.0f),
                                              fmaxf(__uint_as_float(r[8 * i + 3]), 0.0f)),
                                   pack_f32x2(c0.z, c0.w), sum4[1]);
              sum4[2] = ffma_f32x2(pack_f32x2(fmaxf(__uint_as_float(r[8 * i + 4]), 0.0f),
                                              fmaxf(__uint_as_float(r[8 * i + 5]), 0.0f)),
                                   pack_f32x2(c1.x, c1.y), sum4[2]);
              sum4[3] = ffma_f32x2(pack_f32x2(fmaxf(__uint_as_float(r[8 * i + 6]), 0.0f),
                                              fmaxf(__uint_as_float(r[8 * i + 7]), 0.0f)),
                                   pack_f32x2(c1.z, c1.w), sum4[3]);
            }
            if (u & 1) {
              const float2 p0 = unpack_f32x2(sum4[0]), p1 = unpack_f32x2(sum4[1]);
              const float2 p2 = unpack_f32x2(sum4[2]), p3 = unpack_f32x2(sum4[3]);
              const float sum = ((p0.x + p0.y) + (p1.x + p1.y)) + ((p2.x + p2.y) + (p3.x + p3.y));
              const int vis = __shfl_sync(0xffffffffu, vis_l, t);
              if (j < a.T) a.scores[(size_t(m.b) * a.S + s0 + t) * a.T + j] = (j < vis) ? sum * skj : -INFINITY;
            }
          };
          const int nu = 2 * t1;  // halves of this warp's tokens: [2 t0, 2 t1)
          if constexpr (MODE == 2) {
            // 16 columns at a time, double-buffered (96 registers a thread): the next load is
            // in flight while these are summed, so the buffer is released one load latency
            // after its last load instead of after every earlier column's math -- the MMA
            // of the tile two ahead waits on that release.  Same summation order as `half`.
            auto quarter = [&](const uint32_t (&r)[16], int qq) {  // qq = 4 t + (quarter of token t)
              const int t = qq >> 2;
              if ((qq & 3) == 0) sum4[0] = sum4[1] = sum4[2] = sum4[3] = 0ull;
              const float4* cq4 = reinterpret_cast<const float4*>(cwp + (qq - 4 * t0) * 16);
#pragma unroll
              for (int i = 0; i < 2; ++i) {
                const float4 c0 = cq4[2 * i], c1 = cq4[2 * i + 1];
                sum4[0] = ffma_f32x2(pack_f32x2(fmaxf(__uint_as_float(r[8 * i + 0]), 0.0f),
                                                fmaxf(__uint_as_float(r[8 * i + 1]), 0.0f)),
                                     pack_f32x2(c0.x, c0.y), sum4[0]);
                sum4[1] = ffma_f32x2(pack_f32x2(fmaxf(__uint_as_float(r[8 * i + 2]), 0.0f),
                                                fmaxf(__uint_as_float(r[8 * i + 3]), 0.0f)),
                                     pack_f32x2(c0.z, c0.w), sum4[1]);
                sum4[2] = ffma_f32x2(pack_f32x2(fmaxf(__uint_as_float(r[8 * i + 4]), 0.0f),
                                                fmaxf(__uint_as_float(r[8 * i + 5]), 0.0f)),
                                     pack_f32x2(c1.x, c1.y), sum4[2]);
                sum4[3] = ffma_f32x2(pack_f32x2(fmaxf(__uint_as_float(r[8 * i + 6]), 0.0f),
                                                fmaxf(__uint_as_float(r[8 * i + 7]), 0.0f)),
                                     pack_f32x2(c1.z, c1.w), sum4[3]);
              }
              if ((qq & 3) == 3) {
                const float2 p0 = unpack_f32x2(sum4[0]), p1 = unpack_f32x2(sum4[1]);
                const float2 p2 = unpack_f32x2(sum4[2]), p3 = unpack_f32x2(sum4[3]);
                const float sum = ((p0.x + p0.y) + (p1.x + p1.y)) + ((p2.x + p2.y) + (p3.x + p3.y));
                const int vis = __shfl_sync(0xffffffffu, vis_l, t);
                if (j < a.T) a.scores[(size_t(m.b) * a.S + s0 + t) * a.T + j] = (j < vis) ? sum * skj : -INFINITY;
              }
            };
            uint32_t ra[16], rb[16];
            const int q0 = 4 * t0, cnt = 4 * (t1 - t0);  // this warp's token quarters: 0 or 4
            if (cnt > 0) tc::tmem_ld16(tbase + q0 * 16, ra);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              if (k >= cnt) break;
              uint32_t (&cur)[16] = (k & 1) ? rb : ra;
              uint32_t (&nxt)[16] = (k & 1) ? ra : rb;
              tc::tmem_wait_ld();
              tc::reg_after_wait(cur);
              if (k + 1 < cnt) tc::tmem_ld16(tbase + (q0 + k + 1) * 16, nxt);
              else release();
              quarter(cur, q0 + k);
            }
          } else {
            for (int u = 2 * t0; u < nu; u += 2) {
              uint32_t ra[32], rb[32];
              tc::tmem_ld32(tbase + u * 32, ra);
              tc::tmem_ld32(tbase + (u + 1) * 32, rb);
              tc::tmem_wait_ld();
              tc::reg_after_wait(ra);
              tc::reg_after_wait(rb);
              if (u + 2 == nu) release();
              half(ra, u);
              half(rb, u + 1);
            }
          }
        } else {
          for (int t = 0; t < tq_n; ++t) {
            // four independent partial sums (one per 16-head chunk) keep the FMA chains short
            float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};
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
                  const float4* cq4 = reinterpret_cast<const float4*>(cwp + t * a.Hi + h0 + c * 16);
  #pragma unroll
                  for (int q4 = 0; q4 < 4; ++q4) {
                    const float4 cc = cq4[q4];
                    part[c] = fmaf(fmaxf(__uint_as_float(r[c][q4 * 4 + 0]), 0.0f), cc.x, part[c]);
                    part[c] = fmaf(fmaxf(__uint_as_float(r[c][q4 * 4 + 1]), 0.0f), cc.y, part[c]);
                    part[c] = fmaf(fmaxf(__uint_as_float(r[c][q4 * 4 + 2]), 0.0f), cc.z, part[c]);
                    part[c] = fmaf(fmaxf(__uint_as_float(r[c][q4 * 4 + 3]), 0.0f), cc.w, part[c]);
                  }
                }
              }
            }
            const float sum = (part[0] + part[1]) + (part[2] + part[3]);
            const int vis = __shfl_sync(0xffffffffu, vis_l, t);
            if (j < a.T) a.scores[(size_t(m.b) * a.S + s0 + t) * a.T + j] = (j < vis) ? sum * skj : -INFINITY;
          }
        }
        if (!released) {
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&acc_empty[acc]);
        }
      }
      if (!ok) { *abort_flag = 1; break; }
      __syncwarp();  // every lane is done with cwp before the next item rewrites it
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
  const float* qnorm;  // [B * S]: A_s = sum_h |w_h sq_h| ||q_h||_2 per query row
  const int32_t* q_pos;
  int32_t* out;
  int B, S, T, Hi, Di, topk, ratio;
  long long q_offset;
  float scale, eps;
  int fp8;
  const int32_t* k_pt;  // page table of 64-key pages, or null (dense keys)
  int k_ptw, k_npages;
  int fused_bound;  // decode: each row's block computes its own bound factors (no bound_kernel)
  int* err;
};

constexpr int CAND_MAX = 512;  // band keys re-scored exactly (the band holds ~0-2)

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

// sum of squares of the 16 bytes at p (16 e4m3 codes or 8 bf16 values)
__device__ __forceinline__ float sumsq16(const uint4 v, int fp8) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (fp8) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[i] >> (16 * hh)), __NV_E4M3);
        const float2 f = __half22float2(__half2(hr));
        ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
      }
    } else {
      const float lo = __uint_as_float(w[i] << 16), hi = __uint_as_float(w[i] & 0xFFFF0000u);
      ss = fmaf(lo, lo, fmaf(hi, hi, ss));
    }
  }
  return ss;
}

// Upper bound of B_t = |scale| * sk_t * ||k_t||_2 over the keys any query of batch b can
// see, as partial maxima per (batch, part).  Exact norms (one 16-byte vector per lane) when
// many queries share the keys; for one- or few-query rows (decode) with e4m3 keys, the
// bound ||k_t|| <= 448 * sqrt(Di) (448 = largest finite e4m3) so that only the per-key
// scales are read -- that widens the exactly re-scored band by at most sqrt(Di) times,
// which costs little with so few rows.
__device__ void key_bound(const TopkArgs& a, int b, int part) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  __shared__ float red[8];
  __shared__ int red_v[8];
  int tv = 0;
  if (a.q_pos) {
    for (int s = tid; s < a.S; s += blockDim.x) tv = max(tv, visible_of(a.q_pos, a.q_offset, b, a.S, s, a.ratio, a.T));
  } else {
    tv = visible_keys(a.q_offset, a.S - 1, a.ratio, a.T);  // visibility grows with s
  }
  for (int o = 16; o; o >>= 1) tv = max(tv, __shfl_xor_sync(0xffffffffu, tv, o));
  if (lane == 0) red_v[warp] = tv;
  __syncthreads();
  tv = 0;
  for (int i = 0; i < 8; ++i) tv = max(tv, red_v[i]);
  const int per = (tv + KB_PARTS - 1) / KB_PARTS;
  const int t_lo = part * per, t_hi = min(tv, t_lo + per);
  const float asc = fabsf(a.scale);
  const int eb = a.fp8 ? 1 : 2;
  const int rb = a.Di * eb;  // row bytes
  const int lpr = rb / 16;   // lanes per row
  float m = 0.0f;
  if (a.fp8 && a.S <= 16) {
    float mk = 0.0f;
    for (int t = t_lo + tid; t < t_hi; t += blockDim.x)
      mk = fmaxf(mk, fabsf(a.sk[key_row(a.k_pt, a.k_ptw, a.k_npages, a.T, b, t)]));
    m = asc * mk * (448.0f * sqrtf(float(a.Di))) * 1.0001f;
  } else if (rb % 16 == 0 && lpr <= 32 && (lpr & (lpr - 1)) == 0) {
    const int rows = blockDim.x / lpr;
    for (int t0 = t_lo; t0 < t_hi; t0 += rows) {  // uniform trip count: shuffles see full warps
      const int t = t0 + tid / lpr;
      float ss = 0.0f;
      if (t < t_hi)
        ss = sumsq16(*reinterpret_cast<const uint4*>(a.k + key_row(a.k_pt, a.k_ptw, a.k_npages, a.T, b, t) * rb +
                                                     (tid % lpr) * 16),
                     a.fp8);
      for (int o = lpr >> 1; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (t < t_hi) {
        const float sk = a.sk ? fabsf(a.sk[key_row(a.k_pt, a.k_ptw, a.k_npages, a.T, b, t)]) : 1.0f;
        m = fmaxf(m, asc * sk * sqrtf(ss));
      }
    }
  } else {
    for (int t = t_lo + warp; t < t_hi; t += blockDim.x >> 5) {
      const uint8_t* kr = a.k + key_row(a.k_pt, a.k_ptw, a.k_npages, a.T, b, t) * rb;
      float ss = 0.0f;
      for (int i = lane; i < a.Di; i += 32) {
        const float v = elem_f(kr, i, a.fp8);
        ss = fmaf(v, v, ss);
      }
      for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float sk = a.sk ? fabsf(a.sk[key_row(a.k_pt, a.k_ptw, a.k_npages, a.T, b, t)]) : 1.0f;
      m = fmaxf(m, asc * sk * sqrtf(ss));
    }
  }
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (tid == 0) {
    float r = 0.0f;
    for (int i = 0; i < 8; ++i) r = fmaxf(r, red[i]);
    const_cast<float*>(a.kbmax)[b * KB_PARTS + part] = r;
  }
}

// A_s = sum_h |c_h| ||q_h||_2 (c_h = w_h sq_h) of one query row, by one warp, for the rows
// whose selection can need the error bound (more visible keys than topk).  Rows of whole
// 16-byte vectors: lpr = rb / 16 lanes per head row, QB vectors per lane in flight.
__device__ void query_bound(const TopkArgs& a, int row) {
  const int lane = threadIdx.x & 31;
  const int b = row / a.S, s = row % a.S;
  if (visible_of(a.q_pos, a.q_offset, b, a.S, s, a.ratio, a.T) <= a.topk) return;
  const int rb = a.Di * (a.fp8 ? 1 : 2);
  const uint8_t* qg = a.q + size_t(row) * a.Hi * rb;
  const float* wr = a.w + size_t(row) * a.Hi;
  const float* sqr = a.sq ? a.sq + size_t(row) * a.Hi : nullptr;
  const int lpr = rb >> 4;
  float part = 0.0f;
  if ((rb & 15) == 0 && lpr <= 32 && (lpr & (lpr - 1)) == 0) {
    constexpr int QB = 4;
    const int nv = a.Hi * lpr, sh = __ffs(lpr) - 1;
    for (int v0 = 0; v0 < nv; v0 += 32 * QB) {  // warp-uniform trip count: full-warp shuffles
      uint4 qv[QB];
      float cabs[QB];
#pragma unroll
      for (int u = 0; u < QB; ++u) {
        const int v = v0 + 32 * u + lane;
        qv[u] = make_uint4(0u, 0u, 0u, 0u);
        cabs[u] = 0.0f;
        if (v < nv) {
          const int h = v >> sh;
          qv[u] = __ldg(reinterpret_cast<const uint4*>(qg + size_t(h) * rb + (v & (lpr - 1)) * 16));
          if ((v & (lpr - 1)) == 0) cabs[u] = fabsf(__ldg(wr + h) * (sqr ? __ldg(sqr + h) : 1.0f));
        }
      }
#pragma unroll
      for (int u = 0; u < QB; ++u) {
        float ss = sumsq16(qv[u], a.fp8);
        for (int o = lpr >> 1; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        part += cabs[u] * sqrtf(ss);  // cabs is 0 off the head leaders
      }
    }
  } else {
    for (int h = lane; h < a.Hi; h += 32) {
      const uint8_t* qh = qg + size_t(h) * rb;
      float ss = 0.0f;
      for (int i = 0; i < a.Di; ++i) {
        const float v = elem_f(qh, i, a.fp8);
        ss = fmaf(v, v, ss);
      }
      part += fabsf(wr[h] * (sqr ? sqr[h] : 1.0f)) * sqrtf(ss);
    }
  }
  for (int o = 16; o; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if (lane == 0) const_cast<float*>(a.qnorm)[row] = part;
}

// The two bound factors of one decode row, computed by its own top-k block (one query per
// sequence, so nothing is shared between rows): B = |scale| * max_t |sk_t| * 448 sqrt(Di)
// over the row's visible keys (the e4m3 form of key_bound) and A_s of query_bound, one
// 16-byte vector of q per thread.  Needs e4m3 rows of a power-of-two number (<= 32) of
// 16-byte vectors.  Returns both through `red` (2 x 32 floats of shared memory).
template <int NT>
__device__ void row_bound(const TopkArgs& a, int row, int b, int V, float* red, float& kb, float& qn) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float mk = 0.0f;
  if (a.k_pt) {
    // Paged keys, page by page: lane l first reads the id of the warp's l-th page (one
    // load per lane, all in flight together), then the warp's pages are swept with the ids
    // broadcast from the lanes, two coalesced 128-byte scale loads per page.  No load waits
    // on another's result except once on the ids (key_row per key would chain a page-table
    // read before every scale read).
    constexpr int NW = NT / 32;
    const int npg = (V + 63) >> 6;
    for (int p0 = warp; p0 < npg; p0 += NW * 32) {
      const int pl = p0 + NW * lane;
      int pg = 0;
      if (pl < npg) {
        pg = __ldg(a.k_pt + (long long)b * a.k_ptw + min(pl, a.k_ptw - 1));
        pg = pg < 0 ? 0 : (pg >= a.k_npages ? a.k_npages - 1 : pg);
      }
      const int cnt = min(32, (npg - p0 + NW - 1) / NW);  // this warp's pages in this sweep
      for (int i0 = 0; i0 < cnt; i0 += 8) {  // eight pages' loads in flight per batch
        float sv[16];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int pgi = __shfl_sync(0xffffffffu, pg, (i0 + u) & 31);
          const float* sp = a.sk + (long long)pgi * 64 + lane;
          const bool ok = i0 + u < cnt;
          sv[2 * u] = ok ? __ldg(sp) : 0.0f;
          sv[2 * u + 1] = ok ? __ldg(sp + 32) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int t = (p0 + NW * (i0 + u)) * 64 + lane;
          if (i0 + u < cnt && t < V) mk = fmaxf(mk, fabsf(sv[2 * u]));
          if (i0 + u < cnt && t + 32 < V) mk = fmaxf(mk, fabsf(sv[2 * u + 1]));
        }
      }
    }
  } else {
    for (int t = tid; t < V; t += NT) mk = fmaxf(mk, fabsf(a.sk[key_row(a.k_pt, a.k_ptw, a.k_npages, a.T, b, t)]));
  }
  const int lpr = a.Di >> 4, nv = a.Hi * lpr;
  const uint8_t* qg = a.q + size_t(row) * a.Hi * a.Di;
  float part = 0.0f;
  for (int v0 = 0; v0 < nv; v0 += NT) {  // block-uniform trip count: full-warp shuffles
    const int v = v0 + tid;
    float ss = 0.0f, cabs = 0.0f;
    if (v < nv) {
      const int h = v / lpr;
      ss = sumsq16(*reinterpret_cast<const uint4*>(qg + size_t(h) * a.Di + (v % lpr) * 16), 1);
      if (v % lpr == 0) cabs = fabsf(a.w[size_t(row) * a.Hi + h] * a.sq[size_t(row) * a.Hi + h]);
    }
    for (int o = lpr >> 1; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    part += cabs * sqrtf(ss);  // cabs is 0 off the head leaders
  }
  for (int o = 16; o; o >>= 1) {
    mk = fmaxf(mk, __shfl_xor_sync(0xffffffffu, mk, o));
    part += __shfl_xor_sync(0xffffffffu, part, o);
  }
  if (lane == 0) {
    red[warp] = mk;
    red[32 + warp] = part;
  }
  __syncthreads();
  mk = 0.0f;
  part = 0.0f;
  for (int i = 0; i < NT / 32; ++i) {
    mk = fmaxf(mk, red[i]);
    part += red[32 + i];
  }
  kb = fabsf(a.scale) * mk * (448.0f * sqrtf(float(a.Di))) * 1.0001f;
  qn = part;
  __syncthreads();
}

// The error-bound factors of the selection, one launch: blocks [0, B * KB_PARTS) bound
// the keys (per batch and part), the rest the query rows (8 per block, one per warp).
__global__ void __launch_bounds__(256) bound_kernel(TopkArgs a) {
  const int nkb = a.B * KB_PARTS;
  if (int(blockIdx.x) < nkb) {
    key_bound(a, blockIdx.x / KB_PARTS, blockIdx.x % KB_PARTS);
  } else {
    const int row = (int(blockIdx.x) - nkb) * 8 + int(threadIdx.x >> 5);
    if (row < a.B * a.S) query_bound(a, row);
  }
}

// An e4m3 code as an integer in units of 2^-9: value = M * 2^(e' - 10) with M = 8 + m
// (normal) or m (subnormal) and e' = max(e, 1), i.e. (M << (e' - 1)) * 2^-9, |.| < 2^18.  A
// product of two is an integer in units of 2^-18 below 2^36 and a 128-term sum stays below
// 2^43, so an int64 dot product is exact and equals the fp64 sum of the products.  NaN codes
// (0x7F / 0xFF) are reported through `nan` (the caller keeps the fp64 path for them).
__device__ __forceinline__ int e4m3_int(uint32_t c, bool& nan) {
  const int e = int(c >> 3) & 15, m = int(c) & 7;
  nan |= (c & 0x7Fu) == 0x7Fu;
  const int v = (e ? (8 | m) : m) << (e ? e - 1 : 0);
  return (c & 0x80u) ? -v : v;
}

// exact fp64 value of an e4m3 code pair (the low and high byte of a 16-bit word)
__device__ __forceinline__ void e4m3x2_to_f64(uint32_t w16, double& lo, double& hi) {
  const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w16 & 0xFFFFu), __NV_E4M3);
  const float2 f = __half22float2(__half2(hr));
  lo = double(f.x);
  hi = double(f.y);
}

constexpr int BLIST = 256;  // keys of the selected linear bin ranked directly

// bytes of the region shared by the bin bytes of V keys and the fp64 re-scoring buffers
// (exact scores: CAND_MAX doubles, head weights: Hi doubles, per-warp head products:
// rw x Hi doubles, per-warp key rows: rw x Di floats), rounded up to 16
// qint: bytes of the integer copy of an e4m3 query row (wide blocks, see e4m3_int)
__host__ __device__ constexpr int topk_rescore_bytes(int Hi, int Di, int rw, int qint) {
  return CAND_MAX * 8 + Hi * 8 + rw * Hi * 8 + rw * Di * 4 + qint;
}
__host__ __device__ constexpr int topk_region_bytes(int V, int Hi, int Di, int rw, int qint) {
  return ((V > topk_rescore_bytes(Hi, Di, rw, qint) ? V : topk_rescore_bytes(Hi, Di, rw, qint)) + 15) & ~15;
}

// exclusive prefix (over the block, in thread order) of `cnt`; also returns the total.
// Uses sh[0..NW) and sh[32..32+NW], sh[64]; two __syncthreads.
template <int NT>
__device__ __forceinline__ int block_exclusive_scan(int cnt, int* sh, int& total) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = cnt;
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) sh[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int v0 = lane < NW ? sh[lane] : 0;
    int x = v0;
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += v;
    }
    if (lane < NW) sh[32 + lane] = x - v0;
    if (lane == NW - 1) sh[64] = x;
  }
  __syncthreads();
  total = sh[64];
  return sh[32 + warp] + incl - cnt;
}

template <int TK_THREADS>
__global__ void __launch_bounds__(TK_THREADS, TK_THREADS == 128 ? 12 : 1) topk_kernel(TopkArgs a) {
  constexpr int NW = TK_THREADS / 32;
  constexpr int RW = NW < 8 ? NW : 8;  // warps that re-score band keys
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
  const int rb = a.Di * eb;  // bytes per q head row / k row
  float fkb = 0.0f, fqn = 0.0f;
  if (a.fused_bound) {
    __shared__ float fred[64];
    row_bound<TK_THREADS>(a, row, b, V, fred, fkb, fqn);
  }
  // smem carve-up: one bin byte per key; the fp64 re-scoring buffers are used only once
  // the bins are dead and share their region
  // wide blocks with e4m3 rows re-score the band in integers (e4m3_int): the query row's
  // integer copy [Di][Hi] follows the per-warp key rows
  const bool int_dot = TK_THREADS == 1024 && a.fp8;
  const int region = topk_region_bytes(V, a.Hi, a.Di, RW, int_dot ? a.Hi * a.Di * 4 : 0);
  uint8_t* bins = sm;                                                       // V (padded to 4)
  double* exact = reinterpret_cast<double*>(sm);                            // CAND_MAX
  double* cq = exact + CAND_MAX;                                            // Hi
  double* phall = cq + a.Hi;                                                // RW warps x Hi
  float* kdall = reinterpret_cast<float*>(phall + RW * a.Hi);               // RW warps x Di
  int* qint = reinterpret_cast<int*>(kdall + RW * a.Di);                    // [Di][Hi] (int_dot)
  uint32_t* sel = reinterpret_cast<uint32_t*>(sm + region);                 // ceil(V/32)
  const int nsel = (V + 31) >> 5;
  uint32_t* bl_key = sel + nsel;                                            // BLIST
  int* bl_idx = reinterpret_cast<int*>(bl_key + BLIST);                     // BLIST
  int* cand = bl_idx + BLIST;                                               // CAND_MAX
  __shared__ int hist[256];
  __shared__ uint32_t sh_kk, sh_theta;
  __shared__ int sh_bin, n_in, n_cand, n_bl, sh_scan[96];
  __shared__ uint32_t sh_kmin, sh_kmax, sh_bmin, sh_bmax;
  if (tid == 0) {
    sh_kmin = 0xFFFFFFFFu; sh_kmax = 0u; sh_bmin = 0xFFFFFFFFu; sh_bmax = 0u;
    n_in = 0; n_cand = 0; n_bl = 0;
  }
  for (int i = tid; i < 256; i += TK_THREADS) hist[i] = 0;
  __syncthreads();

  const float* srow = a.scores + size_t(row) * a.T;
  const uint8_t* qg = a.q + size_t(row) * a.Hi * rb;
  auto range_reduce = [&](uint32_t kmin, uint32_t kmax) {
    for (int o = 16; o; o >>= 1) {
      kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
      kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
    }
    if (lane == 0) { atomicMin(&sh_kmin, kmin); atomicMax(&sh_kmax, kmax); }
  };
  // The bins' range comes from one strided sample per thread.  Any range is correct (keys
  // outside it are clamped into the end bins, and the bin map stays monotone); a sample of
  // TK_THREADS keys leaves ~V / TK_THREADS keys beyond either end.
  {
    const int j = int((long long)tid * V / TK_THREADS);
    const uint32_t kx = tid < V ? f2key(srow[j]) : 0u;
    range_reduce(tid < V ? kx : 0xFFFFFFFFu, tid < V ? kx : 0u);
  }
  __syncthreads();
  float vmin = key2f(sh_kmin), vmax = key2f(sh_kmax);
  float inv = 256.0f / (vmax - vmin);
  bool binned = vmax > vmin && inv < 1e30f;
  if (!binned) {
    // a flat sample: take the exact range (all keys equal -> no bins)
    __syncthreads();
    if (tid == 0) { sh_kmin = 0xFFFFFFFFu; sh_kmax = 0u; }
    __syncthreads();
    uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
    for (int j = tid; j < V; j += TK_THREADS) {
      const uint32_t kx = f2key(srow[j]);
      kmin = min(kmin, kx);
      kmax = max(kmax, kx);
    }
    range_reduce(kmin, kmax);
    __syncthreads();
    vmin = key2f(sh_kmin);
    vmax = key2f(sh_kmax);
    inv = 256.0f / (vmax - vmin);
    binned = vmax > vmin && inv < 1e30f;
  }

  // The topk-th largest key, exactly.  Pass 1 histograms the scores into 256 linear bins
  // over [vmin, vmax] -- a monotone map, so the k-th largest lies in one bin -- and keeps
  // each key's bin.  Pass 2 writes the selection words of the bins above that bin and
  // gathers the bin's keys; up to BLIST of them are ranked directly, more fall back to a
  // radix select (MSB first, 8-bit digits, below the bits the bin's keys share).
  auto bin_f = [&](float x) {  // monotone non-decreasing in x; always in [0, 255]
    const float f = (x - vmin) * inv;
    return f >= 255.0f ? 255 : (f > 0.0f ? int(f) : 0);
  };
  // warp 0: the digit (bin) holding the kk-th largest of `hist`, counting from the top
  auto pick = [&](uint32_t kk_in) {
    int cnt[8], tot = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) { cnt[i] = hist[255 - 8 * lane - i]; tot += cnt[i]; }
    int incl = tot;
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const int excl = incl - tot;
    if (excl < int(kk_in) && int(kk_in) <= incl) {
      int run = excl;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (run < int(kk_in) && int(kk_in) <= run + cnt[i]) {
          sh_bin = 255 - 8 * lane - i;
          sh_kk = kk_in - run;
        }
        run += cnt[i];
      }
    }
  };
  uint32_t kk = a.topk;
  uint32_t prefix = sh_kmin;  // all keys equal: that key
  int bsel = -1, nb = 0;
  if (binned) {
    // pass 1: global loads batched UNR vectors deep
    if ((a.T & 3) == 0) {  // rows are 16-byte aligned; V rounded up to 4 stays in the row
      constexpr int UNR = 4;
      for (int j0 = 4 * tid; j0 < V; j0 += 4 * TK_THREADS * UNR) {
        float4 f[UNR];
#pragma unroll
        for (int u = 0; u < UNR; ++u) {
          const int j = j0 + 4 * TK_THREADS * u;
          if (j < V) f[u] = __ldg(reinterpret_cast<const float4*>(srow + j));
        }
#pragma unroll
        for (int u = 0; u < UNR; ++u) {
          const int j = j0 + 4 * TK_THREADS * u;
          if (j < V) {
            const float fv[4] = {f[u].x, f[u].y, f[u].z, f[u].w};
            uint32_t packed = 0u;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              if (j + e < V) {
                const int bn = bin_f(fv[e]);
                atomicAdd(&hist[bn], 1);
                packed |= uint32_t(bn) << (8 * e);
              }
            }
            *reinterpret_cast<uint32_t*>(bins + j) = packed;
          }
        }
      }
    } else {
      for (int j = tid; j < V; j += TK_THREADS) {
        const int bn = bin_f(srow[j]);
        atomicAdd(&hist[bn], 1);
        bins[j] = uint8_t(bn);
      }
    }
    __syncthreads();
    if (warp == 0) pick(kk);
    __syncthreads();
    bsel = sh_bin;
    kk = sh_kk;
    if (tid == 0) n_in = a.topk - int(kk);  // every key of the bins above bsel
    // pass 2: selection words of the bins above bsel (a lane's 4 keys are a nibble of a
    // word shared by 8 lanes); bin bsel's indices (its keys are re-read from the row after)
    for (int j0 = 0; j0 < V; j0 += 4 * TK_THREADS) {  // block-uniform trip count
      const int j = j0 + 4 * tid;
      uint32_t nib = 0u;
      if (j < V) {
        const uint32_t b4 = *reinterpret_cast<const uint32_t*>(bins + j);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int bn = int((b4 >> (8 * e)) & 0xFFu);
          if (j + e < V) {
            if (bn > bsel) {
              nib |= 1u << e;
            } else if (bn == bsel) {
              const int at = atomicAdd(&n_bl, 1);
              if (at < BLIST) bl_idx[at] = j + e;
            }
          }
        }
      }
      uint32_t word = nib << (4 * (lane & 7));
      word |= __shfl_xor_sync(0xffffffffu, word, 1);
      word |= __shfl_xor_sync(0xffffffffu, word, 2);
      word |= __shfl_xor_sync(0xffffffffu, word, 4);
      const int wi = j >> 5;
      if ((lane & 7) == 0 && wi < nsel) sel[wi] = word;
    }
    __syncthreads();
    nb = n_bl;
    if (nb <= BLIST) {
      for (int i = tid; i < nb; i += TK_THREADS) bl_key[i] = f2key(srow[bl_idx[i]]);  // one round trip
      __syncthreads();
      // rank directly: the kk-th largest has (#greater < kk <= #greater + #equal)
      for (int i = tid; i < nb; i += TK_THREADS) {
        const uint32_t kx = bl_key[i];
        int gt = 0, eq = 0;
        for (int o = 0; o < nb; ++o) {
          const uint32_t y = bl_key[o];
          gt += y > kx;
          eq += y == kx;
        }
        if (gt < int(kk) && int(kk) <= gt + eq) sh_theta = kx;  // equal keys write equal values
      }
      __syncthreads();
      prefix = sh_theta;
    } else {
      {
        uint32_t bmn = 0xFFFFFFFFu, bmx = 0u;
        for (int j = tid; j < V; j += TK_THREADS) {
          if (bins[j] == bsel) {
            const uint32_t kx = f2key(srow[j]);
            bmn = min(bmn, kx);
            bmx = max(bmx, kx);
          }
        }
        for (int o = 16; o; o >>= 1) {
          bmn = min(bmn, __shfl_xor_sync(0xffffffffu, bmn, o));
          bmx = max(bmx, __shfl_xor_sync(0xffffffffu, bmx, o));
        }
        if (lane == 0) { atomicMin(&sh_bmin, bmn); atomicMax(&sh_bmax, bmx); }
        __syncthreads();
      }
      prefix = sh_bmin;
      const uint32_t kdiff = sh_bmin ^ sh_bmax;
      int hi_bit = kdiff ? 31 - __clz(kdiff) : -1;
      // bits above hi_bit are common to the bin's keys (all of them when they are equal)
      uint32_t mask = hi_bit < 0 ? 0xFFFFFFFFu : (hi_bit >= 31 ? 0u : ~((2u << hi_bit) - 1u));
      prefix &= mask;
      while (hi_bit >= 0) {
        const int width = min(8, hi_bit + 1);
        const int shift = hi_bit - width + 1;
        const uint32_t dmask = (1u << width) - 1u;
        for (int i = tid; i < 256; i += TK_THREADS) hist[i] = 0;
        __syncthreads();
        for (int j = tid; j < V; j += TK_THREADS) {
          if (bins[j] == bsel) {
            const uint32_t kx = f2key(srow[j]);
            if ((kx & mask) == prefix) atomicAdd(&hist[(kx >> shift) & dmask], 1);
          }
        }
        __syncthreads();
        if (warp == 0) pick(kk);
        __syncthreads();
        prefix |= uint32_t(sh_bin) << shift;
        kk = sh_kk;
        mask |= dmask << shift;
        hi_bit -= width;
      }
    }
  }
  const float theta = key2f(prefix);
  float kbm = fkb, qn = fqn;
  if (!a.fused_bound) {
    for (int i = 0; i < KB_PARTS; ++i) kbm = fmaxf(kbm, a.kbmax[b * KB_PARTS + i]);
    qn = a.qnorm[row];
  }
  const float delta = a.eps * qn * kbm * 1.0001f;
  const float hi_thr = __fadd_ru(theta, 2.0f * delta), lo_thr = __fsub_rd(theta, 2.0f * delta);
  // pass 3: certain keys into `sel`, the band between the thresholds into `cand`.  When the
  // band lies in bin bsel and the list holds all of that bin, the keys above it are exactly
  // the bins above bsel (written by pass 2: bin_f is monotone) plus the list's keys above
  // hi_thr, and the band is in the list -- only the list is scanned.  Otherwise the row.
  const bool in_bin = binned && nb <= BLIST && bin_f(lo_thr) == bsel && bin_f(hi_thr) == bsel;
  if (in_bin) {
    for (int i = tid; i < nb; i += TK_THREADS) {
      const float v = key2f(bl_key[i]);
      const int j = bl_idx[i];
      if (v > hi_thr) {
        atomicOr(&sel[j >> 5], 1u << (j & 31));
        atomicAdd(&n_in, 1);
      } else if (v >= lo_thr) {
        const int c = atomicAdd(&n_cand, 1);
        if (c < CAND_MAX) cand[c] = j;
      }
    }
  } else {
    if (tid == 0) n_in = 0;
    __syncthreads();
    for (int j0 = 0; j0 < V; j0 += TK_THREADS) {  // one word per warp iteration, no atomics on sel
      const int j = j0 + tid;
      const float v = j < V ? srow[j] : -INFINITY;
      const uint32_t in_w = __ballot_sync(0xffffffffu, j < V && v > hi_thr);
      const bool is_c = j < V && !(v > hi_thr) && v >= lo_thr;
      const uint32_t c_w = __ballot_sync(0xffffffffu, is_c);
      if (j - lane < V && lane == 0) {
        sel[j >> 5] = in_w;
        if (in_w) atomicAdd(&n_in, __popc(in_w));
      }
      if (c_w) {
        int base = 0;
        if (lane == 0) base = atomicAdd(&n_cand, __popc(c_w));
        base = __shfl_sync(0xffffffffu, base, 0);
        const int c = base + __popc(c_w & ((1u << lane) - 1u));
        if (is_c && c < CAND_MAX) cand[c] = j;
      }
    }
  }
  __syncthreads();
  const int nin = n_in, nc = n_cand;
  const int need = a.topk - nin;
  if (need < 0 || need > nc || (nc > CAND_MAX && delta != 0.0f)) {
    if (tid == 0) atomicExch(a.err, MZB_ERR_BOUND);
    for (int i = tid; i < a.topk; i += TK_THREADS) out[i] = -1;
    return;
  }
  if (need == nc && nc <= CAND_MAX) {
    // the whole band is selected: its exact order does not matter
    for (int c = tid; c < nc; c += TK_THREADS) atomicOr(&sel[cand[c] >> 5], 1u << (cand[c] & 31));
    __syncthreads();
  } else if (nc > CAND_MAX) {
    // delta == 0: every score is exactly 0 (all weights or all keys zero), so the band is
    // one exact tie -- take its lowest indices.  Warp 0 walks the words in order.
    if (warp == 0) {
      int running = 0;
      for (int w0 = 0; w0 < nsel; w0 += 32) {
        const int w = w0 + lane;
        uint32_t bits = 0;
        if (w < nsel)
          for (int bit = 0; bit < 32; ++bit) {
            const int j = w * 32 + bit;
            if (j < V) {
              const float v = srow[j];
              if (!(v > hi_thr) && v >= lo_thr) bits |= 1u << bit;
            }
          }
        const int c = __popc(bits);
        int incl = c;
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += v;
        }
        const int take = max(0, min(c, need - (running + incl - c)));
        uint32_t kept = 0;
        for (int t = 0; t < take; ++t) {
          const uint32_t low = bits & (~bits + 1u);
          kept |= low;
          bits ^= low;
        }
        if (w < nsel) sel[w] |= kept;
        running += __shfl_sync(0xffffffffu, incl, 31);
      }
    }
    __syncthreads();
  } else {
    // exact fp64 re-scoring of the band, RW warps, one candidate per warp; lane l owns
    // heads l + 32 m; q is read from global memory (L1-resident after the first use).  The
    // head products go to the warp's shared-memory row and lane 0 sums them in head order
    // (independent loads feeding one chain of adds).
    for (int h = tid; h < a.Hi; h += TK_THREADS) {
      const size_t o = size_t(row) * a.Hi + h;
      cq[h] = double(a.w[o]) * double(a.sq ? a.sq[o] : 1.0f);
    }
    // wide e4m3 rows: the query row as integers, transposed so a warp's lanes (heads) read
    // consecutive words; fp64 conversions per product were the re-scoring's throughput limit
    bool q_nan = false;
    if (int_dot)  // one 16-code vector per thread; consecutive threads = consecutive heads
      for (int v = tid; v < a.Hi * (a.Di >> 4); v += TK_THREADS) {
        const int h = v % a.Hi, i0 = (v / a.Hi) << 4;
        const uint4 w4 = *reinterpret_cast<const uint4*>(qg + size_t(h) * a.Di + i0);
        const uint32_t w[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
        for (int k = 0; k < 16; ++k) qint[(i0 + k) * a.Hi + h] = e4m3_int((w[k >> 2] >> (8 * (k & 3))) & 0xFFu, q_nan);
      }
    const bool row_int = int_dot && !__syncthreads_or(q_nan);
    float* kd = kdall + warp * a.Di;
    double* ph = phall + warp * a.Hi;
    for (int c = warp; c < nc && warp < RW; c += RW) {
      const int j = cand[c];
      const long long krow = key_row(a.k_pt, a.k_ptw, a.k_npages, a.T, b, j);
      const uint8_t* kr = a.k + krow * rb;
      const float skf = (lane == 0 && a.sk) ? a.sk[krow] : 1.0f;  // with the key row's loads
      __syncwarp();
      bool k_nan = false;
      if (row_int) {
        int* ki = reinterpret_cast<int*>(kd);
        for (int i = lane; i < a.Di; i += 32) ki[i] = e4m3_int(kr[i], k_nan);
      } else {
        for (int i = lane; i < a.Di; i += 32) kd[i] = elem_f(kr, i, a.fp8);  // exact in fp32
      }
      const bool use_int = row_int && !__any_sync(0xffffffffu, k_nan);
      if (row_int && !use_int)  // a NaN code in the key row: its fp64 path
        for (int i = lane; i < a.Di; i += 32) kd[i] = elem_f(kr, i, a.fp8);
      __syncwarp();
      if (use_int) {  // two heads per lane per pass: each key word read once for both
        const int* ki = reinterpret_cast<const int*>(kd);
        for (int m = 0; 32 * m < a.Hi; m += 2) {
          const int h0 = 32 * m + lane, h1 = h0 + 32;
          const int c0 = min(h0, a.Hi - 1), c1 = min(h1, a.Hi - 1);  // clamped reads, results dropped
          long long s0 = 0, s1 = 0;
#pragma unroll 4
          for (int i = 0; i < a.Di; ++i) {
            const long long kv = ki[i];
            s0 += qint[i * a.Hi + c0] * kv;
            s1 += qint[i * a.Hi + c1] * kv;
          }
          if (h0 < a.Hi) ph[h0] = __dmul_rn(cq[h0], s0 > 0 ? double(s0) * 3.814697265625e-06 : 0.0);  // 2^-18
          if (h1 < a.Hi) ph[h1] = __dmul_rn(cq[h1], s1 > 0 ? double(s1) * 3.814697265625e-06 : 0.0);
        }
      }
      for (int m = 0; 32 * m < a.Hi && !use_int; ++m) {
        const int h = 32 * m + lane;
        double pv = 0.0;
        if (h < a.Hi) {
          const uint8_t* qh = qg + size_t(h) * rb;
          double dot = 0.0;
          if (a.fp8) {
            // e4m3 products are multiples of 2^-18 below 2^18 and the sums stay below 2^53
            // units: exact in any order, so four chains
            double d0 = 0.0, d1 = 0.0, d2 = 0.0, d3 = 0.0;
            auto word = [&](uint32_t w, int i) {
              double q0, q1, q2, q3;
              e4m3x2_to_f64(w, q0, q1);
              e4m3x2_to_f64(w >> 16, q2, q3);
              d0 = fma(q0, double(kd[i]), d0);
              d1 = fma(q1, double(kd[i + 1]), d1);
              d2 = fma(q2, double(kd[i + 2]), d2);
              d3 = fma(q3, double(kd[i + 3]), d3);
            };
            if ((rb & 15) == 0) {
              for (int i = 0; i < a.Di; i += 16) {
                const uint4 w4 = __ldg(reinterpret_cast<const uint4*>(qh + i));
                word(w4.x, i);
                word(w4.y, i + 4);
                word(w4.z, i + 8);
                word(w4.w, i + 12);
              }
            } else {
              for (int i = 0; i < a.Di; i += 4) word(__ldg(reinterpret_cast<const uint32_t*>(qh + i)), i);
            }
            dot = (d0 + d1) + (d2 + d3);
          } else {
            for (int i = 0; i < a.Di; ++i) dot = fma(double(elem_f(qh, i, 0)), double(kd[i]), dot);  // sequential
          }
          pv = __dmul_rn(cq[h], dot > 0.0 ? dot : 0.0);
          ph[h] = pv;
        }
      }
      __syncwarp();
      if (lane == 0) {
        double acc = 0.0;
        for (int h = 0; h < a.Hi; ++h) acc = __dadd_rn(acc, ph[h]);  // heads in order
        exact[c] = __dmul_rn(__dmul_rn(acc, double(skf)), double(a.scale));
      }
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
  }
  // ascending compaction of the selected bits (per-thread word ranges in thread order)
  const int per = (nsel + TK_THREADS - 1) / TK_THREADS;
  const int w0 = tid * per, w1 = min(nsel, w0 + per);
  int cnt = 0;
  for (int i = w0; i < w1; ++i) cnt += __popc(sel[i]);
  int total = 0;
  int pos = block_exclusive_scan<TK_THREADS>(cnt, sh_scan, total);
  for (int i = w0; i < w1; ++i) {
    uint32_t bits = sel[i];
    while (bits) {
      const int bit = __ffs(bits) - 1;
      bits &= bits - 1;
      if (pos < a.topk) out[pos] = i * 32 + bit;
      ++pos;
    }
  }
  for (int i = total + tid; i < a.topk; i += TK_THREADS) out[i] = -1;
}

static size_t topk_smem(int T, int Hi, int Di, int eb, int threads) {
  const int rw = std::min(threads / 32, 8);
  const int qint = (threads == 1024 && eb == 1) ? Hi * Di * 4 : 0;
  return size_t(topk_region_bytes(T, Hi, Di, rw, qint)) + size_t((T + 31) / 32) * 4 + BLIST * 8 + CAND_MAX * 4;
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
  if (a.k_pt) {  // the page pool's rows, one 64-key page per load
    const uint64_t dims[2] = {uint64_t(DI), uint64_t(a.k_npages) * 64};
    const uint64_t str[1] = {uint64_t(C::R)};
    const uint32_t box[2] = {uint32_t(C::SW / C::EB), 64};
    int e = encode_tmap(&tk, dt, 2, k, dims, str, box, swz);
    if (e) return e;
  } else {
    const uint64_t dims[3] = {uint64_t(DI), uint64_t(a.T), uint64_t(a.B)};
    const uint64_t str[2] = {uint64_t(C::R), uint64_t(a.T) * C::R};
    const uint32_t box[3] = {uint32_t(C::SW / C::EB), uint32_t(BM), 1};
    int e = encode_tmap(&tk, dt, 3, k, dims, str, box, swz);
    if (e) return e;
  }
  const int mode = a.Hi != 64 ? 0 : (a.Tq == 4 ? 2 : 1);
  const bool paged = a.k_pt != nullptr;
  auto kern = paged ? (mode == 2 ? score_kernel<FP8, DI, 2, true>
                                 : (mode == 1 ? score_kernel<FP8, DI, 1, true> : score_kernel<FP8, DI, 0, true>))
                    : (mode == 2 ? score_kernel<FP8, DI, 2, false>
                                 : (mode == 1 ? score_kernel<FP8, DI, 1, false> : score_kernel<FP8, DI, 0, false>));
  const int smem = paged ? C::SMEM_PAGED : C::SMEM;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return launch_status("indexer_scores(smem attr)");
  // Few (batch, query block) pairs -- decode, short prefill -- would leave SMs idle while
  // each walks its whole key range: split the keys into chunks so there are about 8 items
  // per SM.  A chunk reloads its block's queries (one Q tile per chunk).
  ScoreArgs b = a;
  const int n_tb = (a.S + a.Tq - 1) / a.Tq;
  const long long base = (long long)a.B * n_tb;
  const int sms = num_sms();
  const int max_tiles = (a.T + BM - 1) / BM;
  int n_kc = 1;
  if (base < 2LL * sms && max_tiles > 1) n_kc = int(std::min<long long>(max_tiles, (8LL * sms + base - 1) / base));
  b.kc = (max_tiles + n_kc - 1) / n_kc;
  if (b.kc < 1) b.kc = 1;
  b.n_kc = (max_tiles + b.kc - 1) / b.kc;
  if (b.n_kc < 1) b.n_kc = 1;
  const long long items = base * b.n_kc;
  MZB_REQUIRE(items < (1LL << 31), MZB_ERR_SHAPE, "indexer: too many work items");
  // few units: every CTA takes an equal share of all key tiles instead of whole chunks
  b.bal = (n_kc > 1 && base <= BAL_MAX) ? 1 : 0;
  const int grid = b.bal ? sms : (items < sms ? int(items) : sms);
  kern<<<grid, score_nthreads(mode), smem, st>>>(tq, tk, b);
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

static int indexer_page_checks(const int32_t* k_page_table, int k_ptw, int64_t k_pages, int64_t T) {
  if (!k_page_table) return MZB_OK;
  MZB_REQUIRE(k_ptw >= 1 && k_pages >= 1 && k_pages * 64 < (int64_t(1) << 31), MZB_ERR_SHAPE,
              "indexer: paged keys need k_ptw >= 1 and 1 <= k_pages < 2^25 (got %d, %lld)", k_ptw,
              (long long)k_pages);
  MZB_REQUIRE(T <= int64_t(k_ptw) * 64, MZB_ERR_SHAPE, "indexer: T=%lld exceeds the page table's %d pages of 64",
              (long long)T, k_ptw);
  return MZB_OK;
}

extern "C" int mzb_indexer_scores(const void* q, const void* k, const float* w, const float* sq, const float* sk,
                                  const int32_t* q_pos, float* scores, int64_t B, int64_t S, int64_t T, int Hi,
                                  int Di, int dtype, int ratio, int64_t q_offset, float scale, int write_tail,
                                  const int32_t* k_page_table, int k_ptw, int64_t k_pages, int* err,
                                  void* stream) {
  int e = indexer_common_checks(q, k, B, S, T, Hi, Di, dtype, ratio);
  if (e) return e;
  if ((e = indexer_page_checks(k_page_table, k_ptw, k_pages, T))) return e;
  MZB_REQUIRE(dtype == MZB_BF16 || (sq && sk), MZB_ERR_SHAPE, "indexer: fp8 inputs need sq and sk scales");
  if (T == 0) return MZB_OK;
  idx::ScoreArgs a{};
  a.w = w; a.sq = sq; a.sk = sk; a.q_pos = q_pos; a.scores = scores;
  a.B = int(B); a.S = int(S); a.T = int(T); a.Hi = Hi;
  const int nmax = (Di * (dtype == MZB_E4M3 ? 1 : 2) <= 256) ? 256 : 128;
  a.Tq = nmax / Hi;
  MZB_REQUIRE(a.Tq >= 1, MZB_ERR_SHAPE, "indexer: Hi=%d too large for Di=%d", Hi, Di);
  if (a.Tq > S) a.Tq = int(S);  // one-token decode: N = Hi columns, not a padded block
  a.N = a.Tq * Hi;
  a.ratio = ratio; a.q_offset = q_offset; a.scale = scale; a.write_tail = write_tail; a.err = err;
  a.k_pt = k_page_table; a.k_ptw = k_ptw; a.k_npages = int(k_pages);
  a.sk_ring = (k_page_table && sk && reinterpret_cast<uintptr_t>(sk) % 16 == 0) ? 1 : 0;
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
                                float eps, const int32_t* k_page_table, int k_ptw, int64_t k_pages, int* err,
                                void* stream) {
  int e = indexer_common_checks(q, k, B, S, T, Hi, Di, dtype, ratio);
  if (e) return e;
  if ((e = indexer_page_checks(k_page_table, k_ptw, k_pages, T))) return e;
  MZB_REQUIRE(topk >= 1, MZB_ERR_SHAPE, "indexer topk: topk must be >= 1, got %d", topk);
  MZB_REQUIRE(err != nullptr, MZB_ERR_SHAPE, "indexer topk: needs an error word");
  MZB_REQUIRE(dtype == MZB_BF16 || (sq && sk), MZB_ERR_SHAPE, "indexer: fp8 inputs need sq and sk scales");
  const int eb = dtype == MZB_E4M3 ? 1 : 2;
  MZB_REQUIRE((Di * eb) % 4 == 0, MZB_ERR_UNSUPPORTED, "indexer topk: index rows must be a multiple of 4 bytes");
  // few rows (decode: one query per sequence) -> wide blocks, else 128 threads per row
  const bool wide = B * S < 2LL * num_sms();
  const size_t smem = idx::topk_smem(int(T), Hi, Di, eb, wide ? 1024 : 128);
  MZB_REQUIRE(smem <= 200 * 1024, MZB_ERR_UNSUPPORTED, "indexer topk: T=%lld needs %zu B of shared memory",
              (long long)T, smem);
  idx::TopkArgs a{};
  a.scores = scores; a.q = static_cast<const uint8_t*>(q); a.k = static_cast<const uint8_t*>(k);
  a.w = w; a.sq = sq; a.sk = sk; a.q_pos = q_pos; a.kbmax = kbmax_ws; a.qnorm = kbmax_ws + B * idx::KB_PARTS;
  a.out = out;
  a.B = int(B); a.S = int(S); a.T = int(T); a.Hi = Hi; a.Di = Di; a.topk = topk; a.ratio = ratio;
  a.q_offset = q_offset; a.scale = scale; a.eps = eps; a.fp8 = dtype == MZB_E4M3; a.err = err;
  a.k_pt = k_page_table; a.k_ptw = k_ptw; a.k_npages = int(k_pages);
  // decode rows (few queries, e4m3 keys, the scale-only key bound): each top-k block computes
  // its own row's bound factors, so no separate bound launch
  const int lpr = Di / 16;
  a.fused_bound = wide && dtype == MZB_E4M3 && S <= 16 && Di % 16 == 0 && lpr <= 32 && (lpr & (lpr - 1)) == 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (B == 0 || S == 0) return MZB_OK;
  if (T > 0 && !a.fused_bound) {
    const long long blocks = B * idx::KB_PARTS + (B * S + 7) / 8;
    idx::bound_kernel<<<unsigned(blocks), 256, 0, st>>>(a);
    if (int r = launch_status("indexer_bound")) return r;
  }
  auto kern = wide ? idx::topk_kernel<1024> : idx::topk_kernel<128>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
    return launch_status("indexer_topk(smem attr)");
  kern<<<unsigned(B * S), wide ? 1024 : 128, smem, st>>>(a);
  return launch_status("indexer_topk");
}
