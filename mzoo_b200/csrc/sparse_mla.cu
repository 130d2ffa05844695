// Sparse latent-MQA attention over FP8 KV rows (DeepSeek-V4.1 576/512 layout): prefill
// forward and paged decode, one kernel.
//
// Reference semantics: src/mzoo/layers/attn/csa2_attn/fwd.py:70-219 (one online softmax over
// a causal window of raw latent tokens and per-token gathered compressed entries; an index
// outside [0, G) contributes nothing; duplicates count twice; lse in natural log) and
// golden_ref.py:149-168 (`golden(level="sparse")`), widened to the 576-dim latent with
// V = its first 512 channels and FP8 no-rope storage (BASELINE configs 3 and 4; the
// reference itself stops at D <= 256, csa2_attn/fwd.py:56-61).
//
// KV row (672 B): [0,512) e4m3 codes, [512,544) 8 fp32 scales (one per 64 channels),
// [544,672) 64 bf16 rope channels.
//
// Work item = one query token (all 128 heads).  A cluster of two CTAs owns an item:
// tcgen05.mma.cta_group::2 with M = 128 heads (64 per CTA), so each SM keeps its heads'
// fp32 O (64 x 512) in TMEM as 128 lanes x 256 columns.  Keys come in tiles of 128, 64 per
// CTA (the QK^T B operand's N half): S (64 heads x 128 keys) is 128 lanes x 64 columns,
// lanes 0-63 holding the leader's 64 keys and lanes 64-127 the peer's, double-buffered.
// A 2-CTA MMA instruction costs about the same at N = 64 and N = 128 (~45 cycles), and
// each QK^T tile re-reads this CTA's 73.7 KB Q block from shared memory, so 128-key tiles
// halve both the QK^T instruction count and the Q reads per key against 64-key tiles.
//
// Warp roles per CTA (512 threads):
//   0      TMA of this CTA's Q half (64 heads x 576, 9 swizzled 64-column blocks)
//   1      TMEM allocation; in the leader CTA, the thread issuing the QK^T MMAs
//   2      paged rows (decode): L2 prefetch of this CTA's 64 rows of the tile two ahead of
//          the producers (a hint only: nothing waits on it)
//   3      in the leader CTA, the thread issuing the PV MMAs
//   4-7    softmax / O correction / epilogue (thread = TMEM lane = (head, key half))
//   8-15   producers: gather + dequantise this CTA's 64 keys x 576 channels into the K
//          tile, and fill this CTA's two V halves (below)
// Shared memory (227 KB): Q 72 KB, one K tile 72 KB, V 2 x 32 KB, P 2 x 8 KB.
// The PV B operand of CTA r is all 128 keys of the tile x CTA r's 256 output channels (its
// N half of each 256-channel PV chunk), in two key halves.  Half r (its own keys) is a copy
// of four 8 KB blocks of its K tile (identical 128-byte swizzle); half 1 - r (the peer's
// keys) is gathered from the FP8 rows in L2 and dequantised again.  Moving those blocks
// between the pair's shared memories instead (cp.async.bulk shared::cta -> shared::cluster)
// ran at ~29 bytes per cycle per SM through the cluster crossbar, local copies included,
// and held each K tile until its copies had landed: that cost a quarter of the run time.
// Now the K tile waits only for the previous QK^T and the V halves only for the previous
// PV.  P (64 heads x 128 keys bf16) is written by the softmax threads in two halves: lanes
// 0-63 the leader's keys, lanes 64-127 the peer's.
// QK^T and PV are issued by two threads, so one thread's barrier waits overlap the other's
// MMAs and the pipe takes QK^T of the next tile while the softmax of this one runs.  The
// running max is only raised when it grows by more than 2^8 (in exp2 units), which skips
// most O corrections.
#include "tc.cuh"

namespace mzb {
namespace mla {

constexpr int H = 128, HC = 64, DQK = 576, DV = 512, ROWB = 672, ROPE_OFF = 544, SCALE_OFF = 512;
constexpr int NT = 128, NTH = 64;          // keys per tile, per CTA
constexpr int QBLK = 9;
constexpr int BLK = NTH * 128;             // one 64-channel block of a K tile / V half (8 KB)
constexpr int Q_BYTES = QBLK * HC * 128;   // 73728
constexpr int K_BYTES = QBLK * BLK;        // 73728
constexpr int VH_BYTES = 4 * BLK;          // 32768: one key half x this CTA's 256 channels
constexpr int PH_BYTES = HC * 128;         // 8192: 64 heads x 64 keys bf16
constexpr int TILE_BYTES = Q_BYTES + K_BYTES + 2 * VH_BYTES + 2 * PH_BYTES;  // 229376
// misc (barriers, exchange buffers) after the tiles; no static shared memory, so the
// dynamic window starts 1024-aligned (checked at run time) and the total stays under the
// 227 KB per-block limit.
constexpr int MISC_BYTES = 512 + 2 * 2 * 128 * 4;
constexpr int SMEM_DYN = TILE_BYTES + MISC_BYTES;
constexpr int NTHREADS = 512;
constexpr int TMEM_COLS = 512;
constexpr int S_COL0 = 256, S_COLS = NTH;  // S buffers at columns 256 and 320
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;

enum Bar {
  Q_FULL = 0, Q_READY, Q_EMPTY,
  K_FULL,             // leader: both CTAs' K tiles written (8 producer warps each)
  K_EMPTY,            // local (multicast commit): QK^T of the tile done
  V_FULL,             // leader: both CTAs' V halves written (8 producer warps each)
  S_FULL, S_FULL1, S_EMPTY, S_EMPTY1,
  P_FULL,             // leader: P written and O corrected (4 softmax warps x 2 CTAs)
  O_DONE,             // local (multicast commit): PV of the tile done (P, V and O free)
  O_EMPTY,
  XCH, XCH1, XCH2, XCH3,  // row-max exchange per (S buffer, warp pair {4,6} / {5,7}), local
  XL, XL1,                // row-sum exchange per warp pair, local
  O_FINAL,            // multicast commit after an item's last PV (epilogue, item parity)
  NBAR
};
static_assert(8 * NBAR + 12 <= 512, "barriers + TMEM slot + abort flag + progress fit the first 512 misc bytes");
constexpr int PF_AHEAD = 2;  // the prefetch warp stays up to this many tiles ahead of the K writes
static_assert(SMEM_DYN <= 232448, "shared memory budget");

struct Args {
  const uint8_t* raw;
  const uint8_t* cmp;
  const int32_t* idx;      // [n_tok, topk]
  const int32_t* pos;      // [n_tok] absolute position of each query token
  const int32_t* n_slots;  // [n_tok] window length + last valid compressed slot + 1
  const int32_t* raw_pt;   // [B, raw_ptw] page table (64-row pages) or null (dense)
  const int32_t* cmp_pt;   // [B, cmp_ptw] or null
  const int32_t* cmp_lens; // [B] valid compressed entries per sequence, or null (= cmp_len)
  __nv_bfloat16* o;        // [n_tok, 128, 512]
  float* lse;              // [n_tok, 128]
  int n_tok, tok_per_seq, topk, window;
  long long raw_len, cmp_len;  // rows per sequence of the dense layouts
  int raw_ptw, cmp_ptw;
  float scale_log2;
  int n_split;      // key-range splits per token (1: write o/lse directly)
  float* o_part;    // [n_split, n_tok, 128, 512] fp32, each split's normalised output
  float* lse_part;  // [n_split, n_tok, 128] fp32 natural-log lse (-inf: empty split)
  int* err;
};

struct Slot {
  int b, pos, ws, n_win, g_lim;
};

__device__ __forceinline__ Slot item_info(const Args& a, int tk) {
  Slot s;
  s.b = tk / a.tok_per_seq;
  s.pos = a.pos[tk];
  s.ws = max(0, s.pos - a.window + 1);
  s.n_win = s.pos - s.ws + 1;
  s.g_lim = a.cmp_lens ? a.cmp_lens[s.b] : int(a.cmp_len);
  return s;
}

// Loads issued where they are written: asm volatile keeps the compiler from sinking a
// prefetch down to its first use.
__device__ __forceinline__ int ld_nc_s32(const int32_t* p) {
  int v;
  asm volatile("ld.global.nc.b32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ float ld_nc_f32(const void* p) {
  float v;
  asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ float4 ld_nc_f32x4(const void* p) {
  float4 v;
  asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}

// Key slot p of token tk is window row ws + p for p < n_win, else compressed entry
// idx[tk][p - n_win] (empty when that is out of range).  Its row address is found in two
// steps, so the index load can be issued well before the row is needed: the compressed
// index of slot p (-1 for a window slot or past the list) ...
__device__ __forceinline__ int slot_index(const Args& a, const Slot& s, int tk, int p) {
  const int c = p - s.n_win;
  return (p >= s.n_win && c < a.topk) ? ld_nc_s32(a.idx + (long long)tk * a.topk + c) : -1;
}

// ... and the row pointer of slot p given that index (nullptr for an empty slot).
__device__ __forceinline__ const uint8_t* slot_row_at(const Args& a, const Slot& s, int p, int g) {
  if (p < s.n_win) {
    const int r = s.ws + p;
    const long long row = a.raw_pt ? (long long)a.raw_pt[(long long)s.b * a.raw_ptw + (r >> 6)] * 64 + (r & 63)
                                   : (long long)s.b * a.raw_len + r;
    return a.raw + row * ROWB;
  }
  if (g < 0 || g >= s.g_lim) return nullptr;
  const long long row = a.cmp_pt ? (long long)a.cmp_pt[(long long)s.b * a.cmp_ptw + (g >> 6)] * 64 + (g & 63)
                                 : (long long)s.b * a.cmp_len + g;
  return a.cmp + row * ROWB;
}

// 16 e4m3 codes * scale -> 16 bf16 (two 16-byte chunks): e4m3 pairs -> f16x2 (exact) ->
// two f32 (exact), one packed f32x2 multiply by the scale, round to bf16x2 (the same value
// as fp32 code * scale rounded to bf16).
__device__ __forceinline__ uint32_t dequant2(uint32_t pair16, float scale) {
  uint32_t h2, out;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"((unsigned short)pair16));
  asm("{\n\t.reg .b16 l, h;\n\t.reg .f32 fl, fh;\n\t.reg .b64 v, sc;\n\t"
      "mov.b32 {l, h}, %1;\n\t"
      "cvt.f32.f16 fl, l;\n\tcvt.f32.f16 fh, h;\n\t"
      "mov.b64 v, {fl, fh};\n\tmov.b64 sc, {%2, %2};\n\t"
      "mul.rn.f32x2 v, v, sc;\n\t"
      "mov.b64 {fl, fh}, v;\n\t"
      "cvt.rn.bf16x2.f32 %0, fh, fl;\n\t}"
      : "=r"(out) : "r"(h2), "f"(scale));
  return out;
}

__device__ __forceinline__ void dequant16(const uint4 raw, float scale, uint4& lo, uint4& hi) {
  lo = make_uint4(dequant2(raw.x, scale), dequant2(raw.x >> 16, scale), dequant2(raw.y, scale),
                  dequant2(raw.y >> 16, scale));
  hi = make_uint4(dequant2(raw.z, scale), dequant2(raw.z >> 16, scale), dequant2(raw.w, scale),
                  dequant2(raw.w >> 16, scale));
}

__device__ __forceinline__ void st_shared16(uint8_t* p, const uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(p)), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ uint4 ld_nc16(const uint8_t* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Every wait is CTA-scope, including on barriers the peer CTA or the pair's MMA commits
// arrive on: the operands behind them sit in each CTA's own shared memory / TMEM (written
// by its own threads and fenced to the async proxy, or by bulk copies and TMA that complete
// on the barrier's transaction count), never read by the other CTA's threads.  A
// cluster-scope acquire costs ~130 cycles per check on the MMA issuers' critical path.
#define MLA_WAIT(bar, par, code)                                      \
  if (!tc::mbar_wait(&bars[bar], (par), a.err, (code))) {             \
    abort_flag = 1;                                                   \
    break;                                                            \
  }

// Phases: every role walks the same (item, tile) sequence and counts tiles in g.  A barrier
// completing once per tile is waited with parity g & 1 for tile g, and with (g & 1) ^ 1 for
// the completion of tile g - 1 (immediate at g = 0).  Each waiter has already seen the
// completion before the one it waits for, so a parity wait can never match an older phase.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NTHREADS, 1)
    mla_fwd_kernel(const __grid_constant__ CUtensorMap tq, Args a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = smem_raw;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + TILE_BYTES);
  uint32_t& tmem_slot = *reinterpret_cast<uint32_t*>(sm + TILE_BYTES + 8 * NBAR);
  volatile int& abort_flag = *reinterpret_cast<volatile int*>(sm + TILE_BYTES + 8 * NBAR + 4);
  // K tiles this CTA's producers have written (written by producer warp 8, read by warp 2)
  volatile int& k_progress = *reinterpret_cast<volatile int*>(sm + TILE_BYTES + 8 * NBAR + 8);
  float (*red_m)[128] = reinterpret_cast<float (*)[128]>(sm + TILE_BYTES + 512);
  float (*red_l)[128] = reinterpret_cast<float (*)[128]>(sm + TILE_BYTES + 512 + 1024);
  if (smem_u32(smem_raw) & 1023) {  // swizzled tiles need 1024-byte alignment
    if (threadIdx.x == 0) atomicExch(a.err, MZB_ERR_ALIGN);
    return;
  }
  uint8_t* qs = sm;
  uint8_t* ks = qs + Q_BYTES;
  uint8_t* vs = ks + K_BYTES;
  uint8_t* ps = vs + 2 * VH_BYTES;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = tc::cluster_ctarank();
  const int pair = int(tc::cluster_id_x()), npairs = int(tc::nclusters_x());

  if (threadIdx.x == 0) {
    const uint32_t counts[NBAR] = {1, 2, 1,           // Q_FULL, Q_READY, Q_EMPTY
                                   16, 1, 16,         // K_FULL, K_EMPTY, V_FULL
                                   1, 1, 8, 8,        // S_FULL x2, S_EMPTY x2
                                   8, 1, 8,           // P_FULL, O_DONE, O_EMPTY
                                   2, 2, 2, 2, 2, 2,  // XCH x4, XL x2 (the two warps holding one head's key halves)
                                   1};                // O_FINAL
    for (int i = 0; i < NBAR; ++i) tc::mbar_init(&bars[i], counts[i]);
    abort_flag = 0;
    k_progress = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) tc::tmem_alloc2(&tmem_slot, TMEM_COLS);
  if (warp == 0 && lane == 0) tc::prefetch_tmap(&tq);
  tc::fence_before_sync();
  __syncthreads();
  tc::cluster_sync();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_slot;
  auto leader_bar = [&](int i) { return tc::mapa(smem_u32(&bars[i]), 0); };
  // arrive on a leader-CTA barrier: a local arrive from the leader itself, a remote one
  // (CTA-scope release, see tc::mbar_arrive_remote) from the peer
  auto arrive_leader = [&](int i) {
    if (rank == 0) tc::mbar_arrive(&bars[i]);
    else tc::mbar_arrive_remote(leader_bar(i));
  };
  auto n_tiles = [&](int tk) { return (a.n_slots[tk] + NT - 1) / NT; };
  // work item = (token, key-range split), heaviest tokens first; tiles [t0, t1) of the
  // token's key list (an empty range when the token has fewer tiles than splits)
  const int items = a.n_tok * a.n_split;
  auto item_range = [&](int it, int& tk, int& sp, int& t0, int& t1) {
    tk = a.n_tok - 1 - it / a.n_split;
    sp = it % a.n_split;
    const int n = n_tiles(tk), per = (n + a.n_split - 1) / a.n_split;
    t0 = sp * per;
    t1 = min(n, t0 + per);
  };

  if (warp == 0) {
    // ------------------------------------------------------------------ Q loader
    if (lane == 0) {
      int ii = 0;
      bool issued = false;
      for (int it = pair; it < items && !abort_flag; it += npairs) {
        int tk, sp, t0, t1;
        item_range(it, tk, sp, t0, t1);
        if (t0 >= t1) continue;
        MLA_WAIT(Q_EMPTY, (ii & 1) ^ 1, 201);
        tc::mbar_expect_tx(&bars[Q_FULL], Q_BYTES);
        for (int cb = 0; cb < QBLK; ++cb)
          tc::tma_load_2d(qs + cb * HC * 128, &tq, &bars[Q_FULL], cb * 64, tk * H + int(rank) * HC);
        issued = true;
        MLA_WAIT(Q_FULL, ii & 1, 202);
        issued = false;
        arrive_leader(Q_READY);
        // the next item's Q block into L2 now, so its load at the item boundary (once this
        // item's last QK^T has read Q) does not wait on HBM
        for (int nx = it + npairs; nx < items; nx += npairs) {
          int tk2, sp2, u0, u1;
          item_range(nx, tk2, sp2, u0, u1);
          if (u0 >= u1) continue;
          for (int cb = 0; cb < QBLK; ++cb) tc::tma_prefetch_2d(&tq, cb * 64, tk2 * H + int(rank) * HC);
          break;
        }
        ++ii;
      }
      if (issued) tc::mbar_wait(&bars[Q_FULL], (ii & 1), nullptr, 0);  // drain before exit
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ QK^T issuer (leader)
    if (rank == 0 && lane == 0) {
      const uint32_t idesc_qk = tc::make_idesc(128, NT, 1, 1);
      // descriptors built once; the unrolled loop adds compile-time offsets (a single
      // thread issues every MMA, so per-MMA descriptor arithmetic would throttle issue)
      const uint64_t qd = tc::make_sdesc<128>(smem_u32(qs), 16, 1024);
      const uint64_t kd = tc::make_sdesc<128>(smem_u32(ks), 16, 1024);
      int g = 0, ii = 0;
      for (int it = pair; it < items && !abort_flag; it += npairs) {
        int tk, sp, t0, t1;
        item_range(it, tk, sp, t0, t1);
        if (t0 >= t1) continue;
        MLA_WAIT(Q_READY, ii & 1, 210);
        bool ok = true;
        for (int j = t0; j < t1; ++j, ++g) {
          const int st = g & 1, ph = (g >> 1) & 1;
          if (!tc::mbar_wait(&bars[K_FULL], g & 1, a.err, 214) ||
              !tc::mbar_wait(&bars[S_EMPTY + st], ph ^ 1, a.err, 215)) { ok = false; break; }
          tc::fence_after_sync();
          const uint32_t d = tmem + S_COL0 + st * S_COLS;
#pragma unroll
          for (int kk = 0; kk < 36; ++kk) {
            const int cb = kk >> 2, off = (kk & 3) * 32;
            tc::mma2_f16(d, tc::sdesc_add(qd, cb * 8192 + off), tc::sdesc_add(kd, cb * BLK + off), idesc_qk,
                         kk > 0 ? 1u : 0u);
          }
          tc::mma2_commit_mc(&bars[K_EMPTY], 3);
          tc::mma2_commit_mc(&bars[S_FULL + st], 3);
          if (j == t1 - 1) tc::mma2_commit_mc(&bars[Q_EMPTY], 3);
        }
        if (!ok) { abort_flag = 1; break; }
        ++ii;
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------------ L2 prefetch (paged)
    // Paged rows come from HBM in random 672-byte pieces, and a producer requests a tile's
    // rows only one tile ahead, when the chain index -> page table -> row is still an HBM
    // round trip.  This warp walks the same (item, tile) sequence and, while the producers
    // write K tile g, issues an L2 prefetch of every row of this CTA's keys of tile
    // g + PF_AHEAD, so the producers' own loads hit L2.  It only ever reads: if it falls
    // behind it prefetches rows already loaded, and a stalled pipeline (a bounded wait that
    // gave up) ends its wait after a bounded spin.
    if (a.raw_pt || a.cmp_pt) {
      int g = 0;
      for (int it = pair; it < items && !abort_flag; it += npairs) {
        int tk, sp, t0, t1;
        item_range(it, tk, sp, t0, t1);
        if (t0 >= t1) continue;
        const Slot s = item_info(a, tk);
        bool stop = false;
        for (int j = t0; j < t1; ++j, ++g) {
          for (int spin = 0; k_progress + PF_AHEAD < g; ++spin) {
            if (abort_flag || spin > (1 << 16)) { stop = true; break; }
            __nanosleep(128);
          }
          if (stop) break;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int p = j * NT + int(rank) * NTH + h * 32 + lane;
            const uint8_t* rp = slot_row_at(a, s, p, slot_index(a, s, tk, p));
            if (rp) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(rp), "n"(ROWB) : "memory");
          }
        }
        if (stop) break;
      }
    }
  } else if (warp == 3) {
    // ------------------------------------------------------------------ PV issuer (leader)
    if (rank == 0 && lane == 0) {
      const uint32_t idesc_pv = tc::make_idesc(128, 256, 1, 1, false, true);
      const uint64_t pd[2] = {tc::make_sdesc<128>(smem_u32(ps), 16, 1024),
                              tc::make_sdesc<128>(smem_u32(ps + PH_BYTES), 16, 1024)};
      const uint64_t vd[2] = {tc::make_sdesc<128>(smem_u32(vs), BLK, 1024),
                              tc::make_sdesc<128>(smem_u32(vs + VH_BYTES), BLK, 1024)};
      int g = 0, ii = 0;
      for (int it = pair; it < items && !abort_flag; it += npairs) {
        int tk, sp, t0, t1;
        item_range(it, tk, sp, t0, t1);
        if (t0 >= t1) continue;
        // the previous item's epilogue has read O
        MLA_WAIT(O_EMPTY, (ii & 1) ^ 1, 211);
        bool ok = true;
        for (int j = t0; j < t1 && ok; ++j, ++g) {
          if (!tc::mbar_wait(&bars[P_FULL], g & 1, a.err, 213) ||
              !tc::mbar_wait(&bars[V_FULL], g & 1, a.err, 212)) { ok = false; break; }
          tc::fence_after_sync();
#pragma unroll
          for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int i = 0; i < 2; ++i) {
#pragma unroll
              for (int jj = 0; jj < 4; ++jj)
                tc::mma2_f16(tmem + i * 128, tc::sdesc_add(pd[h], jj * 32), tc::sdesc_add(vd[h], 2 * i * BLK + jj * 2048),
                             idesc_pv, (j == t0 && h == 0 && jj == 0) ? 0u : 1u);
            }
          }
          tc::mma2_commit_mc(&bars[O_DONE], 3);
        }
        if (!ok) { abort_flag = 1; break; }
        tc::mma2_commit_mc(&bars[O_FINAL], 3);
        ++ii;
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------------ softmax / epilogue
    const int sw = warp - 4;
    const int l = sw * 32 + lane;  // TMEM lane
    const int kh = l >> 6, hrow = l & 63;
    const int head = int(rank) * HC + hrow;
    const float sl = a.scale_log2;
    int g = 0, ii = 0;
    for (int it = pair; it < items && !abort_flag; it += npairs) {
      int tk, sp, t0, t1;
      item_range(it, tk, sp, t0, t1);
      if (t0 >= t1) {  // a split with no keys: an empty partial for the combine
        float* orow = a.o_part + (((long long)sp * a.n_tok + tk) * H + head) * DV;
        for (int c = kh * 128; c < DV; c += 256)
          for (int q = 0; q < 128; q += 4) *reinterpret_cast<float4*>(orow + c + q) = make_float4(0.f, 0.f, 0.f, 0.f);
        if (kh == 0) a.lse_part[((long long)sp * a.n_tok + tk) * H + head] = -INFINITY;
        continue;
      }
      const Slot s = item_info(a, tk);
      float m = -1e30f, lsum = 0.0f;
      bool ok = true;
      // key validity: this lane's two keys of tile j + 1 (slots kofs and kofs + 32 of the
      // warp's key half) are looked up while tile j is processed (window slots need no load)
      auto slot_code = [&](int p) -> int {
        if (p < s.n_win) return 0;
        const int c = p - s.n_win;
        return c < a.topk ? ld_nc_s32(a.idx + (long long)tk * a.topk + c) : -1;
      };
      auto slot_ok = [&](int p, int code) { return p < s.n_win || (code >= 0 && code < s.g_lim); };
      const int kofs = kh * NTH + lane;
      int cn0 = slot_code(t0 * NT + kofs), cn1 = slot_code(t0 * NT + kofs + 32);
      for (int j = t0; j < t1; ++j, ++g) {
        const int st = g & 1, ph = (g >> 1) & 1;
        const int c0 = cn0, c1 = cn1;
        if (j + 1 < t1) {
          cn0 = slot_code((j + 1) * NT + kofs);
          cn1 = slot_code((j + 1) * NT + kofs + 32);
        }
        const int p = j * NT + kofs;
        const uint32_t vm0 = __ballot_sync(0xffffffffu, slot_ok(p, c0));
        const uint32_t vm1 = __ballot_sync(0xffffffffu, slot_ok(p + 32, c1));
        if (!tc::mbar_wait(&bars[S_FULL + st], ph, a.err, 220)) { ok = false; break; }
        tc::fence_after_sync();
        uint32_t sr[64];
        tc::tmem_ld32(tc::taddr(tmem, sw * 32, S_COL0 + st * S_COLS), *reinterpret_cast<uint32_t(*)[32]>(sr));
        tc::tmem_ld32(tc::taddr(tmem, sw * 32, S_COL0 + st * S_COLS + 32), *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
        tc::tmem_wait_ld();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) arrive_leader(S_EMPTY + st);
        float sv[64];
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const uint32_t vm = i < 32 ? vm0 : vm1;
          sv[i] = (vm >> (i & 31) & 1u) ? __uint_as_float(sr[i]) : -INFINITY;
          mx4[i & 3] = fmaxf(mx4[i & 3], sv[i]);
        }
        float mt = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
        // exchange with the thread holding the other key half of this head (mbarrier, bounded)
        red_m[st][l] = mt;
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bars[XCH + 2 * st + (sw & 1)]);
        if (!tc::mbar_wait(&bars[XCH + 2 * st + (sw & 1)], ph, a.err, 223)) { ok = false; break; }
        mt = fmaxf(mt, red_m[st][l ^ 64]);
        const bool need = mt * sl > m * sl + 8.0f;
        // both PV halves of the previous tile are done: P may be rewritten and O rescaled
        if (!tc::mbar_wait(&bars[O_DONE], (g & 1) ^ 1, a.err, 225)) { ok = false; break; }
        tc::fence_after_sync();
        const float m_new = need ? mt : m;
        const float alpha = fast_exp2((m - m_new) * sl);
        const float ms = m_new * sl;
        float ps4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        uint8_t* prow = ps + kh * PH_BYTES + hrow * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t pk[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float p0 = fast_exp2(fmaf(sv[8 * c + 2 * i], sl, -ms));
            const float p1 = fast_exp2(fmaf(sv[8 * c + 2 * i + 1], sl, -ms));
            ps4[i] += p0 + p1;
            pk[i] = pack_bf16(p0, p1);
          }
          st_shared16(prow + ((c ^ (hrow & 7)) * 16), make_uint4(pk[0], pk[1], pk[2], pk[3]));
        }
        const float psum = (ps4[0] + ps4[1]) + (ps4[2] + ps4[3]);
        lsum = lsum * alpha + psum;
        if (j > t0 && __any_sync(0xffffffffu, need)) {
          for (int c0 = 0; c0 < 256; c0 += 32) {
            uint32_t ov[32];
            tc::tmem_ld32(tc::taddr(tmem, sw * 32, c0), ov);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
            tc::tmem_st32(tc::taddr(tmem, sw * 32, c0), ov);
          }
          tc::tmem_wait_st();
        }
        m = m_new;
        tc::fence_async_smem();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) arrive_leader(P_FULL);
      }
      if (!ok) { abort_flag = 1; break; }
      // epilogue: O / l, lse.  O_FINAL, not O_DONE: the item's last PV can still be in flight
      // here, and the epilogue's parity is per item.
      MLA_WAIT(O_FINAL, ii & 1, 222);
      tc::fence_after_sync();
      red_l[ii & 1][l] = lsum;
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&bars[XL + (sw & 1)]);
      MLA_WAIT(XL + (sw & 1), ii & 1, 224);
      const float ltot = lsum + red_l[ii & 1][l ^ 64];
      const float inv = 1.0f / ltot;
      if (a.n_split > 1) {  // this split's normalised output and lse, merged by combine_kernel
        float* orow = a.o_part + (((long long)sp * a.n_tok + tk) * H + head) * DV;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          for (int c = 0; c < 4; ++c) {
            uint32_t ov[32];
            tc::tmem_ld32(tc::taddr(tmem, sw * 32, i * 128 + c * 32), ov);
            tc::tmem_wait_ld();
            float4* dst = reinterpret_cast<float4*>(orow + i * 256 + kh * 128 + c * 32);
#pragma unroll
            for (int q = 0; q < 8; ++q)
              dst[q] = make_float4(__uint_as_float(ov[4 * q + 0]) * inv, __uint_as_float(ov[4 * q + 1]) * inv,
                                   __uint_as_float(ov[4 * q + 2]) * inv, __uint_as_float(ov[4 * q + 3]) * inv);
          }
        }
        if (kh == 0) a.lse_part[((long long)sp * a.n_tok + tk) * H + head] = (m * sl + log2f(ltot)) * LN2;
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) arrive_leader(O_EMPTY);
        ++ii;
        continue;
      }
      // O / l to bf16: the eight 32-column TMEM loads double-buffered (the next one in flight
      // while this one is scaled and stored); each lane's 64 contiguous bytes as two 32-byte
      // stores (each warp store touches 32 head rows, so fewer, wider stores mean fewer
      // L1 wavefronts -- this epilogue stalls the pipeline at every item boundary)
      __nv_bfloat16* orow = a.o + ((long long)tk * H + head) * DV;
      const bool wide_st = (reinterpret_cast<uintptr_t>(a.o) & 31) == 0;
      uint32_t ov[2][32];
      auto ocol = [&](int it) { return tc::taddr(tmem, sw * 32, (it >> 2) * 128 + (it & 3) * 32); };
      tc::tmem_ld32(ocol(0), ov[0]);
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        uint32_t (&cur)[32] = ov[it & 1];
        tc::tmem_wait_ld();
        tc::reg_after_wait(cur);
        if (it + 1 < 8) tc::tmem_ld32(ocol(it + 1), ov[(it + 1) & 1]);
        uint32_t w[16];
#pragma unroll
        for (int q = 0; q < 16; ++q)
          w[q] = pack_bf16(__uint_as_float(cur[2 * q]) * inv, __uint_as_float(cur[2 * q + 1]) * inv);
        __nv_bfloat16* dst = orow + (it >> 2) * 256 + kh * 128 + (it & 3) * 32;
        if (wide_st) {
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2)
            asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst + h2 * 16),
                         "r"(w[8 * h2 + 0]), "r"(w[8 * h2 + 1]), "r"(w[8 * h2 + 2]), "r"(w[8 * h2 + 3]),
                         "r"(w[8 * h2 + 4]), "r"(w[8 * h2 + 5]), "r"(w[8 * h2 + 6]), "r"(w[8 * h2 + 7])
                         : "memory");
        } else {
          uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
          for (int q = 0; q < 4; ++q) d4[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
        }
      }
      if (kh == 0) a.lse[(long long)tk * H + head] = (m * sl + log2f(ltot)) * LN2;
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) arrive_leader(O_EMPTY);
      ++ii;
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------------ producers
    // Thread t: key kk = t / 4 of this CTA's 64, 16-byte chunks sub, sub + 4, ... of its row
    // (K tile), and chunks sub of each of this CTA's four V channel blocks of the peer's key
    // kk (V half `peer`).  Per tile:
    //   1. once QK^T of the previous tile is done: dequantise and write this CTA's K tile;
    //      then load the next tile's own rows (held in registers until step 1 comes again);
    //   2. once PV of the previous tile is done: copy this CTA's own V blocks out of its K
    //      tile into V half `rank` (bf16 already, shared memory to shared memory), dequantise
    //      the peer keys' chunks into V half `peer`; then load the next tile's peer chunks.
    // The K tile waits only for QK^T and the V halves only for PV; nothing crosses the pair.
    // The compressed indices of tile g + 2 are requested at the end of tile g, so no row
    // address waits on a dependent index load.
    const int t = threadIdx.x - 256;  // 0..255
    const int kk = t >> 2, sub = t & 3;
    const int peer = int(rank) ^ 1;
    // this CTA's V channel blocks: gb(lb) = (lb >> 1) * 4 + 2 rank + (lb & 1)
    auto vblock = [&](int lb) { return (lb >> 1) * 4 + 2 * int(rank) + (lb & 1); };
    // cursor over this pair's (item, tile) sequence, items without tiles skipped
    int it = pair, j = 0, tk = 0, sp = 0, t0 = 0, t1 = 0;
    Slot s{};
    auto next_item = [&]() -> bool {  // first item at or after `it` that has tiles
      for (; it < items; it += npairs) {
        item_range(it, tk, sp, t0, t1);
        if (t0 < t1) {
          s = item_info(a, tk);
          j = t0;
          return true;
        }
      }
      return false;
    };
    auto advance = [&]() -> bool {
      if (++j < t1) return true;
      it += npairs;
      return next_item();
    };
    const int pk_ofs = int(rank) * NTH + kk, pr_ofs = peer * NTH + kk;  // own / peer key of the tile
    uint4 kraw[10], rraw[4];
    float ksc[8], rsc[4];
    auto load_k = [&](const uint8_t* rp) {
#pragma unroll
      for (int q = 0; q < 10; ++q) {
        const int c = sub + 4 * q;
        kraw[q] = make_uint4(0, 0, 0, 0);
        if (rp) kraw[q] = ld_nc16(rp + (c < 32 ? 16 * c : ROPE_OFF + 16 * (c - 32)));
      }
#pragma unroll
      if (rp) {  // the row's 8 scales: two 16-byte loads
        const float4 s0 = ld_nc_f32x4(rp + SCALE_OFF), s1 = ld_nc_f32x4(rp + SCALE_OFF + 16);
        ksc[0] = s0.x; ksc[1] = s0.y; ksc[2] = s0.z; ksc[3] = s0.w;
        ksc[4] = s1.x; ksc[5] = s1.y; ksc[6] = s1.z; ksc[7] = s1.w;
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) ksc[q] = 0.0f;
      }
    };
    auto load_r = [&](const uint8_t* rp) {
#pragma unroll
      for (int lb = 0; lb < 4; ++lb) {
        rraw[lb] = make_uint4(0, 0, 0, 0);
        if (rp) rraw[lb] = ld_nc16(rp + vblock(lb) * 64 + sub * 16);
        rsc[lb] = rp ? ld_nc_f32(rp + SCALE_OFF + 4 * vblock(lb)) : 0.0f;
      }
    };
    // rows of tile 0 now; then the cursor moves to tile 1 and its two indices are requested
    // (they arrive while tile 0 is written)
    bool have = next_item(), have_next = false;
    int nk = -1, nr = -1;
    if (have) {
      const int p0 = j * NT;
      load_k(slot_row_at(a, s, p0 + pk_ofs, slot_index(a, s, tk, p0 + pk_ofs)));
      load_r(slot_row_at(a, s, p0 + pr_ofs, slot_index(a, s, tk, p0 + pr_ofs)));
      have_next = advance();
      if (have_next) {
        nk = slot_index(a, s, tk, j * NT + pk_ofs);
        nr = slot_index(a, s, tk, j * NT + pr_ofs);
      }
    }
    uint8_t* kt = ks + kk * 128;
    int g = 0;
    while (have && !abort_flag) {
      // 1. K tile g
      if (!tc::mbar_wait(&bars[K_EMPTY], (g & 1) ^ 1, a.err, 230)) { abort_flag = 1; break; }
#pragma unroll
      for (int q = 0; q < 10; ++q) {
        const int c = sub + 4 * q;
        if (c < 32) {
          uint4 lo, hi;
          dequant16(kraw[q], ksc[c >> 2], lo, hi);
          const int cb = c >> 2, ch = (c & 3) * 2;
          st_shared16(kt + cb * BLK + ((ch ^ (kk & 7)) * 16), lo);
          st_shared16(kt + cb * BLK + (((ch + 1) ^ (kk & 7)) * 16), hi);
        } else {
          st_shared16(kt + 8 * BLK + (((c - 32) ^ (kk & 7)) * 16), kraw[q]);
        }
      }
      tc::fence_async_smem();
      __syncwarp();
      if (lane == 0) arrive_leader(K_FULL);
      if (warp == 8 && lane == 0) k_progress = g + 1;
      if (have_next) load_k(slot_row_at(a, s, j * NT + pk_ofs, nk));  // own rows of tile g + 1
      // 2. V halves of tile g
      if (!tc::mbar_wait(&bars[O_DONE], (g & 1) ^ 1, a.err, 231)) { abort_flag = 1; break; }
      {
        // this thread's own K-tile chunks of the four V blocks (row kk, positions 2 sub and
        // 2 sub + 1 of each block): the same places in V half `rank`, so each thread reads
        // back only what it wrote itself and no producer waits for another
        uint8_t* vd = vs + int(rank) * VH_BYTES + kk * 128;
        uint4 cp[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const int lb = m >> 1, pos = ((2 * sub + (m & 1)) ^ (kk & 7)) * 16;
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(cp[m].x), "=r"(cp[m].y), "=r"(cp[m].z), "=r"(cp[m].w)
                       : "r"(smem_u32(kt + vblock(lb) * BLK + pos)));
        }
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const int lb = m >> 1, pos = ((2 * sub + (m & 1)) ^ (kk & 7)) * 16;
          st_shared16(vd + lb * BLK + pos, cp[m]);
        }
      }
      {
        uint8_t* vt = vs + peer * VH_BYTES + kk * 128;
#pragma unroll
        for (int lb = 0; lb < 4; ++lb) {
          uint4 lo, hi;
          dequant16(rraw[lb], rsc[lb], lo, hi);
          st_shared16(vt + lb * BLK + (((2 * sub) ^ (kk & 7)) * 16), lo);
          st_shared16(vt + lb * BLK + (((2 * sub + 1) ^ (kk & 7)) * 16), hi);
        }
      }
      tc::fence_async_smem();
      __syncwarp();
      if (lane == 0) arrive_leader(V_FULL);
      if (have_next) load_r(slot_row_at(a, s, j * NT + pr_ofs, nr));  // peer rows of tile g + 1
      // the cursor moves to tile g + 2 and its indices are requested
      have = have_next;
      if (have_next) {
        have_next = advance();
        if (have_next) {
          nk = slot_index(a, s, tk, j * NT + pk_ofs);
          nr = slot_index(a, s, tk, j * NT + pr_ofs);
        }
      }
      ++g;
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  tc::cluster_sync();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_free2(tmem, TMEM_COLS);
  }
}


// n_slots[tk] = window length + (last valid compressed slot + 1): the key-list length the
// fwd kernel walks (empty tail tiles are skipped).
__global__ void slots_kernel(Args a) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= a.n_tok) return;
  const Slot s = item_info(a, warp);
  int last = -1;
  for (int c = lane; c < a.topk; c += 32) {
    const int g = a.idx[(long long)warp * a.topk + c];
    if (g >= 0 && g < s.g_lim) last = c;
  }
  for (int o = 16; o; o >>= 1) last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
  if (lane == 0) const_cast<int32_t*>(a.n_slots)[warp] = s.n_win + last + 1;
}

// Merge the key-range splits of each (token, head): o = sum_i e^(lse_i) o_i / sum_i e^(lse_i),
// lse = log sum_i e^(lse_i).  One warp per (token, head), 16 channels per lane.
__global__ void __launch_bounds__(256) combine_kernel(Args a) {
  const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= (long long)a.n_tok * H) return;
  const long long row = wid;  // tk * H + head
  const long long stride = (long long)a.n_tok * H;
  float mx = -INFINITY;
  for (int sp = 0; sp < a.n_split; ++sp) mx = fmaxf(mx, a.lse_part[sp * stride + row]);
  float acc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i] = 0.0f;
  float wsum = 0.0f;
  for (int sp = 0; sp < a.n_split; ++sp) {
    const float l = a.lse_part[sp * stride + row];
    if (l == -INFINITY) continue;
    const float wgt = __expf(l - mx);
    wsum += wgt;
    const float4* src = reinterpret_cast<const float4*>(a.o_part + (sp * stride + row) * DV + lane * 16);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 v = src[q];
      acc[4 * q + 0] = fmaf(wgt, v.x, acc[4 * q + 0]);
      acc[4 * q + 1] = fmaf(wgt, v.y, acc[4 * q + 1]);
      acc[4 * q + 2] = fmaf(wgt, v.z, acc[4 * q + 2]);
      acc[4 * q + 3] = fmaf(wgt, v.w, acc[4 * q + 3]);
    }
  }
  const float inv = 1.0f / wsum;
  uint4* dst = reinterpret_cast<uint4*>(a.o + row * DV + lane * 16);
  dst[0] = make_uint4(pack_bf16(acc[0] * inv, acc[1] * inv), pack_bf16(acc[2] * inv, acc[3] * inv),
                      pack_bf16(acc[4] * inv, acc[5] * inv), pack_bf16(acc[6] * inv, acc[7] * inv));
  dst[1] = make_uint4(pack_bf16(acc[8] * inv, acc[9] * inv), pack_bf16(acc[10] * inv, acc[11] * inv),
                      pack_bf16(acc[12] * inv, acc[13] * inv), pack_bf16(acc[14] * inv, acc[15] * inv));
  if (lane == 0) a.lse[row] = mx + logf(wsum);
}

// Splits per token: only when the tokens alone would leave more than half of the SM pairs
// idle (decode of a few sequences per GPU); then floor(pairs / n_tok), at most 8, so all
// (token, split) items run in one wave.  A split costs a Q reload, an fp32 partial output
// round trip through HBM and the combine kernel, which outweigh the gain otherwise.
static int choose_splits(long long n_tok) {
  const long long pairs = num_sms() / 2;
  if (n_tok <= 0 || 2 * n_tok > pairs) return 1;
  const long long s = pairs / n_tok;
  return int(s > 8 ? 8 : (s < 1 ? 1 : s));
}

}  // namespace mla
}  // namespace mzb

using namespace mzb;

extern "C" int mzb_sparse_mla_splits(int64_t n_tok) { return mla::choose_splits(n_tok); }

extern "C" int mzb_sparse_mla_fwd(const void* q, const void* kv_raw, const void* kv_cmp, const int32_t* indices,
                                  const int32_t* q_pos, const int32_t* raw_page_table,
                                  const int32_t* cmp_page_table, const int32_t* cmp_lens, int32_t* slots_ws,
                                  void* o, float* lse, int64_t n_tok, int tok_per_seq, int topk, int window,
                                  int64_t raw_len, int64_t cmp_len, int raw_ptw, int cmp_ptw, float softmax_scale,
                                  int splits, float* part_ws, int* err, void* stream) {
  MZB_REQUIRE(splits >= 1 && splits <= 64 && (splits == 1 || part_ws != nullptr), MZB_ERR_SHAPE,
              "sparse_mla: splits=%d needs 1..64 and a partial-output workspace when > 1", splits);
  MZB_REQUIRE(n_tok >= 0 && tok_per_seq >= 1 && topk >= 0 && window >= 1, MZB_ERR_SHAPE,
              "sparse_mla: bad sizes n_tok=%lld tok_per_seq=%d topk=%d window=%d", (long long)n_tok, tok_per_seq,
              topk, window);
  MZB_REQUIRE(n_tok * 128 < (int64_t(1) << 31), MZB_ERR_SHAPE, "sparse_mla: too many tokens");
  MZB_REQUIRE(reinterpret_cast<uintptr_t>(q) % 16 == 0 && reinterpret_cast<uintptr_t>(kv_raw) % 16 == 0 &&
                  (kv_cmp == nullptr || reinterpret_cast<uintptr_t>(kv_cmp) % 16 == 0) &&
                  reinterpret_cast<uintptr_t>(o) % 16 == 0,
              MZB_ERR_ALIGN, "sparse_mla: q, kv rows and o must be 16-byte aligned");
  MZB_REQUIRE(err != nullptr && slots_ws != nullptr, MZB_ERR_SHAPE, "sparse_mla: needs err and slots workspace");
  if (n_tok == 0) return MZB_OK;
  mla::Args a{};
  a.raw = static_cast<const uint8_t*>(kv_raw);
  a.cmp = static_cast<const uint8_t*>(kv_cmp);
  a.idx = indices; a.pos = q_pos; a.n_slots = slots_ws;
  a.raw_pt = raw_page_table; a.cmp_pt = cmp_page_table; a.cmp_lens = cmp_lens;
  a.o = static_cast<__nv_bfloat16*>(o); a.lse = lse;
  a.n_tok = int(n_tok); a.tok_per_seq = tok_per_seq; a.topk = topk; a.window = window;
  a.raw_len = raw_len; a.cmp_len = cmp_len; a.raw_ptw = raw_ptw; a.cmp_ptw = cmp_ptw;
  a.scale_log2 = softmax_scale * mla::LOG2E;
  a.n_split = splits;
  a.o_part = part_ws;
  a.lse_part = part_ws ? part_ws + (long long)splits * n_tok * mla::H * mla::DV : nullptr;
  a.err = err;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  mla::slots_kernel<<<unsigned((n_tok * 32 + 255) / 256), 256, 0, st>>>(a);
  if (int r = launch_status("sparse_mla_slots")) return r;

  CUtensorMap tq;
  const uint64_t dims[2] = {uint64_t(mla::DQK), uint64_t(n_tok) * mla::H};
  const uint64_t str[1] = {uint64_t(mla::DQK) * 2};
  const uint32_t box[2] = {64, uint32_t(mla::HC)};
  if (int r = encode_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, q, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
    return r;
  if (cudaFuncSetAttribute(mla::mla_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, mla::SMEM_DYN) !=
      cudaSuccess)
    return launch_status("sparse_mla(smem attr)");
  int pairs = num_sms() / 2;
  if (pairs > n_tok * splits) pairs = int(n_tok * splits);
  mla::mla_fwd_kernel<<<unsigned(2 * pairs), mla::NTHREADS, mla::SMEM_DYN, st>>>(tq, a);
  if (int r = launch_status("sparse_mla_fwd")) return r;
  if (splits > 1) {
    const long long warps = n_tok * mla::H;
    mla::combine_kernel<<<unsigned((warps * 32 + 255) / 256), 256, 0, st>>>(a);
    return launch_status("sparse_mla_combine");
  }
  return MZB_OK;
}

// ------------------------------------------------------------------------------------------
// Allocation-free variant of mzb_sparse_mla_fwd.
//
// Some callers cannot allocate device memory when they launch attention: a serving engine
// that has already handed every free byte of HBM to its paged KV-cache pool, or a C/C++
// host with its own memory manager, where a cudaMalloc would implicitly synchronise the
// device and stall every other stream.  mzb_sparse_mla_fwd itself allocates nothing, but
// it asks the caller for an int32 workspace of n_tok entries (the per-token key-list
// lengths).  This entry point takes that workspace from a fixed array in the library's own
// device memory instead, so the caller passes only inputs and outputs.
//
// The array holds MZB_NOALLOC_MAX_TOKENS entries (256 KB) and exists on every GPU that
// loads the library, for the life of the process.  Larger calls are rejected.  The array
// is shared by every call on a device and keeps the last call's contents; each call
// rewrites every entry it reads, so nothing needs clearing, but two calls whose kernels
// overlap on the GPU (different streams, no ordering between them) race on it.  The first
// call on each device looks up the array's device address (cudaGetSymbolAddress, with that
// device current) and caches it; make that first call before any stream capture.
// ------------------------------------------------------------------------------------------
#include <mutex>

#define MZB_NOALLOC_MAX_TOKENS 65536

static __device__ __align__(256) int32_t g_noalloc_slots[MZB_NOALLOC_MAX_TOKENS];

namespace {
constexpr int kMaxDevices = 64;
int32_t* g_noalloc_addr[kMaxDevices] = {nullptr};
std::mutex g_noalloc_mu;

int noalloc_scratch(int32_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    mzb::set_error("sparse_mla_fwd_noalloc: no usable current device");
    return MZB_ERR_LAUNCH;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_slots);
    if (e != cudaSuccess || p == nullptr) {
      mzb::set_error("sparse_mla_fwd_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return MZB_ERR_LAUNCH;
    }
    g_noalloc_addr[dev] = static_cast<int32_t*>(p);
  }
  *out = g_noalloc_addr[dev];
  return MZB_OK;
}
}  // namespace

extern "C" int mzb_sparse_mla_fwd_noalloc(const void* q, const void* kv_raw, const void* kv_cmp,
                                          const int32_t* indices, const int32_t* q_pos,
                                          const int32_t* raw_page_table, const int32_t* cmp_page_table,
                                          const int32_t* cmp_lens, void* o, float* lse, int64_t n_tok,
                                          int tok_per_seq, int topk, int window, int64_t raw_len, int64_t cmp_len,
                                          int raw_ptw, int cmp_ptw, float softmax_scale, int* err, void* stream) {
  MZB_REQUIRE(n_tok >= 0 && n_tok <= MZB_NOALLOC_MAX_TOKENS, MZB_ERR_SHAPE,
              "sparse_mla_fwd_noalloc: n_tok=%lld exceeds the fixed scratch of %d tokens (use mzb_sparse_mla_fwd "
              "with a caller workspace)",
              (long long)n_tok, MZB_NOALLOC_MAX_TOKENS);
  int32_t* slots = nullptr;
  if (int r = noalloc_scratch(&slots)) return r;
  return mzb_sparse_mla_fwd(q, kv_raw, kv_cmp, indices, q_pos, raw_page_table, cmp_page_table, cmp_lens, slots, o,
                            lse, n_tok, tok_per_seq, topk, window, raw_len, cmp_len, raw_ptw, cmp_ptw, softmax_scale,
                            1, nullptr, err, stream);
}
