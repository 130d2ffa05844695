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
// fp32 O (64 x 512) in TMEM as 128 lanes x 256 columns and S (64 x 64 keys) as 128 lanes x
// 32 columns.  Keys come in tiles of 64 (32 per CTA for the QK^T B operand).
//
// Warp roles per CTA (512 threads):
//   0      TMA of this CTA's Q half (64 heads x 576, 9 swizzled 64-column blocks)
//   1      TMEM allocation; in the leader CTA, the single MMA-issuing thread
//   4-7    softmax / O correction / epilogue (thread = TMEM lane = (head, key half))
//   8-11   K producers: gather + dequantise this CTA's 32 keys x 576 channels to bf16
//   12-15  V producers: gather + dequantise all 64 keys x this CTA's 256 V channels
// MMA order per item: QK_0, QK_1, PV_0, QK_2, PV_1, ...; tile g's S completion implies
// PV_{g-2} finished (in-order tensor pipe), so P is double-buffered without extra waits.
// The running max is only raised when it grows by more than 2^8 (in exp2 units), which
// skips most O corrections.
#include "tc.cuh"

namespace mzb {
namespace mla {

constexpr int H = 128, HC = 64, DQK = 576, DV = 512, ROWB = 672, ROPE_OFF = 544, SCALE_OFF = 512;
constexpr int NT = 64, NTH = 32;
constexpr int QBLK = 9;
constexpr int Q_BYTES = QBLK * HC * 128;   // 73728
constexpr int K_BYTES = QBLK * NTH * 128;  // 36864
constexpr int V_BYTES = 4 * NT * 128;      // 32768
constexpr int P_BYTES = HC * 128;          // 8192
constexpr int TILE_BYTES = Q_BYTES + 2 * K_BYTES + 2 * V_BYTES + 2 * P_BYTES;  // 229376
// misc (barriers, exchange buffers) after the tiles; no static shared memory, so the
// dynamic window starts 1024-aligned (checked at run time) and the total stays under the
// 227 KB per-block limit.
constexpr int MISC_BYTES = 256 + 2 * 2 * 128 * 4;
constexpr int SMEM_DYN = TILE_BYTES + MISC_BYTES;
constexpr int NTHREADS = 512;
constexpr int TMEM_COLS = 512;
constexpr int S_COL0 = 256;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;

enum Bar {
  Q_FULL = 0, Q_READY, Q_EMPTY,
  K_FULL, K_FULL1, K_EMPTY, K_EMPTY1,
  V_FULL, V_FULL1, V_EMPTY, V_EMPTY1,
  S_FULL, S_FULL1, S_EMPTY, S_EMPTY1,
  P_FULL, P_FULL1, O_DONE, O_EMPTY, XCH, XCH1, XL, NBAR
};

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

// Row pointer of key slot p of token tk (window first, then the compressed list), or
// nullptr for an empty / out-of-range slot.
__device__ __forceinline__ const uint8_t* slot_row(const Args& a, const Slot& s, int tk, int p) {
  if (p < s.n_win) {
    const int r = s.ws + p;
    const long long row = a.raw_pt ? (long long)a.raw_pt[(long long)s.b * a.raw_ptw + (r >> 6)] * 64 + (r & 63)
                                   : (long long)s.b * a.raw_len + r;
    return a.raw + row * ROWB;
  }
  const int c = p - s.n_win;
  if (c >= a.topk) return nullptr;
  const int g = a.idx[(long long)tk * a.topk + c];
  if (g < 0 || g >= s.g_lim) return nullptr;
  const long long row = a.cmp_pt ? (long long)a.cmp_pt[(long long)s.b * a.cmp_ptw + (g >> 6)] * 64 + (g & 63)
                                 : (long long)s.b * a.cmp_len + g;
  return a.cmp + row * ROWB;
}

__device__ __forceinline__ bool slot_valid(const Args& a, const Slot& s, int tk, int p) {
  if (p < s.n_win) return true;
  const int c = p - s.n_win;
  if (c >= a.topk) return false;
  const int g = a.idx[(long long)tk * a.topk + c];
  return g >= 0 && g < s.g_lim;
}

// 16 e4m3 codes * scale -> 16 bf16 (two 16-byte chunks).
__device__ __forceinline__ void dequant16(const uint4 raw, float scale, uint4& lo, uint4& hi) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  uint32_t out[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[i] >> (16 * h)), __NV_E4M3);
      const float2 f = __half22float2(__half2(hr));
      const __nv_bfloat162 bb = __floats2bfloat162_rn(f.x * scale, f.y * scale);
      out[i * 2 + h] = *reinterpret_cast<const uint32_t*>(&bb);
    }
  }
  lo = make_uint4(out[0], out[1], out[2], out[3]);
  hi = make_uint4(out[4], out[5], out[6], out[7]);
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

#define MLA_WAIT(bar, par, code)                                      \
  if (!tc::mbar_wait(&bars[bar], (par), a.err, (code))) {             \
    abort_flag = 1;                                                   \
    break;                                                            \
  }

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NTHREADS, 1)
    mla_fwd_kernel(const __grid_constant__ CUtensorMap tq, Args a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = smem_raw;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + TILE_BYTES);
  uint32_t& tmem_slot = *reinterpret_cast<uint32_t*>(sm + TILE_BYTES + 8 * NBAR);
  volatile int& abort_flag = *reinterpret_cast<volatile int*>(sm + TILE_BYTES + 8 * NBAR + 4);
  float (*red_m)[128] = reinterpret_cast<float (*)[128]>(sm + TILE_BYTES + 256);
  float (*red_l)[128] = reinterpret_cast<float (*)[128]>(sm + TILE_BYTES + 256 + 1024);
  if (smem_u32(smem_raw) & 1023) {  // swizzled tiles need 1024-byte alignment
    if (threadIdx.x == 0) atomicExch(a.err, MZB_ERR_ALIGN);
    return;
  }
  uint8_t* qs = sm;
  uint8_t* ks = qs + Q_BYTES;
  uint8_t* vs = ks + 2 * K_BYTES;
  uint8_t* ps = vs + 2 * V_BYTES;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = tc::cluster_ctarank();
  const int pair = int(tc::cluster_id_x()), npairs = int(tc::nclusters_x());

  if (threadIdx.x == 0) {
    const uint32_t counts[NBAR] = {1, 2, 1, 8, 8, 1, 1, 8, 8, 1, 1, 1, 1, 8, 8, 8, 8, 1, 8, 4, 4, 4};
    for (int i = 0; i < NBAR; ++i) tc::mbar_init(&bars[i], counts[i]);
    abort_flag = 0;
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
  auto n_tiles = [&](int tk) { return (a.n_slots[tk] + NT - 1) / NT; };

  if (warp == 0) {
    // ------------------------------------------------------------------ Q loader
    if (lane == 0) {
      int ii = 0;
      bool issued = false;
      for (int it = pair; it < a.n_tok && !abort_flag; it += npairs, ++ii) {
        const int tk = a.n_tok - 1 - it;
        MLA_WAIT(Q_EMPTY, (ii & 1) ^ 1, 201);
        tc::mbar_expect_tx(&bars[Q_FULL], Q_BYTES);
        for (int cb = 0; cb < QBLK; ++cb)
          tc::tma_load_2d(qs + cb * HC * 128, &tq, &bars[Q_FULL], cb * 64, tk * H + int(rank) * HC);
        issued = true;
        MLA_WAIT(Q_FULL, ii & 1, 202);
        issued = false;
        tc::mbar_arrive_cluster(leader_bar(Q_READY));
      }
      if (issued) tc::mbar_wait(&bars[Q_FULL], (ii & 1), nullptr, 0);  // drain before exit
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (leader)
    if (rank == 0 && lane == 0) {
      const uint32_t idesc_qk = tc::make_idesc(128, NT, 1, 1);
      const uint32_t idesc_pv = tc::make_idesc(128, 256, 1, 1, false, true);
      const uint32_t q_base = smem_u32(qs), k_base = smem_u32(ks), v_base = smem_u32(vs), p_base = smem_u32(ps);
      int g = 0, ii = 0;
      auto pv = [&](int gg, bool first, int item) -> bool {
        const int st = gg & 1, ph = (gg >> 1) & 1;
        if (first && !tc::mbar_wait(&bars[O_EMPTY], (item & 1) ^ 1, a.err, 211)) return false;
        if (!tc::mbar_wait(&bars[V_FULL + st], ph, a.err, 212)) return false;
        if (!tc::mbar_wait(&bars[P_FULL + st], ph, a.err, 213)) return false;
        tc::fence_after_sync();
#pragma unroll
        for (int i = 0; i < 2; ++i) {
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const uint64_t ad = tc::make_sdesc<128>(p_base + st * P_BYTES + jj * 32, 16, 1024);
            const uint64_t bd = tc::make_sdesc<128>(v_base + st * V_BYTES + 2 * i * 8192 + jj * 2048, 8192, 1024);
            tc::mma2_f16(tmem + i * 128, ad, bd, idesc_pv, (first && jj == 0) ? 0u : 1u);
          }
        }
        tc::mma2_commit_mc(&bars[V_EMPTY + st], 3);
        tc::mma2_commit_mc(&bars[O_DONE], 3);
        return true;
      };
      for (int it = pair; it < a.n_tok && !abort_flag; it += npairs, ++ii) {
        const int tk = a.n_tok - 1 - it;
        const int n = n_tiles(tk);
        MLA_WAIT(Q_READY, ii & 1, 210);
        bool ok = true;
        for (int j = 0; j < n; ++j, ++g) {
          const int st = g & 1, ph = (g >> 1) & 1;
          if (!tc::mbar_wait(&bars[K_FULL + st], ph, a.err, 214) ||
              !tc::mbar_wait(&bars[S_EMPTY + st], ph ^ 1, a.err, 215)) { ok = false; break; }
          tc::fence_after_sync();
          const uint32_t d = tmem + S_COL0 + st * 32;
#pragma unroll 4
          for (int kk = 0; kk < 36; ++kk) {
            const int cb = kk >> 2, off = (kk & 3) * 32;
            const uint64_t ad = tc::make_sdesc<128>(q_base + cb * 8192 + off, 16, 1024);
            const uint64_t bd = tc::make_sdesc<128>(k_base + st * K_BYTES + cb * 4096 + off, 16, 1024);
            tc::mma2_f16(d, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
          }
          tc::mma2_commit_mc(&bars[K_EMPTY + st], 3);
          tc::mma2_commit_mc(&bars[S_FULL + st], 3);
          if (j == n - 1) tc::mma2_commit_mc(&bars[Q_EMPTY], 3);
          if (j >= 1 && !pv(g - 1, j == 1, ii)) { ok = false; break; }
        }
        if (!ok || !pv(g - 1, n == 1, ii)) { abort_flag = 1; break; }
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
    for (int it = pair; it < a.n_tok && !abort_flag; it += npairs, ++ii) {
      const int tk = a.n_tok - 1 - it;
      const int n = n_tiles(tk);
      const Slot s = item_info(a, tk);
      float m = -1e30f, lsum = 0.0f;
      bool ok = true;
      for (int j = 0; j < n; ++j, ++g) {
        const int st = g & 1, ph = (g >> 1) & 1;
        // key validity (global index loads) before waiting on the MMA
        const uint32_t vmask = __ballot_sync(0xffffffffu, slot_valid(a, s, tk, j * NT + kh * NTH + lane));
        if (!tc::mbar_wait(&bars[S_FULL + st], ph, a.err, 220)) { ok = false; break; }
        tc::fence_after_sync();
        uint32_t sr[32];
        tc::tmem_ld32(tc::taddr(tmem, sw * 32, S_COL0 + st * 32), sr);
        tc::tmem_wait_ld();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive_cluster(leader_bar(S_EMPTY + st));
        float sv[32];
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          sv[i] = (vmask >> i & 1u) ? __uint_as_float(sr[i]) : -INFINITY;
          mx4[i & 3] = fmaxf(mx4[i & 3], sv[i]);
        }
        float mt = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
        // exchange with the thread holding the other key half of this head (mbarrier, bounded)
        red_m[st][l] = mt;
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bars[XCH + st]);
        if (!tc::mbar_wait(&bars[XCH + st], ph, a.err, 223)) { ok = false; break; }
        mt = fmaxf(mt, red_m[st][l ^ 64]);
        const bool need = mt * sl > m * sl + 8.0f;
        const float m_new = need ? mt : m;
        const float alpha = fast_exp2((m - m_new) * sl);
        const float ms = m_new * sl;
        uint32_t pk[16];
        float ps4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float p0 = fast_exp2(fmaf(sv[2 * i], sl, -ms));
          const float p1 = fast_exp2(fmaf(sv[2 * i + 1], sl, -ms));
          ps4[i & 3] += p0 + p1;
          pk[i] = pack_bf16(p0, p1);
        }
        const float psum = (ps4[0] + ps4[1]) + (ps4[2] + ps4[3]);
        lsum = lsum * alpha + psum;
        uint8_t* prow = ps + st * P_BYTES + hrow * 128;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          st_shared16(prow + (((kh * 4 + c) ^ (hrow & 7)) * 16), make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]));
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          if (!tc::mbar_wait(&bars[O_DONE], (g - 1) & 1, a.err, 221)) { ok = false; break; }
          tc::fence_after_sync();
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
        if (lane == 0) tc::mbar_arrive_cluster(leader_bar(P_FULL + st));
      }
      if (!ok) { abort_flag = 1; break; }
      // epilogue: O / l, lse
      MLA_WAIT(O_DONE, (g - 1) & 1, 222);
      tc::fence_after_sync();
      red_l[ii & 1][l] = lsum;
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&bars[XL]);
      MLA_WAIT(XL, ii & 1, 224);
      const float ltot = lsum + red_l[ii & 1][l ^ 64];
      const float inv = 1.0f / ltot;
      __nv_bfloat16* orow = a.o + ((long long)tk * H + head) * DV;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        for (int c = 0; c < 4; ++c) {
          uint32_t ov[32];
          tc::tmem_ld32(tc::taddr(tmem, sw * 32, i * 128 + c * 32), ov);
          tc::tmem_wait_ld();
          uint4* dst = reinterpret_cast<uint4*>(orow + i * 256 + kh * 128 + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            dst[q] = make_uint4(pack_bf16(__uint_as_float(ov[8 * q + 0]) * inv, __uint_as_float(ov[8 * q + 1]) * inv),
                                pack_bf16(__uint_as_float(ov[8 * q + 2]) * inv, __uint_as_float(ov[8 * q + 3]) * inv),
                                pack_bf16(__uint_as_float(ov[8 * q + 4]) * inv, __uint_as_float(ov[8 * q + 5]) * inv),
                                pack_bf16(__uint_as_float(ov[8 * q + 6]) * inv, __uint_as_float(ov[8 * q + 7]) * inv));
        }
      }
      if (kh == 0) a.lse[(long long)tk * H + head] = (m * sl + log2f(ltot)) * LN2;
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive_cluster(leader_bar(O_EMPTY));
    }
  } else if (warp >= 8 && warp < 12) {
    // ------------------------------------------------------------------ K producers
    const int t = threadIdx.x - 256;  // 0..127
    const int kk = t >> 2, sub = t & 3;
    int g = 0;
    for (int it = pair; it < a.n_tok && !abort_flag; it += npairs) {
      const int tk = a.n_tok - 1 - it;
      const int n = n_tiles(tk);
      const Slot s = item_info(a, tk);
      bool ok = true;
      for (int j = 0; j < n; ++j, ++g) {
        const int st = g & 1, ph = (g >> 1) & 1;
        const uint8_t* rp = slot_row(a, s, tk, j * NT + int(rank) * NTH + kk);
        uint4 raw[10];
        float sc[8];
#pragma unroll
        for (int q = 0; q < 10; ++q) {
          const int c = sub + 4 * q;
          raw[q] = make_uint4(0, 0, 0, 0);
          if (rp) raw[q] = ld_nc16(rp + (c < 32 ? 16 * c : ROPE_OFF + 16 * (c - 32)));
        }
#pragma unroll
        for (int q = 0; q < 8; ++q) sc[q] = rp ? __ldg(reinterpret_cast<const float*>(rp + SCALE_OFF) + q) : 0.0f;
        if (!tc::mbar_wait(&bars[K_EMPTY + st], ph ^ 1, a.err, 230)) { ok = false; break; }
        uint8_t* kt = ks + st * K_BYTES + kk * 128;
#pragma unroll
        for (int q = 0; q < 10; ++q) {
          const int c = sub + 4 * q;
          if (c < 32) {
            uint4 lo, hi;
            dequant16(raw[q], sc[c >> 2], lo, hi);
            const int cb = c >> 2, ch = (c & 3) * 2;
            st_shared16(kt + cb * 4096 + ((ch ^ (kk & 7)) * 16), lo);
            st_shared16(kt + cb * 4096 + (((ch + 1) ^ (kk & 7)) * 16), hi);
          } else {
            st_shared16(kt + 8 * 4096 + (((c - 32) ^ (kk & 7)) * 16), raw[q]);
          }
        }
        tc::fence_async_smem();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive_cluster(leader_bar(K_FULL + st));
      }
      if (!ok) { abort_flag = 1; break; }
    }
  } else if (warp >= 12) {
    // ------------------------------------------------------------------ V producers
    const int t = threadIdx.x - 384;  // 0..127
    const int key = t >> 1, sub = t & 1;
    int g = 0;
    for (int it = pair; it < a.n_tok && !abort_flag; it += npairs) {
      const int tk = a.n_tok - 1 - it;
      const int n = n_tiles(tk);
      const Slot s = item_info(a, tk);
      bool ok = true;
      for (int j = 0; j < n; ++j, ++g) {
        const int st = g & 1, ph = (g >> 1) & 1;
        const uint8_t* rp = slot_row(a, s, tk, j * NT + key);
        uint4 raw[8];
        float sc[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int cc = sub * 8 + q, lb = cc >> 2, w = cc & 3;
          const int gb = (lb >> 1) * 4 + int(rank) * 2 + (lb & 1);
          raw[q] = make_uint4(0, 0, 0, 0);
          sc[q] = 0.0f;
          if (rp) {
            raw[q] = ld_nc16(rp + gb * 64 + w * 16);
            sc[q] = __ldg(reinterpret_cast<const float*>(rp + SCALE_OFF) + gb);
          }
        }
        if (!tc::mbar_wait(&bars[V_EMPTY + st], ph ^ 1, a.err, 240)) { ok = false; break; }
        uint8_t* vt = vs + st * V_BYTES + key * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int cc = sub * 8 + q, lb = cc >> 2, w = cc & 3;
          uint4 lo, hi;
          dequant16(raw[q], sc[q], lo, hi);
          st_shared16(vt + lb * 8192 + (((2 * w) ^ (key & 7)) * 16), lo);
          st_shared16(vt + lb * 8192 + (((2 * w + 1) ^ (key & 7)) * 16), hi);
        }
        tc::fence_async_smem();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive_cluster(leader_bar(V_FULL + st));
      }
      if (!ok) { abort_flag = 1; break; }
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

}  // namespace mla
}  // namespace mzb

using namespace mzb;

extern "C" int mzb_sparse_mla_fwd(const void* q, const void* kv_raw, const void* kv_cmp, const int32_t* indices,
                                  const int32_t* q_pos, const int32_t* raw_page_table,
                                  const int32_t* cmp_page_table, const int32_t* cmp_lens, int32_t* slots_ws,
                                  void* o, float* lse, int64_t n_tok, int tok_per_seq, int topk, int window,
                                  int64_t raw_len, int64_t cmp_len, int raw_ptw, int cmp_ptw, float softmax_scale,
                                  int* err, void* stream) {
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
  if (pairs > n_tok) pairs = int(n_tok);
  mla::mla_fwd_kernel<<<unsigned(2 * pairs), mla::NTHREADS, mla::SMEM_DYN, st>>>(tq, a);
  return launch_status("sparse_mla_fwd");
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
                            err, stream);
}
