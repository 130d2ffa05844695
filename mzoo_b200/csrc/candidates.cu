// Two-level (hierarchical) indexer selection: level-one candidate blocks and the level-two
// top-k restricted to them.
//
// Reference: src/mzoo/archs/dsv4/modeling_deepseek_v41.py:427-454 `select_candidate_blocks`
// (identical in src/mzoo/archs/owlet1/indexer.py:14-41) and its use in
// `DeepseekV41Indexer.forward` :558-578:
//   level one   block score = amax of `block_size` consecutive logits (the row padded with
//               -inf to a multiple of block_size); the block holding the newest visible
//               position, (compress_len - 1) // block_size, is pinned to +inf; keep the
//               top `topk_blocks` blocks whose score is > -inf (fewer reachable blocks
//               than topk_blocks is normal); the mask repeats each block's flag over its
//               positions, truncated to T.
//   level two   a later index source sets its scores outside the candidates to -inf and
//               keeps its top `topk` positions, dropping picks whose score is -inf.
// Ties: torch.topk leaves their order unspecified; here equal keys go to the lower index
// (block index at level one, position at level two).  NaN scores count as -inf.
//
// One CTA of 1024 threads per query row.  Values become order-preserving uint32 keys (0 =
// not selectable); a 3-pass radix select over 12-, 10- and 10-bit digits (shared-memory
// histograms scanned by the whole CTA) finds the K-th largest key, and one ordered pass keeps
// the keys above it plus the lowest-index ties, writing ascending indices (-1 padded).  Level
// one holds the row's block keys in shared memory (up to NB_MAX blocks).  Level two with a
// block list gathers the listed blocks' scores into shared memory once (up to GK_MAX keys)
// and selects there; with a bool mask, or a list too long for that, it reads the score row
// from global memory in every pass.
#include "common.cuh"

namespace mzb {
namespace cand {

constexpr int NT = 1024;
constexpr int NW = NT / 32;
constexpr int NB_MAX = 16384;  // blocks per row (level-one keys, level-two bitmap)

// order-preserving float -> uint32 (larger value, larger key); -inf and NaN -> 0; -0 and +0
// get the same key (they compare equal, so they are a tie)
__device__ __forceinline__ uint32_t fkey(float x) {
  if (!(x > -INFINITY)) return 0u;
  uint32_t u = __float_as_uint(x);
  if (u == 0x80000000u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
constexpr uint32_t KEY_POS_INF = 0xFF800000u;  // fkey(+inf)

constexpr int NBIN = 4096;  // first radix digit: 12 bits (sign, exponent, 3 mantissa bits)

struct Smem {
  int hist[NBIN];
  int red[NW + 2];
  int wsum[NW];
  uint32_t bits[NB_MAX / 32];  // level one: kept blocks; level two: candidate blocks
};

__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ int block_sum(int v, Smem& sm) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  v = warp_sum(v);
  if (lane == 0) sm.red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int t = lane < NW ? sm.red[lane] : 0;
    t = warp_sum(t);
    if (lane == 0) sm.red[NW] = t;
  }
  __syncthreads();
  const int r = sm.red[NW];
  __syncthreads();
  return r;
}

// Exclusive prefix count of a per-thread flag over the CTA in thread order; returns the total.
__device__ int block_scan(bool f, int& prefix, Smem& sm) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t b = __ballot_sync(0xffffffffu, f);
  if (lane == 0) sm.wsum[warp] = __popc(b);
  __syncthreads();
  if (warp == 0) {
    const int c = lane < NW ? sm.wsum[lane] : 0;
    int inc = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += y;
    }
    if (lane < NW) sm.wsum[lane] = inc - c;
    if (lane == 31) sm.red[NW + 1] = inc;
  }
  __syncthreads();
  prefix = sm.wsum[warp] + __popc(b & ((1u << lane) - 1u));
  const int total = sm.red[NW + 1];
  __syncthreads();
  return total;
}

// Exclusive prefix counts of two per-thread flags in one CTA scan (the counts share an int
// as two 16-bit halves: a tile holds at most 1024 of each); totals through t0 / t1.
__device__ void block_scan2(bool f0, bool f1, int& p0, int& p1, int& t0, int& t1, Smem& sm) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t b0 = __ballot_sync(0xffffffffu, f0), b1 = __ballot_sync(0xffffffffu, f1);
  const uint32_t below = (1u << lane) - 1u;
  if (lane == 0) sm.wsum[warp] = __popc(b0) | (__popc(b1) << 16);
  __syncthreads();
  if (warp == 0) {
    const int c = lane < NW ? sm.wsum[lane] : 0;
    int inc = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += y;
    }
    if (lane < NW) sm.wsum[lane] = inc - c;
    if (lane == 31) sm.red[NW + 1] = inc;
  }
  __syncthreads();
  const int base = sm.wsum[warp], tot = sm.red[NW + 1];
  p0 = (base & 0xFFFF) + __popc(b0 & below);
  p1 = (base >> 16) + __popc(b1 & below);
  t0 = tot & 0xFFFF;
  t1 = tot >> 16;
  __syncthreads();
}

struct Sel {
  uint32_t kth;  // keep keys > kth ...
  int ties;      // ... and the first `ties` keys == kth in index order
  bool all;      // every selectable key fits: keep all keys != 0
};

// Exclusive prefix sum of a per-thread count over the CTA in thread order; returns the total.
__device__ int block_excl_sum(int v, int& prefix, Smem& sm) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) sm.wsum[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const int c = lane < NW ? sm.wsum[lane] : 0;
    int wi = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    if (lane < NW) sm.wsum[lane] = wi - c;
    if (lane == 31) sm.red[NW + 1] = wi;
  }
  __syncthreads();
  prefix = sm.wsum[warp] + inc - v;
  const int total = sm.red[NW + 1];
  __syncthreads();
  return total;
}

// K-th largest non-zero key of src.key(0..n) (K >= 1): three digits of 12, 10 and 10 bits.
// The 12-bit first digit spreads real scores (which share a handful of exponents) over many
// bins, so the shared-memory histogram atomics rarely collide.
template <class Src>
__device__ Sel radix_select(const Src& src, int n, int K, Smem& sm) {
  uint32_t prefix = 0u, pmask = 0u;
  int k = K;
#pragma unroll 1
  for (int pass = 0; pass < 3; ++pass) {
    const int shift = pass == 0 ? 20 : (pass == 1 ? 10 : 0);
    const uint32_t dmask = pass == 0 ? 0xFFFu : 0x3FFu;
    const int nbins = int(dmask) + 1, per = nbins / NT;  // bins per thread: 4, then 1
    for (int b = threadIdx.x; b < nbins; b += NT) sm.hist[b] = 0;
    __syncthreads();
    int cnt = 0;  // selectable keys (first pass)
    for (int i = threadIdx.x; i < n; i += NT) {
      const uint32_t key = src.key(i);
      if (key != 0u && (key & pmask) == prefix) {
        atomicAdd(&sm.hist[(key >> shift) & dmask], 1);
        ++cnt;
      }
    }
    __syncthreads();
    if (pass == 0 && block_sum(cnt, sm) <= K) return Sel{0u, 0, true};  // every selectable key fits
    // thread t owns bins nbins-1-t*per .. nbins-(t+1)*per (descending)
    int c[4], own = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      c[j] = j < per ? sm.hist[nbins - 1 - (threadIdx.x * per + j)] : 0;
      own += c[j];
    }
    int exc;
    block_excl_sum(own, exc, sm);
    if (exc < k && k <= exc + own) {  // exactly one thread: the bin holding the k-th key
      int acc = exc, bin = -1, above = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (bin < 0 && j < per && acc + c[j] >= k) {
          bin = nbins - 1 - (threadIdx.x * per + j);
          above = acc;
        }
        acc += c[j];
      }
      sm.red[0] = bin;
      sm.red[1] = above;
    }
    __syncthreads();
    prefix |= uint32_t(sm.red[0]) << shift;
    pmask |= dmask << shift;
    k -= sm.red[1];
    __syncthreads();
  }
  return Sel{prefix, k, false};
}

// Ordered pass: emit(rank, i) for every kept i, ranks ascending with i; returns the count.
template <class Src, class Emit>
__device__ int select_ordered(const Src& src, int n, const Sel& sel, Smem& sm, Emit emit) {
  int kept = 0, ties_before = 0;
  for (int t0 = 0; t0 < n; t0 += NT) {
    const int i = t0 + threadIdx.x;
    const uint32_t key = i < n ? src.key(i) : 0u;
    const bool gt = key != 0u && (sel.all || key > sel.kth);
    const bool eq = !sel.all && key != 0u && key == sel.kth;
    int pg, pe, tg, te;
    block_scan2(gt, eq, pg, pe, tg, te, sm);
    const int room = max(0, sel.ties - ties_before);  // ties still to take, lowest index first
    if (gt || (eq && pe < room)) emit(kept + pg + min(pe, room), i);
    kept += tg + min(te, room);
    ties_before += te;
  }
  return kept;
}

// ------------------------------------------------------------------ level one
struct BlockKeys {  // keys of the row's blocks, in shared memory
  const uint32_t* k;
  __device__ __forceinline__ uint32_t key(int i) const { return k[i]; }
};

__global__ void __launch_bounds__(NT) blocks_kernel(const float* __restrict__ logits, const int32_t* __restrict__ clens,
                                                    int32_t* __restrict__ blocks, uint8_t* __restrict__ mask, int T,
                                                    int bs, int nb, int topk_blocks, bool vec) {
  extern __shared__ __align__(16) uint8_t dsm[];
  __shared__ Smem sm;
  uint32_t* keys = reinterpret_cast<uint32_t*>(dsm);
  const long long row = blockIdx.x;
  const float* lrow = logits + row * T;
  const int clen = clens[row];
  const int last = clen >= 1 ? (clen - 1) / bs : -1;  // floor((clen - 1) / bs)
  for (int b = threadIdx.x; b < nb; b += NT) {
    const int t0 = b * bs, t1 = min(T, t0 + bs);
    float m = -INFINITY;  // fmaxf skips NaN
    if (vec) {  // host-checked: 16-byte aligned base, T and bs multiples of 4
      for (int t = t0; t < t1; t += 4) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(lrow + t));
        m = fmaxf(fmaxf(m, fmaxf(v.x, v.y)), fmaxf(v.z, v.w));
      }
    } else {
      for (int t = t0; t < t1; ++t) m = fmaxf(m, __ldg(lrow + t));
    }
    keys[b] = b == last ? KEY_POS_INF : fkey(m);
  }
  for (int w = threadIdx.x; w < (nb + 31) / 32; w += NT) sm.bits[w] = 0u;
  __syncthreads();
  const BlockKeys src{keys};
  const Sel sel = radix_select(src, nb, topk_blocks, sm);
  int32_t* brow = blocks + row * topk_blocks;
  const int kept = select_ordered(src, nb, sel, sm, [&](int r, int i) {
    brow[r] = i;
    atomicOr(&sm.bits[i >> 5], 1u << (i & 31));
  });
  for (int r = kept + threadIdx.x; r < topk_blocks; r += NT) brow[r] = -1;
  if (mask) {
    __syncthreads();
    uint8_t* mrow = mask + row * T;
    for (int t = threadIdx.x; t < T; t += NT) {
      const int b = t / bs;
      mrow[t] = uint8_t((sm.bits[b >> 5] >> (b & 31)) & 1u);
    }
  }
}

// ------------------------------------------------------------------ level two
struct MaskedScores {  // score of position i if it is a candidate, else not selectable
  const float* s;
  const uint8_t* m;       // bool mask row, or null
  const uint32_t* bits;   // candidate-block bitmap (when m is null)
  int bs;
  __device__ __forceinline__ uint32_t key(int i) const {
    bool c;
    if (m) {
      c = m[i] != 0;
    } else {
      const int b = i / bs;
      c = (bits[b >> 5] >> (b & 31)) & 1u;
    }
    return c ? fkey(__ldg(s + i)) : 0u;
  }
};

__global__ void __launch_bounds__(NT) topk_kernel(const float* __restrict__ scores, const int32_t* __restrict__ blocks,
                                                  const uint8_t* __restrict__ mask, int32_t* __restrict__ out, int T,
                                                  int bs, int nblk, int topk) {
  __shared__ Smem sm;
  const long long row = blockIdx.x;
  if (!mask) {
    const int nb = (T + bs - 1) / bs;
    for (int w = threadIdx.x; w < (nb + 31) / 32; w += NT) sm.bits[w] = 0u;
    __syncthreads();
    const int32_t* brow = blocks + row * nblk;
    for (int j = threadIdx.x; j < nblk; j += NT) {
      const int b = brow[j];
      if (b >= 0 && b < nb) atomicOr(&sm.bits[b >> 5], 1u << (b & 31));
    }
    __syncthreads();
  }
  const MaskedScores src{scores + row * T, mask ? mask + row * T : nullptr, sm.bits, bs};
  const Sel sel = radix_select(src, T, topk, sm);
  int32_t* orow = out + row * topk;
  const int kept = select_ordered(src, T, sel, sm, [&](int r, int i) { orow[r] = i; });
  for (int r = kept + threadIdx.x; r < topk; r += NT) orow[r] = -1;
}

// Level two from a block list, gathered: the candidate blocks (ascending, duplicates and
// out-of-range entries dropped) are read once into shared memory as keys, in position order,
// so the radix passes and the ordered pass never touch global memory again.
constexpr int GK_MAX = 16384;   // gathered keys per row (64 KB)
constexpr int GB_MAX = 4096;    // gathered blocks per row

struct SmemKeys {
  const uint32_t* k;
  __device__ __forceinline__ uint32_t key(int i) const { return k[i]; }
};

__global__ void __launch_bounds__(NT) topk_gather_kernel(const float* __restrict__ scores,
                                                         const int32_t* __restrict__ blocks, int32_t* __restrict__ out,
                                                         int T, int bs, int nblk, int topk) {
  extern __shared__ __align__(16) uint8_t dsm[];
  __shared__ Smem sm;
  uint32_t* keys = reinterpret_cast<uint32_t*>(dsm);
  int32_t* blist = reinterpret_cast<int32_t*>(dsm + GK_MAX * 4);
  const long long row = blockIdx.x;
  const float* srow = scores + row * T;
  const int nb = (T + bs - 1) / bs;
  for (int w = threadIdx.x; w < (nb + 31) / 32; w += NT) sm.bits[w] = 0u;
  __syncthreads();
  const int32_t* brow = blocks + row * nblk;
  for (int j = threadIdx.x; j < nblk; j += NT) {
    const int b = brow[j];
    if (b >= 0 && b < nb) atomicOr(&sm.bits[b >> 5], 1u << (b & 31));
  }
  __syncthreads();
  // ascending list of the set blocks (the caller guarantees at most GB_MAX of them)
  int nsel = 0;
  for (int b0 = 0; b0 < nb; b0 += NT) {
    const int b = b0 + threadIdx.x;
    const bool set = b < nb && ((sm.bits[b >> 5] >> (b & 31)) & 1u);
    int r;
    const int tot = block_scan(set, r, sm);
    if (set) blist[nsel + r] = b;
    nsel += tot;
  }
  __syncthreads();
  const int n = nsel * bs;
  for (int j = threadIdx.x; j < n; j += NT) {
    const int s = j / bs, t = blist[s] * bs + (j - s * bs);
    keys[j] = t < T ? fkey(__ldg(srow + t)) : 0u;
  }
  __syncthreads();
  const SmemKeys src{keys};
  const Sel sel = radix_select(src, n, topk, sm);
  int32_t* orow = out + row * topk;
  const int kept = select_ordered(src, n, sel, sm, [&](int r, int j) {
    const int s = j / bs;
    orow[r] = blist[s] * bs + (j - s * bs);
  });
  for (int r = kept + threadIdx.x; r < topk; r += NT) orow[r] = -1;
}

}  // namespace cand
}  // namespace mzb

using namespace mzb;

extern "C" int mzb_candidate_blocks(const float* logits, const int32_t* compress_lens, int32_t* blocks, uint8_t* mask,
                                    int64_t rows, int64_t T, int block_size, int topk_blocks, void* stream) {
  MZB_REQUIRE(rows >= 0 && T >= 0 && rows < (int64_t(1) << 31), MZB_ERR_SHAPE,
              "candidate_blocks: bad sizes rows=%lld T=%lld", (long long)rows, (long long)T);
  MZB_REQUIRE(block_size >= 1 && topk_blocks >= 1, MZB_ERR_SHAPE,
              "candidate_blocks: block_size=%d and topk_blocks=%d must be >= 1", block_size, topk_blocks);
  const int64_t nb = (T + block_size - 1) / block_size;
  MZB_REQUIRE(nb <= cand::NB_MAX, MZB_ERR_UNSUPPORTED,
              "candidate_blocks: %lld blocks per row exceed the %d this kernel holds on chip", (long long)nb,
              cand::NB_MAX);
  MZB_REQUIRE(rows == 0 || (logits && compress_lens && blocks), MZB_ERR_SHAPE,
              "candidate_blocks: logits, compress_lens and blocks are required");
  if (rows == 0) return MZB_OK;
  const size_t dyn = size_t(nb > 0 ? nb : 1) * 4;
  if (cudaFuncSetAttribute(cand::blocks_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(dyn)) != cudaSuccess)
    return launch_status("candidate_blocks(smem attr)");
  const bool vec = (T % 4) == 0 && (block_size % 4) == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0;
  cand::blocks_kernel<<<unsigned(rows), cand::NT, dyn, static_cast<cudaStream_t>(stream)>>>(
      logits, compress_lens, blocks, mask, int(T), block_size, int(nb), topk_blocks, vec);
  return launch_status("candidate_blocks");
}

extern "C" int mzb_candidate_topk(const float* scores, const int32_t* blocks, const uint8_t* mask, int64_t rows,
                                  int64_t T, int block_size, int nblk, int topk, int32_t* out, void* stream) {
  MZB_REQUIRE(rows >= 0 && T >= 0 && rows < (int64_t(1) << 31) && T < (int64_t(1) << 31), MZB_ERR_SHAPE,
              "candidate_topk: bad sizes rows=%lld T=%lld", (long long)rows, (long long)T);
  MZB_REQUIRE(topk >= 1, MZB_ERR_SHAPE, "candidate_topk: topk=%d must be >= 1", topk);
  MZB_REQUIRE((blocks == nullptr) != (mask == nullptr), MZB_ERR_SHAPE,
              "candidate_topk: pass exactly one of a block list and a bool mask");
  if (blocks) {
    MZB_REQUIRE(block_size >= 1 && nblk >= 1, MZB_ERR_SHAPE, "candidate_topk: block_size=%d nblk=%d", block_size,
                nblk);
    MZB_REQUIRE((T + block_size - 1) / block_size <= cand::NB_MAX, MZB_ERR_UNSUPPORTED,
                "candidate_topk: more than %d blocks per row", cand::NB_MAX);
  }
  MZB_REQUIRE(rows == 0 || (scores && out), MZB_ERR_SHAPE, "candidate_topk: scores and out are required");
  if (rows == 0) return MZB_OK;
  const int64_t nb = blocks ? (T + block_size - 1) / block_size : 0;
  const int64_t gblocks = nb < nblk ? nb : nblk;  // distinct in-range blocks a row can list
  if (blocks && gblocks <= cand::GB_MAX && gblocks * block_size <= cand::GK_MAX) {
    const int dyn = cand::GK_MAX * 4 + cand::GB_MAX * 4;
    if (cudaFuncSetAttribute(cand::topk_gather_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn) !=
        cudaSuccess)
      return launch_status("candidate_topk(smem attr)");
    cand::topk_gather_kernel<<<unsigned(rows), cand::NT, dyn, static_cast<cudaStream_t>(stream)>>>(
        scores, blocks, out, int(T), block_size, nblk, topk);
    return launch_status("candidate_topk");
  }
  cand::topk_kernel<<<unsigned(rows), cand::NT, 0, static_cast<cudaStream_t>(stream)>>>(
      scores, blocks, mask, out, int(T), blocks ? block_size : 1, blocks ? nblk : 0, topk);
  return launch_status("candidate_topk");
}
