/*
 * mzb200.h -- C ABI of libmzb200.so, the B200 (sm_100a) kernels behind mzoo_b200.
 *
 * Every entry point takes raw device pointers, shapes and scalar parameters plus a
 * CUDA stream (as void*, NULL = legacy default stream), launches asynchronously on that
 * stream and returns MZB_OK (0) or a negative MZB_ERR_* code; mzb_last_error() then
 * holds a message.  The library never allocates or frees caller memory: outputs and
 * workspaces are passed in.  All tensors are dense row-major (C-contiguous) unless a
 * stride argument says otherwise.  Calls are re-entrant; a call only touches the
 * memory its arguments name.
 *
 * Each declaration cites the reference function (pmonad/mzoo, path within the project)
 * whose arithmetic it replaces.  The Python host layer (mzoo_b200/) mirrors the
 * reference's call signatures on top of these.
 */
#ifndef MZB200_H_
#define MZB200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MZB_VERSION 1

#if defined(__GNUC__)
#define MZB_API __attribute__((visibility("default")))
#else
#define MZB_API
#endif

/* status codes */
#define MZB_OK 0
#define MZB_ERR_SHAPE (-1)       /* shape / size / divisibility violated */
#define MZB_ERR_UNSUPPORTED (-2) /* dtype, head dim or mode not built */
#define MZB_ERR_LAUNCH (-3)      /* CUDA launch or attribute failure */
#define MZB_ERR_TIMEOUT (-4)     /* a bounded device-side wait gave up */
#define MZB_ERR_ALIGN (-5)       /* pointer not 16-byte aligned where required */
#define MZB_ERR_BOUND (-6)       /* a device-side error-bound check failed */

/* element type codes */
#define MZB_F32 0
#define MZB_BF16 1
#define MZB_F16 2
#define MZB_E4M3 3 /* float8_e4m3fn codes (uint8) */

MZB_API const char* mzb_last_error(void);
MZB_API int mzb_version(void);

/* ------------------------------------------------------------------ fake quant
 * y = dequant(quant(x)) along the last axis in blocks of `block_size`; x, y are
 * [rows, n] of element type `dtype` (y may alias x).  n % block_size must be 0 (mzoo
 * returns x unchanged otherwise; the Python layer does that without calling here).
 *
 * mzb_fq_fp4 -- replaces `_fake_quant_fp4_block(x, block_size, e4m3_scales)`
 *               (src/mzoo/archs/owlet1/quant.py:49, = archs/dsv4/modeling_deepseek_v41.py:383).
 *   rule 0: ue8m0 scale 2^ceil(log2(max(amax, 6*2^-126)/6))          (e4m3_scales=False)
 *   rule 1: e4m3 scale e4m3(max(amax, 6*2^-9)/6)                      (e4m3_scales=True)
 *   rule 2: OCP MX e8m0 scale 2^(floor(log2 amax) - 2), saturating    (no mzoo counterpart)
 * mzb_fq_fp8 -- replaces `_fake_quant_fp8_block(x, block_size)` (quant.py:72,
 *               = modeling_deepseek_v41.py:616).
 *   rule 0: ue8m0 scale 2^ceil(log2(max(amax, 1e-4)/448))
 *   rule 1: absmax scale amax/448 per tile (1 if amax == 0)          (no mzoo counterpart)
 */
MZB_API int mzb_fq_fp4(const void* x, void* y, int64_t rows, int64_t n, int dtype, int block_size, int rule,
               void* stream);
MZB_API int mzb_fq_fp8(const void* x, void* y, int64_t rows, int64_t n, int dtype, int block_size, int rule,
               void* stream);

/* ------------------------------------------------------------------ lightning indexer
 * mzb_indexer_scores -- replaces `indexer.fwd.fwd` / kernel `index_score`
 *   (src/mzoo/layers/attn/indexer/fwd.py:48-132; golden_ref.py:213 `indexer_scores`).
 *   scores[b,s,t] = scale * sk[b,t] * sum_h w[b,s,h]*sq[b,s,h] * relu(q[b,s,h,:].k[b,t,:])
 *   for t < (q_offset + s + 1) / ratio, else -inf (q_offset = 0 is the reference's
 *   prefill positions 0..S-1; the model uses absolute positions,
 *   archs/dsv4/modeling_deepseek_v41.py:555).  q [B,S,Hi,Di], k [B,T,Di] are bf16
 *   (dtype MZB_BF16; sq, sk may be NULL) or e4m3 codes (MZB_E4M3; sq [B,S,Hi], sk [B,T]
 *   fp32 required); w [B,S,Hi] fp32; scores [B,S,T] fp32.  Hi % 16 == 0 (the host pads
 *   smaller head counts with zero weights); Di in {32,64,96,128,256} (bf16) or
 *   {64,128} (e4m3).  q_pos [B*S] int32 (may be NULL) gives each query's absolute position
 *   (decode: one query per sequence at seq_len-1) and overrides q_offset + s.  write_tail = 0 skips the -inf fill of keys past the block's causal
 *   frontier (the top-k path never reads them).  `err` (device int, may be NULL)
 *   receives a non-zero code if a bounded device wait gives up.
 * mzb_indexer_topk -- replaces `indexer.attn.attn` (indexer/attn.py:67-81: torch.topk on
 *   the score matrix, -inf -> -1) and `golden_ref.topk_indices` (golden_ref.py:230).
 *   Reads `scores` from mzb_indexer_scores (same arguments) and writes out [B,S,topk]
 *   int32: the top-k keys of the exact fp64 canonical score (ties to the lower index),
 *   ascending, -1 padded when fewer than topk keys are visible.  kbmax_ws is a float
 *   workspace of B*16 + B*S entries (key and query-row error-bound factors).  eps bounds the relative error of the fp32 scores (see
 *   indexer.cu); *err = MZB_ERR_BOUND if the bound leaves too many candidates.
 * Paged keys (both entry points; a paged KV cache for decode, no counterpart in the
 *   reference): with k_page_table != NULL, k holds k_pages pages of 64 key rows
 *   [k_pages, 64, Di] and sk [k_pages, 64]; key t of batch b is row t % 64 of page
 *   k_page_table[b * k_ptw + t / 64]; T <= 64 * k_ptw.  Entries past a sequence's visible
 *   keys are never used (ids outside [0, k_pages) are clamped).  NULL: dense k [B,T,Di].
 */
MZB_API int mzb_indexer_scores(const void* q, const void* k, const float* w, const float* sq, const float* sk,
                               const int32_t* q_pos, float* scores, int64_t B, int64_t S, int64_t T, int Hi, int Di,
                               int dtype, int ratio, int64_t q_offset, float scale, int write_tail,
                               const int32_t* k_page_table, int k_ptw, int64_t k_pages, int* err, void* stream);
/* mzb_indexer_bwd -- replaces `indexer.bwd.bwd` / kernel `index_score_bwd`
 *   (src/mzoo/layers/attn/indexer/bwd.py:38-133): with r = q.k recomputed and d = dl on the
 *   group-causal visible keys (masked entries ignored whatever they hold), scale given:
 *   dw = sum_t relu(r)*scale*d (fp32), dr = d*w*scale*[r > 0], dq = sum_t dr k (bf16),
 *   dk = sum_{s,h} dr q (bf16; deterministic here, fp32 atomics in the reference).
 *   q bf16 [B,S,Hi,Di], k bf16 [B,T,Di], w / dl fp32 [B,S,Hi] / [B,S,T]; Hi divides 256 and is a
 *   multiple of 16 (the host pads with zero weights); Di in {64, 128}; T >= 1.
 */
MZB_API int mzb_indexer_bwd(const void* q, const void* k, const float* w, const float* dl, void* dq, void* dk,
                            float* dw, int64_t B, int64_t S, int64_t T, int Hi, int Di, int ratio, int64_t q_offset,
                            float scale, int* err, void* stream);
MZB_API int mzb_indexer_topk(const float* scores, const void* q, const void* k, const float* w, const float* sq,
                             const float* sk, const int32_t* q_pos, float* kbmax_ws, int32_t* out, int64_t B,
                             int64_t S, int64_t T, int Hi, int Di, int dtype, int ratio, int64_t q_offset, float scale,
                             int topk, float eps, const int32_t* k_page_table, int k_ptw, int64_t k_pages, int* err,
                             void* stream);

/* ------------------------------------------------------------------ shared-latent MQA (D <= 256)
 * mzb_attn_fwd -- replaces `swa_attn.fwd` / kernel `flashattn` (src/mzoo/layers/attn/
 *   swa_attn/fwd.py:55-208) and `csa2_attn.fwd` (csa2_attn/fwd.py:70-286).
 *   q bf16 [B, S*H, D] (BSHD packed rows), kv bf16 [B, S, D] (K == V latent), v bf16
 *   [B, S, D] or NULL (= kv; a distinct v only without gathered entries), main_kv bf16
 *   [B, G, D] + indices int32 [B, S, topk] or NULL (window-only), sinks fp32 [H] or NULL.
 *   Row (t, h) attends keys t-window < k <= t plus main_kv[indices[t, :]] (out-of-range =
 *   empty, duplicates count twice); one softmax (+ sink column in the denominator).
 *   o bf16 [B, S*H, D]; lse fp32 [B, S*H] (natural log, packed token-major).
 *   H must divide 128; D in {64, 128, 256}.
 */
MZB_API int mzb_attn_fwd(const void* q, const void* kv, const void* v, const void* main_kv, const int32_t* indices,
                         const float* sinks, void* o, float* lse, int64_t B, int64_t S, int H, int D, int window,
                         int64_t G, int topk, float softmax_scale, int* err, void* stream);

/* mzb_attn_bwd -- replaces `swa_attn.bwd` (swa_attn/bwd.py:79-119: preprocess, bwd_kv,
 *   bwd_dq) and `csa2_attn.bwd` (csa2_attn/bwd.py:67-130, bwd_dq.py:60-187).  Inputs as
 *   mzb_attn_fwd plus o, lse (packed [B, S*H]) and dout bf16 [B, S*H, D].  Outputs: dq bf16
 *   [B, S*H, D]; dk bf16 [B, S, D] (= dK + dV when v is NULL, i.e. K == V); dv bf16 [B, S, D]
 *   (separate v only); dmain_f32 fp32 [B, G, D] accumulated with atomics (caller zeroes it;
 *   not bit-reproducible, as in the reference).  delta_ws, lse2_ws: fp32 workspaces of
 *   B * ceil(S*H/128)*128 entries; dkv_part_ws: splits * B * S * 2 * D fp32 (the split
 *   partials of dK/dV, summed in a fixed order: dq / dk / dv are deterministic).  D in {64, 128}.  dsinks is a host-side reduction of lse
 *   and delta (as in the reference).
 */
MZB_API int mzb_attn_bwd(const void* q, const void* kv, const void* v, const void* main_kv, const int32_t* indices,
                         const void* o, const float* lse, const void* dout, void* dq, void* dk, void* dv,
                         float* dmain_f32, float* delta_ws, float* lse2_ws, float* dkv_part_ws, int splits,
                         int64_t B, int64_t S, int H, int D, int window, int64_t G, int topk, float softmax_scale,
                         int* err, void* stream);
/* Query-loop split count mzb_attn_bwd expects for these sizes (the key-owner kernel's
 * partial sums; dkv_part_ws holds splits * B * S * 2 * D floats).  Host-only, no launch. */
MZB_API int mzb_attn_bwd_splits(int64_t B, int64_t S, int H, int window);

/* ------------------------------------------------------------------ sparse latent attention
 * mzb_sparse_mla_fwd -- the 576/512 FP8-latent form of `csa2_attn.fwd` / kernel `flashattn`
 *   (src/mzoo/layers/attn/csa2_attn/fwd.py:70-286; golden_ref.py:149-168 level "sparse"),
 *   prefill and paged decode.  Per query token tk (sequence b = tk / tok_per_seq, absolute
 *   position q_pos[tk]): one softmax over the raw-latent window [q_pos-window+1, q_pos] and
 *   the compressed entries indices[tk, 0..topk) (-1 or >= the sequence's compressed length
 *   = empty; duplicates count twice), logits = softmax_scale * q . k (576 channels),
 *   o = P V with V = the first 512 channels.
 *   q bf16 [n_tok, 128, 576]; KV rows of 672 B ([0,512) e4m3, [512,544) 8 fp32 scales per
 *   64 channels, [544,672) 64 bf16 rope) in kv_raw / kv_cmp: dense [B, raw_len] /
 *   [B, cmp_len] rows when the page table is NULL, else 64-row pages addressed through
 *   raw_page_table [B, raw_ptw] / cmp_page_table [B, cmp_ptw].  cmp_lens [B] (or NULL =
 *   cmp_len) bounds valid compressed indices.  Outputs o bf16 [n_tok, 128, 512] and
 *   lse fp32 [n_tok, 128] (natural log).  slots_ws: int32 workspace [n_tok].
 *   splits: key-range splits per token (1, or mzb_sparse_mla_splits(n_tok) for calls with
 *   few tokens such as decode); with splits > 1, part_ws holds splits * n_tok * 128 * 513
 *   floats (each split's normalised output and lse, merged by a second kernel).
 */
MZB_API int mzb_sparse_mla_fwd(const void* q, const void* kv_raw, const void* kv_cmp, const int32_t* indices,
                               const int32_t* q_pos, const int32_t* raw_page_table, const int32_t* cmp_page_table,
                               const int32_t* cmp_lens, int32_t* slots_ws, void* o, float* lse, int64_t n_tok,
                               int tok_per_seq, int topk, int window, int64_t raw_len, int64_t cmp_len, int raw_ptw,
                               int cmp_ptw, float softmax_scale, int splits, float* part_ws, int* err, void* stream);
/* Key-range splits per token mzb_sparse_mla_fwd should use for n_tok tokens (1 unless the
 * tokens alone leave SM pairs idle).  Host-only, no launch. */
MZB_API int mzb_sparse_mla_splits(int64_t n_tok);

/* mzb_sparse_mla_fwd_noalloc -- no counterpart in the reference.  Same arguments and
 *   result as mzb_sparse_mla_fwd minus `slots_ws`, `splits` and `part_ws` (one split): for callers that cannot allocate device
 *   memory at launch time (a serving engine whose free HBM all belongs to its KV-cache
 *   pool, or a host whose own memory manager must not be bypassed).  The workspace comes
 *   from a fixed 65536-entry (256 KB) array inside the library, present on every GPU that
 *   loads it until the process exits; n_tok above 65536 is rejected with MZB_ERR_SHAPE.
 *   Calls share that array: two calls that overlap on the GPU race.  The first call on a
 *   device resolves the array's address; make it before any stream capture.
 */
MZB_API int mzb_sparse_mla_fwd_noalloc(const void* q, const void* kv_raw, const void* kv_cmp, const int32_t* indices,
                                       const int32_t* q_pos, const int32_t* raw_page_table,
                                       const int32_t* cmp_page_table, const int32_t* cmp_lens, void* o, float* lse,
                                       int64_t n_tok, int tok_per_seq, int topk, int window, int64_t raw_len,
                                       int64_t cmp_len, int raw_ptw, int cmp_ptw, float softmax_scale, int* err,
                                       void* stream);

/* mzb_candidate_blocks -- replaces `select_candidate_blocks`
 *   (src/mzoo/archs/dsv4/modeling_deepseek_v41.py:427-454, identical in
 *   archs/owlet1/indexer.py:14-41), level one of the two-level indexer top-k.  logits fp32
 *   [rows, T] with unreachable positions at -inf; compress_lens int32 [rows] (the query's
 *   visible compressed length).  Block score = max of block_size consecutive logits; the block
 *   (compress_len - 1) / block_size is pinned in; the top topk_blocks blocks with a score
 *   above -inf are kept (ties to the lower block index).  blocks int32 [rows, topk_blocks]:
 *   kept block indices ascending, -1 padded; mask uint8 [rows, T] (may be NULL): 1 where the
 *   position's block is kept -- the reference's bool mask.  At most 16384 blocks per row.
 * mzb_candidate_topk -- level two (modeling_deepseek_v41.py:566-578: scores outside the
 *   candidates set to -inf, top-k, -inf picks dropped).  scores fp32 [rows, T]; candidates
 *   as a block list int32 [rows, nblk] of block_size-position blocks (-1 = none; at most
 *   16384 blocks per row) or as a uint8 mask [rows, T] -- exactly one of the two.  out int32
 *   [rows, topk]: the candidate positions with the topk largest scores above -inf (ties to
 *   the lower position), ascending, -1 padded.  NaN scores count as -inf in both calls.
 */
MZB_API int mzb_candidate_blocks(const float* logits, const int32_t* compress_lens, int32_t* blocks, uint8_t* mask,
                                 int64_t rows, int64_t T, int block_size, int topk_blocks, void* stream);
MZB_API int mzb_candidate_topk(const float* scores, const int32_t* blocks, const uint8_t* mask, int64_t rows,
                               int64_t T, int block_size, int nblk, int topk, int32_t* out, void* stream);

/* mzb_compress -- replaces the elementwise part of `DeepseekV41Compressor.forward`
 *   (src/mzoo/archs/dsv4/modeling_deepseek_v41.py:318-340) and of the compressed-cache
 *   write (:745-753): per group of `ratio` tokens, latent = sum_r kv_r softmax_r(gate_r) (fp32),
 *   cast to bf16, RMSNorm (:58-63; x * rsqrt(mean(x^2) + eps) -> bf16, times the bf16
 *   weight) -> `latent` bf16 [B, G, D] (the pre-RoPE latent); optionally `cache` bf16
 *   [B, G, D] = _fake_quant_fp4_block(apply_rotary_pos_emb(latent, cos, sin), 16,
 *   e4m3_scales=True) (:405-425, :753).  kv, gate fp32 [B, G*ratio, D] (the projections;
 *   gate NULL at ratio 1, where the latent is kv itself); norm_w bf16 [D]; cos, sin fp32
 *   [B, G, rope_dim/2] (needed with `cache`).  D a multiple of 16, at most 4096; rope_dim a
 *   multiple of 4; kv / gate 16-byte aligned, the bf16 buffers 8-byte aligned.
 */
MZB_API int mzb_compress(const float* kv, const float* gate, const void* norm_w, const float* cos_v,
                         const float* sin_v, void* latent, void* cache, int64_t B, int64_t G, int ratio, int D,
                         int rope_dim, float eps, void* stream);

/* ------------------------------------------------------------------ RMSNorm + RoPE prologue
 * mzb_norm_rope_fwd -- replaces `qk_norm_rope` / kernel `make_fwd`
 *   (src/mzoo/layers/attn/norm_rope.py:52-110, 183-230; contract `qk_norm_rope_eager` :37-44 =
 *   archs/dsv4/modeling_deepseek_v41.py:49-63 RMSNorm then :405-425 apply_rotary_pos_emb).
 *   x, out bf16 [rows, dim] (rows = B*S*H, row r of token r / heads), w bf16 [dim], cos / sin
 *   fp32 [rows / heads, rope_dim / 2] (NULL when rope_dim == 0); rstd fp32 [rows] (saved for
 *   the backward).  dim in {64, 96, 128, 256}; rope_dim even; x, w, out 16-byte aligned.
 * mzb_norm_rope_bwd -- replaces kernel `make_bwd` (norm_rope.py:113-180): dx bf16 [rows, dim],
 *   dw fp32 [dim] = sum over rows, summed in a fixed order through dw_part, a float workspace
 *   of parts * dim entries with parts >= mzb_norm_rope_bwd_parts(rows, dim).
 */
MZB_API int mzb_norm_rope_fwd(const void* x, const void* w, const float* cos, const float* sin, void* out,
                              float* rstd, int64_t rows, int heads, int dim, int rope_dim, float eps, void* stream);
MZB_API int mzb_norm_rope_bwd_parts(int64_t rows, int dim);
MZB_API int mzb_norm_rope_bwd(const void* x, const void* dy, const void* w, const float* rstd, const float* cos,
                              const float* sin, void* dx, float* dw_part, float* dw, int64_t rows, int heads,
                              int dim, int rope_dim, int parts, void* stream);

/* ------------------------------------------------------------------ quantised KV caches
 * The cache formats of the DeepSeek-V4.1 attention (src/mzoo/layers/attn/csa_attn/README.md:
 * 215-235, tickets/0010-csa2-fp-cache.md), bit-identical to the model's fake quantisers
 * (archs/dsv4/modeling_deepseek_v41.py:359-402, :668-683): unpack(pack(x)) equals
 * `_fake_quant_fp8_block(x, 32)` / `_fake_quant_fp4_block(x, 16, e4m3_scales=True)`.
 * mzb_kv_pack_fp8   -- window cache: x bf16 [rows, D] -> e4m3 codes [rows, D] + ue8m0 scale
 *                      bytes [rows, D/32] (scale = 2^(byte - 127)); D % 32 == 0.
 * mzb_kv_unpack_fp8 -- codes + scales -> bf16 [rows, D].
 * mzb_kv_pack_fp4   -- main cache: x bf16 [rows, D] -> e2m1 codes two per byte (low nibble =
 *                      even channel) [rows, D/2] + e4m3 scale bytes [rows, D/16]; D % 16 == 0.
 * mzb_kv_unpack_fp4 -- packed codes + scales -> bf16 [rows, D].
 */
MZB_API int mzb_kv_pack_fp8(const void* x, uint8_t* codes, uint8_t* scales, int64_t rows, int D, void* stream);
MZB_API int mzb_kv_unpack_fp8(const uint8_t* codes, const uint8_t* scales, void* out, int64_t rows, int D,
                              void* stream);
MZB_API int mzb_kv_pack_fp4(const void* x, uint8_t* codes, uint8_t* scales, int64_t rows, int D, void* stream);
MZB_API int mzb_kv_unpack_fp4(const uint8_t* codes, const uint8_t* scales, void* out, int64_t rows, int D,
                              void* stream);

/* Self-test of the bounded device waits (no counterpart in the reference: it checks this
 * library's own failure path).  One thread waits on an mbarrier nothing arrives on; after
 * limit_ns (<= 2e9) the wait gives up, writes 901 (scope 0: CTA-scope wait) or 902
 * (scope 1: cluster-scope wait) into *err and the kernel returns normally. */
MZB_API int mzb_selftest_bounded_wait(int64_t limit_ns, int scope, int* err, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MZB200_H_ */
