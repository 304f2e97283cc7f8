/*
 * srswa.h -- C ABI of the B200 (sm_100a) SR-SWA hot-path library (libsrswa.so).
 *
 * SR-SWA = Sparse-Reference Sliding-Window Attention of Unlimited-OCR 2: every
 * query attends a token-level local window plus K remote key blocks chosen by
 * a single-head router.  This library implements the router (block summaries,
 * scores, top-M 1.5-entmax, top-K, centred log-prior bias), the fused
 * gather-attention forward/backward, and the paged decode attend with its
 * split-KV log-sum-exp merge.
 *
 * Conventions (all entry points):
 *   - pointers are device pointers; shapes/strides are int64 element counts;
 *     the innermost (feature) dimension of every tensor is contiguous;
 *   - work is enqueued on `stream`; nothing blocks the host; nothing allocates:
 *     any scratch memory is passed in by the caller (size from the matching
 *     *_workspace_size query);
 *   - return 0 on success, a negative SRSWA_E* code for invalid or unsupported
 *     arguments (nothing was launched), or a positive cudaError_t value.
 *
 * Reference citations are paths inside the reference project; "whl:" paths are
 * files inside its wheel sglang-0.5.20.dev10+g8d62f5fb9c-py3-none-any.whl.
 */
#ifndef SRSWA_H
#define SRSWA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define SRSWA_API __attribute__((visibility("default")))
#else
#define SRSWA_API
#endif

typedef struct CUstream_st* srswa_stream_t; /* == cudaStream_t */

/* element types */
enum { SRSWA_F32 = 0, SRSWA_BF16 = 1, SRSWA_F16 = 2, SRSWA_F8E4M3 = 3, SRSWA_F8E5M2 = 4 };
/* (the fp8 codes are accepted where an entry point says so: the decode /
 * prefill attend's K/V caches) */

/* negative status codes */
enum {
  SRSWA_OK = 0,
  SRSWA_EINVAL = -1,       /* bad pointer / negative size / inconsistent shape */
  SRSWA_EUNSUPPORTED = -2, /* valid but unsupported (head dim, block size, ...) */
  SRSWA_EALIGN = -3,       /* pointer or stride not 16-byte aligned where needed */
  SRSWA_EWORKSPACE = -4,   /* caller workspace too small */
  SRSWA_ETOOLARGE = -5     /* size above a compiled-in maximum */
};

/* A peer-memory exchange region (see "peer exchange" below); entry points
 * that take one accept NULL = no exchange.  ll selects the protocol: 0 =
 * payload + per-source flags, 1 = LL words (see below). */
typedef struct {
  void* const* regions;
  void* own_region;
  int64_t slot_bytes, rank, world;
  uint64_t* counter;
  uint32_t* tickets;
  int32_t* status;
  int64_t ll;
} srswa_peer;

/* Library version (major*10000 + minor*100 + patch) and status text. */
SRSWA_API int srswa_version(void);
SRSWA_API const char* srswa_status_string(int status);

/* ------------------------------------------------------------------ a1 --
 * head_cls block summaries k_bar of index keys, contiguous sequences.
 * idx_k [B,S,d] (strides sb, st; d contiguous) -> kbar [B,nblk,d] fp32
 * contiguous, nblk = ceil(S/block_size); chunk_valid [B,nblk] (optional,
 * 1 = block holds >= 1 token).
 * Replaces the head_cls branch of modeling_deepseekv2._block_scores_infer
 * (hf-model-code/modeling_deepseekv2.py:391-408) and Stage 0 of
 * DashAttention._block_scores_headcls (hf-model-code/dash_attention.py:1079-1119). */
SRSWA_API int srswa_kbar_contig(const void* idx_k, int dtype, int64_t sb, int64_t st, int64_t B,
                      int64_t S, int64_t d, int64_t block_size, const float* head_cls,
                      float* kbar, uint8_t* chunk_valid, srswa_stream_t stream);

/* head_cls summaries of pages of a paged index-key cache.
 * idx_cache [P, block_size, d] (strides s_page, s_tok); block_table [R, W]
 * int32 (row stride s_bt); seq_lens [R] int32.  Refreshes, for each request,
 * the summaries of its last `tail_pages` pages in use (all pages in use when
 * tail_pages <= 0) into kbar_cache [P, d] fp32 (row stride s_kbar).
 * Replaces KBarCache.put/refresh_tail + K11 _kbar_page_kernel
 * (whl:sglang/srt/layers/attention/unlimited_dash_ops/dash_stage0.py:106-150,
 *  route_triton.py:36-72, 681-726). */
SRSWA_API int srswa_kbar_paged(const void* idx_cache, int dtype, int64_t s_page, int64_t s_tok,
                     int64_t d, int64_t block_size, const int32_t* block_table, int64_t s_bt,
                     int64_t W, const int32_t* seq_lens, int64_t R, int64_t tail_pages,
                     const float* head_cls, float* kbar_cache, int64_t s_kbar,
                     srswa_stream_t stream);

/* k_bar of an explicit page plan: page pages[i] (int64) from its first tok[i]
 * tokens (int32); entries with tok[i] <= 0 store nothing (plan padding, other
 * requests' pages).  The plans are the reference's kbar_tail_plan /
 * kbar_all_plan outputs.  Replaces _kbar_page_kernel driven by a plan
 * (whl:.../unlimited_dash_ops/route_triton.py:36-72, 706-726). */
SRSWA_API int srswa_kbar_pages(const void* idx_cache, int dtype, int64_t s_page, int64_t s_tok, int64_t d,
                     int64_t block_size, const int64_t* pages, const int32_t* tok, int64_t n,
                     const float* head_cls, float* kbar_cache, int64_t s_kbar, srswa_stream_t stream);

/* --------------------------------------------------------------- a2+a4 --
 * Router parameters (the per-layer _infer_params dict of
 * configure_dash_inference, hf-model-code/modeling_deepseekv2.py:296-335). */
typedef struct {
  int64_t block_size;   /* BS */
  int64_t local_blocks; /* L: remote candidates are blocks c <= q_pos/BS - L */
  int64_t topk;         /* K: slots returned (the reference clamps to <= M) */
  int64_t topm;         /* M: entmax window (<= 0: whole row) */
  float idx_scale;      /* entmax input scale (dash_scaling_factor / sqrt(d)) */
  float prior_floor;    /* log-prior floor */
  float sigma;          /* bias divisor */
} srswa_route_params;

/* Fused router over a set of query rows.
 * Scores: z[n,c] = clamp(idx_q[n] . kbar_c / sqrt(d), +-1e4) for remote blocks
 * c <= q_pos[n]/BS - L that hold a token, SCORE_NEG (-1e9) elsewhere.  kbar_c
 * comes either from a contiguous kbar [B, nblk, d] (block_table == NULL; row n
 * belongs to batch n / rows_per_seq) or from a paged kbar cache [P, d] through
 * block_table [R, W] (row n belongs to request n / rows_per_seq, or to
 * row_seq[n] when row_seq [N] int32 is given: varlen prefill rows, which then
 * need q_pos).
 * q_pos [N] int64, or NULL to use seq_lens[r] - rows_per_seq + n % rows_per_seq.
 * seq_lens (NULL allowed when q_pos is given and blocks are contiguous) bounds
 * blocks holding tokens.  cand [N, nblk] uint8 (row stride s_cand, 0 = shared
 * row; NULL = all remote blocks) is the page-aware candidate domain.
 * Selection: _infer_route_select semantics (hf-model-code/modeling_deepseekv2.py:339-362):
 * top-M by x = cand ? z*idx_scale : -1e4, exact 1.5-entmax over those M,
 * first K slots, bias = (log max(p, floor) - mean_valid)/sigma.
 * Outputs (each optional, [N, K] row-major): topi64 (raw indices, score-desc),
 * topi32 (-1 on invalid slots: the serving layout), bias (0 on invalid),
 * valid (uint8); scores [N, nblk] fp32 (the _block_scores_infer output).
 * workspace: caller scratch of srswa_route_workspace_size(N, nblk, params,
 * cand != NULL) bytes: N*nblk*4 (one fp32 score per row and block) where the
 * rows may take the chunked score pass (>= 512 blocks, or too few rows to
 * give the row-packed kernel a CTA per SM), else 0.  Rows of one sequence
 * (prefill) take the tiled routers whenever they apply and then leave the
 * workspace unused.
 * Replaces _block_scores_infer + _infer_route_select (modeling_deepseekv2.py:339-430)
 * and route_decode_triton / route_prefill_triton
 * (whl:.../unlimited_dash_ops/route_triton.py:624-680, 729-847). */
SRSWA_API size_t srswa_route_workspace_size(int64_t N, int64_t nblk, int64_t d, srswa_route_params params,
                                            int has_cand);
SRSWA_API int srswa_route(const void* idx_q, int q_dtype, int64_t s_q, int64_t N, int64_t d,
                const float* kbar, int64_t s_kbar_b, int64_t s_kbar_c, int64_t nblk,
                const int32_t* block_table, int64_t s_bt, const int32_t* seq_lens,
                int64_t rows_per_seq, const int32_t* row_seq, const int64_t* q_pos,
                const uint8_t* cand, int64_t s_cand, srswa_route_params params, int64_t* topi64, int32_t* topi32,
                float* bias, uint8_t* valid, float* scores, void* workspace,
                size_t workspace_bytes, srswa_stream_t stream);

/* Selection only, from given block scores [N, nblk] (row stride s_sc):
 * _infer_route_select (hf-model-code/modeling_deepseekv2.py:339-362) and
 * DashRouterMath.route_and_select (whl:.../unlimited_dash_ops/dash_router.py:131-174). */
SRSWA_API int srswa_route_select(const float* scores, int64_t s_sc, int64_t N, int64_t nblk,
                       const uint8_t* cand, int64_t s_cand, srswa_route_params params,
                       int64_t* topi64, int32_t* topi32, float* bias, uint8_t* valid,
                       srswa_stream_t stream);

/* ------------------------------------------------------------ split-KV --
 * Router for rows whose blocks are spread over shards (the GPUs of a
 * split-KV decode, where GPU g owns a contiguous block range), or too many for
 * one CTA (a 1M-token row has 16384 blocks).
 *
 * Stage 1, per shard: srswa_route_shard_keys scores the blocks the shard owns,
 * global ids [block_offset, block_offset + nblk_local), with the global
 * candidacy rule (c <= q_pos/BS - L, block holds a token; nblk_total = blocks
 * of the whole row) and writes each row's best M as packed keys, keys_out
 * [N, M] uint64.  kbar is the shard's own: contiguous [B, nblk_local, d]
 * (block_table NULL, local index) or a paged cache [P, d] through
 * block_table [R, W] indexed by GLOBAL block id (only the owned range is
 * read).  d = 128.  workspace: srswa_route_shard_workspace_size bytes.
 *
 * Keys travel between processes (an all-gather), so their format is part of
 * this interface: bits 63..32 = order-preserving bits of the fp32 entmax input
 * x (z * idx_scale, or -1e4 off-candidate), bits 31..1 = 0x7fffffff - global
 * block id, bit 0 = candidate flag.  A larger key ranks first (x descending,
 * then block id ascending, the reference's tie order); 0 = no key.
 *
 * push (optional): the row keys also go into slot `rank` of every region of
 * that exchange (the producer side of the split-KV key all-gather), keys
 * [N, M] per slot.
 *
 * Stage 2: srswa_route_merge_keys reads nlists key lists per row (list l of
 * row n at keys[l * s_list + n * s_row], M keys each), keeps the global top-M
 * and runs the selection epilogue of srswa_route (exact entmax over the M,
 * first K slots, centred log-prior bias).  The lists must come from shards
 * that together cover [0, nblk_total) once; the top-M of the whole row is then
 * inside the union of the shards' top-Ms and the outputs equal srswa_route on
 * the whole row.  topi32_own (optional, [N, K]) is topi32 with -1 for blocks
 * outside [own_lo, own_hi): the slots the calling shard attends.
 * No candidate mask in this form (the reference's empty-row fallback needs
 * the whole row).  wait (optional): every CTA first acquires the flags of
 * that exchange (keys then point at own_region's slots), bounded.
 * Serves the per-GPU local top-M + global merge of the 1M-token split-KV
 * decode, over _infer_route_select semantics
 * (hf-model-code/modeling_deepseekv2.py:339-362) and
 * DashRouterMath.route_and_select (whl:.../unlimited_dash_ops/dash_router.py:131-174). */
SRSWA_API size_t srswa_route_shard_workspace_size(int64_t N, int64_t nblk_local, srswa_route_params params);
SRSWA_API int srswa_route_shard_keys(const void* idx_q, int q_dtype, int64_t s_q, int64_t N, int64_t d,
                           const float* kbar, int64_t s_kbar_b, int64_t s_kbar_c, int64_t nblk_local,
                           int64_t block_offset, int64_t nblk_total, const int32_t* block_table,
                           int64_t s_bt, const int32_t* seq_lens, int64_t rows_per_seq,
                           const int64_t* q_pos, srswa_route_params params, uint64_t* keys_out,
                           void* workspace, size_t workspace_bytes, const srswa_peer* push,
                           srswa_stream_t stream);
SRSWA_API int srswa_route_merge_keys(const uint64_t* keys, int64_t nlists, int64_t s_list, int64_t s_row,
                           int64_t N, int64_t nblk_total, srswa_route_params params, int64_t* topi64,
                           int32_t* topi32, float* bias, uint8_t* valid, int64_t own_lo,
                           int64_t own_hi, int32_t* topi32_own, const srswa_peer* wait,
                           srswa_stream_t stream);
/* Both stages in one launch: stage 1 as srswa_route_shard_keys (same
 * arguments and workspace), then the last CTA of each row merges the lists
 * and writes the outputs of srswa_route_merge_keys.  exchange NULL: this
 * shard covers [0, nblk_total) alone.  exchange given: that CTA pushes the
 * row's keys into every region of the exchange, waits (bounded, status 501
 * on expiry) for every rank's keys in its own region and merges the world
 * lists; every rank of the exchange makes the same call.  N <= 128 with an
 * exchange (each waiting CTA stays resident), else SRSWA_ETOOLARGE.  No
 * reference counterpart: it fuses the two stages above and the key
 * all-gather between them. */
SRSWA_API int srswa_route_shard_select(const void* idx_q, int q_dtype, int64_t s_q, int64_t N, int64_t d,
                           const float* kbar, int64_t s_kbar_b, int64_t s_kbar_c, int64_t nblk_local,
                           int64_t block_offset, int64_t nblk_total, const int32_t* block_table,
                           int64_t s_bt, const int32_t* seq_lens, int64_t rows_per_seq,
                           const int64_t* q_pos, srswa_route_params params, int64_t* topi64,
                           int32_t* topi32, float* bias, uint8_t* valid, int64_t own_lo, int64_t own_hi,
                           int32_t* topi32_own, void* workspace, size_t workspace_bytes,
                           const srswa_peer* exchange, srswa_stream_t stream);

/* ------------------------------------------------------------------ a3 --
 * Token block-max scores.  q [B,C,D] (strides), k [B,Sk,D], pos/seg [B,C]
 * int64 (seg may be NULL = 0) -> out [B,C,nblk] fp32 contiguous:
 * max over keys j of the block with seg <= j < pos - LW + 1, j < Sk, of q.k.
 * mode 0: triton_block_max_score (hf-model-code/sparse_gather_triton.py:445-524):
 *         unscaled, ls clamped at 0, -inf where empty.
 * mode 1: stage0 "indexer" _block_scores_infer
 *         (hf-model-code/modeling_deepseekv2.py:418-430): clamp(+-1e4),
 *         SCORE_NEG where empty. */
SRSWA_API int srswa_block_max_score(const void* q, int q_dtype, int64_t sqb, int64_t sqc, const void* k,
                          int k_dtype, int64_t skb, int64_t sks, const int64_t* pos,
                          const int64_t* seg, int64_t B, int64_t C, int64_t Sk, int64_t D,
                          int64_t block_size, int64_t nblk, int64_t local_window, int mode,
                          float* out, srswa_stream_t stream);

/* ------------------------------------------------------------------ a5 --
 * Selection packing: sel [B,HI,T,S] (int32 or int64, is64) -> out int32 with
 * ids < 0 or >= nblk and repeated ids inside a row set to -1 (the first slot
 * of an id survives).  Replaces the dedup of triton_gather_attention /
 * triton_gather_attention_e2e (hf-model-code/sparse_gather_triton.py:418-428,
 * sparse_gather_e2e_triton.py:383-394). */
SRSWA_API int srswa_pack_selection(const void* sel, int is64, int64_t rows, int64_t S, int64_t nblk,
                         int32_t* out, srswa_stream_t stream);

/* --------------------------------------------------------------- a6/a7 --
 * Fused gather-attention over (selected blocks' keys < local start) U window.
 * q [B,T,HQ,D], k/v [B,T,Hkv,D] (strides sb, st, sh; D contiguous), sel
 * [B,HI,T,S] int32 packed (srswa_pack_selection), bias [B,T,S] fp32 per-slot
 * remote bias or NULL, seg [B,T] int32 segment starts or NULL.
 * Outputs o [B,T,HQ,D] (o_dtype, strides), lse [B,T,HQ] fp32 natural log.
 * Replaces K1 _gather_attn_fwd_kernel / K5 _e2e_attn_fwd_kernel
 * (hf-model-code/sparse_gather_triton.py:35-122, 308-321;
 *  sparse_gather_e2e_triton.py:36-121, 303-322). */
typedef struct {
  int64_t B, T, HQ, Hkv, HI, D, S;
  int64_t block_size, local_window;
  float scale;
  int dtype; /* q/k/v element type */
  int64_t sqb, sqt, sqh;
  int64_t skb, skt, skh;
  int64_t svb, svt, svh;
} srswa_gather_desc;

SRSWA_API size_t srswa_gather_fwd_workspace_size(const srswa_gather_desc* g);
SRSWA_API int srswa_gather_fwd(const srswa_gather_desc* g, const void* q, const void* k, const void* v,
                     const int32_t* sel, const float* bias, const int32_t* seg, void* o,
                     int o_dtype, int64_t sob, int64_t sot, int64_t soh, float* lse,
                     void* workspace, size_t workspace_bytes, srswa_stream_t stream);

/* Forward of one sequence (B = 1) over paged K / V, on the tensor cores: the
 * long requests of the paged prefill attend K8 (whl:sglang/srt/layers/
 * attention/unlimited_dash_ops/attend_triton.py:88-292, 523-597), same
 * semantics as srswa_prefill_attend for one request.  k_cache / v_cache
 * [num_pages, 64, Hkv, 128] bf16, strides in the descriptor's k / v fields
 * (skb = svb: page, skt = svt: slot, skh = svh: head); key block j is page
 * pages[j] (pages covers ceil((qoff + T) / 64) blocks); query row t sits at
 * position qoff + t (a cached prefix of qoff tokens).  q / o [T, HQ, 128]
 * with the descriptor's sqt / sqh and o's sot / soh (sqb, sob unused).
 * sel [HI, T, S] int32 packed (srswa_pack_selection), bias [T, S] fp32 or
 * NULL, lse [T, HQ] (natural log) or NULL.  Slots of the last page past the
 * sequence's last token are never read.  D = 128, bf16, 64-token pages and
 * 8-element-aligned strides only: SRSWA_EUNSUPPORTED otherwise (nothing
 * launched; the row kernel of srswa_prefill_attend takes any shape).
 * workspace: srswa_gather_fwd_paged_workspace_size(g, qoff) bytes (0: not
 * a supported shape). */
SRSWA_API size_t srswa_gather_fwd_paged_workspace_size(const srswa_gather_desc* g, int64_t qoff);
SRSWA_API int srswa_gather_fwd_paged(const srswa_gather_desc* g, const void* q, const void* k_cache,
                     const void* v_cache, int64_t num_pages, const int32_t* pages, int64_t qoff,
                     const int32_t* sel, const float* bias, void* o, int64_t sob, int64_t sot,
                     int64_t soh, float* lse, void* workspace, size_t workspace_bytes,
                     srswa_stream_t stream);

/* Backward.  do [B,T,HQ,D] (strides as o), o and lse from the forward.
 * Outputs dq/dk/dv (dtype of q, same strides as q/k/v), d_bias [B,T,S] fp32
 * (required iff bias != NULL; 0 on -1/deduped slots).  Deterministic, no
 * atomics.  Replaces K2/K3 (hf-model-code/sparse_gather_triton.py:125-279,
 * 324-353) and K6/K7 (sparse_gather_e2e_triton.py:124-275, 324-352). */
SRSWA_API size_t srswa_gather_bwd_workspace_size(const srswa_gather_desc* g);
SRSWA_API int srswa_gather_bwd(const srswa_gather_desc* g, const void* q, const void* k, const void* v,
                     const void* o, int64_t sob, int64_t sot, int64_t soh, const void* dout,
                     const float* lse, const int32_t* sel, const float* bias,
                     const int32_t* seg, void* dq, void* dk, void* dv, float* d_bias,
                     void* workspace, size_t workspace_bytes, srswa_stream_t stream);

/* Backward that allocates nothing and takes no workspace.  No counterpart in
 * the reference (whose Triton path always allocates through torch).  For
 * callers that cannot allocate device memory at all (a runtime that reserves
 * all device memory up front, a plugin/FFI host that passes only input and
 * output buffers): the scratch is a 32 MiB array inside this library
 * (srswa_gather_bwd_noalloc_max_scratch()), present on every device that loads
 * it until exit.  Shapes needing more scratch than that return
 * SRSWA_ETOOLARGE.  The first call on a device looks up the array's device
 * address (make it outside stream capture).  Calls share the array: calls
 * whose GPU work overlaps race and must be serialised by the caller.
 * Results equal srswa_gather_bwd's, bit for bit.  The looked-up address is
 * kept for the life of the process: a cudaDeviceReset (or any teardown of the
 * device's primary context) while this library is loaded is not supported.
 * srswa_gather_bwd_noalloc_status reads the last call's status word (the head
 * of the array), as srswa_workspace_status does for a workspace. */
SRSWA_API size_t srswa_gather_bwd_noalloc_max_scratch(void);
SRSWA_API int srswa_gather_bwd_noalloc(const srswa_gather_desc* g, const void* q, const void* k,
                                       const void* v, const void* o, int64_t sob, int64_t sot, int64_t soh,
                                       const void* dout, const float* lse, const int32_t* sel,
                                       const float* bias, const int32_t* seg, void* dq, void* dk, void* dv,
                                       float* d_bias, srswa_stream_t stream);
SRSWA_API int srswa_gather_bwd_noalloc_status(int* out, srswa_stream_t stream);

/* ------------------------------------------------------------------ a9 --
 * Block-sparse decode attend over a paged (or contiguous) KV cache.
 * q [N,H,D] (row stride s_qn, head stride s_qh).  k/v caches: element of
 * (page, pos-in-page, kv head, d) at page*s_page + pos*s_pos + h*s_head + d.
 * block_table [R,W] int32 maps (request, block) -> page; NULL means one
 * contiguous cache per request: block blk of request r starts at element
 * r*s_req + blk*s_page.
 * Row n belongs to request n / rows_per_req and sits at position
 * q_pos[n] (int64, optional) or seq_lens[r] - rows_per_req + n % rows_per_req.
 * topk_idx [.., N, K] (int32 or int64; head stride s_ti_h may be 0; -1 or
 * valid==0 = unused slot; repeated ids count once), bias same layout (NULL =
 * no bias), valid uint8 same layout as topk_idx (NULL = all slots with id >= 0).
 * Remote keys of a selected block: pos <= p and pos < max(0, p-LW+1) (biased);
 * local keys: max(0, p-LW+1) <= pos <= p (unbiased), LW = L*BS.
 * out [N,H,D] (out_dtype, strides), lse_out [N,H] fp32 natural log (optional).
 * nsplit: CTAs per (row, head) merged on-chip through a thread-block cluster
 * (0 = choose).  kv_dtype: SRSWA_BF16, SRSWA_F16, or SRSWA_F8E4M3 /
 * SRSWA_F8E5M2 caches (converted exactly to fp32 in the kernel; the
 * reference's use_fp8 path casts them to the query dtype, attend_triton.py:545,
 * 626).  Replaces dash_sparse_attn_decode + K9/K10
 * (whl:.../unlimited_dash_ops/attend_triton.py:307-518, 600-715; common.py:43-89)
 * and _decode_attend (hf-model-code/modeling_deepseekv2.py:455-481). */
typedef struct {
  int64_t N, H, Hkv, D, K;
  int64_t block_size, local_blocks;
  float sm_scale;
  int q_dtype, kv_dtype, out_dtype;
  int64_t s_qn, s_qh;
  int64_t s_page, s_pos, s_head;
  int64_t s_on, s_oh;
  int64_t R, W, s_req, rows_per_req;
  int idx_is64;
  int64_t s_ti_h, s_ti_n; /* topk_idx / bias / valid strides (head, row) */
  int64_t s_b_h, s_b_n;
  int nsplit;
  int skip_local; /* 1: attend the selected remote blocks only, not the window
                     (split-KV shards that do not own the window) */
  int overlap;    /* 1: the launch may begin before the kernel issued just
                     before it on the stream has finished (programmatic
                     dependent launch) and attends the window keys meanwhile:
                     q, the caches, block_table and seq_lens / q_pos must have
                     been written before that kernel began; topk_idx, bias and
                     valid are read after it has completed.  The library's
                     routers, called right before on the same stream, are such
                     kernels.  0: nothing is read before that kernel has
                     completed.  Results are identical either way. */
} srswa_decode_desc;

SRSWA_API int srswa_decode_attend(const srswa_decode_desc* dd, const void* q, const void* k_cache,
                        const void* v_cache, const int32_t* block_table,
                        const int32_t* seq_lens, const int64_t* q_pos, const void* topk_idx,
                        const float* bias, const uint8_t* valid, void* out, float* lse_out,
                        srswa_stream_t stream);
/* srswa_decode_attend whose results also travel to the peers: out (fp32,
 * contiguous [N, H, D]) and lse_out ([N, H]).  Flag protocol: out and lse_out
 * must lie in this rank's own slot of the exchange `push` (srswa_peer
 * below); every (row, head) result is stored at the same offset of every
 * region, and the storing CTAs are the exchange's producer units (the last
 * releases the flags).  LL protocol: out / lse_out are any buffers (the local
 * copy); element e of the packed o-then-lse partial goes to LL word e of
 * every region.  The consumer is srswa_lse_merge with the same exchange as
 * its wait (LL: o_parts / lse_parts may be NULL, C = world).  The split-KV decode's
 * partial all-gather fused into the attend; no reference counterpart. */
/* srswa_decode_attend_push with an LL exchange whose log-sum-exp merge is
 * done by the attend itself: each (row, head)'s storing CTA, after its own
 * puts, waits (bounded) for every rank's partial of that (row, head) and
 * writes the merge to final_out ([N, H, D] contiguous, final_dtype F32 /
 * BF16 / F16) and final_lse ([N, H], optional) -- the same values as
 * srswa_lse_merge.  The CTAs of one rank wait for the peers' CTAs, so the
 * whole grid must be resident at once (N * H * split CTAs within the GPU's
 * resident slots), else SRSWA_ETOOLARGE and the caller takes
 * srswa_decode_attend_push + srswa_lse_merge.  No reference counterpart: the
 * split-KV decode's partial all-gather and combine fused into the attend. */
SRSWA_API int srswa_decode_attend_exchange(const srswa_decode_desc* dd, const void* q, const void* k_cache,
                        const void* v_cache, const int32_t* block_table, const int32_t* seq_lens,
                        const int64_t* q_pos, const void* topk_idx, const float* bias, const uint8_t* valid,
                        float* out, float* lse_out, const srswa_peer* exchange, void* final_out,
                        int final_dtype, float* final_lse, srswa_stream_t stream);
SRSWA_API int srswa_decode_attend_push(const srswa_decode_desc* dd, const void* q, const void* k_cache,
                        const void* v_cache, const int32_t* block_table,
                        const int32_t* seq_lens, const int64_t* q_pos, const void* topk_idx,
                        const float* bias, const uint8_t* valid, float* out, float* lse_out,
                        const srswa_peer* push, srswa_stream_t stream);

/* Paged varlen prefill attend (the SGLang prefill op): rows n of request r
 * are cu_seqlens_q[r] <= n < cu_seqlens_q[r + 1] (int32 [R + 1], device), row
 * n sits at position prefix_lens[r] + n - cu_seqlens_q[r] (prefix_lens int32
 * [R], device) and reads block table row r.  Per row, remote keys are the
 * selected blocks' keys below the window start, local keys the window
 * [p - LW + 1, p]; bias on remote keys only.  The descriptor is the decode
 * one with N = total rows and R = requests (rows_per_req, s_req ignored).
 * Replaces _dash_sparse_fwd_kernel / dash_sparse_attn
 * (whl:.../unlimited_dash_ops/attend_triton.py:88-292, 523-597). */
SRSWA_API int srswa_prefill_attend(const srswa_decode_desc* dd, const void* q, const void* k_cache,
                         const void* v_cache, const int32_t* block_table, const int32_t* cu_seqlens_q,
                         const int32_t* prefix_lens, const void* topk_idx, const float* bias, void* out,
                         float* lse_out, srswa_stream_t stream);

/* Status of the last gather call that used `workspace`: the first 4 bytes of
 * every gather workspace (srswa_gather_fwd / srswa_gather_bwd; the workspace
 * sizes include them) are that call's status word, cleared when the call is
 * enqueued.  0 = ok; otherwise the code of a tensor-core kernel's bounded
 * wait on a completion barrier that expired (the kernel then skipped its
 * outputs and exited cleanly).  Reads the word on `stream` and waits for that
 * stream only.  Status is per call: concurrent calls on other workspaces never
 * see each other's codes.  No reference counterpart. */
SRSWA_API int srswa_workspace_status(const void* workspace, int* out, srswa_stream_t stream);

/* Log-sum-exp merge of C split-KV partials: part c of o at o_parts + c *
 * s_o_part ([N,H,D] fp32, contiguous inside the part), of the log-sum-exp at
 * lse_parts + c * s_l_part ([N,H] fp32 natural log, -inf = empty part); the
 * strides let the parts come straight out of one packed all-gather buffer
 * (0 = tightly stacked: N*H*D and N*H).  -> out [N,H,D] (out_dtype,
 * contiguous) and lse_out [N,H] (optional).  Replaces
 * _merge_topk_attn_out_kernel (whl:.../unlimited_dash_ops/common.py:43-89);
 * also the cross-GPU combine of the split-KV decode, where wait (optional)
 * makes every CTA first acquire the flags of the partials' exchange. */
SRSWA_API int srswa_lse_merge(const float* o_parts, const float* lse_parts, int64_t C, int64_t N,
                    int64_t H, int64_t D, int64_t s_o_part, int64_t s_l_part, void* out,
                    int out_dtype, float* lse_out, const srswa_peer* wait, srswa_stream_t stream);

/* ------------------------------------------------------------------ f4 --
 * DSA gather-KL distillation (training stage "sparse", one index head).
 * Per query row (b, c): KL(P || P_idx) over the keys of the row's selected
 * blocks sel [B,C,S] (int32, -1 pad; a repeated block counts once) that lie
 * in [seg, pos] and below max(pos - LW + 1, 0): P_idx = softmax of
 * idx_q . idx_k[j], P = the mean over the H main heads of the softmaxes of
 * (q_main[h] . k_main[j, h / (H/Hkv)]) * scaling; both logits rounded to bf16
 * first when logits_bf16 (the reference's bf16 matmul outputs).
 * idx_q [B,C,d], idx_k [B,Sk,d], q_main [B,C,H,D], k_main [B,Sk,Hkv,D] (the
 * strides below; features contiguous; any of f32 / bf16 / f16), pos / seg
 * [B,C] int64 (global position, segment start; seg may be NULL = 0); d, D
 * multiples of 8 up to 128; block_size <= 64, S * block_size <= 2048.
 * fwd -> kl [B,C] fp32 (0 for rows with no key), valid [B,C] uint8.
 * bwd: grad [B,C] = dLoss/dkl per row -> d_idx_q [B,C,d], d_idx_k [B,Sk,d]
 * fp32 (contiguous, fully written; deterministic, no atomics); workspace of
 * srswa_gather_kl_bwd_workspace_size bytes.  Replaces the gather-KL of
 * select_and_kl_loss and _kl_chunk_core / _KLChunkFn
 * (hf-model-code/_sparse_base_impl.py:3397-3450, 2071-2191). */
typedef struct {
  int64_t B, C, Sk, H, Hkv, D, d, S, block_size, local_window;
  float scaling;
  int logits_bf16;
  int iq_dtype, ik_dtype, qm_dtype, km_dtype;
  int64_t s_iq_b, s_iq_c, s_ik_b, s_ik_s, s_qm_b, s_qm_c, s_qm_h, s_km_b, s_km_s, s_km_h;
} srswa_kl_desc;

SRSWA_API int srswa_gather_kl_fwd(const srswa_kl_desc* g, const void* idx_q, const void* idx_k, const void* q_main,
                        const void* k_main, const int32_t* sel, const int64_t* pos, const int64_t* seg,
                        float* kl, uint8_t* valid, srswa_stream_t stream);
SRSWA_API size_t srswa_gather_kl_bwd_workspace_size(const srswa_kl_desc* g);
SRSWA_API int srswa_gather_kl_bwd(const srswa_kl_desc* g, const void* idx_q, const void* idx_k, const void* q_main,
                        const void* k_main, const int32_t* sel, const int64_t* pos, const int64_t* seg,
                        const float* grad, float* d_idx_q, float* d_idx_k, void* workspace,
                        size_t workspace_bytes, srswa_stream_t stream);
/* The same pair keeping the teacher: srswa_gather_kl_fwd_save also writes
 * each row's averaged teacher probabilities over its S * block_size key
 * slots, teacher [B, C, S * block_size] fp32 (0 on slots that keep no key),
 * and srswa_gather_kl_bwd_saved reads them instead of recomputing the H
 * teacher softmaxes (the gather of every head's main keys, most of the
 * backward's work).  Results equal the recomputing pair bit for bit; the
 * price is the teacher buffer kept between the two calls.  No reference
 * counterpart (the reference recomputes inside its chunked autograd
 * function). */
SRSWA_API int srswa_gather_kl_fwd_save(const srswa_kl_desc* g, const void* idx_q, const void* idx_k,
                        const void* q_main, const void* k_main, const int32_t* sel, const int64_t* pos,
                        const int64_t* seg, float* kl, uint8_t* valid, float* teacher, srswa_stream_t stream);
SRSWA_API int srswa_gather_kl_bwd_saved(const srswa_kl_desc* g, const void* idx_q, const void* idx_k,
                        const int32_t* sel, const int64_t* pos, const int64_t* seg, const float* teacher,
                        const float* grad, float* d_idx_q, float* d_idx_k, void* workspace,
                        size_t workspace_bytes, srswa_stream_t stream);

/* --------------------------------------------------- peer exchange ------
 * All-gather through peer memory for the split-KV decode across the GPUs of
 * one node (the two exchanges per layer of the reference plan's per-GPU
 * top-M + LSE combine; no reference counterpart: the reference decodes on
 * one GPU).  Every rank owns one exchange region of
 * srswa_peer_region_size(world, slot_bytes) bytes: 256 bytes of flags (one
 * uint64 epoch per source rank), then one slot_bytes slot per source rank.
 * Set-up (outside the decode loop; the only entry points here that
 * allocate): srswa_peer_region_alloc (cudaMalloc + zero fill, so the IPC
 * handle maps exactly the region), srswa_peer_ipc_handle (64 bytes to send to
 * the peers), srswa_peer_ipc_open / _close on each peer's handle.
 *
 * A region is described by srswa_peer (declared above; all pointers device
 * memory):
 *   regions     [world] the regions' base addresses as mapped in this process
 *               (regions[rank] = own_region);
 *   counter     exchanges completed on this region (zero at set-up; the
 *               producer publishes epoch = *counter + 1, the consumer waits
 *               for it on every source's flag and then advances *counter);
 *   tickets     2 words, zero at set-up: the producer units' and the
 *               consumer CTAs' arrival counts (reset by the last arrival);
 *   status      0, or 501 when a wait expired (2 s bound; the kernel then
 *               goes on with whatever the slots hold and returns).
 * Producers copy their payload with plain stores into slot `rank` of every
 * region, and the last producer unit releases flag `rank` of every region
 * (system scope); consumers acquire all flags before reading the slots.  The
 * payload of rank r is then slot r of own_region.  Producers and consumers
 * are the library's kernels themselves: srswa_route_shard_keys (push of the
 * router keys), srswa_route_merge_keys and srswa_lse_merge (wait), or the
 * stand-alone srswa_peer_push / srswa_peer_allgather (push; push + wait).
 * No NCCL, no TMA, no multicast: peer bytes move only by plain stores.  A
 * rank must not start exchange e+1 on a region before its consumers of e
 * have read it; stream order gives this when two regions alternate (router
 * keys, then attention partials).
 *
 * LL protocol (ll = 1): every 32-bit payload word travels as one 8-byte
 * word (payload, epoch = low 32 bits of *counter + 1) in one aligned store,
 * which is single-copy atomic; a consumer polls each word it reads until its
 * epoch matches (bounded, status 501 on expiry), so no fence, flag or
 * producer ticket is needed and the flag header is unused.  The consumer
 * CTAs still count themselves (tickets[1]) and the last advances *counter.
 * Slot k of a region is then 8-byte word k of the payload's 32-bit word k.
 * Taken by srswa_route_shard_select (the router keys: row n, key j as words
 * 2 (n M + j) and 2 (n M + j) + 1, low half first), srswa_decode_attend_push
 * (partial element e of the packed [N, H, D] o then [N, H] lse) and
 * srswa_lse_merge (wait); the other entry points refuse an LL region
 * (SRSWA_EUNSUPPORTED). */
SRSWA_API int srswa_peer_region_size(int64_t world, int64_t slot_bytes, size_t* out);
SRSWA_API int srswa_peer_region_alloc(size_t bytes, void** out);
SRSWA_API int srswa_peer_region_free(void* region);
SRSWA_API int srswa_peer_ipc_handle(const void* region, void* handle64);
SRSWA_API int srswa_peer_ipc_open(const void* handle64, void** mapped);
SRSWA_API int srswa_peer_ipc_close(void* mapped);
/* nbytes (multiple of 16, <= slot_bytes) from src into slot `rank` of every
 * region, then the flags; srswa_peer_allgather also waits (one more launch)
 * and advances the counter. */
SRSWA_API int srswa_peer_push(const void* src, int64_t nbytes, const srswa_peer* peer, srswa_stream_t stream);
SRSWA_API int srswa_peer_allgather(const void* src, int64_t nbytes, const srswa_peer* peer, srswa_stream_t stream);

/* ------------------------------------------------------- PageGate ------
 * Page-aware remote candidates.  Token ids are int64 [B, n] rows (row stride
 * s_row); img_id / page_id are the <image> and <PAGE> token ids; per_page is
 * the image tokens per page when the prompt carries no <PAGE> markers.
 * Page ids must stay below 2^31. */

/* Scratch of srswa_page_ids / srswa_decode_allow_state for B rows of n_tok
 * tokens (16 bytes per 2048-token chunk and row). */
SRSWA_API size_t srswa_page_scan_workspace_size(int64_t B, int64_t n_tok);

/* Page-aware token ids: itm [B, key_length] (1 = image token), ipi [B,
 * key_length] int64 (image page, -1 = not an image token), qpi [B,
 * key_length] int64 (query page, -1 = unconstrained), all contiguous; ids
 * beyond n_ids are padding (-1), beyond key_length ignored.  flags[0] /
 * flags[1] (int32, zeroed here) become 1 when the rows hold an image token /
 * a query with a page (the reference returns None otherwise).
 * page_scope_prefill: prefill queries (up to the row's last image token) get
 * their raw page (1) or stay unconstrained (0).
 * Replaces DeepseekV2Indexer._build_page_aware_ids
 * (hf-model-code/_sparse_base_impl.py:2404-2497). */
SRSWA_API int srswa_page_ids(const int64_t* ids, int64_t s_row, int64_t B, int64_t n_ids,
                             int64_t key_length, int64_t img_id, int64_t page_id, int64_t per_page,
                             int page_scope_prefill, uint8_t* itm, int64_t* ipi, int64_t* qpi,
                             int32_t* flags, void* workspace, size_t workspace_bytes,
                             srswa_stream_t stream);

/* Per key block of nblk blocks of block_size tokens: desc [B, nblk, 4] int32
 * (16-byte aligned) = {min image page (-1: none), max page, page set low /
 * high 32 bits}.  Source: page ids ipi [B, n_tok] (row stride s_row), or,
 * for the any-page ("flat") candidates, an image-token mask itm [B, n_tok]
 * (exactly one of the two non-null).  Tokens past n_tok are padding.
 * Replaces the block reductions of _build_page_aware_image_block_mask and
 * _build_image_block_allow_mask (_sparse_base_impl.py:2629-2648, 2392-2402). */
SRSWA_API int srswa_page_block_desc(const int64_t* ipi, const uint8_t* itm, int64_t s_row, int64_t B,
                                    int64_t n_tok, int64_t block_size, int64_t nblk, int32_t* desc,
                                    srswa_stream_t stream);

/* Candidate mask cand [B, cq, nblk] (uint8, contiguous) of cq query rows:
 * query i of row b has page qpi[b, clamp(pos[b, i], 0, n_q - 1)] and block c
 * is a candidate when it holds an image token of that page (flat = 1: when
 * it holds any image token).  fallback = 1: a query without a candidate gets
 * every block (the reference's per-query fallback).  ipi (the descriptors'
 * source) is read only for blocks whose pages span 64 or more.
 * Replaces _build_kl_candidate_mask (_sparse_base_impl.py:2697-2730) and the
 * query-chunk loop of _dash_block_cand (modeling_deepseekv2.py:108-122). */
SRSWA_API int srswa_page_cand_mask(const int32_t* desc, const int64_t* ipi, int64_t s_ipi, int64_t n_tok,
                                   int64_t block_size, int64_t B, int64_t nblk, const int64_t* qpi,
                                   int64_t s_qpi, int64_t n_q, const int64_t* pos, int64_t s_pos,
                                   int64_t cq, int flat, int fallback, uint8_t* cand,
                                   srswa_stream_t stream);

/* Decode-allow state of a prefill of L tokens: per block of block_size
 * (dividing 2048) the [min, max] image page it holds (bmin = bmax = -1
 * without image tokens; [B, ceil(L/block_size)] int64 contiguous), the prompt
 * page count pp [B] and the marker count mcum [B].
 * Replaces the prefill branch of _uocr_dash_decode_allow
 * (hf-model-code/modeling_unlimitedocr.py:497-514). */
SRSWA_API int srswa_decode_allow_state(const int64_t* ids, int64_t s_row, int64_t B, int64_t L,
                                       int64_t img_id, int64_t page_id, int64_t per_page,
                                       int64_t block_size, int64_t* bmin, int64_t* bmax, int64_t* pp,
                                       int64_t* mcum, void* workspace, size_t workspace_bytes,
                                       srswa_stream_t stream);

/* Decode allow mask of one new token per request: mcum[b] += (last_ids[b *
 * s_ids] == page_id) in place; query page = mcum - 1 - pp (-1 if negative);
 * allow [B, nblk] uint8 = block c < nblk_state with bmin <= page <= bmax, or
 * every block when the query has no page or no such block.
 * Replaces the decode branch of _uocr_dash_decode_allow
 * (modeling_unlimitedocr.py:515-528). */
SRSWA_API int srswa_decode_allow(const int64_t* last_ids, int64_t s_ids, int64_t B, int64_t page_id,
                                 const int64_t* bmin, const int64_t* bmax, int64_t s_state,
                                 int64_t nblk_state, const int64_t* pp, int64_t* mcum, int64_t nblk,
                                 uint8_t* allow, srswa_stream_t stream);

/* Decode scan window: for each decode row (row of request row / dql at
 * position seq_lens[r] - dql + row % dql), the span [lo, hi) of blocks
 * allowed by allow [nd, WQ] uint8 (row stride s_allow) among the live remote
 * blocks (c <= q_blk - L, c * bs < seq_len, c < min(W, WQ)); with none,
 * lo = 0 and hi = 0 (no remote block) or the live width min(W, max(nblk, 1));
 * fit = (hi - lo) <= tile.  lo / hi int32 [nd], fit int8 [nd].  Replaces
 * _win_bounds_kernel / win_bounds_decode
 * (whl:.../unlimited_dash_ops/route_triton.py:466-526). */
SRSWA_API int srswa_win_bounds_decode(const uint8_t* allow, int64_t s_allow, int64_t WQ, const int32_t* seq_lens,
                            int64_t nd, int64_t W, int64_t block_size, int64_t local_blocks,
                            int64_t decode_query_len, int64_t tile, int32_t* lo, int32_t* hi, int8_t* fit,
                            srswa_stream_t stream);

/* ---------------------------------------------------- page2d RoPE -------
 * Two-axis rotary coordinates (token-in-page, page) of the indexer and the
 * main branch.  Token ids as for PageGate. */

/* Scratch of srswa_rope2d_pos for B rows of n_tok tokens. */
SRSWA_API size_t srswa_rope2d_pos_workspace_size(int64_t B, int64_t n_tok);

/* Coordinates of key_length tokens per row: page [B, key_length] int64 =
 * marker count (prefill: up to the row's last image token) or marker count
 * minus the prompt pages (response); tok [B, key_length] int64 = running
 * count inside the token's page bucket (span > 0: each page's prefill mapped
 * onto span steps, page 0 raw); pf_cnt [B, pf_cap] int64 (pf_cap >=
 * key_length + 1) = prefill tokens of each page.  flags (int32 [4], zeroed
 * here): [0] an image token, [1] a <PAGE> marker, [2] rows without prompt
 * pages, [3] the page count n_pg; the reference returns None unless [0] and
 * [1] are set and [2] is 0.
 * Replaces DeepseekV2Indexer._build_page_rope_pos + _page_rope_offsets
 * (hf-model-code/_sparse_base_impl.py:2511-2570). */
SRSWA_API int srswa_rope2d_pos(const int64_t* ids, int64_t s_row, int64_t B, int64_t n_ids,
                               int64_t key_length, int64_t img_id, int64_t page_id, int64_t span,
                               int64_t* tok, int64_t* page, int64_t* pf_cnt, int64_t pf_cap,
                               int32_t* flags, void* workspace, size_t workspace_bytes,
                               srswa_stream_t stream);

/* cos / sin tables [B, S, 2 * (n_tok + page_pairs)] (dtype, contiguous) of
 * coordinates tok / page [B, S] (row stride s_pos): pair i < n_tok turns by
 * tok * inv_tok[i], pair n_tok + i by (page mod page_mod, if > 0) *
 * inv_page[i]; the table is [angles, angles].
 * Replaces DeepseekV2IndexerRotary2D.forward (_sparse_base_impl.py:2043-2058). */
SRSWA_API int srswa_rope2d_table(const int64_t* tok, const int64_t* page, int64_t s_pos, int64_t B,
                                 int64_t S, const float* inv_tok, int64_t n_tok, const float* inv_page,
                                 int64_t page_pairs, int64_t page_mod, void* cos_out, void* sin_out,
                                 int dtype, srswa_stream_t stream);

/* In place x <- x * cos + rotate_half(x) * sin over x [B, S, H, D] (fp32 or
 * bf16; strides s_b, s_s, s_h, D contiguous, D % 16 == 0), feature f using
 * pair f mod (n_tok + page_pairs), with the table values rounded to
 * table_dtype first.  Fuses srswa_rope2d_table with the rotary application
 * of the reference (apply_rotary_pos_emb at _sparse_base_impl.py:1537, and
 * modeling_deepseekv2.py:183, 374, 508) without materialising the tables. */
SRSWA_API int srswa_rope2d_apply(void* x, int dtype, int64_t B, int64_t S, int64_t H, int64_t D,
                                 int64_t s_b, int64_t s_s, int64_t s_h, const int64_t* tok,
                                 const int64_t* page, int64_t s_pos, const float* inv_tok, int64_t n_tok,
                                 const float* inv_page, int64_t page_pairs, int64_t page_mod,
                                 int table_dtype, srswa_stream_t stream);

/* Decode update of one new token per row, in place on page [B] / tok [B]: a
 * <PAGE> token moves to the next page (at most n_pg - 1) and restarts tok at
 * that page's prefill count pf_cnt[b, page] (row stride s_pf); any other
 * token advances tok.
 * Replaces the decode branch of SlidingWindowLlamaAttention._main_rope_coords
 * (_sparse_base_impl.py:1482-1489). */
SRSWA_API int srswa_rope2d_decode(const int64_t* new_ids, int64_t s_ids, int64_t B, int64_t page_id,
                                  int64_t* page, int64_t* tok, const int64_t* pf_cnt, int64_t s_pf,
                                  int64_t n_pg, srswa_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* SRSWA_H */
