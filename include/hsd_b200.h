/*
 * hsd_b200 -- C ABI of the B200 (sm_100a) verification hot path of HSD.
 *
 * Plain pointers and sizes only.  Every entry point is asynchronous on the
 * stream it is given, never synchronises, and returns an HSD_* status code
 * for host-side argument errors (hsd_last_error() holds the message).
 * Problems found on the device (a bounded wait that ran out, an index out of
 * range) are written with atomicCAS into the caller's int32 `status` word in
 * device memory (first error wins; NULL disables reporting); the host reads
 * it after its next synchronisation.  Every device pointer is caller-owned.
 *
 * The step's kernels (tile plan, attention, KV append, RoPE + cache update,
 * acceptance + KMP, keep indices, compaction, bit remap) are launched with
 * programmatic stream serialization: each waits for the previous work on the
 * stream to complete before touching memory and lets the next kernel be
 * scheduled early.  A caller's kernel that follows on the same stream with
 * programmatic stream serialization of its own must wait for its predecessor
 * (griddepcontrol.wait / cudaGridDependencySynchronize) before reading these
 * kernels' outputs; ordinary launches, copies and events need nothing.
 *
 * Reference interfaces replaced (paths inside whlscut/HSD):
 *   D  = hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py
 *   H  = hsd/hunyuan_ocr_pipeline/modeling_hunyuan_vl_hsd.py
 */
#ifndef HSD_B200_H
#define HSD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *hsd_stream_t;

/* host status codes */
#define HSD_OK 0
#define HSD_ERR_INVALID_ARG 1
#define HSD_ERR_UNSUPPORTED 2
#define HSD_ERR_CUDA 3
#define HSD_ERR_TOO_LARGE 4

/* device status codes (low 16 bits: where; high bits: what) */
#define HSD_DEV_TIMEOUT 0x10000
#define HSD_DEV_BAD_INDEX 0x20000
#define HSD_DEV_CAPACITY 0x40000

/* segment kinds: the intra-segment pattern over the segment's new columns */
#define HSD_SEG_CAUSAL 0 /* speculative / prefill block: tril (D:1442-1447, RD:234-245) */
#define HSD_SEG_TREE 1   /* tree block: ancestor sets (D:1519-1533) */
#define HSD_SEG_SINGLE 2 /* normal block: only its first row sees its first column (D:1021-1025) */
#define HSD_SEG_NONE 3   /* no new columns (e.g. HunYuan tight-pack tail rows, H:2290-2293) */

/* block modes of the verification loop (D:979, `decode_modes`) */
#define HSD_MODE_NORMAL 0
#define HSD_MODE_SPEC 1
#define HSD_MODE_TREE 2
#define HSD_MODE_FINISHED 3

/* One segment of the packed query.  Every row q in [q_start, q_start+q_len)
 * sees the columns set in the segment's row of `seg_kv_bits`, plus the
 * pattern `kind` over the segment's own new columns, which start at column
 * kv_len - q_len_total + q_start.  Replaces the dense float mask the
 * reference rebuilds each step (D:1634-1667, D:1737-1748). */
typedef struct {
  int32_t q_start;
  int32_t q_len;
  int32_t kind;
  int32_t tree_off;   /* HSD_SEG_TREE: offset (in uint64 words) of q_len ancestor rows */
  int32_t tree_words; /* HSD_SEG_TREE: words per ancestor row, >= ceil(q_len / 64) */
  int32_t reserved;
} hsd_segment_t;

/* Tile plan of one packed mask: the same information as FlexAttention's
 * BlockMask at BLOCK_SIZE (128, 64) (D:94-106, H:1213-1221) plus the per-row
 * 64-bit masks of every tile and the list of 128-column blocks the attention
 * kernel visits.  All pointers are device memory carved from one workspace by
 * hsd_plan_init(). */
typedef struct {
  int32_t q_len, kv_len;
  int32_t n_qtiles;   /* ceil(q_len / 128) */
  int32_t n_kv64;     /* ceil(kv_len / 64) */
  int32_t n_kv128;    /* ceil(kv_len / 128) */
  int32_t reserved;
  uint64_t *mask_words;      /* [n_qtiles][n_kv64][128] bit c of row r = column 64t+c allowed */
  uint8_t *tile_class;       /* [n_qtiles][n_kv64] 0 empty, 1 partial, 2 full */
  int32_t *kv_num_blocks;    /* [n_qtiles]  BlockMask.kv_num_blocks (partial tiles) */
  int32_t *kv_indices;       /* [n_qtiles][n_kv64] ascending */
  int32_t *full_kv_num_blocks; /* [n_qtiles] */
  int32_t *full_kv_indices;  /* [n_qtiles][n_kv64] ascending */
  int32_t *blk_count;        /* [n_qtiles] 128-column blocks visited */
  uint32_t *blk_list;        /* [n_qtiles][n_kv128] block | flags << 24 */
  int32_t *tile_order;       /* [n_qtiles] query tiles, most blocks first */
  int32_t *blk_prefix;       /* [n_qtiles + 1] exclusive prefix of blk_count in tile_order */
} hsd_plan_t;

/* Per-block state and inputs of the acceptance / re-alignment kernel.  Mirrors
 * the per-block Python lists of `batch_generate` (D:979-992). */
typedef struct {
  int32_t mode;        /* HSD_MODE_* this step ran in */
  int32_t q_start;     /* block_start in the packed query (D:1101) */
  int32_t q_len;       /* block_end - block_start */
  int32_t valid_count; /* block_valid_counts[b] (D:992) */
  int32_t gen_off;     /* generated tokens live at gen_pool[gen_off, gen_off + gen_cap) */
  int32_t gen_len;     /* in: tokens so far; out: after this step */
  int32_t gen_cap;
  int32_t draft_off;   /* tokenized draft at draft_pool[draft_off, + draft_len) */
  int32_t draft_len;
  int32_t mws;         /* match_window_sizes[b] (in/out) */
  int32_t matches_len; /* matches_length[b] (in/out) */
  int32_t tree_off;    /* HSD_MODE_TREE: packed BFS nodes at tree_tokens/parents[tree_off..] */
  int32_t tree_nodes;
  int32_t seg;         /* row of seg_kv_bits holding this block's KV visibility */
  int32_t flags;       /* bit 0: page block (no repetition stop, no token KMP);
                          bit 1: text mode (parser.text_mode, D:1229), enables the
                          tree logit-ratio fallback */
  int32_t reserved;
} hsd_block_t;

typedef struct {
  int32_t finished;    /* 0 running, 1 EOS (D:1299-1305), 2 repetition stop (D:1306-1319), 3 was finished */
  int32_t increment;   /* generated_tokens_increment[b] */
  int32_t pointer;     /* packed row of the last accepted token */
  int32_t next_token;  /* next_token_int */
  int32_t match_count; /* len(matches) of the re-alignment (D:1419) */
  int32_t match_start; /* draft index of the first match, -1 if none */
  int32_t slice_begin; /* unique match: next speculative input is draft[slice_begin, slice_end) */
  int32_t slice_end;
} hsd_block_result_t;

typedef struct {
  int32_t n_blocks;
  int32_t kv_len;          /* columns of the current mask */
  int32_t kv_base;         /* first new column: kv_len - q_len (D:1089) */
  int32_t kv_words_stride; /* uint64 words per row of seg_kv_bits / out_kv_bits */
  int32_t match_window_size;            /* default 3 */
  int32_t match_window_size_upper_bound;/* default 10 */
  int32_t max_spec_len;    /* HSD_MAX_SPEC_LEN, 0 = unlimited */
  int32_t repeat_sentinel; /* 20993 (dots) / 41153 (HunYuan) */
  int32_t n_eos;
  int32_t eos_ids[8];
} hsd_accept_config_t;

/* Inputs of the logit-ratio acceptance the reference applies below
 * HSD_SPEC_THRESH / HSD_TREE_THRESH = 1 (D:970-971).  Ratios are bf16
 * quotients (float32 quotient rounded to bf16) compared with the threshold
 * rounded to bf16, as torch does on the bf16 logits tensor. */
typedef struct {
  /* [q_len] logits[r, next_ids[r]]: each packed row's maximal logit (bf16
   * value; hsd_lm_head_argmax's max_logit) */
  const float *max_logit;
  /* [q_len] per packed row r: in a speculative block logits[r, input_ids[r + 1]];
   * for node c >= 1 of a tree block starting at row bs,
   * logits[bs + parent(c), token(c)] (row bs + c); hsd_probe_logits computes them */
  const float *probe_logit;
  /* < 1: a speculative row that misses also passes when
   * probe_logit / max_logit >= thresh and max_logit > 0 (D:1147-1174) */
  float spec_thresh;
  /* < 1: in text-mode blocks (flags bit 1), a tree node whose target token is
   * no child moves to the child of first maximal ratio
   * probe_logit(child) / max_logit(node) if one reaches thresh (D:1228-1238,
   * D:1256-1266) */
  float tree_thresh;
  /* HSD_ACCEPT_DOTS or HSD_ACCEPT_HUNYUAN.  HunYuan (H:1653-1858): the
   * speculative ratio applies to the last block only, never inside a
   * formula (rows whose draft token is a formula delimiter or lies between
   * delimiters, counting from the block's generated tokens), and accepted
   * rows keep the model's tokens; the tree fallback runs in text-mode
   * blocks at any tree_thresh (H:1791-1800, no `< 1` guard) */
  int32_t variant;
  int32_t formula_tokens[2]; /* HunYuan formula delimiters: 3 ('$'), 1099 ('$$') */
  /* HunYuan SPEC_MODE (H:1668-1743) for the last block's missed rows, where
   * the ratio rule applies (spec_thresh < 1, outside formulas):
   * HSD_SPEC_FMST (0, default) the ratio; HSD_SPEC_TOPK the draft token is
   * among the row's spec_topk best logits (rank[r] < spec_topk, ranks from
   * hsd_lm_head_rank); HSD_SPEC_ADAPTIVE the ratio, or
   * bf16(max_logit - second) < bf16(spec_margin) with probe_logit > 0
   * (second[r]: the row's second best logit, hsd_lm_head_rank).  Ignored for
   * HSD_ACCEPT_DOTS. */
  int32_t spec_mode;
  int32_t spec_topk;   /* SPEC_TOPK, default 3 */
  float spec_margin;   /* SPEC_MARGIN, default 2.0 */
  const int32_t *rank; /* [q_len], HSD_SPEC_TOPK */
  const float *second; /* [q_len], HSD_SPEC_ADAPTIVE */
} hsd_accept_logits_t;

#define HSD_ACCEPT_DOTS 0
#define HSD_ACCEPT_HUNYUAN 1
#define HSD_SPEC_FMST 0
#define HSD_SPEC_TOPK 1
#define HSD_SPEC_ADAPTIVE 2

/* ---- library ---------------------------------------------------------- */
const char *hsd_version(void);
const char *hsd_last_error(void);

/* Self-test of the device-side failure path: one thread waits for
 * *flag == 1 (a device word nothing sets) with the same bounded wait every
 * kernel of this library uses, gives up after 1 s and writes
 * HSD_DEV_TIMEOUT | 0x7F0 into *status; the context stays usable.  Shows on
 * a device that a wait which cannot finish ends in an error code, not a
 * hang. */
int hsd_selftest_bounded_wait(const uint32_t *flag, int32_t *status, hsd_stream_t stream);

/* ---- (4) packing metadata ---------------------------------------------- */

/* Bytes of device workspace a plan for (q_len, kv_len) needs. */
size_t hsd_plan_workspace_bytes(int32_t q_len, int32_t kv_len);

/* Carve `plan` out of `workspace` (device memory, 256-byte aligned). */
int hsd_plan_init(void *workspace, size_t bytes, int32_t q_len, int32_t kv_len,
                  hsd_plan_t *plan);

/* Tile plan from segment descriptors; replaces create_block_mask(make_mask_mod(
 * dense mask), BLOCK_SIZE=(128,64)) (D:94-106, D:148-153, H:1213-1221) without
 * ever materialising the dense mask.  row_seg[q] is the segment of row q
 * (-1: no segment, row fully masked).  seg_kv_bits has kv_words_stride words
 * per segment. */
int hsd_build_plan_segments(const hsd_segment_t *segs, int32_t n_segs,
                            const int32_t *row_seg,
                            const uint64_t *seg_kv_bits, int32_t kv_words_stride,
                            const uint64_t *tree_bits, hsd_plan_t *plan,
                            int32_t *status, hsd_stream_t stream);

/* Tile plan from the reference's dense float mask [.., q_len, >=kv_len]
 * (allowed <=> value > -0.1, make_mask_mod D:148-153). */
int hsd_build_plan_dense(const float *mask, int64_t row_stride, hsd_plan_t *plan,
                         int32_t *status, hsd_stream_t stream);

/* ---- (1) packed verification attention ---------------------------------- */

/* Device workspace of the load-balanced (stream-K) attention schedule: per SM
 * of the current device and head slot, the bf16 partial rows of the piece
 * that continues an item begun by the previous SM, their ready flags, and a
 * launch generation.  Zero-fill it before first use. */
size_t hsd_attention_workspace_bytes(int32_t q_len, int32_t num_q_heads, int32_t num_kv_heads);

/* out = softmax(q k^T * scale + mask) v per query head with grouped KV heads,
 * lse = natural log-sum-exp; replaces flex_attention_forward (D:72-135,
 * H:103-180) including repeat_kv (D:137-146).  q: bf16 [num_q_heads][q_len]
 * [128] at the given element strides (row, head); k, v likewise with
 * num_kv_heads; out: bf16 [q_len][num_q_heads][128] contiguous (the
 * reference's transposed output, D:134); lse: fp32 [num_q_heads][q_len] or
 * NULL.  Fully masked rows give 0 and -inf.  head_dim must be 128.
 * workspace (256-byte aligned, hsd_attention_workspace_bytes) enables the
 * stream-K schedule -- one CTA per SM, equal shares of the tile plan's work;
 * the CTA holding the first blocks of a (query tile, head pair) item that the
 * shares cut merges the item's other pieces through the workspace.  The
 * workspace must be zero-filled before its first use; each call leaves it
 * ready for the next, and calls sharing one must not overlap in time.  With
 * workspace NULL each item gets its own CTA. */
int hsd_verify_attention(const void *q, int64_t q_row_stride, int64_t q_head_stride,
                         const void *k, int64_t k_row_stride, int64_t k_head_stride,
                         const void *v, int64_t v_row_stride, int64_t v_head_stride,
                         void *out, float *lse, int32_t q_len, int32_t kv_len,
                         int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                         float scale, const hsd_plan_t *plan, void *workspace,
                         size_t workspace_bytes, int32_t *status, hsd_stream_t stream);

/* No counterpart in the reference (it allocates through PyTorch on every
 * call).  hsd_verify_attention with the stream-K scratch taken from a static
 * device array of hsd_attention_static_scratch_bytes() bytes (20 MiB, enough
 * for devices of up to 310 SMs) instead of a caller workspace, so the call
 * allocates nothing: for bindings without a device allocator of their own,
 * and for serving loops that must not reach an allocator between steps.  The
 * first call on each device (that device current) looks up the array's
 * address -- make it before any stream capture.  A scratch need above the
 * array's size returns HSD_ERR_TOO_LARGE.  The array keeps the last call's
 * contents; each call first clears the flags and counters that must start at
 * zero (a few KB, on its stream).  One scratch per device: calls on one
 * device must not overlap on the GPU (one stream, or ordered by events), or
 * they race on it.  Other arguments as hsd_verify_attention. */
size_t hsd_attention_static_scratch_bytes(void);
int hsd_verify_attention_static_scratch(const void *q, int64_t q_row_stride,
                                        int64_t q_head_stride, const void *k,
                                        int64_t k_row_stride, int64_t k_head_stride,
                                        const void *v, int64_t v_row_stride,
                                        int64_t v_head_stride, void *out, float *lse,
                                        int32_t q_len, int32_t kv_len, int32_t num_q_heads,
                                        int32_t num_kv_heads, int32_t head_dim, float scale,
                                        const hsd_plan_t *plan, int32_t *status,
                                        hsd_stream_t stream);

/* ---- (2) KV-cache compaction -------------------------------------------- */

/* In place, for every plane p (one layer's K or V of one KV head, rows of
 * row_bytes contiguous bytes): row i <- row keep_idx[i] for i < n_keep.
 * keep_idx is ascending (so keep_idx[i] >= i); rows already in place are not
 * touched.  Replaces the per-layer index_select(-2, keep_indices) of
 * D:1705-1722 / H:2262-2269.  plane_ptrs: device array of n_planes addresses.
 * counts: device {n_keep, first_moved} as written by hsd_keep_indices (then
 * n_keep is ignored), or NULL to use the host n_keep from row 0. */
int hsd_compact_kv(const uint64_t *plane_ptrs, int32_t n_planes, int32_t row_bytes,
                   const int32_t *keep_idx, int32_t n_keep,
                   const int32_t *counts, int32_t *status, hsd_stream_t stream);

/* KV-cache append: for every plane p, rows [dst_row0, dst_row0 + n_rows) of
 * dst_planes[p] <- rows [0, n_rows) of src_planes[p] (row_bytes contiguous
 * bytes each).  The per-layer cache update the reference gets from
 * DynamicCache.update, a torch.cat along the sequence (D:356-359). */
int hsd_kv_append(const uint64_t *dst_planes, const uint64_t *src_planes, int32_t n_planes,
                  int32_t row_bytes, int32_t dst_row0, int32_t n_rows, hsd_stream_t stream);

/* keep = (OR of live_bits rows [0, n_live)) & ~filter_bits, then the ascending
 * indices of set bits (keep_idx), their count and the first index that moves
 * (D:1679-1707).  Counts land in counts[0] = n_keep, counts[1] = first_moved. */
int hsd_keep_indices(const uint64_t *live_bits, int32_t n_live, int32_t live_stride,
                     const uint64_t *filter_bits, int32_t kv_len,
                     uint64_t *keep_bits, int32_t *keep_idx, int32_t *counts,
                     hsd_stream_t stream);

/* Remap visibility rows after compaction: out[r] bit i = in[r] bit keep_idx[i]
 * (the mask's index_select(-1, keep) of D:1723), rows of `stride` words. */
int hsd_compact_bits(const uint64_t *in_bits, uint64_t *out_bits, int32_t n_rows,
                     int32_t stride, const int32_t *keep_idx, const int32_t *counts,
                     int32_t out_words, hsd_stream_t stream);

/* Rotary position embedding + cache update of one layer's new rows, one
 * launch.  Replaces transformers' apply_rotary_pos_emb on the query and key
 * states (D:345-346) and the DynamicCache.update torch.cat (D:348-351).
 * q: [n_rows][num_q_heads][128] bf16 at q_row_stride (the q_proj output),
 * rotated in place; k, v: [n_rows][num_kv_heads][128] at kv_row_stride (read
 * only); cos_emb, sin_emb: [n_rows][128] bf16 at cs_row_stride (the model's
 * position embeddings).  Rotated k rows and v rows go to rows
 * [dst_row0, dst_row0 + n_rows) of the caches (head h at
 * cache + h * head_stride, rows at cache_row_stride).  Arithmetic as torch's
 * bf16 ops: y = bf16(bf16(x * cos) + bf16(rotate_half(x) * sin)), so the
 * result is bit-identical.  num_q_heads may be 0 (keys and values only).
 * All strides in elements, multiples of 8; pointers 16-byte aligned. */
int hsd_rope_append(void *q, int64_t q_row_stride, const void *k, const void *v,
                    int64_t kv_row_stride, const void *cos_emb, const void *sin_emb,
                    int64_t cs_row_stride, int32_t n_rows, int32_t num_q_heads,
                    int32_t num_kv_heads, int32_t head_dim, void *k_cache,
                    int64_t k_cache_head_stride, void *v_cache, int64_t v_cache_head_stride,
                    int64_t cache_row_stride, int32_t dst_row0, hsd_stream_t stream);

/* ---- (3) acceptance + KMP re-alignment ----------------------------------- */

/* One warp per block: acceptance by mode (D:1107-1293, H:1633-1858 at
 * threshold >= 1), EOS / repetition stop (D:1299-1319), KMP re-alignment of
 * region blocks (compute_lps / kmp_search / find_all_matches_kmp, D:543-618,
 * call site D:1326-1336) and the window update.  next_ids = argmax of the
 * target model per packed row; input_ids = the packed input.  Appends the
 * accepted tokens to gen_pool, ORs rejected columns into filter_bits and
 * writes each block's new visibility (segment row | accepted path) to
 * out_kv_bits[b]. */
int hsd_accept_kmp(const hsd_accept_config_t *cfg, hsd_block_t *blocks,
                   hsd_block_result_t *results, const int32_t *next_ids,
                   const int32_t *input_ids, int32_t *gen_pool,
                   const int32_t *draft_pool, const int32_t *tree_tokens,
                   const int32_t *tree_parents, const uint64_t *seg_kv_bits,
                   uint64_t *out_kv_bits, uint64_t *filter_bits, int32_t *status,
                   hsd_stream_t stream);

/* hsd_accept_kmp with the logit-ratio rules (thresholds below 1; at 1 or
 * above, or logits == NULL, it equals hsd_accept_kmp).  A tree block's
 * result next_token stays next_ids of its last walked row
 * (next_token_int = group[new_index], D:1292); its generated token is the
 * fallback's choice. */
int hsd_accept_kmp_logits(const hsd_accept_config_t *cfg, hsd_block_t *blocks,
                          hsd_block_result_t *results, const int32_t *next_ids,
                          const int32_t *input_ids, int32_t *gen_pool,
                          const int32_t *draft_pool, const int32_t *tree_tokens,
                          const int32_t *tree_parents, const uint64_t *seg_kv_bits,
                          uint64_t *out_kv_bits, uint64_t *filter_bits,
                          const hsd_accept_logits_t *logits, int32_t *status,
                          hsd_stream_t stream);

/* Continuation tries of tree decoding, one CTA per tree.  Tree i: the draft
 * draft_pool[draft_off[i] .. + draft_len[i]) and the root token
 * last_tokens[i] (the match window's last token).  After every draft
 * position p holding the root token the next min(max_depth, len - 1 - p)
 * draft tokens are inserted (kmp_search's trie, D:573-586; children in
 * insertion order) and the trie is packed breadth-first, at most cap nodes
 * (D:1488-1543).  Outputs, row i at i * cap: tokens, depths, parents (-1
 * for the root) and counts[i] nodes; anc_bits[i][node][ceil(cap / 64)]: the
 * node and its ancestors, the tree's attention-mask rows (D:1506-1533).
 * cap <= 1024; more than 2048 root occurrences in one draft sets
 * HSD_DEV_CAPACITY and counts[i] = 0. */
int hsd_continuation_trees(const int32_t *draft_pool, const int32_t *draft_off,
                           const int32_t *draft_len, const int32_t *last_tokens,
                           int32_t n_trees, int32_t max_depth, int32_t cap, int32_t *tokens,
                           int32_t *depths, int32_t *parents, int32_t *counts,
                           uint64_t *anc_bits, int32_t *status, hsd_stream_t stream);

/* ---- (5) next tokens: fused lm_head + argmax ------------------------------ */

/* Workspace of hsd_lm_head_argmax: 8 bytes per row + 256, 256-byte aligned. */
size_t hsd_lm_head_argmax_workspace_bytes(int32_t q_len);

/* Next token of every packed row: argmax over the vocabulary of
 * hidden[q_len, hidden_dim] . weight[vocab, hidden_dim]^T (bf16 in, fp32
 * accumulation), each logit rounded to bf16 as the logits tensor holds it,
 * ties to the lowest id.  Replaces `logits = lm_head(hidden)` followed by
 * `logits.argmax(dim=-1)` (D:1057-1064) without writing the logits.  ids32
 * and/or ids64 receive the ids (one may be NULL); max_logit (nullable) the
 * maximal logit per row.  NaN logits never win (torch's argmax would return
 * a NaN's index).  The workspace must be zero-filled before its first use;
 * each call leaves it ready for the next (after an error status, zero it
 * again), and calls sharing one must not overlap in time.  Pointers 16-byte
 * aligned, row strides (elements) >= hidden_dim and multiples of 8. */
int hsd_lm_head_argmax(const void *hidden, int64_t hidden_row_stride, const void *weight,
                       int64_t weight_row_stride, int32_t q_len, int32_t vocab,
                       int32_t hidden_dim, int32_t *ids32, int64_t *ids64, float *max_logit,
                       void *workspace, size_t workspace_bytes, int32_t *status,
                       hsd_stream_t stream);

/* Second pass of the fused lm_head for HunYuan's SPEC_MODE=topk / adaptive
 * acceptance (H:1712-1736, which call logits.topk on the materialised bf16
 * logits): over the rows given (typically the last block's), with the
 * logits of each row rounded to bf16 as in hsd_lm_head_argmax and never
 * written,
 *   rank[r]   = #columns other than ref_col[r] whose logit exceeds
 *               probe_logit[r], plus #columns below ref_col[r] whose logit
 *               equals it (a NaN probe_logit[r] gives vocab - 1): the 0-based
 *               position of the draft token ref_col[r] in a descending order
 *               that puts lower columns first among equal logits (torch
 *               leaves that order unspecified); rank[r] < k <=> the token is
 *               among topk(k).indices;
 *   second[r] = the largest logit outside column excl_col[r] (the row's
 *               argmax), i.e. topk(2).values[1].
 * probe_logit[r] = logits[r, ref_col[r]] (hsd_probe_logits).  Same
 * workspace contract as hsd_lm_head_argmax (the two may share one). */
int hsd_lm_head_rank(const void *hidden, int64_t hidden_row_stride, const void *weight,
                     int64_t weight_row_stride, int32_t q_len, int32_t vocab, int32_t hidden_dim,
                     const float *probe_logit, const int32_t *ref_col, const int32_t *excl_col,
                     int32_t *rank, float *second, void *workspace, size_t workspace_bytes,
                     int32_t *status, hsd_stream_t stream);

/* Single logits of the logit-ratio acceptance: out[k] = logits[rows[k],
 * toks[k]] = hidden[rows[k]] . weight[toks[k]] (bf16 in, fp32 accumulation,
 * rounded to bf16 and returned as float), the entries the reference reads
 * from the logits tensor (D:1167-1168, D:1231-1232); toks[k] < 0 gives 0.
 * A row outside [0, q_len) or a token >= vocab writes NaN and sets
 * HSD_DEV_BAD_INDEX.  One warp per entry; rows 16-byte aligned, strides
 * (elements) multiples of 8, hidden_dim a multiple of 8. */
int hsd_probe_logits(const void *hidden, int64_t hidden_row_stride, const void *weight,
                     int64_t weight_row_stride, int32_t q_len, int32_t vocab,
                     int32_t hidden_dim, const int32_t *rows, const int32_t *toks, int32_t n,
                     float *out, int32_t *status, hsd_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* HSD_B200_H */
