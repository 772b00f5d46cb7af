// (3) Draft-target acceptance fused with KMP re-alignment: one warp per block.
//
// Restates the per-block body of the reference's verification loop
// (hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py):
//   normal 1-token step                 D:1107-1124
//   speculative longest accepted prefix D:1126-1213 (logit ratio D:1147-1174)
//   tree walk                           D:1215-1293 (logit ratio D:1228-1238, D:1256-1266)
//   EOS and repetition stop             D:1299-1319
//   KMP re-alignment (token mode)       D:1321-1336, window D:1121-1124
// The KMP scan of the reference (compute_lps / kmp_search, D:543-604) reports
// every occurrence of the window in the draft; the warp tests all candidate
// starts at once, which yields the same set (and so the same count and first
// start).  The continuation tries for tree mode come packed as input
// (hsd_continuation_trees builds them on the device).
#include <cooperative_groups.h>

#include "common.cuh"

namespace hsd {
namespace acc {

struct Params {
  hsd_accept_config_t cfg;
  hsd_block_t* blocks;
  hsd_block_result_t* results;
  const int32_t* next_ids;
  const int32_t* input_ids;
  int32_t* gen_pool;
  const int32_t* draft_pool;
  const int32_t* tree_tokens;
  const int32_t* tree_parents;
  const uint64_t* seg_kv_bits;
  uint64_t* out_kv_bits;
  uint64_t* filter_bits;
  int32_t* status;
  // logit-ratio acceptance (off at the default thresholds >= 1)
  const float* max_logit;
  const float* probe_logit;
  float spec_thresh, tree_thresh;  // rounded to bf16
  int32_t spec_ratio, tree_ratio;
  int32_t hunyuan;            // HSD_ACCEPT_HUNYUAN rules
  int32_t formula[2];         // HunYuan formula delimiters
  int32_t spec_mode;          // HunYuan SPEC_MODE: HSD_SPEC_FMST / _TOPK / _ADAPTIVE
  int32_t spec_topk;
  float spec_margin;          // rounded to bf16
  const int32_t* rank;
  const float* second;
};

__device__ __forceinline__ bool is_formula(const Params& p, int tok) {
  return tok == p.formula[0] || tok == p.formula[1];
}

// torch's bf16 quotient: the float32 quotient rounded to bf16 (D:1171, D:1233).
__device__ __forceinline__ float logit_ratio(float num, float den) {
  return __bfloat162float(__float2bfloat16_rn(__fdiv_rn(num, den)));
}

// A speculative row that missed the exact match passes when the draft
// token's logit over the row's maximal logit reaches the threshold and the
// maximal logit is positive (D:1163-1174).
__device__ __forceinline__ bool spec_ratio_pass(const Params& p, int row) {
  const float pred = p.max_logit[row];
  if (p.spec_mode == HSD_SPEC_TOPK) return p.rank[row] < p.spec_topk;  // H:1712-1717
  const bool ratio = pred > 0.f && logit_ratio(p.probe_logit[row], pred) >= p.spec_thresh;
  if (p.spec_mode != HSD_SPEC_ADAPTIVE) return ratio;
  // H:1718-1733: top1 - top2 in bf16, compared with the bf16 margin
  const float margin = __bfloat162float(__float2bfloat16_rn(pred - p.second[row]));
  return ratio || (margin < p.spec_margin && p.probe_logit[row] > 0.f);
}

// Tree walk fallback (D:1228-1238, D:1256-1266, H:1791-1800, H:1821-1830):
// when the target's token
// `decode` is not a child of `node`, the child with the first maximal ratio
// logits[row, child] / logits[row, decode] (torch.argmax; a NaN ratio counts
// as maximal) replaces it, if any ratio reaches the threshold.  Children are
// the packed nodes with parent `node`, in BFS (insertion) order.
__device__ int tree_ratio_fallback(const Params& p, int bs, int node, int decode,
                                   const int32_t* tok, const int32_t* par, int n, int lane) {
  for (int base = node + 1; base < n; base += 32) {
    const int c = base + lane;
    if (__any_sync(0xffffffffu, c < n && par[c] == node && tok[c] == decode)) return decode;
  }
  const float den = p.max_logit[bs + node];
  bool pass = false;
  int nan_c = -1, best_c = -1;
  float best = 0.f;
  for (int base = node + 1; base < n; base += 32) {
    const int c = base + lane;
    const bool kid = c < n && par[c] == node;
    const float r = kid ? logit_ratio(p.probe_logit[bs + c], den) : 0.f;
    pass |= __any_sync(0xffffffffu, kid && r >= p.tree_thresh);
    const uint32_t nb = __ballot_sync(0xffffffffu, kid && isnan(r));
    if (nan_c < 0 && nb) nan_c = base + __ffs(nb) - 1;
    if (kid && !isnan(r) && (best_c < 0 || r > best)) {
      best = r;
      best_c = c;
    }
  }
  if (!pass) return decode;
  if (nan_c >= 0) return tok[nan_c];
  for (int off = 16; off; off >>= 1) {  // maximal ratio, lowest index among equals
    const float ob = __shfl_xor_sync(0xffffffffu, best, off);
    const int oc = __shfl_xor_sync(0xffffffffu, best_c, off);
    if (oc >= 0 && (best_c < 0 || ob > best || (ob == best && oc < best_c))) {
      best = ob;
      best_c = oc;
    }
  }
  return tok[best_c];
}


__device__ __forceinline__ uint64_t word_range(int w, int lo, int hi) {  // [lo, hi]
  const int a = max(lo, 64 * w), b = min(hi, 64 * w + 63);
  if (a > b) return 0;
  const int n = b - a + 1;
  return ((n >= 64) ? ~0ull : ((1ull << n) - 1ull)) << (a - 64 * w);
}

// OR columns [lo, hi] into a bit row (atomic: blocks share filter words).
__device__ void or_range(uint64_t* bits, int lo, int hi, int lane, bool atomic) {
  if (lo > hi) return;
  for (int w = (lo >> 6) + lane; w <= (hi >> 6); w += 32) {
    const uint64_t m = word_range(w, lo, hi);
    if (atomic)
      atomicOr(reinterpret_cast<unsigned long long*>(bits + w), m);
    else
      bits[w] |= m;
  }
}

__device__ __forceinline__ bool is_eos(const hsd_accept_config_t& c, int tok) {
  bool r = false;
  for (int i = 0; i < c.n_eos && i < 8; ++i) r |= (c.eos_ids[i] == tok);
  return r;
}

// Number of starts s (ascending) with text[s, s+m) == pat and s + m <= n - 1,
// and the first such s (-1 if none) -- the matches find_all_matches_kmp keeps
// (D:592-598).  Lane i tests start base + i.  For m <= 32 the pattern sits in
// the lanes and each round of 32 starts needs one new coalesced load of the
// text (lane i holds text[base + i] and text[base + 32 + i]; text[s + k] is
// a shuffle), the next round's load issued before this round's compares.
__device__ void count_matches(const int32_t* text, int n, const int32_t* pat, int m, int lane,
                              int& count, int& first) {
  count = 0;
  first = -1;
  const int last_start = n - 1 - m;  // inclusive
  if (last_start < 0) return;
  if (m > 32) {
    for (int base = 0; base <= last_start; base += 32) {
      const int s = base + lane;
      bool hit = false;
      if (s <= last_start) {
        hit = true;
        for (int k = 0; k < m; ++k)
          if (text[s + k] != pat[k]) {
            hit = false;
            break;
          }
      }
      const uint32_t bal = __ballot_sync(0xffffffffu, hit);
      if (bal && first < 0) first = base + __ffs(bal) - 1;
      count += __popc(bal);
    }
    return;
  }
  const int pk = lane < m ? pat[lane] : 0;
  int t0 = lane < n ? text[lane] : 0;
  int t1 = 32 + lane < n ? text[32 + lane] : 0;
  for (int base = 0; base <= last_start; base += 32) {
    const int s = base + lane;
    const int t2 = s + 64 < n ? text[s + 64] : 0;  // the next round's second half
    bool hit = s <= last_start;
    for (int k = 0; k < m; ++k) {  // every lane takes part in every shuffle
      const int src = (lane + k) & 31;
      const int a0 = __shfl_sync(0xffffffffu, t0, src);
      const int a1 = __shfl_sync(0xffffffffu, t1, src);
      const int pv = __shfl_sync(0xffffffffu, pk, k);
      hit &= (lane + k < 32 ? a0 : a1) == pv;
    }
    const uint32_t bal = __ballot_sync(0xffffffffu, hit);
    if (bal && first < 0) first = base + __ffs(bal) - 1;
    count += __popc(bal);
    t0 = t1;
    t1 = t2;
  }
}

// The reference updates one filter mask block after block: a speculative
// block sets its rejected columns (D:1196-1200), a tree block sets its walked
// path and then inverts its column range (D:1266-1286), a finished block ORs
// in its pointer row's visibility (D:1299-1319).  Setting bits commutes with
// setting bits, so the rejected columns and tree paths go straight into the
// filter words (atomics on masked words: neighbours may share a word).  Only
// the inversions and the finished rows depend on the block order (a row may
// reach another block's columns); each block records those two as a
// FilterRec and one thread per filter word replays them in block order at
// the end.
struct FilterRec {
  int32_t lo, hi;    // inverted columns [lo, hi] (none if lo > hi)
  int32_t finished;  // OR the block's visibility row
};

__device__ __forceinline__ void filter_or(unsigned long long* f, int lo, int hi, int lane) {
  if (lo > hi) return;
  for (int w = (lo >> 6) + lane; w <= (hi >> 6); w += 32) atomicOr(f + w, word_range(w, lo, hi));
}

// One thread-block cluster; warp w of the cluster (CTA rank x warps per CTA
// + warp) handles blocks w, w + cluster warps, ... in parallel.  The blocks'
// commuting filter updates are atomic ORs on the filter words in global
// memory; one FilterRec per block lives in the first CTA's dynamic shared
// memory, which the others reach through distributed shared memory (plain
// stores), and the first CTA replays the order-dependent updates.
__global__ void __launch_bounds__(1024) accept_kmp_kernel(Params p) {
  pdl_wait_then_release();  // launched with launch_pdl
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ uint8_t smem_raw[];
  const bool leader = cluster.block_rank() == 0;
  uint8_t* lead = cluster.map_shared_rank(smem_raw, 0);
  unsigned long long* filt = reinterpret_cast<unsigned long long*>(p.filter_bits);
  const int lane = lane_id();
  const int nwarps = blockDim.x >> 5;
  const int cwarps = nwarps * int(cluster.num_blocks());
  const hsd_accept_config_t& cfg = p.cfg;
  const int stride = cfg.kv_words_stride;
  const int nwords = (cfg.kv_len + 63) / 64;
  const int kvb = cfg.kv_base;
  FilterRec* recs = reinterpret_cast<FilterRec*>(lead);
  cluster.sync();  // every CTA of the cluster runs before any reaches the first one's memory
  for (int b = int(cluster.block_rank()) * nwarps + warp_id(); b < cfg.n_blocks; b += cwarps) {
    if (lane == 0) recs[b] = FilterRec{1, 0, 0};
    hsd_block_t blk = p.blocks[b];
    hsd_block_result_t res;
    res.finished = 0;
    res.increment = 0;
    res.pointer = -1;
    res.next_token = -1;
    res.match_count = 0;
    res.match_start = -1;
    res.slice_begin = -1;
    res.slice_end = -1;
    if (blk.mode == HSD_MODE_FINISHED) {
      // a block finished in an earlier step sees nothing any more
      uint64_t* dead = p.out_kv_bits + size_t(b) * stride;
      for (int w = lane; w < nwords; w += 32) dead[w] = 0;
      res.finished = 3;
      if (lane == 0) p.results[b] = res;
      continue;
    }
    const int bs = blk.q_start, blen = blk.q_len;
    int32_t* gen = p.gen_pool + blk.gen_off;
    int glen = blk.gen_len;
    uint64_t* vis = p.out_kv_bits + size_t(b) * stride;
    const uint64_t* seg_row = p.seg_kv_bits + size_t(blk.seg) * stride;
    for (int w = lane; w < nwords; w += 32) vis[w] = seg_row[w];
    __syncwarp();

    int ptr = bs, nxt = 0, inc = 0;
    bool bad = false;
    if (blk.mode == HSD_MODE_NORMAL) {
      ptr = bs + blk.valid_count - 1;
      nxt = p.next_ids[ptr];
      if (glen + 1 > blk.gen_cap) {
        bad = true;
      } else {
        if (lane == 0) gen[glen] = nxt;
        glen += 1;
        inc = 1;
        or_range(vis, kvb + bs, kvb + ptr, lane, false);
      }
    } else if (blk.mode == HSD_MODE_SPEC) {
      ptr = bs + blk.valid_count - 1;
      int diff = blen - 1;
      // dots: every block (D:1147-1174); HunYuan: the last block only (H:1671)
      const bool ratio = p.spec_ratio && (!p.hunyuan || b == cfg.n_blocks - 1);
      // HunYuan formula state before the block's draft (H:1683-1688): the
      // parity of delimiters among the generated tokens
      int in_formula = 0;
      if (ratio && p.hunyuan) {
        int cnt = 0;
        for (int i = lane; i < glen; i += 32) cnt += is_formula(p, gen[i]);
        for (int off = 16; off; off >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, off);
        in_formula = cnt & 1;
      }
      for (int base = 0; base < blen - 1; base += 32) {
        const int i = base + lane;
        bool can_ratio = ratio;
        if (ratio && p.hunyuan) {
          // row i may use the ratio unless its draft token is a delimiter or
          // the delimiters up to it leave a formula open (H:1689-1695)
          const bool dollar = i < blen && is_formula(p, p.input_ids[bs + i]);
          const uint32_t dm = __ballot_sync(0xffffffffu, dollar);
          const int upto = in_formula + __popc(dm & (0xffffffffu >> (31 - lane)));
          in_formula = (in_formula + __popc(dm)) & 1;
          can_ratio = !dollar && !(upto & 1);
        }
        const bool miss = (i < blen - 1) && (p.next_ids[bs + i] != p.input_ids[bs + i + 1]) &&
                          !(can_ratio && spec_ratio_pass(p, bs + i));
        const uint32_t bal = __ballot_sync(0xffffffffu, miss);
        if (bal) {
          diff = base + __ffs(bal) - 1;
          break;
        }
      }
      if (glen + diff + 1 > blk.gen_cap) {
        bad = true;
      } else {
        nxt = p.next_ids[bs + diff];
        // accepted rows keep the draft's tokens (D:1184-1186); HunYuan keeps
        // the model's (H:1750-1754)
        for (int i = lane; i <= diff; i += 32)
          gen[glen + i] = (i < diff && !p.hunyuan) ? p.input_ids[bs + i + 1] : p.next_ids[bs + i];
        glen += diff + 1;
        inc = diff + 1;
        if (diff != blen - 1) {
          ptr = bs + diff;
          filter_or(filt, kvb + bs + diff + 1, kvb + bs + blen - 1, lane);  // rejected rows
        }
        or_range(vis, kvb + bs, kvb + ptr, lane, false);
      }
    } else if (blk.mode == HSD_MODE_TREE) {
      const int32_t* tok = p.tree_tokens + blk.tree_off;
      const int32_t* par = p.tree_parents + blk.tree_off;
      const int n = min(blk.tree_nodes, blen);
      const bool ratio = p.tree_ratio && (blk.flags & 2);
      int decode = p.next_ids[bs];
      int node = 0, walked = 0;
      if (glen + n > blk.gen_cap) {
        bad = true;
      } else {
        if (ratio) decode = tree_ratio_fallback(p, bs, 0, decode, tok, par, n, lane);
        if (lane == 0) {
          gen[glen] = decode;
          // the visited path (root first) is kept: set here, inverted below
          const int c = kvb + bs;
          atomicOr(filt + (c >> 6), 1ull << (c & 63));
          vis[c >> 6] |= 1ull << (c & 63);
        }
        glen += 1;
        for (int guard = 0; guard < n; ++guard) {
          int child = -1;
          for (int base = node + 1; base < n; base += 32) {
            const int c = base + lane;
            const bool hit = c < n && par[c] == node && tok[c] == decode;
            const uint32_t bal = __ballot_sync(0xffffffffu, hit);
            if (bal) {
              child = base + __ffs(bal) - 1;
              break;
            }
          }
          if (child < 0) break;
          node = child;
          decode = p.next_ids[bs + child];
          if (ratio) decode = tree_ratio_fallback(p, bs, child, decode, tok, par, n, lane);
          if (lane == 0) {
            gen[glen] = decode;
            const int c = kvb + bs + child;
            atomicOr(filt + (c >> 6), 1ull << (c & 63));
            vis[c >> 6] |= 1ull << (c & 63);
          }
          glen += 1;
          ++walked;
        }
        ptr = bs + node;
        nxt = p.next_ids[bs + node];  // next_token_int = group[new_index] (D:1292)
        inc = 1 + walked;
        if (lane == 0) {  // unvisited nodes filtered: the range is inverted
          recs[b].lo = kvb + bs;
          recs[b].hi = kvb + bs + blen - 1;
        }
      }
    } else {
      bad = true;
    }
    if (bad) {
      report(p.status, HSD_DEV_CAPACITY | 1);
      continue;
    }
    __syncwarp();

    // window update (D:1121-1124, D:1201-1204, D:1288-1291)
    const int mws = (blk.matches_len == 0 || blk.matches_len == 1) ? cfg.match_window_size
                                                                   : blk.mws + inc;
    res.increment = inc;
    res.pointer = ptr;
    res.next_token = nxt;

    // EOS stop (D:1299-1305) and repetition stop (D:1306-1319); the block's
    // visibility row joins the filter.
    const bool page_block = (blk.flags & 1) != 0;
    int finished = 0;
    if (is_eos(cfg, gen[glen - 1])) {
      finished = 1;
      glen -= 1;
    } else if (!page_block) {
      const int tl = min(10, glen);
      int count, first;
      count_matches(gen, glen, gen + glen - tl, tl, lane, count, first);
      bool sentinel = false;
      for (int i = lane; i < glen; i += 32) sentinel |= (gen[i] == cfg.repeat_sentinel);
      sentinel = __any_sync(0xffffffffu, sentinel);
      if (count > 10 && !sentinel) {
        if (blk.draft_len > blk.gen_cap) {
          report(p.status, HSD_DEV_CAPACITY | 4);
        } else {
          finished = 2;
          __syncwarp();
          for (int i = lane; i < blk.draft_len; i += 32) gen[i] = p.draft_pool[blk.draft_off + i];
          glen = blk.draft_len;
        }
      }
    }
    __syncwarp();
    if (finished) {
      if (lane == 0) recs[b].finished = 1;
      blk.mode = HSD_MODE_FINISHED;
    } else if (!page_block) {
      // KMP re-alignment (D:1321-1336)
      const int w = min(cfg.match_window_size_upper_bound, mws);
      const int wl = min(w, glen);
      int count, first;
      count_matches(p.draft_pool + blk.draft_off, blk.draft_len, gen + glen - wl, wl, lane,
                    count, first);
      res.match_count = count;
      res.match_start = first;
      blk.matches_len = count;
      if (count == 1) {
        res.slice_begin = first + wl - 1;
        int end = blk.draft_len;
        if (cfg.max_spec_len > 0 && end - res.slice_begin > cfg.max_spec_len)
          end = res.slice_begin + cfg.max_spec_len;
        res.slice_end = end;
      }
    }
    res.finished = finished;
    blk.gen_len = glen;
    blk.mws = mws;
    __syncwarp();
    if (lane == 0) {
      p.results[b] = res;
      p.blocks[b] = blk;
    }
  }
  cluster.sync();
  if (!leader) return;
  // Order-dependent updates, per word in block order (the visibility rows
  // are complete: every warp of the cluster passed the barrier after writing
  // its own).
  for (int w = threadIdx.x; w < nwords; w += blockDim.x) {
    uint64_t v = __ldcg(p.filter_bits + w);
    for (int b = 0; b < cfg.n_blocks; ++b) {
      const FilterRec r = recs[b];
      if (r.lo <= r.hi && (r.lo >> 6) <= w && w <= (r.hi >> 6)) v ^= word_range(w, r.lo, r.hi);
      if (r.finished) v |= __ldcg(p.out_kv_bits + size_t(b) * stride + w);  // other SMs wrote it
    }
    p.filter_bits[w] = v;
  }
}

}  // namespace acc
}  // namespace hsd

using namespace hsd;

static constexpr int kMaxBlocks = 1024;

static int accept_launch(const hsd_accept_config_t* cfg, hsd_block_t* blocks,
                         hsd_block_result_t* results, const int32_t* next_ids,
                         const int32_t* input_ids, int32_t* gen_pool, const int32_t* draft_pool,
                         const int32_t* tree_tokens, const int32_t* tree_parents,
                         const uint64_t* seg_kv_bits, uint64_t* out_kv_bits,
                         uint64_t* filter_bits, const hsd_accept_logits_t* logits,
                         int32_t* status, hsd_stream_t stream) {
  if (!cfg || cfg->n_blocks <= 0 || !blocks || !results || !next_ids || !input_ids ||
      !gen_pool || !draft_pool || !seg_kv_bits || !out_kv_bits || !filter_bits ||
      cfg->kv_words_stride < (cfg->kv_len + 63) / 64 || cfg->n_eos < 0 || cfg->n_eos > 8 ||
      cfg->match_window_size_upper_bound <= 0 || cfg->match_window_size <= 0) {
    hsd_host::set_error("hsd_accept_kmp: bad arguments");
    return HSD_ERR_INVALID_ARG;
  }
  if (logits && logits->variant != HSD_ACCEPT_DOTS && logits->variant != HSD_ACCEPT_HUNYUAN) {
    hsd_host::set_error("hsd_accept_kmp_logits: unknown variant %d", logits->variant);
    return HSD_ERR_INVALID_ARG;
  }
  const bool hunyuan = logits && logits->variant == HSD_ACCEPT_HUNYUAN;
  const bool spec_ratio = logits && logits->spec_thresh < 1.0f;
  // HunYuan's tree fallback has no `< 1` guard (H:1791, H:1821)
  const bool tree_ratio = logits && (hunyuan || logits->tree_thresh < 1.0f);
  if ((spec_ratio || tree_ratio) && (!logits->max_logit || !logits->probe_logit)) {
    hsd_host::set_error("hsd_accept_kmp_logits: a threshold below 1 needs max_logit and "
                        "probe_logit");
    return HSD_ERR_INVALID_ARG;
  }
  const int spec_mode = hunyuan ? logits->spec_mode : HSD_SPEC_FMST;
  if (spec_mode != HSD_SPEC_FMST && spec_mode != HSD_SPEC_TOPK &&
      spec_mode != HSD_SPEC_ADAPTIVE) {
    hsd_host::set_error("hsd_accept_kmp_logits: unknown spec_mode %d", spec_mode);
    return HSD_ERR_INVALID_ARG;
  }
  if (spec_ratio && ((spec_mode == HSD_SPEC_TOPK && !logits->rank) ||
                     (spec_mode == HSD_SPEC_ADAPTIVE && !logits->second))) {
    hsd_host::set_error("hsd_accept_kmp_logits: spec_mode %d needs %s", spec_mode,
                        spec_mode == HSD_SPEC_TOPK ? "rank" : "second");
    return HSD_ERR_INVALID_ARG;
  }
  acc::Params p;
  p.max_logit = logits ? logits->max_logit : nullptr;
  p.probe_logit = logits ? logits->probe_logit : nullptr;
  p.spec_ratio = spec_ratio;
  p.tree_ratio = tree_ratio;
  // the reference compares bf16 ratios with the threshold rounded to bf16
  p.spec_thresh = spec_ratio ? __bfloat162float(__float2bfloat16_rn(logits->spec_thresh)) : 1.f;
  p.tree_thresh = tree_ratio ? __bfloat162float(__float2bfloat16_rn(logits->tree_thresh)) : 1.f;
  p.hunyuan = hunyuan;
  p.formula[0] = hunyuan ? logits->formula_tokens[0] : -1;
  p.formula[1] = hunyuan ? logits->formula_tokens[1] : -1;
  p.spec_mode = spec_ratio ? spec_mode : HSD_SPEC_FMST;
  p.spec_topk = spec_mode == HSD_SPEC_TOPK ? logits->spec_topk : 0;
  p.spec_margin = spec_mode == HSD_SPEC_ADAPTIVE
                      ? __bfloat162float(__float2bfloat16_rn(logits->spec_margin))
                      : 0.f;
  p.rank = spec_mode == HSD_SPEC_TOPK ? logits->rank : nullptr;
  p.second = spec_mode == HSD_SPEC_ADAPTIVE ? logits->second : nullptr;
  p.cfg = *cfg;
  p.blocks = blocks;
  p.results = results;
  p.next_ids = next_ids;
  p.input_ids = input_ids;
  p.gen_pool = gen_pool;
  p.draft_pool = draft_pool;
  p.tree_tokens = tree_tokens;
  p.tree_parents = tree_parents;
  p.seg_kv_bits = seg_kv_bits;
  p.out_kv_bits = out_kv_bits;
  p.filter_bits = filter_bits;
  p.status = status;
  if (cfg->n_blocks > kMaxBlocks) {
    hsd_host::set_error("hsd_accept_kmp: %d blocks > %d", cfg->n_blocks, kMaxBlocks);
    return HSD_ERR_TOO_LARGE;
  }
  // up to 32 blocks per CTA, up to 8 CTAs in the cluster (beyond 256 blocks
  // the warps take several blocks each)
  const int ctas = (cfg->n_blocks + 31) / 32 < 8 ? (cfg->n_blocks + 31) / 32 : 8;
  const int per_cta = (cfg->n_blocks + ctas - 1) / ctas;
  const int warps = per_cta < 32 ? per_cta : 32;
  // one FilterRec per block (at most 12 KB: within the default limit)
  const size_t smem = size_t(cfg->n_blocks) * sizeof(acc::FilterRec);
  return hsd_host::launch_pdl(acc::accept_kmp_kernel, dim3(unsigned(ctas)),
                              dim3(unsigned(warps * 32)), smem,
                              reinterpret_cast<cudaStream_t>(stream), "accept_kmp_kernel launch",
                              unsigned(ctas), p);
}

extern "C" int hsd_accept_kmp(const hsd_accept_config_t* cfg, hsd_block_t* blocks,
                              hsd_block_result_t* results, const int32_t* next_ids,
                              const int32_t* input_ids, int32_t* gen_pool,
                              const int32_t* draft_pool, const int32_t* tree_tokens,
                              const int32_t* tree_parents, const uint64_t* seg_kv_bits,
                              uint64_t* out_kv_bits, uint64_t* filter_bits, int32_t* status,
                              hsd_stream_t stream) {
  return accept_launch(cfg, blocks, results, next_ids, input_ids, gen_pool, draft_pool,
                       tree_tokens, tree_parents, seg_kv_bits, out_kv_bits, filter_bits, nullptr,
                       status, stream);
}

extern "C" int hsd_accept_kmp_logits(const hsd_accept_config_t* cfg, hsd_block_t* blocks,
                                     hsd_block_result_t* results, const int32_t* next_ids,
                                     const int32_t* input_ids, int32_t* gen_pool,
                                     const int32_t* draft_pool, const int32_t* tree_tokens,
                                     const int32_t* tree_parents, const uint64_t* seg_kv_bits,
                                     uint64_t* out_kv_bits, uint64_t* filter_bits,
                                     const hsd_accept_logits_t* logits, int32_t* status,
                                     hsd_stream_t stream) {
  return accept_launch(cfg, blocks, results, next_ids, input_ids, gen_pool, draft_pool,
                       tree_tokens, tree_parents, seg_kv_bits, out_kv_bits, filter_bits, logits,
                       status, stream);
}
