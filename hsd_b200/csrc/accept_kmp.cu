// (3) Draft-target acceptance fused with KMP re-alignment: one warp per block.
//
// Restates, at HSD_SPEC_THRESH / HSD_TREE_THRESH >= 1 (exact match), the
// per-block body of the reference's verification loop
// (hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py):
//   normal 1-token step                 D:1107-1124
//   speculative longest accepted prefix D:1126-1213
//   tree walk                           D:1215-1293
//   EOS and repetition stop             D:1299-1319
//   KMP re-alignment (token mode)       D:1321-1336, window D:1121-1124
// The KMP scan of the reference (compute_lps / kmp_search, D:543-604) reports
// every occurrence of the window in the draft; the warp tests all candidate
// starts at once, which yields the same set (and so the same count and first
// start).  The continuation trie for tree mode is built by the host.
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
};

constexpr int kMaxTreeNodes = 1024;  // 32 lanes x 32 bits of "visited"

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
// (D:592-598).
__device__ void count_matches(const int32_t* text, int n, const int32_t* pat, int m, int lane,
                              int& count, int& first) {
  count = 0;
  first = -1;
  const int last_start = n - 1 - m;  // inclusive
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
}

__global__ void __launch_bounds__(128) accept_kmp_kernel(Params p) {
  const int lane = lane_id();
  const int b = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const hsd_accept_config_t& cfg = p.cfg;
  if (b >= cfg.n_blocks) return;
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
    res.finished = 3;
    if (lane == 0) p.results[b] = res;
    return;
  }
  const int stride = cfg.kv_words_stride;
  const int nwords = (cfg.kv_len + 63) / 64;
  const int kvb = cfg.kv_base;
  const int bs = blk.q_start, blen = blk.q_len;
  int32_t* gen = p.gen_pool + blk.gen_off;
  int glen = blk.gen_len;
  uint64_t* vis = p.out_kv_bits + size_t(b) * stride;
  const uint64_t* seg_row = p.seg_kv_bits + size_t(blk.seg) * stride;
  for (int w = lane; w < nwords; w += 32) vis[w] = seg_row[w];
  __syncwarp();

  int ptr, nxt, inc;
  uint32_t visited = 0;  // tree mode: bit k of lane l = node 32*l + k on the accepted path
  if (blk.mode == HSD_MODE_NORMAL) {
    ptr = bs + blk.valid_count - 1;
    nxt = p.next_ids[ptr];
    if (glen + 1 > blk.gen_cap) {
      report(p.status, HSD_DEV_CAPACITY | 1);
      return;
    }
    if (lane == 0) gen[glen] = nxt;
    glen += 1;
    inc = 1;
    or_range(vis, kvb + bs, kvb + ptr, lane, false);
  } else if (blk.mode == HSD_MODE_SPEC) {
    ptr = bs + blk.valid_count - 1;
    int diff = blen - 1;
    for (int base = 0; base < blen - 1; base += 32) {
      const int i = base + lane;
      const bool bad = (i < blen - 1) && (p.next_ids[bs + i] != p.input_ids[bs + i + 1]);
      const uint32_t bal = __ballot_sync(0xffffffffu, bad);
      if (bal) {
        diff = base + __ffs(bal) - 1;
        break;
      }
    }
    if (glen + diff + 1 > blk.gen_cap) {
      report(p.status, HSD_DEV_CAPACITY | 2);
      return;
    }
    nxt = p.next_ids[bs + diff];
    for (int i = lane; i <= diff; i += 32)
      gen[glen + i] = (i < diff) ? p.input_ids[bs + i + 1] : nxt;
    glen += diff + 1;
    inc = diff + 1;
    if (diff != blen - 1) {
      ptr = bs + diff;
      or_range(p.filter_bits, kvb + bs + diff + 1, kvb + bs + blen - 1, lane, true);
    }
    or_range(vis, kvb + bs, kvb + ptr, lane, false);
  } else if (blk.mode == HSD_MODE_TREE) {
    const int32_t* tok = p.tree_tokens + blk.tree_off;
    const int32_t* par = p.tree_parents + blk.tree_off;
    const int n = min(blk.tree_nodes, min(blen, kMaxTreeNodes));
    int decode = p.next_ids[bs];
    int node = 0, new_index = 0, walked = 0;
    if (lane == 0) visited |= 1u;
    // the walk appends 1 + walked tokens; reserve capacity up front
    if (glen + n > blk.gen_cap) {
      report(p.status, HSD_DEV_CAPACITY | 3);
      return;
    }
    if (lane == 0) gen[glen] = decode;
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
      new_index = child;
      decode = p.next_ids[bs + child];
      if (lane == 0) gen[glen] = decode;
      glen += 1;
      ++walked;
      if (lane == (child >> 5)) visited |= 1u << (child & 31);
    }
    ptr = bs + new_index;
    nxt = decode;
    inc = 1 + walked;
    // every column of the block off the accepted path is filtered (D:1271-1279)
    for (int j0 = 0; j0 < blen; j0 += 64) {
      // build the 64-column word for block columns [j0, j0+64) from the visited bits
      const uint32_t lo = __shfl_sync(0xffffffffu, visited, (j0 >> 5) & 31);
      const uint32_t hi = __shfl_sync(0xffffffffu, visited, ((j0 >> 5) + 1) & 31);
      uint64_t v = (j0 < kMaxTreeNodes) ? ((uint64_t(j0 + 32 < kMaxTreeNodes ? hi : 0) << 32) | lo)
                                        : 0ull;
      const int rem = blen - j0;
      const uint64_t span = rem >= 64 ? ~0ull : ((1ull << rem) - 1ull);
      const uint64_t dead = ~v & span, keep = v & span;
      if (lane == 0) {
        // columns kvb + bs + j0 + k, k < 64: may straddle two words
        const int c0 = kvb + bs + j0;
        const int w = c0 >> 6, sh = c0 & 63;
        if (dead) {
          atomicOr(reinterpret_cast<unsigned long long*>(p.filter_bits + w), dead << sh);
          if (sh && (dead >> (64 - sh)))
            atomicOr(reinterpret_cast<unsigned long long*>(p.filter_bits + w + 1),
                     dead >> (64 - sh));
        }
        if (keep) {
          vis[w] |= keep << sh;
          if (sh && (keep >> (64 - sh))) vis[w + 1] |= keep >> (64 - sh);
        }
      }
    }
  } else {
    report(p.status, HSD_DEV_BAD_INDEX | 3);
    return;
  }
  __syncwarp();

  // window update (D:1121-1124, D:1201-1204, D:1288-1291)
  int mws = (blk.matches_len == 0 || blk.matches_len == 1) ? cfg.match_window_size
                                                           : blk.mws + inc;
  res.increment = inc;
  res.pointer = ptr;
  res.next_token = nxt;

  // EOS stop (D:1299-1305): the pointer row's columns are filtered.
  const bool page_block = (blk.flags & 1) != 0;
  int finished = 0;
  if (is_eos(cfg, gen[glen - 1])) {
    finished = 1;
    glen -= 1;
  } else if (!page_block) {
    // repetition stop (D:1306-1319)
    const int tl = min(10, glen);
    int count, first;
    count_matches(gen, glen, gen + glen - tl, tl, lane, count, first);
    bool sentinel = false;
    for (int i = lane; i < glen; i += 32) sentinel |= (gen[i] == cfg.repeat_sentinel);
    sentinel = __any_sync(0xffffffffu, sentinel);
    if (count > 10 && !sentinel) {
      finished = 2;
      if (blk.draft_len > blk.gen_cap) {
        report(p.status, HSD_DEV_CAPACITY | 4);
        return;
      }
      __syncwarp();
      for (int i = lane; i < blk.draft_len; i += 32) gen[i] = p.draft_pool[blk.draft_off + i];
      glen = blk.draft_len;
    }
  }
  __syncwarp();
  if (finished) {
    for (int w = lane; w < nwords; w += 32)
      atomicOr(reinterpret_cast<unsigned long long*>(p.filter_bits + w), vis[w]);
    blk.mode = HSD_MODE_FINISHED;
  } else if (!page_block) {
    // KMP re-alignment (D:1321-1336)
    const int w = min(cfg.match_window_size_upper_bound, mws);
    const int wl = min(w, glen);
    int count, first;
    count_matches(p.draft_pool + blk.draft_off, blk.draft_len, gen + glen - wl, wl, lane, count,
                  first);
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
  if (lane == 0) {
    p.results[b] = res;
    p.blocks[b] = blk;
  }
}

}  // namespace acc
}  // namespace hsd

using namespace hsd;

extern "C" int hsd_accept_kmp(const hsd_accept_config_t* cfg, hsd_block_t* blocks,
                              hsd_block_result_t* results, const int32_t* next_ids,
                              const int32_t* input_ids, int32_t* gen_pool,
                              const int32_t* draft_pool, const int32_t* tree_tokens,
                              const int32_t* tree_parents, const uint64_t* seg_kv_bits,
                              uint64_t* out_kv_bits, uint64_t* filter_bits, int32_t* status,
                              hsd_stream_t stream) {
  if (!cfg || cfg->n_blocks <= 0 || !blocks || !results || !next_ids || !input_ids ||
      !gen_pool || !draft_pool || !seg_kv_bits || !out_kv_bits || !filter_bits ||
      cfg->kv_words_stride < (cfg->kv_len + 63) / 64 || cfg->n_eos < 0 || cfg->n_eos > 8 ||
      cfg->match_window_size_upper_bound <= 0 || cfg->match_window_size <= 0) {
    hsd_host::set_error("hsd_accept_kmp: bad arguments");
    return HSD_ERR_INVALID_ARG;
  }
  acc::Params p;
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
  const int threads = 128;
  const int grid = (cfg->n_blocks * 32 + threads - 1) / threads;
  acc::accept_kmp_kernel<<<grid, threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  return hsd_host::cuda_check(cudaGetLastError(), "accept_kmp_kernel launch");
}
