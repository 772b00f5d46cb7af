// (4) Packing metadata on the device.
//
// Replaces the reference's per-step dense mask build + create_block_mask
// (D:94-106 with make_mask_mod D:148-153; H:1213-1221): from segment
// descriptors (or, for drop-in use, from the dense float mask) it writes
//   * the 64-bit row masks of every 128x64 tile (tile-major, 1 KB per tile),
//   * the tile classes (empty / partial / full) and FlexAttention-style
//     ascending partial / full index lists per 128-row query tile,
//   * the list of 128-column KV blocks the attention kernel visits, with a
//     present/partial flag per 64-column half,
//   * a query-tile order, most blocks first, for the attention grid.
// Padding rows (>= q_len) and padding columns (>= kv_len) are never allowed,
// exactly as create_block_mask pads its tiles.
#include "common.cuh"

namespace hsd {
namespace meta {

struct SegSource {
  const hsd_segment_t* segs;
  const int32_t* row_seg;
  const uint64_t* seg_kv_bits;
  const uint64_t* tree_bits;
  int32_t stride;  // words per seg_kv_bits row
  int32_t q_len, kv_len, kv_base, n_segs;
  int32_t* status;
};

// Bits of columns [lo, hi] (inclusive) that fall into word t.
__device__ __forceinline__ uint64_t range_bits(int t, int lo, int hi) {
  const int a = max(lo, 64 * t), b = min(hi, 64 * t + 63);
  if (a > b) return 0;
  const int n = b - a + 1;
  const uint64_t m = (n >= 64) ? ~0ull : ((1ull << n) - 1ull);
  return m << (a - 64 * t);
}

// 64 bits of a packed bit row starting at bit `off` (may be negative).
__device__ __forceinline__ uint64_t extract64(const uint64_t* row, int nwords, int off) {
  if (off <= -64) return 0;
  if (off < 0) return nwords > 0 ? (row[0] << (-off)) : 0;
  const int wi = off >> 6, sh = off & 63;
  const uint64_t lo = wi < nwords ? row[wi] : 0;
  if (sh == 0) return lo;
  const uint64_t hi = wi + 1 < nwords ? row[wi + 1] : 0;
  return (lo >> sh) | (hi << (64 - sh));
}

__device__ __forceinline__ uint64_t clip_word(uint64_t w, int t, int kv_len) {
  const int rem = kv_len - 64 * t;
  if (rem <= 0) return 0;
  if (rem < 64) w &= (1ull << rem) - 1ull;
  return w;
}

// A packed row's segment, looked up once per row (row_seg, then the
// descriptor) so that the per-word loop has one load per word.
struct RowSeg {
  int s;  // segment, < 0: the row sees nothing
  hsd_segment_t seg;
};

__device__ __forceinline__ RowSeg row_segment(const SegSource& S, int q) {
  RowSeg r;
  r.s = -1;
  if (q >= S.q_len) return r;
  const int s = S.row_seg[q];
  if (s < 0) return r;
  if (s >= S.n_segs) {
    report(S.status, HSD_DEV_BAD_INDEX | 1);
    return r;
  }
  r.s = s;
  r.seg = S.segs[s];
  return r;
}

__device__ __forceinline__ uint64_t seg_row_word(const SegSource& S, const RowSeg& rs, int q,
                                                 int t) {
  if (rs.s < 0) return 0;
  const int s = rs.s;
  const hsd_segment_t& seg = rs.seg;
  uint64_t w = S.seg_kv_bits[size_t(s) * S.stride + t];
  const int i = q - seg.q_start;
  const int lo = S.kv_base + seg.q_start;
  if (seg.kind == HSD_SEG_CAUSAL) {
    w |= range_bits(t, lo, lo + i);
  } else if (seg.kind == HSD_SEG_SINGLE) {
    if (i == 0) w |= range_bits(t, lo, lo);
  } else if (seg.kind == HSD_SEG_TREE) {
    const int off = 64 * t - lo;
    if (off > -64 && off < seg.q_len && i >= 0 && i < seg.q_len) {
      const uint64_t* row = S.tree_bits + seg.tree_off + size_t(i) * seg.tree_words;
      uint64_t a = extract64(row, seg.tree_words, off);
      // nodes beyond the segment are not its columns
      const int span = seg.q_len - off;  // nodes available from bit 0 of this word
      if (span < 64) a &= (span <= 0) ? 0ull : ((1ull << span) - 1ull);
      w |= a;
    }
  }
  return clip_word(w, t, S.kv_len);
}

__device__ __forceinline__ uint64_t warp_and64(uint64_t v) {
  uint32_t lo = __reduce_and_sync(0xffffffffu, uint32_t(v));
  uint32_t hi = __reduce_and_sync(0xffffffffu, uint32_t(v >> 32));
  return (uint64_t(hi) << 32) | lo;
}
__device__ __forceinline__ uint64_t warp_or64(uint64_t v) {
  uint32_t lo = __reduce_or_sync(0xffffffffu, uint32_t(v));
  uint32_t hi = __reduce_or_sync(0xffffffffu, uint32_t(v >> 32));
  return (uint64_t(hi) << 32) | lo;
}

// Row words and tile classes: CTA (qt, part) covers query tile qt's 64-column
// tiles part, part + parts, ...; a warp per tile, each lane 4 rows.
// kFromSegments: compute the row words from segment descriptors and store
// them; otherwise read the words the dense kernel stored.
template <bool kFromSegments>
__global__ void __launch_bounds__(256) classify_kernel(SegSource S, hsd_plan_t P) {
  pdl_wait_then_release();  // launched with launch_pdl
  const int qt = blockIdx.x;
  const int parts = gridDim.y;
  const int warp = warp_id(), lane = lane_id();
  const int n64 = P.n_kv64;
  uint64_t* words = P.mask_words + size_t(qt) * n64 * 128;
  uint8_t* gcls = P.tile_class + size_t(qt) * n64;
  // lane's rows: lane + 32 k, their segments looked up once
  RowSeg rs[4];
  if (kFromSegments) {
#pragma unroll
    for (int k = 0; k < 4; ++k) rs[k] = row_segment(S, qt * 128 + lane + 32 * k);
  }
  for (int t = int(blockIdx.y) + parts * warp; t < n64; t += parts * 8) {
    uint64_t acc_and = ~0ull, acc_or = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int r = lane + 32 * k;
      const int q = qt * 128 + r;
      uint64_t w;
      if (kFromSegments) {
        w = seg_row_word(S, rs[k], q, t);
        words[size_t(t) * 128 + r] = w;
      } else {
        w = (q < P.q_len) ? words[size_t(t) * 128 + r] : 0ull;
      }
      acc_and &= w;
      acc_or |= w;
    }
    acc_and = warp_and64(acc_and);
    acc_or = warp_or64(acc_or);
    if (lane == 0) gcls[t] = acc_or == 0 ? 0 : (acc_and == ~0ull ? 2 : 1);
  }
}

// One CTA: a warp per query tile turns its tile classes into the
// FlexAttention-style ascending partial / full lists and the 128-column block
// list; then the query tiles are ranked by descending block count (ties:
// lower tile first), so the attention grid starts the longest tiles first,
// with the exclusive prefix of block counts in that order (the work offsets
// of the stream-K schedule).
__global__ void __launch_bounds__(1024) order_kernel(hsd_plan_t P) {
  pdl_wait_then_release();  // launched with launch_pdl
  __shared__ int cnt_sorted[1024];
  const int n = P.n_qtiles;
  const int n64 = P.n_kv64;
  const int warp = warp_id(), lane = lane_id(), nwarps = blockDim.x >> 5;
  for (int qt = warp; qt < n; qt += nwarps) {
    const uint8_t* cls = P.tile_class + size_t(qt) * n64;
    int n_part = 0, n_full = 0;
    int32_t* kvi = P.kv_indices + size_t(qt) * n64;
    int32_t* fvi = P.full_kv_indices + size_t(qt) * n64;
    for (int base = 0; base < n64; base += 32) {
      const int t = base + lane;
      const int c = t < n64 ? cls[t] : 0;
      const uint32_t bp = __ballot_sync(0xffffffffu, c == 1);
      const uint32_t bf = __ballot_sync(0xffffffffu, c == 2);
      const uint32_t below = (1u << lane) - 1u;
      if (c == 1) kvi[n_part + __popc(bp & below)] = t;
      if (c == 2) fvi[n_full + __popc(bf & below)] = t;
      n_part += __popc(bp);
      n_full += __popc(bf);
    }
    int n_blk = 0;
    uint32_t* bl = P.blk_list + size_t(qt) * P.n_kv128;
    for (int base = 0; base < P.n_kv128; base += 32) {
      const int b = base + lane;
      int c0 = 0, c1 = 0;
      if (b < P.n_kv128) {
        c0 = cls[2 * b];
        c1 = (2 * b + 1 < n64) ? cls[2 * b + 1] : 0;
      }
      const bool present = (c0 | c1) != 0;
      const uint32_t bb = __ballot_sync(0xffffffffu, present);
      if (present) {
        const uint32_t e = uint32_t(b) | (uint32_t(c0 != 0) << 24) | (uint32_t(c0 == 1) << 25) |
                           (uint32_t(c1 != 0) << 26) | (uint32_t(c1 == 1) << 27);
        bl[n_blk + __popc(bb & ((1u << lane) - 1u))] = e;
      }
      n_blk += __popc(bb);
    }
    if (lane == 0) {
      P.kv_num_blocks[qt] = n_part;
      P.full_kv_num_blocks[qt] = n_full;
      P.blk_count[qt] = n_blk;
    }
  }
  __syncthreads();  // every tile's block count is written
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int ci = P.blk_count[i];
    int rank = 0;
    for (int j = 0; j < n; ++j) {
      const int cj = P.blk_count[j];
      rank += (cj > ci) || (cj == ci && j < i);
    }
    P.tile_order[rank] = i;
    if (rank < 1024) cnt_sorted[rank] = ci;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int t = 0; t < n; ++t) {
      P.blk_prefix[t] = acc;
      acc += (n <= 1024) ? cnt_sorted[t] : P.blk_count[P.tile_order[t]];
    }
    P.blk_prefix[n] = acc;
  }
}

// Dense float mask -> row words.  One warp per (row, 64-column word); the two
// 32-column halves are read as coalesced 128-byte lines.
__global__ void __launch_bounds__(256) dense_words_kernel(const float* mask, int64_t row_stride,
                                                          hsd_plan_t P) {
  pdl_wait_then_release();  // launched with launch_pdl
  const int n64 = P.n_kv64;
  const int64_t total = int64_t(P.n_qtiles) * 128 * n64;
  const int lane = lane_id();
  for (int64_t w = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; w < total;
       w += (int64_t(gridDim.x) * blockDim.x) >> 5) {
    const int q = int(w / n64);
    const int t = int(w % n64);
    bool a = false, b = false;
    if (q < P.q_len) {
      const float* row = mask + int64_t(q) * row_stride;
      const int c0 = 64 * t + lane, c1 = c0 + 32;
      if (c0 < P.kv_len) a = row[c0] > -0.1f;
      if (c1 < P.kv_len) b = row[c1] > -0.1f;
    }
    const uint32_t lo = __ballot_sync(0xffffffffu, a);
    const uint32_t hi = __ballot_sync(0xffffffffu, b);
    if (lane == 0) {
      const int qt = q >> 7, r = q & 127;
      P.mask_words[(size_t(qt) * n64 + t) * 128 + r] = (uint64_t(hi) << 32) | lo;
    }
  }
}

}  // namespace meta
}  // namespace hsd

using namespace hsd;

static int check_plan(const hsd_plan_t* p) {
  if (!p || !p->mask_words || !p->tile_class || !p->blk_list || p->q_len <= 0 ||
      p->kv_len <= 0) {
    hsd_host::set_error("plan is not initialised (hsd_plan_init)");
    return HSD_ERR_INVALID_ARG;
  }
  return HSD_OK;
}

static int launch_classify(bool from_segments, const meta::SegSource& S, const hsd_plan_t& P,
                           cudaStream_t st) {
  // enough CTAs to cover the SMs twice, at most one warp per 64-column tile
  const int max_parts = (P.n_kv64 + 7) / 8;
  int parts = (296 + P.n_qtiles - 1) / P.n_qtiles;
  if (parts > max_parts) parts = max_parts;
  if (parts < 1) parts = 1;
  const dim3 grid(unsigned(P.n_qtiles), unsigned(parts));
  int rc = from_segments
               ? hsd_host::launch_pdl(meta::classify_kernel<true>, grid, dim3(256), 0, st,
                                      "classify_kernel launch", 0u, S, P)
               : hsd_host::launch_pdl(meta::classify_kernel<false>, grid, dim3(256), 0, st,
                                      "classify_kernel launch", 0u, S, P);
  if (rc) return rc;
  return hsd_host::launch_pdl(meta::order_kernel, dim3(1), dim3(1024), 0, st,
                              "order_kernel launch", 0u, P);
}

extern "C" {

int hsd_build_plan_segments(const hsd_segment_t* segs, int32_t n_segs, const int32_t* row_seg,
                            const uint64_t* seg_kv_bits, int32_t kv_words_stride,
                            const uint64_t* tree_bits, hsd_plan_t* plan, int32_t* status,
                            hsd_stream_t stream) {
  int rc = check_plan(plan);
  if (rc) return rc;
  if (!segs || n_segs <= 0 || !row_seg || !seg_kv_bits ||
      kv_words_stride < plan->n_kv64) {
    hsd_host::set_error("hsd_build_plan_segments: bad segment arguments (n_segs=%d stride=%d "
                        "n_kv64=%d)",
                        n_segs, kv_words_stride, plan->n_kv64);
    return HSD_ERR_INVALID_ARG;
  }
  if (plan->kv_len < plan->q_len) {
    hsd_host::set_error("kv_len (%d) must include the %d new columns", plan->kv_len,
                        plan->q_len);
    return HSD_ERR_INVALID_ARG;
  }
  meta::SegSource S;
  S.segs = segs;
  S.row_seg = row_seg;
  S.seg_kv_bits = seg_kv_bits;
  S.tree_bits = tree_bits;
  S.stride = kv_words_stride;
  S.q_len = plan->q_len;
  S.kv_len = plan->kv_len;
  S.kv_base = plan->kv_len - plan->q_len;
  S.n_segs = n_segs;
  S.status = status;
  return launch_classify(true, S, *plan, reinterpret_cast<cudaStream_t>(stream));
}

int hsd_build_plan_dense(const float* mask, int64_t row_stride, hsd_plan_t* plan,
                         int32_t* status, hsd_stream_t stream) {
  int rc = check_plan(plan);
  if (rc) return rc;
  if (!mask || row_stride < plan->kv_len) {
    hsd_host::set_error("hsd_build_plan_dense: row_stride %lld < kv_len %d",
                        (long long)row_stride, plan->kv_len);
    return HSD_ERR_INVALID_ARG;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t warps = int64_t(plan->n_qtiles) * 128 * plan->n_kv64;
  const int64_t blocks = (warps * 32 + 255) / 256;
  const int grid = int(blocks < 148 * 16 ? blocks : 148 * 16);
  rc = hsd_host::launch_pdl(meta::dense_words_kernel, dim3(unsigned(grid)), dim3(256), 0, st,
                            "dense_words_kernel launch", 0u, mask, row_stride, *plan);
  if (rc) return rc;
  meta::SegSource S{};
  S.status = status;
  return launch_classify(false, S, *plan, st);
}

}  // extern "C"
