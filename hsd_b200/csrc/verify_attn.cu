// (1) Packed block-sparse verification attention, sm_100a.
//
// Replaces the torch.compile'd FlexAttention call of the reference
// (flex_attention_forward, D:72-135 / H:103-180, BlockMask at 128x64 built by
// create_block_mask) including the K/V expansion repeat_kv (D:137-146):
// grouped KV heads are read once per CTA for two query heads.
//
// One CTA = one 128-row query tile x two query heads of the same KV group.
// It walks the tile's list of 128-column KV blocks (built by pack_meta.cu;
// empty 128x64 tiles never appear, partial 64-column halves carry per-row
// 64-bit masks, absent halves are masked out).
//
//   warp 8      TMA producer: Q per piece, then K and V tiles into a 3-stage
//               FIFO in the order the MMAs consume them: K_b0, then per block
//               j: K_{j+1}, V_j
//   warps 9, 11 MMA issuers (one thread each), slot 0 and slot 1: tcgen05
//               with both operands in smem, S = Q K^T and O += P V
//   warp 10     publisher: copies a partial record staged by the softmax in
//               shared memory out to the workspace and raises its flags, so
//               the softmax goes on to its next piece at once
//   warps 0-3   softmax + epilogue of head slot 0 (thread = query row)
//   warps 4-7   softmax + epilogue of head slot 1
//
// TMEM (512 columns): slot s holds S_s at columns [256 s, 256 s + 128) and
// O_s at [256 s + 128, 256 s + 256), fp32, lane = query row.  The softmax
// reads S_s(j) into registers and releases the S columns at once (s_free), so
// the MMA thread computes S_s(j+1) while the softmax of block j is still
// running; P_s(j) goes to shared memory (bf16, the K-major 128-byte swizzled
// layout of an MMA A operand) and O_s += P_s(j) V_j follows when the softmax
// signals p_full.  The chain per slot is therefore softmax(j) -> softmax(j+1)
// with the MMAs in its shadow.  Before the softmax rescales O or overwrites
// P_s it waits for the previous PV (o_done).  Softmax keeps a running max in
// log2 units and rescales O only when the max grows by more than
// kRescaleLog2 (exact: the final O / l and LSE use the same stale max).
//
// Stream-K: with a workspace, one CTA per SM takes an equal share of the
// cost-ordered work, so (query tile, head pair) items get cut between
// consecutive CTAs.  The CTA holding an item's first blocks (its last piece,
// finished at the end of its range) owns the item: the later pieces sit at
// the start of the following CTAs' ranges, finished early, and each publishes
// its normalised rows with one flag per (CTA, slot, warp).  The owner merges
// them into its own O in the epilogue; no second kernel.  Flags hold the
// launch generation + 1 (the generation lives in the workspace and the last
// CTA to exit advances it), so they never need clearing.  Each role walks its
// pieces from the previous one (the next head pair or tile) after one binary
// search for the first.  The MMA thread releases Q after the piece's last S,
// so the next piece's Q loads under the last block's softmax and PV.
#include <atomic>

#include "common.cuh"

namespace hsd {
namespace attn {

constexpr int BM = 128;  // query rows per tile
constexpr int BN = 128;  // KV columns per block
constexpr int HD = 128;  // head dim
constexpr int NSLOT = 2;
constexpr int NSTAGE = 3;
constexpr int TILE_BYTES = BN * HD * 2;  // 32 KB: a 128x128 bf16 tile
constexpr int SUB_BYTES = 128 * 128;     // one 64-column swizzled sub-tile of 128 rows
constexpr int kThreads = 384;  // 3 warpgroups: softmax slot 0, slot 1, producer + MMA
constexpr float kRescaleLog2 = 8.0f;
// P is packed to bf16 by truncation (pack_bf16x2_trunc).  Truncation lowers a
// value by 0.28% on average, so every exponent gets +log2(1 + k) with
// k = 0.00282 and the row sum is divided by (1 + k): the packed weights are
// then unbiased against the exact sum (mean relative error ~1e-6, RMS
// 1.75e-3 vs 1.66e-3 for round-to-nearest), and l stays the exact sum of
// exp2(s * scale - m), so O / l and the LSE need no other correction.
constexpr float kPackBiasLog2 = 0.0040626743f;   // log2(1.00282)
constexpr float kPackBiasInv = 0.99718800f;      // 1 / 1.00282

constexpr int kMaxTiles = 1024;  // query tiles per launch (q_len <= 131072)
// Partial record of one (CTA, slot): the normalised O / l in bf16 of the
// CTA's first piece when that piece continues an item begun by an earlier CTA,
// as [16 chunks][128 rows] of 16-byte vectors (a warp reads or writes 512
// contiguous bytes per access), then (m, l) per row in fp32.  Units of 4 bytes.
constexpr int kRecWords = 128 * 64 + 128 * 2;

struct __align__(1024) Smem {
  uint8_t q[NSLOT][TILE_BYTES];
  uint8_t pb[NSLOT][TILE_BYTES];  // P of the current block per slot (MMA A operand)
  uint8_t kv[NSTAGE][TILE_BYTES];
  uint64_t bar_q;
  uint64_t bar_q_free;
  uint64_t bar_full[NSTAGE];
  uint64_t bar_empty[NSTAGE];
  uint64_t bar_s_full[NSLOT];
  uint64_t bar_s_free[NSLOT];
  uint64_t bar_p_full[NSLOT];
  uint64_t bar_o_done[NSLOT];
  uint64_t bar_o_free[NSLOT];
  uint64_t bar_mufu[NSLOT];  // exponential phases alternate between the slots
  uint64_t bar_final[NSLOT];
  uint64_t bar_ostage[NSLOT];  // the slot's O rows are staged in its P buffer
  uint64_t bar_ofree[NSLOT];   // their bulk stores have read the buffer
  uint64_t bar_pub[NSLOT];       // a partial record is staged in the slot's P buffer
  uint64_t bar_pub_free[NSLOT];  // warp 10 has read it
  uint32_t tmem_base;
  int abort;
};

// 227 KB of opt-in shared memory per CTA, plus up to 1 KB lost aligning the
// dynamic base to the 1024-byte swizzle atom.
static_assert(sizeof(Smem) + 1024 <= 232448, "shared memory budget exceeded");

struct Params {
  __nv_bfloat16* out;
  float* lse;
  const uint32_t* blk_list;
  const int32_t* blk_count;
  const uint64_t* mask_words;
  const int32_t* tile_order;
  const int32_t* blk_prefix;  // [n_qtiles + 1] blocks before each ordered tile
  int32_t* status;
  uint32_t* partials;  // stream-K partial records [G][NSLOT][kRecWords], or null
  uint32_t* flags;     // [G][NSLOT][4]: record rows of warp w published (= generation + 1)
  uint32_t* sync;      // {generation, CTAs finished}: the last CTA to exit bumps the generation
  int q_len, kv_len, hq, hkv, group, pairs;
  int n_qtiles, n_kv64, n_kv128;
  float scale_log2;
  int split;  // 1: stream-K over gridDim.x CTAs; 0: one item per CTA
};

// A piece: blocks [b0, b1) of one item (query tile x head pair).
struct Piece {
  int qt, kvh, h0, nslot, b0, b1, nblk, item, start;
  int lo = -1, hp = 0;  // ordered tile index and head pair of the piece (lo < 0: none yet)
};

// Next piece of the work range [w, w1) (advances w).  Items are the query
// tiles in tile_order, each split into hkv x pairs head-pair items of
// blk_count[tile] blocks; W = sum of all items' blocks.  pc holds the
// previous piece of the walk (pc.lo < 0 before the first), which ended at an
// item boundary unless the range is exhausted.
__device__ __forceinline__ bool next_piece(const Params& p, int& w, int w1, Piece& pc) {
  if (w >= w1) return false;
  const int per_tile = p.hkv * p.pairs;
  int lo, hp, c, b0;
  if (pc.lo >= 0) {
    // the walk continues where the previous piece ended (an item boundary):
    // the next head pair of the same tile, or the next non-empty tile
    b0 = 0;
    lo = pc.lo;
    c = pc.nblk;
    hp = pc.hp + 1;
    if (hp == per_tile) {
      hp = 0;
      do {
        ++lo;
        c = p.blk_prefix[lo + 1] - p.blk_prefix[lo];
      } while (c == 0);
      pc.qt = p.tile_order[lo];
    }
  } else {
    lo = 0;
    int hi = p.n_qtiles - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.blk_prefix[mid] * per_tile <= w)
        lo = mid;
      else
        hi = mid - 1;
    }
    pc.qt = p.tile_order[lo];
    c = p.blk_count[pc.qt];
    const int off = w - p.blk_prefix[lo] * per_tile;
    hp = off / c;
    b0 = off - hp * c;
  }
  pc.lo = lo;
  pc.hp = hp;
  pc.nblk = c;
  pc.b0 = b0;
  pc.b1 = min(c, b0 + (w1 - w));
  pc.item = lo * per_tile + hp;
  pc.start = w - b0;
  pc.kvh = hp / p.pairs;
  const int pair = hp - pc.kvh * p.pairs;
  pc.h0 = pc.kvh * p.group + 2 * pair;
  pc.nslot = (2 * pair + 1 < p.group) ? 2 : 1;
  w += pc.b1 - pc.b0;
  return true;
}

// First work index of CTA k in stream-K mode.
__device__ __forceinline__ int range_start(int k, int total, int g) {
  return int((int64_t(k) * total) / g);
}

constexpr uint32_t kIdescS = idesc_bf16_f32(BM, BN, false, false);  // Q K^T: both K-major
constexpr uint32_t kIdescO = idesc_bf16_f32(BM, HD, false, true);   // P V: V is MN-major

// S = Q K^T for one 128x128 block: 8 MMAs of K = 16.  Descriptors advance
// inside a 128-byte swizzle atom by adding the byte offset >> 4 to the start
// address field (two 64-column sub-tiles of 16 KB each).
__device__ __forceinline__ void issue_s(uint32_t d_tmem, uint32_t q_smem, uint32_t k_smem) {
  const uint64_t a = sdesc_sw128(q_smem, 16, 1024);
  const uint64_t b = sdesc_sw128(k_smem, 16, 1024);
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) {
    const uint64_t off = uint64_t(((kk >> 2) * SUB_BYTES + (kk & 3) * 32) >> 4);
    umma_bf16_ss(d_tmem, a + off, b + off, kIdescS, kk > 0);
  }
}

// O (+)= P V: P K-major in smem (the layout of Q), V MN-major in smem;
// K step = 16 KV rows.
__device__ __forceinline__ void issue_pv(uint32_t d_tmem, uint32_t p_smem, uint32_t v_smem,
                                         bool acc) {
  const uint64_t a = sdesc_sw128(p_smem, 16, 1024);
  const uint64_t b = sdesc_sw128(v_smem, SUB_BYTES, 1024);
#pragma unroll
  for (int kk = 0; kk < BN / 16; ++kk) {
    const uint64_t a_off = uint64_t(((kk >> 2) * SUB_BYTES + (kk & 3) * 32) >> 4);
    umma_bf16_ss(d_tmem, a + a_off, b + uint64_t((kk * 2048) >> 4), kIdescO,
                 (acc || kk > 0) ? 1u : 0u);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    verify_attn_kernel(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v,
                       const __grid_constant__ CUtensorMap tm_o, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                      ~uintptr_t(1023));
  const int warp = warp_id(), lane = lane_id();
  const int per_tile = p.hkv * p.pairs;

  if (threadIdx.x == 0) {
    // Q and every K/V stage are released by both MMA issuers (one per slot;
    // the slot-0 issuer releases twice when slot 1 has no head in a piece)
    mbar_init(&sm.bar_q, 1);
    mbar_init(&sm.bar_q_free, NSLOT);
    for (int i = 0; i < NSTAGE; ++i) {
      mbar_init(&sm.bar_full[i], 1);
      mbar_init(&sm.bar_empty[i], NSLOT);
    }
    for (int i = 0; i < NSLOT; ++i) {
      mbar_init(&sm.bar_s_full[i], 1);
      mbar_init(&sm.bar_s_free[i], 128);
      mbar_init(&sm.bar_p_full[i], 128);
      mbar_init(&sm.bar_o_done[i], 1);
      mbar_init(&sm.bar_o_free[i], 128);
      mbar_init(&sm.bar_mufu[i], 128);
    }
    for (int i = 0; i < NSLOT; ++i) {
      mbar_init(&sm.bar_final[i], 1);
      mbar_init(&sm.bar_ostage[i], 128);
      mbar_init(&sm.bar_ofree[i], 1);
      mbar_init(&sm.bar_pub[i], 4);
      mbar_init(&sm.bar_pub_free[i], 1);
    }
    sm.abort = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Launched with programmatic dependent launch: the setup above overlaps
  // the previous kernel's tail; nothing global is read before this point.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort = &sm.abort;
  const int total = p.blk_prefix[p.n_qtiles] * per_tile;
  const int G = gridDim.x;
  const uint32_t gen = p.split ? __ldcg(p.sync) : 0u;  // launch generation (stream-K flags)
  int w0, w1;
  if (p.split) {
    w0 = range_start(blockIdx.x, total, G);
    w1 = range_start(blockIdx.x + 1, total, G);
  } else {
    // one item per CTA: item blockIdx.x of the ordered item list
    const int t = blockIdx.x / per_tile, hp = blockIdx.x % per_tile;
    const int c = t < p.n_qtiles ? p.blk_count[p.tile_order[t]] : 0;
    w0 = t < p.n_qtiles ? p.blk_prefix[t] * per_tile + hp * c : total;
    w1 = w0 + c;
  }

  // Register split across warpgroups (launch: 384 x 168 = 64512): the
  // producer/MMA warpgroup keeps 120, each softmax warpgroup gets 192
  // (2 x 128 x 192 + 128 x 120 = 64512).  Each role's code sits inside the
  // branch of its own setmaxnreg.
  if (warp >= 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 120;\n" ::: "memory");
    if (warp == 8 && lane == 0) {
      // ---------------------------------------------------------- producer
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;  // K/V tiles issued; ring slot i was used ceil((issued - i) / NSTAGE) times
      int pieces = 0;
      bool ok = true;
      int w = w0;
      Piece pc;
      while (ok && next_piece(p, w, w1, pc)) {
        if (pieces > 0)  // the previous piece's S MMAs no longer read Q
          ok = mbar_wait(&sm.bar_q_free, uint32_t(pieces - 1) & 1u, abort, p.status, 0x101);
        if (!ok) break;
        mbar_arrive_expect_tx(&sm.bar_q, pc.nslot * TILE_BYTES);
        for (int s = 0; s < pc.nslot; ++s)
          for (int d = 0; d < 2; ++d)
            tma_load_3d(sm.q[s] + d * SUB_BYTES, &tm_q, &sm.bar_q, d * 64, pc.qt * BM, pc.h0 + s);
        ++pieces;
        const uint32_t* list = p.blk_list + size_t(pc.qt) * p.n_kv128;
        // consumption order of the MMA thread: K_b0, then per block j
        // K_{j+1} (if any) before V_j
        const int n_loads = 2 * (pc.b1 - pc.b0);
        for (int i = 0; i < n_loads && ok; ++i) {
          const bool is_v = i > 0 && (i == n_loads - 1 || (i & 1) == 0);
          const int j = pc.b0 + (i == 0 ? 0 : (is_v ? (i - 1) / 2 : (i + 1) / 2));
          const int kb = int(list[j] & 0xFFFFFFu);
          ok = mbar_wait(&sm.bar_empty[stage], phase ^ 1u, abort, p.status, 0x100 + int(is_v));
          if (!ok) break;
          mbar_arrive_expect_tx(&sm.bar_full[stage], TILE_BYTES);
          const CUtensorMap* tm = is_v ? &tm_v : &tm_k;
          for (int d = 0; d < 2; ++d)
            tma_load_3d(sm.kv[stage] + d * SUB_BYTES, tm, &sm.bar_full[stage], d * 64, kb * BN,
                        pc.kvh);
          ++issued;
          if (++stage == NSTAGE) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: every issued load must have landed before the CTA exits, also
      // on the abort path (bounded; the last use u of slot i completes the
      // phase of parity u & 1).
      for (int i = 0; i < NSTAGE; ++i) {
        const int uses = issued > i ? (issued - i + NSTAGE - 1) / NSTAGE : 0;
        if (uses > 0)
          mbar_wait(&sm.bar_full[i], uint32_t(uses - 1) & 1u, abort, p.status, 0x110 + i, false);
      }
      if (pieces > 0)
        mbar_wait(&sm.bar_q, uint32_t(pieces - 1) & 1u, abort, p.status, 0x120, false);
    } else if ((warp == 9 || warp == 11) && lane == 0) {
      // ---------------------------------------------------------- MMA issuers
      // One thread per slot (warp 9: slot 0, warp 11: slot 1), so each slot's
      // MMAs follow its own softmax.  tcgen05.commit tracks the MMAs of the
      // committing thread only; K/V stages and Q are released by both.
      const int s = warp == 9 ? 0 : 1;
      const uint32_t qa = smem_u32(sm.q[s]);
      const uint32_t pa = smem_u32(sm.pb[s]);
      const uint32_t kv0 = smem_u32(sm.kv[0]);
      const uint32_t t_sl = tmem + s * 256;
      int stage = 0;
      uint32_t phase = 0;
      int ns = 0;  // S issued (s_free parity)
      int gs = 0;  // PV issued (p_full parity)
      int ps = 0;  // pieces done (o_free parity)
      int pieces = 0;
      bool ok = true;
      bool issued_any = false;
      int w = w0;
      Piece pc;
      while (ok && next_piece(p, w, w1, pc)) {
        const int n_loads = 2 * (pc.b1 - pc.b0);
        if (s >= pc.nslot) {  // no head of this piece in slot 1: skip its FIFO entries
          for (int i = 0; i < n_loads; ++i)
            if (++stage == NSTAGE) {
              stage = 0;
              phase ^= 1u;
            }
          ++pieces;
          continue;
        }
        const int rel = pc.nslot == NSLOT ? 1 : NSLOT;  // releases owed per stage
        ok = mbar_wait(&sm.bar_q, uint32_t(pieces) & 1u, abort, p.status, 0x200 + s);
        if (!ok) break;
        tc_fence_after();
        for (int i = 0; i < n_loads && ok; ++i) {
          // FIFO entry i of the piece: K_b0, then per block j K_{j+1}, V_j
          const bool is_v = i > 0 && (i == n_loads - 1 || (i & 1) == 0);
          const int j = pc.b0 + (i == 0 ? 0 : (is_v ? (i - 1) / 2 : (i + 1) / 2));
          const int st = stage;
          ok = mbar_wait(&sm.bar_full[st], phase, abort, p.status, 0x202 + s);
          if (!ok) break;
          if (++stage == NSTAGE) {
            stage = 0;
            phase ^= 1u;
          }
          if (!is_v) {
            // S(j) once the softmax has read S(j-1) of this slot
            if (ns > 0) {
              ok = mbar_wait(&sm.bar_s_free[s], uint32_t(ns - 1) & 1u, abort, p.status,
                             0x204 + s);
              if (!ok) break;
            }
            tc_fence_after();
            issue_s(t_sl, qa, kv0 + st * TILE_BYTES);
            umma_commit(&sm.bar_s_full[s]);
            ++ns;
            // the piece's last S: Q is free once it completes, so the next
            // piece's Q loads under this block's softmax and PV
            if (j == pc.b1 - 1)
              for (int k = 0; k < rel; ++k) umma_commit(&sm.bar_q_free);
          } else {
            ok = mbar_wait(&sm.bar_p_full[s], uint32_t(gs) & 1u, abort, p.status, 0x206 + s);
            if (!ok) break;
            if (j == pc.b0 && ps > 0) {
              // the softmax has read O of this slot's previous piece
              ok = mbar_wait(&sm.bar_o_free[s], uint32_t(ps - 1) & 1u, abort, p.status,
                             0x208 + s);
              if (!ok) break;
            }
            tc_fence_after();
            issue_pv(t_sl + 128, pa, kv0 + st * TILE_BYTES, j > pc.b0);
            umma_commit(&sm.bar_o_done[s]);
            ++gs;
          }
          issued_any = true;
          for (int k = 0; k < rel; ++k) umma_commit(&sm.bar_empty[st]);
        }
        if (!ok) break;
        ++ps;
        ++pieces;
      }
      // every MMA this thread issued has completed once its bar_final fires
      if (issued_any) {
        umma_commit(&sm.bar_final[s]);
        mbar_wait(&sm.bar_final[s], 0, abort, p.status, 0x20a + s, false);
      }
    } else if (warp == 10) {
      // ---------------------------------------------------------- publisher
      // When the CTA's first piece continues an item begun by an earlier CTA,
      // copy each slot's staged rows (16 chunks x 128 rows of 16 bytes) to its
      // record, release the buffer, then raise the slot's four flags.
      Piece pc;
      int wq = w0;
      if (p.split && next_piece(p, wq, w1, pc) && !(pc.b0 == 0 && pc.b1 == pc.nblk) &&
          pc.start < w0) {
        for (int s = 0; s < pc.nslot; ++s) {
          const bool ok = mbar_wait(&sm.bar_pub[s], 0, abort, p.status, 0x140 + s);
          uint32_t* rec = p.partials + (size_t(blockIdx.x) * NSLOT + s) * kRecWords;
          if (ok) {
            const int4* src = reinterpret_cast<const int4*>(sm.pb[s]);
            int4* dst = reinterpret_cast<int4*>(rec);
#pragma unroll 1
            for (int k0 = 0; k0 < 2048; k0 += 256) {
              int4 v[8];
#pragma unroll
              for (int u = 0; u < 8; ++u) v[u] = src[k0 + 32 * u + lane];
#pragma unroll
              for (int u = 0; u < 8; ++u) dst[k0 + 32 * u + lane] = v[u];
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.bar_pub_free[s]);  // also after an abort
          if (ok) {
            // the rows above, and the softmax's (m, l) stores ordered before
            // bar_pub, are visible before any flag
            __threadfence();
            __syncwarp();
            if (lane < 4)
              st_release_u32(p.flags + (size_t(blockIdx.x) * NSLOT + s) * 4 + lane, gen + 1u);
          }
        }
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 192;\n" ::: "memory");
    // ------------------------------------------------------------ softmax
    const int s = warp >> 2;       // head slot
    const int quarter = warp & 3;  // TMEM lane quarter
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = uint32_t(quarter * 32) << 16;
    const uint32_t t_s = tmem + lane_off + s * 256;
    const uint32_t t_o = t_s + 128;
    int gs = 0;  // blocks this slot has processed (barrier parity)
    int fo = 0;  // final outputs this slot has stored (barrier parity)
    int hs = 0;  // blocks with both slots active (exponential-phase handshakes)
    bool ok = true;
    bool pub_wait = false;  // the P buffer holds a staged record warp 10 may not have read
    int w = w0;
    Piece pc;
    while (ok && next_piece(p, w, w1, pc)) {
      if (s >= pc.nslot) continue;
      const int qt = pc.qt;
      const int q = qt * BM + r;
      const int h = pc.h0 + s;
      const uint32_t* list = p.blk_list + size_t(qt) * p.n_kv128;
      float m = -INFINITY, l = 0.f;
      // Mask words of a block: absent half = 0, full half = ~0, partial half =
      // this row's word.  Block j + 1's list entry and words are fetched
      // during block j, so no global-load latency sits on the block chain.
      const uint64_t* mrow = p.mask_words + size_t(qt) * p.n_kv64 * 128 + r;
      auto load_words = [&](uint32_t e, uint64_t (&wd)[2]) {
        const int kb = int(e & 0xFFFFFFu);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          wd[hf] = ((e >> (24 + 2 * hf)) & 1u) ? ~0ull : 0ull;
          if ((e >> (25 + 2 * hf)) & 1u) wd[hf] = mrow[size_t(2 * kb + hf) * 128];
        }
      };
      uint32_t e_next = pc.b0 < pc.b1 ? list[pc.b0] : 0u;
      uint64_t wd_next[2];
      load_words(e_next, wd_next);
      for (int j = pc.b0; j < pc.b1 && ok; ++j) {
        uint32_t mw[4] = {uint32_t(wd_next[0]), uint32_t(wd_next[0] >> 32), uint32_t(wd_next[1]),
                          uint32_t(wd_next[1] >> 32)};
        if (j + 1 < pc.b1) e_next = list[j + 1];
        ok = __all_sync(0xffffffffu, mbar_wait(&sm.bar_s_full[s], uint32_t(gs) & 1u, abort,
                                               p.status, 0x300 + s));
        if (!ok) break;
        tc_fence_after();
        // S row -> registers: four loads in flight, one wait
        uint32_t u[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(t_s + c * 32, u[c]);
        tmem_wait_ld(u[0]);
        tmem_wait_ld(u[1]);
        tmem_wait_ld(u[2]);
        tmem_wait_ld(u[3]);
        // S is in registers: the MMA thread may overwrite the S columns
        tc_fence_before();
        mbar_arrive(&sm.bar_s_free[s]);
        float x[128];
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) x[c * 32 + i] = __uint_as_float(u[c][i]);
        if ((mw[0] & mw[1] & mw[2] & mw[3]) != 0xffffffffu) {
#pragma unroll
          for (int i = 0; i < 128; ++i)
            x[i] = ((mw[i >> 5] >> (i & 31)) & 1u) ? x[i] : -INFINITY;
        }
        // row max: eight independent chains, then a tree
        float mx8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) mx8[k] = x[k];
#pragma unroll
        for (int i = 8; i < 128; i += 16)
#pragma unroll
          for (int k = 0; k < 8; ++k) mx8[k] = fmax3(mx8[k], x[i + k], x[i + 8 + k]);
        const float mx = fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]),
                               fmaxf(mx8[6], mx8[7]));
        const float m_new = fmaxf(m, mx * p.scale_log2);
        const bool need = m_new > m + kRescaleLog2;  // also true for m = -inf, m_new finite
        const float alpha = need ? ex2_approx(m - m_new) : 1.f;
        if (need) m = m_new;
        const float nm = ((m == -INFINITY) ? 0.f : -m) + kPackBiasLog2;
        // O holds sum_{i<j} P_i V_i of this piece once PV(j-1) completes;
        // rescale it when this block raised the max.  PV of the previous block
        // must also be done before P is overwritten below.
        bool pv_done = gs == 0;
        if (j > pc.b0 && __any_sync(0xffffffffu, need)) {
          ok = __all_sync(0xffffffffu, mbar_wait(&sm.bar_o_done[s], uint32_t(gs - 1) & 1u, abort,
                                                 p.status, 0x310 + s));
          if (!ok) break;
          pv_done = true;
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint32_t o[16];
            tmem_ld16(t_o + c * 16, o);
            tmem_wait_ld16(o);
            const uint64_t al2 = f2_pack(alpha, alpha);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              float lo, hi;
              f2_unpack(f2_mul(f2_pack(__uint_as_float(o[2 * i]), __uint_as_float(o[2 * i + 1])),
                               al2),
                        lo, hi);
              o[2 * i] = __float_as_uint(lo);
              o[2 * i + 1] = __float_as_uint(hi);
            }
            tmem_st16(t_o + c * 16, o);
          }
        }
        if (!pv_done) {
          ok = __all_sync(0xffffffffu, mbar_wait(&sm.bar_o_done[s], uint32_t(gs - 1) & 1u, abort,
                                                 p.status, 0x312 + s));
          if (!ok) break;
        }
        if (j + 1 < pc.b1) load_words(e_next, wd_next);
        // When both slots are active their exponential phases take turns on
        // the MUFU (slot 0 first): each slot's max / load / wait phases then
        // run under the other slot's exponentials instead of in lockstep.
        const bool pingpong = pc.nslot == 2;
        if (pingpong && (s == 1 || hs > 0)) {
          ok = __all_sync(0xffffffffu,
                          mbar_wait(&sm.bar_mufu[s], uint32_t(s == 0 ? hs - 1 : hs) & 1u, abort,
                                    p.status, 0x314 + s));
          if (!ok) break;
        }
        if (pub_wait) {  // P is overwritten below: warp 10 has copied the staged record
          ok = __all_sync(0xffffffffu,
                          mbar_wait(&sm.bar_pub_free[s], 0, abort, p.status, 0x316 + s));
          pub_wait = false;
          if (!ok) break;
        }
        // P = exp2(s * scale - m) -> bf16 pairs -> row r of the slot's P tile
        // (two 64-column sub-tiles, 128-byte rows, 16-byte chunk c stored at
        // chunk c ^ (r & 7): the TMA / MMA 128-byte swizzle).  The scale,
        // subtract and row sums run on packed fp32 pairs.
        const uint64_t sc2 = f2_pack(p.scale_log2, p.scale_log2);
        const uint64_t nm2 = f2_pack(nm, nm);
        uint64_t sum2[4] = {0ull, 0ull, 0ull, 0ull};
        const uint32_t prow = smem_u32(sm.pb[s]) + uint32_t(r) * 128u;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
            uint32_t pk[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int col = 64 * c + 8 * ch + 2 * i;
              float xa, xb;
              f2_unpack(f2_fma(f2_pack(x[col], x[col + 1]), sc2, nm2), xa, xb);
              const float a = ex2_approx(xa);
              const float b = ex2_approx(xb);
              sum2[i] = f2_add(sum2[i], f2_pack(a, b));
              pk[i] = pack_bf16x2_trunc(a, b);
            }
            st_shared_v4(prow + uint32_t(c * SUB_BYTES) + (uint32_t(ch ^ (r & 7)) << 4), pk[0],
                         pk[1], pk[2], pk[3]);
          }
        }
        if (pingpong) {
          mbar_arrive(&sm.bar_mufu[s ^ 1]);
          ++hs;
        }
        float s0, s1, s2, s3, s4, s5, s6, s7;
        f2_unpack(sum2[0], s0, s1);
        f2_unpack(sum2[1], s2, s3);
        f2_unpack(sum2[2], s4, s5);
        f2_unpack(sum2[3], s6, s7);
        l = l * alpha + (((s0 + s1) + (s2 + s3)) + ((s4 + s5) + (s6 + s7))) * kPackBiasInv;
        tmem_wait_st();  // O rescale stores, if any
        tc_fence_before();
        fence_async_shared();  // P stores -> visible to the MMA (async proxy)
        mbar_arrive(&sm.bar_p_full[s]);
        ++gs;
      }
      if (!ok) break;
      // ---- epilogue of the piece: O -> registers, then release O
      ok = __all_sync(0xffffffffu, mbar_wait(&sm.bar_o_done[s], uint32_t(gs - 1) & 1u, abort,
                                             p.status, 0x320 + s));
      if (!ok) break;
      tc_fence_after();
      float o[128];
      {
        uint32_t u[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(t_o + c * 32, u[c]);
        tmem_wait_ld(u[0]);
        tmem_wait_ld(u[1]);
        tmem_wait_ld(u[2]);
        tmem_wait_ld(u[3]);
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) o[c * 32 + i] = __uint_as_float(u[c][i]);
      }
      tc_fence_before();
      mbar_arrive(&sm.bar_o_free[s]);
      const bool whole = pc.b0 == 0 && pc.b1 == pc.nblk;
      if (!whole && pc.start < w0) {
        // a later piece of an item begun by an earlier CTA (this CTA's first
        // piece): O / l in bf16, in the record's layout, goes to the slot's P
        // buffer (free: the last PV has completed) and (m, l) straight to the
        // record; warp 10 copies the rows out and raises the flags.
        uint32_t* rec = p.partials + (size_t(blockIdx.x) * NSLOT + s) * kRecWords;
        const float invl = (l > 0.f) ? 1.f / l : 0.f;
        const uint32_t stg = smem_u32(sm.pb[s]) + uint32_t(r) * 16u;
#pragma unroll
        for (int c = 0; c < 16; ++c)
          st_shared_v4(stg + uint32_t(c) * 2048u, pack_bf16x2(o[8 * c] * invl, o[8 * c + 1] * invl),
                       pack_bf16x2(o[8 * c + 2] * invl, o[8 * c + 3] * invl),
                       pack_bf16x2(o[8 * c + 4] * invl, o[8 * c + 5] * invl),
                       pack_bf16x2(o[8 * c + 6] * invl, o[8 * c + 7] * invl));
        reinterpret_cast<float2*>(rec + 128 * 64)[r] = make_float2(m, l);
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.bar_pub[s]);
        pub_wait = true;
        continue;
      }
      if (!whole) {
        // this piece holds the item's first blocks: merge the later pieces,
        // the first pieces of the non-empty ranges blockIdx.x+1 .. khi
        const int ib = pc.start + pc.nblk - 1;  // the item's last work unit
        int khi = blockIdx.x;
        while (khi + 1 < G && range_start(khi + 1, total, G) <= ib) ++khi;
        for (int k = blockIdx.x + 1; k <= khi && ok; ++k) {
          if (range_start(k + 1, total, G) == range_start(k, total, G)) continue;  // empty
          const uint32_t* rec = p.partials + (size_t(k) * NSLOT + s) * kRecWords;
          // acquire poll: the record reads below are ordered after the flag
          ok = wait_flag(p.flags + (size_t(k) * NSLOT + s) * 4 + quarter, gen + 1u, abort,
                         p.status, 0x330 + s, true);
          if (!ok) break;
          // (m, l) and all 16 chunks in one round of loads; a row the later
          // piece saw nothing of (l = 0) leaves O, m and l as they are
          const float2 ml = __ldcg(reinterpret_cast<const float2*>(rec + 128 * 64) + r);
          const int4* rec4 = reinterpret_cast<const int4*>(rec);
          int4 v[16];
#pragma unroll
          for (int c = 0; c < 16; ++c) v[c] = __ldcg(rec4 + c * 128 + r);
          const bool use = ml.y > 0.f;
          const float nm = use ? fmaxf(m, ml.x) : m;
          const float a = use ? ex2_approx(m - nm) : 1.f;  // 0 when this row had nothing yet
          const float b = use ? ex2_approx(ml.x - nm) * ml.y : 0.f;
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const uint32_t wv[4] = {uint32_t(v[c].x), uint32_t(v[c].y), uint32_t(v[c].z),
                                    uint32_t(v[c].w)};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              o[8 * c + 2 * i] = o[8 * c + 2 * i] * a + __uint_as_float(wv[i] << 16) * b;
              o[8 * c + 2 * i + 1] =
                  o[8 * c + 2 * i + 1] * a + __uint_as_float(wv[i] & 0xffff0000u) * b;
            }
          }
          l = l * a + b;
          m = nm;
        }
        if (!ok) break;
      }
      // ---- final output of the item: O / l rows staged in this slot's P
      // buffer (free: the last PV has completed) in the 128-byte-swizzled TMA
      // layout, then two bulk tensor stores of 64 columns x 128 rows (rows
      // past q_len are not written).  The buffer is free again for the next
      // piece's P once the stores have read it.
      const float inv = (l > 0.f) ? 1.f / l : 0.f;
      if (pub_wait) {  // the output is staged in the P buffer below
        ok = __all_sync(0xffffffffu,
                        mbar_wait(&sm.bar_pub_free[s], 0, abort, p.status, 0x318 + s));
        pub_wait = false;
        if (!ok) break;
      }
      {
        const uint32_t orow = smem_u32(sm.pb[s]) + uint32_t(r) * 128u;
#pragma unroll
        for (int v = 0; v < 16; ++v)
          st_shared_v4(orow + uint32_t((v >> 3) * SUB_BYTES) + (uint32_t((v & 7) ^ (r & 7)) << 4),
                       pack_bf16x2(o[8 * v] * inv, o[8 * v + 1] * inv),
                       pack_bf16x2(o[8 * v + 2] * inv, o[8 * v + 3] * inv),
                       pack_bf16x2(o[8 * v + 4] * inv, o[8 * v + 5] * inv),
                       pack_bf16x2(o[8 * v + 6] * inv, o[8 * v + 7] * inv));
        fence_async_shared();
        mbar_arrive(&sm.bar_ostage[s]);
        if (r == 0) {
          if (mbar_wait(&sm.bar_ostage[s], uint32_t(fo) & 1u, abort, p.status, 0x340 + s)) {
            tma_store_3d(&tm_o, sm.pb[s], 0, qt * BM, h);
            tma_store_3d(&tm_o, sm.pb[s] + SUB_BYTES, 64, qt * BM, h);
            bulk_commit_group();
            bulk_wait_group_read0();
          }
          mbar_arrive(&sm.bar_ofree[s]);  // also after an abort, so no thread waits long
        }
        ok = __all_sync(0xffffffffu, mbar_wait(&sm.bar_ofree[s], uint32_t(fo) & 1u, abort,
                                               p.status, 0x342 + s));
        ++fo;
        if (!ok) break;
      }
      if (q < p.q_len && p.lse)
        p.lse[size_t(h) * p.q_len + q] =
            (l > 0.f) ? (m + __log2f(l)) * 0.69314718055994530942f : -INFINITY;
    }
    bulk_wait_group0();  // this thread's output stores (if any) have completed
    // query tiles without any visible block: all their rows are fully masked
    if (ok) {
      const int tid = threadIdx.x;  // 0..255
      for (int t = blockIdx.x; t < p.n_qtiles; t += G) {
        const int qt = p.tile_order[t];
        if (p.blk_count[qt] != 0) continue;
        for (int idx = tid; idx < 128 * p.hq; idx += 256) {
          const int rr = idx / p.hq, hh = idx % p.hq;
          const int qq = qt * BM + rr;
          if (qq >= p.q_len) continue;
          int4* dst = reinterpret_cast<int4*>(p.out + (size_t(qq) * p.hq + hh) * HD);
          for (int v = 0; v < 16; ++v) dst[v] = make_int4(0, 0, 0, 0);
          if (p.lse) p.lse[size_t(hh) * p.q_len + qq] = -INFINITY;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (p.split && threadIdx.x == 0) {
    // the last CTA to finish advances the generation for the next launch
    __threadfence();
    if (atomicAdd(p.sync + 1, 1u) == uint32_t(G) - 1u) {
      p.sync[1] = 0u;
      __threadfence();
      st_release_u32(p.sync, gen + 1u);
    }
  }
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace attn
}  // namespace hsd

using namespace hsd;

namespace {

// [heads][rows][128] bf16 at element strides (row, head); box 64 x 128 rows x 1 head.
int make_map(CUtensorMap* map, const void* base, int rows, int heads, int64_t row_stride,
             int64_t head_stride, const char* what) {
  hsd_host::EncodeTiledFn enc = hsd_host::tensor_map_encoder();
  if (!enc) {
    hsd_host::set_error("cuTensorMapEncodeTiled unavailable");
    return HSD_ERR_CUDA;
  }
  cuuint64_t dims[3] = {cuuint64_t(attn::HD), cuuint64_t(rows), cuuint64_t(heads)};
  cuuint64_t strides[2] = {cuuint64_t(row_stride) * 2, cuuint64_t(head_stride) * 2};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    hsd_host::set_error("cuTensorMapEncodeTiled(%s) failed: %d", what, int(r));
    return HSD_ERR_CUDA;
  }
  return HSD_OK;
}

bool strides_ok(const void* p, int64_t rs, int64_t hs) {
  return p && (reinterpret_cast<uintptr_t>(p) & 15) == 0 && rs > 0 && hs > 0 && (rs % 8) == 0 &&
         (hs % 8) == 0;
}

}  // namespace

namespace {

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return 148;
  return n;
}

// Stream-K workspace: partial records [G][NSLOT][kRecWords], flags
// [G][NSLOT][4], then {generation, CTAs finished}.  G = SMs of the device.
struct WsLayout {
  size_t partials, flags, sync, total;
  int items, grid;
};

WsLayout ws_layout(int32_t q_len, int32_t hq, int32_t hkv) {
  WsLayout L{};
  const int n_qtiles = (q_len + attn::BM - 1) / attn::BM;
  const int group = hq / hkv, pairs = (group + 1) / 2;
  L.items = n_qtiles * hkv * pairs;
  L.grid = sm_count();
  L.partials = 0;
  L.flags = size_t(L.grid) * attn::NSLOT * attn::kRecWords * sizeof(uint32_t);
  L.sync = L.flags + size_t(L.grid) * attn::NSLOT * 4 * sizeof(uint32_t);
  L.total = L.sync + 256;
  return L;
}

constexpr int kMaxDevices = 64;
// Per-device "attribute set" flags, atomic: host threads driving different
// devices or streams may reach them at once (setting the attribute twice is
// harmless).
std::atomic<bool> g_attr_set[kMaxDevices];

}  // namespace

namespace hsd_host {
size_t attention_flags_offset(int32_t q_len, int32_t num_q_heads, int32_t num_kv_heads) {
  return ws_layout(q_len, num_q_heads, num_kv_heads).flags;
}
}  // namespace hsd_host

extern "C" size_t hsd_attention_workspace_bytes(int32_t q_len, int32_t num_q_heads,
                                                int32_t num_kv_heads) {
  if (q_len <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads)
    return 0;
  return ws_layout(q_len, num_q_heads, num_kv_heads).total;
}

extern "C" int hsd_verify_attention(const void* q, int64_t q_row_stride, int64_t q_head_stride,
                                    const void* k, int64_t k_row_stride, int64_t k_head_stride,
                                    const void* v, int64_t v_row_stride, int64_t v_head_stride,
                                    void* out, float* lse, int32_t q_len, int32_t kv_len,
                                    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                    float scale, const hsd_plan_t* plan, void* workspace,
                                    size_t workspace_bytes, int32_t* status,
                                    hsd_stream_t stream) {
  if (head_dim != attn::HD) {
    hsd_host::set_error("hsd_verify_attention: head_dim %d unsupported (128 only)", head_dim);
    return HSD_ERR_UNSUPPORTED;
  }
  if (!plan || plan->q_len != q_len || plan->kv_len != kv_len || q_len <= 0 || kv_len <= 0 ||
      num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads || !out ||
      (reinterpret_cast<uintptr_t>(out) & 15) || !strides_ok(q, q_row_stride, q_head_stride) ||
      !strides_ok(k, k_row_stride, k_head_stride) || !strides_ok(v, v_row_stride, v_head_stride)) {
    hsd_host::set_error(
        "hsd_verify_attention: bad arguments (q_len=%d kv_len=%d heads=%d/%d, plan %d/%d; "
        "pointers must be 16-byte aligned, strides multiples of 8 elements)",
        q_len, kv_len, num_q_heads, num_kv_heads, plan ? plan->q_len : -1,
        plan ? plan->kv_len : -1);
    return HSD_ERR_INVALID_ARG;
  }
  if (plan->n_qtiles > attn::kMaxTiles) {
    hsd_host::set_error("hsd_verify_attention: q_len %d exceeds %d query tiles", q_len,
                        attn::kMaxTiles);
    return HSD_ERR_TOO_LARGE;
  }
  const WsLayout W = ws_layout(q_len, num_q_heads, num_kv_heads);
  const bool split = workspace != nullptr;
  if (split && ((reinterpret_cast<uintptr_t>(workspace) & 255) || workspace_bytes < W.total)) {
    hsd_host::set_error("hsd_verify_attention: workspace %zu bytes (need %zu, 256-byte aligned)",
                        workspace_bytes, W.total);
    return HSD_ERR_INVALID_ARG;
  }
  CUtensorMap tq, tk, tv;
  int rc = make_map(&tq, q, q_len, num_q_heads, q_row_stride, q_head_stride, "q");
  if (!rc) rc = make_map(&tk, k, kv_len, num_kv_heads, k_row_stride, k_head_stride, "k");
  if (!rc) rc = make_map(&tv, v, kv_len, num_kv_heads, v_row_stride, v_head_stride, "v");
  CUtensorMap to;
  if (!rc)
    rc = make_map(&to, out, q_len, num_q_heads, int64_t(num_q_heads) * attn::HD, attn::HD, "out");
  if (rc) return rc;
  attn::Params p;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.lse = lse;
  p.blk_list = plan->blk_list;
  p.blk_count = plan->blk_count;
  p.mask_words = plan->mask_words;
  p.tile_order = plan->tile_order;
  p.blk_prefix = plan->blk_prefix;
  p.status = status;
  p.q_len = q_len;
  p.kv_len = kv_len;
  p.hq = num_q_heads;
  p.hkv = num_kv_heads;
  p.group = num_q_heads / num_kv_heads;
  p.pairs = (p.group + 1) / 2;
  p.n_qtiles = plan->n_qtiles;
  p.n_kv64 = plan->n_kv64;
  p.n_kv128 = plan->n_kv128;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.split = split ? 1 : 0;
  char* ws = static_cast<char*>(workspace);
  p.partials = split ? reinterpret_cast<uint32_t*>(ws + W.partials) : nullptr;
  p.flags = split ? reinterpret_cast<uint32_t*>(ws + W.flags) : nullptr;
  p.sync = split ? reinterpret_cast<uint32_t*>(ws + W.sync) : nullptr;
  const size_t smem = sizeof(attn::Smem) + 1024;
  int dev = 0;
  rc = hsd_host::cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= kMaxDevices) {
    hsd_host::set_error("hsd_verify_attention: device ordinal %d >= %d", dev, kMaxDevices);
    return HSD_ERR_UNSUPPORTED;
  }
  if (!g_attr_set[dev].load(std::memory_order_acquire)) {
    rc = hsd_host::cuda_check(
        cudaFuncSetAttribute(attn::verify_attn_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
        "cudaFuncSetAttribute(verify_attn_kernel)");
    if (rc) return rc;
    g_attr_set[dev].store(true, std::memory_order_release);
  }
  // stream-K: one CTA per SM sharing the total work evenly; otherwise one CTA
  // per (query tile, head pair) item.
  const int grid = split ? W.grid : W.items;
  // Programmatic dependent launch: the CTAs may start their setup while the
  // previous kernel on the stream finishes (griddepcontrol.wait in the
  // kernel holds every read of global memory until it has completed).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(attn::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return hsd_host::cuda_check(cudaLaunchKernelEx(&cfg, attn::verify_attn_kernel, tq, tk, tv, to, p),
                              "verify_attn_kernel launch");
}
