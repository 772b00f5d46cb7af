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
//   warp 8      TMA producer: Q (once), then K_j and V_j into a 5-slot ring
//   warp 9      MMA issuer (one thread): S = Q K^T (A, B in smem) and
//               O += P V (P from TMEM, V in smem) on tcgen05
//   warps 10-11 idle (complete the third warpgroup for setmaxnreg)
//   warps 0-3   softmax + epilogue of head slot 0 (thread = query row)
//   warps 4-7   softmax + epilogue of head slot 1
//
// TMEM (512 columns): slot s holds S_s at columns [256 s, 256 s + 128) and
// O_s at [256 s + 128, 256 s + 256), fp32, lane = query row.  The softmax
// overwrites the first 64 columns of S_s with P_s (bf16 pairs), which the PV
// MMA reads as its A operand.  Per slot the MMA thread issues
// PV_s(j) before S_s(j+1); tcgen05 MMAs of one thread complete in order, so
// when the softmax sees S_s(j) complete, PV_s(j-1) is complete too -- O can be
// rescaled and the S/P columns reused without further waits.  Softmax keeps a
// running max in log2 units and rescales O only when the max grows by more
// than kRescaleLog2 (exact: the final O / l and LSE use the same stale max).
#include "common.cuh"

namespace hsd {
namespace attn {

constexpr int BM = 128;  // query rows per tile
constexpr int BN = 128;  // KV columns per block
constexpr int HD = 128;  // head dim
constexpr int NSLOT = 2;
constexpr int NSTAGE = 5;
constexpr int TILE_BYTES = BN * HD * 2;  // 32 KB: a 128x128 bf16 tile
constexpr int SUB_BYTES = 128 * 128;     // one 64-column swizzled sub-tile of 128 rows
constexpr int kThreads = 384;  // 3 warpgroups: softmax slot 0, slot 1, producer + MMA
constexpr float kRescaleLog2 = 8.0f;

struct __align__(1024) Smem {
  uint8_t q[NSLOT][TILE_BYTES];
  uint8_t kv[NSTAGE][TILE_BYTES];
  uint64_t bar_q;
  uint64_t bar_full[NSTAGE];
  uint64_t bar_empty[NSTAGE];
  uint64_t bar_s_full[NSLOT];
  uint64_t bar_p_full[NSLOT];
  uint64_t bar_o_done[NSLOT];
  uint64_t bar_final;
  uint32_t tmem_base;
  int abort;
};

struct Params {
  __nv_bfloat16* out;
  float* lse;
  const uint32_t* blk_list;
  const int32_t* blk_count;
  const uint64_t* mask_words;
  const int32_t* tile_order;
  int32_t* status;
  int q_len, kv_len, hq, hkv, group, pairs;
  int n_qtiles, n_kv64, n_kv128;
  float scale_log2;
};

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

// O (+)= P V: P (bf16 pairs) from TMEM, V MN-major in smem; K step = 16 rows.
__device__ __forceinline__ void issue_pv(uint32_t d_tmem, uint32_t p_tmem, uint32_t v_smem,
                                         bool acc) {
  const uint64_t b = sdesc_sw128(v_smem, SUB_BYTES, 1024);
#pragma unroll
  for (int kk = 0; kk < BN / 16; ++kk)
    umma_bf16_ts(d_tmem, p_tmem + kk * 8, b + uint64_t((kk * 2048) >> 4), kIdescO,
                 (acc || kk > 0) ? 1u : 0u);
}

__global__ void __launch_bounds__(kThreads, 1)
    verify_attn_kernel(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                      ~uintptr_t(1023));
  const int warp = warp_id(), lane = lane_id();

  // ---- work item: heaviest query tiles first
  const int per_tile = p.hkv * p.pairs;
  const int qt = p.tile_order[blockIdx.x / per_tile];
  const int hp = blockIdx.x % per_tile;
  const int kvh = hp / p.pairs, pair = hp % p.pairs;
  const int h0 = kvh * p.group + 2 * pair;
  const int nslot = (2 * pair + 1 < p.group) ? 2 : 1;
  const int nblk = p.blk_count[qt];
  const uint32_t* list = p.blk_list + size_t(qt) * p.n_kv128;

  if (threadIdx.x == 0) {
    mbar_init(&sm.bar_q, 1);
    for (int i = 0; i < NSTAGE; ++i) {
      mbar_init(&sm.bar_full[i], 1);
      mbar_init(&sm.bar_empty[i], 1);
    }
    for (int i = 0; i < NSLOT; ++i) {
      mbar_init(&sm.bar_s_full[i], 1);
      mbar_init(&sm.bar_p_full[i], 128);
      mbar_init(&sm.bar_o_done[i], 1);
    }
    mbar_init(&sm.bar_final, 1);
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
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort = &sm.abort;

  // Register split across warpgroups (launch: 384 x 168 = 64512): the
  // producer/MMA warpgroup keeps 120, each softmax warpgroup gets 192
  // (2 x 128 x 192 + 128 x 120 = 64512).  Each role's code sits inside the
  // branch of its own setmaxnreg.
  if (warp >= 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 120;\n" ::: "memory");
    if (warp == 8 && lane == 0 && nblk > 0) {
      // ---------------------------------------------------------- producer
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(&sm.bar_q, nslot * TILE_BYTES);
      for (int s = 0; s < nslot; ++s)
        for (int d = 0; d < 2; ++d)
          tma_load_3d(sm.q[s] + d * SUB_BYTES, &tm_q, &sm.bar_q, d * 64, qt * BM, h0 + s);
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;  // K/V tiles issued; ring slot i was used ceil((issued - i) / NSTAGE) times
      bool ok = true;
      for (int j = 0; j < nblk && ok; ++j) {
        const int kb = int(list[j] & 0xFFFFFFu);
        for (int which = 0; which < 2 && ok; ++which) {
          ok = mbar_wait(&sm.bar_empty[stage], phase ^ 1u, abort, p.status, 0x100 + which);
          if (!ok) break;
          mbar_arrive_expect_tx(&sm.bar_full[stage], TILE_BYTES);
          const CUtensorMap* tm = which ? &tm_v : &tm_k;
          for (int d = 0; d < 2; ++d)
            tma_load_3d(sm.kv[stage] + d * SUB_BYTES, tm, &sm.bar_full[stage], d * 64, kb * BN,
                        kvh);
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
      mbar_wait(&sm.bar_q, 0, abort, p.status, 0x120, false);
    } else if (warp == 9 && lane == 0 && nblk > 0) {
      // ---------------------------------------------------------- MMA issuer
      const uint32_t qa0 = smem_u32(sm.q[0]);
      bool ok = mbar_wait(&sm.bar_q, 0, abort, p.status, 0x200);
      tc_fence_after();
      int stage = 0;
      uint32_t phase = 0;
      const uint32_t kv0 = smem_u32(sm.kv[0]);
      // prologue: S_s(0)
      const int k0 = stage;
      if (ok) ok = mbar_wait(&sm.bar_full[k0], phase, abort, p.status, 0x201);
      if (ok) {
        tc_fence_after();
        for (int s = 0; s < nslot; ++s) {
          issue_s(tmem + s * 256, qa0 + s * TILE_BYTES, kv0 + k0 * TILE_BYTES);
          umma_commit(&sm.bar_s_full[s]);
        }
        umma_commit(&sm.bar_empty[k0]);
      }
      if (++stage == NSTAGE) { stage = 0; phase ^= 1u; }
      for (int j = 0; j < nblk && ok; ++j) {
        const int vstage = stage;
        const uint32_t vphase = phase;
        if (++stage == NSTAGE) { stage = 0; phase ^= 1u; }
        const bool more = j + 1 < nblk;
        const int nk = stage;
        const uint32_t nkph = phase;
        if (more) if (++stage == NSTAGE) { stage = 0; phase ^= 1u; }
        ok = mbar_wait(&sm.bar_full[vstage], vphase, abort, p.status, 0x202);
        if (!ok) break;
        for (int s = 0; s < nslot && ok; ++s) {
          ok = mbar_wait(&sm.bar_p_full[s], j & 1, abort, p.status, 0x205);
          if (!ok) break;
          tc_fence_after();
          issue_pv(tmem + s * 256 + 128, tmem + s * 256, kv0 + vstage * TILE_BYTES, j > 0);
          umma_commit(&sm.bar_o_done[s]);
          if (more) {
            if (s == 0) {
              ok = mbar_wait(&sm.bar_full[nk], nkph, abort, p.status, 0x203);
              if (!ok) break;
              tc_fence_after();
            }
            issue_s(tmem + s * 256, qa0 + s * TILE_BYTES, kv0 + nk * TILE_BYTES);
            umma_commit(&sm.bar_s_full[s]);
          }
        }
        if (!ok) break;
        umma_commit(&sm.bar_empty[vstage]);
        if (more) umma_commit(&sm.bar_empty[nk]);
      }
      // every MMA this thread issued has completed once bar_final fires
      umma_commit(&sm.bar_final);
      mbar_wait(&sm.bar_final, 0, abort, p.status, 0x206, false);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 192;\n" ::: "memory");
    // ------------------------------------------------------------ softmax
    const int s = warp >> 2;       // head slot
    const int quarter = warp & 3;  // TMEM lane quarter
    const int r = quarter * 32 + lane;
    const int q = qt * BM + r;
    const int h = h0 + s;
    const uint32_t lane_off = uint32_t(quarter * 32) << 16;
    const uint32_t t_s = tmem + lane_off + s * 256;
    const uint32_t t_o = t_s + 128;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    if (s < nslot) {
      for (int j = 0; j < nblk && ok; ++j) {
        const uint32_t e = list[j];
        const int kb = int(e & 0xFFFFFFu);
        // mask words: absent half = 0, full half = ~0, partial half = its row word
        uint32_t mw[4];
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const bool present = (e >> (24 + 2 * hf)) & 1u;
          const bool partial = (e >> (25 + 2 * hf)) & 1u;
          uint64_t w = present ? ~0ull : 0ull;
          if (partial) w = p.mask_words[(size_t(qt) * p.n_kv64 + 2 * kb + hf) * 128 + r];
          mw[2 * hf] = uint32_t(w);
          mw[2 * hf + 1] = uint32_t(w >> 32);
        }
        ok = __all_sync(0xffffffffu, mbar_wait(&sm.bar_s_full[s], j & 1, abort, p.status,
                                               0x300 + s));
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
        for (int i = 8; i < 128; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], x[i]);
        const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        const float m_new = fmaxf(m, mx * p.scale_log2);
        const bool need = m_new > m + kRescaleLog2;  // also true for m = -inf, m_new finite
        const float alpha = need ? ex2_approx(m - m_new) : 1.f;
        if (need) m = m_new;
        const float nm = (m == -INFINITY) ? 0.f : -m;
        // O holds sum_{i<j} P_i V_i (PV(j-1) completed before S(j)); rescale it
        // when this block raised the max.
        if (j > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint32_t o[16];
            tmem_ld16(t_o + c * 16, o);
            tmem_wait_ld16(o);
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st16(t_o + c * 16, o);
          }
        }
        // P = exp2(s * scale - m) -> bf16 pairs -> TMEM columns [0, 64) of S
        float sum4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t pk[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float a = ex2_approx(fmaf(x[64 * c + 2 * i], p.scale_log2, nm));
            const float b = ex2_approx(fmaf(x[64 * c + 2 * i + 1], p.scale_log2, nm));
            sum4[i & 3] += a + b;
            pk[i] = pack_bf16x2(a, b);
          }
          tmem_st32(t_s + c * 32, pk);
        }
        l = l * alpha + ((sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&sm.bar_p_full[s]);
      }
      // ---- epilogue
      if (ok && nblk > 0)
        ok = __all_sync(0xffffffffu, mbar_wait(&sm.bar_o_done[s], (nblk - 1) & 1, abort, p.status,
                                               0x320 + s));
      tc_fence_after();
      const float inv = (l > 0.f) ? 1.f / l : 0.f;
      __nv_bfloat16* orow = p.out + (size_t(q) * p.hq + h) * HD;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t u[32];
        if (nblk > 0 && ok) {
          tmem_ld32(t_o + c * 32, u);
          tmem_wait_ld(u);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) u[i] = 0u;
        }
        uint32_t o[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          o[i] = pack_bf16x2(__uint_as_float(u[2 * i]) * inv, __uint_as_float(u[2 * i + 1]) * inv);
        if (q < p.q_len) {
          int4* dst = reinterpret_cast<int4*>(orow + c * 32);
#pragma unroll
          for (int v = 0; v < 4; ++v)
            dst[v] = make_int4(int(o[4 * v]), int(o[4 * v + 1]), int(o[4 * v + 2]), int(o[4 * v + 3]));
        }
      }
      if (p.lse && q < p.q_len)
        p.lse[size_t(h) * p.q_len + q] =
            (l > 0.f) ? (m + __log2f(l)) * 0.69314718055994530942f : -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace attn
}  // namespace hsd

using namespace hsd;

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// [heads][rows][128] bf16 at element strides (row, head); box 64 x 128 rows x 1 head.
int make_map(CUtensorMap* map, const void* base, int rows, int heads, int64_t row_stride,
             int64_t head_stride, const char* what) {
  EncodeTiledFn enc = get_encode();
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

extern "C" int hsd_verify_attention(const void* q, int64_t q_row_stride, int64_t q_head_stride,
                                    const void* k, int64_t k_row_stride, int64_t k_head_stride,
                                    const void* v, int64_t v_row_stride, int64_t v_head_stride,
                                    void* out, float* lse, int32_t q_len, int32_t kv_len,
                                    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                    float scale, const hsd_plan_t* plan, int32_t* status,
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
  CUtensorMap tq, tk, tv;
  int rc = make_map(&tq, q, q_len, num_q_heads, q_row_stride, q_head_stride, "q");
  if (!rc) rc = make_map(&tk, k, kv_len, num_kv_heads, k_row_stride, k_head_stride, "k");
  if (!rc) rc = make_map(&tv, v, kv_len, num_kv_heads, v_row_stride, v_head_stride, "v");
  if (rc) return rc;
  attn::Params p;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.lse = lse;
  p.blk_list = plan->blk_list;
  p.blk_count = plan->blk_count;
  p.mask_words = plan->mask_words;
  p.tile_order = plan->tile_order;
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
  const size_t smem = sizeof(attn::Smem) + 1024;
  static bool attr_set = false;
  if (!attr_set) {
    rc = hsd_host::cuda_check(
        cudaFuncSetAttribute(attn::verify_attn_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
        "cudaFuncSetAttribute(verify_attn_kernel)");
    if (rc) return rc;
    attr_set = true;
  }
  const int grid = plan->n_qtiles * num_kv_heads * p.pairs;
  attn::verify_attn_kernel<<<grid, attn::kThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      tq, tk, tv, p);
  return hsd_host::cuda_check(cudaGetLastError(), "verify_attn_kernel launch");
}
