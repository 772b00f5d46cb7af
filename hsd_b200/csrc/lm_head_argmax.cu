// Fused lm_head + argmax: the next token of every packed row without
// materialising the logits.
//
// The reference computes logits = lm_head(hidden) ([1, Q, V] bf16: a GEMM with
// fp32 accumulation whose result is rounded to bf16) and then
// logits.argmax(-1), which returns the first maximal index
// (hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py D:1057-1064).  At
// Q = 2176, V = 151936 that tensor is 661 MB written and read back every
// step.  Here one persistent kernel computes 128 x 256 tiles of
// hidden . weight^T with tcgen05 MMAs into TMEM and reduces each tile to
// (max, first column of the max) per row, the fp32 accumulators rounded to
// bf16 exactly as the logits tensor would hold them.  The tiles of a row
// combine through one 64-bit atomicMax per (row, tile) on a key ordered by
// value and then by lowest column; the last CTA to finish turns the keys into
// ids and clears them for the next call.
//
// Warp roles (192 threads, one CTA per SM):
//   warp 0     TMA producer: hidden (128 x 64) and weight (256 x 64) tiles
//              into a 4-stage ring
//   warp 1     TMEM owner and MMA issuer (one thread)
//   warps 2-5  epilogue, one accumulator row per thread (TMEM lane quarter
//              warp % 4); two accumulators, so the epilogue of a tile
//              overlaps the MMAs of the next
// Tiles are visited row-tile fastest (every 128-row tile of one 256-column
// weight tile back to back), so each weight tile comes from HBM once and is
// re-read from L2.
#include <atomic>

#include "common.cuh"

namespace hsd {
namespace lmh {

constexpr int BM = 128;  // rows of hidden per tile
constexpr int BN = 256;  // vocabulary columns per tile
constexpr int BK = 64;   // hidden elements per stage (one 128-byte swizzle row)
constexpr int NSTAGE = 4;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int kThreads = 192;
constexpr uint32_t kIdesc = idesc_bf16_f32(BM, BN, false, false);  // both K-major

struct __align__(1024) Smem {
  uint8_t a[NSTAGE][A_BYTES];
  uint8_t b[NSTAGE][B_BYTES];
  uint64_t full[NSTAGE];
  uint64_t empty[NSTAGE];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int consumed;  // stages the MMA thread took (for the producer's drain)
  int abort;
  int last;
};

struct Params {
  unsigned long long* keys;  // [q_len] best (value, column) key per row, 0 = none
  uint32_t* done;            // CTAs finished in this call
  int32_t* ids32;
  int64_t* ids64;
  float* max_logit;
  int32_t* status;
  int q_len, vocab, k_steps, m_tiles, tiles;
  // rank pass (hsd_lm_head_rank): per row the threshold logit, its column
  // and the column left out of the second best; outputs
  const float* probe;
  const int32_t* ref_col;
  const int32_t* excl_col;
  int32_t* rank;
  float* second;
};

// bf16 bit pattern -> unsigned order-preserving code (larger value, larger code).
__device__ __forceinline__ uint32_t ordered_bf16(uint32_t b) {
  return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
}
__device__ __forceinline__ float from_ordered_bf16(uint32_t o) {
  const uint32_t b = (o & 0x8000u) ? (o & 0x7FFFu) : (~o & 0xFFFFu);
  return __uint_as_float(b << 16);
}

// Row best of 32 accumulator columns starting at column c0 of the tile; only
// columns < ncols exist.  Values are compared after rounding to bf16; the
// strict '>' in column order keeps the first maximum.
template <bool kFull>
__device__ __forceinline__ void scan32(const uint32_t (&u)[32], int c0, int ncols, float& best,
                                       int& bcol) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    uint32_t pk;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;"
        : "=r"(pk)
        : "f"(__uint_as_float(u[2 * i + 1])), "f"(__uint_as_float(u[2 * i])));
    const float v0 = __uint_as_float(pk << 16);
    const float v1 = __uint_as_float(pk & 0xFFFF0000u);
    const int c = c0 + 2 * i;
    if (v0 > best && (kFull || c < ncols)) {
      best = v0;
      bcol = c;
    }
    if (v1 > best && (kFull || c + 1 < ncols)) {
      best = v1;
      bcol = c + 1;
    }
  }
}

// Rank pass over 32 accumulator columns (global column gc0, tile column c0):
// counts the columns other than rc whose bf16 logit ranks above (thr, rc) --
// a larger value, or the same value at a lower column -- and keeps the
// largest value outside column ex.  Column rc itself never counts: thr comes
// from hsd_probe_logits, whose summation order differs from the GEMM's, so
// the GEMM's own value at rc may sit one bf16 unit above thr.  A NaN thr (a
// probe of a bad index) counts every column, so the token ranks last.
template <bool kFull>
__device__ __forceinline__ void rank32(const uint32_t (&u)[32], int c0, int gc0, int ncols,
                                       float thr, int rc, int ex, int& cnt, float& best2) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    uint32_t pk;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;"
        : "=r"(pk)
        : "f"(__uint_as_float(u[2 * i + 1])), "f"(__uint_as_float(u[2 * i])));
    const float v[2] = {__uint_as_float(pk << 16), __uint_as_float(pk & 0xFFFF0000u)};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int col = gc0 + 2 * i + h;
      if (kFull || c0 + 2 * i + h < ncols) {
        cnt += (col != rc && (v[h] > thr || (v[h] == thr && col < rc) || thr != thr)) ? 1 : 0;
        if (col != ex && v[h] > best2) best2 = v[h];
      }
    }
  }
}

template <bool kRank>
__global__ void __launch_bounds__(kThreads, 1)
    lm_head_argmax_kernel(const __grid_constant__ CUtensorMap tm_h,
                          const __grid_constant__ CUtensorMap tm_w, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                      ~uintptr_t(1023));
  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sm.acc_full[a], 1);
      mbar_init(&sm.acc_empty[a], 128);
    }
    mbar_init(&sm.drain, 1);
    sm.consumed = 0;
    sm.abort = 0;
    sm.last = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tm_h);
    tma_prefetch_desc(&tm_w);
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort = &sm.abort;
  int issued = 0;

  if (warp == 0) {
    // ---- producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
        const int m = t % p.m_tiles, n = t / p.m_tiles;
        for (int k = 0; k < p.k_steps; ++k) {
          if (!mbar_wait(&sm.empty[stage], phase ^ 1u, abort, p.status, 0x600)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&sm.full[stage], A_BYTES + B_BYTES);
          tma_load_2d(sm.a[stage], &tm_h, &sm.full[stage], k * BK, m * BM);
          tma_load_2d(sm.b[stage], &tm_w, &sm.full[stage], k * BK, n * BN);
          ++issued;
          if (++stage == NSTAGE) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer
    if (lane == 0) {
      int stage = 0, acc = 0, taken = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&sm.acc_empty[acc], acc_phase ^ 1u, abort, p.status, 0x610)) break;
        tc_fence_after();
        const uint32_t d = tmem + uint32_t(acc * BN);
        for (int k = 0; k < p.k_steps; ++k) {
          if (!mbar_wait(&sm.full[stage], phase, abort, p.status, 0x611)) {
            ok = false;
            break;
          }
          ++taken;
          tc_fence_after();
          const uint64_t ad = sdesc_sw128(smem_u32(sm.a[stage]), 16, 1024);
          const uint64_t bd = sdesc_sw128(smem_u32(sm.b[stage]), 16, 1024);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_bf16_ss(d, ad + uint64_t(kk * 2), bd + uint64_t(kk * 2), kIdesc,
                         (k > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&sm.empty[stage]);
          if (++stage == NSTAGE) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&sm.acc_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      sm.consumed = taken;
      // every MMA this thread issued has finished before TMEM is released
      umma_commit(&sm.drain);
      mbar_wait(&sm.drain, 0, abort, p.status, 0x612, false);
    }
  } else {
    // ---- epilogue: thread = accumulator row (warp % 4) * 32 + lane
    const int quarter = warp & 3;
    const int trow = quarter * 32 + lane;
    const uint32_t lane_addr = tmem + (uint32_t(quarter * 32) << 16);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < p.tiles; t += gridDim.x) {
      const int m = t % p.m_tiles, n = t / p.m_tiles;
      if (!__all_sync(0xffffffffu,
                      mbar_wait(&sm.acc_full[acc], acc_phase, abort, p.status, 0x620)))
        break;
      tc_fence_after();
      const int ncols = min(BN, p.vocab - n * BN);
      const int row = m * BM + trow;
      float best = -INFINITY;
      int bcol = -1;
      // rank pass: this row's threshold, its column and the excluded column
      float thr = INFINITY;
      int rc = -1, ex = -1, cnt = 0;
      if (kRank && row < p.q_len) {
        thr = p.probe[row];
        rc = p.ref_col[row];
        ex = p.excl_col[row];
      }
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t u[32];
        tmem_ld32(lane_addr + uint32_t(acc * BN + c * 32), u);
        tmem_wait_ld(u);
        if (kRank) {
          if (ncols == BN)
            rank32<true>(u, c * 32, n * BN + c * 32, ncols, thr, rc, ex, cnt, best);
          else
            rank32<false>(u, c * 32, n * BN + c * 32, ncols, thr, rc, ex, cnt, best);
        } else if (ncols == BN) {
          scan32<true>(u, c * 32, ncols, best, bcol);
        } else {
          scan32<false>(u, c * 32, ncols, best, bcol);
        }
      }
      tc_fence_before();
      mbar_arrive(&sm.acc_empty[acc]);
      if (kRank) {
        // workspace: [q_len] rank counts, then [q_len] codes of the second best (+1, 0 = none)
        uint32_t* ranks = reinterpret_cast<uint32_t*>(p.keys);
        if (row < p.q_len) {
          if (cnt) atomicAdd(&ranks[row], uint32_t(cnt));
          if (best > -INFINITY)
            atomicMax(&ranks[p.q_len + row], ordered_bf16(__float_as_uint(best) >> 16) + 1u);
        }
      } else if (row < p.q_len && bcol >= 0) {
        const uint32_t code = ordered_bf16(__float_as_uint(best) >> 16);
        const uint32_t col = uint32_t(n * BN + bcol);
        atomicMax(&p.keys[row], (static_cast<unsigned long long>(code) << 32) | uint32_t(~col));
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    __threadfence();
  }
  __syncthreads();
  if (warp == 0 && lane == 0) {
    // loads issued but never consumed (after an abort) must land before exit
    for (int i = sm.consumed; i < issued; ++i)
      mbar_wait(&sm.full[i % NSTAGE], uint32_t(i / NSTAGE) & 1u, abort, p.status, 0x601, false);
  }
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
  if (threadIdx.x == 0) {
    __threadfence();
    sm.last = atomicAdd(p.done, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (sm.last && kRank) {
    __threadfence();
    uint32_t* ranks = reinterpret_cast<uint32_t*>(p.keys);
    for (int r = threadIdx.x; r < p.q_len; r += blockDim.x) {
      p.rank[r] = int32_t(atomicExch(&ranks[r], 0u));
      const uint32_t code = atomicExch(&ranks[p.q_len + r], 0u);
      p.second[r] = code ? from_ordered_bf16(code - 1u) : -INFINITY;
    }
    if (threadIdx.x == 0) *p.done = 0;
  } else if (sm.last) {
    __threadfence();
    for (int r = threadIdx.x; r < p.q_len; r += blockDim.x) {
      const unsigned long long key = atomicExch(&p.keys[r], 0ull);
      const int32_t id = key ? int32_t(~uint32_t(key)) : 0;
      if (p.ids32) p.ids32[r] = id;
      if (p.ids64) p.ids64[r] = id;
      if (p.max_logit) p.max_logit[r] = key ? from_ordered_bf16(uint32_t(key >> 32)) : -INFINITY;
    }
    if (threadIdx.x == 0) *p.done = 0;
  }
}

}  // namespace lmh
}  // namespace hsd

namespace {

using namespace hsd;

size_t keys_bytes(int32_t q_len) { return (size_t(q_len) * 8 + 255) & ~size_t(255); }

// [rows][cols] bf16 with a row stride in elements; box BK x box_rows, 128-byte swizzle.
int make_map2d(CUtensorMap* map, const void* base, int cols, int rows, int64_t row_stride,
               int box_rows, const char* what) {
  hsd_host::EncodeTiledFn enc = hsd_host::tensor_map_encoder();
  if (!enc) {
    hsd_host::set_error("cuTensorMapEncodeTiled unavailable");
    return HSD_ERR_CUDA;
  }
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(row_stride) * 2};
  cuuint32_t box[2] = {cuuint32_t(lmh::BK), cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    hsd_host::set_error("cuTensorMapEncodeTiled(%s) failed: %d", what, int(r));
    return HSD_ERR_CUDA;
  }
  return HSD_OK;
}

constexpr int kMaxDevices = 64;
// Per-device "attribute set" flags, atomic: host threads driving different
// devices or streams may reach them at once (setting the attribute twice is
// harmless).
std::atomic<bool> g_attr_set[kMaxDevices];

}  // namespace

extern "C" size_t hsd_lm_head_argmax_workspace_bytes(int32_t q_len) {
  if (q_len <= 0) return 0;
  return keys_bytes(q_len) + 256;
}

namespace {

std::atomic<bool> g_rank_attr_set[kMaxDevices];

// Shared argument checks, tensor maps and launch of both passes.
int lm_head_launch(bool rank, const char* name, const void* hidden, int64_t hidden_row_stride,
                   const void* weight, int64_t weight_row_stride, int32_t q_len, int32_t vocab,
                   int32_t hidden_dim, lmh::Params p, void* workspace, size_t workspace_bytes,
                   hsd_stream_t stream) {
  auto aligned16 = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15) == 0; };
  if (!hidden || !weight || q_len <= 0 || vocab <= 0 || hidden_dim <= 0 ||
      !aligned16(hidden) || !aligned16(weight) || hidden_row_stride < hidden_dim ||
      weight_row_stride < hidden_dim || (hidden_row_stride % 8) || (weight_row_stride % 8)) {
    hsd_host::set_error(
        "%s: bad arguments (q_len=%d vocab=%d hidden=%d; pointers 16-byte aligned, row "
        "strides >= hidden and multiples of 8 elements)",
        name, q_len, vocab, hidden_dim);
    return HSD_ERR_INVALID_ARG;
  }
  const size_t need = hsd_lm_head_argmax_workspace_bytes(q_len);
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255) || workspace_bytes < need) {
    hsd_host::set_error("%s: workspace %zu bytes (need %zu, 256-byte aligned)", name,
                        workspace_bytes, need);
    return HSD_ERR_INVALID_ARG;
  }
  const int64_t m_tiles = (int64_t(q_len) + lmh::BM - 1) / lmh::BM;
  const int64_t n_tiles = (int64_t(vocab) + lmh::BN - 1) / lmh::BN;
  if (m_tiles * n_tiles > (int64_t(1) << 30)) {
    hsd_host::set_error("%s: %lld tiles", name, (long long)(m_tiles * n_tiles));
    return HSD_ERR_TOO_LARGE;
  }
  CUtensorMap th, tw;
  int rc = make_map2d(&th, hidden, hidden_dim, q_len, hidden_row_stride, lmh::BM, "hidden");
  if (!rc) rc = make_map2d(&tw, weight, hidden_dim, vocab, weight_row_stride, lmh::BN, "weight");
  if (rc) return rc;
  char* ws = static_cast<char*>(workspace);
  p.keys = reinterpret_cast<unsigned long long*>(ws);
  p.done = reinterpret_cast<uint32_t*>(ws + keys_bytes(q_len));
  p.q_len = q_len;
  p.vocab = vocab;
  p.k_steps = (hidden_dim + lmh::BK - 1) / lmh::BK;
  p.m_tiles = int(m_tiles);
  p.tiles = int(m_tiles * n_tiles);
  const size_t smem = sizeof(lmh::Smem) + 1024;
  int dev = 0, sms = 0;
  rc = hsd_host::cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  if (!rc)
    rc = hsd_host::cuda_check(
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev),
        "cudaDeviceGetAttribute");
  if (rc) return rc;
  if (dev < 0 || dev >= kMaxDevices) {
    hsd_host::set_error("%s: device ordinal %d >= %d", name, dev, kMaxDevices);
    return HSD_ERR_UNSUPPORTED;
  }
  std::atomic<bool>& attr = rank ? g_rank_attr_set[dev] : g_attr_set[dev];
  if (!attr.load(std::memory_order_acquire)) {
    rc = hsd_host::cuda_check(
        rank ? cudaFuncSetAttribute(lmh::lm_head_argmax_kernel<true>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem))
             : cudaFuncSetAttribute(lmh::lm_head_argmax_kernel<false>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
        "cudaFuncSetAttribute(lm_head_argmax_kernel)");
    if (rc) return rc;
    attr.store(true, std::memory_order_release);
  }
  const int grid = int(std::min<int64_t>(p.tiles, sms));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (rank)
    lmh::lm_head_argmax_kernel<true><<<grid, lmh::kThreads, smem, st>>>(th, tw, p);
  else
    lmh::lm_head_argmax_kernel<false><<<grid, lmh::kThreads, smem, st>>>(th, tw, p);
  return hsd_host::cuda_check(cudaGetLastError(), "lm_head_argmax_kernel launch");
}

}  // namespace

extern "C" int hsd_lm_head_argmax(const void* hidden, int64_t hidden_row_stride,
                                  const void* weight, int64_t weight_row_stride, int32_t q_len,
                                  int32_t vocab, int32_t hidden_dim, int32_t* ids32,
                                  int64_t* ids64, float* max_logit, void* workspace,
                                  size_t workspace_bytes, int32_t* status,
                                  hsd_stream_t stream) {
  if (!ids32 && !ids64) {
    hsd_host::set_error("hsd_lm_head_argmax: bad arguments (no id output)");
    return HSD_ERR_INVALID_ARG;
  }
  lmh::Params p = {};
  p.ids32 = ids32;
  p.ids64 = ids64;
  p.max_logit = max_logit;
  p.status = status;
  return lm_head_launch(false, "hsd_lm_head_argmax", hidden, hidden_row_stride, weight,
                        weight_row_stride, q_len, vocab, hidden_dim, p, workspace,
                        workspace_bytes, stream);
}

extern "C" int hsd_lm_head_rank(const void* hidden, int64_t hidden_row_stride,
                                const void* weight, int64_t weight_row_stride, int32_t q_len,
                                int32_t vocab, int32_t hidden_dim, const float* probe_logit,
                                const int32_t* ref_col, const int32_t* excl_col, int32_t* rank,
                                float* second, void* workspace, size_t workspace_bytes,
                                int32_t* status, hsd_stream_t stream) {
  if (!probe_logit || !ref_col || !excl_col || !rank || !second) {
    hsd_host::set_error("hsd_lm_head_rank: bad arguments (probe_logit, ref_col, excl_col, "
                        "rank and second are all required)");
    return HSD_ERR_INVALID_ARG;
  }
  lmh::Params p = {};
  p.status = status;
  p.probe = probe_logit;
  p.ref_col = ref_col;
  p.excl_col = excl_col;
  p.rank = rank;
  p.second = second;
  return lm_head_launch(true, "hsd_lm_head_rank", hidden, hidden_row_stride, weight,
                        weight_row_stride, q_len, vocab, hidden_dim, p, workspace,
                        workspace_bytes, stream);
}
