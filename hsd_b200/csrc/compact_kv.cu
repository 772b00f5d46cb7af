// (2) KV-cache compaction on the device.
//
// The reference compacts with one index_select(-2, keep_indices) per layer
// and per K/V (D:1705-1722, H:2262-2269), which allocates a new cache and
// copies every kept row.  Here the cache is compacted in place and only rows
// that actually move (i >= first_moved) are read and written.
//
// In place is safe because keep_idx is ascending, so keep_idx[i] >= i: a
// "wave" of destination rows [w0, w1) reads sources >= w0 and earlier waves
// only wrote rows < w0.  Within a wave every source is read before any
// destination is written.  Two launch shapes:
//  * many planes (>= kPlaneCtaMinPlanes): one CTA per plane moving rows with
//    the bulk-copy engine through a ring of shared-memory buffers
//    (compact_plane_bulk_kernel);
//  * few planes: a thread-block cluster per plane staging a wave in
//    registers, the cluster's hardware barrier separating the read and write
//    phases (compact_planes_kernel) -- no global spin-waits in either.
#include <cooperative_groups.h>

#include <atomic>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace hsd {
namespace compact {

constexpr int kThreads = 256;
constexpr int kVec = 16;  // 16-byte vectors staged per thread per wave

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_nrank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// grid = n_planes * cluster, one cluster per plane.
__global__ void __launch_bounds__(kThreads) compact_planes_kernel(
    const uint64_t* __restrict__ plane_ptrs, int n_planes, int row_bytes,
    const int32_t* __restrict__ keep_idx, int n_keep_host, const int32_t* counts,
    int32_t* status) {
  pdl_wait_then_release();  // launched with launch_pdl
  const int cs = int(cluster_nrank());
  const int crank = int(cluster_rank());
  const int plane = blockIdx.x / cs;
  const int n_keep = counts ? counts[0] : n_keep_host;
  const int first = counts ? counts[1] : 0;
  if (plane >= n_planes) return;  // whole cluster exits together (same plane)
  char* base = reinterpret_cast<char*>(plane_ptrs[plane]);
  const int vpr = row_bytes >> 4;                 // 16-byte vectors per row
  const int cta_vecs = kThreads * kVec;           // vectors staged per CTA per wave
  const int rows_per_cta = cta_vecs / vpr;        // rows per CTA per wave (>= 1)
  const int rows_per_wave = rows_per_cta * cs;
  for (int w0 = first; w0 < n_keep; w0 += rows_per_wave) {
    const int r0 = w0 + crank * rows_per_cta;
    int4 stage[kVec];
    int dst_row[kVec];
#pragma unroll
    for (int k = 0; k < kVec; ++k) {
      const int v = threadIdx.x + k * kThreads;
      const int r = r0 + v / vpr;
      dst_row[k] = -1;
      if (v < rows_per_cta * vpr && r < n_keep) {
        const int src = keep_idx[r];
        if (src != r) {
          if (src < r) report(status, HSD_DEV_BAD_INDEX | 2);  // not ascending
          const int c = v % vpr;
          stage[k] = *reinterpret_cast<const int4*>(base + size_t(src) * row_bytes + size_t(c) * 16);
          dst_row[k] = r;
        }
      }
    }
    cluster_sync_all();
#pragma unroll
    for (int k = 0; k < kVec; ++k) {
      if (dst_row[k] >= 0) {
        const int v = threadIdx.x + k * kThreads;
        const int c = v % vpr;
        *reinterpret_cast<int4*>(base + size_t(dst_row[k]) * row_bytes + size_t(c) * 16) = stage[k];
      }
    }
    cluster_sync_all();
  }
}

constexpr int kIdxCache = 8192;  // staged keep indices (32 KB); the rest read from global

// ---- bulk-copy (TMA engine) variant of the one-CTA-per-plane compaction
//
// The copy engine keeps far more bytes in flight per SM than 16-byte register
// loads, so one CTA per plane streams close to HBM speed.  Waves of destination rows
// [d0, d1) go round a ring of shared-memory buffers: the sources of a wave
// are fetched as runs of consecutive rows (at most 32 rows per run, found
// with one warp ballot per 32 destinations) completing on the buffer's
// mbarrier, then the whole wave goes back with one contiguous bulk store.  The
// hazard argument is the one above: a wave's sources lie at or above its first
// destination, which is above every row an earlier wave stores, and a wave's
// store is issued only after its own loads have landed (after the loads of
// every earlier wave).  Before a buffer is refilled, the store that read it
// must have finished reading shared memory.
constexpr int kBulkThreads = 256;
#ifndef HSD_COMPACT_NBUF
#define HSD_COMPACT_NBUF 4
#endif
constexpr int kBulkNBuf = HSD_COMPACT_NBUF;            // staging buffers (a ring)
constexpr int kBulkData = 192 * 1024;                  // bytes of all staging buffers
constexpr int kBulkBuf = kBulkData / kBulkNBuf / 256 * 256;  // bytes per buffer
constexpr int kBulkSmem = kBulkNBuf * kBulkBuf + kIdxCache * 4 + 8 * (kBulkNBuf + 1);


__device__ __forceinline__ void bulk_store(void* dst, const void* src_smem, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
               ::"l"(reinterpret_cast<uint64_t>(dst)), "r"(smem_u32(src_smem)), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Every committed bulk store but the most recent one has read shared memory.
__device__ __forceinline__ void bulk_wait_read_but_last() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__global__ void __launch_bounds__(kBulkThreads, 1) compact_plane_bulk_kernel(
    const uint64_t* __restrict__ plane_ptrs, int n_planes, int row_bytes,
    const int32_t* __restrict__ keep_idx, int n_keep_host, const int32_t* counts,
    int32_t* status) {
  pdl_wait_then_release();  // launched with launch_pdl
  extern __shared__ __align__(128) unsigned char smem[];
  int32_t* s_idx = reinterpret_cast<int32_t*>(smem + kBulkNBuf * kBulkBuf);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kBulkNBuf * kBulkBuf + kIdxCache * 4);
  volatile int* abort = reinterpret_cast<volatile int*>(bar + kBulkNBuf);
  const int plane = blockIdx.x;
  const int n_keep = counts ? counts[0] : n_keep_host;
  const int first = counts ? counts[1] : 0;
  if (plane >= n_planes || first >= n_keep) return;
  char* base = reinterpret_cast<char*>(plane_ptrs[plane]);
  if (reinterpret_cast<uintptr_t>(base) & 15) {  // bulk copies need 16-byte alignment
    if (threadIdx.x == 0) report(status, HSD_DEV_BAD_INDEX | 5);
    return;
  }
  const int n_moved = n_keep - first;
  const int n_cached = n_moved < kIdxCache ? n_moved : kIdxCache;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kBulkNBuf; ++i) mbar_init(&bar[i], 1);
    *abort = 0;
    fence_barrier_init();
  }
  // Stage the indices with eight loads in flight per thread (one round of
  // global latency for up to 2048 indices) before the first wave is issued.
  constexpr int kFill = 8;
  for (int i0 = 0; i0 < n_cached; i0 += kFill * kBulkThreads) {
    int v[kFill];
#pragma unroll
    for (int u = 0; u < kFill; ++u) {
      const int i = i0 + u * kBulkThreads + int(threadIdx.x);
      v[u] = i < n_cached ? keep_idx[first + i] : 0;
    }
#pragma unroll
    for (int u = 0; u < kFill; ++u) {
      const int i = i0 + u * kBulkThreads + int(threadIdx.x);
      if (i < n_cached) s_idx[i] = v[u];
    }
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rows_per_wave = kBulkBuf / row_bytes;
  const int n_waves = (n_moved + rows_per_wave - 1) / rows_per_wave;
  // Waves go round kBulkNBuf buffers with the loads of up to kBulkNBuf - 1
  // waves in flight.  Wave wv's store is issued once its loads have landed
  // (the loads of every earlier wave have landed before); a later wave's
  // sources lie above every row an earlier wave stores, so its loads may be
  // in flight during those stores.  A buffer is refilled once the store that
  // last read it has read it.
  int issued = 0;
  auto issue_wave = [&](int wv) {
    const int b = wv % kBulkNBuf;
    const int d0 = first + wv * rows_per_wave;
    const int d1 = d0 + rows_per_wave < n_keep ? d0 + rows_per_wave : n_keep;
    if (threadIdx.x == 0) {
      // buffer b was last read by the store of wave wv - kBulkNBuf, issued
      // before the most recent store (wave wv - kBulkNBuf + 1, or none yet)
      bulk_wait_read_but_last();
      mbar_arrive_expect_tx(&bar[b], uint32_t(d1 - d0) * uint32_t(row_bytes));
    }
    __syncthreads();
    for (int g0 = d0 + warp * 32; g0 < d1; g0 += kBulkThreads) {
      const int d = g0 + lane;
      const bool valid = d < d1;
      const int j = d - first;
      const int src = valid ? (j < kIdxCache ? s_idx[j] : keep_idx[d]) : 0;
      const int prev = __shfl_up_sync(0xffffffffu, src, 1);
      const bool start = valid && (lane == 0 || src != prev + 1);
      const uint32_t starts = __ballot_sync(0xffffffffu, start);
      if (start) {
        if (src < d) report(status, HSD_DEV_BAD_INDEX | 4);  // not ascending
        const uint32_t above = starts & ~((2u << lane) - 1u);
        const int end = g0 + (above ? __ffs(above) - 1 : 32);
        const int e = end < d1 ? end : d1;
        bulk_load(smem + size_t(b) * kBulkBuf + size_t(d - d0) * row_bytes,
                  base + size_t(src) * row_bytes, uint32_t(e - d) * uint32_t(row_bytes), &bar[b]);
      }
    }
    issued = wv + 1;
  };
  for (int x = 0; x < kBulkNBuf - 1 && x < n_waves; ++x) issue_wave(x);
  for (int wv = 0; wv < n_waves; ++wv) {
    const int b = wv % kBulkNBuf;
    const uint32_t parity = uint32_t(wv / kBulkNBuf) & 1u;
    const int d0 = first + wv * rows_per_wave;
    const int d1 = d0 + rows_per_wave < n_keep ? d0 + rows_per_wave : n_keep;
    if (threadIdx.x == 0) {
      if (!mbar_wait(&bar[b], parity, abort, status, 0x500 + b, false)) {
        // loads still in flight (this wave's and the ones issued after it)
        // land before the CTA's shared memory goes away
        for (int x = wv; x < issued; ++x)
          mbar_wait(&bar[x % kBulkNBuf], uint32_t(x / kBulkNBuf) & 1u, abort, nullptr, 0, false);
        *abort = 1;
      } else {
        bulk_store(base + size_t(d0) * row_bytes, smem + size_t(b) * kBulkBuf,
                   uint32_t(d1 - d0) * uint32_t(row_bytes));
      }
    }
    __syncthreads();
    if (*abort) break;
    if (wv + kBulkNBuf - 1 < n_waves) issue_wave(wv + kBulkNBuf - 1);
  }
  if (threadIdx.x == 0) bulk_wait_all();
}

// keep = OR(live rows) & ~filter; ascending indices of set bits; n_keep and
// the first index i with keep_idx[i] != i.  One CTA of 1024 threads.
__global__ void __launch_bounds__(1024) keep_kernel(const uint64_t* live, int n_live,
                                                    int live_stride, const uint64_t* filter,
                                                    int kv_len, uint64_t* keep_bits,
                                                    int32_t* keep_idx, int32_t* counts) {
  pdl_wait_then_release();  // launched with launch_pdl
  __shared__ int warp_sums[32];
  __shared__ int carry;
  __shared__ int first_moved;
  __shared__ unsigned long long acc[1024];  // OR of the live rows, one chunk of words
  const int nw = (kv_len + 63) / 64;
  if (threadIdx.x == 0) {
    carry = 0;
    first_moved = 0x7fffffff;
  }
  for (int base = 0; base < nw; base += blockDim.x) {
    // OR of the live rows over this chunk of words: all threads share the
    // (row, word) pairs, so the loads are in flight together
    const int cw = min(int(blockDim.x), nw - base);
    acc[threadIdx.x] = 0ull;
    __syncthreads();
    for (int k = threadIdx.x; k < n_live * cw; k += blockDim.x) {
      const int r = k / cw, wi = k - r * cw;
      const uint64_t v = live[size_t(r) * live_stride + base + wi];
      if (v) atomicOr(&acc[wi], static_cast<unsigned long long>(v));
    }
    __syncthreads();
    const int t = base + threadIdx.x;
    uint64_t w = 0;
    if (t < nw) {
      w = acc[threadIdx.x];
      if (filter) w &= ~filter[t];
      const int rem = kv_len - 64 * t;
      if (rem < 64) w &= (1ull << rem) - 1ull;
      keep_bits[t] = w;
    }
    const int c = __popcll(w);
    // block-wide exclusive scan of c
    int x = c;
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane_id() >= o) x += y;
    }
    if (lane_id() == 31) warp_sums[warp_id()] = x;
    __syncthreads();
    if (warp_id() == 0) {
      int s = lane_id() < (blockDim.x >> 5) ? warp_sums[lane_id()] : 0;
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, s, o);
        if (lane_id() >= o) s += y;
      }
      warp_sums[lane_id()] = s;  // inclusive
    }
    __syncthreads();
    const int excl = carry + (warp_id() ? warp_sums[warp_id() - 1] : 0) + x - c;
    int pos = excl;
    int moved = 0x7fffffff;  // col - pos never decreases: the first mismatch is the one
    uint64_t m = w;
    while (m) {
      const int b = __ffsll(static_cast<long long>(m)) - 1;
      const int col = 64 * t + b;
      keep_idx[pos] = col;
      if (col != pos && moved == 0x7fffffff) moved = pos;
      ++pos;
      m &= m - 1;
    }
    if (moved != 0x7fffffff) atomicMin(&first_moved, moved);
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = excl + c;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    counts[0] = carry;
    counts[1] = first_moved == 0x7fffffff ? carry : first_moved;
  }
}

// out[r] bit i = in[r] bit keep_idx[i], i < n_keep; words past n_keep cleared.
// One warp per output word: lane l fetches bits l and l + 32, two ballots
// assemble the word.
__global__ void compact_bits_kernel(const uint64_t* in, uint64_t* out, int n_rows, int stride,
                                    const int32_t* keep_idx, const int32_t* counts,
                                    int out_words) {
  pdl_wait_then_release();  // launched with launch_pdl
  const int n_keep = counts[0];
  const int total = n_rows * out_words;
  const int lane = lane_id();
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int idx = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; idx < total; idx += warps) {
    const int r = idx / out_words, t = idx % out_words;
    const uint64_t* row = in + size_t(r) * stride;
    const int i0 = 64 * t + lane, i1 = i0 + 32;
    bool b0 = false, b1 = false;
    if (i0 < n_keep) {
      const int src = keep_idx[i0];
      b0 = (row[src >> 6] >> (src & 63)) & 1ull;
    }
    if (i1 < n_keep) {
      const int src = keep_idx[i1];
      b1 = (row[src >> 6] >> (src & 63)) & 1ull;
    }
    const uint32_t lo = __ballot_sync(0xffffffffu, b0), hi = __ballot_sync(0xffffffffu, b1);
    if (lane == 0) out[size_t(r) * stride + t] = (uint64_t(hi) << 32) | lo;
  }
}

// Batched row append: plane p gets n_rows rows at dst_row0 from src plane p.
// One CTA streams a contiguous span of one plane with 16-byte vectors, four
// loads in flight per thread.
__global__ void __launch_bounds__(256) append_kernel(const uint64_t* __restrict__ dst_planes,
                                                     const uint64_t* __restrict__ src_planes,
                                                     int n_planes, int row_bytes, int dst_row0,
                                                     int n_rows, int chunks) {
  pdl_wait_then_release();  // launched with launch_pdl
  const int plane = blockIdx.x / chunks, chunk = blockIdx.x % chunks;
  if (plane >= n_planes) return;
  const size_t nvec = size_t(n_rows) * (row_bytes >> 4);
  const size_t per = (nvec + chunks - 1) / chunks;
  const size_t v0 = size_t(chunk) * per, v1 = v0 + per < nvec ? v0 + per : nvec;
  const int4* src = reinterpret_cast<const int4*>(src_planes[plane]);
  int4* dst = reinterpret_cast<int4*>(reinterpret_cast<char*>(dst_planes[plane]) +
                                      size_t(dst_row0) * row_bytes);
  // eight 16-byte loads in flight per thread, then their stores
  constexpr int kU = 8;
  size_t v = v0 + threadIdx.x;
  for (; v + (kU - 1) * blockDim.x < v1; v += kU * blockDim.x) {
    int4 t[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) t[u] = __ldcs(src + v + u * blockDim.x);
#pragma unroll
    for (int u = 0; u < kU; ++u) dst[v + u * blockDim.x] = t[u];
  }
  for (; v < v1; v += blockDim.x) dst[v] = __ldcs(src + v);
}

}  // namespace compact
}  // namespace hsd

using namespace hsd;

namespace {
// With at least this many planes one CTA per plane keeps most SMs streaming.
constexpr int kPlaneCtaMinPlanes = 64;
constexpr int kMaxDevices = 64;
// Per-device "attribute set" flags, atomic: host threads driving different
// devices or streams may reach them at once (setting it twice is harmless).
std::atomic<bool> g_bulk_attr_set[kMaxDevices];
}  // namespace

extern "C" {

int hsd_compact_kv(const uint64_t* plane_ptrs, int32_t n_planes, int32_t row_bytes,
                   const int32_t* keep_idx, int32_t n_keep, const int32_t* counts,
                   int32_t* status, hsd_stream_t stream) {
  if (!plane_ptrs || n_planes <= 0 || !keep_idx || row_bytes <= 0 || (row_bytes & 15) ||
      row_bytes > compact::kThreads * compact::kVec * 16) {
    hsd_host::set_error("hsd_compact_kv: bad arguments (n_planes=%d row_bytes=%d)", n_planes,
                        row_bytes);
    return HSD_ERR_INVALID_ARG;
  }
  if (!counts && n_keep < 0) {
    hsd_host::set_error("hsd_compact_kv: n_keep < 0 needs the device counts");
    return HSD_ERR_INVALID_ARG;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // the bulk kernel stages whole rows; larger rows take the cluster kernel
  if (n_planes >= kPlaneCtaMinPlanes && row_bytes <= compact::kBulkBuf) {
    int dev = 0;
    int rc = hsd_host::cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
    if (rc) return rc;
    if (dev < 0 || dev >= kMaxDevices) {
      hsd_host::set_error("hsd_compact_kv: device ordinal %d >= %d", dev, kMaxDevices);
      return HSD_ERR_UNSUPPORTED;
    }
    if (!g_bulk_attr_set[dev].load(std::memory_order_acquire)) {
      rc = hsd_host::cuda_check(
          cudaFuncSetAttribute(compact::compact_plane_bulk_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, compact::kBulkSmem),
          "cudaFuncSetAttribute(compact_plane_bulk_kernel)");
      if (rc) return rc;
      g_bulk_attr_set[dev].store(true, std::memory_order_release);
    }
    return hsd_host::launch_pdl(compact::compact_plane_bulk_kernel, dim3(unsigned(n_planes)),
                                dim3(compact::kBulkThreads), compact::kBulkSmem, st,
                                "compact_plane_bulk_kernel launch", 0u, plane_ptrs,
                                int(n_planes), int(row_bytes), keep_idx, int(n_keep), counts,
                                status);
  }

  // Few planes: a cluster of CTAs per plane, enough to cover the SMs a few
  // times over, at most 8 (portable cluster size).
  int cs = 1;
  while (cs < 8 && n_planes * cs < 148 * 4) cs <<= 1;
  return hsd_host::launch_pdl(compact::compact_planes_kernel, dim3(unsigned(n_planes * cs)),
                              dim3(compact::kThreads), 0, reinterpret_cast<cudaStream_t>(stream),
                              "compact_planes_kernel launch", unsigned(cs), plane_ptrs,
                              int(n_planes), int(row_bytes), keep_idx, int(n_keep), counts,
                              status);
}

int hsd_kv_append(const uint64_t* dst_planes, const uint64_t* src_planes, int32_t n_planes,
                  int32_t row_bytes, int32_t dst_row0, int32_t n_rows, hsd_stream_t stream) {
  if (!dst_planes || !src_planes || n_planes <= 0 || row_bytes <= 0 || (row_bytes & 15) ||
      dst_row0 < 0 || n_rows < 0) {
    hsd_host::set_error("hsd_kv_append: bad arguments (n_planes=%d row_bytes=%d)", n_planes,
                        row_bytes);
    return HSD_ERR_INVALID_ARG;
  }
  if (n_rows == 0) return HSD_OK;
  const int64_t nvec = int64_t(n_rows) * (row_bytes >> 4);
  int chunks = int((nvec + 8191) / 8192);  // ~128 KB per CTA
  if (chunks < 1) chunks = 1;
  return hsd_host::launch_pdl(compact::append_kernel, dim3(unsigned(n_planes * chunks)), dim3(256),
                              0, reinterpret_cast<cudaStream_t>(stream), "append_kernel launch",
                              0u, dst_planes, src_planes, int(n_planes), int(row_bytes),
                              int(dst_row0), int(n_rows), chunks);
}

int hsd_keep_indices(const uint64_t* live_bits, int32_t n_live, int32_t live_stride,
                     const uint64_t* filter_bits, int32_t kv_len, uint64_t* keep_bits,
                     int32_t* keep_idx, int32_t* counts, hsd_stream_t stream) {
  if (!live_bits || n_live < 0 || kv_len <= 0 || !keep_bits || !keep_idx || !counts ||
      live_stride < (kv_len + 63) / 64) {
    hsd_host::set_error("hsd_keep_indices: bad arguments");
    return HSD_ERR_INVALID_ARG;
  }
  return hsd_host::launch_pdl(compact::keep_kernel, dim3(1), dim3(1024), 0,
                              reinterpret_cast<cudaStream_t>(stream), "keep_kernel launch", 0u,
                              live_bits, int(n_live), int(live_stride), filter_bits, int(kv_len),
                              keep_bits, keep_idx, counts);
}

int hsd_compact_bits(const uint64_t* in_bits, uint64_t* out_bits, int32_t n_rows, int32_t stride,
                     const int32_t* keep_idx, const int32_t* counts, int32_t out_words,
                     hsd_stream_t stream) {
  if (!in_bits || !out_bits || in_bits == out_bits || n_rows <= 0 || out_words > stride ||
      !keep_idx || !counts) {
    hsd_host::set_error("hsd_compact_bits: bad arguments (in-place remap is not supported)");
    return HSD_ERR_INVALID_ARG;
  }
  const int total = n_rows * out_words;  // one warp per output word
  const int grid = (total + 7) / 8 < 1184 ? (total + 7) / 8 : 1184;
  return hsd_host::launch_pdl(compact::compact_bits_kernel, dim3(unsigned(grid > 0 ? grid : 1)),
                              dim3(256), 0, reinterpret_cast<cudaStream_t>(stream),
                              "compact_bits_kernel launch", 0u, in_bits, out_bits, int(n_rows),
                              int(stride), keep_idx, counts, int(out_words));
}

}  // extern "C"
