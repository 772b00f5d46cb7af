// Continuation tries of tree decoding, built and BFS-packed on the device.
//
// When KMP re-alignment does not find exactly one match, the reference
// proposes a prefix tree of the block's draft (hsd/dots_ocr_pipeline/
// modeling_dots_ocr_hsd.py): kmp_search inserts, after every position p whose
// token equals the window's last token, the next min(depth, len - 1 - p)
// draft tokens into a trie rooted at that token (D:573-586, children in
// insertion order), and the loop packs the trie breadth-first, at most
// max_tree_len nodes, each node seeing itself and its ancestors
// (D:1488-1543).  Here one CTA builds one block's packed tree without a
// pointer-chasing trie:
//   * the occurrences p_0 < p_1 < ... of the root token are compacted in order;
//   * level d holds one node per distinct (parent node, draft[p + d]) over the
//     occurrences still inside the draft: a shared-memory hash table groups
//     them and keeps each group's first occurrence (atomicMin);
//   * BFS order of level d = by parent BFS index, then by first occurrence
//     (the insertion order of the parent's children): children per parent are
//     counted, scanned into per-parent bases, bucketed, and each node's rank
//     among its siblings is the number of siblings that occur first;
//   * a node's ancestor row is its parent's row plus its own bit, written
//     level by level (the parent rows are complete one barrier earlier).
// Levels stop at max_depth or once the BFS index passes the cap.
#include <climits>

#include <atomic>

#include "common.cuh"

namespace hsd {
namespace trie {

constexpr int kThreads = 512;
constexpr int kMaxOcc = 2048;  // occurrences of the root token per draft
constexpr int kHash = 4096;    // hash slots (power of two, > kMaxOcc)
constexpr int kMaxCap = 1024;  // packed nodes per tree

struct Smem {
  unsigned long long hkey[kHash];  // (parent + 1) << 32 | token; 0 = empty
  int hmin[kHash];                 // first occurrence (index into occ) of the group
  int hidx[kHash];                 // BFS index of the group's node
  int occ[kMaxOcc];                // draft positions of the root token, ascending
  int prank[kMaxOcc];              // BFS index of the occurrence's node one level up
  int nrank[kMaxOcc];              // hash slot, then BFS index at this level (-1: none)
  int cbase[kMaxOcc];              // children per parent of the previous level -> base
  int cfill[kMaxOcc];
  int bucket[kMaxOcc];             // first occurrences grouped by parent
  int scan[kThreads + 32];
  int n_occ, level_count;
};

struct Params {
  const int32_t* draft_pool;
  const int32_t* draft_off;
  const int32_t* draft_len;
  const int32_t* last_tokens;
  int32_t* tokens;
  int32_t* depths;
  int32_t* parents;
  int32_t* counts;
  unsigned long long* anc;
  int32_t* status;
  int max_depth, cap, anc_words;
};

__device__ __forceinline__ int hash_slot(unsigned long long key) {
  return int((key * 0x9E3779B97F4A7C15ull) >> 52) & (kHash - 1);
}

// In-place exclusive prefix sum of a[0..n), n <= kMaxOcc, by all threads.
__device__ void block_exclusive_scan(int* a, int n, int* tmp) {
  constexpr int per = kMaxOcc / kThreads;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  int v[per];
  int sum = 0;
#pragma unroll
  for (int k = 0; k < per; ++k) {
    const int i = tid * per + k;
    v[k] = i < n ? a[i] : 0;
    sum += v[k];
  }
  int incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) tmp[kThreads + wid] = incl;
  __syncthreads();
  if (wid == 0) {
    int w = lane < kThreads / 32 ? tmp[kThreads + lane] : 0;
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += t;
    }
    if (lane < kThreads / 32) tmp[kThreads + lane] = wi - w;
  }
  __syncthreads();
  int run = tmp[kThreads + wid] + incl - sum;
#pragma unroll
  for (int k = 0; k < per; ++k) {
    const int i = tid * per + k;
    if (i < n) a[i] = run;
    run += v[k];
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kThreads) trie_kernel(const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int32_t* draft = p.draft_pool + p.draft_off[b];
  const int n = p.draft_len[b];
  const int32_t root = p.last_tokens[b];
  int32_t* tok = p.tokens + size_t(b) * p.cap;
  int32_t* dep = p.depths + size_t(b) * p.cap;
  int32_t* par = p.parents + size_t(b) * p.cap;
  unsigned long long* anc = p.anc + size_t(b) * p.cap * p.anc_words;
  const int aw = p.anc_words;

  // ---- occurrences of the root token with at least one follower, in order
  if (tid == 0) sm.n_occ = 0;
  __syncthreads();
  for (int base = 0; base < n - 1; base += kThreads) {
    const int pos = base + tid;
    const bool hit = pos < n - 1 && draft[pos] == root;
    const unsigned bal = __ballot_sync(0xffffffffu, hit);
    if (lane == 0) sm.scan[wid] = __popc(bal);
    __syncthreads();
    if (tid == 0) {
      int s = sm.n_occ;
      for (int w = 0; w < kThreads / 32; ++w) {
        const int c = sm.scan[w];
        sm.scan[w] = s;
        s += c;
      }
      sm.level_count = s;
    }
    __syncthreads();
    if (hit) {
      const int idx = sm.scan[wid] + __popc(bal & ((1u << lane) - 1u));
      if (idx < kMaxOcc) sm.occ[idx] = pos;
    }
    __syncthreads();
    if (tid == 0) sm.n_occ = sm.level_count;
    __syncthreads();
  }
  const int K = sm.n_occ;
  if (K > kMaxOcc) {
    if (tid == 0) {
      report(p.status, HSD_DEV_CAPACITY | 0x700);
      p.counts[b] = 0;
    }
    return;
  }
  // ---- root
  if (tid == 0) {
    tok[0] = root;
    dep[0] = 0;
    par[0] = -1;
  }
  for (int w = tid; w < aw; w += kThreads) anc[w] = w == 0 ? 1ull : 0ull;
  for (int i = tid; i < K; i += kThreads) sm.prank[i] = 0;
  int prev_off = 0, prev_cnt = 1, off = 1;
  __syncthreads();

  for (int d = 1; d <= p.max_depth && off < p.cap; ++d) {
    for (int s = tid; s < kHash; s += kThreads) {
      sm.hkey[s] = 0ull;
      sm.hmin[s] = INT_MAX;
    }
    for (int s = tid; s < prev_cnt; s += kThreads) {
      sm.cbase[s] = 0;
      sm.cfill[s] = 0;
    }
    if (tid == 0) sm.level_count = 0;
    __syncthreads();
    // group the occurrences still inside the draft by (parent, next token)
    for (int i = tid; i < K; i += kThreads) {
      const int pr = sm.prank[i];
      const int o = sm.occ[i];
      int slot = -1;
      if (pr >= 0 && o + d <= n - 1) {
        const unsigned long long key =
            (static_cast<unsigned long long>(pr + 1) << 32) | uint32_t(draft[o + d]);
        slot = hash_slot(key);
        while (true) {
          const unsigned long long prev = atomicCAS(&sm.hkey[slot], 0ull, key);
          if (prev == 0ull || prev == key) break;
          slot = (slot + 1) & (kHash - 1);
        }
        atomicMin(&sm.hmin[slot], i);
      }
      sm.nrank[i] = slot;
    }
    __syncthreads();
    // one node per group, owned by its first occurrence: children per parent
    for (int i = tid; i < K; i += kThreads) {
      const int slot = sm.nrank[i];
      if (slot >= 0 && sm.hmin[slot] == i) {
        atomicAdd(&sm.cbase[sm.prank[i] - prev_off], 1);
        atomicAdd(&sm.level_count, 1);
      }
    }
    __syncthreads();
    block_exclusive_scan(sm.cbase, prev_cnt, sm.scan);
    for (int i = tid; i < K; i += kThreads) {
      const int slot = sm.nrank[i];
      if (slot >= 0 && sm.hmin[slot] == i) {
        const int pl = sm.prank[i] - prev_off;
        sm.bucket[sm.cbase[pl] + atomicAdd(&sm.cfill[pl], 1)] = i;
      }
    }
    __syncthreads();
    // BFS index = level start + parent's children base + rank among siblings
    for (int i = tid; i < K; i += kThreads) {
      const int slot = sm.nrank[i];
      if (slot >= 0 && sm.hmin[slot] == i) {
        const int pl = sm.prank[i] - prev_off;
        const int b0 = sm.cbase[pl], nb = sm.cfill[pl];
        int r = 0;
        for (int k = 0; k < nb; ++k) r += sm.bucket[b0 + k] < i;
        const int idx = off + b0 + r;
        sm.hidx[slot] = idx;
        if (idx < p.cap) {
          tok[idx] = draft[sm.occ[i] + d];
          dep[idx] = d;
          par[idx] = sm.prank[i];
          const unsigned long long* pa = anc + size_t(sm.prank[i]) * aw;
          unsigned long long* me = anc + size_t(idx) * aw;
          for (int w = 0; w < aw; ++w)
            me[w] = pa[w] | (w == (idx >> 6) ? 1ull << (idx & 63) : 0ull);
        }
      }
    }
    __syncthreads();
    for (int i = tid; i < K; i += kThreads) {
      const int slot = sm.nrank[i];
      const int idx = slot >= 0 ? sm.hidx[slot] : -1;
      sm.prank[i] = idx >= 0 && idx < p.cap ? idx : -1;  // nodes past the cap have no children
    }
    prev_off = off;
    prev_cnt = sm.level_count;
    off += prev_cnt;
    __syncthreads();
    if (prev_cnt == 0) break;
  }
  if (tid == 0) p.counts[b] = off < p.cap ? off : p.cap;
}

}  // namespace trie
}  // namespace hsd

namespace {
constexpr int kMaxDevices = 64;
// Per-device "attribute set" flags, atomic: host threads driving different
// devices or streams may reach them at once (setting it twice is harmless).
std::atomic<bool> g_trie_attr[kMaxDevices];
}  // namespace

extern "C" int hsd_continuation_trees(const int32_t* draft_pool, const int32_t* draft_off,
                                      const int32_t* draft_len, const int32_t* last_tokens,
                                      int32_t n_trees, int32_t max_depth, int32_t cap,
                                      int32_t* tokens, int32_t* depths, int32_t* parents,
                                      int32_t* counts, uint64_t* anc_bits, int32_t* status,
                                      hsd_stream_t stream) {
  using namespace hsd;
  if (n_trees < 0 || max_depth < 0 || cap < 1 || cap > trie::kMaxCap ||
      (n_trees > 0 && (!draft_pool || !draft_off || !draft_len || !last_tokens || !tokens ||
                       !depths || !parents || !counts || !anc_bits))) {
    hsd_host::set_error(
        "hsd_continuation_trees: bad arguments (n_trees=%d max_depth=%d cap=%d; cap 1..%d)",
        n_trees, max_depth, cap, trie::kMaxCap);
    return HSD_ERR_INVALID_ARG;
  }
  if (n_trees == 0) return HSD_OK;
  trie::Params p;
  p.draft_pool = draft_pool;
  p.draft_off = draft_off;
  p.draft_len = draft_len;
  p.last_tokens = last_tokens;
  p.tokens = tokens;
  p.depths = depths;
  p.parents = parents;
  p.counts = counts;
  p.anc = reinterpret_cast<unsigned long long*>(anc_bits);
  p.status = status;
  p.max_depth = max_depth;
  p.cap = cap;
  p.anc_words = (cap + 63) / 64;
  const size_t smem = sizeof(trie::Smem);
  int dev = 0;
  int rc = hsd_host::cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= kMaxDevices) {
    hsd_host::set_error("hsd_continuation_trees: device ordinal %d >= %d", dev, kMaxDevices);
    return HSD_ERR_UNSUPPORTED;
  }
  if (!g_trie_attr[dev].load(std::memory_order_acquire)) {
    rc = hsd_host::cuda_check(cudaFuncSetAttribute(trie::trie_kernel,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   int(smem)),
                              "cudaFuncSetAttribute(trie_kernel)");
    if (rc) return rc;
    g_trie_attr[dev].store(true, std::memory_order_release);
  }
  trie::trie_kernel<<<n_trees, trie::kThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  return hsd_host::cuda_check(cudaGetLastError(), "trie_kernel launch");
}
