// Library-wide C ABI pieces: version, error message, plan workspace layout.
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

namespace hsd_host {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return HSD_OK;
  set_error("%s: %s", what, cudaGetErrorString(e));
  return HSD_ERR_CUDA;
}

EncodeTiledFn tensor_map_encoder() {
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

}  // namespace hsd_host

namespace {

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct PlanLayout {
  size_t mask_words, tile_class, kv_num, kv_idx, full_num, full_idx, blk_count, blk_list,
      tile_order, blk_prefix, total;
};

PlanLayout plan_layout(int32_t q_len, int32_t kv_len) {
  const size_t nq = (q_len + 127) / 128, n64 = (kv_len + 63) / 64, n128 = (kv_len + 127) / 128;
  PlanLayout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t at = off;
    off = align256(off + bytes);
    return at;
  };
  L.mask_words = take(nq * n64 * 128 * sizeof(uint64_t));
  L.tile_class = take(nq * n64);
  L.kv_num = take(nq * 4);
  L.kv_idx = take(nq * n64 * 4);
  L.full_num = take(nq * 4);
  L.full_idx = take(nq * n64 * 4);
  L.blk_count = take(nq * 4);
  L.blk_list = take(nq * n128 * 4);
  L.tile_order = take(nq * 4);
  L.blk_prefix = take((nq + 1) * 4);
  L.total = off;
  return L;
}

}  // namespace

extern "C" {

const char* hsd_version(void) { return "hsd_b200 0.1.0 sm_100a"; }

const char* hsd_last_error(void) { return hsd_host::g_err; }

size_t hsd_plan_workspace_bytes(int32_t q_len, int32_t kv_len) {
  if (q_len <= 0 || kv_len <= 0) return 0;
  return plan_layout(q_len, kv_len).total;
}

int hsd_plan_init(void* workspace, size_t bytes, int32_t q_len, int32_t kv_len,
                  hsd_plan_t* plan) {
  if (!plan || !workspace || q_len <= 0 || kv_len <= 0) {
    hsd_host::set_error("hsd_plan_init: bad arguments (q_len=%d kv_len=%d)", q_len, kv_len);
    return HSD_ERR_INVALID_ARG;
  }
  if (reinterpret_cast<uintptr_t>(workspace) & 255) {
    hsd_host::set_error("hsd_plan_init: workspace must be 256-byte aligned");
    return HSD_ERR_INVALID_ARG;
  }
  PlanLayout L = plan_layout(q_len, kv_len);
  if (bytes < L.total) {
    hsd_host::set_error("hsd_plan_init: workspace %zu bytes < %zu needed", bytes, L.total);
    return HSD_ERR_TOO_LARGE;
  }
  char* base = static_cast<char*>(workspace);
  plan->q_len = q_len;
  plan->kv_len = kv_len;
  plan->n_qtiles = (q_len + 127) / 128;
  plan->n_kv64 = (kv_len + 63) / 64;
  plan->n_kv128 = (kv_len + 127) / 128;
  plan->reserved = 0;
  plan->mask_words = reinterpret_cast<uint64_t*>(base + L.mask_words);
  plan->tile_class = reinterpret_cast<uint8_t*>(base + L.tile_class);
  plan->kv_num_blocks = reinterpret_cast<int32_t*>(base + L.kv_num);
  plan->kv_indices = reinterpret_cast<int32_t*>(base + L.kv_idx);
  plan->full_kv_num_blocks = reinterpret_cast<int32_t*>(base + L.full_num);
  plan->full_kv_indices = reinterpret_cast<int32_t*>(base + L.full_idx);
  plan->blk_count = reinterpret_cast<int32_t*>(base + L.blk_count);
  plan->blk_list = reinterpret_cast<uint32_t*>(base + L.blk_list);
  plan->tile_order = reinterpret_cast<int32_t*>(base + L.tile_order);
  plan->blk_prefix = reinterpret_cast<int32_t*>(base + L.blk_prefix);
  return HSD_OK;
}

}  // extern "C"

namespace {

// One thread waits for *flag == 1 with the library's bounded wait; nothing
// sets the flag, so the wait gives up after hsd::kWaitLimitNs and records
// HSD_DEV_TIMEOUT | where in the status word.
__global__ void selftest_wait_kernel(const uint32_t* flag, int32_t* status, int32_t where) {
  __shared__ int abort;
  if (threadIdx.x == 0) {
    abort = 0;
    hsd::wait_flag(flag, 1u, &abort, status, where);
  }
}

}  // namespace

extern "C" int hsd_selftest_bounded_wait(const uint32_t* flag, int32_t* status,
                                         hsd_stream_t stream) {
  if (!flag || !status) {
    hsd_host::set_error("hsd_selftest_bounded_wait: flag and status are required");
    return HSD_ERR_INVALID_ARG;
  }
  selftest_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(flag, status,
                                                                              0x7F0);
  return hsd_host::cuda_check(cudaGetLastError(), "selftest_wait_kernel launch");
}
