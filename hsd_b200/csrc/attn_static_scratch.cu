// Verification attention whose stream-K scratch lives in a static device
// array instead of a caller-allocated workspace.
//
// For callers that cannot allocate device memory where they call it: a
// binding in another language that has no device allocator of its own, or a
// serving loop that keeps every allocation at start-up and must not reach an
// allocator (or pay for cudaMalloc's implicit synchronisation) between steps.
// The kernels and the schedule are those of hsd_verify_attention; only where
// the scratch comes from differs.
//
// Setup: the first call on each device (that device current) looks up the
// array's device address with cudaGetSymbolAddress and caches it; this may
// load the module, so make that first call before any stream capture.
// Later calls only read the cached address.
//
// Limits: the scratch holds kStaticScratchBytes (20 MiB), enough for the
// stream-K schedule on devices of up to 310 SMs (each SM's CTA needs a 33 KB
// partial record per head slot and 32 bytes of flags).  A call whose scratch
// need exceeds it returns HSD_ERR_TOO_LARGE and launches nothing.  The array
// keeps whatever the last call left in it, so every call first clears, on
// its stream, the part that must start at zero (the ready flags and the
// launch counters, a few KB; cudaMemsetAsync allocates nothing): a call never
// depends on an earlier one, not even on one that stopped on an error.  The
// partial records need no clearing -- each is written before it is read.
// There is one scratch per device, so calls on one device must not overlap
// in time -- issue them on one stream (or order them with events); two
// overlapping calls race on the scratch and corrupt each other's output.
#include <mutex>

#include "common.cuh"

namespace {

constexpr size_t kStaticScratchBytes = size_t(20) << 20;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_attn_scratch[kStaticScratchBytes];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

int scratch_for_current_device(void** out) {
  int dev = 0;
  int rc = hsd_host::cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= kMaxDevices) {
    hsd_host::set_error("hsd_verify_attention_static_scratch: device ordinal %d >= %d", dev,
                        kMaxDevices);
    return HSD_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    rc = hsd_host::cuda_check(cudaGetSymbolAddress(&p, g_attn_scratch),
                              "cudaGetSymbolAddress(static attention scratch)");
    if (rc) return rc;
    if (!p || (reinterpret_cast<uintptr_t>(p) & 255)) {
      hsd_host::set_error("hsd_verify_attention_static_scratch: scratch address %p not "
                          "256-byte aligned", p);
      return HSD_ERR_CUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return HSD_OK;
}

}  // namespace

extern "C" size_t hsd_attention_static_scratch_bytes(void) { return kStaticScratchBytes; }

extern "C" int hsd_verify_attention_static_scratch(
    const void* q, int64_t q_row_stride, int64_t q_head_stride, const void* k,
    int64_t k_row_stride, int64_t k_head_stride, const void* v, int64_t v_row_stride,
    int64_t v_head_stride, void* out, float* lse, int32_t q_len, int32_t kv_len,
    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, float scale,
    const hsd_plan_t* plan, int32_t* status, hsd_stream_t stream) {
  const size_t need = hsd_attention_workspace_bytes(q_len, num_q_heads, num_kv_heads);
  if (need == 0) {
    hsd_host::set_error("hsd_verify_attention_static_scratch: bad sizes (q_len=%d heads=%d/%d)",
                        q_len, num_q_heads, num_kv_heads);
    return HSD_ERR_INVALID_ARG;
  }
  if (need > kStaticScratchBytes) {
    hsd_host::set_error("hsd_verify_attention_static_scratch: needs %zu bytes of scratch on "
                        "this device, the static scratch holds %zu; use hsd_verify_attention "
                        "with a workspace",
                        need, kStaticScratchBytes);
    return HSD_ERR_TOO_LARGE;
  }
  void* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc) return rc;
  // the flags and launch counters start at zero on every call
  const size_t flags = hsd_host::attention_flags_offset(q_len, num_q_heads, num_kv_heads);
  rc = hsd_host::cuda_check(
      cudaMemsetAsync(static_cast<unsigned char*>(scratch) + flags, 0, need - flags,
                      reinterpret_cast<cudaStream_t>(stream)),
      "cudaMemsetAsync(static attention scratch flags)");
  if (rc) return rc;
  return hsd_verify_attention(q, q_row_stride, q_head_stride, k, k_row_stride, k_head_stride, v,
                              v_row_stride, v_head_stride, out, lse, q_len, kv_len, num_q_heads,
                              num_kv_heads, head_dim, scale, plan, scratch, kStaticScratchBytes,
                              status, stream);
}
