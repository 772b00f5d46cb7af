// Single logits for the logit-ratio acceptance.
//
// Below HSD_SPEC_THRESH / HSD_TREE_THRESH = 1 the reference reads a few
// entries of the logits tensor besides the argmax: logits[r, draft token]
// for the speculative rows from the first miss on (D:1163-1168) and
// logits[row, child token] for the children of a tree node whose target
// token is no child (D:1228-1232, D:1256-1260).  The fused lm_head + argmax
// never writes that tensor, so each such entry is one dot product
// hidden[row] . weight[token] here: a warp per entry, 16-byte loads of both
// rows, fp32 accumulation and the bf16 rounding the logits tensor applies.
// The summation order differs from a GEMM's, so an entry can differ from
// the GEMM's bf16 logit by one bf16 unit when the exact value lies near a
// rounding boundary.
#include "common.cuh"

namespace hsd {
namespace probe {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) probe_logits_kernel(
    const __nv_bfloat16* __restrict__ hidden, int64_t hs, const __nv_bfloat16* __restrict__ weight,
    int64_t ws, int q_len, int vocab, int hidden_dim, const int32_t* __restrict__ rows,
    const int32_t* __restrict__ toks, int n, float* __restrict__ out, int32_t* status) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int chunks = hidden_dim >> 3;  // 8 bf16 per 16-byte load
  for (int k = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; k < n; k += warps) {
    const int t = toks[k];
    if (t < 0) {
      if (lane == 0) out[k] = 0.f;
      continue;
    }
    const int r = rows[k];
    if (r < 0 || r >= q_len || t >= vocab) {
      if (lane == 0) {
        out[k] = __int_as_float(0x7fc00000);
        report(status, HSD_DEV_BAD_INDEX | 0x7A0);
      }
      continue;
    }
    const uint4* h = reinterpret_cast<const uint4*>(hidden + int64_t(r) * hs);
    const uint4* w = reinterpret_cast<const uint4*>(weight + int64_t(t) * ws);
    float acc = 0.f;
    for (int j = lane; j < chunks; j += 32) {
      const uint4 a = h[j];
      const uint4 b = __ldg(w + j);
      const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
      const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 x = __bfloat1622float2(a2[e]);
        const float2 y = __bfloat1622float2(b2[e]);
        acc = fmaf(x.x, y.x, acc);
        acc = fmaf(x.y, y.y, acc);
      }
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) out[k] = __bfloat162float(__float2bfloat16_rn(acc));
  }
}

}  // namespace probe
}  // namespace hsd

using namespace hsd;

extern "C" int hsd_probe_logits(const void* hidden, int64_t hidden_row_stride, const void* weight,
                                int64_t weight_row_stride, int32_t q_len, int32_t vocab,
                                int32_t hidden_dim, const int32_t* rows, const int32_t* toks,
                                int32_t n, float* out, int32_t* status, hsd_stream_t stream) {
  auto aligned16 = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15) == 0; };
  if (n < 0 || (n > 0 && (!hidden || !weight || !rows || !toks || !out || !status)) ||
      q_len <= 0 || vocab <= 0 || hidden_dim <= 0 || (hidden_dim % 8) ||
      hidden_row_stride < hidden_dim || weight_row_stride < hidden_dim ||
      (hidden_row_stride % 8) || (weight_row_stride % 8) || !aligned16(hidden) ||
      !aligned16(weight)) {
    hsd_host::set_error(
        "hsd_probe_logits: bad arguments (n=%d q_len=%d vocab=%d hidden=%d; pointers 16-byte "
        "aligned, hidden and row strides multiples of 8 elements)",
        n, q_len, vocab, hidden_dim);
    return HSD_ERR_INVALID_ARG;
  }
  if (n == 0) return 0;
  const int warps_per_cta = probe::kThreads / 32;
  const int grid = (n + warps_per_cta - 1) / warps_per_cta < 148 * 8
                       ? (n + warps_per_cta - 1) / warps_per_cta
                       : 148 * 8;
  probe::probe_logits_kernel<<<grid, probe::kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(hidden), hidden_row_stride,
      static_cast<const __nv_bfloat16*>(weight), weight_row_stride, q_len, vocab, hidden_dim, rows,
      toks, n, out, status);
  return hsd_host::cuda_check(cudaGetLastError(), "probe_logits_kernel launch");
}
