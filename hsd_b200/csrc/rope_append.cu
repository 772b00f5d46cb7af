// Rotary position embedding of a layer's new query / key rows fused with the
// KV-cache update, in one launch.
//
// The reference's patched Qwen2 attention (hsd/dots_ocr_pipeline/
// modeling_dots_ocr_hsd.py D:337-351) projects the step's rows, applies
// transformers' apply_rotary_pos_emb -- q * cos + rotate_half(q) * sin in
// bf16 tensor ops, rotate_half(x) = cat(-x[d/2:], x[:d/2]) -- to the query
// and key states, and appends key and value states to the DynamicCache with
// torch.cat (a copy of the layer's whole cache).  Here the query rows are
// rotated in place in the projection output (the attention kernel reads them
// with row stride Hq * D and head stride D), and the rotated key rows and the
// value rows are written straight into the cache planes at their final rows.
// The arithmetic is the one torch's bf16 kernels perform: each product
// rounded to bf16, the two bf16 products summed in fp32 and rounded to bf16,
// so the results are bit-identical.
//
// Work unit: 8 consecutive dimensions i..i+7 of the first half of one head of
// one row together with their partners i+64..i+71 (16-byte loads and
// stores), for query and key heads; 16 bytes of one value row.  HBM bound:
// per row, query rows are read and written once, key and value rows read
// once and written once, cos / sin read once per row (L2 serves the heads).
#include "common.cuh"

namespace hsd {
namespace rope {

constexpr int kThreads = 256;

struct Params {
  __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  const __nv_bfloat16* cos;
  const __nv_bfloat16* sin;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  int64_t q_row_stride, kv_row_stride, cs_row_stride;
  int64_t kc_head_stride, vc_head_stride, cache_row_stride;
  int n_rows, hq, hkv, dst_row0;
  int n_q, n_k, n_v;  // work units of each kind
};

__device__ __forceinline__ uint4 ld16(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}
__device__ __forceinline__ void st16(void* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }

__device__ __forceinline__ float lo_f(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_f(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ float rn(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(lo))) |
         (uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(hi))) << 16);
}

// y1 = x1 * c1 - x2 * s1, y2 = x2 * c2 + x1 * s2 on 8 lanes, with torch's
// bf16 rounding of each product and of the sum.
__device__ __forceinline__ void rotate8(uint4 a, uint4 b, uint4 c1, uint4 c2, uint4 s1, uint4 s2,
                                        uint4& y1, uint4& y2) {
  const uint32_t* A = &a.x;
  const uint32_t* B = &b.x;
  const uint32_t* C1 = &c1.x;
  const uint32_t* C2 = &c2.x;
  const uint32_t* S1 = &s1.x;
  const uint32_t* S2 = &s2.x;
  uint32_t* Y1 = &y1.x;
  uint32_t* Y2 = &y2.x;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    float r1[2], r2[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float x1 = h ? hi_f(A[w]) : lo_f(A[w]);
      const float x2 = h ? hi_f(B[w]) : lo_f(B[w]);
      const float cc1 = h ? hi_f(C1[w]) : lo_f(C1[w]);
      const float cc2 = h ? hi_f(C2[w]) : lo_f(C2[w]);
      const float ss1 = h ? hi_f(S1[w]) : lo_f(S1[w]);
      const float ss2 = h ? hi_f(S2[w]) : lo_f(S2[w]);
      r1[h] = __fadd_rn(rn(__fmul_rn(x1, cc1)), rn(__fmul_rn(-x2, ss1)));
      r2[h] = __fadd_rn(rn(__fmul_rn(x2, cc2)), rn(__fmul_rn(x1, ss2)));
    }
    Y1[w] = pack2(r1[0], r1[1]);
    Y2[w] = pack2(r2[0], r2[1]);
  }
}

// One work unit's operands: kind 0 = query / key (a, b = the two halves'
// 8 lanes, c1..s2 = cos / sin), kind 1 = value (a = 16 bytes), kind 2 = none.
struct Unit {
  uint4 a, b, c1, c2, s1, s2;
  __nv_bfloat16* dst;
  int kind;
};

__device__ __forceinline__ void load_unit(const Params& p, int u, Unit& w) {
  const int nqk = p.n_q + p.n_k;
  if (u >= p.n_q + p.n_k + p.n_v) {
    w.kind = 2;
  } else if (u < nqk) {
    const bool is_q = u < p.n_q;
    const int t = is_q ? u : u - p.n_q;
    const int heads = is_q ? p.hq : p.hkv;
    const int c = t & 7;  // 8-lane group of the first half
    const int rh = t >> 3;
    const int row = rh / heads, head = rh - (rh / heads) * heads;
    const __nv_bfloat16* cs = p.cos + size_t(row) * p.cs_row_stride + c * 8;
    const __nv_bfloat16* sn = p.sin + size_t(row) * p.cs_row_stride + c * 8;
    const __nv_bfloat16* src =
        is_q ? p.q + size_t(row) * p.q_row_stride + head * 128 + c * 8
             : p.k + size_t(row) * p.kv_row_stride + head * 128 + c * 8;
    w.a = ld16(src);
    w.b = ld16(src + 64);
    w.c1 = ld16(cs);
    w.c2 = ld16(cs + 64);
    w.s1 = ld16(sn);
    w.s2 = ld16(sn + 64);
    w.dst = is_q ? p.q + size_t(row) * p.q_row_stride + head * 128 + c * 8
                 : p.k_cache + size_t(head) * p.kc_head_stride +
                       size_t(p.dst_row0 + row) * p.cache_row_stride + c * 8;
    w.kind = 0;
  } else {
    const int t = u - nqk;
    const int c = t & 15;  // 16-byte chunk of the row
    const int rh = t >> 4;
    const int row = rh / p.hkv, head = rh - (rh / p.hkv) * p.hkv;
    w.a = ld16(p.v + size_t(row) * p.kv_row_stride + head * 128 + c * 8);
    w.dst = p.v_cache + size_t(head) * p.vc_head_stride +
            size_t(p.dst_row0 + row) * p.cache_row_stride + c * 8;
    w.kind = 1;
  }
}

__device__ __forceinline__ void store_unit(const Unit& w) {
  if (w.kind == 0) {
    uint4 y1, y2;
    rotate8(w.a, w.b, w.c1, w.c2, w.s1, w.s2, y1, y2);
    st16(w.dst, y1);
    st16(w.dst + 64, y2);
  } else if (w.kind == 1) {
    st16(w.dst, w.a);
  }
}

// One wave of CTAs (eight of 256 threads per SM) walks the units a grid
// apart; more units per thread, or more CTAs than one wave, measured slower.
__global__ void __launch_bounds__(kThreads) rope_append_kernel(const Params p) {
  // Launched with programmatic dependent launch: the CTAs are scheduled
  // while the previous kernel on the stream finishes, and nothing is read
  // before it has completed.  The next kernel may be scheduled at once: it
  // waits for this one's completion in its own griddepcontrol.wait.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int total = p.n_q + p.n_k + p.n_v;
  const int stride = int(gridDim.x) * kThreads;
  for (int u = int(blockIdx.x) * kThreads + int(threadIdx.x); u < total; u += stride) {
    Unit w;
    load_unit(p, u, w);
    store_unit(w);
  }
}

}  // namespace rope
}  // namespace hsd

extern "C" int hsd_rope_append(void* q, int64_t q_row_stride, const void* k, const void* v,
                               int64_t kv_row_stride, const void* cos_emb, const void* sin_emb,
                               int64_t cs_row_stride, int32_t n_rows, int32_t num_q_heads,
                               int32_t num_kv_heads, int32_t head_dim, void* k_cache,
                               int64_t k_cache_head_stride, void* v_cache,
                               int64_t v_cache_head_stride, int64_t cache_row_stride,
                               int32_t dst_row0, hsd_stream_t stream) {
  using namespace hsd;
  if (head_dim != 128) {
    hsd_host::set_error("hsd_rope_append: head_dim %d unsupported (128 only)", head_dim);
    return HSD_ERR_UNSUPPORTED;
  }
  auto a16 = [](const void* x) { return x && (reinterpret_cast<uintptr_t>(x) & 15) == 0; };
  if (n_rows < 0 || num_q_heads < 0 || num_kv_heads <= 0 || dst_row0 < 0 ||
      (num_q_heads > 0 && (!a16(q) || q_row_stride < int64_t(num_q_heads) * 128)) ||
      !a16(k) || !a16(v) || !a16(cos_emb) || !a16(sin_emb) || !a16(k_cache) || !a16(v_cache) ||
      kv_row_stride < int64_t(num_kv_heads) * 128 || cs_row_stride < 128 ||
      cache_row_stride < 128 || (q_row_stride % 8) || (kv_row_stride % 8) ||
      (cs_row_stride % 8) || (cache_row_stride % 8) || (k_cache_head_stride % 8) ||
      (v_cache_head_stride % 8)) {
    hsd_host::set_error(
        "hsd_rope_append: bad arguments (rows=%d heads=%d/%d; pointers 16-byte aligned, "
        "strides multiples of 8 elements covering the heads)",
        n_rows, num_q_heads, num_kv_heads);
    return HSD_ERR_INVALID_ARG;
  }
  if (n_rows == 0) return HSD_OK;
  rope::Params p;
  p.q = static_cast<__nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.cos = static_cast<const __nv_bfloat16*>(cos_emb);
  p.sin = static_cast<const __nv_bfloat16*>(sin_emb);
  p.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  p.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  p.q_row_stride = q_row_stride;
  p.kv_row_stride = kv_row_stride;
  p.cs_row_stride = cs_row_stride;
  p.kc_head_stride = k_cache_head_stride;
  p.vc_head_stride = v_cache_head_stride;
  p.cache_row_stride = cache_row_stride;
  p.n_rows = n_rows;
  p.hq = num_q_heads;
  p.hkv = num_kv_heads;
  p.dst_row0 = dst_row0;
  const int64_t total = int64_t(n_rows) * (num_q_heads * 8 + num_kv_heads * 24);
  if (total >= (int64_t(1) << 30)) {
    hsd_host::set_error("hsd_rope_append: %d rows x %d heads exceed the launch's index range",
                        n_rows, num_q_heads + num_kv_heads);
    return HSD_ERR_TOO_LARGE;
  }
  p.n_q = n_rows * num_q_heads * 8;
  p.n_k = n_rows * num_kv_heads * 8;
  p.n_v = n_rows * num_kv_heads * 16;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    sms = 148;
  const int64_t blocks = (total + rope::kThreads - 1) / rope::kThreads;
  const int grid = int(blocks < int64_t(sms) * 8 ? blocks : int64_t(sms) * 8);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(rope::kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return hsd_host::cuda_check(cudaLaunchKernelEx(&cfg, rope::rope_append_kernel, p),
                              "rope_append_kernel launch");
}
