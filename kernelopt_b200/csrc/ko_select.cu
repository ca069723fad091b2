// Query selection on the device: the top-NQ proposals by class score and their refined reference boxes.
//
// Semantics: RFDETR.select_queries, fast_rfdetr/model.py:175-185:
//   scores[b, i] = max_c logits[b, i, c]
//   coord[b, i]  = (delta_xy * prop_wh + prop_xy, exp(delta_wh) * prop_wh)
//   idx[b, :]    = argsort(-scores[b])[:NQ]
//   ref[b, q]    = (rp_xy[q] * coord_wh + coord_xy, rp_ewh[q] * coord_wh)   with coord = coord[b, idx[b, q]]
// Ties in score (-0 and +0 included) are ordered by ascending proposal index (the order of a stable sort), so the
// selection is deterministic; NaN scores rank last.
//
// B200 design: one CTA per frame. Each proposal's score becomes a 64-bit key (an order-reversing map of the fp32
// score in the high word, the index in the low word), so one ascending bitonic sort in shared memory yields
// descending scores with ties by index. Up to 4096 proposals (32 KB of keys); 1024 threads. Only the NQ selected
// proposals get their boxes refined.
#include "ko_common.cuh"

namespace {

constexpr int kThreads = 1024;
constexpr int kMaxProposals = 4096;

// Monotone map of fp32 to uint32 (a < b  =>  key(a) < key(b)) for non-NaN values.
__device__ __forceinline__ uint32_t ordered(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void __launch_bounds__(kThreads) select_kernel(const float* __restrict__ logits,
                                                          const float* __restrict__ delta,
                                                          const float* __restrict__ prop,
                                                          const float* __restrict__ rp_xy,
                                                          const float* __restrict__ rp_ewh, int np, int nc, int nq,
                                                          int n2, float* __restrict__ ref, int* __restrict__ idx_out) {
  extern __shared__ unsigned long long keys[];
  const int b = blockIdx.x;
  const float* lg = logits + static_cast<int64_t>(b) * np * nc;
  for (int i = threadIdx.x; i < n2; i += kThreads) {
    unsigned long long key = ~0ull;  // padding sorts last
    if (i < np) {
      float s = lg[static_cast<int64_t>(i) * nc];
      for (int c = 1; c < nc; ++c) s = fmaxf(s, lg[static_cast<int64_t>(i) * nc + c]);
      if (s == 0.0f) s = 0.0f;  // -0 ties with +0
      // a NaN score ranks below every number (the place a sort of -score puts it)
      const uint32_t hi = s != s ? 0xFFFFFFFEu : ~ordered(s);
      key = (static_cast<unsigned long long>(hi) << 32) | static_cast<uint32_t>(i);
    }
    keys[i] = key;
  }
  __syncthreads();
  // ascending bitonic sort of n2 (a power of two) keys
  for (int k = 2; k <= n2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n2; i += kThreads) {
        const int l = i ^ j;
        if (l > i) {
          const unsigned long long a = keys[i], c = keys[l];
          const bool up = (i & k) == 0;
          if ((a > c) == up) {
            keys[i] = c;
            keys[l] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int q = threadIdx.x; q < nq; q += kThreads) {
    const int i = static_cast<int>(keys[q] & 0xFFFFFFFFull);
    const float4 d = reinterpret_cast<const float4*>(delta)[static_cast<int64_t>(b) * np + i];
    const float4 p = reinterpret_cast<const float4*>(prop)[i];
    const float cx = d.x * p.z + p.x, cy = d.y * p.w + p.y;
    const float w = expf(d.z) * p.z, h = expf(d.w) * p.w;
    const float2 rxy = reinterpret_cast<const float2*>(rp_xy)[q];
    const float2 rwh = reinterpret_cast<const float2*>(rp_ewh)[q];
    reinterpret_cast<float4*>(ref)[static_cast<int64_t>(b) * nq + q] =
        make_float4(rxy.x * w + cx, rxy.y * h + cy, rwh.x * w, rwh.y * h);
    if (idx_out) idx_out[static_cast<int64_t>(b) * nq + q] = i;
  }
}

}  // namespace

extern "C" int ko_select_queries(const float* logits, const float* delta, const float* proposals, const float* rp_xy,
                                 const float* rp_ewh, int64_t B, int64_t NP, int64_t NC, int64_t NQ, float* ref,
                                 int32_t* idx, ko_stream_t stream) {
  const char* who = "ko_select_queries";
  if (B < 0 || NP < 1 || NP > kMaxProposals || NC < 1 || NQ < 1 || NQ > NP)
    return ko::fail(KO_ERR_INVALID_ARGUMENT,
                    std::string(who) + ": need 1 <= NQ <= NP <= 4096 proposals and NC >= 1 classes");
  if (B == 0) return KO_OK;
  if (!logits || !delta || !proposals || !rp_xy || !rp_ewh || !ref)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": null pointer");
  if (!ko::aligned16(delta) || !ko::aligned16(proposals) || !ko::aligned16(ref) ||
      (reinterpret_cast<uintptr_t>(rp_xy) & 7) != 0 || (reinterpret_cast<uintptr_t>(rp_ewh) & 7) != 0)
    return ko::fail(KO_ERR_INVALID_ARGUMENT,
                    std::string(who) + ": delta, proposals, ref 16-byte aligned; rp_xy, rp_ewh 8-byte aligned");
  if (B > 0x7fffffff) return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": batch too large");
  int n2 = 2;
  while (n2 < NP) n2 <<= 1;
  const size_t smem = static_cast<size_t>(n2) * sizeof(unsigned long long);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return ko::fail(static_cast<int>(e), std::string(who) + ": cudaFuncSetAttribute failed");
  }
  select_kernel<<<static_cast<unsigned>(B), kThreads, smem, st>>>(logits, delta, proposals, rp_xy, rp_ewh,
                                                                   static_cast<int>(NP), static_cast<int>(NC),
                                                                   static_cast<int>(NQ), n2, ref, idx);
  return ko::check_launch(who);
}
