// The decoder's small steps as kernels: the sine embedding of the reference boxes, and the narrow linear layers
// of the heads (11 classes, 4 box coordinates) with the box refinement fused into the last one.
//
// Semantics:
//   ko_sine_embed      fast_rfdetr/model.py:188-194 (sine_embed): for the coordinates (y, x, w, h) of each box,
//                      v = coord * 2*pi / dim_t[k] (k < 128), emb = sin(v) at even k and cos(v) at odd k,
//                      the four 128-wide groups side by side -> [rows, 512]. The same fp32 operations in the same
//                      order (a multiply, then a division; sinf / cosf), with no contraction.
//   ko_linear_small_f32  x @ W + bias for outputs narrower than the tensor-core GEMM takes (N <= 32): the class
//                      heads (model.py:179, :269) and the last layer of the box MLPs (model.py:180, :270).
//   ko_box_head_f32    the last box-MLP layer (N = 4) and the refinement of model.py:271-272:
//                      boxes = (d0 * r2 + r0, d1 * r3 + r1, exp(d2) * r2, exp(d3) * r3) with d = x @ W + bias and r
//                      the reference box, as a multiply then an add (no fused multiply-add), like the reference's
//                      separate array operations.
//
// B200 design. The narrow layers are memory-bound and tiny (a [rows, 256] read and a few floats written per row):
// one warp per row, the lanes splitting K, the weight transposed into shared memory as [N][K], and fixed
// butterfly reductions — deterministic, and a tree sum over K rather than one long chain. For the model's K = 256
// (linear_small_vec_kernel) the grid is resident, each lane holds its 8 values of the row from two 128-bit loads
// and loads the next row's under the current row's arithmetic, and the N column sums share one transposed
// butterfly (each exchange halves the columns a lane carries: 16 shuffles for up to 16 columns instead of 5 per
// column); the 11-class head on 102 400 rows 112.6 -> 55.4 us. Other K take the general kernel (each lane reads 32
// consecutive floats of the row per step, one butterfly per column). The sine embedding is one thread per output
// element with 128-bit stores of four.
#include <algorithm>
#include <cmath>
#include <string>

#include "ko_common.cuh"

namespace {

constexpr int kWarps = 8;

__global__ void __launch_bounds__(256) sine_embed_kernel(const float* __restrict__ ref, const float* __restrict__ dim_t,
                                                         int64_t rows, float* __restrict__ out) {
  // thread -> four consecutive outputs of one row: group g (of 4 coordinates), frequencies k0..k0+3
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= rows * 128) return;
  const int64_t r = t >> 7;
  const int within = static_cast<int>(t & 127);  // 4-float chunk of the 512 outputs
  const int g = within >> 5, k0 = (within & 31) * 4;
  const int coord = g == 0 ? 1 : g == 1 ? 0 : g;  // (y, x, w, h)
  const float c = __fmul_rn(__ldg(ref + r * 4 + coord), 6.28318530717958647692f);
  float o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float v = __fdiv_rn(c, __ldg(dim_t + k0 + j));
    o[j] = ((k0 + j) & 1) ? cosf(v) : sinf(v);
  }
  reinterpret_cast<float4*>(out + r * 512)[within] = make_float4(o[0], o[1], o[2], o[3]);
}

// One warp per row (warps stride over the rows, so each CTA stages the weight once for many rows); acc[n] for
// the NMAX columns, lanes split K, butterfly-reduced. BOX: N == 4 and the box refinement with ref[row].
template <int NMAX, bool BOX>
__global__ void __launch_bounds__(kWarps * 32) linear_small_kernel(const float* __restrict__ x,
                                                                   const float* __restrict__ w,
                                                                   const float* __restrict__ bias,
                                                                   const float* __restrict__ ref, int64_t M, int K,
                                                                   int N, int act, float* __restrict__ out) {
  extern __shared__ float wt[];  // [N][K]
  for (int i = threadIdx.x; i < K * N; i += blockDim.x) {
    const int k = i / N, n = i - k * N;
    wt[n * K + k] = __ldg(w + i);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + warp; row < M;
       row += static_cast<int64_t>(gridDim.x) * kWarps) {
    const float* xr = x + row * K;
    float acc[NMAX];
#pragma unroll
    for (int n = 0; n < NMAX; ++n) acc[n] = 0.f;
    for (int k = lane; k < K; k += 32) {
      const float xv = __ldg(xr + k);
#pragma unroll
      for (int n = 0; n < NMAX; ++n)
        if (n < N) acc[n] = fmaf(xv, wt[n * K + k], acc[n]);
    }
#pragma unroll
    for (int n = 0; n < NMAX; ++n) {
      if (n >= N) break;
#pragma unroll
      for (int s = 16; s > 0; s >>= 1) acc[n] += __shfl_xor_sync(0xffffffffu, acc[n], s);
    }
    if (lane != 0) continue;
    if constexpr (BOX) {
      float d[4];
#pragma unroll
      for (int n = 0; n < 4; ++n) d[n] = acc[n] + (bias ? __ldg(bias + n) : 0.f);
      const float4 rb = __ldg(reinterpret_cast<const float4*>(ref) + row);
      float4 b;
      b.x = __fadd_rn(__fmul_rn(d[0], rb.z), rb.x);
      b.y = __fadd_rn(__fmul_rn(d[1], rb.w), rb.y);
      b.z = __fmul_rn(expf(d[2]), rb.z);
      b.w = __fmul_rn(expf(d[3]), rb.w);
      reinterpret_cast<float4*>(out)[row] = b;
    } else {
#pragma unroll
      for (int n = 0; n < NMAX; ++n) {
        if (n >= N) break;
        float v = acc[n] + (bias ? __ldg(bias + n) : 0.f);
        if (act == KO_ACT_RELU) v = fmaxf(v, 0.f);
        out[row * N + n] = v;
      }
    }
  }
}

// The same for K = 128 * KV (the model's K = 256) and 16-byte aligned rows: each lane holds its 4 * KV values of the
// row (128-bit loads, lane l reading columns 4l..4l+3 of every 128), loads the next row's while it computes this
// one, and reads the weight as float4 from shared memory. Sums a different grouping of the K terms than the
// general kernel, deterministically.
template <int NMAX, bool BOX, int KV>
__global__ void __launch_bounds__(kWarps * 32) linear_small_vec_kernel(const float* __restrict__ x,
                                                                       const float* __restrict__ w,
                                                                       const float* __restrict__ bias,
                                                                       const float* __restrict__ ref, int64_t M,
                                                                       int N, int act, float* __restrict__ out) {
  constexpr int K = 128 * KV;
  extern __shared__ float wt[];  // [N][K]
  for (int i = threadIdx.x; i < K * N; i += blockDim.x) {
    const int k = i / N, n = i - k * N;
    wt[n * K + k] = __ldg(w + i);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kWarps;
  int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
  float4 xv[KV];
  if (row < M) {
#pragma unroll
    for (int i = 0; i < KV; ++i) xv[i] = __ldg(reinterpret_cast<const float4*>(x + row * K) + 32 * i + lane);
  }
  for (; row < M; row += stride) {
    float4 cur[KV];
#pragma unroll
    for (int i = 0; i < KV; ++i) cur[i] = xv[i];
    if (row + stride < M) {  // the next row's values, in flight while this row is computed
#pragma unroll
      for (int i = 0; i < KV; ++i)
        xv[i] = __ldg(reinterpret_cast<const float4*>(x + (row + stride) * K) + 32 * i + lane);
    }
    float acc[NMAX];
#pragma unroll
    for (int n = 0; n < NMAX; ++n) {
      acc[n] = 0.f;
      if (n >= N) continue;
#pragma unroll
      for (int i = 0; i < KV; ++i) {
        const float4 wv = reinterpret_cast<const float4*>(wt + n * K)[32 * i + lane];
        acc[n] = fmaf(cur[i].x, wv.x, acc[n]);
        acc[n] = fmaf(cur[i].y, wv.y, acc[n]);
        acc[n] = fmaf(cur[i].z, wv.z, acc[n]);
        acc[n] = fmaf(cur[i].w, wv.w, acc[n]);
      }
    }
    if constexpr (BOX) {
#pragma unroll
      for (int n = 0; n < 4; ++n) {
#pragma unroll
        for (int s = 16; s > 0; s >>= 1) acc[n] += __shfl_xor_sync(0xffffffffu, acc[n], s);
      }
      if (lane != 0) continue;
      float d[4];
#pragma unroll
      for (int n = 0; n < 4; ++n) d[n] = acc[n] + (bias ? __ldg(bias + n) : 0.f);
      const float4 rb = __ldg(reinterpret_cast<const float4*>(ref) + row);
      float4 b;
      b.x = __fadd_rn(__fmul_rn(d[0], rb.z), rb.x);
      b.y = __fadd_rn(__fmul_rn(d[1], rb.w), rb.y);
      b.z = __fmul_rn(expf(d[2]), rb.z);
      b.w = __fmul_rn(expf(d[3]), rb.w);
      reinterpret_cast<float4*>(out)[row] = b;
    } else {
      // Transposed butterfly: each exchange halves the columns a lane carries (keeping the half its lane bit
      // selects, adding the partner's copy of it), so the NMAX sums take NMAX - 1 + log2(32 / NMAX) + 1
      // shuffles instead of 5 * NMAX. Afterwards lanes of column c hold its sum: c = (lane >> (5 - log2 NMAX)).
      static_assert(NMAX == 4 || NMAX == 16, "column counts of the transposed reduction");
#pragma unroll
      for (int width = NMAX / 2, bit = 16; width >= 1; width /= 2, bit /= 2) {
        const bool upper = (lane & bit) != 0;
#pragma unroll
        for (int j = 0; j < width; ++j) {
          const float keep = upper ? acc[width + j] : acc[j];
          const float give = upper ? acc[j] : acc[width + j];
          acc[j] = keep + __shfl_xor_sync(0xffffffffu, give, bit);
        }
      }
      constexpr int kLog = NMAX == 16 ? 4 : 2;
#pragma unroll
      for (int bit = 16 >> kLog; bit > 0; bit >>= 1) acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], bit);
      const int col = lane >> (5 - kLog);
      if ((lane & ((1 << (5 - kLog)) - 1)) == 0 && col < N) {
        float v = acc[0] + (bias ? __ldg(bias + col) : 0.f);
        if (act == KO_ACT_RELU) v = fmaxf(v, 0.f);
        out[row * N + col] = v;
      }
    }
  }
}

int check_small(const float* x, const float* w, int64_t M, int64_t K, int64_t N, const float* out, const char* who) {
  if (M < 0 || K < 1 || N < 1 || N > 32 || K > 4096 || K * N > 12288 || M > (int64_t(1) << 31))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": need 1 <= N <= 32, K <= 4096 and K*N <= 12288");
  if (M > 0 && (!x || !w || !out)) return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": null pointer");
  return KO_OK;
}

}  // namespace

extern "C" int ko_sine_embed(const float* ref, const float* dim_t, int64_t rows, float* out, ko_stream_t stream) {
  const char* who = "ko_sine_embed";
  if (rows < 0 || rows > (int64_t(1) << 28)) return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": bad rows");
  if (rows == 0) return KO_OK;
  if (!ref || !dim_t || !out || !ko::aligned16(out))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": null pointer or out not 16-byte aligned");
  const int64_t threads = rows * 128;
  sine_embed_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      ref, dim_t, rows, out);
  return ko::check_launch(who);
}

extern "C" int ko_linear_small_f32(const float* x, const float* w, const float* bias, int64_t M, int64_t K,
                                   int64_t N, int act, float* out, ko_stream_t stream) {
  const char* who = "ko_linear_small_f32";
  if (int st = check_small(x, w, M, K, N, out, who)) return st;
  if (act != KO_ACT_NONE && act != KO_ACT_RELU)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": act must be KO_ACT_NONE or KO_ACT_RELU");
  if (M == 0) return KO_OK;
  const ko::DeviceInfo* info = nullptr;
  if (int st = ko::device_or_fail(&info, who)) return st;
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((M + kWarps - 1) / kWarps, 8 * info->sm_count));
  const size_t smem = static_cast<size_t>(K * N) * 4;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int k = static_cast<int>(K), n = static_cast<int>(N);
  if (K == 256 && ko::aligned16(x) && N <= 16) {
    auto kern = N <= 4 ? linear_small_vec_kernel<4, false, 2> : linear_small_vec_kernel<16, false, 2>;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kWarps * 32, smem) != cudaSuccess || per_sm < 1)
      per_sm = 1;
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>((M + kWarps - 1) / kWarps,
                                                                  static_cast<int64_t>(per_sm) * info->sm_count));
    kern<<<grid, kWarps * 32, smem, s>>>(x, w, bias, nullptr, M, n, act, out);
    return ko::check_launch(who);
  }
  if (N <= 4)
    linear_small_kernel<4, false><<<blocks, kWarps * 32, smem, s>>>(x, w, bias, nullptr, M, k, n, act, out);
  else if (N <= 16)
    linear_small_kernel<16, false><<<blocks, kWarps * 32, smem, s>>>(x, w, bias, nullptr, M, k, n, act, out);
  else
    linear_small_kernel<32, false><<<blocks, kWarps * 32, smem, s>>>(x, w, bias, nullptr, M, k, n, act, out);
  return ko::check_launch(who);
}

extern "C" int ko_box_head_f32(const float* x, const float* w, const float* bias, const float* ref, int64_t M,
                               int64_t K, float* boxes, ko_stream_t stream) {
  const char* who = "ko_box_head_f32";
  if (int st = check_small(x, w, M, K, 4, boxes, who)) return st;
  if (M == 0) return KO_OK;
  if (!ref || !ko::aligned16(ref) || !ko::aligned16(boxes))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": ref and boxes must be 16-byte aligned");
  const ko::DeviceInfo* info = nullptr;
  if (int st = ko::device_or_fail(&info, who)) return st;
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((M + kWarps - 1) / kWarps, 8 * info->sm_count));
  if (K == 256 && ko::aligned16(x)) {
    linear_small_vec_kernel<4, true, 2><<<blocks, kWarps * 32, static_cast<size_t>(K * 4) * 4,
                                          reinterpret_cast<cudaStream_t>(stream)>>>(x, w, bias, ref, M, 4, KO_ACT_NONE,
                                                                                    boxes);
    return ko::check_launch(who);
  }
  linear_small_kernel<4, true><<<blocks, kWarps * 32, static_cast<size_t>(K * 4) * 4,
                                 reinterpret_cast<cudaStream_t>(stream)>>>(x, w, bias, ref, M, static_cast<int>(K), 4,
                                                                           KO_ACT_NONE, boxes);
  return ko::check_launch(who);
}
