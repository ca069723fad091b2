// Fused residual add + LayerNorm, fp32:  h_out = h + (o + bias) * scale;  y = LN(h_out) * gamma + beta.
//
// Semantics: the reference kernel fast_rfdetr/kernels.py:9-48 (residual_layernorm) and its unfused form
// model.py:140-141 / 144-145 with mx.fast.layer_norm (biased variance, eps inside the square root).
//
// B200 design: one warp per row; each lane keeps its V = C/128 float4 slices of the row in registers, so every
// byte of h and o is read once and every byte of h_out and y written once with 128-bit accesses. Mean and
// variance are two-pass (mean first, then the sum of squared deviations) with butterfly shuffles, a fixed
// reduction order, so results are deterministic run to run.
#include "ko_common.cuh"

namespace {

constexpr int kRowsPerBlock = 8;

template <int V>
__global__ void __launch_bounds__(32 * kRowsPerBlock) residual_ln_kernel(
    const float* h, const float* __restrict__ o, const float* __restrict__ bias, const float* __restrict__ scale,
    const float* __restrict__ gamma, const float* __restrict__ beta, float eps, int64_t rows, int C4,
    float* h_out, float* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kRowsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;
  // h may alias h_out, so it is read through the coherent path.
  const float4* h4 = reinterpret_cast<const float4*>(h) + row * C4;
  const float4* o4 = reinterpret_cast<const float4*>(o) + row * C4;
  float4 v[V];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + i * 32;
    if (c < C4) {
      const float4 hv = h4[c];
      const float4 ov = __ldg(o4 + c);
      const float4 bv = bias ? __ldg(reinterpret_cast<const float4*>(bias) + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 sv = scale ? __ldg(reinterpret_cast<const float4*>(scale) + c) : make_float4(1.f, 1.f, 1.f, 1.f);
      v[i].x = hv.x + (ov.x + bv.x) * sv.x;
      v[i].y = hv.y + (ov.y + bv.y) * sv.y;
      v[i].z = hv.z + (ov.z + bv.z) * sv.z;
      v[i].w = hv.w + (ov.w + bv.w) * sv.w;
      sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    } else {
      v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, s);
  const float inv_c = 1.0f / static_cast<float>(C4 * 4);
  const float mean = sum * inv_c;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + i * 32;
    if (c < C4) {
      const float dx = v[i].x - mean, dy = v[i].y - mean, dz = v[i].z - mean, dw = v[i].w - mean;
      sq += (dx * dx + dy * dy) + (dz * dz + dw * dw);
    }
  }
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, s);
  const float rstd = 1.0f / sqrtf(sq * inv_c + eps);
  float4* ho4 = reinterpret_cast<float4*>(h_out) + row * C4;
  float4* y4 = reinterpret_cast<float4*>(y) + row * C4;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + i * 32;
    if (c < C4) {
      const float4 g = __ldg(reinterpret_cast<const float4*>(gamma) + c);
      const float4 b = __ldg(reinterpret_cast<const float4*>(beta) + c);
      ho4[c] = v[i];
      float4 r;
      r.x = (v[i].x - mean) * rstd * g.x + b.x;
      r.y = (v[i].y - mean) * rstd * g.y + b.y;
      r.z = (v[i].z - mean) * rstd * g.z + b.z;
      r.w = (v[i].w - mean) * rstd * g.w + b.w;
      y4[c] = r;
    }
  }
}

template <int V>
int launch(const float* h, const float* o, const float* bias, const float* scale, const float* gamma,
           const float* beta, float eps, int64_t rows, int C4, float* h_out, float* y, cudaStream_t s) {
  const int64_t blocks = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
  residual_ln_kernel<V><<<static_cast<unsigned>(blocks), 32 * kRowsPerBlock, 0, s>>>(h, o, bias, scale, gamma, beta,
                                                                                   eps, rows, C4, h_out, y);
  return ko::check_launch("ko_residual_layernorm");
}

}  // namespace

extern "C" int ko_residual_layernorm(const float* h, const float* o, const float* bias, const float* scale,
                                     const float* gamma, const float* beta, float eps, int64_t rows, int64_t C,
                                     float* h_out, float* y, ko_stream_t stream) {
  if (rows < 0 || C < 4 || C % 4 != 0 || C > 1024)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_residual_layernorm: C must be a multiple of 4 in [4, 1024]");
  if (rows == 0) return KO_OK;
  if (!h || !o || !gamma || !beta || !h_out || !y)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_residual_layernorm: null pointer");
  const void* ptrs[] = {h, o, bias, scale, gamma, beta, h_out, y};
  for (const void* p : ptrs)
    if (p && !ko::aligned16(p)) return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_residual_layernorm: pointers must be 16-byte aligned");
  if (rows > (int64_t(1) << 31) * kRowsPerBlock)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_residual_layernorm: too many rows");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int C4 = static_cast<int>(C / 4);
  const int V = (C4 + 31) / 32;
  switch (V) {
    case 1: return launch<1>(h, o, bias, scale, gamma, beta, eps, rows, C4, h_out, y, s);
    case 2: return launch<2>(h, o, bias, scale, gamma, beta, eps, rows, C4, h_out, y, s);
    case 3: return launch<3>(h, o, bias, scale, gamma, beta, eps, rows, C4, h_out, y, s);
    case 4: return launch<4>(h, o, bias, scale, gamma, beta, eps, rows, C4, h_out, y, s);
    case 5: return launch<5>(h, o, bias, scale, gamma, beta, eps, rows, C4, h_out, y, s);
    case 6: return launch<6>(h, o, bias, scale, gamma, beta, eps, rows, C4, h_out, y, s);
    case 7: return launch<7>(h, o, bias, scale, gamma, beta, eps, rows, C4, h_out, y, s);
    default: return launch<8>(h, o, bias, scale, gamma, beta, eps, rows, C4, h_out, y, s);
  }
}
