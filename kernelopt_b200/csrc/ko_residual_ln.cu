// Fused residual add + LayerNorm, fp32:  h_out = h + (o + bias) * scale;  y = LN(h_out) * gamma + beta.
// The same kernel without the residual (ko_layernorm) is the plain LayerNorm of the model's other norms, with an
// optional SiLU on its output (the projector's conv -> channel LayerNorm -> SiLU blocks, model.py:148-158).
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

__device__ __forceinline__ float apply_act(float r, int act) {
  return act == KO_ACT_SILU ? r / (1.0f + expf(-r)) : r;
}

// RESID: h_out = h + (o + bias) * scale is normalised (and written); otherwise h itself is normalised and h_out is
// not written (plain LayerNorm). ACT: KO_ACT_NONE or KO_ACT_SILU on the normalised output.
template <int V, bool RESID>
__global__ void __launch_bounds__(32 * kRowsPerBlock) residual_ln_kernel(
    const float* h, const float* __restrict__ o, const float* __restrict__ bias, const float* __restrict__ scale,
    const float* __restrict__ gamma, const float* __restrict__ beta, float eps, int64_t rows, int C4,
    float* h_out, float* __restrict__ y, int act) {
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
    if (c < C4 && !RESID) {
      v[i] = h4[c];
      sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    } else if (c < C4) {
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
      if (RESID) ho4[c] = v[i];
      float4 r;
      r.x = apply_act((v[i].x - mean) * rstd * g.x + b.x, act);
      r.y = apply_act((v[i].y - mean) * rstd * g.y + b.y, act);
      r.z = apply_act((v[i].z - mean) * rstd * g.z + b.z, act);
      r.w = apply_act((v[i].w - mean) * rstd * g.w + b.w, act);
      y4[c] = r;
    }
  }
}

template <int V>
int launch(const float* h, const float* o, const float* bias, const float* scale, const float* gamma,
           const float* beta, float eps, int64_t rows, int C4, float* h_out, float* y, int act, cudaStream_t s) {
  const int64_t blocks = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
  if (o)
    residual_ln_kernel<V, true><<<static_cast<unsigned>(blocks), 32 * kRowsPerBlock, 0, s>>>(
        h, o, bias, scale, gamma, beta, eps, rows, C4, h_out, y, act);
  else
    residual_ln_kernel<V, false><<<static_cast<unsigned>(blocks), 32 * kRowsPerBlock, 0, s>>>(
        h, o, bias, scale, gamma, beta, eps, rows, C4, h_out, y, act);
  return ko::check_launch(o ? "ko_residual_layernorm" : "ko_layernorm");
}

int dispatch(const float* h, const float* o, const float* bias, const float* scale, const float* gamma,
             const float* beta, float eps, int64_t rows, int64_t C, float* h_out, float* y, int act,
             cudaStream_t s) {
  const int C4 = static_cast<int>(C / 4);
  const int V = (C4 + 31) / 32;
  switch (V) {
    case 1: return launch<1>(h, o, bias, scale, gamma, beta, eps, rows, C4, h_out, y, act, s);
    case 2: return launch<2>(h, o, bias, scale, gamma, beta, eps, rows, C4, h_out, y, act, s);
    case 3: return launch<3>(h, o, bias, scale, gamma, beta, eps, rows, C4, h_out, y, act, s);
    case 4: return launch<4>(h, o, bias, scale, gamma, beta, eps, rows, C4, h_out, y, act, s);
    case 5: return launch<5>(h, o, bias, scale, gamma, beta, eps, rows, C4, h_out, y, act, s);
    case 6: return launch<6>(h, o, bias, scale, gamma, beta, eps, rows, C4, h_out, y, act, s);
    case 7: return launch<7>(h, o, bias, scale, gamma, beta, eps, rows, C4, h_out, y, act, s);
    default: return launch<8>(h, o, bias, scale, gamma, beta, eps, rows, C4, h_out, y, act, s);
  }
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
  return dispatch(h, o, bias, scale, gamma, beta, eps, rows, C, h_out, y, KO_ACT_NONE,
                  reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int ko_layernorm(const float* x, const float* gamma, const float* beta, float eps, int64_t rows, int64_t C,
                            int act, float* y, ko_stream_t stream) {
  if (rows < 0 || C < 4 || C % 4 != 0 || C > 1024)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_layernorm: C must be a multiple of 4 in [4, 1024]");
  if (act != KO_ACT_NONE && act != KO_ACT_SILU)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_layernorm: act must be KO_ACT_NONE or KO_ACT_SILU");
  if (rows == 0) return KO_OK;
  if (!x || !gamma || !beta || !y) return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_layernorm: null pointer");
  const void* ptrs[] = {x, gamma, beta, y};
  for (const void* p : ptrs)
    if (!ko::aligned16(p)) return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_layernorm: pointers must be 16-byte aligned");
  if (rows > (int64_t(1) << 31) * kRowsPerBlock) return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_layernorm: too many rows");
  return dispatch(x, nullptr, nullptr, nullptr, gamma, beta, eps, rows, C, nullptr, y, act,
                  reinterpret_cast<cudaStream_t>(stream));
}
