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
// The backbone's window entry (ko_window_partition_ln: pos add, window partition, class token, first LayerNorm)
// and window merge (ko_window_merge_ln: final LayerNorm of a tapped layer into its channel slice of the projector
// input) use the same one-warp-per-row scheme, with the row's source or destination remapped.
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

// ---------------------------------------------------------------------------------------------------------
// Window merge (+ LayerNorm) into a channel slice: the ViT backbone keeps its tokens in window order
// [B * nwin][1 + win*win][C] (a class token, then the window's pixels row by row; windows row-major over the
// grid). A feature map for the projector wants them as an NHWC image; the projector then concatenates four such
// maps along channels. This kernel writes, for every pixel (b, py, px),
//   out[((b * H + py) * W + px) * ldo + col_off + c] = LN(h[(b * nwin + w) * (1 + win*win) + 1 + iy * win + ix][c])
// (or the row itself with normalize = 0), where w = (py / win) * (W / win) + px / win, iy = py % win,
// ix = px % win: the reference's window merge (fast_rfdetr/model.py:104-105) fused with the final LayerNorm of
// the tapped layers (model.py:101-103) and the channel concatenation of the projector input (model.py:161), in
// one pass per tapped layer. One warp per pixel; the LayerNorm is the two-pass one of residual_ln_kernel.
// ---------------------------------------------------------------------------------------------------------
namespace {

template <int V>
__global__ void __launch_bounds__(32 * kRowsPerBlock) window_merge_kernel(
    const float* __restrict__ h, const float* __restrict__ gamma, const float* __restrict__ beta, float eps,
    int64_t pixels, int H, int W, int win, int C4, int normalize, float* __restrict__ out, int64_t ldo4,
    int64_t col4) {
  const int lane = threadIdx.x & 31;
  const int64_t p = static_cast<int64_t>(blockIdx.x) * kRowsPerBlock + (threadIdx.x >> 5);
  if (p >= pixels) return;
  const int64_t b = p / (static_cast<int64_t>(H) * W);
  const int rem = static_cast<int>(p - b * H * W);
  const int py = rem / W, px = rem - py * W;
  const int nwx = W / win, nwin = (H / win) * nwx;
  const int w = (py / win) * nwx + px / win;
  const int64_t row = (b * nwin + w) * (1 + win * win) + 1 + (py % win) * win + (px % win);
  const float4* src = reinterpret_cast<const float4*>(h) + row * C4;
  float4* dst = reinterpret_cast<float4*>(out) + p * ldo4 + col4;
  float4 v[V];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + i * 32;
    v[i] = c < C4 ? __ldg(src + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
  if (!normalize) {
#pragma unroll
    for (int i = 0; i < V; ++i)
      if (lane + i * 32 < C4) dst[lane + i * 32] = v[i];
    return;
  }
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, s);
  const float inv_c = 1.0f / static_cast<float>(C4 * 4);
  const float mean = sum * inv_c;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    if (lane + i * 32 < C4) {
      const float dx = v[i].x - mean, dy = v[i].y - mean, dz = v[i].z - mean, dw = v[i].w - mean;
      sq += (dx * dx + dy * dy) + (dz * dz + dw * dw);
    }
  }
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, s);
  const float rstd = 1.0f / sqrtf(sq * inv_c + eps);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + i * 32;
    if (c < C4) {
      const float4 g = __ldg(reinterpret_cast<const float4*>(gamma) + c);
      const float4 bt = __ldg(reinterpret_cast<const float4*>(beta) + c);
      dst[c] = make_float4((v[i].x - mean) * rstd * g.x + bt.x, (v[i].y - mean) * rstd * g.y + bt.y,
                           (v[i].z - mean) * rstd * g.z + bt.z, (v[i].w - mean) * rstd * g.w + bt.w);
    }
  }
}

}  // namespace

extern "C" int ko_window_merge_ln(const float* h, const float* gamma, const float* beta, float eps, int64_t B,
                                  int64_t H, int64_t W, int64_t win, int64_t C, int normalize, float* out,
                                  int64_t ldo, int64_t col_off, ko_stream_t stream) {
  const char* who = "ko_window_merge_ln";
  if (B < 0 || H < 1 || W < 1 || win < 1 || H % win != 0 || W % win != 0 || C < 4 || C % 4 != 0 || C > 1024 ||
      ldo % 4 != 0 || col_off % 4 != 0 || col_off < 0 || col_off + C > ldo)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": need H, W multiples of win, C % 4 == 0, "
                                                                "C <= 1024, col_off + C <= ldo (multiples of 4)");
  if (B == 0) return KO_OK;
  if (!h || !out || (normalize && (!gamma || !beta)))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": null pointer");
  if (!ko::aligned16(h) || !ko::aligned16(out) || (normalize && (!ko::aligned16(gamma) || !ko::aligned16(beta))))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": pointers must be 16-byte aligned");
  const int64_t pixels = B * H * W;
  const int64_t blocks = (pixels + kRowsPerBlock - 1) / kRowsPerBlock;
  if (blocks > 0x7fffffff) return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": too many pixels");
  const int C4 = static_cast<int>(C / 4);
  const int V = (C4 + 31) / 32;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned g = static_cast<unsigned>(blocks);
#define KO_WM(VV)                                                                                           \
  window_merge_kernel<VV><<<g, 32 * kRowsPerBlock, 0, s>>>(h, gamma, beta, eps, pixels, static_cast<int>(H), \
                                                            static_cast<int>(W), static_cast<int>(win), C4,   \
                                                            normalize, out, ldo / 4, col_off / 4)
  switch (V) {
    case 1: KO_WM(1); break;
    case 2: KO_WM(2); break;
    case 3: KO_WM(3); break;
    case 4: KO_WM(4); break;
    case 5: KO_WM(5); break;
    case 6: KO_WM(6); break;
    case 7: KO_WM(7); break;
    default: KO_WM(8); break;
  }
#undef KO_WM
  return ko::check_launch(who);
}

// ---------------------------------------------------------------------------------------------------------
// Window partition of the patch embedding + the first layer's LayerNorm (ko_window_partition_ln).
// Semantics: fast_rfdetr/model.py:88-90 and :94 — t + pos over the H x W token grid, cut into (H/win) x (W/win)
// windows of win x win tokens (row-major), each window preceded by the class token, then y = LayerNorm(h) with
// the first layer's norm1. One warp per output token row: it reads the patch-embedding row and the pos row (or the
// class token), writes h and the two-pass LayerNorm of it. Replaces the pos add, the window permute copy, the class
// token concatenation and the separate LayerNorm pass.
// ---------------------------------------------------------------------------------------------------------
namespace {

template <int V>
__global__ void __launch_bounds__(32 * kRowsPerBlock) window_partition_kernel(
    const float* __restrict__ t, const float* __restrict__ pos, const float* __restrict__ cls,
    const float* __restrict__ gamma, const float* __restrict__ beta, float eps, int64_t rows, int H, int W, int win,
    int C4, float* __restrict__ h, float* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kRowsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int per = 1 + win * win, nwx = W / win, nwin = (H / win) * nwx;
  const int64_t n = row / per;  // window index over the batch
  const int r = static_cast<int>(row - n * per);
  const float4* src;
  const float4* add = nullptr;
  if (r == 0) {
    src = reinterpret_cast<const float4*>(cls);
  } else {
    const int64_t bi = n / nwin;
    const int w = static_cast<int>(n - bi * nwin);
    const int py = (w / nwx) * win + (r - 1) / win, px = (w % nwx) * win + (r - 1) % win;
    src = reinterpret_cast<const float4*>(t) + ((bi * H + py) * W + px) * C4;
    add = reinterpret_cast<const float4*>(pos) + (static_cast<int64_t>(py) * W + px) * C4;
  }
  float4 v[V];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + i * 32;
    v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c < C4) {
      v[i] = __ldg(src + c);
      if (add) {
        const float4 p = __ldg(add + c);
        v[i] = make_float4(v[i].x + p.x, v[i].y + p.y, v[i].z + p.z, v[i].w + p.w);
      }
      reinterpret_cast<float4*>(h)[row * C4 + c] = v[i];
    }
    sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, s);
  const float inv_c = 1.0f / static_cast<float>(C4 * 4);
  const float mean = sum * inv_c;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    if (lane + i * 32 < C4) {
      const float dx = v[i].x - mean, dy = v[i].y - mean, dz = v[i].z - mean, dw = v[i].w - mean;
      sq += (dx * dx + dy * dy) + (dz * dz + dw * dw);
    }
  }
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, s);
  const float rstd = 1.0f / sqrtf(sq * inv_c + eps);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + i * 32;
    if (c < C4) {
      const float4 g = __ldg(reinterpret_cast<const float4*>(gamma) + c);
      const float4 bt = __ldg(reinterpret_cast<const float4*>(beta) + c);
      reinterpret_cast<float4*>(y)[row * C4 + c] =
          make_float4((v[i].x - mean) * rstd * g.x + bt.x, (v[i].y - mean) * rstd * g.y + bt.y,
                      (v[i].z - mean) * rstd * g.z + bt.z, (v[i].w - mean) * rstd * g.w + bt.w);
    }
  }
}

}  // namespace

extern "C" int ko_window_partition_ln(const float* t, const float* pos, const float* cls, const float* gamma,
                                      const float* beta, float eps, int64_t B, int64_t H, int64_t W, int64_t win,
                                      int64_t C, float* h, float* y, ko_stream_t stream) {
  const char* who = "ko_window_partition_ln";
  if (B < 0 || H < 1 || W < 1 || win < 1 || H % win != 0 || W % win != 0 || C < 4 || C % 4 != 0 || C > 1024 ||
      H * W > (int64_t(1) << 30))
    return ko::fail(KO_ERR_INVALID_ARGUMENT,
                    std::string(who) + ": need H, W multiples of win, C % 4 == 0 and C <= 1024");
  if (B == 0) return KO_OK;
  if (!t || !pos || !cls || !gamma || !beta || !h || !y)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": null pointer");
  if (!ko::aligned16(t) || !ko::aligned16(pos) || !ko::aligned16(cls) || !ko::aligned16(gamma) ||
      !ko::aligned16(beta) || !ko::aligned16(h) || !ko::aligned16(y))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": pointers must be 16-byte aligned");
  const int64_t rows = B * (H / win) * (W / win) * (1 + win * win);
  const int64_t blocks = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
  if (blocks > 0x7fffffff) return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": too many rows");
  const int C4 = static_cast<int>(C / 4);
  const int V = (C4 + 31) / 32;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned g = static_cast<unsigned>(blocks);
#define KO_WP(VV)                                                                                                \
  window_partition_kernel<VV><<<g, 32 * kRowsPerBlock, 0, s>>>(t, pos, cls, gamma, beta, eps, rows,                \
                                                               static_cast<int>(H), static_cast<int>(W),          \
                                                               static_cast<int>(win), C4, h, y)
  switch (V) {
    case 1: KO_WP(1); break;
    case 2: KO_WP(2); break;
    case 3: KO_WP(3); break;
    case 4: KO_WP(4); break;
    case 5: KO_WP(5); break;
    case 6: KO_WP(6); break;
    case 7: KO_WP(7); break;
    default: KO_WP(8); break;
  }
#undef KO_WP
  return ko::check_launch(who);
}
