// Deformable-attention bilinear sampling with the attention-weighted sum over points (single feature level).
//
// Semantics: the reference kernel fast_rfdetr/kernels.py:124-162 (deform_attn_sample) and the unfused form
// model.py:196-216 + 228-229, i.e. ONNX GridSample (bilinear, zero padding, align_corners=False) on the grid
// 2*loc - 1, then sum_p aw * sample:
//   x = loc_x * GW - 0.5, y = loc_y * GH - 0.5, x0 = floor(x), fx = x - x0 (same for y); taps outside the
//   GH x GW map contribute 0; s_p = sum over the 4 taps of w_x * w_y * value; out = sum_p aw_p * s_p.
//
// B200 design. The value map of one frame and layer is 40x40 tokens x 256 channels (1.6 MB); the batch's maps
// stay resident in the 126 MB L2 while they are sampled, so the kernels gather straight from global memory.
// Four lanes serve one (query, head): each lane owns 4 of the head's 16 channels, so a tap is one 64-byte
// contiguous read by a lane quad (128-bit loads, 2 full sectors), the quad's sampling coordinates are broadcast
// loads, and the output of a warp (8 heads x 64 bytes) is one contiguous 512-byte store. With the model's two
// points per head, every thread issues all 8 of its tap loads before its first multiply, which keeps enough loads
// in flight to cover the HBM latency of the gather. The grid is resident (deform_vec4_np2_grid_kernel: one wave of
// CTAs whose threads stride over the items and load the next item's locations and weights under the current
// gathers): 64 frames 30.7 -> 26.6 us against one short CTA per 64 items (deform_vec4_np2_kernel, kept for
// problems past 2^31 items). (A tile::gather4 TMA version, each point's four tap rows in one TMA load issued by a
// producer warp, measured 68 us: the SM's TMA unit issues 64-byte-row gathers far more slowly than the load path.) (Staging each head's 100 KB slice
// of the map in shared memory, one CTA per (frame, head), measured slower on B200: 45 us against 31 us at
// 64 frames — two such CTAs per SM alternate between copying and sampling instead of overlapping many gathers.)
// A scalar kernel covers head sizes or column offsets that are not multiples of 4.
// ko_deform_prep builds the sampler's inputs from the merged offset / logit projection: the sampling locations
// and the softmax over each head's points (model.py:222-225), one thread per (frame, query, head).
#include <algorithm>

#include "ko_common.cuh"

namespace {

struct DeformShape {
  int64_t B, NQ, NH, HD, NP, GH, GW, ROW, offset;
};

__device__ __forceinline__ void fma4(float4& acc, float w, const float4& v) {
  acc.x += w * v.x;
  acc.y += w * v.y;
  acc.z += w * v.z;
  acc.w += w * v.w;
}

// One thread per (b, q, h, 4-channel group).
__global__ void __launch_bounds__(256) deform_vec4_kernel(const float* __restrict__ value,
                                                          const float* __restrict__ loc,
                                                          const float* __restrict__ aw, DeformShape s,
                                                          float* __restrict__ out) {
  const int64_t groups = s.HD >> 2;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = s.B * s.NQ * s.NH * groups;
  if (t >= total) return;
  const int64_t g = t % groups;
  const int64_t qh = t / groups;            // (b*NQ + q)*NH + h
  const int64_t h = qh % s.NH;
  const int64_t b = qh / (s.NH * s.NQ);
  const int GW = static_cast<int>(s.GW), GH = static_cast<int>(s.GH);
  const float* vb = value + b * (s.GH * s.GW * s.ROW) + s.offset + h * s.HD + g * 4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int p = 0; p < s.NP; ++p) {
    const int64_t li = qh * s.NP + p;
    const float2 lxy = __ldg(reinterpret_cast<const float2*>(loc) + li);
    const float lx = lxy.x * static_cast<float>(GW) - 0.5f;
    const float ly = lxy.y * static_cast<float>(GH) - 0.5f;
    const float x0f = floorf(lx), y0f = floorf(ly);
    const float fx = lx - x0f, fy = ly - y0f;
    const int x0 = static_cast<int>(x0f), y0 = static_cast<int>(y0f);
    const float w = __ldg(aw + li);
    float4 sacc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int dy = 0; dy < 2; ++dy) {
      const int yy = y0 + dy;
      if (yy < 0 || yy >= GH) continue;
      const float wy = dy ? fy : 1.0f - fy;
#pragma unroll
      for (int dx = 0; dx < 2; ++dx) {
        const int xx = x0 + dx;
        if (xx < 0 || xx >= GW) continue;
        const float wx = dx ? fx : 1.0f - fx;
        const float4 v = __ldg(reinterpret_cast<const float4*>(vb + static_cast<int64_t>(yy * GW + xx) * s.ROW));
        fma4(sacc, wx * wy, v);
      }
    }
    fma4(acc, w, sacc);
  }
  reinterpret_cast<float4*>(out)[t] = acc;
}

// Two points per (query, head), the model's layout: each thread reads its (query, head)'s locations (16 bytes)
// and weights (8 bytes) with one load each and then issues all 8 of its tap loads before the first multiply, so
// a thread keeps its whole gather in flight at once instead of one point at a time.
__global__ void __launch_bounds__(256) deform_vec4_np2_kernel(const float* __restrict__ value,
                                                              const float* __restrict__ loc,
                                                              const float* __restrict__ aw, DeformShape s,
                                                              float* __restrict__ out) {
  const int64_t groups = s.HD >> 2;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = s.B * s.NQ * s.NH * groups;
  if (t >= total) return;
  const int64_t g = t % groups;
  const int64_t qh = t / groups;  // (b*NQ + q)*NH + h
  const int64_t h = qh % s.NH;
  const int64_t b = qh / (s.NH * s.NQ);
  const int GW = static_cast<int>(s.GW), GH = static_cast<int>(s.GH);
  const float* vb = value + b * (s.GH * s.GW * s.ROW) + s.offset + h * s.HD + g * 4;
  const float4 l = __ldg(reinterpret_cast<const float4*>(loc) + qh);   // (x0, y0, x1, y1)
  const float2 w = __ldg(reinterpret_cast<const float2*>(aw) + qh);
  float4 v[8];
  float wt[8];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const float lx = (p ? l.z : l.x) * static_cast<float>(GW) - 0.5f;
    const float ly = (p ? l.w : l.y) * static_cast<float>(GH) - 0.5f;
    const float x0f = floorf(lx), y0f = floorf(ly);
    const float fx = lx - x0f, fy = ly - y0f;
    const int x0 = static_cast<int>(x0f), y0 = static_cast<int>(y0f);
#pragma unroll
    for (int dy = 0; dy < 2; ++dy) {
#pragma unroll
      for (int dx = 0; dx < 2; ++dx) {
        const int k = p * 4 + dy * 2 + dx;
        const int yy = y0 + dy, xx = x0 + dx;
        const bool in = yy >= 0 && yy < GH && xx >= 0 && xx < GW;
        wt[k] = in ? (dx ? fx : 1.0f - fx) * (dy ? fy : 1.0f - fy) : 0.0f;
        v[k] = in ? __ldg(reinterpret_cast<const float4*>(vb + static_cast<int64_t>(yy * GW + xx) * s.ROW))
                  : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  }
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    float4 sacc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < 4; ++k) fma4(sacc, wt[p * 4 + k], v[p * 4 + k]);
    fma4(acc, p ? w.y : w.x, sacc);
  }
  reinterpret_cast<float4*>(out)[t] = acc;
}

// The same sampling with a resident grid: every thread walks (query, head, channel group) items with a stride of
// the whole grid and loads the next item's locations and weights while its current gathers are in flight, so the
// SMs stay full for the whole launch instead of cycling ~32 short CTAs each.
__global__ void __launch_bounds__(256) deform_vec4_np2_grid_kernel(const float* __restrict__ value,
                                                                   const float* __restrict__ loc,
                                                                   const float* __restrict__ aw, DeformShape s,
                                                                   float* __restrict__ out) {
  const int groups = static_cast<int>(s.HD >> 2);
  const int NH = static_cast<int>(s.NH), NQ = static_cast<int>(s.NQ);
  const int total = static_cast<int>(s.B * s.NQ * s.NH) * groups;
  const int stride = gridDim.x * blockDim.x;
  const int GW = static_cast<int>(s.GW), GH = static_cast<int>(s.GH);
  int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= total) return;
  float4 l = __ldg(reinterpret_cast<const float4*>(loc) + t / groups);
  float2 w = __ldg(reinterpret_cast<const float2*>(aw) + t / groups);
  for (; t < total; t += stride) {
    const int g = t % groups, qh = t / groups;
    const int h = qh % NH, b = qh / (NH * NQ);
    const float* vb = value + static_cast<int64_t>(b) * (s.GH * s.GW * s.ROW) + s.offset + h * s.HD + g * 4;
    float4 v[8];
    float wt[8];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const float lx = (p ? l.z : l.x) * static_cast<float>(GW) - 0.5f;
      const float ly = (p ? l.w : l.y) * static_cast<float>(GH) - 0.5f;
      const float x0f = floorf(lx), y0f = floorf(ly);
      const float fx = lx - x0f, fy = ly - y0f;
      const int x0 = static_cast<int>(x0f), y0 = static_cast<int>(y0f);
#pragma unroll
      for (int dy = 0; dy < 2; ++dy) {
#pragma unroll
        for (int dx = 0; dx < 2; ++dx) {
          const int k = p * 4 + dy * 2 + dx;
          const int yy = y0 + dy, xx = x0 + dx;
          const bool in = yy >= 0 && yy < GH && xx >= 0 && xx < GW;
          wt[k] = in ? (dx ? fx : 1.0f - fx) * (dy ? fy : 1.0f - fy) : 0.0f;
          v[k] = in ? __ldg(reinterpret_cast<const float4*>(vb + static_cast<int64_t>(yy * GW + xx) * s.ROW))
                    : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
    const float2 wc = w;
    if (t + stride < total) {  // the next item's inputs, while the gathers above are in flight
      l = __ldg(reinterpret_cast<const float4*>(loc) + (t + stride) / groups);
      w = __ldg(reinterpret_cast<const float2*>(aw) + (t + stride) / groups);
    }
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      float4 sacc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int k = 0; k < 4; ++k) fma4(sacc, wt[p * 4 + k], v[p * 4 + k]);
      fma4(acc, p ? wc.y : wc.x, sacc);
    }
    reinterpret_cast<float4*>(out)[t] = acc;
  }
}

// General layout: one thread per (b, q, h, d).
__global__ void __launch_bounds__(256) deform_scalar_kernel(const float* __restrict__ value,
                                                            const float* __restrict__ loc,
                                                            const float* __restrict__ aw, DeformShape s,
                                                            float* __restrict__ out) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = s.B * s.NQ * s.NH * s.HD;
  if (t >= total) return;
  const int64_t d = t % s.HD;
  const int64_t qh = t / s.HD;
  const int64_t h = qh % s.NH;
  const int64_t b = qh / (s.NH * s.NQ);
  const int GW = static_cast<int>(s.GW), GH = static_cast<int>(s.GH);
  const float* vb = value + b * (s.GH * s.GW * s.ROW) + s.offset + h * s.HD + d;
  float acc = 0.f;
  for (int p = 0; p < s.NP; ++p) {
    const int64_t li = qh * s.NP + p;
    const float lx = __ldg(loc + li * 2) * static_cast<float>(GW) - 0.5f;
    const float ly = __ldg(loc + li * 2 + 1) * static_cast<float>(GH) - 0.5f;
    const float x0f = floorf(lx), y0f = floorf(ly);
    const float fx = lx - x0f, fy = ly - y0f;
    const int x0 = static_cast<int>(x0f), y0 = static_cast<int>(y0f);
    float sacc = 0.f;
    for (int dy = 0; dy < 2; ++dy) {
      const int yy = y0 + dy;
      if (yy < 0 || yy >= GH) continue;
      const float wy = dy ? fy : 1.0f - fy;
      for (int dx = 0; dx < 2; ++dx) {
        const int xx = x0 + dx;
        if (xx < 0 || xx >= GW) continue;
        const float wx = dx ? fx : 1.0f - fx;
        sacc += wx * wy * __ldg(vb + static_cast<int64_t>(yy * GW + xx) * s.ROW);
      }
    }
    acc += __ldg(aw + li) * sacc;
  }
  out[t] = acc;
}

}  // namespace

extern "C" int ko_deform_attn(const float* value, const float* loc, const float* aw, int64_t B, int64_t NQ,
                              int64_t NH, int64_t HD, int64_t NP, int64_t GH, int64_t GW, int64_t ROW,
                              int64_t offset, float* out, ko_stream_t stream) {
  if (B < 0 || NQ < 0 || NH < 1 || HD < 1 || NP < 1 || GH < 1 || GW < 1 || offset < 0 || offset + NH * HD > ROW)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_deform_attn: bad shape (need offset + NH*HD <= ROW)");
  if (GH * GW > (int64_t(1) << 30) / 1) return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_deform_attn: map too large");
  if (B == 0 || NQ == 0) return KO_OK;
  if (!value || !loc || !aw || !out) return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_deform_attn: null pointer");
  if ((reinterpret_cast<uintptr_t>(loc) & 7) != 0)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_deform_attn: loc must be 8-byte aligned");
  DeformShape s{B, NQ, NH, HD, NP, GH, GW, ROW, offset};
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool vec = HD % 4 == 0 && offset % 4 == 0 && ROW % 4 == 0 && ko::aligned16(value) && ko::aligned16(out);
  const int64_t total = B * NQ * NH * (vec ? HD / 4 : HD);
  const int64_t blocks = (total + 255) / 256;
  if (blocks > 0x7fffffff) return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_deform_attn: problem too large");
  const bool np2 = vec && NP == 2 && (reinterpret_cast<uintptr_t>(loc) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(aw) & 7) == 0;
  if (np2 && total < (int64_t(1) << 31)) {
    const ko::DeviceInfo* dinfo = nullptr;
    if (int rc = ko::device_or_fail(&dinfo, "ko_deform_attn")) return rc;
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, deform_vec4_np2_grid_kernel, 256, 0);
    if (e != cudaSuccess || per_sm < 1) per_sm = 1;
    const int64_t grid = std::min<int64_t>(blocks, static_cast<int64_t>(per_sm) * dinfo->sm_count);
    deform_vec4_np2_grid_kernel<<<static_cast<unsigned>(grid), 256, 0, st>>>(value, loc, aw, s, out);
  } else if (np2)
    deform_vec4_np2_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(value, loc, aw, s, out);
  else if (vec)
    deform_vec4_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(value, loc, aw, s, out);
  else
    deform_scalar_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(value, loc, aw, s, out);
  return ko::check_launch("ko_deform_attn");
}

// ---------------------------------------------------------------------------------------------------------
// Sampling locations and point weights from the cross-attention's projection (ko_deform_prep).
// Semantics: fast_rfdetr/model.py:222-225 —
//   off = oa[..., :NH*NP*2] as [NH][NP][2],   aw = softmax over points of oa[..., NH*NP*2:] as [NH][NP],
//   loc = ref_xy + off / NP * ref_wh * 0.5   (the same fp32 operations in the same order as the reference,
//   so loc is bit-identical to it; the softmax is max-subtracted with expf).
// One thread per (frame, query, head); replaces the softmax and the four elementwise launches per layer.
// ---------------------------------------------------------------------------------------------------------
namespace {

constexpr int kPrepMaxPoints = 8;

__global__ void __launch_bounds__(256) deform_prep_kernel(const float* __restrict__ oa,
                                                          const float* __restrict__ ref, int64_t rows, int NH,
                                                          int NP, int64_t ld_oa, float* __restrict__ loc,
                                                          float* __restrict__ aw) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= rows * NH) return;
  const int64_t r = t / NH;  // (frame, query) row
  const int h = static_cast<int>(t - r * NH);
  const float* o = oa + r * ld_oa;
  const float4 rb = reinterpret_cast<const float4*>(ref)[r];
  const float np = static_cast<float>(NP);
  float* lp = loc + t * NP * 2;
  for (int p = 0; p < NP; ++p) {
    const float ox = o[(h * NP + p) * 2], oy = o[(h * NP + p) * 2 + 1];
    lp[2 * p] = rb.x + ox / np * rb.z * 0.5f;
    lp[2 * p + 1] = rb.y + oy / np * rb.w * 0.5f;
  }
  const float* lg = o + NH * NP * 2 + h * NP;
  float e[kPrepMaxPoints];
  float mx = lg[0];
  for (int p = 1; p < NP; ++p) mx = fmaxf(mx, lg[p]);
  float sum = 0.f;
  for (int p = 0; p < NP; ++p) {
    e[p] = expf(lg[p] - mx);
    sum += e[p];
  }
  for (int p = 0; p < NP; ++p) aw[t * NP + p] = e[p] / sum;
}

}  // namespace

extern "C" int ko_deform_prep(const float* oa, const float* ref, int64_t B, int64_t NQ, int64_t NH, int64_t NP,
                              int64_t ld_oa, float* loc, float* aw, ko_stream_t stream) {
  const char* who = "ko_deform_prep";
  if (B < 0 || NQ < 0 || NH < 1 || NH > 4096 || NP < 1 || NP > kPrepMaxPoints || ld_oa < NH * NP * 3)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": need 1 <= NH <= 4096 heads, 1 <= NP <= 8 points "
                                                                "and a row of at least NH * NP * 3 values");
  const int64_t rows = B * NQ;
  if (rows == 0) return KO_OK;
  if (!oa || !ref || !loc || !aw) return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": null pointer");
  if (!ko::aligned16(ref)) return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": ref must be 16-byte aligned");
  const int64_t blocks = (rows * NH + 255) / 256;
  if (blocks > 0x7fffffff) return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": too many rows");
  deform_prep_kernel<<<static_cast<unsigned>(blocks), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      oa, ref, rows, static_cast<int>(NH), static_cast<int>(NP), ld_oa, loc, aw);
  return ko::check_launch(who);
}
