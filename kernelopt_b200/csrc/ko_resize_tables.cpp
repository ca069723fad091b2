// Host-side generator of the cv2.resize(INTER_LINEAR, uint8, 3 channels) interpolation tables consumed by the
// preprocessing kernel. Two arithmetic models are produced, in the same 4-tap form:
//
//   mode 0 (KleidiCV):  left  = (A*256 + (C-A)*fy + 128) >> 8,  right = (B*256 + (D-B)*fy + 128) >> 8,
//                       v     = (left*256 + (right-left)*fx + 128) >> 8
//   mode 1 (OpenCV):    h0 = A*a0 + B*a1,  h1 = C*a0 + D*a1,
//                       v  = (((h0>>4)*b0 >> 16) + ((h1>>4)*b1 >> 16) + 2) >> 2
//
// A, B are the top-row taps and C, D the bottom-row taps of an output element. The element-level x table exists
// because KleidiCV steps its 16.16 source coordinate once per 16-lane vector of interleaved BGR bytes, so the
// tap of an element depends on the lane it lands in, not only on its pixel.
//
// This is the algorithm of the reference's table model (fast_rfdetr/resize_tables.py:28-184), restated:
//   - the 16.16 helpers        resize_tables.py:33-38
//   - the KleidiCV selection   resize_tables.py:41-43
//   - KleidiCV x / y tables    resize_tables.py:46-145
//   - OpenCV x / y tables      resize_tables.py:148-162
// The steps have to stay alike because they model one library's exact integer behaviour; the code is written
// independently. Compiled with -ffp-contract=off so the float32 arithmetic of the OpenCV model rounds like numpy.
#include <cmath>
#include <cstdint>
#include <string>
#include <vector>

#include "../../include/kernelopt.h"

namespace ko {
int fail(int code, const std::string& msg);
}

namespace {

constexpr int kFrac = 16;                     // 16.16 fixed point
constexpr int64_t kHalf = int64_t(1) << (kFrac - 1);
constexpr int kLanes = 16;                    // bytes per NEON vector
constexpr int kHalfLanes = 8;
constexpr int kCh = 3;

// Python-style floor division for the non-negative/negative mix the 16.16 helpers can produce.
inline int64_t floordiv(int64_t a, int64_t b) {
  int64_t q = a / b;
  if ((a % b != 0) && ((a < 0) != (b < 0))) --q;
  return q;
}
inline int64_t round_div(int64_t num, int64_t den) { return floordiv(num + den / 2, den); }

// Source coordinate (16.16) of the centre of destination pixel d, KleidiCV's half-pixel alignment.
inline int64_t centre_coord(int64_t d, int64_t src, int64_t dst) {
  return round_div(((d << kFrac) + kHalf) * src, dst) - kHalf + (int64_t(1) << (kFrac - 9));
}

bool kleidicv_applies(int64_t sw, int64_t sh, int64_t dw, int64_t dh) {
  return dw * 3 >= sw && dw < sw && dh < sh && dw * kCh >= 8 && sw * kCh >= 32;
}

struct KleidiX {
  int64_t sw, dw, ratio, n_el, one;
  std::vector<int64_t>& el;
  std::vector<int64_t>& fx;

  int64_t step_of(int64_t k) const { return round_div((k * sw) << kFrac, dw); }  // offset of k pixels (16.16)

  // One 16-lane vector whose first element is channel `ip` of the pixel at coordinate sx.
  void vector_lanes(int64_t e0, int64_t sx, int ip) {
    const int64_t base = sx >> kFrac, f0 = sx & 0xFFFF;
    for (int lane = 0; lane < kLanes; ++lane) {
      const int k = (ip + lane) / kCh;     // pixel offset of this lane inside the vector
      const int ch = (ip + lane) % kCh;    // channel of this lane
      const int64_t pos = f0 + step_of(k);
      const int64_t lane_px = (pos >> kFrac) & 0xFF;
      // u8 multiply by 3 (wraps), saturating subtract of the start channel, then the lane's channel delta
      int64_t idx = ((lane_px * 3) & 0xFF) - ip;
      if (idx < 0) idx = 0;
      idx += (k == 0) ? (ch - ip) : ch;
      el[e0 + lane] = base * kCh + ip + idx;
      fx[e0 + lane] = (pos >> 8) & 0xFF;
    }
  }

  // Scalar tail: the first pixel from sx, every further pixel one source step further.
  void scalar_lanes(int64_t e0, int n, int ip, int64_t sx) {
    int j = 0;
    {
      const int64_t s = (sx >> kFrac) * kCh + ip, f = (sx & 0xFFFF) >> 8;
      for (; j < kCh - ip && j < n; ++j) {
        el[e0 + j] = s + j;
        fx[e0 + j] = f;
      }
    }
    while (j < n) {
      sx += one;
      const int64_t s = (sx >> kFrac) * kCh, f = (sx & 0xFFFF) >> 8;
      for (int c = 0; c < kCh && j < n; ++c, ++j) {
        el[e0 + j] = s + c;
        fx[e0 + j] = f;
      }
    }
  }

  // True when a vector starting at element e would read past the end of the source row.
  bool overruns(int64_t e) const {
    const int64_t src_el = (centre_coord(e / kCh, sw, dw) >> kFrac) * kCh + e % kCh;
    return src_el + kLanes * ratio > sw * kCh;
  }

  void run() {
    const int64_t pairs = (sw * kCh >= kLanes * ratio) ? n_el / (2 * kLanes) : 0;
    const int64_t n_vec = pairs * 2;
    const int64_t rest = n_el - pairs * 2 * kLanes;
    const int64_t n_tail = (rest + kHalfLanes - 1) / kHalfLanes;
    int64_t e = 0, done = 0;
    if (n_vec > 0) {
      if (n_vec > 3) {
        // the vector loop runs over whole groups of three vectors that stay inside the row
        int64_t last = n_vec - 1;
        while (overruns(last * kLanes)) {
          if (--last <= 0) break;
        }
        const int64_t n_inside = (last == 0 && overruns(0)) ? 0 : last + 1;
        int64_t sx = centre_coord(0, sw, dw);
        const int64_t five = round_div((sw * 5) << kFrac, dw), six = round_div((sw * 6) << kFrac, dw);
        int resync = 0;
        for (int64_t g = 0; g < n_inside / 3; ++g) {
          if (resync == 170) {  // the coordinate is recomputed from scratch every 171 groups
            sx = centre_coord(e / kCh, sw, dw);
            resync = 0;
          } else {
            ++resync;
          }
          vector_lanes(e, sx, 0);
          sx += five;
          vector_lanes(e + kLanes, sx, 1);
          sx += five;
          vector_lanes(e + 2 * kLanes, sx, 2);
          sx += six;
          done += 3;
          e += 3 * kLanes;
        }
      }
      for (; done < n_vec; ++done, e += kLanes) scalar_lanes(e, kLanes, static_cast<int>(e % kCh),
                                                             centre_coord(e / kCh, sw, dw));
    }
    for (int64_t t = 0; t < n_tail; ++t) {
      if (e > n_el - kHalfLanes) e = n_el - kHalfLanes;
      scalar_lanes(e, kHalfLanes, static_cast<int>(e % kCh), centre_coord(e / kCh, sw, dw));
      e += kHalfLanes;
    }
  }
};

// OpenCV fixed-point axis: float32 source coordinate, 11-bit weights. clamp_coord: the x axis clamps
// out-of-range coordinates (weight moves fully to the edge pixel); the y axis only clips the row indices.
void opencv_axis(int64_t src, int64_t dst, bool clamp_coord, std::vector<int64_t>& i0, std::vector<int64_t>& i1,
                 std::vector<int64_t>& w0, std::vector<int64_t>& w1) {
  const double scale = static_cast<double>(src) / static_cast<double>(dst);
  for (int64_t d = 0; d < dst; ++d) {
    const float f = static_cast<float>((static_cast<double>(d) + 0.5) * scale - 0.5);
    int64_t s = static_cast<int64_t>(std::floor(f));
    float frac = f - static_cast<float>(s);
    if (clamp_coord) {
      if (s < 0) {
        frac = 0.f;
        s = 0;
      }
      if (s >= src - 1) {
        frac = 0.f;
        s = src - 1;
      }
    }
    const float one = 1.0f, unit = 2048.0f;
    const float p1 = frac * unit;
    const float p0 = (one - frac) * unit;
    w1[d] = static_cast<int64_t>(std::nearbyint(p1));
    w0[d] = static_cast<int64_t>(std::nearbyint(p0));
    i0[d] = s < 0 ? 0 : (s > src - 1 ? src - 1 : s);
    const int64_t s1 = s + 1;
    i1[d] = s1 < 0 ? 0 : (s1 > src - 1 ? src - 1 : s1);
  }
}

}  // namespace

extern "C" int ko_resize_tables(int64_t src_w, int64_t src_h, int64_t dst_w, int64_t dst_h, int policy,
                                int32_t* xtab, int32_t* ytab, int* mode) {
  if (src_w < 1 || src_h < 1 || dst_w < 1 || dst_h < 1 || src_w > (1 << 20) || src_h > (1 << 20) ||
      dst_w > (1 << 16) || dst_h > (1 << 16))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_resize_tables: sizes out of range");
  if (policy != KO_RESIZE_REFERENCE && policy != KO_RESIZE_OPENCV)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_resize_tables: unknown policy");
  if (!xtab || !ytab || !mode) return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_resize_tables: null output");
  const int64_t n_el = dst_w * kCh;
  if (policy == KO_RESIZE_REFERENCE && kleidicv_applies(src_w, src_h, dst_w, dst_h)) {
    std::vector<int64_t> el(n_el, 0), fx(n_el, 0);
    KleidiX kx{src_w, dst_w, (static_cast<double>(src_w) / static_cast<double>(dst_w) < 1.8) ? 2 : 3, n_el,
               round_div(src_w << kFrac, dst_w), el, fx};
    kx.run();
    for (int64_t e = 0; e < n_el; ++e) {
      xtab[e * 4 + 0] = static_cast<int32_t>(el[e]);
      xtab[e * 4 + 1] = static_cast<int32_t>(el[e] + kCh);
      xtab[e * 4 + 2] = static_cast<int32_t>(fx[e]);
      xtab[e * 4 + 3] = 0;
    }
    for (int64_t d = 0; d < dst_h; ++d) {
      const int64_t sy = centre_coord(d, src_h, dst_h);
      const int64_t row = sy >> kFrac;
      const int64_t fy = (sy - (row << kFrac)) >> (kFrac - 8);
      ytab[d * 4 + 0] = static_cast<int32_t>(row);
      ytab[d * 4 + 1] = static_cast<int32_t>(row + 1 < src_h - 1 ? row + 1 : src_h - 1);
      ytab[d * 4 + 2] = static_cast<int32_t>(fy);
      ytab[d * 4 + 3] = 0;
    }
    *mode = 0;
    return KO_OK;
  }
  std::vector<int64_t> x0(dst_w), x1(dst_w), a0(dst_w), a1(dst_w);
  opencv_axis(src_w, dst_w, true, x0, x1, a0, a1);
  for (int64_t x = 0; x < dst_w; ++x)
    for (int c = 0; c < kCh; ++c) {
      const int64_t e = x * kCh + c;
      xtab[e * 4 + 0] = static_cast<int32_t>(x0[x] * kCh + c);
      xtab[e * 4 + 1] = static_cast<int32_t>(x1[x] * kCh + c);
      xtab[e * 4 + 2] = static_cast<int32_t>(a0[x]);
      xtab[e * 4 + 3] = static_cast<int32_t>(a1[x]);
    }
  std::vector<int64_t> y0(dst_h), y1(dst_h), b0(dst_h), b1(dst_h);
  opencv_axis(src_h, dst_h, false, y0, y1, b0, b1);
  for (int64_t d = 0; d < dst_h; ++d) {
    ytab[d * 4 + 0] = static_cast<int32_t>(y0[d]);
    ytab[d * 4 + 1] = static_cast<int32_t>(y1[d]);
    ytab[d * 4 + 2] = static_cast<int32_t>(b0[d]);
    ytab[d * 4 + 3] = static_cast<int32_t>(b1[d]);
  }
  *mode = 1;
  return KO_OK;
}
