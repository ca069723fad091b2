// uint8 BGR frame -> resized (cv2 INTER_LINEAR, bit-exact through the 4-tap tables), RGB, normalised float32.
//
// Semantics follow the reference kernel fast_rfdetr/kernels.py:74-103 (bgr_resize_normalize): for output row y
// and BGR element e = x*3 + c the taps are A = top[xt.x], B = top[xt.y], C = bot[xt.x], D = bot[xt.y] with
// xt = xtab[e], (top, bot) = rows ytab[y].x / ytab[y].y; the tap arithmetic is mode 0 (KleidiCV) or mode 1
// (OpenCV); v is clamped to 0..255 and the RGB output channel 2-c receives lut[(2-c)*256 + v].
//
// B200 design: every thread produces 4 consecutive outputs and writes them with one 128-bit store, from source
// rows staged in shared memory with 16-byte copies, so both the row reads and the output writes are fully
// coalesced. Three kernels share that scheme:
//   - the segment kernel (640-wide HWC / PATCH16 outputs from 16-byte aligned rows: the model's case): persistent
//     warps, each working alone on (image, band of 4-16 rows, 128-element segment) tasks with its own cp.async ring of
//     source-row windows; no CTA-wide barrier. Where the right-hand x tap has weight zero everywhere in a segment
//     (1920 -> 640, an exact 3:1 ratio, in both table modes) it loads and weighs the left taps only.
//   - the band kernel (other outputs up to 682 wide, CHW, unaligned rows): one CTA per band of output rows with
//     the x taps in registers, the LUT in shared memory and the next row pair prefetched with cp.async into a
//     ring of three buffers while the current one is computed;
//   - one CTA per output row for wider outputs.
// All images of a batch (any sizes) go in one launch. Three output layouts share the kernels: HWC (the
// reference's), CHW (NCHW batches) and PATCH16 (the im2col of the ViT 16x16 patch embedding, which turns that
// convolution into a plain GEMM).
#include <cstring>
#include <type_traits>

#include "ko_common.cuh"

namespace {

constexpr int kMaxImages = 64;
constexpr int kThreads = 128;

struct ImageParams {
  const uint8_t* src;
  const int4* xtab;
  const int4* ytab;
  int64_t src_h, src_w, src_stride;
  int32_t mode;
  int32_t vec_ok;  // rows start 16-byte aligned and src_w*3 is a multiple of 16
};

struct BatchParams {
  ImageParams img[kMaxImages];
};

__device__ __forceinline__ int tap_value(int mode, const uint8_t* top, const uint8_t* bot, int4 xt, int4 yt,
                                         int last) {
  const int l = min(max(xt.x, 0), last), r = min(max(xt.y, 0), last);
  const int A = top[l], B = top[r], C = bot[l], D = bot[r];
  int v;
  if (mode == 0) {
    const int left = (A * 256 + (C - A) * yt.z + 128) >> 8;
    const int right = (B * 256 + (D - B) * yt.z + 128) >> 8;
    v = (left * 256 + (right - left) * xt.z + 128) >> 8;
  } else {
    const int h0 = A * xt.z + B * xt.w;
    const int h1 = C * xt.z + D * xt.w;
    v = ((((h0 >> 4) * yt.z) >> 16) + (((h1 >> 4) * yt.w) >> 16) + 2) >> 2;
  }
  return min(max(v, 0), 255);
}

__global__ void __launch_bounds__(kThreads) preprocess_kernel(const __grid_constant__ BatchParams p,
                                                              const float* __restrict__ lut, int dst, int layout,
                                                              float* __restrict__ out, int row_cap) {
  extern __shared__ __align__(16) uint8_t rows[];  // [2][row_cap]
  const ImageParams& im = p.img[blockIdx.y];
  const int y = blockIdx.x;
  const int4 yt = __ldg(im.ytab + y);
  const int rmax = static_cast<int>(im.src_h) - 1;
  const int r0 = min(max(yt.x, 0), rmax), r1 = min(max(yt.y, 0), rmax);
  const int row_bytes = static_cast<int>(im.src_w) * 3;
  const uint8_t* g0 = im.src + static_cast<int64_t>(r0) * im.src_stride;
  const uint8_t* g1 = im.src + static_cast<int64_t>(r1) * im.src_stride;
  uint8_t* s0 = rows;
  uint8_t* s1 = rows + row_cap;

  if (im.vec_ok) {
    const int n16 = row_bytes >> 4;
    const uint4* a = reinterpret_cast<const uint4*>(g0);
    const uint4* b = reinterpret_cast<const uint4*>(g1);
    for (int i = threadIdx.x; i < n16; i += kThreads) {
      const uint4 va = __ldg(a + i), vb = __ldg(b + i);
      reinterpret_cast<uint4*>(s0)[i] = va;
      reinterpret_cast<uint4*>(s1)[i] = vb;
    }
  } else {
    for (int i = threadIdx.x; i < row_bytes; i += kThreads) {
      s0[i] = __ldg(g0 + i);
      s1[i] = __ldg(g1 + i);
    }
  }
  __syncthreads();

  const int n_items = dst * 3 / 4;  // float4 outputs per row
  const int per_ch = dst / 4;
  const int last = row_bytes - 1;
  const int64_t img_base = static_cast<int64_t>(blockIdx.y) * dst * dst * 3;
  for (int i = threadIdx.x; i < n_items; i += kThreads) {
    float v[4];
    int64_t addr;
    if (layout == KO_LAYOUT_CHW) {
      const int c_rgb = i / per_ch, x0 = (i - c_rgb * per_ch) * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int e = (x0 + j) * 3 + (2 - c_rgb);
        const int t = tap_value(im.mode, s0, s1, __ldg(im.xtab + e), yt, last);
        v[j] = __ldg(lut + c_rgb * 256 + t);
      }
      addr = img_base + static_cast<int64_t>(c_rgb) * dst * dst + static_cast<int64_t>(y) * dst + x0;
    } else {
      const int o0 = i * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int o = o0 + j, x = o / 3, c_rgb = o - x * 3;
        const int e = x * 3 + (2 - c_rgb);
        const int t = tap_value(im.mode, s0, s1, __ldg(im.xtab + e), yt, last);
        v[j] = __ldg(lut + c_rgb * 256 + t);
      }
      if (layout == KO_LAYOUT_HWC) {
        addr = img_base + static_cast<int64_t>(y) * dst * 3 + o0;
      } else {  // PATCH16: token (y/16, px) holds 16 rows of 48 floats
        const int px = o0 / 48, within = o0 - px * 48;
        const int token = (y >> 4) * (dst >> 4) + px;
        addr = img_base + static_cast<int64_t>(token) * 768 + (y & 15) * 48 + within;
      }
    }
    *reinterpret_cast<float4*>(out + addr) = make_float4(v[0], v[1], v[2], v[3]);
  }
}

// ---------------------------------------------------------------------------------------------------------
// Band kernel (dst * 3 / 4 <= 2 * kBandThreads float4 outputs per row, i.e. dst <= 682; the 640 of the model).
//
// One CTA per (band of `band` consecutive output rows, image); each thread owns one or two float4 slots of the
// output row.
// Everything that does not depend on the row is set up once per CTA and kept on chip: each thread's x taps (the
// clamped xtab entries of its 4 output elements), their RGB channels and output column offset live in registers, the
// 768-entry LUT in shared memory. The two source rows of output row y+1 are fetched with cp.async (16-byte,
// L2-only) into the next buffer of a ring of three while row y is computed, so the HBM reads of the next row
// overlap the arithmetic of this one. Per output element the loop does 4 byte loads from shared memory, the
// integer tap arithmetic, one LUT load from shared memory and a quarter of a 128-bit store.
// ---------------------------------------------------------------------------------------------------------
// Threads per band CTA; measurement builds may override it (-DKO_PRE_BAND_THREADS=n, a multiple of 32, <= 1024).
#ifndef KO_PRE_BAND_THREADS
#define KO_PRE_BAND_THREADS 256
#endif
constexpr int kBandThreads = KO_PRE_BAND_THREADS;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(kodev::smem_addr(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// Offset of output element 0 of row y for a layout, relative to the image base (the column part is separate).
__device__ __forceinline__ int64_t row_term(int layout, int y, int dst) {
  if (layout == KO_LAYOUT_HWC) return static_cast<int64_t>(y) * dst * 3;
  if (layout == KO_LAYOUT_CHW) return static_cast<int64_t>(y) * dst;
  return static_cast<int64_t>(y >> 4) * (dst >> 4) * 768 + (y & 15) * 48;  // PATCH16
}

// The 4 outputs of one item from the staged rows s0 (top) and s1 (bottom).
template <int MODE>
__device__ __forceinline__ float4 item_values(const uint8_t* s0, const uint8_t* s1, const int4 (&tap)[4],
                                              uint32_t chans, int4 yt, const float* slut) {
  float v[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int4 t = tap[j];
    const int A = s0[t.x], B = s0[t.y], C = s1[t.x], D = s1[t.y];
    int q;
    if (MODE == 0) {
      const int left = (A * 256 + (C - A) * yt.z + 128) >> 8;
      const int right = (B * 256 + (D - B) * yt.z + 128) >> 8;
      q = (left * 256 + (right - left) * t.z + 128) >> 8;
    } else {
      const int h0 = A * t.z + B * t.w;
      const int h1 = C * t.z + D * t.w;
      q = ((((h0 >> 4) * yt.z) >> 16) + (((h1 >> 4) * yt.w) >> 16) + 2) >> 2;
    }
    q = min(max(q, 0), 255);
    v[j] = slut[(((chans >> (2 * j)) & 3u) << 8) + q];  // RGB channel of element j: 2 bits each
  }
  return make_float4(v[0], v[1], v[2], v[3]);
}

template <int IPT>
__global__ void __launch_bounds__(kBandThreads, kBandThreads <= 256 ? 3 : 2) preprocess_band_kernel(const __grid_constant__ BatchParams p,
                                                                       const float* __restrict__ lut, int dst,
                                                                       int layout, float* __restrict__ out,
                                                                       int row_cap, int band) {
  extern __shared__ __align__(16) uint8_t smem[];
  float* slut = reinterpret_cast<float*>(smem);  // [3][256]
  uint8_t* rowbuf = smem + 768 * 4;              // [3 buffers][2 rows][row_cap]
  const ImageParams& im = p.img[blockIdx.y];
  const int tid = threadIdx.x;
  const int y_begin = blockIdx.x * band;
  const int y_end = min(y_begin + band, dst);
  if (y_begin >= dst) return;
  const int row_bytes = static_cast<int>(im.src_w) * 3;
  const int last = row_bytes - 1;
  const int rmax = static_cast<int>(im.src_h) - 1;
  const int n_items = dst * 3 / 4;
  const int per_ch = dst / 4;
  const int64_t img_base = static_cast<int64_t>(blockIdx.y) * dst * dst * 3;
  const int mode = im.mode;
  const bool vec = im.vec_ok != 0;
  const int n16 = row_bytes >> 4;

  // Stage the two source rows of output row y into buffer `buf` (vector path: cp.async, 16 bytes per copy);
  // returns the row's ytab entry, which the compute step of that row needs again.
  auto stage = [&](int y, int buf) -> int4 {
    const int4 yt = __ldg(im.ytab + y);
    const int r0 = min(max(yt.x, 0), rmax), r1 = min(max(yt.y, 0), rmax);
    const uint8_t* g0 = im.src + static_cast<int64_t>(r0) * im.src_stride;
    const uint8_t* g1 = im.src + static_cast<int64_t>(r1) * im.src_stride;
    uint8_t* s0 = rowbuf + (2 * buf) * row_cap;
    uint8_t* s1 = s0 + row_cap;
    if (vec) {
      for (int i = tid; i < n16; i += kBandThreads) {
        cp_async16(s0 + 16 * i, g0 + 16 * i);
        cp_async16(s1 + 16 * i, g1 + 16 * i);
      }
    } else {
      for (int i = tid; i < row_bytes; i += kBandThreads) {
        s0[i] = __ldg(g0 + i);
        s1[i] = __ldg(g1 + i);
      }
    }
    cp_async_commit();
    return yt;
  };

  int4 yt_next = stage(y_begin, 0);
  for (int i = tid; i < 768; i += kBandThreads) slut[i] = __ldg(lut + i);

  // Per-thread column set-up: clamped taps (l, r), weights, RGB channel and output column offset of each element.
  int4 tap[IPT][4];
  uint32_t chans[IPT];
  float* obase[IPT];
  bool live[IPT];
#pragma unroll
  for (int k = 0; k < IPT; ++k) {
    const int i = tid + k * kBandThreads;
    live[k] = i < n_items;
    chans[k] = 0;
    int64_t col_off = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) tap[k][j] = make_int4(0, 0, 0, 0);
    if (live[k]) {
      if (layout == KO_LAYOUT_CHW) {
        const int c_rgb = i / per_ch, x0 = (i - c_rgb * per_ch) * 4;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          tap[k][j] = __ldg(im.xtab + (x0 + j) * 3 + (2 - c_rgb));
          chans[k] |= static_cast<uint32_t>(c_rgb) << (2 * j);
        }
        col_off = static_cast<int64_t>(c_rgb) * dst * dst + x0;
      } else {
        const int o0 = i * 4;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int o = o0 + j, x = o / 3, c_rgb = o - x * 3;
          tap[k][j] = __ldg(im.xtab + x * 3 + (2 - c_rgb));
          chans[k] |= static_cast<uint32_t>(c_rgb) << (2 * j);
        }
        if (layout == KO_LAYOUT_HWC) {
          col_off = o0;
        } else {
          const int px = o0 / 48;
          col_off = static_cast<int64_t>(px) * 768 + (o0 - px * 48);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        tap[k][j].x = min(max(tap[k][j].x, 0), last);
        tap[k][j].y = min(max(tap[k][j].y, 0), last);
      }
    }
    obase[k] = out + img_base + col_off;
  }

  // Three row-pair buffers: the pair of row y+1 is staged into the buffer row y-2 used, which every thread has
  // finished reading before it passed the barrier of row y-1; so one barrier per row suffices. The loop is
  // unrolled over the ring (the buffer of each step is a constant) and specialised for the table mode, which is
  // the same for the whole CTA (one image).
  auto rows = [&](auto mode_c) {
    constexpr int MODE = decltype(mode_c)::value;
    int y = y_begin;
    auto step = [&](auto buf_c) -> bool {
      constexpr int BUF = decltype(buf_c)::value;
      if (y >= y_end) return false;
      const int4 yt = yt_next;
      if (y + 1 < y_end) {
        yt_next = stage(y + 1, (BUF + 1) % 3);
      } else {
        cp_async_commit();  // empty group keeps the wait count uniform
      }
      cp_async_wait_1();
      __syncthreads();
      const uint8_t* s0 = rowbuf + (2 * BUF) * row_cap;
      const uint8_t* s1 = s0 + row_cap;
      const int64_t rt = row_term(layout, y, dst);
#pragma unroll
      for (int k = 0; k < IPT; ++k) {
        if (!live[k]) continue;
        *reinterpret_cast<float4*>(obase[k] + rt) = item_values<MODE>(s0, s1, tap[k], chans[k], yt, slut);
      }
      ++y;
      return true;
    };
    while (step(std::integral_constant<int, 0>{}) && step(std::integral_constant<int, 1>{}) &&
           step(std::integral_constant<int, 2>{})) {
    }
  };
  if (mode == 0)
    rows(std::integral_constant<int, 0>{});
  else
    rows(std::integral_constant<int, 1>{});
}

// ---------------------------------------------------------------------------------------------------------
// Segment kernel (640-wide outputs from 16-byte aligned sources: the model's case). Every warp works alone:
// no CTA-wide barrier after the LUT is loaded.
//
// A task is (image, band of 4-16 output rows, segment of 32 float4 items = 128 output elements). Warps are
// persistent and take tasks round-robin, so the 15 segments of a band run at the same time on neighbouring
// warps and each source row comes from HBM once. For a task the warp loads its lanes' taps, reduces them to the
// byte window of a source row that the segment reads (about 400 bytes for a 1920-pixel row) and walks the band:
// the windows of the two source rows of row y + kSegAhead are copied with 16-byte cp.async into the warp's own
// ring of kSegBufs row-pair slots while row y is computed from its slot; the rows' ytab entries ride along in
// registers a row ahead of their use. cp.async.wait_group and __syncwarp are the only waits. A window wider than
// a slot (tables this kernel was not sized for) makes the warp read that task's taps from global memory instead.
// ---------------------------------------------------------------------------------------------------------
constexpr int kSegDst = 640;
constexpr int kSegItems = kSegDst * 3 / 4;        // float4 items per output row
constexpr int kSegPerRow = kSegItems / 32;        // segments per output row
constexpr int kSegWarps = 8;
constexpr int kSegBandMax = 16;                   // output rows per task (4, 8 or 16: fewer for small batches)
constexpr int kSegWin = 512;                      // bytes of a staged source-row window
constexpr int kSegBufs = 4;
constexpr int kSegAhead = kSegBufs - 2;
constexpr int kSegSmem = 768 * 4 + kSegWarps * kSegBufs * 2 * kSegWin;
static_assert(kSegItems % 32 == 0 && kSegDst % kSegBandMax == 0 && kSegBandMax % kSegBufs == 0, "segment tiling");

template <int MODE>
__device__ __forceinline__ int seg_value(int A, int B, int C, int D, int4 t, int yz, int yw) {
  int q;
  if (MODE == 0) {
    const int left = (A * 256 + (C - A) * yz + 128) >> 8;
    const int right = (B * 256 + (D - B) * yz + 128) >> 8;
    q = (left * 256 + (right - left) * t.z + 128) >> 8;
  } else {
    const int h0 = A * t.z + B * t.w;
    const int h1 = C * t.z + D * t.w;
    q = ((((h0 >> 4) * yz) >> 16) + (((h1 >> 4) * yw) >> 16) + 2) >> 2;
  }
  return min(max(q, 0), 255);
}

// The same value when the right-hand x tap has weight zero (t.w == 0 in mode 1, t.z == 0 in mode 0): exactly
// the full formula with B = D = anything, without their loads and products. 1920-pixel rows resized to 640 (an
// exact 3:1 ratio) have such tables in both modes.
template <int MODE>
__device__ __forceinline__ int seg_value_left(int A, int C, int4 t, int yz, int yw) {
  int q;
  if (MODE == 0) {
    q = (A * 256 + (C - A) * yz + 128) >> 8;
  } else {
    q = ((((A * t.z) >> 4) * yz >> 16) + (((C * t.z) >> 4) * yw >> 16) + 2) >> 2;
  }
  return min(max(q, 0), 255);
}

__global__ void __launch_bounds__(kSegWarps * 32, 4) preprocess_seg_kernel(const __grid_constant__ BatchParams p,
                                                                           const float* __restrict__ lut,
                                                                           int layout, float* __restrict__ out,
                                                                           int n_tasks, int band_rows) {
  extern __shared__ __align__(16) uint8_t smem[];
  float* slut = reinterpret_cast<float*>(smem);  // [3][256]
  for (int i = threadIdx.x; i < 768; i += blockDim.x) slut[i] = __ldg(lut + i);
  __syncthreads();  // the only CTA-wide barrier: the LUT is in place
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ring = smem + 768 * 4 + warp * kSegBufs * 2 * kSegWin;  // [kSegBufs][2][kSegWin]
  const int bands = kSegDst / band_rows;
  const int n_warps = gridDim.x * kSegWarps;

  for (int task = blockIdx.x * kSegWarps + warp; task < n_tasks; task += n_warps) {
    const int seg = task % kSegPerRow;
    const int band = (task / kSegPerRow) % bands;
    const int image = task / (kSegPerRow * bands);
    const ImageParams& im = p.img[image];
    const int item = seg * 32 + lane;
    const int last = static_cast<int>(im.src_w) * 3 - 1;
    const int rmax = static_cast<int>(im.src_h) - 1;

    // The item's taps (as in the band kernel) and the segment's source window [wlo, whi).
    int4 tap[4];
    int lut_off[4];
    int64_t col_off;
    if (layout == KO_LAYOUT_CHW) {
      constexpr int per_ch = kSegDst / 4;
      const int c_rgb = item / per_ch, x0 = (item - c_rgb * per_ch) * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        tap[j] = __ldg(im.xtab + (x0 + j) * 3 + (2 - c_rgb));
        lut_off[j] = c_rgb << 8;
      }
      col_off = static_cast<int64_t>(c_rgb) * kSegDst * kSegDst + x0;
    } else {
      const int o0 = item * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int o = o0 + j, x = o / 3, c_rgb = o - x * 3;
        tap[j] = __ldg(im.xtab + x * 3 + (2 - c_rgb));
        lut_off[j] = c_rgb << 8;
      }
      if (layout == KO_LAYOUT_HWC) {
        col_off = o0;
      } else {
        const int px = o0 / 48;
        col_off = static_cast<int64_t>(px) * 768 + (o0 - px * 48);
      }
    }
    int lo = last, hi = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      tap[j].x = min(max(tap[j].x, 0), last);
      tap[j].y = min(max(tap[j].y, 0), last);
      lo = min(lo, min(tap[j].x, tap[j].y));
      hi = max(hi, max(tap[j].x, tap[j].y));
    }
    lo = __reduce_min_sync(0xffffffffu, lo);
    hi = __reduce_max_sync(0xffffffffu, hi);
    const int wlo = lo & ~15;
    const int whi = min((hi + 16) & ~15, last + 1);  // rows are whole 16-byte chunks (vec_ok)
    const int n16 = (whi - wlo) >> 4;
    float* obase = out + static_cast<int64_t>(image) * kSegDst * kSegDst * 3 + col_off;
    const int y0 = band * band_rows;

    if (whi - wlo > kSegWin) {  // window wider than a slot: taps straight from global memory
      for (int y = y0; y < y0 + band_rows; ++y) {
        const int4 yt = __ldg(im.ytab + y);
        const uint8_t* top = im.src + static_cast<int64_t>(min(max(yt.x, 0), rmax)) * im.src_stride;
        const uint8_t* bot = im.src + static_cast<int64_t>(min(max(yt.y, 0), rmax)) * im.src_stride;
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int4 t = tap[j];
          const int A = top[t.x], B = top[t.y], C = bot[t.x], D = bot[t.y];
          const int q =
              im.mode == 0 ? seg_value<0>(A, B, C, D, t, yt.z, yt.w) : seg_value<1>(A, B, C, D, t, yt.z, yt.w);
          v[j] = slut[lut_off[j] + q];
        }
        *reinterpret_cast<float4*>(obase + row_term(layout, y, kSegDst)) = make_float4(v[0], v[1], v[2], v[3]);
      }
      continue;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      tap[j].x -= wlo;
      tap[j].y -= wlo;
    }
    const uint8_t* src = im.src + wlo;
    const int64_t stride = im.src_stride;

    // Copy the two source windows of output row y into slot `buf` (n16 <= 32 chunks per window: one per lane).
    auto stage = [&](int y, int4 yt, int buf) {
      if (y < y0 + band_rows && lane < n16) {
        uint8_t* s = ring + buf * 2 * kSegWin + 16 * lane;
        cp_async16(s, src + static_cast<int64_t>(min(max(yt.x, 0), rmax)) * stride + 16 * lane);
        cp_async16(s + kSegWin, src + static_cast<int64_t>(min(max(yt.y, 0), rmax)) * stride + 16 * lane);
      }
      cp_async_commit();
    };
    // ytab entries: rows y (weights), y + 1, and y + kSegAhead (its copies are issued at step y).
    int4 yt0 = __ldg(im.ytab + y0), yt1 = __ldg(im.ytab + y0 + 1);
    int4 yt2 = __ldg(im.ytab + y0 + kSegAhead);
    static_assert(kSegAhead == 2, "the ytab register ring holds rows y .. y + 2");
    stage(y0, yt0, 0);
    stage(y0 + 1, yt1, 1);

    auto rows = [&](auto mode_c, auto left_c) {
      constexpr int MODE = decltype(mode_c)::value;
      constexpr bool LEFT = decltype(left_c)::value;
      int y = y0;
      auto step = [&](auto buf_c) {
        constexpr int BUF = decltype(buf_c)::value;
        stage(y + kSegAhead, yt2, (BUF + kSegAhead) % kSegBufs);
        const int yz = yt0.z, yw = yt0.w;
        yt0 = yt1;
        yt1 = yt2;
        yt2 = __ldg(im.ytab + min(y + kSegAhead + 1, kSegDst - 1));
        asm volatile("cp.async.wait_group %0;" ::"n"(kSegAhead) : "memory");
        __syncwarp();
        const uint8_t* s = ring + BUF * 2 * kSegWin;
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int4 t = tap[j];
          const int q = LEFT ? seg_value_left<MODE>(s[t.x], s[kSegWin + t.x], t, yz, yw)
                             : seg_value<MODE>(s[t.x], s[t.y], s[kSegWin + t.x], s[kSegWin + t.y], t, yz, yw);
          v[j] = slut[lut_off[j] + q];
        }
        *reinterpret_cast<float4*>(obase + row_term(layout, y, kSegDst)) = make_float4(v[0], v[1], v[2], v[3]);
        ++y;
      };
      for (int k = 0; k < band_rows / kSegBufs; ++k) {
        step(std::integral_constant<int, 0>{});
        step(std::integral_constant<int, 1>{});
        step(std::integral_constant<int, 2>{});
        step(std::integral_constant<int, 3>{});
      }
    };
    bool left_only = true;
#pragma unroll
    for (int j = 0; j < 4; ++j) left_only = left_only && (im.mode == 0 ? tap[j].z == 0 : tap[j].w == 0);
    left_only = __all_sync(0xffffffffu, left_only);
    using F = std::false_type;
    using T = std::true_type;
    if (im.mode == 0) {
      if (left_only)
        rows(std::integral_constant<int, 0>{}, T{});
      else
        rows(std::integral_constant<int, 0>{}, F{});
    } else {
      if (left_only)
        rows(std::integral_constant<int, 1>{}, T{});
      else
        rows(std::integral_constant<int, 1>{}, F{});
    }
    asm volatile("cp.async.wait_all;" ::: "memory");  // the next task refills the slots
    __syncwarp();
  }
}

int validate_image(const ko_image_desc& d, int64_t dst, const char* who) {
  if (!d.src || !d.xtab || !d.ytab) return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": null pointer");
  if (d.src_h < 1 || d.src_w < 1 || d.src_stride < d.src_w * 3 || d.src_w > (1 << 20) || d.src_h > (1 << 20))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": bad image size or stride");
  if (d.mode != 0 && d.mode != 1) return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": mode must be 0 or 1");
  if (!ko::aligned16(d.xtab) || !ko::aligned16(d.ytab))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": tables must be 16-byte aligned");
  (void)dst;
  return KO_OK;
}

}  // namespace

extern "C" int ko_preprocess_batch(const ko_image_desc* images, int n, const float* lut, int64_t dst, int layout,
                                   float* out, ko_stream_t stream) {
  const char* who = "ko_preprocess";
  if (n < 1 || n > kMaxImages || !images) return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_preprocess: 1..64 images per call");
  if (!lut || !out || !ko::aligned16(out)) return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_preprocess: lut/out null or out unaligned");
  if (layout != KO_LAYOUT_HWC && layout != KO_LAYOUT_CHW && layout != KO_LAYOUT_PATCH16)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_preprocess: unknown layout");
  if (dst < 4 || dst > 8192 || dst % 4 != 0 || (layout == KO_LAYOUT_PATCH16 && dst % 16 != 0))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_preprocess: dst must be a multiple of 4 (16 for PATCH16)");
  BatchParams p;
  std::memset(&p, 0, sizeof p);
  int64_t row_cap = 16;
  for (int i = 0; i < n; ++i) {
    const ko_image_desc& d = images[i];
    int st = validate_image(d, dst, who);
    if (st) return st;
    ImageParams& q = p.img[i];
    q.src = d.src;
    q.xtab = reinterpret_cast<const int4*>(d.xtab);
    q.ytab = reinterpret_cast<const int4*>(d.ytab);
    q.src_h = d.src_h;
    q.src_w = d.src_w;
    q.src_stride = d.src_stride;
    q.mode = d.mode;
    q.vec_ok = ko::aligned16(d.src) && d.src_stride % 16 == 0 && (d.src_w * 3) % 16 == 0;
    row_cap = std::max<int64_t>(row_cap, (d.src_w * 3 + 15) / 16 * 16);
  }
  const ko::DeviceInfo* dinfo = nullptr;
  if (int rc = ko::device_or_fail(&dinfo, "ko_preprocess")) return rc;
  const ko::DeviceInfo& info = *dinfo;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t n_items = dst * 3 / 4;
  bool seg_ok = dst == kSegDst && layout != KO_LAYOUT_CHW;  // CHW items span 4 pixels of one channel: wide windows
  for (int i = 0; i < n && seg_ok; ++i) seg_ok = p.img[i].vec_ok;
  if (seg_ok) {
    cudaError_t e = cudaFuncSetAttribute(preprocess_seg_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                         cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return ko::fail(static_cast<int>(e), "ko_preprocess: cannot set the shared-memory carveout");
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, preprocess_seg_kernel, kSegWarps * 32, kSegSmem);
    if (e != cudaSuccess || per_sm < 1) return ko::fail(KO_ERR_UNSUPPORTED, "ko_preprocess: segment kernel does not fit");
    // Bands of 16 rows, or 8 / 4 when the batch is too small to give every resident warp two tasks.
    int band_rows = kSegBandMax;
    while (band_rows > kSegBufs &&
           static_cast<int64_t>(n) * (kSegDst / band_rows) * kSegPerRow < 2LL * per_sm * info.sm_count * kSegWarps)
      band_rows /= 2;
    const int n_tasks = n * (kSegDst / band_rows) * kSegPerRow;
    const int64_t grid = std::min<int64_t>(static_cast<int64_t>(per_sm) * info.sm_count,
                                           (n_tasks + kSegWarps - 1) / kSegWarps);
    preprocess_seg_kernel<<<static_cast<unsigned>(grid), kSegWarps * 32, kSegSmem, st>>>(p, lut, layout, out,
                                                                                         n_tasks, band_rows);
    return ko::check_launch("ko_preprocess");
  }
  if (n_items <= 2 * kBandThreads) {
    // Band kernel: the largest band (rows per CTA) that still gives every SM about eight CTAs.
    const int64_t target = 8 * static_cast<int64_t>(info.sm_count);
    int band = 16;
    while (band > 1 && n * ((dst + band - 1) / band) < target) band /= 2;
    const int64_t smem = 768 * 4 + 6 * row_cap;
    if (smem > info.max_smem_optin) return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_preprocess: source rows too wide");
    dim3 grid(static_cast<unsigned>((dst + band - 1) / band), static_cast<unsigned>(n));
    auto kern = n_items <= kBandThreads ? preprocess_band_kernel<1> : preprocess_band_kernel<2>;
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (e != cudaSuccess) return ko::fail(static_cast<int>(e), "ko_preprocess: cannot enable large shared memory");
    }
    kern<<<grid, kBandThreads, smem, st>>>(p, lut, static_cast<int>(dst), layout, out, static_cast<int>(row_cap),
                                           band);
    return ko::check_launch("ko_preprocess");
  }
  // Wider outputs: one CTA per (output row, image), row pair staged synchronously.
  const int64_t smem = 2 * row_cap;
  if (smem > info.max_smem_optin) return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_preprocess: source rows too wide");
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(preprocess_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return ko::fail(static_cast<int>(e), "ko_preprocess: cannot enable large shared memory");
  }
  dim3 grid(static_cast<unsigned>(dst), static_cast<unsigned>(n));
  preprocess_kernel<<<grid, kThreads, smem, st>>>(
      p, lut, static_cast<int>(dst), layout, out, static_cast<int>(row_cap));
  return ko::check_launch("ko_preprocess");
}

extern "C" int ko_preprocess(const uint8_t* src, int64_t src_h, int64_t src_w, int64_t src_stride,
                             const int32_t* xtab, const int32_t* ytab, const float* lut, int mode, int64_t dst,
                             int layout, float* out, ko_stream_t stream) {
  ko_image_desc d;
  d.src = src;
  d.xtab = xtab;
  d.ytab = ytab;
  d.src_h = src_h;
  d.src_w = src_w;
  d.src_stride = src_stride;
  d.mode = mode;
  d._pad = 0;
  return ko_preprocess_batch(&d, 1, lut, dst, layout, out, stream);
}
