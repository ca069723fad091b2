// im2col of a 3x3, stride-1, zero-padded convolution on an NHWC fp32 tensor, written as the A operand of the
// tcgen05 GEMM:   cols[(b*H + y)*W + x][tap*C + c] = x[b][y + dy - 1][x + dx - 1][c]  (tap = dy*3 + dx; 0 outside).
//
// Semantics: the projector's 3x3 convolutions (fast_rfdetr/model.py:148-158, mx.conv2d with padding 1) as im2col +
// GEMM, the column order matching the conv weight [out][kh][kw][in] flattened to [out][9*in].
//
// B200 design: one thread per 16-byte output chunk, consecutive threads on consecutive chunks of an output row
// (coalesced 128-bit stores; the 9 taps of a pixel read 9 neighbouring 16-byte chunks of the input, served by L2),
// a grid of whole waves striding over the output. Padding is written as zeros in the same pass, so the padded copy
// and the concatenation of nine shifted views that a framework would make are one kernel.
#include <algorithm>
#include <climits>

#include "ko_common.cuh"

namespace {

__global__ void __launch_bounds__(256) im2col3x3_kernel(const float4* __restrict__ x, int B, int H, int W, int C4,
                                                        float4* __restrict__ cols) {
  const int64_t row_chunks = 9LL * C4;
  const int64_t total = static_cast<int64_t>(B) * H * W * row_chunks;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t pix = i / row_chunks;
    const int k = static_cast<int>(i - pix * row_chunks);
    const int tap = k / C4, c = k - tap * C4;
    const int px = static_cast<int>(pix % W);
    const int64_t by = pix / W;
    const int py = static_cast<int>(by % H);
    const int yy = py + tap / 3 - 1, xx = px + tap % 3 - 1;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (yy >= 0 && yy < H && xx >= 0 && xx < W) v = __ldg(x + ((by - py + yy) * W + xx) * C4 + c);
    cols[i] = v;
  }
}

}  // namespace

extern "C" int ko_im2col3x3(const float* x, int64_t B, int64_t H, int64_t W, int64_t C, float* cols,
                            ko_stream_t stream) {
  if (B < 0 || H < 0 || W < 0 || C < 4 || C % 4 != 0 || B > INT32_MAX || H > INT32_MAX || W > INT32_MAX ||
      C > (int64_t(1) << 20))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_im2col3x3: need C % 4 == 0 and non-negative sizes");
  if (B == 0 || H == 0 || W == 0) return KO_OK;
  if (!x || !cols || !ko::aligned16(x) || !ko::aligned16(cols))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_im2col3x3: pointers must be non-null and 16-byte aligned");
  const int64_t total = B * H * W * 9 * (C / 4);
  const ko::DeviceInfo* info = nullptr;
  if (int st = ko::device_or_fail(&info, "ko_im2col3x3")) return st;
  const int64_t sms = info->sm_count;
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, sms * 8);
  im2col3x3_kernel<<<static_cast<unsigned>(blocks), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const float4*>(x), static_cast<int>(B), static_cast<int>(H), static_cast<int>(W),
      static_cast<int>(C / 4), reinterpret_cast<float4*>(cols));
  return ko::check_launch("ko_im2col3x3");
}
