/*
 * kernelopt.h — C ABI of libkernelopt.so, the sm_100a (B200) kernels of the RF-DETR-Medium inference hot path.
 *
 * The reference (ishaanzee/kernelopt) reaches its four GPU kernels through Python wrappers around
 * mx.fast.metal_kernel in fast_rfdetr/kernels.py. Each entry point below replaces one of those wrappers (or the
 * host helper it relies on); the comment on each cites the reference interface it stands in for.
 *
 * Conventions shared by every entry point:
 *   - All tensor arguments are raw device pointers to contiguous, row-major buffers owned by the caller.
 *     No entry point allocates device memory; scratch space, where needed, is passed in by the caller.
 *   - Sizes are int64_t. Scalars (eps, mode, offset) are passed by value.
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream). Work is enqueued asynchronously.
 *   - The return value is KO_OK (0), a cudaError_t value (1..999) from a failed launch, or one of the KO_ERR_*
 *     codes below. ko_last_error_string() describes the most recent failure on the calling host thread.
 *   - Kernels that wait on on-chip barriers (the tcgen05 GEMM) bound every wait. When a wait runs out the
 *     kernel writes KO_ERR_DEVICE_TIMEOUT into *dev_status (an int in device memory, may be NULL) and returns;
 *     the caller reads it after synchronising.
 */
#ifndef KERNELOPT_H_
#define KERNELOPT_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* ko_stream_t; /* identical to cudaStream_t */

#define KO_OK 0
#define KO_ERR_INVALID_ARGUMENT 1001 /* a size, layout or alignment precondition does not hold */
#define KO_ERR_UNSUPPORTED 1002      /* the device is not sm_100 or a driver entry point is missing */
#define KO_ERR_DEVICE_TIMEOUT 1003   /* written to *dev_status by a kernel whose bounded wait ran out */

/* Output layouts of ko_preprocess / ko_preprocess_batch. */
#define KO_LAYOUT_HWC 0     /* [dst, dst, 3] RGB, the reference's preprocess_gpu output */
#define KO_LAYOUT_CHW 1     /* [3, dst, dst] RGB, the NCHW tensor Ballform's cv2 path produces */
#define KO_LAYOUT_PATCH16 2 /* [(dst/16)^2, 16*16*3]: 16x16 patches flattened as (ky, kx, c) — the im2col of the
                               ViT patch-embedding convolution, so that convolution becomes one GEMM */

/* Table policies of ko_resize_tables. */
#define KO_RESIZE_REFERENCE 0 /* the reference's model of the macOS arm64 cv2 wheel: KleidiCV arithmetic for the
                                 sizes that wheel hands to KleidiCV, OpenCV's fixed-point arithmetic otherwise */
#define KO_RESIZE_OPENCV 1    /* OpenCV's own fixed-point path for every size: cv2 builds without KleidiCV,
                                 such as the x86-64 wheels */

/* Activations of ko_linear_f32_packed. */
#define KO_ACT_NONE 0
#define KO_ACT_GELU 1 /* GELU 0.5 v (1 + erf(v / sqrt 2)), erf by A&S 7.1.26 (|error| < 1.5e-7) */
#define KO_ACT_RELU 2
#define KO_ACT_SILU 3 /* v / (1 + exp(-v)); ko_layernorm only */

/* --- status / version ------------------------------------------------------------------------------------- */

/* Text of the last failure on the calling host thread ("" if none). */
const char* ko_last_error_string(void);
/* ABI version, bumped whenever a signature below changes. */
int ko_abi_version(void);
/* 0 when the current device is an sm_100-class GPU this library was built for, else KO_ERR_UNSUPPORTED. */
int ko_check_device(void);
/* Runs the bounded on-chip wait of the tcgen05 kernels on a barrier that nothing completes: after limit_ns the
 * wait gives up, a second warp waiting on the same barrier leaves on the CTA's abort flag, and
 * KO_ERR_DEVICE_TIMEOUT is written to *dev_status (device memory) — the failure path of every kernel with
 * on-chip waits, without a fault. For tests and health checks; no counterpart in the reference. */
int ko_wait_probe(int64_t limit_ns, int* dev_status, ko_stream_t stream);

/* --- preprocessing: uint8 BGR frame -> resized, RGB, normalised float32 ------------------------------------ */

/* Host function. Fills the interpolation tables that reproduce cv2.resize(INTER_LINEAR) of a uint8 3-channel
 * image from src_w x src_h to dst_w x dst_h. Replaces resize_tables.tables (fast_rfdetr/resize_tables.py:165-184).
 *   xtab: int32 [dst_w*3][4] = (left element, right element, weight a, weight b) per output element x*3+c
 *   ytab: int32 [dst_h][4]   = (top row, bottom row, weight a, weight b) per output row
 *   *mode: 0 = KleidiCV arithmetic, 1 = OpenCV arithmetic (the `mode` argument of ko_preprocess). */
int ko_resize_tables(int64_t src_w, int64_t src_h, int64_t dst_w, int64_t dst_h, int policy, int32_t* xtab,
                     int32_t* ytab, int* mode);

/* One frame. Replaces preprocess_gpu (fast_rfdetr/kernels.py:106-116; kernel source :74-103).
 * src: uint8 [src_h][src_stride] holding BGR pixels (src_stride >= src_w*3 bytes); xtab/ytab from
 * ko_resize_tables (device copies); lut: float32 [3][256] with lut[c][v] = (v/255 - mean[c]) / std[c] for RGB
 * channel c; out: float32 in `layout`. Output is bit-identical to the reference kernel on the same tables. */
int ko_preprocess(const uint8_t* src, int64_t src_h, int64_t src_w, int64_t src_stride, const int32_t* xtab,
                  const int32_t* ytab, const float* lut, int mode, int64_t dst, int layout, float* out,
                  ko_stream_t stream);

/* One image of a batch for ko_preprocess_batch (all pointers are device pointers). */
typedef struct ko_image_desc {
  const uint8_t* src;
  const int32_t* xtab;
  const int32_t* ytab;
  int64_t src_h, src_w, src_stride;
  int32_t mode;
  int32_t _pad;
} ko_image_desc;

/* Several frames of any sizes in one launch; image i is written at out + i*dst*dst*3. Replaces the per-image
 * preprocess_gpu loop of FastBasketballDetector.raw_batch (fast_rfdetr/detector.py:100). `images` is a HOST
 * array of n descriptors; n <= 64 per call. */
int ko_preprocess_batch(const ko_image_desc* images, int n, const float* lut, int64_t dst, int layout, float* out,
                        ko_stream_t stream);

/* --- fused residual add + LayerNorm ------------------------------------------------------------------------- */

/* h_out = h + (o + bias) * scale;  y = (h_out - mean) / sqrt(var + eps) * gamma + beta  (row statistics in fp32,
 * biased variance). h, o, h_out, y: float32 [rows][C]; bias, scale, gamma, beta: float32 [C]. C % 4 == 0.
 * bias and scale may be NULL (0 and 1). h_out may alias h. Replaces residual_layernorm
 * (fast_rfdetr/kernels.py:53-67; kernel source :9-48). */
int ko_residual_layernorm(const float* h, const float* o, const float* bias, const float* scale, const float* gamma,
                          const float* beta, float eps, int64_t rows, int64_t C, float* h_out, float* y,
                          ko_stream_t stream);

/* y = act(LayerNorm(x) * gamma + beta) over rows of C (biased variance, eps inside the square root), act
 * KO_ACT_NONE or KO_ACT_SILU. x, y: float32 [rows][C], C % 4 == 0, C <= 1024; y may alias x. Replaces the plain
 * mx.fast.layer_norm calls of the model (fast_rfdetr/model.py:80-82) and, with SiLU, the channel LayerNorm + SiLU
 * of the projector's conv blocks (model.py:157-158). */
int ko_layernorm(const float* x, const float* gamma, const float* beta, float eps, int64_t rows, int64_t C, int act,
                 float* y, ko_stream_t stream);

/* The ViT backbone's tokens, kept in window order h: float32 [B * nwin][1 + win*win][C] (a class token, then the
 * window's pixels row by row; windows row-major over the H x W grid, nwin = (H/win) * (W/win)), written as an
 * NHWC image into channels [col_off, col_off + C) of out: float32 [B][H][W][ldo]:
 *   out[b][py][px][col_off + c] = LN(h[(b*nwin + w)*(1 + win*win) + 1 + (py%win)*win + (px%win)][c])
 * with w = (py/win)*(W/win) + px/win and LN = (v - mean) / sqrt(var + eps) * gamma + beta over C (biased variance),
 * or the value itself when normalize == 0 (gamma, beta may then be NULL). C % 4 == 0, C <= 1024, ldo and col_off
 * multiples of 4, 16-byte aligned pointers. Replaces the window merge (fast_rfdetr/model.py:104-105), the final
 * LayerNorm of the tapped layers (model.py:101-103) and the channel concatenation of the projector input
 * (model.py:161) with one pass per tapped layer. */
int ko_window_merge_ln(const float* h, const float* gamma, const float* beta, float eps, int64_t B, int64_t H,
                       int64_t W, int64_t win, int64_t C, int normalize, float* out, int64_t ldo, int64_t col_off,
                       ko_stream_t stream);

/* The backbone's entry: t: float32 [B][H][W][C] (the patch embedding, bias included), pos: [H][W][C], cls: [C]
 * -> h: float32 [B * nwin][1 + win*win][C] in window order (nwin = (H/win) * (W/win), windows row-major, each
 * row block led by the class token), h = cls for the first row of a window and t + pos for its pixels (row by
 * row), and y = LayerNorm(h) over C with gamma, beta, eps (biased variance). C % 4 == 0, C <= 1024, 16-byte
 * aligned pointers. Replaces the pos add, window partition and class-token concatenation of fast_rfdetr/model.py:88-90
 * and the first layer's LayerNorm (model.py:94) with one pass. */
int ko_window_partition_ln(const float* t, const float* pos, const float* cls, const float* gamma,
                           const float* beta, float eps, int64_t B, int64_t H, int64_t W, int64_t win, int64_t C,
                           float* h, float* y, ko_stream_t stream);

/* cols[(b*H + y)*W + x][tap*C + c] = x[b][y + dy - 1][x + dx - 1][c] (tap = 3*dy + dx, zero outside the image):
 * the im2col of a 3x3, stride-1, padding-1 convolution on an NHWC float32 tensor, in the column order of a conv
 * weight [out][3][3][in] flattened to [out][9*in]. C % 4 == 0; x, cols 16-byte aligned. Replaces the padded
 * mx.conv2d of the projector's 3x3 convolutions (fast_rfdetr/model.py:154-156) as the A operand of
 * ko_linear_f32_packed. */
int ko_im2col3x3(const float* x, int64_t B, int64_t H, int64_t W, int64_t C, float* cols, ko_stream_t stream);

/* --- deformable-attention sampling (single level) ----------------------------------------------------------- */

/* out[b,q,h*HD+d] = sum_p aw[b,q,h,p] * bilinear(value[b, :, offset + h*HD + d] viewed as GH x GW, loc[b,q,h,p])
 * with grid_sample semantics (align_corners=False, zero padding): x = loc_x*GW - 0.5, y = loc_y*GH - 0.5.
 * value: float32 [B][GH*GW][ROW]; loc: float32 [B][NQ][NH][NP][2] (x, y in [0,1]); aw: float32 [B][NQ][NH][NP];
 * out: float32 [B][NQ][NH*HD]. offset + NH*HD <= ROW. Replaces deform_attn (fast_rfdetr/kernels.py:165-181;
 * kernel source :124-162). */
int ko_deform_attn(const float* value, const float* loc, const float* aw, int64_t B, int64_t NQ, int64_t NH,
                   int64_t HD, int64_t NP, int64_t GH, int64_t GW, int64_t ROW, int64_t offset, float* out,
                   ko_stream_t stream);

/* The sampling inputs of one decoder cross-attention layer from its projection: oa: float32 [B*NQ rows][ld_oa]
 * holding NH*NP*2 sampling offsets (head, point, x/y) then NH*NP attention logits (head, point); ref: float32
 * [B*NQ][4] (cx, cy, w, h), 16-byte aligned. Writes loc: [B*NQ][NH][NP][2] = ref_xy + off / NP * ref_wh * 0.5 and
 * aw: [B*NQ][NH][NP] = softmax over the points of the logits. NP <= 8, NH <= 4096. Replaces the reshape /
 * softmax / location arithmetic of fast_rfdetr/model.py:222-225 with one launch. */
int ko_deform_prep(const float* oa, const float* ref, int64_t B, int64_t NQ, int64_t NH, int64_t NP, int64_t ld_oa,
                   float* loc, float* aw, ko_stream_t stream);

/* --- fp32-grade GEMM on tcgen05 tensor cores (3xTF32 split) ------------------------------------------------- */

/* Bytes of scratch that ko_linear_gelu_f32 needs for a [K, N] weight (its split, transposed copy). */
int64_t ko_linear_workspace_bytes(int64_t K, int64_t N);

/* Splits w (float32 [K][N], the x @ W convention) into w_packed = float32 [2][N][K]: w_packed[0] = tf32(w)^T,
 * w_packed[1] = tf32(w - tf32(w))^T. Run once per weight; the result feeds ko_linear_f32_packed. No reference
 * counterpart (the reference's GEMM reads w directly, fast_rfdetr/kernels.py:245). */
int ko_pack_weight_tf32x3(const float* w, int64_t K, int64_t N, float* w_packed, ko_stream_t stream);

/* out = act(x @ W + bias) with x float32 [M][K], W given pre-split by ko_pack_weight_tf32x3, bias float32 [N]
 * (may be NULL), out float32 [M][N]. Three TF32 tensor-core products (hi*hi + hi*lo + lo*hi) with fp32
 * accumulation in TMEM give fp32-grade results. K % 4 == 0, N % 4 == 0, 16-byte aligned pointers. */
int ko_linear_f32_packed(const float* x, const float* w_packed, const float* bias, int64_t M, int64_t K, int64_t N,
                         int act, float* out, int* dev_status, ko_stream_t stream);

/* out = act(x @ W + bias + A) where A[i][j] = addend[i * ld_addend + j] for j < add_cols and 0 beyond: the GEMM
 * of ko_linear_f32_packed with a per-element term added in its epilogue. add_cols and ld_addend multiples of 4,
 * 4 <= add_cols <= N, ld_addend >= add_cols, addend 16-byte aligned and not aliasing
 * out. The decoder uses it for (tgt + qpos) @ W = tgt @ W + qpos @ W, with qpos @ W of all four layers computed
 * once: it replaces the `tgt + qpos` additions before the self-attention q / k projections and the
 * cross-attention offset / weight projections (fast_rfdetr/model.py:251, :256) and lets the value projection
 * of tgt share the q / k GEMM. */
int ko_linear_add_f32_packed(const float* x, const float* w_packed, const float* bias, const float* addend,
                             int64_t ld_addend, int64_t add_cols, int64_t M, int64_t K, int64_t N, int act,
                             float* out, int* dev_status, ko_stream_t stream);

/* GEMM with the residual add and LayerNorm in its epilogue, whole rows at a time:
 *   v = resid + (x @ W + bias) * scale;   y = act((v - mean(v)) / sqrt(var(v) + eps) * gamma + beta)
 * with the mean and biased variance over the N columns of each row. x float32 [M][K]; W pre-split by
 * ko_pack_weight_tf32x3; bias, scale, gamma, beta float32 [N] (bias NULL = 0, scale NULL = 1); resid float32
 * [M][N] or NULL (no residual); h_out float32 [M][N] receives v, or NULL (not written); h_out may alias resid,
 * y must alias none of x, resid, h_out; row r of y starts at y + r * ldy (ldy 0 = N; else a multiple of 4 >= N,
 * so y may be a column slice of a wider buffer). act KO_ACT_NONE or KO_ACT_SILU. N one of 128, 192, 256, 384, 512 (a
 * row spans one CTA, or a cluster of two that exchange row statistics); K % 4 == 0; 16-byte aligned pointers.
 * The GEMM is the 3xTF32 product of ko_linear_f32_packed. Fuses the reference's next step: its attention
 * out-projection and fc2 GEMMs followed by residual_layernorm (fast_rfdetr/model.py:121-123, 129-132,
 * kernels.py:9-67), and also GEMM + LayerNorm + SiLU (model.py:148-158) and GEMM + LayerNorm (model.py:178). */
int ko_linear_residual_ln_f32_packed(const float* x, const float* w_packed, const float* bias, const float* scale,
                                     const float* resid, const float* gamma, const float* beta, float eps,
                                     int64_t M, int64_t K, int64_t N, int act, float* h_out, float* y, int64_t ldy,
                                     int* dev_status, ko_stream_t stream);

/* out = GELU_erf(x @ w + bias): packs w into `workspace` (ko_linear_workspace_bytes(K, N) bytes, 16-byte
 * aligned) and runs ko_linear_f32_packed. Replaces linear_gelu_f32 (fast_rfdetr/kernels.py:271-285; kernel
 * source :188-266). */
int ko_linear_gelu_f32(const float* x, const float* w, const float* bias, int64_t M, int64_t K, int64_t N,
                       float* out, void* workspace, int64_t workspace_bytes, int* dev_status, ko_stream_t stream);

/* out = GELU_erf(x @ w + bias) like ko_linear_gelu_f32, but needing no workspace: for callers that cannot
 * allocate device memory at run time — applications whose allocator owns all GPU memory and forbids libraries
 * to allocate, real-time per-frame paths where cudaMalloc/cudaFree can synchronise the device, plugin hosts that
 * pass only input and output buffers. The weight split (2*K*N floats) goes to an 8 MiB array in the library's
 * static device memory, held by every GPU that loads the library until exit; nothing is allocated per call.
 * Limits: K*N <= KO_NOALLOC_MAX_WEIGHT_ELEMS, else KO_ERR_INVALID_ARGUMENT. All calls on a device share the
 * array: calls that overlap on the GPU race and must be ordered (one stream, or events). Each call rewrites the
 * part it reads first, so nothing needs clearing. The first call on a device looks up the array's address; make
 * it before any stream capture on that device. No counterpart in the reference (its kernels run inside MLX,
 * which allocates every buffer itself). */
#define KO_NOALLOC_MAX_WEIGHT_ELEMS 1048576
int ko_linear_gelu_f32_noalloc(const float* x, const float* w, const float* bias, int64_t M, int64_t K, int64_t N,
                               float* out, int* dev_status, ko_stream_t stream);

/* A 3x3 convolution (stride 1, zero padding 1) as an implicit GEMM on the same tensor cores, with the LayerNorm
 * (+ SiLU) of ko_linear_residual_ln_f32_packed in its epilogue and no residual:
 *   y[p] = act(LN(sum_{ky,kx,c} x[b][py+ky-1][px+kx-1][c] * w[(ky*3+kx)*C + c][:] + bias) * gamma + beta)
 * x: float32 NHWC [B][H][W][C] with pixel p at x + p * ldx, C % 16 == 0; w_packed: ko_pack_weight_tf32x3 of the
 * weight as [9*C][N] in (ky, kx, c) row order (the conv weight [N][3][3][C] flattened and transposed); y: float32
 * [B*H*W][N] with row p at y + p * ldy; N one of 128, 192, 256, 384, 512; ldx / ldy 0 (= C / N) or multiples of 4
 * not below C / N, so that x and y can be channel slices of wider NHWC buffers (the projector's concatenation,
 * fast_rfdetr/model.py:161, is written in place). No im2col buffer: each k-block's TMA load reads x shifted by
 * the tap, and rows whose shifted pixel lies outside the image are zeroed on chip. Replaces the projector's conv
 * -> channel LayerNorm -> SiLU blocks (fast_rfdetr/model.py:148-158) with one kernel each. */
int ko_conv3x3_ln_f32_packed(const float* x, int64_t ldx, const float* w_packed, const float* bias,
                             const float* gamma, const float* beta, float eps, int64_t B, int64_t H, int64_t W,
                             int64_t C, int64_t N, int act, float* y, int64_t ldy, int* dev_status,
                             ko_stream_t stream);

/* --- query selection ------------------------------------------------------------------------------------------ */

/* The top-NQ proposals of each frame by class score, and their refined reference boxes:
 *   score[b, i] = max_c logits[b, i, c];   order = proposals by descending score, ties by ascending index
 *   c = coord(b, idx[b, q]) with coord = (delta_xy * prop_wh + prop_xy, exp(delta_wh) * prop_wh)
 *   ref[b, q] = (rp_xy[q] * c_wh + c_xy, rp_ewh[q] * c_wh)
 * logits: float32 [B][NP][NC]; delta: float32 [B][NP][4]; proposals: float32 [NP][4] (cx, cy, w, h);
 * rp_xy, rp_ewh: float32 [NQ][2]; ref: float32 [B][NQ][4]; idx: int32 [B][NQ] or NULL. 1 <= NQ <= NP <= 4096.
 * delta, proposals and ref 16-byte aligned, rp_xy and rp_ewh 8-byte aligned. Replaces select_queries'
 * max / argsort / take_along_axis / box refinement (fast_rfdetr/model.py:175-185). */
int ko_select_queries(const float* logits, const float* delta, const float* proposals, const float* rp_xy,
                      const float* rp_ewh, int64_t B, int64_t NP, int64_t NC, int64_t NQ, float* ref, int32_t* idx,
                      ko_stream_t stream);

/* --- multi-head attention, fp32 grade (3xTF32 on tcgen05, flash style) ------------------------------------- */

/* o[b, i, h, :] = sum_j softmax_j(scale * q[b, i, h, :] . k[b, j, h, :]) v[b, j, h, :], no mask.
 * Element (b, i, h, d) of q lives at q + b*q_bstride + i*q_row + h*head_dim + d; k, v and o likewise with their
 * own strides (in elements), so q, k and v can be column slices of one fused QKV projection.
 * head_dim 32 or 64; batch, heads <= 65535; every stride a multiple of 4; pointers 16-byte aligned; scale > 0.
 * Replaces mx.fast.scaled_dot_product_attention at fast_rfdetr/model.py:110 and :119-120 (backbone, windowed and
 * global layers) and :238 (decoder self-attention). dev_status as for ko_linear_f32_packed. */
int ko_attention_f32(const float* q, const float* k, const float* v, float* o, int64_t batch, int64_t L,
                     int64_t heads, int64_t head_dim, int64_t q_bstride, int64_t q_row, int64_t k_bstride,
                     int64_t k_row, int64_t v_bstride, int64_t v_row, int64_t o_bstride, int64_t o_row, float scale,
                     int* dev_status, ko_stream_t stream);

/* --- decoder and head steps --------------------------------------------------------------------------------- */

/* out[r][g*128 + k] = sin(v) for even k, cos(v) for odd k, v = ref[r][c_g] * 2*pi / dim_t[k], with coordinates
 * c_g = (1, 0, 2, 3) for the four groups g (y, x, w, h): ref float32 [rows][4], dim_t float32 [128], out
 * float32 [rows][512], 16-byte aligned. Replaces sine_embed (fast_rfdetr/model.py:188-194). */
int ko_sine_embed(const float* ref, const float* dim_t, int64_t rows, float* out, ko_stream_t stream);

/* out = act(x @ w + bias) for narrow outputs, fp32 FMA (not the tensor cores): x float32 [M][K], w float32
 * [K][N] row-major, bias float32 [N] or NULL, out float32 [M][N]; 1 <= N <= 32, K*N <= 12288, act KO_ACT_NONE or
 * KO_ACT_RELU. Deterministic (fixed reduction order). Replaces the class heads' matmuls (fast_rfdetr/model.py:179,
 * :269) and the 4-wide last layer of the encoder's box MLP (:180). */
int ko_linear_small_f32(const float* x, const float* w, const float* bias, int64_t M, int64_t K, int64_t N,
                        int act, float* out, ko_stream_t stream);

/* boxes[r] = (d0 * ref2 + ref0, d1 * ref3 + ref1, exp(d2) * ref2, exp(d3) * ref3) with d = x[r] @ w + bias:
 * the last layer of the box MLP (K inputs, 4 outputs) and the box refinement in one kernel. x float32 [M][K], w
 * float32 [K][4], bias float32 [4] or NULL, ref float32 [M][4] (cx, cy, w, h), boxes float32 [M][4]; ref and boxes
 * 16-byte aligned, K <= 3072. Replaces bbox_embed's last layer and the box arithmetic of fast_rfdetr/model.py:270-272. */
int ko_box_head_f32(const float* x, const float* w, const float* bias, const float* ref, int64_t M, int64_t K,
                    float* boxes, ko_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* KERNELOPT_H_ */
