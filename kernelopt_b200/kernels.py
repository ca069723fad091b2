"""The four hot-path kernels, with the reference's call signatures (fast_rfdetr/kernels.py), on torch CUDA tensors.

    residual_layernorm(h, o, bias, scale, gamma, beta, eps) -> (h_out, y)     kernels.py:53
    preprocess_gpu(img_u8, xtab, ytab, lut, mode, dst=640) -> [dst,dst,3]      kernels.py:106
    deform_attn(value, loc, aw, grid_hw, nh, hd, offset=0) -> [B,NQ,NH*HD]     kernels.py:165
    linear_gelu_f32(x, w, bias) -> [..., N]                                    kernels.py:271
plus attention(q, k, v, heads, scale), which replaces the reference's mx.fast.scaled_dot_product_attention calls.

Every call goes to libkernelopt.so (hand-written sm_100a CUDA) on the caller's current CUDA stream. Outputs
are freshly allocated unless the function takes an `out` (or `h` / `y`) buffer; inputs are read-only and must be
contiguous float32 (uint8/int32 for preprocessing) CUDA tensors. There is no CPU path: CPU tensors raise
ValueError, a missing library raises RuntimeError.
Beyond the reference's API, the model's other fused steps: batched preprocessing (`preprocess_batch`); the
pre-split weight form of the GEMM (`pack_weight` / `linear`) used for every dense layer, with its residual +
LayerNorm epilogue (`linear_residual_layernorm`) and the implicit 3x3 convolution (`conv3x3_layernorm`);
`layernorm`, `im2col3x3`; the backbone's `window_partition_layernorm` / `window_merge_layernorm`; the decoder's
`select_queries` and `deform_prep`.
"""
from __future__ import annotations

import threading
import weakref

import torch

from . import _lib
from ._lib import call

LAYOUTS = {"hwc": _lib.KO_LAYOUT_HWC, "chw": _lib.KO_LAYOUT_CHW, "patch16": _lib.KO_LAYOUT_PATCH16}
ACTS = {None: _lib.KO_ACT_NONE, "none": _lib.KO_ACT_NONE, "gelu": _lib.KO_ACT_GELU, "relu": _lib.KO_ACT_RELU}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _need(t: torch.Tensor, name: str, dtype=torch.float32):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (there is no CPU path)")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# ---- device-side status word for kernels with bounded waits ----
_status: dict[int, torch.Tensor] = {}
_status_lock = threading.Lock()


def _dev_index(device) -> int:
    if device is None:
        return torch.cuda.current_device()
    if isinstance(device, int):
        return device
    d = torch.device(device)
    return d.index if d.index is not None else torch.cuda.current_device()


def status_word(device=None) -> torch.Tensor:
    """The int32 device word that bounded-wait kernels write KO_ERR_DEVICE_TIMEOUT into."""
    idx = _dev_index(device)
    with _status_lock:
        if idx not in _status:
            _status[idx] = torch.zeros(1, dtype=torch.int32, device=f"cuda:{idx}")
        return _status[idx]


def check_device_status(device=None) -> None:
    """Synchronising check of the status word; raises KernelError (and clears it) if a kernel timed out."""
    w = status_word(device)
    v = int(w.item())
    if v != 0:
        w.zero_()
        raise _lib.KernelError("device kernel", v, "an on-chip wait ran out; the results of that launch are invalid")


# ---- residual + LayerNorm ----
def residual_layernorm(h, o, bias, scale, gamma, beta, eps):
    """Returns (h + (o + bias) * scale, LayerNorm of that). h, o: [..., C] float32, C % 4 == 0.

    bias / scale may be None (0 / 1). Same contract as the reference (kernels.py:53-67), fp32 only."""
    _need(h, "h")
    _need(o, "o")
    if h.shape != o.shape:
        raise ValueError("h and o must have the same shape")
    c = h.shape[-1]
    for name, t in (("bias", bias), ("scale", scale), ("gamma", gamma), ("beta", beta)):
        if t is None and name in ("gamma", "beta"):
            raise ValueError(f"{name} is required")
        if t is not None and (_need(t, name).numel() != c):
            raise ValueError(f"{name} must have {c} elements")
    rows = h.numel() // c if c else 0
    h_out = torch.empty_like(h)
    y = torch.empty_like(h)
    call("ko_residual_layernorm", h.data_ptr(), o.data_ptr(), _ptr(bias), _ptr(scale), gamma.data_ptr(),
         beta.data_ptr(), float(eps), rows, c, h_out.data_ptr(), y.data_ptr(), _stream())
    return h_out, y


def layernorm(x, gamma, beta, eps, act=None, out=None):
    """act(LayerNorm(x) * gamma + beta) over the last dimension (C % 4 == 0, C <= 1024), act None or 'silu'.
    The plain mx.fast.layer_norm of the reference (model.py:80-82); with 'silu', the projector's channel
    LayerNorm + SiLU (model.py:157-158) in one pass."""
    _need(x, "x")
    c = x.shape[-1]
    for name, t in (("gamma", gamma), ("beta", beta)):
        if _need(t, name).numel() != c:
            raise ValueError(f"{name} must have {c} elements")
    if act not in (None, "none", "silu"):
        raise ValueError("act must be None or 'silu'")
    if out is None:
        out = torch.empty_like(x)
    call("ko_layernorm", x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), float(eps), x.numel() // c if c else 0, c,
         _lib.KO_ACT_SILU if act == "silu" else _lib.KO_ACT_NONE, out.data_ptr(), _stream())
    return out


def window_merge_layernorm(h, grid_hw, win, out, col_off, gamma=None, beta=None, eps=1e-6, normalize=True):
    """Writes the backbone's window-ordered tokens h [B*nwin, 1 + win*win, C] (class token first) as an NHWC
    image into channels [col_off, col_off + C) of out [B, H, W, ldo], LayerNorm'd over C when normalize is set:
    the window merge (model.py:104-105), the tapped layers' final LayerNorm (model.py:101-103) and the projector's
    channel concatenation (model.py:161) in one pass. Returns out."""
    _need(h, "h")
    _need(out, "out")
    gh, gw = grid_hw
    nwin = (gh // win) * (gw // win)
    n, lw, c = h.shape
    if lw != 1 + win * win or n % nwin != 0:
        raise ValueError(f"h must be [B * {nwin}, {1 + win * win}, C]")
    b = n // nwin
    if out.dim() != 4 or tuple(out.shape[:3]) != (b, gh, gw):
        raise ValueError(f"out must be [{b}, {gh}, {gw}, channels]")
    if normalize:
        if gamma is None or beta is None:
            raise ValueError("gamma and beta are required to normalize")
        for name, t in (("gamma", gamma), ("beta", beta)):
            if _need(t, name).numel() != c:
                raise ValueError(f"{name} must have {c} elements")
    call("ko_window_merge_ln", h.data_ptr(), _ptr(gamma), _ptr(beta), float(eps), b, gh, gw, win, c,
         1 if normalize else 0, out.data_ptr(), out.shape[-1], col_off, _stream())
    return out


def window_partition_layernorm(t, pos, cls, win, gamma, beta, eps=1e-6, h=None, y=None):
    """The backbone's entry in one pass: t [B, H, W, C] (patch embedding) plus pos [H, W, C], cut into win x win
    windows each led by the class token cls [C] -> (h [B*nwin, 1 + win*win, C], LayerNorm(h)) — the pos add,
    window partition and concatenation of model.py:88-90 and the first LayerNorm of model.py:94."""
    for a, n in ((t, "t"), (pos, "pos"), (cls, "cls"), (gamma, "gamma"), (beta, "beta")):
        _need(a, n)
    if t.dim() != 4:
        raise ValueError("t must be [B, H, W, C]")
    b, gh, gw, c = t.shape
    if tuple(pos.shape) != (gh, gw, c) or cls.numel() != c:
        raise ValueError("pos must be [H, W, C] and cls [C]")
    if gamma.numel() != c or beta.numel() != c:
        raise ValueError(f"gamma and beta must have {c} elements")
    if gh % win or gw % win:
        raise ValueError("H and W must be multiples of win")
    shape = (b * (gh // win) * (gw // win), 1 + win * win, c)
    h = torch.empty(shape, dtype=torch.float32, device=t.device) if h is None else h
    y = torch.empty(shape, dtype=torch.float32, device=t.device) if y is None else y
    _need(h, "h")
    _need(y, "y")
    if tuple(h.shape) != shape or tuple(y.shape) != shape:
        raise ValueError(f"h and y must be {list(shape)}")
    call("ko_window_partition_ln", t.data_ptr(), pos.data_ptr(), cls.data_ptr(), gamma.data_ptr(),
         beta.data_ptr(), float(eps), b, gh, gw, win, c, h.data_ptr(), y.data_ptr(), _stream())
    return h, y


def im2col3x3(x, out=None):
    """x: float32 NHWC [B, H, W, C] -> [B*H*W, 9*C], the im2col of a 3x3 / stride 1 / padding 1 convolution in the
    column order of a [out][3][3][in] weight (the projector's mx.conv2d, model.py:154-156, as a GEMM operand)."""
    _need(x, "x")
    if x.dim() != 4:
        raise ValueError("x must be [B, H, W, C]")
    b, h, w, c = x.shape
    if out is None:
        out = torch.empty((b * h * w, 9 * c), dtype=torch.float32, device=x.device)
    call("ko_im2col3x3", x.data_ptr(), b, h, w, c, out.data_ptr(), _stream())
    return out


# ---- preprocessing ----
def preprocess_gpu(img_u8, xtab, ytab, lut, mode, dst=640, layout="hwc", out=None):
    """img_u8: uint8 [H, W, 3] (row-contiguous) CUDA tensor. Returns float32 [dst, dst, 3] normalised RGB
    (layout 'hwc', as the reference), or [3, dst, dst] ('chw') or [(dst/16)^2, 768] ('patch16')."""
    return preprocess_batch([(img_u8, xtab, ytab, mode)], lut, dst, layout, out=out)[0]


def preprocess_batch(items, lut, dst=640, layout="hwc", out=None):
    """items: list of (img_u8 [H,W,3], xtab, ytab, mode) of any sizes; one launch per 64 images.

    Returns float32 [N, ...] in `layout` (written into `out` when given)."""
    if layout not in LAYOUTS:
        raise ValueError(f"layout must be one of {sorted(LAYOUTS)}")
    _need(lut, "lut")
    n = len(items)
    shape = {"hwc": (n, dst, dst, 3), "chw": (n, 3, dst, dst), "patch16": (n, (dst // 16) ** 2, 768)}[layout]
    if out is None:
        out = torch.empty(shape, dtype=torch.float32, device=lut.device)
    elif tuple(out.shape) != shape or out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous float32 tensor of shape {shape}")
    for start in range(0, n, 64):
        chunk = items[start:start + 64]
        descs = (_lib.ImageDesc * len(chunk))()
        for d, (img, xt, yt, mode) in zip(descs, chunk):
            _need(img, "img_u8", torch.uint8)
            _need(xt, "xtab", torch.int32)
            _need(yt, "ytab", torch.int32)
            if img.dim() != 3 or img.shape[2] != 3:
                raise ValueError("expected a uint8 BGR image of shape (H, W, 3)")
            if xt.numel() != dst * 3 * 4 or yt.numel() != dst * 4:
                raise ValueError("tables do not match dst")
            d.src, d.xtab, d.ytab = img.data_ptr(), xt.data_ptr(), yt.data_ptr()
            d.src_h, d.src_w, d.src_stride = img.shape[0], img.shape[1], img.shape[1] * 3
            d.mode = int(mode)
        call("ko_preprocess_batch", descs, len(chunk), lut.data_ptr(), dst, LAYOUTS[layout],
             out[start].data_ptr(), _stream())
    return out


# ---- deformable sampling ----
def deform_attn(value, loc, aw, grid_hw, nh, hd, offset=0):
    """value [B, H*W, ROW] with this layer's heads at columns [offset, offset + nh*hd); loc [B, NQ, NH, NP, 2]
    normalised x, y; aw [B, NQ, NH, NP]. Returns [B, NQ, NH*HD] float32 (kernels.py:165-181)."""
    _need(value, "value")
    loc = _need(loc.contiguous() if loc.dtype == torch.float32 else loc.float().contiguous(), "loc")
    aw = _need(aw.contiguous() if aw.dtype == torch.float32 else aw.float().contiguous(), "aw")
    b, n_tok, row = value.shape
    nq, npts = loc.shape[1], loc.shape[-2]
    gh, gw = grid_hw
    if n_tok != gh * gw or loc.numel() != b * nq * nh * npts * 2 or aw.numel() != b * nq * nh * npts:
        raise ValueError("deform_attn: inconsistent shapes")
    out = torch.empty((b, nq, nh * hd), dtype=torch.float32, device=value.device)
    call("ko_deform_attn", value.data_ptr(), loc.data_ptr(), aw.data_ptr(), b, nq, nh, hd, npts, gh, gw, row,
         offset, out.data_ptr(), _stream())
    return out


def deform_prep(oa, ref, nh, npts):
    """oa [B, NQ, >= NH*NP*3] (sampling offsets, then attention logits), ref [B, NQ, 4] -> (loc [B, NQ, NH, NP, 2],
    aw [B, NQ, NH, NP]): the location arithmetic and point softmax of model.py:222-225 in one launch."""
    _need(oa, "oa")
    _need(ref, "ref")
    b, nq, w = oa.shape
    if tuple(ref.shape) != (b, nq, 4) or w < nh * npts * 3:
        raise ValueError("deform_prep: oa must be [B, NQ, >= NH*NP*3] and ref [B, NQ, 4]")
    loc = torch.empty((b, nq, nh, npts, 2), dtype=torch.float32, device=oa.device)
    aw = torch.empty((b, nq, nh, npts), dtype=torch.float32, device=oa.device)
    call("ko_deform_prep", oa.data_ptr(), ref.data_ptr(), b, nq, nh, npts, w, loc.data_ptr(), aw.data_ptr(),
         _stream())
    return loc, aw


# ---- multi-head attention ----
def attention(q, k, v, heads, scale, out=None):
    """softmax(scale * q k^T) v for every head, fp32 grade (the 3xTF32 tcgen05 flash kernel; the reference uses
    mx.fast.scaled_dot_product_attention, model.py:110, :119-120, :238).

    q, k, v: [B, L, heads * head_dim] float32 CUDA tensors (head_dim 32 or 64) whose last dimension is contiguous
    — column slices of one fused QKV projection need no copy. Returns [B, L, heads * head_dim] contiguous, or
    writes `out` (same shape, last dimension contiguous)."""
    for name, t in (("q", q), ("k", k), ("v", v)):
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor (there is no CPU path)")
        if t.dtype != torch.float32 or t.dim() != 3 or t.stride(2) != 1:
            raise ValueError(f"{name} must be float32 [B, L, heads*head_dim] with a contiguous last dimension")
    if k.shape != q.shape or v.shape != q.shape:
        raise ValueError("q, k and v must have the same shape")
    b, n, width = q.shape
    hd = width // heads
    if hd * heads != width or hd not in (32, 64):
        raise ValueError("head_dim = width / heads must be 32 or 64")
    if out is None:
        out = torch.empty((b, n, width), dtype=torch.float32, device=q.device)
    elif tuple(out.shape) != (b, n, width) or out.dtype != torch.float32 or out.stride(2) != 1:
        raise ValueError("out must be float32 [B, L, heads*head_dim] with a contiguous last dimension")
    call("ko_attention_f32", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), b, n, heads, hd,
         q.stride(0), q.stride(1), k.stride(0), k.stride(1), v.stride(0), v.stride(1), out.stride(0), out.stride(1),
         float(scale), status_word(q.device).data_ptr(), _stream())
    return out


# ---- 3xTF32 GEMM ----
class PackedWeight:
    """A [K, N] weight split once into tf32 hi/lo halves, transposed ([2, N, K]) for the tcgen05 GEMM."""

    __slots__ = ("packed", "k", "n", "bias", "__weakref__")

    def __init__(self, w: torch.Tensor, bias: torch.Tensor | None = None):
        _need(w, "w")
        if w.dim() != 2:
            raise ValueError("w must be [K, N]")
        self.k, self.n = w.shape
        self.packed = torch.empty((2, self.n, self.k), dtype=torch.float32, device=w.device)
        call("ko_pack_weight_tf32x3", w.data_ptr(), self.k, self.n, self.packed.data_ptr(), _stream())
        self.bias = None if bias is None else _need(bias, "bias")


def pack_weight(w, bias=None) -> PackedWeight:
    return PackedWeight(w, bias)


def linear(x, pw: PackedWeight, act=None, out=None):
    """act(x @ W + bias) for x [..., K] float32 with W pre-split (fp32-grade 3xTF32 tcgen05 GEMM)."""
    _need(x, "x")
    if x.shape[-1] != pw.k:
        raise ValueError(f"x has {x.shape[-1]} features, the weight expects {pw.k}")
    m = x.numel() // pw.k
    if out is None:
        out = torch.empty((*x.shape[:-1], pw.n), dtype=torch.float32, device=x.device)
    call("ko_linear_f32_packed", x.data_ptr(), pw.packed.data_ptr(), _ptr(pw.bias), m, pw.k, pw.n, ACTS[act],
         out.data_ptr(), status_word(x.device).data_ptr(), _stream())
    return out


def linear_add(x, pw: PackedWeight, addend, act=None, out=None):
    """act(x @ W + bias + addend) in one GEMM: addend [..., add_cols] (add_cols <= N, a multiple of 4) is added to
    the first add_cols output columns in the epilogue; its last dimension must be contiguous (any row stride, a
    multiple of 4), e.g. a column slice of a wider precomputed product. The decoder's (tgt + qpos) @ W =
    tgt @ W + qpos @ W (fast_rfdetr/model.py:251, :256) with qpos @ W computed once for all layers."""
    _need(x, "x")
    if x.shape[-1] != pw.k:
        raise ValueError(f"x has {x.shape[-1]} features, the weight expects {pw.k}")
    if not isinstance(addend, torch.Tensor) or not addend.is_cuda or addend.dtype != torch.float32 \
            or addend.dim() != 2 or addend.stride(1) != 1:
        raise ValueError("addend must be a float32 CUDA [M, add_cols] tensor with a contiguous last dimension")
    m = x.numel() // pw.k
    if addend.shape[0] != m:
        raise ValueError(f"addend has {addend.shape[0]} rows, x has {m}")
    if out is None:
        out = torch.empty((*x.shape[:-1], pw.n), dtype=torch.float32, device=x.device)
    call("ko_linear_add_f32_packed", x.data_ptr(), pw.packed.data_ptr(), _ptr(pw.bias), addend.data_ptr(),
         addend.stride(0), addend.shape[1], m, pw.k, pw.n, ACTS[act], out.data_ptr(), status_word(x.device).data_ptr(),
         _stream())
    return out


def sine_embed(ref, dim_t, out=None):
    """ref [..., 4] (cx, cy, w, h) -> [..., 512]: the sine embedding of the (y, x, w, h) coordinates with the
    frequency divisors dim_t [128] (fast_rfdetr/model.py:188-194) in one kernel."""
    _need(ref, "ref")
    _need(dim_t, "dim_t")
    if ref.shape[-1] != 4 or dim_t.numel() != 128:
        raise ValueError("ref must be [..., 4] and dim_t [128]")
    rows = ref.numel() // 4
    if out is None:
        out = torch.empty((*ref.shape[:-1], 512), dtype=torch.float32, device=ref.device)
    call("ko_sine_embed", ref.data_ptr(), dim_t.data_ptr(), rows, out.data_ptr(), _stream())
    return out


def linear_small(x, w, bias=None, act=None):
    """act(x @ w + bias) for narrow outputs (N <= 32; the 11-class and 4-wide heads) on fp32 FMA: x [..., K],
    w [K, N] row-major, bias [N] or None, act None or 'relu'."""
    _need(x, "x")
    _need(w, "w")
    k, n = w.shape
    if x.shape[-1] != k:
        raise ValueError(f"x has {x.shape[-1]} features, the weight expects {k}")
    if bias is not None and _need(bias, "bias").numel() != n:
        raise ValueError(f"bias must have {n} elements")
    if act not in (None, "none", "relu"):
        raise ValueError("act must be None or 'relu'")
    out = torch.empty((*x.shape[:-1], n), dtype=torch.float32, device=x.device)
    call("ko_linear_small_f32", x.data_ptr(), w.data_ptr(), _ptr(bias), x.numel() // k, k, n, ACTS[act],
         out.data_ptr(), _stream())
    return out


def box_head(x, w, bias, ref):
    """Boxes from the box MLP's last layer and the reference boxes: d = x @ w + bias (w [K, 4]), then
    (d0 * r2 + r0, d1 * r3 + r1, exp(d2) * r2, exp(d3) * r3) with r = ref [..., 4] (fast_rfdetr/model.py:270-272)."""
    _need(x, "x")
    _need(w, "w")
    _need(ref, "ref")
    k = w.shape[0]
    if tuple(w.shape) != (k, 4) or x.shape[-1] != k:
        raise ValueError("w must be [K, 4] and x [..., K]")
    if tuple(ref.shape) != (*x.shape[:-1], 4):
        raise ValueError("ref must be [..., 4] with the rows of x")
    if bias is not None and _need(bias, "bias").numel() != 4:
        raise ValueError("bias must have 4 elements")
    out = torch.empty((*x.shape[:-1], 4), dtype=torch.float32, device=x.device)
    call("ko_box_head_f32", x.data_ptr(), w.data_ptr(), _ptr(bias), ref.data_ptr(), x.numel() // k, k, out.data_ptr(),
         _stream())
    return out


def select_queries(logits, delta, proposals, rp_xy, rp_ewh, nq, ref=None, idx=None):
    """The reference's query selection (model.py:175-185) in one kernel: per frame the nq proposals with the
    highest class score (max over the last dimension of logits; ties by ascending index), and their reference
    boxes refined with rp_xy / rp_ewh. logits [B, NP, NC], delta [B, NP, 4], proposals [NP, 4], rp_xy and
    rp_ewh [nq, 2]. Returns (ref [B, nq, 4], idx [B, nq] int32)."""
    for name, t in (("logits", logits), ("delta", delta), ("proposals", proposals), ("rp_xy", rp_xy),
                    ("rp_ewh", rp_ewh)):
        _need(t, name)
    b, n_p, n_c = logits.shape
    if tuple(delta.shape) != (b, n_p, 4) or tuple(proposals.shape) != (n_p, 4):
        raise ValueError("delta must be [B, NP, 4] and proposals [NP, 4]")
    if tuple(rp_xy.shape) != (nq, 2) or tuple(rp_ewh.shape) != (nq, 2):
        raise ValueError("rp_xy and rp_ewh must be [nq, 2]")
    if ref is None:
        ref = torch.empty((b, nq, 4), dtype=torch.float32, device=logits.device)
    if idx is None:
        idx = torch.empty((b, nq), dtype=torch.int32, device=logits.device)
    call("ko_select_queries", logits.data_ptr(), delta.data_ptr(), proposals.data_ptr(), rp_xy.data_ptr(),
         rp_ewh.data_ptr(), b, n_p, n_c, nq, ref.data_ptr(), idx.data_ptr(), _stream())
    return ref, idx


LN_WIDTHS = (128, 192, 256, 384, 512)


def linear_residual_layernorm(x, pw: PackedWeight, gamma, beta, eps, resid=None, scale=None, act=None,
                              h_out=None, y=None, write_h=True):
    """One GEMM with the residual add and LayerNorm in its epilogue:
        h_out = resid + (x @ W + bias) * scale;   y = act(LayerNorm(h_out) * gamma + beta)
    bias is the PackedWeight's (None = 0), scale None = 1, resid None = no residual, act None or 'silu'.
    Returns (h_out, y); h_out is None when write_h is False. h_out may be resid (in place). y may be given as a
    column slice of a wider buffer (last dimension contiguous, rows any multiple of 4 floats apart). W's width
    must be one of LN_WIDTHS. Fuses the reference's out-projection / fc2 GEMM + residual_layernorm pairs
    (model.py:121-123, 129-132) and the projector's conv GEMM + LayerNorm + SiLU (model.py:148-158)."""
    _need(x, "x")
    if x.shape[-1] != pw.k:
        raise ValueError(f"x has {x.shape[-1]} features, the weight expects {pw.k}")
    n = pw.n
    if n not in LN_WIDTHS:
        raise ValueError(f"output width {n} is not one of {LN_WIDTHS}")
    for name, t in (("gamma", gamma), ("beta", beta), ("scale", scale)):
        if t is not None and _need(t, name).numel() != n:
            raise ValueError(f"{name} must have {n} elements")
    if act not in (None, "none", "silu"):
        raise ValueError("act must be None or 'silu'")
    shape = (*x.shape[:-1], n)
    if resid is not None and tuple(_need(resid, "resid").shape) != shape:
        raise ValueError(f"resid must have shape {shape}")
    m = x.numel() // pw.k
    if y is None:
        y = torch.empty(shape, dtype=torch.float32, device=x.device)
    ldy = _row_pitch(y, m, n, "y")
    if write_h and h_out is None:
        h_out = torch.empty(shape, dtype=torch.float32, device=x.device)
    call("ko_linear_residual_ln_f32_packed", x.data_ptr(), pw.packed.data_ptr(), _ptr(pw.bias), _ptr(scale),
         _ptr(resid), gamma.data_ptr(), beta.data_ptr(), float(eps), m, pw.k, n,
         _lib.KO_ACT_SILU if act == "silu" else _lib.KO_ACT_NONE, _ptr(h_out if write_h else None), y.data_ptr(),
         ldy, status_word(x.device).data_ptr(), _stream())
    return (h_out if write_h else None), y


def _row_pitch(t, rows: int, cols: int, name: str) -> int:
    """Elements between consecutive rows of t viewed as [rows, cols] (its last dimension contiguous, its rows
    evenly spaced): a dense tensor or a column slice of a wider one."""
    if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dtype != torch.float32:
        raise ValueError(f"{name} must be a float32 CUDA tensor")
    if t.dim() < 2 or t.shape[-1] != cols or t.numel() != rows * cols or t.stride(-1) != 1:
        raise ValueError(f"{name} must hold [{rows}, {cols}] with a contiguous last dimension")
    pitch = t.stride(-2)
    step = pitch
    for d in range(t.dim() - 2, -1, -1):  # every leading dimension steps by whole rows
        if t.shape[d] > 1 and t.stride(d) != step:
            raise ValueError(f"{name}: rows are not evenly spaced")
        step *= t.shape[d]
    if pitch < cols or pitch % 4:
        raise ValueError(f"{name}: row pitch {pitch} must be a multiple of 4 and at least {cols}")
    return pitch


def conv3x3_layernorm(x, pw: PackedWeight, gamma, beta, eps, act=None, out=None):
    """act(LayerNorm(conv3x3(x) + bias) * gamma + beta) for an NHWC float32 x [B, H, W, C] (C % 16 == 0): the
    3x3 / stride 1 / padding 1 convolution as an implicit GEMM (no im2col buffer) with the LayerNorm epilogue.
    pw: the weight as [9*C, N] in (ky, kx, c) row order (PackedWeight; its bias is the conv bias). Returns out,
    [B*H*W, N] (or the [B, H, W, N] channel slice of a wider NHWC buffer given as `out`). x may be a channel slice
    of a wider NHWC buffer too. The projector's conv -> channel LayerNorm -> SiLU block (model.py:148-158)."""
    if x.dim() != 4:
        raise ValueError("x must be [B, H, W, C]")
    b, h, w, c = x.shape
    ldx = _row_pitch(x, b * h * w, c, "x")
    if pw.k != 9 * c:
        raise ValueError(f"the weight has {pw.k} rows, a 3x3 convolution over {c} channels needs {9 * c}")
    if pw.n not in LN_WIDTHS:
        raise ValueError(f"output width {pw.n} is not one of {LN_WIDTHS}")
    for name, t in (("gamma", gamma), ("beta", beta)):
        if _need(t, name).numel() != pw.n:
            raise ValueError(f"{name} must have {pw.n} elements")
    if act not in (None, "none", "silu"):
        raise ValueError("act must be None or 'silu'")
    if out is None:
        out = torch.empty((b * h * w, pw.n), dtype=torch.float32, device=x.device)
    ldy = _row_pitch(out, b * h * w, pw.n, "out")
    call("ko_conv3x3_ln_f32_packed", x.data_ptr(), ldx, pw.packed.data_ptr(), _ptr(pw.bias), gamma.data_ptr(),
         beta.data_ptr(), float(eps), b, h, w, c, pw.n, _lib.KO_ACT_SILU if act == "silu" else _lib.KO_ACT_NONE,
         out.data_ptr(), ldy, status_word(x.device).data_ptr(), _stream())
    return out


_pack_cache: "weakref.WeakKeyDictionary[torch.Tensor, tuple[int, PackedWeight]]" = weakref.WeakKeyDictionary()
_pack_lock = threading.Lock()


def linear_gelu_f32(x, w, bias):
    """GELU(x @ w + bias) for float32 x [..., K], w [K, N], bias [N] (kernels.py:271-285).

    The split of w is cached per weight tensor (and redone if the tensor is modified in place). A new split is
    complete before it enters the cache, so callers on other streams can use it at once. During CUDA graph
    capture a missing split is recorded into the graph for this call only and not cached: it holds data only
    once the graph replays, so an eager call must not find it."""
    _need(x, "x")
    _need(w, "w")
    _need(bias, "bias")
    with _pack_lock:
        hit = _pack_cache.get(w)
        if hit is None or hit[0] != w._version:
            if torch.cuda.is_current_stream_capturing():
                pw = PackedWeight(w)                  # part of the captured graph; lives as long as this call
            else:
                hit = (w._version, PackedWeight(w))
                torch.cuda.current_stream().synchronize()
                _pack_cache[w] = hit
                pw = hit[1]
        else:
            pw = hit[1]
    m = x.numel() // pw.k
    out = torch.empty((*x.shape[:-1], pw.n), dtype=torch.float32, device=x.device)
    call("ko_linear_f32_packed", x.data_ptr(), pw.packed.data_ptr(), bias.data_ptr(), m, pw.k, pw.n,
         _lib.KO_ACT_GELU, out.data_ptr(), status_word(x.device).data_ptr(), _stream())
    return out
