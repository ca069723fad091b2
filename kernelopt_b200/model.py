"""RF-DETR-Medium forward pass on B200: the reference's graph (fast_rfdetr/model.py) in torch CUDA ops, with
the hot path on libkernelopt's sm_100a kernels.

Call sites of the reference's kernels (model.py:122, 125, 131, 226) use the same kernels here:
  residual_layernorm   after the attention out-projection and after fc2 (24 calls per frame) — here inside the
                       epilogue of those two GEMMs (ko_linear_residual_ln: the reference's listed next step); the
                       decoder's post-norms LN(tgt + linear(x)), the projector's conv GEMM -> LN -> SiLU and the
                       encoder-output linear + LN run through the same fused kernel
  linear_gelu_f32      backbone fc1 (the 3xTF32 tcgen05 GEMM with the GELU epilogue)
  deform_attn          decoder cross-attention sampling, on the one fused [B,1600,1024] value projection
Every other dense layer (QKV, out-proj, fc2, the patch embedding, the projector's 1x1 convs, the decoder
linears) runs on the same fp32-grade tcgen05 GEMM. The projector's 3x3 convs run on it as an implicit GEMM with
LayerNorm + SiLU in the epilogue, and its C2f concatenation is written in place (each block's output lands in its
channel slice of one buffer). The heads' 11- and 4-wide outputs run on a narrow fp32 kernel, the box refinement
fused into the last box layer. Attention — the backbone's windowed and global self-attention and the decoder's
self-attention (the reference's mx.fast.scaled_dot_product_attention) — runs on the fp32-grade 3xTF32 tcgen05
flash-attention kernel, straight on column slices of the fused QKV projection, softmax included. The backbone's
entry (pos add, windows, class token, first LayerNorm) and each tapped layer's merge + LayerNorm are one kernel
each. The top-300 query selection is one kernel, and so are the sine embedding and the sampler's input step
(locations + point softmax). The decoder's `tgt + qpos` (model.py:251, :256) becomes tgt @ W + qpos @ W: one GEMM
per forward computes qpos @ W for all four layers and each layer's GEMM adds its slice in the epilogue.

The input is the patch layout the preprocessing kernel writes (PATCH16: [B, 1600, 768]), which makes the
16x16/16 patch-embedding convolution one GEMM; NHWC [B, 640, 640, 3] (the reference's input) is accepted too.
Everything is shape-static, so a whole forward is captured in one CUDA graph per batch size (detector.py).
"""
from __future__ import annotations

import math

import numpy as np
import torch

from . import kernels as K
from .weights import BB, CA_HEADS, CA_POINTS, DEC, LAYER, PROJ

FULL_ATTN = (3, 6, 9)
TAPS = (2, 5, 8, 11)
GRID, WIN, C, HEADS = 40, 20, 384, 6
D_MODEL, SA_HEADS, N_QUERIES = 256, 8, 300


def configure_numerics() -> None:
    """fp32 everywhere: no TF32 in torch matmul/cuDNN (single-pass TF32 reorders the top-300 ranking)."""
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    torch.set_float32_matmul_precision("highest")


class Dense:
    """A linear layer x @ W + b: the tcgen05 3xTF32 GEMM when the widths are multiples of 4, the narrow-output
    fp32 kernel (ko_linear_small_f32) for the heads' 11- and 4-wide outputs."""

    def __init__(self, w: torch.Tensor, b: torch.Tensor | None):
        self.k, self.n = w.shape
        self.native = self.n % 4 == 0 and self.k % 4 == 0
        self.w, self.b = w.contiguous(), (None if b is None else b.contiguous())
        if self.native:
            self.pw = K.pack_weight(self.w, self.b)
        elif not (self.n <= 32 and self.k * self.n <= 12288):
            raise ValueError(f"no kernel for a {self.k} x {self.n} linear layer")

    def ln(self, x: torch.Tensor, ln, resid=None, scale=None, act=None, write_h=None):
        """(h_out, y) with h_out = resid + (x @ W + b) * scale and y = act(LayerNorm(h_out)): one GEMM whose
        epilogue does the residual add and the LayerNorm when the output width allows it (ko_linear_residual_ln),
        else the GEMM and then the LayerNorm kernel. h_out is returned only when there is a residual."""
        w, b, eps = ln
        if write_h is None:
            write_h = resid is not None
        # Fused at every size, K > 512 included: its correction accumulator leaves TMEM for one accumulator
        # buffer, so the epilogue does not overlap the next tile's MMAs, but the separate LayerNorm pass goes
        # (fc2 at 102 656 rows: 572 us fused against 588 us for the GEMM + LayerNorm pair on B200; over the
        # whole 64-frame step 41.50 against 41.68 ms).
        if self.native and self.n in K.LN_WIDTHS:
            return K.linear_residual_layernorm(x.contiguous(), self.pw, w, b, eps, resid=resid, scale=scale,
                                               act=act, write_h=write_h)
        o = self(x)
        if resid is None and scale is None:
            return None, K.layernorm(o.contiguous(), w, b, eps, act)
        h = torch.zeros_like(o) if resid is None else resid
        h_out, y = K.residual_layernorm(h.contiguous(), o.contiguous(), None, scale, w, b, eps)
        return h_out, (K.layernorm(h_out, w, b, eps, act) if act else y)

    def __call__(self, x: torch.Tensor, act=None, addend=None) -> torch.Tensor:
        """act(x @ W + b [+ addend on the first addend.shape[-1] columns])."""
        if addend is not None:
            return K.linear_add(x.contiguous(), self.pw, addend, act)
        if self.native:
            return K.linear(x.contiguous(), self.pw, act)
        return K.linear_small(x.contiguous(), self.w, self.b, act)


class RFDETR:
    def __init__(self, weights: dict[str, np.ndarray], device: torch.device | str = "cuda"):
        configure_numerics()
        self.device = torch.device(device)
        dev = self.device
        self.eps = {k[5:]: float(np.asarray(v).reshape(())) for k, v in weights.items() if k.startswith("_eps.")}
        p = {}
        for k, v in weights.items():
            if k.startswith("_eps."):
                continue
            if k.endswith("self_attn.out_proj.weight"):  # stored [out, in]
                v = v.T
            p[k] = torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32)).to(dev)
        self.p = p
        K.status_word(dev)  # allocate before any graph capture
        self._prepare()

    # ---- parameters -------------------------------------------------------------------------------------
    def _ln(self, key):
        return self.p[key + ".weight"], self.p[key + ".bias"], self.eps[key + ".weight"]

    def _prepare(self):
        p = self.p
        pos = p[BB + "embeddings.position_embeddings"][0]
        self.cls = (p[BB + "embeddings.cls_token"][0, 0] + pos[0]).reshape(1, 1, C)
        self.pos = pos[1:].contiguous()                                                     # [1600, C]
        pw = p[BB + "embeddings.patch_embeddings.projection.weight"]                         # [C, 16, 16, 3]
        self.patch = Dense(pw.reshape(C, 768).t().contiguous(), p[BB + "embeddings.patch_embeddings.projection.bias"])
        self.layers = []
        for i in range(12):
            pre = LAYER.format(i)
            att = pre + "attention.attention."
            wqkv = torch.cat([p[att + n + ".weight"] for n in ("query", "key", "value")], 1)
            bqkv = torch.cat([p[att + n + ".bias"] for n in ("query", "key", "value")])
            nxt = LAYER.format(i + 1) + "norm1" if i < 11 else BB + "layernorm"
            self.layers.append(dict(
                qkv=Dense(wqkv, bqkv),
                out=Dense(p[pre + "attention.output.dense.weight"], p[pre + "attention.output.dense.bias"]),
                ls1=p[pre + "layer_scale1.lambda1"],
                norm2=self._ln(pre + "norm2"),
                fc1=K.pack_weight(p[pre + "mlp.fc1.weight"], p[pre + "mlp.fc1.bias"]),
                fc2=Dense(p[pre + "mlp.fc2.weight"], p[pre + "mlp.fc2.bias"]),
                ls2=p[pre + "layer_scale2.lambda1"],
                next_norm=self._ln(nxt)))
        self.norm1_0 = self._ln(LAYER.format(0) + "norm1")
        self.final_ln = self._ln(BB + "layernorm")

        def conv(key):
            w = p[key + ".conv.weight"]                                                      # [out, kh, kw, in]
            k = w.shape[1]
            return dict(dense=Dense(w.reshape(w.shape[0], -1).t().contiguous(), None), k=k, ln=self._ln(key + ".bn"))

        self.cv1 = conv(PROJ + "0.cv1")
        self.bottlenecks = [(conv(PROJ + f"0.m.{j}.cv1"), conv(PROJ + f"0.m.{j}.cv2")) for j in range(3)]
        self.cv2 = conv(PROJ + "0.cv2")
        self.proj_ln = self._ln(PROJ + "1")

        d = lambda key: Dense(p[key + ".weight"], p.get(key + ".bias"))  # noqa: E731
        self.enc_output = d("transformer.enc_output.0")
        self.enc_norm = self._ln("transformer.enc_output_norm.0")
        self.enc_class = d("transformer.enc_out_class_embed.0")
        self.enc_bbox = [d(f"transformer.enc_out_bbox_embed.0.layers.{j}") for j in range(3)]
        self.valid = p["proposal_valid"]
        # Masked proposals (valid = 0) enter the encoder head as zero rows, whose output is the same constant row
        # for every frame: LayerNorm(enc_output(0)). It is computed once here; the per-frame mask multiply of the
        # reference (model.py:177) then becomes a copy of that row into the masked rows, and nothing at all for
        # weights whose proposals are all valid (the reference's own).
        self.masked = torch.nonzero(self.valid[:, 0] == 0)[:, 0]
        self.enc_zero_row = None
        if self.masked.numel():
            _, self.enc_zero_row = self.enc_output.ln(torch.zeros((1, D_MODEL), device=self.device), self.enc_norm)
        self.props = p["proposals"]
        rp = p["refpoint_embed"]
        self.rp_xy, self.rp_ewh = rp[:, :2].contiguous(), torch.exp(rp[:, 2:]).contiguous()
        self.dim_t = p["dim_t"]
        self.query_feat = p["query_feat"]
        self.rph = [d(DEC + f"ref_point_head.layers.{j}") for j in range(2)]
        vp = [DEC + f"layers.{i}.cross_attn.value_proj" for i in range(4)]
        self.vproj = Dense(torch.cat([p[k + ".weight"] for k in vp], 1), torch.cat([p[k + ".bias"] for k in vp]))
        # (tgt + qpos) @ W = tgt @ W + qpos @ W: qpos is the same in all four layers, so its products with each
        # layer's q | k and offset | weight projections come from one GEMM per forward ([rows, 4 * 608]), which
        # the layers' GEMMs of tgt add in their epilogues; the value projection of tgt joins the q | k GEMM.
        self.dec = []
        pos_w = []
        for i in range(4):
            pre = DEC + f"layers.{i}."
            sa = pre + "self_attn."
            wqk = torch.cat([p[sa + "q.weight"], p[sa + "k.weight"]], 1)
            wqkv = torch.cat([wqk, p[sa + "v.weight"]], 1)
            bqkv = torch.cat([p[sa + "q.bias"], p[sa + "k.bias"], p[sa + "v.bias"]])
            ca = pre + "cross_attn."
            woff = torch.cat([p[ca + "sampling_offsets.weight"], p[ca + "attention_weights.weight"]], 1)
            boff = torch.cat([p[ca + "sampling_offsets.bias"], p[ca + "attention_weights.bias"]])
            pos_w += [wqk, woff]
            self.dec.append(dict(
                qkv=Dense(wqkv, bqkv), out=d(sa + "out_proj"), norm1=self._ln(pre + "norm1"),
                offaw=Dense(woff, boff), oproj=d(ca + "output_proj"), norm2=self._ln(pre + "norm2"),
                l1=d(pre + "linear1"), l2=d(pre + "linear2"), norm3=self._ln(pre + "norm3")))
        self.pos_proj = Dense(torch.cat(pos_w, 1), None)                      # [256, 4 * (512 + 96)]
        self.pos_cols = 2 * D_MODEL + woff.shape[1]                            # 608 columns per layer
        self._tgt0: dict[int, torch.Tensor] = {}
        self.dec_norm = self._ln(DEC + "norm")
        self.class_embed = d("class_embed")
        self.bbox_embed = [d(f"bbox_embed.layers.{j}") for j in range(3)]

    # ---- backbone -----------------------------------------------------------------------------------------
    @staticmethod
    def _ln_op(x, ln, act=None):
        w, b, eps = ln
        return K.layernorm(x.contiguous(), w, b, eps, act)

    def backbone(self, patches: torch.Tensor):
        """patches [B, 1600, 768] -> the four tapped feature maps [B, 40, 40, C], concatenated along channels as
        the projector takes them: [B, 40, 40, 4C] (model.py:84-105, fused path, and the concatenation of :161).
        Each tap is written straight into its channel slice by the window-merge (+ LayerNorm) kernel."""
        b = patches.shape[0]
        t = self.patch(patches.reshape(b * GRID * GRID, 768)).reshape(b, GRID, GRID, C)
        w0, b0, eps0 = self.norm1_0        # + pos, 2 x 2 windows led by the class token, first LayerNorm: one pass
        h, y = K.window_partition_layernorm(t, self.pos.view(GRID, GRID, C), self.cls.reshape(C), WIN, w0, b0,
                                            eps0)                                               # [4B, 401, C]
        feats = h.new_empty((b, GRID, GRID, len(TAPS) * C))
        w, bt, eps = self.final_ln
        for i, lyr in enumerate(self.layers):
            h, y = self._vit_layer(i, lyr, h, y, b)
            if i in TAPS:
                k = TAPS.index(i)
                if i == 11:  # the last layer's epilogue already applied the final LayerNorm (its next norm)
                    K.window_merge_layernorm(y, (GRID, GRID), WIN, feats, k * C, normalize=False)
                else:
                    K.window_merge_layernorm(h, (GRID, GRID), WIN, feats, k * C, w, bt, eps)
        return feats

    def _vit_layer(self, i, lyr, h, y, b):
        """model.py:113-132: attention, residual+LN, fc1+GELU, fc2, residual+LN (next layer's norm1)."""
        n, L, _ = h.shape
        nb, Lb = (b, 4 * L) if i in FULL_ATTN else (n, L)                                      # global: merge windows
        qkv = lyr["qkv"](y.reshape(nb * Lb, C)).reshape(nb, Lb, 3 * C)                         # q | k | v columns
        o = K.attention(qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:], HEADS, 1 / math.sqrt(C // HEADS))
        # out-projection + bias, * layer scale, + residual, norm2: one kernel (and fc2 + next norm1 likewise)
        h, y = lyr["out"].ln(o.reshape(n, L, C), lyr["norm2"], resid=h, scale=lyr["ls1"])
        m = K.linear(y, lyr["fc1"], "gelu")
        return lyr["fc2"].ln(m, lyr["next_norm"], resid=h, scale=lyr["ls2"])

    # ---- projector ----------------------------------------------------------------------------------------
    def _convx(self, x, cv, out=None):
        """conv (1x1 as GEMM, 3x3 as implicit GEMM) + channel LayerNorm + SiLU (model.py:148-158) in one kernel.
        x may be a channel slice of a wider NHWC buffer, and `out` ([B, H, W, N], possibly such a slice) receives
        the result; returns it."""
        b, hh, ww, cin = x.shape
        dense = cv["dense"]
        w, bt, eps = cv["ln"]
        if out is None:
            out = x.new_empty((b, hh, ww, dense.n))
        if cv["k"] == 1:
            K.linear_residual_layernorm(x.reshape(b * hh * ww, cin), dense.pw, w, bt, eps, act="silu", y=out,
                                        write_h=False)
        else:
            K.conv3x3_layernorm(x, dense.pw, w, bt, eps, "silu", out=out)
        return out

    def projector(self, feats):
        """feats: the backbone's concatenated feature maps [B, 40, 40, 4C] -> [B, 40, 40, 256] (model.py:148-167).
        The C2f concatenation (model.py:161-162) is never copied: cv1 writes channels [0, 256) of one
        [B, 40, 40, 640] buffer, each bottleneck reads the previous 128-channel slice in place and writes the next
        slice, and cv2 reads the whole buffer."""
        b = feats.shape[0]
        cat = feats.new_empty((b, GRID, GRID, 128 * (2 + len(self.bottlenecks))))
        self._convx(feats, self.cv1, out=cat[..., :256])
        for j, (cv_a, cv_b) in enumerate(self.bottlenecks):
            t = self._convx(cat[..., 128 * (j + 1):128 * (j + 2)], cv_a)
            self._convx(t, cv_b, out=cat[..., 128 * (j + 2):128 * (j + 3)])
        y = self._convx(cat, self.cv2)
        return self._ln_op(y, self.proj_ln)

    # ---- query selection ------------------------------------------------------------------------------------
    def _mlp3(self, x, layers):
        x = layers[0](x, "relu")
        x = layers[1](x, "relu")
        return layers[2](x)

    def select_queries(self, memory, with_scores=True):
        """model.py:175-185: class score per proposal, box refinement, top-300 by score. The score maximum, the
        ranking (ties by ascending proposal index), the gather and the box refinement are one kernel
        (ko_select_queries). Returns (ref [B, 300, 4], scores [B, 1600] or None, idx [B, 300])."""
        _, om = self.enc_output.ln(memory, self.enc_norm)
        if self.enc_zero_row is not None:                   # masked proposals: the head's output for a zero row
            om[:, self.masked] = self.enc_zero_row
        logits = self.enc_class(om)                                                             # [B, 1600, 11]
        delta = self._mlp3(om, self.enc_bbox)                                                   # [B, 1600, 4]
        ref, idx = K.select_queries(logits.contiguous(), delta.contiguous(), self.props, self.rp_xy, self.rp_ewh,
                                    N_QUERIES)
        return ref, (logits.amax(-1) if with_scores else None), idx

    # ---- decoder ----------------------------------------------------------------------------------------------
    def sine_embed(self, ref):
        """model.py:188-194 in one kernel: [B, 300, 4] boxes -> [B, 300, 512]."""
        return K.sine_embed(ref.contiguous(), self.dim_t)

    def _query_feat(self, b: int) -> torch.Tensor:
        """query_feat broadcast over the batch: a constant, made once per batch size outside graph capture (the
        layers never write it) and made afresh inside a capture that meets a new size."""
        t = self._tgt0.get(b)
        if t is None:
            t = self.query_feat.expand(b, N_QUERIES, D_MODEL).contiguous()
            if not (t.is_cuda and torch.cuda.is_current_stream_capturing()):
                self._tgt0[b] = t
        return t

    def decoder(self, memory, ref):
        b = memory.shape[0]
        qpos = self.rph[1](self.rph[0](self.sine_embed(ref), "relu"))
        qp = self.pos_proj(qpos).reshape(b * N_QUERIES, -1)                    # qpos @ W of every layer
        tgt = self._query_feat(b)
        values = self.vproj(memory)                                                              # [B, 1600, 1024]
        hd = D_MODEL // SA_HEADS
        for i, lyr in enumerate(self.dec):
            c0 = i * self.pos_cols
            # (tgt + qpos) @ [Wq | Wk] and tgt @ Wv in one GEMM: q | k | v columns
            qkv = lyr["qkv"](tgt, addend=qp[:, c0:c0 + 2 * D_MODEL]).reshape(b, N_QUERIES, 3 * D_MODEL)
            o = K.attention(qkv[..., :D_MODEL], qkv[..., D_MODEL:2 * D_MODEL], qkv[..., 2 * D_MODEL:], SA_HEADS,
                            1 / math.sqrt(hd))
            _, tgt = lyr["out"].ln(o, lyr["norm1"], resid=tgt, write_h=False)                  # LN(tgt + out(o))
            oa = lyr["offaw"](tgt, addend=qp[:, c0 + 2 * D_MODEL:c0 + self.pos_cols])          # [B, 300, 96]
            loc, aw = K.deform_prep(oa, ref.contiguous(), CA_HEADS, CA_POINTS)  # locations + point softmax
            s = K.deform_attn(values, loc, aw, (GRID, GRID), CA_HEADS, D_MODEL // CA_HEADS, offset=i * D_MODEL)
            _, tgt = lyr["oproj"].ln(s, lyr["norm2"], resid=tgt, write_h=False)
            _, tgt = lyr["l2"].ln(lyr["l1"](tgt, "relu"), lyr["norm3"], resid=tgt, write_h=False)
        return self._ln_op(tgt, self.dec_norm)

    # ---- full forward -------------------------------------------------------------------------------------------
    def forward(self, x: torch.Tensor):
        """x: PATCH16 [B, 1600, 768] or NHWC [B, 640, 640, 3] normalised RGB.
        Returns (boxes [B,300,4] cxcywh, logits [B,300,11]) float32 (model.py:261-272)."""
        if x.dim() == 4:
            b = x.shape[0]
            x = x.reshape(b, GRID, 16, GRID, 16, 3).permute(0, 1, 3, 2, 4, 5).reshape(b, GRID * GRID, 768)
        x = x.contiguous()
        b = x.shape[0]
        feats = self.backbone(x)
        memory = self.projector(feats).reshape(b, GRID * GRID, D_MODEL)
        ref, _, _ = self.select_queries(memory, with_scores=False)
        hs = self.decoder(memory, ref)
        logits = self.class_embed(hs)
        h2 = self.bbox_embed[1](self.bbox_embed[0](hs, "relu"), "relu")
        last = self.bbox_embed[2]                                 # the last box layer + the box refinement
        boxes = K.box_head(h2, last.w, last.b, ref.contiguous())
        return boxes, logits

    __call__ = forward
