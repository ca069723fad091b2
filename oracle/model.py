"""CPU oracle (test infrastructure): RF-DETR-Medium forward on torch CPU with the reference's UNFUSED semantics.

Restates fast_rfdetr/model.py with fused=False: backbone vit_layer (:134-145), attention (:107-111), projector
(:148-167), select_queries (:175-185), sine_embed (:188-194), grid_sample (:196-216), cross_attn (:218-230,
unfused branch), self_attn (:232-239), decoder (:241-259), heads (:261-272). No custom kernels, no fused value
projection, no head-major QKV: each op as the reference's plain path writes it.

dtype=torch.float64 is the parity checker; dtype=torch.float32 with all host threads is the timed CPU baseline
(a stand-in for "plain MLX on MLX's Linux CPU backend", which cannot be installed here).
Parity unpinned at the MLX boundary.
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

BB = "backbone.0.encoder.encoder."
LAYER = BB + "encoder.layer.{}."
PROJ = "backbone.0.projector.stages.0."
DEC = "transformer.decoder."
FULL_ATTN = (3, 6, 9)
TAPS = (2, 5, 8, 11)
GRID, WIN, C, HEADS = 40, 20, 384, 6
D_MODEL, CA_HEADS, CA_POINTS, SA_HEADS = 256, 16, 2, 8


class OracleRFDETR:
    def __init__(self, weights: dict[str, np.ndarray], dtype=torch.float64):
        self.dtype = dtype
        self.eps = {k[5:]: float(np.asarray(v).reshape(())) for k, v in weights.items() if k.startswith("_eps.")}
        p = {}
        for k, v in weights.items():
            if k.startswith("_eps."):
                continue
            if k.endswith("self_attn.out_proj.weight"):
                v = v.T
            p[k] = torch.from_numpy(np.ascontiguousarray(v)).to(dtype)
        for i in range(12):
            pre = LAYER.format(i) + "attention.attention."
            p[f"_qkv{i}.w"] = torch.cat([p[pre + n + ".weight"] for n in ("query", "key", "value")], 1)
            p[f"_qkv{i}.b"] = torch.cat([p[pre + n + ".bias"] for n in ("query", "key", "value")])
        pos = p[BB + "embeddings.position_embeddings"][0]
        p["_cls"] = (p[BB + "embeddings.cls_token"][0, 0] + pos[0]).reshape(1, 1, C)
        p["_pos"] = pos[1:].reshape(1, GRID, GRID, C)
        self.p = p

    def lin(self, x, key):
        y = x @ self.p[key + ".weight"]
        b = self.p.get(key + ".bias")
        return y if b is None else y + b

    def ln(self, x, key):
        return F.layer_norm(x, (x.shape[-1],), self.p[key + ".weight"], self.p[key + ".bias"], self.eps[key + ".weight"])

    @staticmethod
    def conv_nhwc(x, w, padding):
        """x NHWC, w [out, kh, kw, in] (the reference's MLX layout) -> NHWC."""
        y = F.conv2d(x.permute(0, 3, 1, 2), w.permute(0, 3, 1, 2), padding=padding)
        return y.permute(0, 2, 3, 1)

    # backbone (model.py:84-111, 134-145)
    def backbone(self, x):
        p, b = self.p, x.shape[0]
        w = p[BB + "embeddings.patch_embeddings.projection.weight"]
        t = F.conv2d(x.permute(0, 3, 1, 2), w.permute(0, 3, 1, 2), stride=16).permute(0, 2, 3, 1)
        t = t + p[BB + "embeddings.patch_embeddings.projection.bias"] + p["_pos"]
        t = t.reshape(b, 2, WIN, 2, WIN, C).permute(0, 1, 3, 2, 4, 5).reshape(b * 4, WIN * WIN, C)
        h = torch.cat([p["_cls"].expand(b * 4, 1, C), t], 1)
        feats = []
        for i in range(12):
            h = self.vit_layer(i, h, b)
            if i in TAPS:
                feats.append(self.ln(h, BB + "layernorm"))
        return [f[:, 1:].reshape(b, 2, 2, WIN, WIN, C).permute(0, 1, 3, 2, 4, 5).reshape(b, GRID, GRID, C)
                for f in feats]

    def attention(self, i, qkv, n, L, b):
        qkv = qkv.reshape(b, 4 * L, 3, HEADS, C // HEADS) if i in FULL_ATTN else qkv.reshape(n, L, 3, HEADS, C // HEADS)
        qkv = qkv.permute(2, 0, 3, 1, 4)
        o = F.scaled_dot_product_attention(qkv[0], qkv[1], qkv[2], scale=1 / math.sqrt(C // HEADS))
        return o.permute(0, 2, 1, 3).reshape(n, L, C)

    def vit_layer(self, i, h, b):
        pre = LAYER.format(i)
        n, L, _ = h.shape
        y = self.ln(h, pre + "norm1")
        o = self.attention(i, y @ self.p[f"_qkv{i}.w"] + self.p[f"_qkv{i}.b"], n, L, b)
        o = self.lin(o, pre + "attention.output.dense")
        h = h + o * self.p[pre + "layer_scale1.lambda1"]
        y = self.ln(h, pre + "norm2")
        y = self.lin(y, pre + "mlp.fc1")
        y = 0.5 * y * (1 + torch.erf(y / math.sqrt(2)))
        y = self.lin(y, pre + "mlp.fc2")
        return h + y * self.p[pre + "layer_scale2.lambda1"]

    # projector (model.py:148-167)
    def convx(self, x, key):
        w = self.p[key + ".conv.weight"]
        y = self.conv_nhwc(x, w, w.shape[1] // 2)
        y = self.ln(y, key + ".bn")
        return y * torch.sigmoid(y)

    def projector(self, feats):
        pre = PROJ + "0."
        y = self.convx(torch.cat(feats, -1), pre + "cv1")
        parts = [y[..., :128], y[..., 128:]]
        for j in range(3):
            parts.append(self.convx(self.convx(parts[-1], pre + f"m.{j}.cv1"), pre + f"m.{j}.cv2"))
        y = self.convx(torch.cat(parts, -1), pre + "cv2")
        return self.ln(y, PROJ + "1")

    # query selection (model.py:170-185)
    def mlp3(self, x, key):
        x = torch.relu(self.lin(x, key + ".layers.0"))
        x = torch.relu(self.lin(x, key + ".layers.1"))
        return self.lin(x, key + ".layers.2")

    def select_queries(self, memory):
        p = self.p
        om = memory * p["proposal_valid"]
        om = self.ln(self.lin(om, "transformer.enc_output.0"), "transformer.enc_output_norm.0")
        scores = self.lin(om, "transformer.enc_out_class_embed.0").amax(-1)
        delta = self.mlp3(om, "transformer.enc_out_bbox_embed.0")
        prop = p["proposals"]
        coord = torch.cat([delta[..., :2] * prop[:, 2:] + prop[:, :2], torch.exp(delta[..., 2:]) * prop[:, 2:]], -1)
        idx = torch.argsort(-scores, dim=-1, stable=True)[:, :300]
        ts = torch.gather(coord, 1, idx[..., None].expand(-1, -1, 4))
        rp = p["refpoint_embed"]
        ref = torch.cat([rp[:, :2] * ts[..., 2:] + ts[..., :2], torch.exp(rp[:, 2:]) * ts[..., 2:]], -1)
        return ref, scores, idx

    # decoder (model.py:188-259)
    def sine_embed(self, ref):
        dim_t = self.p["dim_t"]
        outs = []
        for c in (1, 0, 2, 3):
            v = (ref[..., c] * (2 * math.pi))[..., None] / dim_t
            outs.append(torch.stack([torch.sin(v[..., 0::2]), torch.cos(v[..., 1::2])], -1).reshape(*v.shape[:2], 128))
        return torch.cat(outs, -1)

    def grid_sample(self, value, loc):
        """value [B,1600,16,16]; loc [B,300,16,P,2] -> [B,300,16,P,16] (zero padding, align_corners=False)."""
        b = value.shape[0]
        v = value.permute(0, 2, 1, 3).reshape(b * CA_HEADS * GRID * GRID, D_MODEL // CA_HEADS)
        loc = loc.permute(0, 2, 1, 3, 4)
        x = loc[..., 0] * GRID - 0.5
        y = loc[..., 1] * GRID - 0.5
        x0, y0 = torch.floor(x), torch.floor(y)
        fx, fy = x - x0, y - y0
        base = (torch.arange(b * CA_HEADS) * (GRID * GRID)).reshape(b, CA_HEADS, 1, 1)
        out = 0
        for dy, wy in ((0, 1 - fy), (1, fy)):
            for dx, wx in ((0, 1 - fx), (1, fx)):
                xi, yi = x0 + dx, y0 + dy
                ok = (xi >= 0) & (xi < GRID) & (yi >= 0) & (yi < GRID)
                idx = base + (yi.clamp(0, GRID - 1) * GRID + xi.clamp(0, GRID - 1)).long()
                g = v[idx.reshape(-1)].reshape(*idx.shape, -1)
                out = out + g * torch.where(ok, wx * wy, torch.zeros_like(wx))[..., None]
        return out.permute(0, 2, 1, 3, 4)

    def cross_attn(self, q, ref, value, key):
        b, nq, _ = q.shape
        off = self.lin(q, key + ".sampling_offsets").reshape(b, nq, CA_HEADS, CA_POINTS, 2)
        aw = torch.softmax(self.lin(q, key + ".attention_weights").reshape(b, nq, CA_HEADS, CA_POINTS), -1)
        r = ref[:, :, None, None, :]
        loc = r[..., :2] + off / CA_POINTS * r[..., 2:] * 0.5
        s = self.grid_sample(value, loc)
        o = (s * aw[..., None]).sum(3).reshape(b, nq, D_MODEL)
        return self.lin(o, key + ".output_proj")

    def self_attn(self, qk, v, key):
        b, n, _ = qk.shape
        hd = D_MODEL // SA_HEADS
        q = self.lin(qk, key + ".q").reshape(b, n, SA_HEADS, hd).transpose(1, 2)
        k = self.lin(qk, key + ".k").reshape(b, n, SA_HEADS, hd).transpose(1, 2)
        v = self.lin(v, key + ".v").reshape(b, n, SA_HEADS, hd).transpose(1, 2)
        o = F.scaled_dot_product_attention(q, k, v, scale=1 / math.sqrt(hd))
        return self.lin(o.transpose(1, 2).reshape(b, n, D_MODEL), key + ".out_proj")

    def decoder(self, memory, ref):
        p = self.p
        b = memory.shape[0]
        emb = self.sine_embed(ref)
        qpos = self.lin(torch.relu(self.lin(emb, DEC + "ref_point_head.layers.0")), DEC + "ref_point_head.layers.1")
        tgt = p["query_feat"].expand(b, 300, D_MODEL)
        for i in range(4):
            pre = DEC + f"layers.{i}."
            tgt = self.ln(tgt + self.self_attn(tgt + qpos, tgt, pre + "self_attn"), pre + "norm1")
            value = self.lin(memory, pre + "cross_attn.value_proj").reshape(b, GRID * GRID, CA_HEADS, D_MODEL // CA_HEADS)
            tgt = self.ln(tgt + self.cross_attn(tgt + qpos, ref, value, pre + "cross_attn"), pre + "norm2")
            ffn = self.lin(torch.relu(self.lin(tgt, pre + "linear1")), pre + "linear2")
            tgt = self.ln(tgt + ffn, pre + "norm3")
        return self.ln(tgt, DEC + "norm")

    @torch.no_grad()
    def forward(self, x, return_selection: bool = False):
        """x [B,640,640,3] normalised RGB (NHWC). Returns (boxes [B,300,4], logits [B,300,11])."""
        x = torch.as_tensor(x).to(self.dtype)
        b = x.shape[0]
        memory = self.projector(self.backbone(x)).reshape(b, GRID * GRID, D_MODEL)
        ref, scores, idx = self.select_queries(memory)
        hs = self.decoder(memory, ref)
        logits = self.lin(hs, "class_embed")
        delta = self.mlp3(hs, "bbox_embed")
        boxes = torch.cat([delta[..., :2] * ref[..., 2:] + ref[..., :2], torch.exp(delta[..., 2:]) * ref[..., 2:]], -1)
        if return_selection:
            return boxes, logits, scores, idx
        return boxes, logits

    __call__ = forward
