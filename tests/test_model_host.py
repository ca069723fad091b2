"""Host-side wiring of the GPU model graph (kernelopt_b200.model) on the CPU: the kernel layer is replaced by
float64 torch fakes (test doubles of the CUDA calls), so windowing, head splits, im2col ordering, the fused
value projection and the decoder plumbing are checked against the oracle's unfused graph without a GPU."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle.kernels as OKn
import oracle.resize as OR
from kernelopt_b200.weights import random_weights
from oracle.model import OracleRFDETR


class _Packed:
    def __init__(self, w, b=None):
        self.w, self.b = w, b
        self.k, self.n = w.shape


def _linear(x, pw, act=None, out=None):
    y = x @ pw.w
    if pw.b is not None:
        y = y + pw.b
    if act == "gelu":
        y = 0.5 * y * (1 + torch.erf(y / math.sqrt(2)))
    elif act == "relu":
        y = torch.relu(y)
    return y


def _rln(h, o, bias, scale, g, b, eps):
    ho = h + (o + (0 if bias is None else bias)) * (1 if scale is None else scale)
    return ho, F.layer_norm(ho, (ho.shape[-1],), g, b, eps)


def _deform(value, loc, aw, grid_hw, nh, hd, offset=0):
    return torch.from_numpy(OKn.deform_attn(value.numpy(), loc.numpy(), aw.numpy(), grid_hw, nh, hd, offset))


def _attention(q, k, v, heads, scale, out=None):
    b, n, w = q.shape
    hd = w // heads
    qh, kh, vh = (t.reshape(b, n, heads, hd).transpose(1, 2) for t in (q, k, v))
    p = torch.softmax((qh @ kh.transpose(-1, -2)) * scale, dim=-1)
    return (p @ vh).transpose(1, 2).reshape(b, n, w)


def _layernorm(x, g, b, eps, act=None, out=None):
    y = F.layer_norm(x, (x.shape[-1],), g, b, eps)
    return F.silu(y) if act == "silu" else y


def _lrln(x, pw, gamma, beta, eps, resid=None, scale=None, act=None, h_out=None, y=None, write_h=True):
    o = _linear(x, pw)
    ho = (0 if resid is None else resid) + o * (1 if scale is None else scale)
    yy = F.layer_norm(ho, (ho.shape[-1],), gamma, beta, eps)
    yy = F.silu(yy) if act == "silu" else yy
    if y is not None:                     # written into the caller's buffer (possibly a channel slice)
        y.copy_(yy.reshape(y.shape))
        yy = y
    return (ho if write_h else None), yy


def _linear_add(x, pw, addend, act=None, out=None):
    y = x @ pw.w + (0 if pw.b is None else pw.b)
    y = y.reshape(-1, pw.n)
    y = torch.cat([y[:, :addend.shape[1]] + addend, y[:, addend.shape[1]:]], 1)
    return _linear(y.reshape(*x.shape[:-1], pw.n), _Packed(torch.eye(pw.n, dtype=y.dtype)), act)


def _sine_embed(ref, dim_t, out=None):
    outs = []
    for c in (1, 0, 2, 3):
        v = (ref[..., c] * (2 * math.pi))[..., None] / dim_t
        outs.append(torch.stack([torch.sin(v[..., 0::2]), torch.cos(v[..., 1::2])], -1).reshape(*v.shape[:-1], 128))
    return torch.cat(outs, -1)


def _linear_small(x, w, bias=None, act=None):
    return _linear(x, _Packed(w, bias), act)


def _box_head(x, w, bias, ref):
    d = x @ w + bias
    return torch.cat([d[..., :2] * ref[..., 2:] + ref[..., :2], torch.exp(d[..., 2:]) * ref[..., 2:]], -1)


def _select(logits, delta, prop, rp_xy, rp_ewh, nq, ref=None, idx=None):
    scores = logits.amax(-1)
    coord = torch.cat([delta[..., :2] * prop[:, 2:] + prop[:, :2], torch.exp(delta[..., 2:]) * prop[:, 2:]], -1)
    i = torch.from_numpy(np.argsort(-scores.numpy(), axis=-1, kind="stable")[:, :nq].copy())
    ts = torch.gather(coord, 1, i[..., None].expand(-1, -1, 4))
    return torch.cat([rp_xy * ts[..., 2:] + ts[..., :2], rp_ewh * ts[..., 2:]], -1), i


def _conv3x3_ln(x, pw, gamma, beta, eps, act=None, out=None):
    return _lrln(_im2col3x3(x), pw, gamma, beta, eps, act=act, y=out, write_h=False)[1]


def _window_merge(h, grid_hw, win, out, col_off, gamma=None, beta=None, eps=1e-6, normalize=True):
    gh, gw = grid_hw
    nwin = (gh // win) * (gw // win)
    b = h.shape[0] // nwin
    c = h.shape[-1]
    v = F.layer_norm(h, (c,), gamma, beta, eps) if normalize else h
    img = v[:, 1:].reshape(b, gh // win, gw // win, win, win, c).permute(0, 1, 3, 2, 4, 5).reshape(b, gh, gw, c)
    out[..., col_off:col_off + c] = img
    return out


def _window_partition(t, pos, cls, win, gamma, beta, eps=1e-6, h=None, y=None):
    b, gh, gw, c = t.shape
    v = (t + pos).reshape(b, gh // win, win, gw // win, win, c).permute(0, 1, 3, 2, 4, 5)
    v = v.reshape(-1, win * win, c)
    hh = torch.cat([cls.reshape(1, 1, c).expand(v.shape[0], 1, c), v], 1)
    return hh, F.layer_norm(hh, (c,), gamma, beta, eps)


def _deform_prep(oa, ref, nh, npts):
    b, nq, _ = oa.shape
    off = oa[..., :nh * npts * 2].reshape(b, nq, nh, npts, 2)
    aw = torch.softmax(oa[..., nh * npts * 2:nh * npts * 3].reshape(b, nq, nh, npts), -1)
    r = ref[:, :, None, None, :]
    return r[..., :2] + off / npts * r[..., 2:] * 0.5, aw


def _im2col3x3(x, out=None):
    b, h, w, c = x.shape
    xp = F.pad(x, (0, 0, 1, 1, 1, 1))
    return torch.cat([xp[:, dy:dy + h, dx:dx + w] for dy in range(3) for dx in range(3)], -1).reshape(b * h * w, 9 * c)


@pytest.fixture()
def cpu_model(monkeypatch):
    import kernelopt_b200.kernels as K
    import kernelopt_b200.model as M
    monkeypatch.setattr(K, "pack_weight", lambda w, b=None: _Packed(w, b))
    monkeypatch.setattr(K, "linear", _linear)
    monkeypatch.setattr(K, "residual_layernorm", _rln)
    monkeypatch.setattr(K, "deform_attn", _deform)
    monkeypatch.setattr(K, "attention", _attention)
    monkeypatch.setattr(K, "layernorm", _layernorm)
    monkeypatch.setattr(K, "im2col3x3", _im2col3x3)
    monkeypatch.setattr(K, "linear_residual_layernorm", _lrln)
    monkeypatch.setattr(K, "select_queries", _select)
    monkeypatch.setattr(K, "conv3x3_layernorm", _conv3x3_ln)
    monkeypatch.setattr(K, "window_merge_layernorm", _window_merge)
    monkeypatch.setattr(K, "window_partition_layernorm", _window_partition)
    monkeypatch.setattr(K, "deform_prep", _deform_prep)
    monkeypatch.setattr(K, "linear_add", _linear_add)
    monkeypatch.setattr(K, "sine_embed", _sine_embed)
    monkeypatch.setattr(K, "linear_small", _linear_small)
    monkeypatch.setattr(K, "box_head", _box_head)
    monkeypatch.setattr(K, "status_word", lambda *a: None)
    w = random_weights(0)

    class CPUModel(M.RFDETR):
        def __init__(self, weights):
            self.device = torch.device("cpu")
            self.eps = {k[5:]: float(np.asarray(v).reshape(())) for k, v in weights.items() if k.startswith("_eps.")}
            self.p = {k: torch.from_numpy(np.ascontiguousarray(v.T if k.endswith("self_attn.out_proj.weight") else v))
                      .double() for k, v in weights.items() if not k.startswith("_eps.")}
            self._prepare()

    return CPUModel(w), OracleRFDETR(w, torch.float64)


def test_model_graph_matches_oracle(cpu_model):
    model, orc = cpu_model
    img = np.random.default_rng(1).integers(0, 256, (720, 1280, 3), dtype=np.uint8)
    x = torch.from_numpy(OR.preprocess(img))[None].double()
    patches = torch.from_numpy(OR.preprocess(img, layout="patch16"))[None].double()
    b1, l1 = model(patches)
    b2, l2 = orc(x)
    assert (b1 - b2).abs().max() < 1e-9 and (l1 - l2).abs().max() < 1e-9
    b3, l3 = model(x)                     # NHWC input is accepted too
    assert (b3 - b2).abs().max() < 1e-9 and (l3 - l2).abs().max() < 1e-9
