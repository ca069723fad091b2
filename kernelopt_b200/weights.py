"""RF-DETR-Medium weights as a flat {name: np.ndarray} dict in the reference's key schema.

The reference extracts this dict from Ballform's ONNX export (fast_rfdetr/weights.py:23-78) and caches it as
safetensors (detector.py:40-56). Neither the ONNX model nor the `onnx` package exists here, so this module
provides what the rest of the path needs:

  * `random_weights(seed)`  seeded random-init weights with the exact keys, shapes and conventions the model
    reads (linear weights [in, out] for x @ W; convs [out, kh, kw, in]; LayerNorm eps under "_eps.<key>").
    Init: truncated normal (std 0.02, cut at 2 std) for every weight matrix, conv kernel and embedding;
    biases 0; LayerNorm gamma 1, beta 0; layer-scale lambdas 1.0; decoder FFN width 2048 (the RF-DETR default,
    not pinned by the reference). LayerNorm eps: 1e-6 in the backbone and projector, 1e-5 in the transformer.
    `random_weights(seed, varied=True)` exercises every parameter the init above leaves at an identity value:
    biases ~ 0.02 * tn, LayerNorm gamma ~ 1 + 0.1 * tn and beta ~ 0.05 * tn, layer-scale lambdas ~ 1 + 0.2 * tn
    (tn: standard normal cut at 2), and a proposal mask with the four corner proposals marked invalid (the
    reference's proposals are all valid, fast_rfdetr/weights.py:81-88; the model still multiplies by the mask,
    model.py:177).
  * `proposals()`  the fixed 40x40 encoder proposals and validity mask (fast_rfdetr/weights.py:81-88).
  * `save` / `load`  safetensors files with the same schema — including the reference's own weight cache
    (mlx-cache/<digest>/weights.safetensors), which therefore loads here unchanged.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

BB = "backbone.0.encoder.encoder."
LAYER = BB + "encoder.layer.{}."
PROJ = "backbone.0.projector.stages.0."
DEC = "transformer.decoder."
C, MLP, D_MODEL, FFN, N_CLASSES, N_QUERIES = 384, 1536, 256, 2048, 11, 300
CA_HEADS, CA_POINTS = 16, 2


def proposals(h: int = 40, w: int = 40) -> dict[str, np.ndarray]:
    """Fixed cxcywh anchors at the patch centres (wh = 0.05) and their validity mask (all inside (0.01, 0.99))."""
    ys, xs = np.meshgrid(np.arange(h, dtype=np.float32), np.arange(w, dtype=np.float32), indexing="ij")
    cxcy = (np.stack([xs, ys], -1).reshape(-1, 2) + 0.5) / np.asarray([w, h], np.float32)
    boxes = np.concatenate([cxcy, np.full_like(cxcy, 0.05)], -1).astype(np.float32)
    valid = np.all((boxes > 0.01) & (boxes < 0.99), axis=-1, keepdims=True).astype(np.float32)
    return {"proposals": boxes, "proposal_valid": valid}


def dim_t(n: int = 128, temperature: float = 10000.0) -> np.ndarray:
    """Sine-embedding frequency divisors: temperature ** (2 * (i // 2) / n)."""
    i = np.arange(n, dtype=np.float32)
    return (temperature ** (2 * (i // 2) / n)).astype(np.float32)


def random_weights(seed: int = 0, varied: bool = False) -> dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    # the varied parameters come from a second stream, so the weight matrices equal those of varied=False
    vrng = np.random.default_rng([seed, 1]) if varied else None
    w: dict[str, np.ndarray] = {}

    def tn(*shape, std=0.02):
        return np.clip(rng.standard_normal(shape), -2.0, 2.0).astype(np.float32) * np.float32(std)

    def around(n, centre, std):
        if vrng is None:
            return np.full(n, centre, np.float32)
        return (np.float32(centre) + np.clip(vrng.standard_normal(n), -2.0, 2.0).astype(np.float32)
                * np.float32(std)).astype(np.float32)

    def bias(n):
        return around(n, 0.0, 0.02)

    def scale(n):
        return around(n, 1.0, 0.2)

    def lin(key, n_in, n_out, with_bias=True):
        w[key + ".weight"] = tn(n_in, n_out)
        if with_bias:
            w[key + ".bias"] = bias(n_out)

    def ln(key, n, eps):
        w[key + ".weight"] = around(n, 1.0, 0.1)
        w[key + ".bias"] = around(n, 0.0, 0.05)
        w["_eps." + key + ".weight"] = np.asarray(eps, np.float32)

    # backbone (DINOv2-small style windowed ViT)
    w[BB + "embeddings.cls_token"] = tn(1, 1, C)
    w[BB + "embeddings.position_embeddings"] = tn(1, 1601, C)
    w[BB + "embeddings.patch_embeddings.projection.weight"] = tn(C, 16, 16, 3)
    w[BB + "embeddings.patch_embeddings.projection.bias"] = bias(C)
    for i in range(12):
        pre = LAYER.format(i)
        ln(pre + "norm1", C, 1e-6)
        for n in ("query", "key", "value"):
            lin(pre + "attention.attention." + n, C, C)
        lin(pre + "attention.output.dense", C, C)
        w[pre + "layer_scale1.lambda1"] = scale(C)
        ln(pre + "norm2", C, 1e-6)
        lin(pre + "mlp.fc1", C, MLP)
        lin(pre + "mlp.fc2", MLP, C)
        w[pre + "layer_scale2.lambda1"] = scale(C)
    ln(BB + "layernorm", C, 1e-6)

    # projector: C2f with 3 bottlenecks, channel LayerNorm + SiLU after every conv
    def convx(key, c_in, c_out, k):
        w[key + ".conv.weight"] = tn(c_out, k, k, c_in)
        ln(key + ".bn", c_out, 1e-6)

    convx(PROJ + "0.cv1", 4 * C, 2 * 128, 1)
    for j in range(3):
        convx(PROJ + f"0.m.{j}.cv1", 128, 128, 3)
        convx(PROJ + f"0.m.{j}.cv2", 128, 128, 3)
    convx(PROJ + "0.cv2", 5 * 128, D_MODEL, 1)
    ln(PROJ + "1", D_MODEL, 1e-6)

    # two-stage query selection
    w.update(proposals())
    if varied:
        w["proposal_valid"] = w["proposal_valid"].copy()
        w["proposal_valid"][[0, 39, 1560, 1599]] = 0.0
    lin("transformer.enc_output.0", D_MODEL, D_MODEL)
    ln("transformer.enc_output_norm.0", D_MODEL, 1e-5)
    lin("transformer.enc_out_class_embed.0", D_MODEL, N_CLASSES)
    for j, n_out in enumerate((D_MODEL, D_MODEL, 4)):
        lin(f"transformer.enc_out_bbox_embed.0.layers.{j}", D_MODEL, n_out)
    w["refpoint_embed"] = tn(N_QUERIES, 4)
    w["query_feat"] = tn(N_QUERIES, D_MODEL)
    w["dim_t"] = dim_t()

    # decoder
    lin(DEC + "ref_point_head.layers.0", 2 * D_MODEL, D_MODEL)
    lin(DEC + "ref_point_head.layers.1", D_MODEL, D_MODEL)
    for i in range(4):
        pre = DEC + f"layers.{i}."
        for n in ("q", "k", "v"):
            lin(pre + "self_attn." + n, D_MODEL, D_MODEL)
        w[pre + "self_attn.out_proj.weight"] = tn(D_MODEL, D_MODEL)  # stored [out, in] (ONNX Gemm transB=1)
        w[pre + "self_attn.out_proj.bias"] = bias(D_MODEL)
        ln(pre + "norm1", D_MODEL, 1e-5)
        lin(pre + "cross_attn.sampling_offsets", D_MODEL, CA_HEADS * CA_POINTS * 2)
        lin(pre + "cross_attn.attention_weights", D_MODEL, CA_HEADS * CA_POINTS)
        lin(pre + "cross_attn.value_proj", D_MODEL, D_MODEL)
        lin(pre + "cross_attn.output_proj", D_MODEL, D_MODEL)
        ln(pre + "norm2", D_MODEL, 1e-5)
        lin(pre + "linear1", D_MODEL, FFN)
        lin(pre + "linear2", FFN, D_MODEL)
        ln(pre + "norm3", D_MODEL, 1e-5)
    ln(DEC + "norm", D_MODEL, 1e-5)

    # heads
    lin("class_embed", D_MODEL, N_CLASSES)
    for j, n_out in enumerate((D_MODEL, D_MODEL, 4)):
        lin(f"bbox_embed.layers.{j}", D_MODEL, n_out)
    return {k: np.ascontiguousarray(v) for k, v in w.items()}


def save(weights: dict[str, np.ndarray], path: str | Path) -> None:
    """Atomic safetensors write (tmp file + rename), as the reference's cache does (detector.py:52-55)."""
    from safetensors.numpy import save_file
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(".tmp.safetensors")
    save_file({k: np.ascontiguousarray(v) for k, v in weights.items()}, str(tmp))
    tmp.replace(path)


def load(path: str | Path) -> dict[str, np.ndarray]:
    from safetensors.numpy import load_file
    return {k: np.asarray(v) for k, v in load_file(str(path)).items()}
