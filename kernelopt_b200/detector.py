"""FastBasketballDetector on B200: the reference's public API (fast_rfdetr/detector.py) over libkernelopt.

    det = FastBasketballDetector(model_path)            # weights file; see load_weights
    boxes, logits = det.raw(frame_bgr)                  # [1,300,4], [1,300,11] float32 numpy
    boxes, logits = det.raw_batch([frame, crop, crop])  # up to 3 images of any sizes

Differences from the reference, all additive: `device`, `resize_policy` ("reference" = the reference's cv2
model, "opencv" = bit-exact with cv2 builds without KleidiCV) and `cuda_graphs` keyword arguments, and
`detect_batch` for larger batches (the reference caps raw_batch at 3, detector.py:97-98).

Execution: each instance owns a CUDA stream and one CUDA graph per batch size (the analogue of the
reference's mx.compile per warm-up batch size). A module-level lock serialises graph capture and launch
(detector.py:29-32); waiting for the GPU happens outside it, so two instances on two threads overlap on the GPU
and return bitwise the same results as one thread (all kernels are deterministic: no float atomics).
"""
from __future__ import annotations

import hashlib
import threading
from pathlib import Path

import numpy as np
import torch

from . import kernels as K
from . import weights as W
from .model import RFDETR
from .resize_tables import tables

MEAN = np.asarray([.485, .456, .406], dtype=np.float32)
STD = np.asarray([.229, .224, .225], dtype=np.float32)
INPUT = 640
MAX_BATCH = 3
PRECISIONS = ("fp32",)

_GPU_LOCK = threading.Lock()


def _file_sha256(path: Path) -> str:
    with path.open("rb") as f:
        return hashlib.file_digest(f, "sha256").hexdigest()


def load_weights(model_path: str | Path, cache_dir: str | Path | None = None) -> dict[str, np.ndarray]:
    """Weights as {name: ndarray} in the reference's key schema (detector.py:40-56).

    model_path may be
      * "random:<seed>"           seeded random-init weights (weights.random_weights)
      * "random-varied:<seed>"    the same with non-identity biases, norms, layer scales and proposal mask
                                  (weights.random_weights(seed, varied=True))
      * a .safetensors file       e.g. the reference's own cache, mlx-cache/<digest>/weights.safetensors
      * an .onnx file             read through the reference's cache layout: <cache_dir or
                                  model_dir/mlx-cache/<sha256[:20]>>/weights.safetensors must exist (extracting
                                  from ONNX itself needs the `onnx` package, which this environment lacks)."""
    s = str(model_path)
    if s.startswith("random:"):
        return W.random_weights(int(s.split(":", 1)[1] or 0))
    if s.startswith("random-varied:"):
        return W.random_weights(int(s.split(":", 1)[1] or 0), varied=True)
    path = Path(model_path)
    if path.suffix == ".safetensors":
        return W.load(path)
    if path.suffix == ".onnx":
        digest = _file_sha256(path)[:20]
        cache = Path(cache_dir) if cache_dir else path.parent / "mlx-cache" / digest
        cached = cache / "weights.safetensors"
        if cached.exists():
            return W.load(cached)
        raise RuntimeError(f"no weight cache at {cached}; extracting weights from an ONNX file needs the `onnx` "
                           "package (run the reference once to create the cache, or pass a .safetensors file)")
    raise ValueError(f"unsupported model file {model_path!r} (expected .safetensors, .onnx or 'random:<seed>')")


class _GraphRunner:
    """Static input/output buffers and one captured forward for a fixed batch size."""

    def __init__(self, model: RFDETR, batch: int, stream: torch.cuda.Stream, use_graph: bool):
        dev = model.device
        self.model = model
        self.x = torch.zeros((batch, 1600, 768), dtype=torch.float32, device=dev)
        self.graph = None
        with torch.cuda.stream(stream):
            self.boxes, self.logits = model(self.x)                      # eager warm-up (also loads kernels)
        stream.synchronize()
        if use_graph:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream, capture_error_mode="thread_local"):
                self.boxes, self.logits = model(self.x)
            self.graph = g

    def run(self):
        if self.graph is not None:
            self.graph.replay()
        else:
            self.boxes, self.logits = self.model(self.x)
        return self.boxes, self.logits


class FastBasketballDetector:
    def __init__(self, model_path: str, precision: str = "fp32", warmup_batch_sizes=(1,), cache_dir=None, *,
                 device: str | torch.device | None = None, resize_policy: str = "reference",
                 cuda_graphs: bool = True):
        """model_path: see load_weights. warmup_batch_sizes: batch sizes captured and run once now."""
        if precision not in PRECISIONS:
            raise ValueError(f"precision must be one of {list(PRECISIONS)}")
        if not torch.cuda.is_available():
            raise RuntimeError("FastBasketballDetector needs a CUDA (sm_100) device; there is no CPU path")
        self.precision = precision
        self.resize_policy = resize_policy
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.cuda_graphs = cuda_graphs
        with _GPU_LOCK, torch.cuda.device(self.device):
            self.model = RFDETR(load_weights(model_path, cache_dir), self.device)
            lut = (np.arange(256, dtype=np.float32)[:, None] / 255. - MEAN) / STD   # same float32 ops as Ballform
            self._lut = torch.from_numpy(np.ascontiguousarray(lut.T)).to(self.device)
            # The weight splits were launched on this thread's current stream; the instance's own stream is
            # non-blocking and would not wait for them.
            torch.cuda.current_stream(self.device).synchronize()
            self.stream = torch.cuda.Stream(self.device)
        self._tables: dict[tuple[int, int], tuple[int, torch.Tensor, torch.Tensor]] = {}
        self._runners: dict[int, _GraphRunner] = {}
        dummy = np.zeros((1080, 1920, 3), np.uint8)
        for b in warmup_batch_sizes:
            self.detect_batch([dummy] * b)

    def _taps(self, w: int, h: int):
        key = (w, h)
        if key not in self._tables:
            mode, xt, yt = tables(w, h, INPUT, INPUT, self.resize_policy)
            self._tables[key] = (mode, torch.from_numpy(np.array(xt)).to(self.device),
                                 torch.from_numpy(np.array(yt)).to(self.device))
        return self._tables[key]

    @staticmethod
    def _check_image(image_bgr) -> np.ndarray:
        if not isinstance(image_bgr, np.ndarray) or image_bgr.dtype != np.uint8 or image_bgr.ndim != 3 \
                or image_bgr.shape[2] != 3:
            raise ValueError("expected a uint8 BGR image of shape (H, W, 3)")
        return np.ascontiguousarray(image_bgr)

    def _preprocess(self, image_bgr: np.ndarray) -> torch.Tensor:
        """float32 [640, 640, 3] normalised RGB on the device (the reference's _preprocess, detector.py:84-89)."""
        img = self._check_image(image_bgr)
        h, w, _ = img.shape
        mode, xt, yt = self._taps(w, h)
        with torch.cuda.device(self.device), torch.cuda.stream(self.stream):
            out = K.preprocess_gpu(torch.from_numpy(img).to(self.device, non_blocking=False), xt, yt, self._lut, mode,
                                   INPUT)
        self.stream.synchronize()
        return out

    def _runner(self, b: int) -> _GraphRunner:
        if b not in self._runners:
            self._runners[b] = _GraphRunner(self.model, b, self.stream, self.cuda_graphs)
        return self._runners[b]

    def raw(self, image_bgr: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
        """Returns (boxes [1,300,4] f32, logits [1,300,11] f32), the same as the ONNX outputs."""
        return self.raw_batch([image_bgr])

    def raw_batch(self, images: list[np.ndarray]) -> tuple[np.ndarray, np.ndarray]:
        """Images of any sizes (each resized to 640x640). Returns boxes [N,300,4], logits [N,300,11]."""
        if not 1 <= len(images) <= MAX_BATCH:
            raise ValueError(f"batch size must be 1..{MAX_BATCH}")
        return self.detect_batch(images)

    def detect_batch(self, images: list[np.ndarray]) -> tuple[np.ndarray, np.ndarray]:
        """raw_batch without the batch cap of 3 (one CUDA graph per distinct batch size)."""
        if len(images) < 1:
            raise ValueError("need at least one image")
        imgs = [self._check_image(im) for im in images]
        with _GPU_LOCK, torch.cuda.device(self.device), torch.cuda.stream(self.stream):
            runner = self._runner(len(imgs))
            items = []
            for img in imgs:
                h, w, _ = img.shape
                mode, xt, yt = self._taps(w, h)
                src = torch.from_numpy(img).pin_memory().to(self.device, non_blocking=True)
                items.append((src, xt, yt, mode))
            K.preprocess_batch(items, self._lut, INPUT, "patch16", out=runner.x)
            boxes, logits = runner.run()
            hb = torch.empty(boxes.shape, dtype=torch.float32, pin_memory=True)
            hl = torch.empty(logits.shape, dtype=torch.float32, pin_memory=True)
            hb.copy_(boxes, non_blocking=True)
            hl.copy_(logits, non_blocking=True)
            done = torch.cuda.Event()
            done.record(self.stream)
            keep = items  # device copies of the frames must live until the stream has consumed them
        done.synchronize()
        del keep
        K.check_device_status(self.device)
        return hb.numpy().copy(), hl.numpy().copy()

    def detect_stream(self, batches):
        """Pipelined detection over a stream of frame batches (a video decoder's output): yields
        (boxes [N,300,4], logits [N,300,11]) numpy arrays for each uint8 tensor [N, H, W, 3] of `batches`, in order.

        All batches must have one shape; host tensors should be pinned. The host-to-device copy of batch i+1 runs
        on its own stream while batch i is preprocessed and run on this instance's stream, and the outputs of
        batch i come back on a third stream (device-to-device into a slot buffer, then to pinned host memory)
        while batch i+1 computes.
        Two slots of device frames and outputs alternate; events order every reuse. Results are identical to
        detect_frames on the same batch."""
        it = iter(batches)
        first = next(it, None)
        if first is None:
            return
        if first.dtype != torch.uint8 or first.dim() != 4 or first.shape[-1] != 3:
            raise ValueError("frames must be a uint8 tensor of shape (N, H, W, 3)")
        shape = tuple(first.shape)
        n, h, w, _ = shape
        with _GPU_LOCK, torch.cuda.device(self.device):
            runner = self._runner(n)
            mode, xt, yt = self._taps(w, h)
            h2d = torch.cuda.Stream(self.device)   # copies in; never waits for compute of earlier batches
            d2h = torch.cuda.Stream(self.device)   # copies out; waits for each batch's compute
            dev = [torch.empty(shape, dtype=torch.uint8, device=self.device) for _ in range(2)]
            out_dev = [(torch.empty_like(runner.boxes), torch.empty_like(runner.logits)) for _ in range(2)]
            out_host = [(torch.empty(runner.boxes.shape, dtype=torch.float32, pin_memory=True),
                         torch.empty(runner.logits.shape, dtype=torch.float32, pin_memory=True)) for _ in range(2)]
            ev = {k: [torch.cuda.Event() for _ in range(2)] for k in ("h2d", "free", "comp", "d2h")}
        used = [False, False]
        keep = [None, None]  # host batches stay referenced until their copy has certainly completed

        def enqueue(i: int, frames: torch.Tensor):
            if tuple(frames.shape) != shape or frames.dtype != torch.uint8:
                raise ValueError("every batch of a stream must have the first batch's shape and dtype")
            s = i & 1
            with _GPU_LOCK, torch.cuda.device(self.device):
                with torch.cuda.stream(h2d):
                    if used[s]:
                        h2d.wait_event(ev["free"][s])           # the slot's previous frames were preprocessed
                    dev[s].copy_(frames, non_blocking=True)
                    ev["h2d"][s].record(h2d)
                    keep[s] = frames
                with torch.cuda.stream(self.stream):
                    self.stream.wait_event(ev["h2d"][s])
                    K.preprocess_batch([(dev[s][k], xt, yt, mode) for k in range(n)], self._lut, INPUT, "patch16",
                                       out=runner.x)
                    ev["free"][s].record(self.stream)
                    boxes, logits = runner.run()
                    if used[s]:
                        self.stream.wait_event(ev["d2h"][s])     # the slot's previous outputs reached the host
                    out_dev[s][0].copy_(boxes)
                    out_dev[s][1].copy_(logits)
                    ev["comp"][s].record(self.stream)
                with torch.cuda.stream(d2h):
                    d2h.wait_event(ev["comp"][s])
                    out_host[s][0].copy_(out_dev[s][0], non_blocking=True)
                    out_host[s][1].copy_(out_dev[s][1], non_blocking=True)
                    ev["d2h"][s].record(d2h)
                used[s] = True

        def collect(i: int):
            s = i & 1
            ev["d2h"][s].synchronize()
            keep[s] = None
            K.check_device_status(self.device)
            return out_host[s][0].numpy().copy(), out_host[s][1].numpy().copy()

        try:
            enqueue(0, first)
            i = 0
            for frames in it:
                enqueue(i + 1, frames)
                yield collect(i)
                i += 1
            yield collect(i)
        finally:
            # A consumer that stops early (break, an exception) must not free the slot buffers while copies or
            # preprocessing that use them are still queued: the caching allocator would hand them out again.
            h2d.synchronize()
            self.stream.synchronize()
            d2h.synchronize()

    def detect_frames(self, frames: torch.Tensor) -> tuple[np.ndarray, np.ndarray]:
        """Frames already in a uint8 tensor [N, H, W, 3] (one size), ideally in pinned host memory (a video
        decoder's output buffer) or on this device. One H2D copy, preprocessing, the captured forward and one
        D2H copy of the outputs, all on this instance's stream. Returns boxes [N,300,4], logits [N,300,11]."""
        if frames.dtype != torch.uint8 or frames.dim() != 4 or frames.shape[-1] != 3:
            raise ValueError("frames must be a uint8 tensor of shape (N, H, W, 3)")
        n, h, w, _ = frames.shape
        with _GPU_LOCK, torch.cuda.device(self.device), torch.cuda.stream(self.stream):
            runner = self._runner(n)
            mode, xt, yt = self._taps(w, h)
            dev = frames if frames.device == self.device else frames.to(self.device, non_blocking=True)
            K.preprocess_batch([(dev[i], xt, yt, mode) for i in range(n)], self._lut, INPUT, "patch16", out=runner.x)
            boxes, logits = runner.run()
            hb = torch.empty(boxes.shape, dtype=torch.float32, pin_memory=True)
            hl = torch.empty(logits.shape, dtype=torch.float32, pin_memory=True)
            hb.copy_(boxes, non_blocking=True)
            hl.copy_(logits, non_blocking=True)
            done = torch.cuda.Event()
            done.record(self.stream)
        done.synchronize()
        del dev
        K.check_device_status(self.device)
        return hb.numpy(), hl.numpy()
