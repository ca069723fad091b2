"""fast_rfdetr.weights: the weight key schema and the fixed encoder proposals (fast_rfdetr/weights.py:81-88), from
kernelopt_b200.weights (ONNX extraction is not available here; see kernelopt_b200.detector.load_weights)."""
from kernelopt_b200.weights import BB, DEC, LAYER, PROJ, load, proposals, random_weights, save

__all__ = ["BB", "LAYER", "PROJ", "DEC", "proposals", "random_weights", "save", "load"]
