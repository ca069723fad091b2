"""fast_rfdetr.detector: FastBasketballDetector and load_weights (fast_rfdetr/detector.py:40, :59) and the module
constants the reference exports, from kernelopt_b200.detector."""
from kernelopt_b200.detector import INPUT, MAX_BATCH, MEAN, STD, FastBasketballDetector, load_weights

__all__ = ["FastBasketballDetector", "load_weights", "MEAN", "STD", "INPUT", "MAX_BATCH"]
