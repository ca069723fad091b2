"""The reference's import path, `fast_rfdetr`, served by kernelopt_b200 (the B200 implementation).

A caller of the reference switches by putting this repository on sys.path in place of the reference's package;
its imports stay as they are (fast_rfdetr/__init__.py:2-4, fast_rfdetr/model.py:9):

    from fast_rfdetr import FastBasketballDetector, load_weights
    from fast_rfdetr.kernels import residual_layernorm, linear_gelu_f32, deform_attn, preprocess_gpu
    from fast_rfdetr.resize_tables import tables, uses_kleidicv

Every name resolves to the kernelopt_b200 object itself (not a copy), so both import paths share one library,
one set of caches and one device status word. The detector (and torch) load on first use, as in kernelopt_b200.
"""
__all__ = ["FastBasketballDetector", "load_weights"]


def __getattr__(name):
    if name in __all__:
        from . import detector
        return getattr(detector, name)
    raise AttributeError(name)
