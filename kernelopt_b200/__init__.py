"""B200-native (sm_100a) RF-DETR-Medium inference hot path: a drop-in for the reference's fast_rfdetr package.

Exports the reference's public API (fast_rfdetr/__init__.py:2-4). The detector module (and torch) load on
first use, so the table generator and the C ABI can be used without them.
"""
__all__ = ["FastBasketballDetector", "load_weights"]


def __getattr__(name):
    if name in __all__:
        from . import detector
        return getattr(detector, name)
    raise AttributeError(name)
