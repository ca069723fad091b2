"""fast_rfdetr.model: the RFDETR forward (fast_rfdetr/model.py:26) and its layout constants, from kernelopt_b200.model."""
from kernelopt_b200.model import C, FULL_ATTN, GRID, HEADS, RFDETR, SA_HEADS, TAPS, WIN, D_MODEL

__all__ = ["RFDETR", "FULL_ATTN", "TAPS", "GRID", "WIN", "C", "HEADS", "D_MODEL", "SA_HEADS"]
