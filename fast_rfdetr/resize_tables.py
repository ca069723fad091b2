"""fast_rfdetr.resize_tables: `tables` and `uses_kleidicv` (fast_rfdetr/resize_tables.py:41, :165), from
kernelopt_b200.resize_tables (computed by the native table generator)."""
from kernelopt_b200.resize_tables import tables, uses_kleidicv

__all__ = ["tables", "uses_kleidicv"]
