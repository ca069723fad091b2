"""CPU oracle of the RF-DETR-Medium hot path — TEST INFRASTRUCTURE ONLY.

This package restates the reference's algorithms (ishaanzee/kernelopt, fast_rfdetr/) on the CPU so that the
CUDA kernels can be checked against them. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs
import it; the product package kernelopt_b200 never does, and never falls back to it.

    oracle.resize   numpy restatement of the cv2.resize table model and its evaluation + normalisation
                    (fast_rfdetr/resize_tables.py, kernels.py:74-103, detector.py:70-71).
                    PINNED: golden tables and output digests generated from the reference's own
                    resize_tables.py (tests/golden/make_golden.py), and cv2.resize on this machine.
    oracle.kernels  float64 numpy restatements of residual+LayerNorm, GEMM+bias+GELU and deformable sampling
                    (model.py unfused path). Parity unpinned at the MLX boundary: MLX (the reference's
                    runtime) cannot be installed here and the reference ships no golden vectors for these
                    kernels; the restatements are cross-checked against torch's independent CPU operators.
    oracle.model    torch-CPU restatement of RFDETR.__call__ with the reference's unfused semantics
                    (model.py:84-272), in float32 (the timed CPU baseline) or float64 (the parity checker).
                    Parity unpinned at the MLX boundary, for the same reason.
"""
