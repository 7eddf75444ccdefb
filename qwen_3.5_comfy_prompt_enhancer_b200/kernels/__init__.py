"""Drop-in replacements for the reference engine's ``kernels`` package entry
points on the quantised-linear hot path (``gemm.py``, ``w4.py``) plus the
activation quantiser they consume (``norm.quant_row``)."""
