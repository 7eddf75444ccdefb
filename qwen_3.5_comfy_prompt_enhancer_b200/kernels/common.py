"""Constants shared with the reference engine (kernels/common.py:5-9)."""

# Activation quantisation granularity along K: one fp32 scale per 64 int8
# activations.  Every GEMM consumes activations on this grid.
GROUP = 64


def next_pow2(n):
    """Smallest power of two >= n (kernels/common.py:57-58)."""
    return 1 << max(0, (n - 1)).bit_length()
