"""B200-native (sm_100a) quantised-linear hot path of a Qwen3.5 hybrid engine.

Drop-in for the reference engine's ``kernels/gemm.py`` and ``kernels/w4.py``
entry points, the activation producers of ``kernels/norm.py`` and the decode /
prefill neighbours of ``kernels/attention.py`` and ``kernels/linear_attn.py``:
the same names and signatures, backed
by hand-written CUDA in ``libqlin.so`` behind the C ABI of ``include/qlin.h``.

The directory name contains a dot, so import it through
``__graft_entry__.load_package()`` (registers it as ``qwen35_b200``) or any
other importlib alias; all imports inside the package are relative.
"""
from . import _lib, decode_step, tp  # noqa: F401
from .kernels.attention import attn_decode, attn_prefill, qk_norm_rope  # noqa: F401
from .kernels.common import GROUP  # noqa: F401
from .kernels.linear_attn import (conv_silu, conv_silu_update, conv_state_update, delta_decode,  # noqa: F401
                                  delta_prefill)
from .kernels.gemm import gemm_i8, mlp_gate_up, mlp_gate_up_quant, proj3  # noqa: F401
from .kernels.norm import (gate_mul_quant, gate_proj, norm_gated, norm_gated_quant, quant_row,  # noqa: F401
                           rmsnorm_quant, silu_mul_quant)
from .kernels.w4 import gemm_w4, mlp_gate_up_quant_w4, proj3_w4  # noqa: F401

__all__ = ["GROUP", "gemm_i8", "mlp_gate_up", "mlp_gate_up_quant", "proj3", "gemm_w4",
           "proj3_w4", "mlp_gate_up_quant_w4", "quant_row", "rmsnorm_quant", "norm_gated_quant", "norm_gated",
           "gate_mul_quant", "silu_mul_quant", "gate_proj", "qk_norm_rope", "attn_decode", "conv_silu",
           "conv_state_update", "conv_silu_update", "delta_decode", "attn_prefill", "delta_prefill"]
