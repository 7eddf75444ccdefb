"""Host-side logic of the Python mirror: dispatch and argument validation
(no kernels are launched: every case fails before reaching the C ABI)."""
import pytest
import torch


def test_reference_names_exported(pkg):
    for name in ("gemm_i8", "mlp_gate_up", "mlp_gate_up_quant", "proj3", "gemm_w4", "proj3_w4",
                 "mlp_gate_up_quant_w4", "quant_row", "GROUP"):
        assert hasattr(pkg, name)
    assert pkg.GROUP == 64


def test_cpu_tensors_rejected(pkg):
    a = torch.zeros(1, 64, dtype=torch.int8)
    s = torch.zeros(1, 1)
    b = torch.zeros(64, 128, dtype=torch.int8)
    bs = torch.zeros(128)
    out = torch.zeros(1, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        pkg.gemm_i8(a, s, b, bs, out)


def test_w4_dispatch_on_uint8(pkg, monkeypatch):
    """uint8 weights route gemm_i8 / mlp_gate_up_quant / proj3 to the W4 entry
    points, int8 weights to the W8 ones (kernels/gemm.py:15-17, 69-72)."""
    from qwen35_b200.kernels import gemm as G
    calls = []

    class FakeExt:
        def __getattr__(self, name):
            def call(*args):
                calls.append(name)
                return 0
            return call

    monkeypatch.setattr(G._lib, "ext", lambda: FakeExt())
    b4 = torch.zeros(32, 128, dtype=torch.uint8)
    b8 = torch.zeros(64, 128, dtype=torch.int8)
    G.gemm_i8(None, None, b4, None, None)
    G.mlp_gate_up_quant(None, None, b4, None, b4, None, None, None)
    G.proj3(None, None, b4, None, None, None, None, None, None)
    G.gemm_i8(None, None, b8, None, None)
    G.mlp_gate_up_quant(None, None, b8, None, b8, None, None, None)
    G.proj3(None, None, b8, None, None, None, None, None, None)
    assert calls == ["gemm_w4", "mlp_gate_up_quant_w4", "proj3_w4", "gemm_i8", "mlp_gate_up_quant", "proj3"]


def test_block_k_must_be_group(pkg):
    a = torch.zeros(1, 64, dtype=torch.int8)
    with pytest.raises(ValueError, match="block_k"):
        pkg.gemm_i8(a, None, torch.zeros(64, 16, dtype=torch.int8), None, None, block_k=32)


def test_binding_exports_every_entry_point(pkg):
    ext = pkg._lib.ext()
    for name in ("gemm_i8", "mlp_gate_up", "mlp_gate_up_quant", "proj3", "gemm_w4", "proj3_w4",
                 "mlp_gate_up_quant_w4", "quant_row"):
        assert callable(getattr(ext, name)), name


def _cpu_calls(pkg):
    a = torch.zeros(1, 128, dtype=torch.int8)
    s = torch.zeros(1, 2)
    b8 = torch.zeros(128, 64, dtype=torch.int8)
    s8 = torch.zeros(64)
    b4 = torch.zeros(64, 64, dtype=torch.uint8)
    s4 = torch.zeros(2, 64, dtype=torch.bfloat16)
    out = torch.zeros(1, 64, dtype=torch.bfloat16)
    q = torch.zeros(1, 64, dtype=torch.int8)
    qs = torch.zeros(1, 1)
    x = torch.zeros(1, 128, dtype=torch.bfloat16)
    return {
        "gemm_i8": lambda: pkg.gemm_i8(a, s, b8, s8, out),
        "mlp_gate_up": lambda: pkg.mlp_gate_up(a, s, b8, s8, b8, s8, out),
        "mlp_gate_up_quant": lambda: pkg.mlp_gate_up_quant(a, s, b8, s8, b8, s8, q, qs),
        "proj3": lambda: pkg.proj3(a, s, b8, s8, None, None, None, None, out),
        "gemm_w4": lambda: pkg.gemm_w4(a, s, b4, s4, out),
        "proj3_w4": lambda: pkg.proj3_w4(a, s, b4, s4, None, None, None, None, out),
        "mlp_gate_up_quant_w4": lambda: pkg.mlp_gate_up_quant_w4(a, s, b4, s4, b4, s4, q, qs),
        "quant_row": lambda: pkg.quant_row(x, torch.zeros(1, 128, dtype=torch.int8), s),
    }


@pytest.mark.parametrize("name", ["gemm_i8", "mlp_gate_up", "mlp_gate_up_quant", "proj3", "gemm_w4",
                                  "proj3_w4", "mlp_gate_up_quant_w4", "quant_row"])
def test_every_entry_point_rejects_cpu_tensors(pkg, name):
    """No CPU path: the binding refuses host tensors before reaching the C ABI."""
    with pytest.raises(ValueError, match="CUDA tensor"):
        _cpu_calls(pkg)[name]()
