"""Argument checks of the compiled binding (``_qlin_ext``) and the C ABI on CUDA
tensors.  Every case here is refused on the host: no kernel is launched."""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _w8_args(M=2, K=128, N=64):
    a = torch.zeros(M, K, dtype=torch.int8, device=DEV)
    s = torch.ones(M, K // 64, device=DEV)
    b = torch.zeros(K, N, dtype=torch.int8, device=DEV)
    bs = torch.ones(N, device=DEV)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    return a, s, b, bs, out


def _w4_args(M=2, K=128, N=64, wg=64):
    a = torch.zeros(M, K, dtype=torch.int8, device=DEV)
    s = torch.ones(M, K // 64, device=DEV)
    w = torch.zeros(K // 2, N, dtype=torch.uint8, device=DEV)
    ws = torch.ones(K // wg, N, dtype=torch.bfloat16, device=DEV)
    wz = torch.full((K // wg, N), 8, dtype=torch.uint8, device=DEV)
    return a, s, w, ws, wz


def test_wrong_dtype_is_type_error(pkg):
    a, s, b, bs, out = _w8_args()
    with pytest.raises(TypeError, match="a_s must be torch.float32"):
        pkg.gemm_i8(a, s.double(), b, bs, out)
    with pytest.raises(TypeError, match="out must be torch.bfloat16"):
        pkg.gemm_i8(a, s, b, bs, out.float())


def test_wrong_shapes_are_value_errors(pkg):
    a, s, b, bs, out = _w8_args()
    with pytest.raises(ValueError, match="a_s must be"):
        pkg.gemm_i8(a, s[:, :1].contiguous(), b, bs, out)
    with pytest.raises(ValueError, match="out must be"):
        pkg.gemm_i8(a, s, b, bs, out[:1])
    with pytest.raises(ValueError, match="b must be"):
        pkg.gemm_i8(a, s, b[:64].contiguous(), bs, out)
    a4, s4, w, ws, wz = _w4_args()
    with pytest.raises(ValueError, match="zeros must match"):
        pkg.gemm_w4(a4, s4, w, ws, out, b_z=wz[:, :32].contiguous())
    q = torch.empty(2, 64, dtype=torch.int8, device=DEV)
    qs = torch.empty(2, 2, device=DEV)
    with pytest.raises(ValueError, match="out_q/out_s"):
        pkg.mlp_gate_up_quant_w4(a4, s4, w, ws, w, ws, q, qs)


def test_non_contiguous_weight_rejected(pkg):
    a, s, b, bs, out = _w8_args()
    bt = torch.zeros(64, 128, dtype=torch.int8, device=DEV).t()
    with pytest.raises(ValueError, match="contiguous"):
        pkg.gemm_i8(a, s, bt, bs, out)


def test_strided_last_dim_rejected(pkg):
    a, s, b, bs, _ = _w8_args()
    wide = torch.empty(2, 128, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError, match="unit stride"):
        pkg.gemm_i8(a, s, b, bs, wide[:, ::2])


def test_misaligned_activation_refused_by_c_abi(pkg):
    """A contiguous view starting 1 byte into its buffer passes the Python-level
    checks; the C ABI refuses it (QLIN_ERR_ALIGNMENT) before any launch."""
    _, s, b, bs, out = _w8_args()
    buf = torch.zeros(2 * 128 + 16, dtype=torch.int8, device=DEV)
    a = buf[1:1 + 2 * 128].view(2, 128)
    with pytest.raises(pkg._lib.QlinError) as e:
        pkg.gemm_i8(a, s, b, bs, out)
    assert e.value.status == 3 and "aligned" in str(e.value)


def test_block_k_rule(pkg):
    a, s, b, bs, out = _w8_args()
    with pytest.raises(ValueError, match="block_k"):
        pkg.gemm_i8(a, s, b, bs, out, block_k=128)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_operands_on_two_devices_rejected(pkg):
    a, s, b, bs, out = _w8_args()
    with pytest.raises(ValueError, match="cuda:1"):
        pkg.gemm_i8(a, s, b.to("cuda:1"), bs, out)


def test_binding_and_library_loaded_in_tree(pkg):
    import os
    ext = pkg._lib.ext()
    here = os.path.dirname(os.path.abspath(pkg._lib.__file__))
    assert os.path.dirname(os.path.abspath(ext.__file__)) == here
    with open("/proc/self/maps") as f:
        maps = f.read()
    assert os.path.join(here, "libqlin.so") in maps
