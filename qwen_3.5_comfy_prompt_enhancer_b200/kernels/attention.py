"""Full-attention decode neighbours -- drop-in for the reference's
``kernels/attention.py`` (``qk_norm_rope``, ``attn_decode``), backed by the
sm_100a kernels of ``libqlin.so``.

Extension over the reference: a position (``pos0`` / ``pos``) may be given as
a one-element int32 CUDA tensor instead of an int, read by the kernels at run
time, so that a decode step is captured in a CUDA graph once and replayed at
every position (``max_pos`` then bounds the positions a replay will see).
"""
import torch

from .. import _lib


def _pos(p):
    if isinstance(p, torch.Tensor):
        return 0, p
    return int(p), None


def qk_norm_rope(proj, qn, kn, invf, qout, kvc, kvs, pos0, eps=1e-6, kv_int8=False,
                 batch=False, kv_stride=None, kvs_stride=None):
    """Norm + RoPE the q/k/v heads; k/v go to the KV cache (bf16 or int8)
    (kernels/attention.py:70-133).

    In batch mode each row is one candidate at the *shared* position `pos0`;
    the cache is laid out as per-row slices of `kv_stride` elements
    (`kvs_stride` for the scales).
    """
    if kv_int8 and kvs is None:
        raise ValueError("kv_int8=True requires the kvs scales tensor")
    p, pd = _pos(pos0)
    rc = _lib.ext().qk_norm_rope(proj, qn, kn, invf, qout, kvc, kvs if kv_int8 else None, p, pd, float(eps),
                                 bool(kv_int8), bool(batch), int(kv_stride or 0), int(kvs_stride or 0))
    if rc:
        raise _lib.QlinError("qlin_qk_norm_rope", rc)


def attn_decode(q, kvc, out, pos, kvs=None, kv_int8=False, batch=1, block_n=32,
                nq=8, nkv=2, hd=256, max_pos=None):
    """Single-query decode read of the KV cache (bf16 or int8), batched
    (kernels/attention.py:209-267).  ``block_n`` is accepted and ignored."""
    if kv_int8 and kvs is None:
        raise ValueError("kv_int8=True requires the kvs scales tensor")
    p, pd = _pos(pos)
    if pd is not None and max_pos is None:
        max_pos = kvc.shape[0] // batch - 1   # the cache's last row
    rc = _lib.ext().attn_decode(q, kvc, out, p, pd, int(max_pos or 0), kvs if kv_int8 else None, bool(kv_int8),
                                int(batch), int(nq), int(nkv), int(hd))
    if rc:
        raise _lib.QlinError("qlin_attn_decode", rc)
    return out


def attn_prefill(q, kvc, out, T, pos0=0, kvs=None, kv_int8=False, block_m=32,
                 block_n=32, nq=8, nkv=2, hd=256):
    """Causal prefill over the KV cache; reads the int8 cache when kv_int8
    (kernels/attention.py:136-206).  Tile keywords are accepted and ignored.
    Returns ``out``."""
    if kv_int8 and kvs is None:
        raise ValueError("kv_int8=True requires the kvs scales tensor")
    rc = _lib.ext().attn_prefill(q, kvc, out, int(T), int(pos0), kvs if kv_int8 else None, bool(kv_int8), int(nq),
                                 int(nkv), int(hd))
    if rc:
        raise _lib.QlinError("qlin_attn_prefill", rc)
    return out
