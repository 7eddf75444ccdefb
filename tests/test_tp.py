"""Column-split (tensor-parallel) W4 MLP: host logic on CPU with gloo ranks.

The compute calls are replaced by the CPU oracle, so these tests check the
sharding, the all-gathers and the column reassembly: every rank must end
with exactly the single-process result (a column split does not change any
per-column arithmetic).  The CUDA path of the same class runs in
tests/test_gpu_tp.py and bench.py on real GPUs.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import qlin_oracle as O
from qlin_testutil import bits, from_bits, gen, w4

K, I, H, WG = 256, 512, 256, 128


class OracleOps:
    """CPU stand-ins for the CUDA entry points (test infrastructure)."""

    @staticmethod
    def gate_up_quant_w4(a_q, a_s, wg, sg, wu, su, out_q, out_s, zg=None, zu=None):
        q, s = O.mlp_gate_up_quant_w4(a_q.numpy(), a_s.numpy(), wg.numpy(), bits(sg), wu.numpy(), bits(su),
                                      None if zg is None else zg.numpy(), None if zu is None else zu.numpy())
        out_q.copy_(torch.from_numpy(q))
        out_s.copy_(torch.from_numpy(s))

    @staticmethod
    def gemm_w4(a_q, a_s, b, b_s, out, b_z=None):
        r = O.gemm_w4(a_q.numpy(), a_s.numpy(), b.numpy(), bits(b_s), None if b_z is None else b_z.numpy())
        out.copy_(from_bits(r))


def make_layer(seed, zeros=True):
    g = gen(seed)
    return w4(g, K, I, WG, zeros), w4(g, K, I, WG, zeros), w4(g, I, H, WG, zeros)


def reference(M, seed, zeros):
    gate, up, down = make_layer(seed, zeros)
    g = gen(seed + 1)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    a_q, a_s = O.quant_row(bits(x))
    hq, hs = O.mlp_gate_up_quant_w4(a_q, a_s, gate[0].numpy(), bits(gate[1]), up[0].numpy(), bits(up[1]),
                                    None if gate[2] is None else gate[2].numpy(),
                                    None if up[2] is None else up[2].numpy())
    out = O.gemm_w4(hq, hs, down[0].numpy(), bits(down[1]), None if down[2] is None else down[2].numpy())
    return torch.from_numpy(a_q), torch.from_numpy(a_s), out


def _rank_main(rank, world, port, M, seed, zeros, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import __graft_entry__
        pkg = __graft_entry__.load_package()
        gate, up, down = make_layer(seed, zeros)
        layer = pkg.tp.ColumnParallelW4MLP(gate, up, down, "cpu", ops=OracleOps())
        a_q, a_s, _ = reference(M, seed, zeros)
        out = torch.empty(M, H, dtype=torch.bfloat16)
        layer(a_q, a_s, out)
        q.put((rank, bits(out), layer.i_loc, layer.h_loc))
    finally:
        dist.destroy_process_group()


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [1, 2, 4])
@pytest.mark.parametrize("M,zeros", [(1, True), (4, False), (3, True)])
def test_column_split_matches_single_process(world, M, zeros):
    seed = 7000 + world * 10 + M
    _, _, ref = reference(M, seed, zeros)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, M, seed, zeros, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, out_bits, i_loc, h_loc in results:
        assert i_loc == I // world and h_loc == H // world
        np.testing.assert_array_equal(out_bits, ref, err_msg=f"rank {rank} of {world}")


def test_shard_range_rules(pkg):
    assert pkg.tp.shard_range(17408, 3, 8) == (6528, 8704)
    assert pkg.tp.shard_range(5120, 7, 8) == (4480, 5120)
    with pytest.raises(ValueError):
        pkg.tp.shard_range(5120, 0, 3)     # 5120 / 3 is not a multiple of 64
    with pytest.raises(ValueError):
        pkg.tp.shard_range(192, 0, 2)      # 96 is not a multiple of 64
