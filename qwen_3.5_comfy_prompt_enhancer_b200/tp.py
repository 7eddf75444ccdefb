"""Column-split (tensor-parallel) W4 MLP layer over the ranks of one node.

The gate/up projection and the down projection are split by OUTPUT columns:
rank r of g owns gate and up columns [r*I/g, (r+1)*I/g) and down columns
[r*H/g, (r+1)*H/g).  Every output element is computed by the same formula as
on one GPU (only the fp32 order of the kernels' K split, which they choose per
launch shape, can differ):

  1. fused gate/up + SiLU + per-64 requantisation on the local columns
     (``mlp_gate_up_quant_w4``; the 64-column quantisation groups stay on one
     rank because I/g is a multiple of 64);
  2. one all-gather of the int8 codes and their scales (packed in one byte
     buffer per rank) -> the full h [M, I] on every rank (NCCL over NVLink);
  3. down projection of the full h against the local down columns
     (``gemm_w4``);
  4. all-gather of the bf16 outputs -> [M, H] on every rank.

A K (row) split would add an all-reduce of fp32 partial sums across ranks, so
it is not used.  Weights are given in the engine layouts (packed uint8 [K/2, N],
bf16 scales [K/WG, N], optional uint8 zeros [K/WG, N]); each rank keeps a
contiguous copy of its columns only.

The compute calls go through ``ops`` (default: this package's CUDA kernels);
collectives use ``torch.distributed`` on the given process group.
"""
import torch
import torch.distributed as dist

from .kernels.common import GROUP


def shard_range(n, rank, world):
    """Column range [lo, hi) of ``rank``; shards are equal and multiples of 64."""
    if n % (GROUP * world) != 0:
        raise ValueError(f"{n} columns do not split into {world} shards of a multiple of {GROUP}")
    w = n // world
    return rank * w, (rank + 1) * w


def _cols(t, lo, hi):
    return None if t is None else t[:, lo:hi].contiguous()


class _KernelOps:
    """The package's CUDA entry points (imported lazily: the package's
    top-level module name is an alias chosen by the importer)."""

    def __init__(self):
        from .kernels import w4
        self.gate_up_quant_w4 = w4.mlp_gate_up_quant_w4
        self.gemm_w4 = w4.gemm_w4


class ColumnParallelW4MLP:
    """One W4 MLP (gate/up fused with SiLU + int8 requant, then down) with its
    output columns split over the ranks of ``group``.

    ``gate``, ``up``, ``down`` are (packed, scales, zeros-or-None) triples of
    the full layer; ``device`` is this rank's GPU.
    """

    def __init__(self, gate, up, down, device, group=None, ops=None):
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.device = torch.device(device)
        self.ops = ops if ops is not None else _KernelOps()
        self.inter = gate[0].shape[1]
        self.hidden = down[0].shape[1]
        self.k = 2 * gate[0].shape[0]
        if up[0].shape != gate[0].shape or 2 * down[0].shape[0] != self.inter:
            raise ValueError("gate/up/down shapes do not form an MLP")
        lo, hi = shard_range(self.inter, self.rank, self.world)
        dlo, dhi = shard_range(self.hidden, self.rank, self.world)
        self.i_loc = hi - lo
        self.h_loc = dhi - dlo
        put = (lambda t: None if t is None else t.to(self.device))
        self.gate = tuple(put(_cols(t, lo, hi)) for t in gate)
        self.up = tuple(put(_cols(t, lo, hi)) for t in up)
        self.down = tuple(put(_cols(t, dlo, dhi)) for t in down)
        self._ws = {}

    def _workspace(self, M):
        ws = self._ws.get(M)
        if ws is None:
            d, g = self.device, self.world
            nq, ns = M * self.i_loc, M * (self.i_loc // GROUP) * 4
            # The local int8 codes and their fp32 scales share one byte buffer,
            # so a single all-gather moves both.
            pack = torch.empty(nq + ns, dtype=torch.uint8, device=d)
            ws = {
                "pack": pack,
                "hq_loc": pack[:nq].view(torch.int8).view(M, self.i_loc),
                "hs_loc": pack[nq:].view(torch.float32).view(M, self.i_loc // GROUP),
                "pack_all": torch.empty(g * (nq + ns), dtype=torch.uint8, device=d),
                "hq": torch.empty(M, self.inter, dtype=torch.int8, device=d),
                "hs": torch.empty(M, self.inter // GROUP, dtype=torch.float32, device=d),
                "o_loc": torch.empty(M, self.h_loc, dtype=torch.bfloat16, device=d),
                "o_all": torch.empty(g * M, self.h_loc, dtype=torch.bfloat16, device=d),
            }
            self._ws[M] = ws
        return ws

    def _gather_h(self, ws, M):
        """All-gather the packed (codes, scales) shards; reassemble h [M, I] and its scales."""
        if self.world == 1:
            ws["hq"].copy_(ws["hq_loc"])
            ws["hs"].copy_(ws["hs_loc"])
            return ws["hq"], ws["hs"]
        dist.all_gather_into_tensor(ws["pack_all"], ws["pack"], group=self.group)
        g, n, ng = self.world, self.i_loc, self.i_loc // GROUP
        nq = M * n
        allp = ws["pack_all"].view(g, -1)
        codes = allp[:, :nq].view(torch.int8).view(g, M, n)
        scales = allp[:, nq:].contiguous().view(torch.float32).view(g, M, ng)
        ws["hq"].view(M, g, n).copy_(codes.permute(1, 0, 2))
        ws["hs"].view(M, g, ng).copy_(scales.permute(1, 0, 2))
        return ws["hq"], ws["hs"]

    def _gather_cols(self, loc, allbuf, full):
        """all-gather [M, n] shards into [M, world * n] (rank r at columns r*n)."""
        if self.world == 1:
            full.copy_(loc)
            return full
        dist.all_gather_into_tensor(allbuf, loc, group=self.group)   # [world * M, n], rank-major
        M, n = loc.shape
        full.view(M, self.world, n).copy_(allbuf.view(self.world, M, n).permute(1, 0, 2))
        return full

    def forward(self, a_q, a_s, out):
        """a_q int8 [M, K], a_s fp32 [M, K/64] -> out bf16 [M, H] (every rank)."""
        M = a_q.shape[0]
        if a_q.shape[1] != self.k or out.shape != (M, self.hidden):
            raise ValueError("activation / output shape does not match the layer")
        ws = self._workspace(M)
        g, u, d = self.gate, self.up, self.down
        self.ops.gate_up_quant_w4(a_q, a_s, g[0], g[1], u[0], u[1], ws["hq_loc"], ws["hs_loc"], zg=g[2], zu=u[2])
        hq, hs = self._gather_h(ws, M)
        self.ops.gemm_w4(hq, hs, d[0], d[1], ws["o_loc"], b_z=d[2])
        return self._gather_cols(ws["o_loc"], ws["o_all"], out)

    __call__ = forward

    def capture(self, a_q, a_s, out, warmup=2):
        """CUDA graph of ``forward`` on these buffers (kernels and NCCL
        collectives).  Replay it after refilling ``a_q``/``a_s`` in place;
        release the graph before the process group is destroyed."""
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.forward(a_q, a_s, out)
        torch.cuda.current_stream(self.device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            self.forward(a_q, a_s, out)
        return graph
