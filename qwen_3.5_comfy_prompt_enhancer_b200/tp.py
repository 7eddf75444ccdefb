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
     buffer per rank) -> the full h [M, I] on every rank: by default this
     package's kernel storing straight into the peers' memory over NVLink
     (``PeerGather``), or torch.distributed's all-gather (NCCL / gloo);
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


class PeerGather:
    """All-gather of equal byte shards over NVLink peer memory with this
    package's own kernel (``qlin_peer_allgather``): each rank stores its shard
    straight into every rank's gather buffer and bumps arrival counters held
    in the peers' memory; no NCCL call on the data path.

    One cudaMalloc'd allocation per rank and gather holds the gather buffer
    (world x shard bytes) and the arrival counters; its CUDA IPC handle is
    exchanged once through the process group (``group`` must reach every
    rank).  Each call copies the gathered bytes, rank-major like
    ``all_gather_into_tensor``, into the torch tensor ``buf``."""

    def __init__(self, shard_bytes, device, group=None):
        import ctypes
        from . import _lib
        self._lib = _lib.load()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.shard = -(-shard_bytes // 16) * 16
        self.device = torch.device(device)
        gbytes = self.world * self.shard
        with torch.cuda.device(self.device):
            own = ctypes.c_void_p()
            _lib.check("qlin_dev_alloc", self._lib.qlin_dev_alloc(gbytes + 256, ctypes.byref(own)))
            self._own = own.value
            handle = (ctypes.c_ubyte * 64)()
            off = ctypes.c_int64()
            _lib.check("qlin_ipc_get_handle", self._lib.qlin_ipc_get_handle(self._own, handle, ctypes.byref(off)))
        self.buf = torch.empty(gbytes, dtype=torch.uint8, device=self.device)
        self.expected = torch.zeros(self.world, dtype=torch.int32, device=self.device)
        mine = torch.tensor(list(bytes(handle)) + list(off.value.to_bytes(8, "little")), dtype=torch.uint8,
                            device=self.device)
        allh = torch.empty(self.world * 72, dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(allh, mine, group=group)
        allh = allh.view(self.world, 72).cpu()
        self._opened = []
        bufs, arrive = [], []
        with torch.cuda.device(self.device):
            for q in range(self.world):
                if q == self.rank:
                    base = self._own
                else:
                    h = (ctypes.c_ubyte * 64)(*allh[q, :64].tolist())
                    qoff = int.from_bytes(bytes(allh[q, 64:].tolist()), "little")
                    ptr = ctypes.c_void_p()
                    _lib.check("qlin_ipc_open", self._lib.qlin_ipc_open(h, qoff, ctypes.byref(ptr)))
                    base = ptr.value
                    self._opened.append((base, qoff))
                bufs.append(base)
                arrive.append(base + gbytes)
        self._bufs = (ctypes.c_void_p * self.world)(*bufs)
        self._arrive = (ctypes.c_void_p * self.world)(*arrive)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)   # every rank's counters are zero before anyone writes

    def __call__(self, src):
        """Gather ``src`` (``shard`` bytes, contiguous) from every rank; returns ``buf``,
        the rank-major bytes [world * shard]."""
        from .kernels._host import stream_of
        from . import _lib
        rc = self._lib.qlin_peer_allgather(self._bufs, self._arrive, self.expected.data_ptr(), src.data_ptr(),
                                           self.shard, self.world, self.rank, self.buf.data_ptr(), stream_of(src))
        _lib.check("qlin_peer_allgather", rc)
        return self.buf

    def close(self):
        """Unmap the peers' buffers and free this rank's (after every rank stopped using them)."""
        with torch.cuda.device(self.device):
            for base, off in self._opened:
                self._lib.qlin_ipc_close(base, off)
            self._opened = []
            if self._own:
                self._lib.qlin_dev_free(self._own)
                self._own = None


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

    def __init__(self, gate, up, down, device, group=None, ops=None, gather=None):
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
        # "peer": this package's NVLink peer-memory all-gather (CUDA, world > 1);
        # "dist": torch.distributed's all_gather_into_tensor (NCCL or gloo).
        if gather is None:
            gather = "peer" if (self.world > 1 and self.device.type == "cuda") else "dist"
        if gather not in ("peer", "dist"):
            raise ValueError(f"gather must be 'peer' or 'dist', got {gather!r}")
        self.gather = gather

    def _workspace(self, M):
        ws = self._ws.get(M)
        if ws is None:
            d, g = self.device, self.world
            nq, ns = M * self.i_loc, M * (self.i_loc // GROUP) * 4
            # The local int8 codes and their fp32 scales share one byte buffer
            # (padded to 16 bytes), so a single all-gather moves both.
            pack = torch.zeros(-(-(nq + ns) // 16) * 16, dtype=torch.uint8, device=d)
            ws = {
                "pack": pack,
                "hq_loc": pack[:nq].view(torch.int8).view(M, self.i_loc),
                "hs_loc": pack[nq:nq + ns].view(torch.float32).view(M, self.i_loc // GROUP),
                "pack_all": torch.empty(g * pack.numel(), dtype=torch.uint8, device=d),
                "hq": torch.empty(M, self.inter, dtype=torch.int8, device=d),
                "hs": torch.empty(M, self.inter // GROUP, dtype=torch.float32, device=d),
                "o_loc": torch.empty(M, self.h_loc, dtype=torch.bfloat16, device=d),
                "o_all": torch.empty(g * M, self.h_loc, dtype=torch.bfloat16, device=d),
            }
            if self.gather == "peer":
                ws["peer_h"] = PeerGather(pack.numel(), d, self.group)
                ws["peer_o"] = PeerGather(M * self.h_loc * 2, d, self.group)
            self._ws[M] = ws
        return ws

    def _gather_h(self, ws, M):
        """All-gather the packed (codes, scales) shards; reassemble h [M, I] and its scales."""
        if self.world == 1:
            ws["hq"].copy_(ws["hq_loc"])
            ws["hs"].copy_(ws["hs_loc"])
            return ws["hq"], ws["hs"]
        if self.gather == "peer":
            allp = ws["peer_h"](ws["pack"]).view(self.world, -1)
        else:
            dist.all_gather_into_tensor(ws["pack_all"], ws["pack"], group=self.group)
            allp = ws["pack_all"].view(self.world, -1)
        g, n, ng = self.world, self.i_loc, self.i_loc // GROUP
        nq = M * n
        codes = allp[:, :nq].view(torch.int8).view(g, M, n)
        scales = allp[:, nq:nq + M * ng * 4].contiguous().view(torch.float32).view(g, M, ng)
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
        if self.gather == "peer" and self.world > 1:
            allo = ws["peer_o"](ws["o_loc"]).view(torch.bfloat16).view(self.world, M, self.h_loc)
            out.view(M, self.world, self.h_loc).copy_(allo.permute(1, 0, 2))
            return out
        return self._gather_cols(ws["o_loc"], ws["o_all"], out)

    def close(self):
        """Release the peer mappings (before the process group is destroyed)."""
        for ws in self._ws.values():
            for k in ("peer_h", "peer_o"):
                if k in ws:
                    ws[k].close()
        self._ws = {}

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
