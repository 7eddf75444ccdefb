"""Column-split (tensor-parallel) W4 MLP layer over the ranks of one node.

The gate/up projection and the down projection are split by OUTPUT columns:
rank r of g owns gate and up columns [r*I/g, (r+1)*I/g) and down columns
[r*H/g, (r+1)*H/g).  Every output element is computed by the same formula as
on one GPU (only the fp32 order of the kernels' K split, which they choose per
launch shape, can differ):

  1. fused gate/up + SiLU + per-64 requantisation on the local columns
     (``mlp_gate_up_quant_w4``; the 64-column quantisation groups stay on one
     rank because I/g is a multiple of 64);
  2. all-gather of the int8 codes and their scales -> the full h [M, I] and
     its scales [M, I/64] on every rank;
  3. down projection of the full h against the local down columns
     (``gemm_w4``);
  4. all-gather of the bf16 outputs -> [M, H] on every rank.

With CUDA and world > 1 the gathers are this package's own kernel
(``qlin_peer_allgather_ll``): each rank stores its column shard as flagged
8-byte words into every peer's exchange buffer over NVLink (CUDA IPC buffers,
no NCCL on the data path), and every rank's kernel writes each peer's words,
once they carry the call's number, into their column range of its own h /
output matrix -- the down projection reads h where it landed and the output
gather writes ``out`` itself: four launches per forward.  ``gather="dist"`` uses
``torch.distributed.all_gather_into_tensor`` (NCCL or gloo) and a column
reassembly instead; that is the path the CPU tests take.

A K (row) split would add an all-reduce of fp32 partial sums across ranks, so
it is not used.  Weights are given in the engine layouts (packed uint8 [K/2, N],
bf16 scales [K/WG, N], optional uint8 zeros [K/WG, N]); each rank keeps a
contiguous copy of its columns only.
"""
import copy
import ctypes

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


def _pad16(n):
    return -(-n // 16) * 16


class _DeviceBytes:
    """``__cuda_array_interface__`` over raw device memory, so that torch can
    view a buffer this package allocated (``torch.as_tensor``, no copy)."""

    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "strides": None, "version": 3}


# Gathers of at least this many bytes per rank move each byte once (arrival
# counters) instead of twice (flagged words).  Measured on 2 GPUs (graph of
# gathers, us per call, flagged words / counters): 256 KB 5.8 / 13.9, 1 MB
# 8.2 / 15.3, 4 MB 26.6 / 21.4.
FENCED_MIN_BYTES = 4 * 1024 * 1024


class PeerBuffer:
    """A gather destination of ``nbytes`` on every rank of ``group``, filled
    by ``qlin_peer_allgather_ll`` over NVLink peer memory.

    ``local`` (torch uint8) is this rank's destination.  Behind it sits an
    exchange buffer that every other rank stores its flagged words into: one
    allocation of its own per rank, shared through one CUDA IPC handle
    exchanged once over the process group, sized for gathers of at most
    ``nbytes`` in all, plus a small state array (the call count)."""

    def __init__(self, nbytes, device, group=None):
        from . import _lib
        self._lib = _lib.load()
        self._check = _lib.check
        init = dist.is_initialized()
        self.world = dist.get_world_size(group) if init else 1
        self.rank = dist.get_rank(group) if init else 0
        self.nbytes = _pad16(nbytes)
        self.device = torch.device(device)
        # per sender: two 8-byte words per 8 data bytes, each part padded to 16
        self.ll_bytes = 2 * self.world * (2 * _pad16(-(-self.nbytes // self.world)) + 16 * 4)
        # one allocation: the destination, arrival counters of the fenced
        # protocol, the exchange buffer of the flagged words
        self._ll_off = self.nbytes + 256
        with torch.cuda.device(self.device):
            own = ctypes.c_void_p()
            _lib.check("qlin_dev_alloc", self._lib.qlin_dev_alloc(self._ll_off + self.ll_bytes, ctypes.byref(own)))
            self._own = own.value
            handle = (ctypes.c_ubyte * 64)()
            off = ctypes.c_int64()
            _lib.check("qlin_ipc_get_handle", self._lib.qlin_ipc_get_handle(self._own, handle, ctypes.byref(off)))
        self.local = torch.as_tensor(_DeviceBytes(self._own, self.nbytes), device=self.device)
        self.state = torch.zeros(_lib.PEER_STATE_WORDS, dtype=torch.int32, device=self.device)
        mine = torch.tensor(list(bytes(handle)) + list(off.value.to_bytes(8, "little")), dtype=torch.uint8)
        if self.world > 1:
            # the handles travel as device tensors over NCCL, as CPU tensors otherwise
            where = self.device if dist.get_backend(group) == "nccl" else torch.device("cpu")
            allh = torch.empty(self.world * 72, dtype=torch.uint8, device=where)
            dist.all_gather_into_tensor(allh, mine.to(where), group=group)
            allh = allh.view(self.world, 72).cpu()
        else:
            allh = mine.view(1, 72)
        self._opened = []
        ll = []
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
                ll.append(base)
        self._bufs = (ctypes.c_void_p * self.world)(*ll)
        self._arrive = (ctypes.c_void_p * self.world)(*[b + self.nbytes for b in ll])
        self._ll = (ctypes.c_void_p * self.world)(*[b + self._ll_off for b in ll])
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=group)   # every rank's exchange buffer is zero before anyone writes

    def gather(self, parts, dst=None, fenced=False):
        """All-gather ``parts`` (a list of ``_lib.GatherPart`` whose offsets
        refer to the destination) into ``dst`` (a CUDA tensor; default
        ``local``) on every rank, on the current stream.  With ``fenced``
        (every rank must pass the same), gathers into ``local`` of at least
        FENCED_MIN_BYTES per rank take the arrival-counter protocol, which
        stores each byte once (``qlin_peer_allgather_fenced``)."""
        from .kernels._host import stream_of
        arr = (type(parts[0]) * len(parts))(*parts)
        if fenced and dst is None and sum(p.rows * p.row_bytes for p in parts) >= FENCED_MIN_BYTES:
            rc = self._lib.qlin_peer_allgather_fenced(self._bufs, self._arrive, self.state[8:].data_ptr(), arr,
                                                      len(parts), self.world, self.rank, stream_of(self.local))
            self._check("qlin_peer_allgather_fenced", rc)
            return
        dst = self.local if dst is None else dst
        rc = self._lib.qlin_peer_allgather_ll(self._ll, self.ll_bytes, self.state.data_ptr(), arr, len(parts),
                                              self.world, self.rank, dst.data_ptr(), stream_of(self.local))
        self._check("qlin_peer_allgather_ll", rc)

    def send(self, parts):
        """The sending half of ``gather``: this rank's parts go to every rank's
        exchange buffer (its own included) as words of the next call number;
        nothing waits and nothing advances (``qlin_peer_ll_send``)."""
        from .kernels._host import stream_of
        arr = (type(parts[0]) * len(parts))(*parts)
        rc = self._lib.qlin_peer_ll_send(self._ll, self.ll_bytes, self.state.data_ptr(), arr, len(parts),
                                         self.world, self.rank, stream_of(self.local))
        self._check("qlin_peer_ll_send", rc)

    def recv(self, parts, dst=None, state2=None):
        """The receiving half: every rank's words of the next call number
        (own included) into ``dst`` (default ``local``); then the call count
        advances, and ``state2``'s by one if given (``qlin_peer_ll_recv``)."""
        from .kernels._host import stream_of
        dst = self.local if dst is None else dst
        arr = (type(parts[0]) * len(parts))(*parts)
        rc = self._lib.qlin_peer_ll_recv(self._ll, self.ll_bytes, self.state.data_ptr(), arr, len(parts),
                                         self.world, self.rank, dst.data_ptr(),
                                         None if state2 is None else state2.data_ptr(), stream_of(self.local))
        self._check("qlin_peer_ll_recv", rc)

    def close(self):
        """Unmap the peers' exchange buffers and free this rank's.  The caller
        must make sure every rank has stopped using them first (GPU work
        synchronised, then a barrier), as ColumnParallelW4MLP.close does."""
        with torch.cuda.device(self.device):
            for base, off in self._opened:
                self._lib.qlin_ipc_close(base, off)
            self._opened = []
            self.local = None
            if self._own:
                self._lib.qlin_dev_free(self._own)
                self._own = None


def _part(src, rows, row_bytes, src_ld, dst_off, dst_ld):
    from ._lib import GatherPart
    return GatherPart(src.data_ptr(), src_ld, rows, row_bytes, dst_off, dst_ld)


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

    def __init__(self, gate, up, down, device, group=None, ops=None, gather=None, fused=True):
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
        # "peer" gathers around a 1-2-row down projection that the decode-row
        # kernel serves run inside it (qlin_tp_gemm_w4_ll): it polls h's words
        # in its prologue and sends its output rows from its epilogue.
        # Measured on 2 GPUs (graph replay, us per forward, separate / fused):
        # M = 1 35.3 / 33.1, M = 2 40.5 / 39.2, M = 4 47.5 / 48.1 (not taken).
        self.fused = fused
        self.down_wg = self.inter // down[1].shape[0]

    def sharing(self, gate, up, down):
        """The same layer shape with other weights (full-layer triples, sharded
        like the constructor's), sharing this layer's workspaces: gather
        buffers and their call counts.  Forwards of the layers that share them
        must run one after another on one stream, in the same order on every
        rank; only the first layer's ``close`` releases the buffers."""
        other = copy.copy(self)
        lo, hi = shard_range(self.inter, self.rank, self.world)
        dlo, dhi = shard_range(self.hidden, self.rank, self.world)
        put = (lambda t: None if t is None else t.to(self.device))
        other.gate = tuple(put(_cols(t, lo, hi)) for t in gate)
        other.up = tuple(put(_cols(t, lo, hi)) for t in up)
        other.down = tuple(put(_cols(t, dlo, dhi)) for t in down)
        if other.gate[0].shape != self.gate[0].shape or other.down[0].shape != self.down[0].shape:
            raise ValueError("weights of another shape")
        return other

    def _workspace(self, M):
        ws = self._ws.get(M)
        if ws is not None:
            return ws
        d, g, r = self.device, self.world, self.rank
        ng_loc, ng = self.i_loc // GROUP, self.inter // GROUP
        ws = {
            "hq_loc": torch.empty(M, self.i_loc, dtype=torch.int8, device=d),
            "hs_loc": torch.empty(M, ng_loc, dtype=torch.float32, device=d),
        }
        if g == 1:
            # nothing to gather: h is the local h, the output is written in place
            ws["hq"], ws["hs"] = ws["hq_loc"], ws["hs_loc"]
        elif self.gather == "peer":
            # h codes at byte 0 and h scales at hs_off of one gather buffer;
            # the output matrix in a second one.  Rank r's shards land in their
            # column ranges, so hq / hs / out_full are ordinary row-major views.
            hs_off = _pad16(M * self.inter)
            hbuf = PeerBuffer(hs_off + M * ng * 4, d, self.group)
            obuf = PeerBuffer(M * self.hidden * 2, d, self.group)
            out_full = obuf.local[:M * self.hidden * 2].view(torch.bfloat16).view(M, self.hidden)
            ws.update(
                hbuf=hbuf, obuf=obuf,
                hq=hbuf.local[:M * self.inter].view(torch.int8).view(M, self.inter),
                hs=hbuf.local[hs_off:hs_off + M * ng * 4].view(torch.float32).view(M, ng),
                out_full=out_full,
                o_slot=out_full[:, r * self.h_loc:(r + 1) * self.h_loc],
                h_parts=[_part(ws["hq_loc"], M, self.i_loc, self.i_loc, 0, self.inter),
                         _part(ws["hs_loc"], M, ng_loc * 4, ng_loc * 4, hs_off, ng * 4)])
            ws["o_parts"] = [_part(ws["o_slot"], M, self.h_loc * 2, self.hidden * 2, 0, self.hidden * 2)]
            ws["fused"] = self.fused and self._fused_ok(M)
            if ws["fused"]:
                from ._lib import GatherPart
                ws["h_arr"] = (GatherPart * 2)(*ws["h_parts"])
                ws["o_arr"] = (GatherPart * 1)(*ws["o_parts"])
        else:
            nq, ns = M * self.i_loc, M * ng_loc * 4
            # the local codes and scales share one byte buffer, so a single
            # all-gather moves both
            pack = torch.zeros(_pad16(nq + ns), dtype=torch.uint8, device=d)
            ws.update(
                pack=pack,
                hq_loc=pack[:nq].view(torch.int8).view(M, self.i_loc),
                hs_loc=pack[nq:nq + ns].view(torch.float32).view(M, ng_loc),
                pack_all=torch.empty(g * pack.numel(), dtype=torch.uint8, device=d),
                hq=torch.empty(M, self.inter, dtype=torch.int8, device=d),
                hs=torch.empty(M, ng, dtype=torch.float32, device=d),
                o_loc=torch.empty(M, self.h_loc, dtype=torch.bfloat16, device=d),
                o_all=torch.empty(g * M, self.h_loc, dtype=torch.bfloat16, device=d))
        self._ws[M] = ws
        return ws

    def _fused_ok(self, M):
        """Whether the down projection of M rows runs on the decode-row kernel
        (the only one with the gathers inside) and the shard sizes fit it."""
        if M > 2 or self.i_loc % 128 or self.h_loc % 16:
            return False
        from . import _lib
        plan = (ctypes.c_int64 * 4)()
        with torch.cuda.device(self.device):
            _lib.check("qlin_plan_dp", _lib.load().qlin_plan_dp(4, 0, M, self.inter, -(-self.h_loc // 128),
                                                                self.down_wg, 0, plan))
        return plan[0] > 0

    def _down_fused(self, ws, M):
        from . import _lib
        from .kernels._host import stream_of
        d, hb, ob = self.down, ws["hbuf"], ws["obuf"]
        rc = _lib.load().qlin_tp_gemm_w4_ll(
            M, self.inter, d[0].data_ptr(), d[1].data_ptr(), None if d[2] is None else d[2].data_ptr(), self.h_loc,
            self.down_wg, ws["o_slot"].data_ptr(), self.hidden, hb._ll, hb.ll_bytes, hb.state.data_ptr(),
            ws["h_arr"], 2, ob._ll, ob.ll_bytes, ob.state.data_ptr(), ws["o_arr"], 1, self.world, self.rank,
            ws["hq"].data_ptr(), ws["hs"].data_ptr(), stream_of(d[0]))
        _lib.check("qlin_tp_gemm_w4_ll", rc)

    def _gather_h_dist(self, ws, M):
        """torch.distributed all-gather of the packed (codes, scales) shards,
        then the column reassembly of h [M, I] and its scales."""
        dist.all_gather_into_tensor(ws["pack_all"], ws["pack"], group=self.group)
        allp = ws["pack_all"].view(self.world, -1)
        g, n, ng = self.world, self.i_loc, self.i_loc // GROUP
        nq = M * n
        codes = allp[:, :nq].view(torch.int8).view(g, M, n)
        scales = allp[:, nq:nq + M * ng * 4].contiguous().view(torch.float32).view(g, M, ng)
        ws["hq"].view(M, g, n).copy_(codes.permute(1, 0, 2))
        ws["hs"].view(M, g, ng).copy_(scales.permute(1, 0, 2))

    def forward(self, a_q, a_s, out, events=None):
        """a_q int8 [M, K], a_s fp32 [M, K/64] -> out bf16 [M, H] (every rank).

        ``events``: optional list of five CUDA events, recorded before the
        gate/up projection and after it, the h gather, the down projection
        and the output gather (per-stage timing)."""
        M = a_q.shape[0]
        if a_q.shape[1] != self.k or out.shape != (M, self.hidden):
            raise ValueError("activation / output shape does not match the layer")
        ws = self._workspace(M)
        g, u, d = self.gate, self.up, self.down
        rec = (lambda i: events[i].record()) if events else (lambda i: None)
        rec(0)
        self.ops.gate_up_quant_w4(a_q, a_s, g[0], g[1], u[0], u[1], ws["hq_loc"], ws["hs_loc"], zg=g[2], zu=u[2])
        rec(1)
        if self.world == 1:
            rec(2)
            self.ops.gemm_w4(ws["hq"], ws["hs"], d[0], d[1], out, b_z=d[2])
            rec(3)
            rec(4)
            return out
        if self.gather == "peer" and ws["fused"]:
            # h's words leave now; the down projection polls them, sends its
            # output rows, and the receive lands every rank's rows in out
            ws["hbuf"].send(ws["h_parts"])
            rec(2)
            self._down_fused(ws, M)
            rec(3)
            direct = out.is_contiguous() and out.data_ptr() % 8 == 0
            ws["obuf"].recv(ws["o_parts"], out if direct else None, state2=ws["hbuf"].state)
            if not direct:
                out.copy_(ws["out_full"])
            rec(4)
            return out
        if self.gather == "peer":
            ws["hbuf"].gather(ws["h_parts"], fenced=True)
            rec(2)
            self.ops.gemm_w4(ws["hq"], ws["hs"], d[0], d[1], ws["o_slot"], b_z=d[2])
            rec(3)
            # the output gather lands in ``out`` itself when it can
            direct = out.is_contiguous() and out.data_ptr() % 8 == 0
            ws["obuf"].gather(ws["o_parts"], out if direct else None)
            if not direct:
                out.copy_(ws["out_full"])
            rec(4)
            return out
        self._gather_h_dist(ws, M)
        rec(2)
        self.ops.gemm_w4(ws["hq"], ws["hs"], d[0], d[1], ws["o_loc"], b_z=d[2])
        rec(3)
        # [world * M, h_loc] rank-major -> columns of out
        dist.all_gather_into_tensor(ws["o_all"], ws["o_loc"], group=self.group)
        out.view(M, self.world, self.h_loc).copy_(ws["o_all"].view(self.world, M, self.h_loc).permute(1, 0, 2))
        rec(4)
        return out

    __call__ = forward

    def close(self):
        """Release the peer mappings (before the process group is destroyed).

        Peers write into this rank's gather buffers directly, so every rank
        must have finished using them first: this waits for this rank's GPU
        work, then for every rank (a barrier on the layer's group), and only
        then unmaps and frees.  Every rank of the group must call it."""
        peers = [ws[k] for ws in self._ws.values() for k in ("hbuf", "obuf") if k in ws]
        if peers:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
        for p in peers:
            p.close()
        self._ws = {}

    def capture(self, a_q, a_s, out, warmup=2):
        """CUDA graph of ``forward`` on these buffers (kernels and, with the
        dist gather, NCCL collectives).  Replay it after refilling
        ``a_q``/``a_s`` in place; release the graph before the process group
        is destroyed."""
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
