"""Row-sharded pair stack: one process per GPU, NCCL between the phases.

Rank ``r`` of ``W`` owns rows ``[r0, r0 + rows)`` of the pair tensor
``z [n, n, 128]``, held in a ``[chunk, n, 128]`` buffer. ``chunk`` is the
common padded row count (``ceil(n / W)`` rounded up to 32 rows, so that a
rank's rows are whole column tiles of the outgoing contraction); the last
ranks may hold fewer valid rows, or none.

Every operator of the block needs at most one exchange step (the reference
runs each operator on one device; its only multi-device code is the outer
batch split of ``python/fireprot/backends/amd/two_gcd_attention.py:53-101``):

* TriMul outgoing ``x_ij = sum_k a_ik b_jk``: ``a`` rows are local, every
  ``j`` needs all rows of ``b`` -> all-gather of the projected ``b`` planes,
  then the local rows of ``x``.
* TriMul incoming ``x_ij = sum_k a_ki b_kj``: the rank holds rows ``k`` of
  ``a`` and ``b`` -> partial contraction over its ``k`` for all ``(i, j)``,
  reduce-scatter of ``x`` by rows.
* TriMul, channel-group scheme (``trimul_scheme``: four or more ranks): the
  channels of the contraction are independent, so rank ``g`` takes channel
  group ``g`` (``128 / W`` planes) of every rank's projected ``a`` and ``b``
  (one all-to-all each), contracts it over the whole ``n x n`` grid and
  returns each rank its rows of ``x`` (a third all-to-all). Per rank that
  moves ``3/W`` of the row scheme's bytes.
* TriAttn starting node: q/k/v/gate of row ``i`` come from row ``i``; only
  the pair bias ``b[h, j, k]`` spans all rows -> all-gather of the rank's
  rows of the row-blocked bias.
* TriAttn ending node: the starting form on ``z^T`` -> all-to-all transpose
  of ``z``, starting form, all-to-all transpose back.
* Transition: per position, local.

The phase kernels are the single-GPU kernels run on row ranges
(``fpb_trimul_shard_*``, ``fpb_triattn_shard_*``, ``fpb_transition``);
``CudaPhases`` is the only compute provider in the package. ``Comm`` wraps
the three collectives so the orchestration is independent of the transport.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib, ops

ROW_ALIGN = 32


@dataclass(frozen=True)
class RowShard:
    """Rows of the pair tensor owned by one rank."""
    n: int
    world: int
    rank: int

    @property
    def chunk(self) -> int:
        per = -(-self.n // self.world)
        return -(-per // ROW_ALIGN) * ROW_ALIGN

    @property
    def r0(self) -> int:
        return min(self.rank * self.chunk, self.n)

    @property
    def rows(self) -> int:
        return max(0, min(self.n, (self.rank + 1) * self.chunk) - self.r0)


def shard_plan(n: int, world: int, rank: int) -> RowShard:
    if n <= 0 or world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad shard plan n={n} world={world} rank={rank}")
    return RowShard(n, world, rank)


def local_rows(z: torch.Tensor, shard: RowShard) -> torch.Tensor:
    """This rank's padded ``[chunk, n, c]`` slice of a full pair tensor."""
    out = z.new_zeros((shard.chunk,) + tuple(z.shape[1:]))
    out[:shard.rows] = z[shard.r0:shard.r0 + shard.rows]
    return out


class DistComm:
    """Collectives of a ``torch.distributed`` process group (NCCL on GPUs).

    Buffers are contiguous and rank-major along their first dimension; they
    are passed flat, since only their sizes matter to the exchange."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self._dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def all_gather(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        self._dist.all_gather_into_tensor(out.view(-1), inp.reshape(-1), group=self.group)

    def reduce_scatter(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        self._dist.reduce_scatter_tensor(out.view(-1), inp.reshape(-1),
                                         op=self._dist.ReduceOp.SUM, group=self.group)

    def all_to_all(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        self._dist.all_to_all_single(out.view(-1), inp.reshape(-1), group=self.group)


class PeerComm:
    """The exchanges over CUDA peer memory between the GPUs of one node.

    Every rank registers the receive buffers once (an IPC handle per buffer,
    swapped with ``all_gather_object``; the peers map them into their own
    context), after which an all-to-all or all-gather is one kernel
    (``fpb_peer_scatter``) whose SMs store every peer's block straight into
    the peer's buffer over NVLink, all peers side by side, and the
    transposed exchange of the ending-node operator is one kernel
    (``fpb_peer_transpose_rows``) that stores each 512-byte channel vector
    at its transposed place on its owner: no packing, staging or unpacking
    pass. ``owner_buffer`` hands phase kernels every rank's address of a
    buffer, so the channel-group TriMul's projection and contraction store
    their outputs at the owning ranks themselves. A one-element NCCL
    all-reduce on the current stream orders the transfers: after them
    (every peer's stores into this rank have landed), and before them
    (every peer is done with the buffer's previous contents) unless the
    caller passes ``fresh=True``. The reduce-scatter of the row TriMul
    scheme stays on NCCL.

    A buffer obtained from ``recv_buffer`` is filled in place; any other
    destination is filled through a registered scratch buffer plus one local
    copy. Registered buffers live as long as the object: ``close()`` unmaps
    the peers' buffers (call it, after a device synchronise, before the
    process group is destroyed).

    ``dist``, ``lib`` and ``device`` default to ``torch.distributed``, the
    CUDA library and the current CUDA device; another process-group API (with
    ``get_world_size``, ``get_rank``, ``all_gather_object``, ``all_reduce``,
    ``reduce_scatter_tensor`` and ``ReduceOp``) or an object with the
    library's peer entry points can stand in for them."""

    def __init__(self, group=None, *, dist=None, lib=None, device=None):
        if dist is None:
            import torch.distributed as dist
        self._dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 16:
            raise ValueError(f"the peer transport spans at most 16 ranks (world={self.world})")
        self.lib = _lib.load() if lib is None else lib
        self.dev = (torch.device("cuda", torch.cuda.current_device()) if device is None
                    else torch.device(device))
        self._tick = torch.zeros(1, device=self.dev)
        self._bufs: dict = {}     # (tag, shape, dtype) -> (tensor, [device pointer per rank])
        self._by_ptr: dict = {}   # data_ptr -> (tag, shape, dtype)
        self._opened: dict = {}   # handle bytes -> mapped base (peer segments)
        self._hbytes = int(self.lib.fpb_ipc_handle_bytes())

    # -- registration -----------------------------------------------------
    def _register(self, tag, shape, dtype):
        t = torch.zeros(shape, dtype=dtype, device=self.dev)
        handle = ctypes.create_string_buffer(self._hbytes)
        off = ctypes.c_size_t(0)
        _lib.check(self.lib.fpb_ipc_export(ctypes.c_void_p(t.data_ptr()), handle,
                                           ctypes.pointer(off)), "fpb_ipc_export")
        mine = (bytes(handle.raw), int(off.value), t.numel() * t.element_size())
        got = [None] * self.world
        self._dist.all_gather_object(got, mine, group=self.group)
        ptrs = []
        for r, (h, o, nbytes) in enumerate(got):
            if nbytes != mine[2]:
                raise RuntimeError(f"peer buffer {tag!r}: rank {r} registered {nbytes} bytes, "
                                   f"rank {self.rank} {mine[2]}")
            if r == self.rank:
                ptrs.append(t.data_ptr())
                continue
            base = self._opened.get(h)
            ptr = ctypes.c_void_p()
            if base is None:
                b = ctypes.c_void_p()
                _lib.check(self.lib.fpb_ipc_import(h, o, ctypes.pointer(b), ctypes.pointer(ptr)),
                           "fpb_ipc_import")
                self._opened[h] = base = b.value
            ptrs.append(base + o)
        self._bufs[(tag, shape, dtype)] = (t, ptrs)
        self._by_ptr[t.data_ptr()] = (tag, shape, dtype)
        return t, ptrs

    def _buffer(self, tag, shape, dtype):
        """The registered buffer of ``(tag, shape, dtype)``: one per distinct
        shape, so operators whose exchanges differ in shape (the outgoing and
        incoming TriMul) each keep theirs instead of re-registering."""
        shape = tuple(int(d) for d in shape)
        ent = self._bufs.get((tag, shape, dtype))
        if ent is None:
            ent = self._register(tag, shape, dtype)
        return ent

    def owner_buffer(self, tag: str, shape, dtype):
        """Registered buffer of this rank plus every rank's address of its
        own (``(tensor, [pointer per rank])``), for kernels that store
        straight at the owners."""
        return self._buffer(tag, shape, dtype)

    def recv_buffer(self, tag: str, like: torch.Tensor) -> torch.Tensor:
        """Registered buffer shaped like ``like`` (collective on first use of
        ``tag`` or a new shape); filled in place by the exchanges."""
        return self._buffer(tag, like.shape, like.dtype)[0]

    def _target(self, out):
        key = self._by_ptr.get(out.data_ptr())
        if key is not None and self._bufs[key][0].numel() == out.numel():
            return self._bufs[key], False
        return self._buffer("scratch", (out.numel(),), out.dtype), True

    # -- ordering ---------------------------------------------------------
    def barrier(self) -> None:
        """Stream-ordered barrier: work queued on every rank's current stream
        before it is complete once it returns on any stream after it."""
        self._dist.all_reduce(self._tick, group=self.group)

    def _scatter(self, copies):
        """``copies``: ``(peer, dst_ptr, src_ptr, nbytes)``. One kernel on the
        current stream (``fpb_peer_scatter``) writes every peer's block side
        by side; a copy that is not 16-byte aligned goes through the copy
        engine on the same stream instead."""
        cur = self._stream()
        fast = [(d, s, b) for _, d, s, b in copies
                if b and d != s and not (d | s | b) & 15]
        slow = [(d, s, b) for _, d, s, b in copies
                if b and d != s and (d | s | b) & 15]
        for i in range(0, len(fast), 16):
            part = fast[i:i + 16]
            k = len(part)
            _lib.check(self.lib.fpb_peer_scatter(
                (ctypes.c_void_p * k)(*[s for _, s, _ in part]),
                (ctypes.c_void_p * k)(*[d for d, _, _ in part]),
                (ctypes.c_size_t * k)(*[b for _, _, b in part]), k, cur), "fpb_peer_scatter")
        for d, s, b in slow:
            _lib.check(self.lib.fpb_copy_async(ctypes.c_void_p(d), ctypes.c_void_p(s), b, cur),
                       "fpb_copy_async")

    def _order(self):
        return [(self.rank + k) % self.world for k in range(self.world)]

    # -- collectives ------------------------------------------------------
    # ``fresh=True``: the caller's schedule guarantees that every rank's
    # reads of the destination buffers' previous contents were queued before
    # a barrier that has since been passed (typically the closing barrier of
    # a later exchange), so the opening barrier is skipped. The closing
    # barrier is always issued.
    def all_to_all(self, out: torch.Tensor, inp: torch.Tensor, *, fresh: bool = False) -> None:
        self.all_to_all_many([(out, inp)], fresh=fresh)

    def all_to_all_many(self, pairs, *, fresh: bool = False) -> None:
        """Several all-to-alls ``(out, inp)`` in one kernel and one barrier."""
        copies, backs = [], []
        for out, inp in pairs:
            (buf, ptrs), copy_back = self._target(out)
            inp = inp.contiguous()
            m = inp.numel() * inp.element_size() // self.world
            copies += [(d, ptrs[d] + self.rank * m, inp.data_ptr() + d * m, m)
                       for d in self._order()]
            if copy_back:
                backs.append((out, buf))
        if not fresh:
            self.barrier()
        self._scatter(copies)
        self.barrier()
        for out, buf in backs:
            out.view(-1).copy_(buf)

    def all_gather(self, out: torch.Tensor, inp: torch.Tensor, *, fresh: bool = False) -> None:
        (buf, ptrs), copy_back = self._target(out)
        inp = inp.contiguous()
        m = inp.numel() * inp.element_size()
        if not fresh:
            self.barrier()
        self._scatter([(d, ptrs[d] + self.rank * m, inp.data_ptr(), m) for d in self._order()])
        self.barrier()
        if copy_back:
            out.view(-1).copy_(buf)

    def reduce_scatter(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        """NCCL's reduce-scatter (the row scheme's incoming TriMul)."""
        self._dist.reduce_scatter_tensor(out.view(-1), inp.reshape(-1),
                                         op=self._dist.ReduceOp.SUM, group=self.group)

    def _stream(self) -> int:
        return ops._stream_ptr(self.dev) if self.dev.type == "cuda" else 0

    def transpose_rows(self, z_loc, shard: RowShard, out=None, tag="transpose", *,
                       fresh: bool = False):
        """``transpose_rows`` in one kernel over peer memory (see there)."""
        c, n, ch = shard.chunk, shard.n, z_loc.shape[-1]
        words = ch * z_loc.element_size() // 4  # the kernel moves 4-byte words
        if not z_loc.is_contiguous() or (ch * z_loc.element_size()) % 16:
            raise ValueError("peer transpose takes a contiguous [chunk, n, c] tensor whose "
                             "rows are a multiple of 16 bytes")
        buf, ptrs = self._buffer(tag, (c, n, ch), z_loc.dtype)
        arr = (ctypes.c_void_p * self.world)(*ptrs)
        if not fresh:
            self.barrier()
        _lib.check(self.lib.fpb_peer_transpose_rows(
            ctypes.c_void_p(z_loc.data_ptr()), n, c, words, self.rank, self.world, arr,
            self._stream()), "fpb_peer_transpose_rows")
        self.barrier()
        if out is None:
            return buf
        out[:shard.rows].copy_(buf[:shard.rows])
        return out

    def close(self) -> None:
        """Unmap every peer buffer (after a device synchronise)."""
        for base in self._opened.values():
            self.lib.fpb_ipc_close(ctypes.c_void_p(base))
        self._opened.clear()
        self._bufs.clear()
        self._by_ptr.clear()


def _recv_like(comm, tag: str, like: torch.Tensor) -> torch.Tensor:
    """Receive buffer of an exchange: the transport's registered buffer when
    it has one (filled in place), else a fresh tensor."""
    get = getattr(comm, "recv_buffer", None)
    return torch.empty_like(like) if get is None else get(tag, like)


def gather_rows(z_loc: torch.Tensor, shard: RowShard, comm) -> torch.Tensor:
    """Full ``[n, n, c]`` pair tensor on every rank (tests and checkpoints)."""
    full = z_loc.new_empty((shard.world * shard.chunk,) + tuple(z_loc.shape[1:]))
    comm.all_gather(full, z_loc.contiguous())
    return full[:shard.n]


def transpose_rows(z_loc: torch.Tensor, shard: RowShard, comm, out=None, *,
                   fresh: bool = False) -> torch.Tensor:
    """Rows of ``z^T`` owned by this rank: ``zt[i, j] = z[j, i]`` for the
    rank's ``i``. One all-to-all of ``[chunk, chunk, c]`` blocks, packed and
    unpacked in one pass each; padded columns travel as zeros and padded rows
    of the result are zero. ``out``: optional ``[chunk, n, c]`` destination
    (may be ``z_loc`` itself: the send block is packed before it is written).
    A transport with its own ``transpose_rows`` (``PeerComm``) does it in one
    pass; its result without ``out`` is a registered buffer, valid until the
    next transpose into it; ``fresh`` as for ``PeerComm`` exchanges."""
    peer = getattr(comm, "transpose_rows", None)
    if peer is not None:
        return peer(z_loc, shard, out=out, tag="transpose" if out is None else "transpose_out",
                    fresh=fresh)
    w, c, n = shard.world, shard.chunk, shard.n
    ch = z_loc.shape[-1]
    send = z_loc.new_empty(w, c, c, ch)  # [dest][my i][dest j]
    for d in range(w):
        cols = max(0, min(c, n - d * c))
        if cols:
            send[d, :, :cols].copy_(z_loc[:, d * c:d * c + cols])
        if cols < c:
            send[d, :, cols:].zero_()
    recv = torch.empty_like(send)
    comm.all_to_all(recv, send)  # [src][src rows][my cols]
    del send
    res = z_loc.new_empty(c, n, ch) if out is None else out
    for src in range(w):
        rows = max(0, min(c, n - src * c))
        if rows:
            res[:, src * c:src * c + rows].copy_(recv[src, :rows].transpose(0, 1))
    return res


class CudaPhases:
    """Phase kernels of the row-sharded operators (C-ABI entry points).

    Buffers are allocated with torch on the current stream. Each phase keeps
    one workspace, reused by its later calls on the same stream (each call
    restarts its status word), so ``check()`` reports the latest call of
    every phase. ``stores_at_owners``: the TriMul projection and contraction
    can store straight into every rank's buffers (the peer transport's
    fused exchanges).
    """

    stores_at_owners = True

    def __init__(self, precision="strict", eps: float = 1e-5):
        self.p = ops.precision_code(precision)
        self.strict = self.p == ops.STRICT
        self.eps = float(eps)
        self.lib = _lib.load()
        self._ws = {}

    # ---------------------------------------------------------------- helpers
    def _dtype(self):
        return torch.float32 if self.strict else torch.bfloat16

    def _planes(self, rows, ld, device):
        n_planes = 2 if self.strict else 1
        return [torch.empty(128, rows, ld, dtype=self._dtype(), device=device)
                for _ in range(n_planes)]

    def _ws_take(self, name, nbytes, device):
        ws = self._ws.get(name)
        if ws is None or ws.numel() < nbytes or ws.device != device:
            ws = ops.workspace(nbytes, device)
            self._ws[name] = ws
        return ws

    @staticmethod
    def _ptr(t):
        return 0 if t is None else t.data_ptr()

    def _pair(self, planes):
        return planes[0].data_ptr(), (planes[1].data_ptr() if self.strict else 0)

    # ---------------------------------------------------------------- TriMul
    def trimul_proj(self, z_loc, mask, shard: RowShard, outgoing: bool, w: dict):
        """Gated, masked a/b planes of the rank's rows: outgoing ``[128][chunk][ld(n)]``
        (the b planes are the all-gather chunk; in strict mode one unsplit FP32
        plane, split after the gather: half the bytes), incoming
        ``[128][n][ld(rows)]``."""
        n, rows = shard.n, shard.rows
        dev = z_loc.device
        if outgoing:
            ld = int(self.lib.fpb_trimul_plane_ld(n, self.p))
            plane_rows = shard.chunk
        else:
            if rows == 0:
                return None, None, 0
            ld = int(self.lib.fpb_trimul_plane_ld(rows, self.p))
            plane_rows = n
        a = self._planes(plane_rows, ld, dev)
        if outgoing and self.strict:
            b = [torch.empty(128, plane_rows, ld, dtype=torch.float32, device=dev)]
        else:
            b = self._planes(plane_rows, ld, dev)
        if rows == 0:
            return a, b, ld
        ws = self._ws_take("trimul_proj", self.lib.fpb_trimul_shard_workspace_size(self.p), dev)
        keys = ("ln_in_w", "ln_in_b", "w_a_p", "w_a_g", "w_b_p", "w_b_g")
        wt = [w[k].contiguous() for k in keys]
        _lib.check(self.lib.fpb_trimul_shard_proj(
            z_loc.data_ptr(), self._ptr(mask), n, rows, shard.r0, int(not outgoing),
            *[t.data_ptr() for t in wt], self.eps, *self._pair(a), b[0].data_ptr(),
            (b[1].data_ptr() if len(b) > 1 else 0), ld, plane_rows,
            self.p, ws.data_ptr(), ws.numel(), ops._stream_ptr(dev)), "fpb_trimul_shard_proj")
        return a, b, ld

    def new_x(self, rows: int, shard: RowShard, device):
        njb = (shard.n + 127) // 128
        return torch.empty(rows, njb, 128, 128, dtype=self._dtype(), device=device)

    def _contract(self, a, m, a_plane_rows, b, nn, b_chunk_rows, b_chunks, b_chunk_stride, k,
                  ld, x, device):
        ws = self._ws_take("trimul_contract", 256, device)
        _lib.check(self.lib.fpb_trimul_shard_contract(
            *self._pair(a), m, a_plane_rows, *self._pair(b), nn, b_chunk_rows, b_chunks,
            b_chunk_stride, k, ld, x.data_ptr(), self.p, ws.data_ptr(), ws.numel(),
            ops._stream_ptr(device)), "fpb_trimul_shard_contract")

    def trimul_contract_out(self, a, b_full, shard: RowShard, ld):
        """Local rows of ``x = a b^T`` with ``b_full`` the gathered chunks
        (strict: unsplit FP32, split in place into hi + a new lo here)."""
        dev = b_full[0].device
        if self.strict and len(b_full) == 1:
            hi = b_full[0]
            lo = torch.empty_like(hi)
            _lib.check(self.lib.fpb_split_tf32(hi.data_ptr(), hi.data_ptr(), lo.data_ptr(),
                                               hi.numel(), ops._stream_ptr(dev)),
                       "fpb_split_tf32")
            b_full = [hi, lo]
        x = self.new_x(shard.chunk, shard, dev)
        if shard.rows:
            self._contract(a, shard.rows, shard.chunk, b_full, shard.n, shard.chunk, shard.world,
                           b_full[0][0].numel(), shard.n, ld, x, dev)
        return x

    def trimul_contract_in(self, a, b, shard: RowShard, ld, device):
        """Partial ``x = a^T b`` over the rank's k rows, all ``world*chunk`` rows
        (padding rows zero), ready for the reduce-scatter."""
        x = self.new_x(shard.world * shard.chunk, shard, device)
        if shard.rows:
            self._contract(a, shard.n, shard.n, b, shard.n, shard.n, 1, 0, shard.rows, ld, x,
                           device)
            x[shard.n:].zero_()
        else:
            x.zero_()
        return x

    def trimul_finish(self, z_loc, shard: RowShard, x_loc, w: dict, add: bool):
        if shard.rows == 0:
            return
        dev = z_loc.device
        ws = self._ws_take("trimul_finish", self.lib.fpb_trimul_shard_workspace_size(self.p), dev)
        keys = ("ln_in_w", "ln_in_b", "w_g", "ln_out_w", "ln_out_b", "w_z")
        wt = [w[k].contiguous() for k in keys]
        _lib.check(self.lib.fpb_trimul_shard_finish(
            z_loc.data_ptr(), shard.n, shard.rows, x_loc.data_ptr(), *[t.data_ptr() for t in wt],
            self.eps, int(bool(add)), self.p, ws.data_ptr(), ws.numel(), ops._stream_ptr(dev)),
            "fpb_trimul_shard_finish")

    # ---------------------------------------------------------------- TriAttn
    def triattn_bias_buffer(self, shard: RowShard, device):
        """Row-blocked pair bias for ``world*chunk`` rows, viewed ``[rows, 4*ldb]``:
        a rank's ``chunk`` rows (a multiple of 32) are one contiguous range."""
        ldb = int(self.lib.fpb_triattn_bias_ld(shard.n))
        return torch.empty(shard.world * shard.chunk, 4 * ldb, dtype=torch.float32,
                           device=device)

    def triattn_proj(self, z_loc, mask, shard: RowShard, w: dict, bias_full):
        if shard.rows == 0:
            return None
        dev = z_loc.device
        ws = self._ws_take("triattn", self.lib.fpb_triattn_shard_workspace_size(
            shard.n, shard.rows, self.p, int(mask is not None)), dev)
        wt = [None if w.get(k) is None else w[k].contiguous()
              for k in ("ln_w", "ln_b", "w_q", "w_k", "w_v", "w_bias", "w_g", "b_g")]
        _lib.check(self.lib.fpb_triattn_shard_proj(
            z_loc.data_ptr(), self._ptr(mask), shard.n, shard.rows, shard.r0,
            *[self._ptr(t) for t in wt], self.eps, bias_full.data_ptr(), self.p, ws.data_ptr(),
            ws.numel(), ops._stream_ptr(dev)), "fpb_triattn_shard_proj")
        return ws

    def triattn_finish(self, z_loc, shard: RowShard, with_mask: bool, bias_full, w: dict, state):
        if shard.rows == 0:
            return
        ws = state
        keep = [None if w.get(k) is None else w[k].contiguous() for k in ("w_o", "b_o")]
        _lib.check(self.lib.fpb_triattn_shard_finish(
            z_loc.data_ptr(), 0, shard.n, shard.rows, int(bool(with_mask)), bias_full.data_ptr(),
            *[self._ptr(t) for t in keep], self.p, ws.data_ptr(), ws.numel(),
            ops._stream_ptr(z_loc.device)), "fpb_triattn_shard_finish")

    # ---------------------------------------------------------------- transition
    def transition(self, z_loc, shard: RowShard, w: dict):
        if shard.rows == 0:
            return
        ws = self._ws_take("transition", self.lib.fpb_transition_workspace_size(128, 4, self.p),
                           z_loc.device)
        keys = ("ln_w", "ln_b", "w_a", "w_b", "w_out")
        wt = [w[k].contiguous() for k in keys]
        _lib.check(self.lib.fpb_transition(
            z_loc.data_ptr(), 0, shard.rows * shard.n, 128, 4, *[t.data_ptr() for t in wt],
            self.eps, self.p, ws.data_ptr(), ws.numel(), ops._stream_ptr(z_loc.device)),
            "fpb_transition")

    # ---------------------------------------------------------- single stack
    def single_block(self, s, z_loc, mask, shard: RowShard, w: dict):
        """``s [n, 384]`` (every row) += the single stack on the rank's rows;
        ``z_loc`` holds the rank's pair rows."""
        if shard.rows == 0:
            return
        from .modules import SingleBlockWeights, _fill
        key = tuple((k, t.data_ptr(), t._version) for k, t in w.items())
        cached = self._ws.get("_single_weights")
        if cached is None or cached[0] != key:
            keep: list = []
            cw = SingleBlockWeights()
            _fill(cw, w, keep)
            cached = (key, cw, keep)
            self._ws["_single_weights"] = cached
        ws = self._ws_take("single", self.lib.fpb_single_block_workspace_size(
            shard.n, shard.rows, 384), s.device)
        ops.single_block(s, z_loc[:shard.rows], mask, cached[1], r0=shard.r0, precision=self.p,
                         eps=self.eps, workspace=ws)

    # ------------------------------------------------ TriMul, channel groups
    def trimul_group_plane(self, shard: RowShard, outgoing: bool):
        """``(rows_p, ld)`` of the channel-group a/b planes (see
        ``trimul_proj_groups``)."""
        if outgoing:
            return shard.chunk, int(self.lib.fpb_trimul_plane_ld(shard.n, self.p))
        return shard.n, int(self.lib.fpb_trimul_plane_ld(shard.chunk, self.p))

    def trimul_proj_groups(self, z_loc, mask, shard: RowShard, outgoing: bool, w: dict,
                           a_owner=None, b_owner=None):
        """Gated, masked a/b planes of the rank's rows, unsplit (FP32 strict,
        BF16 fast) and channel-first ``[128][rows_p][ld]``, so that channel
        group ``g`` is the ``g``-th contiguous block of the all-to-all:
        outgoing ``rows_p = chunk``, ``ld = ld(n)``; incoming ``rows_p = n``,
        ``ld = ld(chunk)`` with the columns past the rank's rows zero (they
        are terms of the concatenated contraction index). With ``a_owner`` /
        ``b_owner`` (every rank's ``[world][G][rows_p][ld]`` receive buffer,
        zero where no rank writes) group ``g`` is stored straight into block
        ``rank`` of rank ``g``'s buffers and ``(None, None, ld)`` returned."""
        n, rows, chunk = shard.n, shard.rows, shard.chunk
        dev = z_loc.device
        plane_rows, ld = self.trimul_group_plane(shard, outgoing)
        if a_owner is not None:
            # stored straight into every rank's receive buffers
            if rows:
                ws = self._ws_take("trimul_proj",
                                   self.lib.fpb_trimul_shard_workspace_size(self.p), dev)
                keys = ("ln_in_w", "ln_in_b", "w_a_p", "w_a_g", "w_b_p", "w_b_g")
                wt = [w[k].contiguous() for k in keys]
                W = shard.world
                _lib.check(self.lib.fpb_trimul_shard_proj_scatter(
                    z_loc.data_ptr(), self._ptr(mask), n, rows, shard.r0, int(not outgoing),
                    *[t.data_ptr() for t in wt], self.eps, (ctypes.c_void_p * W)(*a_owner),
                    (ctypes.c_void_p * W)(*b_owner), W, shard.rank, ld, plane_rows, self.p,
                    ws.data_ptr(), ws.numel(), ops._stream_ptr(dev)),
                    "fpb_trimul_shard_proj_scatter")
            return None, None, ld
        a = torch.empty(128, plane_rows, ld, dtype=self._dtype(), device=dev)
        b = torch.empty_like(a)
        if rows:
            ws = self._ws_take("trimul_proj", self.lib.fpb_trimul_shard_workspace_size(self.p),
                               dev)
            keys = ("ln_in_w", "ln_in_b", "w_a_p", "w_a_g", "w_b_p", "w_b_g")
            wt = [w[k].contiguous() for k in keys]
            _lib.check(self.lib.fpb_trimul_shard_proj(
                z_loc.data_ptr(), self._ptr(mask), n, rows, shard.r0, int(not outgoing),
                *[t.data_ptr() for t in wt], self.eps, a.data_ptr(), 0, b.data_ptr(), 0, ld,
                plane_rows, self.p, ws.data_ptr(), ws.numel(), ops._stream_ptr(dev)),
                "fpb_trimul_shard_proj")
        if not outgoing and rows < chunk:
            a[:, :, rows:chunk].zero_()
            b[:, :, rows:chunk].zero_()
        return a, b, ld

    def _split(self, t):
        """Strict: ``[t (now hi), lo]`` split in place; fast: ``[t]``."""
        if not self.strict:
            return [t]
        lo = torch.empty_like(t)
        _lib.check(self.lib.fpb_split_tf32(t.data_ptr(), t.data_ptr(), lo.data_ptr(), t.numel(),
                                           ops._stream_ptr(t.device)), "fpb_split_tf32")
        return [t, lo]

    def trimul_contract_groups(self, ra, rb, shard: RowShard, outgoing: bool, ld: int,
                               x_owner=None):
        """This rank's channel group contracted over the whole grid. ``ra``,
        ``rb``: the received ``[world][G][rows_p][ld]`` blocks. Returns x
        blocked ``[world * chunk][njb][G][128]``; rows ``[r * chunk, (r + 1) *
        chunk)`` are rank ``r``'s (the send block of the return all-to-all).
        With ``x_owner`` (rank ``r``'s ``[chunk][njb][128][128]`` x buffer
        address, for every rank) the rows are stored at their owners instead,
        in this rank's channel group, and nothing is returned."""
        W, n, chunk = shard.world, shard.n, shard.chunk
        G = 128 // W
        dev = ra.device
        def gather(r, rows, seg, cols_mode, dst_rows, dst_ld):
            # reorder + hi/lo split (strict) of a received block, one pass
            out = [torch.empty(G, dst_rows, dst_ld, dtype=r.dtype, device=dev)
                   for _ in range(2 if self.strict else 1)]
            _lib.check(self.lib.fpb_trimul_group_gather(
                r.data_ptr(), W, G, rows, ld, seg, cols_mode, out[0].data_ptr(),
                out[1].data_ptr() if self.strict else 0, dst_ld, self.p,
                ops._stream_ptr(dev)), "fpb_trimul_group_gather")
            return out

        if outgoing:
            # A: the row blocks of every rank stacked; B: read as W chunks
            a_op = gather(ra, chunk, ld, 0, W * chunk, ld)
            b_op = self._split(rb)
            geo = dict(m=n, a_rows=W * chunk, nn=n, b_chunk_rows=chunk, b_chunks=W,
                       b_chunk_stride=G * chunk * ld, k=n, ld=ld)
        else:
            # the contraction index k runs over every rank's rows: concatenate
            # the ranks' column blocks
            ldk = int(self.lib.fpb_trimul_plane_ld(W * chunk, self.p))
            a_op = gather(ra, n, chunk, 1, n, ldk)
            b_op = gather(rb, n, chunk, 1, n, ldk)
            geo = dict(m=n, a_rows=n, nn=n, b_chunk_rows=n, b_chunks=1, b_chunk_stride=0,
                       k=W * chunk, ld=ldk)
        ws = self._ws_take("trimul_contract", 256, dev)
        if x_owner is not None:
            _lib.check(self.lib.fpb_trimul_group_contract_scatter(
                *self._pair(a_op), geo["m"], geo["a_rows"], *self._pair(b_op), geo["nn"],
                geo["b_chunk_rows"], geo["b_chunks"], geo["b_chunk_stride"], geo["k"], geo["ld"],
                G, (ctypes.c_void_p * W)(*x_owner), W, chunk, shard.rank * G, self.p,
                ws.data_ptr(), ws.numel(), ops._stream_ptr(dev)),
                "fpb_trimul_group_contract_scatter")
            return None
        x = torch.empty(W * chunk, (n + 127) // 128, G, 128, dtype=self._dtype(), device=dev)
        _lib.check(self.lib.fpb_trimul_group_contract(
            *self._pair(a_op), geo["m"], geo["a_rows"], *self._pair(b_op), geo["nn"],
            geo["b_chunk_rows"], geo["b_chunks"], geo["b_chunk_stride"], geo["k"], geo["ld"], G,
            x.data_ptr(), self.p, ws.data_ptr(), ws.numel(), ops._stream_ptr(dev)),
            "fpb_trimul_group_contract")
        return x

    def trimul_ungroup_x(self, rx, shard: RowShard):
        """The rank's x rows ``[chunk][njb][128][128]`` from the received
        ``[world][chunk][njb][G][128]`` (block ``g``: channel group ``g``)."""
        W, chunk = shard.world, shard.chunk
        njb = (shard.n + 127) // 128
        return (rx.view(W, chunk, njb, 128 // W, 128).permute(1, 2, 0, 3, 4)
                .reshape(chunk, njb, 128, 128))

    def check(self) -> None:
        """Raise if any wait of any phase kernel gave up (reads status words)."""
        for name, ws in self._ws.items():
            if name.startswith("_"):
                continue
            st = ops.workspace_status(ws)
            if st:
                raise RuntimeError(f"{name} phase kernel status {st}")


# ---------------------------------------------------------------------------
# rank-local orchestration (every rank runs the same collective sequence)
# ---------------------------------------------------------------------------
TRIMUL_SCHEMES = ("rows", "channels")


def trimul_scheme(world: int, transport: str = "nccl") -> str:
    """Exchange scheme of the TriMul contraction for ``world`` ranks. Per rank
    and operator the row scheme moves ``(W-1)/W`` of the full ``n x n x 128``
    planes (the all-gather of ``b`` or the reduce-scatter of ``x``); the
    channel scheme moves ``(W-1)/W`` of three rank shares (``a``, ``b`` and
    ``x``, each ``1/W`` of the planes), ``3/W`` of it, and splits only its own
    group for the strict operands. Over NCCL: channels from four ranks up;
    over peer memory (``transport="peer"``), where the projection and the
    contraction store their outputs straight at the owners, channels from
    two ranks up. Both need the 128 channels to divide evenly."""
    if 128 % world:
        return "rows"
    return "channels" if world >= (2 if transport == "peer" else 4) else "rows"


def _trimul_channels(z_loc, mask, w, shard, comm, phases, outgoing, add):
    owners = getattr(comm, "owner_buffer", None)
    if owners is not None and getattr(phases, "stores_at_owners", False):
        # Peer transport: the projection stores a / b straight into the
        # owners' receive buffers and the contraction stores each x row at
        # its owner, so both exchanges ride on the kernels' own stores. The
        # receive buffers were last read by the contraction of an earlier
        # call of this direction and the x buffers by the finish of an
        # earlier call; every call closes its projection and its contraction
        # with a barrier, after any earlier reader, so no opening barriers.
        rows_p, ld = phases.trimul_group_plane(shard, outgoing)
        dtype = phases._dtype()
        ra, pa = owners("trimul_a", (128, rows_p, ld), dtype)
        rb, pb = owners("trimul_b", (128, rows_p, ld), dtype)
        phases.trimul_proj_groups(z_loc, mask, shard, outgoing, w, a_owner=pa, b_owner=pb)
        comm.barrier()
        njb = (shard.n + 127) // 128
        x_loc, px = owners("trimul_x", (shard.chunk, njb, 128, 128), dtype)
        phases.trimul_contract_groups(ra, rb, shard, outgoing, ld, x_owner=px)
        comm.barrier()
        phases.trimul_finish(z_loc, shard, x_loc, w, add)
        return z_loc
    a, b, ld = phases.trimul_proj_groups(z_loc, mask, shard, outgoing, w)
    ra = _recv_like(comm, "trimul_a", a)
    rb = _recv_like(comm, "trimul_b", b)
    comm.all_to_all(ra, a)
    del a
    comm.all_to_all(rb, b)
    del b
    xg = phases.trimul_contract_groups(ra, rb, shard, outgoing, ld)
    del ra, rb
    rx = _recv_like(comm, "trimul_x", xg)
    comm.all_to_all(rx, xg)
    del xg
    phases.trimul_finish(z_loc, shard, phases.trimul_ungroup_x(rx, shard), w, add)
    return z_loc


def sharded_trimul(z_loc, mask, w: dict, shard: RowShard, comm, phases, *, outgoing: bool,
                   add: bool = True, scheme: str | None = None):
    """Triangle multiplicative update of the rank's rows, in place on ``z_loc``.
    ``scheme``: ``"rows"`` or ``"channels"`` (default ``trimul_scheme``)."""
    if scheme is None:
        scheme = trimul_scheme(shard.world, "peer" if isinstance(comm, PeerComm) else "nccl")
    if scheme not in TRIMUL_SCHEMES:
        raise ValueError(f"unknown TriMul scheme {scheme!r}")
    if scheme == "channels":
        if 128 % shard.world:
            raise ValueError(f"channel scheme needs 128 % world == 0 (world={shard.world})")
        return _trimul_channels(z_loc, mask, w, shard, comm, phases, outgoing, add)
    a, b, ld = phases.trimul_proj(z_loc, mask, shard, outgoing, w)
    if outgoing:
        b_full = []
        for i, t in enumerate(b):
            full = _recv_like(comm, f"trimul_b_full{i}", t.new_empty((shard.world,) + tuple(t.shape)))
            comm.all_gather(full, t)
            b_full.append(full)
        x_loc = phases.trimul_contract_out(a, b_full, shard, ld)
    else:
        x_full = phases.trimul_contract_in(a, b, shard, ld, z_loc.device)
        x_loc = phases.new_x(shard.chunk, shard, z_loc.device)
        comm.reduce_scatter(x_loc, x_full)
    phases.trimul_finish(z_loc, shard, x_loc, w, add)
    return z_loc


def sharded_triattn(z_loc, mask, w: dict, shard: RowShard, comm, phases, *,
                    starting: bool = True):
    """Triangle attention update added to the rank's rows of ``z_loc``."""
    if not starting:
        # Peer transport: the forward destination was last read by an
        # earlier call's attention and backward transpose, the backward
        # destination by an earlier call's copy out of it; the backward
        # transpose and this call's forward transpose close with barriers
        # after those reads, so neither transpose needs an opening barrier.
        zt = transpose_rows(z_loc, shard, comm, fresh=True)
        mt = None if mask is None else mask.transpose(0, 1).contiguous()
        sharded_triattn(zt, mt, w, shard, comm, phases, starting=True)
        transpose_rows(zt, shard, comm, out=z_loc, fresh=True)
        return z_loc
    bias_full = _recv_like(comm, "triattn_bias", phases.triattn_bias_buffer(shard, z_loc.device))
    state = phases.triattn_proj(z_loc, mask, shard, w, bias_full)
    own = bias_full[shard.rank * shard.chunk:(shard.rank + 1) * shard.chunk]
    comm.all_gather(bias_full, own.clone())
    phases.triattn_finish(z_loc, shard, mask is not None, bias_full, w, state)
    return z_loc


def sharded_pair_block(z_loc, mask, weights: dict, shard: RowShard, comm, phases, *,
                       scheme: str | None = None):
    """Pair stack of one Pairformer block on the rank's rows (AF3 Algorithm 17
    order): TriMul out, TriMul in, TriAttn start, TriAttn end, transition.
    ``weights`` maps ``tri_mul_out, tri_mul_in, tri_att_start, tri_att_end,
    pair_transition`` to the operators' weight dicts; ``scheme`` the TriMul
    exchange scheme (default ``trimul_scheme`` for the world and transport)."""
    sharded_trimul(z_loc, mask, weights["tri_mul_out"], shard, comm, phases, outgoing=True,
                   scheme=scheme)
    sharded_trimul(z_loc, mask, weights["tri_mul_in"], shard, comm, phases, outgoing=False,
                   scheme=scheme)
    sharded_triattn(z_loc, mask, weights["tri_att_start"], shard, comm, phases, starting=True)
    sharded_triattn(z_loc, mask, weights["tri_att_end"], shard, comm, phases, starting=False)
    phases.transition(z_loc, shard, weights["pair_transition"])
    return z_loc


def single_buffer(s: torch.Tensor, shard: RowShard) -> torch.Tensor:
    """``[W * chunk, 384]`` buffer holding ``s`` in its first ``n`` rows: the
    all-gather target of ``sharded_single_block``."""
    buf = s.new_zeros((shard.world * shard.chunk, s.shape[1]))
    buf[:shard.n] = s
    return buf


def sharded_single_block(s_buf, z_loc, mask, w: dict, shard: RowShard, comm, phases):
    """Single stack of one Pairformer block on the rank's query rows, then an
    all-gather of the updated rows so that every rank holds all of ``s``.
    ``s_buf`` is a ``single_buffer`` (rows past ``n`` are padding); ``w`` is
    ``PairformerSingleBlock.weight_dict()``. Keys and values read every row
    of ``s``, which is why ``s`` is replicated rather than sharded."""
    phases.single_block(s_buf[:shard.n], z_loc, mask, shard, w)
    local = s_buf[shard.r0:shard.r0 + shard.chunk].clone()
    comm.all_gather(s_buf, local)
    return s_buf


def block_weight_dicts(block) -> dict:
    """Weight dicts of a ``modules.PairformerPairBlock`` for ``sharded_pair_block``."""
    return {name: getattr(block, name).weight_dict()
            for name in ("tri_mul_out", "tri_mul_in", "tri_att_start", "tri_att_end",
                         "pair_transition")}
