"""Host logic of the peer-memory transport (``sharded.PeerComm``) on CPU.

Ranks are threads of one process, so a peer "mapping" is the buffer's own
address: a stand-in library exports a buffer's address as its IPC handle,
imports it back, and runs the peer copy and transpose entry points as host
memory moves with the same argument contract as the CUDA ones; a stand-in
process group gives every thread its rank and implements the object
all-gather, the barrier all-reduce and the reduce-scatter over threads.
What is checked: buffer registration and the handle exchange, the pointer
tables, the segment arithmetic of the all-to-all and all-gather, the
transpose, the opening / closing barriers (``fresh``), and the whole
sharded block through the transport against the single-device oracle (the
phase math is ``tests/sharded_util.OraclePhases``, float64, tolerance
1e-10)."""
import ctypes
import threading

import numpy as np
import pytest
import torch

from fireprot_b200 import sharded as S
from oracle import pairformer_oracle as O

from sharded_util import OraclePhases, oracle_weight_dicts, single_weight_dict

TOL = 1e-10


class Hub:
    def __init__(self, world):
        self.world = world
        self.barrier = threading.Barrier(world, timeout=120)
        self.slots = [None] * world
        self.barriers = [0] * world


class FakeDist:
    """One rank's view of a thread process group."""

    class ReduceOp:
        SUM = "sum"

    def __init__(self, hub, rank):
        self.hub, self.rank = hub, rank

    def get_world_size(self, group=None):
        return self.hub.world

    def get_rank(self, group=None):
        return self.rank

    def _exchange(self, obj):
        h = self.hub
        h.slots[self.rank] = obj
        h.barrier.wait()
        got = list(h.slots)
        h.barrier.wait()
        return got

    def all_gather_object(self, out, obj, group=None):
        out[:] = self._exchange(obj)

    def all_reduce(self, t, group=None):
        self.hub.barriers[self.rank] += 1
        self._exchange(None)

    def reduce_scatter_tensor(self, out, inp, op=None, group=None):
        got = self._exchange(inp.clone())
        acc = sum(g.view(self.hub.world, -1)[self.rank] for g in got)
        out.copy_(acc)


def _floats(addr, count):
    return np.ctypeslib.as_array((ctypes.c_float * count).from_address(addr))


class FakePeerLib:
    """The peer entry points as host-memory moves (threads share memory)."""

    def __init__(self):
        self.closed = []

    def fpb_ipc_handle_bytes(self):
        return 16

    def fpb_ipc_export(self, ptr, handle, off_ptr):
        ctypes.memmove(handle, (ctypes.c_uint64 * 2)(ptr.value, 0), 16)
        off_ptr.contents.value = 0
        return 0

    def fpb_ipc_import(self, handle, off, base_ptr, ptr_ptr):
        base = int.from_bytes(bytes(handle)[:8], "little")
        base_ptr.contents.value = base
        ptr_ptr.contents.value = base + off
        return 0

    def fpb_ipc_close(self, base):
        self.closed.append(base.value)
        return 0

    def fpb_copy_async(self, dst, src, nbytes, stream):
        ctypes.memmove(dst.value, src.value, nbytes)
        return 0

    def fpb_peer_scatter(self, srcs, dsts, sizes, count, stream):
        assert 0 < count <= 16
        for k in range(count):
            assert srcs[k] % 16 == 0 and dsts[k] % 16 == 0 and sizes[k] % 16 == 0
            ctypes.memmove(dsts[k], srcs[k], sizes[k])
        return 0

    def fpb_peer_transpose_rows(self, z, n, chunk, ch, rank, world, dst, stream):
        r0 = rank * chunk
        rows = max(0, min(chunk, n - r0))
        if rows == 0:
            return 0
        src = _floats(z.value, rows * n * ch).reshape(rows, n, ch)
        for d in range(world):
            j0 = d * chunk
            cols = max(0, min(chunk, n - j0))
            if cols == 0:
                continue
            out = _floats(dst[d], chunk * n * ch).reshape(chunk, n, ch)
            out[:cols, r0:r0 + rows] = src[:, j0:j0 + cols].transpose(1, 0, 2)
        return 0

    def fpb_status_string(self, status):
        return b"error"


def run_ranks(world, fn):
    hub, lib = Hub(world), FakePeerLib()
    results, errors = [None] * world, []

    def body(r):
        try:
            comm = S.PeerComm(dist=FakeDist(hub, r), lib=lib, device="cpu")
            results[r] = fn(r, comm)
            comm.close()
        except BaseException as e:  # noqa: BLE001 - surfaced below
            errors.append(e)
            hub.barrier.abort()

    threads = [threading.Thread(target=body, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    if errors:
        raise errors[0]
    return results, hub, lib


@pytest.mark.parametrize("world", [1, 2, 3, 4])
def test_peer_comm_exchanges(world):
    g = torch.Generator().manual_seed(world)
    per = 12  # float32 elements per rank block (48 bytes: 16-byte multiples)
    sends = [torch.randn(world * per, generator=g) for _ in range(world)]
    owns = [torch.randn(per, generator=g) for _ in range(world)]

    def rank_fn(r, comm):
        # all-to-all into a registered buffer (filled in place) ...
        recv = comm.recv_buffer("a2a", sends[r])
        comm.all_to_all(recv, sends[r])
        a2a = recv.clone()
        # ... and into a plain tensor (through the scratch buffer)
        plain = torch.empty_like(sends[r])
        comm.all_to_all(plain, sends[r], fresh=False)
        full = torch.empty(world * per)
        comm.all_gather(full, owns[r])
        return a2a, plain, full

    res, hub, lib = run_ranks(world, rank_fn)
    for r, (a2a, plain, full) in enumerate(res):
        want = torch.cat([sends[s].view(world, per)[r] for s in range(world)])
        assert torch.equal(a2a, want) and torch.equal(plain, want)
        assert torch.equal(full, torch.cat(owns))
    # opening + closing barrier per exchange, three exchanges
    assert hub.barriers == [6] * world
    # every imported peer segment is unmapped by close()
    assert len(lib.closed) == world * (world - 1) * 2  # "a2a" and the scratch buffer


@pytest.mark.parametrize("n,world,dtype", [(40, 2, torch.float32), (70, 3, torch.float64),
                                           (33, 4, torch.float32), (33, 8, torch.float64)])
def test_peer_comm_transpose(n, world, dtype):
    z = torch.randn(n, n, 8, generator=torch.Generator().manual_seed(n)).to(dtype)

    def rank_fn(r, comm):
        sh = S.shard_plan(n, world, r)
        zl = S.local_rows(z, sh)
        zt = S.transpose_rows(zl, sh, comm, fresh=True)
        got_t = zt.clone()
        back = torch.zeros_like(zl)
        S.transpose_rows(zt, sh, comm, out=back, fresh=True)
        return sh, got_t, back

    res, hub, _ = run_ranks(world, rank_fn)
    for sh, zt, back in res:
        assert torch.equal(zt[:sh.rows], z.transpose(0, 1)[sh.r0:sh.r0 + sh.rows])
        assert not zt[sh.rows:].any()  # padding rows of the registered buffer stay zero
        assert torch.equal(back[:sh.rows], z[sh.r0:sh.r0 + sh.rows])
    assert hub.barriers == [2] * world  # fresh: closing barriers only


def test_peer_comm_rejects_unaligned_transpose_rows():
    def rank_fn(r, comm):
        sh = S.shard_plan(8, 1, 0)
        with pytest.raises(ValueError):
            S.transpose_rows(torch.zeros(32, 8, 3), sh, comm)  # 12-byte pair rows
    run_ranks(1, rank_fn)


@pytest.mark.parametrize("n,world,mask_kind", [(40, 2, "padding"), (70, 3, "none"),
                                               (33, 4, "padding")])
def test_sharded_block_over_peer_comm(n, world, mask_kind):
    z = O.make_pair(n, seed=5, dtype=torch.float64)
    p = O.make_block_params(seed=6, dtype=torch.float64)
    mask = O.make_padding_mask(n, n - 5, dtype=torch.float64) if mask_kind == "padding" else None
    w = oracle_weight_dicts(p)
    s = O.make_single(n, seed=n, dtype=torch.float64)
    ps = O.make_single_params(seed=7, ln_affine_random=True, dtype=torch.float64)
    ws = single_weight_dict(ps)
    ref = O.pair_block(z, mask, p)
    s_ref = O.single_block(s, ref, mask, ps)

    def rank_fn(r, comm):
        sh = S.shard_plan(n, world, r)
        z_loc = S.local_rows(z, sh)
        s_buf = S.single_buffer(s, sh)
        ph = OraclePhases()
        S.sharded_pair_block(z_loc, mask, w, sh, comm, ph)
        S.sharded_single_block(s_buf, z_loc, mask, ws, sh, comm, ph)
        return S.gather_rows(z_loc, sh, comm), s_buf[:n].clone()

    res, _, _ = run_ranks(world, rank_fn)
    for full, s_out in res:
        assert O.rel_max_err(full, ref) <= TOL
        assert O.rel_max_err(s_out, s_ref) <= TOL
