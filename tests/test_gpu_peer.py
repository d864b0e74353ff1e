"""The transposed peer exchange kernel (``fpb_peer_transpose_rows``) on one
GPU: every emulated rank's destination is a local buffer, so one launch per
rank writes the rows of ``z^T`` exactly as it would write into the other
ranks' mapped buffers. Bit-exact: the kernel only moves bytes."""
import ctypes

import pytest
import torch

from fireprot_b200 import _lib, ops
from fireprot_b200 import sharded as S

pytestmark = pytest.mark.gpu


def _transpose_all(z, world):
    n, ch = z.shape[0], z.shape[-1]
    lib = _lib.load()
    dev = torch.device("cuda")
    shards = [S.shard_plan(n, world, r) for r in range(world)]
    locs = [S.local_rows(z, sh).to(dev) for sh in shards]
    c = shards[0].chunk
    outs = [torch.full((c, n, ch), 7.0, device=dev) for _ in range(world)]
    ptrs = (ctypes.c_void_p * world)(*[o.data_ptr() for o in outs])
    for r, sh in enumerate(shards):
        _lib.check(lib.fpb_peer_transpose_rows(
            ctypes.c_void_p(locs[r].data_ptr()), n, c, ch, r, world, ptrs,
            ops._stream_ptr(dev)), "fpb_peer_transpose_rows")
    torch.cuda.synchronize()
    return shards, [o.cpu() for o in outs]


@pytest.mark.parametrize("n,world,ch", [(150, 1, 128), (150, 2, 128), (150, 3, 128),
                                        (97, 4, 128), (40, 4, 128), (300, 8, 128),
                                        (64, 2, 4), (66, 3, 260)])
def test_peer_transpose_matches_transpose(n, world, ch):
    g = torch.Generator().manual_seed(n * 31 + world)
    z = torch.randn(n, n, ch, generator=g)
    zt = z.transpose(0, 1)
    shards, outs = _transpose_all(z, world)
    for sh, o in zip(shards, outs):
        assert torch.equal(o[:sh.rows], zt[sh.r0:sh.r0 + sh.rows])
        # rows past n are not written
        assert torch.all(o[sh.rows:] == 7.0)


def test_peer_transpose_rejects_bad_arguments():
    lib = _lib.load()
    dev = torch.device("cuda")
    z = torch.zeros(32, 64, 128, device=dev)
    ptrs = (ctypes.c_void_p * 2)(z.data_ptr(), z.data_ptr())
    st = ops._stream_ptr(dev)
    zp = ctypes.c_void_p(z.data_ptr())
    assert lib.fpb_peer_transpose_rows(zp, 64, 32, 126, 0, 2, ptrs, st) != 0  # ch % 4
    assert lib.fpb_peer_transpose_rows(zp, 64, 16, 128, 0, 2, ptrs, st) != 0  # chunk*world < n
    assert lib.fpb_peer_transpose_rows(zp, 64, 32, 128, 2, 2, ptrs, st) != 0  # rank
    assert lib.fpb_peer_transpose_rows(zp, 64, 32, 128, 0, 17, ptrs, st) != 0  # world
    nul = (ctypes.c_void_p * 2)(z.data_ptr(), None)
    assert lib.fpb_peer_transpose_rows(zp, 64, 32, 128, 0, 2, nul, st) != 0
    mis = (ctypes.c_void_p * 2)(z.data_ptr(), z.data_ptr() + 4)
    assert lib.fpb_peer_transpose_rows(zp, 64, 32, 128, 0, 2, mis, st) != 0
    torch.cuda.synchronize()


def test_peer_scatter_copies_every_segment():
    lib = _lib.load()
    dev = torch.device("cuda")
    sizes = [0, 16, 4096, 1 << 20, (3 << 20) + 48, 7 * 16]
    src = [torch.randint(0, 255, (max(b, 16),), dtype=torch.uint8, device=dev) for b in sizes]
    dst = [torch.zeros(max(b, 16) + 32, dtype=torch.uint8, device=dev) for b in sizes]
    k = len(sizes)
    _lib.check(lib.fpb_peer_scatter(
        (ctypes.c_void_p * k)(*[t.data_ptr() for t in src]),
        (ctypes.c_void_p * k)(*[t.data_ptr() + 16 for t in dst]),
        (ctypes.c_size_t * k)(*sizes), k, ops._stream_ptr(dev)), "fpb_peer_scatter")
    torch.cuda.synchronize()
    for b, s_, d_ in zip(sizes, src, dst):
        assert torch.equal(d_[16:16 + b], s_[:b])
        assert not d_[:16].any() and not d_[16 + b:].any()  # nothing outside the segment


def test_peer_scatter_rejects_bad_arguments():
    lib = _lib.load()
    dev = torch.device("cuda")
    t = torch.zeros(1024, dtype=torch.uint8, device=dev)
    st = ops._stream_ptr(dev)

    def call(src_off, dst_off, nbytes, count=1):
        return lib.fpb_peer_scatter((ctypes.c_void_p * 1)(t.data_ptr() + src_off),
                                    (ctypes.c_void_p * 1)(t.data_ptr() + 512 + dst_off),
                                    (ctypes.c_size_t * 1)(nbytes), count, st)
    assert call(0, 0, 24) != 0     # size not a multiple of 16
    assert call(8, 0, 32) != 0     # misaligned source
    assert call(0, 4, 32) != 0     # misaligned destination
    assert call(0, 0, 32, count=17) != 0
    assert call(0, 0, 32, count=-1) != 0
    torch.cuda.synchronize()
