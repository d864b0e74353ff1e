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


def _split_hi_lo(x):
    hi = (x.view(torch.int32) & -8192).view(torch.float32)  # top 11 significand bits
    return hi, x - hi


@pytest.mark.parametrize("precision", ["strict", "fast"])
@pytest.mark.parametrize("m,nn,k,owners,chunk", [(200, 200, 96, 3, 96), (256, 300, 64, 2, 128),
                                                 (90, 70, 40, 4, 32)])
def test_group_contract_scatter_matches_local(precision, m, nn, k, owners, chunk):
    """The contraction storing its rows at their owners (the row-sharded
    TriMul's fused return exchange, emulated with local buffers) writes
    exactly the rows and channels the plain call writes, and nothing else."""
    lib = _lib.load()
    dev = torch.device("cuda")
    st = ops._stream_ptr(dev)
    p = 0 if precision == "strict" else 1
    G, ch_off = 16, 32
    ld = int(lib.fpb_trimul_plane_ld(k, p))
    g = torch.Generator().manual_seed(m + nn + k)
    a = torch.zeros(G, m, ld)
    b = torch.zeros(G, nn, ld)
    a[:, :, :k] = torch.randn(G, m, k, generator=g)
    b[:, :, :k] = torch.randn(G, nn, k, generator=g)
    a, b = a.to(dev), b.to(dev)
    if p == 0:
        (a_hi, a_lo), (b_hi, b_lo) = _split_hi_lo(a), _split_hi_lo(b)
        ops_ = [a_hi, a_lo, b_hi, b_lo]
        odt = torch.float32
    else:
        a_hi, b_hi = a.to(torch.bfloat16), b.to(torch.bfloat16)
        ops_ = [a_hi, None, b_hi, None]
        odt = torch.bfloat16
    ptr = [ctypes.c_void_p(t.data_ptr() if t is not None else 0) for t in ops_]
    njb = (nn + 127) // 128
    ws = torch.zeros(256, dtype=torch.uint8, device=dev)
    ref = torch.zeros(m, njb, G, 128, dtype=odt, device=dev)
    _lib.check(lib.fpb_trimul_group_contract(
        ptr[0], ptr[1], m, m, ptr[2], ptr[3], nn, nn, 1, 0, k, ld, G,
        ctypes.c_void_p(ref.data_ptr()), p, ctypes.c_void_p(ws.data_ptr()), 256, st),
        "fpb_trimul_group_contract")
    outs = [torch.full((chunk, njb, 128, 128), 7.0, dtype=odt, device=dev) for _ in range(owners)]
    arr = (ctypes.c_void_p * owners)(*[o.data_ptr() for o in outs])
    _lib.check(lib.fpb_trimul_group_contract_scatter(
        ptr[0], ptr[1], m, m, ptr[2], ptr[3], nn, nn, 1, 0, k, ld, G, arr, owners, chunk,
        ch_off, p, ctypes.c_void_p(ws.data_ptr()), 256, st),
        "fpb_trimul_group_contract_scatter")
    torch.cuda.synchronize()
    ref = ref.cpu()
    for d, o in enumerate(outs):
        o = o.cpu()
        rows = max(0, min(chunk, m - d * chunk))
        got = o[:rows, :, ch_off:ch_off + G]
        want = ref[d * chunk:d * chunk + rows]
        # columns past nn inside the last 128-column block are not written
        full = njb * 128
        for jb in range(njb):
            cols = min(128, nn - jb * 128)
            assert torch.equal(got[:, jb, :, :cols], want[:, jb, :, :cols])
            assert torch.all(got[:, jb, :, cols:] == 7.0)
        assert full >= nn
        assert torch.all(o[rows:] == 7.0)
        assert torch.all(o[:, :, :ch_off] == 7.0) and torch.all(o[:, :, ch_off + G:] == 7.0)
