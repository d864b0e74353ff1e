"""Allocation-free pair transition (``fpb_transition_noalloc``) against the
workspace entry point ``fpb_transition``, both called through the C ABI.

The two run the same kernels on the same inputs, so the results are expected
to agree to the bit; the test holds them to 1e-6 of the output scale. Two
calls in a row (the second with other weights, in delta mode) show that each
call repacks the weights and restarts the status word in the static scratch.
This file is collected last so it also runs after every other GPU test.
"""
import ctypes

import pytest
import torch

from fireprot_b200 import _lib

pytestmark = pytest.mark.gpu

TOL = 1e-6
ROWS = 37 * 61  # ragged: not a multiple of the 128-row tile


def _weights(seed, device):
    g = torch.Generator().manual_seed(seed)

    def rnd(*shape, scale):
        return (torch.randn(*shape, generator=g) * scale).to(device)

    return {"ln_w": 1.0 + rnd(128, scale=0.1), "ln_b": rnd(128, scale=0.1),
            "w_a": rnd(512, 128, scale=128 ** -0.5), "w_b": rnd(512, 128, scale=128 ** -0.5),
            "w_out": rnd(128, 512, scale=512 ** -0.5)}


def _ptrs(w):
    return [w[k].data_ptr() for k in ("ln_w", "ln_b", "w_a", "w_b", "w_out")]


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream


def _reference(lib, z, delta, w, precision, device):
    nbytes = lib.fpb_transition_workspace_size(128, 4, precision)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=device)
    rc = lib.fpb_transition(z.data_ptr(), 0 if delta is None else delta.data_ptr(), ROWS, 128,
                            4, *_ptrs(w), 1e-5, precision, ws.data_ptr(), nbytes,
                            _stream(device))
    assert rc == 0, lib.fpb_status_string(rc)
    st = ctypes.c_int(-1)
    assert lib.fpb_workspace_status(ws.data_ptr(), _stream(device), ctypes.byref(st)) == 0
    assert st.value == 0


def _noalloc(lib, z, delta, w, precision, device):
    st = ctypes.c_int(-1)
    rc = lib.fpb_transition_noalloc(z.data_ptr(), 0 if delta is None else delta.data_ptr(),
                                    ROWS, 128, 4, *_ptrs(w), 1e-5, precision, ctypes.byref(st),
                                    _stream(device))
    assert rc == 0, lib.fpb_status_string(rc)
    assert st.value == 0


def _rel(a, b):
    return ((a - b).abs().max() / b.abs().max()).item()


@pytest.mark.parametrize("precision", [0, 1])
def test_noalloc_matches_workspace_entry_point(cuda_device, precision):
    lib = _lib.load()
    g = torch.Generator().manual_seed(3 + precision)
    z0 = torch.randn(ROWS, 128, generator=g).to(cuda_device)
    z1 = torch.randn(ROWS, 128, generator=g).to(cuda_device)
    w0, w1 = _weights(10 + precision, cuda_device), _weights(20 + precision, cuda_device)

    # call 1: in place, z += update
    ref0 = z0.clone()
    _reference(lib, ref0, None, w0, precision, cuda_device)
    out0 = z0.clone()
    _noalloc(lib, out0, None, w0, precision, cuda_device)
    assert _rel(out0, ref0) <= TOL

    # call 2 right after: other weights, delta mode (z left unchanged)
    ref1 = torch.empty_like(z1)
    _reference(lib, z1, ref1, w1, precision, cuda_device)
    out1 = torch.full_like(z1, float("nan"))
    z1_before = z1.clone()
    _noalloc(lib, z1, out1, w1, precision, cuda_device)
    assert _rel(out1, ref1) <= TOL
    assert torch.equal(z1, z1_before)

    # a repeat call changes nothing in the device's free memory
    torch.cuda.synchronize(cuda_device)
    free_before, _ = torch.cuda.mem_get_info(cuda_device)
    _noalloc(lib, z1, out1, w1, precision, cuda_device)
    torch.cuda.synchronize(cuda_device)
    free_after, _ = torch.cuda.mem_get_info(cuda_device)
    assert free_after == free_before
    assert _rel(out1, ref1) <= TOL


def test_noalloc_rejects_bad_requests(cuda_device):
    lib = _lib.load()
    z = torch.zeros(ROWS, 128, device=cuda_device)
    w = _weights(1, cuda_device)
    st = ctypes.c_int(-1)
    stream = _stream(cuda_device)
    # unsupported channel count / expansion -> unsupported shape (2)
    assert lib.fpb_transition_noalloc(z.data_ptr(), 0, ROWS, 64, 4, *_ptrs(w), 1e-5, 0,
                                      ctypes.byref(st), stream) == 2
    assert lib.fpb_transition_noalloc(z.data_ptr(), 0, ROWS, 128, 2, *_ptrs(w), 1e-5, 0,
                                      ctypes.byref(st), stream) == 2
    # unknown precision -> invalid argument (4)
    assert lib.fpb_transition_noalloc(z.data_ptr(), 0, ROWS, 128, 4, *_ptrs(w), 1e-5, 7,
                                      ctypes.byref(st), stream) == 4
    assert lib.fpb_status_string(8).decode() == "request exceeds the static scratch capacity"
    # a null input or weight -> invalid argument (4)
    assert lib.fpb_transition_noalloc(0, 0, ROWS, 128, 4, *_ptrs(w), 1e-5, 0,
                                      ctypes.byref(st), stream) == 4
    bad = _ptrs(w)
    bad[2] = 0
    assert lib.fpb_transition_noalloc(z.data_ptr(), 0, ROWS, 128, 4, *bad, 1e-5, 0,
                                      ctypes.byref(st), stream) == 4
    # z or delta_out off a 16-byte boundary -> misaligned (3)
    assert lib.fpb_transition_noalloc(z.data_ptr() + 4, 0, ROWS - 1, 128, 4, *_ptrs(w), 1e-5,
                                      0, ctypes.byref(st), stream) == 3
    d = torch.zeros(ROWS, 128, device=cuda_device)
    assert lib.fpb_transition_noalloc(z.data_ptr(), d.data_ptr() + 4, ROWS - 1, 128, 4,
                                      *_ptrs(w), 1e-5, 0, ctypes.byref(st), stream) == 3
    # no rows -> unsupported shape (2)
    assert lib.fpb_transition_noalloc(z.data_ptr(), 0, 0, 128, 4, *_ptrs(w), 1e-5, 0,
                                      ctypes.byref(st), stream) == 2
    torch.cuda.synchronize(cuda_device)
    assert torch.count_nonzero(z).item() == 0 and torch.count_nonzero(d).item() == 0


def test_noalloc_status_out_refused_while_capturing(cuda_device):
    """Reporting the status waits for the stream, which a capture forbids:
    the call is refused before it enqueues anything."""
    lib = _lib.load()
    z = torch.zeros(ROWS, 128, device=cuda_device)
    w = _weights(2, cuda_device)
    x = torch.zeros(4, device=cuda_device)
    side = torch.cuda.Stream(cuda_device)
    graph = torch.cuda.CUDAGraph()
    st = ctypes.c_int(-1)
    rcs = []
    torch.cuda.synchronize(cuda_device)
    with torch.cuda.stream(side):
        graph.capture_begin()
        x.add_(1.0)
        rcs.append(lib.fpb_transition_noalloc(z.data_ptr(), 0, ROWS, 128, 4, *_ptrs(w), 1e-5, 0,
                                              ctypes.byref(st), side.cuda_stream))
        graph.capture_end()
    assert rcs == [4]
    assert st.value == -1
    graph.replay()
    torch.cuda.synchronize(cuda_device)
    assert x.tolist() == [1.0] * 4
    assert torch.count_nonzero(z).item() == 0
    del graph


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs a second GPU")
def test_noalloc_second_device():
    """Each device has its own array; a call on device 1 after one on device
    0 uses device 1's copy and matches the workspace entry point there."""
    lib = _lib.load()
    for dev_index in (0, 1):
        dev = torch.device("cuda", dev_index)
        with torch.cuda.device(dev):
            g = torch.Generator().manual_seed(40 + dev_index)
            z = torch.randn(ROWS, 128, generator=g).to(dev)
            w = _weights(30 + dev_index, dev)
            ref = z.clone()
            _reference(lib, ref, None, w, 0, dev)
            out = z.clone()
            _noalloc(lib, out, None, w, 0, dev)
            assert _rel(out, ref) <= TOL
