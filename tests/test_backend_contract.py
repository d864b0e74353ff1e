"""CPU contract tests of the b200 backend boundary (no GPU needed): the C-ABI
library loads and exports every symbol ``include/fireprot_b200.h`` declares,
capability predicates accept exactly the supported signatures, CPU tensors
never reach the C ABI (native fallback), and the ops refuse CPU tensors
(``tests/operators/test_softmax_fp32_contract.py:52-59`` pattern)."""
from __future__ import annotations

import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def _declared_symbols():
    text = (ROOT / "include" / "fireprot_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fpb_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    import ctypes
    from fireprot_b200 import _lib
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    names = _declared_symbols()
    assert len(names) >= 20
    for name in names:
        assert hasattr(lib, name), name
    # the Python binding covers every declared entry point
    assert set(names) <= set(_lib.SIGNATURES), set(names) - set(_lib.SIGNATURES)


def test_abi_version_and_status_strings():
    from fireprot_b200 import _lib
    lib = _lib.load()
    assert lib.fpb_abi_version() == 1
    assert lib.fpb_status_string(0) == b"ok"
    assert b"workspace" in lib.fpb_status_string(7)


def test_entry_points_reject_bad_arguments_without_a_gpu():
    """Argument validation happens on the host before any launch."""
    from fireprot_b200 import _lib
    lib = _lib.load()
    assert lib.fpb_trimul_workspace_size(64, 64, 0) == 0       # c_z must be 128
    assert lib.fpb_triattn_workspace_size(64, 128, 8, 32, 0, 0) == 0
    assert lib.fpb_transition_workspace_size(128, 2, 0) == 0
    assert lib.fpb_pair_block_workspace_size(0, 0, 0) == 0
    # strict: a/b hi/lo channel-first planes (4 x 1.21 GB) + the x tiles (1.21 GB)
    assert lib.fpb_trimul_workspace_size(1536, 128, 0) > 5 * 1536 * 1536 * 128 * 4
    # null pointers / bad shapes are status codes, not crashes
    assert lib.fpb_trimul(None, None, 8, 128, *([None] * 10), 1e-5, 1, 1, 0, None, 0, None) == 4
    assert lib.fpb_transition(None, None, 0, 128, 4, *([None] * 5), 1e-5, 0, None, 0, None) == 4


def _base_sig(**kw):
    from fireprot_b200.registry import OperationSignature
    base = dict(operation="triangle_multiplication", device_type="cuda", architecture="sm_100",
                dtype="float32", shape=(1536, 1536, 128), layout="contiguous", mode="inference",
                mask="none", inplace=True,
                attributes={"c_z": 128, "c_hidden": 128, "weights": "ok"})
    base.update(kw)
    return OperationSignature.create(**base)


def test_trimul_capability_accepts_only_supported_signatures():
    from fireprot_b200 import backend as b
    assert b._supports_trimul(_base_sig()) is True
    assert b._supports_trimul(_base_sig(mask="dense")) is True
    assert b._supports_trimul(_base_sig(shape=(7, 7, 128))) is True  # any N
    for change in ({"device_type": "cpu"}, {"architecture": "gfx90a"}, {"dtype": "bfloat16"},
                   {"layout": "strided"}, {"mode": "training"}, {"inplace": False},
                   {"shape": (1, 64, 64, 128)}, {"shape": (64, 64, 64)},
                   {"attributes": {"c_z": 128, "c_hidden": 64, "weights": "ok"}},
                   {"attributes": {"c_z": 128, "c_hidden": 128, "weights": "unsupported"}}):
        res = b._supports_trimul(_base_sig(**change))
        assert res is not True and isinstance(res[1], str), change


def test_attention_core_capability():
    from fireprot_b200 import backend as b
    from fireprot_b200.registry import OperationSignature
    n = 124
    ok = dict(operation="triangle_attention", device_type="cuda", architecture="sm_100",
              dtype="float32", shape=(n, 4, n, 32), layout="strided", mode="inference",
              mask="additive-mask-and-triangle-bias", inplace=False,
              attributes={"bias_shapes": repr(((n, 1, 1, n), (1, 4, n, n))),
                          "qkv_shapes_match": True})
    assert b._supports_attention_core(OperationSignature.create(**ok)) is True
    tri_only = dict(ok, attributes={"bias_shapes": repr(((1, 4, n, n),)),
                                    "qkv_shapes_match": True})
    assert b._supports_attention_core(OperationSignature.create(**tri_only)) is True
    for change in ({"shape": (n, 2, n, 32)}, {"shape": (n, 4, n, 16)}, {"mode": "training"},
                   {"attributes": {"bias_shapes": repr(((n, 1, 1, n),)),
                                   "qkv_shapes_match": True}},
                   {"attributes": {"bias_shapes": repr(((1, 4, n, n),)),
                                   "qkv_shapes_match": False}}):
        assert b._supports_attention_core(OperationSignature.create(**dict(ok, **change))) \
            is not True


def test_cpu_tensors_fall_back_to_native():
    from fireprot_b200 import backend as b
    from fireprot_b200.modules import PairformerPairBlock
    blk = PairformerPairBlock().init_random_(1).eval()
    z = torch.randn(6, 6, 128)
    with torch.no_grad():
        assert b.dispatch_triangle_multiplication(
            module=blk.tri_mul_out, z=z, mask=None, inplace_safe=True, add_with_inplace=True,
            inplace_chunk_size=None, native=lambda **_: "native") == "native"
        q = torch.randn(6, 4, 6, 32)
        assert b.dispatch_triangle_attention(
            module=None, q=q, k=q, v=q, biases=[torch.randn(1, 4, 6, 6)],
            native=lambda **_: "native") == "native"
        assert b.dispatch_transition(module=blk.pair_transition, x=z,
                                     native=lambda: "native") == "native"
        assert b.triangle_attention_module(module=blk.tri_att_start, z=z, mask=None,
                                           starting=True, native=lambda **_: "native") == "native"
    assert b.transpose_pair(z, training=False).is_contiguous()


def test_ops_refuse_cpu_tensors():
    from fireprot_b200 import ops
    from fireprot_b200.modules import PairformerPairBlock
    blk = PairformerPairBlock().init_random_(1)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.trimul(torch.randn(4, 4, 128), None, blk.tri_mul_out.weight_dict(), outgoing=True)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.transition(torch.randn(4, 4, 128), blk.pair_transition.weight_dict())
    with pytest.raises(ValueError):
        ops.precision_code("tf32")
