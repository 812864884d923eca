"""CPU-only checks of the drop-in boundary: the C-ABI library loads, exports
every symbol include/hkb_mpnn.h declares, and its host-only logic (decoding
orders, synthetic inputs, weight-image validation, argument checks) behaves
like the reference without touching a GPU."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


def header_functions():
    text = (ROOT / "include" / "hkb_mpnn.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(hkb_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from hikoboshi_b200 import _lib
    lib = _lib.load()
    declared = header_functions()
    assert declared, "no declarations parsed"
    for name in declared:
        assert hasattr(lib, name), name
    assert sorted(_lib.EXPORTED) == declared
    assert lib.hkb_mpnn_abi_version() == 1


def test_decode_order_matches_reference_goldens(refsyn):
    from hikoboshi_b200 import decode_order
    for name in refsyn["cases"]:
        s = refsyn[f"{name}/sources"]
        mask = (s[:, :4].min(axis=1) > 0).astype(np.float32)
        got = decode_order(s.shape[0], 99, mask=mask)
        assert (got == refsyn[f"{name}/order_seed99"]).all(), name


def test_decode_order_modes_and_permutation_check():
    from hikoboshi_b200 import HkbError, decode_order
    assert (decode_order(5, 0, mode="n_to_c") == np.arange(5)).all()
    assert (decode_order(4, 0, mode="input", input_order=[2, 0, 3, 1]) == [2, 0, 3, 1]).all()
    for bad in ([0, 0, 1, 2], [0, 1, 2, 4], [-1, 0, 1, 2]):
        with pytest.raises(HkbError) as e:
            decode_order(4, 0, mode="input", input_order=bad)
        assert e.value.code == 1 and "permutation" in e.value.detail


def test_synthetic_backbone_is_deterministic_and_ideal():
    from hikoboshi_b200 import synthetic_backbone
    a, sa = synthetic_backbone(3, 200)
    b, sb = synthetic_backbone(3, 200)
    c, _ = synthetic_backbone(4, 200)
    assert (a == b).all() and (sa == sb).all() and not (a == c).all()
    n, ca, cc, o = a[:, 0], a[:, 1], a[:, 2], a[:, 3]
    assert np.allclose(np.linalg.norm(ca - n, axis=1), 1.458, atol=1e-4)
    assert np.allclose(np.linalg.norm(cc - ca, axis=1), 1.525, atol=1e-4)
    assert np.allclose(np.linalg.norm(n[1:] - cc[:-1], axis=1), 1.329, atol=1e-4)
    assert np.allclose(np.linalg.norm(o - cc, axis=1), 1.231, atol=1e-4)
    assert (sa[:, :4] == 1).all() and (sa[:, 4] == 3).all()


def test_weight_image_validation_runs_before_device_use():
    """Broken safetensors images are rejected as InvalidArgument on the host
    (no GPU needed), like the reference's package validation."""
    from hikoboshi_b200 import _lib
    lib = _lib.load()
    h = ctypes.c_void_p()
    for blob in (b"", b"\x10\x00\x00\x00\x00\x00\x00\x00{}", b"\x02\x00\x00\x00\x00\x00\x00\x00{}"):
        buf = ctypes.create_string_buffer(blob, max(1, len(blob)))
        st = lib.hkb_mpnn_create(buf, len(blob), 0, 0, ctypes.byref(h))
        assert st.code == 1, blob
        assert not h.value
    buf = ctypes.create_string_buffer(b"x", 1)
    assert lib.hkb_mpnn_create(buf, 1, 0, 7, ctypes.byref(h)).code == 1  # bad precision


def test_null_engine_calls_are_rejected():
    from hikoboshi_b200 import _lib
    lib = _lib.load()
    st = lib.hkb_mpnn_design(None, None, None)
    assert st.code == 1
    st = lib.hkb_mpnn_score(None, None, None)
    assert st.code == 1
    assert lib.hkb_mpnn_last_launch_count(None) == -1


def test_full_weight_image_parses_on_host(weights_path):
    """A valid image passes parsing and shape checks; without a GPU the call
    stops at device discovery with Unavailable (never a crash)."""
    import torch
    from hikoboshi_b200 import _lib
    lib = _lib.load()
    blob = Path(weights_path).read_bytes()
    buf = ctypes.create_string_buffer(blob, len(blob))
    h = ctypes.c_void_p()
    st = lib.hkb_mpnn_create(buf, len(blob), 0, 0, ctypes.byref(h))
    if torch.cuda.is_available():
        assert st.code == 0
        lib.hkb_mpnn_destroy(h)
    else:
        assert st.code == 3, st.detail
