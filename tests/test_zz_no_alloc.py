"""The allocation-free entry point, hkb_mpnn_design_noalloc.

It serves callers that may not allocate device memory while they run (a
plugin whose host application owns every byte of GPU memory through its own
pool, or a loop that cannot pay cudaMalloc's implicit synchronisation).  Its
scratch is one fixed device array inside the library, so this test checks
that two calls in a row -- the second reusing whatever the first left in
that array -- both reproduce the allocating device entry point
(hkb_mpnn_design_device) on the same fp32 engine, and that a batch over the
limit is refused with InvalidArgument.

This file is named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

P = ctypes.POINTER


def _batch(hl, L, S, seeds, temps, modes, coords_ptr, src_ptr):
    return hl.DesignBatch(len(L), L.ctypes.data_as(P(ctypes.c_int32)), coords_ptr, src_ptr,
                          S.ctypes.data_as(P(ctypes.c_int32)),
                          seeds.ctypes.data_as(P(ctypes.c_uint64)),
                          temps.ctypes.data_as(P(ctypes.c_float)),
                          modes.ctypes.data_as(P(ctypes.c_int32)), None)


def _outputs(torch, hl, Q, NS):
    t = torch.full((Q,), -7, dtype=torch.int32, device="cuda")
    lp = torch.full((Q * 21,), 123.0, dtype=torch.float32, device="cuda")
    o = torch.full((Q,), -7, dtype=torch.int32, device="cuda")
    sc = torch.full((NS,), 123.0, dtype=torch.float32, device="cuda")
    out = hl.DesignOut(ctypes.c_void_p(t.data_ptr()), ctypes.c_void_p(lp.data_ptr()),
                       ctypes.c_void_p(o.data_ptr()), ctypes.c_void_p(sc.data_ptr()))
    return out, (t, lp, o, sc)


def test_noalloc_design_matches_device_design_twice(weights_path):
    import torch
    from hikoboshi_b200 import DesignEngine, synthetic_backbone
    from hikoboshi_b200 import _lib as hl

    lib = hl.load()
    eng = DesignEngine(weights_path, device=0, precision="fp32")
    try:
        Ls = [24, 40]                      # 64 residues: the limit
        L = np.array(Ls, np.int32)
        S = np.array([3, 2], np.int32)
        seeds = np.array([11, 500], np.uint64)
        temps = np.array([0.1, 0.0], np.float32)
        modes = np.array([0, 0], np.int32)
        bb = [synthetic_backbone(40 + i, n) for i, n in enumerate(Ls)]
        coords = torch.from_numpy(np.concatenate([b[0] for b in bb])).cuda()
        srcs = torch.from_numpy(np.concatenate([b[1] for b in bb])).cuda()
        Q = int((L * S).sum())
        NS = int(S.sum())
        batch = _batch(hl, L, S, seeds, temps, modes, ctypes.c_void_p(coords.data_ptr()),
                       ctypes.c_void_p(srcs.data_ptr()))

        ref_out, ref = _outputs(torch, hl, Q, NS)
        hl.check(lib.hkb_mpnn_design_device(eng._h, ctypes.byref(batch), ctypes.byref(ref_out),
                                            None))
        torch.cuda.synchronize()
        ref = [x.cpu().numpy() for x in ref]

        for call in range(2):
            out, got = _outputs(torch, hl, Q, NS)
            hl.check(lib.hkb_mpnn_design_noalloc(eng._h, ctypes.byref(batch), ctypes.byref(out),
                                                 None))
            torch.cuda.synchronize()
            tok, lp, order, sc = [x.cpu().numpy() for x in got]
            assert (order == ref[2]).all(), call
            assert (tok == ref[0]).all(), call
            # same kernels and same inputs: within the fp32 parity tolerance
            # on temperature-scaled log-probs (1e-4 / T, T = 0.1)
            assert np.abs(lp - ref[1]).max() <= 1e-3, call
            assert np.abs(sc - ref[3]).max() <= 1e-3, call
            assert np.isfinite(lp).all() and ((tok >= 0) & (tok < 21)).all()
    finally:
        eng.close()


def test_noalloc_rejects_batches_over_the_limit(weights_path):
    import torch
    from hikoboshi_b200 import DesignEngine
    from hikoboshi_b200 import _lib as hl

    lib = hl.load()
    eng = DesignEngine(weights_path, device=0, precision="fp32")
    try:
        L = np.array([65], np.int32)
        S = np.array([1], np.int32)
        seeds = np.array([0], np.uint64)
        temps = np.array([0.1], np.float32)
        modes = np.array([0], np.int32)
        coords = torch.zeros((65, 5, 3), dtype=torch.float32, device="cuda")
        srcs = torch.ones((65, 5), dtype=torch.uint8, device="cuda")
        batch = _batch(hl, L, S, seeds, temps, modes, ctypes.c_void_p(coords.data_ptr()),
                       ctypes.c_void_p(srcs.data_ptr()))
        out, _keep = _outputs(torch, hl, 65, 1)
        st = lib.hkb_mpnn_design_noalloc(eng._h, ctypes.byref(batch), ctypes.byref(out), None)
        assert st.code == hl.HKB_INVALID_ARGUMENT
        assert b"allocation-free limits" in st.detail
    finally:
        eng.close()
