"""The allocation-free entry point, hkb_mpnn_design_noalloc.

It serves callers that may not allocate device memory while they run (a
plugin whose host application owns every byte of GPU memory through its own
pool, or a loop that cannot pay cudaMalloc's implicit synchronisation).  Its
scratch is one fixed device array inside the library, so this test checks
that two calls in a row -- the second reusing whatever the first left in
that array -- both reproduce the allocating device entry point
(hkb_mpnn_design_device) on the same fp32 engine, and that a batch over the
limit is refused with InvalidArgument.  The two entry points run the same
kernels on the same inputs, so their outputs must be bit-identical; the
random, N-to-C and caller-given decoding orders are all exercised, and the
device's free memory must not move across a call.

This file is named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

P = ctypes.POINTER


def _batch(hl, L, S, seeds, temps, modes, coords_ptr, src_ptr, input_orders=None):
    io = None if input_orders is None else input_orders.ctypes.data_as(P(ctypes.c_int32))
    return hl.DesignBatch(len(L), L.ctypes.data_as(P(ctypes.c_int32)), coords_ptr, src_ptr,
                          S.ctypes.data_as(P(ctypes.c_int32)),
                          seeds.ctypes.data_as(P(ctypes.c_uint64)),
                          temps.ctypes.data_as(P(ctypes.c_float)),
                          modes.ctypes.data_as(P(ctypes.c_int32)), io)


def _outputs(torch, hl, Q, NS):
    t = torch.full((Q,), -7, dtype=torch.int32, device="cuda")
    lp = torch.full((Q * 21,), 123.0, dtype=torch.float32, device="cuda")
    o = torch.full((Q,), -7, dtype=torch.int32, device="cuda")
    sc = torch.full((NS,), 123.0, dtype=torch.float32, device="cuda")
    out = hl.DesignOut(ctypes.c_void_p(t.data_ptr()), ctypes.c_void_p(lp.data_ptr()),
                       ctypes.c_void_p(o.data_ptr()), ctypes.c_void_p(sc.data_ptr()))
    return out, (t, lp, o, sc)


@pytest.mark.parametrize("modes", [(0, 0), (1, 2)], ids=["random", "n_to_c+input"])
def test_noalloc_design_matches_device_design_twice(weights_path, modes):
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
        modes_a = np.array(modes, np.int32)
        # a caller permutation for every protein (read where the mode is INPUT)
        rng = np.random.default_rng(5)
        io = np.concatenate([rng.permutation(n).astype(np.int32) for n in Ls])
        bb = [synthetic_backbone(40 + i, n) for i, n in enumerate(Ls)]
        coords = torch.from_numpy(np.concatenate([b[0] for b in bb])).cuda()
        srcs = torch.from_numpy(np.concatenate([b[1] for b in bb])).cuda()
        Q = int((L * S).sum())
        NS = int(S.sum())
        batch = _batch(hl, L, S, seeds, temps, modes_a, ctypes.c_void_p(coords.data_ptr()),
                       ctypes.c_void_p(srcs.data_ptr()), io)

        ref_out, ref = _outputs(torch, hl, Q, NS)
        hl.check(lib.hkb_mpnn_design_device(eng._h, ctypes.byref(batch), ctypes.byref(ref_out),
                                            None))
        torch.cuda.synchronize()
        ref = [x.cpu().numpy() for x in ref]
        if modes[1] == 2:
            assert (ref[2][3 * 24:].reshape(2, 40) == io[24:]).all()
        if modes[0] == 1:
            assert (ref[2][:3 * 24].reshape(3, 24) == np.arange(24)).all()

        outs = [_outputs(torch, hl, Q, NS) for _ in range(2)]   # allocated up front
        free = []
        for call, (out, got) in enumerate(outs):
            hl.check(lib.hkb_mpnn_design_noalloc(eng._h, ctypes.byref(batch), ctypes.byref(out),
                                                 None))
            torch.cuda.synchronize()
            free.append(torch.cuda.mem_get_info()[0])
            tok, lp, order, sc = [x.cpu().numpy() for x in got]
            # same kernels on the same inputs: bit-identical outputs
            assert (order == ref[2]).all(), call
            assert (tok == ref[0]).all(), call
            assert (lp.view(np.uint32) == ref[1].view(np.uint32)).all(), call
            assert (sc.view(np.uint32) == ref[3].view(np.uint32)).all(), call
            assert np.isfinite(lp).all() and ((tok >= 0) & (tok < 21)).all()
        # nothing was allocated on the device by the second call
        assert free[0] == free[1]
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
