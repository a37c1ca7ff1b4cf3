"""ksd8_ks3_vjp_static (partials in a static device array, no allocation)
against the two-call path ksd8_ks3_vjp + ksd8_ks3_vjp_reduce with caller
scratch.  The static entry point serves callers that cannot allocate device
memory (a binding or plugin host handed its buffers by an owner that reserved
all memory up front); it must produce the same bits as the path whose
partials buffer the caller provides.  Named to be collected last; every test builds its own inputs, so the
file also passes alone in a fresh process."""

import numpy as np
import pytest
import torch

FP16 = torch.float16


def _lib():
    from ksdraft_b200 import _lib
    return _lib


def _inputs(m, charts, seed):
    from ksdraft_b200.kernels.ks3_int8 import pack_small
    rng = np.random.default_rng(seed)
    coeffs = (rng.standard_normal((charts, 6)) * 0.05).astype(np.float32)
    rs = rng.uniform(-1, 1, charts).astype(np.float32)
    rh = rng.uniform(-1, 1, charts).astype(np.float32)
    packed = pack_small(*(torch.from_numpy(t).cuda() for t in (coeffs, rs, rh)))
    value = torch.from_numpy((rng.standard_normal((m, charts)) * 1e-2).astype(np.float16)).cuda()
    coords = torch.from_numpy((rng.standard_normal((m, charts)) * 2).astype(np.float16)).cuda()
    return value, coords, packed, torch.from_numpy(rs).cuda(), torch.from_numpy(rh).cuda()


def _outputs(m, charts):
    nt = (m + 127) // 128
    return dict(dcq=torch.full((m, charts), 77, dtype=torch.int8, device="cuda"),
                dcs=torch.full((m, charts // 128), 7.0, dtype=FP16, device="cuda"),
                dctq=torch.full((charts, m), 77, dtype=torch.int8, device="cuda"),
                dcts=torch.full((charts, nt), 7.0, dtype=FP16, device="cuda"),
                dcoeff=torch.full((charts, 6), 7.0, dtype=FP16, device="cuda"),
                dscale=torch.full((charts,), 7.0, dtype=FP16, device="cuda"),
                dshift=torch.full((charts,), 7.0, dtype=FP16, device="cuda"),
                status=torch.zeros(1, dtype=torch.int32, device="cuda"))


def _ptr(t):
    return t.data_ptr() if t.numel() else None


def _two_call(m, charts, inp):
    lib = _lib()
    value, coords, p, rs, rh = inp
    o = _outputs(m, charts)
    nt = (m + 127) // 128
    partials = torch.empty(max(nt, 1), 8, charts, device="cuda")  # non-NULL when m == 0
    rc = lib.lib().ksd8_ks3_vjp(_ptr(value), _ptr(coords), m, charts, *(t.data_ptr() for t in p),
                                _ptr(o["dcq"]), _ptr(o["dcs"]), _ptr(o["dctq"]),
                                _ptr(o["dcts"]), partials.data_ptr(), None, lib.stream_ptr())
    lib.check(rc, "ks3_vjp")
    rc = lib.lib().ksd8_ks3_vjp_reduce(partials.data_ptr(), nt, charts, rs.data_ptr(), rh.data_ptr(),
                                       o["dcoeff"].data_ptr(), o["dscale"].data_ptr(),
                                       o["dshift"].data_ptr(), o["status"].data_ptr(),
                                       lib.stream_ptr())
    lib.check(rc, "ks3_vjp_reduce")
    return o


def _static(m, charts, inp):
    lib = _lib()
    value, coords, p, rs, rh = inp
    o = _outputs(m, charts)
    rc = lib.lib().ksd8_ks3_vjp_static(
        _ptr(value), _ptr(coords), m, charts, *(t.data_ptr() for t in p), _ptr(o["dcq"]),
        _ptr(o["dcs"]), _ptr(o["dctq"]), _ptr(o["dcts"]), rs.data_ptr(), rh.data_ptr(),
        o["dcoeff"].data_ptr(), o["dscale"].data_ptr(), o["dshift"].data_ptr(),
        o["status"].data_ptr(), lib.stream_ptr())
    lib.check(rc, "ks3_vjp_static")
    return o


def _assert_same(a, b):
    torch.cuda.synchronize()
    for k in a:
        x, y = a[k].cpu(), b[k].cpu()
        if x.dtype == FP16:
            x, y = x.view(torch.int16), y.view(torch.int16)
        assert torch.equal(x, y), k


@pytest.mark.gpu
def test_static_matches_two_call_path_on_consecutive_calls():
    # two different problems back to back: the second call must not see the
    # first call's partials (ragged token count, then a larger one)
    first, second = (300, 384, 11), (1000, 640, 12)
    for m, charts, seed in (first, second):
        inp = _inputs(m, charts, seed)
        ref = _two_call(m, charts, inp)
        got = _static(m, charts, inp)
        _assert_same(got, ref)
        assert int(got["status"][0]) == 0
    # and the same problem twice in a row gives the same bits
    m, charts, seed = first
    inp = _inputs(m, charts, seed)
    _assert_same(_static(m, charts, inp), _static(m, charts, inp))


@pytest.mark.gpu
def test_static_at_capacity_and_empty():
    lib = _lib()
    charts = 2048
    m = lib.VJP_STATIC_MAX_PARTIALS // (8 * charts) * 128  # exactly fills the array
    inp = _inputs(m, charts, 13)
    _assert_same(_static(m, charts, inp), _two_call(m, charts, inp))
    inp0 = _inputs(0, 256, 14)
    got = _static(0, 256, inp0)
    _assert_same(got, _two_call(0, 256, inp0))
    assert not got["dcoeff"].any()


def test_static_rejects_requests_beyond_the_array():
    """Host-side size check: returns before any CUDA call (runs without a GPU)."""
    lib = _lib()
    L = lib.load()
    charts = 2048
    m = lib.VJP_STATIC_MAX_PARTIALS // (8 * charts) * 128 + 1
    rc = L.ksd8_ks3_vjp_static(*([None] * 2), m, charts, *([None] * 16), None)
    assert rc == lib.ERR_SCRATCH_LIMIT
    assert lib.status_string(rc) == "request exceeds the static scratch capacity"
    rc = L.ksd8_ks3_vjp_static(*([None] * 2), 128, lib.VJP_STATIC_MAX_PARTIALS // 4,
                               *([None] * 16), None)
    assert rc == lib.ERR_SCRATCH_LIMIT
    with pytest.raises(RuntimeError, match="static scratch"):
        lib.check(rc, "ks3_vjp_static")
