"""The calibration observer (esmcu_observer) against the reference's
ActivationObserver compiled from its own sources (observer.cpp:8-51), on the
CPU.  Both keep, per site, a 65536-value reservoir filled by Algorithm R with
a std::mt19937 seeded 0xc1b1ce; fed the same values in the same order they
must keep the same sample, so every percentile is bit-identical.  The cases
cross the reservoir size within one call and across calls, interleave sites,
and include zeros, negatives and a site observed with no values."""
import ctypes as C

import numpy as np
import pytest


def _feeds(rng):
    sizes = [10, 65530, 3, 70000, 1, 200000, 0, 65536, 12345]
    out = []
    for i, n in enumerate(sizes):
        site = f"layer{i % 3}.attn_out"
        v = (rng.standard_normal(n) * (1 + 5 * (i % 2))).astype(np.float32)
        if n > 100:
            v[::97] = 0.0
            v[::131] = -np.abs(v[::131]) * 20
        out.append((site, v))
    return out


def test_observer_matches_reference_bit_exactly(O, R):
    from esm_b200 import ActivationObserver

    rng = np.random.default_rng(41)
    ours = ActivationObserver()
    theirs = R.ref_observer_new()
    try:
        for site, v in _feeds(rng):
            ours.observe(site, v)
            O.ref_check(R.ref_observer_observe(theirs, site.encode(), v.ctypes.data, v.size))
        for pct in (0.0, 1.0, 50.0, 99.0, 99.9, 99.99, 100.0, 150.0):
            got = ours.percentile(pct)
            assert set(got) == {"layer0.attn_out", "layer1.attn_out", "layer2.attn_out"}
            for site, val in got.items():
                want = C.c_float()
                O.ref_check(R.ref_observer_percentile(theirs, site.encode(), C.c_float(pct),
                                                      C.byref(want)))
                assert np.float32(val) == np.float32(want.value), (site, pct, val, want.value)
    finally:
        R.ref_observer_free(theirs)


def test_observer_sites_and_clear():
    from esm_b200 import ActivationObserver

    obs = ActivationObserver()
    obs.observe("a", np.zeros(0, np.float32))  # no values: no site (observer.cpp:10)
    assert obs.percentile(99.9) == {}
    obs.observe("b", np.array([-3.0, 1.0, 2.0], np.float32))
    obs.observe("a", np.array([5.0], np.float32))
    got = obs.percentile(100.0)
    assert list(got) == ["b", "a"]  # first-observed order
    assert got == {"b": 3.0, "a": 5.0}
    assert obs.percentile(0.0)["b"] == 1.0
    obs.clear()
    assert obs.percentile(50.0) == {}


def test_observer_percentile_of_unknown_site_is_not_found():
    from esm_b200 import ActivationObserver, EsmCudaError, _lib

    obs = ActivationObserver()
    v = C.c_float()
    with pytest.raises(EsmCudaError) as ei:
        _lib.call("esmcu_observer_percentile", obs.handle, b"nope", 99.9, C.byref(v))
    assert _lib.STATUS[ei.value.code] == "NOT_FOUND"
