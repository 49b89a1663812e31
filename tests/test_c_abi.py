"""The C-ABI library on the CPU: it loads, exports exactly what
include/esm_b200.h declares, and its host-side functions (PlanBatches,
BatchView validation, RoPE tables) equal the reference's.  No compute call
needs a GPU here; device calls report NO_DEVICE cleanly."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


def _declared():
    h = (ROOT / "include" / "esm_b200.h").read_text()
    return sorted(set(re.findall(r"^(?:int|void\*|const char\*) (esmcu_\w+)\(", h, re.M)))


def test_library_exports_every_declared_symbol():
    from esm_b200 import _lib

    L = _lib.lib()
    declared = _declared()
    assert len(declared) >= 35
    for name in declared:
        assert hasattr(L, name), f"{name} declared in include/esm_b200.h but not exported"
    assert declared == _lib.exported_symbols(), "ctypes signature table out of sync with the header"


def test_exports_have_no_torch_or_cxx_types():
    h = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / "esm_b200.h").read_text(), flags=re.S)
    for bad in ("torch", "std::", "at::", "Tensor", "template"):
        assert bad not in h


def test_version_and_no_device_error():
    import torch

    from esm_b200 import _lib

    L = _lib.lib()
    assert b"sm_100a" in L.esmcu_version()
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = C.c_void_p()
    rc = L.esmcu_open(0, C.byref(h))
    assert rc in (7, 9) and not h.value
    assert L.esmcu_last_error()


def test_plan_batches_equals_reference(O, R):
    from esm_b200 import ops

    rng = np.random.default_rng(0)
    for n, thr, mb in [(1, 1.2, 256), (300, 1.2, 64), (257, 1.2, 256), (100, 1.5, 7), (64, 1.2, 0)]:
        lens = rng.integers(1, 500, n).astype(np.int32)
        lens[: n // 3] = 122  # plenty of ties
        order = np.zeros(n, np.int32)
        sizes = np.zeros(n, np.int32)
        ng = R.ref_plan_batches(lens.ctypes.data, n, thr, mb, order.ctypes.data, sizes.ctypes.data)
        want = []
        p = 0
        for s in sizes[:ng]:
            want.append(order[p:p + s].tolist())
            p += s
        assert ops.plan_batches(lens, thr, mb) == want
    assert ops.plan_batches(np.zeros(0, np.int32)) == []


def test_plan_batches_golden(O):
    from esm_b200 import ops

    G = np.load(ROOT / "tests" / "golden" / "ops_golden.npz")
    plan = ops.plan_batches(G["plan_lengths"], 1.2, 64)
    assert [len(g) for g in plan] == G["plan_sizes"].tolist()
    assert sum(plan, []) == G["plan_order"].tolist()


@pytest.mark.parametrize("T,n_masks,cu,B,ok", [
    (5, 0, [0, 2, 5], 2, True), (5, 5, [0, 5], 1, True), (0, 0, [0], 0, False),
    (5, 0, [1, 5], 1, False), (5, 0, [0, 3, 2, 5], 3, False), (5, 0, [0, 4], 1, False),
    (5, 3, [0, 5], 1, False), (5, 0, [0, 5], 2, False), (0, 0, [0, 0, 0], 2, True)])
def test_batch_view_validation_matches_reference(R, T, n_masks, cu, B, ok):
    from esm_b200 import EsmCudaError, ops

    cu = np.array(cu, np.int32)
    ids = np.zeros(max(T, 1), np.int32)
    masks = np.ones(max(n_masks, 1), np.int32)
    rc = R.ref_batch_view_check(ids.ctypes.data, T, masks.ctypes.data, n_masks, cu.ctypes.data,
                                cu.size, B)
    assert (rc == 0) == ok
    if ok:
        ops.batch_view_check(T, n_masks, cu, B)
    else:
        with pytest.raises(EsmCudaError) as e:
            ops.batch_view_check(T, n_masks, cu, B)
        assert R.ref_last_error().decode() in str(e.value)


def test_rope_tables_equal_reference(R):
    from esm_b200 import ops

    for L_, dh in [(1, 64), (1024, 64), (300, 16), (77, 24)]:
        c, s = ops.rope_build_tables(L_, dh)
        cr = np.zeros((L_, dh), np.float32)
        sr = np.zeros((L_, dh), np.float32)
        R.ref_rope_build_tables(L_, dh, cr.ctypes.data, sr.ctypes.data)
        assert np.array_equal(c, cr) and np.array_equal(s, sr)


def test_rope_tables_golden():
    from esm_b200 import ops

    G = np.load(ROOT / "tests" / "golden" / "ops_golden.npz")
    c, s = ops.rope_build_tables(256, 64)
    assert np.array_equal(c, G["rope_cos"]) and np.array_equal(s, G["rope_sin"])


def test_bad_arguments_are_rejected_without_a_device():
    from esm_b200 import EsmCudaError, ops

    with pytest.raises(EsmCudaError):
        ops.rope_build_tables(4, 3)  # odd head_dim


def test_model_entry_points_reject_null_handles_without_a_device():
    """The model-level entry points added for hidden states, scoring, the
    INT8 LM head, the fc1 fp16 flag and device quantisation return
    ESMCU_ERR_INVALID_ARGUMENT for a null handle before touching a device."""
    from esm_b200 import _lib

    L = _lib.lib()
    bad = 1  # ESMCU_ERR_INVALID_ARGUMENT
    assert L.esmcu_model_forward_hidden_states(None, None, None, 0, None, 0, None, None) == bad
    assert L.esmcu_model_masked_marginals(None, None, None, None, None, 1, 1.2, 256, None) == bad
    assert L.esmcu_model_set_head_int8(None, None, None) == bad
    assert L.esmcu_model_set_first_block_fc1_fp16(None, 1) == bad
    assert L.esmcu_quantize_weights(None, None, 4, 4, None, None) == bad
    assert L.esmcu_last_error()


def test_plan_batches_fuzz_against_reference_and_oracle(O, R):
    """PlanBatches (scheduler.cpp:13-75) under property-based inputs: the
    C-ABI host packer, the oracle and the compiled reference make the same
    groups in the same order (per-tensor W8A8 numerics depend on them)."""
    from hypothesis import HealthCheck, given, settings
    from hypothesis import strategies as st

    from esm_b200 import ops

    @settings(max_examples=150, deadline=None, suppress_health_check=list(HealthCheck))
    @given(lens=st.lists(st.integers(0, 1024), min_size=1, max_size=600),
           thr=st.sampled_from([1.0, 1.05, 1.2, 1.5, 3.0]),
           mb=st.sampled_from([0, 1, 7, 64, 256, 1000]))
    def check(lens, thr, mb):
        a = np.array(lens, np.int32)
        order = np.zeros(a.size, np.int32)
        sizes = np.zeros(a.size, np.int32)
        ng = R.ref_plan_batches(a.ctypes.data, a.size, thr, mb, order.ctypes.data, sizes.ctypes.data)
        want, p = [], 0
        for s in sizes[:ng]:
            want.append(order[p:p + s].tolist())
            p += s
        assert ops.plan_batches(a, thr, mb) == want
        assert O.plan_batches(a, thr, mb) == want

    check()


def test_batch_view_validation_fuzz_against_reference(R):
    """BatchView (batch.cpp:8-45) under property-based views, valid and not:
    the C-ABI check accepts exactly what the reference accepts and rejects
    the rest with the reference's message."""
    from hypothesis import HealthCheck, given, settings
    from hypothesis import strategies as st

    from esm_b200 import EsmCudaError, ops

    @settings(max_examples=200, deadline=None, suppress_health_check=list(HealthCheck))
    # Perturbations weighted towards zero: about a fifth of the views are valid,
    # the rest reach the reference's different rejection messages.
    @given(lens=st.lists(st.integers(-1, 40), min_size=0, max_size=12),
           dT=st.sampled_from([0, 0, 0, 0, 0, -1, 1, 2]),
           masks=st.sampled_from(["none", "match", "match", "short"]),
           dB=st.sampled_from([0, 0, 0, 0, -1, 1]), first=st.sampled_from([0, 0, 0, 0, 1]))
    def check(lens, dT, masks, dB, first):
        cu = np.concatenate([[first], first + np.cumsum(lens, dtype=np.int64)]).astype(np.int32)
        B = len(lens) + dB
        T = max(int(cu[-1]) + dT, 0)
        n_masks = {"none": 0, "match": T, "short": max(T - 1, 0)}[masks]
        ids = np.zeros(max(T, 1), np.int32)
        mk = np.ones(max(n_masks, 1), np.int32)
        rc = R.ref_batch_view_check(ids.ctypes.data, T, mk.ctypes.data, n_masks, cu.ctypes.data,
                                    cu.size, B)
        if rc == 0:
            ops.batch_view_check(T, n_masks, cu, B)
        else:
            with pytest.raises(EsmCudaError) as e:
                ops.batch_view_check(T, n_masks, cu, B)
            assert R.ref_last_error().decode() in str(e.value)

    check()
