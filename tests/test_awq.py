"""AWQ alpha search: the oracle against the reference's fixtures (CPU), and the
C-ABI validation of the AWQ reductions (no launch, no GPU).

Fixtures: tests/golden/make_awq.py ran ptqkit's awq_quantize (src/ptqkit/awq.py:39-81)
and replayed its loop to record every candidate's pre-scale and score; the inputs
are regenerated here from their seeds and checked against the recorded digests.

Tolerances: the score (awq.py:76-77) is checked to 1e-6 relative when it is
evaluated with the reference's own pre-scales (then the codes are bit-exact and
only the fp32-vs-fp64 arithmetic differs), and to 5e-3 relative end to end,
where a pre-scale a few ulp away can flip a handful of codes; the pre-scales
themselves to 5e-7 relative (a few fp32 ulp: m^alpha and the mean are rounded
differently).
"""

from __future__ import annotations

import ctypes
import importlib.util
import json
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN

import oracle


def awq_cases() -> tuple[list[dict], list[dict], dict[str, np.ndarray]]:
    spec = importlib.util.spec_from_file_location("make_awq", os.path.join(GOLDEN, "make_awq.py"))
    assert spec is not None and spec.loader is not None
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    with torch.random.fork_rng():
        cases = mod.cases()
    with open(os.path.join(GOLDEN, "awq_cases.json")) as f:
        meta = json.load(f)
    with np.load(os.path.join(GOLDEN, "awq_cases.npz")) as z:
        arrays = {k: z[k] for k in z.files}
    assert [c["name"] for c in cases] == [m["name"] for m in meta]
    for c, m in zip(cases, meta):
        assert mod.sha(c["w"]) == m["sha_w"] and mod.sha(c["x"]) == m["sha_x"], m["name"]
        if c["mean_abs"] is not None:
            assert mod.sha(c["mean_abs"]) == m["sha_mean_abs"], m["name"]
    return cases, meta, arrays


def search_rows(x: np.ndarray) -> np.ndarray:
    n = x.shape[0]
    return x if n <= 2048 else x[:: max(n // 2048, 1)][:2048]


def score(w: np.ndarray, x: np.ndarray, r: dict) -> float:
    s = search_rows(x).astype(np.float64)
    hat = oracle.dequantize(r["codes"], r["scales"], r["zeros"], r["channel_scale"], int(r["group_size"]))
    err = s @ hat.astype(np.float64).T - s @ w.astype(np.float64).T
    return float((err * err).mean())


def test_oracle_awq_matches_reference() -> None:
    cases, meta, z = awq_cases()
    for c, m in zip(cases, meta):
        name = m["name"]
        w, x = c["w"].numpy(), c["x"].numpy()
        ma = None if c["mean_abs"] is None else c["mean_abs"].numpy()
        r = oracle.awq_search(w, x, m["bits"], m["symmetric"], m["group_size"], tuple(m["alphas"]), ma)
        assert r["alpha"] == m["alpha"], name
        np.testing.assert_allclose(r["mag"], z[f"{name}.mag"], rtol=5e-7, err_msg=name)
        for i, a in enumerate(m["alphas"]):
            ref_pre = z[f"{name}.pre{i}"]
            np.testing.assert_allclose(r["pre_scale"][i], ref_pre, rtol=5e-7, err_msg=f"{name} pre alpha={a}")
            assert abs(r["mse"][i] - m["mse"][i]) <= 5e-3 * m["mse"][i], (name, a)
            # with the reference's pre-scale: bit-exact codes, score to fp32-vs-fp64 rounding
            rr = oracle.rtn_quantize(w, m["bits"], m["symmetric"], m["group_size"], ref_pre)
            assert abs(score(w, x, rr) - m["mse"][i]) <= 1e-6 * m["mse"][i], (name, a)
            if a == m["alpha"]:
                q = oracle.pack_int4(rr["codes"]) if m["bits"] == 4 else rr["codes"].astype(np.uint8)
                assert np.array_equal(q, z[f"{name}.q"]), name
                assert np.array_equal(rr["scales"].view(np.int32), z[f"{name}.scales"].view(np.int32)), name
                assert np.array_equal(rr["zeros"].view(np.int32), z[f"{name}.zeros"].view(np.int32)), name
                assert np.array_equal(rr["channel_scale"].view(np.int32), z[f"{name}.channel"].view(np.int32)), name


def test_oracle_alpha_zero_is_plain_rtn() -> None:
    # tests/test_awq.py:12-25 of the reference: alpha 0 gives s = 1, i.e. RTN
    cases, meta, _ = awq_cases()
    c, m = cases[0], meta[0]
    assert m["alphas"] == [0.0]
    r = oracle.awq_search(c["w"].numpy(), c["x"].numpy(), 4, True, 16, (0.0,))
    plain = oracle.rtn_quantize(c["w"].numpy(), 4, True, 16)
    assert np.array_equal(r["rtn"]["codes"], plain["codes"])
    assert np.array_equal(r["rtn"]["scales"], plain["scales"])


def test_awq_reduction_validation(wq) -> None:
    lib = wq._kernels.library()
    vp = ctypes.c_void_p
    dummy = vp(16)
    assert lib.wq_channel_abs_sum_f64(dummy, -1, 4, 4, dummy, None) == 5
    assert lib.wq_channel_abs_sum_f64(dummy, 2, 4, 3, dummy, None) == 20
    assert lib.wq_channel_abs_sum_f64(None, 2, 4, 4, dummy, None) == 11
    assert lib.wq_channel_abs_sum_f64(dummy, 2, 4, 4, None, None) == 11
    assert lib.wq_channel_abs_sum_f64(None, 0, 0, 0, None, None) == 0
    assert lib.wq_awq_pre_scale_f32(dummy, -3, 0.5, dummy, None) == 5
    assert lib.wq_awq_pre_scale_f32(None, 3, 0.5, dummy, None) == 11
    assert lib.wq_awq_pre_scale_f32(dummy, 3, 0.5, None, None) == 11
    ws = int(lib.wq_sq_err_workspace_bytes())
    assert ws > 0
    assert lib.wq_sq_err_sum_f64(dummy, dummy, -1, dummy, dummy, ws, None) == 5
    assert lib.wq_sq_err_sum_f64(dummy, dummy, 8, None, dummy, ws, None) == 11
    assert lib.wq_sq_err_sum_f64(dummy, dummy, 8, dummy, dummy, ws - 1, None) == 12
    assert lib.wq_sq_err_sum_f64(dummy, dummy, 8, dummy, None, ws, None) == 12


def test_awq_python_argument_errors(wq) -> None:
    awq = pytest.importorskip("weight-quantizer_b200.awq")
    cfg = wq.QuantConfig(bits=4, group_size=8, method=wq.Method.AWQ)
    with pytest.raises(ValueError, match="weight must have shape"):
        awq.awq_quantize(torch.zeros(4), torch.zeros(3, 4), cfg)
    with pytest.raises(ValueError, match=r"activations must have shape \[n, in\]"):
        awq.awq_quantize(torch.zeros(2, 4), torch.zeros(3, 5), cfg)
