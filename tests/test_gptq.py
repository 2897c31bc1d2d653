"""GPTQ: the oracle against the reference's fixtures (CPU), and the C-ABI
validation of the GPTQ sweep entry points (no launch, no GPU).

Fixtures: tests/golden/make_gptq.py ran ptqkit's gptq_quantize
(src/ptqkit/gptq.py:128-191); inputs are regenerated from their seeds and
checked against the recorded digests. The oracle (numpy fp64, LAPACK
factorization) reproduces the reference's stored codes, scales and zeros bit
for bit on every case.
"""

from __future__ import annotations

import ctypes
import importlib.util
import json
import os

import numpy as np
import torch

from conftest import GOLDEN

import oracle


def gptq_cases() -> tuple[list[dict], list[dict], dict[str, np.ndarray]]:
    spec = importlib.util.spec_from_file_location("make_gptq", os.path.join(GOLDEN, "make_gptq.py"))
    assert spec is not None and spec.loader is not None
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    with torch.random.fork_rng():
        cases = mod.cases()
    with open(os.path.join(GOLDEN, "gptq_cases.json")) as f:
        meta = json.load(f)
    with np.load(os.path.join(GOLDEN, "gptq_cases.npz")) as z:
        arrays = {k: z[k] for k in z.files}
    assert [c["name"] for c in cases] == [m["name"] for m in meta]
    for c, m in zip(cases, meta):
        assert mod.sha(c["w"]) == m["sha_w"] and mod.sha(c["x"]) == m["sha_x"] and mod.sha(c["h"]) == m["sha_h"]
    return cases, meta, arrays


def unpacked(q: np.ndarray, bits: int, k: int) -> np.ndarray:
    return oracle.unpack_int4(q, k).astype(np.int32) if bits == 4 else q.astype(np.int32)


def out_err(x: np.ndarray, w: np.ndarray, hat: np.ndarray) -> float:
    e = x.astype(np.float64) @ (hat.astype(np.float64) - w.astype(np.float64)).T
    return float((e * e).mean())


def test_oracle_gptq_matches_reference() -> None:
    cases, meta, z = gptq_cases()
    for c, m in zip(cases, meta):
        name = m["name"]
        w = c["w"].numpy()
        r = oracle.gptq_quantize(w, c["h"].numpy(), m["bits"], m["symmetric"], m["group_size"], m["percdamp"],
                                 m["blocksize"])
        assert np.array_equal(r["codes"], unpacked(z[f"{name}.q"], m["bits"], w.shape[1])), name
        assert np.array_equal(r["scales"].view(np.int32), z[f"{name}.scales"].view(np.int32)), name
        assert np.array_equal(r["zeros"], z[f"{name}.zeros"]), name
        assert r["group_size"] == m["stored_group"]
        hat = oracle.dequantize(r["codes"], r["scales"], r["zeros"], None, int(r["group_size"]))
        assert abs(out_err(c["x"].numpy(), w, hat) - m["out_err"]) <= 1e-6 * m["out_err"], name


def test_gptq_entry_point_validation(wq) -> None:
    lib = wq._kernels.library()
    d = ctypes.c_void_p(16)
    assert lib.wq_gptq_qparams_f64(d, -1, 4, 0, 4, 4, 1, 0, d, d, 1, None, 0, None) == 5
    assert lib.wq_gptq_qparams_f64(d, 2, 4, 3, 2, 4, 1, 0, d, d, 1, None, 0, None) == 5
    assert lib.wq_gptq_qparams_f64(d, 2, 4, 0, 4, 5, 1, 0, d, d, 1, None, 0, None) == 3
    assert lib.wq_gptq_qparams_f64(d, 2, 3, 0, 4, 4, 1, 0, d, d, 1, None, 0, None) == 20
    assert lib.wq_gptq_qparams_f64(d, 2, 4, 0, 4, 4, 1, 1, d, d, 1, None, 0, None) == 12
    assert lib.wq_gptq_qparams_f64(None, 2, 4, 0, 4, 4, 1, 0, d, d, 1, None, 0, None) == 11
    assert lib.wq_gptq_block_f64(d, 2, 256, d, 256, 0, 129, d, d, 1, 4, d, 256, d, None, None, None) == 13
    assert lib.wq_gptq_block_f64(d, 2, 64, d, 256, 0, 128, d, d, 1, 4, d, 256, d, None, None, None) == 20
    assert lib.wq_gptq_block_f64(d, 2, 256, d, 256, 0, 64, d, d, 1, 8, None, 256, d, None, None, None) == 11
    assert lib.wq_gptq_block_f64(d, -2, 256, d, 256, 0, 64, d, d, 1, 8, d, 256, d, None, None, None) == 5
    assert lib.wq_gptq_block_f64(d, 2, 256, d, 256, 0, 64, d, d, 1, 6, d, 256, d, None, None, None) == 3
    # the tail update: negative sizes, short strides, null pointers
    assert lib.wq_gptq_tail_f64(d, -1, 8, 0, 8, d, 4, d, 8, 0, None) == 5
    assert lib.wq_gptq_tail_f64(d, 2, 8, 4, 8, d, 4, d, 16, 0, None) == 20
    assert lib.wq_gptq_tail_f64(None, 2, 16, 4, 8, d, 4, d, 16, 0, None) == 11
    # the factor of the inverse: sizes, strides, pointers, workspace (no GPU work)
    assert lib.wq_chol_inverse_upper_workspace_bytes(100) == 2 * 100 * 100 * 8
    assert lib.wq_chol_inverse_upper_workspace_bytes(0) == 0
    assert lib.wq_chol_inverse_upper_f64(d, -1, 4, d, 4, d, 1 << 20, d, None) == 5
    assert lib.wq_chol_inverse_upper_f64(d, 4, 4, d, 4, d, 1 << 20, None, None) == 11
    assert lib.wq_chol_inverse_upper_f64(d, 8, 4, d, 8, d, 1 << 20, d, None) == 20
    assert lib.wq_chol_inverse_upper_f64(d, 8, 8, d, 7, d, 1 << 20, d, None) == 20
    assert lib.wq_chol_inverse_upper_f64(None, 8, 8, d, 8, d, 1 << 20, d, None) == 11
    assert lib.wq_chol_inverse_upper_f64(d, 8, 8, d, 8, d, 2 * 8 * 8 * 8 - 1, d, None) == 12
    assert lib.wq_chol_inverse_upper_f64(d, 50000, 50000, d, 50000, d, 1 << 62, d, None) == 13
