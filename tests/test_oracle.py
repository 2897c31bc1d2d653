"""The CPU oracle pinned against outputs of the reference itself.

The fixtures in tests/golden were produced by ptqkit's own Python RTN
(src/ptqkit/quant.py:225-289) and its compiled C++ kernel
(src/ptqkit/csrc/dequant_gemm.cpp) by tests/golden/make_golden.py. The oracle
must reproduce them bit for bit before it is trusted as the checker of the
CUDA path.
"""

from __future__ import annotations

import importlib

import numpy as np
import pytest

from conftest import sha, small_cases, workload_digests


def _group_arg(meta: dict) -> int | None:
    return meta["group"]


def test_pack_known_answer(orc) -> None:
    # tests/test_pack.py:6-13: bytes 0x21, 0x0F and 0xF0
    data, _ = small_cases()
    packed = orc.pack_int4(data["kat_pack.codes"])
    assert packed[0, 0] == 0x21 and packed[0, 1] == 0x0F and packed[1, 0] == 0xF0
    assert np.array_equal(packed, data["kat_pack.packed"])
    assert np.array_equal(orc.unpack_int4(packed, 4), data["kat_pack.codes"].astype(np.uint8))
    odd = orc.pack_int4(data["pack_odd.codes"])
    assert odd.shape == (5, 4)
    assert np.array_equal(odd, data["pack_odd.packed"])
    assert np.array_equal(orc.unpack_int4(odd, 7), data["pack_odd.codes"].astype(np.uint8))


def test_nibble_dot_known_answer(orc) -> None:
    # tests/test_gemm.py:13-32
    data, _ = small_cases()
    y = orc.dequant_gemm(data["kat_nibble.x"], data["kat_nibble.q"], data["kat_nibble.scales"],
                         data["kat_nibble.zeros"], None, 2, 4)
    assert np.allclose(y, [[1.0, 15.0], [2.0, 0.0], [3.0, 15.0]], atol=1e-6)
    assert np.array_equal(y.view(np.int32), data["kat_nibble.y_kernel"].view(np.int32))


def test_rtn_bit_exact_small(orc) -> None:
    data, meta = small_cases()
    n = 0
    for m in meta:
        if m["kind"] != "rtn":
            continue
        name = m["name"]
        pre = data.get(f"{name}.pre")
        r = orc.quantize_stored(data[f"{name}.w"], m["bits"], m["symmetric"], _group_arg(m), pre)
        assert np.array_equal(r["q"], data[f"{name}.q"]), name
        assert np.array_equal(r["scales"].view(np.int32), data[f"{name}.scales"].view(np.int32)), name
        assert np.array_equal(r["zeros"].view(np.int32), data[f"{name}.zeros"].view(np.int32)), name
        assert r["group_size"] == m["stored_group"], name
        if pre is not None:
            assert np.array_equal(r["channel_scale"].view(np.int32), data[f"{name}.channel"].view(np.int32))
        n += 1
    assert n > 200


def test_gemm_bit_exact_with_reference_kernel(orc) -> None:
    data, meta = small_cases()
    rtn = {m["name"]: m for m in meta if m["kind"] in ("rtn", "kat")}
    n = 0
    for m in meta:
        if m["kind"] != "gemm":
            continue
        name = m["name"]
        r = rtn[name]
        y = orc.dequant_gemm(data[f"{name}.x"], data[f"{name}.q"], data[f"{name}.scales"],
                             data[f"{name}.zeros"], data.get(f"{name}.channel"), r["stored_group"], r["bits"])
        assert np.array_equal(y.view(np.int32), data[f"{name}.y_kernel"].view(np.int32)), name
        # the reference's own kernel vs its dense formulation (tests/test_gemm.py:62)
        assert np.allclose(y, data[f"{name}.y_reference"], rtol=1e-4, atol=1e-4), name
        # thread-count invariance (tests/test_gemm.py:63-65)
        y1 = orc.dequant_gemm(data[f"{name}.x"], data[f"{name}.q"], data[f"{name}.scales"],
                              data[f"{name}.zeros"], data.get(f"{name}.channel"), r["stored_group"], r["bits"], 1)
        assert np.array_equal(y, y1)
        n += 1
    assert n > 30


def test_reference_kernel_module_matches_oracle(orc) -> None:
    """When the reference kernel was compiled here (oracle/_ref), compare directly."""
    kern = orc.reference_kernels()
    if kern is None:
        pytest.skip("reference kernel not built in this checkout")
    assert kern.kernel_info()["openmp"] is True
    data, meta = small_cases()
    for m in meta:
        if m["kind"] != "gemm":
            continue
        name = m["name"]
        r = next(x for x in meta if x["name"] == name and x["kind"] in ("rtn", "kat"))
        ch = data.get(f"{name}.channel")
        y = kern.dequant_gemm(data[f"{name}.x"], data[f"{name}.q"], data[f"{name}.scales"],
                              data[f"{name}.zeros"], ch, r["stored_group"], r["bits"], 1)
        assert np.array_equal(y, data[f"{name}.y_kernel"]), name


WORKLOADS_CPU = ["gpt2_c_fc_int4_g128", "gpt2_small_int8_asym", "awq_11008x4096", "oddk_4096x4095_g64"]


def _check_workload(orc, wname: str, max_batch: int) -> None:
    wl = importlib.import_module("weight-quantizer_b200.workloads")
    dig = workload_digests()[wname]
    layers = wl.WORKLOADS[wname]()
    assert len(layers) == len(dig)
    for layer, d in zip(layers, dig):
        assert sha(layer.weight) == d["w"], f"{wname}: seeded weight changed"
        cfg = layer.config
        pre = None if layer.pre_scale is None else layer.pre_scale.numpy()
        r = orc.quantize_stored(layer.weight.numpy(), cfg.bits, cfg.symmetric, cfg.group_size, pre)
        assert sha(r["q"]) == d["q"], f"{wname}/{layer.name}: codes"
        assert sha(r["scales"]) == d["scales"], f"{wname}/{layer.name}: scales"
        assert sha(r["zeros"]) == d["zeros"], f"{wname}/{layer.name}: zeros"
        if pre is not None:
            assert sha(r["channel_scale"]) == d["channel"]
        for b, x in layer.x.items():
            assert sha(x) == d["x"][str(b)]
            if b > max_batch:
                continue
            y = orc.dequant_gemm(x.numpy(), r["q"], r["scales"], r["zeros"], r["channel_scale"],
                                 int(r["group_size"]), cfg.bits)
            assert sha(y) == d["y"][str(b)], f"{wname}/{layer.name}: y at batch {b}"


@pytest.mark.parametrize("wname", WORKLOADS_CPU)
def test_oracle_matches_reference_on_workloads(orc, wname: str) -> None:
    _check_workload(orc, wname, max_batch=64)


@pytest.mark.slow
def test_oracle_matches_reference_on_sharded_workload(orc) -> None:
    _check_workload(orc, "sharded_28672x8192", max_batch=32)
