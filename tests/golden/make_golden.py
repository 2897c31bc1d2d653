"""Generate the golden fixtures from the reference itself.

Run in a checkout where the ptqkit reference tree is mounted (default
WQ_REFERENCE_ROOT) after ``make -C oracle ref`` built its C++ kernel:

    python tests/golden/make_golden.py [--reference <ptqkit tree>]   (or WQ_REFERENCE_ROOT=<ptqkit tree>)

Writes, next to this script:

* ``small_cases.npz``  inputs and the reference's outputs for the known-answer
  cases of ptqkit's own tests (tests/test_gemm.py:13-65, tests/test_pack.py:6-25,
  tests/test_quant.py:13-60), RTN edge cases (zero blocks, constant blocks,
  signed zeros in narrow blocks, odd K, odd group sizes, pre_scale) and odd-shape
  dequant-GEMM cases. RTN outputs come from ptqkit.quant.quantize_weight; GEMM
  outputs from ptqkit._kernels.dequant_gemm (the compiled reference kernel) and
  from the reference's dense formulation (impl="reference").
* ``workload_digests.json``  SHA-256 digests of the seeded inputs of the five
  benchmark workloads (weight-quantizer_b200/workloads.py), of the reference's
  RTN outputs for them (stored codes, scales, zeros, channel scale) and of the
  reference kernel's outputs y per batch.

The GPU tests compare the CUDA path with these without needing the reference.
"""

from __future__ import annotations

import argparse
import hashlib
import importlib
import json
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.abspath(os.path.join(HERE, "..", ".."))


def sha(a: np.ndarray | torch.Tensor) -> str:
    if isinstance(a, torch.Tensor):
        a = a.detach().cpu().contiguous().numpy()
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def load_reference(ref_root: str):  # type: ignore[no-untyped-def]
    sys.path.insert(0, os.path.join(ref_root, "src"))
    sys.path.insert(0, REPO)
    import oracle

    kern = oracle.reference_kernels()
    if kern is None:
        raise SystemExit("build the reference kernel first: make -C oracle ref")
    sys.modules["ptqkit._kernels"] = kern
    ptq = importlib.import_module("ptqkit")
    return ptq, kern


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("WQ_REFERENCE_ROOT"),
                    help="ptqkit source tree (default: $WQ_REFERENCE_ROOT)")
    ap.add_argument("--skip-workloads", action="store_true")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set WQ_REFERENCE_ROOT to the ptqkit source tree")
    ptq, kern = load_reference(args.reference)
    from ptqkit.gemm import dequant_gemm as ref_gemm
    from ptqkit.pack import pack_int4 as ref_pack
    from ptqkit.quant import QuantConfig, assemble_quantized, quantize_weight

    out: dict[str, np.ndarray] = {}
    meta: list[dict[str, object]] = []

    def add_rtn(name: str, w: torch.Tensor, bits: int, sym: bool, group: int | None,
                pre: torch.Tensor | None = None) -> object:
        qw = quantize_weight(w, QuantConfig(bits=bits, symmetric=sym, group_size=group), pre_scale=pre)
        out[f"{name}.w"] = w.numpy().astype(np.float32)
        if pre is not None:
            out[f"{name}.pre"] = pre.numpy().astype(np.float32)
            out[f"{name}.channel"] = qw.channel_scale.numpy()
        out[f"{name}.q"] = qw.codes.numpy()
        out[f"{name}.scales"] = qw.scales.numpy()
        out[f"{name}.zeros"] = qw.zeros.numpy()
        meta.append({"name": name, "kind": "rtn", "bits": bits, "symmetric": sym, "group": group,
                     "stored_group": qw.group_size, "pre": pre is not None})
        return qw

    def add_gemm(name: str, qw: object, x: torch.Tensor) -> None:
        ch = None if qw.channel_scale is None else qw.channel_scale.numpy()  # type: ignore[attr-defined]
        y = kern.dequant_gemm(x.numpy(), qw.codes.numpy(), qw.scales.numpy(), qw.zeros.numpy(),  # type: ignore[attr-defined]
                              ch, int(qw.group_size), int(qw.bits), 1)  # type: ignore[attr-defined]
        y2 = kern.dequant_gemm(x.numpy(), qw.codes.numpy(), qw.scales.numpy(), qw.zeros.numpy(),  # type: ignore[attr-defined]
                               ch, int(qw.group_size), int(qw.bits), 2)  # type: ignore[attr-defined]
        assert np.array_equal(y, y2), "reference kernel must not depend on nthreads"
        out[f"{name}.x"] = x.numpy().astype(np.float32)
        out[f"{name}.y_kernel"] = y
        out[f"{name}.y_reference"] = ref_gemm(x, qw, impl="reference").numpy()
        meta.append({"name": name, "kind": "gemm", "rtn": name})

    # --- KAT: nibble dot (tests/test_gemm.py:13-32) ---------------------------
    codes = torch.tensor([[1, 2], [15, 0]], dtype=torch.int32)
    qw = assemble_quantized(codes, torch.tensor([[1.0], [1.0]]), torch.zeros(2, 1), bits=4,
                            group_size=2, symmetric=True, granularity="channel")
    out["kat_nibble.codes"] = codes.numpy()
    out["kat_nibble.q"] = qw.codes.numpy()
    out["kat_nibble.scales"] = qw.scales.numpy()
    out["kat_nibble.zeros"] = qw.zeros.numpy()
    add_gemm("kat_nibble", qw, torch.tensor([[1.0, 0.0], [0.0, 1.0], [1.0, 1.0]]))
    meta.append({"name": "kat_nibble", "kind": "kat", "bits": 4, "stored_group": 2})

    # --- KAT: nibble layout (tests/test_pack.py:6-13) --------------------------
    codes = torch.tensor([[1, 2, 15, 0], [0, 15, 8, 8]], dtype=torch.int32)
    out["kat_pack.codes"] = codes.numpy()
    out["kat_pack.packed"] = ref_pack(codes).numpy()
    g = torch.Generator().manual_seed(7)
    codes = torch.randint(0, 16, (5, 7), generator=g, dtype=torch.int32)
    out["pack_odd.codes"] = codes.numpy()
    out["pack_odd.packed"] = ref_pack(codes).numpy()

    # --- differential cases of tests/test_gemm.py:35-65 ------------------------
    cases = [
        (4, 8, 1, 8, True, None, False),
        (5, 7, 3, 8, True, 0, False),
        (8, 16, 4, 4, True, 8, False),
        (3, 13, 1, 4, False, 4, False),
        (6, 32, 5, 4, True, 16, True),
        (32, 128, 2, 4, True, 128, False),
        (4, 1, 2, 8, True, None, False),
        (7, 17, 8, 8, False, None, False),
    ]
    g = torch.Generator().manual_seed(0)
    for i, (o, inn, batch, bits, sym, group, use_pre) in enumerate(cases):
        w = torch.randn(o, inn, generator=g)
        pre = torch.rand(inn, generator=g) + 0.25 if use_pre else None
        qw = add_rtn(f"refcase{i}", w, bits, sym, group, pre)
        add_gemm(f"refcase{i}", qw, torch.randn(batch, inn, generator=g))

    # --- RTN edge tensors (tests/test_quant.py:13-44 shapes) and signed zeros --
    g = torch.Generator().manual_seed(1)
    tensors = {
        "randn17x32": torch.randn(17, 32, generator=g),
        "randn4x7": torch.randn(4, 7, generator=g),
        "randn8x128": torch.randn(8, 128, generator=g),
        "linspace": torch.linspace(-1.5, 2.0, 128).reshape(4, 32),
        "zeros": torch.zeros(4, 8),
        "half": torch.full((3, 16), 0.5),
        "neghalf": torch.full((3, 16), -0.5),
        "negzero_first": torch.tensor([[-0.0, 0.0, 1.0, 2.0], [0.0, -0.0, 3.0, 1.0], [-0.0, -0.0, 0.5, 0.25]]),
        "allnegzero": torch.tensor([[-0.0] * 6] * 3),
        "mixed_zero_neg": torch.tensor([[-0.0, -1.0, 0.0, 2.0, 0.0, -0.0]] * 2),
        "tiny": torch.randn(5, 24, generator=g) * 1e-30,
        "huge": torch.randn(5, 24, generator=g) * 1e30,
    }
    for tname, w in tensors.items():
        for bits in (4, 8):
            for sym in (True, False):
                for group in (0, None, 2, 16):
                    add_rtn(f"edge.{tname}.{bits}.{int(sym)}.{group}", w, bits, sym, group)
    # odd K, odd group sizes, K = 1, pre_scale with every granularity
    g = torch.Generator().manual_seed(2)
    for (o, inn, group) in [(5, 13, 3), (7, 33, 5), (3, 1, 1), (6, 31, 7), (9, 65, 64), (4, 127, 128)]:
        for bits in (4, 8):
            for sym in (True, False):
                w = torch.randn(o, inn, generator=g)
                qw = add_rtn(f"odd.{o}x{inn}.g{group}.{bits}.{int(sym)}", w, bits, sym, group)
                add_gemm(f"odd.{o}x{inn}.g{group}.{bits}.{int(sym)}", qw, torch.randn(3, inn, generator=g))
    for group in (0, None, 8):
        for sym in (True, False):
            w = torch.randn(6, 40, generator=g)
            pre = torch.rand(40, generator=g) + 0.2
            qw = add_rtn(f"pre.g{group}.{int(sym)}", w, 4, sym, group, pre)
            add_gemm(f"pre.g{group}.{int(sym)}", qw, torch.randn(4, 40, generator=g))

    np.savez_compressed(os.path.join(HERE, "small_cases.npz"), **out)
    with open(os.path.join(HERE, "small_cases.json"), "w") as f:
        json.dump(meta, f, indent=0)
    print(f"small cases: {len(meta)} entries, {len(out)} arrays")

    if args.skip_workloads:
        return
    # --- full-size workload digests -------------------------------------------
    wl = importlib.import_module("weight-quantizer_b200.workloads")
    threads = os.cpu_count() or 1
    digests: dict[str, object] = {"reference_kernel_threads": threads}
    for wname, fn in wl.WORKLOADS.items():
        t0 = time.time()
        layers = fn()
        entries = []
        for layer in layers:
            cfg = layer.config
            qw = quantize_weight(layer.weight, QuantConfig(bits=cfg.bits, symmetric=cfg.symmetric,
                                                           group_size=cfg.group_size),
                                 pre_scale=layer.pre_scale)
            e: dict[str, object] = {
                "name": layer.name,
                "w": sha(layer.weight),
                "q": sha(qw.codes),
                "scales": sha(qw.scales),
                "zeros": sha(qw.zeros),
                "group_size": int(qw.group_size),
                "y": {},
            }
            if layer.pre_scale is not None:
                e["pre"] = sha(layer.pre_scale)
                e["channel"] = sha(qw.channel_scale)
            ch = None if qw.channel_scale is None else qw.channel_scale.numpy()
            for b, x in layer.x.items():
                e.setdefault("x", {})[str(b)] = sha(x)  # type: ignore[index]
                y = kern.dequant_gemm(x.numpy(), qw.codes.numpy(), qw.scales.numpy(), qw.zeros.numpy(), ch,
                                      int(qw.group_size), int(qw.bits), threads)
                e["y"][str(b)] = sha(y)  # type: ignore[index]
            entries.append(e)
        digests[wname] = entries
        print(f"{wname}: {len(entries)} layers, {time.time() - t0:.1f}s", flush=True)
    with open(os.path.join(HERE, "workload_digests.json"), "w") as f:
        json.dump(digests, f, indent=1)


if __name__ == "__main__":
    main()
