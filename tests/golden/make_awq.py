"""Generate the AWQ golden fixtures from the reference itself.

Run where the ptqkit reference tree is mounted (the --reference argument or WQ_REFERENCE_ROOT):

    python tests/golden/make_awq.py [--reference <ptqkit tree>]   (or WQ_REFERENCE_ROOT=<ptqkit tree>)

For each case, the inputs are seeded CPU tensors, and the outputs come from
ptqkit's own code: ``ptqkit.awq.awq_quantize`` gives the winning alpha and the
quantized weight, and the search loop of src/ptqkit/awq.py:53-79 is replayed
with ptqkit's functions (``_subsample``, ``quantize_weight``,
``dequantize_weight``) to record every candidate's pre-scale and score. The
replay must pick the same alpha and codes as awq_quantize.

Writes ``awq_cases.npz`` (per-alpha pre-scales, the channel magnitudes, the
reference's stored codes/scales/zeros/channel scale) and ``awq_cases.json``
(configs, alphas, per-alpha scores, the winning alpha, SHA-256 digests of the
inputs) next to this script. The inputs themselves are not stored: ``cases()``
regenerates them from their seeds (the tests call it and check the digests).
"""

from __future__ import annotations

import argparse
import hashlib
import importlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(np.ascontiguousarray(t.detach().cpu().numpy()).tobytes()).hexdigest()


def cases() -> list[dict]:
    out = []
    # tests/test_awq.py:12-25 and :28-41 of the reference, same seeds and shapes
    torch.manual_seed(0)
    w = torch.randn(6, 32)
    x = torch.randn(40, 32)
    out.append(dict(name="kat_alpha_zero", w=w, x=x, bits=4, sym=True, group=16, alphas=(0.0,), mean_abs=None))
    torch.manual_seed(0)
    w = torch.randn(6, 32) * 0.1
    w[:, 1] = 3.0
    x = torch.randn(48, 32)
    x[:, 0] *= 20
    out.append(dict(name="kat_search", w=w, x=x, bits=4, sym=True, group=16, alphas=None, mean_abs=None))

    def acts(g: torch.Generator, n: int, k: int) -> torch.Tensor:
        # channel magnitudes ~ LogNormal(0, 1), 1% of channels x20
        m = torch.exp(torch.randn(k, generator=g))
        x = torch.randn(n, k, generator=g) * m
        idx = torch.randperm(k, generator=g)[: max(1, round(0.01 * k))]
        x[:, idx] *= 20
        return x

    g = torch.Generator().manual_seed(11)
    out.append(dict(name="g128_asym", w=torch.randn(96, 256, generator=g) * 0.02, x=acts(g, 600, 256),
                    bits=4, sym=False, group=128, alphas=None, mean_abs=None))
    g = torch.Generator().manual_seed(12)
    out.append(dict(name="int8_g64_sym", w=torch.randn(64, 192, generator=g) * 0.02, x=acts(g, 500, 192),
                    bits=8, sym=True, group=64, alphas=None, mean_abs=None))
    g = torch.Generator().manual_seed(13)
    x = acts(g, 700, 128)
    # mean_abs the way ActivationStats produces it (convert.py:47-63): fp64 sums, then fp32
    mean_abs = (x.double().abs().sum(dim=0) / x.shape[0]).to(torch.float32)
    out.append(dict(name="channel_asym_meanabs", w=torch.randn(48, 128, generator=g) * 0.02, x=x,
                    bits=4, sym=False, group=None, alphas=None, mean_abs=mean_abs))
    g = torch.Generator().manual_seed(14)
    out.append(dict(name="tensor_sym", w=torch.randn(40, 128, generator=g) * 0.02, x=acts(g, 300, 128),
                    bits=4, sym=True, group=0, alphas=None, mean_abs=None))
    g = torch.Generator().manual_seed(15)
    out.append(dict(name="oddk_g64", w=torch.randn(33, 255, generator=g) * 0.02, x=acts(g, 200, 255),
                    bits=4, sym=True, group=64, alphas=(0.0, 0.3, 0.6, 0.9), mean_abs=None))
    g = torch.Generator().manual_seed(16)
    # more than 2 x 2048 rows: the search takes every second row (awq.py:31-36)
    out.append(dict(name="subsample_stride2", w=torch.randn(24, 32, generator=g) * 0.02, x=acts(g, 4100, 32),
                    bits=4, sym=False, group=32, alphas=None, mean_abs=None))
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("WQ_REFERENCE_ROOT"),
                    help="ptqkit source tree (default: $WQ_REFERENCE_ROOT)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set WQ_REFERENCE_ROOT to the ptqkit source tree")
    sys.path.insert(0, os.path.join(args.reference, "src"))
    awq = importlib.import_module("ptqkit.awq")
    quant = importlib.import_module("ptqkit.quant")

    arrays: dict[str, np.ndarray] = {}
    meta = []
    for c in cases():
        kw = {} if c["alphas"] is None else {"awq_alphas": c["alphas"]}
        cfg = quant.QuantConfig(bits=c["bits"], symmetric=c["sym"], group_size=c["group"], method=quant.Method.AWQ, **kw)
        qw, alpha = awq.awq_quantize(c["w"], c["x"], cfg, mean_abs=c["mean_abs"])
        # replay of awq.py:53-79 with the reference's own functions
        w = c["w"].to(torch.float32)
        x_all = c["x"].to(torch.float32)
        if c["mean_abs"] is None:
            mag = x_all.abs().mean(dim=0).clamp(min=1e-8)
        else:
            mag = c["mean_abs"].to(torch.float32).reshape(-1).clamp(min=1e-8)
        search = awq._subsample(x_all, awq._SEARCH_ROWS)
        target = search @ w.transpose(0, 1)
        mses, best, best_mse = [], None, float("inf")
        for i, a in enumerate(cfg.awq_alphas):
            a = float(a)
            if a == 0.0:
                pre = torch.ones(w.shape[1], dtype=torch.float32)
            else:
                pre = mag.pow(a)
                pre = pre / pre.mean().clamp(min=1e-8)
            cand = quant.quantize_weight(w, cfg, pre_scale=pre)
            hat = quant.dequantize_weight(cand)
            mse = float((search @ hat.transpose(0, 1) - target).square().mean().item())
            mses.append(mse)
            arrays[f"{c['name']}.pre{i}"] = pre.numpy()
            if mse < best_mse:
                best_mse, best = mse, (a, cand)
        assert best is not None and best[0] == alpha, (c["name"], best[0], alpha)
        assert torch.equal(best[1].codes, qw.codes)
        arrays[f"{c['name']}.mag"] = mag.numpy()
        arrays[f"{c['name']}.q"] = qw.codes.numpy()
        arrays[f"{c['name']}.scales"] = qw.scales.numpy()
        arrays[f"{c['name']}.zeros"] = qw.zeros.numpy()
        arrays[f"{c['name']}.channel"] = qw.channel_scale.numpy()
        meta.append({"name": c["name"], "bits": c["bits"], "symmetric": c["sym"], "group_size": c["group"],
                     "stored_group": qw.group_size, "alphas": [float(a) for a in cfg.awq_alphas],
                     "mse": mses, "alpha": alpha, "has_mean_abs": c["mean_abs"] is not None,
                     "sha_w": sha(c["w"]), "sha_x": sha(c["x"]),
                     "sha_mean_abs": None if c["mean_abs"] is None else sha(c["mean_abs"])})
        print(c["name"], "alpha", alpha, "mse", ["%.6g" % m for m in mses])
    np.savez_compressed(os.path.join(HERE, "awq_cases.npz"), **arrays)
    with open(os.path.join(HERE, "awq_cases.json"), "w") as f:
        json.dump(meta, f, indent=1)


if __name__ == "__main__":
    main()
