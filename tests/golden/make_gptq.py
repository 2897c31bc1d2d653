"""Generate the GPTQ golden fixtures from the reference itself.

Run where the ptqkit reference tree is mounted (the --reference argument or WQ_REFERENCE_ROOT):

    python tests/golden/make_gptq.py [--reference <ptqkit tree>]   (or WQ_REFERENCE_ROOT=<ptqkit tree>)

Each case is a seeded weight and Hessian (the three cases of the reference's
tests/test_gptq.py, then group, channel and tensor grids with correlated
inputs, a dead input channel, an odd last group and a group wider than 128
columns); inputs sit on a 1/64 grid so that the Hessians are exact; the outputs are ptqkit's own ``gptq_quantize`` (src/ptqkit/gptq.py:128-191):
stored codes, fp32 scales and zeros, and the output error
mean((X W_hat^T - X W^T)^2) on the case's inputs.

Writes ``gptq_cases.npz`` (outputs) and ``gptq_cases.json`` (configs, errors,
SHA-256 digests of the inputs) next to this script. ``cases()`` regenerates
the inputs; the tests call it and check the digests.
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


def _grid(x: torch.Tensor) -> torch.Tensor:
    """x rounded to multiples of 1/64: with |x| < 512 every product x_i x_j and every
    partial sum of up to 2^11 of them is exact in fp64, so X^T X is the same on any
    CPU whatever the summation order of its BLAS."""
    return torch.round(x * 64) / 64


def _hessian(x: torch.Tensor) -> torch.Tensor:
    return x.double().transpose(0, 1) @ x.double() / x.shape[0]


def cases() -> list[dict]:
    out = []
    # The three cases of the reference's tests/test_gptq.py, same seeds and shapes;
    # inputs on the 1/64 grid and the rank-2 product formed elementwise, so that
    # inputs and Hessians are reproducible bit for bit on any CPU.
    torch.manual_seed(0)
    w = torch.randn(8, 32)
    x = _grid(torch.randn(64, 32))
    out.append(dict(name="ref_identity", w=w, x=x, h=torch.eye(32, dtype=torch.float64),
                    bits=4, sym=True, group=16, percdamp=0.0, blocksize=128))
    torch.manual_seed(0)
    a, b = torch.randn(2048, 2), torch.randn(2, 32)
    latent = a[:, 0:1] * b[0:1, :] + a[:, 1:2] * b[1:2, :]
    latent[:, 0] *= 5
    latent = _grid(latent)
    w = torch.randn(8, 32) * 0.1
    w[:, 3] = 6
    out.append(dict(name="ref_latent", w=w, x=latent, h=_hessian(latent),
                    bits=4, sym=True, group=32, percdamp=0.01, blocksize=128))
    torch.manual_seed(1)
    x = _grid(torch.randn(64, 16))
    x[:, 3] = 0
    w = torch.randn(4, 16)
    out.append(dict(name="ref_dead", w=w, x=x, h=_hessian(x),
                    bits=4, sym=False, group=None, percdamp=0.01, blocksize=128))

    def correlated(g: torch.Generator, n: int, k: int, rank: int) -> torch.Tensor:
        # column j follows latent factor j % rank, plus per-channel noise of magnitude 2^e
        z = torch.randn(n, rank, generator=g)
        coef = torch.randn(k, generator=g)
        mag = torch.pow(2.0, torch.randint(-2, 3, (k,), generator=g).to(torch.float32))
        idx = torch.arange(k) % rank
        return _grid(z[:, idx] * coef + 0.3 * torch.randn(n, k, generator=g) * mag)

    specs = [
        ("g128_sym", 48, 256, 4, True, 128, 128, None),
        ("g64_asym_oddk", 40, 200, 4, False, 64, 128, 7),
        ("int8_channel_b32", 32, 160, 8, True, None, 32, None),
        ("tensor_sym", 24, 96, 4, True, 0, 128, None),
        ("wide_group256", 16, 256, 4, True, 256, 128, None),
        ("int8_g128_asym", 24, 384, 8, False, 128, 128, 100),
    ]
    for i, (name, m, k, bits, sym, group, bs, dead) in enumerate(specs):
        g = torch.Generator().manual_seed(100 + i)
        x = correlated(g, 4 * k, k, max(2, k // 16))
        if dead is not None:
            x[:, dead] = 0
        w = torch.randn(m, k, generator=g) * 0.05
        out.append(dict(name=name, w=w, x=x, h=_hessian(x), bits=bits, sym=sym, group=group, percdamp=0.01,
                        blocksize=bs))
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("WQ_REFERENCE_ROOT"),
                    help="ptqkit source tree (default: $WQ_REFERENCE_ROOT)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set WQ_REFERENCE_ROOT to the ptqkit source tree")
    sys.path.insert(0, os.path.join(args.reference, "src"))
    gptq = importlib.import_module("ptqkit.gptq")
    quant = importlib.import_module("ptqkit.quant")
    arrays: dict[str, np.ndarray] = {}
    meta = []
    for c in cases():
        cfg = quant.QuantConfig(bits=c["bits"], symmetric=c["sym"], group_size=c["group"], method=quant.Method.GPTQ,
                                percdamp=c["percdamp"], blocksize=c["blocksize"])
        qw = gptq.gptq_quantize(c["w"], c["h"], cfg)
        hat = quant.dequantize_weight(qw)
        err = float((c["x"] @ (hat - c["w"]).transpose(0, 1)).square().mean().item())
        rtn = quant.dequantize_weight(quant.quantize_weight(c["w"], quant.QuantConfig(
            bits=c["bits"], symmetric=c["sym"], group_size=c["group"])))
        err_rtn = float((c["x"] @ (rtn - c["w"]).transpose(0, 1)).square().mean().item())
        arrays[f"{c['name']}.q"] = qw.codes.numpy()
        arrays[f"{c['name']}.scales"] = qw.scales.numpy()
        arrays[f"{c['name']}.zeros"] = qw.zeros.numpy()
        meta.append({"name": c["name"], "bits": c["bits"], "symmetric": c["sym"], "group_size": c["group"],
                     "percdamp": c["percdamp"], "blocksize": c["blocksize"], "stored_group": qw.group_size,
                     "out_err": err, "rtn_err": err_rtn,
                     "sha_w": sha(c["w"]), "sha_x": sha(c["x"]), "sha_h": sha(c["h"])})
        print(c["name"], "gptq err %.6g  rtn err %.6g" % (err, err_rtn))
    np.savez_compressed(os.path.join(HERE, "gptq_cases.npz"), **arrays)
    with open(os.path.join(HERE, "gptq_cases.json"), "w") as f:
        json.dump(meta, f, indent=1)


if __name__ == "__main__":
    main()
