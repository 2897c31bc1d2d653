"""Generate the compressed-format fixtures from the reference itself.

Run where the ptqkit reference tree is mounted (the --reference argument or WQ_REFERENCE_ROOT),
after ``make -C oracle ref`` built its C++ kernel:

    python tests/golden/make_compressed.py [--reference <ptqkit tree>]   (or WQ_REFERENCE_ROOT=<ptqkit tree>)

For each case below a ``CompressedNet`` (defined here; the tests import this
file for the class) is built from a seed, quantized by ptqkit's
``quantize_model`` (src/ptqkit/convert.py:236-293) and written by ptqkit's
``save_compressed`` (convert.py:364-370), i.e. the version-1 payload of
``compressed_state`` (convert.py:296-336) through ``torch.save``. Writes, next
to this script:

* ``compressed_<case>.pt``  the reference's file, byte for byte.
* ``compressed_ref.npz``  per case and quantized layer: an input
  ``<case>.x.<layer>`` with the reference kernel's output
  ``<case>.y.<layer>`` for the layer as stored in the file (fp16 scales, zeros
  and channel scale widened to fp32, the fp32 bias added after the GEMM as in
  linear.py:99-100).
* ``compressed_ref.json``  per case: the quantization config, file size, the
  SHA-256 of the model's fp32 state_dict before quantization (``make_model``
  rebuilds it from the seed) and the reference's ``payload_nbytes``, ``matrix_nbytes`` and
  ``state_dict_nbytes`` (convert.py:339-374).
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
from torch import nn

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.abspath(os.path.join(HERE, "..", ".."))

# case -> (bits, symmetric, group_size, method, seed)
CASES: dict[str, tuple[int, bool, int | None, str, int]] = {
    "rtn_int4_g32": (4, True, 32, "rtn", 1),
    "rtn_int8_channel": (8, False, None, "rtn", 2),
    "rtn_int4_tensor": (4, False, 0, "rtn", 3),
    "awq_int4_g16": (4, False, 16, "awq", 4),
}


class Conv1D(nn.Module):
    """GPT-2's Conv1D layout: weight [in, out], y = x @ W + b."""

    def __init__(self, nf: int, nx: int) -> None:
        super().__init__()
        self.nf = nf
        self.weight = nn.Parameter(torch.empty(nx, nf))
        self.bias = nn.Parameter(torch.empty(nf))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return x @ self.weight + self.bias


class CompressedNet(nn.Module):
    """Quantized targets: attn (Conv1D), up (bias), down (no bias), odd (K = 63).
    Plain parameters (embedding, layer norm) and a buffer stay as they are."""

    def __init__(self) -> None:
        super().__init__()
        self.embed = nn.Embedding(32, 64)
        self.ln = nn.LayerNorm(64)
        self.attn = Conv1D(96, 64)
        self.up = nn.Linear(64, 128)
        self.down = nn.Linear(128, 64, bias=False)
        self.odd = nn.Linear(63, 40)
        self.register_buffer("position", torch.arange(16, dtype=torch.int64))

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        h = self.ln(self.embed(ids))
        a = self.attn(h)[..., :64]
        y = self.down(torch.relu(self.up(h + a)))
        return y + self.odd(h[..., :63]).sum(dim=-1, keepdim=True)


def make_model(seed: int) -> CompressedNet:
    model = CompressedNet()
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for _, p in sorted(model.named_parameters()):
            p.copy_(torch.randn(p.shape, generator=g) * 0.05)
        model.ln.weight.add_(1.0)
    return model


def state_digest(model: nn.Module) -> str:
    h = hashlib.sha256()
    for name, t in sorted(model.state_dict().items()):
        h.update(name.encode())
        h.update(t.detach().cpu().contiguous().numpy().tobytes())
    return h.hexdigest()


def calibration(seed: int) -> list[torch.Tensor]:
    g = torch.Generator().manual_seed(1000 + seed)
    return [torch.randint(0, 32, (4, 8), generator=g) for _ in range(3)]


def load_reference(ref_root: str):  # type: ignore[no-untyped-def]
    sys.path.insert(0, os.path.join(ref_root, "src"))
    sys.path.insert(0, REPO)
    import oracle

    kern = oracle.reference_kernels()
    if kern is None:
        raise SystemExit("build the reference kernel first: make -C oracle ref")
    sys.modules["ptqkit._kernels"] = kern
    return importlib.import_module("ptqkit")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("WQ_REFERENCE_ROOT"),
                    help="ptqkit source tree (default: $WQ_REFERENCE_ROOT)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set WQ_REFERENCE_ROOT to the ptqkit source tree")
    load_reference(args.reference)
    from ptqkit.convert import (
        matrix_nbytes,
        payload_nbytes,
        quantize_model,
        save_compressed,
        state_dict_nbytes,
    )
    from ptqkit.gemm import dequant_gemm
    from ptqkit.linear import QuantizedLinear
    from ptqkit.quant import Method, QuantConfig, QuantizedWeight

    arrays: dict[str, np.ndarray] = {}
    info: dict[str, dict[str, object]] = {}
    for case, (bits, sym, group, method, seed) in CASES.items():
        model = make_model(seed)
        digest = state_digest(model)
        config = QuantConfig(bits=bits, symmetric=sym, group_size=group, method=Method(method))
        batches = calibration(seed) if method != "rtn" else None
        quantize_model(model, config, batches)
        path = os.path.join(HERE, f"compressed_{case}.pt")
        size = save_compressed(model, path)
        state = torch.load(path, weights_only=True)
        g = torch.Generator().manual_seed(2000 + seed)
        for name, module in model.named_modules():
            if not isinstance(module, QuantizedLinear):
                continue
            t = state["tensors"]
            m = state["meta"][name]
            channel = t.get(f"{name}.channel_scale")
            qw = QuantizedWeight(
                codes=t[f"{name}.codes"],
                scales=t[f"{name}.scales"].float(),
                zeros=t[f"{name}.zeros"].float(),
                bits=m["bits"],
                group_size=m["group_size"],
                in_features=m["in_features"],
                out_features=m["out_features"],
                symmetric=m["symmetric"],
                packed=m["packed"],
                granularity=m["granularity"],
                channel_scale=None if channel is None else channel.float(),
            )
            x = torch.randn(5, m["in_features"], generator=g)
            y = dequant_gemm(x, qw, impl="kernel")
            if f"{name}.bias" in t:
                y = y + t[f"{name}.bias"]
            arrays[f"{case}.x.{name}"] = x.numpy()
            arrays[f"{case}.y.{name}"] = y.numpy()
        info[case] = {
            "bits": bits,
            "symmetric": sym,
            "group_size": group,
            "method": method,
            "seed": seed,
            "file_bytes": size,
            "state_sha256": digest,
            "payload_nbytes": payload_nbytes(state),
            "matrix_nbytes": matrix_nbytes(model),
            "state_dict_nbytes": state_dict_nbytes(model),
            "layers": sorted(state["meta"]),
        }
        print(case, size, "bytes")
    np.savez_compressed(os.path.join(HERE, "compressed_ref.npz"), **arrays)
    with open(os.path.join(HERE, "compressed_ref.json"), "w") as f:
        json.dump(info, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
