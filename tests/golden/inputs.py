"""Regenerate a reference problem's inputs from a recorded spec.

make_golden.py runs each reference ``get_inputs()`` with torch.randn /
torch.randint replaced by seeded CPU generators and records, per returned
input, how to rebuild it: the base tensor (kind, numel/shape, dtype, range,
seed) and the view applied to it (shape, stride, storage offset).  This file
replays those specs anywhere (no reference checkout needed), on any device.
"""
from __future__ import annotations

import torch

# bound at import, so replaying specs works while torch.randn is patched
_randn = torch.randn
_randint = torch.randint

DTYPES = {
    "bfloat16": torch.bfloat16,
    "float32": torch.float32,
    "complex64": torch.complex64,
    "int64": torch.int64,
    "int32": torch.int32,
}


def base_tensor(spec: dict) -> torch.Tensor:
    """The seeded base tensor of one input, on the CPU."""
    g = torch.Generator().manual_seed(int(spec["seed"]))
    dt = DTYPES[spec["dtype"]]
    size = tuple(spec["size"])
    if spec["kind"] == "randn":
        if dt == torch.complex64:
            return _randn(size, dtype=torch.complex64, generator=g)
        return _randn(size, dtype=torch.float32, generator=g).to(dt)
    if spec["kind"] == "randint":
        return _randint(int(spec["low"]), int(spec["high"]), size, dtype=dt, generator=g)
    raise ValueError(f"unknown input kind {spec['kind']}")


def make_input(spec: dict, device="cpu") -> torch.Tensor:
    base = base_tensor(spec).to(device)
    v = spec.get("view")
    if v is None:
        return base
    return base.as_strided(tuple(v["shape"]), tuple(v["stride"]), int(v["offset"]))


# Inputs rebuilt for problems whose own get_inputs() does not match their
# graph (see make_golden.py's INPUT_FIXUPS):
#   "fused_rms_norm": the (y, rstd) pair that
#     aten._fused_rms_norm(inputs[x], [N], inputs[w], eps) returns on the CPU;
#   "tuple_slot": a tuple of `len` entries whose entry `slot` is the tensor
#     described by `item` (a seeded spec like any other input), the rest None.
DERIVED = ("fused_rms_norm", "tuple_slot")


def make_inputs(specs: list[dict], device="cpu") -> list:
    out = [None if s["kind"] in DERIVED else make_input(s, device) for s in specs]
    for i, s in enumerate(specs):
        if s["kind"] == "tuple_slot":
            item = make_input(s["item"], device)
            out[i] = tuple(item if j == s["slot"] else None for j in range(s["len"]))
        if s["kind"] == "fused_rms_norm":
            x, w = out[s["x"]].cpu(), out[s["w"]].cpu()
            y, rstd = torch.ops.aten._fused_rms_norm.default(x, [w.numel()], w, float(s["eps"]))
            out[i] = (y.to(device), rstd.to(device))
    return out
