"""Shared loaders for the golden fixtures (tests/golden/*.npz + manifest.json)."""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np
import torch

from oracle.synth import make_inputs
from fftsparse_b200.params import derive_mask_params

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
DT = {"fp32": torch.float32, "bf16": torch.bfloat16}


def manifest():
    with open(os.path.join(GOLDEN, "manifest.json")) as f:
        return json.load(f)


def sha(t: torch.Tensor) -> str:
    t = t.contiguous()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def load_case(name: str):
    """(spec, q, k, v, params, fixture arrays) for one golden case."""
    spec = manifest()[name]
    q, k, v = make_inputs(spec["L"], dtype=DT[spec["dtype"]], batch=spec["batch"],
                          num_q_heads=spec.get("hq", 32), num_kv_heads=spec.get("hkv", 8),
                          rope_base=spec.get("rope_base", 500000.0))
    kw = dict(spec["kwargs"], block_size=spec["block_size"])
    params = derive_mask_params(spec["L"], **kw)
    fx = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    return spec, q, k, v, params, {key: fx[key] for key in fx.files}


def is_large(spec) -> bool:
    """The BASELINE config 3 / 5 shaped cases (131072 tokens per case): their
    inputs take tens of seconds to generate on the CPU, so each test module
    loads them once."""
    return spec["L"] * spec["batch"] >= 131072


def case_names(large=None):
    """Golden case names; ``large`` True / False selects the large / small ones."""
    m = manifest()
    return sorted(n for n in m if large is None or is_large(m[n]) == large)
