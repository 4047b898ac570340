"""Loads the golden fixtures written by tests/golden/make_golden.py."""
import os

import numpy as np
import torch

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = ["fastmka_mha_gelu", "fastmka_mha_l3_pad", "fastmka_mha_l3_single", "fastmka_mha_cache",
         "fastmka_mha_decode", "hf_qwen_rope", "hf_qwen_decode", "hf_llama_norope"]


def load(name: str) -> dict:
    """Returns {key: tensor or python scalar/str}; bf16-exact tensors come back as fp32."""
    z = np.load(os.path.join(GOLDEN_DIR, f"{name}.npz"))
    out = {}
    for k in z.files:
        a = z[k]
        if k.endswith("__bf16"):
            t = torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).to(torch.float32)
            out[k[: -len("__bf16")]] = t
        elif a.dtype.kind in "fc" and a.ndim > 0:
            out[k] = torch.from_numpy(a.copy())
        elif a.dtype.kind in "U":
            out[k] = str(a)
        else:
            out[k] = a.item() if a.ndim == 0 else torch.from_numpy(a.copy())
    if "weights_from" in out:
        src = load(out["weights_from"])
        out.update({k: v for k, v in src.items() if k.startswith("p.")})
    return out


def params(case: dict) -> dict:
    """The module state_dict stored under p.<name>."""
    return {k[2:]: v for k, v in case.items() if k.startswith("p.")}
