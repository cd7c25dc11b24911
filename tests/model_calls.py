"""Loading of the recorded model calls (tests/golden/model_calls/*.npz, made by
tests/golden/make_model_calls.py from the reference model)."""
import glob
import json
import os

import numpy as np
import torch

DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "model_calls")
FILES = sorted(glob.glob(os.path.join(DIR, "*.npz")))
IDS = [os.path.basename(f)[:-4] for f in FILES]


def load(path):
    d = np.load(path)
    meta = json.loads(bytes(d["meta"]).decode())
    return d, meta


def array(d, key, dtype=None, device="cpu"):
    """A stored array as a tensor: b* keys hold bf16 bit patterns, f* fp32."""
    a = d[key]
    t = torch.from_numpy(np.array(a)).view(torch.bfloat16) if key.startswith("b") else torch.from_numpy(np.array(a))
    t = t.to(device)
    return t.to(dtype) if dtype is not None else t


def rebuild(spec, leaves):
    if "t" in spec:
        return leaves[spec["t"]]
    if "l" in spec:
        return [rebuild(e, leaves) for e in spec["l"]]
    return spec["v"]


def call_args(d, call, device="cpu"):
    """(leaf tensors, args, kwargs) of one recorded call, leaves requiring
    grad as recorded."""
    leaves = []
    for lf in call["leaves"]:
        t = array(d, lf["a"], getattr(torch, lf["dtype"]), device)
        leaves.append(t.requires_grad_(lf["requires_grad"]))
    args = rebuild(call["args"], leaves)
    kwargs = {k: rebuild(v, leaves) for k, v in call["kwargs"].items()}
    return leaves, args, kwargs
