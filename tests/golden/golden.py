"""Reader for the golden fixtures written by ``make_golden.py``."""
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load(name):
    """Return {key: torch.Tensor} with bf16 / fp16-packed entries restored exactly."""
    out = {}
    with np.load(os.path.join(HERE, name + ".npz")) as z:
        for k in z.files:
            a = z[k]
            if k.endswith("@bf16"):
                out[k[:-5]] = torch.from_numpy(a.copy()).view(torch.bfloat16)
            elif k.endswith("@f16"):
                out[k[:-4]] = torch.from_numpy(a.copy()).float()
            else:
                out[k] = torch.from_numpy(a.copy())
    return out


def state_dict(g, prefix):
    """Collect ``<prefix>sd.<name>`` entries into a state_dict."""
    p = prefix + "sd."
    return {k[len(p):]: v for k, v in g.items() if k.startswith(p)}
