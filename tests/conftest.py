import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name: str) -> dict:
    """Golden fixture -> dict of torch tensors (fp16 arrays widened to fp32) plus 'W' (weights)."""
    z = np.load(GOLDEN / f"{name}.npz")
    out, W = {}, {}
    for k in z.files:
        a = z[k]
        t = torch.from_numpy(a.astype(np.float32) if a.dtype == np.float16 else a)
        if k.startswith("w."):
            W[k[2:]] = t
        else:
            out[k] = t
    H, heads, FM, L, T, V, R, rank, B = (int(x) for x in out["cfg"])
    out.update(W=W, H=H, heads=heads, FM=FM, L=L, T=T, V=V, R=R, rank=rank, B=B)
    return out


def golden_flow_config(g):
    from oracle import FlowConfig
    return FlowConfig(hidden=g["H"], num_heads=g["heads"], ffn_multiplier=g["FM"],
                      num_layers=g["L"], num_flow_steps=g["T"], markov_rank=g["rank"])


@pytest.fixture(params=["g64", "g128"])
def golden(request):
    return load_golden(request.param)


def has_gpu() -> bool:
    return torch.cuda.is_available()
