"""Shared helpers of the test-suite (inputs, tolerances, comparisons)."""
import os

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden", "kat.pt")

# float32 parity bar of the hot path (rel-L2 against the reference build)
REL_L2_F32 = 1e-5


def load_golden():
    return torch.load(GOLDEN, weights_only=False)


def rel_l2(a, b) -> float:
    a = torch.as_tensor(a).double().cpu()
    b = torch.as_tensor(b).double().cpu()
    den = b.norm().item()
    num = (a - b).norm().item()
    return num / den if den > 0 else num


def cuda(t, dtype=None):
    t = t.cuda()
    return t if dtype is None else t.to(dtype)
