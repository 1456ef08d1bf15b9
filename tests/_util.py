"""Shared helpers for the parity tests."""
import glob
import os

import numpy as np
import torch

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


def golden_cases(kind):
    out = []
    for f in sorted(glob.glob(os.path.join(GOLDEN_DIR, "*.npz"))):
        z = np.load(f)
        if str(z["kind"]) == kind:
            out.append(f)
    return out


def load_golden(path):
    """Return (dict of float32 torch tensors, input dtype, scalars)."""
    z = np.load(path)
    dt = DTYPES[str(z["dtype"])]
    t = {k: torch.from_numpy(np.array(z[k])) for k in z.files
         if z[k].dtype == np.float32 and z[k].ndim > 0}
    sc = {k: z[k].item() for k in z.files if z[k].ndim == 0}
    return t, dt, sc


def rel_err(a, b):
    """Normwise relative error max|a-b| / max|b| (fp64 on CPU)."""
    a = a.detach().to(torch.float64).cpu()
    b = b.detach().to(torch.float64).cpu()
    den = b.abs().max().item()
    if den == 0.0:
        return a.abs().max().item()
    return (a - b).abs().max().item() / den


def abs_err(a, b):
    a = a.detach().to(torch.float64).cpu()
    b = b.detach().to(torch.float64).cpu()
    return (a - b).abs().max().item()


# Tolerances (normwise relative unless stated) -- the bar the kernels must meet
TOL_FP32 = 1e-5          # fp32 outputs
TOL_BF16 = 2e-2          # bf16 / fp16 stored outputs, fp32 accumulation
TOL_SINKHORN_ABS = 1e-4  # Sinkhorn matrices, absolute
