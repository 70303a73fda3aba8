"""Helpers shared by the GPU tests: NumPy <-> CUDA tensors in the oracle's
storage convention (16-bit types as raw uint16 bits)."""
import numpy as np
import torch

import oracle as O

TORCH_OF = {O.F32: torch.float32, O.F16: torch.float16, O.BF16: torch.bfloat16}


def dev(a: np.ndarray, t: int = O.F32) -> torch.Tensor:
    """Upload an oracle-storage array (f32, or uint16 bits of f16/bf16)."""
    a = np.ascontiguousarray(a)
    if t == O.F32:
        return torch.from_numpy(a.astype(np.float32, copy=False)).cuda()
    return torch.from_numpy(a.view(np.int16)).cuda().view(TORCH_OF[t])


def host(x: torch.Tensor) -> np.ndarray:
    """Download to the oracle's storage convention."""
    x = x.detach().contiguous()
    if x.dtype == torch.float32:
        return x.cpu().numpy()
    if x.dtype in (torch.float16, torch.bfloat16):
        return x.view(torch.int16).cpu().numpy().view(np.uint16)
    return x.cpu().numpy()


def host_f32(x: torch.Tensor) -> np.ndarray:
    return x.detach().float().cpu().numpy()


def normal_with_outliers(rng, shape, frac=0.01, mag=20.0):
    """N(0,1) with `frac` of the elements set to +-mag (random sign)."""
    x = rng.standard_normal(shape).astype(np.float32)
    n = x.size
    k = int(n * frac)
    if k:
        idx = rng.choice(n, size=k, replace=False)
        x.reshape(-1)[idx] = np.where(rng.random(k) < 0.5, -mag, mag).astype(np.float32)
    return x
