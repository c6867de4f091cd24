"""Low-rank delta compression (the reference's negative result, core/model/src/lowrank.rs:54-230).

Per 2-D tensor: randomized range finder with a Gaussian test matrix drawn from splitmix64 + Box-Muller
(same seeds as the reference: m * 0x9e3779b97f4a7c15 + n + r), one pass, modified Gram-Schmidt in
float64, D ~= Q (Q^T D); the residual goes to the error buffer. 1-D tensors pass through exactly.
Runs where the delta lives: CUDA tensors are compressed on the GPU (the test matrix comes from the
native runtime - the draws form one sequential chain, each state being the previous output - and is
copied over; the products and the Gram-Schmidt run on the device in float64), and only the factors cross
to the host for the JSON payload.
JSON shape: {"tensors": {name: {u, v, m, n, rank}}, "rank": r}.
"""
from __future__ import annotations

import math
from typing import Dict, List, Tuple

import torch

_M64 = (1 << 64) - 1


def _splitmix64(s: int) -> int:
    s = (s + 0x9e3779b97f4a7c15) & _M64
    z = s
    z = ((z ^ (z >> 30)) * 0xbf58476d1ce4e5b9) & _M64
    z = ((z ^ (z >> 27)) * 0x94d049bb133111eb) & _M64
    return z ^ (z >> 31)


def _omega_loop(m: int, n: int, r: int) -> torch.Tensor:
    """The test matrix draw by draw (the reference's loop, lowrank.rs:54-80); kept as the oracle."""
    rng = ((m * 0x9e3779b97f4a7c15) & _M64)
    rng = (rng + n + r) & _M64
    vals = []
    for _ in range(n * r):
        rng = _splitmix64(rng)
        u1 = (rng & 0xFFFFFFFF) / 4294967296.0 + 1e-10
        rng = _splitmix64(rng)
        u2 = (rng & 0xFFFFFFFF) / 4294967296.0
        vals.append(math.sqrt(-2.0 * math.log(u1)) * math.cos(2.0 * math.pi * u2))
    return torch.tensor(vals, dtype=torch.float64).view(n, r)


def _omega(m: int, n: int, r: int, device="cpu") -> torch.Tensor:
    """The test matrix from the native runtime (the same draws as ``_omega_loop``), on ``device``."""
    from ..utils import native
    out = torch.empty(n, r, dtype=torch.float64)
    native.rt().dtr_lowrank_omega(m, n, r, out.data_ptr())
    return out.to(device)


def truncated_svd(mat: torch.Tensor, m: int, n: int, r: int) -> Tuple[torch.Tensor, torch.Tensor]:
    D = mat.reshape(m, n).double()
    Y = D @ _omega(m, n, r, D.device)
    for j in range(r):  # modified Gram-Schmidt, as the reference
        Y[:, j] /= Y[:, j].norm().clamp_min(1e-15)
        if j + 1 < r:
            dots = Y[:, j] @ Y[:, j + 1:]
            Y[:, j + 1:] -= Y[:, j:j + 1] * dots[None, :]
    B = Y.t() @ D
    return Y.float(), B.t().contiguous().float()


def compress_lowrank(delta: Dict[str, torch.Tensor], shapes: Dict[str, List[int]], rank: int,
                     error_buffer: Dict[str, torch.Tensor]):
    tensors, orig, comp, err_sq, norm_sq = {}, 0, 0, 0.0, 0.0
    for name, v in delta.items():
        v = v.reshape(-1).float()
        shape = shapes.get(name, [v.numel()])
        orig += v.numel() * 4
        eff = v + error_buffer[name] if name in error_buffer else v
        if len(shape) == 2 and shape[0] > 1 and shape[1] > 1:
            m, n = shape
            r = min(rank, m, n)
            u, vv = truncated_svd(eff, m, n, r)
            rec = (u.double() @ vv.double().t()).float().reshape(-1)
            res = eff - rec
            err_sq += float((res.double() ** 2).sum())
            norm_sq += float((eff.double() ** 2).sum())
            error_buffer[name] = res
            comp += (m * r + n * r) * 4
            tensors[name] = {"u": u.reshape(-1).tolist(), "v": vv.reshape(-1).tolist(), "m": m, "n": n, "rank": r}
        else:
            comp += eff.numel() * 4
            tensors[name] = {"u": eff.tolist(), "v": [], "m": eff.numel(), "n": 0, "rank": 0}
            error_buffer.pop(name, None)
    stats = {"rank": rank, "original_bytes": orig, "compressed_bytes": comp,
             "compression_ratio": orig / comp if comp else 1.0,
             "reconstruction_error": math.sqrt(err_sq / norm_sq) if norm_sq > 0 else 0.0}
    return {"tensors": tensors, "rank": rank}, stats


def decompress_lowrank(lr: dict) -> Dict[str, torch.Tensor]:
    out = {}
    for name, f in lr["tensors"].items():
        if f["rank"] == 0 or f["n"] == 0:
            out[name] = torch.tensor(f["u"], dtype=torch.float32)
        else:
            u = torch.tensor(f["u"], dtype=torch.float64).view(f["m"], f["rank"])
            v = torch.tensor(f["v"], dtype=torch.float64).view(f["n"], f["rank"])
            out[name] = (u @ v.t()).float().reshape(-1)
    return out
