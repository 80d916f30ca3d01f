"""Checks of a full-size convolution that stay cheap on the host.

A benchmark-sized convolution (up to 10M rows x 1024 channels) is too large for the fp32 oracle
to recompute on the CPU and too large to copy to the host. Two checks cover it:

* :func:`oracle_rows` -- the fp32 oracle (the gather-matmul fallback of
  ``src/mlx_diffuser/kernels/sparse.py:39-55``) on a sample of output rows. Only the sampled
  rows' neighbour features leave the device (gathered there), so the oracle's cost does not
  grow with the scene.
* :func:`projection_error` -- every output row, projected on random vectors. The convolution is
  linear, so for a vector v over the output channels

      out[p] . v = bias . v + sum_k f[nbr[p, k]] . (W[k] v)

  The right side needs one pass over the features (f @ (W[k] v) for all k at once, one value
  per source row and offset) and a gather of those values through the map; both sides are
  evaluated in float64 on the device. The error is reported as max_p |lhs - rhs| / max_p |rhs|,
  the tests' max-relative-error measure, for every row of the scene: a single wrong row shows
  up at the size of the outputs themselves, while half-precision output rounding stays near
  1e-3.
"""

from __future__ import annotations

import numpy as np
import torch

ROW_CHUNK = 1 << 18


def device_features(n: int, channels: int, seed: int, dtype, device) -> torch.Tensor:
    """N(0, 1) features generated on the device (a 10M x 1024 scene never exists on the host)."""

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.randn((n, channels), generator=g, device=device, dtype=dtype)


def oracle_rows(feats: torch.Tensor, nbr: torch.Tensor, rows: np.ndarray, w_kio: np.ndarray,
                bias: np.ndarray | None) -> np.ndarray:
    """fp32 oracle of the convolution for output rows ``rows``: features and map stay on the
    device, only the gathered neighbour rows ([len(rows), K, Cin]) come to the host."""

    idx = nbr[torch.from_numpy(np.asarray(rows, np.int64)).to(nbr.device)].long()  # [R, K]
    gathered = feats[idx.clamp(min=0)].float().cpu().numpy()  # [R, K, Cin]
    valid = (idx >= 0).cpu().numpy()
    out = np.zeros((len(rows), w_kio.shape[2]), np.float32)
    if bias is not None:
        out += np.asarray(bias, np.float32)
    for k in range(w_kio.shape[0]):
        ok = valid[:, k]
        if ok.any():
            out[ok] += gathered[ok, k] @ w_kio[k]
    return out


def projection_error(out: torch.Tensor, feats: torch.Tensor, nbr: torch.Tensor,
                     w_kio: torch.Tensor, bias: torch.Tensor | None, seed: int = 0,
                     vectors: int = 2) -> float:
    """max_p |out[p] . v - ref[p] . v| / max_p |ref[p] . v| over every row p and ``vectors``
    random N(0, 1) vectors v (see the module docstring); float64 on the device."""

    dev = out.device
    n, kvol = nbr.shape
    cout = out.shape[1]
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    v = torch.randn((cout, vectors), generator=g, device=dev, dtype=torch.float64)
    w = w_kio.to(device=dev, dtype=torch.float64)  # [K, Cin, Cout]
    u = (w @ v).permute(1, 0, 2).reshape(w.shape[1], kvol * vectors)  # [Cin, K*J]
    lhs = torch.empty((n, vectors), dtype=torch.float64, device=dev)
    s = torch.empty((n, kvol * vectors), dtype=torch.float64, device=dev)
    for a in range(0, n, ROW_CHUNK):
        lhs[a : a + ROW_CHUNK] = out[a : a + ROW_CHUNK].double() @ v
        s[a : a + ROW_CHUNK] = feats[a : a + ROW_CHUNK].double() @ u
    rhs = torch.zeros((n, vectors), dtype=torch.float64, device=dev)
    if bias is not None:
        rhs += bias.to(dev, torch.float64) @ v
    nb = nbr.long()
    for k in range(kvol):
        src = nb[:, k]
        ok = src >= 0
        rhs[ok] += s[src[ok], k * vectors : (k + 1) * vectors]
    return float((lhs - rhs).abs().max() / rhs.abs().max().clamp(min=1e-300))
