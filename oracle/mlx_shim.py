"""Test infrastructure only: a NumPy stand-in for the parts of ``mlx.core`` / ``mlx.nn``
that mlx_diffuser's sparse-voxel path touches.

MLX has no Linux wheel in this environment, so the reference's own Python for the hot path
(``src/mlx_diffuser/layers/sparse.py`` and ``src/mlx_diffuser/kernels/sparse.py``) is executed
unmodified on top of this shim to produce golden vectors (``tests/golden/make_golden.py``).
Nothing in the product package imports this module.

Covered surface (each item is what those two reference files call):

* ``mx.array`` -- an ``ndarray`` subclass; ``x.at[idx].add(v)`` returns a copy with
  ``np.add.at`` applied (MLX scatter-add semantics: duplicates accumulate);
* dtypes ``int32 / float32 / float16 / bfloat16`` (bfloat16 is carried as float32: NumPy
  has no bfloat16, and every golden vector is generated in float32);
* ``zeros / ones / full / max / maximum / broadcast_to / array_equal / allclose``;
* ``random.uniform / random.normal / random.seed``;
* ``fast.metal_kernel`` -- returns a callable that raises, so only the reference's pure
  fallback (``use_metal=False``) can run;
* ``fast.scaled_dot_product_attention`` -- a float64 softmax attention, for the reference's
  ``sparse_self_attention`` / ``sparse_cross_attention``;
* ``arange / split / mean / square / rsqrt``;
* ``nn.Linear``, ``nn.SiLU`` and ``nn.silu``, for the residual block around the convolutions;
* ``nn.Module`` with ``training`` / ``eval()`` / ``train()``.
"""

from __future__ import annotations

import sys
import types

import numpy as np


class array(np.ndarray):  # noqa: N801 - mirrors ``mx.array``
    """ndarray subclass constructed like ``mx.array(data, dtype=...)``."""

    def __new__(cls, data, dtype=None):
        return np.asarray(data, dtype=dtype).view(cls)

    @property
    def at(self):
        return _At(self)

    def item(self):  # noqa: D401 - numpy-compatible
        return np.ndarray.item(self)


class _At:
    def __init__(self, base: np.ndarray):
        self._base = base

    def __getitem__(self, index):
        return _AtIndex(self._base, index)


class _AtIndex:
    def __init__(self, base: np.ndarray, index):
        self._base = base
        self._index = index

    def add(self, values):
        out = np.array(self._base, copy=True)
        index = self._index
        if isinstance(index, tuple):
            index = tuple(np.asarray(i) for i in index)
        else:
            index = np.asarray(index)
        np.add.at(out, index, np.asarray(values, dtype=out.dtype))
        return out.view(array)


Dtype = np.dtype
int32 = np.dtype(np.int32)
int64 = np.dtype(np.int64)
float32 = np.dtype(np.float32)
float16 = np.dtype(np.float16)
bfloat16 = np.dtype(np.float32)
bool_ = np.dtype(np.bool_)


def _wrap(x):
    return np.asarray(x).view(array)


def zeros(shape, dtype=float32):
    return _wrap(np.zeros(shape, dtype=dtype))


def ones(shape, dtype=float32):
    return _wrap(np.ones(shape, dtype=dtype))


def full(shape, value, dtype=float32):
    return _wrap(np.full(shape, value, dtype=dtype))


def zeros_like(x):
    return _wrap(np.zeros_like(np.asarray(x)))


def ones_like(x):
    return _wrap(np.ones_like(np.asarray(x)))


def max(x, axis=None, keepdims=False):  # noqa: A001 - mirrors ``mx.max``
    return _wrap(np.max(np.asarray(x), axis=axis, keepdims=keepdims))


def maximum(a, b):
    return _wrap(np.maximum(np.asarray(a), np.asarray(b)))


def broadcast_to(x, shape):
    return _wrap(np.broadcast_to(np.asarray(x), shape))


def array_equal(a, b):
    return bool(np.array_equal(np.asarray(a), np.asarray(b)))


def allclose(a, b, rtol=1e-5, atol=1e-8):
    return bool(np.allclose(np.asarray(a), np.asarray(b), rtol=rtol, atol=atol))


def split(a, sections, axis=0):
    return [_wrap(p) for p in np.split(np.asarray(a), sections, axis=axis)]


def mean(a, axis=None, keepdims=False):
    return _wrap(np.mean(np.asarray(a), axis=axis, keepdims=keepdims))


def square(a):
    return _wrap(np.square(np.asarray(a)))


def rsqrt(a):
    a = np.asarray(a)
    return _wrap((1.0 / np.sqrt(a)).astype(a.dtype))


def arange(start, stop=None, step=1, dtype=None):
    return _wrap(np.arange(start, stop, step, dtype=dtype))


def eval(*_args):  # noqa: A001 - mirrors ``mx.eval``
    return None


class _Random(types.ModuleType):
    def __init__(self):
        super().__init__("mlx.core.random")
        self._rng = np.random.default_rng(0)

    def seed(self, value: int) -> None:
        self._rng = np.random.default_rng(value)

    def uniform(self, low=0.0, high=1.0, shape=(), dtype=float32):
        return _wrap(self._rng.uniform(low, high, size=shape).astype(dtype))

    def normal(self, shape=(), dtype=float32):
        return _wrap(self._rng.standard_normal(size=shape).astype(dtype))


random = _Random()


class _Fast(types.ModuleType):
    def __init__(self):
        super().__init__("mlx.core.fast")

    @staticmethod
    def metal_kernel(**_kwargs):
        def _unavailable(*_a, **_k):
            raise RuntimeError("Metal kernels cannot run under the NumPy shim")

        return _unavailable

    @staticmethod
    def scaled_dot_product_attention(q, k, v, *, scale, mask=None):
        """softmax(q k^T * scale) v over the last two axes of (B, heads, L, D) arrays, in
        float64 and returned in q's dtype."""

        if mask is not None:
            raise NotImplementedError("masks are not used by the sparse path")
        q64, k64, v64 = (np.asarray(t, np.float64) for t in (q, k, v))
        s = np.einsum("bhld,bhmd->bhlm", q64, k64) * scale
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=-1, keepdims=True)
        return _wrap(np.einsum("bhlm,bhmd->bhld", p, v64).astype(np.asarray(q).dtype))


fast = _Fast()


def _silu(x):
    x = np.asarray(x)
    return _wrap((x / (1.0 + np.exp(-x))).astype(x.dtype))


class Module:
    """Minimal ``mlx.nn.Module``: attribute container with a training flag."""

    def __init__(self):
        self.training = True

    def eval(self):
        self.training = False
        return self

    def train(self, mode: bool = True):
        self.training = mode
        return self


class SiLU(Module):
    def __call__(self, x):
        return _silu(x)


class Linear(Module):
    """``mlx.nn.Linear``: weight (out, in) uniform in ±1/sqrt(in), bias zeros."""

    def __init__(self, input_dims: int, output_dims: int, bias: bool = True):
        super().__init__()
        bound = 1.0 / np.sqrt(input_dims)
        self.weight = random.uniform(-bound, bound, (output_dims, input_dims))
        if bias:
            self.bias = zeros((output_dims,))

    def __call__(self, x):
        y = np.asarray(x) @ np.asarray(self.weight).T
        if hasattr(self, "bias"):
            y = y + np.asarray(self.bias)
        return _wrap(y)


def install() -> None:
    """Register this shim as ``mlx`` / ``mlx.core`` / ``mlx.nn`` in ``sys.modules``."""

    core = sys.modules[__name__]
    nn = types.ModuleType("mlx.nn")
    nn.Module = Module
    nn.Linear = Linear
    nn.SiLU = SiLU
    nn.silu = _silu
    pkg = types.ModuleType("mlx")
    pkg.__path__ = []
    pkg.core = core
    pkg.nn = nn
    sys.modules["mlx"] = pkg
    sys.modules["mlx.core"] = core
    sys.modules["mlx.core.random"] = random
    sys.modules["mlx.core.fast"] = fast
    sys.modules["mlx.nn"] = nn
