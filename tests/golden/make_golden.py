"""Generate the golden fixtures by running the reference's own sparse-voxel code.

Run from the repository root, with the mlx_diffuser sources available:

    python tests/golden/make_golden.py [--reference /path/to/mlx_diffuser]

MLX cannot be installed here, so the reference files ``src/mlx_diffuser/kernels/sparse.py``
and ``src/mlx_diffuser/layers/sparse.py`` are executed unmodified on top of the NumPy stand-in
``oracle/mlx_shim.py``: ``build_neighbor_map``, ``SparseConv3D`` (its pure fallback,
``use_metal=False``), ``sparse_downsample``, ``sparse_upsample``, ``sparse_subdivide``,
``_attention_groups``, ``sparse_self_attention`` and ``sparse_cross_attention``; the
residual block ``_SparseResBlock3D`` (``src/mlx_diffuser/models/trellis_slat.py:43-92``) with
``LayerNorm32`` and ``SparseLinear`` is compiled from its files by ``ast``, as written. The
occupancy step ``TrellisSparseStructureDecoder.occupied_coordinates``
(``src/mlx_diffuser/models/trellis.py:278-285``) is taken out of its file by ``ast`` and run as
written, with a stand-in ``self`` whose call returns the logits. Outputs are written to
``tests/golden/*.npz``. The fixtures travel with the repository; the reference does not.
"""

from __future__ import annotations

import __future__
import argparse
import ast
import importlib.util
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from mlx_diffuser_b200 import scenes  # noqa: E402
from oracle import mlx_shim  # noqa: E402


def load_reference(reference_root: str):
    """Import the reference's two hot-path modules under the shim; returns (kernels, layers)."""

    mlx_shim.install()
    src = os.path.join(reference_root, "src", "mlx_diffuser")
    for name, path in (
        ("mlx_diffuser", src),
        ("mlx_diffuser.kernels", os.path.join(src, "kernels")),
        ("mlx_diffuser.layers", os.path.join(src, "layers")),
    ):
        pkg = types.ModuleType(name)
        pkg.__path__ = [path]
        sys.modules[name] = pkg

    def load(name: str, path: str):
        spec = importlib.util.spec_from_file_location(name, path)
        module = importlib.util.module_from_spec(spec)
        sys.modules[name] = module
        spec.loader.exec_module(module)
        return module

    kernels_sparse = load("mlx_diffuser.kernels.sparse", os.path.join(src, "kernels", "sparse.py"))
    sys.modules["mlx_diffuser.kernels"].sparse_conv3d = kernels_sparse.sparse_conv3d
    layers_sparse = load("mlx_diffuser.layers.sparse", os.path.join(src, "layers", "sparse.py"))
    return kernels_sparse, layers_sparse


def run_case(ref, coords, features, weight, bias, *, kernel_size=3, dilation=1, factors=(2,),
             spatial_shape=None, extra_maps=()):
    """Run the reference path on one input and collect every output as numpy arrays."""

    _, L = ref
    mx = sys.modules["mlx.core"]
    out: dict[str, np.ndarray] = {
        "coords": coords.astype(np.int32),
        "features": features.astype(np.float32),
        "weight": weight.astype(np.float32),
        "bias": bias.astype(np.float32),
        "kernel_size": np.int32(kernel_size),
        "dilation": np.int32(dilation),
    }
    tensor = L.SparseTensor(mx.array(features), mx.array(coords), spatial_shape=spatial_shape)
    out["batch_size"] = np.int32(tensor.batch_size)
    out["spatial_shape"] = np.asarray(tensor.spatial_shape, np.int32)
    out["nbr"] = np.asarray(L.build_neighbor_map(tensor.coords, kernel_size, dilation), np.int32)
    for i, (ks, dl) in enumerate(extra_maps):
        out[f"nbr_extra{i}"] = np.asarray(L.build_neighbor_map(tensor.coords, ks, dl), np.int32)
        out[f"nbr_extra{i}_kernel"] = np.asarray(ks if not isinstance(ks, int) else (ks,) * 3)
        out[f"nbr_extra{i}_dilation"] = np.asarray(dl if not isinstance(dl, int) else (dl,) * 3)
    conv = L.SparseConv3D(weight.shape[-1], weight.shape[0], kernel_size, dilation=dilation,
                          use_metal=False)
    conv.conv.weight = mx.array(weight)
    conv.conv.bias = mx.array(bias)
    out["conv_out"] = np.asarray(conv(tensor).features, np.float32)
    for f in factors:
        down = L.sparse_downsample(tensor, f)
        up = L.sparse_upsample(down, f)
        out[f"down{f}_coords"] = np.asarray(down.coords, np.int32)
        out[f"down{f}_inverse"] = np.asarray(
            down.cache[f"upsample_{f}_{down.scale}"][1], np.int32
        ).reshape(-1)
        out[f"down{f}_features"] = np.asarray(down.features, np.float32)
        out[f"down{f}_spatial_shape"] = np.asarray(down.spatial_shape, np.int32)
        out[f"down{f}_scale"] = np.asarray(down.scale, np.int32)
        out[f"up{f}_features"] = np.asarray(up.features, np.float32)
    return out


def cases(ref):
    rng = np.random.default_rng(1234)
    yield "ref_test_four_points", run_case(
        ref,
        np.array([[0, 0, 0, 0], [0, 0, 0, 1], [0, 0, 1, 0], [0, 1, 0, 0]], np.int32),
        np.arange(12, dtype=np.float32).reshape(4, 3),
        rng.uniform(-0.3, 0.3, (2, 3, 3, 3, 3)).astype(np.float32),
        np.array([0.5, -0.25], np.float32),
    )
    block = np.array([[0, z, y, x] for z in range(2) for y in range(2) for x in range(2)], np.int32)
    yield "ref_test_block2", run_case(
        ref,
        block,
        np.arange(16, dtype=np.float32).reshape(8, 2),
        rng.uniform(-0.3, 0.3, (2, 3, 3, 3, 2)).astype(np.float32),
        np.zeros(2, np.float32),
        spatial_shape=(2, 2, 2),
    )
    # duplicates, negative coordinates, three batch elements, odd factors
    c = rng.integers(-6, 6, size=(400, 4)).astype(np.int32)
    c[:, 0] = rng.integers(0, 3, size=400)
    c = np.concatenate([c, c[rng.integers(0, 400, 40)]], axis=0)  # 40 duplicate rows
    yield "duplicates_negative", run_case(
        ref,
        c,
        rng.standard_normal((len(c), 5)).astype(np.float32),
        rng.standard_normal((7, 3, 3, 3, 5)).astype(np.float32) * 0.1,
        rng.standard_normal(7).astype(np.float32),
        factors=(2, 3),
        extra_maps=(((3, 1, 5), (2, 1, 1)), (1, 1), (5, 2)),
    )
    s = scenes.shell(16, 5.5, 2.0, 1.0, seed=7)
    s = scenes.batched([s, scenes.shell(16, 6.0, 2.0, 1.0, seed=8)])
    yield "shell16_pair", run_case(
        ref,
        s,
        scenes.normal_features(len(s), 16, seed=11),
        scenes.conv_weight(24, 16, 3, seed=12),
        rng.standard_normal(24).astype(np.float32) * 0.1,
    )
    s = scenes.shell(20, 7.0, 2.5, 1.0, seed=21)
    yield "shell20_kernel5", run_case(
        ref,
        s,
        scenes.normal_features(len(s), 8, seed=22),
        scenes.conv_weight(8, 8, 5, seed=23),
        np.zeros(8, np.float32),
        kernel_size=5,
        dilation=1,
    )
    s = scenes.shell(24, 8.0, 2.5, 1.0, seed=31)
    yield "shell24_dilation2", run_case(
        ref,
        s,
        scenes.normal_features(len(s), 64, seed=32),
        scenes.conv_weight(64, 64, 3, seed=33),
        rng.standard_normal(64).astype(np.float32) * 0.1,
        dilation=2,
    )
    s = scenes.shell32(seed=41)
    yield "shell32_c64", run_case(
        ref,
        s,
        scenes.normal_features(len(s), 64, seed=42),
        scenes.conv_weight(64, 64, 3, seed=43),
        np.zeros(64, np.float32),
    )


def load_occupied_coordinates(reference_root: str):
    """The reference's ``occupied_coordinates`` method, compiled alone from its source file."""

    path = os.path.join(reference_root, "src", "mlx_diffuser", "models", "trellis.py")
    with open(path) as f:
        tree = ast.parse(f.read(), path)
    for node in tree.body:
        if isinstance(node, ast.ClassDef) and node.name == "TrellisSparseStructureDecoder":
            for item in node.body:
                if isinstance(item, ast.FunctionDef) and item.name == "occupied_coordinates":
                    module = ast.Module(body=[item], type_ignores=[])
                    code = compile(module, path, "exec",
                                   flags=__future__.annotations.compiler_flag, dont_inherit=True)
                    namespace = {"mx": sys.modules["mlx.core"], "np": np}
                    exec(code, namespace)
                    return namespace["occupied_coordinates"]
    raise RuntimeError("occupied_coordinates not found in the reference")


class _LogitsModel:
    """Stand-in ``self`` for ``occupied_coordinates``: calling it returns the logits with a
    trailing channel axis, like the decoder's (B, D, H, W, 1) output."""

    def __init__(self, logits):
        self.logits = logits

    def __call__(self, _latent):
        return self.logits[..., None]


def load_classes(reference_root: str, relpath: str, names: tuple[str, ...], namespace: dict):
    """Compile the named classes of one reference file, as written, into ``namespace``."""

    path = os.path.join(reference_root, "src", "mlx_diffuser", relpath)
    with open(path) as f:
        tree = ast.parse(f.read(), path)
    body = [n for n in tree.body if isinstance(n, ast.ClassDef) and n.name in names]
    if len(body) != len(names):
        raise RuntimeError(f"{names} not all found in {relpath}")
    code = compile(ast.Module(body=body, type_ignores=[]), path, "exec",
                   flags=__future__.annotations.compiler_flag, dont_inherit=True)
    exec(code, namespace)


def resblock_case(ref, reference_root: str) -> dict[str, np.ndarray]:
    """The reference's _SparseResBlock3D (with its LayerNorm32 and SparseLinear) in float32 on
    seeded parameters: a plain block with a linear skip, a downsampling block and an upsampling
    block fed by the downsampling block's output."""

    _, L = ref
    mx = sys.modules["mlx.core"]
    ns = {"mx": mx, "nn": sys.modules["mlx.nn"], "math": __import__("math"), "np": np,
          "SparseTensor": L.SparseTensor, "SparseConv3D": L.SparseConv3D,
          "sparse_downsample": L.sparse_downsample, "sparse_upsample": L.sparse_upsample}
    load_classes(reference_root, "layers/trellis.py", ("LayerNorm32",), ns)
    load_classes(reference_root, "layers/trellis_sparse.py", ("SparseLinear",), ns)
    load_classes(reference_root, "models/trellis_slat.py", ("_SparseResBlock3D",), ns)
    block_cls = ns["_SparseResBlock3D"]
    rng = np.random.default_rng(99)
    out: dict[str, np.ndarray] = {}

    def build(prefix, cin, cout, emb_ch, **kw):
        blk = block_cls(cin, emb_ch, out_channels=cout, use_metal=False, **kw)
        p = {
            "norm1_w": (1 + 0.1 * rng.standard_normal(cin)).astype(np.float32),
            "norm1_b": (0.1 * rng.standard_normal(cin)).astype(np.float32),
            "conv1_w": scenes.conv_weight(cout, cin, 3, int(rng.integers(1 << 30))),
            "conv1_b": (0.1 * rng.standard_normal(cout)).astype(np.float32),
            "conv2_w": scenes.conv_weight(cout, cout, 3, int(rng.integers(1 << 30))),
            "conv2_b": (0.1 * rng.standard_normal(cout)).astype(np.float32),
            "emb_w": (rng.standard_normal((2 * cout, emb_ch)) / np.sqrt(emb_ch)).astype(np.float32),
            "emb_b": (0.1 * rng.standard_normal(2 * cout)).astype(np.float32),
        }
        blk.norm1.weight, blk.norm1.bias = mx.array(p["norm1_w"]), mx.array(p["norm1_b"])
        blk.conv1.conv.weight, blk.conv1.conv.bias = mx.array(p["conv1_w"]), mx.array(p["conv1_b"])
        blk.conv2.conv.weight, blk.conv2.conv.bias = mx.array(p["conv2_w"]), mx.array(p["conv2_b"])
        blk.emb_layers[1].weight = mx.array(p["emb_w"])
        blk.emb_layers[1].bias = mx.array(p["emb_b"])
        if blk.skip_connection is not None:
            p["skip_w"] = (rng.standard_normal((cout, cin)) / np.sqrt(cin)).astype(np.float32)
            p["skip_b"] = (0.1 * rng.standard_normal(cout)).astype(np.float32)
            blk.skip_connection.weight = mx.array(p["skip_w"])
            blk.skip_connection.bias = mx.array(p["skip_b"])
        for k, v in p.items():
            out[f"{prefix}_{k}"] = v
        return blk

    coords = scenes.batched([scenes.shell(16, 5.5, 2.0, 1.0, seed=51),
                             scenes.shell(16, 6.5, 2.0, 1.0, seed=52)])
    feats = rng.standard_normal((len(coords), 8)).astype(np.float32)
    emb = rng.standard_normal((2, 12)).astype(np.float32)
    out["rb_coords"], out["rb_features"], out["rb_emb"] = coords, feats, emb
    x = L.SparseTensor(mx.array(feats), mx.array(coords))
    plain = build("plain", 8, 16, 12)
    y = plain(x, mx.array(emb))
    out["plain_out"] = np.asarray(y.features, np.float32)
    down = build("down", 16, 16, 12, downsample=True)
    d = down(y, mx.array(emb))
    out["down_coords"] = np.asarray(d.coords, np.int32)
    out["down_out"] = np.asarray(d.features, np.float32)
    up = build("up", 16, 8, 12, upsample=True)
    u = up(d, mx.array(emb))
    out["up_out"] = np.asarray(u.features, np.float32)
    return out


def topology_case(ref, reference_root: str) -> dict[str, np.ndarray]:
    _, L = ref
    mx = sys.modules["mlx.core"]
    rng = np.random.default_rng(77)
    out: dict[str, np.ndarray] = {}

    # sparse_subdivide: negative coordinates, two batch elements, 2-D feature rows, and a scale
    # that halves (4 -> 2) next to one that clamps (1 -> 1)
    c = rng.integers(-5, 6, size=(37, 4)).astype(np.int32)
    c[:, 0] = rng.integers(0, 2, size=37)
    f = rng.standard_normal((37, 2, 3)).astype(np.float32)
    t = L.SparseTensor(mx.array(f), mx.array(c), spatial_shape=(11, 12, 13), scale=(4, 1, 2))
    sub = L.sparse_subdivide(t)
    out["sub_coords_in"] = c
    out["sub_features_in"] = f
    out["sub_coords"] = np.asarray(sub.coords, np.int32)
    out["sub_features"] = np.asarray(sub.features, np.float32)
    out["sub_spatial_shape"] = np.asarray(sub.spatial_shape, np.int32)
    out["sub_scale"] = np.asarray(sub.scale, np.int32)

    # attention windows: three batch elements, negative coordinates, shifted windows
    c = rng.integers(-9, 17, size=(300, 4)).astype(np.int32)
    c[:, 0] = rng.integers(0, 3, size=300)
    c = np.concatenate([c, c[:17]])  # duplicate rows land in one group
    out["win_coords"] = c
    t = L.SparseTensor(mx.zeros((len(c), 1)), mx.array(c))
    cases = [(None, (0, 0, 0)), (8, (0, 0, 0)), (8, (4, 4, 4)), (3, (1, -2, 5))]
    for i, (window, shift) in enumerate(cases):
        groups = L._attention_groups(t, window, shift)
        out[f"win{i}_window"] = np.int32(-1 if window is None else window)
        out[f"win{i}_shift"] = np.asarray(shift, np.int32)
        out[f"win{i}_perm"] = np.concatenate(groups).astype(np.int32)
        out[f"win{i}_offsets"] = np.cumsum([0] + [len(g) for g in groups]).astype(np.int32)

    # windowed self-attention and cross-attention through the reference's own code
    heads, dim = 2, 8
    q = rng.standard_normal((len(c), heads, dim)).astype(np.float32)
    k = rng.standard_normal((len(c), heads, dim)).astype(np.float32)
    v = rng.standard_normal((len(c), heads, dim)).astype(np.float32)
    out["attn_q"], out["attn_k"], out["attn_v"] = q, k, v
    for i, (window, shift) in enumerate(cases[1:3]):
        o = L.sparse_self_attention(t, mx.array(q), mx.array(k), mx.array(v), window_size=window,
                                    shift_window=shift)
        out[f"attn{i}_out"] = np.asarray(o, np.float32)
    order = np.argsort(c[:, 0], kind="stable")  # cross-attention wants batch-contiguous rows
    cb = c[order]
    tb = L.SparseTensor(mx.zeros((len(cb), 1)), mx.array(cb))
    ctx_k = rng.standard_normal((3, 5, heads, dim)).astype(np.float32)
    ctx_v = rng.standard_normal((3, 5, heads, dim)).astype(np.float32)
    o = L.sparse_cross_attention(tb, mx.array(q), mx.array(ctx_k), mx.array(ctx_v))
    out["cross_coords"] = cb
    out["cross_k"], out["cross_v"] = ctx_k, ctx_v
    out["cross_out"] = np.asarray(o, np.float32)

    # occupancy -> coordinates, float32 and float16 logits, thresholds that need rounding
    occupied = load_occupied_coordinates(reference_root)
    logits = rng.standard_normal((2, 9, 10, 11)).astype(np.float32)
    logits[0, 3, 4, 5] = np.nan
    logits[1, 0, 0, 0] = np.float32(0.3)
    out["occ_logits"] = logits
    for i, thr in enumerate((0.0, 0.3, -1.25)):
        out[f"occ{i}_threshold"] = np.float64(thr)
        out[f"occ{i}_coords"] = np.asarray(occupied(_LogitsModel(mx.array(logits)), None, thr),
                                           np.int32)
    # float16(0.3) is above 0.3: a logit equal to it is above 0.3 but not above the rounded
    # threshold the comparison uses
    half = (rng.standard_normal((1, 7, 8, 9)) * 0.4).astype(np.float16)
    half[0, 1, 2, 3] = np.float16(0.3)
    out["occ_half_logits"] = half
    out["occ_half_threshold"] = np.float64(0.3)
    out["occ_half_coords"] = np.asarray(occupied(_LogitsModel(mx.array(half)), None, 0.3),
                                        np.int32)
    return out


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.environ.get("MLX_DIFFUSER_REF", "/root/reference"))
    args = parser.parse_args()
    ref = load_reference(args.reference)
    for name, data in cases(ref):
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **data)
        print(f"{name}: N={len(data['coords'])} -> {os.path.relpath(path, ROOT)}")
    path = os.path.join(HERE, "topology.npz")
    np.savez_compressed(path, **topology_case(ref, args.reference))
    print(f"topology -> {os.path.relpath(path, ROOT)}")
    path = os.path.join(HERE, "resblock.npz")
    np.savez_compressed(path, **resblock_case(ref, args.reference))
    print(f"resblock -> {os.path.relpath(path, ROOT)}")


if __name__ == "__main__":
    main()
