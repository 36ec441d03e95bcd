"""Writes tests/golden/golden.npz from the reference's own CPU implementation.

Run in a checkout where the Cu-Vit sources are available and oracle/_ref is built
(`make -C oracle ref`); the GPU box never runs this. Inputs are generated from numpy seeds;
the fixture stores each input's SHA-256 so tests can regenerate them and prove they are the
same bytes, plus the reference's outputs (whole for small cases, sampled rows for large
ones). Every output comes from oracle/_ref/libcuvit_ref_cpu.so -- the reference's
tests/reference/*.hpp and src/runtime/weights.cpp compiled in place -- never from this
repository's restatement, which the fixture exists to pin.

    python tests/golden/make_golden.py
"""

from __future__ import annotations

import hashlib
import pathlib
import sys
import tempfile

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "cu-vit_b200"))

import oracle  # noqa: E402
from cuvit import cvw  # noqa: E402
from cuvit.vit import VitConfig, random_weights, tensor_specs  # noqa: E402

OUT = pathlib.Path(__file__).resolve().parent / "golden.npz"


def digest(array: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(array, np.float32).tobytes()).hexdigest()


# ---- seeded inputs (tests regenerate them with the same functions) -------------------------

def gemm_inputs(m, n, k, seed, distribution="normal"):
    rng = np.random.default_rng(seed)
    draw = (lambda size: rng.uniform(-1.0, 1.0, size)) if distribution == "uniform" else (
        lambda size: rng.standard_normal(size))
    a = draw(m * k).astype(np.float32)
    b = draw(k * n).astype(np.float32)
    bias = draw(n).astype(np.float32)
    existing = draw(m * n).astype(np.float32)
    return a, b, bias, existing


GEMM_CASES = [
    # (label, m, n, k, transposed, alpha, bias, epilogue, distribution, seed)
    ("1x1x1", 1, 1, 1, True, 1.0, True, "none", "normal", 11),
    ("small odd", 17, 33, 7, False, 1.0, True, "none", "normal", 12),
    ("just under a tile", 63, 63, 63, True, 1.0, False, "none", "normal", 13),
    ("just over a tile", 65, 65, 65, False, 1.0, True, "none", "normal", 14),
    ("negative scale", 32, 48, 16, False, -2.5, True, "none", "normal", 15),
    ("scaled attention logits", 197, 197, 64, True, 0.125, False, "none", "normal", 16),
    # The single-GEMM benchmark case: ViT-Tiny QKV shape, U(-1, 1) from seed 0, then GELU and
    # accumulate.
    ("config1 qkv", 197, 576, 192, True, 1.0, True, "none", "uniform", 0),
    ("config1 gelu", 197, 768, 192, True, 1.0, True, "gelu", "uniform", 0),
    ("config1 accumulate", 197, 192, 768, True, 1.0, True, "accumulate", "uniform", 0),
]

SAMPLE_ROWS = 9  # rows kept for large outputs: the first 8 and the last


def sample_rows(m: int) -> np.ndarray:
    if m <= 24:
        return np.arange(m)
    return np.concatenate([np.arange(8), [m - 1]])


LN_CASES = [("ln 1x192", 1, 192, 0.0, 101), ("ln 197x192", 197, 192, 0.0, 102),
            ("ln 3x1", 3, 1, 0.0, 103), ("ln 5x31", 5, 31, 0.0, 104),
            ("ln 2x1024", 2, 1024, 0.0, 105), ("ln offset 1000", 197, 192, 1000.0, 106)]


def ln_inputs(rows, columns, offset, seed):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(rows * columns) + offset).astype(np.float32)
    gamma = (1.0 + 0.2 * rng.standard_normal(columns)).astype(np.float32)
    beta = (0.2 * rng.standard_normal(columns)).astype(np.float32)
    if offset != 0.0:
        gamma[:] = 1.0
        beta[:] = 0.0
    return x, gamma, beta


SOFTMAX_CASES = [("sm 1x2", 1, 2, 201), ("sm 4x1", 4, 1, 202), ("sm 8x33", 8, 33, 203),
                 ("sm 3x1000", 3, 1000, 204), ("sm 197x197", 197, 197, 205)]


def softmax_inputs(rows, columns, seed):
    rng = np.random.default_rng(seed)
    return (4.0 * rng.standard_normal(rows * columns)).astype(np.float32)


def gelu_inputs():
    rng = np.random.default_rng(31)
    x = (3.0 * rng.standard_normal(4099)).astype(np.float32)
    landmarks = [-30.0, -8.0, -2.7, -2.0, -1.0, -0.5, 0.0, 0.5, 1.0, 2.0, 2.7, 8.0, 30.0]
    x[:len(landmarks)] = landmarks
    return x


# Model cases: the reference vit_test's small config (tests/vit_test.cu:36-47), a head_dim-64
# config that exercises the fused attention path, and ViT-Tiny/16 itself (the TF32 benchmark
# configuration).
VIT_CASES = [
    ("vit small", VitConfig(32, 8, 3, 24, 3, 4, 48, 7), 1234, 0.2, 3, 1),
    ("vit hd64", VitConfig(32, 8, 3, 128, 2, 2, 256, 10), 77, 0.05, 3, 2),
    ("vit tiny", VitConfig(), 1, 0.02, 2, 3),
]


# Image preprocessing (src/runtime/image.cpp:90-135): (label, height, width, size,
# crop_fraction, mean, stddev, seed). Landscape, square, portrait, a single pixel (every tap
# clamps) and a wide strip; the timm defaults (0.5) and the ImageNet statistics.
IMAGENET_MEAN = (0.485, 0.456, 0.406)
IMAGENET_STD = (0.229, 0.224, 0.225)
PREPROCESS_CASES = [
    ("landscape 375x500", 375, 500, 224, 0.9, (0.5, 0.5, 0.5), (0.5, 0.5, 0.5), 41),
    ("square 224", 224, 224, 224, 1.0, IMAGENET_MEAN, IMAGENET_STD, 42),
    ("portrait 61x37 to 32", 61, 37, 32, 0.875, IMAGENET_MEAN, IMAGENET_STD, 43),
    ("single pixel to 8", 1, 1, 8, 0.9, (0.5, 0.5, 0.5), (0.5, 0.5, 0.5), 44),
    ("wide 100x300", 100, 300, 224, 0.95, (0.5, 0.5, 0.5), (0.25, 0.5, 1.0), 45),
]


def preprocess_image(height: int, width: int, seed: int) -> np.ndarray:
    """Interleaved 8-bit RGB [height, width, 3]."""
    return np.random.default_rng(seed).integers(0, 256, (height, width, 3), dtype=np.uint8)


def vit_images(config: VitConfig, count: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.standard_normal(count * config.image_elements()).astype(np.float32)


def main() -> None:
    if not oracle.ref_cpu_available():
        raise SystemExit("oracle/_ref/libcuvit_ref_cpu.so is missing: make -C oracle ref")
    ref = oracle.ref_cpu()
    out: dict[str, np.ndarray] = {}

    for label, m, n, k, transposed, alpha, with_bias, epilogue, dist, seed in GEMM_CASES:
        a, b, bias, existing = gemm_inputs(m, n, k, seed, dist)
        product = np.empty(m * n, np.float32)
        ref.ref_gemm(a, b, bias.ctypes.data if with_bias else None, product, m, n, k,
                     int(transposed), alpha)
        if epilogue == "gelu":
            ref.ref_gelu(product, product, product.size)
        elif epilogue == "accumulate":
            product = (existing + product).astype(np.float32)
        scale = np.empty(m * n, np.float32)
        ref.ref_gemm_term_magnitudes(a, b, scale, m, n, k, int(transposed), alpha)
        rows = sample_rows(m)
        key = f"gemm/{label}"
        out[key + "/rows"] = rows
        out[key + "/c"] = product.reshape(m, n)[rows]
        out[key + "/scale"] = scale.reshape(m, n)[rows]
        out[key + "/sha"] = np.array([digest(a), digest(b), digest(bias), digest(existing)])

    for label, rows, columns, offset, seed in LN_CASES:
        x, gamma, beta = ln_inputs(rows, columns, offset, seed)
        y = np.empty_like(x)
        ref.ref_layer_norm(x, gamma, beta, y, rows, columns, 1e-6)
        keep = sample_rows(rows)
        out[f"ln/{label}/rows"] = keep
        out[f"ln/{label}/y"] = y.reshape(rows, columns)[keep]
        out[f"ln/{label}/sha"] = np.array([digest(x), digest(gamma), digest(beta)])

    for label, rows, columns, seed in SOFTMAX_CASES:
        x = softmax_inputs(rows, columns, seed)
        y = np.empty_like(x)
        ref.ref_softmax(x, y, rows, columns)
        keep = sample_rows(rows)
        out[f"softmax/{label}/rows"] = keep
        out[f"softmax/{label}/y"] = y.reshape(rows, columns)[keep]
        out[f"softmax/{label}/sha"] = np.array([digest(x)])

    x = gelu_inputs()
    y = np.empty_like(x)
    ref.ref_gelu(x, y, x.size)
    out["gelu/y"] = y
    out["gelu/sha"] = np.array([digest(x)])

    for label, height, width, size, crop, mean, stddev, seed in PREPROCESS_CASES:
        pixels = preprocess_image(height, width, seed)
        tensor = oracle.ref_preprocess(pixels, size, crop, mean, stddev)
        keep = sample_rows(size)
        out[f"preprocess/{label}/rows"] = keep
        out[f"preprocess/{label}/y"] = tensor[:, keep, :]
        out[f"preprocess/{label}/sha"] = np.array(
            [hashlib.sha256(pixels.tobytes()).hexdigest()])

    with tempfile.TemporaryDirectory() as tmp:
        for label, config, weight_seed, std, count, image_seed in VIT_CASES:
            weights = random_weights(config, weight_seed, std=std)
            writer = cvw.WeightFileWriter()
            for name, extents in tensor_specs(config):
                writer.add(name, extents, weights[name])
            path = pathlib.Path(tmp) / "weights.cvw"
            writer.write(path)
            images = vit_images(config, count, image_seed)
            logits = oracle.ref_vit_forward(path, config, images)
            out[f"vit/{label}/logits"] = logits
            out[f"vit/{label}/sha"] = np.array(
                [digest(images)] + [digest(weights[n]) for n, _ in tensor_specs(config)])

    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()
