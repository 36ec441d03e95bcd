"""Device preprocessing (cuvit_preprocess) against the reference's cuvit::preprocess
(src/runtime/image.cpp:90-135): bit for bit against the C restatement (pinned to the
reference's own output by the golden vectors) and, where oracle/_ref is built, against the
reference's compiled code itself; batches with padded strides; and the preprocessed tensor
feeding the model gives the same logits as the host-preprocessed one."""

from __future__ import annotations

import numpy as np
import pytest

import make_golden as mg
import oracle
from cuvit import VisionTransformer, kernels
from cuvit.vit import PRECISION_BF16, VitConfig, random_weights
from helpers import to_host

pytestmark = pytest.mark.gpu


def device_preprocess(cuda, pixels, size, crop, mean, stddev, stride=0):
    """pixels: uint8 [batch, H, W, 3] (or one [H, W, 3]); returns float [batch, 3, size, size]."""
    if pixels.ndim == 3:
        pixels = pixels[None]
    batch, height, width, _ = pixels.shape
    flat = pixels.reshape(batch, -1)
    if stride:
        padded = np.zeros((batch, stride), np.uint8)
        padded[:, :flat.shape[1]] = flat
        flat = padded
    d_pixels = cuda.from_numpy(np.ascontiguousarray(flat)).cuda()
    out = cuda.full((batch, 3, size, size), float("nan"), device="cuda")
    kernels.launch_preprocess(d_pixels, out, batch, width, height, size, crop, mean, stddev,
                              image_stride=stride)
    cuda.cuda.synchronize()
    return to_host(out)


@pytest.mark.parametrize("case", mg.PREPROCESS_CASES, ids=[c[0] for c in mg.PREPROCESS_CASES])
def test_preprocess_is_bitwise_the_reference(case, golden, cuda):
    label, height, width, size, crop, mean, stddev, seed = case
    pixels = mg.preprocess_image(height, width, seed)
    got = device_preprocess(cuda, pixels, size, crop, mean, stddev)[0]
    want = oracle.preprocess(pixels, size, crop, mean, stddev)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    rows = golden[f"preprocess/{label}/rows"]
    np.testing.assert_array_equal(got[:, rows, :], golden[f"preprocess/{label}/y"])
    if oracle.ref_cpu_available():
        np.testing.assert_array_equal(got, oracle.ref_preprocess(pixels, size, crop, mean,
                                                                 stddev))


def test_batches_and_strides(cuda):
    """Three images of one size, packed and with a padded stride, against per-image oracle
    runs; odd sizes and a non-unit scale in both directions."""
    rng = np.random.default_rng(7)
    for height, width, size, crop in ((120, 90, 64, 0.875), (33, 257, 48, 1.0),
                                      (480, 640, 224, 0.9)):
        pixels = rng.integers(0, 256, (3, height, width, 3), dtype=np.uint8)
        want = np.stack([oracle.preprocess(p, size, crop, mg.IMAGENET_MEAN, mg.IMAGENET_STD)
                         for p in pixels])
        for stride in (0, height * width * 3 + 40):
            got = device_preprocess(cuda, pixels, size, crop, mg.IMAGENET_MEAN,
                                    mg.IMAGENET_STD, stride)
            np.testing.assert_array_equal(got, want, err_msg=f"{height}x{width} {stride}")


def test_preprocessed_images_feed_the_model(cuda):
    """Real-image path on the device: RGB bytes -> cuvit_preprocess -> forward gives the logits
    of the same model on the host-preprocessed tensor, bitwise."""
    config = VitConfig(image_size=32, patch_size=8, channels=3, embed_dim=128, depth=2,
                       heads=2, mlp_hidden=256, classes=10)
    weights = random_weights(config, 12, std=0.05)
    rng = np.random.default_rng(8)
    pixels = rng.integers(0, 256, (4, 50, 70, 3), dtype=np.uint8)
    host = np.stack([oracle.preprocess(p, 32, 0.9) for p in pixels]).astype(np.float32)
    model = VisionTransformer(config, weights, max_batch=4, precision=PRECISION_BF16)
    d_pixels = cuda.from_numpy(pixels.reshape(4, -1)).cuda()
    d_images = cuda.empty((4, 3, 32, 32), device="cuda")
    kernels.launch_preprocess(d_pixels, d_images, 4, 70, 50, 32, 0.9)
    from_device = cuda.zeros((4, 10), device="cuda")
    model.forward(d_images, from_device, 4)
    from_host = cuda.zeros((4, 10), device="cuda")
    model.forward(cuda.from_numpy(host).cuda(), from_host, 4)
    cuda.cuda.synchronize()
    np.testing.assert_array_equal(to_host(from_device), to_host(from_host))
    model.close()
