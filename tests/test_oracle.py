"""The CPU oracle pinned against golden vectors the reference's own code produced.

tests/golden/golden.npz was written by tests/golden/make_golden.py from the reference's
tests/reference/*.hpp compiled in place (oracle/_ref). The oracle (oracle/cuvit_oracle.c)
restates those algorithms in C with the same floating-point operation order, so it must
reproduce the golden values bit for bit.
"""

from __future__ import annotations

import hashlib
import pathlib
import sys
import tempfile

import numpy as np
import pytest

sys.path.insert(0, str(pathlib.Path(__file__).resolve().parent / "golden"))
import make_golden as mg  # noqa: E402

from cuvit import cvw  # noqa: E402
from cuvit.vit import VitConfig, random_weights, tensor_specs  # noqa: E402


def digest(array) -> str:
    return hashlib.sha256(np.ascontiguousarray(array, np.float32).tobytes()).hexdigest()


@pytest.mark.parametrize("case", mg.GEMM_CASES, ids=[c[0] for c in mg.GEMM_CASES])
def test_gemm_matches_reference_bitwise(case, golden, oracle_lib):
    label, m, n, k, transposed, alpha, with_bias, epilogue, dist, seed = case
    a, b, bias, existing = mg.gemm_inputs(m, n, k, seed, dist)
    key = f"gemm/{label}"
    assert list(golden[key + "/sha"]) == [digest(a), digest(b), digest(bias), digest(existing)]
    c = oracle_lib.gemm(a, b, bias if with_bias else None,
                        existing if epilogue == "accumulate" else np.zeros(m * n, np.float32),
                        m, n, k, transposed, alpha=alpha, accumulate=epilogue == "accumulate",
                        gelu=epilogue == "gelu")
    rows = golden[key + "/rows"]
    np.testing.assert_array_equal(c.reshape(m, n)[rows], golden[key + "/c"])
    scale = oracle_lib.gemm_term_magnitudes(a, b, m, n, k, transposed, alpha)
    np.testing.assert_array_equal(scale.reshape(m, n)[rows], golden[key + "/scale"])


@pytest.mark.parametrize("case", mg.LN_CASES, ids=[c[0] for c in mg.LN_CASES])
def test_layer_norm_matches_reference_bitwise(case, golden, oracle_lib):
    label, rows, columns, offset, seed = case
    x, gamma, beta = mg.ln_inputs(rows, columns, offset, seed)
    assert list(golden[f"ln/{label}/sha"]) == [digest(x), digest(gamma), digest(beta)]
    y = oracle_lib.layer_norm(x, gamma, beta, rows, columns, 1e-6).reshape(rows, columns)
    keep = golden[f"ln/{label}/rows"]
    np.testing.assert_array_equal(y[keep], golden[f"ln/{label}/y"])


@pytest.mark.parametrize("case", mg.SOFTMAX_CASES, ids=[c[0] for c in mg.SOFTMAX_CASES])
def test_softmax_matches_reference_bitwise(case, golden, oracle_lib):
    label, rows, columns, seed = case
    x = mg.softmax_inputs(rows, columns, seed)
    assert list(golden[f"softmax/{label}/sha"]) == [digest(x)]
    y = oracle_lib.softmax(x, rows, columns).reshape(rows, columns)
    keep = golden[f"softmax/{label}/rows"]
    np.testing.assert_array_equal(y[keep], golden[f"softmax/{label}/y"])


def test_gelu_matches_reference_bitwise(golden, oracle_lib):
    x = mg.gelu_inputs()
    assert list(golden["gelu/sha"]) == [digest(x)]
    np.testing.assert_array_equal(oracle_lib.gelu(x), golden["gelu/y"])
    # The erf and tanh forms must be distinguishable at the tolerance tests use
    # (the reference's own check, tests/elementwise_test.cu:51-60).
    probe = np.float32(-2.7)
    tanh_form = 0.5 * probe * (1 + np.tanh(0.7978845608 * (probe + 0.044715 * probe ** 3)))
    assert abs(tanh_form - oracle_lib.gelu(np.array([probe]))[0]) > 4.0e-4


@pytest.mark.parametrize("case", mg.VIT_CASES, ids=[c[0] for c in mg.VIT_CASES])
def test_vit_forward_matches_reference_bitwise(case, golden, oracle_lib):
    label, config, weight_seed, std, count, image_seed = case
    weights = random_weights(config, weight_seed, std=std)
    images = mg.vit_images(config, count, image_seed)
    assert list(golden[f"vit/{label}/sha"]) == (
        [digest(images)] + [digest(weights[n]) for n, _ in tensor_specs(config)])
    logits = oracle_lib.vit_forward(config, weights, tensor_specs(config), images)
    np.testing.assert_array_equal(logits, golden[f"vit/{label}/logits"])


@pytest.mark.parametrize("case", mg.PREPROCESS_CASES, ids=[c[0] for c in mg.PREPROCESS_CASES])
def test_preprocess_matches_reference_bitwise(case, golden, oracle_lib):
    """src/runtime/image.cpp:90-135 -- resize, centre crop, normalise -- bit for bit."""
    import hashlib

    label, height, width, size, crop, mean, stddev, seed = case
    pixels = mg.preprocess_image(height, width, seed)
    assert list(golden[f"preprocess/{label}/sha"]) == [hashlib.sha256(pixels.tobytes()).hexdigest()]
    got = oracle_lib.preprocess(pixels, size, crop, mean, stddev)
    rows = golden[f"preprocess/{label}/rows"]
    np.testing.assert_array_equal(got[:, rows, :], golden[f"preprocess/{label}/y"])


def test_preprocess_rejects_what_the_reference_rejects(oracle_lib):
    pixels = np.zeros((4, 4, 3), np.uint8)
    for size, crop, stddev in ((0, 0.9, (1, 1, 1)), (8, 0.0, (1, 1, 1)), (8, 1.5, (1, 1, 1)),
                               (8, 0.9, (1, 0, 1))):
        with pytest.raises(ValueError):
            oracle_lib.preprocess(pixels, size, crop, (0, 0, 0), stddev)


def test_extract_patches_is_the_documented_gather(oracle_lib):
    # patches[b*P + p][c*pp + r*patch + q] = images[b][c][pr*patch + r][pc*patch + q]
    rng = np.random.default_rng(5)
    batch, channels, size, patch = 2, 3, 32, 8
    images = rng.standard_normal((batch, channels, size, size)).astype(np.float32)
    across = size // patch
    expected = images.reshape(batch, channels, across, patch, across, patch)
    expected = expected.transpose(0, 2, 4, 1, 3, 5).reshape(batch * across * across, -1)
    got = oracle_lib.extract_patches(images, batch, channels, size, size, patch)
    np.testing.assert_array_equal(got.reshape(expected.shape), expected)


def test_top_k_report_is_the_documented_selection(oracle_lib):
    """report_top (src/main.cpp:90-114): the k largest logits per row in descending order
    (equal logits by ascending class index) and softmax probabilities in double."""
    rng = np.random.default_rng(9)
    logits = rng.standard_normal((6, 1000)).astype(np.float32) * 3
    logits[1, [10, 20, 30]] = 50.0          # a three-way tie at the top
    logits[2, :] = 1.0                      # every logit equal
    logits[3, 5] = -np.inf
    logits[4, 7] = np.nan                   # never reported
    for k in (1, 5, 40):
        indices, values, probabilities = oracle_lib.top_k(logits, k)
        for row in range(logits.shape[0]):
            x = logits[row]
            keep = np.flatnonzero(~np.isnan(x))
            order = keep[np.lexsort((keep, -x[keep].astype(np.float64)))][:k]
            np.testing.assert_array_equal(indices[row], order)
            np.testing.assert_array_equal(values[row], x[order])
            top = np.nanmax(x).astype(np.float64)
            total = np.exp(x[keep].astype(np.float64) - top).sum()
            if row != 4:  # the reference's sum runs over every logit; a NaN poisons it
                np.testing.assert_allclose(probabilities[row],
                                           np.exp(x[order].astype(np.float64) - top) / total,
                                           rtol=1e-12)
    indices, _, _ = oracle_lib.top_k(logits, 3)
    assert list(indices[1]) == [10, 20, 30]
    assert list(indices[2]) == [0, 1, 2]


def test_attention_matches_float64_definition(oracle_lib):
    rng = np.random.default_rng(9)
    tokens, embed, heads = 17, 32, 4
    d = embed // heads
    qkv = rng.standard_normal((tokens, 3 * embed)).astype(np.float32)
    got = oracle_lib.attention(qkv, tokens, embed, heads).reshape(tokens, embed)
    q = qkv[:, :embed].reshape(tokens, heads, d).astype(np.float64)
    k = qkv[:, embed:2 * embed].reshape(tokens, heads, d).astype(np.float64)
    v = qkv[:, 2 * embed:].reshape(tokens, heads, d).astype(np.float64)
    s = np.einsum("qhd,khd->hqk", q, k) / np.sqrt(d)
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    want = np.einsum("hqk,khd->qhd", p, v).reshape(tokens, embed)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5)


def test_elementwise_helpers(oracle_lib):
    rng = np.random.default_rng(3)
    acc = rng.standard_normal(40).astype(np.float32)
    addend = rng.standard_normal(10).astype(np.float32)
    np.testing.assert_array_equal(oracle_lib.add_broadcast(acc, addend, 10, 4),
                                  acc + np.tile(addend, 4))
    np.testing.assert_array_equal(oracle_lib.add(acc, acc), acc + acc)
    dst = np.zeros(30, np.float32)
    out = oracle_lib.broadcast(dst, addend[:4], 4, 10, 3).reshape(3, 10)
    np.testing.assert_array_equal(out[:, :4], np.tile(addend[:4], (3, 1)))
    assert not out[:, 4:].any()


@pytest.mark.skipif(not __import__("oracle").ref_cpu_available(),
                    reason="oracle/_ref not built (needs the reference sources)")
def test_oracle_matches_reference_library_directly(oracle_lib):
    """Beyond the fixture: the restatement against the reference's compiled code on fresh
    inputs, including a .cvw file written by this package and read by the reference."""
    rng = np.random.default_rng(2024)
    ref = oracle_lib.ref_cpu()
    for m, n, k, transposed in [(7, 9, 5, True), (40, 24, 32, False), (197, 64, 197, False)]:
        a = rng.standard_normal(m * k).astype(np.float32)
        b = rng.standard_normal(k * n).astype(np.float32)
        bias = rng.standard_normal(n).astype(np.float32)
        want = np.empty(m * n, np.float32)
        ref.ref_gemm(a, b, bias.ctypes.data, want, m, n, k, int(transposed), 0.5)
        got = oracle_lib.gemm(a, b, bias, np.zeros(m * n, np.float32), m, n, k, transposed,
                              alpha=0.5)
        np.testing.assert_array_equal(got, want)
    config = VitConfig(16, 4, 3, 16, 2, 2, 32, 5)
    weights = random_weights(config, 42, std=0.3)
    images = rng.standard_normal(2 * config.image_elements()).astype(np.float32)
    with tempfile.TemporaryDirectory() as tmp:
        path = pathlib.Path(tmp) / "w.cvw"
        writer = cvw.WeightFileWriter()
        for name, extents in tensor_specs(config):
            writer.add(name, extents, weights[name])
        writer.write(path)
        want = oracle_lib.ref_vit_forward(path, config, images, threads=2)
    got = oracle_lib.vit_forward(config, weights, tensor_specs(config), images)
    np.testing.assert_array_equal(got, want)
