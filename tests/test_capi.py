"""The C ABI on the CPU: the library loads, exports every symbol include/*.h declares, and
rejects bad arguments on the host -- with the reference launchers' outcome classes and
messages -- before touching a GPU. No compute call is made here."""

from __future__ import annotations

import ctypes
import pathlib
import re
import tempfile

import numpy as np
import pytest

import cuvit
from cuvit import _lib, cvw, kernels
from cuvit.errors import InvalidArgument, LengthError, Unsupported, WeightError
from cuvit.vit import VitConfig, random_weights, tensor_specs

ROOT = pathlib.Path(__file__).resolve().parents[1]
FAKE = 0x10000  # a non-null address that is never dereferenced: validation fails first


def declared_functions() -> set[str]:
    header = (ROOT / "include" / "cuvit_b200.h").read_text()
    header = re.sub(r"/\*.*?\*/", "", header, flags=re.S)
    return set(re.findall(r"\b(cuvit_[a-z0-9_]+)\s*\(", header))


def test_library_exports_every_declared_symbol():
    lib = cuvit.library()
    declared = declared_functions()
    assert len(declared) >= 39
    for name in sorted(declared):
        assert hasattr(lib, name), f"{name} is declared in cuvit_b200.h but not exported"
    assert declared == set(_lib.SIGNATURES), "ctypes signatures drifted from the header"


def test_status_strings():
    lib = cuvit.library()
    assert lib.cuvit_status_string(0) == b"ok"
    assert lib.cuvit_status_string(1) == b"invalid argument"
    assert lib.cuvit_status_string(4) == b"device-side wait timed out"
    assert lib.cuvit_version() >= 100


def test_gemm_validation_matches_reference():
    # empty problems are no-ops (src/kernels/gemm.cu:205-207), even with null pointers
    kernels.launch_gemm(None, None, None, None, kernels.gemm_problem(0, 4, 4, 0))
    kernels.launch_gemm(None, None, None, None, kernels.gemm_problem(4, 0, 4, 0))
    problem = kernels.gemm_problem(4, 4, 4, 0)
    problem.batch.count = 0
    kernels.launch_gemm(None, None, None, None, problem)
    with pytest.raises(InvalidArgument, match="cannot be negative"):
        kernels.launch_gemm(FAKE, FAKE, None, FAKE, kernels.gemm_problem(-1, 4, 4, 0))
    with pytest.raises(InvalidArgument, match="cannot be null"):
        kernels.launch_gemm(None, FAKE, None, FAKE, kernels.gemm_problem(4, 4, 4, 0))
    split = kernels.gemm_problem(4, 4, 4, 0)
    split.batch.count = 5
    split.batch.inner = 2
    with pytest.raises(InvalidArgument, match="whole inner groups"):
        kernels.launch_gemm(FAKE, FAKE, None, FAKE, split)
    narrow = kernels.gemm_problem(4, 4, 8, 1)
    narrow.lda = 4
    with pytest.raises(InvalidArgument, match="leading dimension"):
        kernels.launch_gemm(FAKE, FAKE, None, FAKE, narrow)
    with pytest.raises(ValueError):  # InvalidArgument is a ValueError, as invalid_argument
        kernels.launch_gemm_ex(FAKE, FAKE, None, FAKE, kernels.gemm_problem(4, 4, 4, 0),
                               c_dtype=7)


def test_math_mode():
    assert kernels.get_math_mode() == kernels.MATH_FP32
    kernels.set_math_mode(kernels.MATH_TF32)
    assert kernels.get_math_mode() == kernels.MATH_TF32
    kernels.set_math_mode(kernels.MATH_FP32)
    with pytest.raises(InvalidArgument):
        kernels.set_math_mode(kernels.MATH_BF16)


def test_elementwise_validation_matches_reference():
    kernels.launch_gelu(None, None, 0)
    kernels.launch_softmax(None, None, 0, 4)
    kernels.launch_layer_norm(None, None, None, None, 0, 4)
    kernels.launch_add(None, None, 0)
    kernels.launch_add_broadcast(None, None, 0, 3)
    kernels.launch_broadcast(None, None, 4, 4, 0)
    kernels.launch_extract_patches(None, None, 0, 3, 32, 32, 8)
    with pytest.raises(InvalidArgument, match="GELU operands cannot be null"):
        kernels.launch_gelu(None, FAKE, 4)
    with pytest.raises(InvalidArgument, match="Layer norm operands cannot be null"):
        kernels.launch_layer_norm(FAKE, None, FAKE, FAKE, 2, 4)
    with pytest.raises(InvalidArgument, match="cannot be negative"):
        kernels.launch_softmax(FAKE, FAKE, -1, 4)
    with pytest.raises(InvalidArgument, match="whole patches"):
        kernels.launch_extract_patches(FAKE, FAKE, 1, 3, 30, 32, 8)
    with pytest.raises(InvalidArgument, match="must be positive"):
        kernels.launch_extract_patches(FAKE, FAKE, 1, 0, 32, 32, 8)
    with pytest.raises(InvalidArgument, match="inconsistent"):
        kernels.launch_broadcast(FAKE, FAKE, 8, 4, 2)
    with pytest.raises(InvalidArgument, match="cannot be negative"):
        kernels.launch_add(FAKE, FAKE, -3)
    with pytest.raises(InvalidArgument, match="cannot be negative"):
        kernels.launch_add_broadcast(FAKE, FAKE, 4, -1)
    with pytest.raises(LengthError, match="grid limit"):
        kernels.launch_gelu(FAKE, FAKE, 1 << 62)


def test_top_k_report_validation():
    """cuvit_logits_top_k (the CLI's report_top on device logits): empty batches are no-ops,
    bad extents and null operands fail on the host."""
    kernels.launch_logits_top_k(None, None, None, None, 0, 1000, 5)
    with pytest.raises(InvalidArgument, match="1 <= k <= classes"):
        kernels.launch_logits_top_k(FAKE, FAKE, FAKE, FAKE, 2, 10, 11)
    with pytest.raises(InvalidArgument, match="1 <= k <= classes"):
        kernels.launch_logits_top_k(FAKE, FAKE, FAKE, FAKE, 2, 10, 0)
    with pytest.raises(InvalidArgument, match="1 <= k <= classes"):
        kernels.launch_logits_top_k(FAKE, FAKE, FAKE, FAKE, -1, 10, 3)
    with pytest.raises(InvalidArgument, match="cannot be null"):
        kernels.launch_logits_top_k(FAKE, None, FAKE, FAKE, 2, 10, 3)
    lib = _lib.library()
    assert lib.cuvit_vit_host_image_bytes(None) == 0


def test_attention_validation():
    kernels.launch_attention(None, None, kernels.DTYPE_BF16, 0, 197, 12, 64, 0.125)
    with pytest.raises(Unsupported, match="head_dim 64"):
        kernels.launch_attention(FAKE, FAKE, kernels.DTYPE_BF16, 1, 197, 12, 32, 0.125)
    with pytest.raises(Unsupported, match="256 tokens"):
        kernels.launch_attention(FAKE, FAKE, kernels.DTYPE_BF16, 1, 300, 12, 64, 0.125)
    with pytest.raises(InvalidArgument, match="aligned"):
        kernels.launch_attention(FAKE + 4, FAKE, kernels.DTYPE_BF16, 1, 197, 12, 64, 0.125)
    with pytest.raises(InvalidArgument, match="BF16, F32 or TF32"):
        kernels.launch_attention(FAKE, FAKE, 9, 1, 197, 12, 64, 0.125)


def test_config_validation_matches_reference():
    VitConfig().validate()
    with pytest.raises(InvalidArgument, match="divide across the heads"):
        VitConfig(32, 8, 3, 25, 3, 4, 48, 7).validate()
    with pytest.raises(InvalidArgument, match="whole patches"):
        VitConfig(30, 8, 3, 24, 3, 4, 48, 7).validate()
    with pytest.raises(InvalidArgument, match="must be positive"):
        VitConfig(32, 8, 3, 24, 0, 4, 48, 7).validate()


def test_tensor_table_matches_reference_names():
    config = VitConfig(32, 8, 3, 24, 3, 4, 48, 7)
    lib = cuvit.library()
    c_config = config.to_c()
    count = lib.cuvit_vit_tensor_count(ctypes.byref(c_config))
    specs = tensor_specs(config)
    assert count == len(specs) == 4 + 12 * 3 + 4
    name = ctypes.create_string_buffer(128)
    extents = (ctypes.c_int64 * 4)()
    rank = ctypes.c_int(0)
    for index, (want_name, want_extents) in enumerate(specs):
        status = lib.cuvit_vit_tensor_info(ctypes.byref(c_config), index, name, 128, extents,
                                           ctypes.byref(rank))
        assert status == 0
        assert name.value.decode() == want_name
        assert tuple(extents[:rank.value]) == tuple(want_extents)
    assert specs[0][0] == "cls_token" and specs[-1][0] == "head.bias"


def test_weight_file_errors_are_reported_before_any_device_work():
    config = VitConfig(32, 8, 3, 24, 3, 4, 48, 7)
    with tempfile.TemporaryDirectory() as tmp:
        missing = pathlib.Path(tmp) / "missing.cvw"
        with pytest.raises(WeightError, match="Cannot open"):
            cuvit.VisionTransformer.from_file(config, missing)
        bogus = pathlib.Path(tmp) / "bogus.cvw"
        bogus.write_bytes(b"NOPE" + bytes(60))
        with pytest.raises(WeightError, match="Not a Cu-Vit weight file"):
            cuvit.VisionTransformer.from_file(config, bogus)
        # Weights written for one shape, loaded with another (tests/vit_test.cu:347-367).
        weights = random_weights(config, 3)
        writer = cvw.WeightFileWriter()
        for tensor, extents in tensor_specs(config):
            writer.add(tensor, extents, weights[tensor])
        path = pathlib.Path(tmp) / "small.cvw"
        writer.write(path)
        wrong = VitConfig(32, 8, 3, 48, 3, 4, 48, 7)
        with pytest.raises(WeightError, match="has shape"):
            cuvit.VisionTransformer.from_file(wrong, path)
        deeper = VitConfig(32, 8, 3, 24, 4, 4, 48, 7)
        with pytest.raises(WeightError, match="no tensor named 'blocks.3"):
            cuvit.VisionTransformer.from_file(deeper, path)


def test_model_creation_validation():
    config = VitConfig(32, 8, 3, 24, 3, 4, 48, 7)
    weights = random_weights(config, 3)
    with pytest.raises(InvalidArgument, match="at least one"):
        cuvit.VisionTransformer(config, weights, max_batch=0)
    with pytest.raises(Unsupported, match="head_dim 64"):
        cuvit.VisionTransformer(config, weights, max_batch=1, precision=cuvit.PRECISION_BF16)
    bad = dict(weights)
    bad["head.bias"] = np.zeros(8, np.float32)
    with pytest.raises(RuntimeError, match="has shape"):
        cuvit.VisionTransformer(config, bad, max_batch=1, precision=cuvit.PRECISION_FP32)


def test_cvw_round_trip_and_rejections():
    rng = np.random.default_rng(0)
    with tempfile.TemporaryDirectory() as tmp:
        path = pathlib.Path(tmp) / "w.cvw"
        writer = cvw.WeightFileWriter()
        a = rng.standard_normal((3, 5)).astype(np.float32)
        b = rng.standard_normal(7).astype(np.float32)
        writer.add("a", (3, 5), a)
        writer.add("b", (7,), b)
        with pytest.raises(ValueError, match="added twice"):
            writer.add("a", (1,), [1.0])
        with pytest.raises(ValueError, match="unsupported rank"):
            writer.add("c", (1, 1, 1, 1, 1), [1.0])
        writer.write(path)
        blob = path.read_bytes()
        assert blob[:4] == b"CVIT"
        loaded = cvw.WeightFile.load(path)
        assert len(loaded) == 2 and "a" in loaded
        np.testing.assert_array_equal(loaded.float_data("a", (3, 5)), a.reshape(-1))
        with pytest.raises(RuntimeError, match="has shape"):
            loaded.float_data("a", (5, 3))
        with pytest.raises(RuntimeError, match="no tensor named"):
            loaded.float_data("z", (1,))
        versioned = bytearray(blob)
        versioned[4] = 2
        path.write_bytes(bytes(versioned))
        with pytest.raises(RuntimeError, match="version 2"):
            cvw.WeightFile.load(path)


def test_preprocess_validation_matches_reference():
    """cuvit_preprocess rejects what cuvit::preprocess rejects (src/runtime/image.cpp:91-99,
    116-119), with its messages, before touching a device; an empty batch is a no-op."""
    def call(batch=1, width=8, height=8, size=4, crop=0.9, stddev=(1.0, 1.0, 1.0)):
        kernels.launch_preprocess(FAKE, FAKE, batch, width, height, size, crop, (0.0, 0.0, 0.0),
                                  stddev)

    call(batch=0)
    cases = [(dict(width=0), "Cannot preprocess an empty image"),
             (dict(height=-1), "Cannot preprocess an empty image"),
             (dict(size=0), "The preprocessing size must be positive"),
             (dict(crop=0.0), "The crop fraction must lie in (0, 1]"),
             (dict(crop=1.01), "The crop fraction must lie in (0, 1]"),
             (dict(crop=float("nan")), "The crop fraction must lie in (0, 1]"),
             (dict(stddev=(1.0, 0.0, 1.0)), "A preprocessing standard deviation cannot be zero"),
             (dict(batch=-1), "The batch cannot be negative")]
    for kwargs, message in cases:
        with pytest.raises(InvalidArgument, match=re.escape(message)):
            call(**kwargs)
    with pytest.raises(InvalidArgument):
        kernels.launch_preprocess(FAKE, FAKE, 2, 8, 8, 4, image_stride=8 * 8 * 3 - 1)
    with pytest.raises(InvalidArgument):
        kernels.launch_preprocess(None, FAKE, 1, 8, 8, 4)
    # The device kernel's own limits (exact float/int conversions below 2^22, 32-bit planes).
    with pytest.raises(LengthError, match="4194304"):
        kernels.launch_preprocess(FAKE, FAKE, 1, 1 << 22, 8, 4)
    with pytest.raises(LengthError, match="46340"):
        kernels.launch_preprocess(FAKE, FAKE, 1, 8, 8, 46341)
    settings = _lib.PreprocessingC()
    _lib.library().cuvit_preprocessing_default(ctypes.byref(settings))
    assert settings.size == 224 and abs(settings.crop_fraction - 0.9) < 1e-7
    assert list(settings.mean) == [0.5] * 3 and list(settings.stddev) == [0.5] * 3


def test_multi_gpu_entry_points_validate_on_the_host():
    """The communicator's id comes from NCCL without a GPU; bad ranks, worlds and buffers are
    rejected before NCCL or a device is touched."""
    from cuvit.replicas import Comm

    first, second = Comm.unique_id(), Comm.unique_id()
    assert len(first) == 128 and first != second
    lib = cuvit.library()
    handle = ctypes.c_void_p(0)
    buffer = ctypes.create_string_buffer(first, 128)
    for world, rank, device in ((0, 0, 0), (2, 2, 0), (2, -1, 0), (1, 0, -1)):
        assert lib.cuvit_comm_create(buffer, world, rank, device,
                                     ctypes.byref(handle)) == _lib.INVALID_ARGUMENT
        assert not handle.value
    assert lib.cuvit_comm_unique_id(buffer, 64) == _lib.INVALID_ARGUMENT
    assert lib.cuvit_gather_logits(None, FAKE, FAKE, 4, 10, 0, None) == _lib.INVALID_ARGUMENT
    assert lib.cuvit_comm_destroy(None) == _lib.OK
    assert lib.cuvit_replicas_destroy(None) == _lib.OK
    assert lib.cuvit_replicas_device_count(None) == 0
    assert lib.cuvit_replicas_forward_host(None, FAKE, FAKE, 1) == _lib.INVALID_ARGUMENT
