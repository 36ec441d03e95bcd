"""TEST INFRASTRUCTURE ONLY: the CPU oracle for Cu-Vit's hot path.

Wraps liboracle.so (cuvit_oracle.c, a C restatement of the reference's CPU algorithms) and,
when built, oracle/_ref/libcuvit_ref_cpu.so / libcuvit_ref_gpu.so (the reference's own CPU
and FP32 GPU code compiled from its sources). Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference legs may import this package; the product never does.
"""

from __future__ import annotations

import ctypes
import pathlib
import subprocess
import threading

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ORACLE_LIB = HERE / "liboracle.so"
REF_CPU_LIB = HERE / "_ref" / "libcuvit_ref_cpu.so"
REF_GPU_LIB = HERE / "_ref" / "libcuvit_ref_gpu.so"

_lock = threading.Lock()
_libs: dict[str, ctypes.CDLL] = {}

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i = ctypes.c_int
_i64 = ctypes.c_int64
_f = ctypes.c_float


def build(reference: bool = False, source=None) -> None:
    """Builds liboracle.so (and, when reference=True, the _ref libraries from the Cu-Vit
    source checkout `source`; the Makefile's default is a checkout beside this repository)."""
    targets = ["oracle"] + (["ref", "ref-tests"] if reference else [])
    extra = [f"REF={source}"] if reference and source is not None else []
    subprocess.run(["make", "-s", "-C", str(HERE), *extra, *targets], check=True)


def _load(path: pathlib.Path, key: str) -> ctypes.CDLL:
    with _lock:
        if key not in _libs:
            if not path.exists():
                raise FileNotFoundError(f"{path} is not built (make -C oracle)")
            _libs[key] = ctypes.CDLL(str(path))
        return _libs[key]


def lib() -> ctypes.CDLL:
    library = _load(ORACLE_LIB, "oracle")
    library.oracle_gemm.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_void_p, _i, _i, _i, _i, _f, _i64, _i64, _i64, _i, _i,
                                    _i64, _i64, _i64, _i64, _i64, _i64, _i, _i]
    library.oracle_gemm_term_magnitudes.argtypes = [_f32p, _f32p, _f32p, _i, _i, _i, _i, _f]
    library.oracle_layer_norm.argtypes = [ctypes.c_void_p, _i64, _f32p, _f32p, ctypes.c_void_p,
                                          _i64, _i, _i, _f]
    library.oracle_softmax.argtypes = [ctypes.c_void_p, ctypes.c_void_p, _i, _i, _i64]
    library.oracle_top_k.argtypes = [_f32p, _i, _i, _i, ctypes.c_void_p, ctypes.c_void_p,
                                     ctypes.c_void_p]
    library.oracle_gelu.restype = _f
    library.oracle_gelu.argtypes = [_f]
    library.oracle_gelu_array.argtypes = [_f32p, _f32p, _i64]
    library.oracle_extract_patches.argtypes = [_f32p, _f32p, _i, _i, _i, _i, _i]
    library.oracle_add.argtypes = [_f32p, _f32p, _i64]
    library.oracle_add_broadcast.argtypes = [_f32p, _f32p, _i64, _i]
    library.oracle_broadcast.argtypes = [_f32p, _f32p, _i64, _i64, _i]
    library.oracle_attention.argtypes = [_f32p, _f32p, _i, _i, _i]
    library.oracle_vit_forward_batch.argtypes = [ctypes.c_void_p, _f, ctypes.c_void_p,
                                                 ctypes.c_void_p, _i, ctypes.c_void_p, _i]
    library.oracle_max_threads.restype = _i
    library.oracle_preprocess.restype = _i
    library.oracle_preprocess.argtypes = [ctypes.c_void_p, _i, _i, _i, _f, _f32p, _f32p, _f32p]
    return library


def _f32(array) -> np.ndarray:
    return np.ascontiguousarray(array, dtype=np.float32)


def gemm(a, b, bias, c, m, n, k, transposed, alpha=1.0, lda=0, ldb=0, ldc=0, count=1, inner=0,
         stride_a=0, stride_b=0, stride_c=0, outer_a=0, outer_b=0, outer_c=0,
         accumulate=False, gelu=False) -> np.ndarray:
    """GemmProblem semantics; returns the new C (c is copied, not modified)."""
    a, b = _f32(a), _f32(b)
    out = _f32(c).copy()
    bias_arr = None if bias is None else _f32(bias)
    lda = lda or k
    ldb = ldb or (k if transposed else n)
    ldc = ldc or n
    lib().oracle_gemm(a.ctypes.data, b.ctypes.data,
                      None if bias_arr is None else bias_arr.ctypes.data, out.ctypes.data, m, n,
                      k, int(transposed), alpha, lda, ldb, ldc, count, inner, stride_a, stride_b,
                      stride_c, outer_a, outer_b, outer_c, int(accumulate), int(gelu))
    return out


def gemm_term_magnitudes(a, b, m, n, k, transposed, alpha=1.0) -> np.ndarray:
    scale = np.empty(m * n, np.float32)
    lib().oracle_gemm_term_magnitudes(_f32(a).reshape(-1), _f32(b).reshape(-1), scale, m, n, k,
                                      int(transposed), alpha)
    return scale


def layer_norm(x, gamma, beta, rows, columns, epsilon=1e-6, in_stride=0) -> np.ndarray:
    x = _f32(x)
    out = np.empty(rows * columns, np.float32)
    lib().oracle_layer_norm(x.ctypes.data, in_stride or columns, _f32(gamma), _f32(beta),
                            out.ctypes.data, columns, rows, columns, epsilon)
    return out


def softmax(x, rows, columns) -> np.ndarray:
    x = _f32(x)
    out = np.empty(rows * columns, np.float32)
    lib().oracle_softmax(x.ctypes.data, out.ctypes.data, rows, columns, columns)
    return out


def top_k(logits, k: int):
    """report_top (src/main.cpp:90-114) per row: (indices int32, logits float32,
    probabilities float64), each [rows, k]; equal logits by ascending class index."""
    logits = _f32(logits)
    rows, classes = logits.shape
    indices = np.empty((rows, k), np.int32)
    values = np.empty((rows, k), np.float32)
    probabilities = np.empty((rows, k), np.float64)
    lib().oracle_top_k(logits.reshape(-1), rows, classes, k, indices.ctypes.data,
                       values.ctypes.data, probabilities.ctypes.data)
    return indices, values, probabilities


def gelu(x) -> np.ndarray:
    x = _f32(x).reshape(-1)
    out = np.empty_like(x)
    lib().oracle_gelu_array(x, out, x.size)
    return out


def extract_patches(images, batch, channels, height, width, patch) -> np.ndarray:
    per_image = (height // patch) * (width // patch)
    out = np.empty(batch * per_image * channels * patch * patch, np.float32)
    lib().oracle_extract_patches(_f32(images).reshape(-1), out, batch, channels, height, width,
                                 patch)
    return out


def add(acc, addend) -> np.ndarray:
    out = _f32(acc).reshape(-1).copy()
    addend = _f32(addend).reshape(-1)
    lib().oracle_add(out, addend, out.size)
    return out


def add_broadcast(acc, addend, count, batch) -> np.ndarray:
    out = _f32(acc).reshape(-1).copy()
    lib().oracle_add_broadcast(out, _f32(addend).reshape(-1), count, batch)
    return out


def broadcast(dst, src, count, stride, batch) -> np.ndarray:
    out = _f32(dst).reshape(-1).copy()
    lib().oracle_broadcast(out, _f32(src).reshape(-1), count, stride, batch)
    return out


def attention(qkv, tokens, embed, heads) -> np.ndarray:
    out = np.empty(tokens * embed, np.float32)
    lib().oracle_attention(_f32(qkv).reshape(-1), out, tokens, embed, heads)
    return out


def config_ints(config) -> np.ndarray:
    return np.array([config.image_size, config.patch_size, config.channels, config.embed_dim,
                     config.depth, config.heads, config.mlp_hidden, config.classes], np.int32)


def vit_forward(config, weights: dict, specs, images, threads: int = 0) -> np.ndarray:
    """Logits [n, classes] of the reference's forward pass (tests/reference/vit.hpp:57-112),
    one image per worker thread. specs: [(name, extents)] in load order."""
    arrays = [_f32(weights[name]).reshape(-1) for name, _ in specs]
    pointers = (ctypes.c_void_p * len(arrays))(*[a.ctypes.data for a in arrays])
    images = _f32(images)
    per_image = config.channels * config.image_size * config.image_size
    count = images.size // per_image
    logits = np.empty((count, config.classes), np.float32)
    ints = config_ints(config)
    failures = lib().oracle_vit_forward_batch(ints.ctypes.data, config.layer_norm_epsilon,
                                              pointers, images.ctypes.data, count,
                                              logits.ctypes.data, threads)
    if failures:
        raise MemoryError(f"oracle forward failed on {failures} images")
    return logits


def preprocess(pixels, size: int = 224, crop_fraction: float = 0.9, mean=(0.5, 0.5, 0.5),
               stddev=(0.5, 0.5, 0.5)) -> np.ndarray:
    """preprocess (src/runtime/image.cpp:90-135) of one interleaved uint8 RGB image [H, W, 3]
    into a planar float32 [3, size, size] tensor."""
    pixels = np.ascontiguousarray(pixels, dtype=np.uint8)
    height, width = pixels.shape[:2]
    out = np.empty(3 * size * size, np.float32)
    status = lib().oracle_preprocess(pixels.ctypes.data, width, height, size, crop_fraction,
                                     _f32(mean), _f32(stddev), out)
    if status != 0:
        raise ValueError("preprocessing arguments rejected")
    return out.reshape(3, size, size)


def ref_preprocess(pixels, size: int = 224, crop_fraction: float = 0.9, mean=(0.5, 0.5, 0.5),
                   stddev=(0.5, 0.5, 0.5)) -> np.ndarray:
    """The reference's own cuvit::preprocess (oracle/_ref), same contract as preprocess()."""
    pixels = np.ascontiguousarray(pixels, dtype=np.uint8)
    height, width = pixels.shape[:2]
    out = np.empty(3 * size * size, np.float32)
    status = ref_cpu().ref_preprocess(pixels.ctypes.data, width, height, size, crop_fraction,
                                      _f32(mean), _f32(stddev), out)
    if status != 0:
        raise ValueError("the reference rejected the preprocessing arguments")
    return out.reshape(3, size, size)


def max_threads() -> int:
    return int(lib().oracle_max_threads())


# ---- the reference's own code (oracle/_ref), when built --------------------------------

def ref_cpu_available() -> bool:
    return REF_CPU_LIB.exists()


def ref_cpu() -> ctypes.CDLL:
    library = _load(REF_CPU_LIB, "ref_cpu")
    library.ref_gemm.argtypes = [_f32p, _f32p, ctypes.c_void_p, _f32p, _i, _i, _i, _i, _f]
    library.ref_gemm_term_magnitudes.argtypes = [_f32p, _f32p, _f32p, _i, _i, _i, _i, _f]
    library.ref_layer_norm.argtypes = [_f32p, _f32p, _f32p, _f32p, _i, _i, _f]
    library.ref_softmax.argtypes = [_f32p, _f32p, _i, _i]
    library.ref_gelu.argtypes = [_f32p, _f32p, _i64]
    library.ref_vit_forward.argtypes = [ctypes.c_char_p, ctypes.c_void_p, _f, ctypes.c_void_p,
                                        _i, ctypes.c_void_p, _i]
    library.ref_vit_forward.restype = _i
    library.ref_preprocess.argtypes = [ctypes.c_void_p, _i, _i, _i, _f, _f32p, _f32p, _f32p]
    library.ref_preprocess.restype = _i
    return library


def ref_vit_forward(weights_path, config, images, threads: int = 0) -> np.ndarray:
    """The reference's VitReference::forward over images, loading a .cvw file."""
    images = _f32(images)
    per_image = config.channels * config.image_size * config.image_size
    count = images.size // per_image
    logits = np.empty((count, config.classes), np.float32)
    ints = config_ints(config)
    if threads <= 0:
        threads = max_threads()
    status = ref_cpu().ref_vit_forward(str(weights_path).encode(), ints.ctypes.data,
                                       config.layer_norm_epsilon, images.ctypes.data, count,
                                       logits.ctypes.data, threads)
    if status != 0:
        raise RuntimeError("the reference's CPU forward pass failed")
    return logits


def ref_gpu_available() -> bool:
    return REF_GPU_LIB.exists()


def ref_gpu() -> ctypes.CDLL:
    library = _load(REF_GPU_LIB, "ref_gpu")
    library.ref_gpu_gemm.argtypes = [ctypes.c_void_p] * 4 + [_i, _i, _i, _i, _f, _i, _i]
    library.ref_gpu_gemm.restype = _i
    library.ref_gpu_gemm_async.argtypes = [ctypes.c_void_p] * 4 + [_i, _i, _i, _i, _f, _i, _i,
                                                                  ctypes.c_void_p]
    library.ref_gpu_gemm_async.restype = _i
    library.ref_gpu_vit_create.argtypes = [ctypes.c_char_p, ctypes.c_void_p, _f, _i]
    library.ref_gpu_vit_create.restype = ctypes.c_void_p
    library.ref_gpu_vit_forward.argtypes = [ctypes.c_void_p] * 3 + [_i, ctypes.c_void_p]
    library.ref_gpu_vit_forward.restype = _i
    library.ref_gpu_vit_destroy.argtypes = [ctypes.c_void_p]
    return library


class RefGpuModel:
    """The reference's own VisionTransformer (FP32 GPU path, oracle/_ref/libcuvit_ref_gpu.so)
    for `config` and host `weights`, loaded through a temporary .cvw file. forward() takes
    device pointers (integers) and runs on `stream` (a cudaStream_t as an integer, 0 for the
    legacy default stream)."""

    def __init__(self, config, weights: dict, specs, max_batch: int):
        import tempfile

        from cuvit import cvw

        self.config = config
        with tempfile.TemporaryDirectory() as tmp:
            path = pathlib.Path(tmp) / "weights.cvw"
            writer = cvw.WeightFileWriter()
            for name, extents in specs:
                writer.add(name, extents, weights[name])
            writer.write(path)
            ints = config_ints(config)
            self._handle = ref_gpu().ref_gpu_vit_create(str(path).encode(), ints.ctypes.data,
                                                        config.layer_norm_epsilon, max_batch)
        if not self._handle:
            raise RuntimeError("the reference's VisionTransformer could not be created")

    def forward(self, images_ptr: int, logits_ptr: int, batch: int, stream: int = 0) -> None:
        status = ref_gpu().ref_gpu_vit_forward(self._handle, ctypes.c_void_p(images_ptr),
                                               ctypes.c_void_p(logits_ptr), batch,
                                               ctypes.c_void_p(stream or None))
        if status != 0:
            raise RuntimeError("the reference's GPU forward pass failed")

    def close(self) -> None:
        if self._handle:
            ref_gpu().ref_gpu_vit_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown
            pass

