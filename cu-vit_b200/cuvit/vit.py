"""VitConfig and VisionTransformer over the C ABI (reference: include/cuvit/vit.hpp)."""

from __future__ import annotations

import ctypes
import dataclasses

import numpy as np

from . import _lib
from .errors import InvalidArgument, check
from .kernels import _ptr, _stream

PRECISION_FP32 = _lib.MATH_FP32
PRECISION_TF32 = _lib.MATH_TF32
PRECISION_BF16 = _lib.MATH_BF16


@dataclasses.dataclass
class VitConfig:
    """Shape of a ViT; defaults describe ViT-Tiny/16 at 224x224 (vit.hpp:15-35)."""

    image_size: int = 224
    patch_size: int = 16
    channels: int = 3
    embed_dim: int = 192
    depth: int = 12
    heads: int = 3
    mlp_hidden: int = 768
    classes: int = 1000
    layer_norm_epsilon: float = 1.0e-6

    def patches_per_side(self) -> int:
        return self.image_size // self.patch_size

    def patch_count(self) -> int:
        return self.patches_per_side() ** 2

    def token_count(self) -> int:
        return self.patch_count() + 1

    def head_dim(self) -> int:
        return self.embed_dim // self.heads

    def patch_elements(self) -> int:
        return self.channels * self.patch_size * self.patch_size

    def image_elements(self) -> int:
        return self.channels * self.image_size * self.image_size

    def to_c(self) -> _lib.VitConfigC:
        return _lib.VitConfigC(self.image_size, self.patch_size, self.channels, self.embed_dim,
                               self.depth, self.heads, self.mlp_hidden, self.classes,
                               self.layer_norm_epsilon)

    def validate(self) -> None:
        """reference: VitConfig::validate (src/model/vit.cu:36-47)."""
        config = self.to_c()
        check(_lib.library().cuvit_vit_config_validate(ctypes.byref(config)))

    def gflop_per_image(self) -> float:
        """Algorithmic FLOPs of one forward pass (2 per multiply-add)."""
        e, t, p, f = self.embed_dim, self.token_count(), self.patch_count(), self.mlp_hidden
        per_block = 2 * t * e * 3 * e + 4 * t * t * e + 2 * t * e * e + 4 * t * e * f
        return (2 * p * self.patch_elements() * e + self.depth * per_block +
                2 * e * self.classes) / 1e9


def tensor_specs(config: VitConfig) -> list[tuple[str, tuple[int, ...]]]:
    """timm tensor names and extents in load order (reference: vit.cu:49-63, 114-143)."""
    e, t, f = config.embed_dim, config.token_count(), config.mlp_hidden
    specs = [
        ("cls_token", (1, 1, e)),
        ("pos_embed", (1, t, e)),
        ("patch_embed.proj.weight", (e, config.channels, config.patch_size, config.patch_size)),
        ("patch_embed.proj.bias", (e,)),
    ]
    for i in range(config.depth):
        prefix = f"blocks.{i}."
        specs += [
            (prefix + "norm1.weight", (e,)), (prefix + "norm1.bias", (e,)),
            (prefix + "attn.qkv.weight", (3 * e, e)), (prefix + "attn.qkv.bias", (3 * e,)),
            (prefix + "attn.proj.weight", (e, e)), (prefix + "attn.proj.bias", (e,)),
            (prefix + "norm2.weight", (e,)), (prefix + "norm2.bias", (e,)),
            (prefix + "mlp.fc1.weight", (f, e)), (prefix + "mlp.fc1.bias", (f,)),
            (prefix + "mlp.fc2.weight", (e, f)), (prefix + "mlp.fc2.bias", (e,)),
        ]
    specs += [("norm.weight", (e,)), ("norm.bias", (e,)),
              ("head.weight", (config.classes, e)), ("head.bias", (config.classes,))]
    return specs


def random_weights(config: VitConfig, seed: int, std: float = 0.02) -> dict[str, np.ndarray]:
    """Random-init weights as the benchmark configurations specify: matrices, class token and
    position embedding ~ truncated normal (std, cut at +-2 std), LN gamma = 1, beta = 0,
    biases 0."""
    rng = np.random.default_rng(seed)
    weights = {}
    for name, extents in tensor_specs(config):
        count = int(np.prod(extents))
        if name.endswith("norm1.weight") or name.endswith("norm2.weight") or name == "norm.weight":
            values = np.ones(count, np.float32)
        elif name.endswith(".bias"):
            values = np.zeros(count, np.float32)
        else:
            values = rng.standard_normal(count).astype(np.float32)
            bad = np.abs(values) > 2.0
            while bad.any():
                values[bad] = rng.standard_normal(int(bad.sum())).astype(np.float32)
                bad = np.abs(values) > 2.0
            values *= np.float32(std)
        weights[name] = values.reshape(extents)
    return weights


def host_tensors(config: VitConfig, weights) -> list[np.ndarray]:
    """The model's tensors as contiguous float32 arrays in load order, from a dict name ->
    array or a cvw.WeightFile; names and shapes are checked against config."""
    arrays = []
    for name, extents in tensor_specs(config):
        if hasattr(weights, "float_data"):
            data = weights.float_data(name, extents)
        else:
            if name not in weights:
                raise RuntimeError(f"Weight file has no tensor named '{name}'")
            data = np.asarray(weights[name], dtype=np.float32)
            if tuple(data.shape) != tuple(extents):
                raise RuntimeError(f"Tensor '{name}' has shape {list(data.shape)}, but "
                                   f"{list(extents)} was expected")
        arrays.append(np.ascontiguousarray(data, dtype=np.float32))
    return arrays


class VisionTransformer:
    """reference: cuvit::VisionTransformer (include/cuvit/vit.hpp:63-120).

    weights: a dict name -> array, or a cvw.WeightFile; shapes are checked against config.
    precision: PRECISION_FP32 (FP32-faithful), PRECISION_TF32 or PRECISION_BF16.
    """

    def __init__(self, config: VitConfig, weights, max_batch: int = 1,
                 precision: int = PRECISION_BF16, device: int = 0):
        self.config = config
        lib = _lib.library()
        c_config = config.to_c()
        check(lib.cuvit_vit_config_validate(ctypes.byref(c_config)))
        arrays = host_tensors(config, weights)
        pointers = (ctypes.c_void_p * len(arrays))(*[a.ctypes.data for a in arrays])
        handle = ctypes.c_void_p(0)
        check(lib.cuvit_vit_create_from_host(ctypes.byref(c_config), pointers, len(arrays),
                                             max_batch, precision, device, ctypes.byref(handle)))
        self._handle = handle
        self.precision = precision
        self.device = device

    @classmethod
    def from_file(cls, config: VitConfig, path, max_batch: int = 1,
                  precision: int = PRECISION_BF16, device: int = 0) -> "VisionTransformer":
        """Loads a .cvw file in C++ (reference: WeightFile::load + constructor)."""
        self = cls.__new__(cls)
        self.config = config
        lib = _lib.library()
        c_config = config.to_c()
        handle = ctypes.c_void_p(0)
        check(lib.cuvit_vit_create_from_file(ctypes.byref(c_config), str(path).encode(),
                                             max_batch, precision, device,
                                             ctypes.byref(handle)))
        self._handle = handle
        self.precision = precision
        self.device = device
        return self

    def close(self) -> None:
        if getattr(self, "_handle", None) and self._handle.value:
            _lib.library().cuvit_vit_destroy(self._handle)
            self._handle = ctypes.c_void_p(0)

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass

    def forward(self, images, logits, batch: int, stream=None) -> None:
        """Device pointers in, device logits out; queued on stream (vit.hpp:80-87)."""
        check(_lib.library().cuvit_vit_forward(self._handle, _ptr(images), _ptr(logits), batch,
                                               _stream(stream)))

    def forward_graph(self, images, logits, batch: int, stream=None) -> None:
        """forward() replayed from a CUDA graph captured on first use for these pointers."""
        check(_lib.library().cuvit_vit_forward_graph(self._handle, _ptr(images), _ptr(logits),
                                                     batch, _stream(stream)))

    def forward_host(self, images: np.ndarray, stream=None) -> np.ndarray:
        """Host array in, host logits out, synchronised (vit.hpp:89-91)."""
        per_image = self.image_elements()
        flat = np.ascontiguousarray(images, dtype=np.float32).reshape(-1)
        if per_image == 0 or flat.size % per_image != 0:
            raise InvalidArgument(_lib.INVALID_ARGUMENT,
                                  f"The input holds {flat.size} elements, which is not a whole "
                                  f"number of {per_image}-element images")
        batch = flat.size // per_image
        if batch > self.max_batch:
            raise InvalidArgument(_lib.INVALID_ARGUMENT,
                                  f"This model was built for at most {self.max_batch} images, "
                                  f"but {batch} were given")
        logits = np.empty((batch, self.config.classes), np.float32)
        check(_lib.library().cuvit_vit_forward_host(self._handle, flat.ctypes.data,
                                                    logits.ctypes.data, batch, _stream(stream)))
        return logits

    def forward_host_ptr(self, images_ptr: int, logits_ptr: int, batch: int, stream=None) -> None:
        """forward_host() on caller-owned (e.g. pinned) host buffers given as addresses."""
        check(_lib.library().cuvit_vit_forward_host(self._handle, ctypes.c_void_p(images_ptr),
                                                    ctypes.c_void_p(logits_ptr), batch,
                                                    _stream(stream)))

    def forward_host_async(self, images_ptr: int, logits_ptr: int, batch: int,
                           stream=None) -> None:
        """Queues copy-in, pass and copy-out on caller-owned pinned host buffers and returns;
        the copy of the next call overlaps this call's pass. Results are valid once `stream`
        has been synchronised."""
        check(_lib.library().cuvit_vit_forward_host_async(
            self._handle, ctypes.c_void_p(images_ptr), ctypes.c_void_p(logits_ptr), batch,
            _stream(stream)))

    def set_host_chunk(self, images: int) -> None:
        """Images per forward_host() chunk (copy of chunk i+1 overlaps chunk i); 0 = automatic."""
        check(_lib.library().cuvit_vit_set_host_chunk(self._handle, images))

    def forward_profiled(self, images, logits, batch: int, stream=None) -> list[dict]:
        """forward() with CUDA events around every launch; returns one record per launch:
        kind, layer, algorithmic flops and bytes, and device milliseconds."""
        capacity = self.launches_per_forward(batch) + 8
        records = (_lib.LaunchRecordC * capacity)()
        count = ctypes.c_int(0)
        check(_lib.library().cuvit_vit_forward_profiled(self._handle, _ptr(images), _ptr(logits),
                                                        batch, _stream(stream), records,
                                                        capacity, ctypes.byref(count)))
        return [{"kind": _lib.LAUNCH_KINDS[r.kind], "layer": r.layer, "flops": r.flops,
                 "bytes": r.bytes, "ms": r.milliseconds} for r in records[:count.value]]

    @property
    def max_batch(self) -> int:
        return _lib.library().cuvit_vit_max_batch(self._handle)

    def image_elements(self) -> int:
        return int(_lib.library().cuvit_vit_image_elements(self._handle))

    def host_image_bytes(self) -> int:
        """Bytes per image that forward_host_async moves host -> device: 2 per element where
        the model rounds images to bfloat16 on the host (BF16 models created with
        CUVIT_HOST_ROUNDING=1), else 4."""
        return int(_lib.library().cuvit_vit_host_image_bytes(self._handle))

    def weight_bytes(self) -> int:
        return int(_lib.library().cuvit_vit_weight_bytes(self._handle))

    def activation_bytes(self) -> int:
        return int(_lib.library().cuvit_vit_activation_bytes(self._handle))

    def launches_per_forward(self, batch: int) -> int:
        return int(_lib.library().cuvit_vit_launches_per_forward(self._handle, batch))

    @staticmethod
    def expected_tensor_names(config: VitConfig) -> list[str]:
        return [name for name, _ in tensor_specs(config)]
