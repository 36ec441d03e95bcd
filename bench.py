#!/usr/bin/env python
"""ViT forward-pass throughput on B200, one process per GPU (by default the headline
benchmark configuration: ViT-B/16, BF16, batch 256 per GPU, logits gathered to rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config vit-b|vit-s|vit-ti|vit-l]

Under torchrun (N > 1) every rank runs its own replica on its own batch shard; the only
collective is the per-step gather of the logits to rank 0 (NCCL). A step is one forward
pass over one batch. Rank 0 prints one JSON line.

  value   images/s over all ranks, inputs resident in HBM, CUDA-graph replay, timed with CUDA
          events on the launching stream, max over ranks
  e2e     the same through the public host-buffer call (VisionTransformer.forward_host_async,
          the serving-loop form of forward_host): every step copies its pinned host images to
          the device, runs the pass and copies the logits back to pinned host memory; the copy
          of step i+1 overlaps the pass of step i, and the timed region ends when the last
          step's logits are on the host
  roofline  the tcgen05 GEMMs (the dominant kernel): algorithmic FLOPs / device time of every
          GEMM launch, from CUDA events around each launch over profiled passes
  cpu_baseline  the reference's own CPU forward pass (oracle/_ref, compiled from its sources)
          on this host's cores, one image per core, rank 0 at N = 1

--impl reference times that CPU implementation alone (rank 0; other ranks exit).
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "cu-vit_b200"))

import numpy as np  # noqa: E402

METRIC = "ViT-B/16 images/s at 1/2/4/8 B200; batched-GEMM % of tensor-core peak"

CONFIGS = {
    # name: (model label, VitConfig kwargs, batch per GPU, precision, seed)
    "vit-b": ("ViT-B/16", dict(embed_dim=768, heads=12, mlp_hidden=3072), 256, "bf16", 3),
    "vit-s": ("ViT-S/16", dict(embed_dim=384, heads=6, mlp_hidden=1536), 128, "bf16", 2),
    "vit-ti": ("ViT-Ti/16", dict(), 32, "tf32", 1),
    "vit-l": ("ViT-L/16", dict(embed_dim=1024, depth=24, heads=16, mlp_hidden=4096), 128,
              "bf16", 4),
}

# Measurements beside the headline on one GPU (all by default).
EXTRAS = ("configs", "single_gemms", "fp32_baselines", "preprocess")

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse_args():
    parser = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=50)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--config", choices=sorted(CONFIGS), default="vit-b")
    parser.add_argument("--precision", choices=["bf16", "tf32", "fp32"], default=None,
                        help="override the configuration's precision (profiling runs)")
    parser.add_argument("--profile-passes", type=int, default=5)
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--timeline", action="store_true",
                        help="device timeline of one graph-replayed pass (instrumented build)")
    parser.add_argument("--no-extras", action="store_true",
                        help="skip the other configurations, single GEMMs and FP32 baselines")
    parser.add_argument("--extra", action="append", choices=EXTRAS, default=None,
                        help="run only the named extra measurements (repeatable; profiling runs)")
    return parser.parse_args()


def peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons, every 100 ms, with timestamps."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.samples: list[tuple[float, list[str]]] = []
        self._process = None
        self._thread = None

    def start(self) -> None:
        try:
            self._process = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self._process = None
            return
        self._thread = threading.Thread(target=self._read, daemon=True)
        self._thread.start()

    def _read(self) -> None:
        for line in self._process.stdout:
            self.samples.append((time.monotonic(), [f.strip() for f in line.split(",")]))

    def stop(self) -> None:
        if self._process is not None:
            self._process.terminate()
            try:
                self._process.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._process.kill()
        if self._thread is not None:
            self._thread.join(timeout=5)

    def summary(self, start: float, end: float) -> dict:
        window = [s for t, s in self.samples if start <= t <= end]
        if len(window) < 3:  # short timed region: widen into the warm-up, same load
            window = [s for t, s in self.samples if start - 2.0 <= t <= end]
        if not window:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({name for s in window for name, value in zip(names, s[5:9])
                          if value.lower().startswith("active")})

        def number(text):
            try:
                return float(text)
            except ValueError:
                return None

        sm = [number(s[1]) for s in window if number(s[1]) is not None]
        power = [number(s[3]) for s in window if number(s[3]) is not None]
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": number(window[0][2]), "reasons": reasons,
                "power_w_median": statistics.median(power) if power else None,
                "samples": len(window)}


def write_cvw(config, weights, path) -> None:
    from cuvit import cvw
    from cuvit.vit import tensor_specs

    writer = cvw.WeightFileWriter()
    for name, extents in tensor_specs(config):
        writer.add(name, extents, weights[name])
    writer.write(path)


def cpu_model() -> str:
    """The host CPU's model name (from /proc/cpuinfo), for the CPU baseline's record."""
    try:
        for line in pathlib.Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_reference_step(config, weights_path, images, threads):
    """One bounded sample of the workload through the reference's CPU code: returns
    (seconds, images, kind)."""
    import oracle

    start = time.perf_counter()
    if oracle.ref_cpu_available():
        oracle.ref_vit_forward(weights_path, config, images, threads=threads)
        kind = "reference"
    else:
        raise RuntimeError("oracle/_ref/libcuvit_ref_cpu.so is not built")
    return time.perf_counter() - start, images.size // config.image_elements(), kind


def reference_arm(args) -> None:
    """Times the reference's own CPU implementation (oracle/_ref) on this host's cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from cuvit.vit import VitConfig, random_weights

    label, kwargs, batch, precision, seed = CONFIGS[args.config]
    config = VitConfig(**kwargs)
    threads = os.cpu_count() or 1
    weights = random_weights(config, seed)
    rng = np.random.default_rng([seed, 0])
    # A step is one image through VitReference::forward (single-threaded, ~10 s for ViT-B).
    # Steps run `threads` at a time, one per host thread, in whole rounds so that no thread
    # idles in a partial round: the K timed steps become the nearest whole number of rounds
    # (at least one), the warm-up one round of min(W, threads) images.
    rounds = max(1, round(args.steps / threads))
    timed = rounds * threads
    images = rng.standard_normal(timed * config.image_elements()).astype(np.float32)
    with tempfile.TemporaryDirectory() as tmp:
        path = pathlib.Path(tmp) / "weights.cvw"
        write_cvw(config, weights, path)
        if args.warmup > 0:
            warm = min(args.warmup, threads)
            cpu_reference_step(config, path, images[:warm * config.image_elements()], threads)
        total, count, kind = cpu_reference_step(config, path, images, threads)
    value = count / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "images/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * total / count, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic N(0,1) images, random-init trunc-normal(0.02) weights",
        "config": {"workload": f"{label} forward, reference CPU implementation (FP32)",
                   "model": label, "seq_len": config.token_count()},
        "cpu_baseline": {"value": value, "unit": "images/s", "cores": threads, "kind": kind,
                         "cpu": cpu_model(),
                         "sample": f"{count} images in {rounds} rounds of {threads}, one per "
                                   "host thread, VitReference::forward "
                                   "(tests/reference/vit.hpp)"},
        "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def profile_pass_kinds(model, images, logits, batch, stream, passes: int) -> dict:
    """Per launch kind, the median over `passes` profiled passes (CUDA events around every
    launch, after one discarded pass) of launches, ms, FLOPs and bytes per pass."""
    model.forward_profiled(images, logits, batch, stream)
    per_pass: list[dict[str, dict]] = []
    for _ in range(max(passes, 1)):
        kinds: dict[str, dict] = {}
        for r in model.forward_profiled(images, logits, batch, stream):
            entry = kinds.setdefault(r["kind"], {"launches": 0, "ms": 0.0, "flops": 0.0,
                                                 "bytes": 0.0})
            entry["launches"] += 1
            entry["ms"] += r["ms"]
            entry["flops"] += r["flops"]
            entry["bytes"] += r["bytes"]
        per_pass.append(kinds)
    by_kind = {}
    for kind in per_pass[0]:
        times = sorted(k[kind]["ms"] for k in per_pass)
        by_kind[kind] = dict(per_pass[0][kind], ms=times[len(times) // 2])
    return by_kind


def gemm_summary(by_kind: dict) -> tuple[float, float, int]:
    """(GEMM FLOPs, GEMM ms, GEMM launches) of one pass."""
    gemm = [e for k, e in by_kind.items() if k.startswith("gemm")]
    return (sum(e["flops"] for e in gemm), sum(e["ms"] for e in gemm),
            sum(e["launches"] for e in gemm))


def event_ms(torch, stream, fn, repeats: int) -> float:
    """Mean device milliseconds of fn() over `repeats` back-to-back calls on `stream`."""
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(repeats):
        fn()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) / repeats


def measure_tf32_peak(torch, device) -> float:
    """Dense TF32 tensor-core throughput of torch.matmul (cuBLAS) at 8192^3, best of 10,
    CUDA events: the denominator of the TF32 configuration's roofline."""
    previous = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    a = torch.randn(8192, 8192, device=device)
    b = torch.randn(8192, 8192, device=device)
    stream = torch.cuda.current_stream(device)
    torch.matmul(a, b)
    best = min(event_ms(torch, stream, lambda: torch.matmul(a, b), 1) for _ in range(10))
    torch.backends.cuda.matmul.allow_tf32 = previous
    del a, b
    return 2 * 8192 ** 3 / (best * 1e-3) / 1e12


def measure_other_configs(torch, device, peak_bf16: float, peak_tf32: float) -> dict:
    """The benchmark configurations other than the headline one, each on one GPU with its own
    model: images/s over 20 graph replays (inputs resident), GEMM TFLOP/s from 3 profiled
    passes, and that as a fraction of the measured tensor peak of its precision."""
    import cuvit
    from cuvit.vit import PRECISION_BF16, PRECISION_TF32, VisionTransformer, VitConfig, random_weights

    results = {}
    stream = torch.cuda.current_stream(device)
    for name in ("vit-ti", "vit-s", "vit-l"):
        label, kwargs, batch, precision_name, seed = CONFIGS[name]
        config = VitConfig(**kwargs)
        precision = PRECISION_BF16 if precision_name == "bf16" else PRECISION_TF32
        model = VisionTransformer(config, random_weights(config, seed), max_batch=batch,
                                  precision=precision, device=device.index)
        rng = np.random.default_rng([seed, 0])
        images = torch.from_numpy(rng.standard_normal(batch * config.image_elements())
                                  .astype(np.float32)).to(device)
        logits = torch.zeros(batch, config.classes, device=device)
        for _ in range(5):
            model.forward_graph(images, logits, batch, stream)
        ms = event_ms(torch, stream, lambda: model.forward_graph(images, logits, batch, stream),
                      20)
        flops, gemm_ms, _ = gemm_summary(profile_pass_kinds(model, images, logits, batch,
                                                            stream, 3))
        cuvit.kernels.device_status()  # raises if any kernel gave up on a bounded wait
        peak = peak_bf16 if precision == PRECISION_BF16 else peak_tf32
        tflops = flops / (gemm_ms * 1e-3) / 1e12
        results[name] = {
            "workload": f"{label} {precision_name.upper()}, batch {batch}", "batch": batch,
            "images_per_s": batch / (ms * 1e-3), "ms_per_pass": ms,
            "gemm_tflops": tflops, "gemm_frac": tflops / peak,
            "peak": peak, "peak_kind": ("measured bf16 burst (MEASURED_PEAKS.json)"
                                        if precision == PRECISION_BF16 else
                                        "measured tf32 burst (torch.matmul 8192^3, this run)"),
            "pass_tflops": batch * config.gflop_per_image() / ms,
        }
        model.close()
        del images, logits
    return results


def measure_single_gemms(torch, device, peak_tf32: float) -> dict:
    """the three single FP32 GEMMs of ViT-Tiny (QKV shape without
    epilogue, FC1 shape with GELU, FC2 shape accumulating), A, B, bias ~ U(-1, 1) from seed 0,
    through launch_gemm in the FP32-faithful (3xTF32) and TF32 modes. Mean device time per
    launch over 100 launches captured in one CUDA graph (so host call overhead does not
    appear), 5 replays; each launch is one wave or less, so this is a latency figure."""
    import oracle
    from cuvit import kernels

    ref = oracle.ref_gpu() if oracle.ref_gpu_available() else None
    stream = torch.cuda.current_stream(device)
    rng = np.random.default_rng(0)
    shapes = [("qkv", 197, 576, 192, False, False), ("fc1_gelu", 197, 768, 192, True, False),
              ("fc2_accumulate", 197, 192, 768, False, True)]
    results = {}
    previous = kernels.get_math_mode()
    for math_name, math in (("fp32", kernels.MATH_FP32), ("tf32", kernels.MATH_TF32)):
        kernels.set_math_mode(math)
        for name, m, n, k, gelu, accumulate in shapes:
            a = torch.from_numpy(rng.uniform(-1, 1, m * k).astype(np.float32)).to(device)
            b = torch.from_numpy(rng.uniform(-1, 1, n * k).astype(np.float32)).to(device)
            bias = torch.from_numpy(rng.uniform(-1, 1, n).astype(np.float32)).to(device)
            c = torch.zeros(m * n, device=device)
            problem = kernels.gemm_problem(m, n, k, kernels.LAYOUT_TRANSPOSED)
            problem.epilogue.gelu = int(gelu)
            problem.epilogue.accumulate = int(accumulate)

            side = torch.cuda.Stream(device)
            side.wait_stream(stream)
            with torch.cuda.stream(side):
                for _ in range(3):  # one-time set-up happens outside the capture
                    kernels.launch_gemm(a, b, bias, c, problem, side)
            stream.wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                for _ in range(100):
                    kernels.launch_gemm(a, b, bias, c, problem, side)
            graph.replay()
            ms = event_ms(torch, stream, graph.replay, 5) / 100
            del graph
            flops = 2.0 * m * n * k
            results[f"{name}_{math_name}"] = {
                "m": m, "n": n, "k": k, "us_per_launch": ms * 1e3,
                "tflops": flops / (ms * 1e-3) / 1e12,
                "frac_of_tf32_peak": flops / (ms * 1e-3) / 1e12 / peak_tf32}
            if math_name == "fp32" and ref is not None:
                # The reference's own launch_gemm (SIMT FP32, src/kernels/gemm.cu) on the same
                # operands, captured and timed the same way.
                def ref_launch():
                    status = ref.ref_gpu_gemm_async(a.data_ptr(), b.data_ptr(), bias.data_ptr(),
                                                    c.data_ptr(), m, n, k, 1, 1.0,
                                                    int(accumulate), int(gelu), side.cuda_stream)
                    assert status == 0

                with torch.cuda.stream(side):
                    for _ in range(3):
                        ref_launch()
                stream.wait_stream(side)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=side):
                    for _ in range(100):
                        ref_launch()
                graph.replay()
                ms_ref = event_ms(torch, stream, graph.replay, 5) / 100
                del graph
                results[f"{name}_reference_fp32_gpu"] = {
                    "m": m, "n": n, "k": k, "us_per_launch": ms_ref * 1e3,
                    "tflops": flops / (ms_ref * 1e-3) / 1e12}
    kernels.set_math_mode(previous)
    kernels.device_status()
    return results


def measure_preprocess(torch, device) -> dict:
    """Image preprocessing (the input pipeline): 256 interleaved 8-bit RGB images of 500 x 375
    pixels to the ViT-B input tensor (resize of the shorter side to 248, centre crop 224,
    normalisation) by cuvit_preprocess on the device, 20 launches timed with CUDA events,
    against the reference's host preprocess (src/runtime/image.cpp:90-135, compiled into
    oracle/_ref) on one image per host thread over a sample of 2 x threads images."""
    import concurrent.futures

    import oracle
    from cuvit import kernels

    batch, height, width, size = 256, 375, 500, 224
    rng = np.random.default_rng(17)
    pixels = rng.integers(0, 256, (batch, height, width, 3), dtype=np.uint8)
    d_pixels = torch.from_numpy(pixels.reshape(batch, -1)).to(device)
    out = torch.empty((batch, 3, size, size), device=device)
    stream = torch.cuda.current_stream(device)

    def launch():
        kernels.launch_preprocess(d_pixels, out, batch, width, height, size, 0.9, stream=stream)

    for _ in range(3):
        launch()
    ms = event_ms(torch, stream, launch, 20)
    kernels.device_status()
    moved = pixels.nbytes + out.numel() * 4
    result = {"workload": f"{batch} RGB images {width}x{height} -> 3x{size}x{size} FP32",
              "us_per_batch": ms * 1e3, "images_per_s": batch / (ms * 1e-3),
              "gbs": moved / (ms * 1e-3) / 1e9}
    if oracle.ref_cpu_available():
        threads = os.cpu_count() or 1
        sample = pixels[: min(batch, 2 * threads)]
        start = time.perf_counter()
        with concurrent.futures.ThreadPoolExecutor(threads) as pool:
            list(pool.map(lambda p: oracle.ref_preprocess(p, size, 0.9), sample))
        seconds = time.perf_counter() - start
        result["reference_host"] = {"images_per_s": len(sample) / seconds, "threads": threads,
                                    "kind": "reference (oracle/_ref, cuvit::preprocess)"}
    return result


def measure_fp32_baselines(torch, device) -> dict:
    """ViT-B/16 at batch 256 in FP32 on one GPU: the reference's own FP32 GPU path
    (src/model/vit.cu built for sm_100a into oracle/_ref; a second baseline, never the
    product) beside this library's FP32-faithful mode (3xTF32 tensor cores, the reference's
    unfused attention steps)."""
    import oracle
    import cuvit
    from cuvit.vit import PRECISION_FP32, VisionTransformer, VitConfig, random_weights, tensor_specs

    label, kwargs, batch, _, seed = CONFIGS["vit-b"]
    config = VitConfig(**kwargs)
    weights = random_weights(config, seed)
    stream = torch.cuda.current_stream(device)
    rng = np.random.default_rng([seed, 0])
    images = torch.from_numpy(rng.standard_normal(batch * config.image_elements())
                              .astype(np.float32)).to(device)
    logits = torch.zeros(batch, config.classes, device=device)
    results = {"workload": f"{label} FP32, batch {batch}"}
    ours = VisionTransformer(config, weights, max_batch=batch, precision=PRECISION_FP32,
                             device=device.index)
    for _ in range(2):
        ours.forward_graph(images, logits, batch, stream)
    ms = event_ms(torch, stream, lambda: ours.forward_graph(images, logits, batch, stream), 3)
    cuvit.kernels.device_status()
    ours.close()
    results["ours_fp32_faithful"] = {"images_per_s": batch / (ms * 1e-3), "ms_per_pass": ms}
    del images, logits
    if not oracle.ref_gpu_available():
        results["reference_fp32_gpu"] = None
        return results
    # The reference's FP32 GPU path on every model configuration at its batch (one GPU).
    results["reference_fp32_gpu"] = {}
    for name in ("vit-ti", "vit-s", "vit-b", "vit-l"):
        ref_label, ref_kwargs, ref_batch, _, ref_seed = CONFIGS[name]
        ref_config = VitConfig(**ref_kwargs)
        ref_weights = weights if name == "vit-b" else random_weights(ref_config, ref_seed)
        ref_rng = np.random.default_rng([ref_seed, 0])
        ref_images = torch.from_numpy(ref_rng.standard_normal(
            ref_batch * ref_config.image_elements()).astype(np.float32)).to(device)
        ref_logits = torch.zeros(ref_batch, ref_config.classes, device=device)
        ref = oracle.RefGpuModel(ref_config, ref_weights, tensor_specs(ref_config), ref_batch)
        handle = stream.cuda_stream

        def ref_pass():
            ref.forward(ref_images.data_ptr(), ref_logits.data_ptr(), ref_batch, handle)

        ref_pass()
        ms_ref = event_ms(torch, stream, ref_pass, 3)
        ref.close()
        results["reference_fp32_gpu"][name] = {
            "workload": f"{ref_label} FP32, batch {ref_batch}",
            "images_per_s": ref_batch / (ms_ref * 1e-3), "ms_per_pass": ms_ref,
            "kind": "reference (oracle/_ref/libcuvit_ref_gpu.so)"}
        if name == "vit-b":
            results["ratio_ours_over_reference"] = ms_ref / ms
        del ref_images, ref_logits
    return results


def our_arm(args) -> None:
    import torch
    import torch.distributed as dist

    import cuvit
    from cuvit.replicas import Comm, bind_to_gpu_cpus
    from cuvit.vit import (PRECISION_BF16, PRECISION_FP32, PRECISION_TF32, VisionTransformer,
                           VitConfig, random_weights)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        # Each rank on its GPU's NUMA node, so its pinned images feed the copy engine from
        # local memory (N = 1 keeps every core: the CPU baseline runs there).
        bind_to_gpu_cpus(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=device)

    label, kwargs, batch, precision_name, seed = CONFIGS[args.config]
    precision_name = args.precision or precision_name
    config = VitConfig(**kwargs)
    precision = {"bf16": PRECISION_BF16, "tf32": PRECISION_TF32,
                 "fp32": PRECISION_FP32}[precision_name]
    weights = random_weights(config, seed)
    model = VisionTransformer(config, weights, max_batch=batch, precision=precision,
                              device=local_rank)
    rng = np.random.default_rng([seed, rank])
    host_images = rng.standard_normal(batch * config.image_elements()).astype(np.float32)
    images = torch.from_numpy(host_images).to(device)
    logits = torch.zeros(batch, config.classes, device=device)
    stream = torch.cuda.current_stream(device)
    # N > 1: the logits gather goes through the library's own NCCL communicator (C ABI);
    # torch.distributed only hands the communicator's unique id around and keeps the
    # barriers and the max-over-ranks timing.
    comm = None
    gathered = None
    if world > 1:
        unique = [Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(unique, src=0)
        comm = Comm(unique[0], world, rank, local_rank)
        if rank == 0:
            gathered = torch.zeros(world * batch, config.classes, device=device)

    def gather(local, on_stream):
        if comm is not None:  # the path's only collective
            comm.gather_logits(local, gathered, batch, config.classes, 0, on_stream)

    def step():
        model.forward_graph(images, logits, batch, stream)
        gather(logits, stream)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(device)

    def max_over_ranks(value: float) -> float:
        if world == 1:
            return value
        t = torch.tensor([value], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    sampler = ClockSampler(local_rank)
    sampler.start()
    for _ in range(args.warmup):
        step()
    barrier()
    launches_before = cuvit.kernels.launch_count()
    start_event = torch.cuda.Event(enable_timing=True)
    end_event = torch.cuda.Event(enable_timing=True)
    t0 = time.monotonic()
    start_event.record(stream)
    for _ in range(args.steps):
        step()
    end_event.record(stream)
    barrier()
    t1 = time.monotonic()
    elapsed_ms = max_over_ranks(start_event.elapsed_time(end_event))
    clocks = sampler.summary(t0, t1)
    sampler.stop()
    gpu_launches = model.launches_per_forward(batch) * args.steps
    launches_issued = cuvit.kernels.launch_count() - launches_before  # 0 under graph replay

    cuvit.kernels.device_status()  # raises if any kernel of the timed passes gave up a wait

    # Per-kernel device time over profiled passes (events around each launch), after one
    # discarded pass; per launch kind, the median pass (clocks drift under the power cap).
    by_kind = profile_pass_kinds(model, images, logits, batch, stream, args.profile_passes)
    passes = 1  # by_kind holds one (median) pass
    profiled_ms = sum(e["ms"] for e in by_kind.values())
    kernels = {}
    for kind, e in sorted(by_kind.items()):
        kernels[kind] = {
            "launches_per_pass": e["launches"],
            "ms_per_pass": e["ms"],
            "share": e["ms"] / profiled_ms if profiled_ms else None,
            "tflops": e["flops"] / (e["ms"] * 1e-3) / 1e12 if e["flops"] else None,
            "gbs": e["bytes"] / (e["ms"] * 1e-3) / 1e9,
        }
    gemm_flops, gemm_ms, gemm_launches = gemm_summary(by_kind)
    cuvit.kernels.device_status()
    achieved_tflops = gemm_flops / (gemm_ms * 1e-3) / 1e12
    peak, peak_kind = peaks()
    traffic, traffic_launch = gemm_traffic(args.config, label, batch, precision_name)

    # End to end through the public host-buffer API: pinned host images in, logits out.
    # N > 1: each step's host logits go back to the device and to rank 0 on a side stream,
    # overlapping the next step's pass (two logits buffers alternate; events order the reuse).
    pinned_images = torch.from_numpy(host_images).pin_memory()
    pinned_logits = [torch.zeros(batch, config.classes).pin_memory() for _ in range(2)]
    device_logits = [torch.zeros_like(logits) for _ in range(2)]
    side = torch.cuda.Stream(device)
    landed = [torch.cuda.Event() for _ in range(2)]  # the step's logits are on the host
    handed = [torch.cuda.Event() for _ in range(2)]  # ... and back on the device for the gather
    calls = [0]

    def e2e_step():
        k = calls[0] % 2
        calls[0] += 1
        if world > 1:
            stream.wait_event(handed[k])  # buffer k's previous logits have been handed over
        model.forward_host_async(pinned_images.data_ptr(), pinned_logits[k].data_ptr(), batch,
                                 stream)
        if world > 1:
            landed[k].record(stream)
            with torch.cuda.stream(side):
                side.wait_event(landed[k])
                device_logits[k].copy_(pinned_logits[k], non_blocking=True)
                handed[k].record(side)
                gather(device_logits[k], side)

    for _ in range(args.warmup):
        e2e_step()
    barrier()
    e2e_start = torch.cuda.Event(enable_timing=True)
    e2e_end = torch.cuda.Event(enable_timing=True)
    e2e_start.record(stream)
    for _ in range(args.steps):
        e2e_step()
    stream.wait_stream(side)  # the last gather is part of the step
    e2e_end.record(stream)
    barrier()
    e2e_ms = max_over_ranks(e2e_start.elapsed_time(e2e_end))
    cuvit.kernels.device_status()

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_baseline = measure_cpu_baseline(config, weights, seed)

    # One GPU only: the other benchmark configurations, the single-GEMM configuration and the
    # FP32 comparison with the reference's own GPU path, each timed in this run beside the
    # headline (which they do not touch).
    extras = {}
    wanted = set() if args.no_extras else set(args.extra or EXTRAS)
    if world == 1 and wanted:
        peak_tf32 = None
        if wanted & {"configs", "single_gemms"}:
            peak_tf32 = measure_tf32_peak(torch, device)
            extras["tf32_peak_tflops"] = peak_tf32
        if "configs" in wanted:
            extras["configs"] = measure_other_configs(
                torch, device, peak.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]),
                peak_tf32)
        if "single_gemms" in wanted:
            extras["single_gemms"] = measure_single_gemms(torch, device, peak_tf32)
        if "fp32_baselines" in wanted:
            extras["fp32_baselines"] = measure_fp32_baselines(torch, device)
        if "preprocess" in wanted:
            extras["preprocess"] = measure_preprocess(torch, device)

    total_images = world * batch * args.steps
    value = total_images / (elapsed_ms * 1e-3)
    if rank == 0:
        bf16 = precision == PRECISION_BF16
        sustained = peak.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
        burst = peak.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
        line = {
            "metric": METRIC, "value": value, "unit": "images/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": precision_name,
            "data": "synthetic N(0,1) images, random-init trunc-normal(0.02) weights",
            "config": {
                "workload": f"{label} forward, {precision_name.upper()} operands / FP32 "
                            f"accumulate, batch {batch} per GPU",
                "model": label, "global_batch": batch * world, "seq_len": config.token_count(),
                "parallelism": f"dp{world} (replicas; logits gathered to rank 0 each step "
                               "by cuvit_gather_logits over NCCL)",
                "l2": f"inputs {host_images.nbytes / 1e6:.0f} MB per GPU (> 126 MB L2), "
                      "weights re-read each pass; no flush",
                "gflop_per_image": config.gflop_per_image(),
            },
            "e2e": {"value": total_images / (e2e_ms * 1e-3), "unit": "images/s",
                    "h2d_bytes_per_step": int(batch * model.host_image_bytes()),
                    "d2h_bytes_per_step": int(batch * config.classes * 4)},
            "gpu_launches": gpu_launches,
            "roofline": {
                "kernel": "tcgen05 GEMMs, all launches of a pass (tc_gemm_pair_kernel: patch, "
                          "QKV, proj, FC2; tc_gemm_kernel: FC1 with GELU, head)",
                "bound": "tensor", "achieved": achieved_tflops,
                "peak": burst, "unit": "TFLOP/s", "frac": achieved_tflops / burst,
                "peak_kind": f"{peak_kind} bf16 burst (each GEMM timed per launch with CUDA "
                             "events inside ~11 ms profiled passes)",
                "frac_of_sustained": achieved_tflops / sustained,
                "frac_of_nominal_2250": achieved_tflops / 2250.0,
                "traffic": traffic,
                "traffic_launch": traffic_launch,
                "launches_per_pass": gemm_launches // passes,
                "flops_per_launch": gemm_flops / max(gemm_launches, 1),
            },
            "kernels": kernels,
            "clocks": clocks,
            "cpu_baseline": cpu_baseline,
            "launches_issued_in_timed_region": launches_issued,
            **extras,
        }
        print(json.dumps(line), flush=True)
    model.close()
    if world > 1:
        torch.cuda.synchronize(device)
        comm.close()
        dist.destroy_process_group()


def gemm_traffic(config_name: str, label: str, batch: int, precision: str):
    """DRAM bytes (read + write) of one launch of the dominant GEMM kernel from the committed
    ncu summary, if any: profiles/tc_gemm_pair_qkv_<config>_b<batch>_<precision>.md, line
    'traffic_bytes_per_launch'."""
    import re

    path = ROOT / "profiles" / f"tc_gemm_pair_qkv_{config_name}_b{batch}_{precision}.md"
    if not path.exists():
        return None, None
    match = re.search(r"^traffic_bytes_per_launch:\s*(\d+)", path.read_text(), re.M)
    if not match:
        return None, None
    return int(match.group(1)), (f"{label} block-0 QKV GEMM (tc_gemm_pair_kernel), one ncu "
                                 f"capture ({path.name})")


def measure_cpu_baseline(config, weights, seed) -> dict | None:
    """The reference's CPU forward on one image per host core (about 10-30 s)."""
    import oracle

    threads = os.cpu_count() or 1
    rng = np.random.default_rng([seed, 99])
    images = rng.standard_normal(threads * config.image_elements()).astype(np.float32)
    try:
        with tempfile.TemporaryDirectory() as tmp:
            path = pathlib.Path(tmp) / "weights.cvw"
            write_cvw(config, weights, path)
            seconds, count, kind = cpu_reference_step(config, path, images, threads)
    except (RuntimeError, FileNotFoundError) as error:
        return {"value": None, "unit": "images/s", "cores": threads, "kind": None,
                "sample": f"unavailable: {error}"}
    return {"value": count / seconds, "unit": "images/s", "cores": threads, "kind": kind,
            "cpu": cpu_model(),
            "sample": f"{count} images, one per host thread, VitReference::forward "
                      f"(tests/reference/vit.hpp), {seconds:.1f} s"}


def timeline_arm(args) -> None:
    """Where a graph-replayed pass spends its time between and inside kernels (one GPU).

    Needs the instrumented library (python cu-vit_b200/build.py --timeline): every
    forward-path kernel stamps the global timer at its first CTA's entry and its last warp's
    exit, and CTA 0 its SM cycle counter, so each launch gives its span, the gap before it
    and the SM clock it ran at. Three passes are replayed back to back as in the timed region
    of the benchmark; the device is synchronized once after them and one more replay is
    recorded (a graph node keeps its grid id across replays, so one replay is recorded at a
    time); then one profiled pass (CUDA events around every launch) for comparison."""
    import ctypes

    import torch

    import cuvit
    from cuvit import _lib
    from cuvit.errors import check
    from cuvit.vit import PRECISION_BF16, PRECISION_TF32, VisionTransformer, VitConfig, random_weights

    lib = _lib.library()
    if not lib.cuvit_timeline_available():
        raise SystemExit("the timeline build is not loaded (build it with "
                         "python cu-vit_b200/build.py --timeline)")
    label, kwargs, batch, precision_name, seed = CONFIGS[args.config]
    config = VitConfig(**kwargs)
    precision = PRECISION_BF16 if precision_name == "bf16" else PRECISION_TF32
    device = torch.device("cuda", 0)
    model = VisionTransformer(config, random_weights(config, seed), max_batch=batch,
                              precision=precision)
    rng = np.random.default_rng([seed, 0])
    images = torch.from_numpy(rng.standard_normal(batch * config.image_elements())
                              .astype(np.float32)).to(device)
    logits = torch.zeros(batch, config.classes, device=device)
    stream = torch.cuda.current_stream(device)
    kinds = [r["kind"] for r in model.forward_profiled(images, logits, batch, stream)]
    per_pass = len(kinds)

    def capture(run, passes):
        check(lib.cuvit_timeline_reset())
        run()
        torch.cuda.synchronize()
        records = (_lib.TimelineRecordC * (per_pass * passes + 16))()
        count = ctypes.c_int(0)
        check(lib.cuvit_timeline_read(records, len(records), ctypes.byref(count)))
        got = records[:count.value]
        if len(got) != per_pass * passes:
            raise SystemExit(f"expected {per_pass * passes} launches, recorded {len(got)}")
        return got[-per_pass:]

    def analyse(records):
        rows = []
        for i, (kind, r) in enumerate(zip(kinds, records)):
            span = (r.last_ns - r.first_ns) / 1e3
            gap = (r.first_ns - records[i - 1].last_ns) / 1e3 if i else 0.0
            ns = r.cta0_exit_ns - r.cta0_entry_ns
            mhz = (r.cta0_exit_clock - r.cta0_entry_clock) / ns * 1e3 if ns > 0 else None
            rows.append({"kind": kind, "span_us": span, "gap_before_us": gap, "sm_mhz": mhz,
                         # CTA 0 from its entry to its exit; the rest of the span is the
                         # launch skew of later CTAs plus the tail of the last ones
                         "cta0_us": ns / 1e3,
                         "cycles": span * mhz if mhz else 0.0})
        summary = {}
        for row in rows:
            entry = summary.setdefault(row["kind"], {"launches": 0, "span_us": 0.0,
                                                     "gap_before_us": 0.0, "cta0_us": 0.0,
                                                     "mcycles": 0.0, "mhz": []})
            entry["launches"] += 1
            entry["span_us"] += row["span_us"]
            entry["gap_before_us"] += row["gap_before_us"]
            entry["cta0_us"] += row["cta0_us"]
            entry["mcycles"] += row["cycles"] / 1e6
            if row["sm_mhz"]:
                entry["mhz"].append(row["sm_mhz"])
        for entry in summary.values():
            mhz = entry.pop("mhz")
            entry["sm_mhz_mean"] = sum(mhz) / len(mhz) if mhz else None
        total = (records[-1].last_ns - records[0].first_ns) / 1e3
        spans = sum(r["span_us"] for r in rows)
        gaps = sum(r["gap_before_us"] for r in rows)
        return {"pass_us": total, "kernel_spans_us": spans, "gaps_us": gaps,
                "gaps_per_launch_us": gaps / max(len(rows) - 1, 1), "by_kind": summary}

    for _ in range(5):
        model.forward_graph(images, logits, batch, stream)
    graph = capture(lambda: model.forward_graph(images, logits, batch, stream), 1)
    profiled_ms = {}
    profiled = capture(lambda: profiled_ms.setdefault(
        "records", model.forward_profiled(images, logits, batch, stream)), 1)
    event_us = sum(r["ms"] for r in profiled_ms["records"]) * 1e3
    cuvit.kernels.device_status()
    line = {"mode": "timeline", "workload": f"{label} {precision_name.upper()}, batch {batch}",
            "launches_per_pass": per_pass, "graph_replay": analyse(graph),
            "profiled_pass": dict(analyse(profiled), event_sum_us=event_us)}
    print(json.dumps(line), flush=True)
    model.close()


def main() -> None:
    args = parse_args()
    if args.timeline:
        os.environ["CUVIT_LIBRARY_VARIANT"] = "timeline"
        timeline_arm(args)
    elif args.impl == "reference":
        reference_arm(args)
    else:
        our_arm(args)


if __name__ == "__main__":
    main()
