"""Benchmark: ResNet-50 FP32 inference img/s (+ FFN FP16 tokens/s) on B200.

One process per GPU (torchrun for N > 1), one Engine + ExecutionContext per
GPU with replicated constants and a batch shard of 256 images per GPU (weak
scaling, no collective on the data path). Each step is one pass of the
compiled ResNet-50 (batch 256, 224x224, FP32) through
ExecutionContext::RunAsync; the timed region is K steps bracketed by a
barrier + device synchronize, timed with CUDA events on the launching
stream, max over ranks. Inputs (154 MB per step) are larger than L2.

The line also reports: the end-to-end rate through the C ABI with host
buffers (pinned H2D of the step's images + D2H of the logits inside the
timed region), the roofline of the dominant kernel family (the FP32
convolutions), the FFN FP16 block at config 1 (M=4096, H=768, I=3072, per
rank) and config 4 (H=1024, I=4096, global M=65536 split over the ranks),
SM clocks sampled during the timed region, and — from the CPU leg on rank 0,
after all GPU timing — the PyTorch-eager CPU baseline on a bounded sample and
a parity check of the bench's own GPU outputs against the CPU results
(sampled bs256 logits; the whole config-1 FFN output).

``--impl reference`` times the reference's CPU comparison path (the PyTorch
eager ResNet-50 of the reference's benchmarks/resnet50_compare.py, restated
in oracle/torch_ref.py) on the host cores, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

PEAKS_FILE = REPO / "MEASURED_PEAKS.json"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
RN_BATCH_PER_GPU = 256
UNFUSED = "unfused:"  # candidate-id prefix of the unfused decompositions
CONV_DRAM_BYTES_PER_STEP_BS256 = 25.669e9  # ncu, the 53 conv kernels of one tuned bs256 step (see roofline.traffic)
FFN = dict(tokens=4096, hidden=768, inner=3072)


def parse_args() -> argparse.Namespace:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=30)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--batch", type=int, default=RN_BATCH_PER_GPU, help="images per GPU")
    p.add_argument("--no-ffn", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--tuning", choices=["TuneOnMiss", "Disabled"], default="TuneOnMiss",
                   help="ResNet-50 candidate selection: tuned during warm-up into a per-run cache (default, "
                        "as a deployment tunes once and then runs from the cache) or the pack defaults")
    p.add_argument("--tuning-cache", default=None,
                   help="tuning cache directory (default: a fresh one per run); a run with a filled cache "
                        "reads its choices instead of timing candidates")
    p.add_argument("--profile-case", choices=sorted(PROFILE_CASES),
                   help="run one small kernel case three times (for ncu captures) and exit")
    p.add_argument("--config", type=int, choices=[2, 3, 4],
                   help="2: dynamic-batch ResNet-50 (profile 1/32/128, graph LRU 4, TuneOnMiss); "
                        "3: per-layer conv sweep at N=256; 4: FFN H=1024 I=4096 M=65536 (sharded over ranks)")
    return p.parse_args()


def _conv_case(n, c, h, k, r, stride, pad, op="FusedConvBatchNormRelu", residual=False, **engine_options):
    """One convolution node through the engine; returns (engine, ctx, tensors).
    Default: no CUDA graph, no tuning (the default candidate)."""
    import torch
    import cutriton_b200 as ct

    rng = np.random.default_rng(0)
    m = ct.Model()
    m.add_input("x", [n, c, h, h])
    m.add_constant("w", (rng.standard_normal((k, c, r, r)) * 0.05).astype(np.float32), layout="OIHW")
    for nm in ("s", "b", "mu", "v"):
        m.add_constant(nm, np.ones(k, np.float32), layout="")
    ho = (h + 2 * pad - r) // stride + 1
    names = ["x", "w", "s", "b", "mu", "v"]
    if residual:
        op = "FusedConvBatchNormAddRelu"
        m.add_input("res", [n, k, ho, ho])
        names.append("res")
    m.add_node("conv", op, names, ["y"], strides=[stride, stride],
               pads=[pad] * 4, dilations=[1, 1], batchnorm_epsilon=1e-5)
    m.add_output("y")
    e = ct.build_engine(m, **{"enable_cuda_graph": False, "tuning_mode": ct.TUNING_DISABLED, **engine_options})
    ctx = e.create_context()
    x = torch.randn(n, c, h, h, device="cuda")
    y = torch.empty(n, k, ho, ho, device="cuda")
    ctx.bind_tensor("x", x)
    ctx.bind_tensor("y", y, output=True)
    keep = [x, y]
    if residual:
        keep.append(torch.randn(n, k, ho, ho, device="cuda"))
        ctx.bind_tensor("res", keep[-1])
    return e, ctx, keep


def _ffn_case():
    import torch
    import cutriton_b200 as ct
    from cutriton_b200 import workloads

    t, h, i = FFN["tokens"], FFN["hidden"], FFN["inner"]
    e = ct.build_engine(workloads.build_ffn(workloads.ffn_weights(h, i), t, h, i),
                        enable_cuda_graph=False, tuning_mode=ct.TUNING_DISABLED)
    ctx = e.create_context()
    x = torch.from_numpy(workloads.ffn_input(t, h)).cuda()
    y = torch.empty(t, h, dtype=torch.float16, device="cuda")
    ctx.bind_tensor("x", x)
    ctx.bind_tensor("output", y, output=True)
    return e, ctx, (x, y)


def _single_op_case(op: str, shapes: list[tuple[str, list[int]]], out_shape: list[int], dtype: str = "float32",
                    constants: dict | None = None, **attrs):
    """One node `op` over inputs of `shapes` through the engine; returns (engine, ctx, tensors)."""
    import torch
    import cutriton_b200 as ct

    np_dtype = np.float16 if dtype == "float16" else np.float32
    layout = "NCHW" if len(out_shape) == 4 else ""
    m = ct.Model()
    names = []
    for name, shape in shapes:
        m.add_input(name, shape, dtype=np_dtype, layout=layout)
        names.append(name)
    for name, value in (constants or {}).items():
        m.add_constant(name, value, layout="")
        names.append(name)
    m.add_node("op", op, names, ["y"], **attrs)
    m.add_output("y")
    e = ct.build_engine(m, enable_cuda_graph=False, tuning_mode=ct.TUNING_DISABLED)
    ctx = e.create_context()
    tdtype = getattr(torch, dtype)
    keep = []
    for name, shape in shapes:
        keep.append(torch.randn(*shape, device="cuda").to(tdtype))
        ctx.bind_tensor(name, keep[-1])
    keep.append(torch.empty(*out_shape, device="cuda", dtype=tdtype))
    ctx.bind_tensor("y", keep[-1], output=True)
    return e, ctx, keep


def _skip_ln_case(rows: list[int]):
    import torch
    import cutriton_b200 as ct

    m = ct.Model()
    m.add_input("x", rows, dtype=np.float16, layout="")
    m.add_input("r", rows, dtype=np.float16, layout="")
    m.add_constant("g", np.ones(rows[1], np.float16), layout="")
    m.add_constant("b", np.zeros(rows[1], np.float16), layout="")
    m.add_node("add", "Add", ["x", "r"], ["s"])
    m.add_node("ln", "LayerNormalization", ["s", "g", "b"], ["y"], axis=-1, epsilon=1e-5)
    m.add_output("y")
    e = ct.build_engine(m, enable_cuda_graph=False, tuning_mode=ct.TUNING_DISABLED)
    ctx = e.create_context()
    keep = [torch.randn(*rows, device="cuda").half() for _ in range(3)]
    ctx.bind_tensor("x", keep[0])
    ctx.bind_tensor("r", keep[1])
    ctx.bind_tensor("y", keep[2], output=True)
    return e, ctx, keep


def _bandwidth_cases():
    """Every bandwidth-bound kernel of the pack at a size above L2 (126 MB)
    and a few hundred MB on the device, plus the FC GEMM at bs256."""
    nchw = [64, 256, 56, 56]  # 205.5 MB per FP32 tensor
    rows = [65536, 1024]      # 134 MB per FP16 tensor
    bn = {n: np.ones(256, np.float32) for n in ("s", "b", "m", "v")}
    ln = {"g": np.ones(1024, np.float16), "b": np.zeros(1024, np.float16)}
    return [
        ("max_pool_3x3s2_f32_64x64x112x112", lambda: _single_op_case(
            "MaxPool", [("x", [64, 64, 112, 112])], [64, 64, 56, 56], kernel_shape=[3, 3], strides=[2, 2],
            pads=[1, 1, 1, 1], dilations=[1, 1])),
        ("global_average_pool_f32_512x2048x7x7", lambda: _single_op_case(
            "GlobalAveragePool", [("x", [512, 2048, 7, 7])], [512, 2048, 1, 1])),
        ("add_relu_f32_64x256x56x56", lambda: _single_op_case("AddRelu", [("a", nchw), ("b", nchw)], nchw)),
        ("add_f32_64x256x56x56", lambda: _single_op_case("Add", [("a", nchw), ("b", nchw)], nchw)),
        ("relu_f32_64x256x56x56", lambda: _single_op_case("Relu", [("a", nchw)], nchw)),
        ("batch_norm_f32_64x256x56x56", lambda: _single_op_case(
            "BatchNormalization", [("x", nchw)], nchw, constants=bn, epsilon=1e-5)),
        ("gelu_f16_65536x1024", lambda: _single_op_case("Gelu", [("x", rows)], rows, dtype="float16")),
        ("add_f16_65536x1024", lambda: _single_op_case("Add", [("a", rows), ("b", rows)], rows, dtype="float16")),
        ("layer_norm_f16_65536x1024", lambda: _single_op_case(
            "LayerNormalization", [("x", rows)], rows, dtype="float16", constants=ln, axis=-1, epsilon=1e-5)),
        ("skip_layer_norm_f16_65536x1024", lambda: _skip_ln_case(rows)),
        ("fc_gemm_f32_256x2048x1000", lambda: _single_op_case(
            "Gemm", [("a", [256, 2048])], [256, 1000], constants={"w": np.full((2048, 1000), 0.01, np.float32)})),
    ]


def _gemm_f16_case(m: int, n: int, k: int, kernel_id: str):
    """One FP16 Gemm node (B constant) with candidate `kernel_id` selected."""
    rng = np.random.default_rng(0)
    b = (rng.standard_normal((k, n)) * 0.02).astype(np.float16)
    e, ctx, keep = _single_op_case("Gemm", [("a", [m, k])], [m, n], dtype="float16", constants={"b": b})
    ids = [c.split(":")[1] for c in e.ops()[0]["candidates"]]
    ctx.select_candidate(0, ids.index(kernel_id))
    return e, ctx, keep


def _with_candidate(case, kernel_id: str):
    """Selects the candidate of op 0 whose kernel id is `kernel_id`."""
    e, ctx, keep = case
    ids = [c.split(":")[1] for c in e.ops()[0]["candidates"]]
    ctx.select_candidate(0, ids.index(kernel_id))
    return e, ctx, keep


def _resnet_case(batch: int):
    import torch
    import cutriton_b200 as ct
    from cutriton_b200 import workloads

    model = workloads.build_resnet50(workloads.resnet50_weights("baseline", seed=0), batch=batch)
    e = ct.build_engine(model, enable_cuda_graph=False, enable_residual_fusion=True, tuning_mode=ct.TUNING_DISABLED)
    ctx = e.create_context()
    x = torch.from_numpy(workloads.resnet50_input(batch, seed=0)).cuda()
    y = torch.empty(batch, 1000, device="cuda")
    ctx.bind_tensor("input", x)
    ctx.bind_tensor("output", y, output=True)
    return e, ctx, (x, y)


# Cases for ncu captures: inputs + outputs above L2 (126 MB), at most a few GB
# on the device. A single-kernel case runs three times; "bandwidth_ops" runs
# each of its graphs once, one after the other (built, run, freed);
# "resnet50_bs32" / "resnet50_bs64" run the whole network once each (per-layer
# DRAM traffic at two batch sizes, extrapolated to bs256 by a fit linear in
# the batch).
PROFILE_CASES = {
    "conv3x3_128ch_28x28_bs256": lambda: _conv_case(256, 128, 28, 128, 3, 1, 1),
    "conv3x3_64ch_56x56_bs64": lambda: _conv_case(64, 64, 56, 64, 3, 1, 1),
    "conv1x1_256to64_56x56_bs64": lambda: _conv_case(64, 256, 56, 64, 1, 1, 0),
    "conv1x1_64to256_add_56x56_bs64": lambda: _conv_case(64, 64, 56, 256, 1, 1, 0, residual=True),
    "conv1x1_mn_64to256_add_56x56_bs64": lambda: _with_candidate(
        _conv_case(64, 64, 56, 256, 1, 1, 0, residual=True), "conv_bn_add_relu.fp32.nchw.tcgen05_mn"),
    "stem7x7_bs64": lambda: _conv_case(64, 3, 224, 64, 7, 2, 3),
    "ffn_4096x768x3072": _ffn_case,
    # FFN config-4 down-projection shape at M=16384 (A 134 MB): CTA pair vs single CTA.
    "gemm_f16_pair_16384x1024x4096": lambda: _gemm_f16_case(16384, 1024, 4096, "gemm.fp16.tcgen05_pair"),
    "gemm_f16_tp_16384x1024x4096": lambda: _gemm_f16_case(16384, 1024, 4096, "gemm.fp16.tcgen05_persistent"),
    "bandwidth_ops": None,
    "resnet50_bs32": lambda: _resnet_case(32),
    "resnet50_bs64": lambda: _resnet_case(64),
}


def run_profile_case(name: str) -> None:
    import torch

    if name == "bandwidth_ops":
        for case, make in _bandwidth_cases():
            keep = make()
            keep[1].run()
            torch.cuda.synchronize()
            print(json.dumps({"profile_case": case, "runs": 1}), flush=True)
            del keep
        return
    keep = PROFILE_CASES[name]()
    runs = 1 if name.startswith("resnet50_") else 3
    for _ in range(runs):
        keep[1].run()
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": name, "runs": runs}), flush=True)


def conv_shapes() -> list[tuple[int, int, int, int, int, int]]:
    """Distinct ResNet-50 conv shapes (cin, cout, kernel, stride, pad, input H=W), in network order."""
    from cutriton_b200 import workloads

    shapes, h, block_in = [], 224, 224
    for kind, item in workloads.resnet50_layers():
        if kind == "maxpool":
            h = (h + 2 - 3) // 2 + 1
            block_in = h
            continue
        if kind == "block_add":
            block_in = h
            continue
        ih = block_in if item.prefix.endswith(("_conv1", "_downsample")) else h
        key = (item.cin, item.cout, item.kernel, item.stride, item.pad, ih)
        if key not in shapes:
            shapes.append(key)
        if not item.prefix.endswith("_downsample"):
            h = (ih + 2 * item.pad - item.kernel) // item.stride + 1
    return shapes


def time_context(ctx, stream, steps: int, warmup: int, all_times: bool = False):
    """Median ms of `steps` RunAsync calls timed with CUDA events on `stream`
    (every step's ms with `all_times`)."""
    import torch

    for _ in range(max(3, warmup)):
        ctx.run_async(stream.cuda_stream)
        ctx.synchronize()
    times = []
    for _ in range(steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        ctx.run_async(stream.cuda_stream)
        b.record(stream)
        ctx.synchronize()
        b.synchronize()
        times.append(a.elapsed_time(b))
    return times if all_times else float(np.median(times))


def run_config2(args, tuning: str = "TuneOnMiss") -> dict:
    """Config 2: one engine with a dynamic batch profile min/opt/max = 1/32/128, a CUDA-graph LRU of
    capacity 4 and the tuner in TuneOnMiss mode (fused vs unfused candidates), run at 32, 64, 128."""
    import tempfile

    import torch
    import cutriton_b200 as ct
    from cutriton_b200 import workloads

    weights = workloads.resnet50_weights("baseline", seed=0)
    model = workloads.build_resnet50(weights, dynamic_batch=True)
    model.add_shape_profile("batch", "input", [1, 3, 224, 224], [32, 3, 224, 224], [128, 3, 224, 224])
    cache = tempfile.mkdtemp(prefix="ctb_tuning_")
    mode = ct.TUNING_TUNE_ON_MISS if tuning == "TuneOnMiss" else ct.TUNING_DISABLED
    engine = ct.build_engine(model, enable_cuda_graph=True, enable_residual_fusion=True,
                             tuning_mode=mode, tuning_cache_dir=cache, cuda_graph_cache_capacity=4)
    ctx = engine.create_context()
    stream = torch.cuda.Stream()
    results = {}
    for batch in (32, 64, 128):
        ctx.set_input_shape("input", [batch, 3, 224, 224])
        ctx.resolve_shapes()
        x = torch.from_numpy(workloads.resnet50_input(batch, seed=0)).cuda()
        y = torch.empty(batch, 1000, device="cuda")
        ctx.bind_tensor("input", x)
        ctx.bind_tensor("output", y, output=True)
        ms = time_context(ctx, stream, args.steps, args.warmup)
        results[str(batch)] = {"ms": ms, "img_s": batch / ms * 1e3}
    ops = engine.ops()
    chosen = [op["candidates"][ctx.selected_candidate(i)] for i, op in enumerate(ops)]
    unfused = sum(1 for c in chosen if c.startswith(UNFUSED))
    # Which ops the tuner moved off their default candidate at the last batch
    # run (128; each batch shape is tuned on its first run and cached).
    moved = [{"op": op["node"], "default": op["candidates"][op["default"]].split(":", 1)[-1],
              "chosen": chosen[i].split(":", 1)[-1]}
             for i, op in enumerate(ops) if ctx.selected_candidate(i) != op["default"]]
    kinds: dict[str, int] = {}
    for c in chosen:
        kind = c.split(":")[1] if ":" in c else c
        kinds[kind] = kinds.get(kind, 0) + 1
    return {"metric": "ResNet-50 FP32 img/s, dynamic batch profile (config 2)", "unit": "img/s",
            "higher_is_better": True, "config": {"workload": "resnet50_dynamic_batch", "profile": [1, 32, 128],
                                                "graph_lru": 4, "tuning": tuning},
            "batches": results, "cached_graphs": ctx.cached_graph_count(), "ops": engine.num_ops(),
            "ops_tuned_to_unfused": unfused, "selected_kernels": kinds, "tuned_off_default": moved}


def run_config3(args, peaks) -> dict:
    """Config 3: one FusedConvBatchNormRelu graph per distinct ResNet-50 conv
    shape at N=256, on the candidate the tuner picks (--tuning TuneOnMiss, the
    default; the warm-up runs tune) or the default one (--tuning Disabled).
    Device time of the op: the engine's per-op events inside the captured
    graph, median over the timed runs."""
    import torch

    peak_tf = peaks["bf16_tflops"] / 6.0  # burst: each layer runs for well under a millisecond
    rows = []
    tuning = bench_tuning(args, 0)
    stream = torch.cuda.Stream()
    for cin, cout, kernel, stride, pad, h in conv_shapes():
        e, ctx, keep = _conv_case(256, cin, h, cout, kernel, stride, pad, enable_cuda_graph=True,
                                  enable_profiling=True, **tuning)
        samples = []
        for step in range(max(3, args.warmup) + args.steps):
            ctx.run_async(stream.cuda_stream)
            ctx.synchronize()
            if step >= max(3, args.warmup):
                samples.append(ctx.profile_events()[0][1])
        ms = float(np.median(samples))
        ho = (h + 2 * pad - kernel) // stride + 1
        flops = 2.0 * 256 * ho * ho * cout * cin * kernel * kernel
        nbytes = 4.0 * 256 * (cin * h * h + cout * ho * ho)
        rows.append({"shape": f"{cin}->{cout} k{kernel} s{stride} {h}x{h}", "ms": round(ms, 4),
                     "tflops": round(flops / ms / 1e9, 1), "tensor_frac": round(flops / ms / 1e9 / peak_tf, 3),
                     "gbs": round(nbytes / ms / 1e6, 1), "hbm_frac": round(nbytes / ms / 1e6 / peaks["hbm_gbs"], 3),
                     "candidate": e.ops()[0]["candidates"][ctx.selected_candidate(0)]})
        del ctx, e, keep
    return {"metric": "per-layer FusedConvBatchNormRelu sweep, N=256 (config 3)", "unit": "TFLOP/s",
            "peak_basis": f"3xTF32 = bf16_tflops (burst) / 6 = {peak_tf:.1f} TFLOP/s; HBM {peaks['hbm_gbs']} GB/s",
            "tuning": args.tuning, "timing": "per-op CUDA events inside the captured graph, median",
            "layers": rows}


def bench_tuning(args, rank: int) -> dict:
    """Engine options for the candidate choice of every timed engine:
    TuneOnMiss times every numerically valid candidate of each op on its
    first run (a warm-up, outside the timed region) and caches the choice in
    this rank's cache directory, which every later engine of the run reads."""
    import tempfile

    import cutriton_b200 as ct

    tuning_dir = (os.path.join(args.tuning_cache, f"rank{rank}") if args.tuning_cache
                  else tempfile.mkdtemp(prefix=f"ctb_bench_tuning_{rank}_"))
    return dict(tuning_mode=ct.TUNING_TUNE_ON_MISS if args.tuning == "TuneOnMiss" else ct.TUNING_DISABLED,
                tuning_cache_dir=tuning_dir)


def chosen_kernels(engine, ctx) -> list[str]:
    """Kernel (candidate id without the backend prefix) each op runs."""
    return [op["candidates"][ctx.selected_candidate(i)].split(":", 1)[-1] for i, op in enumerate(engine.ops())]


def run_config4(args, world, rank, local, peaks, peak_kind) -> dict:
    """Config 4: FFN H=1024, I=4096, global M=65536 split over the ranks (no collective)."""
    import torch
    import cutriton_b200 as ct
    from cutriton_b200 import workloads

    h, i, global_m = 1024, 4096, 65536
    m_rank = global_m // world
    w = workloads.ffn_weights(h, i, seed=0)
    engine = ct.build_engine(workloads.build_ffn(w, m_rank, h, i), device_id=local, enable_cuda_graph=True,
                             **bench_tuning(args, rank))
    ctx = engine.create_context()
    x = torch.from_numpy(workloads.ffn_input(m_rank, h, seed=rank)).cuda(local)
    y = torch.empty(m_rank, h, dtype=torch.float16, device=f"cuda:{local}")
    ctx.bind_tensor("x", x)
    ctx.bind_tensor("output", y, output=True)
    times = time_context(ctx, torch.cuda.Stream(local), args.steps, args.warmup, all_times=True)
    kernels = chosen_kernels(engine, ctx)
    ms = max_over_ranks(float(np.median(times)), world)
    p95 = max_over_ranks(float(np.percentile(times, 95)), world)
    flops = 4.0 * h * i * global_m
    tflops = flops / ms / 1e9
    return {"metric": "FFN FP16 tokens/s (config 4: H=1024, I=4096, global M=65536)", "unit": "tokens/s",
            "value": global_m / ms * 1e3, "ms_per_step": ms, "ms_p95": p95, "tflops": tflops,
            "tflops_per_gpu": tflops / world, "roofline": ffn_roofline(tflops / world, peaks, peak_kind, kernels),
            "rows_per_gpu": m_rank, "n_gpus": world, "scaling": "strong", "higher_is_better": True,
            "l2": "inputs larger than L2 at 1 GPU (M=65536: 128 MB in, 512 MB intermediate)"}


def load_peaks() -> tuple[dict, str]:
    if PEAKS_FILE.exists():
        return json.loads(PEAKS_FILE.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the
    timed region (100 ms period); entering waits for the first sample so the
    samples fall inside the region rather than in nvidia-smi's start-up."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        # nvidia-smi numbers GPUs its own way (it ignores CUDA_VISIBLE_DEVICES),
        # so the timed GPU is named by its UUID rather than the CUDA ordinal.
        self.device_index = str(device_index)
        try:
            import torch

            self.device_index = "GPU-" + str(torch.cuda.get_device_properties(device_index).uuid)
        except Exception:  # noqa: BLE001 - keep the ordinal when the UUID is unavailable
            pass
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"ctb_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-i", self.device_index, "-lms", "100"], stdout=self.out,
                                         stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
            return self
        deadline = time.monotonic() + 5.0
        while time.monotonic() < deadline and self.proc.poll() is None:
            if self.path.stat().st_size > 0:
                break
            time.sleep(0.02)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.out.close()

    def summary(self) -> dict:
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = [r.split(",") for r in self.path.read_text().strip().splitlines() if r.strip()]
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].strip().replace(".", "").isdigit()]
        sm_max = [float(r[2]) for r in rows if len(r) >= 9 and r[2].strip().replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            if len(r) < 9:
                continue
            for name, value in zip(names, r[5:9]):
                if value.strip().lower() == "active":
                    reasons.add(name)
        self.path.unlink(missing_ok=True)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(sm_max) if sm_max else None,
                "samples": len(rows), "reasons": sorted(reasons), "gpu": self.device_index}


def dist_setup(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        from datetime import timedelta

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    """Slowest rank's value (device time of the timed region)."""
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def shard(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous batch shard of `rank`: (first image, image count). Every
    rank gets global_batch // world images; the first global_batch % world
    ranks take one more."""
    base, extra = divmod(global_batch, world)
    count = base + (1 if rank < extra else 0)
    start = rank * base + min(rank, extra)
    return start, count


def kernel_launches_per_run(engine, ctx) -> int:
    total = 0
    for i, op in enumerate(engine.ops()):
        cand = op["candidates"][ctx.selected_candidate(i)]
        if cand == "view:flatten":
            continue
        total += 3 if cand == "unfused:conv_bn_relu" else (2 if cand.startswith("unfused:") else 1)
    return total


def resnet_work(batch: int) -> dict:
    """Per-step algorithmic work of ResNet-50 at `batch` (FLOPs per conv
    family and minimal bytes), from the layer table."""
    from cutriton_b200.workloads import resnet50_layers

    conv_flops = 0.0
    conv_bytes = 0.0
    h = 224
    block_h = h
    for kind, item in resnet50_layers():
        if kind == "maxpool":
            h = (h + 2 - 3) // 2 + 1
            block_h = h
            continue
        if kind == "block_add":
            block_h = h
            continue
        layer = item
        in_h = block_h if layer.prefix.endswith(("_conv1", "_downsample")) else h
        out_h = (in_h + 2 * layer.pad - layer.kernel) // layer.stride + 1
        conv_flops += 2.0 * batch * out_h * out_h * layer.cout * layer.cin * layer.kernel ** 2
        conv_bytes += 4.0 * (batch * layer.cin * in_h * in_h + layer.cout * layer.cin * layer.kernel ** 2
                             + batch * layer.cout * out_h * out_h)
        if not layer.prefix.endswith("_downsample"):
            h = out_h
    return {"conv_flops": conv_flops, "conv_bytes": conv_bytes,
            "total_flops": conv_flops + 2.0 * batch * 2048 * 1000}


def run_resnet(args, world, rank, local, peaks, peak_kind) -> dict:
    import torch

    import cutriton_b200 as ct
    from cutriton_b200 import workloads

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    batch = args.batch
    weights = workloads.resnet50_weights("baseline", seed=0)
    model = workloads.build_resnet50(weights, batch=batch)
    # The headline runs without per-op profiling events (as a user would run
    # it); a second engine with profiling gives the per-op conv times for the
    # roofline afterwards, outside the timed region.
    # Candidate choice: TuneOnMiss times every numerically valid candidate of
    # each op on its first run (the warm-up, outside the timed region) and
    # caches the choice; every later engine and context of this run reads it.
    tuning = bench_tuning(args, rank)
    engine = ct.build_engine(model, device_id=local, enable_cuda_graph=True, enable_profiling=False,
                             enable_residual_fusion=True, **tuning)
    ctx = engine.create_context()
    x_host = workloads.resnet50_input(batch, seed=rank)
    x = torch.from_numpy(x_host).to(device)
    y = torch.empty(batch, 1000, device=device)
    ctx.bind_tensor("input", x)
    ctx.bind_tensor("output", y, output=True)
    stream = torch.cuda.Stream(device)
    for _ in range(max(3, args.warmup)):
        ctx.run_async(stream.cuda_stream)
        ctx.synchronize()

    launches = kernel_launches_per_run(engine, ctx)
    tuned_off_default = [{"op": op["node"], "default": op["candidates"][op["default"]].split(":", 1)[-1],
                          "chosen": op["candidates"][ctx.selected_candidate(i)].split(":", 1)[-1]}
                         for i, op in enumerate(engine.ops()) if ctx.selected_candidate(i) != op["default"]]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        # One event per step boundary (same stream, no extra synchronisation)
        # for the per-step median / p95 the reference harness reports.
        marks = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
        start.record(stream)
        marks[0].record(stream)
        for i in range(args.steps):
            ctx.run_async(stream.cuda_stream)
            marks[i + 1].record(stream)
            ctx.synchronize()  # the reference harness synchronizes every run
        end.record(stream)
        torch.cuda.synchronize()
        barrier(world)
    elapsed_ms = max_over_ranks(start.elapsed_time(end), world)
    step_ms = [marks[i].elapsed_time(marks[i + 1]) for i in range(args.steps)]
    clock_summary = clocks.summary()
    logits = y.cpu().numpy()  # after the timed region: the parity check's input

    # Per-op conv times (engine profiler: CUDA events around each op).
    prof_engine = ct.build_engine(model, device_id=local, enable_cuda_graph=True, enable_profiling=True,
                                  enable_residual_fusion=True, **tuning)
    prof_ctx = prof_engine.create_context()
    prof_ctx.bind_tensor("input", x)
    prof_ctx.bind_tensor("output", y, output=True)
    op_types = [o["op_type"] for o in prof_engine.ops()]
    conv_ops = [i for i, t in enumerate(op_types) if "Conv" in t]
    conv_ms = []
    for step in range(3 + min(args.steps, 5)):
        prof_ctx.run_async(stream.cuda_stream)
        prof_ctx.synchronize()
        if step >= 3:
            events = prof_ctx.profile_events()
            conv_ms.append(sum(events[i][1] for i in conv_ops))
    del prof_ctx, prof_engine
    ms_per_step = elapsed_ms / args.steps
    value = world * batch * args.steps / (elapsed_ms / 1e3)

    work = resnet_work(batch)
    conv_ms_avg = float(np.mean(conv_ms))
    achieved_tflops = work["conv_flops"] / (conv_ms_avg / 1e3) / 1e12
    # FP32 convolutions run as 3xTF32 on the tensor cores: 3 TF32 MMAs (TF32
    # = half the BF16 rate) per FP32 multiply-add, so the FP32-equivalent
    # ceiling is bf16_tflops / 6 of the measured BF16 peak. Each conv launch
    # lasts 0.1-1 ms at full clock, so the burst figure is the basis; the
    # sustained (power-capped, seconds-long) one is reported beside it.
    peak_tflops = peaks["bf16_tflops"] / 6.0
    peak_sustained = peaks["bf16_tflops_sustained"] / 6.0
    result = {
        "value": value, "ms_per_step": ms_per_step, "launches_per_step": launches, "clocks": clock_summary,
        "step_ms": {"median": float(np.median(step_ms)), "p95": float(np.percentile(step_ms, 95)),
                    "note": "this rank's per-step event times; value uses the whole timed region, max over ranks"},
        "roofline": {
            "bound": "tensor", "kernel": "FP32 convolution family (all conv ops of one step)",
            "achieved": achieved_tflops, "peak": peak_tflops, "unit": "TFLOP/s",
            "frac": achieved_tflops / peak_tflops,
            "frac_sustained_basis": achieved_tflops / peak_sustained,
            # For transparency: the same FLOPs against a plain (1xTF32) basis,
            # half the measured BF16 rate; 3xTF32 issues three MMAs per MAC.
            "frac_vs_plain_tf32": achieved_tflops / (peaks["bf16_tflops"] / 2.0),
            "peak_basis": f"{peak_kind} bf16_tflops (burst) {peaks['bf16_tflops']} / 6 (3xTF32 FP32-equivalent); "
                          f"frac_sustained_basis uses bf16_tflops_sustained {peaks['bf16_tflops_sustained']} / 6",
            "conv_ms_per_step": conv_ms_avg, "algorithmic_gflop_per_step": work["conv_flops"] / 1e9,
            "hbm_frac_at_min_bytes": (work["conv_bytes"] / (conv_ms_avg / 1e3) / 1e9) / peaks["hbm_gbs"],
            # DRAM bytes (read + write) of the 53 conv launches of one bs256 step
            # from an ncu capture (not measured live).
            "traffic": CONV_DRAM_BYTES_PER_STEP_BS256 * batch / 256,
            "traffic_unit": "bytes per step (ncu dram__bytes_read.sum + dram__bytes_write.sum)",
            "min_bytes": work["conv_bytes"],
        },
        "whole_net_tflops": work["total_flops"] / (ms_per_step / 1e3) / 1e12,
        "images": x_host, "logits": logits,
        "tuning": {"mode": args.tuning, "ops": len(engine.ops()), "tuned_off_default": tuned_off_default},
    }

    if not args.no_e2e:
        pinned = torch.from_numpy(x_host).pin_memory()
        host_in = pinned.numpy()
        host_outs = [torch.empty(batch, 1000).pin_memory().numpy() for _ in range(2)]
        steps = max(6, args.steps)
        # Serial: one context, each call waits for its own copies.
        ctx.run_host({"input": host_in}, {"output": host_outs[0]}, stream=stream.cuda_stream)
        barrier(world)
        torch.cuda.synchronize()
        e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_start.record(stream)
        for _ in range(steps):
            ctx.run_host({"input": host_in}, {"output": host_outs[0]}, stream=stream.cuda_stream)
        e_end.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        serial_ms = max_over_ranks(e_start.elapsed_time(e_end), world)
        # Pipelined: two contexts of the engine on two streams; step i+1's
        # host->device copy runs under step i's kernels.
        ctx2 = engine.create_context()
        ctx2.bind_tensor("input", torch.empty_like(x))
        ctx2.bind_tensor("output", torch.empty_like(y), output=True)
        stream2 = torch.cuda.Stream(device=device)
        ctxs, streams = [ctx, ctx2], [stream, stream2]
        for j in range(2):
            ctxs[j].run_host({"input": host_in}, {"output": host_outs[j]}, stream=streams[j].cuda_stream)
        barrier(world)
        torch.cuda.synchronize()
        e_start.record(stream)
        stream2.wait_event(e_start)
        for i in range(steps):
            j = i % 2
            if i >= 2:
                ctxs[j].synchronize()
            ctxs[j].run_host_async({"input": host_in}, {"output": host_outs[j]}, streams[j].cuda_stream)
        tail = torch.cuda.Event()
        tail.record(stream2)
        stream.wait_event(tail)
        e_end.record(stream)
        for c in ctxs:
            c.synchronize()
        torch.cuda.synchronize()
        barrier(world)
        e_ms = max_over_ranks(e_start.elapsed_time(e_end), world)
        del ctx2
        result["e2e"] = {"value": world * batch * steps / (e_ms / 1e3), "unit": "img/s",
                         "h2d_bytes_per_step": int(x_host.nbytes), "d2h_bytes_per_step": int(host_outs[0].nbytes),
                         "steps": steps,
                         "path": "ctb_context_run_host_async (C ABI): two contexts on two streams, pinned host buffers",
                         "h2d_gbs_per_rank": x_host.nbytes * steps / (e_ms / 1e3) / 1e9,
                         "h2d_gbs_all_ranks": world * x_host.nbytes * steps / (e_ms / 1e3) / 1e9,
                         "serial_value": world * batch * steps / (serial_ms / 1e3),
                         "serial_path": "ctb_context_run_host (C ABI), one context, waits every step"}
    return result


def run_ffn(args, world, rank, local, peaks, peak_kind) -> dict:
    import torch

    import cutriton_b200 as ct
    from cutriton_b200 import workloads

    device = torch.device("cuda", local)
    t, h, i = FFN["tokens"], FFN["hidden"], FFN["inner"]
    w = workloads.ffn_weights(h, i, seed=0)
    engine = ct.build_engine(workloads.build_ffn(w, t, h, i), device_id=local, enable_cuda_graph=True,
                             enable_profiling=False, **bench_tuning(args, rank))
    ctx = engine.create_context()
    x = torch.from_numpy(workloads.ffn_input(t, h, seed=rank)).to(device)
    y = torch.empty(t, h, dtype=torch.float16, device=device)
    ctx.bind_tensor("x", x)
    ctx.bind_tensor("output", y, output=True)
    # L2 flush buffer (inputs of this config fit in L2).
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)
    stream = torch.cuda.Stream(device)
    for _ in range(max(3, args.warmup)):
        ctx.run_async(stream.cuda_stream)
        ctx.synchronize()
    steps = max(20, args.steps * 5)
    times = []
    with torch.cuda.stream(stream):
        for _ in range(steps):
            flush.fill_(1.0)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            ctx.run_async(stream.cuda_stream)
            e.record(stream)
            ctx.synchronize()
            times.append(s.elapsed_time(e))
    kernels = chosen_kernels(engine, ctx)
    med = max_over_ranks(float(np.median(times)), world)
    p95 = max_over_ranks(float(np.percentile(times, 95)), world)
    flops = 4.0 * t * h * i
    tflops = flops / (med / 1e3) / 1e12
    return {"metric": "FFN FP16 tokens/s (M=4096, H=768, I=3072)", "value": world * t / (med / 1e3),
            "unit": "tokens/s", "ms_per_step": med, "ms_p95": p95, "tflops": tflops,
            "roofline": ffn_roofline(tflops, peaks, peak_kind, kernels),
            "scaling": "weak (config 1 per rank)", "l2": "flushed (256 MB write) before every timed step",
            "input": x.cpu().numpy(), "output": y.cpu().numpy(), "weights": w}


def ffn_roofline(tflops: float, peaks: dict, peak_kind: str, kernels: list[str]) -> dict:
    """FFN block (GemmGelu + Gemm + SkipLayerNorm) against the FP16 tensor
    peak: 4*H*I FLOPs per token; the kernels run well under a millisecond at
    full clock, so the burst BF16 figure (= FP16 rate) is the basis."""
    return {"bound": "tensor", "kernel": "FFN block: " + " + ".join(kernels),
            "achieved": tflops, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
            "frac": tflops / peaks["bf16_tflops"], "peak_basis": f"{peak_kind} bf16_tflops (burst)"}


def host_cpu() -> dict:
    """Model name and core count of the host CPU (lscpu), recorded with the CPU legs."""
    info = {"logical_cpus": os.cpu_count()}
    try:
        out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
        for row in out.splitlines():
            key, _, value = row.partition(":")
            if key.strip() in ("Model name", "Socket(s)", "Core(s) per socket", "Thread(s) per core"):
                info[key.strip().lower().replace("(s)", "s").replace(" ", "_")] = value.strip()
    except (OSError, subprocess.SubprocessError):
        pass
    return info


def resnet_parity_sample(batch: int) -> np.ndarray:
    """Images of the bs256 step whose logits are checked: the first and last
    eight (first and last pixel tiles of every layer) and the three around
    image 128 (tiles that straddle two images)."""
    picked = set(range(min(8, batch))) | set(range(max(0, batch - 8), batch))
    picked.update(i for i in (127, 128, 129) if i < batch)
    return np.array(sorted(picked), dtype=np.int64)


def cpu_resnet(steps: int | None, batch: int, seconds: float | None = None, threads: int | None = None,
               images: np.ndarray | None = None) -> dict:
    """The reference's CPU comparison path for ResNet-50 (PyTorch eager FP32,
    benchmarks/resnet50_compare.py:118-141, restated in oracle/torch_ref.py)
    on all host threads: one untimed warm-up step, then `steps` timed steps of
    `batch` images (or as many as fit in `seconds`, at least two). `images`
    replaces the seeded batch (the bench's own images). Both CPU legs of this
    file call it, so they measure the same thing; the logits of the last step
    come back under "logits"."""
    import torch

    from cutriton_b200 import workloads
    from oracle import torch_ref

    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    weights = workloads.resnet50_weights("baseline", seed=0)
    x = workloads.resnet50_input(batch, seed=0) if images is None else np.ascontiguousarray(images)
    batch = x.shape[0]
    torch_ref.resnet50_logits(x, weights)  # warm-up: one full step
    times = []
    t_end = time.perf_counter() + (seconds or 0.0)
    while True:
        t0 = time.perf_counter()
        logits = torch_ref.resnet50_logits(x, weights)
        times.append(time.perf_counter() - t0)
        if steps is not None and len(times) >= steps:
            break
        if steps is None and len(times) >= 2 and time.perf_counter() >= t_end:
            break
    total = sum(times)
    return {"value": batch * len(times) / total, "unit": "img/s", "cores": threads, "kind": "port",
            "ms_per_step": total / len(times) * 1e3, "steps": len(times), "batch_per_step": batch,
            "sample": f"PyTorch eager FP32 ResNet-50 on {threads} host threads, {len(times)} steps x {batch} images "
                      f"(bounded sample of the bs{RN_BATCH_PER_GPU} step)", "logits": logits}


def cpu_ffn(seconds: float = 3.0, threads: int | None = None, x: np.ndarray | None = None,
            weights: dict | None = None) -> dict:
    """The reference's PyTorch FFN (benchmarks/transformer_ffn_compare.py:52-60,
    restated as the two-GEMM block of config 1) in FP16 on the host CPU,
    full M=4096 per step; the output of the last step under "output"."""
    import torch

    from cutriton_b200 import workloads
    from oracle import torch_ref

    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    t, h, i = FFN["tokens"], FFN["hidden"], FFN["inner"]
    w = weights if weights is not None else workloads.ffn_weights(h, i, seed=0)
    x = x if x is not None else workloads.ffn_input(t, h, seed=0)
    torch_ref.ffn_output(x, w, dtype=torch.float16)
    times = []
    t_end = time.perf_counter() + seconds
    while len(times) < 2 or time.perf_counter() < t_end:
        t0 = time.perf_counter()
        out = torch_ref.ffn_output(x, w, dtype=torch.float16)
        times.append(time.perf_counter() - t0)
    med = float(np.median(times))
    return {"value": t / med, "unit": "tokens/s", "cores": threads, "kind": "port", "dtype": "f16",
            "sample": f"PyTorch eager FP16 FFN M={t} H={h} I={i} on {threads} host threads, median of {len(times)}",
            "output": out}


def cpu_baseline(rn: dict, ffn: dict | None, seconds: float = 10.0, timed: bool = True) -> dict:
    """The CPU leg of the main line (rank 0). Times the reference's CPU path
    for about `seconds` on the parity sample of this rank's own bs256 images
    (and the FFN block on the bench's FFN input), and checks the GPU results
    of the bench against those CPU results:

    * ResNet-50 logits: max|d| <= 1e-3 * max|logit|, identical top-1;
    * FFN output: max|d| <= 2e-2.

    With `timed` False (N > 1) only the parity part runs and no baseline is
    reported."""
    picked = resnet_parity_sample(rn["logits"].shape[0])
    cpu = cpu_resnet(None if timed else 1, len(picked), seconds=seconds if timed else None,
                     images=rn["images"][picked])
    ref = cpu.pop("logits").astype(np.float64)
    got = rn["logits"][picked].astype(np.float64)
    bound = 1e-3 * float(np.abs(ref).max())
    err = float(np.abs(got - ref).max())
    top1 = bool((got.argmax(axis=1) == ref.argmax(axis=1)).all())
    parity = {"resnet50": {"images": picked.tolist(), "max_abs": err, "bound": bound, "top1_equal": top1,
                           "pass": bool(err <= bound and top1 and np.isfinite(got).all()),
                           "against": "PyTorch eager FP32 on the host (oracle/torch_ref.py)"}}
    line = cpu if timed else {}
    if ffn is not None:
        fcpu = cpu_ffn(seconds=3.0 if timed else 0.0, x=ffn["input"], weights=ffn["weights"])
        fref = fcpu.pop("output").astype(np.float64)
        fgot = ffn["output"].astype(np.float64)
        ferr = float(np.abs(fgot - fref).max())
        parity["ffn"] = {"rows": int(fgot.shape[0]), "max_abs": ferr, "bound": 2e-2,
                         "pass": bool(ferr <= 2e-2 and np.isfinite(fgot).all()),
                         "against": "PyTorch eager FP16 on the host (oracle/torch_ref.py)"}
        if timed:
            line["ffn"] = fcpu
    if timed:
        line["host_cpu"] = host_cpu()
    return {"baseline": line if timed else None, "parity": parity}


def base_line(args, world) -> dict:
    return {
        "metric": "ResNet-50 FP32 inference img/s (bs256 per GPU, 224x224)",
        "unit": "img/s", "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) images, seeded Kaiming/BN/FC weights)",
        "config": {"workload": "resnet50_fp32_inference", "model": "ResNet-50 v1.5", "global_batch": args.batch * world,
                   "batch_per_gpu": args.batch, "image": "3x224x224 NCHW", "parallelism": f"dp{world} (batch shards)",
                   "l2": "inputs larger than L2 (154 MB/step)", "cuda_graph": True, "residual_fusion": True,
                   "tuning": args.tuning},
    }


def run_reference_arm(args) -> None:
    """`--impl reference`: the reference's CPU comparison path (cpu_resnet) on
    the host cores, rank 0 only; the other ranks of a torchrun launch exit
    at once. Each step runs as many images of the bs256 step as keep the whole
    run within about 150 s (all 256 when the host is fast enough)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    probe = cpu_resnet(1, 8)
    per_image_s = probe["ms_per_step"] / 1e3 / 8
    budget_s = 150.0
    batch = int(budget_s / max(1, args.steps) / per_image_s) // 8 * 8
    batch = max(8, min(RN_BATCH_PER_GPU, batch))
    cpu = cpu_resnet(args.steps, batch)
    line = base_line(args, world)
    line.update({"impl": "reference", "value": cpu["value"], "ms_per_step": cpu["ms_per_step"],
                 "batch_per_step": batch, "gpus_used": 0,
                 "compute": "host CPU on rank 0; the value does not depend on the number of GPUs launched",
                 "cpu_baseline": {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
                 "host_cpu": host_cpu(),
                 "e2e": {"value": cpu["value"], "unit": "img/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
    print(json.dumps(line), flush=True)


def main() -> None:
    args = parse_args()
    if args.profile_case:
        run_profile_case(args.profile_case)
        return
    if args.impl == "reference":
        run_reference_arm(args)
        return

    world, rank, local = dist_setup(args)
    peaks, peak_kind = load_peaks()
    if args.config is not None:
        if args.config == 4:
            line = run_config4(args, world, rank, local, peaks, peak_kind)
        elif rank == 0:
            line = run_config2(args) if args.config == 2 else run_config3(args, peaks)
        else:
            line = None
        if rank == 0:
            print(json.dumps(line), flush=True)
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
            dist.destroy_process_group()
        return
    rn = run_resnet(args, world, rank, local, peaks, peak_kind)
    ffn = None if args.no_ffn else run_ffn(args, world, rank, local, peaks, peak_kind)
    ffn4 = None if args.no_ffn else run_config4(args, world, rank, local, peaks, peak_kind)
    if rank == 0:
        line = base_line(args, world)
        line.update({"value": rn["value"], "ms_per_step": rn["ms_per_step"], "roofline": rn["roofline"],
                     "clocks": rn["clocks"], "gpu_launches": rn["launches_per_step"] * args.steps,
                     "whole_net_tflops": rn["whole_net_tflops"], "step_ms": rn["step_ms"], "tuning": rn["tuning"]})
        if "e2e" in rn:
            line["e2e"] = rn["e2e"]
        if ffn is not None:
            line["ffn"] = {k: v for k, v in ffn.items() if k not in ("input", "output", "weights")}
            line["ffn_config4"] = ffn4
        if not args.no_cpu_baseline:
            leg = cpu_baseline(rn, ffn, timed=(world == 1))
            line["parity"] = leg["parity"]
            if leg["baseline"] is not None:
                line["cpu_baseline"] = leg["baseline"]
        line["peaks"] = peak_kind
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
