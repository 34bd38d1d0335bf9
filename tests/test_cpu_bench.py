"""CPU checks of the benchmark's accounting: the algorithmic work behind
`roofline.achieved`, the 23 distinct ResNet-50 conv shapes of config 3, and
the batch sharding of the multi-GPU runs. No GPU is touched."""

from __future__ import annotations

import bench


def test_resnet50_algorithmic_work_matches_the_stated_figures():
    # bs256: 4.0871 G conv MACs + 2.048 M FC MACs per image, multiply-add = 2 FLOP,
    # FP32 math counted once (not x3 for the split); conv I/O 22.39 GB minimum.
    work = bench.resnet_work(256)
    assert abs(work["total_flops"] / 1e9 - 2093.66) < 0.01
    assert abs(work["conv_flops"] / 1e9 - 2092.61) < 0.01
    assert abs(work["conv_bytes"] / 1e9 - 22.39) < 0.01
    # Work scales linearly with the batch (FLOPs exactly; bytes up to the constant weights).
    assert abs(bench.resnet_work(1)["total_flops"] * 256 - work["total_flops"]) < 1.0


def test_resnet50_has_23_distinct_conv_shapes():
    shapes = bench.conv_shapes()
    assert len(shapes) == 23
    assert shapes[0] == (3, 64, 7, 2, 3, 224)  # the stem
    assert (512, 512, 3, 1, 1, 7) in shapes  # last stage 3x3
    assert len(set(shapes)) == len(shapes)


def test_batch_shards_cover_the_global_batch_once():
    for global_batch in (256, 512, 2048, 1000, 7):
        for world in (1, 2, 3, 4, 8):
            spans = [bench.shard(global_batch, world, r) for r in range(world)]
            assert sum(count for _, count in spans) == global_batch
            starts = [start for start, _ in spans]
            assert starts == sorted(starts)
            for (s0, c0), (s1, _) in zip(spans, spans[1:]):
                assert s0 + c0 == s1
            counts = [count for _, count in spans]
            assert max(counts) - min(counts) <= 1


def test_peaks_come_from_the_measured_file_when_present():
    peaks, kind = bench.load_peaks()
    for key in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained"):
        assert peaks[key] > 0
    assert kind == ("measured" if bench.PEAKS_FILE.exists() else "fallback")


def test_reference_arm_under_torchrun_prints_one_line():
    """`bench.py --impl reference` launched like the GPU arm at N=2: rank 0
    times the CPU path and prints one JSON line, the other rank exits 0."""
    import json
    import socket
    import subprocess
    import sys

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), str(bench.REPO / "bench.py"),
           "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "1"]
    done = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=bench.REPO)
    assert done.returncode == 0, done.stderr[-2000:]
    lines = [l for l in done.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["n_gpus"] == 2 and line["value"] > 0
    assert line["cpu_baseline"]["value"] == line["value"] and line["e2e"]["h2d_bytes_per_step"] == 0


def test_cpu_leg_parity_check_passes_and_fails():
    """The CPU leg's parity check of the bench's GPU logits, fed CPU logits
    (pass) and the same logits with one entry pushed past the bound (fail)."""
    import numpy as np

    from cutriton_b200 import workloads
    from oracle import torch_ref

    batch = 16
    images = workloads.resnet50_input(batch, seed=0)
    picked = bench.resnet_parity_sample(batch)
    assert picked.tolist() == list(range(16))
    logits = np.zeros((batch, 1000), np.float32)
    logits[picked] = torch_ref.resnet50_logits(images[picked], workloads.resnet50_weights("baseline", seed=0))
    ok = bench.cpu_baseline({"images": images, "logits": logits}, None, timed=False)
    assert ok["baseline"] is None and ok["parity"]["resnet50"]["pass"]
    bad = logits.copy()
    bad[3, 7] += 10 * ok["parity"]["resnet50"]["bound"] + 1.0
    fail = bench.cpu_baseline({"images": images, "logits": bad}, None, timed=False)
    assert not fail["parity"]["resnet50"]["pass"]
