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
