"""Kernel descriptors of the sm_100a pack (consumed by :mod:`kernel_sdk`).

Argument lists bind exactly the values the reference kernels bind
(python/cutriton/triton_kernels/resnet.py:216-400, transformer.py:193-396),
so graphs lower to the same op set; the kernels themselves are this
package's CUDA sources under ``csrc/kernels``.
"""

from __future__ import annotations

from typing import Any

from .kernel_sdk import Arg, KernelSpec, Variant


def arg(arg_name: str, type_: str, kind: str, **source: Any) -> Arg:
    return Arg(arg_name, type_, {"kind": kind, **source})


RESERVED = (arg("runtime_scratch", "*i8", "runtime_reserved"), arg("profile_scratch", "*i8", "runtime_reserved"))


def literal(value: int) -> dict[str, Any]:
    return {"kind": "literal", "value": value}


def meta(name: str) -> dict[str, Any]:
    return {"kind": "meta", "name": name}


def ceil_div(a: dict[str, Any], b: dict[str, Any]) -> dict[str, Any]:
    return {"kind": "ceil_div", "args": [a, b]}


def mul(a: dict[str, Any], b: dict[str, Any]) -> dict[str, Any]:
    return {"kind": "mul", "args": [a, b]}


def out_dim(axis: int, index: int = 0) -> dict[str, Any]:
    return {"kind": "output_dim", "index": index, "axis": axis}


def out_numel(index: int = 0) -> dict[str, Any]:
    return {"kind": "output_numel", "index": index}


CONV_DIMS = (
    arg("n", "i32", "input_dim", index=0, axis=0),
    arg("c", "i32", "input_dim", index=0, axis=1),
    arg("h", "i32", "input_dim", index=0, axis=2),
    arg("w", "i32", "input_dim", index=0, axis=3),
    arg("k", "i32", "input_dim", index=1, axis=0),
    arg("r", "i32", "input_dim", index=1, axis=2),
    arg("s", "i32", "input_dim", index=1, axis=3),
    arg("out_h", "i32", "output_dim", index=0, axis=2),
    arg("out_w", "i32", "output_dim", index=0, axis=3),
    arg("stride_h", "i32", "attribute_i64", name="strides", index=0, default=1),
    arg("stride_w", "i32", "attribute_i64", name="strides", index=1, default=1),
    arg("pad_h", "i32", "attribute_i64", name="pads", index=0, default=0),
    arg("pad_w", "i32", "attribute_i64", name="pads", index=1, default=0),
    arg("dilation_h", "i32", "attribute_i64", name="dilations", index=0, default=1),
    arg("dilation_w", "i32", "attribute_i64", name="dilations", index=1, default=1),
)
BN_TENSORS = tuple(arg(n, "*fp32", "input", index=i + 2) for i, n in enumerate(("scale", "bias", "mean", "variance")))
EPSILON = arg("epsilon", "fp32", "attribute_f64", name="batchnorm_epsilon", alternate_name="epsilon", default=1e-5)
# Output pixels (n * oh * ow) tiled by BLOCK_M, channels by BLOCK_N.
CONV_GRID = (
    ceil_div(mul(out_dim(0), mul(out_dim(2), out_dim(3))), meta("BLOCK_M")),
    ceil_div(out_dim(1), meta("BLOCK_N")),
)
SIMT_TILE = {"BLOCK_M": 64, "BLOCK_N": 64}


def _conv_specs() -> list[KernelSpec]:
    x_w = (arg("x", "*fp32", "input", index=0), arg("weight", "*fp32", "input", index=1))
    out = (arg("output", "*fp32", "output", index=0),)
    families = [
        ("conv.fp32.nchw", "Conv", "ctb_conv_f32_simt", x_w + out + CONV_DIMS + RESERVED),
        ("conv_bn.fp32.nchw", "FusedConvBatchNorm", "ctb_conv_bn_f32_simt",
         x_w + BN_TENSORS + out + CONV_DIMS + (EPSILON,) + RESERVED),
        ("conv_bn_relu.fp32.nchw", "FusedConvBatchNormRelu", "ctb_conv_bn_relu_f32_simt",
         x_w + BN_TENSORS + out + CONV_DIMS + (EPSILON,) + RESERVED),
        ("conv_bn_add_relu.fp32.nchw", "FusedConvBatchNormAddRelu", "ctb_conv_bn_add_relu_f32_simt",
         x_w + BN_TENSORS + (arg("residual", "*fp32", "input", index=6),) + out + CONV_DIMS + (EPSILON,) + RESERVED),
    ]
    specs = []
    for kernel_id, op_type, symbol, arguments in families:
        specs.append(KernelSpec(
            kernel_id=kernel_id, op_type=op_type, version=1, source="conv_simt.cu", symbol=symbol,
            arguments=arguments, grid=CONV_GRID, layout="NCHW",
            variants=(Variant("simt_m64n64", num_warps=8, meta=SIMT_TILE, default=False),),
        ))
    # 3xTF32 tcgen05 implicit GEMM: output channels on M, output pixels on N.
    tma_w = arg("tma_w", "tensormap", "tensor_map", tensor="input", index=1, box=[32, 128, 1], swizzle=128,
                prepack="conv_w_tf32x2_okpad")
    x = (arg("x", "*fp32", "input", index=0),)
    tc_families = [
        ("conv.fp32.nchw.tcgen05", "Conv", "ctb_conv_f32_tc", (tma_w,) + x + out + CONV_DIMS + RESERVED),
        ("conv_bn.fp32.nchw.tcgen05", "FusedConvBatchNorm", "ctb_conv_bn_f32_tc",
         (tma_w,) + x + BN_TENSORS + out + CONV_DIMS + (EPSILON,) + RESERVED),
        ("conv_bn_relu.fp32.nchw.tcgen05", "FusedConvBatchNormRelu", "ctb_conv_bn_relu_f32_tc",
         (tma_w,) + x + BN_TENSORS + out + CONV_DIMS + (EPSILON,) + RESERVED),
        ("conv_bn_add_relu.fp32.nchw.tcgen05", "FusedConvBatchNormAddRelu", "ctb_conv_bn_add_relu_f32_tc",
         (tma_w,) + x + BN_TENSORS + (arg("residual", "*fp32", "input", index=6),) + out + CONV_DIMS
         + (EPSILON,) + RESERVED),
    ]
    # Persistent: min(#tiles, #SMs) CTAs walk the 128-channel x 128-pixel tiles.
    tiles = mul(ceil_div(mul(out_dim(0), mul(out_dim(2), out_dim(3))), meta("BLOCK_PIXELS")),
                ceil_div(out_dim(1), meta("BLOCK_CHANNELS")))
    tc_grid = ({"kind": "min", "args": [tiles, {"kind": "sm_count"}]},)
    # Activation operand in TMEM (pixels on M, channels on N): the default.
    # BLOCK_CHANNELS=128 counts the tiles for both of the kernel's channel
    # tilings (64 when Cout <= 64, else 128).
    tma_w64 = arg("tma_w", "tensormap", "tensor_map", tensor="input", index=1, box=[32, 64, 1], swizzle=128,
                  prepack="conv_w_tf32x2_cb")
    def tm_smem(n128: int, n64: int, slots: int, a_ring: int) -> int:
        # weight stages + barriers + k-chunk table + epilogue staging ring +
        # activation ring + alignment slack
        return max(n128 * 32768, n64 * 16384) + 512 + 1024 + slots * 16384 + a_ring * 16384 + 1024

    def tm_defines(n128: int, n64: int, slots: int, ahead: int, a_tma: int) -> dict[str, str]:
        return {"CTB_TM_STAGES_N128": str(n128), "CTB_TM_STAGES_N64": str(n64), "CTB_TM_SLOTS": str(slots),
                "CTB_TM_LOAD_AHEAD": str(ahead), "CTB_TM_A_TMA": str(a_tma), "CTB_TM_IMAGE_TILES": "0",
                # One gather group with two epilogue halves (CTB_TM_EPI_WARPS=8) was
                # measured slower for the 1x1 variant too: the gather limits it.
                "CTB_TM_GATHER_GROUPS": "2", "CTB_TM_EPI_WARPS": "4", "CTB_TM_SPLIT_N": "1"}

    # Epilogue tensor copies over the [N][K][H*W] view (optional: bound as
    # zeros when H*W*4 is not a multiple of 16; the kernel then stores from
    # registers). tma_x: activation blocks of the 1x1 variant.
    tma_out = arg("tma_out", "tensormap", "tensor_map", tensor="output", index=0, box=[128, 32, 1], merge_inner=2,
                  optional=1)
    tma_res = arg("tma_res", "tensormap", "tensor_map", tensor="input", index=6, box=[128, 32, 1], merge_inner=2,
                  optional=1)
    tma_x = arg("tma_x", "tensormap", "tensor_map", tensor="input", index=0, box=[128, 32, 1], merge_inner=2,
                optional=1)
    one_by_one = (
        {"kind": "dim_le", "source": "input", "index": 1, "axis": 2, "value": 1},
        {"kind": "dim_le", "source": "input", "index": 1, "axis": 3, "value": 1},
        {"kind": "attribute_list_eq", "name": "strides", "value": [1, 1], "default": [1, 1]},
        {"kind": "attribute_list_eq", "name": "pads", "value": [0, 0, 0, 0], "default": [0, 0, 0, 0]},
        # H a multiple of 4 and W even (the 56x56 and 28x28 layers): H*W % 4 == 0, so every
        # image-aligned tile moves by tensor copies. At 14x14 two of three 128-pixel tiles
        # straddle two images and fall back to global loads anyway; there the general
        # sibling was measured 17 % faster (256->1024, 1024->256 and 1024->512 at N=256),
        # so those layers lower to it.
        {"kind": "dim_multiple_of", "source": "output", "index": 0, "axis": 2, "value": 4},
        {"kind": "dim_multiple_of", "source": "output", "index": 0, "axis": 3, "value": 2},
    )
    # Input windows of the small-channel variant: box {232 columns, 11 rows,
    # 4 channels, 1 image} of the NCHW input (the 7x7/2 stem's tile window).
    tma_xwin = arg("tma_xwin", "tensormap", "tensor_map", tensor="input", index=0, box=[232, 11, 4, 1], optional=1)
    tiny_box = {"tma_xwin": {"box": [4, 1, 1, 1]}}  # unused by the other variants
    window_bytes = 2 * 232 * 11 * 4 * 4
    for kernel_id, op_type, symbol, arguments in tc_families:
        with_window = op_type == "FusedConvBatchNormRelu"
        maps = ((tma_w64, tma_out) + ((tma_res,) if op_type.endswith("AddRelu") else ()) + (tma_x,)
                + ((tma_xwin,) if with_window else ()))
        overrides = tiny_box if with_window else {}
        variants = [
            # Any shape: activations gathered with global loads.
            Variant("persistent_m128n128k32_tmem_a_3xtf32", num_warps=14,
                    shared_memory_bytes=tm_smem(3, 6, 4, 0), defines=tm_defines(3, 6, 4, 2, 0),
                    meta={"BLOCK_PIXELS": 128, "BLOCK_CHANNELS": 128}, arg_overrides=overrides),
            # 1x1 / stride 1 / no padding: activation blocks by TMA. With a
            # residual, the epilogue's residual stream limits these layers: one
            # weight stage less for a 5-slot staging ring loading 3 chunks ahead
            # (measured 4-7.5 % faster on the ResNet shapes; 4.6 % slower without
            # a residual, so only for this family).
            Variant("persistent_m128n128k32_tmem_a_3xtf32_1x1tma", num_warps=14,
                    shared_memory_bytes=tm_smem(2, 5, 5, 4) if op_type.endswith("AddRelu") else tm_smem(3, 5, 4, 4),
                    defines=tm_defines(2, 5, 5, 3, 1) if op_type.endswith("AddRelu") else tm_defines(3, 5, 4, 2, 1),
                    meta={"BLOCK_PIXELS": 128, "BLOCK_CHANNELS": 128}, constraints=one_by_one, default=True,
                    arg_overrides=overrides),
        ]
        if with_window:
            # C <= 4 (the stem): listed first so it leads when the 1x1 default does not apply.
            variants.insert(0, Variant(
                "persistent_m128n128k32_tmem_a_3xtf32_window", num_warps=14,
                shared_memory_bytes=tm_smem(2, 4, 4, 0) + window_bytes,
                defines={**tm_defines(2, 4, 4, 2, 0), "CTB_TM_WINDOW": "1"},
                meta={"BLOCK_PIXELS": 128, "BLOCK_CHANNELS": 128},
                constraints=({"kind": "dim_le", "source": "input", "index": 1, "axis": 1, "value": 4},)))
        specs.append(KernelSpec(
            kernel_id=kernel_id.replace("tcgen05", "tcgen05_tmem"), op_type=op_type, version=1,
            source="conv_tm.cu", symbol=symbol.replace("_tc", "_tm"),
            arguments=maps + arguments[1:], grid=tc_grid, layout="NCHW",
            constraints=({"kind": "input_is_constant", "index": 1},), variants=tuple(variants)))
    for kernel_id, op_type, symbol, arguments in tc_families:
        stages = 3
        smem = stages * 65536 + 4 * 32 * 33 * 4 + 1024 + 256
        specs.append(KernelSpec(
            kernel_id=kernel_id, op_type=op_type, version=1, source="conv_tc.cu", symbol=symbol,
            arguments=arguments, grid=tc_grid, layout="NCHW",
            constraints=({"kind": "input_is_constant", "index": 1},),
            variants=(Variant(f"persistent_m128n128k32s{stages}_3xtf32", num_warps=10, shared_memory_bytes=smem,
                              meta={"BLOCK_PIXELS": 128, "BLOCK_CHANNELS": 128},
                              defines={"CTB_STAGES": str(stages)}, default=False),),
        ))
    specs.extend(_conv1x1_mn_specs(one_by_one))
    return specs


def _conv1x1_mn_specs(one_by_one: tuple[dict[str, Any], ...]) -> list[KernelSpec]:
    """1x1 / stride-1 / unpadded convolutions with the output channels on M
    (conv1x1_mn.cu): activations and results move as {32 px, 32 channel}
    boxes of the [N][C][H*W] view, no gather. Candidates next to the TMEM
    kernel; the tuner picks per layer."""
    box = dict(box=[32, 32, 1], swizzle=128, merge_inner=2, optional=1)
    w = arg("tma_w", "tensormap", "tensor_map", tensor="input", index=1, box=[32, 128, 1], swizzle=128,
            prepack="conv_w_tf32x2_cb")
    # X is the MN-major TF32 operand: 32-byte swizzle atoms (the tensor core's only layout for it).
    maps = (w, arg("tma_x", "tensormap", "tensor_map", tensor="input", index=0, swizzle_atom=32, **box),
            arg("tma_out", "tensormap", "tensor_map", tensor="output", index=0, **box))
    res_map = arg("tma_res", "tensormap", "tensor_map", tensor="input", index=6, **box)
    x = (arg("x", "*fp32", "input", index=0),)
    out = (arg("output", "*fp32", "output", index=0),)
    dims = (arg("n", "i32", "input_dim", index=0, axis=0), arg("c", "i32", "input_dim", index=0, axis=1),
            arg("h", "i32", "input_dim", index=0, axis=2), arg("w", "i32", "input_dim", index=0, axis=3),
            arg("k", "i32", "input_dim", index=1, axis=0))
    families = [
        ("conv.fp32.nchw.tcgen05_mn", "Conv", "ctb_conv1x1_f32_mn", maps + x + out + dims + RESERVED),
        ("conv_bn.fp32.nchw.tcgen05_mn", "FusedConvBatchNorm", "ctb_conv1x1_bn_f32_mn",
         maps + x + BN_TENSORS + out + dims + (EPSILON,) + RESERVED),
        ("conv_bn_relu.fp32.nchw.tcgen05_mn", "FusedConvBatchNormRelu", "ctb_conv1x1_bn_relu_f32_mn",
         maps + x + BN_TENSORS + out + dims + (EPSILON,) + RESERVED),
        ("conv_bn_add_relu.fp32.nchw.tcgen05_mn", "FusedConvBatchNormAddRelu", "ctb_conv1x1_bn_add_relu_f32_mn",
         maps + (res_map,) + x + BN_TENSORS + (arg("residual", "*fp32", "input", index=6),) + out + dims
         + (EPSILON,) + RESERVED),
    ]
    # 128 channels x 128 pixels of one image per tile; persistent.
    tiles = mul(out_dim(0), mul(ceil_div(mul(out_dim(2), out_dim(3)), literal(128)),
                                ceil_div(out_dim(1), literal(128))))
    grid = ({"kind": "min", "args": [tiles, {"kind": "sm_count"}]},)
    # 1x1 / stride 1 / unpadded (the first four of one_by_one), C a multiple
    # of 32, H and W even (H*W % 4 == 0: 16-byte rows for the tensor maps;
    # the 56x56, 28x28 and 14x14 layers).
    constraints = one_by_one[:4] + (
        {"kind": "dim_multiple_of", "source": "output", "index": 0, "axis": 2, "value": 2},
        {"kind": "dim_multiple_of", "source": "output", "index": 0, "axis": 3, "value": 2},
        {"kind": "input_is_constant", "index": 1},
        {"kind": "dim_multiple_of", "source": "input", "index": 0, "axis": 1, "value": 32},
    )
    def smem(op_type: str) -> int:
        # Stages of W_hi, W_lo, X_hi, X_lo (64 KB each: two with a residual,
        # three without) + four epilogue warps x {32 px, 32 channel} boxes
        # (two output boxes, plus four residual slots) + barriers + slack.
        residual = op_type.endswith("AddRelu")
        return (2 if residual else 3) * 65536 + 4 * (6 if residual else 2) * 4096 + 256 + 1024

    return [KernelSpec(kernel_id=kernel_id, op_type=op_type, version=1, source="conv1x1_mn.cu", symbol=symbol,
                       arguments=arguments, grid=grid, layout="NCHW", constraints=constraints,
                       variants=(Variant("persistent_co128px128k32_3xtf32", num_warps=10,
                                         shared_memory_bytes=smem(op_type), meta={"BLOCK_PIXELS": 128}),))
            for kernel_id, op_type, symbol, arguments in families]


def _elementwise_specs() -> list[KernelSpec]:
    specs = []
    chunk_f32 = {"CHUNK": 4096}
    chunk_f16 = {"CHUNK": 8192}
    grid = (ceil_div(out_numel(), meta("CHUNK")),)
    for kernel_id, op_type, symbol, inputs, dtype, chunk, layout in (
        ("relu.fp32", "Relu", "ctb_relu_f32", ("x",), "float32", chunk_f32, ""),
        ("add.fp32", "Add", "ctb_add_f32", ("a", "b"), "float32", chunk_f32, ""),
        ("add_relu.fp32", "AddRelu", "ctb_add_relu_f32", ("a", "b"), "float32", chunk_f32, ""),
        ("gelu.fp16", "Gelu", "ctb_gelu_f16", ("x",), "float16", chunk_f16, ""),
        ("add.fp16", "Add", "ctb_add_f16", ("a", "b"), "float16", chunk_f16, ""),
    ):
        ptr = "*fp32" if dtype == "float32" else "*fp16"
        arguments = tuple(arg(n, ptr, "input", index=i) for i, n in enumerate(inputs)) + (
            arg("output", ptr, "output", index=0),
            arg("total", "i32", "output_numel", index=0),
        ) + RESERVED
        specs.append(KernelSpec(
            kernel_id=kernel_id, op_type=op_type, version=1, source="elementwise.cu", symbol=symbol,
            arguments=arguments, grid=grid, dtype=dtype, layout=layout,
            variants=(Variant("vec16b", num_warps=8, meta=chunk, default=True),),
        ))
    bn_arguments = (
        arg("x", "*fp32", "input", index=0),
        arg("scale", "*fp32", "input", index=1),
        arg("bias", "*fp32", "input", index=2),
        arg("mean", "*fp32", "input", index=3),
        arg("variance", "*fp32", "input", index=4),
        arg("output", "*fp32", "output", index=0),
        arg("total", "i32", "output_numel", index=0),
        arg("channels", "i32", "input_dim", index=0, axis=1),
        arg("spatial", "i32", "input_dim_product", index=0, begin_axis=2),
        arg("epsilon", "fp32", "attribute_f64", name="epsilon", alternate_name="batchnorm_epsilon", default=1e-5),
    ) + RESERVED
    specs.append(KernelSpec(
        kernel_id="batch_norm.fp32.nchw", op_type="BatchNormalization", version=1, source="elementwise.cu",
        symbol="ctb_batch_norm_f32", arguments=bn_arguments, grid=grid, layout="NCHW",
        variants=(Variant("vec16b", num_warps=8, meta=chunk_f32, default=True),),
    ))
    return specs


def _pool_specs() -> list[KernelSpec]:
    pool_arguments = (
        arg("x", "*fp32", "input", index=0),
        arg("output", "*fp32", "output", index=0),
        arg("n", "i32", "input_dim", index=0, axis=0),
        arg("c", "i32", "input_dim", index=0, axis=1),
        arg("h", "i32", "input_dim", index=0, axis=2),
        arg("w", "i32", "input_dim", index=0, axis=3),
        arg("out_h", "i32", "output_dim", index=0, axis=2),
        arg("out_w", "i32", "output_dim", index=0, axis=3),
        arg("kernel_h", "i32", "attribute_i64", name="kernel_shape", index=0, default=1),
        arg("kernel_w", "i32", "attribute_i64", name="kernel_shape", index=1, default=1),
        arg("stride_h", "i32", "attribute_i64", name="strides", index=0, default=1),
        arg("stride_w", "i32", "attribute_i64", name="strides", index=1, default=1),
        arg("pad_h", "i32", "attribute_i64", name="pads", index=0, default=0),
        arg("pad_w", "i32", "attribute_i64", name="pads", index=1, default=0),
        arg("dilation_h", "i32", "attribute_i64", name="dilations", index=0, default=1),
        arg("dilation_w", "i32", "attribute_i64", name="dilations", index=1, default=1),
    ) + RESERVED
    gap_arguments = (
        arg("x", "*fp32", "input", index=0),
        arg("output", "*fp32", "output", index=0),
        arg("n", "i32", "input_dim", index=0, axis=0),
        arg("c", "i32", "input_dim", index=0, axis=1),
        arg("h", "i32", "input_dim", index=0, axis=2),
        arg("w", "i32", "input_dim", index=0, axis=3),
    ) + RESERVED
    return [
        KernelSpec(
            kernel_id="max_pool.fp32.nchw", op_type="MaxPool", version=1, source="pool.cu",
            symbol="ctb_max_pool_f32", arguments=pool_arguments, layout="NCHW",
            grid=(ceil_div(out_numel(), meta("BLOCK")),),
            variants=(Variant("thread_per_output", num_warps=8, meta={"BLOCK": 256}, default=False),),
        ),
        # 3x3/2 pad 1 with W % 4 == 0 and W <= 128: warp per output row, float4 rows.
        KernelSpec(
            kernel_id="max_pool_3x3s2.fp32.nchw", op_type="MaxPool", version=1, source="pool.cu",
            symbol="ctb_max_pool_3x3s2_f32",
            arguments=(arg("x", "*fp32", "input", index=0), arg("output", "*fp32", "output", index=0),
                       arg("n", "i32", "input_dim", index=0, axis=0), arg("c", "i32", "input_dim", index=0, axis=1),
                       arg("h", "i32", "input_dim", index=0, axis=2), arg("w", "i32", "input_dim", index=0, axis=3),
                       arg("out_h", "i32", "output_dim", index=0, axis=2),
                       arg("out_w", "i32", "output_dim", index=0, axis=3)) + RESERVED,
            layout="NCHW", grid=(ceil_div(mul(out_dim(0), mul(out_dim(1), out_dim(2))), meta("ROWS")),),
            constraints=(
                {"kind": "attribute_list_eq", "name": "kernel_shape", "value": [3, 3], "default": [0, 0]},
                {"kind": "attribute_list_eq", "name": "strides", "value": [2, 2], "default": [1, 1]},
                {"kind": "attribute_list_eq", "name": "pads", "value": [1, 1, 1, 1], "default": [0, 0, 0, 0]},
                {"kind": "attribute_list_eq", "name": "dilations", "value": [1, 1], "default": [1, 1]},
                {"kind": "dim_multiple_of", "source": "input", "index": 0, "axis": 3, "value": 4},
                {"kind": "dim_le", "source": "input", "index": 0, "axis": 3, "value": 128},
                {"kind": "dim_multiple_of", "source": "input", "index": 0, "axis": 2, "value": 2},
            ),
            variants=(Variant("warp_per_row_vec4", num_warps=8, meta={"ROWS": 8}, default=True),),
        ),
        KernelSpec(
            kernel_id="global_average_pool.fp32.nchw", op_type="GlobalAveragePool", version=1, source="pool.cu",
            symbol="ctb_global_average_pool_f32", arguments=gap_arguments, layout="NCHW",
            grid=(ceil_div(out_numel(), meta("PLANES")),),
            variants=(Variant("warp_per_plane", num_warps=8, meta={"PLANES": 8}, default=False),),
        ),
        # Planes of at most 81 elements (9x9): 128 planes per block staged in
        # shared memory by cp.async, one serial sum per thread.
        KernelSpec(
            kernel_id="global_average_pool_staged.fp32.nchw", op_type="GlobalAveragePool", version=1,
            source="pool.cu", symbol="ctb_global_average_pool_f32_staged", arguments=gap_arguments, layout="NCHW",
            grid=(ceil_div(out_numel(), meta("PLANES")),),
            constraints=(
                {"kind": "dim_le", "source": "input", "index": 0, "axis": 2, "value": 9},
                {"kind": "dim_le", "source": "input", "index": 0, "axis": 3, "value": 9},
            ),
            variants=(Variant("block_of_128_planes", num_warps=4, meta={"PLANES": 128}, default=True),),
        ),
    ]


GEMM_CONSTRAINTS = (
    {"kind": "input_count_eq", "value": 2},
    {"kind": "attribute_i64_eq", "name": "transA", "value": 0, "default": 0},
    {"kind": "attribute_i64_eq", "name": "transB", "value": 0, "default": 0},
    {"kind": "tensor_rank_eq", "source": "input", "index": 0, "value": 2},
    {"kind": "tensor_rank_eq", "source": "input", "index": 1, "value": 2},
)


def _gemm_specs() -> list[KernelSpec]:
    def gemm_args(ptr: str) -> tuple[Arg, ...]:
        return (
            arg("a", ptr, "input", index=0),
            arg("b", ptr, "input", index=1),
            arg("output", ptr, "output", index=0),
            arg("m", "i32", "output_dim", index=0, axis=0),
            arg("n", "i32", "output_dim", index=0, axis=1),
            arg("k", "i32", "input_dim", index=0, axis=1),
        ) + RESERVED

    grid = (ceil_div(out_dim(0), meta("BLOCK_M")), ceil_div(out_dim(1), meta("BLOCK_N")))

    def tc_args(block_n: int) -> tuple[Arg, ...]:
        return (
            arg("tma_a", "tensormap", "tensor_map", tensor="input", index=0, box=[64, 128], swizzle=128),
            arg("tma_b", "tensormap", "tensor_map", tensor="input", index=1, box=[64, block_n], swizzle=128,
                prepack="transpose_2d"),
            arg("output", "*fp16", "output", index=0),
            arg("m", "i32", "output_dim", index=0, axis=0),
            arg("n", "i32", "output_dim", index=0, axis=1),
            arg("k", "i32", "input_dim", index=0, axis=1),
        ) + RESERVED

    tc_constraints = GEMM_CONSTRAINTS + (
        {"kind": "input_is_constant", "index": 1},
        {"kind": "dim_multiple_of", "source": "input", "index": 0, "axis": 1, "value": 8},
        {"kind": "dim_multiple_of", "source": "output", "index": 0, "axis": 1, "value": 8},
    )

    def tc_variants() -> tuple[Variant, ...]:
        out = []
        for block_n, stages, default in ((128, 4, False), (128, 3, False), (256, 3, False)):
            smem = stages * (128 * 64 * 2 + block_n * 64 * 2) + 1024 + 256
            out.append(Variant(f"m128n{block_n}k64s{stages}", num_warps=4, shared_memory_bytes=smem,
                               meta={"BLOCK_M": 128, "BLOCK_N": block_n},
                               defines={"CTB_BLOCK_N": str(block_n), "CTB_STAGES": str(stages)}, default=default,
                               arg_overrides={"tma_b": {"box": [64, block_n]}}))
        return tuple(out)

    # Persistent: min(#128x128 tiles, #SMs) CTAs; the kernel picks 256- or
    # 128-wide tiles at run time.
    tp_args = (
        arg("tma_a", "tensormap", "tensor_map", tensor="input", index=0, box=[64, 128], swizzle=128),
        arg("tma_b", "tensormap", "tensor_map", tensor="input", index=1, box=[64, 128], swizzle=128,
            prepack="transpose_2d"),
        arg("tma_out", "tensormap", "tensor_map", tensor="output", index=0, box=[32, 32], swizzle=64, optional=1),
        arg("output", "*fp16", "output", index=0),
        arg("m", "i32", "output_dim", index=0, axis=0),
        arg("n", "i32", "output_dim", index=0, axis=1),
        arg("k", "i32", "input_dim", index=0, axis=1),
    ) + RESERVED
    tp_grid = ({"kind": "min", "args": [mul(ceil_div(out_dim(0), meta("BLOCK_M")), ceil_div(out_dim(1), meta("BLOCK_N"))),
                                        {"kind": "sm_count"}]},)
    tp_variant = Variant("persistent_m128n256k64_2acc", num_warps=18, shared_memory_bytes=196608 + 32768 + 256 + 1024,
                         meta={"BLOCK_M": 128, "BLOCK_N": 128}, default=True, programmatic_launch=True)
    # CTA pairs (clusters of two SMs, tcgen05 cta_group::2): 2 x min(#256x128
    # pair tiles, #SMs / 2) CTAs. The kernel picks 256-, 192- or 128-wide
    # tiles at run time; each CTA reads its half of B^T through the map of
    # that half width.
    pair_args = (
        arg("tma_a", "tensormap", "tensor_map", tensor="input", index=0, box=[64, 128], swizzle=128),
        *(arg(f"tma_b{rows}", "tensormap", "tensor_map", tensor="input", index=1, box=[64, rows], swizzle=128,
              prepack="transpose_2d") for rows in (128, 96, 64)),
        arg("tma_out", "tensormap", "tensor_map", tensor="output", index=0, box=[32, 32], swizzle=64, optional=1),
        arg("output", "*fp16", "output", index=0),
        arg("m", "i32", "output_dim", index=0, axis=0),
        arg("n", "i32", "output_dim", index=0, axis=1),
        arg("k", "i32", "input_dim", index=0, axis=1),
    ) + RESERVED
    pair_grid = (mul(literal(2), {"kind": "min", "args": [
        mul(ceil_div(out_dim(0), literal(256)), ceil_div(out_dim(1), literal(128))),
        ceil_div({"kind": "sm_count"}, literal(2))]}),)
    pair_variant = Variant("pair_m256n256k64_2acc", num_warps=18, shared_memory_bytes=196608 + 32768 + 256 + 1024,
                           meta={"BLOCK_M": 256, "BLOCK_N": 128}, programmatic_launch=True)
    tc = [
        KernelSpec(kernel_id="gemm.fp16.tcgen05_persistent", op_type="Gemm", version=1, source="gemm_f16_tp.cu",
                   symbol="ctb_gemm_f16_tp", arguments=tp_args, grid=tp_grid, dtype="float16",
                   constraints=tc_constraints, variants=(tp_variant,)),
        KernelSpec(kernel_id="gemm_gelu.fp16.tcgen05_persistent", op_type="GemmGelu", version=1,
                   source="gemm_f16_tp.cu", symbol="ctb_gemm_gelu_f16_tp", arguments=tp_args, grid=tp_grid,
                   dtype="float16", constraints=tc_constraints, variants=(tp_variant,)),
        KernelSpec(kernel_id="gemm.fp16.tcgen05_pair", op_type="Gemm", version=1, source="gemm_f16_2sm.cu",
                   symbol="ctb_gemm_f16_2sm", arguments=pair_args, grid=pair_grid, dtype="float16",
                   constraints=tc_constraints, variants=(pair_variant,)),
        KernelSpec(kernel_id="gemm_gelu.fp16.tcgen05_pair", op_type="GemmGelu", version=1,
                   source="gemm_f16_2sm.cu", symbol="ctb_gemm_gelu_f16_2sm", arguments=pair_args, grid=pair_grid,
                   dtype="float16", constraints=tc_constraints, variants=(pair_variant,)),
        KernelSpec(kernel_id="gemm.fp16.tcgen05", op_type="Gemm", version=1, source="gemm_f16_tc.cu",
                   symbol="ctb_gemm_f16_tc", arguments=tc_args(128), grid=grid, dtype="float16",
                   constraints=tc_constraints, variants=tc_variants()),
        KernelSpec(kernel_id="gemm_gelu.fp16.tcgen05", op_type="GemmGelu", version=1, source="gemm_f16_tc.cu",
                   symbol="ctb_gemm_gelu_f16_tc", arguments=tc_args(128), grid=grid, dtype="float16",
                   constraints=tc_constraints, variants=tc_variants()),
    ]
    # FP32 Gemm on the tensor cores: the TMEM conv kernel (3xTF32) as a 1x1
    # convolution over M "pixels" with H = W = 1; B [K, N] prepacked to the
    # K-major hi / lo planes [2][N][K] ("gemm_w_tf32x2_nk"). Its tensor maps
    # over the output / input do not fit a rank-2 tensor and are bound as
    # zeros, which selects the kernel's register-path epilogue.
    one = {"default": 1}
    zero = {"default": 0}
    fp32_tm_args = (
        arg("tma_w", "tensormap", "tensor_map", tensor="input", index=1, box=[32, 64, 1], swizzle=128,
            prepack="gemm_w_tf32x2_nk"),
        arg("tma_out", "tensormap", "tensor_map", tensor="output", index=0, box=[128, 32, 1], merge_inner=2,
            optional=1),
        arg("tma_x", "tensormap", "tensor_map", tensor="input", index=0, box=[128, 32, 1], merge_inner=2,
            optional=1),
        arg("x", "*fp32", "input", index=0),
        arg("output", "*fp32", "output", index=0),
        arg("n", "i32", "input_dim", index=0, axis=0),
        arg("c", "i32", "input_dim", index=0, axis=1),
        arg("h", "i32", "literal_i32", **one), arg("w", "i32", "literal_i32", **one),
        arg("k", "i32", "output_dim", index=0, axis=1),
        arg("r", "i32", "literal_i32", **one), arg("s", "i32", "literal_i32", **one),
        arg("out_h", "i32", "literal_i32", **one), arg("out_w", "i32", "literal_i32", **one),
        arg("stride_h", "i32", "literal_i32", **one), arg("stride_w", "i32", "literal_i32", **one),
        arg("pad_h", "i32", "literal_i32", **zero), arg("pad_w", "i32", "literal_i32", **zero),
        arg("dilation_h", "i32", "literal_i32", **one), arg("dilation_w", "i32", "literal_i32", **one),
    ) + RESERVED
    fp32_tm_grid = ({"kind": "min", "args": [mul(ceil_div(out_dim(0), literal(128)), ceil_div(out_dim(1), literal(128))),
                                             {"kind": "sm_count"}]},)
    fp32_tm_smem = 3 * 32768 + 512 + 1024 + 4 * 16384 + 1024
    fp32_tm = KernelSpec(
        kernel_id="gemm.fp32.tcgen05_tmem", op_type="Gemm", version=1, source="conv_tm.cu", symbol="ctb_conv_f32_tm",
        arguments=fp32_tm_args, grid=fp32_tm_grid,
        constraints=GEMM_CONSTRAINTS + ({"kind": "input_is_constant", "index": 1},
                                        {"kind": "dim_multiple_of", "source": "input", "index": 0, "axis": 1,
                                         "value": 4}),
        variants=(Variant("persistent_m128n128k32_tmem_a_3xtf32", num_warps=14, shared_memory_bytes=fp32_tm_smem,
                          defines={"CTB_TM_STAGES_N128": "3", "CTB_TM_STAGES_N64": "6", "CTB_TM_SLOTS": "4",
                                   "CTB_TM_LOAD_AHEAD": "2", "CTB_TM_A_TMA": "0", "CTB_TM_IMAGE_TILES": "0",
                                   "CTB_TM_GATHER_GROUPS": "2", "CTB_TM_EPI_WARPS": "4", "CTB_TM_SPLIT_N": "1"}, default=True),),
    )
    return tc + [fp32_tm] + [
        KernelSpec(
            kernel_id="gemm.fp32", op_type="Gemm", version=1, source="conv_simt.cu", symbol="ctb_gemm_f32_simt",
            arguments=gemm_args("*fp32"), grid=grid, constraints=GEMM_CONSTRAINTS,
            variants=(Variant("simt_m64n64", num_warps=8, meta=SIMT_TILE, default=False),),
        ),
        KernelSpec(
            kernel_id="gemm.fp16.wmma", op_type="Gemm", version=1, source="gemm_f16_wmma.cu",
            symbol="ctb_gemm_f16_wmma", arguments=gemm_args("*fp16"), grid=grid, dtype="float16",
            constraints=GEMM_CONSTRAINTS,
            variants=(Variant("m128n128k32", num_warps=8, meta={"BLOCK_M": 128, "BLOCK_N": 128}, default=False),),
        ),
        KernelSpec(
            kernel_id="gemm_gelu.fp16.wmma", op_type="GemmGelu", version=1, source="gemm_f16_wmma.cu",
            symbol="ctb_gemm_gelu_f16_wmma", arguments=gemm_args("*fp16"), grid=grid, dtype="float16",
            constraints=GEMM_CONSTRAINTS,
            variants=(Variant("m128n128k32", num_warps=8, meta={"BLOCK_M": 128, "BLOCK_N": 128}, default=False),),
        ),
    ]


def _norm_specs() -> list[KernelSpec]:
    def norm_args(skip: bool) -> tuple[Arg, ...]:
        names = ("x", "residual", "scale", "bias") if skip else ("x", "scale", "bias")
        return tuple(arg(n, "*fp16", "input", index=i) for i, n in enumerate(names)) + (
            arg("output", "*fp16", "output", index=0),
            arg("rows", "i32", "input_dim", index=0, axis=0),
            arg("columns", "i32", "input_dim", index=0, axis=1),
            arg("epsilon", "fp32", "attribute_f64", name="epsilon", default=1e-5),
        ) + RESERVED

    def row_constraints(inputs: int | None) -> tuple[dict[str, Any], ...]:
        out: tuple[dict[str, Any], ...] = (
            {"kind": "tensor_rank_eq", "source": "input", "index": 0, "value": 2},
            {"kind": "dim_le", "source": "input", "index": 0, "axis": 1, "value": 1024},
        )
        if inputs is not None:
            out = ({"kind": "input_count_eq", "value": inputs},) + out
        return out

    grid = (ceil_div(out_dim(0), meta("ROWS")),)
    softmax_args = (
        arg("x", "*fp16", "input", index=0),
        arg("output", "*fp16", "output", index=0),
        arg("rows", "i32", "input_dim", index=0, axis=0),
        arg("columns", "i32", "input_dim", index=0, axis=1),
    ) + RESERVED
    variants = (Variant("warp_per_row", num_warps=8, meta={"ROWS": 8}, default=True),)
    return [
        KernelSpec(kernel_id="layer_norm.fp16.last_axis", op_type="LayerNormalization", version=1,
                   source="norm.cu", symbol="ctb_layer_norm_f16", arguments=norm_args(False), grid=grid,
                   dtype="float16", constraints=row_constraints(3), variants=variants),
        KernelSpec(kernel_id="skip_layer_norm.fp16.last_axis", op_type="SkipLayerNormalization", version=1,
                   source="norm.cu", symbol="ctb_skip_layer_norm_f16", arguments=norm_args(True), grid=grid,
                   dtype="float16", constraints=row_constraints(4),
                   variants=(Variant("warp_per_row", num_warps=8, meta={"ROWS": 8}, default=True,
                                     programmatic_launch=True),)),
        KernelSpec(kernel_id="softmax.fp16.last_axis", op_type="Softmax", version=1, source="norm.cu",
                   symbol="ctb_softmax_f16", arguments=softmax_args, grid=grid, dtype="float16",
                   constraints=row_constraints(None), variants=variants),
    ]


def _diag_specs() -> list[KernelSpec]:
    """Failure-detection probe: a bounded wait that always expires, then y = x."""
    arguments = (
        arg("x", "*fp32", "input", index=0),
        arg("output", "*fp32", "output", index=0),
        arg("numel", "i32", "input_numel", index=0),
        arg("limit_us", "i32", "attribute_i64", name="limit_us", default=50000),
    ) + RESERVED
    return [KernelSpec(kernel_id="bounded_wait_probe.fp32", op_type="BoundedWaitProbe", version=1, source="diag.cu",
                       symbol="ctb_bounded_wait_probe_f32", arguments=arguments,
                       grid=({"kind": "min", "args": [ceil_div(out_numel(), literal(256)), literal(1024)]},),
                       variants=(Variant("single_waiter", num_warps=8, default=True),))]


def all_specs() -> list[KernelSpec]:
    return [*_conv_specs(), *_elementwise_specs(), *_pool_specs(), *_gemm_specs(), *_norm_specs(), *_diag_specs()]
