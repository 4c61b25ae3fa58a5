"""The C-ABI library: loads, exports every declared symbol, and applies the
compile-error semantics on the host (no GPU, no compute calls)."""

import ctypes
import re
from pathlib import Path

import pytest

from gpu_optimizer_b200 import _lib
from gpu_optimizer_b200.runner import KernelBuildError, compile_module, render_source

HEADER = Path(__file__).resolve().parent.parent / "include" / "gpo.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gpo_[a-z_]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 9
    for n in names:
        assert hasattr(lib, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"
    assert lib.gpo_abi_version() == _lib.ABI_VERSION
    assert _lib.status_name(_lib.COMPILE_ERROR) == "GPO_COMPILE_ERROR"


def test_struct_layouts_match_header():
    # int32 x 11 (44 B) + pad to 8 + int64 x 4
    assert ctypes.sizeof(_lib.GpoKey) == 48 + 32
    assert ctypes.sizeof(_lib.GpoArgs) == 8 * 4 + 8 + 8 * 2 + 4 + 4


def mm(cfg, shape=(4096, 4096, 4096)):
    base = {"BLOCK_M": 128, "BLOCK_N": 256, "BLOCK_K": 64, "GROUP_M": 8, "num_warps": 8,
            "num_stages": 4, "dtype": "bfloat16"}
    return compile_module("matmul", shape, {**base, **cfg})


def test_tcgen05_matmul_plan():
    res = mm({}).resources()
    assert res["kernel"].startswith("matmul_tc_kernel<bf16,128,256,persistent>")
    assert res["tmem_cols"] == 512  # two 256-column accumulators (double buffer)
    assert res["smem_bytes"] <= 227 * 1024
    assert res["persistent"]
    res4 = mm({"num_warps": 4}).resources()
    assert res4["tmem_cols"] == 256 and not res4["persistent"]
    assert res4["grid"][0] == 32 * 16


def test_block_m_64_uses_m64_tensor_core_mmas_for_16_bit_inputs():
    res = mm({"BLOCK_M": 64, "BLOCK_N": 128, "num_warps": 4}).resources()
    assert res["kernel"] == "matmul_tc_kernel<bf16,64,128,tile>"
    assert res["tmem_cols"] == 128 and res["grid"][0] == 64 * 32
    resp = mm({"BLOCK_M": 64, "BLOCK_N": 256}).resources()
    assert resp["kernel"] == "matmul_tc_kernel<bf16,64,256,persistent>"
    assert resp["tmem_cols"] == 512
    rt = mm({"BLOCK_M": 64, "BLOCK_N": 64, "num_warps": 4, "dtype": "tf32"}).resources()
    assert rt["kernel"] == "matmul_tc_kernel<tf32,64,64,tile>"


def test_shared_memory_overflow_is_a_compile_error():
    with pytest.raises(KernelBuildError) as ei:
        mm({"BLOCK_M": 256, "BLOCK_N": 256, "BLOCK_K": 128, "num_stages": 6})
    assert "GPO_COMPILE_ERROR" in str(ei.value) and "shared memory" in ei.value.log


def test_simt_register_tile_overflow_is_a_compile_error():
    with pytest.raises(KernelBuildError) as ei:
        mm({"BLOCK_M": 256, "BLOCK_N": 256, "dtype": "float32", "num_warps": 4})
    assert "register" in ei.value.log


def test_small_tiles_route_to_cuda_cores():
    # fp32 and 16-row tiles run on the CUDA cores
    res = mm({"BLOCK_M": 32, "BLOCK_N": 32, "BLOCK_K": 16, "num_warps": 4,
              "dtype": "float32"}).resources()
    assert res["kernel"].startswith("matmul_simt")
    res = mm({"BLOCK_M": 16, "BLOCK_N": 32, "BLOCK_K": 16, "num_warps": 4}).resources()
    assert res["kernel"].startswith("matmul_simt")


def test_block_m_32_runs_on_tensor_cores_with_cuda_core_fallback():
    # 16-bit BLOCK_M 32: the M=64 MMA over 64-row A atoms
    res = mm({"BLOCK_M": 32, "BLOCK_N": 32, "BLOCK_K": 16, "num_warps": 4}).resources()
    assert res["kernel"] == "matmul_tc_kernel<bf16,32,32,tile>"
    assert res["grid"][0] == (4096 // 32) * (4096 // 32)
    # A in 64-row atoms: 5 stages x (64 + 32) x 256 bf16 do not fit; the
    # CUDA-core tile (32-row A) does, so the config still compiles
    cfg = {"BLOCK_M": 32, "BLOCK_N": 32, "BLOCK_K": 256, "num_warps": 4, "num_stages": 5}
    res = mm(cfg).resources()
    assert res["kernel"].startswith("matmul_simt"), res["kernel"]


def test_attention_plans():
    base = {"BLOCK_M": 128, "BLOCK_N": 128, "num_warps": 4, "num_stages": 2,
            "dtype": "bfloat16"}
    r = compile_module("attention_causal", (128, 4096, 128), base).resources()
    assert r["kernel"] == "attn_tc_kernel<bf16,BN=128,D=128,causal,wg=1,sbufs=3>"
    assert r["tmem_cols"] == 512 and r["grid"] == [32, 128, 1]
    # 8 warps: two softmax warpgroups split each row's columns
    r2 = compile_module("attention_causal", (128, 4096, 128),
                        {**base, "num_warps": 8}).resources()
    assert r2["kernel"].endswith("wg=2,sbufs=3>") and r2["threads_per_cta"] == 384
    assert r2["grid"] == [32, 128, 1] and r2["tmem_cols"] == 512
    # BLOCK_N 32 keeps one warpgroup (a warp needs 32 S columns)
    r3 = compile_module("attention", (16, 1024, 64),
                        {**base, "BLOCK_N": 32, "num_warps": 8}).resources()
    assert r3["kernel"].endswith("wg=1,sbufs=3>") and r3["threads_per_cta"] == 256
    # BLOCK_M 256: a CTA pair per two query tiles
    r5 = compile_module("attention_causal", (128, 4096, 128),
                        {**base, "BLOCK_M": 256, "num_stages": 4}).resources()
    assert r5["kernel"].endswith("sbufs=3,cta_pair>") and r5["grid"] == [32, 128, 1]
    assert r5["threads_per_cta"] == 256 and r5["tmem_cols"] == 512
    # BLOCK_M 256 with 8 warps: two query tiles per CTA, one softmax
    # warpgroup each (O 2 x 128 + S 2 x 128 columns = all of TMEM)
    rd = compile_module("attention_causal", (128, 4096, 128),
                        {**base, "BLOCK_M": 256, "num_warps": 8}).resources()
    assert rd["kernel"] == "attn_tc_dual_kernel<bf16,BN=128,D=128,causal,two_tiles>"
    # causal: one 1-D grid ordered longest span first over groups of heads
    assert rd["grid"] == [16 * 128, 1, 1] and rd["threads_per_cta"] == 384
    rf = compile_module("attention", (128, 4096, 128),
                        {**base, "BLOCK_M": 256, "num_warps": 8}).resources()
    assert rf["grid"] == [16 * 128, 1, 1] and rf["persistent"]
    assert rd["tmem_cols"] == 512 and rd["smem_bytes"] <= 227 * 1024
    for bad in ({"num_stages": 3}, {"BLOCK_N": 128, "num_stages": 4}):  # shared memory
        with pytest.raises(KernelBuildError, match="shared memory"):
            compile_module("attention", (128, 4096, 128),
                           {**base, "BLOCK_M": 256, "num_warps": 8, **bad})
    with pytest.raises(KernelBuildError, match="TMEM"):  # 2 x 256 + 2 x 32 columns
        compile_module("attention", (4, 512, 256),
                       {**base, "BLOCK_M": 256, "BLOCK_N": 32, "num_warps": 8})
    # BLOCK_N 64 (D 128), one warpgroup, two stages: two S/P buffers keep the
    # CTA within 256 TMEM columns so that two CTAs share an SM
    r6 = compile_module("attention", (128, 4096, 128), {**base, "BLOCK_N": 64}).resources()
    assert r6["kernel"].endswith("wg=1,sbufs=2>") and r6["tmem_cols"] == 256
    assert 2 * (r6["smem_bytes"] + 1024) <= 228 * 1024
    # three stages no longer leave room for two CTAs: three buffers, 512 columns
    r7 = compile_module("attention", (128, 4096, 128),
                        {**base, "BLOCK_N": 64, "num_stages": 3}).resources()
    assert r7["kernel"].endswith("sbufs=3>") and r7["tmem_cols"] == 512
    # BLOCK_M 64: 64-row query tiles on M=64 MMAs, one softmax warpgroup
    r8 = compile_module("attention_causal", (128, 4096, 128),
                        {**base, "BLOCK_M": 64, "num_warps": 8}).resources()
    assert r8["kernel"] == "attn_tc_kernel<bf16,BM=64,BN=128,D=128,causal,wg=1,sbufs=3>"
    assert r8["grid"] == [64, 128, 1] and r8["threads_per_cta"] == 256
    # D = 256 with BLOCK_N 128: O 256 + 2 S buffers x 128 fill TMEM (two buffers)
    r4 = compile_module("attention", (4, 512, 256), {**base, "num_stages": 1}).resources()
    assert r4["kernel"].endswith("sbufs=2>") and r4["tmem_cols"] == 512
    # Q (32 KB) + 3 K/V stages of 64 KB fit (P lives in TMEM); 4 do not
    compile_module("attention_causal", (128, 4096, 128), {**base, "num_stages": 3})
    with pytest.raises(KernelBuildError):
        compile_module("attention_causal", (128, 4096, 128), {**base, "num_stages": 4})
    with pytest.raises(KernelBuildError) as ei:  # fp32 tiles of the CUDA-core family
        compile_module("attention", (16, 1024, 128), {**base, "dtype": "float32"})
    assert "shared memory" in ei.value.log
    with pytest.raises(KernelBuildError) as ei:  # same rule as runner.py:233-234
        compile_module("attention", (16, 1024, 48), base)
    assert "power of two" in str(ei.value)


def test_unknown_task_and_strategy_are_rejected():
    with pytest.raises(KernelBuildError):
        compile_module("conv2d", (8,), {})
    with pytest.raises(KernelBuildError):
        compile_module("reduction", (1000,), {"BLOCK_SIZE": 256, "strategy": "tree",
                                              "dtype": "float32"})
    with pytest.raises(KernelBuildError):
        compile_module("reduction", (1000,), {"BLOCK_SIZE": 256, "strategy": "loop",
                                              "dtype": "bfloat16"})


def test_scratch_requirements():
    r = compile_module("reduction", (100_003,), {"BLOCK_SIZE": 1024, "num_warps": 4,
                                                 "strategy": "two_pass",
                                                 "dtype": "float32"}).resources()
    assert r["scratch_bytes"][0] == 4 * 98 and r["launches_per_call"] == 2
    r = compile_module("fused_elementwise", (1000,), {"BLOCK_SIZE": 256, "num_warps": 4,
                                                      "strategy": "unfused",
                                                      "dtype": "bfloat16"}).resources()
    assert r["scratch_bytes"] == [2000, 2000] and r["launches_per_call"] == 3


def test_render_source_works_without_gpu():
    """tests/test_triton_gpu.py:73-82, for the CUDA backend."""
    src = render_source("matmul", {"BLOCK_M": 128, "BLOCK_N": 128, "BLOCK_K": 64,
                                   "GROUP_M": 4, "num_warps": 4, "num_stages": 3,
                                   "dtype": "float16"})
    assert "tcgen05.mma" in src and "matmul_tc_kernel" in src
    assert "BLOCK_M = 128" in src
    src_red = render_source("reduction", {"strategy": "atomic", "BLOCK_SIZE": 1024})
    assert "reduce_slice_kernel" in src_red


def test_row_kernel_plans():
    r = compile_module("softmax", (16384, 8192), {"BLOCK_N": 8192, "num_warps": 8,
                                                  "num_stages": 1,
                                                  "dtype": "bfloat16"}).resources()
    assert r["kernel"] == "softmax_tile_regs<vpt=4>"
    r = compile_module("softmax", (16384, 8192), {"BLOCK_N": 16384, "num_warps": 4,
                                                  "num_stages": 1,
                                                  "dtype": "bfloat16"}).resources()
    assert r["kernel"] == "softmax_tile_smem<vpt=0>"
    r = compile_module("layernorm", (37, 500), {"BLOCK_N": 128, "num_warps": 4,
                                                "num_stages": 1,
                                                "dtype": "float32"}).resources()
    assert r["kernel"] == "layernorm_twopass<vpt=1>"


def test_row_ring_plans():
    # num_stages rows of shared memory (+ gamma, beta for layernorm)
    r = compile_module("softmax", (16384, 8192), {"BLOCK_N": 8192, "num_warps": 8,
                                                  "num_stages": 3,
                                                  "dtype": "bfloat16"}).resources()
    assert r["kernel"] == "softmax_rows_ring<vpt=4,rows=3>" and r["persistent"]
    assert r["smem_bytes"] >= 3 * 8192 * 2
    r = compile_module("layernorm", (16384, 8192), {"BLOCK_N": 8192, "num_warps": 16,
                                                    "num_stages": 2,
                                                    "dtype": "bfloat16"}).resources()
    assert r["kernel"] == "layernorm_rows_ring<vpt=2,rows=2>"
    assert r["smem_bytes"] >= 4 * 8192 * 2
    # rows whose bytes are not a multiple of 16 cannot be bulk-copied: tile kernel
    r = compile_module("softmax", (64, 1001), {"BLOCK_N": 1024, "num_warps": 4,
                                               "num_stages": 2,
                                               "dtype": "bfloat16"}).resources()
    assert r["kernel"].startswith("softmax_tile_regs")
    # a ring that does not fit shared memory falls back to the register prefetch
    r = compile_module("layernorm", (64, 16384), {"BLOCK_N": 16384, "num_warps": 8,
                                                  "num_stages": 4,
                                                  "dtype": "float32"}).resources()
    assert r["kernel"] == "layernorm_rows_pipe<vpt=16>"
    # 4+ slots per thread need more than 64 registers: CTAs wider than 256
    # threads take the per-row kernel
    r = compile_module("layernorm", (64, 16384), {"BLOCK_N": 16384, "num_warps": 16,
                                                  "num_stages": 4,
                                                  "dtype": "float32"}).resources()
    assert r["kernel"] == "layernorm_tile_regs<vpt=8>"


def test_cta_pair_plan():
    r = mm({"BLOCK_M": 256, "num_warps": 4, "num_stages": 3}).resources()
    assert r["kernel"] == "matmul_tc2_kernel<bf16,256,256,cta_pair>"
    assert r["grid"][0] == 2 * 16 * 16 and r["tmem_cols"] == 256
    # padded so that at most 2 CTAs (2 x 256 TMEM columns) share an SM
    assert 233472 // 3 < r["smem_bytes"] <= 227 * 1024
