"""The relative-error bounds of the B200 benchmark configurations, at their
full sizes: fp32 <= 1e-5, tf32 / bf16 / fp16 <= 1e-2, read as the largest
row-wise normwise error ||c - r||_2 / ||r||_2 against the task's torch
reference on identical seeded inputs (a 1-D output is one row).  Each case
is the configuration the benchmark reports for the task (or the fp32 /
tf32 / fp16 form of the same workload)."""

import pytest
import torch

from gpu_optimizer_b200.correctness import NORMWISE_BOUND, check_correctness
from gpu_optimizer_b200.runner import build_callable, check_device_status
from gpu_optimizer_b200.tasks import get_task

pytestmark = pytest.mark.gpu

MM = {"BLOCK_M": 256, "BLOCK_N": 256, "BLOCK_K": 128, "GROUP_M": 16, "num_warps": 8,
      "num_stages": 3}
CASES = [
    ("vecadd", (1 << 24,), {"BLOCK_SIZE": 2048, "num_warps": 4, "dtype": "float32"}),
    ("reduction", (1 << 28,), {"BLOCK_SIZE": 8192, "num_warps": 16, "strategy": "atomic",
                               "dtype": "float32"}),
    ("reduction", (1 << 28,), {"BLOCK_SIZE": 4096, "num_warps": 8, "strategy": "two_pass",
                               "dtype": "float32"}),
    ("softmax", (16384, 8192), {"BLOCK_N": 8192, "num_warps": 4, "num_stages": 2,
                                "dtype": "bfloat16"}),
    ("softmax", (16384, 8192), {"BLOCK_N": 8192, "num_warps": 4, "num_stages": 2,
                                "dtype": "float16"}),
    ("layernorm", (16384, 8192), {"BLOCK_N": 8192, "num_warps": 4, "num_stages": 2,
                                  "dtype": "bfloat16"}),
    ("layernorm", (16384, 8192), {"BLOCK_N": 2048, "num_warps": 8, "num_stages": 2,
                                  "dtype": "float16"}),
    ("fused_gelu", (1 << 26,), {"BLOCK_SIZE": 4096, "num_warps": 4, "strategy": "fused",
                                "dtype": "bfloat16"}),
    ("fused_gelu", (1 << 26,), {"BLOCK_SIZE": 4096, "num_warps": 4, "strategy": "unfused",
                                "dtype": "bfloat16"}),
    ("matmul", (4096, 4096, 4096), {**MM, "dtype": "bfloat16"}),
    ("matmul", (8192, 8192, 8192), {**MM, "dtype": "bfloat16"}),
    ("matmul", (4096, 4096, 4096), {**MM, "dtype": "float16"}),
    ("matmul", (4096, 4096, 4096), {"BLOCK_M": 256, "BLOCK_N": 128, "BLOCK_K": 32,
                                    "GROUP_M": 8, "num_warps": 4, "num_stages": 3,
                                    "dtype": "tf32"}),
    ("matmul", (2048, 2048, 2048), {"BLOCK_M": 128, "BLOCK_N": 128, "BLOCK_K": 32,
                                    "GROUP_M": 8, "num_warps": 8, "num_stages": 3,
                                    "dtype": "float32"}),
    ("attention", (128, 4096, 128), {"BLOCK_M": 128, "BLOCK_N": 128, "num_warps": 4,
                                     "num_stages": 2, "dtype": "bfloat16"}),
    ("attention_causal", (128, 4096, 128), {"BLOCK_M": 128, "BLOCK_N": 128, "num_warps": 4,
                                            "num_stages": 2, "dtype": "bfloat16"}),
    ("attention_causal", (128, 4096, 128), {"BLOCK_M": 128, "BLOCK_N": 128, "num_warps": 4,
                                            "num_stages": 2, "dtype": "float16"}),
    ("attention", (128, 4096, 128), {"BLOCK_M": 256, "BLOCK_N": 128, "num_warps": 8,
                                     "num_stages": 2, "dtype": "bfloat16"}),
    ("attention_causal", (128, 4096, 128), {"BLOCK_M": 256, "BLOCK_N": 128, "num_warps": 8,
                                            "num_stages": 2, "dtype": "bfloat16"}),
]


@pytest.mark.parametrize("name,shape,cfg", CASES,
                         ids=lambda v: v if isinstance(v, str) else
                         (str(v.get("dtype")) + "-" + str(v.get("strategy", ""))
                          if isinstance(v, dict) else "x".join(map(str, v))))
def test_normwise_error_within_benchmark_bound(name, shape, cfg):
    task = get_task(name, "b200")
    dtype = cfg["dtype"]
    inputs = task.make_inputs(shape, dtype, "cuda", 0)
    out = build_callable(name, shape, cfg, inputs).fn()
    check_device_status()
    ref = task.reference(*inputs)
    rtol, atol = task.tolerance(dtype)
    rep = check_correctness(out, ref, rtol, atol)
    assert rep.passed, rep.summary()
    assert rep.rel_err_normwise <= NORMWISE_BOUND[dtype], rep.summary()
    del inputs, out, ref
    torch.cuda.empty_cache()
