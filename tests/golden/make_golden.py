"""Generate the golden fixtures by running the reference's own code.

Run where a checkout of the reference is readable, giving its path:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py <reference checkout>

For every reference task at the reference's odd-sized test shapes
(tests/test_tasks_and_emulation.py:13-21) and each supported dtype, this
imports the reference's ``benchmarks`` and ``compiler.validation.emulation``
modules, builds inputs with the reference's ``make_inputs`` (seeded), and
stores: the SHA-256 of every input tensor, the reference's
``task.reference`` output, and ``emulate`` outputs for configs that exercise
each algorithm variant (chunked K, tf32, online softmax, two-pass layernorm,
unfused rounding, attention P cast).  It also stores input hashes at the
reference's GPU test shapes (tests/test_triton_gpu.py:21-29).  Outputs are
written bit-exact (bf16 as its uint16 bit pattern) to golden_<task>.npz with
a JSON index.
"""

from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

SMALL_SHAPES = {
    "matmul": (96, 80, 72), "vecadd": (10_007,), "reduction": (100_003,),
    "softmax": (37, 500), "layernorm": (37, 500), "fused_elementwise": (10_007,),
    "attention": (3, 130, 32),
}
GPU_SHAPES = {
    "matmul": (384, 320, 288), "vecadd": (1_000_003,), "reduction": (1_000_003,),
    "softmax": (256, 1000), "layernorm": (256, 1000), "fused_elementwise": (1_000_003,),
    "attention": (4, 512, 64),
}
EMU_CONFIGS = {
    "matmul": [{"BLOCK_K": 16}, {"BLOCK_K": 64}],
    "vecadd": [{}],
    "reduction": [{"BLOCK_SIZE": 1024, "strategy": "two_pass"},
                  {"BLOCK_SIZE": 256, "strategy": "atomic"}],
    "softmax": [{"BLOCK_N": 1024}, {"BLOCK_N": 128}],
    "layernorm": [{"BLOCK_N": 1024}, {"BLOCK_N": 128}],
    "fused_elementwise": [{"strategy": "fused"}, {"strategy": "unfused"}],
    "attention": [{"BLOCK_N": 32}, {"BLOCK_N": 128}],
}
SEEDS = (0, 7)


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(to_np(t).tobytes()).hexdigest()


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from benchmarks import get_task
    from compiler.validation.emulation import emulate

    index = {"torch": torch.__version__, "tasks": {}}
    for name, shape in SMALL_SHAPES.items():
        task = get_task(name)
        arrays: dict[str, np.ndarray] = {}
        entry = {"shape": list(shape), "cases": [], "gpu_shape": list(GPU_SHAPES[name]),
                 "gpu_input_sha": {}}
        for dtype in task.supported_dtypes:
            for seed in SEEDS:
                inputs = task.make_inputs(shape, dtype, "cpu", seed=seed)
                ref = task.reference(*inputs)
                tag = f"{dtype}__s{seed}"
                arrays[f"ref__{tag}"] = to_np(ref)
                case = {"dtype": dtype, "seed": seed, "input_sha": [sha(t) for t in inputs],
                        "ref": f"ref__{tag}", "emulate": []}
                for ci, cfg in enumerate(EMU_CONFIGS[name]):
                    full = {**task.default_config(shape), **cfg, "dtype": dtype}
                    out = emulate(name, shape, full, inputs)
                    key = f"emu{ci}__{tag}"
                    arrays[key] = to_np(out)
                    case["emulate"].append({"config": full, "key": key})
                entry["cases"].append(case)
            gin = task.make_inputs(GPU_SHAPES[name], dtype, "cpu", seed=0)
            entry["gpu_input_sha"][dtype] = [sha(t) for t in gin]
        np.savez_compressed(HERE / f"golden_{name}.npz", **arrays)
        index["tasks"][name] = entry
        print(name, len(arrays), "arrays")
    (HERE / "golden_index.json").write_text(json.dumps(index, indent=1, sort_keys=True))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <path of the reference checkout>")
    main(sys.argv[1])
