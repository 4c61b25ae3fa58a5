"""Host logic: candidate identity, spaces and task analytics (no GPU)."""

import random

import pytest

from gpu_optimizer_b200.space import Candidate
from gpu_optimizer_b200.tasks import REFERENCE_TASKS, TASK_CLASSES, get_task


def test_candidate_id_equals_reference_hash():
    # values computed with the reference's Candidate (space.py:185-191)
    cases = [
        ("matmul", (4096, 4096, 4096), {"BLOCK_M": 128, "BLOCK_N": 256, "BLOCK_K": 64,
                                        "GROUP_M": 8, "num_warps": 8, "num_stages": 4,
                                        "dtype": "bfloat16"}, "11790ea43300322f"),
        ("vecadd", (16777216,), {"BLOCK_SIZE": 1024, "num_warps": 4, "dtype": "float32"},
         "9c45f1ef1127495f"),
        ("reduction", (100003,), {"BLOCK_SIZE": 1024, "num_warps": 4, "strategy": "two_pass",
                                  "dtype": "float32"}, "3435e9e5fff93894"),
    ]
    for task, shape, cfg, want in cases:
        assert Candidate(task=task, shape=shape, config=cfg).candidate_id == want


@pytest.mark.parametrize("name", sorted(TASK_CLASSES))
@pytest.mark.parametrize("profile", ["reference", "b200"])
def test_task_basics(name, profile):
    task = get_task(name, profile)
    shape = task.default_shapes()[0]
    space = task.param_space(shape)
    cfg = task.default_config(shape)
    space.validate(cfg)
    assert space.size() > 10
    assert task.flops(shape) > 0 and task.bytes_moved(shape, cfg["dtype"], cfg) > 0
    assert task.roofline_work(shape, cfg["dtype"]) > 0
    rng = random.Random(0)
    for _ in range(5):
        c = space.sample(rng)
        space.validate(c)
        assert all(n in space for n in c)


def test_b200_spaces_match_workload_definition():
    mm = get_task("matmul", "b200").param_space((4096, 4096, 4096))
    assert mm["BLOCK_M"].choices == (32, 64, 128, 256)
    assert mm["GROUP_M"].choices == (1, 4, 8, 16)
    assert mm["num_stages"].choices == (2, 3, 4, 5, 6)
    assert mm.size() == 4 * 4 * 4 * 4 * 2 * 5 * 4
    sm = get_task("softmax", "b200").param_space((16384, 8192))
    assert sm["BLOCK_N"].choices == (1024, 2048, 4096, 8192, 16384)
    at = get_task("attention_causal", "b200").param_space((128, 4096, 128))
    assert at["BLOCK_M"].choices == (64, 128, 256) and at["BLOCK_N"].choices == (32, 64, 128)


def test_reference_spaces_equal_reference_sizes():
    sizes = {"matmul": 6912, "vecadd": 72, "reduction": 90, "softmax": 360, "layernorm": 360,
             "fused_elementwise": 144, "attention": 432}
    for name in REFERENCE_TASKS:
        t = get_task(name)
        assert t.param_space(t.default_shapes()[0]).size() == sizes[name], name


def test_causal_roofline_work():
    t = get_task("attention_causal", "b200")
    w = t.roofline_work((128, 4096, 128), "bfloat16")
    assert abs(w - 4 * 128 * 128 * 4096 * 4097 / 2) < 1
    assert abs(w / 5.50e11 - 1) < 0.01
