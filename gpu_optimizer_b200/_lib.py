"""ctypes binding of libgpo.so (declarations: include/gpo.h).

The library is loaded from this package directory.  There is no fallback:
if it is missing, ``load()`` raises and the runner reports every candidate
as a build failure.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libgpo.so"
ABI_VERSION = 1

# gpo_status
OK, COMPILE_ERROR, BAD_CONFIG, BAD_ARGS, LAUNCH_ERROR, TIMEOUT, NO_DEVICE, INTERNAL = range(8)

# gpo_task
TASK_IDS = {
    "matmul": 0, "vecadd": 1, "reduction": 2, "softmax": 3, "layernorm": 4,
    "fused_elementwise": 5, "attention": 6, "attention_causal": 7, "fused_gelu": 8,
}
# gpo_dtype
DTYPE_IDS = {"float32": 0, "tf32": 1, "float16": 2, "bfloat16": 3}
# gpo_strategy
STRATEGY_IDS = {"": 0, "loop": 1, "atomic": 2, "two_pass": 3, "fused": 4, "unfused": 5}


class GpoKey(ctypes.Structure):
    _fields_ = [
        ("task", ctypes.c_int32), ("dtype", ctypes.c_int32), ("strategy", ctypes.c_int32),
        ("block_m", ctypes.c_int32), ("block_n", ctypes.c_int32), ("block_k", ctypes.c_int32),
        ("block_size", ctypes.c_int32), ("group_m", ctypes.c_int32),
        ("num_warps", ctypes.c_int32), ("num_stages", ctypes.c_int32),
        ("ndim", ctypes.c_int32), ("shape", ctypes.c_int64 * 4),
    ]


class GpoResources(ctypes.Structure):
    _fields_ = [
        ("smem_bytes", ctypes.c_uint32), ("tmem_cols", ctypes.c_uint32),
        ("threads_per_cta", ctypes.c_uint32), ("grid_x", ctypes.c_uint32),
        ("grid_y", ctypes.c_uint32), ("grid_z", ctypes.c_uint32),
        ("launches_per_call", ctypes.c_uint32), ("persistent", ctypes.c_uint32),
        ("scratch_bytes", ctypes.c_uint64 * 2), ("kernel", ctypes.c_char * 96),
    ]

    def to_dict(self) -> dict:
        return {
            "smem_bytes": self.smem_bytes, "tmem_cols": self.tmem_cols,
            "threads_per_cta": self.threads_per_cta,
            "grid": [self.grid_x, self.grid_y, self.grid_z],
            "launches_per_call": self.launches_per_call,
            "persistent": bool(self.persistent),
            "scratch_bytes": [int(self.scratch_bytes[0]), int(self.scratch_bytes[1])],
            "kernel": self.kernel.decode(),
        }


class GpoArgs(ctypes.Structure):
    _fields_ = [
        ("in_", ctypes.c_void_p * 4), ("out", ctypes.c_void_p),
        ("scratch", ctypes.c_void_p * 2), ("scale", ctypes.c_float), ("eps", ctypes.c_float),
    ]


# Every symbol include/gpo.h declares, with its ctypes signature.
SIGNATURES = {
    "gpo_abi_version": (ctypes.c_int, []),
    "gpo_compile": (ctypes.c_int, [ctypes.POINTER(GpoKey), ctypes.POINTER(ctypes.c_void_p),
                                   ctypes.c_char_p, ctypes.c_size_t]),
    "gpo_query": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(GpoResources)]),
    "gpo_launch": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(GpoArgs), ctypes.c_void_p]),
    "gpo_device_status": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)]),
    "gpo_selftest_timeout": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32,
                                            ctypes.POINTER(ctypes.c_uint32)]),
    "gpo_reduction_sum_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64,
                                                 ctypes.c_void_p, ctypes.c_int32,
                                                 ctypes.c_int32, ctypes.c_void_p]),
    "gpo_destroy": (None, [ctypes.c_void_p]),
    "gpo_source": (ctypes.c_char_p, [ctypes.c_void_p]),
    "gpo_status_name": (ctypes.c_char_p, [ctypes.c_int]),
}

_lib = None
_lock = threading.Lock()


class LibraryMissing(RuntimeError):
    """libgpo.so is absent or does not match this binding."""


def load() -> ctypes.CDLL:
    """Load (once) and return the kernel library; raises LibraryMissing."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise LibraryMissing(
                f"{LIB_PATH} is not built; run `python -m gpu_optimizer_b200.build`")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.gpo_abi_version() != ABI_VERSION:
            raise LibraryMissing(f"libgpo.so ABI {lib.gpo_abi_version()} != {ABI_VERSION}")
        _lib = lib
        return lib


def status_name(code: int) -> str:
    return load().gpo_status_name(code).decode()


def make_key(task: str, shape, config: dict) -> GpoKey:
    """Translate a (task, shape, config dict) candidate into a gpo_key."""
    k = GpoKey()
    k.task = TASK_IDS[task]
    k.dtype = DTYPE_IDS[str(config.get("dtype", "float32"))]
    k.strategy = STRATEGY_IDS[str(config.get("strategy", ""))]
    k.block_m = int(config.get("BLOCK_M", 0))
    k.block_n = int(config.get("BLOCK_N", 0))
    k.block_k = int(config.get("BLOCK_K", 0))
    k.block_size = int(config.get("BLOCK_SIZE", 0))
    k.group_m = int(config.get("GROUP_M", 1))
    k.num_warps = int(config.get("num_warps", 4))
    k.num_stages = int(config.get("num_stages", 1))
    shape = tuple(int(s) for s in shape)
    if len(shape) > 4:
        raise ValueError("at most 4 shape dims")
    k.ndim = len(shape)
    for i, s in enumerate(shape):
        k.shape[i] = s
    return k


class Module:
    """An owned gpo_module handle (compiled candidate)."""

    def __init__(self, task: str, shape, config: dict) -> None:
        lib = load()
        self._lib = lib
        self.key = make_key(task, shape, config)
        handle = ctypes.c_void_p()
        log = ctypes.create_string_buffer(1024)
        self.status = lib.gpo_compile(ctypes.byref(self.key), ctypes.byref(handle), log, 1024)
        self.log = log.value.decode(errors="replace")
        self.handle = handle if self.status == OK else None

    @property
    def ok(self) -> bool:
        return self.handle is not None

    def resources(self) -> dict:
        r = GpoResources()
        rc = self._lib.gpo_query(self.handle, ctypes.byref(r))
        if rc != OK:
            raise RuntimeError(f"gpo_query failed: {status_name(rc)}")
        return r.to_dict()

    def source(self) -> str:
        return self._lib.gpo_source(self.handle).decode(errors="replace")

    def launch(self, args: GpoArgs, stream: int) -> int:
        return self._lib.gpo_launch(self.handle, ctypes.byref(args), ctypes.c_void_p(stream))

    def __del__(self) -> None:
        h = getattr(self, "handle", None)
        if h is not None:
            try:
                self._lib.gpo_destroy(h)
            except Exception:
                pass


def device_status(stream: int) -> tuple[int, int]:
    """(status, flags) of the current device's error word after syncing."""
    flags = ctypes.c_uint32(0)
    rc = load().gpo_device_status(ctypes.c_void_p(stream), ctypes.byref(flags))
    return rc, int(flags.value)


def selftest_timeout(stream: int, limit_ms: int = 100) -> tuple[int, int]:
    """Run the bounded-wait self-test; returns (status, flags)."""
    flags = ctypes.c_uint32(0)
    rc = load().gpo_selftest_timeout(ctypes.c_void_p(stream), limit_ms, ctypes.byref(flags))
    return rc, int(flags.value)


NOALLOC_MAX_PARTIALS = 65536


def reduction_sum_noalloc(x_ptr: int, n: int, out_ptr: int, block_size: int, num_warps: int,
                          stream: int) -> int:
    """gpo_reduction_sum_noalloc: two_pass fp32 sum with the library's fixed
    partial-sum array (no allocation); returns the gpo_status code."""
    return load().gpo_reduction_sum_noalloc(ctypes.c_void_p(x_ptr), n, ctypes.c_void_p(out_ptr),
                                            block_size, num_warps, ctypes.c_void_p(stream))
