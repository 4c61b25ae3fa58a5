"""Hardware description with a B200 catalog entry (hardware/gpu_info.py:24-234).

``HardwareSpec`` keeps the reference's fields and 12-dim ``feature_vector``
so the surrogate / policy hardware embedding is unchanged; the catalog gains
the B200 (sm_100, 148 SMs, 180 GB HBM3e), which the reference's catalog
lacks.  ``detect_hardware`` matches the device name against the catalog and
otherwise derives a spec from queried properties.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass

import numpy as np


@dataclass(frozen=True)
class HardwareSpec:
    name: str
    compute_capability: tuple[int, int]
    sm_count: int
    memory_gb: float
    memory_bandwidth_gbs: float
    fp32_tflops: float
    fp16_tflops: float
    shared_mem_per_sm_kb: int
    registers_per_sm: int
    warp_size: int = 32
    l2_cache_mb: float = 4.0
    supports_bf16: bool = True
    supports_tf32: bool = True
    is_simulated: bool = False
    tmem_kb_per_sm: int = 0
    max_smem_per_cta_kb: int = 0

    def feature_vector(self) -> np.ndarray:
        cc = self.compute_capability[0] + self.compute_capability[1] / 10.0
        return np.array([
            cc / 10.0, self.sm_count / 150.0,
            np.log2(max(self.memory_gb, 1e-3)) / 8.0,
            np.log2(max(self.memory_bandwidth_gbs, 1.0)) / 12.0,
            np.log2(max(self.fp32_tflops, 1e-2)) / 8.0,
            np.log2(max(self.fp16_tflops, 1e-2)) / 10.0,
            self.shared_mem_per_sm_kb / 256.0, self.registers_per_sm / 65536.0,
            self.warp_size / 32.0, np.log2(max(self.l2_cache_mb, 0.5)) / 7.0,
            1.0 if self.supports_bf16 else 0.0, 1.0 if self.supports_tf32 else 0.0,
        ], dtype=np.float32)

    def to_dict(self) -> dict:
        d = asdict(self)
        d["compute_capability"] = list(self.compute_capability)
        return d


HARDWARE_FEATURE_DIM = 12

# Nominal B200 figures (dense tensor peaks; HBM3e bandwidth of the HGX part).
B200 = HardwareSpec(
    name="NVIDIA B200", compute_capability=(10, 0), sm_count=148, memory_gb=180.0,
    memory_bandwidth_gbs=7700.0, fp32_tflops=75.0, fp16_tflops=2250.0,
    shared_mem_per_sm_kb=228, registers_per_sm=65536, l2_cache_mb=126.0,
    tmem_kb_per_sm=256, max_smem_per_cta_kb=227,
)

KNOWN_GPUS: dict[str, HardwareSpec] = {"B200": B200}


def detect_hardware(device_index: int = 0) -> HardwareSpec:
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("detect_hardware() requires CUDA")
    props = torch.cuda.get_device_properties(device_index)
    name = props.name
    for spec in KNOWN_GPUS.values():
        if spec.name.lower() in name.lower():
            return HardwareSpec(**{**spec.to_dict(), "name": name,
                                   "compute_capability": (props.major, props.minor)})
    return HardwareSpec(
        name=name, compute_capability=(props.major, props.minor),
        sm_count=props.multi_processor_count, memory_gb=props.total_memory / 2**30,
        memory_bandwidth_gbs=800.0, fp32_tflops=15.0, fp16_tflops=100.0,
        shared_mem_per_sm_kb=props.shared_memory_per_multiprocessor // 1024,
        registers_per_sm=props.regs_per_multiprocessor, warp_size=props.warp_size,
        supports_bf16=props.major >= 8, supports_tf32=props.major >= 8)
