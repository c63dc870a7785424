"""Multi-GPU plumbing: one process per GPU, independent inferences per rank.

The lowered-op path has no cross-inference reduction, so N GPUs run N full
weight replicas on disjoint work ("replicas only"): either whole
inferences per rank (weak scaling, what the benchmark does) or contiguous
batch rows of one inference per rank through ``emx_b200_run``'s
``batch_begin/batch_count`` (strong scaling).  No collective touches the data
path; ``torch.distributed`` (NCCL on GPUs, gloo in the CPU tests) is used only
for barriers and for reducing timings.
"""
from __future__ import annotations

import hashlib
import os


def world() -> tuple[int, int, int]:
    """(rank, world_size, local_rank) from the torchrun environment."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def shard_rows(batch: int, world_size: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced split of `batch` rows: (batch_begin, batch_count)."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError("bad rank/world")
    base, extra = divmod(batch, world_size)
    begin = rank * base + min(rank, extra)
    return begin, base + (1 if rank < extra else 0)


def parse_cpulist(text: str) -> list[int]:
    """CPU numbers of a sysfs cpulist such as ``"0-3,8,10-11"``."""
    cpus: list[int] = []
    for part in text.strip().split(","):
        part = part.strip()
        if not part:
            continue
        lo, _, hi = part.partition("-")
        cpus.extend(range(int(lo), int(hi or lo) + 1))
    return cpus


def numa_cpus_for_pci(domain: int, bus: int, device: int, sysfs: str = "/sys") -> tuple[int, list[int]]:
    """(NUMA node, its CPUs) of the PCI device ``domain:bus:device.0``;
    (-1, []) where the platform does not say (no sysfs entry, node -1)."""
    dev = os.path.join(sysfs, "bus", "pci", "devices", f"{domain:04x}:{bus:02x}:{device:02x}.0")
    try:
        with open(os.path.join(dev, "numa_node")) as f:
            node = int(f.read().strip())
        if node < 0:
            return -1, []
        with open(os.path.join(sysfs, "devices", "system", "node", f"node{node}", "cpulist")) as f:
            return node, parse_cpulist(f.read())
    except (OSError, ValueError):
        return -1, []


def cpus_from_affinity_words(words) -> list[int]:
    """CPU numbers set in a bitmask given as 64-bit words, lowest word first
    (the form NVML's ``nvmlDeviceGetCpuAffinity`` returns)."""
    return [64 * i + b for i, w in enumerate(words) for b in range(64) if (int(w) >> b) & 1]


def nvml_cpus_for_pci(domain: int, bus: int, device: int, nvml=None) -> list[int]:
    """The CPUs the driver reports as closest to the GPU at ``domain:bus:device``
    (a read-only NVML query); [] when NVML is absent or does not say."""
    try:
        if nvml is None:
            import pynvml as nvml
        nvml.nvmlInit()
        try:
            h = nvml.nvmlDeviceGetHandleByPciBusId(f"{domain:08x}:{bus:02x}:{device:02x}.0".encode())
            n_words = (max(os.cpu_count() or 1, 1) + 63) // 64
            return cpus_from_affinity_words(nvml.nvmlDeviceGetCpuAffinity(h, n_words))
        finally:
            nvml.nvmlShutdown()
    except Exception:  # no NVML, no device entry: placement is unknown
        return []


def _cpu_span(cpus: list[int]) -> str:
    if cpus == list(range(cpus[0], cpus[-1] + 1)):
        return f"{cpus[0]}-{cpus[-1]}"
    return ",".join(map(str, cpus))


def bind_host_to_gpu(device_index: int, sysfs: str = "/sys", nvml=None) -> dict:
    """Pin this process to the CPUs nearest its GPU -- its NUMA node's CPUs from
    sysfs, else the CPU affinity the driver reports through NVML -- so
    page-locked host buffers allocated afterwards (first touch) sit in that
    node's memory, next to the GPU's PCIe root.  Returns what was done; changes
    nothing where neither source says or none of those CPUs is allowed to this
    process."""
    import torch
    pr = torch.cuda.get_device_properties(device_index)
    node, cpus = numa_cpus_for_pci(pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id, sysfs)
    source = "sysfs"
    if node < 0:
        cpus, source = nvml_cpus_for_pci(pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id, nvml), "nvml"
    allowed = os.sched_getaffinity(0)
    cpus = [c for c in cpus if c in allowed]
    if not cpus:
        return {"numa_node": node, "cpus": None}
    if set(cpus) != allowed:
        os.sched_setaffinity(0, cpus)
    return {"numa_node": node, "cpus": _cpu_span(cpus), "source": source}


def replica_seed(rank: int, base: int = 0) -> int:
    """Input seed of a rank's independent inferences."""
    return base + rank


def plan_digest(plan_bytes: bytes, weight_bytes: bytes) -> str:
    return hashlib.sha256(plan_bytes + b"|" + weight_bytes).hexdigest()


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank scalar (timing) across the default process group."""
    import torch
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def check_same_plan(plan_bytes: bytes, weight_bytes: bytes, device=None) -> bool:
    """True when every rank emitted a byte-identical plan (replicas must agree)."""
    import torch
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return True
    d = int(plan_digest(plan_bytes, weight_bytes)[:15], 16)
    t = torch.tensor([d, -d], dtype=torch.int64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return int(t[0].item()) == d and int(t[1].item()) == -d
