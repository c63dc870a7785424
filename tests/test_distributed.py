"""The N>1 path's host logic with world_size-2 gloo ranks on CPU: every rank
emits a byte-identical plan (replicas), batch shards tile the batch exactly,
and timings reduce to the max over ranks."""
import os
import socket

import pytest

from emx_onnx_cgen_b200.distributed import (cpus_from_affinity_words, numa_cpus_for_pci,
                                              nvml_cpus_for_pci, parse_cpulist, shard_rows)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from emx_onnx_cgen_b200 import lowering, workloads as W
        from emx_onnx_cgen_b200.distributed import check_same_plan, max_over_ranks, shard_rows
        from emx_onnx_cgen_b200.plan import B200PlanEmitter
        wl = W.qconv_stack_int8(batch=4, height=10, width=10)
        plan = B200PlanEmitter().emit_plan(lowering.lower(wl.graph))
        same = check_same_plan(plan.plan_bytes, plan.weight_bytes)
        # a rank that emitted something else must be detected
        bad = plan.plan_bytes + (b"x" if rank == 1 else b"")
        differs = not check_same_plan(bad, plan.weight_bytes)
        worst = max_over_ranks(float(10 + rank))
        begin, count = shard_rows(plan.batch, world, rank)
        result_q.put((rank, same, differs, worst, begin, count))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    results = sorted(q.get(timeout=10) for _ in range(2))
    for rank, same, differs, worst, begin, count in results:
        assert same and differs and worst == 11.0
    assert [(b, c) for _, _, _, _, b, c in results] == [(0, 2), (2, 2)]


@pytest.mark.parametrize("batch,world", [(32, 1), (32, 3), (7, 8), (0, 2), (100, 8)])
def test_shards_tile_the_batch(batch, world):
    spans = [shard_rows(batch, world, r) for r in range(world)]
    pos = 0
    for b, c in spans:
        assert b == pos and c >= 0
        pos += c
    assert pos == batch
    assert max(c for _, c in spans) - min(c for _, c in spans) <= 1


def test_cpulist_forms():
    assert parse_cpulist("0-3,8,10-11\n") == [0, 1, 2, 3, 8, 10, 11]
    assert parse_cpulist("5") == [5]
    assert parse_cpulist("") == []


def test_numa_cpus_for_pci_reads_sysfs(tmp_path):
    dev = tmp_path / "bus" / "pci" / "devices" / "0000:1b:00.0"
    dev.mkdir(parents=True)
    (dev / "numa_node").write_text("1\n")
    node = tmp_path / "devices" / "system" / "node" / "node1"
    node.mkdir(parents=True)
    (node / "cpulist").write_text("32-35,96\n")
    assert numa_cpus_for_pci(0, 0x1B, 0, str(tmp_path)) == (1, [32, 33, 34, 35, 96])
    # unknown placement: no entry, or node -1 (single-node platforms)
    assert numa_cpus_for_pci(0, 0x1C, 0, str(tmp_path)) == (-1, [])
    (dev / "numa_node").write_text("-1\n")
    assert numa_cpus_for_pci(0, 0x1B, 0, str(tmp_path)) == (-1, [])


def test_nvml_affinity_fallback():
    assert cpus_from_affinity_words([0xFFFF]) == list(range(16))
    assert cpus_from_affinity_words([0, 1 << 3]) == [67]

    class FakeNvml:
        calls = []

        def nvmlInit(self):
            self.calls.append("init")

        def nvmlShutdown(self):
            self.calls.append("shutdown")

        def nvmlDeviceGetHandleByPciBusId(self, bus_id):
            if bus_id != b"00000000:1b:00.0":
                raise RuntimeError("no such device")
            return "h"

        def nvmlDeviceGetCpuAffinity(self, h, n_words):
            return [0x0F0] + [0] * (n_words - 1)

    fake = FakeNvml()
    assert nvml_cpus_for_pci(0, 0x1B, 0, fake) == [4, 5, 6, 7]
    assert fake.calls == ["init", "shutdown"]
    assert nvml_cpus_for_pci(0, 0x1C, 0, fake) == []  # unknown device: no placement
