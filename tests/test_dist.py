"""Multi-process host logic of the sharded path on CPU (gloo, world size 2):
frame sharding, max-over-ranks timing and the output gather."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from ai_engine_b200 import dist as adist


def test_shard_range_covers_batch_exactly():
    for n in (0, 1, 7, 256, 1000):
        for world in (1, 2, 3, 8):
            spans = [adist.shard_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            for (s0, e0), (s1, e1) in zip(spans, spans[1:]):
                assert e0 == s1
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        adist.shard_range(10, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, n_total, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    adist.init("gloo", timeout_s=30)
    s, e = adist.shard_range(n_total, rank, world)
    # each rank "processes" its frames: out[f] = f (a stand-in for the conv output)
    local = torch.arange(s, e, dtype=torch.float32).view(-1, 1, 1).expand(-1, 2, 3).contiguous()
    t = adist.max_over_ranks(float(rank + 1))
    full = adist.gather_outputs(local, n_total)
    q.put((rank, t, None if full is None else full[:, 0, 0].tolist()))
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


@pytest.mark.parametrize("n_total", [8, 7])
def test_gather_and_max_over_two_ranks(n_total):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n_total, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rank, t, full = q.get(timeout=120)
        res[rank] = (t, full)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0][0] == 2.0 and res[1][0] == 2.0
    assert res[0][1] == [float(i) for i in range(n_total)]
    assert res[1][1] is None


class _FakeNvml:
    """NVML stand-in: GPU i's local CPUs are the bits of a fixed mask."""

    def __init__(self, masks):
        self.masks = masks

    def nvmlInit(self):
        pass

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetCpuAffinity(self, h, words):
        return self.masks[h][:words]


def test_gpu_local_cpus_from_nvml_mask():
    import os
    from ai_engine_b200.dist import gpu_local_cpus
    n = os.cpu_count()
    words = (n + 63) // 64
    lo = [(1 << min(n, 2)) - 1] + [0] * (words - 1)   # CPUs 0, 1
    assert gpu_local_cpus(0, _FakeNvml([lo])) == list(range(min(n, 2)))
    assert gpu_local_cpus(0, _FakeNvml([[0] * words])) is None   # empty mask: unknown

    class Broken(_FakeNvml):
        def nvmlInit(self):
            raise RuntimeError("no NVML")
    assert gpu_local_cpus(0, Broken([lo])) is None
