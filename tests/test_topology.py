"""Topology pre-flight with a fake CUDA runtime and a fake NVML (no GPU needed)."""
import pytest

from qwen38_b200.parallel.topology import TopologyError, check_topology


class FakeCuda:
    def __init__(self, n, blocked=()):
        self.n, self.blocked = n, set(blocked)

    def device_count(self):
        return self.n

    def can_device_access_peer(self, i, j):
        return (i, j) not in self.blocked


class FakeNvml:
    def __init__(self, links):
        self.links = links

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetNvLinkState(self, h, link):
        if link >= 18:
            raise RuntimeError("no such link")
        return 1 if link < self.links[h] else 0


def test_full_nvswitch_node():
    r = check_topology(8, cuda=FakeCuda(8), nvml=FakeNvml([18] * 8))
    assert r["recommended_comm"] == "fused" and r["nvlink_active_links"] == [18] * 8


def test_missing_peer_access_rejects_peer_collectives():
    cuda = FakeCuda(4, blocked={(0, 3), (3, 0)})
    with pytest.raises(TopologyError):
        check_topology(4, cuda=cuda, nvml=FakeNvml([18] * 4))
    r = check_topology(4, comm="nccl", cuda=cuda, nvml=FakeNvml([18] * 4))
    assert r["recommended_comm"] == "nccl"


def test_no_nvlink_recommends_nccl_and_too_few_gpus_raise():
    r = check_topology(2, cuda=FakeCuda(2), nvml=FakeNvml([0, 0]))
    assert r["recommended_comm"] == "nccl"
    with pytest.raises(TopologyError):
        check_topology(4, cuda=FakeCuda(2), nvml=None)
