"""Pre-flight topology check before tensor-parallel weights are loaded.

The in-kernel collectives store to and load from peer GPUs' memory, so every pair of ranks needs
peer access, and they are only fast over NVLink (NVSwitch on HGX B200: every GPU reaches every
peer at full bandwidth).  ``check_topology`` reads peer access from CUDA and the active NVLink
count per GPU from NVML and says which communicator fits; the reference runs an equivalent ring /
mesh degree check before it loads weights (``docs/gotchas.md:33-56``, ``scripts/ci/tp4_mesh.py``).
It only reads state; it changes no device setting.
"""
from __future__ import annotations


class TopologyError(RuntimeError):
    pass


def _nvml():
    try:
        import pynvml
        pynvml.nvmlInit()
        return pynvml
    except Exception:
        return None


def active_nvlinks(nvml, index: int, max_links: int = 18) -> int:
    h = nvml.nvmlDeviceGetHandleByIndex(index)
    n = 0
    for link in range(max_links):
        try:
            if nvml.nvmlDeviceGetNvLinkState(h, link) == 1:
                n += 1
        except Exception:
            break
    return n


def check_topology(world: int, *, comm: str = "fused", cuda=None, nvml="auto") -> dict:
    """Report for ranks 0..world-1 on this node; raises ``TopologyError`` when ``comm`` needs
    peer access that is missing."""
    if cuda is None:
        import torch
        cuda = torch.cuda
    n = cuda.device_count()
    if n < world:
        raise TopologyError(f"{world} ranks need {world} GPUs on the node, {n} visible")
    peer = [[i == j or bool(cuda.can_device_access_peer(i, j)) for j in range(world)] for i in range(world)]
    if nvml == "auto":
        nvml = _nvml()
    links = [active_nvlinks(nvml, i) for i in range(world)] if nvml is not None else None
    all_peer = all(all(r) for r in peer)
    nvlink = links is not None and all(k > 0 for k in links)
    report = dict(world=world, devices=n, peer_access=peer, nvlink_active_links=links,
                  recommended_comm="fused" if (all_peer and (nvlink or links is None)) else "nccl")
    if world > 1 and comm in ("fused", "peer") and not all_peer:
        missing = [(i, j) for i in range(world) for j in range(world) if not peer[i][j]]
        raise TopologyError(f"peer access missing between GPU pairs {missing[:8]}: use parallel.comm=nccl")
    return report
