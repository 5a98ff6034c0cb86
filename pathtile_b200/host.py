"""Host-buffer entry point: the full FWD + dX + dK pass on CPU-resident tensors.

A caller that holds x, k and dy in (pinned) host memory gets y, dX and dK back
in host memory.  The batch is cut into chunks that flow through a ring of
device staging buffers on two streams, so that the host-to-device copy of one
chunk, the kernels of the previous one and the device-to-host copy of the one
before overlap (PCIe is full duplex).  The backward of a chunk is one
ops.dx_dk call (the fused dX + dK kernel where it applies); dK accumulates
over chunks on the device (deterministic per chunk, fixed chunk order) and is
copied back once.  Every kernel is the native library's; nothing is computed
on the host.
"""
from __future__ import annotations

import contextlib
import os
from typing import Iterator, Sequence

import torch

from . import ops


def cpus_from_mask(words: Sequence[int]) -> list[int]:
    """CPU ids set in an NVML CPU-affinity mask (bit i of 64-bit word w is CPU 64 w + i)."""
    return [64 * w + i for w, word in enumerate(words) for i in range(64) if (int(word) >> i) & 1]


def device_local_cpus(device: int | torch.device) -> list[int]:
    """The CPUs NVML reports as local to `device` (its NUMA node), or [] when NVML
    cannot say.  The GPU is found by PCI bus id, so CUDA_VISIBLE_DEVICES
    renumbering does not matter."""
    try:
        import pynvml

        props = torch.cuda.get_device_properties(device)
        bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
        pynvml.nvmlInit()
        try:
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            words = pynvml.nvmlDeviceGetCpuAffinity(handle, ((os.cpu_count() or 64) + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
    except Exception:  # no NVML or no such device: leave placement to the OS
        return []
    return cpus_from_mask(words)


@contextlib.contextmanager
def near_device(device: int | torch.device) -> Iterator[list[int]]:
    """Run the block with the calling thread bound to the CPUs local to `device`.

    Pinned host buffers allocated inside land on the GPU's NUMA node (Linux
    places pages where they are first touched), so their copies do not cross
    the inter-socket link.  With several GPUs per host each rank's buffers then
    sit next to its own GPU.  Yields the CPUs used ([] = unchanged: NVML had no
    answer, or none of its CPUs is allowed to this process); the previous
    affinity is restored on exit.
    """
    before = os.sched_getaffinity(0)
    cpus = [c for c in device_local_cpus(device) if c in before]
    if cpus:
        os.sched_setaffinity(0, cpus)
    try:
        yield cpus
    finally:
        if cpus:
            os.sched_setaffinity(0, before)


class HostPipeline:
    """Reusable staging buffers and streams for one device and one [H, L, K] shape."""

    def __init__(self, H: int, L: int, K: int, chunk_b: int = 1024, device: int | torch.device = 0,
                 depth: int = 3) -> None:
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        self.H, self.L, self.K = H, L, K
        self.chunk_b = int(chunk_b)
        self.depth = int(depth)
        with torch.cuda.device(self.device):
            shape = (self.chunk_b, H, L)
            self.x = [torch.empty(shape, device=self.device) for _ in range(self.depth)]
            self.dy = [torch.empty(shape, device=self.device) for _ in range(self.depth)]
            self.y = [torch.empty(shape, device=self.device) for _ in range(self.depth)]
            self.gx = [torch.empty(shape, device=self.device) for _ in range(self.depth)]
            self.k = torch.empty(H, K, device=self.device)
            self.gk = torch.empty(H, K, device=self.device)
            self.copy_in = torch.cuda.Stream(self.device)
            self.compute = torch.cuda.Stream(self.device)
            self.copy_out = torch.cuda.Stream(self.device)
            self.in_done = [torch.cuda.Event() for _ in range(self.depth)]
            self.comp_done = [torch.cuda.Event() for _ in range(self.depth)]
            self.out_done = [torch.cuda.Event() for _ in range(self.depth)]

    def bytes_per_call(self, B: int) -> tuple[int, int]:
        """(host-to-device, device-to-host) bytes of one call at batch B."""
        act = B * self.H * self.L * 4
        return 2 * act + self.H * self.K * 4, 2 * act + self.H * self.K * 4

    def run(self, x_h: torch.Tensor, k_h: torch.Tensor, dy_h: torch.Tensor, y_h: torch.Tensor,
            gx_h: torch.Tensor, gk_h: torch.Tensor) -> None:
        """y_h, gx_h, gk_h <- FWD, dX, dK of (x_h, k_h, dy_h); all host tensors.

        Asynchronous: returns once everything is queued; the caller synchronises
        (``torch.cuda.synchronize`` or an event on ``self.copy_out``)."""
        B, H, L = map(int, x_h.shape)
        if (H, L) != (self.H, self.L) or tuple(k_h.shape) != (self.H, self.K):
            raise ValueError("shape does not match this pipeline")
        dev = self.device
        cur = torch.cuda.current_stream(dev)
        for s in (self.copy_in, self.compute, self.copy_out):
            s.wait_stream(cur)
        with torch.cuda.device(dev):
            with torch.cuda.stream(self.copy_in):
                self.k.copy_(k_h, non_blocking=True)
                k_ready = torch.cuda.Event()
                k_ready.record(self.copy_in)
            self.compute.wait_event(k_ready)
            n = (B + self.chunk_b - 1) // self.chunk_b
            for i in range(n):
                slot = i % self.depth
                b0, b1 = i * self.chunk_b, min(B, (i + 1) * self.chunk_b)
                nb = b1 - b0
                if i >= self.depth:  # slot reused: its outputs must have left the device
                    self.copy_in.wait_event(self.out_done[slot])
                with torch.cuda.stream(self.copy_in):
                    self.x[slot][:nb].copy_(x_h[b0:b1], non_blocking=True)
                    self.dy[slot][:nb].copy_(dy_h[b0:b1], non_blocking=True)
                    self.in_done[slot].record(self.copy_in)
                self.compute.wait_event(self.in_done[slot])
                with torch.cuda.stream(self.compute):
                    xs, dys = self.x[slot][:nb], self.dy[slot][:nb]
                    ops.fwd(xs, self.k, self.y[slot][:nb])
                    ops.dx_dk(dys, xs, self.k, self.gk, gx=self.gx[slot][:nb], mode="deterministic",
                              accumulate=(i > 0))
                    self.comp_done[slot].record(self.compute)
                self.copy_out.wait_event(self.comp_done[slot])
                with torch.cuda.stream(self.copy_out):
                    y_h[b0:b1].copy_(self.y[slot][:nb], non_blocking=True)
                    gx_h[b0:b1].copy_(self.gx[slot][:nb], non_blocking=True)
                    self.out_done[slot].record(self.copy_out)
            self.copy_out.wait_stream(self.compute)
            with torch.cuda.stream(self.copy_out):
                gk_h.copy_(self.gk, non_blocking=True)
            cur.wait_stream(self.copy_out)

    def launches_per_call(self, B: int) -> int:
        """Native kernel launches of one call: per chunk, FWD and the backward's."""
        n = 0
        for b0 in range(0, B, self.chunk_b):
            nb = min(self.chunk_b, B - b0)
            n += 1 + ops.dx_dk_launches(nb, self.H, self.L, self.K)
        return n
