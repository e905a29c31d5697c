"""Layer-sharded whole-model quantization across the GPUs of one node.

Whole-model weight quantization and KV-cache quantization are independent per
layer, so N ranks (one process per GPU, torch.distributed over NCCL) each
take a contiguous block of layers and run the quantization kernels with no
data-path collective.  The only exchange is the final gather of each rank's
packed results (4-bit codes + scales) to rank 0 over NVLink: one flat byte
buffer per rank, sent point to point at its exact size.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Dict, List, Sequence

import torch
import torch.distributed as dist


def layer_block(num_layers: int, rank: int, world: int) -> range:
    """Contiguous block of layers owned by `rank` (sizes differ by at most one)."""
    if not (0 <= rank < world):
        raise ValueError(f"rank {rank} outside world of {world}")
    base, extra = divmod(num_layers, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


@dataclass
class PackedLayer:
    """Packed NF4 result of one layer: per weight (codes, scales, q_scales, dq_scales)."""
    index: int
    tensors: Dict[str, torch.Tensor]


_ALIGN = 16


def _padded(nb: int) -> int:
    return (nb + _ALIGN - 1) // _ALIGN * _ALIGN


def flatten_bytes(tensors: Sequence[torch.Tensor]) -> torch.Tensor:
    """Concatenate tensors' raw bytes into one uint8 buffer (on their device),
    each part starting on a 16-byte boundary."""
    tensors = list(tensors)
    if not tensors:
        return torch.empty(0, dtype=torch.uint8)
    total = sum(_padded(t.numel() * t.element_size()) for t in tensors)
    buf = torch.zeros(total, dtype=torch.uint8, device=tensors[0].device)
    off = 0
    for t in tensors:
        nb = t.numel() * t.element_size()
        buf[off:off + nb].copy_(t.contiguous().view(-1).view(torch.uint8))
        off += _padded(nb)
    return buf


def unflatten_bytes(buf: torch.Tensor, like: Sequence[torch.Tensor]) -> List[torch.Tensor]:
    """Inverse of flatten_bytes given tensors of the same shapes / dtypes."""
    out, off = [], 0
    for t in like:
        nb = t.numel() * t.element_size()
        out.append(buf[off:off + nb].view(t.dtype).view(t.shape))
        off += _padded(nb)
    return out


def gather_to_rank0(local: torch.Tensor, group=None) -> List[torch.Tensor] | None:
    """Gather each rank's flat uint8 buffer to rank 0, exact sizes.

    One all_gather of the sizes; then every other rank sends its buffer to
    rank 0 point to point, all transfers posted together (batch_isend_irecv)
    so they overlap on rank 0's links.  Nothing is padded: a rank with fewer
    layers sends fewer bytes.  Returns the per-rank buffers on rank 0 (its
    own is `local` itself), None elsewhere."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    dev = local.device
    n = torch.tensor([local.numel()], dtype=torch.int64, device=dev)
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n, group=group)
    sizes = [int(s.item()) for s in sizes]

    def peer(r: int) -> int:
        return r if group is None else dist.get_global_rank(group, r)

    if rank == 0:
        bufs = [local] + [torch.empty(sz, dtype=torch.uint8, device=dev) for sz in sizes[1:]]
        ops = [dist.P2POp(dist.irecv, bufs[r], peer(r), group) for r in range(1, world) if sizes[r]]
    else:
        bufs = None
        ops = [dist.P2POp(dist.isend, local.contiguous(), peer(0), group)] if sizes[rank] else []
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    return bufs


def quantize_layers(num_layers: int, rank: int, world: int,
                    quantize_layer: Callable[[int], PackedLayer]) -> List[PackedLayer]:
    """Run `quantize_layer` on this rank's block of layers (no collective)."""
    return [quantize_layer(i) for i in layer_block(num_layers, rank, world)]
