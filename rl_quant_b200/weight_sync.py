"""Per-iteration weight hand-over across GPUs.

One process per GPU runs its own inference copy; after each PPO update the
source rank refreshes its copy from the fp32 master (cast-copy + requantise,
``InferenceRunner.sync_weights_from``) and every rank receives the result in
ONE collective: all tensors the fused forward reads live in a single
contiguous device blob, broadcast with NCCL over NVLink.

``PackedWeights`` moves a module's parameters and buffers into that blob in
place: parameters keep their ``nn.Parameter`` objects (their ``.data`` becomes
a view of the blob), buffers are re-registered as views, names/shapes/dtypes
are unchanged, so state dicts, ``requantize_`` and the fused kernels keep
working. Pack before capturing CUDA graphs (captured graphs hold addresses).
"""
from __future__ import annotations

import torch
import torch.nn as nn

_ALIGN = 256


def _tensors(model: nn.Module, include_params: bool):
    for mod_name, mod in model.named_modules():
        if include_params:
            for n, p in mod.named_parameters(recurse=False):
                yield mod, n, p, True
        for n, b in mod.named_buffers(recurse=False):
            if b is None or n.startswith("_") or n == "num_batches_tracked":
                continue
            yield mod, n, b, False


def pack_layout(sizes: list[int]) -> tuple[list[int], int]:
    """Offsets of tensors of `sizes` bytes in the blob and its size: each tensor at the
    first 256-byte boundary after the previous one (the rule of glad_pack_layout)."""
    offs, off = [], 0
    for n in sizes:
        offs.append(off)
        off += (n + _ALIGN - 1) // _ALIGN * _ALIGN
    return offs, max(off, _ALIGN)


class PackedWeights:
    def __init__(self, model: nn.Module, include_params: bool = True):
        items = []
        seen = set()
        for mod, name, t, is_param in _tensors(model, include_params):
            if t.data_ptr() in seen:
                continue
            seen.add(t.data_ptr())
            items.append((mod, name, t, is_param))
        offs, off = pack_layout([t.numel() * t.element_size() for _, _, t, _ in items])
        items = [(mod, name, t, is_param, o, t.numel() * t.element_size())
                 for (mod, name, t, is_param), o in zip(items, offs)]
        if not items:
            raise ValueError("nothing to pack")
        device = items[0][2].device
        self.blob = torch.zeros(off, dtype=torch.uint8, device=device)
        self.entries = []
        with torch.no_grad():
            for mod, name, t, is_param, o, nbytes in items:
                if not t.is_contiguous():
                    raise ValueError(f"{name}: only contiguous tensors can be packed")
                view = self.blob[o:o + nbytes].view(t.dtype).view(t.shape)
                view.copy_(t)
                if is_param:
                    getattr(mod, name).data = view
                else:
                    mod._buffers[name] = view
                self.entries.append((name, o, nbytes))
        self.nbytes = off

    def broadcast(self, src: int = 0, group=None) -> None:
        """One collective for every weight (NCCL over NVLink on GPUs)."""
        import torch.distributed as dist
        dist.broadcast(self.blob, src=src, group=group)

    def checksum(self) -> int:
        """Order-independent integer checksum of the packed bytes."""
        return int(self.blob.to(torch.int64).sum().item())
