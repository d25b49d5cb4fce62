"""Q4 weight format (utils/pack_weights.py) -- packing on the host or device.

Format (utils/pack_weights.py:18-46): the tensor is flattened row-major,
zero-padded to a multiple of 32, and split into groups of 32; scale =
max|w|/7 in fp32 (0 -> 1.0); code = round-half-even(w/scale) clamped to
[-8, 7]; nibble = code + 8; byte b = nib[2b] | nib[2b+1] << 4; scales are
stored fp16.  ``pack_q4`` runs the CUDA packer for device tensors and a torch
implementation for host tensors (the offline converter path; decode never
packs).
"""
from __future__ import annotations

import torch

GROUP = 32


def pack_q4_host(w: torch.Tensor):
    """Host packer (offline conversion): returns (uint8[n_pad/2], float16[n_pad/32])."""
    flat = w.detach().to(torch.float32).reshape(-1).cpu()
    pad = (GROUP - flat.numel() % GROUP) % GROUP
    if pad:
        flat = torch.cat([flat, torch.zeros(pad, dtype=torch.float32)])
    blocks = flat.view(-1, GROUP)
    scales = blocks.abs().amax(dim=1) / 7.0
    scales = torch.where(scales == 0, torch.ones_like(scales), scales)
    codes = torch.round(blocks / scales[:, None]).clamp_(-8, 7).to(torch.int16) + 8
    u = codes.to(torch.uint8).reshape(-1)
    packed = u[0::2] | (u[1::2] << 4)
    return packed.contiguous(), scales.to(torch.float16)


def pack_q4(w: torch.Tensor):
    """Pack ``w`` into the Q4 format on the tensor's own device."""
    if w.is_cuda:
        from .kernels import q4_pack_device
        return q4_pack_device(w.detach().to(torch.float32).contiguous())
    return pack_q4_host(w)
