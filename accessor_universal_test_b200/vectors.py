"""Device buffers of encoded vectors (torch supplies the memory, libautdot
does the work).

``encoded(ws, "e8m0", DENSE, kind, seed, vector_id, n)`` generates the seeded
synthetic values on the GPU (aut_generate) and encodes them on the GPU
(aut_encode) into a uint8 tensor of aut_storage_bytes() bytes -- the layout
the reference's kernels read (dense LSB-first words + guard word, or padded
containers).
"""
from __future__ import annotations

import torch

from . import _lib

# Values generated and encoded per step; a multiple of every dense chunk
# (lcm of 32 / gcd(bits, 32) over all widths divides 2^7 * 3 * 5 * 7 ... so a
# power of two times 1 is enough for aligned word offsets: 2^22 * B bits is
# always a whole number of 32-bit words).
_CHUNK = 1 << 22


def encoded(ws: _lib.Workspace, fmt: str | int, layout: int, kind: int, seed: int,
            vector_id: int, n: int, first: int = 0, device=None,
            stream: int = 0) -> torch.Tensor:
    fid = _lib.format_id(fmt) if isinstance(fmt, str) else fmt
    family, bits, _, _ = _lib.format_info(fid)
    device = device if device is not None else torch.device("cuda", ws.device)
    nbytes = _lib.storage_bytes(fid, layout, n)
    out = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=device)
    if n == 0:
        out.zero_()
        return out
    scratch = torch.empty(min(n, _CHUNK), dtype=torch.float64, device=device)
    stride = 64 if family == _lib.FAMILY_RAW_FP64 else (
        bits if layout == _lib.DENSE or family == _lib.FAMILY_RAW_FP32 else
        (8 if bits <= 8 else 16 if bits <= 16 else 32))
    done = 0
    while done < n:
        m = min(_CHUNK, n - done)
        _lib.generate(kind, seed, vector_id, first + done, m, scratch.data_ptr(), stream)
        byte_off = done * stride // 8
        if family == _lib.FAMILY_RAW_FP64:
            out[byte_off:byte_off + m * 8].view(torch.float64).copy_(scratch[:m])
        else:
            ws.encode(fid, layout, scratch.data_ptr(), m, out.data_ptr() + byte_off, stream)
        done += m
    return out


def decoded(ws: _lib.Workspace, fmt: str | int, layout: int, codes: torch.Tensor, n: int,
            target: int = _lib.TARGET_FP64, stream: int = 0) -> torch.Tensor:
    fid = _lib.format_id(fmt) if isinstance(fmt, str) else fmt
    dtype = torch.float64 if target == _lib.TARGET_FP64 else torch.float32
    out = torch.empty(max(n, 1), dtype=dtype, device=codes.device)
    ws.decode(fid, layout, target, codes.data_ptr(), n, out.data_ptr(), stream)
    return out[:n]
