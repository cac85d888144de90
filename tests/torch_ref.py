"""Torch (fp32) references of the expert FFN for GPU-sized checks.

Floating-point kernels are checked against a plain fp32 computation of the
same op on the same inputs; these helpers run it on the GPU for shapes the
numpy oracle would take minutes on (Mixtral-sized experts). The nibble order
is the packed layout of include/phmoe.h (restated by oracle.moe_oracle.
unpack_nibbles, which the CPU test of this module pins it to)."""

from __future__ import annotations

import torch
import torch.nn.functional as F


def unpack_nibbles_torch(q: torch.Tensor) -> torch.Tensor:
    """uint8 [..., K/2] -> int nibbles [..., K] (0..15) in element order."""
    b = q.view(*q.shape[:-1], q.shape[-1] // 4, 4).to(torch.int16)
    lo, hi = b & 15, b >> 4
    # bytes (e0|e2<<4, e4|e6<<4, e1|e3<<4, e5|e7<<4)
    e = torch.stack([lo[..., 0], lo[..., 2], hi[..., 0], hi[..., 2],
                     lo[..., 1], lo[..., 3], hi[..., 1], hi[..., 3]], dim=-1)
    return e.reshape(*q.shape[:-1], q.shape[-1] * 2)


def dequant_torch(q: torch.Tensor, s: torch.Tensor, group: int) -> torch.Tensor:
    """Exact fp32 (nibble - 8) * scale."""
    n = unpack_nibbles_torch(q).float() - 8.0
    K = n.shape[-1]
    return (n.view(*n.shape[:-1], K // group, group) * s.float().unsqueeze(-1)).view(*n.shape[:-1], K)


def ffn_rows_torch(x, row_token, offsets, w13_q, w13_s, w2_q, w2_s, group, *, operand_dtype=None):
    """y[r] for every dispatched row r, expert by expert, in fp32. With
    ``operand_dtype`` (torch.float16 for the prefill GEMMs) the dequantised
    weights and the SwiGLU output are rounded to it, as the kernels do."""
    R = row_token.numel()
    H = x.shape[1]
    y = torch.zeros(R, H, dtype=torch.float32, device=x.device)
    off = offsets.cpu().tolist()
    E = w13_q.shape[0]
    for e in range(E):
        a, b = off[e], off[e + 1]
        if a == b:
            continue
        w13 = dequant_torch(w13_q[e], w13_s[e], group)
        w2 = dequant_torch(w2_q[e], w2_s[e], group)
        if operand_dtype is not None:
            w13, w2 = w13.to(operand_dtype).float(), w2.to(operand_dtype).float()
        xe = x[row_token[a:b].long()].float()
        gu = xe @ w13.T
        I = w13.shape[0] // 2
        h = F.silu(gu[:, :I]) * gu[:, I:]
        if operand_dtype is not None:
            h = h.to(operand_dtype).float()
        y[a:b] = h @ w2.T
    return y


def layer_torch(x, idx, w, offsets, row_token, inv, packed, group):
    """Whole layer on given routing: combine of ffn_rows_torch in slot order."""
    y = ffn_rows_torch(x, row_token, offsets, *packed, group)
    out = torch.zeros(x.shape[0], x.shape[1], dtype=torch.float32, device=x.device)
    for j in range(idx.shape[1]):
        out += w[:, j:j + 1] * y[inv[:, j].long()]
    return out
