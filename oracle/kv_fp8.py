"""Oracle: FP8 KV row quantisation (CPU).  Test infrastructure.

Restates ``act_quant_simulate`` (``flash_sparse/utils/quantization.py:19-36``;
the shipped code drops the call parentheses of ``.abs``) at block 64 on bf16
input, step for step in the input dtype as torch evaluates it:

    amax  = max(max|x| over the block, 1e-4)     (bf16)
    scale = amax / 448                             (bf16)
    q     = e4m3(clamp(x / scale, -448, 448))      (x / scale in bf16)
    deq   = bf16(float(q) * float(scale))

and lays the result out as the FP8 KV row the B200 attention reads
(the V4 production row of ``docs/ir_analysis.md:45-55``):
``[n_nope e4m3 | n_nope/64 fp32 scales | pad to 16 B | rope bf16 | pad to 16 B]``.
"""

from __future__ import annotations

import torch


def row_layout(D: int, n_nope: int):
    nblk = n_nope // 64
    rope_off = (n_nope + 4 * nblk + 15) // 16 * 16
    row_bytes = (rope_off + 2 * (D - n_nope) + 15) // 16 * 16
    return rope_off, row_bytes


def quant_blocks(x: torch.Tensor, block: int = 64):
    """bf16 ``[..., n]`` -> (e4m3 ``[..., n]``, bf16 scales ``[..., n/block]``, bf16 dequantised ``[..., n]``)."""
    assert x.dtype == torch.bfloat16
    *pre, n = x.shape
    b = x.reshape(*pre, n // block, block)
    amax = b.abs().amax(dim=-1, keepdim=True).clamp_min(1e-4)
    scale = amax / 448.0
    q = (b / scale).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    deq = (q.float() * scale).to(torch.bfloat16)
    return q.reshape(*pre, n), scale.squeeze(-1), deq.reshape(*pre, n)


def quantize_rows(kv: torch.Tensor, n_nope: int) -> torch.Tensor:
    """bf16 ``[..., D]`` -> FP8 rows ``[..., row_bytes]`` uint8."""
    D = kv.shape[-1]
    rope_off, rb = row_layout(D, n_nope)
    q, scale, _ = quant_blocks(kv[..., :n_nope].contiguous())
    rows = kv.reshape(-1, D)
    out = torch.zeros((rows.shape[0], rb), dtype=torch.uint8)
    out[:, :n_nope] = q.reshape(-1, n_nope).view(torch.uint8)
    out[:, n_nope:n_nope + 4 * (n_nope // 64)] = scale.float().reshape(-1, n_nope // 64).contiguous().view(torch.uint8)
    out[:, rope_off:rope_off + 2 * (D - n_nope)] = rows[:, n_nope:].contiguous().view(torch.uint8)
    return out.reshape(*kv.shape[:-1], rb)


def dequantize_rows(rows: torch.Tensor, D: int, n_nope: int) -> torch.Tensor:
    """FP8 rows -> bf16 ``[..., D]`` (``bf16(float(e4m3) * scale)`` and the bf16 rope dims)."""
    rope_off, rb = row_layout(D, n_nope)
    r = rows.reshape(-1, rb)
    q = r[:, :n_nope].contiguous().view(torch.float8_e4m3fn).float()
    sc = r[:, n_nope:n_nope + 4 * (n_nope // 64)].contiguous().view(torch.float32)
    deq = (q.reshape(-1, n_nope // 64, 64) * sc.unsqueeze(-1)).reshape(-1, n_nope).to(torch.bfloat16)
    rope = r[:, rope_off:rope_off + 2 * (D - n_nope)].contiguous().view(torch.bfloat16)
    return torch.cat([deq, rope], dim=-1).reshape(*rows.shape[:-1], D)
