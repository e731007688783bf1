"""TEST INFRASTRUCTURE ONLY: numpy restatement of the reference KV codec.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU baseline use this
module, as the checker.  The product path (``secure_infer_b200``) runs the
codec in CUDA and never imports anything under ``oracle/``.

Restated from (paths relative to the reference project):
  * ``settings`` / ``layer_bits``  -- secure_infer/kv_offload/transport_codec.py:9-19
  * ``encode``                      -- secure_infer/kv_offload/transport_codec.py:22-42
  * ``decode_into``                 -- secure_infer/kv_offload/optimized_decode.py:5-27
  * ``encode_torch`` / ``decode_into_torch`` -- the same two steps with the
    reference's torch CPU ops (the CPU baseline's codec, multi-threaded by torch)

Layout of one bf16 KV slice: ``[block][token=128][head][dim]``.  Grouping:
kind 0 (K) reduces 64 consecutive tokens of one (head, dim) channel; kind 1
(V) reduces 64 consecutive dims of one (token, head).  A packet row is
``q || scale fp32[E/64] || low fp32[E/64] || int32{1, layer, kind, bits}``
zero padded to a multiple of 16 bytes, E = 128*heads*dim.

All arithmetic is IEEE fp32 with one rounding per operation, exactly as the
reference's torch CPU ops evaluate it: scale = (high-low)/(2^bits-1) clamped
below at fp32(1e-12), q = clamp(round_half_even((x-low)/scale)), and decode
v = fp32(q*scale) then fp32(v+low) then round-to-nearest-even bf16.
"""
from __future__ import annotations

import math

import numpy as np

GROUP = 64


def layer_bits(mode: str, layer: int, layers: int) -> int:
    """transport_codec.py:18-19."""
    return 8 if mode == "int8" or (mode == "mixed" and layer < math.ceil(layers / 3)) else 4


def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    return (u16.astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_to_bf16(f: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits (finite inputs)."""
    u = np.ascontiguousarray(f, dtype=np.float32).view(np.uint32)
    rounding = ((u >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    return ((u + rounding) >> np.uint32(16)).astype(np.uint16)


def packet_geometry(heads: int, dim: int, bits: int, tokens: int = 128):
    elements = tokens * heads * dim
    qb = elements * bits // 8
    sb = elements // GROUP * 4
    width = (qb + 2 * sb + 16 + 15) // 16 * 16
    return qb, sb, width


def _grouped(x: np.ndarray, kind: int) -> tuple[np.ndarray, int]:
    b, t, h, d = x.shape
    if kind == 0:
        return x.reshape(b, t // GROUP, GROUP, h, d), 2
    return x.reshape(b, t, h, d // GROUP, GROUP), 4


def encode(source_bf16: np.ndarray, indices, bits: int, kind: int, layer: int):
    """source_bf16: uint16 array [num_blocks, 128, heads, dim] (bf16 bits)."""
    idx = np.asarray(indices, dtype=np.int64)
    x = bf16_to_f32(source_bf16[idx])
    if x.ndim != 4 or x.shape[1] != 128:
        raise ValueError(tuple(x.shape))
    b = x.shape[0]
    xg, axis = _grouped(x, kind)
    low = xg.min(axis=axis, keepdims=True)
    high = xg.max(axis=axis, keepdims=True)
    levels = np.float32((1 << bits) - 1)
    scale = np.maximum((high - low) / levels, np.float32(1e-12)).astype(np.float32)
    q = np.clip(np.rint((xg - low) / scale), 0, (1 << bits) - 1).reshape(b, -1)
    if bits == 4:
        q = q[:, 0::2] + 16 * q[:, 1::2]
    q = q.astype(np.uint8)
    qb = q.shape[1]
    sb = scale[0].size * 4
    width = (qb + 2 * sb + 16 + 15) // 16 * 16
    packet = np.zeros((b, width), dtype=np.uint8)
    packet[:, :qb] = q
    packet[:, qb:qb + sb] = np.ascontiguousarray(scale).view(np.uint8).reshape(b, -1)
    packet[:, qb + sb:qb + 2 * sb] = np.ascontiguousarray(low).view(np.uint8).reshape(b, -1)
    header = np.array([1, layer, kind, bits], dtype="<i4").view(np.uint8)
    packet[:, qb + 2 * sb:qb + 2 * sb + 16] = header
    return packet, qb, sb


def encode_torch(source_bf16, indices, bits: int, kind: int, layer: int):
    """transport_codec.py:22-42 with torch CPU ops, as the reference runs it
    (amin/amax over the group axis, true division, round-half-even, clamp);
    multi-threaded by torch.  source_bf16: uint16 numpy array or bf16 tensor
    [num_blocks, 128, heads, dim].  Same packets as ``encode``."""
    import torch
    src = source_bf16 if isinstance(source_bf16, torch.Tensor) else \
        torch.from_numpy(np.ascontiguousarray(source_bf16).view(np.int16)).view(torch.bfloat16)
    x = src[torch.as_tensor(np.asarray(indices, dtype=np.int64))].float()
    b, t, h, d = x.shape
    if kind == 0:
        xg, axis = x.view(b, t // GROUP, GROUP, h, d), 2
    else:
        xg, axis = x.view(b, t, h, d // GROUP, GROUP), 4
    low = xg.amin(dim=axis, keepdim=True)
    high = xg.amax(dim=axis, keepdim=True)
    levels = float((1 << bits) - 1)
    scale = torch.clamp((high - low) / levels, min=1e-12)
    q = torch.clamp(torch.round((xg - low) / scale), 0, levels).reshape(b, -1)
    if bits == 4:
        q = q[:, 0::2] + 16 * q[:, 1::2]
    q = q.to(torch.uint8)
    qb = q.shape[1]
    sb = scale[0].numel() * 4
    width = (qb + 2 * sb + 16 + 15) // 16 * 16
    packet = torch.zeros((b, width), dtype=torch.uint8)
    packet[:, :qb] = q
    packet[:, qb:qb + sb] = scale.reshape(b, -1).contiguous().view(torch.uint8)
    packet[:, qb + sb:qb + 2 * sb] = low.reshape(b, -1).contiguous().view(torch.uint8)
    packet[:, qb + 2 * sb:qb + 2 * sb + 16] = torch.tensor([1, layer, kind, bits], dtype=torch.int32).view(torch.uint8)
    return packet.numpy(), qb, sb


def decode_into(wire: np.ndarray, destination_bf16: np.ndarray, indices, bits: int,
                kind: int, qbytes: int, sbytes: int) -> None:
    """wire: uint8 [b, width]; destination_bf16: uint16 [num_blocks, 128, H, D]."""
    b = wire.shape[0]
    _, tokens, heads, dim = destination_bf16.shape
    q = wire[:, :qbytes]
    if bits == 8:
        full = q.astype(np.float32)
    else:
        lo = (q & 0xF).astype(np.float32)
        hi = (q >> 4).astype(np.float32)
        full = np.stack((lo, hi), axis=-1).reshape(b, -1)
    params = np.ascontiguousarray(wire).view(np.float32)
    scale = params[:, qbytes // 4:(qbytes + sbytes) // 4]
    offset = params[:, (qbytes + sbytes) // 4:(qbytes + 2 * sbytes) // 4]
    if kind == 0:
        shape = (b, tokens // GROUP, GROUP, heads, dim)
        pshape = (b, tokens // GROUP, 1, heads, dim)
    else:
        shape = (b, tokens, heads, dim // GROUP, GROUP)
        pshape = (b, tokens, heads, dim // GROUP, 1)
    values = full.reshape(shape) * scale.reshape(pshape)
    values = (values + offset.reshape(pshape)).astype(np.float32)
    restored = f32_to_bf16(values.reshape(b, tokens, heads, dim))
    destination_bf16[np.asarray(indices, dtype=np.int64)] = restored


def decode_into_torch(wire, destination, indices, bits: int, kind: int, qbytes: int, sbytes: int,
                      temporary=None):
    """optimized_decode.py:5-27 with torch CPU ops, as the reference runs it:
    int8 q -> fp32; int4 hi = floor(p / 16), lo = p - 16 hi, interleaved lo,
    hi; then in place v *= scale, v += offset (two fp32 roundings), RNE to
    the destination's bf16 and ``index_copy_`` along the block axis.
    wire: uint8 tensor [b, width]; destination: bf16 tensor [num_blocks, 128,
    heads, dim]; indices: int64 tensor.  Returns the fp32 work buffer, which a
    caller may pass back as `temporary`."""
    import torch
    b = wire.shape[0]
    _, tokens, heads, dim = destination.shape
    total = b * tokens * heads * dim
    work = temporary if temporary is not None and temporary.numel() >= total else \
        torch.empty(total, dtype=torch.float32)
    q = wire[:, :qbytes]
    full = work[:total].view(b, -1)
    if bits == 8:
        full.copy_(q)
    else:
        p = q.float()
        hi = torch.floor(p / 16)
        torch.stack((p - 16 * hi, hi), dim=-1, out=full.view(b, -1, 2))
    if kind == 0:
        shape, pshape = (b, tokens // GROUP, GROUP, heads, dim), (b, tokens // GROUP, 1, heads, dim)
    else:
        shape, pshape = (b, tokens, heads, dim // GROUP, GROUP), (b, tokens, heads, dim // GROUP, 1)
    params = wire.view(torch.float32)
    scale = params[:, qbytes // 4:(qbytes + sbytes) // 4].reshape(pshape)
    offset = params[:, (qbytes + sbytes) // 4:(qbytes + 2 * sbytes) // 4].reshape(pshape)
    v = full.view(shape)
    v.mul_(scale)
    v.add_(offset)
    destination.index_copy_(0, indices, v.reshape(b, tokens, heads, dim).to(destination.dtype))
    return work
