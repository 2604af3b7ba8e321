"""Kernel layout of MX-format (MXFP4 / MXFP8) expert weights.

Values are stored tile-contiguous: ``[E, ceil(rows/128), Kp/128, 128, 128*bits/8]`` so
that every (128-row, 128-element) block the tensor cores consume is one contiguous
8 KB (fp4) or 16 KB (fp8) run in HBM, which the TMA reads in one sweep.  Rows are
zero-padded to a multiple of 128 and K to ``Kp = roundup(K, 128)``.

The checkpoint stores, per expert, ``blocks [rows, K/32, 16]`` (two e2m1 per byte) and
``scales [rows, K/32]`` (ue8m0).  The tensor-core kernel reads:
* values ``[E, rows, Kp/2]`` (fp4) or ``[E, rows, Kp]`` (fp8) with K zero-padded to
  ``Kp = roundup(K, 128)`` (the TMA unpack-to-shared-memory mode for fp4 needs the
  inner extent to be a multiple of 128 elements);
* scales in 512-byte atoms ``[E, ceil(rows/128), Kp/128, 512]``: byte
  ``(r % 32) * 16 + (r // 32) * 4 + j`` of an atom holds the scale of row ``r`` (of 128)
  and 32-element block ``j`` (of 4); padding scales are 127 (2^0), never NaN.
Both conversions are exact (pure data movement).
"""

from __future__ import annotations

import torch


def round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def pad_k(values: torch.Tensor, K: int, fp4: bool = True) -> torch.Tensor:
    """values [..., rows, K/2] (fp4) or [..., rows, K] -> zero-padded along K to Kp."""
    Kp = round_up(K, 128)
    width = Kp // 2 if fp4 else Kp
    cur = values.shape[-1]
    if cur == width:
        return values.contiguous()
    out = torch.zeros(*values.shape[:-1], width, dtype=values.dtype, device=values.device)
    out[..., :cur] = values
    return out


def scales_to_atoms(scales: torch.Tensor, K: int) -> torch.Tensor:
    """scales [E, rows, K/32] uint8 -> atoms [E, ceil(rows/128), Kp/128, 512] uint8."""
    E, R, nb = scales.shape
    Kp = round_up(K, 128)
    Rp = round_up(R, 128)
    full = torch.full((E, Rp, Kp // 32), 127, dtype=torch.uint8, device=scales.device)
    full[:, :R, :nb] = scales
    # [E, Rb, 4(r//32), 32(r%32), Kg, 4(j)] -> [E, Rb, Kg, r%32, r//32, j]
    v = full.view(E, Rp // 128, 4, 32, Kp // 128, 4).permute(0, 1, 4, 3, 2, 5)
    return v.contiguous().view(E, Rp // 128, Kp // 128, 512)


def atoms_to_scales(atoms: torch.Tensor, rows: int, K: int) -> torch.Tensor:
    E, Rb, Kg, _ = atoms.shape
    v = atoms.view(E, Rb, Kg, 32, 4, 4).permute(0, 1, 4, 3, 2, 5).contiguous()
    full = v.view(E, Rb * 128, Kg * 4)
    return full[:, :rows, : K // 32].contiguous()


def unpad_k(values: torch.Tensor, K: int, fp4: bool = True) -> torch.Tensor:
    return values[..., : (K // 2 if fp4 else K)]


def tile_values(values: torch.Tensor, K: int, fp4: bool = True) -> torch.Tensor:
    """values [E, rows, K/2] (fp4) or [E, rows, K] (fp8) -> [E, Rb, Kb, 128, W] with
    W = 64 (fp4) or 128 (fp8): block (rb, kb) holds rows rb*128.. and K elements kb*128.."""
    E, R, _ = values.shape
    padded = pad_k(values, K, fp4)
    Rp = round_up(R, 128)
    if Rp != R:
        z = torch.zeros(E, Rp, padded.shape[-1], dtype=padded.dtype, device=padded.device)
        z[:, :R] = padded
        padded = z
    W = 64 if fp4 else 128
    Kb = padded.shape[-1] // W
    return padded.view(E, Rp // 128, 128, Kb, W).permute(0, 1, 3, 2, 4).contiguous()


def untile_values(tiled: torch.Tensor, rows: int, K: int, fp4: bool = True) -> torch.Tensor:
    E, Rb, Kb, _, W = tiled.shape
    flat = tiled.permute(0, 1, 3, 2, 4).reshape(E, Rb * 128, Kb * W)
    return flat[:, :rows, : (K // 2 if fp4 else K)].contiguous()


def tiled_shape(E: int, rows: int, K: int, fp4: bool = True) -> tuple[int, int, int, int, int]:
    return (E, -(-rows // 128), round_up(K, 128) // 128, 128, 64 if fp4 else 128)


def tile_bf16(w: torch.Tensor) -> torch.Tensor:
    """bf16 expert weights [E, rows, K] -> tiles [E, ceil(rows/128), Kp/64, 128, 64] (Kp = K
    rounded up to 64, rows and K zero-padded): every (128-row, 64-element) block the
    kind::f16 tensor-core MMA consumes is one contiguous 16 KB run."""
    E, R, K = w.shape
    Rp, Kp = round_up(R, 128), round_up(K, 64)
    full = torch.zeros(E, Rp, Kp, dtype=w.dtype, device=w.device)
    full[:, :R, :K] = w
    return full.view(E, Rp // 128, 128, Kp // 64, 64).permute(0, 1, 3, 2, 4).contiguous()


def untile_bf16(t: torch.Tensor, rows: int, K: int) -> torch.Tensor:
    E, Rb, Kb, _, _ = t.shape
    return t.permute(0, 1, 3, 2, 4).reshape(E, Rb * 128, Kb * 64)[:, :rows, :K]


def interleave_gate_up(w13: torch.Tensor) -> torch.Tensor:
    """[E, 2I, K] with gate rows then up rows -> rows gate0, up0, gate1, up1, ... (the
    kernels' SwiGLU epilogue pairs adjacent rows)."""
    E, I2, K = w13.shape
    I = I2 // 2
    return torch.stack([w13[:, :I], w13[:, I:]], dim=2).reshape(E, I2, K)
