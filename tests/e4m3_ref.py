"""Test-side statement of the FP8 path's storage format (plain torch on any device), used to check the CUDA kernels.

Values are e4m3 (torch.float8_e4m3fn) with one power-of-two scale per block: the UE8M0 byte e gives the scale
2^(e - 127), chosen as the smallest power of two with amax / scale <= 448 (an all-zero block gets e = 127).  With
amax = m 2^E (m in [0.5, 1), torch.frexp), that is e - 127 = E - 9 + (m > 0.875).  Activations use 1 x 32 blocks;
weights 1 x 128 blocks (the scale repeated over the block's four 32-column slots).

Scale atoms: for a [rows, C] matrix, one 512-byte atom per (128-row tile, 128-column block); row r of the tile and
32-column block j sit at byte (r % 32) * 16 + (r // 32) * 4 + j % 4 of atom (r_global // 128) * (C // 128) + j // 4.
"""

import torch

E4M3_MAX = 448.0


def ue8m0(amax: torch.Tensor) -> torch.Tensor:
    """UE8M0 byte (int32 tensor) per block max |x| (>= 0)."""
    m, E = torch.frexp(amax.float())
    e = E - 9 + (m > 0.875).to(E.dtype) + 127
    e = e.clamp(0, 254)
    return torch.where(amax == 0, torch.full_like(e, 127), e)


def quant_blocks(x: torch.Tensor, block: int):
    """x [rows, C] fp32 -> (e4m3 values [rows, C], scale bytes [rows, C // block] int32)."""
    rows, C = x.shape
    xb = x.float().view(rows, C // block, block)
    e = ue8m0(xb.abs().amax(dim=2))
    inv = torch.pow(2.0, (127 - e).double()).float()
    q = (xb * inv[..., None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return q.view(rows, C), e


def dequant(q: torch.Tensor, e: torch.Tensor, block: int) -> torch.Tensor:
    rows, C = q.shape
    s = torch.pow(2.0, (e - 127).double()).float()
    return (q.float().view(rows, C // block, block) * s[..., None]).view(rows, C)


def atom_index(rows: int, C: int, device=None):
    """Byte offset inside the atoms of every (row, 32-block j) entry: int64 tensor [rows, C // 32]."""
    r = torch.arange(rows, device=device)[:, None]
    j = torch.arange(C // 32, device=device)[None, :]
    rr = r % 128
    return ((r // 128) * (C // 128) + j // 4) * 512 + (rr % 32) * 16 + (rr // 32) * 4 + j % 4


def atoms_from_bytes(e32: torch.Tensor, shift: int = 0, tiles: int | None = None) -> torch.Tensor:
    """Scale bytes per (row, 32-block) [rows, C // 32] -> the atoms of row-shifted layout `shift` (row x at x + shift);
    positions no row maps to hold 127."""
    rows, nb = e32.shape
    C = nb * 32
    tiles = tiles if tiles is not None else (rows + shift + 127) // 128
    out = torch.full((tiles * (C // 128) * 512,), 127, dtype=torch.uint8, device=e32.device)
    idx = atom_index(rows + shift, C, e32.device)[shift:]
    out[idx.reshape(-1)] = e32.to(torch.uint8).reshape(-1)
    return out


def bytes_from_atoms(atoms: torch.Tensor, rows: int, C: int, shift: int = 0) -> torch.Tensor:
    idx = atom_index(rows + shift, C, atoms.device)[shift:]
    return atoms[idx.reshape(-1)].view(rows, C // 32).to(torch.int32)


def quant_weight(w: torch.Tensor):
    """W [N, Kt] -> (e4m3 [N, Kt], atoms [Kt // 128][N // 128][512], per-32-column bytes [N, Kt // 32])."""
    N, Kt = w.shape
    q, e128 = quant_blocks(w, 128)
    e32 = e128.repeat_interleave(4, dim=1)
    # weight atoms: (k block, n tile) order
    r = torch.arange(N, device=w.device)[:, None]
    j = torch.arange(Kt // 32, device=w.device)[None, :]
    rr = r % 128
    idx = ((j // 4) * (N // 128) + r // 128) * 512 + (rr % 32) * 16 + (rr // 32) * 4 + j % 4
    atoms = torch.empty(N * Kt // 32, dtype=torch.uint8, device=w.device)
    atoms[idx.reshape(-1)] = e32.to(torch.uint8).reshape(-1)
    return q, atoms, e32
