"""Resident-block and occupancy calculator for B200 (sm_100a).

Given a kernel's launch shape and resources (threads per block, registers per
thread, shared memory per block, TMEM columns per block) this returns how many
blocks of it fit on one SM at once, which resource stops the next one, and
how the grid maps onto waves over the 148 SMs. The per-SM limits are the
published compute-capability 10.0 figures:

* 65,536 32-bit registers, allocated per warp in units of 256 (a thread's
  count rounds up to a multiple of 8), at most 255 per thread;
* 2,048 resident threads (64 warps) and 32 resident blocks;
* 228 KB of shared memory, at most 227 KB per block, and 1 KB per block kept
  by the system; allocation granularity 128 bytes;
* 512 TMEM columns (128 lanes x 32 bits each): a block that allocates N
  columns (a power of two >= 32) leaves room for 512 / N such blocks.

Reference parity: the reference's occupancy estimate for its own GPU
(kore/verifier/pmc.py:335-517, waves per SIMD from VGPR / LDS); this is the
same question asked of the B200's resources.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, asdict
from typing import Optional

SMS = 148
REGS_PER_SM = 65536
REG_ALLOC_UNIT = 256            # registers per warp allocation unit
MAX_REGS_PER_THREAD = 255
MAX_THREADS_PER_SM = 2048
MAX_WARPS_PER_SM = MAX_THREADS_PER_SM // 32
MAX_BLOCKS_PER_SM = 32
SMEM_PER_SM = 228 * 1024
SMEM_PER_BLOCK_MAX = 227 * 1024
SMEM_RESERVED_PER_BLOCK = 1024
SMEM_ALLOC_UNIT = 128
TMEM_COLUMNS = 512
_UNBOUNDED = 1 << 30            # a resource the block does not use


def _ceil_to(x: int, m: int) -> int:
    return -(-int(x) // m) * m


@dataclass
class Occupancy:
    blocks_per_sm: int
    warps_per_sm: int
    occupancy: float              # resident warps / 64
    limiter: str                  # registers | shared_memory | tmem | threads | blocks | invalid
    by_registers: int
    by_shared_memory: int
    by_threads: int
    by_blocks: int
    by_tmem: int
    note: str = ""

    def as_dict(self) -> dict:
        return asdict(self)


def occupancy(threads: int, registers: int = 0, smem_bytes: int = 0, tmem_columns: int = 0) -> Occupancy:
    """Resident blocks per SM for a block of ``threads`` threads using
    ``registers`` per thread, ``smem_bytes`` of shared memory (static +
    dynamic) and ``tmem_columns`` TMEM columns."""
    threads = int(threads)
    if threads <= 0 or threads > 1024:
        return Occupancy(0, 0, 0.0, "invalid", 0, 0, 0, 0, 0, "threads per block must be 1..1024")
    if registers > MAX_REGS_PER_THREAD:
        return Occupancy(0, 0, 0.0, "invalid", 0, 0, 0, 0, 0, "more than 255 registers per thread")
    if smem_bytes > SMEM_PER_BLOCK_MAX:
        return Occupancy(0, 0, 0.0, "invalid", 0, 0, 0, 0, 0, "more than 227 KB of shared memory per block")
    warps = -(-threads // 32)
    by_threads = MAX_WARPS_PER_SM // warps
    if registers > 0:
        per_warp = _ceil_to(registers * 32, REG_ALLOC_UNIT)
        by_regs = REGS_PER_SM // (per_warp * warps)
    else:
        by_regs = _UNBOUNDED
    if smem_bytes > 0:
        per_block = _ceil_to(smem_bytes, SMEM_ALLOC_UNIT) + SMEM_RESERVED_PER_BLOCK
        by_smem = SMEM_PER_SM // per_block
    else:
        by_smem = _UNBOUNDED
    if tmem_columns > 0:
        cols = max(32, 1 << math.ceil(math.log2(tmem_columns)))
        if cols > TMEM_COLUMNS:
            return Occupancy(0, 0, 0.0, "invalid", 0, 0, 0, 0, 0, "more than 512 TMEM columns")
        by_tmem = TMEM_COLUMNS // cols
    else:
        by_tmem = _UNBOUNDED
    limits = {"registers": by_regs, "shared_memory": by_smem, "threads": by_threads,
              "blocks": MAX_BLOCKS_PER_SM, "tmem": by_tmem}
    blocks = min(limits.values())
    limiter = next(k for k in ("registers", "shared_memory", "tmem", "threads", "blocks")
                   if limits[k] == blocks)                     # the first binding resource
    w = blocks * warps
    return Occupancy(blocks, w, w / MAX_WARPS_PER_SM, limiter, by_regs, by_smem, by_threads,
                     MAX_BLOCKS_PER_SM, by_tmem)


@dataclass
class Waves:
    waves: float                  # grid / (blocks_per_sm * SMs)
    full_waves: int
    tail_blocks: int              # blocks of the last, partial wave
    tail_efficiency: float        # busy fraction of the SM slots over all waves


def waves(grid: int, blocks_per_sm: int, sms: int = SMS) -> Waves:
    """How a grid of ``grid`` blocks spreads over ``sms`` SMs at ``blocks_per_sm``."""
    slots = max(1, blocks_per_sm * sms)
    full, tail = divmod(int(grid), slots)
    n = full + (1 if tail else 0)
    eff = grid / (n * slots) if n else 0.0
    return Waves(grid / slots, full, tail, eff)


def persistent_grid(blocks_per_sm: int, sms: int = SMS) -> int:
    """One block per resident slot: the grid of a persistent kernel."""
    return max(1, blocks_per_sm) * sms


def advise(occ: Occupancy, grid: Optional[int] = None) -> str:
    """One line on what bounds residency and how the grid fills the GPU."""
    if occ.limiter == "invalid":
        return f"launch cannot run: {occ.note}"
    s = f"{occ.blocks_per_sm} block(s)/SM, {occ.warps_per_sm} warps ({occ.occupancy:.0%})"
    s += f", limited by {occ.limiter.replace('_', ' ')}"
    if grid:
        w = waves(grid, occ.blocks_per_sm)
        s += f"; grid {grid} = {w.waves:.2f} waves, tail efficiency {w.tail_efficiency:.0%}"
        if w.full_waves >= 1 and w.tail_efficiency < 0.85:
            s += " (a persistent grid of %d or a different tile size removes the tail)" % \
                persistent_grid(occ.blocks_per_sm)
    return s
