"""Splitting work across GPUs: independent objects, and one large volume.

Objects (`assign_objects`): whole objects are dealt to ranks, largest first,
each to the rank with the least voxels so far (longest-processing-time
first); objects never talk to each other, so there is no collective.

One large volume (Morton-ordered slabs + halo; each rank's own rows are
ordered interior first, so the interior rows' conv can run while the halo
is exchanged):

The volume's active voxels are sorted by their 3D Morton code and cut into
`world` contiguous ranges of (nearly) equal voxel count; rank r owns range r.
A submanifold 3x3x3 conv of rank r's voxels reads their 26-neighbours, some of
which belong to other ranks: those "ghost" voxels are received from their
owners before every layer. Coordinates never change across layers, so the
plan (ghost lists and the matching send lists) is computed once, by every
rank on its own from the global coordinate list, with no communication.

Per layer a rank packs the rows its peers need (`HaloPlan.send_rows`), swaps
them with one all-to-all (torch.distributed: NCCL on GPUs, gloo on CPU) into
the ghost region after its own rows, and convolves its own rows over
[own | ghost] rows (`s3dsp_kmap_build_subm3_rows`). The only collective is
that halo exchange.

There is no reference counterpart: sam3d.cpp runs one object on one device.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

def assign_objects(sizes, world: int) -> list[list[int]]:
    """Object indices per rank: largest first, each to the least-loaded rank
    (ties: lowest rank). Deterministic, so every rank computes the same split."""
    load = [0] * world
    out = [[] for _ in range(world)]
    for i in sorted(range(len(sizes)), key=lambda j: (-int(sizes[j]), j)):
        r = min(range(world), key=lambda q: (load[q], q))
        out[r].append(i)
        load[r] += int(sizes[i])
    return out


_OFFSETS = np.array([(dx, dy, dz) for dx in (-1, 0, 1) for dy in (-1, 0, 1) for dz in (-1, 0, 1)
                     if (dx, dy, dz) != (0, 0, 0)], dtype=np.int64)


def _spread21(v: np.ndarray) -> np.ndarray:
    """Bits 0..20 of v moved to bit positions 0, 3, 6, ... (3D Morton interleave)."""
    v = v.astype(np.uint64) & np.uint64(0x1FFFFF)
    v = (v | (v << np.uint64(32))) & np.uint64(0x1F00000000FFFF)
    v = (v | (v << np.uint64(16))) & np.uint64(0x1F0000FF0000FF)
    v = (v | (v << np.uint64(8))) & np.uint64(0x100F00F00F00F00F)
    v = (v | (v << np.uint64(4))) & np.uint64(0x10C30C30C30C30C3)
    v = (v | (v << np.uint64(2))) & np.uint64(0x1249249249249249)
    return v


def morton_codes(coords: np.ndarray) -> np.ndarray:
    """64-bit Morton codes of int32 (b, x, y, z) rows: x, y, z shifted to be
    non-negative, 21 bits each, interleaved x-major; the batch index b goes
    above them, so voxels of one object stay contiguous."""
    c = np.asarray(coords, dtype=np.int64)
    xyz = c[:, 1:4] - c[:, 1:4].min(axis=0)
    if xyz.size and xyz.max() >= (1 << 21):
        raise ValueError("coordinate extent exceeds 2^21 per axis")
    code = (_spread21(xyz[:, 0]) << np.uint64(2)) | (_spread21(xyz[:, 1]) << np.uint64(1)) | _spread21(xyz[:, 2])
    if c.shape[0] and c[:, 0].max() > 0:
        if c[:, 0].max() >= 2:
            raise ValueError("morton_codes orders one object (batch index 0 or 1)")
        code = code | (c[:, 0].astype(np.uint64) << np.uint64(63))
    return code


def slab_bounds(n: int, world: int) -> np.ndarray:
    """Cut points of `world` contiguous ranges of the Morton order, sizes
    differing by at most one voxel."""
    return np.array([(n * r) // world for r in range(world + 1)], dtype=np.int64)


def _packed_keys(c: np.ndarray) -> np.ndarray:
    # (b, x, y, z) -> one int64, order-preserving for |x|, |y|, |z| < 2^20
    return (((c[:, 0] << 21) + (c[:, 1] + (1 << 20))) << 42) + ((c[:, 2] + (1 << 20)) << 21) + (c[:, 3] + (1 << 20))


@dataclass
class HaloPlan:
    rank: int
    world: int
    own: np.ndarray          # global row ids of this rank's voxels: interior, then boundary (Morton order in each)
    ghost: np.ndarray        # global row ids of the halo, grouped by owner rank, Morton order within
    recv_counts: np.ndarray  # [world] ghost rows received from each rank
    send_rows: np.ndarray    # local row indices (into `own`) sent, grouped by destination rank
    send_counts: np.ndarray  # [world]
    n_interior: int = 0      # own rows [0, n_interior) have no neighbour on another rank

    @property
    def n_own(self) -> int:
        return int(self.own.shape[0])

    @property
    def n_ghost(self) -> int:
        return int(self.ghost.shape[0])

    def shard_coords(self, coords: np.ndarray) -> np.ndarray:
        """Coordinates of this rank's rows: own voxels first, then the halo."""
        return np.ascontiguousarray(np.concatenate([coords[self.own], coords[self.ghost]]).astype(np.int32))


def plan_halos(coords: np.ndarray, world: int) -> list[HaloPlan]:
    """Morton slabs and halo exchange lists of every rank.

    Rank r's ghosts from rank p are p's voxels that are 26-neighbours of some
    voxel of r, in Morton order; rank p's send list to r is the same set (the
    neighbour relation is symmetric), in the same order, so one all-to-all
    lands every row in its ghost slot."""
    coords = np.asarray(coords, dtype=np.int64)
    n = coords.shape[0]
    order = np.argsort(morton_codes(coords), kind="stable")
    pos = np.empty(n, dtype=np.int64)
    pos[order] = np.arange(n)
    bounds = slab_bounds(n, world)
    owner = (np.searchsorted(bounds, pos, side="right") - 1).astype(np.int64)

    keys = _packed_keys(coords)
    korder = np.argsort(keys, kind="stable")
    skeys = keys[korder]
    # adjacency between ranks: for every voxel and offset, the owner of the neighbour
    if world > 32767:
        raise ValueError("world too large")
    nb_owner = np.full((n, _OFFSETS.shape[0]), -1, dtype=np.int16)
    for j, d in enumerate(_OFFSETS):
        q = coords.copy()
        q[:, 1:4] += d
        qk = _packed_keys(q)
        at = np.searchsorted(skeys, qk)
        at_c = np.minimum(at, n - 1)
        hit = (at < n) & (skeys[at_c] == qk)
        nb_owner[hit, j] = owner[korder[at_c[hit]]].astype(np.int16)

    plans = []
    for r in range(world):
        own = order[bounds[r]:bounds[r + 1]]
        # interior rows first: their conv needs no halo, so it can run while the halo is in flight
        nb = nb_owner[own]
        boundary = ((nb >= 0) & (nb != r)).any(axis=1)
        own = np.concatenate([own[~boundary], own[boundary]])
        n_interior = int((~boundary).sum())
        # ghosts: voxels of other ranks adjacent to some voxel of r
        # == voxels v with owner != r having a neighbour owned by r
        touches_r = (nb_owner == r).any(axis=1)
        g = np.nonzero(touches_r & (owner != r))[0]
        g = g[np.lexsort((pos[g], owner[g]))]
        recv_counts = np.bincount(owner[g], minlength=world).astype(np.int64)
        # sends: own voxels adjacent to a voxel of p, for each p, in Morton order
        own_local = np.arange(own.shape[0], dtype=np.int64)
        send, send_counts = [], np.zeros(world, dtype=np.int64)
        nb_own = nb_owner[own]
        for p in range(world):
            if p == r:
                continue
            sel = own_local[(nb_own == p).any(axis=1)]
            send.append(sel)
            send_counts[p] = sel.shape[0]
        send_rows = np.concatenate(send) if send else np.zeros(0, dtype=np.int64)
        plans.append(HaloPlan(r, world, own, g, recv_counts, send_rows, send_counts, n_interior))
    return plans


def exchange_halo(x, plan: HaloPlan, group=None):
    """Fill rows [n_own, n_own + n_ghost) of x ([n_own + n_ghost, C], CPU or
    CUDA tensor) with the peers' rows, in place: one all-to-all."""
    import torch
    import torch.distributed as dist

    if plan.world == 1:
        return
    cache = plan.__dict__.setdefault("_send_idx", {})
    idx = cache.get(x.device)
    if idx is None:  # copied to the device once, not every layer
        idx = cache[x.device] = torch.as_tensor(plan.send_rows, device=x.device)
    send = x.index_select(0, idx)
    recv = x[plan.n_own:plan.n_own + plan.n_ghost]
    dist.all_to_all_single(recv, send, output_split_sizes=plan.recv_counts.tolist(),
                           input_split_sizes=plan.send_counts.tolist(), group=group)
